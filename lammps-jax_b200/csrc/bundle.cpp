// Bundle loader. The reference loader (cpp/lammps_jax_model.cpp:12-315) reads the sorted-key
// JSON that python/lammps_jax/export.py:523-566 writes by first-quoted-key lookup; this loader
// keeps that lookup rule, the same required/optional keys, the same validation order and the
// same messages, so it accepts and rejects exactly the bundles the reference does. It adds the
// `potential` keys the engine computes from (the reference's physics lives only inside the
// serialized XLA programs, python/lammps_jax/export.py:524-531):
//   "potential_kind": "eam/alloy" with "setfl_b64" (base64 of the DYNAMO setfl text),
//                     "eam" with "funcfl_b64", or "lj/cut" with "lj_epsilon", "lj_sigma" and
//                     optionally "lj_edge_energy_scale".
// The key names are distinct from every contract key, so first-match lookup stays unambiguous.

#include "bundle.h"

#include <cctype>
#include <cmath>
#include <cstring>
#include <fstream>
#include <iterator>
#include <sstream>
#include <stdexcept>

namespace ljx {
namespace {

bool has_key(const std::string &json, const std::string &key)
{
  return json.find("\"" + key + "\"") != std::string::npos;
}

// Position just past the colon that follows the first occurrence of "key".
size_t value_start(const std::string &json, const std::string &key)
{
  const std::string quoted = "\"" + key + "\"";
  const size_t at = json.find(quoted);
  if (at == std::string::npos) throw std::runtime_error("Missing key in bundle: " + key);
  const size_t colon = json.find(':', at + quoted.size());
  if (colon == std::string::npos) throw std::runtime_error("Malformed key in bundle: " + key);
  size_t pos = colon + 1;
  while (pos < json.size() && std::isspace(static_cast<unsigned char>(json[pos]))) ++pos;
  return pos;
}

std::string read_string(const std::string &json, const std::string &key)
{
  size_t pos = value_start(json, key);
  if (pos >= json.size() || json[pos] != '"') throw std::runtime_error("Expected JSON string");
  std::string out;
  for (++pos; pos < json.size();) {
    const char c = json[pos++];
    if (c == '"') return out;
    if (c != '\\') {
      out.push_back(c);
      continue;
    }
    if (pos >= json.size()) throw std::runtime_error("Invalid JSON escape");
    const char e = json[pos++];
    const char *from = "\"\\/bfnrt";
    const char *to = "\"\\/\b\f\n\r\t";
    const char *hit = std::strchr(from, e);
    if (hit == nullptr || e == '\0')
      throw std::runtime_error("Unsupported JSON escape in model bundle");
    out.push_back(to[hit - from]);
  }
  throw std::runtime_error("Unterminated JSON string");
}

double read_number(const std::string &json, const std::string &key)
{
  const size_t pos = value_start(json, key);
  const size_t end = json.find_first_of(",}\n\r\t ", pos);
  return std::stod(json.substr(pos, end - pos));
}

int read_int_or(const std::string &json, const std::string &key, int fallback)
{
  return has_key(json, key) ? static_cast<int>(read_number(json, key)) : fallback;
}

double read_double_or(const std::string &json, const std::string &key, double fallback)
{
  return has_key(json, key) ? read_number(json, key) : fallback;
}

bool read_bool(const std::string &json, const std::string &key)
{
  const size_t pos = value_start(json, key);
  if (json.compare(pos, 4, "true") == 0) return true;
  if (json.compare(pos, 5, "false") == 0) return false;
  throw std::runtime_error("Expected boolean for key: " + key);
}

bool read_bool_or(const std::string &json, const std::string &key, bool fallback)
{
  return has_key(json, key) ? read_bool(json, key) : fallback;
}

// Flat array of integers or of identifier-like strings; a missing key is an empty array.
std::vector<std::string> read_array_items(const std::string &json, const std::string &key,
                                          bool strings)
{
  std::vector<std::string> items;
  if (!has_key(json, key)) return items;
  size_t pos = value_start(json, key);
  if (pos >= json.size() || json[pos] != '[')
    throw std::runtime_error("Expected JSON array for key: " + key);
  ++pos;
  for (;;) {
    while (pos < json.size() && std::isspace(static_cast<unsigned char>(json[pos]))) ++pos;
    if (pos >= json.size()) throw std::runtime_error("Unterminated JSON array for key: " + key);
    if (json[pos] == ']') break;
    if (strings) {
      if (json[pos] != '"')
        throw std::runtime_error("Expected string in JSON array for key: " + key);
      const size_t end = json.find('"', pos + 1);
      if (end == std::string::npos)
        throw std::runtime_error("Unterminated string in JSON array for key: " + key);
      items.push_back(json.substr(pos + 1, end - pos - 1));
      pos = end + 1;
      while (pos < json.size() && std::isspace(static_cast<unsigned char>(json[pos]))) ++pos;
    } else {
      const size_t end = json.find_first_of(",]", pos);
      if (end == std::string::npos)
        throw std::runtime_error("Unterminated JSON array for key: " + key);
      items.push_back(json.substr(pos, end - pos));
      pos = end;
    }
    if (pos < json.size() && json[pos] == ',') ++pos;
  }
  return items;
}

std::vector<int> read_int_array(const std::string &json, const std::string &key)
{
  std::vector<int> out;
  for (const std::string &item : read_array_items(json, key, false)) out.push_back(std::stoi(item));
  return out;
}

std::string base64_decode(const std::string &text)
{
  int table[256];
  for (int &t : table) t = -1;
  const char *alphabet = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";
  for (int k = 0; alphabet[k]; ++k) table[static_cast<unsigned char>(alphabet[k])] = k;
  std::string out;
  out.reserve(text.size() * 3 / 4);
  unsigned acc = 0;
  int nbits = 0;
  for (const unsigned char c : text) {
    if (std::isspace(c)) continue;
    if (c == '=') break;
    if (table[c] < 0) throw std::runtime_error("Invalid base64 data");
    acc = (acc << 6) | static_cast<unsigned>(table[c]);
    nbits += 6;
    if (nbits >= 8) {
      nbits -= 8;
      out.push_back(static_cast<char>((acc >> nbits) & 0xffu));
    }
  }
  return out;
}

// "<name>_b64" holds base64 VHLO; legacy bundles stored text under "<name>".
std::string read_program(const std::string &json, const std::string &name)
{
  if (has_key(json, name + "_b64")) return base64_decode(read_string(json, name + "_b64"));
  return read_string(json, name);
}

void copy_text(char *dst, size_t cap, const std::string &src)
{
  std::strncpy(dst, src.c_str(), cap - 1);
  dst[cap - 1] = '\0';
}

int parse_layout(const std::string &v)
{
  if (v == "sparse-edge") return LJX_LAYOUT_SPARSE_EDGE;
  if (v == "neighbor-matrix") return LJX_LAYOUT_NEIGHBOR_MATRIX;
  throw std::runtime_error("Unsupported LAMMPS-JAX input layout '" + v +
                           "'; re-export the bundle with the current lammps_jax exporter");
}

int parse_force_layout(const std::string &v)
{
  if (v == "atom-force") return LJX_FORCE_ATOM;
  if (v == "edge-force") return LJX_FORCE_EDGE;
  throw std::runtime_error("Unsupported LAMMPS-JAX force output layout '" + v + "'");
}

int parse_newton(const std::string &v)
{
  if (v == "any") return LJX_NEWTON_ANY;
  if (v == "on") return LJX_NEWTON_ON;
  if (v == "off") return LJX_NEWTON_OFF;
  throw std::runtime_error("Unsupported LAMMPS-JAX newton mode '" + v + "'");
}

int parse_precision(const std::string &v)
{
  if (v == "float32") return LJX_FLOAT32;
  if (v == "float64") return LJX_FLOAT64;
  throw std::runtime_error("Unsupported LAMMPS-JAX precision '" + v +
                           "'; expected float32 or float64");
}

std::vector<std::string> split_tokens(const std::string &text)
{
  std::vector<std::string> tokens;
  std::istringstream in(text);
  std::string tok;
  while (in >> tok) tokens.push_back(tok);
  return tokens;
}

}  // namespace

void spline_coefficients(const std::vector<double> &f, double *out)
{
  // python/lammps_jax/eam.py:115-135 (LAMMPS PairEAM::interpolate).
  const int n = static_cast<int>(f.size());
  if (n < 4) throw std::runtime_error("setfl tables need at least 4 points");
  std::vector<double> d(n);
  d[0] = f[1] - f[0];
  d[1] = 0.5 * (f[2] - f[0]);
  d[n - 2] = 0.5 * (f[n - 1] - f[n - 3]);
  d[n - 1] = f[n - 1] - f[n - 2];
  for (int m = 2; m < n - 2; ++m) d[m] = ((f[m - 2] - f[m + 2]) + 8.0 * (f[m + 1] - f[m - 1])) / 12.0;
  for (int m = 0; m < n; ++m) {
    out[4 * m + 0] = f[m];
    out[4 * m + 1] = d[m];
    if (m + 1 < n) {
      const double step = f[m + 1] - f[m];
      out[4 * m + 2] = 3.0 * step - 2.0 * d[m] - d[m + 1];
      out[4 * m + 3] = d[m] + d[m + 1] - 2.0 * step;
    } else {
      out[4 * m + 2] = 0.0;
      out[4 * m + 3] = 0.0;
    }
  }
}

EamTables parse_setfl(const std::string &text)
{
  // DYNAMO setfl layout as python/lammps_jax/eam.py:174-227 reads it.
  size_t start = 0;
  for (int line = 0; line < 3; ++line) {
    start = text.find('\n', start);
    if (start == std::string::npos) throw std::runtime_error("setfl text has no table body");
    ++start;
  }
  const std::vector<std::string> tok = split_tokens(text.substr(start));
  size_t pos = 0;
  auto need = [&](size_t k) {
    if (pos + k > tok.size()) throw std::runtime_error("setfl text ends early");
  };
  EamTables t;
  need(1);
  t.n_elements = std::stoi(tok[pos++]);
  if (t.n_elements < 1 || t.n_elements > 16) throw std::runtime_error("setfl element count out of range");
  need(t.n_elements + 5);
  for (int e = 0; e < t.n_elements; ++e) t.elements.push_back(tok[pos++]);
  t.nrho = std::stoi(tok[pos++]);
  t.drho = std::stod(tok[pos++]);
  t.nr = std::stoi(tok[pos++]);
  t.dr = std::stod(tok[pos++]);
  t.cutoff = std::stod(tok[pos++]);
  if (t.nrho < 4 || t.nr < 4 || !(t.drho > 0) || !(t.dr > 0))
    throw std::runtime_error("setfl grid sizes out of range");
  const size_t nrho = static_cast<size_t>(t.nrho), nr = static_cast<size_t>(t.nr);
  t.embedding.resize(static_cast<size_t>(t.n_elements) * nrho * 4);
  t.density.resize(static_cast<size_t>(t.n_elements) * nr * 4);
  std::vector<double> values;
  auto take = [&](size_t count) {
    need(count);
    values.resize(count);
    for (size_t k = 0; k < count; ++k) values[k] = std::stod(tok[pos++]);
  };
  for (int e = 0; e < t.n_elements; ++e) {
    need(4);
    t.masses.push_back(std::stod(tok[pos + 1]));
    pos += 4;
    take(nrho);
    spline_coefficients(values, t.embedding.data() + e * nrho * 4);
    take(nr);
    spline_coefficients(values, t.density.data() + e * nr * 4);
  }
  const int n_pairs = t.n_elements * (t.n_elements + 1) / 2;
  t.pair.resize(static_cast<size_t>(n_pairs) * nr * 4);
  for (int p = 0; p < n_pairs; ++p) {
    take(nr);
    spline_coefficients(values, t.pair.data() + p * nr * 4);
  }
  if (pos != tok.size())
    throw std::runtime_error("setfl text: " + std::to_string(tok.size() - pos) +
                             " unparsed trailing values");
  return t;
}

EamTables parse_funcfl(const std::string &text, const std::string &name)
{
  // Single-element funcfl as python/lammps_jax/eam.py:233-262 reads it.
  std::istringstream in(text);
  std::string comment, header;
  std::getline(in, comment);
  std::getline(in, header);
  const std::vector<std::string> head = split_tokens(header);
  if (head.size() < 2) throw std::runtime_error("funcfl header line is malformed");
  std::string rest((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
  const std::vector<std::string> tok = split_tokens(rest);
  if (tok.size() < 5) throw std::runtime_error("funcfl text ends early");
  EamTables t;
  t.n_elements = 1;
  t.elements.push_back(name);
  t.masses.push_back(std::stod(head[1]));
  t.nrho = std::stoi(tok[0]);
  t.drho = std::stod(tok[1]);
  t.nr = std::stoi(tok[2]);
  t.dr = std::stod(tok[3]);
  t.cutoff = std::stod(tok[4]);
  const size_t nrho = static_cast<size_t>(t.nrho), nr = static_cast<size_t>(t.nr);
  if (tok.size() - 5 != nrho + 2 * nr)
    throw std::runtime_error("funcfl: expected " + std::to_string(nrho + 2 * nr) +
                             " table values, got " + std::to_string(tok.size() - 5));
  std::vector<double> emb(nrho), z(nr), rho(nr), z2r(nr);
  for (size_t k = 0; k < nrho; ++k) emb[k] = std::stod(tok[5 + k]);
  for (size_t k = 0; k < nr; ++k) z[k] = std::stod(tok[5 + nrho + k]);
  for (size_t k = 0; k < nr; ++k) rho[k] = std::stod(tok[5 + nrho + nr + k]);
  const double scale = 27.2 * 0.529;  // Hartree*Bohr -> eV*Angstrom
  for (size_t k = 0; k < nr; ++k) z2r[k] = scale * z[k] * z[k];
  t.embedding.resize(nrho * 4);
  t.density.resize(nr * 4);
  t.pair.resize(nr * 4);
  spline_coefficients(emb, t.embedding.data());
  spline_coefficients(rho, t.density.data());
  spline_coefficients(z2r, t.pair.data());
  return t;
}

Bundle parse_bundle(const std::string &json)
{
  Bundle b;
  ljx_contract &c = b.contract;
  const std::string format = read_string(json, "format");
  copy_text(c.format, sizeof c.format, format);
  c.has_force_program = !read_program(json, "force_mlir").empty();
  c.has_energy_program = !read_program(json, "energy_mlir").empty();
  c.has_energy_and_forces_program = !read_program(json, "energy_and_forces_mlir").empty();
  (void) base64_decode(read_string(json, "compile_options_b64"));
  copy_text(c.platform, sizeof c.platform,
            has_key(json, "platform") ? read_string(json, "platform") : std::string("cuda"));
  c.input_layout = parse_layout(read_string(json, "input_layout"));
  c.max_atoms = static_cast<int>(read_number(json, "max_atoms"));
  c.max_edges = read_int_or(json, "max_edges", 0);
  c.max_neighbors = read_int_or(json, "max_neighbors", 0);
  c.cutoff = read_number(json, "cutoff");
  copy_text(c.unit_style, sizeof c.unit_style, read_string(json, "unit_style"));
  c.precision = parse_precision(read_string(json, "precision"));
  c.force_layout = parse_force_layout(read_string(json, "force_output"));
  c.newton = parse_newton(read_string(json, "newton"));
  c.n_hops = read_int_or(json, "n_hops", 1);
  const std::vector<int> widths = read_int_array(json, "comm_widths");
  if (widths.size() > LJX_MAX_COMM_WIDTHS) throw std::runtime_error("too many comm widths in bundle");
  c.n_comm_widths = static_cast<int>(widths.size());
  for (size_t k = 0; k < widths.size(); ++k) c.comm_widths[k] = widths[k];
  const std::vector<int> sites = read_int_array(json, "comm_sites");
  c.n_comm_sites = static_cast<int>(sites.size() < 3 ? sites.size() : 3);
  for (int k = 0; k < c.n_comm_sites; ++k) c.comm_sites[k] = sites[k];
  (void) read_array_items(json, "custom_call_targets", true);
  c.uses_box = read_bool(json, "uses_box");
  c.pair_sum = read_bool_or(json, "pair_sum", false);
  c.n_species = read_int_or(json, "n_species", 0);
  if (c.n_species < 0) throw std::runtime_error("Invalid n_species in bundle");
  c.max_owned = read_int_or(json, "max_owned", 0);
  if (c.max_owned < 0 || c.max_owned > c.max_atoms)
    throw std::runtime_error("Invalid max_owned in bundle");

  // Validation in the order of cpp/lammps_jax_model.cpp:248-313.
  const bool comm = c.n_comm_widths > 0;
  if (format != "lammps-jax-json" && format != "lammps-jax-json-distributed" &&
      format != "lammps-jax-json-half-edge")
    throw std::runtime_error("Unsupported bundle format");
  c.edge_pairing = LJX_PAIRING_FULL;
  if (format == "lammps-jax-json-half-edge") {
    const std::string pairing = read_string(json, "edge_pairing");
    if (pairing == "half") {
      if (comm)
        throw std::runtime_error(
            "Communicating half-edge bundles now pack each boundary pair on "
            "one rank; re-export this bundle");
      c.half_edges = 1;
      c.edge_pairing = LJX_PAIRING_HALF;
    } else if (pairing == "half-unique") {
      if (!comm)
        throw std::runtime_error(
            "Unique-boundary bundles need a communication schedule; the "
            "partner rank's density share arrives through reverse comm");
      c.half_edges = 1;
      c.edge_pairing = LJX_PAIRING_HALF_UNIQUE;
    } else if (pairing != "full") {
      throw std::runtime_error("Invalid edge_pairing in bundle");
    }
  }
  if (c.half_edges && c.n_hops == 1 && !comm)
    throw std::runtime_error(
        "Half-edge bundles require n_hops > 1 or a communication schedule; the "
        "single-hop packer does not deduplicate edge directions");
  const bool matrix = c.input_layout == LJX_LAYOUT_NEIGHBOR_MATRIX;
  if (c.max_atoms <= 0 || (matrix ? c.max_neighbors : c.max_edges) <= 0)
    throw std::runtime_error("Invalid fixed capacities in bundle");
  if (matrix && c.force_layout == LJX_FORCE_EDGE)
    throw std::runtime_error(
        "Neighbor-matrix bundles return per-atom forces; edge-force output needs sparse edges");
  if (c.max_owned > 0 && !comm && !(matrix && c.n_hops == 1))
    throw std::runtime_error(
        "max_owned needs a communicating or single-hop neighbor-matrix bundle; other layouts "
        "hold ghost rows past the owned ones");
  if (matrix && c.half_edges && !comm)
    throw std::runtime_error(
        "Neighbor-matrix half pairing needs a communication schedule; the pair style hands "
        "the model the LAMMPS half list as is");
  if (c.n_hops < 1) throw std::runtime_error("Invalid n_hops in bundle");
  if (c.n_hops > 1 && (c.newton != LJX_NEWTON_ON || c.force_layout != LJX_FORCE_ATOM))
    throw std::runtime_error(
        "Bundles with n_hops > 1 require newton on and atom-force output; ghost force rows "
        "must flow back through the LAMMPS reverse communication");
  for (int k = 0; k < c.n_comm_widths; ++k)
    if (c.comm_widths[k] <= 0) throw std::runtime_error("Invalid communication width in bundle");
  if (comm && c.n_hops != 1)
    throw std::runtime_error(
        "Communicating bundles require a one-cutoff ghost shell (n_hops = 1)");
  if (comm && c.newton != LJX_NEWTON_ON && (c.half_edges || c.force_layout != LJX_FORCE_ATOM))
    throw std::runtime_error(
        "Communicating bundles require newton on unless they pair fully and return atom "
        "forces; ghost force rows flow back through the LAMMPS reverse communication");
  if (comm && c.force_layout == LJX_FORCE_EDGE && !c.half_edges)
    throw std::runtime_error(
        "Communicating edge-force bundles require half-edge packing; full "
        "pairing packs both directions and the newton scatter doubles forces");

  // Potential block.
  c.potential = LJX_POTENTIAL_NONE;
  if (has_key(json, "potential_kind")) {
    const std::string kind = read_string(json, "potential_kind");
    if (kind == "eam/alloy") {
      b.eam = parse_setfl(base64_decode(read_string(json, "setfl_b64")));
      c.potential = LJX_POTENTIAL_EAM;
    } else if (kind == "eam") {
      b.eam = parse_funcfl(base64_decode(read_string(json, "funcfl_b64")),
                           has_key(json, "funcfl_element") ? read_string(json, "funcfl_element")
                                                           : std::string("funcfl"));
      c.potential = LJX_POTENTIAL_EAM;
    } else if (kind == "lj/cut") {
      c.potential = LJX_POTENTIAL_LJ;
      c.lj_epsilon = read_number(json, "lj_epsilon");
      c.lj_sigma = read_number(json, "lj_sigma");
      // examples/export_model.py:107 — whole pair energy per edge only for newton-on edge forces.
      const double fallback =
          (c.force_layout == LJX_FORCE_EDGE && c.newton == LJX_NEWTON_ON) ? 1.0 : 0.5;
      c.lj_edge_energy_scale = read_double_or(json, "lj_edge_energy_scale", fallback);
    } else {
      throw std::runtime_error("Unsupported potential_kind '" + kind +
                               "'; this engine runs eam/alloy, eam and lj/cut bundles");
    }
    if (c.potential == LJX_POTENTIAL_EAM) c.n_elements = b.eam.n_elements;
  }
  return b;
}

Bundle load_bundle(const std::string &path)
{
  std::ifstream file(path);
  if (!file.is_open()) throw std::runtime_error("Could not open model bundle: " + path);
  const std::string json{std::istreambuf_iterator<char>(file), std::istreambuf_iterator<char>()};
  return parse_bundle(json);
}

}  // namespace ljx
