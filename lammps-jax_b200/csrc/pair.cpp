// pair_style jax/kk on the ljx engine: the host side of cpp/pair_jax_kokkos.cpp without LAMMPS
// types (see include/ljx_pair.h). Each method keeps the reference's checks, their order and
// their messages; the kernels and the exchanges are the engine's C ABI (include/ljx.h).

#include "ljx_pair.h"

#include <cuda_runtime.h>

#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>

namespace {

// LAMMPS utils::bounds: "*", "n", "*n", "n*", "m*n" over [nmin, nmax].
bool parse_bounds(const std::string &s, int nmin, int nmax, int &lo, int &hi, std::string &err)
{
  auto number = [&](const std::string &t, int &out) {
    if (t.empty()) return false;
    char *end = nullptr;
    errno = 0;
    const long v = std::strtol(t.c_str(), &end, 10);
    if (errno != 0 || *end != '\0') return false;
    out = static_cast<int>(v);
    return true;
  };
  const size_t star = s.find('*');
  bool ok = true;
  if (star == std::string::npos) {
    ok = number(s, lo);
    hi = lo;
  } else {
    const std::string a = s.substr(0, star), b = s.substr(star + 1);
    lo = nmin;
    hi = nmax;
    if (!a.empty()) ok = number(a, lo);
    if (ok && !b.empty()) ok = number(b, hi);
  }
  if (!ok) {
    err = "Invalid range string: " + s;
    return false;
  }
  if (lo < nmin || hi > nmax || lo > hi) {
    const int bad = lo < nmin || lo > hi ? lo : hi;
    err = "Numeric index " + std::to_string(bad) + " is out of bounds (" + std::to_string(nmin) +
          "-" + std::to_string(nmax) + ")";
    return false;
  }
  return true;
}

// LAMMPS utils::numeric.
bool parse_numeric(const std::string &s, double &out, std::string &err)
{
  char *end = nullptr;
  errno = 0;
  out = std::strtod(s.c_str(), &end);
  if (s.empty() || errno != 0 || *end != '\0') {
    err = "Expected floating point parameter instead of '" + s +
          "' in input script or data file";
    return false;
  }
  return true;
}

bool has(const char *style, const char *what) { return std::strstr(style, what) != nullptr; }

}  // namespace

struct ljx_pair {
  int device = 0;
  double scale = 1.0;
  std::string plugin_path;  // pair_style argument: accepted, unused (no PJRT plugin)
  ljx_bundle *bundle = nullptr;
  ljx_engine *engine = nullptr;
  ljx_contract c{};
  ljx_plan plan{};
  bool model_loaded = false;
  bool planned = false;
  double eng_vdwl = 0.0;
  double virial[6] = {0, 0, 0, 0, 0, 0};
  double *eatom = nullptr;  // LAMMPS's per-atom arrays (device), registered by the plugin
  double *vatom = nullptr;
  std::string error;

  ljx_status fail(ljx_status status, std::string message)
  {
    error = std::move(message);
    return status;
  }
  void release()
  {
    if (engine) ljx_engine_destroy(engine);
    if (bundle) ljx_bundle_free(bundle);
    engine = nullptr;
    bundle = nullptr;
    model_loaded = false;
    planned = false;
  }
  ~ljx_pair() { release(); }
};

extern "C" {

ljx_status ljx_pair_create(int device, ljx_pair **out)
{
  if (out == nullptr) return LJX_ERR_INVALID;
  *out = new (std::nothrow) ljx_pair;
  if (*out == nullptr) return LJX_ERR_INVALID;
  (*out)->device = device;
  return LJX_OK;
}

void ljx_pair_destroy(ljx_pair *pair) { delete pair; }

const char *ljx_pair_error(const ljx_pair *pair) { return pair ? pair->error.c_str() : ""; }

ljx_status ljx_pair_settings(ljx_pair *pair, int narg, const char *const *arg)
{
  if (pair == nullptr) return LJX_ERR_INVALID;
  if (narg > 1) return pair->fail(LJX_ERR_INVALID, "Illegal pair_style jax/kk command");
  if (narg == 1 && arg && arg[0]) pair->plugin_path = arg[0];
  return LJX_OK;
}

ljx_status ljx_pair_coeff(ljx_pair *pair, int narg, const char *const *arg,
                          const char *unit_style, int ntypes)
{
  if (pair == nullptr) return LJX_ERR_INVALID;
  if (narg < 3 || narg > 4 || arg == nullptr)
    return pair->fail(LJX_ERR_INVALID, "Illegal pair_coeff jax/kk command");
  int ilo = 0, ihi = 0, jlo = 0, jhi = 0;
  std::string err;
  if (!parse_bounds(arg[0], 1, ntypes, ilo, ihi, err) ||
      !parse_bounds(arg[1], 1, ntypes, jlo, jhi, err))
    return pair->fail(LJX_ERR_INVALID, err);
  if (narg == 4 && !parse_numeric(arg[3], pair->scale, err))
    return pair->fail(LJX_ERR_INVALID, err);

  pair->release();
  if (ljx_bundle_load(arg[2], &pair->bundle) != LJX_OK)
    return pair->fail(LJX_ERR_BUNDLE,
                      std::string("Failed to load LAMMPS-JAX model: ") + ljx_bundle_error());
  ljx_bundle_contract(pair->bundle, &pair->c);
  const ljx_contract &c = pair->c;
  if (unit_style == nullptr || std::strcmp(c.unit_style, unit_style) != 0)
    return pair->fail(LJX_ERR_INVALID, "LAMMPS-JAX model unit style does not match current units");
  if (c.n_species > 0 && ntypes > c.n_species)
    return pair->fail(LJX_ERR_INVALID,
                      "LAMMPS-JAX model distinguishes " + std::to_string(c.n_species) +
                          " species but the system defines " + std::to_string(ntypes) +
                          " atom types; types beyond the model's range would silently map to "
                          "its last species");
  // ljx runs only on CUDA devices.
  const char *platform = "cuda";
  if (std::strcmp(c.platform, platform) != 0)
    return pair->fail(LJX_ERR_INVALID, std::string("LAMMPS-JAX model was exported for ") +
                                           c.platform + " but this build runs " + platform +
                                           "; re-export it with platform=\"" + platform + "\"");
  if (ljx_engine_create(pair->bundle, pair->device, &pair->engine) != LJX_OK)
    return pair->fail(LJX_ERR_CUDA, std::string("Failed to initialize LAMMPS-JAX runtime: ") +
                                        ljx_bundle_error());
  pair->model_loaded = true;

  int count = 0;
  for (int i = ilo; i <= ihi; ++i)
    for (int j = (jlo > i ? jlo : i); j <= jhi; ++j) ++count;
  if (count == 0) return pair->fail(LJX_ERR_INVALID, "Incorrect args for pair coefficients");
  return LJX_OK;
}

ljx_status ljx_pair_init_style(ljx_pair *pair, int newton_pair, int molecular,
                               const double *special_lj, const double *special_coul, int nfix,
                               const char *const *fix_styles, ljx_plan *plan)
{
  if (pair == nullptr) return LJX_ERR_INVALID;
  if (!pair->model_loaded) return pair->fail(LJX_ERR_INVALID, "LAMMPS-JAX model has not been loaded");
  // Newton mode of the bundle (the engine's plan carries the reference's messages).
  if (ljx_engine_plan(pair->engine, newton_pair, &pair->plan) != LJX_OK)
    return pair->fail(LJX_ERR_INVALID, ljx_engine_error(pair->engine));
  if (molecular && special_lj && special_coul) {
    // Every listed pair gets full weight; partial special_bonds factors would be ignored.
    for (int n = 1; n <= 3; ++n)
      if (special_lj[n] != 1.0 && !(special_lj[n] == 0.0 && special_coul[n] == 0.0))
        return pair->fail(LJX_ERR_INVALID, "pair jax/kk does not apply special_bonds factors; "
                                           "use 1 1 1 or full exclusion");
  }
  if (!newton_pair) {
    // Pair virial needs newton-on ghost force rows; a barostat would see incomplete pressure.
    for (int k = 0; k < nfix && fix_styles; ++k) {
      const char *style = fix_styles[k];
      if (style && (has(style, "npt") || has(style, "nph") || has(style, "press") ||
                    has(style, "box/relax") || has(style, "msst")))
        return pair->fail(LJX_ERR_INVALID, std::string("Fix ") + style +
                                               " requires pair virial; run pair jax/kk with "
                                               "newton pair on");
    }
  }
  if (pair->c.n_comm_widths > 0 && molecular && special_lj) {
    for (int n = 1; n <= 3; ++n)
      if (special_lj[n] != 1.0)
        return pair->fail(LJX_ERR_INVALID,
                          "Communicating LAMMPS-JAX bundles require special_bonds 1 1 1");
  }
  pair->planned = true;
  if (plan) *plan = pair->plan;
  return LJX_OK;
}

double ljx_pair_init_one(const ljx_pair *pair)
{
  return pair && pair->model_loaded ? pair->c.cutoff : 0.0;
}

ljx_status ljx_pair_compute(ljx_pair *pair, void *stream, const ljx_atoms *atoms,
                            const ljx_list *list, int newton_pair, int flags,
                            const ljx_pair_host *host, ljx_result *out)
{
  if (pair == nullptr) return LJX_ERR_INVALID;
  // ev_init: the global tallies this call reports start from zero.
  if (flags & LJX_EFLAG_GLOBAL) pair->eng_vdwl = 0.0;
  if (flags & LJX_VFLAG_GLOBAL)
    for (double &v : pair->virial) v = 0.0;
  if (!pair->model_loaded || pair->engine == nullptr)
    return pair->fail(LJX_ERR_INVALID, "LAMMPS-JAX runtime is not initialized");
  // Per-atom output needs LAMMPS's arrays; without them the reference's refusal stands.
  if ((flags & LJX_EFLAG_ATOM) && pair->eatom == nullptr)
    return pair->fail(LJX_ERR_UNSUPPORTED, "pair jax/kk does not support per-atom energy output");
  if ((flags & LJX_VFLAG_ATOM) && pair->vatom == nullptr)
    return pair->fail(LJX_ERR_UNSUPPORTED, "pair jax/kk does not support per-atom virial output");
  // Energy-only (MC) steps need an energy program in the reference; a bundle's potential block
  // always yields the energy here.
  const bool energy_only = (flags & LJX_EFLAG_ONLY) != 0;
  if (list == nullptr)
    return pair->fail(LJX_ERR_INVALID, "LAMMPS-JAX requires a Kokkos device neighbor list");
  if (atoms == nullptr) return pair->fail(LJX_ERR_INVALID, "atom arrays are missing");
  if (!pair->planned) {
    if (ljx_engine_plan(pair->engine, newton_pair, &pair->plan) != LJX_OK)
      return pair->fail(LJX_ERR_INVALID, ljx_engine_error(pair->engine));
    pair->planned = true;
  }
  const ljx_contract &c = pair->c;
  ljx_engine *e = pair->engine;
  auto reduce = [&](int *values, int n) {
    return host && host->allreduce_max ? host->allreduce_max(host->ctx, values, n) : 0;
  };
  auto compute_failed = [&]() {
    return pair->fail(LJX_ERR_CUDA, std::string("LAMMPS-JAX compute failed: ") + ljx_engine_error(e));
  };

  // Row limits abort before launch, on global values (:1035-1046).
  int rows[2] = {atoms->nlocal + atoms->nghost, atoms->nlocal};
  if (reduce(rows, 2) != 0) return pair->fail(LJX_ERR_INVALID, "LAMMPS-JAX row check failed");
  if (rows[0] > c.max_atoms)
    return pair->fail(LJX_ERR_CAPACITY, "LAMMPS-JAX atom capacity exceeded: global max " +
                                            std::to_string(rows[0]) + " atoms, capacity " +
                                            std::to_string(c.max_atoms));
  if (c.max_owned > 0 && rows[1] > c.max_owned)
    return pair->fail(LJX_ERR_CAPACITY, "LAMMPS-JAX owned-row capacity exceeded: global max " +
                                            std::to_string(rows[1]) + " owned atoms, capacity " +
                                            std::to_string(c.max_owned));

  // ev_setup: the per-atom arrays asked for start from zero over nlocal (+ nghost with newton).
  double *eatom = (flags & LJX_EFLAG_ATOM) ? pair->eatom : nullptr;
  double *vatom = (flags & LJX_VFLAG_ATOM) && !energy_only ? pair->vatom : nullptr;
  const long long tally_rows =
      static_cast<long long>(atoms->nlocal) + (newton_pair ? atoms->nghost : 0);
  auto cs = static_cast<cudaStream_t>(stream);
  if ((eatom && cudaMemsetAsync(eatom, 0, tally_rows * sizeof(double), cs) != cudaSuccess) ||
      (vatom && cudaMemsetAsync(vatom, 0, 6 * tally_rows * sizeof(double), cs) != cudaSuccess))
    return pair->fail(LJX_ERR_CUDA, "LAMMPS-JAX compute failed: per-atom arrays");
  ljx_set_atom_tallies(e, eatom, vatom, pair->scale);
  struct TalliesOff {
    ljx_engine *e;
    ~TalliesOff() { ljx_set_atom_tallies(e, nullptr, nullptr, 1.0); }
  } tallies_off{e};

  if (ljx_pack_atoms(e, stream, atoms) != LJX_OK)
    return pair->fail(LJX_ERR_CAPACITY, ljx_engine_error(e));
  if (ljx_density(e, stream, atoms, list, newton_pair) != LJX_OK) return compute_failed();
  const ljx_plan &plan = pair->plan;
  if (plan.reverse_density) {
    void *rows_ptr = nullptr;
    int width = 0, elem = 0;
    ljx_feature_rows(e, 0, &rows_ptr, &width, &elem);
    if (!host || !host->reverse_comm || host->reverse_comm(host->ctx, rows_ptr, width, elem, stream))
      return pair->fail(LJX_ERR_CUDA, "LAMMPS-JAX compute failed: reverse comm of rho failed");
  }
  if (ljx_embed(e, stream, atoms) != LJX_OK) return compute_failed();
  if (energy_only) {
    if (ljx_energy(e, stream, atoms, list, newton_pair, pair->scale) != LJX_OK)
      return compute_failed();
  } else {
    if (plan.forward_fp) {
      void *rows_ptr = nullptr;
      int width = 0, elem = 0;
      ljx_feature_rows(e, 1, &rows_ptr, &width, &elem);
      if (!host || !host->forward_comm ||
          host->forward_comm(host->ctx, rows_ptr, width, elem, stream))
        return pair->fail(LJX_ERR_CUDA, "LAMMPS-JAX compute failed: forward comm of F' failed");
    }
    if (atoms->f == nullptr) return pair->fail(LJX_ERR_INVALID, "force array is missing");
    // Steps without energy or virial requests (all but thermo steps) run the forces alone, as
    // the reference runs its force program (:1055-1057).
    const bool ev = (flags & (LJX_EFLAG_GLOBAL | LJX_VFLAG_GLOBAL | LJX_EFLAG_ATOM |
                              LJX_VFLAG_ATOM)) != 0;
    if ((ev ? ljx_force(e, stream, atoms, list, newton_pair, pair->scale)
            : ljx_force_only(e, stream, atoms, list, newton_pair, pair->scale)) != LJX_OK)
      return compute_failed();
  }
  ljx_result res{};
  if (ljx_read_result(e, stream, &res) != LJX_OK) return compute_failed();

  // Overflow only truncates the packed rows, so the collective abort waits until here
  // (:1063-1075). Matrix bundles report the widest list row.
  const bool matrix = c.input_layout == LJX_LAYOUT_NEIGHBOR_MATRIX;
  const long long first = matrix ? res.widest_row : res.edge_count;
  int counts[2] = {static_cast<int>(first < 2147483647LL ? first : 2147483647LL), res.overflow};
  if (reduce(counts, 2) != 0) return pair->fail(LJX_ERR_INVALID, "LAMMPS-JAX count check failed");
  if (counts[1] && matrix)
    return pair->fail(LJX_ERR_CAPACITY, "LAMMPS-JAX neighbor capacity exceeded: global max " +
                                            std::to_string(counts[0]) + " neighbors per atom, "
                                            "capacity " + std::to_string(c.max_neighbors));
  if (counts[1])
    return pair->fail(LJX_ERR_CAPACITY, "LAMMPS-JAX edge capacity exceeded: global max " +
                                            std::to_string(counts[0]) + " edges, capacity " +
                                            std::to_string(c.max_edges));

  // Tallies (:1083-1101): the energy (already times scale) whenever it was asked for; the f.r
  // virial unless this was an energy-only step.
  if ((flags & LJX_EFLAG_GLOBAL) || energy_only) pair->eng_vdwl += res.energy;
  if ((flags & LJX_VFLAG_GLOBAL) && !energy_only)
    for (int k = 0; k < 6; ++k) pair->virial[k] += res.virial[k];
  if (out) *out = res;
  return LJX_OK;
}

ljx_status ljx_pair_tally(const ljx_pair *pair, double *eng_vdwl, double *virial)
{
  if (pair == nullptr) return LJX_ERR_INVALID;
  if (eng_vdwl) *eng_vdwl = pair->eng_vdwl;
  if (virial)
    for (int k = 0; k < 6; ++k) virial[k] = pair->virial[k];
  return LJX_OK;
}

ljx_status ljx_pair_set_atom_tallies(ljx_pair *pair, double *eatom, double *vatom)
{
  if (pair == nullptr) return LJX_ERR_INVALID;
  pair->eatom = eatom;
  pair->vatom = vatom;
  return LJX_OK;
}

const ljx_bundle *ljx_pair_bundle(const ljx_pair *pair) { return pair ? pair->bundle : nullptr; }

ljx_engine *ljx_pair_engine(ljx_pair *pair) { return pair ? pair->engine : nullptr; }

}  // extern "C"
