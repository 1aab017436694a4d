// Parsed bundle: the reference contract plus the potential block the engine computes from.
#pragma once

#include <string>
#include <vector>

#include "ljx.h"

namespace ljx {

// EAM tables after the spline build: [n_elements][nrho][4], [n_elements][nr][4],
// [n_pairs][nr][4] with n_pairs = n_elements (n_elements + 1) / 2 in file order.
struct EamTables {
  int n_elements = 0;
  int nrho = 0;
  int nr = 0;
  double drho = 0.0;
  double dr = 0.0;
  double cutoff = 0.0;
  std::vector<std::string> elements;
  std::vector<double> masses;
  std::vector<double> embedding;
  std::vector<double> density;
  std::vector<double> pair;
};

struct Bundle {
  ljx_contract contract{};
  EamTables eam;
};

// Throws std::runtime_error with the reference loader's messages.
Bundle parse_bundle(const std::string &json);
Bundle load_bundle(const std::string &path);

// Cubic coefficients of a uniform table, (f, d, c2, c3) per node.
void spline_coefficients(const std::vector<double> &f, double *out);
EamTables parse_setfl(const std::string &text);
EamTables parse_funcfl(const std::string &text, const std::string &name);

}  // namespace ljx
