/*
 * CPU ORACLE — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the lammps-jax reference's per-step EAM/LJ force path, used by the
 * parity tests, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg as the checker
 * and the CPU stand-in for the reference's own CPU path. Nothing in the product
 * (lammps-jax_b200/) links or calls this file.
 *
 * Parity is pinned: tests/golden/ holds vectors produced by running the reference's own
 * python/lammps_jax/eam.py and examples/export_model.py (under a numpy stand-in for jax.numpy,
 * tests/golden/make_golden.py) plus the reference test suite's independent numpy port of
 * PairEAM::compute (tests/test_eam.py:338-394); tests/test_oracle_golden.py checks this file
 * against them. The packing rule has no runnable reference (it is Kokkos code inside LAMMPS);
 * it is restated line by line from cpp/pair_jax_kokkos.cpp:77-117 and pinned by known-answer
 * cases written from that code.
 *
 * Every routine is written twice through eam_oracle_impl.h: once with REAL = double and once
 * with REAL = float, because the reference's contract precision decides the arithmetic type of
 * positions, tables and model outputs (cpp/lammps_jax_model.h:30-34, eam.py:276-283).
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off, so no fused multiply-adds change
 * the rounding of the double-precision cutoff test).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* LAMMPS keeps special-bond flags in the top bits of neighbor indices (NEIGHMASK). */
#define ORC_NEIGHMASK 0x1FFFFFFF

int orc_num_threads(void)
{
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n)
{
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void) n;
#endif
}

/*
 * Piecewise-cubic coefficients of a uniformly tabulated function, out[n][4] = (f, d, c2, c3).
 * Follows python/lammps_jax/eam.py:115-135 (= LAMMPS PairEAM::interpolate).
 */
void orc_spline_coefficients(const double *f, int n, double *out)
{
  double *d = (double *) malloc(sizeof(double) * (size_t) n);
  d[0] = f[1] - f[0];
  d[1] = 0.5 * (f[2] - f[0]);
  d[n - 2] = 0.5 * (f[n - 1] - f[n - 3]);
  d[n - 1] = f[n - 1] - f[n - 2];
  for (int m = 2; m < n - 2; ++m) d[m] = ((f[m - 2] - f[m + 2]) + 8.0 * (f[m + 1] - f[m - 1])) / 12.0;
  for (int m = 0; m < n; ++m) {
    out[4 * m + 0] = f[m];
    out[4 * m + 1] = d[m];
    if (m < n - 1) {
      const double step = f[m + 1] - f[m];
      out[4 * m + 2] = 3.0 * step - 2.0 * d[m] - d[m + 1];
      out[4 * m + 3] = d[m] + d[m + 1] - 2.0 * step;
    } else {
      out[4 * m + 2] = 0.0;
      out[4 * m + 3] = 0.0;
    }
  }
  free(d);
}

/*
 * Neighbor list over owned rows (the input LAMMPS hands the pair style), built by binning all
 * atoms into cells of side >= cutoff/2 and scanning a +-2 cell stencil. Output layout is
 * LAMMPS/Kokkos LayoutLeft: neighbors[i + jj * stride]. half != 0 keeps each pair once:
 * owned j > i, or a ghost j whose coordinates sort after i in (z, y, x) order — the same
 * one-rank-per-pair rule the reference packer applies (cpp/pair_jax_kokkos.cpp:94-101).
 * Returns the widest row; rows past `maxneigh` are truncated and counted in the return value.
 */
int orc_build_list(const double *x, int nall, int nlocal, double cutoff, int half, int *neighbors,
                   long stride, int maxneigh, int *numneigh)
{
  if (nall <= 0) return 0;
  double lo[3], hi[3];
  for (int k = 0; k < 3; ++k) { lo[k] = x[k]; hi[k] = x[k]; }
  for (int i = 1; i < nall; ++i)
    for (int k = 0; k < 3; ++k) {
      if (x[3 * i + k] < lo[k]) lo[k] = x[3 * i + k];
      if (x[3 * i + k] > hi[k]) hi[k] = x[3 * i + k];
    }
  const double bin = cutoff > 0 ? 0.5 * cutoff : 1.0;
  int nb[3];
  for (int k = 0; k < 3; ++k) {
    nb[k] = (int) floor((hi[k] - lo[k]) / bin) + 1;
    if (nb[k] < 1) nb[k] = 1;
  }
  const long nbins = (long) nb[0] * nb[1] * nb[2];
  int *count = (int *) calloc((size_t) nbins + 1, sizeof(int));
  int *bin_of = (int *) malloc(sizeof(int) * (size_t) nall);
  for (int i = 0; i < nall; ++i) {
    int c[3];
    for (int k = 0; k < 3; ++k) {
      c[k] = (int) floor((x[3 * i + k] - lo[k]) / bin);
      if (c[k] < 0) c[k] = 0;
      if (c[k] >= nb[k]) c[k] = nb[k] - 1;
    }
    bin_of[i] = (c[2] * nb[1] + c[1]) * nb[0] + c[0];
    count[bin_of[i] + 1]++;
  }
  for (long b = 0; b < nbins; ++b) count[b + 1] += count[b];
  int *fill = (int *) malloc(sizeof(int) * (size_t) nbins);
  memcpy(fill, count, sizeof(int) * (size_t) nbins);
  int *sorted = (int *) malloc(sizeof(int) * (size_t) nall);
  for (int i = 0; i < nall; ++i) sorted[fill[bin_of[i]]++] = i;
  free(fill);
  const double cutsq = cutoff * cutoff;
  int widest = 0;
#pragma omp parallel for schedule(dynamic, 256) reduction(max : widest)
  for (int i = 0; i < nlocal; ++i) {
    const int b = bin_of[i];
    const int cx = b % nb[0], cy = (b / nb[0]) % nb[1], cz = b / (nb[0] * nb[1]);
    int n = 0;
    for (int dz = -2; dz <= 2; ++dz) {
      const int zz = cz + dz;
      if (zz < 0 || zz >= nb[2]) continue;
      for (int dy = -2; dy <= 2; ++dy) {
        const int yy = cy + dy;
        if (yy < 0 || yy >= nb[1]) continue;
        for (int dx = -2; dx <= 2; ++dx) {
          const int xx = cx + dx;
          if (xx < 0 || xx >= nb[0]) continue;
          const long bb = ((long) zz * nb[1] + yy) * nb[0] + xx;
          for (int s = count[bb]; s < count[bb + 1]; ++s) {
            const int j = sorted[s];
            if (j == i) continue;
            const double ex = x[3 * i] - x[3 * j], ey = x[3 * i + 1] - x[3 * j + 1],
                         ez = x[3 * i + 2] - x[3 * j + 2];
            if (ex * ex + ey * ey + ez * ez >= cutsq) continue;
            if (half) {
              if (j < nlocal) {
                if (j < i) continue;
              } else {
                const double *xi = x + 3 * i, *xj = x + 3 * j;
                if (xj[2] < xi[2]) continue;
                if (xj[2] == xi[2]) {
                  if (xj[1] < xi[1]) continue;
                  if (xj[1] == xi[1] && xj[0] < xi[0]) continue;
                }
              }
            }
            if (n < maxneigh) neighbors[(long) i + (long) n * stride] = j;
            ++n;
          }
        }
      }
    }
    numneigh[i] = n < maxneigh ? n : maxneigh;
    if (n > widest) widest = n;
  }
  free(count);
  free(bin_of);
  free(sorted);
  return widest;
}

/*
 * Sparse-edge pack of the LAMMPS list: cpp/pair_jax_kokkos.cpp:77-117 (PackNeighborFunctor) with
 * the launch extent and flags of :811-873 (pack_edges) and the padding contract of :157-173
 * (ResetEdgeTailFunctor) / :379-383. The reference reserves slots with one global atomic per
 * kept pair, so its order is nondeterministic; this restatement emits rows in ilist order and
 * slots in list order. Parity is therefore checked after a canonical (receiver, sender) sort.
 * Slots [count, max_edges) are set to the padding (max_atoms, max_atoms, false). Returns the
 * number of kept edges counted by the reference's counter (which keeps growing past max_edges).
 */
int orc_pack_edges(const double *x, const int *ilist, const int *numneigh, const int *neighbors,
                   long atom_stride, long slot_stride, int num_rows, int maxneighs, int max_atoms,
                   int max_edges, double cutsq, int half_edges, int unique_boundary,
                   int duplicate_reverse_edges, int nlocal, int *senders, int *receivers,
                   unsigned char *edge_mask, int *overflow)
{
  int count = 0;
  *overflow = 0;
  const int per = duplicate_reverse_edges ? 2 : 1;
  const int slots = maxneighs > 1 ? maxneighs : 1;
  for (int ii = 0; ii < num_rows; ++ii) {
    const int i = ilist[ii];
    if (i >= max_atoms) continue;
    for (int jj = 0; jj < slots; ++jj) {
      if (jj >= numneigh[i]) break;
      const int j = neighbors[(long) i * atom_stride + (long) jj * slot_stride] & ORC_NEIGHMASK;
      if (j >= max_atoms) continue;
      const double dx = x[3 * i + 0] - x[3 * j + 0];
      const double dy = x[3 * i + 1] - x[3 * j + 1];
      const double dz = x[3 * i + 2] - x[3 * j + 2];
      if (dx * dx + dy * dy + dz * dz > cutsq) continue;
      if (half_edges && j < i) continue;
      if (unique_boundary && j >= nlocal) {
        if (x[3 * j + 2] < x[3 * i + 2]) continue;
        if (x[3 * j + 2] == x[3 * i + 2]) {
          if (x[3 * j + 1] < x[3 * i + 1]) continue;
          if (x[3 * j + 1] == x[3 * i + 1] && x[3 * j + 0] < x[3 * i + 0]) continue;
        }
      }
      const int edge = count;
      count += per;
      if (edge + per > max_edges) {
        *overflow = 1;
        continue;
      }
      senders[edge] = i;
      receivers[edge] = j;
      edge_mask[edge] = 1;
      if (duplicate_reverse_edges) {
        senders[edge + 1] = j;
        receivers[edge + 1] = i;
        edge_mask[edge + 1] = 1;
      }
    }
  }
  for (int e = count; e < max_edges; ++e) {
    senders[e] = max_atoms;
    receivers[e] = max_atoms;
    edge_mask[e] = 0;
  }
  return count;
}

/* f += scale * model_forces over `rows` rows: cpp/pair_jax_kokkos.cpp:176-192 (AddForcesFunctor). */
void orc_add_forces_f64(double *f, const double *model, int rows, double scale)
{
  for (int i = 0; i < 3 * rows; ++i) f[i] += scale * model[i];
}

void orc_add_forces_f32(double *f, const float *model, int rows, double scale)
{
  for (int i = 0; i < 3 * rows; ++i) f[i] += scale * (double) model[i];
}

/*
 * Edge-force scatter over the packed prefix: cpp/pair_jax_kokkos.cpp:195-225 (AddEdgeForcesFunctor).
 */
void orc_add_edge_forces_f64(double *f, const double *edge_forces, const int *senders,
                             const int *receivers, int count, int newton_pair, double scale)
{
  for (int e = 0; e < count; ++e) {
    const int i = senders[e], j = receivers[e];
    for (int k = 0; k < 3; ++k) {
      const double v = scale * edge_forces[3 * e + k];
      f[3 * i + k] += v;
      if (newton_pair) f[3 * j + k] -= v;
    }
  }
}

void orc_add_edge_forces_f32(double *f, const float *edge_forces, const int *senders,
                             const int *receivers, int count, int newton_pair, double scale)
{
  for (int e = 0; e < count; ++e) {
    const int i = senders[e], j = receivers[e];
    for (int k = 0; k < 3; ++k) {
      const double v = scale * (double) edge_forces[3 * e + k];
      f[3 * i + k] += v;
      if (newton_pair) f[3 * j + k] -= v;
    }
  }
}

/*
 * Pair virial by f.r over owned and ghost rows: cpp/pair_jax_kokkos.cpp:228-245
 * (VirialFDotRFunctor, run at :1092-1100). Accumulated in long double so that the check
 * against the engine's per-edge virial is not limited by this sum's own rounding.
 */
void orc_virial_fdotr(const double *x, const double *f, int nall, double *v)
{
  long double acc[6] = {0, 0, 0, 0, 0, 0};
  for (int i = 0; i < nall; ++i) {
    const double *xi = x + 3 * i, *fi = f + 3 * i;
    acc[0] += (long double) fi[0] * xi[0];
    acc[1] += (long double) fi[1] * xi[1];
    acc[2] += (long double) fi[2] * xi[2];
    acc[3] += (long double) fi[1] * xi[0];
    acc[4] += (long double) fi[2] * xi[0];
    acc[5] += (long double) fi[2] * xi[1];
  }
  for (int k = 0; k < 6; ++k) v[k] = (double) acc[k];
}

/*
 * LAMMPS-side comm emulation for one rank with periodic images: ghost row nlocal+g is an image
 * of owned row owner[g]. forward: ghost rows take their owner's value. reverse: ghost rows are
 * summed into their owners and zeroed — the semantics of the reference's comm primitives
 * (python/lammps_jax/comm.py:151-153,190-196; cpp/pjrt/model_comm.cpp:453-466) and of LAMMPS's
 * own reverse comm of ghost forces.
 */
void orc_forward_rows_f64(double *rows, int width, int nlocal, int nghost, const int *owner)
{
  for (int g = 0; g < nghost; ++g)
    for (int w = 0; w < width; ++w)
      rows[(long) (nlocal + g) * width + w] = rows[(long) owner[g] * width + w];
}

void orc_reverse_rows_f64(double *rows, int width, int nlocal, int nghost, const int *owner)
{
  for (int g = 0; g < nghost; ++g)
    for (int w = 0; w < width; ++w) {
      rows[(long) owner[g] * width + w] += rows[(long) (nlocal + g) * width + w];
      rows[(long) (nlocal + g) * width + w] = 0.0;
    }
}

void orc_forward_rows_f32(float *rows, int width, int nlocal, int nghost, const int *owner)
{
  for (int g = 0; g < nghost; ++g)
    for (int w = 0; w < width; ++w)
      rows[(long) (nlocal + g) * width + w] = rows[(long) owner[g] * width + w];
}

void orc_reverse_rows_f32(float *rows, int width, int nlocal, int nghost, const int *owner)
{
  for (int g = 0; g < nghost; ++g)
    for (int w = 0; w < width; ++w) {
      rows[(long) owner[g] * width + w] += rows[(long) (nlocal + g) * width + w];
      rows[(long) (nlocal + g) * width + w] = 0.0f;
    }
}

#define REAL double
#define SUF(name) name##_f64
#include "eam_oracle_impl.h"
#undef REAL
#undef SUF

#define REAL float
#define SUF(name) name##_f32
#include "eam_oracle_impl.h"
#undef REAL
#undef SUF
