// Device neighbor-list build for the harness: one thread per owned atom scans a +-2 stencil of
// bins (bin side >= cutoff / 2) and writes its row in Kokkos LayoutLeft, so a warp's 32 rows
// store each slot as one coalesced 128-byte line.

#include <cuda_runtime.h>

#include "ljx_neigh.h"

namespace {

struct Grid {
  double lo[3];
  double inv_bin;
  int nb[3];
};

__global__ void k_neigh_build(const double *__restrict__ x, int nlocal, double cutsq, int half,
                              Grid g, const int *__restrict__ bin_start,
                              const int *__restrict__ bin_atoms, int *__restrict__ neighbors,
                              long long stride, int maxneigh, int *__restrict__ numneigh,
                              int *__restrict__ widest)
{
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nlocal) return;
  const double xi = x[3 * i], yi = x[3 * i + 1], zi = x[3 * i + 2];
  int c[3];
  const double xyz[3] = {xi, yi, zi};
  for (int k = 0; k < 3; ++k) {
    int v = static_cast<int>(floor((xyz[k] - g.lo[k]) * g.inv_bin));
    c[k] = v < 0 ? 0 : (v >= g.nb[k] ? g.nb[k] - 1 : v);
  }
  int n = 0;
  for (int dz = -2; dz <= 2; ++dz) {
    const int bz = c[2] + dz;
    if (bz < 0 || bz >= g.nb[2]) continue;
    for (int dy = -2; dy <= 2; ++dy) {
      const int by = c[1] + dy;
      if (by < 0 || by >= g.nb[1]) continue;
      for (int dx = -2; dx <= 2; ++dx) {
        const int bx = c[0] + dx;
        if (bx < 0 || bx >= g.nb[0]) continue;
        const long long b = (static_cast<long long>(bz) * g.nb[1] + by) * g.nb[0] + bx;
        const int end = bin_start[b + 1];
        for (int s = bin_start[b]; s < end; ++s) {
          const int j = bin_atoms[s];
          if (j == i) continue;
          const double xj = x[3 * j], yj = x[3 * j + 1], zj = x[3 * j + 2];
          const double ex = xi - xj, ey = yi - yj, ez = zi - zj;
          if (ex * ex + ey * ey + ez * ez >= cutsq) continue;
          if (half) {
            if (j < nlocal) {
              if (j < i) continue;
            } else {
              if (zj < zi) continue;
              if (zj == zi) {
                if (yj < yi) continue;
                if (yj == yi && xj < xi) continue;
              }
            }
          }
          if (n < maxneigh) neighbors[i + static_cast<long long>(n) * stride] = j;
          ++n;
        }
      }
    }
  }
  numneigh[i] = n < maxneigh ? n : maxneigh;
  atomicMax(widest, n);
}

}  // namespace

extern "C" ljx_status ljx_neigh_build(void *stream, const double *x, int nall, int nlocal,
                                      double cutoff, int half, const double *lo, double binsize,
                                      const int *nbins, const int *bin_start,
                                      const int *bin_atoms, int *neighbors,
                                      long long slot_stride, int maxneigh, int *numneigh,
                                      int *widest)
{
  if (nlocal <= 0) return LJX_OK;
  if (!x || !lo || !nbins || !bin_start || !bin_atoms || !neighbors || !numneigh || !widest ||
      nall < nlocal || slot_stride < nlocal || maxneigh <= 0 || !(binsize >= 0.5 * cutoff) ||
      !(binsize > 0))
    return LJX_ERR_INVALID;
  Grid g;
  for (int k = 0; k < 3; ++k) {
    g.lo[k] = lo[k];
    g.nb[k] = nbins[k];
    if (nbins[k] <= 0) return LJX_ERR_INVALID;
  }
  g.inv_bin = 1.0 / binsize;
  auto s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(widest, 0, sizeof(int), s) != cudaSuccess) return LJX_ERR_CUDA;
  k_neigh_build<<<(nlocal + 127) / 128, 128, 0, s>>>(x, nlocal, cutoff * cutoff, half, g,
                                                     bin_start, bin_atoms, neighbors, slot_stride,
                                                     maxneigh, numneigh, widest);
  return cudaGetLastError() == cudaSuccess ? LJX_OK : LJX_ERR_CUDA;
}
