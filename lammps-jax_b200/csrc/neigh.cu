// Device neighbor-list build for the harness: one thread per owned atom scans a +-2 stencil of
// bins (bin side >= cutoff / 2) and writes its row in Kokkos LayoutLeft, so a warp's 32 rows
// store each slot as one coalesced 128-byte line.

#include <cuda_runtime.h>

#include "ljx_neigh.h"

namespace {

struct Grid {
  double lo[3];
  double bin;
  double inv_bin;
  int nb[3];
};

__device__ __forceinline__ long long bin_of(const double *x, int i, const Grid &g)
{
  int c[3];
  for (int k = 0; k < 3; ++k) {
    const int v = static_cast<int>(floor((x[3 * i + k] - g.lo[k]) * g.inv_bin));
    c[k] = v < 0 ? 0 : (v >= g.nb[k] ? g.nb[k] - 1 : v);
  }
  return (static_cast<long long>(c[2]) * g.nb[1] + c[1]) * g.nb[0] + c[0];
}

// Counting sort of atoms into bins: count, exclusive scan (per-block scan, scan of the block
// sums, add back), fill through per-bin cursors, then order each bin by atom index so the lists
// come out the same on every run.
constexpr int kScanBlock = 1024;

__global__ void k_bin_count(const double *__restrict__ x, int nall, Grid g, int *count)
{
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nall; i += gridDim.x * blockDim.x)
    atomicAdd(count + bin_of(x, i, g), 1);
}

__global__ void k_scan_blocks(const int *__restrict__ count, long long nb, int *start,
                              int *block_sums)
{
  __shared__ int s[kScanBlock];
  const long long b = static_cast<long long>(blockIdx.x) * kScanBlock + threadIdx.x;
  const int v = b < nb ? count[b] : 0;
  s[threadIdx.x] = v;
  __syncthreads();
  for (int o = 1; o < kScanBlock; o <<= 1) {
    const int add = threadIdx.x >= o ? s[threadIdx.x - o] : 0;
    __syncthreads();
    s[threadIdx.x] += add;
    __syncthreads();
  }
  if (b < nb) start[b] = s[threadIdx.x] - v;  // exclusive within the block
  if (threadIdx.x == kScanBlock - 1) block_sums[blockIdx.x] = s[threadIdx.x];
}

__global__ void k_scan_sums(int *block_sums, int nblocks, int *total)
{
  if (threadIdx.x != 0) return;
  int run = 0;
  for (int k = 0; k < nblocks; ++k) {
    const int v = block_sums[k];
    block_sums[k] = run;
    run += v;
  }
  *total = run;
}

__global__ void k_scan_add(int *start, long long nb, const int *__restrict__ block_sums,
                           int *cursor)
{
  const long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const int v = start[b] + block_sums[b / kScanBlock];
  start[b] = v;
  cursor[b] = v;
}

__global__ void k_bin_fill(const double *__restrict__ x, int nall, Grid g, int *cursor,
                           int *bin_atoms)
{
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nall; i += gridDim.x * blockDim.x)
    bin_atoms[atomicAdd(cursor + bin_of(x, i, g), 1)] = i;
}

__global__ void k_bin_order(const int *__restrict__ start, long long nb, int *bin_atoms)
{
  const long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const int lo = start[b], hi = start[b + 1];
  for (int s = lo + 1; s < hi; ++s) {
    const int a = bin_atoms[s];
    int t = s - 1;
    while (t >= lo && bin_atoms[t] > a) {
      bin_atoms[t + 1] = bin_atoms[t];
      --t;
    }
    bin_atoms[t + 1] = a;
  }
}

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
  // Distance from the atom to the near face of bin b along one axis (0 inside the slab).
  auto gap = [&](int k, int b) {
    const double blo = g.lo[k] + b * g.bin, bhi = blo + g.bin;
    const double v = xyz[k];
    return v < blo ? blo - v : (v > bhi ? v - bhi : 0.0);
  };
  int n = 0;
  for (int dz = -2; dz <= 2; ++dz) {
    const int bz = c[2] + dz;
    if (bz < 0 || bz >= g.nb[2]) continue;
    const double gz = gap(2, bz);
    for (int dy = -2; dy <= 2; ++dy) {
      const int by = c[1] + dy;
      if (by < 0 || by >= g.nb[1]) continue;
      const double gy = gap(1, by);
      for (int dx = -2; dx <= 2; ++dx) {
        const int bx = c[0] + dx;
        if (bx < 0 || bx >= g.nb[0]) continue;
        // Bins whose box lies beyond the cutoff hold no neighbor (a little slack keeps the
        // pruning conservative against rounding).
        const double gx = gap(0, bx);
        if (gx * gx + gy * gy + gz * gz > cutsq * (1.0 + 1e-9)) continue;
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
  g.bin = binsize;
  g.inv_bin = 1.0 / binsize;
  auto s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(widest, 0, sizeof(int), s) != cudaSuccess) return LJX_ERR_CUDA;
  k_neigh_build<<<(nlocal + 127) / 128, 128, 0, s>>>(x, nlocal, cutoff * cutoff, half, g,
                                                     bin_start, bin_atoms, neighbors, slot_stride,
                                                     maxneigh, numneigh, widest);
  return cudaGetLastError() == cudaSuccess ? LJX_OK : LJX_ERR_CUDA;
}

extern "C" ljx_status ljx_neigh_bin(void *stream, const double *x, int nall, const double *lo,
                                    double binsize, const int *nbins, int *bin_start,
                                    int *bin_atoms, int *scratch)
{
  if (!x || !lo || !nbins || !bin_start || !bin_atoms || !scratch || nall < 0 || !(binsize > 0))
    return LJX_ERR_INVALID;
  Grid g;
  long long nb = 1;
  for (int k = 0; k < 3; ++k) {
    if (nbins[k] <= 0) return LJX_ERR_INVALID;
    g.lo[k] = lo[k];
    g.nb[k] = nbins[k];
    nb *= nbins[k];
  }
  g.bin = binsize;
  g.inv_bin = 1.0 / binsize;
  const long long nblocks = (nb + kScanBlock - 1) / kScanBlock;
  int *count = scratch;                // nb ints, then the per-bin cursors
  int *block_sums = scratch + nb;      // nblocks ints
  auto s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(count, 0, nb * sizeof(int), s) != cudaSuccess) return LJX_ERR_CUDA;
  const int flat = static_cast<int>(nall > 0 ? (nall + 255) / 256 : 1);
  if (nall > 0) k_bin_count<<<flat, 256, 0, s>>>(x, nall, g, count);
  k_scan_blocks<<<static_cast<unsigned>(nblocks), kScanBlock, 0, s>>>(count, nb, bin_start,
                                                                       block_sums);
  k_scan_sums<<<1, 32, 0, s>>>(block_sums, static_cast<int>(nblocks), bin_start + nb);
  k_scan_add<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, s>>>(bin_start, nb, block_sums,
                                                                     count);
  if (nall > 0) k_bin_fill<<<flat, 256, 0, s>>>(x, nall, g, count, bin_atoms);
  k_bin_order<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, s>>>(bin_start, nb, bin_atoms);
  return cudaGetLastError() == cudaSuccess ? LJX_OK : LJX_ERR_CUDA;
}
