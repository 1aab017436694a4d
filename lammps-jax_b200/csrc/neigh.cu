// Device neighbor-list build for the harness: bins of side >= cutoff / 2 (counting sort on the
// device, ljx_neigh_bin, which also leaves a bin-ordered float copy of the positions), then one
// warp per bin scans the +-2 stencil (ljx_neigh_build) and writes the bin's rows in Kokkos
// LayoutLeft.

#include <cuda_runtime.h>

#include <algorithm>

#include "kernels.cuh"
#include "ljx_neigh.h"

namespace {

using ljx::FilterBand;
using ljx::filter_band;

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

// Also the largest |coordinate| (float bits, of the float-rounded values) into *bound, which the
// build's float distance test needs for its rounding band.
__global__ void k_bin_count(const double *__restrict__ x, int nall, Grid g, int *count,
                            unsigned int *bound)
{
  float big = 0.0f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nall; i += gridDim.x * blockDim.x) {
    atomicAdd(count + bin_of(x, i, g), 1);
    for (int k = 0; k < 3; ++k) big = fmaxf(big, fabsf(static_cast<float>(x[3 * i + k])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) big = fmaxf(big, __shfl_xor_sync(0xffffffffu, big, o));
  if ((threadIdx.x & 31) == 0) atomicMax(bound, __float_as_uint(big));
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

// Bin-ordered float copy of the positions: record s holds atom bin_atoms[s] as (x, y, z, the
// atom index's bits), so a stencil row's candidates are one contiguous run of records.
__global__ void k_bin_sorted(const double *__restrict__ x, int nall,
                             const int *__restrict__ bin_atoms, float4 *sorted)
{
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < nall; s += gridDim.x * blockDim.x) {
    const int j = bin_atoms[s];
    sorted[s] = make_float4(static_cast<float>(x[3 * j]), static_cast<float>(x[3 * j + 1]),
                            static_cast<float>(x[3 * j + 2]), __int_as_float(j));
  }
}

// LAMMPS's distance test rsq < cutsq in double (npair: delx = xtmp - x[j][0], rsq = delx*delx +
// dely*dely + delz*delz), without fused multiply-adds, for pairs the float test cannot decide.
__device__ __forceinline__ bool within_exact(const double *xi, const double *__restrict__ x, int j,
                                             double cutsq)
{
  const double ex = __dsub_rn(xi[0], x[3 * j]);
  const double ey = __dsub_rn(xi[1], x[3 * j + 1]);
  const double ez = __dsub_rn(xi[2], x[3 * j + 2]);
  return __dadd_rn(__dadd_rn(__dmul_rn(ex, ex), __dmul_rn(ey, ey)), __dmul_rn(ez, ez)) < cutsq;
}

// One warp per bin: the bin's owned atoms (in index order, up to kRowsPerPass at a time) are
// the rows; the atoms of the +-2 stencil are the candidates. For each (dy, dz) the five bins
// along x are consecutive, so their atoms form one run of the bin-ordered float copy, which the
// lanes read 32 records at a time (coalesced 16-byte loads). Each candidate is tested against
// every row (row positions are shared-memory broadcasts) in float; only a pair whose float r^2
// falls in the rounding band around the cutoff takes the exact double test. Kept neighbors
// append to the rows in shared memory in stencil order; slots past kRowCap go straight to
// global memory. The rows then leave slot-major, so one store covers the same slot of
// consecutive rows (LayoutLeft).
// Row staging capacity: 192 slots (24 KB per 4-warp block) measured faster than 256 (32 KB) at
// 214 and 261 neighbors per row (C3, C5), by more resident blocks; the slots past it go
// straight to global memory. 128 was slower again.
#ifndef LJX_NEIGH_ROW_CAP
#define LJX_NEIGH_ROW_CAP 192
#endif
#ifndef LJX_NEIGH_WARPS
#define LJX_NEIGH_WARPS 4
#endif
constexpr int kRowsPerPass = 8;
constexpr int kRowCap = LJX_NEIGH_ROW_CAP;
constexpr int kNeighWarps = LJX_NEIGH_WARPS;

// HALF: keep each pair once (owned j > i, a ghost j only if it sorts after i in (z, y, x)).
template <bool HALF>
__global__ void __launch_bounds__(kNeighWarps * 32)
k_neigh_bins(const double *__restrict__ x, int nall, int nlocal, double cutsq, Grid g,
             const int *__restrict__ bin_start, const int *__restrict__ bin_atoms,
             const float4 *__restrict__ sorted, int *__restrict__ neighbors, long long stride,
             int maxneigh, int *__restrict__ numneigh, int *__restrict__ widest)
{
  __shared__ int s_row[kNeighWarps][kRowsPerPass][kRowCap];
  __shared__ double s_xi[kNeighWarps][kRowsPerPass][3];
  __shared__ float4 s_xf[kNeighWarps][kRowsPerPass];
  __shared__ int s_i[kNeighWarps][kRowsPerPass];
  __shared__ int s_start[kNeighWarps][32];  // stencil row q: first entry in bin_atoms
  __shared__ int s_off[kNeighWarps][32];    // stencil row q: offset in the candidate stream
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  const long long nbins = static_cast<long long>(g.nb[0]) * g.nb[1] * g.nb[2];
  int (*rows)[kRowCap] = s_row[warp];
  double (*xis)[3] = s_xi[warp];
  float4 *xfs = s_xf[warp];
  int *is = s_i[warp];
  int wide = 0;
  // The largest |coordinate| sits in the record after the last atom.
  const FilterBand band = filter_band(cutsq, __float_as_uint(sorted[nall].x));
  for (long long b = static_cast<long long>(blockIdx.x) * kNeighWarps + warp; b < nbins;
       b += static_cast<long long>(gridDim.x) * kNeighWarps) {
    const int b0 = bin_start[b], b1 = bin_start[b + 1];
    // Owned atoms come first within a bin (index order).
    int owned = 0;
    for (int s0 = b0; s0 < b1; s0 += 32) {
      const bool own = s0 + lane < b1 && bin_atoms[s0 + lane] < nlocal;
      owned += __popc(__ballot_sync(0xffffffffu, own));
    }
    if (owned == 0) continue;
    const int bz = static_cast<int>(b / (static_cast<long long>(g.nb[0]) * g.nb[1]));
    const int by = static_cast<int>((b / g.nb[0]) % g.nb[1]);
    const int bx = static_cast<int>(b % g.nb[0]);
    for (int r0 = 0; r0 < owned; r0 += kRowsPerPass) {
      const int m = min(kRowsPerPass, owned - r0);
      if (lane < m) {
        const float4 rf = sorted[b0 + r0 + lane];
        const int i = __float_as_int(rf.w);
        is[lane] = i;
        xfs[lane] = rf;
        xis[lane][0] = x[3 * i];
        xis[lane][1] = x[3 * i + 1];
        xis[lane][2] = x[3 * i + 2];
      }
      __syncwarp();
      int count[kRowsPerPass] = {0, 0, 0, 0, 0, 0, 0, 0};
      // The 25 (dy, dz) rows of the stencil, in (dz, dy) order, one per lane: the bins
      // bx-2 .. bx+2 of a row are consecutive, so their atoms are one range of bin_atoms. The
      // ranges are walked as one stream of candidates, 32 at a time, so no batch is left mostly
      // empty at the end of a short range (about 33 atoms per range at solid densities).
      int start = 0, len = 0;
      if (lane < 25) {
        const int dz = lane / 5 - 2, dy = lane % 5 - 2;
        const int cz = bz + dz, cy = by + dy;
        // Bins wider than cutoff / 2 can put a whole (dy, dz) row of bins out of range.
        const double gy = (dy > 1 ? dy - 1 : (dy < -1 ? -dy - 1 : 0)) * g.bin;
        const double gz = (dz > 1 ? dz - 1 : (dz < -1 ? -dz - 1 : 0)) * g.bin;
        if (cz >= 0 && cz < g.nb[2] && cy >= 0 && cy < g.nb[1] &&
            !(gy * gy + gz * gz > cutsq * (1.0 + 1e-9))) {
          const long long row0 = (static_cast<long long>(cz) * g.nb[1] + cy) * g.nb[0];
          start = bin_start[row0 + max(bx - 2, 0)];
          len = bin_start[row0 + min(bx + 2, g.nb[0] - 1) + 1] - start;
        }
      }
      int incl = len;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const int total = __shfl_sync(0xffffffffu, incl, 31);
      s_start[warp][lane] = start;
      s_off[warp][lane] = incl - len;
      __syncwarp();
      // Candidate k's stencil row is the last row whose offset is <= k (empty rows share their
      // offset with the next one, so they are never the last). A lane's k grows by 32 per
      // batch, about one row, so the row only moves forward; the next batch's atom and position
      // are fetched before this batch's tests, so their latency overlaps them.
      int q = 0;
      // Past the stream's end a lane holds an atom at infinity (index -1), which no row keeps.
      auto fetch = [&](int k, float4 &c) {
        c = make_float4(INFINITY, INFINITY, INFINITY, __int_as_float(-1));
        if (k < total) {
          while (q < 24 && s_off[warp][q + 1] <= k) ++q;
          c = sorted[s_start[warp][q] + (k - s_off[warp][q])];
        }
      };
      float4 cn;
      fetch(lane, cn);
      for (int s0 = 0; s0 < total; s0 += 32) {
        const float4 c = cn;
        const int j = __float_as_int(c.w);
        fetch(s0 + 32 + lane, cn);
#pragma unroll
        for (int r = 0; r < kRowsPerPass; ++r) {
          if (r >= m) continue;  // m is the same for every lane
          const int i = is[r];
          const float4 rf = xfs[r];
          const float dx = rf.x - c.x, dy = rf.y - c.y, dz = rf.z - c.z;
          const float r2f = dx * dx + dy * dy + dz * dz;
          bool keep = j != i && r2f <= band.hi;
          // Predicated: the rare pair inside the band takes the double test under a warp vote,
          // so the common batch runs without divergent branches.
          const bool unsure = keep && r2f >= band.lo;
          if (__any_sync(0xffffffffu, unsure)) {
            if (unsure) keep = within_exact(xis[r], x, j, cutsq);
          }
          if constexpr (HALF) {
            if (keep) {
              if (j < nlocal) {
                keep = j > i;
              } else {
                const double zi = xis[r][2], yi = xis[r][1], xi = xis[r][0];
                const double xj = x[3 * j], yj = x[3 * j + 1], zj = x[3 * j + 2];
                keep = !(zj < zi || (zj == zi && (yj < yi || (yj == yi && xj < xi))));
              }
            }
          }
          const unsigned mk = __ballot_sync(0xffffffffu, keep);
          const int slot = count[r] + __popc(mk & below);
          if (keep && slot < kRowCap) rows[r][slot] = j;
          if (keep && slot >= kRowCap && slot < maxneigh)
            neighbors[i + static_cast<long long>(slot) * stride] = j;
          count[r] += __popc(mk);
        }
      }
      __syncwarp();
      // Slot-major write-out: lane l takes row l % 8 at slot n + l / 8.
      int longest = 0;
#pragma unroll
      for (int r = 0; r < kRowsPerPass; ++r) longest = max(longest, r < m ? count[r] : 0);
      const int r = lane % kRowsPerPass;
      int mine = 0;
#pragma unroll
      for (int rr = 0; rr < kRowsPerPass; ++rr)
        if (rr == r && rr < m) mine = count[rr];
      const int stop = min(min(longest, kRowCap), maxneigh);
      for (int n0 = 0; n0 < stop; n0 += 32 / kRowsPerPass) {
        const int n = n0 + lane / kRowsPerPass;
        if (r < m && n < mine && n < stop)
          neighbors[is[r] + static_cast<long long>(n) * stride] = rows[r][n];
      }
      if (lane < m) {
        numneigh[is[lane]] = min(mine, maxneigh);
        wide = max(wide, mine);
      }
      __syncwarp();
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wide = max(wide, __shfl_xor_sync(0xffffffffu, wide, o));
  if (lane == 0 && wide > 0) atomicMax(widest, wide);
}

}  // namespace

extern "C" ljx_status ljx_neigh_build(void *stream, const double *x, int nall, int nlocal,
                                      double cutoff, int half, const double *lo, double binsize,
                                      const int *nbins, const int *bin_start,
                                      const int *bin_atoms, const void *sorted, int *neighbors,
                                      long long slot_stride, int maxneigh, int *numneigh,
                                      int *widest)
{
  if (nlocal <= 0) return LJX_OK;
  if (!x || !lo || !nbins || !bin_start || !bin_atoms || !sorted || !neighbors || !numneigh ||
      !widest ||
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
  const long long nb = static_cast<long long>(g.nb[0]) * g.nb[1] * g.nb[2];
  const long long blocks = std::min<long long>((nb + kNeighWarps - 1) / kNeighWarps, 148LL * 64);
  auto kernel = half ? k_neigh_bins<true> : k_neigh_bins<false>;
  kernel<<<static_cast<unsigned>(blocks), kNeighWarps * 32, 0, s>>>(
      x, nall, nlocal, cutoff * cutoff, g, bin_start, bin_atoms,
      static_cast<const float4 *>(sorted), neighbors, slot_stride, maxneigh, numneigh, widest);
  return cudaGetLastError() == cudaSuccess ? LJX_OK : LJX_ERR_CUDA;
}

extern "C" ljx_status ljx_neigh_bin(void *stream, const double *x, int nall, const double *lo,
                                    double binsize, const int *nbins, int *bin_start,
                                    int *bin_atoms, int *scratch, void *sorted)
{
  if (!x || !lo || !nbins || !bin_start || !bin_atoms || !scratch || !sorted || nall < 0 ||
      !(binsize > 0))
    return LJX_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(sorted) % alignof(float4) != 0) return LJX_ERR_INVALID;
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
  float4 *records = static_cast<float4 *>(sorted);
  // The record after the last atom carries the largest |coordinate| (float bits in .x).
  unsigned int *bound = reinterpret_cast<unsigned int *>(records + nall);
  if (cudaMemsetAsync(count, 0, nb * sizeof(int), s) != cudaSuccess ||
      cudaMemsetAsync(records + nall, 0, sizeof(float4), s) != cudaSuccess)
    return LJX_ERR_CUDA;
  const int flat = static_cast<int>(nall > 0 ? (nall + 255) / 256 : 1);
  if (nall > 0) k_bin_count<<<flat, 256, 0, s>>>(x, nall, g, count, bound);
  k_scan_blocks<<<static_cast<unsigned>(nblocks), kScanBlock, 0, s>>>(count, nb, bin_start,
                                                                       block_sums);
  k_scan_sums<<<1, 32, 0, s>>>(block_sums, static_cast<int>(nblocks), bin_start + nb);
  k_scan_add<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, s>>>(bin_start, nb, block_sums,
                                                                     count);
  if (nall > 0) k_bin_fill<<<flat, 256, 0, s>>>(x, nall, g, count, bin_atoms);
  k_bin_order<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, s>>>(bin_start, nb, bin_atoms);
  if (nall > 0) k_bin_sorted<<<flat, 256, 0, s>>>(x, nall, bin_atoms, records);
  return cudaGetLastError() == cudaSuccess ? LJX_OK : LJX_ERR_CUDA;
}
