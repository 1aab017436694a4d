// Device kernels of the ljx engine (sm_100a). One warp owns one LAMMPS list row at a time
// ("warp per row"): lanes take consecutive slots, a ballot compacts the kept pairs, per-row sums
// finish with warp shuffles, and only scatters to a neighbor's row (half lists, newton-on ghost
// rows) use atomics. Grids are persistent: a multiple of the SM count, warps stride over rows.
// The row-group density pass over the candidate cache lives in groups.cuh; k_density here is the
// list pass (cache off, and the compaction behind ljx_pack_edges).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ljx {

constexpr int kWarp = 32;
constexpr int kBlock = 256;
constexpr int kWarpsPerBlock = kBlock / kWarp;
constexpr unsigned kFull = 0xffffffffu;
// LAMMPS keeps special-bond flags in the top bits of neighbor indices.
constexpr int kNeighMask = 0x1FFFFFFF;
// One block's partial sums: [0] energy, [1..6] virial, [7] kept pairs, [8] widest row (max).
constexpr int kPartialWidth = 10;
// List slots of one row staged in shared memory per block row-group (longer rows read the rest
// straight from global memory), and the per-warp queue of kept pairs.
constexpr int kTileSlots = 384;
constexpr int kQueue = 64;
// Minimum resident blocks per SM requested from the compiler for the two row kernels (caps
// their registers per thread); 0 leaves the choice to the compiler.
#ifndef LJX_DENSITY_MIN_BLOCKS
#define LJX_DENSITY_MIN_BLOCKS 7
#endif
#ifndef LJX_FORCE_MIN_BLOCKS
#define LJX_FORCE_MIN_BLOCKS 4
#endif
#if LJX_DENSITY_MIN_BLOCKS > 0
#define LJX_DENSITY_BOUNDS __launch_bounds__(kBlock, LJX_DENSITY_MIN_BLOCKS)
#else
#define LJX_DENSITY_BOUNDS __launch_bounds__(kBlock)
#endif
// The force pass: 4 blocks of 256 per SM (64 registers); the double half-list variant, which
// spills at 64, runs 3 (80 registers) and is faster for it. Force-only passes (no energy or
// virial sums) hold 14 fewer registers per thread.
#ifndef LJX_FORCE_EV_PRELOAD
#define LJX_FORCE_EV_PRELOAD 0
#endif
#ifndef LJX_FORCE_ONLY_MIN_BLOCKS
#define LJX_FORCE_ONLY_MIN_BLOCKS 4
#endif
#define LJX_FORCE_BOUNDS                                                                   \
  __launch_bounds__(kBlock, TALLY ? 2                                                       \
                            : (sizeof(T) == 8 && MODE == kHalf) ? 3                         \
                            : !EV ? LJX_FORCE_ONLY_MIN_BLOCKS : LJX_FORCE_MIN_BLOCKS)

// Density modes. kDensityHalfOwned: a full list with newton off whose rows keep only owned
// neighbors j > i and all ghosts (the filter's half rule); each owned pair is evaluated once and
// its share added to both rows, ghost pairs (also listed from the image's owner) to row i alone.
enum DensityMode { kDensityFull = 0, kDensityHalf = 1, kCompactOnly = 2, kDensityHalfOwned = 3 };
// Force distribution modes.
//  kRowsFull       : full list, newton off; row i takes the whole pair force, no scatter.
//  kGhost          : full list, newton on, plain bundle; each edge carries F'(rho_i) rho_j' +
//                    phi'/2 to both endpoints (the autodiff of the plain energy program).
//  kHalf           : half list, newton on; whole pair force, sender +, receiver -.
//  kRowsHalfOwned  : the rows of kDensityHalfOwned; an owned pair's force goes to both atoms
//                    (Newton's third law; the neighbor's share by atomics) and its energy and
//                    virial count for both directions, a ghost pair's to row i alone. The same
//                    pairs, forces, energy and virial as kRowsFull, from about half the pairs.
enum ForceMode { kRowsFull = 0, kGhost = 1, kHalf = 2, kRowsHalfOwned = 3 };
enum LjMode { kLjEdgeFull = 0, kLjEdgeHalf = 1, kLjAtomFull = 2, kLjAtomHalfPairSum = 3 };
enum RowPart { kRowsAll = 0, kRowsLocal = 1, kRowsGhost = 2 };

template <typename T> struct Vec4;
template <> struct Vec4<float> { using type = float4; };
template <> struct Vec4<double> { using type = double4; };

// One 32-byte record per lane in a single request (sm_100 256-bit vector load through the
// read-only path). Only used on data no kernel writes while the reading kernel runs.
__device__ __forceinline__ double4 load4(const double4 *p)
{
  double4 v;
  asm("ld.global.nc.v4.f64 {%0, %1, %2, %3}, [%4];"
      : "=d"(v.x), "=d"(v.y), "=d"(v.z), "=d"(v.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ float4 load4(const float4 *p) { return __ldg(p); }

// Spline-table rows: the tables (a few hundred KB in all) are re-read by every pair, while the
// position and list data stream through L1; with LJX_L1_HINTS the table rows are kept in L1 in
// preference (evict_last) and the once-read list words are dropped first (evict_first).
#ifndef LJX_L1_HINTS
#define LJX_L1_HINTS 2
#endif
__device__ __forceinline__ double4 load4_tab(const double4 *p)
{
#if LJX_L1_HINTS >= 1
  double4 v;
  asm("ld.global.nc.L1::evict_last.v4.f64 {%0, %1, %2, %3}, [%4];"
      : "=d"(v.x), "=d"(v.y), "=d"(v.z), "=d"(v.w)
      : "l"(p));
  return v;
#else
  return load4(p);
#endif
}
__device__ __forceinline__ float4 load4_tab(const float4 *p)
{
#if LJX_L1_HINTS >= 1
  float4 v;
  asm("ld.global.nc.L1::evict_last.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p));
  return v;
#else
  return __ldg(p);
#endif
}
template <typename W>
__device__ __forceinline__ W load_once(const W *p)
{
#if LJX_L1_HINTS >= 2
  static_assert(sizeof(W) == 4 || sizeof(W) == 2, "list words");
  if constexpr (sizeof(W) == 4) {
    unsigned v;
    asm("ld.global.nc.L1::evict_first.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return *reinterpret_cast<W *>(&v);
  } else {
    unsigned short v;
    asm("ld.global.nc.L1::evict_first.b16 %0, [%1];" : "=h"(v) : "l"(p));
    return *reinterpret_cast<W *>(&v);
  }
#else
  return __ldg(p);
#endif
}

template <typename T>
struct Step {
  // LAMMPS arrays.
  const double *x;
  const int *type;
  double *f;
  int nlocal;
  int nghost;
  int nall;
  // LAMMPS list.
  const int *ilist;
  const int *numneigh;
  const int *neighbors;
  long long atom_stride;
  long long slot_stride;
  int inum;
  int maxneighs;
  // Engine buffers.
  double4 *xd4;                       // x, y, z, species (double), rows < max_atoms
  typename Vec4<T>::type *pos4;       // contract-precision copy (float runs only)
  T *rho;
  T *fp;
  int *cedges;                        // compacted rows: row * row_cap + slot
  int *ccount;                        // kept pairs per row (may exceed row_cap: spilled row)
  int row_cap;
  // Tables: [n_el][n][4] at contract precision.
  const typename Vec4<T>::type *embedding;
  const typename Vec4<T>::type *density;
  const typename Vec4<T>::type *density_slope;  // (c1, 2 c2, 3 c3, 0) / dr per node
  const typename Vec4<T>::type *pair;
  int n_species;                      // table count; species clamp to [0, n_species)
  int nrho;
  int nr;
  T drho;
  T inv_dr;
  // Cutoffs: the pack filter is the reference's double test (r^2 <= rc^2 from LAMMPS x); the
  // model keeps r^2 < rc^2 at contract precision.
  double pack_cutsq;
  T model_cutsq;
  int max_atoms;
  int half_rule;                      // drop j < i (half-edge bundle on a full list)
  int unique_rule;                    // keep a ghost j only if it sorts after i in (z, y, x)
  double scale;
  // LJ.
  T lj_four_eps;
  T lj_sigma_sq;
  T lj_energy_scale;
  // Largest |coordinate| of this step's atoms (float bits), for the float pre-filter bound.
  unsigned int *coord_bound;
  // Row-group candidate cache (groups.cuh): positions when the cache was built, the largest
  // squared displacement since (float bits, rounded up; zeroed with coord_bound), per group of
  // kGroupRows list rows the union of their neighbors (gatom, gcount), and per row its
  // candidates as slots into its group's union (rslot, rcount).
  double4 *xref;
  unsigned int *disp_bound;
  int *gatom;
  int *gcount;
  int gcap;
  unsigned short *rslot;
  int *rcount;
  int rcap;
  // Per-block partial sums.
  double *partials;
  // Per-atom tallies (LAMMPS eatom[nall], vatom[nall][6]; null when not asked for), accumulated
  // with += times tally_scale.
  double *eatom;
  double *vatom;
  double tally_scale;
  // Per list row: 1 when the row keeps a ghost neighbor (written by the density passes). The
  // force pass takes every row (kRowsAll), or only the rows without (kRowsLocal: they need no
  // ghost F', so they can run while the F' exchange is in flight) or with one (kRowsGhost).
  unsigned char *ghost_rows;
  int row_part;
};

__device__ __forceinline__ double warp_sum(double v)
{
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Distance from r^2 for the density spline: r^2 times its reciprocal square root, as the force
// pass forms r. Within 2 ulp of the rounded square root and cheaper than it (measured: density
// phase -2 % at C3).
template <typename T>
__device__ __forceinline__ T pair_distance(T r2)
{
  return r2 > T(0) ? r2 * rsqrt(r2) : T(0);
}

// Warp sums of three per-lane values in 6 exchange steps instead of 15. The first step swaps
// half of (a, b) / (c, 0) between the two half-warps, the second keeps one of the two remaining
// partials per quarter; afterwards each group of 8 lanes sums one of a, b, c, 0. The total of a
// is in lane 0, of b in lane 8 and of c in lane 16.
template <typename T>
__device__ __forceinline__ T warp_sum3(T a, T b, T c, int lane)
{
  const bool hi16 = (lane & 16) != 0;
  const T k0 = (hi16 ? c : a) + __shfl_xor_sync(kFull, hi16 ? a : c, 16);
  const T k1 = (hi16 ? T(0) : b) + __shfl_xor_sync(kFull, hi16 ? b : T(0), 16);
  const bool hi8 = (lane & 8) != 0;
  T m = (hi8 ? k1 : k0) + __shfl_xor_sync(kFull, hi8 ? k0 : k1, 8);
  m += __shfl_xor_sync(kFull, m, 4);
  m += __shfl_xor_sync(kFull, m, 2);
  m += __shfl_xor_sync(kFull, m, 1);
  return m;
}

// Reduce the thread's {energy, virial[6], kept} sums and widest row over the block and store
// one partial row (every slot written, so the finalize step can sum all kernels uniformly).
__device__ __forceinline__ void store_partials(double (&v)[8], int widest, double *partials)
{
  __shared__ double sm[kWarpsPerBlock][9];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = warp_sum(v[k]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) widest = max(widest, __shfl_xor_sync(kFull, widest, o));
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < 8; ++k) sm[warp][k] = v[k];
    sm[warp][8] = static_cast<double>(widest);
  }
  __syncthreads();
  if (threadIdx.x < kPartialWidth) {
    const int k = threadIdx.x;
    double s = 0.0;
    if (k < 8) {
      for (int w = 0; w < kWarpsPerBlock; ++w) s += sm[w][k];
    } else if (k == 8) {
      for (int w = 0; w < kWarpsPerBlock; ++w) s = fmax(s, sm[w][8]);
    }
    partials[static_cast<long long>(blockIdx.x) * kPartialWidth + k] = s;
  }
}

// Value and slope of one spline table at x (python/lammps_jax/eam.py:138-164 without
// extrapolation): node = clip(floor(x/delta), 0, n-2), t = min(x/delta - node, 1).
template <typename T>
__device__ __forceinline__ void spline_vs(const typename Vec4<T>::type *tab, int n, T x,
                                          T inv_delta, T &v, T &s)
{
  const T idx = x * inv_delta;
  T fl = floor(idx);
  fl = fmin(fmax(fl, T(0)), T(n - 2));
  const T t = fmin(idx - fl, T(1));
  const auto c = load4_tab(tab + static_cast<int>(fl));
  v = c.x + t * (c.y + t * (c.z + t * c.w));
  s = (c.y + t * (T(2) * c.z + t * (T(3) * c.w))) * inv_delta;
}

template <typename T>
__device__ __forceinline__ T spline_v(const typename Vec4<T>::type *tab, int n, T x, T inv_delta)
{
  const T idx = x * inv_delta;
  T fl = floor(idx);
  fl = fmin(fmax(fl, T(0)), T(n - 2));
  const T t = fmin(idx - fl, T(1));
  const auto c = load4_tab(tab + static_cast<int>(fl));
  return c.x + t * (c.y + t * (c.z + t * c.w));
}

// spline_v at a distance (x >= 0), where the node's lower clamp is a no-op and is left out, as
// in the force pass (the same node, t and value; cached C3 density phase 1.999 -> 1.956 ms).
template <typename T>
__device__ __forceinline__ T spline_v_dist(const typename Vec4<T>::type *tab, int n, T x,
                                           T inv_delta)
{
  const T idx = x * inv_delta;
  const T fl = fmin(floor(idx), T(n - 2));
  const T t = fmin(idx - fl, T(1));
  const auto c = load4_tab(tab + static_cast<int>(fl));
  return c.x + t * (c.y + t * (c.z + t * c.w));
}

template <typename T>
__device__ __forceinline__ T spline_s(const typename Vec4<T>::type *tab, int n, T x, T inv_delta)
{
  const T idx = x * inv_delta;
  T fl = floor(idx);
  fl = fmin(fmax(fl, T(0)), T(n - 2));
  const T t = fmin(idx - fl, T(1));
  const auto c = load4_tab(tab + static_cast<int>(fl));
  return (c.y + t * (T(2) * c.z + t * (T(3) * c.w))) * inv_delta;
}

__device__ __forceinline__ int pair_row(int a, int b)
{
  const int hi = a > b ? a : b, lo = a > b ? b : a;
  return hi * (hi + 1) / 2 + lo;
}

// r^2 of the reference's distance filter, formed without fused multiply-adds so it is the same
// double the reference computes (cpp/pair_jax_kokkos.cpp:88-91).
__device__ __forceinline__ double pack_r2(const double4 &xi, const double4 &xj)
{
  const double dx = __dsub_rn(xi.x, xj.x);
  const double dy = __dsub_rn(xi.y, xj.y);
  const double dz = __dsub_rn(xi.z, xj.z);
  return __dadd_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)), __dmul_rn(dz, dz));
}

// The reference's pairing rules for a pair within the cutoff (cpp/pair_jax_kokkos.cpp:92-101):
// the j < i half rule, and the unique-boundary rule that keeps a ghost j only if it sorts after
// i in (z, y, x).
template <typename T>
__device__ __forceinline__ bool pair_rules(const Step<T> &p, int i, const double4 &xi, int j,
                                           const double4 &xj)
{
  if (p.half_rule && j < i) return false;
  if (p.unique_rule && j >= p.nlocal) {
    if (xj.z < xi.z) return false;
    if (xj.z == xi.z) {
      if (xj.y < xi.y) return false;
      if (xj.y == xi.y && xj.x < xi.x) return false;
    }
  }
  return true;
}

// The reference's keep decision for list slot (i -> j), cpp/pair_jax_kokkos.cpp:84-101.
template <typename T>
__device__ __forceinline__ bool pack_keep(const Step<T> &p, int i, const double4 &xi, int j,
                                          const double4 &xj)
{
  return pack_r2(xi, xj) <= p.pack_cutsq && pair_rules(p, i, xi, j, xj);
}

// a1: LAMMPS x/type -> xd4 and its float copy (cpp/pair_jax_kokkos.cpp:35-52), plus the
// largest |coordinate| and, when a candidate cache exists, the largest squared displacement since
// it was built (atomic max on float bits; both words are zeroed before the launch).
template <typename T>
__global__ void __launch_bounds__(kBlock) k_pack_atoms(const Step<T> p, int span)
{
  float big = 0.0f;
  double moved = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < span; i += gridDim.x * blockDim.x) {
    const double x0 = p.x[3 * i], x1 = p.x[3 * i + 1], x2 = p.x[3 * i + 2];
    if (p.xref != nullptr) {
      const double4 r = p.xref[i];
      const double d0 = x0 - r.x, d1 = x1 - r.y, d2 = x2 - r.z;
      moved = fmax(moved, d0 * d0 + d1 * d1 + d2 * d2);
    }
    // Types past the table map to the last species (the clamped gather of the reference model).
    const int s = min(max(p.type[i] - 1, 0), p.n_species - 1);
    p.xd4[i] = make_double4(x0, x1, x2, static_cast<double>(s));
    const float4 f = make_float4(static_cast<float>(x0), static_cast<float>(x1),
                                 static_cast<float>(x2), static_cast<float>(s));
    reinterpret_cast<float4 *>(p.pos4)[i] = f;
    big = fmaxf(big, fmaxf(fabsf(f.x), fmaxf(fabsf(f.y), fabsf(f.z))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) big = fmaxf(big, __shfl_xor_sync(kFull, big, o));
  if ((threadIdx.x & 31) == 0) atomicMax(p.coord_bound, __float_as_uint(big));
  if (p.xref != nullptr) {
    // Rounded up, so the float never understates the displacement (non-negative floats order
    // like their bit patterns).
    float m = __double2float_ru(moved);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(p.disp_bound, __float_as_uint(m));
  }
}

// Band around rc^2 inside which a float r^2 cannot decide the reference's double test
// r^2 <= rc^2. Float coordinates carry at most u|x| rounding (u = 2^-24, |x| <= X), so a float
// difference is off by E <= 2uX' + u(R + 2uX') for |d| <= R, and the float r^2 by at most
// 2 sqrt(3) R E + 3 E^2 + 4 u R^2 (three rounded products and two rounded sums). The band is
// twice that plus 1e-6 R^2; pairs inside it take the exact double test.
struct FilterBand {
  float lo;  // float r^2 below: certainly kept
  float hi;  // float r^2 above: certainly dropped
};

__device__ __forceinline__ FilterBand filter_band(double cutsq, unsigned int bound_bits)
{
  const double u = 5.9604644775390625e-8;
  const double X = static_cast<double>(__uint_as_float(bound_bits)) * (1.0 + 4.0 * u);
  const double R = sqrt(cutsq) + 1.0;
  const double E = 2.0 * u * X + u * (R + 2.0 * u * X);
  const double d = 2.0 * (2.0 * 1.7320508075688772 * R * E + 3.0 * E * E + 4.0 * u * R * R) +
                   1e-6 * R * R;
  FilterBand b;
  b.lo = static_cast<float>(cutsq - d);
  b.hi = static_cast<float>(cutsq + d);
  return b;
}

// The reference's keep decision for list pair (i -> j) given its float r^2 (from the float copy
// of the positions) and the band around rc^2: the float value decides outside the band, the
// double test inside it and wherever the unique-boundary rule needs coordinates.
template <typename T>
__device__ __forceinline__ bool keep_pair(const Step<T> &p, const FilterBand &band, float r2f,
                                          int i, const double4 &xi, int j, const double4 &xj)
{
  if (r2f > band.hi) return false;
  if (r2f < band.lo && !p.unique_rule) return !(p.half_rule && j < i);
  return pack_keep(p, i, xi, j, xj);
}

// a2 + a6: filter and compact each list row, accumulating the EAM density.
//
// A block takes 8 consecutive list rows at a time (one per warp). The rows' list slots are first
// staged in shared memory: with the Kokkos LayoutLeft list, slot s of 8 consecutive rows is one
// 32-byte sector, so the staging load is coalesced where a warp walking one row directly would
// touch a different cache line per lane. Each warp then filters its row 32 slots at a time
// (reference distance test and pairing rules). In double runs a ballot appends the kept pairs
// to a per-warp queue in shared memory; every 32 queued pairs are written out as one coalesced
// segment of the compacted row and evaluated by all 32 lanes together (32-byte position gather,
// sqrt, density spline), so that work runs at full lane occupancy instead of at the ~40% keep
// rate. Float runs gather only a species word per kept pair and evaluate kept pairs in place.
template <typename T, int MODE>
__global__ void LJX_DENSITY_BOUNDS k_density(const Step<T> p)
{
  __shared__ int s_tile[kTileSlots][kWarpsPerBlock + 1];
  __shared__ int s_row_i[kWarpsPerBlock];
  __shared__ int s_row_n[kWarpsPerBlock];
  __shared__ int s_qj[kWarpsPerBlock][kQueue];
  __shared__ float s_qr2[kWarpsPerBlock][kQueue];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  int *qj = s_qj[warp];
  float *qr2 = s_qr2[warp];
  double kept_sum = 0.0;
  int widest = 0;
  const int groups = (p.inum + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const bool slot_major = p.atom_stride == 1;
  const FilterBand band = filter_band(p.pack_cutsq, *p.coord_bound);
  const bool exact_rules = p.unique_rule != 0;
  const float4 *pos4f = reinterpret_cast<const float4 *>(p.pos4);
  for (int g = blockIdx.x; g < groups; g += gridDim.x) {
    const int row0 = g * kWarpsPerBlock;
    if (threadIdx.x < kWarpsPerBlock) {
      const int row = row0 + threadIdx.x;
      int i = -1, n = 0;
      if (row < p.inum) {
        i = p.ilist[row];
        if (i < p.max_atoms) {
          const int listed = p.numneigh[i];
          widest = max(widest, listed);
          n = min(listed, p.maxneighs);
        } else {
          i = -1;
        }
      }
      s_row_i[threadIdx.x] = i;
      s_row_n[threadIdx.x] = n;
    }
    __syncthreads();
    int wmax = 0;
#pragma unroll
    for (int r = 0; r < kWarpsPerBlock; ++r) wmax = max(wmax, min(s_row_n[r], kTileSlots));
    for (int t = threadIdx.x; t < wmax * kWarpsPerBlock; t += kBlock) {
      const int r = slot_major ? t % kWarpsPerBlock : t / wmax;
      const int sl = slot_major ? t / kWarpsPerBlock : t % wmax;
      const int ii = s_row_i[r];
      if (ii >= 0 && sl < s_row_n[r])
        s_tile[sl][r] = p.neighbors[static_cast<long long>(ii) * p.atom_stride +
                                    static_cast<long long>(sl) * p.slot_stride] & kNeighMask;
    }
    __syncthreads();
    const int row = row0 + warp;
    const int i = s_row_i[warp];
    const int n = s_row_n[warp];
    if (row < p.inum && i < 0 && lane == 0) {
      p.ccount[row] = 0;
      p.ghost_rows[row] = 0;
    }
    if (row < p.inum && i >= 0) {
      const double4 xi = load4(p.xd4 + i);
      const float4 fi = __ldg(pos4f + i);
      bool ghost = false;  // this lane kept a ghost neighbor
      const int si = static_cast<int>(xi.w);
      int *crow = p.cedges + static_cast<long long>(row) * p.row_cap;
      const long long rowbase = static_cast<long long>(i) * p.atom_stride;
      T rho = T(0);
      int kept = 0;  // pairs already written out
      int kept_twice = 0;
      int q = 0;     // pairs waiting in the queue
      // Write out kept pair (i -> j) at `slot` of the compacted row and add its density.
      auto evaluate = [&](int slot, int j, float r2f) {
        if (MODE == kCompactOnly) {
          if (slot < p.row_cap) crow[slot] = j;
        } else {
          T r2;
          int sj;
          if constexpr (sizeof(T) == 8) {
            // The model's double r^2 is the reference's pack r^2 (same operands and order).
            const double4 xj = load4(p.xd4 + j);
            r2 = pack_r2(xi, xj);
            sj = static_cast<int>(xj.w);
          } else {
            r2 = r2f;
            sj = static_cast<int>(__ldg(&pos4f[j].w));
          }
          if (slot < p.row_cap) crow[slot] = j;
          if (r2 < p.model_cutsq) {
            const T r = pair_distance(r2);
            // f_sj(r) to row i; f_si(r) to the neighbor, the same value for a same-species pair.
            const T fj = spline_v_dist<T>(p.density + sj * p.nr, p.nr, r, p.inv_dr);
            rho += fj;
            if (MODE == kDensityHalf || (MODE == kDensityHalfOwned && j < p.nlocal))
              atomicAdd(p.rho + j, si == sj ? fj
                                            : spline_v_dist<T>(p.density + si * p.nr, p.nr, r,
                                                               p.inv_dr));
          }
        }
      };
      // Write out and evaluate the first `count` queued pairs (count <= 32), then drop them.
      auto flush = [&](int count) {
        __syncwarp();
        int j = 0;
        float r2f = 0.0f;
        if (lane < count) {
          j = qj[lane];
          r2f = qr2[lane];
        }
        int tj = 0;
        float tr2 = 0.0f;
        const int rest = q - count;
        if (lane < rest) {
          tj = qj[count + lane];
          tr2 = qr2[count + lane];
        }
        __syncwarp();
        if (lane < rest) {
          qj[lane] = tj;
          qr2[lane] = tr2;
        }
        __syncwarp();
        if (lane < count) evaluate(kept + lane, j, r2f);
        kept += count;
        q = rest;
      };
      for (int base = 0; base < n; base += kWarp) {
        const int jj = base + lane;
        int j = 0;
        bool keep = false;
        float r2f = 0.0f;
        if (jj < n) {
          j = jj < kTileSlots ? s_tile[jj][warp]
                              : (p.neighbors[rowbase + static_cast<long long>(jj) * p.slot_stride] &
                                 kNeighMask);
          // The half rule needs only the indices: a dropped pair costs no position gather
          // (rows that hold owned pairs once drop about half their list this way).
          if (j < p.max_atoms && !(p.half_rule && j < i)) {
            // Float pre-filter; only pairs inside the rounding band, or rows that need the
            // unique-boundary coordinate rule, read the double coordinates.
            const float4 fj = __ldg(pos4f + j);
            const float dx = fj.x - fi.x, dy = fj.y - fi.y, dz = fj.z - fi.z;
            r2f = dx * dx + dy * dy + dz * dz;
            if (r2f <= band.hi) {
              if (r2f < band.lo && !exact_rules)
                keep = !(p.half_rule && j < i);
              else
                keep = pack_keep(p, i, xi, j, load4(p.xd4 + j));
            }
          }
        }
        const unsigned m = __ballot_sync(kFull, keep);
        ghost |= keep && j >= p.nlocal;
        // Owned pairs held once stand for both directions in the kept-edge count.
        if (MODE == kDensityHalfOwned) kept_twice += __popc(__ballot_sync(kFull, keep && j < p.nlocal));
        if constexpr (sizeof(T) == 4) {
          // Float runs evaluate kept pairs in place: their evaluation gathers only the species
          // word, so idle lanes cost less than the queue's shared-memory round trip.
          if (keep) evaluate(kept + __popc(m & below), j, r2f);
          kept += __popc(m);
        } else {
          // Double runs gather each kept pair's 32-byte position again; the queue runs that
          // gather and the spline at full lane occupancy.
          if (keep) {
            const int at = q + __popc(m & below);
            qj[at] = j;
            qr2[at] = r2f;
          }
          q += __popc(m);
          if (q >= kWarp) flush(kWarp);
        }
      }
      if (q > 0) flush(q);
      if (MODE != kCompactOnly) {
        rho = warp_sum(rho);
        if (lane == 0) {
          if (MODE == kDensityHalf || MODE == kDensityHalfOwned)
            atomicAdd(p.rho + i, rho);
          else
            p.rho[i] = rho;
        }
      }
      const bool ghost_row = __any_sync(kFull, ghost);
      if (lane == 0) {
        p.ccount[row] = kept;
        p.ghost_rows[row] = ghost_row;
      }
      kept_sum += kept + kept_twice;
    }
    __syncthreads();
  }
  // kept_sum is carried by lane 0 of each warp (the other lanes hold copies): count it once.
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, lane == 0 ? kept_sum : 0.0};
  store_partials(acc, widest, p.partials);
}

// a8: F(rho) and F'(rho) of owned rows with linear continuation past rhomax
// (python/lammps_jax/eam.py:138-164 with extrapolate, :319-321, :383-384).
template <typename T>
__global__ void __launch_bounds__(kBlock) k_embed(const Step<T> p)
{
  double e = 0.0;
  const T inv_drho = T(1) / p.drho;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.nlocal;
       i += gridDim.x * blockDim.x) {
    const int s = min(max(p.type[i] - 1, 0), p.n_species - 1);
    const T rho = p.rho[i];
    const T idx = rho / p.drho;
    T fl = floor(idx);
    fl = fmin(fmax(fl, T(0)), T(p.nrho - 2));
    const T t_raw = idx - fl;
    const T t = fmin(t_raw, T(1));
    const auto c = load4(p.embedding + s * p.nrho + static_cast<int>(fl));
    const T end = c.y + T(2) * c.z + T(3) * c.w;
    T v = c.x + t * (c.y + t * (c.z + t * c.w));
    v = v + (t_raw - t) * end;
    T sl = c.y + t * (T(2) * c.z + t * (T(3) * c.w));
    if (t_raw > t) sl = end;
    p.fp[i] = sl * inv_drho;
    e += static_cast<double>(v);
    // Per-atom energy: the embedding term belongs to atom i alone.
    if (p.eatom != nullptr) p.eatom[i] += p.tally_scale * static_cast<double>(v);
  }
  double acc[8] = {e, 0, 0, 0, 0, 0, 0, 0};
  store_partials(acc, 0, p.partials);
}

// One EAM edge (i -> j, neighbor species sj) of the force pass; python/lammps_jax/eam.py:383-398
// for the pair force and :300-309 for the pair energy. r and 1/r come from one reciprocal square root; the density
// and pair tables share the r grid, so one (node, t) serves both lookups; F' of the density
// comes from the pre-scaled slope table. Accumulates the row force and the thread's pair energy
// and virial (both without their constant weights, applied once per block). Without FORCES only
// the pair energy is accumulated (energy-only evaluation).
//
// TALLY adds the per-atom split of LAMMPS's ev_tally: atom i always takes half the pair energy
// phi and half of this edge's -rij (x) F_e into the row sums er / vr; the neighbor j takes the
// other half of the energy when each pair appears once (half list) and the other half of the
// virial when the force acts on j too (newton-on scatter), both by atomics into its rows.
// Without EV (force-only steps) neither the pair energy nor the virial is summed.
template <typename T, int MODE, bool FORCES = true, bool TALLY = false, bool EV = true>
__device__ __forceinline__ void eam_edge(const Step<T> &p, const typename Vec4<T>::type &pi,
                                         int si, T fpi, int j, const typename Vec4<T>::type &pj,
                                         int sj, T fpj, T &fx, T &fy, T &fz, double &e,
                                         double (&v)[6], double &er, double (&vr)[6])
{
  const T dx = pj.x - pi.x, dy = pj.y - pi.y, dz = pj.z - pi.z;
  const T r2 = dx * dx + dy * dy + dz * dz;
  if (!(r2 < p.model_cutsq)) return;
  const T rinv = rsqrt(r2);
  const T r = r2 * rinv;
  const T idx = r * p.inv_dr;
  const T fl = fmin(floor(idx), T(p.nr - 2));
  const int node = static_cast<int>(fl);
  const T t = fmin(idx - fl, T(1));
  const auto c = load4_tab(p.pair + pair_row(si, sj) * p.nr + node);
  const T z2 = c.x + t * (c.y + t * (c.z + t * c.w));
  const T phi = z2 * rinv;
  // An owned pair held once (kRowsHalfOwned) counts for both directions.
  const bool twice = MODE == kRowsHalfOwned && j < p.nlocal;
  if constexpr (EV) e += twice ? 2.0 * static_cast<double>(phi) : static_cast<double>(phi);
  if constexpr (TALLY) {
    er += 0.5 * static_cast<double>(phi);
    if (MODE == kHalf && p.eatom != nullptr && j < p.nall)
      atomicAdd(p.eatom + j, p.tally_scale * 0.5 * static_cast<double>(phi));
  }
  if constexpr (FORCES) {
    const auto dj = load4_tab(p.density_slope + sj * p.nr + node);
    const T rhojp = dj.x + t * (dj.y + t * dj.z);
    const T z2p = (c.y + t * (T(2) * c.z + t * (T(3) * c.w))) * p.inv_dr;
    const T phip = (z2p - phi) * rinv;
    T psip;
    if (MODE == kGhost) {
      psip = fpi * rhojp + T(0.5) * phip;
    } else if (si == sj) {
      psip = (fpi + fpj) * rhojp + phip;
    } else {
      const auto di = load4_tab(p.density_slope + si * p.nr + node);
      psip = fpi * rhojp + fpj * (di.x + t * (di.y + t * di.z)) + phip;
    }
    const T sc = psip * rinv;
    const T ex = sc * dx, ey = sc * dy, ez = sc * dz;
    fx += ex;
    fy += ey;
    fz += ez;
    const double c6[6] = {static_cast<double>(dx * ex), static_cast<double>(dy * ey),
                          static_cast<double>(dz * ez), static_cast<double>(dx * ey),
                          static_cast<double>(dx * ez), static_cast<double>(dy * ez)};
    if constexpr (EV) {
#pragma unroll
      for (int k = 0; k < 6; ++k) v[k] += twice ? 2.0 * c6[k] : c6[k];
    }
    if constexpr (TALLY) {
#pragma unroll
      for (int k = 0; k < 6; ++k) vr[k] -= 0.5 * c6[k];
      if ((MODE == kGhost || MODE == kHalf) && p.vatom != nullptr && j < p.nall)
#pragma unroll
        for (int k = 0; k < 6; ++k) atomicAdd(p.vatom + 6 * j + k, -0.5 * p.tally_scale * c6[k]);
    }
    if (((MODE == kGhost || MODE == kHalf) && j < p.nall) || twice) {
      atomicAdd(p.f + 3 * j + 0, -p.scale * static_cast<double>(ex));
      atomicAdd(p.f + 3 * j + 1, -p.scale * static_cast<double>(ey));
      atomicAdd(p.f + 3 * j + 2, -p.scale * static_cast<double>(ez));
    }
  }
}

// Adds a row's per-atom sums (TALLY) into eatom[i] / vatom[i]: plain adds when no other row
// scatters into atom i (PLAIN: full list without newton-on scatters), atomics otherwise.
template <typename T, bool PLAIN>
__device__ __forceinline__ void tally_row(const Step<T> &p, int lane, int i, double er,
                                          double (&vr)[6])
{
  er = warp_sum(er);
#pragma unroll
  for (int k = 0; k < 6; ++k) vr[k] = warp_sum(vr[k]);
  if (lane != 0 || i >= p.nall) return;
  if (p.eatom != nullptr) {
    if (PLAIN)
      p.eatom[i] += p.tally_scale * er;
    else
      atomicAdd(p.eatom + i, p.tally_scale * er);
  }
  if (p.vatom != nullptr) {
#pragma unroll
    for (int k = 0; k < 6; ++k) {
      if (PLAIN)
        p.vatom[6 * i + k] += p.tally_scale * vr[k];
      else
        atomicAdd(p.vatom + 6 * i + k, p.tally_scale * vr[k]);
    }
  }
}

template <typename T>
__device__ __forceinline__ typename Vec4<T>::type load_pos(const Step<T> &p, int j)
{
  if constexpr (sizeof(T) == 8) {
    return load4(p.xd4 + j);
  } else {
    return load4(p.pos4 + j);
  }
}

// a9..a13: fused force + pair energy + virial over the compacted rows. Spilled rows (more kept
// pairs than row_cap) re-walk the LAMMPS list with the same filter. Without FORCES: the pair
// energy alone (energy-only evaluation; no F', no force or virial). Without EV: the forces
// alone (the steps where LAMMPS asks for neither energy nor virial); no partial sums are written.
template <typename T, int MODE, bool FORCES = true, bool TALLY = false, bool EV = true>
__global__ void LJX_FORCE_BOUNDS k_force(const Step<T> p)
{
  using V = typename Vec4<T>::type;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double e = 0.0;
  double v[6] = {0, 0, 0, 0, 0, 0};
  double er = 0.0;                      // per-atom tallies of the current row (TALLY)
  double vr[6] = {0, 0, 0, 0, 0, 0};
  constexpr bool kNeedFpj = FORCES && MODE != kGhost;
  // Float runs and the half-list mode (80 registers) load the next row's atom and kept count
  // one row ahead, so a row's dependent loads (atom -> position and F') start without waiting
  // on the list. The double full-list modes would spill at 64 registers, and lose.
  constexpr bool kAhead = sizeof(T) == 4 || MODE == kHalf;
  // Double force-only passes load a row's first two batches of compacted neighbor indices
  // together with the row's atom and kept count (they depend on the row alone), so a batch's
  // position gathers do not wait on an index load (C3 force-only 1.744 -> 1.680 ms). With the
  // energy and virial sums the two index registers spill at 64 registers, and at 3 blocks per
  // SM the pass is no faster than without them.
  constexpr int kPreloadIdx = sizeof(T) != 8 || TALLY ? 0 : !EV ? 2 : LJX_FORCE_EV_PRELOAD;
  const int stride = gridDim.x * kWarpsPerBlock;
  int row = blockIdx.x * kWarpsPerBlock + warp;
  int next_i = 0, next_n = 0;
  if (kAhead && row < p.inum) {
    next_i = p.ilist[row];
    next_n = p.ccount[row];
  }
  for (; row < p.inum; row += stride) {
    int i, n;
    int j0 = 0, j1 = 0;
    if constexpr (kPreloadIdx > 0) {
      const int *crow = p.cedges + static_cast<long long>(row) * p.row_cap;
      if (lane < p.row_cap) j0 = load_once(crow + lane);
      if (kPreloadIdx > 1 && lane + kWarp < p.row_cap) j1 = load_once(crow + lane + kWarp);
    }
    if constexpr (kAhead) {
      i = next_i;
      n = next_n;
      if (row + stride < p.inum) {
        next_i = p.ilist[row + stride];
        next_n = p.ccount[row + stride];
      }
    } else {
      i = p.ilist[row];
      n = p.ccount[row];
    }
    if (i >= p.max_atoms) continue;
    if (p.row_part != kRowsAll && (p.ghost_rows[row] != 0) != (p.row_part == kRowsGhost)) continue;
    const V pi = load_pos(p, i);
    const int si = static_cast<int>(pi.w);
    const T fpi = FORCES ? p.fp[i] : T(0);
    T fx = T(0), fy = T(0), fz = T(0);
    if constexpr (TALLY) {
      er = 0.0;
#pragma unroll
      for (int k = 0; k < 6; ++k) vr[k] = 0.0;
    }
    if (n <= p.row_cap) {
      const int *crow = p.cedges + static_cast<long long>(row) * p.row_cap;
      if constexpr (sizeof(T) == 8) {
        // (Pipelining as below spills at 64 registers in double runs and loses.)
        for (int k = lane; k < n; k += kWarp) {
          const int j = kPreloadIdx > 0 && k < kWarp       ? j0
                        : kPreloadIdx > 1 && k < 2 * kWarp ? j1
                                                           : load_once(crow + k);
          const V pj = load_pos(p, j);
          eam_edge<T, MODE, FORCES, TALLY, EV>(p, pi, si, fpi, j, pj, static_cast<int>(pj.w),
                                           kNeedFpj ? __ldg(p.fp + j) : T(0), fx, fy, fz, e, v,
                                           er, vr);
        }
      } else {
        // Float runs are software-pipelined by one pair: the next pair's position and F' gathers
        // are issued before the current pair's spline lookups, so two dependent chains overlap
        // per lane.
        int k = lane;
        int j = 0;
        V pj = V{};
        T fpj = T(0);
        if (k < n) {
          j = load_once(crow + k);
          pj = load_pos(p, j);
          if (kNeedFpj) fpj = __ldg(p.fp + j);
        }
        while (k < n) {
          const int k2 = k + kWarp;
          int j2 = 0;
          V pj2 = V{};
          T fpj2 = T(0);
          if (k2 < n) {
            j2 = load_once(crow + k2);
            pj2 = load_pos(p, j2);
            if (kNeedFpj) fpj2 = __ldg(p.fp + j2);
          }
          eam_edge<T, MODE, FORCES, TALLY, EV>(p, pi, si, fpi, j, pj, static_cast<int>(pj.w), fpj,
                                           fx, fy, fz, e, v, er, vr);
          k = k2;
          j = j2;
          pj = pj2;
          fpj = fpj2;
        }
      }
    } else {
      const double4 xi = load4(p.xd4 + i);
      const int listed = min(p.numneigh[i], p.maxneighs);
      const long long rowbase = static_cast<long long>(i) * p.atom_stride;
      for (int jj = lane; jj < listed; jj += kWarp) {
        const int j = p.neighbors[rowbase + jj * p.slot_stride] & kNeighMask;
        if (j >= p.max_atoms || (p.half_rule && j < i)) continue;
        if (pack_keep(p, i, xi, j, load4(p.xd4 + j))) {
          const V pj = load_pos(p, j);
          eam_edge<T, MODE, FORCES, TALLY, EV>(p, pi, si, fpi, j, pj, static_cast<int>(pj.w),
                                           kNeedFpj ? __ldg(p.fp + j) : T(0), fx, fy, fz, e, v,
                                           er, vr);
        }
      }
    }
    if constexpr (FORCES) {
      // The row force: x in lane 0, y in lane 8, z in lane 16, each stored by its lane.
      const T fc = warp_sum3(fx, fy, fz, lane);
      if ((lane & 7) == 0 && lane < 24 && i < p.nall) {
        double *fi = p.f + 3 * i + (lane >> 3);
        if (MODE == kRowsFull)
          *fi += p.scale * static_cast<double>(fc);
        else
          atomicAdd(fi, p.scale * static_cast<double>(fc));
      }
    }
    if constexpr (TALLY) tally_row<T, MODE == kRowsFull>(p, lane, i, er, vr);
  }
  // Pair energy: phi/2 per directed edge of a full list, phi per edge of a half list. Virial:
  // -1/2 rij (x) F_e when every pair appears in two rows, -rij (x) F_e when the receiver takes
  // -F_e (newton-on scatters).
  if constexpr (EV) {
    const double ew = MODE == kHalf ? 1.0 : 0.5;
    const double vw = (MODE == kRowsFull || MODE == kRowsHalfOwned) ? -0.5 : -1.0;
    double acc[8] = {ew * e, vw * v[0], vw * v[1], vw * v[2], vw * v[3], vw * v[4], vw * v[5],
                     0.0};
    store_partials(acc, 0, p.partials);
  }
}

// LJ 12-6 in one pass over the LAMMPS list: examples/export_model.py:16-74 with the force-add
// conventions of cpp/pair_jax_kokkos.cpp:176-225. Without FORCES: the energy alone.
template <typename T, int MODE, bool FORCES = true, bool TALLY = false>
__global__ void __launch_bounds__(kBlock) k_lj(const Step<T> p)
{
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double e = 0.0, kept_sum = 0.0;
  double v[6] = {0, 0, 0, 0, 0, 0};
  int widest = 0;
  const bool scatter = MODE != kLjEdgeFull;
  // Per-atom split (TALLY): a half list holds each pair once, so its energy goes half to each
  // atom; a scattering mode applies the force to both atoms, so its virial goes half to each.
  constexpr bool kHalfList = MODE == kLjEdgeHalf || MODE == kLjAtomHalfPairSum;
  double er = 0.0;
  double vr[6] = {0, 0, 0, 0, 0, 0};
  // Sender weight (edge-force bundles add dU/drij; atom-force bundles the energy-scaled
  // gradient, doubled for pair-sum half lists that stand for both directions).
  const T fw = MODE == kLjAtomFull ? p.lj_energy_scale
               : MODE == kLjAtomHalfPairSum ? T(2) * p.lj_energy_scale
                                            : T(1);
  const T ew = MODE == kLjAtomHalfPairSum ? T(2) * p.lj_energy_scale : p.lj_energy_scale;
  const double vw = scatter ? 1.0 : 0.5;
  for (int row = blockIdx.x * kWarpsPerBlock + warp; row < p.inum;
       row += gridDim.x * kWarpsPerBlock) {
    const int i = p.ilist[row];
    if (i >= p.max_atoms) continue;
    const int listed = p.numneigh[i];
    widest = max(widest, listed);
    const int n = min(listed, p.maxneighs);
    const double4 xi = load4(p.xd4 + i);
    const long long rowbase = static_cast<long long>(i) * p.atom_stride;
    T fx = T(0), fy = T(0), fz = T(0);
    int kept = 0;
    if constexpr (TALLY) {
      er = 0.0;
#pragma unroll
      for (int k = 0; k < 6; ++k) vr[k] = 0.0;
    }
    for (int base = 0; base < n; base += kWarp) {
      const int jj = base + lane;
      bool keep = false;
      int j = 0;
      double4 xj = make_double4(0, 0, 0, 0);
      if (jj < n) {
        j = p.neighbors[rowbase + jj * p.slot_stride] & kNeighMask;
        if (j < p.max_atoms) {
          xj = load4(p.xd4 + j);
          keep = pack_keep(p, i, xi, j, xj);
        }
      }
      kept += __popc(__ballot_sync(kFull, keep));
      if (!keep) continue;
      const T dx = T(xj.x) - T(xi.x), dy = T(xj.y) - T(xi.y), dz = T(xj.z) - T(xi.z);
      const T r2 = dx * dx + dy * dy + dz * dz;
      if (!(r2 > T(1.0e-12) && r2 < p.model_cutsq)) continue;
      const T inv_r2 = p.lj_sigma_sq / r2;
      const T inv_r6 = inv_r2 * inv_r2 * inv_r2;
      const T u = p.lj_four_eps * (inv_r6 * inv_r6 - inv_r6);
      const double eu = static_cast<double>(ew * u);
      e += eu;
      if constexpr (TALLY) {
        er += kHalfList ? 0.5 * eu : eu;
        if (kHalfList && p.eatom != nullptr && j < p.nall)
          atomicAdd(p.eatom + j, p.tally_scale * 0.5 * eu);
      }
      if constexpr (!FORCES) continue;
      // dU/drij = 2 rij dU/d(r^2), dU/d(r^2) = -4 eps (6 a^6 - 3 a^3) / r^2, a = sigma^2/r^2.
      const T g = T(-2) * p.lj_four_eps * (T(6) * inv_r6 * inv_r6 - T(3) * inv_r6) / r2 * fw;
      const T ex = g * dx, ey = g * dy, ez = g * dz;
      fx += ex;
      fy += ey;
      fz += ez;
      const double c6[6] = {static_cast<double>(dx * ex), static_cast<double>(dy * ey),
                            static_cast<double>(dz * ez), static_cast<double>(dx * ey),
                            static_cast<double>(dx * ez), static_cast<double>(dy * ez)};
#pragma unroll
      for (int k = 0; k < 6; ++k) v[k] -= vw * c6[k];
      if constexpr (TALLY) {
        const double wi = scatter ? 0.5 * vw : vw;
#pragma unroll
        for (int k = 0; k < 6; ++k) vr[k] -= wi * c6[k];
        if (scatter && p.vatom != nullptr && j < p.nall)
#pragma unroll
          for (int k = 0; k < 6; ++k)
            atomicAdd(p.vatom + 6 * j + k, -0.5 * vw * p.tally_scale * c6[k]);
      }
      if (scatter && j < p.nall) {
        atomicAdd(p.f + 3 * j + 0, -p.scale * static_cast<double>(ex));
        atomicAdd(p.f + 3 * j + 1, -p.scale * static_cast<double>(ey));
        atomicAdd(p.f + 3 * j + 2, -p.scale * static_cast<double>(ez));
      }
    }
    if constexpr (FORCES) {
      fx = warp_sum(fx);
      fy = warp_sum(fy);
      fz = warp_sum(fz);
      if (lane == 0 && i < p.nall) {
        double *fi = p.f + 3 * i;
        if (!scatter) {
          fi[0] += p.scale * static_cast<double>(fx);
          fi[1] += p.scale * static_cast<double>(fy);
          fi[2] += p.scale * static_cast<double>(fz);
        } else {
          atomicAdd(fi + 0, p.scale * static_cast<double>(fx));
          atomicAdd(fi + 1, p.scale * static_cast<double>(fy));
          atomicAdd(fi + 2, p.scale * static_cast<double>(fz));
        }
      }
    }
    if constexpr (TALLY) tally_row<T, MODE == kLjEdgeFull>(p, lane, i, er, vr);
    kept_sum += kept;
  }
  double acc[8] = {e, v[0], v[1], v[2], v[3], v[4], v[5], lane == 0 ? kept_sum : 0.0};
  store_partials(acc, widest, p.partials);
}

// Row counts -> exclusive offsets for the reference edge ABI (single block; off the hot path).
static __global__ void k_scan_counts(const int *counts, int n, int per_pair, long long *offsets)
{
  __shared__ long long s_part[1024];
  const int t = threadIdx.x, nt = blockDim.x;
  const long long chunk = (static_cast<long long>(n) + nt - 1) / nt;
  const long long lo = chunk * t;
  const long long hi = lo + chunk < n ? lo + chunk : n;
  long long sum = 0;
  for (long long k = lo; k < hi; ++k) sum += static_cast<long long>(counts[k]) * per_pair;
  s_part[t] = sum;
  __syncthreads();
  if (t == 0) {
    long long run = 0;
    for (int q = 0; q < nt; ++q) {
      const long long c = s_part[q];
      s_part[q] = run;
      run += c;
    }
    offsets[n] = run;
  }
  __syncthreads();
  long long run = s_part[t];
  for (long long k = lo; k < hi; ++k) {
    offsets[k] = run;
    run += static_cast<long long>(counts[k]) * per_pair;
  }
}

// Scatter compacted rows into the reference ABI: senders/receivers/edge_mask at the row's
// offset, duplicated reversed when the bundle asks (cpp/pair_jax_kokkos.cpp:103-116). Rows that
// spilled past row_cap re-walk the list with the same filter.
template <typename T>
__global__ void __launch_bounds__(kBlock)
k_emit_edges(const Step<T> p, const long long *offsets, int duplicate, int max_edges,
             int *senders, int *receivers, uint8_t *mask)
{
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  const int per = duplicate ? 2 : 1;
  for (int row = blockIdx.x * kWarpsPerBlock + warp; row < p.inum;
       row += gridDim.x * kWarpsPerBlock) {
    const int i = p.ilist[row];
    if (i >= p.max_atoms) continue;
    const int n = p.ccount[row];
    const long long base_edge = offsets[row];
    auto put = [&](long long edge, int j) {
      if (edge + per > max_edges) return;
      senders[edge] = i;
      receivers[edge] = j;
      mask[edge] = 1;
      if (duplicate) {
        senders[edge + 1] = j;
        receivers[edge + 1] = i;
        mask[edge + 1] = 1;
      }
    };
    if (n <= p.row_cap) {
      const int *crow = p.cedges + static_cast<long long>(row) * p.row_cap;
      for (int k = lane; k < n; k += kWarp) put(base_edge + static_cast<long long>(k) * per, crow[k]);
    } else {
      const double4 xi = load4(p.xd4 + i);
      const int listed = min(p.numneigh[i], p.maxneighs);
      const long long rowbase = static_cast<long long>(i) * p.atom_stride;
      int kept = 0;
      for (int base = 0; base < listed; base += kWarp) {
        const int jj = base + lane;
        bool keep = false;
        int j = 0;
        if (jj < listed) {
          j = p.neighbors[rowbase + jj * p.slot_stride] & kNeighMask;
          if (j < p.max_atoms) keep = pack_keep(p, i, xi, j, load4(p.xd4 + j));
        }
        const unsigned m = __ballot_sync(kFull, keep);
        if (keep) put(base_edge + static_cast<long long>(kept + __popc(m & below)) * per, j);
        kept += __popc(m);
      }
    }
  }
}

// Padding past the new count up to the previous count (ResetEdgeTailFunctor,
// cpp/pair_jax_kokkos.cpp:157-173); both counts are read on the device.
static __global__ void k_reset_tail(const long long *count_now, long long *count_prev, int max_atoms,
                             int max_edges, int *senders, int *receivers, uint8_t *mask)
{
  const long long now = *count_now;
  const long long prev = *count_prev;
  const long long hi = prev < max_edges ? prev : max_edges;
  for (long long e = now + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < hi;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    senders[e] = max_atoms;
    receivers[e] = max_atoms;
    mask[e] = 0;
  }
}

static __global__ void k_store_prev(const long long *count_now, long long *count_prev)
{
  *count_prev = *count_now;
}

// Step totals from the per-block partials of the kernels that ran, in a fixed order.
// result: [0] energy, [1..6] virial (both times `scale`), [7] kept pairs, [8] widest row.
struct PartialSet {
  const double *ptr[4];
  int blocks[4];
};

static __global__ void __launch_bounds__(kBlock) k_finalize(PartialSet set, double scale, double *result)
{
  __shared__ double s[9][kBlock];
  const int t = threadIdx.x;
  double acc[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  for (int q = 0; q < 4; ++q) {
    for (int b = t; b < set.blocks[q]; b += blockDim.x) {
      const double *row = set.ptr[q] + static_cast<long long>(b) * kPartialWidth;
      for (int k = 0; k < 8; ++k) acc[k] += row[k];
      acc[8] = fmax(acc[8], row[8]);
    }
  }
  for (int k = 0; k < 9; ++k) s[k][t] = acc[k];
  __syncthreads();
  if (t < 9) {
    double total = 0.0;
    for (int q = 0; q < static_cast<int>(blockDim.x); ++q)
      total = (t == 8) ? fmax(total, s[t][q]) : total + s[t][q];
    result[t] = (t < 7) ? scale * total : total;
  }
}

// ---- comm rows (cpp/pair_jax_kokkos.cpp:247-318) ----

static __global__ void k_pack_words_by_list(const uint32_t *rows, int words, const int *sendlist, int n,
                                     double *buf, int slots)
{
  const long long total = static_cast<long long>(n) * words;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(flat / words), w = static_cast<int>(flat % words);
    uint32_t *packed = reinterpret_cast<uint32_t *>(buf + static_cast<long long>(i) * slots);
    packed[w] = rows[static_cast<long long>(sendlist[i]) * words + w];
    if ((words & 1) && w + 1 == words) packed[words] = 0u;
  }
}

static __global__ void k_unpack_words_at(uint32_t *rows, int words, int first, int n, const double *buf,
                                  int slots)
{
  const long long total = static_cast<long long>(n) * words;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(flat / words), w = static_cast<int>(flat % words);
    rows[static_cast<long long>(first + i) * words + w] =
        reinterpret_cast<const uint32_t *>(buf + static_cast<long long>(i) * slots)[w];
  }
}

static __global__ void k_pack_words_at(const uint32_t *rows, int words, int first, int n, double *buf,
                                int slots)
{
  const long long total = static_cast<long long>(n) * words;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(flat / words), w = static_cast<int>(flat % words);
    uint32_t *packed = reinterpret_cast<uint32_t *>(buf + static_cast<long long>(i) * slots);
    packed[w] = rows[static_cast<long long>(first + i) * words + w];
    if ((words & 1) && w + 1 == words) packed[words] = 0u;
  }
}

template <typename S>
__global__ void k_add_rows_by_list(S *rows, int width, const int *sendlist, int n,
                                   const double *buf, int slots)
{
  const long long total = static_cast<long long>(n) * width;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(flat / width), w = static_cast<int>(flat % width);
    // sendlist rows are unique within one swap, so the add needs no atomic.
    rows[static_cast<long long>(sendlist[i]) * width + w] +=
        reinterpret_cast<const S *>(buf + static_cast<long long>(i) * slots)[w];
  }
}

template <typename S>
__global__ void k_zero_rows(S *rows, int width, int first, int n)
{
  const long long total = static_cast<long long>(n) * width;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x)
    rows[static_cast<long long>(first) * width + flat] = S(0);
}

template <typename S>
__global__ void k_forward_self(S *rows, int width, const int *owner, int first, int n)
{
  const long long total = static_cast<long long>(n) * width;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(flat / width), w = static_cast<int>(flat % width);
    rows[static_cast<long long>(first + g) * width + w] =
        rows[static_cast<long long>(owner[g]) * width + w];
  }
}

template <typename S>
__global__ void k_reverse_self(S *rows, int width, const int *owner, int first, int n)
{
  const long long total = static_cast<long long>(n) * width;
  for (long long flat = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; flat < total;
       flat += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(flat / width), w = static_cast<int>(flat % width);
    S *src = rows + static_cast<long long>(first + g) * width + w;
    // Several images can share one owner, so the add is atomic.
    atomicAdd(rows + static_cast<long long>(owner[g]) * width + w, *src);
    *src = S(0);
  }
}

}  // namespace ljx
