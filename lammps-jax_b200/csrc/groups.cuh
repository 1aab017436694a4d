// Row-group density pass over cached neighbor unions (sm_100a).
//
// The list pass (k_density) gathers the float position of every listed pair of every row (about
// 215 per row at the C3 density, each its own L1 sector) and the double position of every kept
// pair. Consecutive list rows are spatial neighbours (LAMMPS sorts atoms by bin), so their
// neighbor sets overlap heavily. When LAMMPS has built a new list (neighbor->ago == 0, the
// signal the reference's neighbor-matrix path also follows, cpp/pair_jax_kokkos.cpp:1011-1012),
// k_build_groups stores for each group of kGroupRows consecutive rows:
//   - the union of the rows' neighbors within rc + margin (about 300 atoms for 8 rows at C3);
//   - for each row, its candidates within rc + margin as 16-bit slots into that union, in the
//     order of the row's LAMMPS list (so the kept pairs come out as the list pass emits them).
// Every step, k_density_groups runs one block per group. The block stages the union's positions
// in shared memory (one global gather per union atom, shared by the eight rows). Then, as in the
// list pass, one warp per row filters its candidates with the reference's exact keep test,
// compacts the kept pairs and evaluates the density spline. Per row that is about 40 position
// gathers from global memory instead of about 300, and about 135 candidates instead of 215 list
// slots.
//
// The kept set is the reference's exactly. A pair the reference keeps is in its row's list and
// lies within rc now. While no atom has moved more than margin / 2 since the build, it lay
// within rc + margin then, so it is among its row's candidates. k_pack_atoms tracks the largest
// displacement; k_build_groups rebuilds on the device when it passes the limit.
#pragma once

#include "kernels.cuh"

namespace ljx {

constexpr int kGroupRows = 8;          // list rows per group: one block, one warp per row
constexpr int kHashSlots = 1024;       // per-warp open-addressing set of neighbor indices
constexpr int kBuildWarps = 8;         // build block: one group per warp
constexpr int kBuildBlock = kBuildWarps * kWarp;
constexpr int kUnionMax = 512;         // largest union a group may cache (shared-memory stage)

static_assert(kGroupRows == kWarpsPerBlock, "one warp per row of a group");
static_assert(kGroupRows <= 8, "row masks are one byte");
static_assert(kUnionMax < kHashSlots, "the set must keep free slots");
// Builds over half rows (half lists, owned pairs held once) use a set of this many slots and
// keep unions of at most three quarters of it; their density passes stage that many atoms.
#ifndef LJX_BUILD_HALF_HASH
#define LJX_BUILD_HALF_HASH 512
#endif
constexpr int kHalfUnion = LJX_BUILD_HALF_HASH * 3 / 4 < kUnionMax ? LJX_BUILD_HALF_HASH * 3 / 4
                                                                   : kUnionMax;

// Rows of owned pairs held once and half lists stage their unions twice over (one stage per
// group in turn, so one block barrier per group instead of two), at most 384 atoms each: their
// builds already mark larger unions past capacity. C3 density phase 2.020 -> 1.998 ms.
#ifndef LJX_OWNED_UNION
#define LJX_OWNED_UNION ljx::kHalfUnion
#endif
// Resident blocks per SM of the cached density pass (caps its registers per thread): 5, at 48
// registers without spills (6 blocks at 40 registers spilled: with owned pairs held once and
// the candidate slots loaded ahead, C3 density phase 2.20 -> 2.02 ms; half lists with two union
// stages, C4 at 80^3 1.605 -> 1.588 ms; full rows 2.975 -> 2.898 ms).
#ifndef LJX_GROUP_MIN_BLOCKS
#define LJX_GROUP_MIN_BLOCKS 5
#endif
// Candidate slots of a row's second and third batches loaded before the staging barrier, per
// mode (owned pairs held once / the others).
#ifndef LJX_DG_PRELOAD_OWNED
#define LJX_DG_PRELOAD_OWNED 1
#endif
#ifndef LJX_DG_PRELOAD
#define LJX_DG_PRELOAD 0
#endif
#ifndef LJX_DG_DOUBLE
#define LJX_DG_DOUBLE 1
#endif
#ifndef LJX_DG_DOUBLE_HALF
#define LJX_DG_DOUBLE_HALF 1
#endif

// Rebuild the group caches when the host asks (new list, first use, changed sizes or pointers)
// or when some atom has moved more than margin / 2 since the last build (disp_limit is that
// squared distance, rounded down). Every block reads the same displacement word, so the
// decision is uniform over the grid. Also records the positions the displacement is measured
// from. cand_cutsq is (rc + margin)^2; the float test uses its rounding band, so a pair whose
// exact distance is within rc + margin is never dropped.
//
// One warp per group. Lane l walks row l % 8, four list slots per step (with LayoutLeft and
// consecutive rows, one step reads slot s of all eight rows as one 32-byte sector). Each
// candidate is looked up in the warp's hash set (a plain read first: most candidates of a group
// are already there, about 3.6 rows share each neighbor) and inserted by compare-and-swap when
// absent; a new atom takes the next union index, in first-seen order, and is written out at
// once. Every candidate then goes straight into its row's slot list as its union index, so a
// row's candidates keep the order of its LAMMPS list.
// HASH: the set's slots. Rows that hold owned pairs once list about half the candidates, so
// their builds use a set half the size (more resident warps); a group whose union passes three
// quarters of the set is marked past capacity.
template <typename T, int HASH = kHashSlots>
__global__ void __launch_bounds__(kBuildBlock)
k_build_groups(const Step<T> p, int span, int force_build, float disp_limit, double cand_cutsq)
{
  static_assert((HASH & (HASH - 1)) == 0 && HASH >= 256 && HASH <= 1024, "power-of-two set");
  constexpr int kHashShift = HASH == 1024 ? 22 : HASH == 512 ? 23 : 24;
  __shared__ __align__(16) int s_key[kBuildWarps][HASH];
  __shared__ unsigned short s_index[kBuildWarps][HASH];
  if (!force_build && !(__uint_as_float(*p.disp_bound) > disp_limit)) return;
  for (int a = blockIdx.x * blockDim.x + threadIdx.x; a < span; a += gridDim.x * blockDim.x)
    p.xref[a] = p.xd4[a];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  volatile int *key = s_key[warp];
  unsigned short *uindex = s_index[warp];
  int4 *key4 = reinterpret_cast<int4 *>(s_key[warp]);
  const float4 *pos4f = reinterpret_cast<const float4 *>(p.pos4);
  const FilterBand band = filter_band(cand_cutsq, *p.coord_bound);
  const int groups = (p.inum + kGroupRows - 1) / kGroupRows;
  // The set starts empty; each group empties it again when done.
  for (int h = lane; h < HASH / 4; h += kWarp) key4[h] = make_int4(-1, -1, -1, -1);
  __syncwarp();
  for (int g = blockIdx.x * kBuildWarps + warp; g < groups; g += gridDim.x * kBuildWarps) {
    const int k = lane & (kGroupRows - 1);
    const int row = g * kGroupRows + k;
    int i = -1, n = 0;
    float4 fi = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < p.inum) {
      i = p.ilist[row];
      if (i < p.max_atoms) {
        n = min(p.numneigh[i], p.maxneighs);
        fi = __ldg(pos4f + i);
      } else {
        i = -1;
      }
    }
    int longest = n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) longest = max(longest, __shfl_xor_sync(kFull, longest, o));
    const unsigned rowlanes = 0x01010101u << k;  // the four lanes of this lane's row
    unsigned short *slots = p.rslot + static_cast<long long>(row) * p.rcap;
    int *out = p.gatom + static_cast<long long>(g) * p.gcap;
    bool lost = false;
    bool ghost = false;  // this lane met a ghost candidate
    int total = 0;  // distinct atoms so far (uniform over the warp)
    int got = 0;    // candidates of this lane's row so far (uniform over the row's lanes)
    const long long rowbase = static_cast<long long>(i) * p.atom_stride;
    for (int s0 = 0; s0 < longest; s0 += kWarp / kGroupRows) {
      const int s = s0 + lane / kGroupRows;
      bool cand = false;
      int j = 0;
      if (i >= 0 && s < n) {
        j = p.neighbors[rowbase + static_cast<long long>(s) * p.slot_stride] & kNeighMask;
        if (j < p.max_atoms && !(p.half_rule && j < i)) {
          const float4 fj = __ldg(pos4f + j);
          const float dx = fj.x - fi.x, dy = fj.y - fi.y, dz = fj.z - fi.z;
          cand = dx * dx + dy * dy + dz * dz <= band.hi;
        }
      }
      // Multiplicative hash, linear probing.
      unsigned h = (static_cast<unsigned>(j) * 0x9E3779B1u) >> kHashShift;
      bool fresh = false;
      if (cand) {
        bool placed = false;
        for (int probe = 0; probe < HASH; ++probe) {
          int cur = key[h];
          if (cur == -1) cur = atomicCAS(const_cast<int *>(key) + h, -1, j);
          if (cur == -1 || cur == j) {
            fresh = cur == -1;
            placed = true;
            break;
          }
          h = (h + 1u) & (HASH - 1);
        }
        lost |= !placed;
      }
      const unsigned fm = __ballot_sync(kFull, fresh);
      if (fresh) {
        const int at = total + __popc(fm & below);
        uindex[h] = static_cast<unsigned short>(min(at, 65535));
        if (at < p.gcap) out[at] = j;
      }
      total += __popc(fm);
      __syncwarp();  // the new atoms' union indices are visible to every lane
      const unsigned cm = __ballot_sync(kFull, cand);
      ghost |= cand && j >= p.nlocal;
      if (cand) {
        const int at = got + __popc(cm & rowlanes & below);
        if (at < p.rcap) slots[at] = uindex[h];
      }
      got += __popc(cm & rowlanes);
    }
    // A group that does not fit is marked past capacity; the density pass then walks its rows'
    // lists instead.
    const bool spilled = __any_sync(kFull, lost || got > p.rcap) || total > kUnionMax ||
                         total > p.gcap || total > HASH * 3 / 4;
    // A row with a ghost among its candidates may keep a ghost pair until the next build (every
    // kept pair is a candidate): ljx_force_rows runs it after the F' exchange. A group past
    // capacity walks its lists, so all its rows are marked.
    const bool row_ghost = (__ballot_sync(kFull, ghost) & rowlanes) != 0;
    if (lane < kGroupRows && row < p.inum) {
      p.rcount[row] = got;
      p.ghost_rows[row] = spilled || row_ghost;
    }
    __syncwarp();
    for (int h = lane; h < HASH / 4; h += kWarp) key4[h] = make_int4(-1, -1, -1, -1);
    __syncwarp();
    if (lane == 0) p.gcount[g] = spilled ? p.gcap + 1 : total;
  }
}

__device__ __forceinline__ double4 staged(const double2 *xy, const double2 *zw, int slot)
{
  const double2 a = xy[slot], b = zw[slot];
  return make_double4(a.x, a.y, b.x, b.y);
}

// a2 + a6 over the group caches: one block per group, one warp per row. The union's positions
// are staged in shared memory; each warp filters its row's candidates with the reference's exact
// keep test, compacts the kept pairs into the row's segment of the compacted buffer (the force
// pass reads it as from k_density) and accumulates the EAM density, scattered to the neighbor as
// well for half lists. Groups past capacity walk their rows' lists.
// RULES: the bundle's packing has a half or unique-boundary rule to apply (half-edge bundles on
// a full list); without one the keep test is the distance alone.
// UNION: the staged union's capacity. Builds over half rows mark unions past three quarters of
// their 512-slot set as past capacity, so their cached groups stage at most 384 atoms; half
// lists stage that much (less shared memory per block, more L1 left to the spline rows of two
// species: C4 density -2 %), and so do rows with owned pairs held once, in two stages.
template <typename T, int MODE, bool RULES = true, int UNION = kUnionMax>
__global__ void __launch_bounds__(kBlock, LJX_GROUP_MIN_BLOCKS) k_density_groups(const Step<T> p)
{
  static_assert(UNION <= kUnionMax, "the union stage holds at most kUnionMax atoms");
  // A row of owned pairs held once has about 72 candidates: with its first three batches'
  // slots loaded before the staging barrier, its whole candidate list is in flight at once.
  constexpr bool kPreload = MODE == kDensityHalfOwned ? LJX_DG_PRELOAD_OWNED : LJX_DG_PRELOAD;
  // Staged positions as two 16-byte halves: consecutive slots then fall on different bank
  // quads (a 32-byte record per slot would reach only 4 of the 8 and conflict at least 2-way).
  // DOUBLE: two stages used in turn, so one barrier per group suffices (the stage written for
  // group g + 2 was last read for group g, and every warp has passed group g + 1's barrier).
  constexpr bool kDouble = (MODE == kDensityHalfOwned && LJX_DG_DOUBLE) ||
                           (MODE == kDensityHalf && LJX_DG_DOUBLE_HALF);
  constexpr int kStages = kDouble ? 2 : 1;
  __shared__ double2 s_xy_all[kStages][UNION];
  __shared__ double2 s_zw_all[kStages][UNION];
  __shared__ int s_j_all[kStages][UNION];
  int stage = 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  const int groups = (p.inum + kGroupRows - 1) / kGroupRows;
  double kept_sum = 0.0;
  int widest = 0;
  for (int g = blockIdx.x; g < groups; g += gridDim.x) {
    const int count = p.gcount[g];
    const bool cached = count <= p.gcap && count <= UNION;
    double2 *s_xy = s_xy_all[stage], *s_zw = s_zw_all[stage];
    int *s_j = s_j_all[stage];
    if constexpr (kDouble) stage ^= 1;
    // The warp's row and its first 32 candidate slots do not depend on the staged union: they
    // are loaded before the staging barrier, so their latency overlaps the staging gathers.
    // (rslot holds rcap >= 32 entries per row; slots past the row's count are not used.)
    const int row = g * kGroupRows + warp;
    int i = -1, listed = 0, n = 0;
    unsigned short slot0 = 0, slot1 = 0, slot2 = 0;
    double4 xi = make_double4(0.0, 0.0, 0.0, 0.0);
    if (row < p.inum) {
      i = p.ilist[row];
      if (i >= p.max_atoms) i = -1;
    }
    if (i >= 0) {
      listed = p.numneigh[i];
      xi = load4(p.xd4 + i);
      if (cached) {
        n = p.rcount[row];
        const unsigned short *first = p.rslot + static_cast<long long>(row) * p.rcap + lane;
        slot0 = load_once(first);
        if constexpr (kPreload) {
          if (lane + kWarp < p.rcap) slot1 = load_once(first + kWarp);
          if (lane + 2 * kWarp < p.rcap) slot2 = load_once(first + 2 * kWarp);
        }
      }
    }
    if (cached) {
      const int *atoms = p.gatom + static_cast<long long>(g) * p.gcap;
      for (int t = threadIdx.x; t < count; t += kBlock) {
        const int j = atoms[t];
        const double4 xj = load4(p.xd4 + j);
        s_xy[t] = make_double2(xj.x, xj.y);
        s_zw[t] = make_double2(xj.z, xj.w);
        s_j[t] = j;
      }
    }
    __syncthreads();
    if (row < p.inum && i < 0 && lane == 0) p.ccount[row] = 0;
    if (i >= 0) {
      widest = max(widest, listed);
      const float fix = static_cast<float>(xi.x), fiy = static_cast<float>(xi.y),
                  fiz = static_cast<float>(xi.z);
      const int si = static_cast<int>(xi.w);
      int *crow = p.cedges + static_cast<long long>(row) * p.row_cap;
      T rho = T(0);
      int kept = 0;
      int kept_twice = 0;  // owned pairs held once (kDensityHalfOwned) count for both directions
      if (cached) {
        // About 80 % of a row's cached candidates are kept, so each batch of 32 evaluates its
        // kept pairs in place: the idle lanes cost little (a gather costs per sector touched,
        // not per lane) and no queue round trip through shared memory is needed. The reference's
        // keep test in double (pair_jax_kokkos.cpp:84-101) runs straight from the staged
        // coordinates. The batch is predicated: every lane runs the keep test and the table-node
        // arithmetic of spline_v_dist (lanes past the row's candidates on slot 0 of the stage),
        // and only the table gather, the compacted store and the neighbor's reduction depend on
        // the lane's pair. (Nested divergent branches had cost 83 branch instructions per row:
        // C3 density phase 1.961 -> 1.843 ms, f32 1.769 -> 1.634 ms, C4 at 80^3 1.582 -> 1.560.)
        const unsigned short *slots = p.rslot + static_cast<long long>(row) * p.rcap;
        for (int base = 0; base < n; base += kWarp) {
          const bool valid = base + lane < n;
          int slot;
          if constexpr (kPreload)
            slot = base == 0           ? slot0
                   : base == kWarp     ? slot1
                   : base == 2 * kWarp ? slot2
                   : valid             ? load_once(slots + base + lane)
                                       : 0;
          else
            slot = base == 0 ? slot0 : valid ? load_once(slots + base + lane) : 0;
          slot = valid ? slot : 0;
          const double4 xj = staged(s_xy, s_zw, slot);
          const double r2d = pack_r2(xi, xj);
          const int j = s_j[slot];
          bool keep = valid && r2d <= p.pack_cutsq;
          if constexpr (RULES) keep = keep && pair_rules(p, i, xi, j, xj);
          const unsigned m = __ballot_sync(kFull, keep);
          const int at = kept + __popc(m & below);
          if (keep && at < p.row_cap) crow[at] = j;
          T r2;
          if constexpr (sizeof(T) == 8) {
            r2 = r2d;
          } else {
            const float dx = static_cast<float>(xj.x) - fix, dy = static_cast<float>(xj.y) - fiy,
                        dz = static_cast<float>(xj.z) - fiz;
            r2 = dx * dx + dy * dy + dz * dz;
          }
          const bool ev = keep && r2 < p.model_cutsq;
          const int sj = static_cast<int>(xj.w);
          const T idx = pair_distance(r2) * p.inv_dr;
          const T fl = fmin(floor(idx), T(p.nr - 2));
          const T t = fmin(idx - fl, T(1));
          const int node = static_cast<int>(fl);
          T fj = T(0);
          if (ev) {
            const auto c = load4_tab(p.density + sj * p.nr + node);
            fj = c.x + t * (c.y + t * (c.z + t * c.w));
          }
          rho += fj;
          if (MODE == kDensityHalf || MODE == kDensityHalfOwned) {
            if (ev && (MODE == kDensityHalf || j < p.nlocal)) {
              T fi = fj;
              if (si != sj) {
                const auto c = load4_tab(p.density + si * p.nr + node);
                fi = c.x + t * (c.y + t * (c.z + t * c.w));
              }
              atomicAdd(p.rho + j, fi);
            }
          }
          if (MODE == kDensityHalfOwned)
            kept_twice += __popc(__ballot_sync(kFull, keep && j < p.nlocal));
          kept += __popc(m);
        }
      } else {
        // Group past capacity: walk the row's list with the exact test.
        const int n = min(listed, p.maxneighs);
        const long long rowbase = static_cast<long long>(i) * p.atom_stride;
        for (int base = 0; base < n; base += kWarp) {
          const int jj = base + lane;
          bool keep = false;
          int j = 0;
          double4 xj = make_double4(0.0, 0.0, 0.0, 0.0);
          if (jj < n) {
            j = p.neighbors[rowbase + static_cast<long long>(jj) * p.slot_stride] & kNeighMask;
            if (j < p.max_atoms && !(p.half_rule && j < i)) {
              xj = load4(p.xd4 + j);
              keep = pack_keep(p, i, xi, j, xj);
            }
          }
          const unsigned m = __ballot_sync(kFull, keep);
          if (keep) {
            const int at = kept + __popc(m & below);
            if (at < p.row_cap) crow[at] = j;
            T r2;
            if constexpr (sizeof(T) == 8) {
              r2 = pack_r2(xi, xj);
            } else {
              const float dx = static_cast<float>(xj.x) - fix, dy = static_cast<float>(xj.y) - fiy,
                          dz = static_cast<float>(xj.z) - fiz;
              r2 = dx * dx + dy * dy + dz * dz;
            }
            if (r2 < p.model_cutsq) {
              const T r = pair_distance(r2);
              const int sj = static_cast<int>(xj.w);
              const T fj = spline_v_dist<T>(p.density + sj * p.nr, p.nr, r, p.inv_dr);
              rho += fj;
              if (MODE == kDensityHalf || (MODE == kDensityHalfOwned && j < p.nlocal))
                atomicAdd(p.rho + j, si == sj ? fj
                                              : spline_v_dist<T>(p.density + si * p.nr, p.nr, r,
                                                                 p.inv_dr));
            }
          }
          if (MODE == kDensityHalfOwned)
            kept_twice += __popc(__ballot_sync(kFull, keep && j < p.nlocal));
          kept += __popc(m);
        }
      }
      rho = warp_sum(rho);
      if (lane == 0) {
        if (MODE == kDensityHalf || MODE == kDensityHalfOwned)
          atomicAdd(p.rho + i, rho);
        else
          p.rho[i] = rho;
        p.ccount[row] = kept;
      }
      kept_sum += kept + kept_twice;
    }
    if constexpr (!kDouble) __syncthreads();
  }
  // kept_sum is carried by every lane of a warp: count it once.
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, lane == 0 ? kept_sum : 0.0};
  store_partials(acc, widest, p.partials);
}

}  // namespace ljx
