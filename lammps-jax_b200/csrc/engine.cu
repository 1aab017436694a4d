// ljx engine: the extern "C" layer of include/ljx.h. Replaces the reference's PJRT runtime
// (cpp/pjrt/runtime.{h,cpp}) and the Kokkos pack/add/virial/comm functors of
// cpp/pair_jax_kokkos.cpp with hand-written sm_100a kernels (kernels.cuh, and groups.cuh for the
// row-group candidate cache). Buffers are sized once from the bundle contract; no call allocates
// or synchronizes except ljx_read_result.

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "bundle.h"
#include "groups.cuh"
#include "halo_internal.h"
#include "kernels.cuh"
#include "ljx.h"

#define LJX_VERSION "0.1.0"

namespace {

thread_local std::string g_bundle_error;

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void check(cudaError_t err, const char *what)
{
  if (err != cudaSuccess)
    throw CudaError(std::string(what) + ": " + cudaGetErrorString(err));
}

// Resident blocks per SM of `kernel` at `block` threads (at most 8), computed once per kernel.
// Engines on several host threads share the cache, hence the lock.
template <typename Kernel>
int blocks_per_sm(Kernel kernel, int block = ljx::kBlock)
{
  static std::mutex lock;
  static std::unordered_map<const void *, int> cache;
  const void *key = reinterpret_cast<const void *>(kernel);
  std::lock_guard<std::mutex> guard(lock);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, block, 0),
        "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  n = std::max(1, std::min(n, 8));
  cache.emplace(key, n);
  return n;
}

// Shared-memory carveout preference (percent of the unified L1/shared array) of the force pass,
// which uses almost no shared memory: 0 leaves the most L1 to its table and position gathers.
// Negative: the driver's choice. Set once per kernel, before its occupancy is computed.
#ifndef LJX_FORCE_CARVEOUT
#define LJX_FORCE_CARVEOUT 0
#endif
template <typename Kernel>
void prefer_carveout(Kernel kernel, int percent)
{
  if (percent < 0) return;
  static std::mutex lock;
  static std::unordered_map<const void *, bool> done;
  const void *key = reinterpret_cast<const void *>(kernel);
  std::lock_guard<std::mutex> guard(lock);
  if (done.count(key)) return;
  check(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, percent),
        "cudaFuncSetAttribute(carveout)");
  done.emplace(key, true);
}

}  // namespace

struct ljx_bundle {
  ljx::Bundle b;
};

struct ljx_engine {
  ljx::Bundle bundle;
  ljx_contract c{};
  int device = 0;
  int sm_count = 148;
  bool f64 = true;
  int rows_cap = 0;     // list rows the compacted buffer holds
  int row_cap = 0;      // kept pairs per compacted row
  int max_grid = 0;     // partial rows per kernel kind
  // Device buffers.
  double4 *xd4 = nullptr;
  void *pos4 = nullptr;
  void *rho = nullptr;
  void *fp = nullptr;
  int *cedges = nullptr;
  int *ccount = nullptr;
  unsigned char *ghost_rows = nullptr;  // per list row: keeps a ghost neighbor (density passes)
  void *embedding = nullptr;
  void *density = nullptr;
  void *density_slope = nullptr;
  void *pair = nullptr;
  unsigned int *coord_bound = nullptr;  // [0] largest |coordinate|, [1] largest displacement^2
  // Row-group candidate cache (EAM bundles).
  double4 *xref = nullptr;
  int *gatom = nullptr;
  int *gcount = nullptr;
  unsigned short *rslot = nullptr;
  int *rcount = nullptr;
  int gcap = 0;
  int rcap = 0;
  int groups_cap = 0;
  struct GroupKey {
    const int *ilist, *numneigh, *neighbors;
    long long atom_stride, slot_stride;
    int inum, maxneighs, nlocal, nall, half_rule, unique_rule;
    bool operator==(const GroupKey &o) const
    {
      return ilist == o.ilist && numneigh == o.numneigh && neighbors == o.neighbors &&
             atom_stride == o.atom_stride && slot_stride == o.slot_stride && inum == o.inum &&
             maxneighs == o.maxneighs && nlocal == o.nlocal && nall == o.nall &&
             half_rule == o.half_rule && unique_rule == o.unique_rule;
    }
  };
  bool groups_valid = false;
  GroupKey groups_key{};
  long long group_builds = 0;  // host-requested cache builds
  int list_age_steps = 0;      // density calls since the last fresh list (ago == 0)
  int list_period = 1 << 30;   // lifetime in steps of the previous list (unknown at first)
  bool period_cached = true;   // the current list's steps run over the candidate cache
  int *senders = nullptr;
  int *receivers = nullptr;
  uint8_t *edge_mask = nullptr;
  long long *offsets = nullptr;
  long long *count_prev = nullptr;
  double *partials = nullptr;   // [4][max_grid][kPartialWidth]: density, embed, force, lj
  double *result = nullptr;     // [9]
  double *host_result = nullptr;
  // Step state: partial rows written by this step's kernels.
  int step_blocks[4] = {0, 0, 0, 0};
  int last_nlocal = 0;
  int last_nall = 0;
  double last_scale = 1.0;
  int last_duplicate = 1;
  // Per-atom tallies (ljx_set_atom_tallies): caller-owned device arrays, null when off.
  double *eatom = nullptr;
  double *vatom = nullptr;
  double tally_scale = 1.0;
  long long launches = 0;
  // ljx_force_to_host: the copy stream and the events that order it after each piece of the
  // force pass; the row-order check word (device, and its pinned landing slot) and whether this
  // step's result read must look at it.
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t piece_done[17] = {};
  int *order_bad = nullptr;       // device: rows r with ilist[r] != r (result slot 12)
  int *host_order_bad = nullptr;  // pinned: its copy (host_result slot 12)
  bool rows_streamed = false;
  bool step_ev = true;            // false after ljx_force_only: the result has no energy/virial
  bool owned_half = true;         // allow owned pairs held once (LJX_OWNED_HALF, default on)
  bool rows_owned_half = false;   // the last ljx_density compacted rows that hold them once
  // ljx_force_rows: partial rows of this step's local-rows pass, which the ghost-rows pass
  // writes after (-1: no local-rows pass since the last ljx_density).
  int local_part_blocks = -1;
  std::string error;

  ~ljx_engine()
  {
    cudaSetDevice(device);
    for (cudaEvent_t ev : piece_done)
      if (ev) cudaEventDestroy(ev);
    if (copy_stream) cudaStreamDestroy(copy_stream);
    void *ptrs[] = {xd4,       pos4,      rho,        fp,          cedges,  ccount,
                    embedding, density,   density_slope, pair,     coord_bound, xref,
                    gatom,     gcount,    rslot,      rcount,      senders,
                    receivers, edge_mask, offsets,    count_prev,  partials, result,
                    ghost_rows};
    for (void *p : ptrs)
      if (p) cudaFree(p);
    if (host_result) cudaFreeHost(host_result);
  }

  double *partial(int kind) const
  {
    return partials + static_cast<long long>(kind) * max_grid * ljx::kPartialWidth;
  }
};

namespace {

enum PartialKind { kDensityPart = 0, kEmbedPart = 1, kForcePart = 2, kLjPart = 3 };

struct DeviceGuard {
  int previous = -1;
  explicit DeviceGuard(int device)
  {
    check(cudaGetDevice(&previous), "cudaGetDevice");
    if (previous != device) check(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceGuard()
  {
    int now = -1;
    if (cudaGetDevice(&now) == cudaSuccess && now != previous && previous >= 0)
      cudaSetDevice(previous);
  }
};

template <typename F>
ljx_status guarded(ljx_engine *e, F &&body)
{
  if (e == nullptr) return LJX_ERR_INVALID;
  try {
    DeviceGuard guard(e->device);
    return body();
  } catch (const CudaError &err) {
    e->error = err.what();
    return LJX_ERR_CUDA;
  } catch (const std::exception &err) {
    e->error = err.what();
    return LJX_ERR_INVALID;
  }
}

ljx_status fail(ljx_engine *e, ljx_status status, const std::string &message)
{
  e->error = message;
  return status;
}

void *device_alloc(size_t bytes, const char *what)
{
  void *p = nullptr;
  if (bytes == 0) bytes = 16;
  check(cudaMalloc(&p, bytes), what);
  return p;
}

template <typename T>
void *upload_table(const std::vector<double> &values)
{
  std::vector<T> cast(values.begin(), values.end());
  void *p = device_alloc(cast.size() * sizeof(T), "cudaMalloc(table)");
  check(cudaMemcpy(p, cast.data(), cast.size() * sizeof(T), cudaMemcpyHostToDevice),
        "cudaMemcpy(table)");
  return p;
}

// Force distribution and list kind, decided as PairJaxKokkos::half_list / compute do.
struct Modes {
  bool half_list = false;
  int density = ljx::kDensityFull;
  int force = ljx::kRowsFull;
  int lj = ljx::kLjEdgeFull;
  bool forward_fp = false;
  bool reverse_density = false;
  bool reverse_force = false;
  bool duplicate = false;
  bool owned_half = false;  // owned pairs held once (kDensityHalfOwned / kRowsHalfOwned)
};

Modes decide_modes(const ljx_contract &c, int newton_pair)
{
  Modes m;
  const bool comm = c.n_comm_widths > 0;
  const bool matrix = c.input_layout == LJX_LAYOUT_NEIGHBOR_MATRIX;
  const bool edge_force = c.force_layout == LJX_FORCE_EDGE;
  // cpp/pair_jax_kokkos.cpp:425-431.
  if (!newton_pair)
    m.half_list = false;
  else if (comm)
    m.half_list = c.half_edges != 0;
  else if (matrix)
    m.half_list = false;
  else
    m.half_list = c.n_hops == 1 && (edge_force || c.pair_sum);
  m.duplicate = newton_pair && c.pair_sum && !edge_force && c.n_hops == 1 && !comm;
  if (c.potential == LJX_POTENTIAL_EAM) {
    if (m.half_list) {
      m.density = ljx::kDensityHalf;
      m.force = ljx::kHalf;
      m.reverse_density = true;
      m.forward_fp = true;
      m.reverse_force = true;
    } else if (newton_pair) {
      m.force = ljx::kGhost;
      m.reverse_force = true;
    } else {
      m.force = ljx::kRowsFull;
      m.forward_fp = true;
    }
  } else if (c.potential == LJX_POTENTIAL_LJ) {
    if (edge_force)
      m.lj = m.half_list ? ljx::kLjEdgeHalf : ljx::kLjEdgeFull;
    else
      m.lj = m.half_list ? ljx::kLjAtomHalfPairSum : ljx::kLjAtomFull;
    m.reverse_force = newton_pair != 0;
  }
  return m;
}

// The modes a step runs with. EAM full lists with newton off hold each owned pair once
// (kDensityHalfOwned / kRowsHalfOwned) unless the bundle has its own pairing rule, per-atom
// tallies are registered, some owned atom has no list row (an owned pair must be held by the row
// of its lower atom), or LJX_OWNED_HALF=0. ljx_density decides and records it; the force and
// energy passes of the step follow the compacted rows it wrote.
Modes density_modes(ljx_engine *e, int newton_pair, int inum, int nlocal)
{
  Modes m = decide_modes(e->c, newton_pair);
  if (e->owned_half && e->c.potential == LJX_POTENTIAL_EAM && m.force == ljx::kRowsFull &&
      !e->c.half_edges && e->eatom == nullptr && e->vatom == nullptr && inum == nlocal) {
    m.owned_half = true;
    m.density = ljx::kDensityHalfOwned;
    m.force = ljx::kRowsHalfOwned;
  }
  e->rows_owned_half = m.owned_half;
  return m;
}

Modes pass_modes(const ljx_engine *e, int newton_pair)
{
  Modes m = decide_modes(e->c, newton_pair);
  if (e->rows_owned_half && m.force == ljx::kRowsFull) {
    m.owned_half = true;
    m.density = ljx::kDensityHalfOwned;
    m.force = ljx::kRowsHalfOwned;
  }
  return m;
}

template <typename T>
ljx::Step<T> make_step(ljx_engine *e, const ljx_atoms *a, const ljx_list *l, double scale)
{
  using V = typename ljx::Vec4<T>::type;
  ljx::Step<T> p{};
  if (a) {
    p.x = a->x;
    p.type = a->type;
    p.f = a->f;
    p.nlocal = a->nlocal;
    p.nghost = a->nghost;
    p.nall = a->nlocal + a->nghost;
  }
  if (l) {
    p.ilist = l->ilist;
    p.numneigh = l->numneigh;
    p.neighbors = l->neighbors;
    p.atom_stride = l->atom_stride;
    p.slot_stride = l->slot_stride;
    p.inum = l->inum;
    p.maxneighs = std::max(1, l->maxneighs);
  }
  p.xd4 = e->xd4;
  p.pos4 = static_cast<V *>(e->pos4);
  p.rho = static_cast<T *>(e->rho);
  p.fp = static_cast<T *>(e->fp);
  p.cedges = e->cedges;
  p.ccount = e->ccount;
  p.ghost_rows = e->ghost_rows;
  p.row_part = ljx::kRowsAll;
  p.row_cap = e->row_cap;
  p.embedding = static_cast<const V *>(e->embedding);
  p.density = static_cast<const V *>(e->density);
  p.density_slope = static_cast<const V *>(e->density_slope);
  p.pair = static_cast<const V *>(e->pair);
  p.coord_bound = e->coord_bound;
  p.disp_bound = e->coord_bound + 1;
  p.xref = e->xref;
  p.gatom = e->gatom;
  p.gcount = e->gcount;
  p.gcap = e->gcap;
  p.rslot = e->rslot;
  p.rcount = e->rcount;
  p.rcap = e->rcap;
  p.n_species = e->c.potential == LJX_POTENTIAL_EAM ? std::max(1, e->bundle.eam.n_elements) : 1;
  p.nrho = e->bundle.eam.nrho;
  p.nr = e->bundle.eam.nr;
  p.drho = static_cast<T>(e->bundle.eam.drho);
  p.inv_dr = e->bundle.eam.dr > 0 ? static_cast<T>(1.0 / e->bundle.eam.dr) : T(0);
  p.pack_cutsq = e->c.cutoff * e->c.cutoff;
  const double model_cut =
      e->c.potential == LJX_POTENTIAL_EAM ? e->bundle.eam.cutoff : e->c.cutoff;
  p.model_cutsq = static_cast<T>(model_cut * model_cut);
  p.max_atoms = e->c.max_atoms;
  p.scale = scale;
  p.lj_four_eps = static_cast<T>(4.0 * e->c.lj_epsilon);
  p.lj_sigma_sq = static_cast<T>(e->c.lj_sigma * e->c.lj_sigma);
  p.lj_energy_scale = static_cast<T>(e->c.lj_edge_energy_scale);
  p.eatom = e->eatom;
  p.vatom = e->vatom;
  p.tally_scale = e->tally_scale;
  return p;
}

// Packer rules of cpp/pair_jax_kokkos.cpp:853-865 for the list the run hands over.
template <typename T>
void set_pack_rules(ljx::Step<T> &p, const ljx_contract &c, const Modes &m)
{
  const bool full_list = !m.half_list;
  // Owned pairs held once keep the owned neighbors j > i and every ghost: the half rule's filter.
  p.half_rule = (c.half_edges && full_list) || m.owned_half;
  p.unique_rule = c.half_edges && c.n_comm_widths > 0 && full_list;
}

int row_grid(ljx_engine *e, int rows, int per_sm)
{
  const int need = (rows + ljx::kWarpsPerBlock - 1) / ljx::kWarpsPerBlock;
  return std::max(1, std::min(need, std::min(e->max_grid, e->sm_count * per_sm)));
}

int flat_grid(long long items)
{
  const long long need = (items + ljx::kBlock - 1) / ljx::kBlock;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(need, 148LL * 16)));
}

void check_launch(const char *what) { check(cudaGetLastError(), what); }

ljx_status check_capacity(ljx_engine *e, const ljx_atoms *a)
{
  // Pre-launch row limits, cpp/pair_jax_kokkos.cpp:1035-1046 (rank-local values; the pair
  // style takes the global max first).
  const int nall = a->nlocal + a->nghost;
  if (nall > e->c.max_atoms)
    return fail(e, LJX_ERR_CAPACITY,
                "LAMMPS-JAX atom capacity exceeded: global max " + std::to_string(nall) +
                    " atoms, capacity " + std::to_string(e->c.max_atoms));
  if (e->c.max_owned > 0 && a->nlocal > e->c.max_owned)
    return fail(e, LJX_ERR_CAPACITY,
                "LAMMPS-JAX owned-row capacity exceeded: global max " +
                    std::to_string(a->nlocal) + " owned atoms, capacity " +
                    std::to_string(e->c.max_owned));
  return LJX_OK;
}

ljx_status check_list(ljx_engine *e, const ljx_list *l)
{
  if (l == nullptr || (l->inum > 0 && (!l->ilist || !l->numneigh || !l->neighbors)))
    return fail(e, LJX_ERR_INVALID, "neighbor list view is incomplete");
  if (l->inum > e->rows_cap)
    return fail(e, LJX_ERR_CAPACITY,
                "LAMMPS-JAX owned-row capacity exceeded: global max " + std::to_string(l->inum) +
                    " list rows, capacity " + std::to_string(e->rows_cap));
  if (l->gnum > 0)
    return fail(e, LJX_ERR_UNSUPPORTED, "ljx runs single-hop bundles; ghost list rows are unused");
  return LJX_OK;
}

template <typename T>
void launch_density(ljx_engine *e, cudaStream_t s, const ljx::Step<T> &p, int mode)
{
  if (p.inum <= 0) return;
  int grid = 0;
  switch (mode) {
    case ljx::kDensityHalf:
      grid = row_grid(e, p.inum, blocks_per_sm(ljx::k_density<T, ljx::kDensityHalf>));
      ljx::k_density<T, ljx::kDensityHalf><<<grid, ljx::kBlock, 0, s>>>(p);
      break;
    case ljx::kDensityHalfOwned:
      grid = row_grid(e, p.inum, blocks_per_sm(ljx::k_density<T, ljx::kDensityHalfOwned>));
      ljx::k_density<T, ljx::kDensityHalfOwned><<<grid, ljx::kBlock, 0, s>>>(p);
      break;
    case ljx::kCompactOnly:
      grid = row_grid(e, p.inum, blocks_per_sm(ljx::k_density<T, ljx::kCompactOnly>));
      ljx::k_density<T, ljx::kCompactOnly><<<grid, ljx::kBlock, 0, s>>>(p);
      break;
    default:
      grid = row_grid(e, p.inum, blocks_per_sm(ljx::k_density<T, ljx::kDensityFull>));
      ljx::k_density<T, ljx::kDensityFull><<<grid, ljx::kBlock, 0, s>>>(p);
  }
  check_launch("k_density");
  e->launches++;
  e->step_blocks[kDensityPart] = grid;
}

// Cache margin as a fraction of the pack cutoff: unions hold pairs within rc (1 + margin) and
// stay valid until some atom has moved rc * margin / 2.
#ifndef LJX_GROUP_MARGIN
#define LJX_GROUP_MARGIN 0.08
#endif
constexpr double kGroupMargin = LJX_GROUP_MARGIN;
// Shortest list lifetime (steps) for which the candidate cache is built.
constexpr int kCacheMinPeriod = 4;

template <typename T>
void launch_groups(ljx_engine *e, cudaStream_t s, const ljx::Step<T> &p, int ago, int mode)
{
  if (p.inum <= 0) return;
  const ljx_engine::GroupKey key{p.ilist,      p.numneigh, p.neighbors, p.atom_stride,
                                 p.slot_stride, p.inum,     p.maxneighs, p.nlocal,
                                 p.nall,        p.half_rule, p.unique_rule};
  const bool rebuild = ago == 0 || !e->groups_valid || !(key == e->groups_key);
  const double rc = std::sqrt(p.pack_cutsq);
  const double half_margin = 0.5 * kGroupMargin * rc;
  // Rounded down: the device rebuilds as soon as the float displacement^2 passes it.
  const float disp_limit = std::nextafter(static_cast<float>(half_margin * half_margin), 0.0f);
  const double cand = rc * (1.0 + kGroupMargin);
  const int span = std::min(p.nall, e->c.max_atoms);
  const int groups = (p.inum + ljx::kGroupRows - 1) / ljx::kGroupRows;
  // Half rows (half lists, owned pairs held once) build with a set half the size.
  auto build = [&](auto kernel) {
    const int bgrid = std::max(1, std::min((groups + ljx::kBuildWarps - 1) / ljx::kBuildWarps,
                                           e->sm_count * blocks_per_sm(kernel, ljx::kBuildBlock)));
    kernel<<<bgrid, ljx::kBuildBlock, 0, s>>>(p, span, rebuild ? 1 : 0, disp_limit, cand * cand);
  };
  if (mode == ljx::kDensityHalf || mode == ljx::kDensityHalfOwned)
    build(ljx::k_build_groups<T, LJX_BUILD_HALF_HASH>);
  else
    build(ljx::k_build_groups<T>);
  check_launch("k_build_groups");
  e->launches++;
  if (rebuild) e->group_builds++;
  e->groups_valid = true;
  e->groups_key = key;
  const int need = groups;  // one block per group
  // The build applied the owned-pairs half rule already; other rules are re-checked each step.
  const bool rules = (p.half_rule && mode != ljx::kDensityHalfOwned) || p.unique_rule;
  auto run = [&](auto kernel) {
    const int grid = std::max(1, std::min(need, std::min(e->max_grid,
                                                         e->sm_count * blocks_per_sm(kernel))));
    kernel<<<grid, ljx::kBlock, 0, s>>>(p);
    return grid;
  };
  int grid = 0;
  if (mode == ljx::kDensityHalf)
    grid = rules ? run(ljx::k_density_groups<T, ljx::kDensityHalf, true, ljx::kHalfUnion>)
                 : run(ljx::k_density_groups<T, ljx::kDensityHalf, false, ljx::kHalfUnion>);
  else if (mode == ljx::kDensityHalfOwned)
    grid = run(ljx::k_density_groups<T, ljx::kDensityHalfOwned, false, LJX_OWNED_UNION>);
  else
    grid = rules ? run(ljx::k_density_groups<T, ljx::kDensityFull, true>)
                 : run(ljx::k_density_groups<T, ljx::kDensityFull, false>);
  check_launch("k_density_groups");
  e->launches++;
  e->step_blocks[kDensityPart] = grid;
}

// block0 / cap: a pass launched in pieces (ljx_force_to_host) writes its partial rows after
// those of the earlier pieces, at most `cap` blocks (0: no cap).
template <typename T, bool FORCES, bool TALLY, bool EV = true>
int launch_force_as(ljx_engine *e, cudaStream_t s, const ljx::Step<T> &p, int mode,
                    int block0 = 0, int cap = 0, int waves = 1)
{
  auto run = [&](auto kernel) {
    prefer_carveout(kernel, LJX_FORCE_CARVEOUT);
    int grid = row_grid(e, p.inum, blocks_per_sm(kernel) * waves);
    if (cap > 0) grid = std::min(grid, cap);
    kernel<<<grid, ljx::kBlock, 0, s>>>(p);
    return grid;
  };
  int grid = 0;
  switch (mode) {
    case ljx::kGhost: grid = run(ljx::k_force<T, ljx::kGhost, FORCES, TALLY, EV>); break;
    case ljx::kHalf: grid = run(ljx::k_force<T, ljx::kHalf, FORCES, TALLY, EV>); break;
    case ljx::kRowsHalfOwned:
      // Never with per-atom tallies: the density pass then keeps full rows.
      if constexpr (!TALLY) grid = run(ljx::k_force<T, ljx::kRowsHalfOwned, FORCES, false, EV>);
      break;
    default: grid = run(ljx::k_force<T, ljx::kRowsFull, FORCES, TALLY, EV>);
  }
  check_launch("k_force");
  e->launches++;
  // A force-only pass writes no partial sums.
  e->step_blocks[kForcePart] = EV ? block0 + grid : 0;
  return grid;
}

template <typename T, bool FORCES = true>
int launch_force(ljx_engine *e, cudaStream_t s, const ljx::Step<T> &p, int mode, int block0 = 0,
                 int cap = 0, int waves = 1)
{
  if (p.inum <= 0) return 0;
  // The per-atom tally variants run only when a caller asked for per-atom output.
  if (p.eatom != nullptr || p.vatom != nullptr)
    return launch_force_as<T, FORCES, true>(e, s, p, mode, block0, cap, waves);
  return launch_force_as<T, FORCES, false>(e, s, p, mode, block0, cap, waves);
}

template <typename T, bool FORCES, bool TALLY>
void launch_lj_as(ljx_engine *e, cudaStream_t s, const ljx::Step<T> &p, int mode)
{
  int grid = 0;
  switch (mode) {
    case ljx::kLjEdgeHalf:
      grid = row_grid(e, p.inum, blocks_per_sm(ljx::k_lj<T, ljx::kLjEdgeHalf, FORCES, TALLY>));
      ljx::k_lj<T, ljx::kLjEdgeHalf, FORCES, TALLY><<<grid, ljx::kBlock, 0, s>>>(p);
      break;
    case ljx::kLjAtomFull:
      grid = row_grid(e, p.inum, blocks_per_sm(ljx::k_lj<T, ljx::kLjAtomFull, FORCES, TALLY>));
      ljx::k_lj<T, ljx::kLjAtomFull, FORCES, TALLY><<<grid, ljx::kBlock, 0, s>>>(p);
      break;
    case ljx::kLjAtomHalfPairSum:
      grid = row_grid(e, p.inum,
                      blocks_per_sm(ljx::k_lj<T, ljx::kLjAtomHalfPairSum, FORCES, TALLY>));
      ljx::k_lj<T, ljx::kLjAtomHalfPairSum, FORCES, TALLY><<<grid, ljx::kBlock, 0, s>>>(p);
      break;
    default:
      grid = row_grid(e, p.inum, blocks_per_sm(ljx::k_lj<T, ljx::kLjEdgeFull, FORCES, TALLY>));
      ljx::k_lj<T, ljx::kLjEdgeFull, FORCES, TALLY><<<grid, ljx::kBlock, 0, s>>>(p);
  }
  check_launch("k_lj");
  e->launches++;
  e->step_blocks[kLjPart] = grid;
}

template <typename T, bool FORCES = true>
void launch_lj(ljx_engine *e, cudaStream_t s, const ljx::Step<T> &p, int mode)
{
  if (p.inum <= 0) return;
  if (p.eatom != nullptr || p.vatom != nullptr)
    launch_lj_as<T, FORCES, true>(e, s, p, mode);
  else
    launch_lj_as<T, FORCES, false>(e, s, p, mode);
}

template <typename T>
ljx_status pack_edges_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a, const ljx_list *l,
                           int newton_pair)
{
  const Modes m = decide_modes(e->c, newton_pair);
  ljx::Step<T> p = make_step<T>(e, a, l, 1.0);
  set_pack_rules(p, e->c, m);
  p.partials = e->partial(kDensityPart);
  launch_density<T>(e, s, p, ljx::kCompactOnly);
  const int rows = std::max(0, p.inum);
  ljx::k_scan_counts<<<1, 1024, 0, s>>>(e->ccount, rows, m.duplicate ? 2 : 1, e->offsets);
  check_launch("k_scan_counts");
  e->launches++;
  if (rows > 0) {
    const int grid = row_grid(e, rows, blocks_per_sm(ljx::k_emit_edges<T>));
    ljx::k_emit_edges<T><<<grid, ljx::kBlock, 0, s>>>(p, e->offsets, m.duplicate ? 1 : 0,
                                                       e->c.max_edges, e->senders, e->receivers,
                                                       e->edge_mask);
    check_launch("k_emit_edges");
    e->launches++;
  }
  ljx::k_reset_tail<<<e->sm_count * 4, ljx::kBlock, 0, s>>>(e->offsets + rows, e->count_prev,
                                                            e->c.max_atoms, e->c.max_edges,
                                                            e->senders, e->receivers, e->edge_mask);
  check_launch("k_reset_tail");
  ljx::k_store_prev<<<1, 1, 0, s>>>(e->offsets + rows, e->count_prev);
  check_launch("k_store_prev");
  e->launches += 2;
  e->last_duplicate = m.duplicate ? 2 : 1;
  return LJX_OK;
}

template <typename T>
ljx_status density_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a, const ljx_list *l,
                        int newton_pair)
{
  const Modes m = density_modes(e, newton_pair, l ? l->inum : 0, a ? a->nlocal : 0);
  e->local_part_blocks = -1;
  if (e->c.potential == LJX_POTENTIAL_LJ) return LJX_OK;  // LJ is one pass (ljx_force)
  ljx::Step<T> p = make_step<T>(e, a, l, 1.0);
  set_pack_rules(p, e->c, m);
  p.partials = e->partial(kDensityPart);
  if (m.density == ljx::kDensityHalf) {
    // Half lists scatter into neighbor rows, ghosts included: start from zero.
    const long long rows = std::min<long long>(p.nall, e->c.max_atoms);
    check(cudaMemsetAsync(e->rho, 0, rows * sizeof(T), s), "cudaMemsetAsync(rho)");
  } else if ((m.density == ljx::kDensityHalfOwned || p.inum < p.nlocal) && p.nlocal > 0) {
    // Owned pairs held once scatter into owned rows only; owned atoms without a list row have
    // no density term (the reference's segment sum over their edges is empty).
    check(cudaMemsetAsync(e->rho, 0, static_cast<long long>(p.nlocal) * sizeof(T), s),
          "cudaMemsetAsync(rho)");
  }
  // Candidate cache policy. A build costs about as much as one list pass plus a third, and each
  // later step over the cache saves about a quarter of a list pass (C3), so a list has to live
  // kCacheMinPeriod steps for the cache to pay. LAMMPS rebuilds lists at a steady rhythm, so
  // the previous list's lifetime decides, at each fresh list, whether its steps use the cache.
  bool cached = l->ago >= 0 && e->xref != nullptr;
  if (cached) {
    if (l->ago == 0) {
      if (e->list_age_steps > 0) e->list_period = e->list_age_steps;
      e->list_age_steps = 0;
      e->period_cached = e->list_period >= kCacheMinPeriod;
    }
    ++e->list_age_steps;
    cached = e->period_cached;
  }
  if (cached)
    launch_groups<T>(e, s, p, l->ago, m.density);
  else
    launch_density<T>(e, s, p, m.density);
  e->last_duplicate = m.duplicate ? 2 : 1;
  return LJX_OK;
}

template <typename T>
ljx_status embed_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a)
{
  if (e->c.potential != LJX_POTENTIAL_EAM) return LJX_OK;
  ljx::Step<T> p = make_step<T>(e, a, nullptr, 1.0);
  p.partials = e->partial(kEmbedPart);
  if (p.nlocal <= 0) return LJX_OK;
  const int per = blocks_per_sm(ljx::k_embed<T>);
  const int need = (p.nlocal + ljx::kBlock - 1) / ljx::kBlock;
  const int grid = std::max(1, std::min(need, std::min(e->max_grid, e->sm_count * per)));
  ljx::k_embed<T><<<grid, ljx::kBlock, 0, s>>>(p);
  check_launch("k_embed");
  e->launches++;
  e->step_blocks[kEmbedPart] = grid;
  return LJX_OK;
}

template <typename T>
ljx_status force_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a, const ljx_list *l,
                      int newton_pair, double scale)
{
  const Modes m = pass_modes(e, newton_pair);
  ljx::Step<T> p = make_step<T>(e, a, l, scale);
  set_pack_rules(p, e->c, m);
  e->last_scale = scale;
  e->step_ev = true;
  if (e->c.potential == LJX_POTENTIAL_LJ) {
    p.partials = e->partial(kLjPart);
    launch_lj<T>(e, s, p, m.lj);
    e->last_duplicate = m.duplicate ? 2 : 1;
    return LJX_OK;
  }
  p.partials = e->partial(kForcePart);
  launch_force<T>(e, s, p, m.force);
  return LJX_OK;
}

// One part of the EAM force pass (ljx_force_rows): the list rows that keep no ghost neighbor
// (LJX_ROWS_LOCAL) or the others (LJX_ROWS_GHOST), as this step's ljx_density marked them. The
// local rows read no ghost F', so they can run while the F' exchange is in flight. The ghost
// part writes its energy and virial partial rows after the local part's, so the step's result
// sums both.
#ifndef LJX_LOCAL_WAVES
#define LJX_LOCAL_WAVES 8
#endif
template <typename T>
ljx_status force_rows_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a, const ljx_list *l,
                           int newton_pair, double scale, int part)
{
  if (e->c.potential != LJX_POTENTIAL_EAM)
    return fail(e, LJX_ERR_UNSUPPORTED, "the force pass splits by ghost rows for EAM bundles only");
  if (part != LJX_ROWS_LOCAL && part != LJX_ROWS_GHOST)
    return fail(e, LJX_ERR_INVALID, "row part must be LJX_ROWS_LOCAL or LJX_ROWS_GHOST");
  if (part == LJX_ROWS_GHOST && e->local_part_blocks < 0)
    return fail(e, LJX_ERR_INVALID,
                "ljx_force_rows(LJX_ROWS_GHOST) must follow ljx_force_rows(LJX_ROWS_LOCAL) after "
                "the same ljx_density");
  const Modes m = pass_modes(e, newton_pair);
  ljx::Step<T> p = make_step<T>(e, a, l, scale);
  set_pack_rules(p, e->c, m);
  p.row_part = part == LJX_ROWS_LOCAL ? ljx::kRowsLocal : ljx::kRowsGhost;
  e->last_scale = scale;
  e->step_ev = true;
  // The local part runs beside the exchange's NCCL kernels, which hold some SMs' block slots
  // when it starts. Launched as one wave of resident blocks, each walking its share of the rows,
  // the blocks that find no slot would start only when others finish and run their whole share
  // after them; as LJX_LOCAL_WAVES waves, a late block takes a small share. Each part writes at
  // most half of the force partial rows.
  const int block0 = part == LJX_ROWS_LOCAL ? 0 : e->local_part_blocks;
  p.partials = e->partial(kForcePart) + static_cast<long long>(block0) * ljx::kPartialWidth;
  const int grid = launch_force<T>(e, s, p, m.force, block0, e->max_grid / 2,
                                   part == LJX_ROWS_LOCAL ? LJX_LOCAL_WAVES : 1);
  e->local_part_blocks = part == LJX_ROWS_LOCAL ? grid : -1;
  return LJX_OK;
}

// Forces alone (ljx_force_only): the EAM force pass without its energy and virial sums; LJ runs
// its one pass as ljx_force does. The step's result then reports no energy or virial.
template <typename T>
ljx_status force_only_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a, const ljx_list *l,
                           int newton_pair, double scale)
{
  if (e->c.potential == LJX_POTENTIAL_LJ || e->eatom != nullptr || e->vatom != nullptr) {
    const ljx_status st = force_impl<T>(e, s, a, l, newton_pair, scale);
    e->step_ev = false;
    return st;
  }
  const Modes m = pass_modes(e, newton_pair);
  ljx::Step<T> p = make_step<T>(e, a, l, scale);
  set_pack_rules(p, e->c, m);
  e->last_scale = scale;
  p.partials = e->partial(kForcePart);
  if (p.inum > 0) launch_force_as<T, true, false, false>(e, s, p, m.force);
  e->step_ev = false;
  return LJX_OK;
}

// Rows r of the list whose atom is not r (ljx_force_to_host copies atom ranges by row ranges).
__global__ void k_rows_in_order(const int *ilist, int inum, int *bad)
{
  int count = 0;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < inum; r += gridDim.x * blockDim.x)
    count += ilist[r] != r;
  count = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(count));
  if ((threadIdx.x & 31) == 0 && count) atomicAdd(bad, count);
}

// The force pass in `pieces` consecutive row ranges; after each, its owned rows of f go to the
// host on the engine's copy stream. Row r is atom r (checked on the device), so a row range is
// an atom range of f.
template <typename T>
ljx_status force_to_host_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a,
                              const ljx_list *l, int newton_pair, double scale, double *f_host,
                              int pieces)
{
  const Modes m = pass_modes(e, newton_pair);
  const bool lj = e->c.potential == LJX_POTENTIAL_LJ;
  // Owned pairs held once scatter only into rows of higher index (j > i), so after each piece
  // every row before its end is final too.
  if (lj ? m.lj != ljx::kLjEdgeFull
         : (m.force != ljx::kRowsFull && m.force != ljx::kRowsHalfOwned))
    return fail(e, LJX_ERR_UNSUPPORTED,
                "force rows stream to the host only when each list row holds its atom's whole "
                "force (full list, newton off)");
  if (e->copy_stream == nullptr)
    check(cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking),
          "cudaStreamCreateWithFlags(copy)");
  for (cudaEvent_t &ev : e->piece_done)
    if (ev == nullptr) check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
  ljx::Step<T> p = make_step<T>(e, a, l, scale);
  set_pack_rules(p, e->c, m);
  e->last_scale = scale;
  const int inum = std::max(0, std::min(p.inum, a->nlocal));
  check(cudaMemsetAsync(e->order_bad, 0, sizeof(int), s), "cudaMemsetAsync(order)");
  if (inum > 0) {
    k_rows_in_order<<<flat_grid(inum), ljx::kBlock, 0, s>>>(p.ilist, inum, e->order_bad);
    check_launch("k_rows_in_order");
    e->launches++;
  }
  check(cudaMemcpyAsync(e->host_order_bad, e->order_bad, sizeof(int), cudaMemcpyDeviceToHost, s),
        "cudaMemcpyAsync(order)");
  const int part = lj ? kLjPart : kForcePart;
  double *partials = e->partial(part);
  const int cap = e->max_grid / pieces;
  const bool tally = p.eatom != nullptr || p.vatom != nullptr;
  int blocks = 0;
  for (int k = 0; k < pieces; ++k) {
    const int r0 = static_cast<int>(static_cast<long long>(inum) * k / pieces);
    const int r1 = static_cast<int>(static_cast<long long>(inum) * (k + 1) / pieces);
    ljx::Step<T> q = p;
    q.ilist = p.ilist + r0;
    q.ccount = p.ccount + r0;
    q.cedges = p.cedges + static_cast<long long>(r0) * p.row_cap;
    q.inum = r1 - r0;
    q.partials = partials + static_cast<long long>(blocks) * ljx::kPartialWidth;
    if (q.inum > 0) {
      if (lj) {
        auto run = [&](auto kernel) {
          const int grid = std::min(row_grid(e, q.inum, blocks_per_sm(kernel)), cap);
          kernel<<<grid, ljx::kBlock, 0, s>>>(q);
          return grid;
        };
        blocks += tally ? run(ljx::k_lj<T, ljx::kLjEdgeFull, true, true>)
                        : run(ljx::k_lj<T, ljx::kLjEdgeFull, true, false>);
        check_launch("k_lj");
        e->launches++;
        e->step_blocks[kLjPart] = blocks;
      } else {
        blocks += launch_force<T>(e, s, q, m.force, blocks, cap);
      }
    }
    // Rows r0..r1-1 of f are final; the last piece also takes owned atoms without a list row.
    const int c1 = k + 1 == pieces ? a->nlocal : r1;
    check(cudaEventRecord(e->piece_done[k], s), "cudaEventRecord(piece)");
    if (c1 > r0) {
      check(cudaStreamWaitEvent(e->copy_stream, e->piece_done[k], 0), "cudaStreamWaitEvent(copy)");
      check(cudaMemcpyAsync(f_host + 3LL * r0, a->f + 3LL * r0,
                            3ULL * static_cast<size_t>(c1 - r0) * sizeof(double),
                            cudaMemcpyDeviceToHost, e->copy_stream),
            "cudaMemcpyAsync(f rows)");
    }
  }
  if (lj) e->last_duplicate = m.duplicate ? 2 : 1;
  check(cudaEventRecord(e->piece_done[16], e->copy_stream), "cudaEventRecord(copies)");
  check(cudaStreamWaitEvent(s, e->piece_done[16], 0), "cudaStreamWaitEvent(stream)");
  e->rows_streamed = true;
  return LJX_OK;
}

// Energy-only evaluation (the reference's execute_energy path for eflag_only steps,
// cpp/pair_jax_kokkos.cpp:997-1001,1051-1053): the pair energy over the compacted rows (EAM,
// after ljx_density and ljx_embed) or the LJ energy over the list. No F' is read and no force or
// virial is written.
template <typename T>
ljx_status energy_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a, const ljx_list *l,
                       int newton_pair, double scale)
{
  const Modes m = pass_modes(e, newton_pair);
  ljx::Step<T> p = make_step<T>(e, a, l, scale);
  set_pack_rules(p, e->c, m);
  e->last_scale = scale;
  if (e->c.potential == LJX_POTENTIAL_LJ) {
    p.partials = e->partial(kLjPart);
    launch_lj<T, false>(e, s, p, m.lj);
    e->last_duplicate = m.duplicate ? 2 : 1;
    return LJX_OK;
  }
  p.partials = e->partial(kForcePart);
  launch_force<T, false>(e, s, p, m.force);
  return LJX_OK;
}

template <typename T>
ljx_status pack_atoms_impl(ljx_engine *e, cudaStream_t s, const ljx_atoms *a)
{
  ljx::Step<T> p = make_step<T>(e, a, nullptr, 1.0);
  const int span = std::min(p.nall, e->c.max_atoms);
  check(cudaMemsetAsync(e->coord_bound, 0, 2 * sizeof(unsigned int), s), "cudaMemsetAsync(bound)");
  if (span <= 0) return LJX_OK;
  ljx::k_pack_atoms<T><<<flat_grid(span), ljx::kBlock, 0, s>>>(p, span);
  check_launch("k_pack_atoms");
  e->launches++;
  return LJX_OK;
}

// The collective result's inputs from this rank's step totals (k_finalize's result): slots 0..7
// are summed over ranks (energy, virial, kept edges), 8..10 max-reduced (kept edges, widest
// row, capacity overflow), 11 stays local (this rank's energy).
__global__ void k_result_collect(const double *result, double *out, int duplicate, int matrix,
                                 double capacity)
{
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const double edges = result[7] * duplicate;
  for (int k = 0; k < 7; ++k) out[k] = result[k];
  out[7] = edges;
  out[8] = edges;
  out[9] = result[8];
  out[10] = (matrix ? result[8] : edges) > capacity ? 1.0 : 0.0;
  out[11] = result[0];
}

template <typename S>
void launch_flat_rows(const char *what, long long items, cudaStream_t s, void (*kernel)(S *, int, const int *, int, int),
                      S *rows, int width, const int *owner, int first, int n)
{
  if (items <= 0) return;
  kernel<<<flat_grid(items), ljx::kBlock, 0, s>>>(rows, width, owner, first, n);
  check_launch(what);
}

}  // namespace

extern "C" {

const char *ljx_version(void) { return LJX_VERSION; }

ljx_status ljx_bundle_load(const char *path, ljx_bundle **out)
{
  if (path == nullptr || out == nullptr) return LJX_ERR_INVALID;
  try {
    auto *b = new ljx_bundle{ljx::load_bundle(path)};
    *out = b;
    return LJX_OK;
  } catch (const std::exception &err) {
    g_bundle_error = err.what();
    *out = nullptr;
    return LJX_ERR_BUNDLE;
  }
}

ljx_status ljx_bundle_load_string(const char *json, size_t length, ljx_bundle **out)
{
  if (json == nullptr || out == nullptr) return LJX_ERR_INVALID;
  try {
    auto *b = new ljx_bundle{ljx::parse_bundle(std::string(json, length))};
    *out = b;
    return LJX_OK;
  } catch (const std::exception &err) {
    g_bundle_error = err.what();
    *out = nullptr;
    return LJX_ERR_BUNDLE;
  }
}

const char *ljx_bundle_error(void) { return g_bundle_error.c_str(); }

ljx_status ljx_bundle_contract(const ljx_bundle *bundle, ljx_contract *out)
{
  if (bundle == nullptr || out == nullptr) return LJX_ERR_INVALID;
  *out = bundle->b.contract;
  return LJX_OK;
}

ljx_status ljx_bundle_eam_tables(const ljx_bundle *bundle, int *n_elements, int *nrho, int *nr,
                                 double *drho, double *dr, double *cutoff, double *embedding,
                                 double *density, double *pair)
{
  if (bundle == nullptr) return LJX_ERR_INVALID;
  const ljx::EamTables &t = bundle->b.eam;
  if (bundle->b.contract.potential != LJX_POTENTIAL_EAM) return LJX_ERR_INVALID;
  if (n_elements) *n_elements = t.n_elements;
  if (nrho) *nrho = t.nrho;
  if (nr) *nr = t.nr;
  if (drho) *drho = t.drho;
  if (dr) *dr = t.dr;
  if (cutoff) *cutoff = t.cutoff;
  if (embedding) std::memcpy(embedding, t.embedding.data(), t.embedding.size() * sizeof(double));
  if (density) std::memcpy(density, t.density.data(), t.density.size() * sizeof(double));
  if (pair) std::memcpy(pair, t.pair.data(), t.pair.size() * sizeof(double));
  return LJX_OK;
}

void ljx_bundle_free(ljx_bundle *bundle) { delete bundle; }

ljx_status ljx_engine_create(const ljx_bundle *bundle, int device, ljx_engine **out)
{
  if (bundle == nullptr || out == nullptr) return LJX_ERR_INVALID;
  *out = nullptr;
  std::unique_ptr<ljx_engine> e(new ljx_engine());
  e->bundle = bundle->b;
  e->c = bundle->b.contract;
  e->device = device;
  const ljx_contract &c = e->c;
  if (c.potential == LJX_POTENTIAL_NONE) {
    g_bundle_error =
        "LAMMPS-JAX bundle carries no potential block; the ljx engine runs eam/alloy, eam and "
        "lj/cut bundles written with their potential parameters";
    return LJX_ERR_UNSUPPORTED;
  }
  if (c.n_hops != 1) {
    g_bundle_error = "ljx runs single-hop (n_hops = 1) bundles; EAM and LJ need one cutoff";
    return LJX_ERR_UNSUPPORTED;
  }
  try {
    DeviceGuard guard(device);
    if (const char *v = std::getenv("LJX_OWNED_HALF")) e->owned_half = std::atoi(v) != 0;
    check(cudaDeviceGetAttribute(&e->sm_count, cudaDevAttrMultiProcessorCount, device),
          "cudaDeviceGetAttribute");
    e->f64 = c.precision == LJX_FLOAT64;
    const size_t real = e->f64 ? sizeof(double) : sizeof(float);
    const long long max_atoms = c.max_atoms;
    const bool matrix = c.input_layout == LJX_LAYOUT_NEIGHBOR_MATRIX;
    e->rows_cap = c.max_owned > 0 ? c.max_owned : c.max_atoms;
    e->row_cap = matrix ? c.max_neighbors
                        : static_cast<int>(std::max<long long>(1, c.max_edges / e->rows_cap));
    // Room for a force pass launched in up to 16 pieces (ljx_force_to_host).
    e->max_grid = e->sm_count * 64;
    e->xd4 = static_cast<double4 *>(device_alloc(max_atoms * sizeof(double4), "cudaMalloc(xd4)"));
    check(cudaMemset(e->xd4, 0, max_atoms * sizeof(double4)), "cudaMemset(xd4)");
    // Float copy of the positions: the distance pre-filter (and the float model) reads it.
    e->pos4 = device_alloc(max_atoms * sizeof(float4), "cudaMalloc(pos4)");
    check(cudaMemset(e->pos4, 0, max_atoms * sizeof(float4)), "cudaMemset(pos4)");
    e->coord_bound = static_cast<unsigned int *>(device_alloc(2 * sizeof(unsigned int), "cudaMalloc(bound)"));
    check(cudaMemset(e->coord_bound, 0, 2 * sizeof(unsigned int)), "cudaMemset(bound)");
    if (c.potential == LJX_POTENTIAL_EAM) {
      // Candidate cache: a group's union holds about 3.5 rows' worth of kept pairs at solid
      // densities and a row's candidates within rc (1 + margin) about 1.6; 4 x and 2 x row_cap
      // leave headroom. Groups that do not fit walk their lists.
      e->groups_cap = (e->rows_cap + ljx::kGroupRows - 1) / ljx::kGroupRows;
      e->gcap = std::max(64, std::min(ljx::kUnionMax, 4 * e->row_cap));
      e->rcap = std::max(32, std::min(ljx::kUnionMax, 2 * e->row_cap));
      e->xref = static_cast<double4 *>(device_alloc(max_atoms * sizeof(double4), "cudaMalloc(xref)"));
      check(cudaMemset(e->xref, 0, max_atoms * sizeof(double4)), "cudaMemset(xref)");
      e->gatom = static_cast<int *>(device_alloc(
          static_cast<size_t>(e->groups_cap) * e->gcap * sizeof(int), "cudaMalloc(group unions)"));
      e->gcount = static_cast<int *>(device_alloc(e->groups_cap * sizeof(int), "cudaMalloc(group counts)"));
      check(cudaMemset(e->gcount, 0, e->groups_cap * sizeof(int)), "cudaMemset(group counts)");
      e->rslot = static_cast<unsigned short *>(device_alloc(
          static_cast<size_t>(e->groups_cap) * ljx::kGroupRows * e->rcap * sizeof(unsigned short),
          "cudaMalloc(row candidates)"));
      e->rcount = static_cast<int *>(device_alloc(
          static_cast<size_t>(e->groups_cap) * ljx::kGroupRows * sizeof(int), "cudaMalloc(row counts)"));
    }
    e->rho = device_alloc(max_atoms * real, "cudaMalloc(rho)");
    e->fp = device_alloc(max_atoms * real, "cudaMalloc(fp)");
    check(cudaMemset(e->rho, 0, max_atoms * real), "cudaMemset(rho)");
    check(cudaMemset(e->fp, 0, max_atoms * real), "cudaMemset(fp)");
    e->cedges = static_cast<int *>(device_alloc(
        static_cast<size_t>(e->rows_cap) * e->row_cap * sizeof(int), "cudaMalloc(compacted rows)"));
    e->ccount = static_cast<int *>(device_alloc(e->rows_cap * sizeof(int), "cudaMalloc(counts)"));
    check(cudaMemset(e->ccount, 0, e->rows_cap * sizeof(int)), "cudaMemset(counts)");
    e->ghost_rows = static_cast<unsigned char *>(device_alloc(e->rows_cap, "cudaMalloc(ghost rows)"));
    check(cudaMemset(e->ghost_rows, 1, e->rows_cap), "cudaMemset(ghost rows)");
    e->offsets = static_cast<long long *>(
        device_alloc((static_cast<size_t>(e->rows_cap) + 1) * sizeof(long long), "cudaMalloc(offsets)"));
    check(cudaMemset(e->offsets, 0, (static_cast<size_t>(e->rows_cap) + 1) * sizeof(long long)),
          "cudaMemset(offsets)");
    e->count_prev = static_cast<long long *>(device_alloc(sizeof(long long), "cudaMalloc(count)"));
    check(cudaMemset(e->count_prev, 0, sizeof(long long)), "cudaMemset(count)");
    if (!matrix) {
      // Padding contract of the sparse edge ABI (cpp/pair_jax_kokkos.cpp:379-383).
      const size_t me = static_cast<size_t>(c.max_edges);
      e->senders = static_cast<int *>(device_alloc(me * sizeof(int), "cudaMalloc(senders)"));
      e->receivers = static_cast<int *>(device_alloc(me * sizeof(int), "cudaMalloc(receivers)"));
      e->edge_mask = static_cast<uint8_t *>(device_alloc(me, "cudaMalloc(edge_mask)"));
      std::vector<int> pad(std::min<size_t>(me, 1 << 20), c.max_atoms);
      for (size_t off = 0; off < me; off += pad.size()) {
        const size_t n = std::min(pad.size(), me - off);
        check(cudaMemcpy(e->senders + off, pad.data(), n * sizeof(int), cudaMemcpyHostToDevice),
              "cudaMemcpy(senders)");
        check(cudaMemcpy(e->receivers + off, pad.data(), n * sizeof(int), cudaMemcpyHostToDevice),
              "cudaMemcpy(receivers)");
      }
      check(cudaMemset(e->edge_mask, 0, me), "cudaMemset(edge_mask)");
    }
    e->partials = static_cast<double *>(device_alloc(
        4ULL * e->max_grid * ljx::kPartialWidth * sizeof(double), "cudaMalloc(partials)"));
    check(cudaMemset(e->partials, 0, 4ULL * e->max_grid * ljx::kPartialWidth * sizeof(double)),
          "cudaMemset(partials)");
    e->result = static_cast<double *>(device_alloc(16 * sizeof(double), "cudaMalloc(result)"));
    check(cudaMallocHost(reinterpret_cast<void **>(&e->host_result), 16 * sizeof(double)),
          "cudaMallocHost(result)");
    e->order_bad = reinterpret_cast<int *>(e->result + 12);
    e->host_order_bad = reinterpret_cast<int *>(e->host_result + 12);
    *e->host_order_bad = 0;
    if (c.potential == LJX_POTENTIAL_EAM) {
      const ljx::EamTables &t = e->bundle.eam;
      // Slope rows (c1, 2 c2, 3 c3, 0) / dr: d rho/dr = s0 + t (s1 + t s2).
      std::vector<double> slope(t.density.size());
      const double inv_dr = 1.0 / t.dr;
      for (size_t k = 0; k < slope.size(); k += 4) {
        slope[k + 0] = t.density[k + 1] * inv_dr;
        slope[k + 1] = 2.0 * t.density[k + 2] * inv_dr;
        slope[k + 2] = 3.0 * t.density[k + 3] * inv_dr;
        slope[k + 3] = 0.0;
      }
      if (e->f64) {
        e->embedding = upload_table<double>(t.embedding);
        e->density = upload_table<double>(t.density);
        e->density_slope = upload_table<double>(slope);
        e->pair = upload_table<double>(t.pair);
      } else {
        e->embedding = upload_table<float>(t.embedding);
        e->density = upload_table<float>(t.density);
        e->density_slope = upload_table<float>(slope);
        e->pair = upload_table<float>(t.pair);
      }
    }
    check(cudaDeviceSynchronize(), "cudaDeviceSynchronize(create)");
  } catch (const std::exception &err) {
    g_bundle_error = err.what();
    return LJX_ERR_CUDA;
  }
  *out = e.release();
  return LJX_OK;
}

void ljx_engine_destroy(ljx_engine *engine) { delete engine; }

const char *ljx_engine_error(const ljx_engine *engine)
{
  return engine ? engine->error.c_str() : "null engine";
}

ljx_status ljx_engine_plan(ljx_engine *e, int newton_pair, ljx_plan *plan)
{
  if (e == nullptr || plan == nullptr) return LJX_ERR_INVALID;
  // init_style newton checks, cpp/pair_jax_kokkos.cpp:668-673.
  if (e->c.newton == LJX_NEWTON_ON && !newton_pair)
    return fail(e, LJX_ERR_INVALID,
                "LAMMPS-JAX bundle was exported for newton pair on; this run uses newton off");
  if (e->c.newton == LJX_NEWTON_OFF && newton_pair)
    return fail(e, LJX_ERR_INVALID,
                "LAMMPS-JAX bundle was exported for newton pair off; this run uses newton on");
  const Modes m = decide_modes(e->c, newton_pair);
  plan->half_list = m.half_list;
  plan->reverse_density = m.reverse_density;
  plan->forward_fp = m.forward_fp;
  plan->reverse_force = m.reverse_force;
  plan->comm_width = 1;
  plan->comm_elem_bytes = e->f64 ? 8 : 4;
  return LJX_OK;
}

ljx_status ljx_pack_atoms(ljx_engine *e, void *stream, const ljx_atoms *atoms)
{
  return guarded(e, [&]() -> ljx_status {
    if (atoms == nullptr || (atoms->nlocal + atoms->nghost > 0 && (!atoms->x || !atoms->type)))
      return fail(e, LJX_ERR_INVALID, "atom arrays are incomplete");
    const ljx_status cap = check_capacity(e, atoms);
    if (cap != LJX_OK) return cap;
    for (int &b : e->step_blocks) b = 0;
    e->last_nlocal = atoms->nlocal;
    e->last_nall = atoms->nlocal + atoms->nghost;
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? pack_atoms_impl<double>(e, s, atoms) : pack_atoms_impl<float>(e, s, atoms);
  });
}

ljx_status ljx_pack_edges(ljx_engine *e, void *stream, const ljx_atoms *atoms,
                          const ljx_list *list, int newton_pair)
{
  return guarded(e, [&]() -> ljx_status {
    if (e->c.input_layout != LJX_LAYOUT_SPARSE_EDGE)
      return fail(e, LJX_ERR_INVALID, "neighbor-matrix bundles have no sparse edge arrays");
    const ljx_status st = check_list(e, list);
    if (st != LJX_OK) return st;
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? pack_edges_impl<double>(e, s, atoms, list, newton_pair)
                  : pack_edges_impl<float>(e, s, atoms, list, newton_pair);
  });
}

ljx_status ljx_edges(ljx_engine *e, const int **senders, const int **receivers,
                     const uint8_t **edge_mask, int *capacity)
{
  if (e == nullptr) return LJX_ERR_INVALID;
  if (e->senders == nullptr) return fail(e, LJX_ERR_INVALID, "no sparse edge arrays");
  if (senders) *senders = e->senders;
  if (receivers) *receivers = e->receivers;
  if (edge_mask) *edge_mask = e->edge_mask;
  if (capacity) *capacity = e->c.max_edges;
  return LJX_OK;
}

ljx_status ljx_density(ljx_engine *e, void *stream, const ljx_atoms *atoms,
                       const ljx_list *list, int newton_pair)
{
  return guarded(e, [&]() -> ljx_status {
    const ljx_status st = check_list(e, list);
    if (st != LJX_OK) return st;
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? density_impl<double>(e, s, atoms, list, newton_pair)
                  : density_impl<float>(e, s, atoms, list, newton_pair);
  });
}

ljx_status ljx_embed(ljx_engine *e, void *stream, const ljx_atoms *atoms)
{
  return guarded(e, [&]() -> ljx_status {
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? embed_impl<double>(e, s, atoms) : embed_impl<float>(e, s, atoms);
  });
}

ljx_status ljx_energy(ljx_engine *e, void *stream, const ljx_atoms *atoms, const ljx_list *list,
                      int newton_pair, double scale)
{
  return guarded(e, [&]() -> ljx_status {
    const ljx_status st = check_list(e, list);
    if (st != LJX_OK) return st;
    if (atoms == nullptr) return fail(e, LJX_ERR_INVALID, "atom arrays are missing");
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? energy_impl<double>(e, s, atoms, list, newton_pair, scale)
                  : energy_impl<float>(e, s, atoms, list, newton_pair, scale);
  });
}

ljx_status ljx_force(ljx_engine *e, void *stream, const ljx_atoms *atoms, const ljx_list *list,
                     int newton_pair, double scale)
{
  return guarded(e, [&]() -> ljx_status {
    const ljx_status st = check_list(e, list);
    if (st != LJX_OK) return st;
    if (atoms == nullptr || atoms->f == nullptr)
      return fail(e, LJX_ERR_INVALID, "force array is missing");
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? force_impl<double>(e, s, atoms, list, newton_pair, scale)
                  : force_impl<float>(e, s, atoms, list, newton_pair, scale);
  });
}

ljx_status ljx_force_rows(ljx_engine *e, void *stream, const ljx_atoms *atoms,
                          const ljx_list *list, int newton_pair, double scale, int part)
{
  return guarded(e, [&]() -> ljx_status {
    const ljx_status st = check_list(e, list);
    if (st != LJX_OK) return st;
    if (atoms == nullptr || atoms->f == nullptr)
      return fail(e, LJX_ERR_INVALID, "force array is missing");
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? force_rows_impl<double>(e, s, atoms, list, newton_pair, scale, part)
                  : force_rows_impl<float>(e, s, atoms, list, newton_pair, scale, part);
  });
}

ljx_status ljx_force_only(ljx_engine *e, void *stream, const ljx_atoms *atoms,
                          const ljx_list *list, int newton_pair, double scale)
{
  return guarded(e, [&]() -> ljx_status {
    const ljx_status st = check_list(e, list);
    if (st != LJX_OK) return st;
    if (atoms == nullptr || atoms->f == nullptr)
      return fail(e, LJX_ERR_INVALID, "force array is missing");
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? force_only_impl<double>(e, s, atoms, list, newton_pair, scale)
                  : force_only_impl<float>(e, s, atoms, list, newton_pair, scale);
  });
}

ljx_status ljx_force_to_host(ljx_engine *e, void *stream, const ljx_atoms *atoms,
                             const ljx_list *list, int newton_pair, double scale, double *f_host,
                             int pieces)
{
  return guarded(e, [&]() -> ljx_status {
    const ljx_status st = check_list(e, list);
    if (st != LJX_OK) return st;
    if (atoms == nullptr || atoms->f == nullptr)
      return fail(e, LJX_ERR_INVALID, "force array is missing");
    if (f_host == nullptr || pieces < 1 || pieces > 16)
      return fail(e, LJX_ERR_INVALID, "f_host is missing or pieces is outside 1..16");
    auto s = static_cast<cudaStream_t>(stream);
    return e->f64 ? force_to_host_impl<double>(e, s, atoms, list, newton_pair, scale, f_host, pieces)
                  : force_to_host_impl<float>(e, s, atoms, list, newton_pair, scale, f_host,
                                              pieces);
  });
}

// After the stream has drained: a streamed force step whose rows were not in atom order.
static ljx_status check_streamed_rows(ljx_engine *e)
{
  if (!e->rows_streamed) return LJX_OK;
  e->rows_streamed = false;
  if (*e->host_order_bad != 0)
    return fail(e, LJX_ERR_INVALID,
                "ljx_force_to_host: " + std::to_string(*e->host_order_bad) +
                    " list rows are not their own atom (ilist[r] != r); the host force rows are "
                    "not usable");
  return LJX_OK;
}

ljx_status ljx_read_result(ljx_engine *e, void *stream, ljx_result *out)
{
  return guarded(e, [&]() -> ljx_status {
    auto s = static_cast<cudaStream_t>(stream);
    ljx::PartialSet set{};
    for (int k = 0; k < 4; ++k) {
      set.ptr[k] = e->partial(k);
      set.blocks[k] = e->step_blocks[k];
    }
    ljx::k_finalize<<<1, ljx::kBlock, 0, s>>>(set, e->last_scale, e->result);
    check_launch("k_finalize");
    e->launches++;
    check(cudaMemcpyAsync(e->host_result, e->result, 9 * sizeof(double), cudaMemcpyDeviceToHost, s),
          "cudaMemcpyAsync(result)");
    check(cudaStreamSynchronize(s), "cudaStreamSynchronize(result)");
    const double *r = e->host_result;
    ljx_result res{};
    if (e->step_ev) {
      res.energy = r[0];
      for (int k = 0; k < 6; ++k) res.virial[k] = r[1 + k];
    }
    e->step_ev = true;
    res.edge_count = static_cast<long long>(r[7]) * e->last_duplicate;
    res.widest_row = static_cast<int>(r[8]);
    if (e->c.input_layout == LJX_LAYOUT_NEIGHBOR_MATRIX)
      res.overflow = res.widest_row > e->c.max_neighbors;
    else
      res.overflow = res.edge_count > e->c.max_edges;
    if (out) *out = res;
    for (int &b : e->step_blocks) b = 0;
    return check_streamed_rows(e);
  });
}

ljx_status ljx_read_result_all(ljx_engine *e, ljx_halo *halo, void *stream, ljx_result_all *out)
{
  return guarded(e, [&]() -> ljx_status {
    if (halo == nullptr) return fail(e, LJX_ERR_INVALID, "halo is missing");
    auto s = static_cast<cudaStream_t>(stream);
    ljx::PartialSet set{};
    for (int k = 0; k < 4; ++k) {
      set.ptr[k] = e->partial(k);
      set.blocks[k] = e->step_blocks[k];
    }
    ljx::k_finalize<<<1, ljx::kBlock, 0, s>>>(set, e->last_scale, e->result);
    check_launch("k_finalize");
    const bool matrix = e->c.input_layout == LJX_LAYOUT_NEIGHBOR_MATRIX;
    const double capacity = matrix ? e->c.max_neighbors : e->c.max_edges;
    k_result_collect<<<1, 32, 0, s>>>(e->result, ljx::halo_scalars(halo), e->last_duplicate,
                                      matrix ? 1 : 0, capacity);
    check_launch("k_result_collect");
    e->launches += 2;
    double r[12];
    std::string why;
    const ljx_status st = ljx::halo_reduce_fetch(halo, s, 8, 3, 12, r, why);
    if (st != LJX_OK) return fail(e, st, why);
    ljx_result_all res{};
    if (e->step_ev) {
      res.energy = r[0];
      for (int k = 0; k < 6; ++k) res.virial[k] = r[1 + k];
    }
    res.edge_count = static_cast<long long>(r[7]);
    res.edge_max = static_cast<long long>(r[8]);
    res.widest_row = static_cast<int>(r[9]);
    res.overflow = r[10] > 0.0 ? 1 : 0;
    res.local_energy = e->step_ev ? r[11] : 0.0;
    e->step_ev = true;
    if (out) *out = res;
    for (int &b : e->step_blocks) b = 0;
    return check_streamed_rows(e);
  });
}

ljx_status ljx_feature_rows(ljx_engine *e, int which, void **rows, int *width, int *elem_bytes)
{
  if (e == nullptr || rows == nullptr) return LJX_ERR_INVALID;
  if (which != 0 && which != 1) return fail(e, LJX_ERR_INVALID, "feature must be 0 (rho) or 1 (F')");
  *rows = which == 0 ? e->rho : e->fp;
  if (width) *width = 1;
  if (elem_bytes) *elem_bytes = e->f64 ? 8 : 4;
  return LJX_OK;
}

ljx_status ljx_set_atom_tallies(ljx_engine *e, double *eatom, double *vatom, double scale)
{
  if (e == nullptr) return LJX_ERR_INVALID;
  e->eatom = eatom;
  e->vatom = vatom;
  e->tally_scale = scale;
  return LJX_OK;
}

long long ljx_engine_launches(const ljx_engine *e) { return e ? e->launches : 0; }

// ---- comm rows ----

static ljx_status comm_status(cudaError_t err)
{
  return err == cudaSuccess ? LJX_OK : LJX_ERR_CUDA;
}

ljx_status ljx_comm_pack_forward(void *stream, const void *rows, int words, const int *sendlist,
                                 int n, double *buf, int slots)
{
  if (n <= 0) return LJX_OK;
  if (!rows || !sendlist || !buf || words <= 0 || slots * 2 < words) return LJX_ERR_INVALID;
  ljx::k_pack_words_by_list<<<flat_grid(static_cast<long long>(n) * words), ljx::kBlock, 0,
                              static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t *>(rows), words, sendlist, n, buf, slots);
  return comm_status(cudaGetLastError());
}

ljx_status ljx_comm_unpack_forward(void *stream, void *rows, int words, int first, int n,
                                   const double *buf, int slots)
{
  if (n <= 0) return LJX_OK;
  if (!rows || !buf || words <= 0 || slots * 2 < words) return LJX_ERR_INVALID;
  ljx::k_unpack_words_at<<<flat_grid(static_cast<long long>(n) * words), ljx::kBlock, 0,
                           static_cast<cudaStream_t>(stream)>>>(static_cast<uint32_t *>(rows),
                                                                words, first, n, buf, slots);
  return comm_status(cudaGetLastError());
}

ljx_status ljx_comm_pack_reverse(void *stream, const void *rows, int words, int first, int n,
                                 double *buf, int slots)
{
  if (n <= 0) return LJX_OK;
  if (!rows || !buf || words <= 0 || slots * 2 < words) return LJX_ERR_INVALID;
  ljx::k_pack_words_at<<<flat_grid(static_cast<long long>(n) * words), ljx::kBlock, 0,
                         static_cast<cudaStream_t>(stream)>>>(static_cast<const uint32_t *>(rows),
                                                              words, first, n, buf, slots);
  return comm_status(cudaGetLastError());
}

ljx_status ljx_comm_unpack_reverse(void *stream, void *rows, int width, int elem_bytes,
                                   const int *sendlist, int n, const double *buf, int slots)
{
  if (n <= 0) return LJX_OK;
  if (!rows || !sendlist || !buf || width <= 0) return LJX_ERR_INVALID;
  auto s = static_cast<cudaStream_t>(stream);
  const int grid = flat_grid(static_cast<long long>(n) * width);
  if (elem_bytes == 8)
    ljx::k_add_rows_by_list<double><<<grid, ljx::kBlock, 0, s>>>(static_cast<double *>(rows),
                                                                 width, sendlist, n, buf, slots);
  else if (elem_bytes == 4)
    ljx::k_add_rows_by_list<float><<<grid, ljx::kBlock, 0, s>>>(static_cast<float *>(rows), width,
                                                                sendlist, n, buf, slots);
  else
    return LJX_ERR_INVALID;
  return comm_status(cudaGetLastError());
}

ljx_status ljx_comm_zero_rows(void *stream, void *rows, int width, int elem_bytes, int first,
                              int n)
{
  if (n <= 0) return LJX_OK;
  if (!rows || width <= 0) return LJX_ERR_INVALID;
  auto s = static_cast<cudaStream_t>(stream);
  const int grid = flat_grid(static_cast<long long>(n) * width);
  if (elem_bytes == 8)
    ljx::k_zero_rows<double><<<grid, ljx::kBlock, 0, s>>>(static_cast<double *>(rows), width, first, n);
  else if (elem_bytes == 4)
    ljx::k_zero_rows<float><<<grid, ljx::kBlock, 0, s>>>(static_cast<float *>(rows), width, first, n);
  else
    return LJX_ERR_INVALID;
  return comm_status(cudaGetLastError());
}

ljx_status ljx_halo_forward_self(void *stream, void *rows, int width, int elem_bytes,
                                 const int *owner, int first, int n)
{
  if (n <= 0) return LJX_OK;
  if (!rows || !owner || width <= 0) return LJX_ERR_INVALID;
  auto s = static_cast<cudaStream_t>(stream);
  const long long items = static_cast<long long>(n) * width;
  try {
    if (elem_bytes == 8)
      launch_flat_rows<double>("k_forward_self", items, s, ljx::k_forward_self<double>,
                               static_cast<double *>(rows), width, owner, first, n);
    else if (elem_bytes == 4)
      launch_flat_rows<float>("k_forward_self", items, s, ljx::k_forward_self<float>,
                              static_cast<float *>(rows), width, owner, first, n);
    else
      return LJX_ERR_INVALID;
  } catch (const std::exception &) {
    return LJX_ERR_CUDA;
  }
  return LJX_OK;
}

ljx_status ljx_halo_reverse_self(void *stream, void *rows, int width, int elem_bytes,
                                 const int *owner, int first, int n)
{
  if (n <= 0) return LJX_OK;
  if (!rows || !owner || width <= 0) return LJX_ERR_INVALID;
  auto s = static_cast<cudaStream_t>(stream);
  const long long items = static_cast<long long>(n) * width;
  try {
    if (elem_bytes == 8)
      launch_flat_rows<double>("k_reverse_self", items, s, ljx::k_reverse_self<double>,
                               static_cast<double *>(rows), width, owner, first, n);
    else if (elem_bytes == 4)
      launch_flat_rows<float>("k_reverse_self", items, s, ljx::k_reverse_self<float>,
                              static_cast<float *>(rows), width, owner, first, n);
    else
      return LJX_ERR_INVALID;
  } catch (const std::exception &) {
    return LJX_ERR_CUDA;
  }
  return LJX_OK;
}

}  // extern "C"
