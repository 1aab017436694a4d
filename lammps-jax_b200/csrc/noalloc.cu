// ljx_lj_force_noalloc: the LJ force pass with its scratch in a fixed device array.
//
// Some callers cannot call cudaMalloc: a process where another framework has already reserved
// the device memory (JAX/XLA preallocates most of the GPU by default, which is why the
// reference's PJRT client turns preallocation off), or a host code that must stay inside a
// memory pool it does not own. This entry point runs the same kernels as ljx_force on an lj/cut
// bundle (position staging, the one-pass LJ kernel, the step reduction) but takes no engine and
// allocates nothing: its scratch lives in a file-scope __device__ array of LJX_NOALLOC_BYTES
// bytes that every GPU which loads the library holds until the process exits.

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "kernels.cuh"
#include "ljx.h"

namespace {

constexpr int kMaxAtoms = LJX_NOALLOC_MAX_ATOMS;
constexpr int kMaxBlocks = 2048;
constexpr size_t kXd4Bytes = static_cast<size_t>(kMaxAtoms) * sizeof(double4);
constexpr size_t kPos4Bytes = static_cast<size_t>(kMaxAtoms) * sizeof(float4);
constexpr size_t kPartialBytes = static_cast<size_t>(kMaxBlocks) * ljx::kPartialWidth * sizeof(double);
constexpr size_t kBoundOffset = kXd4Bytes + kPos4Bytes + kPartialBytes;
static_assert(kBoundOffset + 256 <= LJX_NOALLOC_BYTES, "scratch layout exceeds the array");

// Staged positions (double4 + float4), per-block partial sums, the coordinate bound.
static __device__ __align__(256) unsigned char g_scratch[LJX_NOALLOC_BYTES];

std::mutex g_mutex;
void *g_address[64] = {};

// Device address of g_scratch on the current device, looked up once per device. In host code
// the name g_scratch is only a host-side stand-in, so kernels are always handed this address.
// The cached address belongs to the device's primary context: after cudaDeviceReset the next
// context may place the array elsewhere, so a process that resets a device must not call this
// entry point on that device again.
ljx_status scratch_address(int device, unsigned char **out)
{
  if (device < 0 || device >= 64) return LJX_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_address[device] == nullptr) {
    void *ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_scratch);
    if (err != cudaSuccess)
      return LJX_ERR_CUDA;
    g_address[device] = ptr;
  }
  *out = static_cast<unsigned char *>(g_address[device]);
  return LJX_OK;
}

template <typename T>
ljx_status run(cudaStream_t s, unsigned char *scratch, const ljx_atoms *a, const ljx_list *l,
               double epsilon, double sigma, double cutoff, double edge_energy_scale, int mode,
               double scale, double *result, int sm_count)
{
  ljx::Step<T> p{};
  p.x = a->x;
  p.type = a->type;
  p.f = a->f;
  p.nlocal = a->nlocal;
  p.nghost = a->nghost;
  p.nall = a->nlocal + a->nghost;
  p.ilist = l->ilist;
  p.numneigh = l->numneigh;
  p.neighbors = l->neighbors;
  p.atom_stride = l->atom_stride;
  p.slot_stride = l->slot_stride;
  p.inum = l->inum;
  p.maxneighs = std::max(1, l->maxneighs);
  p.xd4 = reinterpret_cast<double4 *>(scratch);
  p.pos4 = reinterpret_cast<typename ljx::Vec4<T>::type *>(scratch + kXd4Bytes);
  p.partials = reinterpret_cast<double *>(scratch + kXd4Bytes + kPos4Bytes);
  p.coord_bound = reinterpret_cast<unsigned int *>(scratch + kBoundOffset);
  p.n_species = 1;
  p.pack_cutsq = cutoff * cutoff;
  p.model_cutsq = static_cast<T>(cutoff * cutoff);
  // Rows past nall hold whatever an earlier call (possibly of another system) left in the shared
  // array, so list indices >= nall are dropped exactly as indices past an engine's capacity are.
  p.max_atoms = p.nall;
  p.scale = scale;
  p.lj_four_eps = static_cast<T>(4.0 * epsilon);
  p.lj_sigma_sq = static_cast<T>(sigma * sigma);
  p.lj_energy_scale = static_cast<T>(edge_energy_scale);
  // The coordinate bound accumulates with atomic max, so it must start at zero on every call;
  // everything else in the array is fully written before it is read.
  if (cudaMemsetAsync(p.coord_bound, 0, sizeof(unsigned int), s) != cudaSuccess)
    return LJX_ERR_CUDA;
  const int span = p.nall;
  if (span > 0) {
    const int grid = std::max(1, std::min((span + ljx::kBlock - 1) / ljx::kBlock, sm_count * 16));
    ljx::k_pack_atoms<T><<<grid, ljx::kBlock, 0, s>>>(p, span);
  }
  ljx::PartialSet set{};
  if (p.inum > 0) {
    const int need = (p.inum + ljx::kWarpsPerBlock - 1) / ljx::kWarpsPerBlock;
    const int grid = std::max(1, std::min(need, std::min(kMaxBlocks, sm_count * 4)));
    switch (mode) {
      case ljx::kLjEdgeHalf: ljx::k_lj<T, ljx::kLjEdgeHalf><<<grid, ljx::kBlock, 0, s>>>(p); break;
      case ljx::kLjAtomFull: ljx::k_lj<T, ljx::kLjAtomFull><<<grid, ljx::kBlock, 0, s>>>(p); break;
      default: ljx::k_lj<T, ljx::kLjEdgeFull><<<grid, ljx::kBlock, 0, s>>>(p); break;
    }
    set.ptr[3] = p.partials;
    set.blocks[3] = grid;
  }
  ljx::k_finalize<<<1, ljx::kBlock, 0, s>>>(set, scale, result);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return LJX_ERR_CUDA;
  return LJX_OK;
}

}  // namespace

extern "C" ljx_status ljx_lj_force_noalloc(void *stream, const ljx_atoms *atoms,
                                           const ljx_list *list, double epsilon, double sigma,
                                           double cutoff, int precision, int force_layout,
                                           int newton_pair, double scale, double *result)
{
  if (atoms == nullptr || list == nullptr || result == nullptr || atoms->f == nullptr)
    return LJX_ERR_INVALID;
  const long long nall = static_cast<long long>(atoms->nlocal) + atoms->nghost;
  // Past the fixed array: refuse before touching the device (use an engine for such systems).
  if (nall > kMaxAtoms || list->inum > kMaxAtoms) return LJX_ERR_CAPACITY;
  if (list->gnum > 0) return LJX_ERR_UNSUPPORTED;
  if (force_layout == LJX_FORCE_ATOM && !newton_pair)
    return LJX_ERR_INVALID;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return LJX_ERR_CUDA;
  unsigned char *scratch = nullptr;
  const ljx_status st = scratch_address(device, &scratch);
  if (st != LJX_OK) return st;
  int sm_count = 0;
  if (cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      sm_count <= 0)
    return LJX_ERR_CUDA;
  // Force distribution of an lj/cut bundle as ljx_force decides it (full list unless newton-on
  // edge forces, which take the half list), with the exporter's per-edge energy weight.
  int mode = ljx::kLjEdgeFull;
  double energy_scale = 0.5;
  if (force_layout == LJX_FORCE_EDGE && newton_pair) {
    mode = ljx::kLjEdgeHalf;
    energy_scale = 1.0;
  } else if (force_layout == LJX_FORCE_ATOM) {
    mode = ljx::kLjAtomFull;
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (precision == LJX_FLOAT64)
    return run<double>(s, scratch, atoms, list, epsilon, sigma, cutoff, energy_scale, mode, scale,
                       result, sm_count);
  if (precision == LJX_FLOAT32)
    return run<float>(s, scratch, atoms, list, epsilon, sigma, cutoff, energy_scale, mode, scale,
                      result, sm_count);
  return LJX_ERR_INVALID;
}

