// The MD step around the pair style for the standalone harness (include/ljx_md.h): velocity
// Verlet as LAMMPS's FixNVE, the forward comm of positions to periodic images, and the
// displacement test that decides a neighbor rebuild. Each is one streaming pass over per-atom
// rows (HBM-bound, a few tens of bytes per atom), launched on the caller's stream.

#include <cuda_runtime.h>

#include <algorithm>

#include "ljx_md.h"

namespace {

constexpr int kBlock = 256;

struct TypeTable {
  double dtfm[LJX_MD_MAX_TYPES];
};

unsigned grid_for(long long n)
{
  // Grid-stride loops: enough blocks to fill 148 SMs several times over, no more.
  return static_cast<unsigned>(std::max(1LL, std::min((n + kBlock - 1) / kBlock, 148LL * 16)));
}

__global__ void k_nve_initial(double *__restrict__ x, double *__restrict__ v,
                              const double *__restrict__ f, const int *__restrict__ type,
                              int nlocal, double dtv, TypeTable table, int ntypes)
{
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nlocal; i += gridDim.x * blockDim.x) {
    const int t = min(max(type[i], 1), ntypes) - 1;
    const double dtfm = table.dtfm[t];
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const long long k = 3LL * i + d;
      const double vk = v[k] + dtfm * f[k];
      v[k] = vk;
      x[k] += dtv * vk;
    }
  }
}

__global__ void k_nve_final(double *__restrict__ v, const double *__restrict__ f,
                            const int *__restrict__ type, int nlocal, TypeTable table, int ntypes)
{
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nlocal; i += gridDim.x * blockDim.x) {
    const double dtfm = table.dtfm[min(max(type[i], 1), ntypes) - 1];
#pragma unroll
    for (int d = 0; d < 3; ++d) v[3LL * i + d] += dtfm * f[3LL * i + d];
  }
}

__global__ void k_ghost_positions(double *__restrict__ x, int nlocal, int nghost,
                                  const int *__restrict__ owner, const double *__restrict__ shift)
{
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < nghost; g += gridDim.x * blockDim.x) {
    const long long o = 3LL * owner[g];
    const long long k = 3LL * (nlocal + g);
#pragma unroll
    for (int d = 0; d < 3; ++d) x[k + d] = x[o + d] + shift[3LL * g + d];
  }
}

__global__ void k_max_displacement(const double *__restrict__ x, const double *__restrict__ xref,
                                   int n, unsigned long long *__restrict__ out)
{
  double best = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double dx = x[3LL * i] - xref[3LL * i];
    const double dy = x[3LL * i + 1] - xref[3LL * i + 1];
    const double dz = x[3LL * i + 2] - xref[3LL * i + 2];
    best = fmax(best, dx * dx + dy * dy + dz * dz);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = fmax(best, __shfl_xor_sync(0xffffffffu, best, o));
  __shared__ double s_best[kBlock / 32];
  if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < blockDim.x / 32; ++w) best = fmax(best, s_best[w]);
    // Non-negative doubles order as their bit patterns do.
    atomicMax(out, static_cast<unsigned long long>(__double_as_longlong(best)));
  }
}

bool load_table(const double *dtfm, int ntypes, TypeTable *table)
{
  if (!dtfm || ntypes <= 0 || ntypes > LJX_MD_MAX_TYPES) return false;
  for (int t = 0; t < LJX_MD_MAX_TYPES; ++t) table->dtfm[t] = t < ntypes ? dtfm[t] : 0.0;
  return true;
}

ljx_status launched() { return cudaGetLastError() == cudaSuccess ? LJX_OK : LJX_ERR_CUDA; }

}  // namespace

extern "C" ljx_status ljx_nve_initial(void *stream, double *x, double *v, const double *f,
                                      const int *type, int nlocal, double dtv,
                                      const double *dtfm, int ntypes)
{
  TypeTable table;
  if (nlocal < 0 || !load_table(dtfm, ntypes, &table)) return LJX_ERR_INVALID;
  if (nlocal == 0) return LJX_OK;
  if (!x || !v || !f || !type) return LJX_ERR_INVALID;
  k_nve_initial<<<grid_for(nlocal), kBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      x, v, f, type, nlocal, dtv, table, ntypes);
  return launched();
}

extern "C" ljx_status ljx_nve_final(void *stream, double *v, const double *f, const int *type,
                                    int nlocal, const double *dtfm, int ntypes)
{
  TypeTable table;
  if (nlocal < 0 || !load_table(dtfm, ntypes, &table)) return LJX_ERR_INVALID;
  if (nlocal == 0) return LJX_OK;
  if (!v || !f || !type) return LJX_ERR_INVALID;
  k_nve_final<<<grid_for(nlocal), kBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      v, f, type, nlocal, table, ntypes);
  return launched();
}

extern "C" ljx_status ljx_ghost_positions(void *stream, double *x, int nlocal, int nghost,
                                          const int *owner, const double *shift)
{
  if (nlocal < 0 || nghost < 0) return LJX_ERR_INVALID;
  if (nghost == 0) return LJX_OK;
  if (!x || !owner || !shift) return LJX_ERR_INVALID;
  k_ghost_positions<<<grid_for(nghost), kBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      x, nlocal, nghost, owner, shift);
  return launched();
}

extern "C" ljx_status ljx_max_displacement(void *stream, const double *x, const double *xref,
                                           int n, double *out)
{
  if (!out || n < 0 || (n > 0 && (!x || !xref))) return LJX_ERR_INVALID;
  auto s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(out, 0, sizeof(double), s) != cudaSuccess) return LJX_ERR_CUDA;
  if (n == 0) return LJX_OK;
  k_max_displacement<<<grid_for(n), kBlock, 0, s>>>(
      x, xref, n, reinterpret_cast<unsigned long long *>(out));
  return launched();
}
