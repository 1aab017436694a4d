// Internal interface between the engine (engine.cu) and the NCCL halo (halo_nccl.cu): the
// collective step result reduces the engine's step totals through the halo's communicator.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "ljx_halo.h"

namespace ljx {

// Device scratch of the halo for the collective result (kHaloScalars doubles).
constexpr int kHaloScalars = 16;
double *halo_scalars(ljx_halo *halo);

// Sum all-reduce of scalars[0, nsum) and max all-reduce of scalars[nsum, nsum + nmax) as one NCCL
// group on `stream`, then copy scalars[0, ncopy) to `host` and wait for the stream, at most the
// halo's timeout (after which the communicator is aborted). Returns LJX_OK or an error status
// with the message in `error`.
ljx_status halo_reduce_fetch(ljx_halo *halo, cudaStream_t stream, int nsum, int nmax, int ncopy,
                             double *host, std::string &error);

}  // namespace ljx
