/*
 * ljx halo — per-atom row exchange between ranks over NCCL send/recv (one rank per GPU, NVLink /
 * NVSwitch), and the collective step result.
 *
 * Replaces the reference's model-comm bridge (cpp/pjrt/model_comm.cpp:392-472: the XLA FFI
 * handler that stages feature rows, hands them to the LAMMPS thread and waits for
 * PairJaxKokkos's forward/reverse comm over MPI, cpp/pair_jax_kokkos.cpp:444-571) and the
 * per-step MPI_Allreduce of the edge counts (cpp/pair_jax_kokkos.cpp:1059-1075). Everything is
 * ordered on the caller's stream: pack kernels, one grouped ncclSend/ncclRecv per stage, unpack
 * kernels. Nothing waits on the host except ljx_read_result_all.
 *
 * Exchange pattern (LAMMPS CommBrick's swaps): swap s sends the rows sendlist[0..sendnum) to
 * rank send_rank, and receives recvnum rows from rank recv_rank into rows firstrecv.. (forward).
 * The reverse exchange runs the swaps backwards: the rows firstrecv..+recvnum go back to
 * recv_rank and what arrives from send_rank is ADDED into the sendlist rows (then the received
 * ghost rows may be zeroed, as the reference's model comm zeroes forwarded ghost cotangents,
 * cpp/pjrt/model_comm.cpp:463-465). Swaps carry a stage number: swaps of one stage are
 * independent (no sendlist row of a stage is received in the same stage) and run as one NCCL
 * group; stages run in increasing order forward and in decreasing order in reverse. Messages
 * between two ranks within one stage match in posting order. A swap whose send_rank and
 * recv_rank are this rank is a periodic self image: a device copy (an add in reverse), unless
 * the halo was created with LJX_HALO_SELF_BY_NCCL.
 *
 * Failures: every call returns an ljx_status; ljx_halo_error gives the message. A peer that
 * never posts its side leaves the NCCL kernels waiting; ljx_read_result_all waits at most the
 * halo's timeout for the step, then aborts the communicator (ncclCommAbort, which ends the
 * waiting kernels) and returns LJX_ERR_CUDA. An aborted halo refuses further exchanges.
 *
 * NCCL is bound at run time (dlopen): the copy already loaded in the process (for instance by
 * the framework that set up the ranks) if there is one, else libnccl.so.2 from the library path
 * (LJX_NCCL_LIBRARY names another file).
 */
#ifndef LJX_HALO_H
#define LJX_HALO_H

#include "ljx.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LJX_HALO_ID_BYTES 128
/* Route periodic self swaps through NCCL send/recv to this rank instead of a device copy. */
#define LJX_HALO_SELF_BY_NCCL 1

typedef struct ljx_halo ljx_halo;

typedef struct ljx_swap {
  int stage;
  int send_rank;
  int recv_rank;
  const int *sendlist; /* device array of sendnum row indices */
  int sendnum;
  int firstrecv;
  int recvnum;
} ljx_swap;

/* A fresh NCCL unique id (ncclGetUniqueId), made on one rank and broadcast to the others by the
 * caller (MPI_Bcast in LAMMPS, the process group's broadcast in the harness). */
ljx_status ljx_halo_unique_id(unsigned char id[LJX_HALO_ID_BYTES]);
/* Collective over nranks: every rank calls it with the same id. timeout_ms bounds
 * ljx_read_result_all's wait (<= 0: 60000). */
ljx_status ljx_halo_create(const unsigned char id[LJX_HALO_ID_BYTES], int nranks, int rank,
                           int device, int timeout_ms, int flags, ljx_halo **out);
void ljx_halo_destroy(ljx_halo *halo);
const char *ljx_halo_error(const ljx_halo *halo);
/* Message of the last failed ljx_halo_unique_id / ljx_halo_create on this thread. */
const char *ljx_halo_create_error(void);

/* Set (or replace, after a reneighboring) the swap table. Device staging buffers are sized here
 * for rows of up to max_row_bytes bytes (a multiple of 4); exchanges of wider rows are refused.
 * The sendlist arrays stay owned by the caller and must live until the next set_swaps. */
ljx_status ljx_halo_set_swaps(ljx_halo *halo, const ljx_swap *swaps, int nswaps,
                              int max_row_bytes);

/* Forward exchange of rows (width elements of elem_bytes bytes, elem_bytes 4 or 8): owners to
 * ghosts. */
ljx_status ljx_halo_forward(ljx_halo *halo, void *stream, void *rows, int width, int elem_bytes);
/* Reverse exchange: ghost rows added into their owners' rows; zero_ghosts clears every received
 * row afterwards. */
ljx_status ljx_halo_reverse(ljx_halo *halo, void *stream, void *rows, int width, int elem_bytes,
                            int zero_ghosts);

/* Step result over all ranks of the halo. energy and virial are summed over ranks (times the
 * pair_coeff scale); edge_count is summed; edge_max is the largest rank's count (the "global
 * max" of the reference's capacity message); overflow is set when some rank exceeded its edge
 * (or, for neighbor-matrix bundles, neighbor) capacity; widest_row is the global widest list
 * row. One grouped NCCL all-reduce on the stream, one device-to-host copy, one bounded wait. */
typedef struct ljx_result_all {
  double energy;
  double virial[6];
  long long edge_count;
  long long edge_max;
  int overflow;
  int widest_row;
  double local_energy; /* this rank's share of energy */
} ljx_result_all;

ljx_status ljx_read_result_all(ljx_engine *engine, ljx_halo *halo, void *stream,
                               ljx_result_all *out);

/* In-place sum over ranks of n doubles on the stream: the harness's global sums. */
ljx_status ljx_halo_allreduce_sum(ljx_halo *halo, void *stream, double *values, int n);

/* Launches of this library's own halo kernels (row gathers and scatter-adds) so far; the NCCL
 * kernels of the send/recv groups and all-reduces are not counted. */
long long ljx_halo_launches(const ljx_halo *halo);

#ifdef __cplusplus
}
#endif

#endif /* LJX_HALO_H */
