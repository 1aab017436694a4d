/*
 * ljx — B200 (sm_100a) force engine behind `pair_style jax/kk` for EAM and LJ bundles.
 *
 * The C ABI the LAMMPS pair style binds in place of the PJRT runtime. Plain pointers and sizes
 * only; every device pointer is CUDA device memory on the engine's device and every call is
 * ordered on the caller's stream (the Kokkos execution space's stream in LAMMPS). No call
 * allocates or synchronizes on the hot path except ljx_read_result (one small D2H + stream sync,
 * the analogue of the reference's energy readback, cpp/pjrt/runtime.cpp:242-256).
 *
 * Errors: every entry point returns an ljx_status; exceptions never cross the ABI (as the
 * reference's FFI handlers, cpp/pjrt/model_comm.cpp:78-90). ljx_engine_error / ljx_bundle_error
 * give the message, using the reference's wording where the reference has one.
 */
#ifndef LJX_H
#define LJX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int ljx_status;
enum {
  LJX_OK = 0,
  LJX_ERR_INVALID = 1,     /* bad argument or call order */
  LJX_ERR_CUDA = 2,        /* a CUDA call failed; the message names it */
  LJX_ERR_CAPACITY = 3,    /* a contract capacity was exceeded (collective abort upstream) */
  LJX_ERR_BUNDLE = 4,      /* bundle could not be parsed or failed contract validation */
  LJX_ERR_UNSUPPORTED = 5  /* bundle asks for something this engine does not implement */
};

/* Mirrors lammps_jax::InputLayout / ForceLayout / NewtonMode / Precision
 * (cpp/lammps_jax_model.h:11-34). */
enum { LJX_LAYOUT_SPARSE_EDGE = 0, LJX_LAYOUT_NEIGHBOR_MATRIX = 1 };
enum { LJX_FORCE_ATOM = 0, LJX_FORCE_EDGE = 1 };
enum { LJX_NEWTON_ANY = 0, LJX_NEWTON_ON = 1, LJX_NEWTON_OFF = 2 };
enum { LJX_FLOAT32 = 0, LJX_FLOAT64 = 1 };
enum { LJX_PAIRING_FULL = 0, LJX_PAIRING_HALF = 1, LJX_PAIRING_HALF_UNIQUE = 2 };
enum { LJX_POTENTIAL_NONE = 0, LJX_POTENTIAL_EAM = 1, LJX_POTENTIAL_LJ = 2 };

#define LJX_MAX_COMM_WIDTHS 16

/* The bundle contract: lammps_jax::ModelContract (cpp/lammps_jax_model.h:43-76) plus bundle
 * header fields (:78-87) and the potential block this engine reads. */
typedef struct ljx_contract {
  int input_layout;
  int max_atoms;
  int max_edges;
  int max_neighbors;
  double cutoff;
  char unit_style[16];
  int precision;
  int force_layout;
  int newton;
  int n_hops;
  int half_edges;
  int edge_pairing;
  int n_comm_widths;
  int comm_widths[LJX_MAX_COMM_WIDTHS];
  int n_comm_sites;
  int comm_sites[3];
  int uses_box;
  int pair_sum;
  int n_species;
  int max_owned;
  char format[48];
  char platform[16];
  /* Programs the bundle carries (non-empty): force, energy, energy_and_forces. */
  int has_force_program;
  int has_energy_program;
  int has_energy_and_forces_program;
  /* Potential block. */
  int potential;
  int n_elements;
  double lj_epsilon;
  double lj_sigma;
  double lj_edge_energy_scale;
} ljx_contract;

typedef struct ljx_bundle ljx_bundle;
typedef struct ljx_engine ljx_engine;

/* ---------------------------------------------------------------------------------------------
 * Bundle: replaces lammps_jax::load_bundle_file (cpp/lammps_jax_model.cpp:212-315). Same key
 * lookup, same validation and messages, plus the `potential` block (setfl text or LJ
 * parameters) the engine computes from instead of the serialized XLA programs.
 * ------------------------------------------------------------------------------------------- */
ljx_status ljx_bundle_load(const char *path, ljx_bundle **out);
ljx_status ljx_bundle_load_string(const char *json, size_t length, ljx_bundle **out);
/* Message of the last failed load on this thread. */
const char *ljx_bundle_error(void);
ljx_status ljx_bundle_contract(const ljx_bundle *bundle, ljx_contract *out);
/* EAM tables after the setfl parse and spline build (python/lammps_jax/eam.py:115-227):
 * sizes, then [n_elements][nrho][4], [n_elements][nr][4], [n_pairs][nr][4] doubles. Pass NULL
 * arrays to query sizes. */
ljx_status ljx_bundle_eam_tables(const ljx_bundle *bundle, int *n_elements, int *nrho, int *nr,
                                 double *drho, double *dr, double *cutoff, double *embedding,
                                 double *density, double *pair);
void ljx_bundle_free(ljx_bundle *bundle);

/* ---------------------------------------------------------------------------------------------
 * Engine: replaces pjrt::Runtime (cpp/pjrt/runtime.h:66-124) and the pair style's device
 * buffers (cpp/pair_jax_kokkos.cpp:355-387). Sized once from the contract, never resized.
 * ------------------------------------------------------------------------------------------- */
ljx_status ljx_engine_create(const ljx_bundle *bundle, int device, ljx_engine **out);
void ljx_engine_destroy(ljx_engine *engine);
const char *ljx_engine_error(const ljx_engine *engine);

/* LAMMPS per-atom arrays on the device: x double[nall][3] (read), type int[nall] 1-based
 * (read), f double[nall][3] (accumulated with +=, as AddForcesFunctor does). */
typedef struct ljx_atoms {
  const double *x;
  const int *type;
  double *f;
  int nlocal;
  int nghost;
} ljx_atoms;

/* A NeighListKokkos view: row ii lists atom ilist[ii]; its jj-th neighbor is
 * neighbors[i * atom_stride + jj * slot_stride] & NEIGHMASK for jj < numneigh[i] (Kokkos
 * LayoutLeft on CUDA: atom_stride 1, slot_stride = list allocation rows).
 *
 * ago is LAMMPS's neighbor->ago: steps since this list was built, 0 on the step it was built
 * (the reference's neighbor-matrix path repacks on the same signal, cpp/pair_jax_kokkos.cpp:
 * 1011-1012). For EAM, ljx_density caches per group of 8 rows the union of their neighbors
 * within rc plus a margin when ago == 0, and reuses it while ago > 0. It rebuilds by itself when
 * the list pointers or sizes change or when some atom has moved more than half the margin. The
 * kept pairs are the reference's in every case. A negative ago turns the cache off: every step
 * then filters the whole list, as the reference's sparse-edge path does. */
typedef struct ljx_list {
  const int *ilist;
  const int *numneigh;
  const int *neighbors;
  long long atom_stride;
  long long slot_stride;
  int inum;
  int gnum;
  int maxneighs;
  int ago;
} ljx_list;

/* Per-step results; energy and virial already multiplied by the pair_coeff scale. */
typedef struct ljx_result {
  double energy;
  double virial[6];
  long long edge_count;    /* kept edges this step (the reference's edge counter) */
  int overflow;            /* capacity exceeded (edges, or neighbors for matrix bundles) */
  int widest_row;          /* widest LAMMPS list row seen this step */
} ljx_result;

/* Which list the pair style must request and which exchanges the step needs, decided from the
 * contract and the run's newton setting as PairJaxKokkos::half_list / init_style do
 * (cpp/pair_jax_kokkos.cpp:425-431, 665-785). */
typedef struct ljx_plan {
  int half_list;           /* request a half list (1) or a full list (0) */
  int reverse_density;     /* ghost density partials must be reverse-communicated */
  int forward_fp;          /* F'(rho) of owners must be forward-communicated to ghosts */
  int reverse_force;       /* ghost force rows feed LAMMPS's own reverse comm (newton on) */
  int comm_width;          /* exchanged row width in features */
  int comm_elem_bytes;     /* 4 or 8: feature precision */
} ljx_plan;

/* Checks the run against the contract (init_style, cpp/pair_jax_kokkos.cpp:665-693) and fills
 * the plan. newton_pair is LAMMPS's force->newton_pair. */
ljx_status ljx_engine_plan(ljx_engine *engine, int newton_pair, ljx_plan *plan);

/* a1 — positions/species staging: PackAtomsFunctor (cpp/pair_jax_kokkos.cpp:35-52, 794-809).
 * Also runs the pre-launch row-capacity check of :1035-1046 (rank-local values). */
ljx_status ljx_pack_atoms(ljx_engine *engine, void *stream, const ljx_atoms *atoms);

/* a2 — the reference sparse-edge ABI: PackNeighborFunctor + ResetEdgeTailFunctor
 * (cpp/pair_jax_kokkos.cpp:54-118, 157-173, 811-874). Writes senders/receivers/edge_mask of
 * max_edges slots, kept pairs first in (row, slot) order, padding max_atoms/false after. */
ljx_status ljx_pack_edges(ljx_engine *engine, void *stream, const ljx_atoms *atoms,
                          const ljx_list *list, int newton_pair);
ljx_status ljx_edges(ljx_engine *engine, const int **senders, const int **receivers,
                     const uint8_t **edge_mask, int *capacity);

/* a2+a6 — fused pass over the LAMMPS list: distance-filter and compact each row (warp ballot
 * compaction, rows kept in engine scratch) and accumulate the EAM density rho_i += f_j(r)
 * (python/lammps_jax/eam.py:284-314). For half lists the neighbor share is scattered too.
 * For LJ bundles it only compacts.
 * EAM full lists with newton off hold each owned pair once: row i keeps the owned neighbors
 * j > i and every ghost, and the neighbor's density share (here) and force (ljx_force) are added
 * by atomics; the kept pairs, the edge count and all results are the reference's, with sums in
 * an order that can differ between runs in the last bits. The environment variable
 * LJX_OWNED_HALF=0, read by ljx_engine_create, evaluates every pair from both rows instead
 * (bitwise reproducible, slower). Per-atom tallies and lists without a row for every owned atom
 * use both rows too. */
ljx_status ljx_density(ljx_engine *engine, void *stream, const ljx_atoms *atoms,
                       const ljx_list *list, int newton_pair);

/* a8 — embedding F(rho), F'(rho) of owned rows (eam.py:319-321, 383-384) and their energy. */
ljx_status ljx_embed(ljx_engine *engine, void *stream, const ljx_atoms *atoms);

/* a9..a14 — fused force + energy + virial over the compacted rows: per-edge
 * psip = F'(rho_i) f_j'(r) + F'(rho_j) f_i'(r) + phi'(r) (eam.py:383-398), forces added into
 * atoms->f (scaled), pair energy, per-edge virial; LJ 12-6 as the one-pass case
 * (examples/export_model.py:16-74). Newton-on modes also add ghost-row forces for LAMMPS's
 * reverse comm. */
ljx_status ljx_force(ljx_engine *engine, void *stream, const ljx_atoms *atoms,
                     const ljx_list *list, int newton_pair, double scale);

/* ljx_force in two parts, so that a rank's F'(rho) exchange overlaps its force pass (the
 * reference's forward comm of F' runs between its density and force programs, with nothing else
 * in flight: cpp/pair_jax_kokkos.cpp:523-571, cpp/pjrt/model_comm.cpp:392-472).
 * ljx_density marks each list row that keeps a ghost neighbor (over the candidate cache: each
 * row with a ghost candidate, marked when the cache is built). LJX_ROWS_LOCAL runs the force
 * pass over the unmarked rows, which read no ghost F' and may run while the exchange fills the
 * ghost rows of F'; LJX_ROWS_GHOST, after the exchange, runs the marked rows. The two calls, in that
 * order after the same ljx_density, leave atoms->f and the step's energy and virial as one
 * ljx_force call does (sums in another order). EAM bundles only (LJ: LJX_ERR_UNSUPPORTED);
 * a ghost part without its local part fails with LJX_ERR_INVALID. */
#define LJX_ROWS_LOCAL 1
#define LJX_ROWS_GHOST 2
ljx_status ljx_force_rows(ljx_engine *engine, void *stream, const ljx_atoms *atoms,
                          const ljx_list *list, int newton_pair, double scale, int part);

/* Forces alone: the reference's execute_force path, which LAMMPS takes on every step that asks
 * for neither energy nor virial (cpp/pair_jax_kokkos.cpp:1002-1003, 1055-1057, 1092; eflag and vflag
 * are set only on thermo steps). The forces of ljx_force (to the last bit: without the sums the
 * compiler may fuse a multiply-add the full pass keeps apart) from an EAM force pass that sums no
 * pair energy and no virial (fewer registers per thread); LJ runs its one pass as in ljx_force. The next ljx_read_result / ljx_read_result_all reports energy and virial as zero and
 * the edge count and overflow as usual. Per-atom tallies, when registered, run the full pass. */
ljx_status ljx_force_only(ljx_engine *engine, void *stream, const ljx_atoms *atoms,
                          const ljx_list *list, int newton_pair, double scale);

/* ljx_force with the owned force rows streamed to host memory while the pass runs: the pass is
 * launched as `pieces` (1..16) consecutive ranges of list rows, and each range's rows of
 * atoms->f are copied to f_host (double[nlocal][3], pinned host memory for the copies to overlap)
 * on an engine-owned copy stream as soon as that range has finished, so the device-to-host copy
 * of a LAMMPS step's forces (atomKK->sync of f to the host) runs under the rest of the pass.
 * `stream` is ordered after the last copy when this returns, so a synchronize of it (ljx_read_result
 * does one) leaves f_host complete: atoms->f as ljx_force leaves it, rows 0..nlocal-1.
 * Only where a list row holds its atom's whole force: EAM full list with newton off, LJ
 * edge-force bundles on a full list (otherwise LJX_ERR_UNSUPPORTED, nothing launched). Row r of
 * the list must be atom r (ilist[r] == r, as LAMMPS's Kokkos lists are built); a device check
 * runs with the pass and the next ljx_read_result / ljx_read_result_all fails with
 * LJX_ERR_INVALID if a row was out of order (f_host is then not usable; atoms->f is). */
ljx_status ljx_force_to_host(ljx_engine *engine, void *stream, const ljx_atoms *atoms,
                             const ljx_list *list, int newton_pair, double scale, double *f_host,
                             int pieces);

/* Energy-only evaluation: the reference's execute_energy path for LAMMPS eflag_only steps (MC
 * moves; cpp/pair_jax_kokkos.cpp:997-1001, 1051-1053, runtime execute_energy). After ljx_density
 * and ljx_embed (and the reverse rho exchange of half-list plans) it sums the pair energy (EAM)
 * or the LJ energy; ljx_read_result then reports the total energy. No F' is needed and no force
 * or virial is written. */
ljx_status ljx_energy(ljx_engine *engine, void *stream, const ljx_atoms *atoms,
                      const ljx_list *list, int newton_pair, double scale);

/* Per-atom energy and virial: LAMMPS's eatom / vatom under eflag_atom / vflag_atom, which the
 * reference refuses (cpp/pair_jax_kokkos.cpp:995-996). eatom is double[nall], vatom
 * double[nall][6] (xx, yy, zz, xy, xz, yz), device memory on the engine's device; either may be
 * NULL. The ljx_embed, ljx_force and ljx_energy calls that follow ADD into them (LAMMPS's
 * ev_setup zeroes them first), times `scale` (the pair_coeff scale), until the next call here
 * (NULL, NULL turns the tallies off). The split is LAMMPS's ev_tally: the embedding energy
 * F(rho_i) goes to atom i; half of each pair's energy and half of its virial -rij (x) F go to each
 * of the two atoms (a full-list row takes its own half, the pair's other row the other).
 * Newton-on modes also write ghost rows, which LAMMPS's compute pe/atom and stress/atom fold into
 * their owners by reverse comm. Without these arrays the force pass runs without the tally work.
 */
ljx_status ljx_set_atom_tallies(ljx_engine *engine, double *eatom, double *vatom, double scale);

/* Reduces the step's energy/virial/counters and copies them to the host (one stream sync). */
ljx_status ljx_read_result(ljx_engine *engine, void *stream, ljx_result *out);

/* Engine-owned per-atom feature rows of the model comm sites: 0 = density rho, 1 = F'(rho);
 * max_atoms rows of `width` elements of `elem_bytes` bytes (the contract precision). */
ljx_status ljx_feature_rows(ljx_engine *engine, int which, void **rows, int *width,
                            int *elem_bytes);

/* a15 — comm rows as 4-byte words, one row per `slots` doubles of the LAMMPS buffer
 * (cpp/pair_jax_kokkos.cpp:247-318, 523-571; comm_slots :75-78). */
ljx_status ljx_comm_pack_forward(void *stream, const void *rows, int words, const int *sendlist,
                                 int n, double *buf, int slots);
ljx_status ljx_comm_unpack_forward(void *stream, void *rows, int words, int first, int n,
                                   const double *buf, int slots);
ljx_status ljx_comm_pack_reverse(void *stream, const void *rows, int words, int first, int n,
                                 double *buf, int slots);
/* Reverse unpack adds (the adjoint of forward): rows[sendlist[i]] += buf row i. */
ljx_status ljx_comm_unpack_reverse(void *stream, void *rows, int width, int elem_bytes,
                                   const int *sendlist, int n, const double *buf, int slots);
/* Zero ghost rows after a reverse exchange (cpp/pjrt/model_comm.cpp:463-465). */
ljx_status ljx_comm_zero_rows(void *stream, void *rows, int width, int elem_bytes, int first,
                              int n);
/* Same-rank exchange for periodic images: row first+g mirrors row owner[g]. forward copies the
 * owner row into the image; reverse adds the image row into its owner (atomically) and zeroes
 * it. elem_bytes 4 (float) or 8 (double). */
ljx_status ljx_halo_forward_self(void *stream, void *rows, int width, int elem_bytes,
                                 const int *owner, int first, int n);
ljx_status ljx_halo_reverse_self(void *stream, void *rows, int width, int elem_bytes,
                                 const int *owner, int first, int n);

/* ---------------------------------------------------------------------------------------------
 * Allocation-free LJ force pass. No counterpart in the reference: the reference always runs
 * through a PJRT client that owns its buffers. This is for callers that cannot call cudaMalloc
 * — a process where another framework already reserved the device memory (JAX/XLA preallocates
 * most of the GPU by default) or host code bound to a memory pool it does not own. It runs the
 * same kernels as ljx_force on an lj/cut bundle without an engine: the caller passes inputs and
 * outputs (atoms->f is accumulated with +=; `result` is device memory for 9 doubles: energy,
 * virial[6] (both times `scale`), kept pairs, widest list row) and the scratch is a fixed
 * LJX_NOALLOC_BYTES device array inside the library, held by every GPU that loads it until the
 * process exits. nlocal + nghost (and inum) must not exceed LJX_NOALLOC_MAX_ATOMS; larger
 * systems get LJX_ERR_CAPACITY before anything is launched. List entries (rows or neighbors) at
 * or past nlocal + nghost are skipped. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress, once per device): make that first call before any stream
 * capture, and do not call this entry point again on a device the process has reset
 * (cudaDeviceReset), since the address belongs to the old context. Calls share the one array,
 * so calls that overlap on the GPU (other streams, other host threads) race; serialize them.
 * Nothing here calls cudaMalloc or cudaFree.
 * force_layout/newton_pair select the distribution exactly as for an lj/cut bundle.
 * ------------------------------------------------------------------------------------------- */
#define LJX_NOALLOC_MAX_ATOMS 32768
#define LJX_NOALLOC_BYTES (2u << 20)
ljx_status ljx_lj_force_noalloc(void *stream, const ljx_atoms *atoms, const ljx_list *list,
                                double epsilon, double sigma, double cutoff, int precision,
                                int force_layout, int newton_pair, double scale, double *result);

/* Number of this library's kernel launches issued since the engine was created. */
long long ljx_engine_launches(const ljx_engine *engine);

/* Library version string. */
const char *ljx_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LJX_H */
