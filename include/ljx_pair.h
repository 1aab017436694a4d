/*
 * ljx_pair — the host side of pair_style jax/kk on the ljx engine, as a C ABI.
 *
 * It restates PairJaxKokkos (cpp/pair_jax_kokkos.cpp, cpp/pair_jax_kokkos.h) without LAMMPS
 * types: settings / coeff / init_style / init_one / compute keep the reference's argument
 * meaning, checks, order of checks and error messages. A LAMMPS plugin forwards its methods
 * here; the standalone harness (lammps-jax_b200/engine.py PairJax) and the tests drive the same
 * entry points. A failing call returns a non-OK status; ljx_pair_error gives the message the
 * reference passes to error->all / error->one.
 *
 * What LAMMPS provides to the pair style during compute (its comm and MPI) comes in through
 * ljx_pair_host callbacks.
 */
#ifndef LJX_PAIR_H
#define LJX_PAIR_H

#include "ljx.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ljx_pair ljx_pair;

/* LAMMPS services the pair style calls during compute. Each returns 0 on success.
 * forward_comm / reverse_comm: comm->forward_comm(this) / comm->reverse_comm(this) over the
 *   engine's feature rows (`rows`, `width` features of `elem_bytes` each; the pair style's pack
 *   and unpack hooks call ljx_comm_*). reverse_comm adds ghost rows into their owners.
 * allreduce_max: MPI_Allreduce(MPI_IN_PLACE, values, n, MPI_INT, MPI_MAX, world).
 * A null callback means one rank with no exchange (allreduce_max: the values are global). */
typedef struct ljx_pair_host {
  void *ctx;
  int (*forward_comm)(void *ctx, void *rows, int width, int elem_bytes, void *stream);
  int (*reverse_comm)(void *ctx, void *rows, int width, int elem_bytes, void *stream);
  int (*allreduce_max)(void *ctx, int *values, int n);
} ljx_pair_host;

/* Compute flags (LAMMPS's ev_init arguments). */
#define LJX_EFLAG_GLOBAL 1
#define LJX_VFLAG_GLOBAL 2
#define LJX_EFLAG_ATOM 4
#define LJX_VFLAG_ATOM 8
#define LJX_EFLAG_ONLY 16

/* The pair style (PairJaxKokkos constructor); `device` is the CUDA device (exec.cuda_device()). */
ljx_status ljx_pair_create(int device, ljx_pair **out);
void ljx_pair_destroy(ljx_pair *pair);
const char *ljx_pair_error(const ljx_pair *pair);

/* pair_style jax/kk [plugin-path] (:573-580): at most one argument, accepted and ignored. */
ljx_status ljx_pair_settings(ljx_pair *pair, int narg, const char *const *arg);

/* pair_coeff I J bundle.json [scale] (:582-663): type bounds against ntypes, the scale, the
 * bundle load, unit style / species / platform checks, then the engine. */
ljx_status ljx_pair_coeff(ljx_pair *pair, int narg, const char *const *arg,
                          const char *unit_style, int ntypes);

/* init_style (:665-785): newton mode of the bundle, special_bonds factors (molecular systems:
 * special_lj / special_coul hold LAMMPS's force->special_* [0..3], may be null for atomic ones),
 * barostat fixes without newton. *plan receives the list request and the exchanges. */
ljx_status ljx_pair_init_style(ljx_pair *pair, int newton_pair, int molecular,
                               const double *special_lj, const double *special_coul, int nfix,
                               const char *const *fix_styles, ljx_plan *plan);

/* init_one (:787-792): the bundle cutoff. */
double ljx_pair_init_one(const ljx_pair *pair);

/* compute(eflag, vflag) (:989-1102): collective row limits, pack, density, [reverse rho], embed,
 * then [forward F'] + forces (or the energy alone for LJX_EFLAG_ONLY), the collective capacity
 * check, and the energy / f.r virial tallies. Forces are added into atoms->f. The step result is
 * copied to *out when it is not null. */
ljx_status ljx_pair_compute(ljx_pair *pair, void *stream, const ljx_atoms *atoms,
                            const ljx_list *list, int newton_pair, int flags,
                            const ljx_pair_host *host, ljx_result *out);

/* LAMMPS's per-atom arrays for eflag_atom / vflag_atom computes: Pair::eatom double[nmax] and
 * Pair::vatom double[nmax][6] (the Kokkos pair's d_eatom / d_vatom), device memory; either may
 * be NULL. With an array registered, compute accepts the matching flag instead of the
 * reference's refusal (cpp/pair_jax_kokkos.cpp:995-996): it zeroes nlocal (+ nghost with newton
 * on) rows as ev_setup does and fills them as LAMMPS's ev_tally splits pair terms (see
 * ljx_set_atom_tallies). The plugin re-registers them when LAMMPS grows the arrays. */
ljx_status ljx_pair_set_atom_tallies(ljx_pair *pair, double *eatom, double *vatom);

/* Pair::eng_vdwl and Pair::virial[6] after the last compute (reset by its flags, as ev_init). */
ljx_status ljx_pair_tally(const ljx_pair *pair, double *eng_vdwl, double *virial);

/* The bundle and engine behind a coeff'ed pair style (owned by it; null before coeff). */
const ljx_bundle *ljx_pair_bundle(const ljx_pair *pair);
ljx_engine *ljx_pair_engine(ljx_pair *pair);

#ifdef __cplusplus
}
#endif

#endif /* LJX_PAIR_H */
