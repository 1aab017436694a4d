/*
 * ljx_md — the MD step around the pair style, for the standalone harness. In a LAMMPS run this is
 * LAMMPS's own code, outside the reference and unchanged by a drop-in: FixNVE's velocity Verlet
 * (fix_nve.cpp initial_integrate / final_integrate), Comm::forward_comm of positions to the
 * periodic ghost images, and the displacement test of Neighbor::decide ("neigh_modify check yes",
 * Neighbor::check_distance). The harness uses them to run the benchmark configurations' NVE
 * trajectories on the device around ljx_pair_compute.
 *
 * Positions, velocities and forces are LAMMPS's per-atom double [n][3] arrays; type is 1-based.
 * Every pointer is device memory except the per-type dtf/m table, which is a HOST array of
 * ntypes <= LJX_MD_MAX_TYPES doubles passed by value to the kernel.
 */
#ifndef LJX_MD_H
#define LJX_MD_H

#include "ljx.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LJX_MD_MAX_TYPES 16

/* FixNVE::initial_integrate over the nlocal owned atoms: v += dtfm[type-1] * f, then
 * x += dtv * v. dtv = dt; dtfm[t] = 0.5 * dt * ftm2v / mass[t]. */
ljx_status ljx_nve_initial(void *stream, double *x, double *v, const double *f, const int *type,
                           int nlocal, double dtv, const double *dtfm, int ntypes);

/* FixNVE::final_integrate: v += dtfm[type-1] * f over the nlocal owned atoms. */
ljx_status ljx_nve_final(void *stream, double *v, const double *f, const int *type, int nlocal,
                         const double *dtfm, int ntypes);

/* Forward comm of positions to the periodic images one rank holds of its own atoms:
 * x[nlocal + g][d] = x[owner[g]][d] + shift[g][d] (shift: whole box lengths, 0 or +-L per
 * dimension, so each coordinate takes one rounding, as LAMMPS's pbc shift in pack_comm). */
ljx_status ljx_ghost_positions(void *stream, double *x, int nlocal, int nghost, const int *owner,
                               const double *shift);

/* Neighbor::check_distance: *out (one device double) = max over i < n of |x_i - xref_i|^2. */
ljx_status ljx_max_displacement(void *stream, const double *x, const double *xref, int n,
                                double *out);

#ifdef __cplusplus
}
#endif

#endif /* LJX_MD_H */
