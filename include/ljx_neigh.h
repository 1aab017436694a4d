/*
 * ljx_neigh — device neighbor-list build for the standalone harness (the step before the pack;
 * in LAMMPS this is NPairKokkos, outside the reference). Produces the same NeighListKokkos view
 * the pair style receives: owned rows over owned + ghost atoms, Kokkos LayoutLeft
 * (neighbors[i + jj * slot_stride]), pairs with r^2 < cutoff^2 (cutoff = model cutoff + skin).
 *
 * Binning: atoms are pre-sorted into a uniform grid of cubic bins (side `binsize` >= cutoff/2,
 * origin `lo`, `nbins` per dimension); bin b holds bin_atoms[bin_start[b] .. bin_start[b+1]).
 * `lo` (3 doubles) and `nbins` (3 ints) are HOST arrays; every other pointer is device memory.
 * Each owned atom scans the bins of a +-2 stencil whose box lies within the cutoff. half != 0 keeps each pair once: owned j > i, or a
 * ghost j whose (z, y, x) sorts after atom i's — the one-rank-per-pair rule of the reference
 * packer (cpp/pair_jax_kokkos.cpp:94-101).
 *
 * Rows wider than maxneigh are truncated; *widest (device int) receives the widest row so the
 * caller can rebuild with a larger maxneigh.
 */
#ifndef LJX_NEIGH_H
#define LJX_NEIGH_H

#include "ljx.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Device binning for ljx_neigh_build (no counterpart in the reference: LAMMPS bins inside
 * NPairKokkos): counting sort of the nall atoms of x into the grid given by lo, binsize and nbins
 * (HOST arrays), atoms in index order within each bin. bin_start receives nbins_total + 1 ints,
 * bin_atoms nall ints; scratch must hold nbins_total + ceil(nbins_total / 1024) ints. sorted
 * (16-byte aligned) receives nall + 1 records of 16 bytes: the atoms in bin order as float x, y,
 * z and the atom index, then the largest |coordinate| that ljx_neigh_build's float distance test
 * needs. All four are device memory owned by the caller; nothing is allocated. */
ljx_status ljx_neigh_bin(void *stream, const double *x, int nall, const double *lo,
                         double binsize, const int *nbins, int *bin_start, int *bin_atoms,
                         int *scratch, void *sorted);

/* The list itself, from ljx_neigh_bin's bin_start, bin_atoms and sorted for the same x. Pairs are
 * tested in float with a rounding band around the cutoff; those inside it take LAMMPS's double
 * test, so the list is the double test's exactly. */
ljx_status ljx_neigh_build(void *stream, const double *x, int nall, int nlocal, double cutoff,
                           int half, const double *lo, double binsize, const int *nbins,
                           const int *bin_start, const int *bin_atoms, const void *sorted,
                           int *neighbors, long long slot_stride, int maxneigh, int *numneigh,
                           int *widest);

#ifdef __cplusplus
}
#endif

#endif /* LJX_NEIGH_H */
