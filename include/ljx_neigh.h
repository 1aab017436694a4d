/*
 * ljx_neigh — device neighbor-list build for the standalone harness (the step before the pack;
 * in LAMMPS this is NPairKokkos, outside the reference). Produces the same NeighListKokkos view
 * the pair style receives: owned rows over owned + ghost atoms, Kokkos LayoutLeft
 * (neighbors[i + jj * slot_stride]), pairs with r^2 < cutoff^2 (cutoff = model cutoff + skin).
 *
 * Binning: atoms are pre-sorted into a uniform grid of cubic bins (side `binsize` >= cutoff/2,
 * origin `lo`, `nbins` per dimension); bin b holds bin_atoms[bin_start[b] .. bin_start[b+1]).
 * `lo` (3 doubles) and `nbins` (3 ints) are HOST arrays; every other pointer is device memory.
 * Each owned atom scans a +-2 bin stencil. half != 0 keeps each pair once: owned j > i, or a
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

ljx_status ljx_neigh_build(void *stream, const double *x, int nall, int nlocal, double cutoff,
                           int half, const double *lo, double binsize, const int *nbins,
                           const int *bin_start, const int *bin_atoms, int *neighbors,
                           long long slot_stride, int maxneigh, int *numneigh, int *widest);

#ifdef __cplusplus
}
#endif

#endif /* LJX_NEIGH_H */
