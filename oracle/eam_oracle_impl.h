/*
 * CPU ORACLE — TEST INFRASTRUCTURE ONLY (see eam_oracle.c). Included twice with REAL = double and
 * REAL = float; SUF(name) appends the precision suffix.
 */

/*
 * Stacked-spline evaluation at x with spacing delta; python/lammps_jax/eam.py:138-164.
 * c points at one table [n][4]. Past the table the value saturates, or with `extrapolate`
 * continues linearly with the end slope (pair_eam past rhomax), and the slope is the end slope.
 */
static inline void SUF(orc_spline)(const REAL *c, int n, REAL x, REAL delta, int extrapolate,
                                  REAL *value, REAL *slope)
{
  const REAL idx = x / delta;
  REAL fl = (REAL) floor((double) idx);
  if (fl < (REAL) 0) fl = (REAL) 0;
  if (fl > (REAL) (n - 2)) fl = (REAL) (n - 2);
  const int node = (int) fl;
  const REAL t_raw = idx - (REAL) node;
  const REAL t = t_raw < (REAL) 1 ? t_raw : (REAL) 1;
  const REAL *k = c + 4 * (long) node;
  REAL v = k[0] + t * (k[1] + t * (k[2] + t * k[3]));
  REAL s = k[1] + t * ((REAL) 2 * k[2] + t * ((REAL) 3 * k[3]));
  if (extrapolate) {
    const REAL end = k[1] + (REAL) 2 * k[2] + (REAL) 3 * k[3];
    v = v + (t_raw - t) * end;
    if (t_raw > t) s = end;
  }
  if (value) *value = v;
  if (slope) *slope = s / delta;
}

/* Batch evaluation for the spline fixtures (values or slopes at m points). */
void SUF(orc_spline_eval)(const REAL *c, int n, const REAL *x, int m, REAL delta, int extrapolate,
                          int derivative, REAL *out)
{
  for (int i = 0; i < m; ++i) {
    REAL v, s;
    SUF(orc_spline)(c, n, x[i], delta, extrapolate, &v, &s);
    out[i] = derivative ? s : v;
  }
}

/* Row of the setfl pair table for elements a, b; python/lammps_jax/eam.py:167-171. */
static inline int SUF(orc_pair_row)(int a, int b)
{
  const int hi = a > b ? a : b, lo = a > b ? b : a;
  return hi * (hi + 1) / 2 + lo;
}

/* Positions to contract precision and 0-based species: cpp/pair_jax_kokkos.cpp:35-52. */
void SUF(orc_pack_atoms)(const double *x, const int *type, int span, REAL *positions, int *species)
{
  for (int i = 0; i < span; ++i) {
    positions[3 * i + 0] = (REAL) x[3 * i + 0];
    positions[3 * i + 1] = (REAL) x[3 * i + 1];
    positions[3 * i + 2] = (REAL) x[3 * i + 2];
    species[i] = type[i] - 1;
  }
}

#ifndef ORC_ATOMIC_ADD_DEFINED
#define ORC_ATOMIC_ADD_DEFINED
#define ORC_ATOMIC _Pragma("omp atomic")
#endif

/* Sender-segment starts of an edge prefix sorted by sender (returns the segment count). */
static int SUF(orc_segments)(const int *senders, const unsigned char *mask, int n_edges, int *starts)
{
  int nseg = 0;
  for (int e = 0; e < n_edges; ++e)
    if (e == 0 || senders[e] != senders[e - 1]) starts[nseg++] = e;
  (void) mask;
  starts[nseg] = n_edges;
  return nseg;
}

/*
 * One evaluation of the setfl EAM model over a packed edge list, in three distribution modes:
 *
 *  mode 0 — plain ("ghost") bundle: make_setfl_energy on full pairing, python/lammps_jax/eam.py:
 *           265-333, forces = -dE/dx of the selected energy (python/lammps_jax/export.py:153-209),
 *           energy = owned rows unless a valid edge starts on a ghost row (export.py:54-59,194).
 *           Each edge contributes dE/dr = F'(rho_s) rho'_{t(r)}(r) + phi'(r)/2 to both endpoints.
 *  mode 1 — full pairing, newton off, density forward-communicated: the row kernels of
 *           python/lammps_jax/eam_pallas.py:181-250 with half=False and their export
 *           (examples/export_eam_pallas.py:48-94, :336-345): each row owns its complete force
 *           f_i = sum psip/r * rij, psip = fp_i rho'_j + fp_j rho'_i + phi' (eam.py:383-398);
 *           energy = owned rows (export.py:190-192) with phi/2 per edge (eam_pallas.py:215).
 *  mode 2 — communicating half-unique pairing: densities scatter to both endpoints
 *           (eam.py:310-314), reverse comm completes owners and zeroes ghosts, forward comm fills
 *           ghost rows (eam.py:375-381), forces are psip/r*rij on the sender and the negative on
 *           the receiver (eam.py:396-398 plus the newton scatter of pair_jax_kokkos.cpp:219-223);
 *           energy = owned rows with phi to the sender (eam.py:303-305).
 *
 * Comm is emulated for one rank with periodic images: ghost row nlocal+g mirrors owner[g].
 * Outputs (all arrays sized n_rows, zero-initialised here): rho, fp, atom_energy, model_force
 * [n_rows][3] (the program's per-atom force output), edge_force [n_edges][3] (the edge-force
 * builder's psip/r*rij, modes 1-2; dE/dr-weighted one-sided force in mode 0), energy (selected
 * scalar, accumulated in double) and virial[6] = sum over valid edges of -w rij (x) F_e with
 * w = 1/2 for mode 1 (each pair appears in two rows) and 1 otherwise.
 */
void SUF(orc_eam_model)(int n_el, int nrho, int nr, REAL drho, REAL dr, REAL cutoff_sq,
                        const REAL *embedding, const REAL *density, const REAL *pair,
                        const REAL *pos, const int *species, int n_rows, int nlocal, int nghost,
                        const int *senders, const int *receivers, const unsigned char *mask,
                        int n_edges, int mode, const int *owner, REAL *rho, REAL *fp,
                        REAL *atom_energy, REAL *model_force, REAL *edge_force, double *energy,
                        double *virial)
{
  (void) n_el;
  memset(rho, 0, sizeof(REAL) * (size_t) n_rows);
  memset(fp, 0, sizeof(REAL) * (size_t) n_rows);
  memset(atom_energy, 0, sizeof(REAL) * (size_t) n_rows);
  memset(model_force, 0, sizeof(REAL) * 3 * (size_t) n_rows);
  if (edge_force) memset(edge_force, 0, sizeof(REAL) * 3 * (size_t) n_edges);
  const int half = mode == 2;
  int *starts = (int *) malloc(sizeof(int) * ((size_t) n_edges + 1));
  const int nseg = SUF(orc_segments)(senders, mask, n_edges, starts);
  const long nrt = (long) nr * 4, nrhot = (long) nrho * 4;

  /* Density pass (eam.py:284-299, 310-314). */
#pragma omp parallel for schedule(dynamic, 64)
  for (int sg = 0; sg < nseg; ++sg) {
    for (int e = starts[sg]; e < starts[sg + 1]; ++e) {
      const int s = senders[e], r = receivers[e];
      if (!mask[e] || s >= n_rows || r >= n_rows) continue;
      const REAL dx = pos[3 * r] - pos[3 * s], dy = pos[3 * r + 1] - pos[3 * s + 1],
                 dz = pos[3 * r + 2] - pos[3 * s + 2];
      const REAL rsq = dx * dx + dy * dy + dz * dz;
      if (!(rsq < cutoff_sq)) continue;
      const REAL rr = (REAL) sqrt((double) rsq);
      REAL v;
      SUF(orc_spline)(density + species[r] * nrt, nr, rr, dr, 0, &v, NULL);
      ORC_ATOMIC
      rho[s] += v;
      if (half) {
        SUF(orc_spline)(density + species[s] * nrt, nr, rr, dr, 0, &v, NULL);
        ORC_ATOMIC
        rho[r] += v;
      }
    }
  }
  /* Density exchange (eam.py:315-317, 375-381) emulated on periodic images. */
  if (mode == 1) {
    for (int g = 0; g < nghost; ++g) rho[nlocal + g] = rho[owner[g]];
  } else if (mode == 2) {
    for (int g = 0; g < nghost; ++g) {
      rho[owner[g]] += rho[nlocal + g];
      rho[nlocal + g] = 0;
    }
  }
  /* Embedding (eam.py:319-321, 383-384); the forward fill of mode 2 happens after the reverse,
   * and ghost F' in modes 1-2 is the owner's. */
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n_rows; ++i) {
    REAL v, s;
    SUF(orc_spline)(embedding + species[i] * nrhot, nrho, rho[i], drho, 1, &v, &s);
    atom_energy[i] = v;
    fp[i] = s;
  }
  if (mode == 2) {
    /* Energy of mode 2 embeds before the forward fill (eam.py:315-321): ghost rows embed the
     * zeroed density; owned rows are the ones counted. The forces use the forward fill. */
    for (int g = 0; g < nghost; ++g) {
      rho[nlocal + g] = rho[owner[g]];
      fp[nlocal + g] = fp[owner[g]];
    }
  }

  /* Pair and force pass (eam.py:300-309, 383-398). */
  int ghost_sender = 0;
  double vir[6] = {0, 0, 0, 0, 0, 0};
#pragma omp parallel
  {
    double lv[6] = {0, 0, 0, 0, 0, 0};
    int lghost = 0;
#pragma omp for schedule(dynamic, 64)
    for (int sg = 0; sg < nseg; ++sg) {
      for (int e = starts[sg]; e < starts[sg + 1]; ++e) {
        const int s = senders[e], r = receivers[e];
        if (!mask[e] || s >= n_rows || r >= n_rows) continue;
        if (s >= nlocal) lghost = 1;
        const REAL dx = pos[3 * r] - pos[3 * s], dy = pos[3 * r + 1] - pos[3 * s + 1],
                   dz = pos[3 * r + 2] - pos[3 * s + 2];
        const REAL rsq = dx * dx + dy * dy + dz * dz;
        if (!(rsq < cutoff_sq)) continue;
        const REAL rr = (REAL) sqrt((double) rsq);
        const int ss = species[s], sr = species[r];
        REAL rhojp, rhoip, z2, z2p;
        SUF(orc_spline)(density + sr * nrt, nr, rr, dr, 0, NULL, &rhojp);
        SUF(orc_spline)(density + ss * nrt, nr, rr, dr, 0, NULL, &rhoip);
        SUF(orc_spline)(pair + SUF(orc_pair_row)(ss, sr) * nrt, nr, rr, dr, 0, &z2, &z2p);
        const REAL phi = z2 / rr;
        const REAL phip = (z2p - phi) / rr;
        REAL d_e, w;
        REAL pe;
        int scatter;
        if (mode == 0) {
          d_e = fp[s] * rhojp + (REAL) 0.5 * phip;
          pe = (REAL) 0.5 * phi;
          w = 1;
          scatter = 1;
        } else if (mode == 1) {
          d_e = fp[s] * rhojp + fp[r] * rhoip + phip;
          pe = (REAL) 0.5 * phi;
          w = (REAL) 0.5;
          scatter = 0;
        } else {
          d_e = fp[s] * rhojp + fp[r] * rhoip + phip;
          pe = phi;
          w = 1;
          scatter = 1;
        }
        const REAL sc = d_e / rr;
        const REAL fx = sc * dx, fy = sc * dy, fz = sc * dz;
        if (edge_force) {
          edge_force[3 * e] = fx;
          edge_force[3 * e + 1] = fy;
          edge_force[3 * e + 2] = fz;
        }
        atom_energy[s] += pe; /* sender segments belong to one thread */
        if (scatter) {
          /* Receiver rows may be another thread's senders: every force update is atomic. */
          ORC_ATOMIC
          model_force[3 * s] += fx;
          ORC_ATOMIC
          model_force[3 * s + 1] += fy;
          ORC_ATOMIC
          model_force[3 * s + 2] += fz;
          ORC_ATOMIC
          model_force[3 * r] -= fx;
          ORC_ATOMIC
          model_force[3 * r + 1] -= fy;
          ORC_ATOMIC
          model_force[3 * r + 2] -= fz;
        } else {
          model_force[3 * s] += fx;
          model_force[3 * s + 1] += fy;
          model_force[3 * s + 2] += fz;
        }
        lv[0] -= (double) w * dx * fx;
        lv[1] -= (double) w * dy * fy;
        lv[2] -= (double) w * dz * fz;
        lv[3] -= (double) w * dx * fy;
        lv[4] -= (double) w * dx * fz;
        lv[5] -= (double) w * dy * fz;
      }
    }
#pragma omp critical
    {
      for (int k = 0; k < 6; ++k) vir[k] += lv[k];
      ghost_sender |= lghost;
    }
  }
  /* Energy selection: export.py:167-195. */
  const int rows = (mode == 0 && ghost_sender) ? nlocal + nghost : nlocal;
  double etot = 0.0;
  for (int i = 0; i < rows && i < n_rows; ++i) etot += (double) atom_energy[i];
  *energy = etot;
  for (int k = 0; k < 6; ++k) virial[k] = vir[k];
  free(starts);
}

/*
 * Lennard-Jones 12-6, hard cutoff, no shift: examples/export_model.py:16-74.
 * valid = mask & r^2 > 1e-12 & r^2 < rc^2 (:22); per-edge energy scaled by edge_energy_scale
 * (0.5 on full lists, 1.0 for newton-on edge-force exports, :30-50,107) and added to the sender.
 * edge_force = dU/d(rij), rij = x_receiver - x_sender (:53-74), zero on invalid edges.
 * model_force = -dE/dx of the selected energy (the atom-force program), energy selected as in
 * export.py:167-195. virial_edge = -w sum rij (x) F_e with w = 1/2 (full list, newton off:
 * every pair appears twice) or 1 (newton on: the receiver takes -F_e).
 */
void SUF(orc_lj_model)(REAL four_eps, REAL sigma_sq, REAL cutoff_sq, REAL edge_energy_scale,
                       const REAL *pos, int n_rows, int nlocal, int nghost, const int *senders,
                       const int *receivers, const unsigned char *mask, int n_edges,
                       double virial_weight, REAL *atom_energy, REAL *edge_force,
                       REAL *model_force, double *energy, double *virial)
{
  memset(atom_energy, 0, sizeof(REAL) * (size_t) n_rows);
  memset(model_force, 0, sizeof(REAL) * 3 * (size_t) n_rows);
  memset(edge_force, 0, sizeof(REAL) * 3 * (size_t) n_edges);
  int ghost_sender = 0;
  double vir[6] = {0, 0, 0, 0, 0, 0};
  for (int e = 0; e < n_edges; ++e) {
    const int s = senders[e], r = receivers[e];
    if (!mask[e] || s >= n_rows || r >= n_rows) continue;
    if (s >= nlocal) ghost_sender = 1;
    const REAL dx = pos[3 * r] - pos[3 * s], dy = pos[3 * r + 1] - pos[3 * s + 1],
               dz = pos[3 * r + 2] - pos[3 * s + 2];
    const REAL rsq = dx * dx + dy * dy + dz * dz;
    if (!(rsq > (REAL) 1.0e-12 && rsq < cutoff_sq)) continue;
    const REAL inv_r2 = sigma_sq / rsq;
    const REAL inv_r6 = inv_r2 * inv_r2 * inv_r2;
    const REAL u = four_eps * (inv_r6 * inv_r6 - inv_r6);
    atom_energy[s] += edge_energy_scale * u;
    /* dU/d(r^2) = -4eps (6 a^6 - 3 a^3) / r^2 with a = sigma^2/r^2; dU/drij = 2 rij dU/d(r^2). */
    const REAL du_drsq = -four_eps * ((REAL) 6 * inv_r6 * inv_r6 - (REAL) 3 * inv_r6) / rsq;
    const REAL fx = (REAL) 2 * du_drsq * dx, fy = (REAL) 2 * du_drsq * dy,
               fz = (REAL) 2 * du_drsq * dz;
    edge_force[3 * e] = fx;
    edge_force[3 * e + 1] = fy;
    edge_force[3 * e + 2] = fz;
    /* -dE/dx of edge_energy_scale * U: sender += scale * dU/drij, receiver -= it. */
    model_force[3 * s] += edge_energy_scale * fx;
    model_force[3 * s + 1] += edge_energy_scale * fy;
    model_force[3 * s + 2] += edge_energy_scale * fz;
    model_force[3 * r] -= edge_energy_scale * fx;
    model_force[3 * r + 1] -= edge_energy_scale * fy;
    model_force[3 * r + 2] -= edge_energy_scale * fz;
    vir[0] -= virial_weight * dx * fx;
    vir[1] -= virial_weight * dy * fy;
    vir[2] -= virial_weight * dz * fz;
    vir[3] -= virial_weight * dx * fy;
    vir[4] -= virial_weight * dx * fz;
    vir[5] -= virial_weight * dy * fz;
  }
  const int rows = ghost_sender ? nlocal + nghost : nlocal;
  double etot = 0.0;
  for (int i = 0; i < rows && i < n_rows; ++i) etot += (double) atom_energy[i];
  *energy = etot;
  for (int k = 0; k < 6; ++k) virial[k] = vir[k];
}
