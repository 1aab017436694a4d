"""Generate the golden vectors in tests/golden/ by running the lammps-jax reference itself.

Run where the reference checkout exists (a directory named reference beside this repository, or
the path in LJX_REFERENCE):  python tests/golden/make_golden.py

jax is not installed here, so numpy_jax_shim.py stands in for jax.numpy; the reference's own
python/lammps_jax/eam.py and the LJ energy builder of examples/export_model.py then run
unchanged on numpy arrays. Fixture inputs come from the reference test suite's own generators
(tests/helpers.py random_system / edges_within_cutoff / native_interpolate, tests/test_eam.py
synthetic_setfl / native_numpy_reference, tests/test_distributed.py cuzr_cluster), which are
loaded from the reference checkout by name and executed, not copied.

Outputs (small .npz files plus the tiny setfl table the reference test writes):
  tiny.eam.alloy                 synthetic_setfl(nrho=12, nr=10) as the reference writes it
  golden_spline.npz              spline_coefficients / spline_lookup on a sinh table, f64 and f32
  golden_tiny_setfl.npz          make_setfl_energy / make_setfl_edge_force, full and half pairing,
                                 f64 and f32, plus native_numpy_reference and central differences
  golden_cuzr_cluster.npz        same builders on the CuZr Zhou-2004 table and cuzr_cluster
                                 (the table itself is read from the reference checkout at test
                                 time and is not vendored)
  golden_lj.npz                  make_lj_energy per-atom energies, f64 and f32, both scales
"""

from __future__ import annotations

import ast
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("LJX_REFERENCE", HERE.parents[2] / "reference"))

sys.path.insert(0, str(HERE))
import numpy_jax_shim  # noqa: E402

jax, jnp = numpy_jax_shim.install()
sys.path.insert(0, str(REF / "python"))
from lammps_jax import eam  # noqa: E402  (the reference module, run under the shim)


def load_reference_functions(path: Path, names: list[str], namespace: dict) -> dict:
    """Execute the named top-level functions of a reference test file in `namespace`."""
    tree = ast.parse(path.read_text())
    wanted = [node for node in tree.body
              if isinstance(node, ast.FunctionDef) and node.name in names]
    missing = set(names) - {node.name for node in wanted}
    if missing:
        raise RuntimeError(f"{path}: missing {sorted(missing)}")
    module = ast.Module(body=wanted, type_ignores=[])
    exec(compile(module, str(path), "exec"), namespace)
    return namespace


def reference_namespace() -> dict:
    ns = {"np": np, "jnp": jnp, "Path": Path}
    load_reference_functions(REF / "tests" / "helpers.py",
                             ["random_system", "edges_within_cutoff", "native_interpolate"], ns)
    load_reference_functions(REF / "tests" / "test_eam.py",
                             ["synthetic_setfl", "native_numpy_reference"], ns)
    load_reference_functions(REF / "tests" / "test_distributed.py", ["cuzr_cluster"], ns)
    return ns


def lj_builders():
    """make_lj_energy from examples/export_model.py, importing it with the exporter stubbed."""
    stub = types.ModuleType("lammps_jax.export")
    stub.export_model = None
    sys.modules["lammps_jax.export"] = stub
    sys.path.insert(0, str(REF / "examples"))
    import export_model  # noqa: E402  (reference example module)
    return export_model


class Graph:
    def __init__(self, senders, receivers, mask=None):
        self.senders = numpy_jax_shim.wrap(np.asarray(senders, np.int32))
        self.receivers = numpy_jax_shim.wrap(np.asarray(receivers, np.int32))
        m = np.ones(len(senders), bool) if mask is None else np.asarray(mask, bool)
        self.edge_mask = numpy_jax_shim.wrap(m)


def run_setfl(tables, positions, species, senders, receivers, dtype, half=False):
    pos = numpy_jax_shim.wrap(np.asarray(positions, dtype))
    spc = numpy_jax_shim.wrap(np.asarray(species, np.int32))
    graph = Graph(senders, receivers)
    energy = eam.make_setfl_energy(tables, half_edges=half)(pos, spc, graph)
    edge_force = eam.make_setfl_edge_force(tables, half_edges=half)(pos, spc, graph)
    return np.asarray(energy), np.asarray(edge_force)


def central_difference_forces(tables, positions, species, senders, receivers, step=1e-6):
    """-dE/dx of the reference's summed f64 energy by central differences (graph held fixed)."""
    base = np.asarray(positions, np.float64)
    out = np.zeros_like(base)
    fn = eam.make_setfl_energy(tables)
    spc = numpy_jax_shim.wrap(np.asarray(species, np.int32))
    graph = Graph(senders, receivers)
    for i in range(base.shape[0]):
        for k in range(3):
            plus = base.copy()
            minus = base.copy()
            plus[i, k] += step
            minus[i, k] -= step
            ep = float(np.sum(np.asarray(fn(numpy_jax_shim.wrap(plus), spc, graph))))
            em = float(np.sum(np.asarray(fn(numpy_jax_shim.wrap(minus), spc, graph))))
            out[i, k] = -(ep - em) / (2 * step)
    return out


def main() -> None:
    ns = reference_namespace()

    # Spline scheme (eam.py:115-164) on the table of test_embedding_extrapolates_linearly_past_rhomax.
    nodes = np.linspace(0.0, 3.0, 31)
    drho = float(nodes[1] - nodes[0])
    values = np.sinh(nodes)
    coeffs = eam.spline_coefficients(values)
    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.random(64) * 3.0, 3.0 + rng.random(16) * 10.0, [0.0, 3.0, 1.5]])
    spline = {"values": values, "delta": drho, "coeffs": coeffs, "x": xs,
              "native_coeffs": ns["native_interpolate"](values)}
    for tag, dtype in (("f64", np.float64), ("f32", np.float32)):
        c = numpy_jax_shim.wrap(coeffs[None].astype(dtype))
        x = numpy_jax_shim.wrap(xs.astype(dtype))
        ids = numpy_jax_shim.wrap(np.zeros(xs.size, np.int32))
        for ext in (False, True):
            for der in (False, True):
                key = f"{tag}_ext{int(ext)}_der{int(der)}"
                spline[key] = np.asarray(eam.spline_lookup(c, ids, x, drho, extrapolate=ext,
                                                           derivative=der))
    np.savez_compressed(HERE / "golden_spline.npz", **spline)

    # Tiny two-element setfl of the reference tests.
    tiny_path = HERE / "tiny.eam.alloy"
    ns["synthetic_setfl"](tiny_path)
    tables = eam.load_setfl(str(tiny_path))
    out = {"embedding": tables["embedding"], "density": tables["density"],
           "pair": tables["pair"], "pair_index": tables["pair_index"]}
    # Fixture of test_setfl_energy_matches_native_numpy_reference (test_eam.py:397-429).
    positions = ns["random_system"](seed=23, n_atoms=32, box=(3.0, 2.0, 2.0)).astype(np.float64)
    species = np.random.default_rng(29).integers(0, 2, size=32)
    senders, receivers = ns["edges_within_cutoff"](positions, tables["cutoff"])
    out.update(positions=positions, species=species, senders=senders, receivers=receivers)
    for tag, dtype in (("f64", np.float64), ("f32", np.float32)):
        e, fe = run_setfl(tables, positions, species, senders, receivers, dtype)
        out[f"energy_{tag}"], out[f"edge_force_{tag}"] = e, fe
    native_e, native_f, native_rho = ns["native_numpy_reference"](tables, positions, species)
    out.update(native_energy=native_e, native_forces=native_f, native_density=native_rho)
    out["fd_forces"] = central_difference_forces(tables, positions, species, senders, receivers)
    # Half pairing (test_half_edges_match_full_pairing, test_eam.py:467-508).
    hpos = ns["random_system"](seed=31, n_atoms=32, box=(3.0, 2.0, 2.0)).astype(np.float64)
    hspc = np.random.default_rng(37).integers(0, 2, size=32)
    hs, hr = ns["edges_within_cutoff"](hpos, tables["cutoff"])
    keep = hs < hr
    out.update(half_positions=hpos, half_species=hspc, half_senders=hs[keep],
               half_receivers=hr[keep], full_senders=hs, full_receivers=hr)
    for tag, dtype in (("f64", np.float64), ("f32", np.float32)):
        e, fe = run_setfl(tables, hpos, hspc, hs[keep], hr[keep], dtype, half=True)
        out[f"half_energy_{tag}"], out[f"half_edge_force_{tag}"] = e, fe
        e, fe = run_setfl(tables, hpos, hspc, hs, hr, dtype)
        out[f"half_full_energy_{tag}"], out[f"half_full_edge_force_{tag}"] = e, fe
    np.savez_compressed(HERE / "golden_tiny_setfl.npz", **out)

    # Real CuZr table (Zhou 2004) on the reference's cuzr_cluster fixture.
    cuzr = eam.load_setfl(str(REF / "examples" / "potentials" / "CuZr.eam.alloy.gz"))
    cpos, cspc = ns["cuzr_cluster"](cuzr)
    cs, cr = ns["edges_within_cutoff"](cpos, cuzr["cutoff"])
    out = {"positions": cpos, "species": cspc, "senders": cs, "receivers": cr,
           "density_row1000": cuzr["density"][:, 1000], "pair_row1000": cuzr["pair"][:, 1000],
           "embedding_row500": cuzr["embedding"][:, 500]}
    for tag, dtype in (("f64", np.float64), ("f32", np.float32)):
        e, fe = run_setfl(cuzr, cpos, cspc, cs, cr, dtype)
        out[f"energy_{tag}"], out[f"edge_force_{tag}"] = e, fe
    ne, nf, nrho = ns["native_numpy_reference"](cuzr, cpos.astype(np.float64), cspc)
    out.update(native_energy=ne, native_forces=nf, native_density=nrho)
    np.savez_compressed(HERE / "golden_cuzr_cluster.npz", **out)

    # LJ energy builder (examples/export_model.py:16-50) on test_lj_example_padded_edges_... input.
    ex = lj_builders()
    lpos = ns["random_system"](seed=5, n_atoms=32, box=(3.0, 2.0, 2.0)).astype(np.float64)
    ls, lr = ns["edges_within_cutoff"](lpos, 1.6)
    out = {"positions": lpos, "senders": ls, "receivers": lr, "cutoff": 1.6}
    for tag, dtype in (("f64", np.float64), ("f32", np.float32)):
        for scale in (0.5, 1.0):
            fn = ex.make_lj_energy(cutoff=1.6, epsilon=1.0, sigma=1.0, edge_energy_scale=scale)
            e = fn(numpy_jax_shim.wrap(lpos.astype(dtype)), None, Graph(ls, lr))
            out[f"energy_{tag}_s{scale}"] = np.asarray(e)
    # -dE/dx of the f64 full-list energy (scale 0.5) by central differences, graph held fixed.
    fn = ex.make_lj_energy(cutoff=1.6, epsilon=1.0, sigma=1.0, edge_energy_scale=0.5)
    fd = np.zeros_like(lpos)
    step = 1e-6
    for i in range(lpos.shape[0]):
        for k in range(3):
            plus, minus = lpos.copy(), lpos.copy()
            plus[i, k] += step
            minus[i, k] -= step
            ep = float(np.sum(np.asarray(fn(numpy_jax_shim.wrap(plus), None, Graph(ls, lr)))))
            em = float(np.sum(np.asarray(fn(numpy_jax_shim.wrap(minus), None, Graph(ls, lr)))))
            fd[i, k] = -(ep - em) / (2 * step)
    out["fd_forces_s0.5"] = fd
    np.savez_compressed(HERE / "golden_lj.npz", **out)
    print("wrote", sorted(p.name for p in HERE.glob("golden_*.npz")), tiny_path.name)


if __name__ == "__main__":
    main()
