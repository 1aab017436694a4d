"""The exporter side of the potential block (bundles written by the reference's exporter).

- export_potential.patch applies to the reference's python/lammps_jax/export.py and gives
  export_model a `potential=` argument that lands in the bundle (checked on the patched source's
  syntax tree; jax is not installed here, so the exporter itself cannot run);
- a bundle shaped exactly as export_model writes it (VHLO programs as opaque base64, serialized
  compile options, export_info with the jax version and platform, the full contract) plus the
  potential block loads through libljx's loader with the programs, contract and physics read;
- add_potential inserts the block into an already exported bundle;
- on a GPU, a reference-shaped bundle drives the engine to the same forces, bit for bit, as the
  bundle ljx writes itself.
"""

import ast
import base64
import json
import shutil
import subprocess

import numpy as np
import pytest

from conftest import REFERENCE, ROOT, load_package

PATCH = ROOT / "lammps-jax_b200" / "export_potential.patch"
EXPORT_PY = REFERENCE / "python" / "lammps_jax" / "export.py"


def reference_shaped(ljx, potential=None, seed=0, **contract):
    """A bundle dict with every key export_model writes (export.py:523-566), programs and
    compile options as opaque bytes."""
    rng = np.random.default_rng(seed)
    blob = lambda n: base64.b64encode(rng.bytes(n)).decode("ascii")  # noqa: E731
    c = {"input_layout": "sparse-edge", "max_atoms": 4096, "max_edges": 4096 * 128,
         "cutoff": 6.5, "unit_style": "metal", "precision": "float64",
         "force_output": "atom-force", "newton": "off", "n_hops": 1, "edge_pairing": "full",
         "comm_widths": [1], "comm_sites": [1, 0, 1], "custom_call_targets": ["lammps_jax_comm"],
         "uses_box": False, "pair_sum": False, "n_species": 2}
    c.update(contract)
    data = {
        "format": "lammps-jax-json-distributed",
        "programs": {"force_mlir_b64": blob(3000), "energy_mlir_b64": "",
                     "energy_and_forces_mlir_b64": blob(5000)},
        "export_info": {"jax_version": "0.8.1", "platform": "cuda"},
        "compile_options_b64": blob(64),
        "contract": c,
    }
    if potential is not None:
        data["potential"] = potential
    return data


def write(path, data):
    path.write_text(json.dumps(data, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return path


@pytest.mark.skipif(not EXPORT_PY.exists(), reason="needs the reference checkout")
def test_patch_gives_export_model_a_potential_argument(tmp_path):
    target = tmp_path / "python" / "lammps_jax" / "export.py"
    target.parent.mkdir(parents=True)
    shutil.copy(EXPORT_PY, target)
    out = subprocess.run(["patch", "-p1", "-i", str(PATCH)], cwd=tmp_path, capture_output=True,
                         text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    tree = ast.parse(target.read_text())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "export_model")
    assert "potential" in [a.arg for a in fn.args.kwonlyargs]
    stores = [n for n in ast.walk(fn) if isinstance(n, ast.Assign)
              and isinstance(n.targets[0], ast.Subscript)
              and isinstance(n.targets[0].slice, ast.Constant)
              and n.targets[0].slice.value == "potential"]
    assert len(stores) == 1
    # The block is added before the file is written.
    write_calls = [n for n in ast.walk(fn) if isinstance(n, ast.Call)
                   and getattr(n.func, "attr", "") == "write_text"]
    assert stores[0].lineno < min(c.lineno for c in write_calls)


def test_reference_shaped_bundle_with_potential_loads(ljx, tmp_path):
    text = ljx.synth.synthetic_setfl(("Cu", "Zr"), nr=500, nrho=500)
    path = write(tmp_path / "ref.json", reference_shaped(ljx, ljx.eam_potential(text)))
    b = ljx.Bundle.load(path)
    c = b.contract
    assert c["format"] == "lammps-jax-json-distributed" and c["platform"] == "cuda"
    assert (c["has_force_program"], c["has_energy_program"],
            c["has_energy_and_forces_program"]) == (1, 0, 1)
    assert c["comm_widths"] == [1] and c["comm_sites"] == [1, 0, 1]
    assert c["max_edges"] == 4096 * 128 and c["n_species"] == 2
    assert c["potential"] == ljx.abi.POTENTIAL_EAM and c["n_elements"] == 2
    tables = b.eam_tables()
    assert tables["nr"] == 500 and tables["pair"].shape == (3, 500, 4)


def test_add_potential_to_an_exported_bundle(ljx, tmp_path):
    path = write(tmp_path / "ref.json", reference_shaped(ljx, newton="off"))
    assert ljx.Bundle.load(path).contract["potential"] == ljx.abi.POTENTIAL_NONE
    ljx.add_potential(path, ljx.lj_potential(1.0, 1.0))
    raw = path.read_text()
    assert raw == json.dumps(json.loads(raw), indent=2, sort_keys=True) + "\n"
    c = ljx.Bundle.load(path).contract
    assert c["potential"] == ljx.abi.POTENTIAL_LJ and c["lj_sigma"] == 1.0
    assert c["has_force_program"] == 1  # the exporter's programs stay in place


@pytest.mark.gpu
def test_reference_shaped_bundle_drives_the_engine(tmp_path, monkeypatch):
    import torch

    # Every pair from both rows, no atomics (LJX_OWNED_HALF=0): two runs agree bit for bit.
    monkeypatch.setenv("LJX_OWNED_HALF", "0")

    from cases import device_system, eam_case, write_eam_bundle
    ljx = load_package()
    case = eam_case(elements=("Cu", "Zr"), cells=(3, 3, 3), seed=4, nr=1000, nrho=1000)
    nall = len(case.x_all)
    ours = write_eam_bundle(tmp_path, case, mode="rows-full", precision="float64",
                            max_atoms=nall + 64)
    theirs = write(tmp_path / "ref.json", reference_shaped(
        ljx, ljx.eam_potential(case.text), max_atoms=nall + 64, max_edges=(nall + 64) * 128))
    forces = []
    for path in (ours, theirs):
        system = device_system(case, newton=False, half=False)
        pair = ljx.PairJax(device=0)
        pair.coeff(system, "*", "*", str(path))
        pair.init_style(system)
        res = pair.compute(system)
        torch.cuda.synchronize()
        forces.append((system.f.cpu().numpy(), res.energy, list(res.virial)))
    np.testing.assert_array_equal(forces[0][0], forces[1][0])
    assert forces[0][1] == forces[1][1] and forces[0][2] == forces[1][2]
