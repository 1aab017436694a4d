"""The pair style's argument checks and messages (csrc/pair.cpp, the restatement of
cpp/pair_jax_kokkos.cpp:573-663, 665-785, 989-1000). Every case fails before an engine exists,
so these run without a GPU. The messages are the reference's, which its LAMMPS tests match as
negative controls (tests/test_lammps.py:445-461)."""

import ctypes

import pytest

from conftest import load_package


def lj_bundle(ljx, path, **kw):
    args = dict(potential=ljx.lj_potential(1.0, 1.0), max_atoms=1000, max_edges=64000,
                cutoff=2.5, unit_style="lj", precision="float64", force_output="edge-force",
                newton="off")
    args.update(kw)
    ljx.write_bundle(path, **args)
    return path


class Host:
    """The LAMMPS state PairJax reads in coeff / init_style."""

    def __init__(self, unit_style="lj", ntypes=1):
        self.unit_style = unit_style
        self.ntypes = ntypes


def fails(fn, message):
    ljx = load_package()
    with pytest.raises(ljx.LammpsError) as err:
        fn()
    assert str(err.value) == message


def test_settings_takes_at_most_one_argument():
    ljx = load_package()
    pair = ljx.PairJax()
    pair.settings()
    pair.settings("/opt/plugin.so")
    fails(lambda: pair.settings("a", "b"), "Illegal pair_style jax/kk command")


def test_coeff_argument_checks(tmp_path):
    ljx = load_package()
    path = lj_bundle(ljx, tmp_path / "lj.json")
    pair = ljx.PairJax()
    host = Host()
    fails(lambda: pair.coeff(host, "*", "*"), "Illegal pair_coeff jax/kk command")
    fails(lambda: pair.coeff(host, "*", "*", str(path), "1", "2"),
          "Illegal pair_coeff jax/kk command")
    fails(lambda: pair.coeff(host, "1", "3", str(path)), "Numeric index 3 is out of bounds (1-1)")
    fails(lambda: pair.coeff(host, "*", "*", str(path), "x"),
          "Expected floating point parameter instead of 'x' in input script or data file")


def test_coeff_model_checks(tmp_path):
    ljx = load_package()
    pair = ljx.PairJax()
    missing = tmp_path / "none.json"
    with pytest.raises(ljx.LammpsError) as err:
        pair.coeff(Host(), "*", "*", str(missing))
    assert str(err.value).startswith("Failed to load LAMMPS-JAX model: ")
    path = lj_bundle(ljx, tmp_path / "lj.json")
    fails(lambda: pair.coeff(Host(unit_style="metal"), "*", "*", str(path)),
          "LAMMPS-JAX model unit style does not match current units")
    two = lj_bundle(ljx, tmp_path / "two.json", n_species=1)
    fails(lambda: pair.coeff(Host(ntypes=2), "*", "*", str(two)),
          "LAMMPS-JAX model distinguishes 1 species but the system defines 2 atom types; types "
          "beyond the model's range would silently map to its last species")
    cpu = lj_bundle(ljx, tmp_path / "cpu.json", platform="cpu")
    fails(lambda: pair.coeff(Host(), "*", "*", str(cpu)),
          "LAMMPS-JAX model was exported for cpu but this build runs cuda; re-export it with "
          "platform=\"cuda\"")


def test_calls_out_of_order():
    ljx = load_package()
    pair = ljx.PairJax()
    lib = ljx.abi.load()
    plan = ljx.abi.Plan()
    status = lib.ljx_pair_init_style(pair._h, 1, 0, None, None, 0, None, ctypes.byref(plan))
    assert status != ljx.abi.OK
    assert lib.ljx_pair_error(pair._h).decode() == "LAMMPS-JAX model has not been loaded"
    status = lib.ljx_pair_compute(pair._h, None, None, None, 1, 1, None, None)
    assert status != ljx.abi.OK
    assert lib.ljx_pair_error(pair._h).decode() == "LAMMPS-JAX runtime is not initialized"
    assert lib.ljx_pair_init_one(pair._h) == 0.0
