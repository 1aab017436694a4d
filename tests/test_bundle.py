"""Bundle loader (libljx, no GPU needed): same lookup, validation and messages as the
reference loader (cpp/lammps_jax_model.cpp:212-315), plus the potential block."""

import json

import numpy as np
import pytest

from conftest import GOLDEN, CUZR_TABLE


def base(ljx, **kw):
    args = dict(potential=ljx.lj_potential(1.0, 1.0), max_atoms=64, max_edges=512, cutoff=2.5,
                unit_style="lj", precision="float64", force_output="edge-force", newton="off")
    args.update(kw)
    return ljx.bundle_dict(**args)


def load(ljx, data):
    return ljx.Bundle.from_string(json.dumps(data, indent=2, sort_keys=True))


def expect_error(ljx, data, message):
    with pytest.raises(ljx.LjxError, match=message) as err:
        load(ljx, data)
    assert err.value.status == ljx.abi.ERR_BUNDLE


def test_contract_round_trip(ljx):
    c = load(ljx, base(ljx)).contract
    assert c["max_atoms"] == 64 and c["max_edges"] == 512 and c["cutoff"] == 2.5
    assert c["unit_style"] == "lj" and c["precision"] == ljx.abi.FLOAT64
    assert c["force_layout"] == ljx.abi.FORCE_EDGE and c["newton"] == ljx.abi.NEWTON_OFF
    assert c["format"] == "lammps-jax-json" and c["platform"] == "cuda"
    assert c["potential"] == ljx.abi.POTENTIAL_LJ
    assert c["lj_edge_energy_scale"] == 0.5  # full list, newton off (export_model.py:107)
    on = load(ljx, base(ljx, newton="on")).contract
    assert on["lj_edge_energy_scale"] == 1.0


def test_sorted_key_first_match_ignores_later_blocks(ljx):
    data = base(ljx)
    text = json.dumps(data, indent=2, sort_keys=True)
    # A "cutoff" key after the contract (e.g. inside export_info) must not win the lookup.
    data["export_info"]["zz_note"] = {"cutoff": 99.0}
    assert load(ljx, data).contract["cutoff"] == 2.5
    assert json.loads(text)["contract"]["cutoff"] == 2.5


@pytest.mark.parametrize("mutate,message", [
    (lambda d: d.pop("format"), "Missing key in bundle: format"),
    (lambda d: d.update(format="lammps-jax-json-v9"), "Unsupported bundle format"),
    (lambda d: d["contract"].update(precision="float16"), "Unsupported LAMMPS-JAX precision"),
    (lambda d: d["contract"].update(input_layout="dense"), "Unsupported LAMMPS-JAX input layout"),
    (lambda d: d["contract"].update(force_output="virial"), "force output layout"),
    (lambda d: d["contract"].update(newton="maybe"), "Unsupported LAMMPS-JAX newton mode"),
    (lambda d: d["contract"].update(max_edges=0), "Invalid fixed capacities in bundle"),
    (lambda d: d["contract"].update(n_species=-1), "Invalid n_species in bundle"),
    (lambda d: d["contract"].update(max_owned=1000), "Invalid max_owned in bundle"),
    (lambda d: d["contract"].update(max_owned=8), "max_owned needs a communicating"),
    (lambda d: d["contract"].update(n_hops=0), "Invalid n_hops in bundle"),
    (lambda d: d["contract"].update(n_hops=2), "Bundles with n_hops > 1 require newton on"),
    (lambda d: d["contract"].update(uses_box="yes"), "Expected boolean for key: uses_box"),
])
def test_contract_validation_messages(ljx, mutate, message):
    data = base(ljx)
    mutate(data)
    expect_error(ljx, data, message)


def test_half_edge_and_comm_rules(ljx):
    d = base(ljx, newton="on", comm=True, half_edges=True, force_output="atom-force")
    assert load(ljx, d).contract["edge_pairing"] == ljx.abi.PAIRING_HALF_UNIQUE
    d = base(ljx, newton="on", comm=True, half_edges=True)
    d["contract"]["edge_pairing"] = "half"
    expect_error(ljx, d, "Communicating half-edge bundles now pack each boundary pair")
    d = base(ljx, newton="on", comm=False, half_edges=True)
    d["contract"]["edge_pairing"] = "half-unique"
    expect_error(ljx, d, "Unique-boundary bundles need a communication schedule")
    d["contract"]["edge_pairing"] = "quarter"
    expect_error(ljx, d, "Invalid edge_pairing in bundle")
    d = base(ljx, newton="on", half_edges=True)
    expect_error(ljx, d, "Half-edge bundles require n_hops > 1 or a communication schedule")
    d = base(ljx, newton="off", comm=True, half_edges=True)
    expect_error(ljx, d, "Communicating bundles require newton on unless")
    d = base(ljx, newton="on", comm=True)
    expect_error(ljx, d, "Communicating edge-force bundles require half-edge packing")
    d = base(ljx, newton="on", comm=True, comm_widths=[0], force_output="atom-force")
    expect_error(ljx, d, "Invalid communication width in bundle")
    d = base(ljx, max_edges=None, max_neighbors=16)
    expect_error(ljx, d, "Neighbor-matrix bundles return per-atom forces")


def test_setfl_tables_match_oracle(ljx, oracle):
    text = (GOLDEN / "tiny.eam.alloy").read_text()
    b = load(ljx, base(ljx, potential=ljx.eam_potential(text), unit_style="metal",
                       force_output="atom-force", newton="on", cutoff=2.0))
    t = b.eam_tables()
    ref = oracle.parse_setfl_text(text)
    for key in ("embedding", "density", "pair"):
        np.testing.assert_array_equal(t[key], ref[key])
    assert (t["nrho"], t["nr"], t["drho"], t["dr"], t["cutoff"]) == \
        (ref["nrho"], ref["nr"], ref["drho"], ref["dr"], ref["cutoff"])
    assert b.contract["potential"] == ljx.abi.POTENTIAL_EAM and b.contract["n_elements"] == 2


@pytest.mark.skipif(not CUZR_TABLE.exists(), reason="CuZr table lives in the reference checkout")
def test_cuzr_setfl_tables_match_oracle(ljx, oracle):
    text = "\n".join(oracle.read_table_lines(CUZR_TABLE)) + "\n"
    b = load(ljx, base(ljx, potential=ljx.eam_potential(text), unit_style="metal",
                       force_output="atom-force", newton="on", cutoff=7.1553683345038239))
    t = b.eam_tables()
    ref = oracle.load_setfl(CUZR_TABLE)
    for key in ("embedding", "density", "pair"):
        np.testing.assert_array_equal(t[key], ref[key])


def test_funcfl_potential(ljx, oracle, tmp_path):
    nrho, nr = 8, 6
    embed = np.linspace(0.0, -2.0, nrho)
    z = np.linspace(2.0, 0.0, nr)
    rho = np.linspace(1.0, 0.0, nr)
    lines = ["comment", "29 63.55 3.615 fcc", f"{nrho} 0.5 {nr} 0.25 1.5"]
    lines += [repr(float(v)) for v in np.concatenate([embed, z, rho])]
    text = "\n".join(lines) + "\n"
    (tmp_path / "tiny.eam").write_text(text)
    b = load(ljx, base(ljx, potential=ljx.bundle.funcfl_potential(text), unit_style="metal",
                       force_output="atom-force", newton="on", cutoff=1.5))
    t = b.eam_tables()
    ref = oracle.load_funcfl(tmp_path / "tiny.eam")
    for key in ("embedding", "density", "pair"):
        np.testing.assert_array_equal(t[key], ref[key])


def test_engine_rejects_bundle_without_potential(ljx):
    d = base(ljx)
    d.pop("potential")
    b = load(ljx, d)
    with pytest.raises(ljx.LjxError, match="no potential block"):
        ljx.Engine(b)


def test_missing_file_message(ljx, tmp_path):
    with pytest.raises(ljx.LjxError, match="Could not open model bundle"):
        ljx.Bundle.load(tmp_path / "absent.json")
