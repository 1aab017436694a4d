"""The C ABI library loads without a GPU and exports every symbol include/*.h declares."""

import ctypes
import re

from conftest import ROOT


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        for match in re.finditer(r"^\s*(?:const\s+)?[\w ]+?\*?\s*\b(ljx_\w+)\s*\(", text, re.M):
            names.add(match.group(1))
    return names


def test_headers_declare_the_abi():
    names = declared_symbols()
    for required in ("ljx_bundle_load", "ljx_engine_create", "ljx_pack_atoms", "ljx_pack_edges",
                     "ljx_density", "ljx_embed", "ljx_force", "ljx_read_result",
                     "ljx_comm_pack_forward", "ljx_comm_unpack_reverse", "ljx_neigh_build"):
        assert required in names


def test_library_exports_every_declared_symbol(ljx):
    lib = ljx.load()
    names = declared_symbols()
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    # The binding table covers the same set, so Python never calls an undeclared entry.
    bound = {name for name, _, _ in ljx.abi.SIGNATURES}
    assert bound == names
    assert lib.ljx_version().decode().count(".") == 2


def test_build_recipe_targets_sm100a_only(ljx):
    assert ljx.build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "-lineinfo" in ljx.build.FLAGS


def test_loader_rejects_missing_library(ljx, tmp_path):
    import pytest
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ljx.abi.load(tmp_path / "absent.so")
    assert ctypes  # the binding is plain ctypes
