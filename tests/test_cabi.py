"""CPU: the C-ABI library loads, exports exactly the declared entry points,
and rejects invalid requests on the host before touching the device."""
import ctypes as C
import subprocess

import pytest


def test_exports_match_header(pkg):
    lib = pkg._lib.lib()
    declared = pkg._lib.declared_symbols()
    assert len(declared) >= 27
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(pkg._lib.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) == {s for s in exported if s.startswith("l3d_")}
    assert lib.l3d_abi_version() == 1


def test_null_requests_fail_on_host(pkg):
    lib = pkg._lib.lib()
    T = pkg._lib.L3dTensor
    x = T()  # data = NULL
    y = T()
    assert lib.l3d_layer_norm(C.byref(x), None, None, 1e-5, C.byref(y), None) == 6  # E_NULL
    assert b"null" in lib.l3d_last_error()
    assert lib.l3d_layer_norm(None, None, None, 1e-5, None, None) == 6
    assert lib.l3d_gelu_erf(C.byref(x), C.byref(y), None) == 6
    assert lib.l3d_dequantize(None, 8, 4, 32, None, None) == 6
    assert lib.l3d_sparse_neighbor_pairs(None, None, None, None, None, 0, None) == 6


def test_workspace_sizes(pkg):
    lib = pkg._lib.lib()
    assert lib.l3d_sparse_neighbor_pairs_workspace_size(31500) >= 2 * 31500 * 12
    assert lib.l3d_sparse_neighbor_pairs_workspace_size(-1) == 0
    assert lib.l3d_dequant_linear_workspace_size(8, 31500, 4608, 1536) >= 0


@pytest.mark.parametrize("fmt", [8, 2])
def test_block_bytes_contract(orc, fmt):
    import numpy as np

    w = np.zeros((2, 64), np.float32)
    q = orc.quantize(w, "q8_0" if fmt == 8 else "q4_0")
    assert q.size == 2 * 2 * (34 if fmt == 8 else 18)
