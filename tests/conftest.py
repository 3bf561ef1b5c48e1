"""Shared test configuration: the `gpu` marker, package/oracle loading, the
seeded input generator and the parity tolerances.

Tolerances (from the build's parity contract):
  * F32: |gpu - oracle| <= 1e-5 * max(|oracle|, 1) elementwise;
  * BF16 / F16: |gpu - oracle| <= max(2e-2, 2^-8 * |oracle|), the oracle kept
    in f32 — 2e-2 max-abs, widened only where a single output rounding alone
    (half an ulp, 2^-9 relative) can exceed it (|values| >= 8);
  * integer / index outputs: bit-exact.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__ as graft  # noqa: E402

SEED = 20261201


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return graft.load_package()


@pytest.fixture(scope="session")
def ops(pkg):
    return pkg.ops


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def rng(tag: int = 0) -> np.random.Generator:
    return np.random.default_rng(SEED ^ tag)


TORCH_DT = {"f32": "float32", "bf16": "bfloat16", "f16": "float16"}


def to_dev(a: np.ndarray, dt: str, dev):
    """Upload a float32 array as dtype `dt`; returns (tensor, the f32 values it holds)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
    t = t.to(getattr(torch, TORCH_DT[dt]))
    return t, t.float().cpu().numpy()


def assert_close(got, ref, dt: str, what: str = ""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} != {ref.shape}"
    if not np.all(np.isfinite(got) == np.isfinite(ref)):
        raise AssertionError(f"{what}: non-finite mismatch")
    err = np.abs(got - ref)
    if dt == "f32":
        bound = 1e-5 * np.maximum(np.abs(ref), 1.0)
    else:
        bound = np.maximum(2e-2, np.abs(ref) * 2.0 ** -8)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what} [{dt}]: {bad.sum()} of {err.size} outside tolerance; worst at "
                             f"{i}: got {got[i]} ref {ref[i]} (err {err[i]:.3e})")


KQ_BYTES = {"q4_k": 144, "q5_k": 176, "q6_k": 210}


def random_kquant_blocks(r: np.random.Generator, fmt: str, n: int, k: int) -> np.ndarray:
    """Random GGML K-quant super-blocks for an [n, k] weight (k % 256 == 0):
    random quant bits, random 6-bit scales / mins (int8 scales in [-16, 16]
    for Q6_K) and f16 super-block scales d, dmin ~ U(1e-3, 1e-2)."""
    nsb = n * (k // 256)
    bb = KQ_BYTES[fmt]
    blk = r.integers(0, 256, size=(nsb, bb), dtype=np.uint8)
    d = r.uniform(1e-3, 1e-2, size=nsb).astype(np.float16).view(np.uint8).reshape(nsb, 2)
    if fmt == "q6_k":
        blk[:, 192:208] = r.integers(-16, 17, size=(nsb, 16)).astype(np.int8).view(np.uint8)
        blk[:, 208:210] = d
    else:
        dm = r.uniform(1e-3, 1e-2, size=nsb).astype(np.float16).view(np.uint8).reshape(nsb, 2)
        blk[:, 0:2] = d
        blk[:, 2:4] = dm
    return blk.reshape(-1)
