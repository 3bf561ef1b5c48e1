"""TEST INFRASTRUCTURE ONLY — numpy/ctypes front end of the C oracle
(`l3d_oracle.c`), the CPU restatement of the reference's per-token layer ops.

Only the tests, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline /
reference arm may import this module; the product path never does.

All functions take and return float32 numpy arrays (C-contiguous).  For
reduced-precision activations pass `rnd=1` (bf16) / `rnd=2` (f16) to round
every intermediate op output the way Candle materialises each op, or keep
`rnd=0` and round only the final result (see `round_to`).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "l3d_oracle.c"
BUILD = HERE / "_build"
LIB = BUILD / "libl3d_oracle.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i64 = C.c_int64
_int = C.c_int
_flt = C.c_float


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc (OpenMP, no FMA contraction: the restatement
    keeps the reference's separate multiply/add roundings)."""
    BUILD.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        cmd = ["gcc", "-O3", "-std=gnu11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
               "-march=x86-64-v2", str(SRC), "-o", str(LIB), "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()  # compiles only when the library is missing or older than the source
        L = C.CDLL(str(LIB))
        sig = {
            "orc_round_array": [_f32p, _i64, _int],
            "orc_sparse_conv3d": [C.c_void_p, _i64, _f32p, _i64, _f32p, _i64, C.c_void_p, _f32p],
            "orc_num_threads": [],
            "orc_set_num_threads": [_int],
            "orc_layer_norm": [_f32p, _i64, _i64, C.c_void_p, C.c_void_p, _flt, _f32p, _int],
            "orc_layer_norm_modulate": [_f32p, _i64, _i64, _i64, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_void_p, _int, _flt, _f32p,
                                        _int],
            "orc_gated_residual": [_f32p, _f32p, C.c_void_p, _i64, _i64, _i64, _f32p, _int],
            "orc_rms_norm_heads": [_f32p, _i64, _i64, C.c_void_p, _flt, _f32p, _int],
            "orc_rope2d_tables": [_i64p, _i64, _i64, _flt, _int, _f32p, _f32p],
            "orc_layernorm_rope2d": [_f32p, _i64, _i64, _i64, _i64, C.c_void_p, C.c_void_p,
                                     _flt, _f32p, _f32p, _f32p, _int],
            "orc_rope3d_tables": [_i64p, _i64, _int, _flt, _f32p, _f32p],
            "orc_rope3d_apply": [_f32p, _i64, _i64, _i64, _i64, _f32p, _f32p, _f32p, _int],
            "orc_qk_l2norm_rope3d": [_f32p, _i64, _i64, _i64, _i64, C.c_void_p, C.c_void_p,
                                     _flt, _f32p, _int],
            "orc_activation": [_f32p, _i64, _int, _f32p, _int],
            "orc_geglu": [_f32p, _i64, _i64, _f32p, _int],
            "orc_timestep_embedding": [_f32p, _i64, _int, _int, _flt, _f32p, _int],
            "orc_linear": [_f32p, _i64, _i64, _f32p, _i64, C.c_void_p, C.c_void_p, _int, _int,
                           _f32p],
            "orc_patch_embed": [_f32p, _i64, _i64, _i64, _i64, _f32p, _f32p, _f32p, _f32p,
                                C.c_void_p, _i64, _int, _i64, _f32p],
            "orc_dequantize": [_u8p, _int, _i64, _i64, _f32p],
            "orc_quantize": [_f32p, _int, _i64, _i64, _u8p],
            "orc_neighbor_pairs": [_i32p, _i64, _i32p, _i32p, _i32p],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _int
        _lib = L
    return _lib


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def _opt(a):
    """Optional float32 array -> (keepalive, void pointer or None)."""
    if a is None:
        return None, None
    a = _c(a)
    return a, a.ctypes.data_as(C.c_void_p)


def _chk(rc, name):
    if rc != 0:
        raise RuntimeError(f"oracle {name} failed ({rc})")


def num_threads() -> int:
    return lib().orc_num_threads()


def use_all_host_threads() -> int:
    """Run the oracle on every core this process may use; returns the count."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    lib().orc_set_num_threads(n)
    return num_threads()


# ----------------------------------------------------------------- rounding
def round_bf16(a: np.ndarray, inplace: bool = False) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even), kept as f32;
    `inplace` rounds a C-contiguous float32 array in place."""
    if not (inplace and isinstance(a, np.ndarray) and a.dtype == np.float32
            and a.flags.c_contiguous):
        a = np.array(a, dtype=np.float32, copy=True)
    lib().orc_round_array(a, a.size, 1)
    return a


def round_f16(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    return round_bf16(a) if dtype == "bf16" else round_f16(a) if dtype == "f16" else _c(a)


# ---------------------------------------------------------------- LN family
def layer_norm(x, w=None, b=None, eps=1e-5, rnd=0):
    x = _c(x)
    C_ = x.shape[-1]
    y = np.empty_like(x)
    w_, wp = _opt(w)
    b_, bp = _opt(b)
    _chk(lib().orc_layer_norm(x, x.size // C_, C_, wp, bp, eps, y, rnd), "layer_norm")
    return y


def layer_norm_modulate(x, w=None, b=None, shift=None, scale=None, gate=None, add_input=False,
                        eps=1e-6, rnd=0):
    """x: [B, N, C]; shift/scale/gate: [B, C] or [C]."""
    x = _c(x)
    B = x.shape[0] if x.ndim >= 3 else 1
    C_ = x.shape[-1]
    rows = x.size // C_

    def per_batch(v):
        if v is None:
            return None
        v = _c(v).reshape(-1, C_)
        return np.broadcast_to(v, (B, C_)).copy() if v.shape[0] == 1 else v

    keep = [_opt(per_batch(v)) for v in (shift, scale, gate)]
    w_, wp = _opt(w)
    b_, bp = _opt(b)
    y = np.empty_like(x)
    _chk(lib().orc_layer_norm_modulate(x, rows, C_, rows // B, wp, bp, keep[0][1], keep[1][1],
                                       keep[2][1], int(bool(add_input)), eps, y, rnd), "lnm")
    return y


def gated_residual(x, h, gate, rnd=0):
    """out = x + gate * h; gate [B, C] (per batch of x [B, N, C]) or [C]."""
    x = _c(x)
    h = _c(h)
    C_ = x.shape[-1]
    rows = x.size // C_
    g = _c(gate).reshape(-1, C_)
    B = g.shape[0]
    out = np.empty_like(x)
    _, gp = _opt(g)
    _chk(lib().orc_gated_residual(x, h, gp, rows, C_, rows // B, out, rnd), "gated_residual")
    return out


def layerscale_residual(x, h, gamma, rnd=0):
    return gated_residual(x, h, _c(gamma).reshape(1, -1), rnd)


def rms_norm_heads(x, w=None, eps=1e-6, rnd=0):
    x = _c(x)
    D = x.shape[-1]
    y = np.empty_like(x)
    w_, wp = _opt(w)
    _chk(lib().orc_rms_norm_heads(x, x.size // D, D, wp, eps, y, rnd), "rms_norm_heads")
    return y


# -------------------------------------------------------------------- RoPE
def rope2d_tables(positions, theta=100.0, head_dim=64):
    """positions [B, N, 2] -> (cos_full, sin_alt_full) [B, N, head_dim]."""
    p = _c(positions, np.int64)
    B, N, _ = p.shape
    c = np.empty((B, N, head_dim), np.float32)
    s = np.empty_like(c)
    _chk(lib().orc_rope2d_tables(p, B, N, theta, head_dim, c, s), "rope2d_tables")
    return c, s


def layernorm_rope2d(x, w, b, eps, cos_full, sin_alt_full, rnd=0):
    """x [B, H, N, D] contiguous (a copy of the strided view); tables [B, N, D]."""
    x = _c(x)
    B, H, N, D = x.shape
    out = np.empty_like(x)
    w_, wp = _opt(w)
    b_, bp = _opt(b)
    cf = _c(cos_full).reshape(-1, N, D)
    sf = _c(sin_alt_full).reshape(-1, N, D)
    if cf.shape[0] == 1 and B > 1:
        cf = np.broadcast_to(cf, (B, N, D)).copy()
        sf = np.broadcast_to(sf, (B, N, D)).copy()
    _chk(lib().orc_layernorm_rope2d(x, B, H, N, D, wp, bp, eps, cf, sf, out, rnd), "ln_rope2d")
    return out


def rope3d_tables(coords, head_dim=128, theta=10000.0):
    c = _c(coords, np.int64)
    L = c.shape[0]
    cs = np.empty((L, head_dim // 2), np.float32)
    sn = np.empty_like(cs)
    _chk(lib().orc_rope3d_tables(c, L, head_dim, theta, cs, sn), "rope3d_tables")
    return cs, sn


def rope3d_apply(x, cos, sin, rnd=0):
    x = _c(x)
    B, L, H, D = x.shape
    y = np.empty_like(x)
    _chk(lib().orc_rope3d_apply(x, B, L, H, D, _c(cos), _c(sin), y, rnd), "rope3d_apply")
    return y


def qk_l2norm_rope3d(x, gamma, coords, theta=10000.0, rnd=0):
    """x [B, L, H, D]; gamma [H, D] or None; coords [L, 3] or None (norm only)."""
    x = _c(x)
    B, L, H, D = x.shape
    y = np.empty_like(x)
    g_, gp = _opt(gamma)
    c_ = None if coords is None else _c(coords, np.int64)
    cp = None if c_ is None else c_.ctypes.data_as(C.c_void_p)
    _chk(lib().orc_qk_l2norm_rope3d(x, B, L, H, D, gp, cp, theta, y, rnd), "qk_l2norm_rope3d")
    return y


# ------------------------------------------------------------- activations
ACT = {"none": 0, "silu": 1, "gelu_erf": 2, "gelu_tanh": 3}


def activation(x, kind, rnd=0):
    x = _c(x)
    y = np.empty_like(x)
    _chk(lib().orc_activation(x, x.size, ACT[kind], y, rnd), kind)
    return y


def gelu_tanh(x, rnd=0):
    return activation(x, "gelu_tanh", rnd)


def gelu_erf(x, rnd=0):
    return activation(x, "gelu_erf", rnd)


def silu(x, rnd=0):
    return activation(x, "silu", rnd)


def geglu(x, rnd=0):
    x = _c(x)
    F = x.shape[-1] // 2
    y = np.empty(x.shape[:-1] + (F,), np.float32)
    _chk(lib().orc_geglu(x, x.size // (2 * F), F, y, rnd), "geglu")
    return y


# --------------------------------------------------------- timestep, linear
def timestep_embedding(t, dim, order, max_period=10000.0, rnd=0):
    t = _c(np.atleast_1d(t))
    out = np.empty((t.size, dim), np.float32)
    _chk(lib().orc_timestep_embedding(t, t.size, dim, order, max_period, out, rnd), "timestep")
    return out


def linear(x, w, bias=None, addend=None, act_in="none", act_out="none"):
    x = _c(x)
    w = _c(w)
    B, K = x.shape
    N = w.shape[0]
    y = np.empty((B, N), np.float32)
    b_, bp = _opt(bias)
    a_, ap = _opt(addend)
    _chk(lib().orc_linear(x, B, K, w, N, bp, ap, ACT[act_in], ACT[act_out], y), "linear")
    return y


def patch_embed(pixels, weight, bias, pos, cls, reg, patch):
    pix = _c(pixels)
    BS, Cin, H, W = pix.shape
    Cc = weight.shape[0]
    R_ = 0 if reg is None else reg.shape[0]
    np_ = (H // patch) * (W // patch)
    out = np.empty((BS, 1 + R_ + np_, Cc), np.float32)
    r_, rp = _opt(reg)
    _chk(lib().orc_patch_embed(pix, BS, Cin, H, W, _c(weight), _c(bias), _c(pos), _c(cls), rp,
                               R_, patch, Cc, out), "patch_embed")
    return out


# ---------------------------------------------------------------- GGML blocks
QFMT = {"q8_0": 8, "q4_0": 2, "q4_k": 12, "q5_k": 13, "q6_k": 14}
BLOCK_BYTES = {"q8_0": 34, "q4_0": 18, "q4_k": 144, "q5_k": 176, "q6_k": 210}
BLOCK_ELEMS = {"q8_0": 32, "q4_0": 32, "q4_k": 256, "q5_k": 256, "q6_k": 256}


def quantize(w, fmt):
    w = _c(w)
    n, k = w.shape
    out = np.empty(n * (k // 32) * BLOCK_BYTES[fmt], np.uint8)
    _chk(lib().orc_quantize(w, QFMT[fmt], n, k, out), "quantize")
    return out


def dequantize(wq, fmt, n, k):
    out = np.empty((n, k), np.float32)
    _chk(lib().orc_dequantize(_c(wq, np.uint8), QFMT[fmt], n, k, out), "dequantize")
    return out


# ------------------------------------------------------------------- sparse
def neighbor_pairs(coords):
    c = _c(coords, np.int32)
    n = c.shape[0]
    dest = np.full((27, n), -1, np.int32)
    src = np.full((27, n), -1, np.int32)
    counts = np.zeros(27, np.int32)
    _chk(lib().orc_neighbor_pairs(c, n, dest, src, counts), "neighbor_pairs")
    return dest, src, counts


def kernel_offset_delta(k: int):
    """crate/runtime/trellis2_sparse.rs:99-106."""
    return (k // 9 - 1, (k % 9) // 3 - 1, k % 3 - 1)


def sparse_conv3d(coords, feats, w27, bias=None):
    """SparseConv3d::forward in f32: coords [N, 3] int, feats [N, Cin],
    w27 [27, Cout, Cin], bias [Cout] or None -> [N, Cout]."""
    c = _c(coords, np.int32)
    f = _c(feats)
    w = _c(w27)
    n, cin = f.shape
    cout = w.shape[1]
    b = None if bias is None else _c(bias)
    out = np.empty((n, cout), np.float32)
    _chk(lib().orc_sparse_conv3d(c.ctypes.data, n, f, cin, w, cout,
                                 None if b is None else b.ctypes.data, out), "sparse_conv3d")
    return out


if __name__ == "__main__":
    build(force=True)
    print("built", LIB, "threads", num_threads())
