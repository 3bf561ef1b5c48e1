"""ctypes binding of libl3dops.so (the C ABI declared in include/l3d_ops.h).

Tensors cross the boundary as `l3d_tensor` descriptors built from torch
tensors: storage base pointer + Candle-style layout (dims, element strides,
start offset).  torch is used only for device memory and the current stream.

The library is required: importing this module on a machine without the built
`libl3dops.so` raises, and there is no CPU fallback anywhere in the package.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libl3dops.so"
HEADER = PKG.parent / "include" / "l3d_ops.h"

MAX_DIMS = 6
F32, F16, BF16, I32, I64, U32, U8 = 0, 1, 2, 3, 4, 5, 6
Q8_0, Q4_0, Q4_K, Q5_K, Q6_K = 8, 2, 12, 13, 14
STATUS = {0: "OK", 1: "E_SHAPE", 2: "E_DTYPE", 3: "E_ALIGN", 4: "E_UNSUPPORTED", 5: "E_CUDA",
          6: "E_NULL", 7: "E_WORKSPACE", 8: "E_DEVICE"}

_TORCH_TO_L3D = {
    torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int32: I32,
    torch.int64: I64, torch.uint32: U32, torch.uint8: U8,
}


class L3dTensor(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("dtype", C.c_int32),
        ("ndim", C.c_int32),
        ("dims", C.c_int64 * MAX_DIMS),
        ("strides", C.c_int64 * MAX_DIMS),
        ("offset", C.c_int64),
    ]


class L3dError(RuntimeError):
    def __init__(self, status: int, op: str, msg: str):
        super().__init__(f"{op} failed: {STATUS.get(status, status)}: {msg}")
        self.status = status
        self.op = op


def desc(t: torch.Tensor | None):
    """Descriptor for a tensor view (None -> NULL)."""
    if t is None:
        return None
    if t.dim() > MAX_DIMS:
        raise ValueError(f"rank {t.dim()} exceeds {MAX_DIMS}")
    d = L3dTensor()
    d.data = t.untyped_storage().data_ptr() if t.numel() else t.data_ptr()
    d.dtype = _TORCH_TO_L3D[t.dtype]
    d.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        d.dims[i] = s
        d.strides[i] = st
    d.offset = t.storage_offset() if t.numel() else 0
    return d


def ref(d):
    return None if d is None else C.byref(d)


_P = C.POINTER(L3dTensor)
_S = C.c_void_p
_SIGS = {
    "l3d_abi_version": ([], C.c_int),
    "l3d_last_error": ([], C.c_char_p),
    "l3d_layer_norm": ([_P, _P, _P, C.c_float, _P, _S], C.c_int),
    "l3d_layer_norm_modulate": ([_P, _P, _P, _P, _P, _P, C.c_int, C.c_float, _P, _S], C.c_int),
    "l3d_gated_residual": ([_P, _P, _P, _P, _S], C.c_int),
    "l3d_layerscale_residual": ([_P, _P, _P, _P, _S], C.c_int),
    "l3d_residual_layer_norm_modulate": ([_P, _P, _P, _P, _P, _P, _P, C.c_float, _P, _P, _S],
                                         C.c_int),
    "l3d_layernorm_rope2d": ([_P, _P, _P, C.c_float, _P, _P, _P, _S], C.c_int),
    "l3d_qk_layernorm_rope2d_pos": ([_P, _P, _P, _P, _P, _P, C.c_float, _P, C.c_float, _P, _P,
                                     _S], C.c_int),
    "l3d_rope2d_tables": ([_P, C.c_float, C.c_int, _P, _P, _S], C.c_int),
    "l3d_rms_norm_heads": ([_P, _P, C.c_float, _P, _S], C.c_int),
    "l3d_qk_l2norm_rope3d": ([_P, _P, _P, C.c_float, _P, _S], C.c_int),
    "l3d_rope3d_tables": ([_P, C.c_int, C.c_float, _P, _P, _S], C.c_int),
    "l3d_rope3d_apply": ([_P, _P, _P, _P, _S], C.c_int),
    "l3d_gelu_tanh": ([_P, _P, _S], C.c_int),
    "l3d_gelu_erf": ([_P, _P, _S], C.c_int),
    "l3d_silu": ([_P, _P, _S], C.c_int),
    "l3d_geglu": ([_P, _P, _S], C.c_int),
    "l3d_timestep_embedding": ([_P, C.c_int, C.c_int, C.c_float, _P, _S], C.c_int),
    "l3d_linear_small": ([_P, _P, _P, _P, C.c_int, C.c_int, _P, _S], C.c_int),
    "l3d_patch_embed": ([_P, _P, _P, _P, _P, _P, C.c_int, _P, _S], C.c_int),
    "l3d_dequantize": ([C.c_void_p, C.c_int, C.c_int64, C.c_int64, _P, _S], C.c_int),
    "l3d_dequant_linear_workspace_size": ([C.c_int, C.c_int64, C.c_int64, C.c_int64], C.c_size_t),
    "l3d_dequant_linear": ([_P, C.c_void_p, C.c_int, C.c_int64, C.c_int64, _P, _P, C.c_void_p,
                            C.c_size_t, _S], C.c_int),
    "l3d_dequant_linear_ex": ([_P, C.c_void_p, C.c_int, C.c_int64, C.c_int64, _P, C.c_int, _P, _P,
                               _P, C.c_void_p, C.c_size_t, _S], C.c_int),
    "l3d_linear_workspace_size": ([C.c_int64, C.c_int64, C.c_int64], C.c_size_t),
    "l3d_linear_ex": ([_P, _P, _P, C.c_int, _P, _P, _P, C.c_void_p, C.c_size_t, _S], C.c_int),
    "l3d_sparse_neighbor_pairs_workspace_size": ([C.c_int64], C.c_size_t),
    "l3d_sparse_neighbor_pairs": ([_P, _P, _P, _P, C.c_void_p, C.c_size_t, _S], C.c_int),
    "l3d_sparse_neighbor_pairs_noalloc": ([_P, _P, _P, _P, _S], C.c_int),
    "l3d_index_select_rows": ([_P, _P, _P, _S], C.c_int),
    "l3d_sparse_neighbor_map": ([_P, _P, C.c_void_p, C.c_size_t, _S], C.c_int),
    "l3d_sparse_conv3d_workspace_size": ([C.c_int64, C.c_int64, C.c_int], C.c_size_t),
    "l3d_sparse_conv3d": ([_P, _P, _P, _P, _P, C.c_void_p, C.c_size_t, _S], C.c_int),
    "l3d_sparse_conv3d_pairs_workspace_size": ([C.c_int64, C.c_int64, C.c_int64, C.c_void_p],
                                               C.c_size_t),
    "l3d_sparse_conv3d_pairs": ([_P, _P, _P, _P, C.c_void_p, _P, _P, _P, C.c_void_p, C.c_size_t,
                                 _S], C.c_int),
    "l3d_attention_workspace_size": ([C.c_int64, C.c_int64, C.c_int64, C.c_int64], C.c_size_t),
    "l3d_kernel_status": ([C.POINTER(C.c_int), C.c_int], C.c_int),
    "l3d_activation_scatter": ([C.c_int, _P, _P, C.c_int, _S], C.c_int),
    "l3d_attention": ([_P, _P, _P, C.c_float, _P, C.c_void_p, C.c_size_t, _S], C.c_int),
    "l3d_attention_selftest_timeout": ([_P, _P, _P, C.c_float, _P, C.c_void_p, C.c_size_t,
                                        C.c_uint32, _S], C.c_int),
    "l3d_gguf_index": ([C.c_void_p, C.c_uint64, C.c_void_p, C.c_int64, C.POINTER(C.c_int64),
                        C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)], C.c_int),
    "l3d_gguf_metadata_string": ([C.c_void_p, C.c_uint64, C.c_char_p, C.POINTER(C.c_void_p),
                                  C.POINTER(C.c_uint64)], C.c_int),
}


class GgufTensorInfo(C.Structure):
    """l3d_gguf_tensor (include/l3d_ops.h)."""
    _fields_ = [
        ("name", C.c_void_p),
        ("name_len", C.c_uint64),
        ("type", C.c_int32),
        ("n_dims", C.c_int32),
        ("dims", C.c_int64 * 4),
        ("offset", C.c_uint64),
        ("nbytes", C.c_uint64),
    ]

_lib = None


def lib():
    """Load libl3dops.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python candle-3d_b200/build.py`"
                               " (there is no fallback implementation)")
        L = C.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def call(name: str, *args):
    """Invoke an entry point and raise L3dError on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise L3dError(rc, name, lib().l3d_last_error().decode())
    return rc


def declared_symbols() -> list[str]:
    """Every function name declared in include/l3d_ops.h."""
    import re

    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(l3d_\w+)\s*\(", text, re.M)))
