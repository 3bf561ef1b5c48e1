"""GGUF checkpoints for the dequant-linear (the reference's `model.gguf`).

The reference reads GGUF through Candle's `gguf_file::Content::read`
(crate/weights/mod.rs:596-650) and turns every rank-2 `*.weight` into either a
dense Linear (F32 / F16 / BF16 entries) or a `QMatMul` over the packed blocks
(`quantized_linear`, crate/runtime/nn_blocks.rs:123-152).  `GgufFile` indexes
a file through the C ABI (`l3d_gguf_index`, host code over an mmap of the
file) and `quantized_linear` mirrors that split: packed GGML blocks go to the
device unchanged and feed `ops.QMatMul`; float entries become dense weights.
"""
from __future__ import annotations

import ctypes as C
import mmap
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import _lib, ops

# GGML type ids of the formats the dequant-linear runs.
QTYPES = {8: "q8_0", 2: "q4_0", 12: "q4_k", 13: "q5_k", 14: "q6_k"}
FLOAT_TYPES = {0: torch.float32, 1: torch.float16, 30: torch.bfloat16}


@dataclass
class GgufTensor:
    name: str
    type: int
    dims: tuple
    offset: int
    nbytes: int


class GgufFile:
    """A GGUF file mapped read-only, with its tensor index and metadata."""

    def __init__(self, path):
        self.path = Path(path)
        self._f = open(self.path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.buf = np.frombuffer(self._mm, dtype=np.uint8)
        self._addr = self.buf.ctypes.data
        n = C.c_int64(0)
        ver = C.c_uint32(0)
        align = C.c_uint64(0)
        _lib.call("l3d_gguf_index", self._addr, len(self.buf), None, 0, C.byref(n), C.byref(ver),
                  C.byref(align))
        infos = (_lib.GgufTensorInfo * max(n.value, 1))()
        _lib.call("l3d_gguf_index", self._addr, len(self.buf), infos, n.value, C.byref(n),
                  C.byref(ver), C.byref(align))
        self.version, self.alignment = ver.value, align.value
        self.tensors = {}
        for i in range(n.value):
            t = infos[i]
            name = C.string_at(t.name, t.name_len).decode()
            self.tensors[name] = GgufTensor(name, t.type, tuple(t.dims[:t.n_dims]), t.offset,
                                            t.nbytes)

    def metadata_string(self, key: str):
        """String metadata value, or None when the key is absent."""
        v = C.c_void_p()
        n = C.c_uint64(0)
        rc = _lib.lib().l3d_gguf_metadata_string(self._addr, len(self.buf), key.encode(),
                                                 C.byref(v), C.byref(n))
        return None if rc != 0 else C.string_at(v.value, n.value).decode()

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes (a view of the mapping)."""
        t = self.tensors[name]
        if t.nbytes == 0:
            raise ValueError(f"{name}: GGML type {t.type} is not supported")
        return self.buf[t.offset:t.offset + t.nbytes]

    def dense(self, name: str, device, dtype=None) -> torch.Tensor:
        """A float entry (F32 / F16 / BF16) as a device tensor of its dims."""
        t = self.tensors[name]
        if t.type not in FLOAT_TYPES:
            raise ValueError(f"{name}: not a float tensor (GGML type {t.type})")
        host = torch.from_numpy(self.raw(name).copy()).view(FLOAT_TYPES[t.type]).reshape(t.dims)
        return host.to(device, dtype or host.dtype)

    def close(self):
        self.buf = None
        self._mm.close()
        self._f.close()


def quantized_linear(g: GgufFile, prefix: str, in_dim: int, out_dim: int, device,
                     dense_dtype=torch.bfloat16):
    """quantized_linear (crate/runtime/nn_blocks.rs:123-152) for `{prefix}.weight`
    (+ optional `{prefix}.bias`): an `ops.QMatMul` for packed GGML weights, or
    `(weight, bias)` dense tensors for F32 / F16 / BF16 entries."""
    t = g.tensors[f"{prefix}.weight"]
    if t.dims != (out_dim, in_dim):
        raise ValueError(f"quantized linear weight shape {t.dims} does not match expected "
                         f"({out_dim}, {in_dim})")
    bias = None
    if f"{prefix}.bias" in g.tensors:
        bias = g.dense(f"{prefix}.bias", device, torch.float32)
    if t.type in FLOAT_TYPES:
        return g.dense(f"{prefix}.weight", device, dense_dtype), bias
    if t.type not in QTYPES:
        raise ValueError(f"{prefix}.weight: GGML type {t.type} has no dequant-linear path")
    blocks = torch.from_numpy(g.raw(f"{prefix}.weight").copy()).to(device)
    return ops.QMatMul(blocks, QTYPES[t.type], out_dim, in_dim, bias=bias)
