"""candle3d_b200 — B200-native (sm_100a) per-token layer ops of the Lux3D /
candle-3d models behind a C ABI (libl3dops.so, include/l3d_ops.h).

`ops` mirrors the Candle ops the reference model code calls; `_lib` is the
ctypes binding of the C ABI; `blocks` assembles the VGGT, TripoSG and
TRELLIS.2 block stacks from them; `gguf` indexes GGUF checkpoints for the
dequant-linear; `shard` splits token rows across ranks.
"""
from . import _lib, blocks, gguf, ops, shard  # noqa: F401

__all__ = ["ops", "blocks", "gguf", "shard", "_lib"]
