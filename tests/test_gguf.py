"""GGUF tensor index through the C ABI (host code: runs without a GPU).

The files are written here from the public GGUF v3 layout (little-endian:
magic, version, tensor count, metadata count, key/values, tensor infos with
dims fastest-first, data section aligned to general.alignment), with the
metadata keys the reference's quantizer writes (crate/weights/quantize.rs:
255-283: general.architecture, lux3d.family, lux3d.resolved_config, ...).
"""
import struct

import numpy as np
import pytest

from conftest import random_kquant_blocks, rng

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    if t == STRING:
        return _s(v.encode())
    if t == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    fmt = {U8: "B", I8: "b", U16: "H", I16: "h", U32: "I", I32: "i", F32: "f", BOOL: "?",
           U64: "Q", I64: "q", F64: "d"}[t]
    return struct.pack("<" + fmt, v)


def write_gguf(path, metadata, tensors, alignment=32, version=3):
    """metadata: [(key, type, value)]; tensors: [(name, ggml_type, dims_row_major, bytes)]."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, t, v in metadata:
        out += _s(key.encode()) + struct.pack("<I", t) + _value(t, v)
    offsets, off = [], 0
    for _, _, _, data in tensors:
        offsets.append(off)
        off += (len(data) + alignment - 1) // alignment * alignment
    for (name, ty, dims, _), o in zip(tensors, offsets):
        ne = list(reversed(dims))
        out += _s(name.encode()) + struct.pack("<I", len(ne))
        out += b"".join(struct.pack("<Q", d) for d in ne) + struct.pack("<IQ", ty, o)
    out += b"\0" * ((-len(out)) % alignment)
    data_start = len(out)
    for (_, _, _, data), o in zip(tensors, offsets):
        out += b"\0" * (data_start + o - len(out)) + data
    path.write_bytes(bytes(out))
    return data_start, offsets


@pytest.fixture
def sample(tmp_path, orc):
    r = rng(900)
    w = (r.standard_normal((64, 256)) * 0.05).astype(np.float32)
    q8 = orc.quantize(w, "q8_0").tobytes()
    q4k = random_kquant_blocks(r, "q4_k", 32, 512).tobytes()
    bias = r.standard_normal(64).astype(np.float32).tobytes()
    norm = r.standard_normal(256).astype(np.float16).tobytes()
    tbl = r.standard_normal((3, 5)).astype(np.float32)
    tensors = [
        ("blocks.0.attn.to_qkv.weight", 8, (64, 256), q8),
        ("blocks.0.attn.to_qkv.bias", 0, (64,), bias),
        ("blocks.0.mlp.0.weight", 12, (32, 512), q4k),
        ("blocks.0.norm.weight", 1, (256,), norm),
        ("blocks.0.table", 0, (3, 5), tbl.tobytes()),
        ("blocks.0.proj.weight", 1, (16, 256), r.standard_normal((16, 256)).astype(np.float16).tobytes()),
    ]
    meta = [
        ("general.architecture", STRING, "trellis2"),
        ("general.alignment", U32, 64),
        ("lux3d.family", STRING, "trellis2"),
        ("lux3d.quantization.dtype", STRING, "q8_0"),
        ("lux3d.tensor_count", U32, 6),
        ("some.array", ARRAY, (I32, [1, -2, 3])),
        ("some.strings", ARRAY, (STRING, ["a", "bc"])),
        ("some.flag", BOOL, True),
        ("some.f64", F64, 0.5),
        ("lux3d.resolved_config", STRING, '{"width": 1536}'),
    ]
    path = tmp_path / "model.gguf"
    data_start, offsets = write_gguf(path, meta, tensors, alignment=64)
    return path, tensors, data_start, offsets


def test_gguf_index_reads_tensors_and_metadata(pkg, sample):
    path, tensors, data_start, offsets = sample
    g = pkg.gguf.GgufFile(path)
    assert g.version == 3 and g.alignment == 64
    assert list(g.tensors) == [t[0] for t in tensors]
    for (name, ty, dims, data), o in zip(tensors, offsets):
        t = g.tensors[name]
        assert t.type == ty and t.dims == dims
        assert t.offset == data_start + o and t.offset % 64 == 0
        assert t.nbytes == len(data)
        assert g.raw(name).tobytes() == data
    assert g.metadata_string("general.architecture") == "trellis2"
    assert g.metadata_string("lux3d.family") == "trellis2"
    assert g.metadata_string("lux3d.resolved_config") == '{"width": 1536}'
    assert g.metadata_string("lux3d.tensor_count") is None  # not a string
    assert g.metadata_string("missing.key") is None


def test_gguf_rejects_bad_and_truncated_buffers(pkg, sample):
    import ctypes as C

    path, _, data_start, _ = sample
    blob = path.read_bytes()
    L = pkg._lib.lib()
    n = C.c_int64(0)

    def index(b):
        a = np.frombuffer(b, np.uint8)
        return L.l3d_gguf_index(a.ctypes.data, len(a), None, 0, C.byref(n), None, None)

    assert index(blob) == 0 and n.value == 6
    assert index(b"GGUX" + blob[4:]) != 0            # bad magic
    assert index(blob[:40]) != 0                      # truncated metadata
    assert index(blob[: data_start + 16]) != 0        # truncated data section
    bad_version = blob[:4] + struct.pack("<I", 9) + blob[8:]
    assert index(bad_version) != 0
    assert b"version" in L.l3d_last_error()


def test_gguf_partial_index_reports_full_count(pkg, sample):
    import ctypes as C

    path, tensors, _, _ = sample
    blob = np.frombuffer(path.read_bytes(), np.uint8)
    L = pkg._lib.lib()
    infos = (pkg._lib.GgufTensorInfo * 2)()
    n = C.c_int64(0)
    assert L.l3d_gguf_index(blob.ctypes.data, len(blob), infos, 2, C.byref(n), None, None) == 0
    assert n.value == len(tensors)
    assert C.string_at(infos[1].name, infos[1].name_len).decode() == tensors[1][0]


def test_gguf_blocks_decode_like_the_packed_source(pkg, orc, sample):
    """The Q8_0 / Q4_K bytes found through the index decode (oracle) to the
    same weights as the buffers they were written from."""
    path, tensors, _, _ = sample
    g = pkg.gguf.GgufFile(path)
    for name, fmt in (("blocks.0.attn.to_qkv.weight", "q8_0"), ("blocks.0.mlp.0.weight", "q4_k")):
        t = g.tensors[name]
        src = next(d for nm, _, _, d in tensors if nm == name)
        n, k = t.dims
        a = orc.dequantize(np.frombuffer(src, np.uint8), fmt, n, k)
        b = orc.dequantize(g.raw(name).copy(), fmt, n, k)
        assert np.array_equal(a, b)


@pytest.mark.gpu
def test_gguf_quantized_linear_runs_on_device(pkg, orc, dev, sample):
    """quantized_linear -> QMatMul over the file's Q8_0 blocks, against the
    oracle's decode of the same bytes."""
    import torch

    path, tensors, _, _ = sample
    g = pkg.gguf.GgufFile(path)
    mm = pkg.gguf.quantized_linear(g, "blocks.0.attn.to_qkv", 256, 64, dev)
    x = torch.randn(40, 256, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    y = mm(x.to(dev), out_dtype=torch.float32).cpu().numpy().astype(np.float64)
    w = orc.round_bf16(orc.dequantize(g.raw("blocks.0.attn.to_qkv.weight").copy(), "q8_0", 64, 256))
    bias = np.frombuffer(next(d for nm, _, _, d in tensors if nm.endswith("to_qkv.bias")), np.float32)
    xv = x.float().numpy().astype(np.float64)
    ref = xv @ w.astype(np.float64).T + bias
    bound = 2e-5 * (np.abs(xv) @ np.abs(w.astype(np.float64)).T) + 1e-6
    assert np.all(np.abs(y - ref) <= bound)
    with pytest.raises(ValueError):
        pkg.gguf.quantized_linear(g, "blocks.0.attn.to_qkv", 128, 64, dev)


def test_gguf_float_linear_stays_dense(pkg, sample):
    """F16 / F32 / BF16 weights take the dense path (nn_blocks.rs:136-145)."""
    import torch

    path, tensors, _, _ = sample
    g = pkg.gguf.GgufFile(path)
    w, b = pkg.gguf.quantized_linear(g, "blocks.0.proj", 256, 16, "cpu", dense_dtype=torch.float32)
    src = np.frombuffer(next(d for nm, _, _, d in tensors if nm == "blocks.0.proj.weight"), np.float16)
    assert b is None and w.shape == (16, 256)
    assert np.array_equal(w.numpy(), src.astype(np.float32).reshape(16, 256))
