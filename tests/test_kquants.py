"""GGML K-quant super-blocks (Q4_K, Q5_K, Q6_K): the C oracle's decode
against an independent numpy restatement of the public block layouts, and a
hand-built known answer.  The reference loads these types through Candle's
GGUF reader (crate/weights/quantize.rs:355-393 names them); the decode order
is GGML's (d * sc, dmin * m, then w = d1 * q - m1; Q6_K w = (d * sc) * q)."""
import numpy as np
import pytest

from conftest import KQ_BYTES, random_kquant_blocks, rng


def _scale_min(s, j):
    """6-bit (scale, min) of sub-block j for every super-block; s [nsb, 12]."""
    s = s.astype(np.int32)
    if j < 4:
        return s[:, j] & 63, s[:, j + 4] & 63
    return ((s[:, j + 4] & 15) | ((s[:, j - 4] >> 6) << 4),
            (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4))


def _np_decode(blk, fmt):
    """[nsb, bytes] -> [nsb, 256] float32, vectorised over super-blocks."""
    f32 = np.float32
    out = np.empty((blk.shape[0], 256), f32)
    if fmt == "q6_k":
        ql, qh = blk[:, :128].astype(np.int32), blk[:, 128:192].astype(np.int32)
        sc = blk[:, 192:208].view(np.int8).astype(f32)
        d = blk[:, 208:210].copy().view(np.float16).astype(f32)[:, 0]
        for h in range(2):
            for g in range(4):
                lo_src = ql[:, 64 * h + 32 * (g & 1): 64 * h + 32 * (g & 1) + 32]
                nib = (lo_src & 15) if g < 2 else (lo_src >> 4)
                hi = (qh[:, 32 * h: 32 * h + 32] >> (2 * g)) & 3
                q = (nib | (hi << 4)) - 32
                for l in range(32):
                    s = sc[:, 8 * h + l // 16 + 2 * g]
                    out[:, 128 * h + 32 * g + l] = (d * s).astype(f32) * q[:, l].astype(f32)
        return out
    q5 = fmt == "q5_k"
    d = blk[:, 0:2].copy().view(np.float16).astype(f32)[:, 0]
    dmin = blk[:, 2:4].copy().view(np.float16).astype(f32)[:, 0]
    scales = blk[:, 4:16]
    qh = blk[:, 16:48].astype(np.int32)
    qs = blk[:, 48:176].astype(np.int32) if q5 else blk[:, 16:144].astype(np.int32)
    for c in range(4):
        for half in range(2):
            j = 2 * c + half
            sc, m = _scale_min(scales, j)
            d1 = (d * sc.astype(f32)).astype(f32)
            m1 = (dmin * m.astype(f32)).astype(f32)
            src = qs[:, 32 * c: 32 * c + 32]
            q = (src >> 4) if half else (src & 15)
            if q5:
                q = q + (((qh >> j) & 1) << 4)
            out[:, 64 * c + 32 * half: 64 * c + 32 * half + 32] = (
                (d1[:, None] * q.astype(f32)).astype(f32) - m1[:, None]).astype(f32)
    return out


@pytest.mark.parametrize("fmt", ["q4_k", "q5_k", "q6_k"])
def test_kquant_oracle_matches_numpy_restatement(orc, fmt):
    n, k = 24, 1024
    blk = random_kquant_blocks(rng(300 + len(fmt)), fmt, n, k)
    got = orc.dequantize(blk, fmt, n, k)
    ref = _np_decode(blk.reshape(-1, KQ_BYTES[fmt]), fmt).reshape(n, k)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_kquant_q4k_known_answer(orc):
    # d = 1, dmin = 0.5; sub-block j: scale j + 1, min j (6-bit packing of
    # get_scale_min_k4); every qs byte = 0x21 (low nibble 1, high nibble 2).
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.array([1.0], np.float16).view(np.uint8)
    blk[2:4] = np.array([0.5], np.float16).view(np.uint8)
    sc = [j + 1 for j in range(8)]
    mn = list(range(8))
    s = np.zeros(12, np.int32)
    for j in range(4):
        s[j] |= sc[j]
        s[j + 4] |= mn[j]
    for j in range(4, 8):
        s[j + 4] |= (sc[j] & 15) | ((mn[j] & 15) << 4)
        s[j - 4] |= (sc[j] >> 4) << 6
        s[j] |= (mn[j] >> 4) << 6
    blk[4:16] = s.astype(np.uint8)
    blk[16:144] = 0x21
    w = orc.dequantize(blk, "q4_k", 1, 256)[0]
    for c in range(4):
        for half in range(2):
            j = 2 * c + half
            q = 2 if half else 1
            expect = np.float32(sc[j]) * q - np.float32(0.5) * mn[j]
            assert np.all(w[64 * c + 32 * half: 64 * c + 32 * half + 32] == expect), (j, w[64 * c])


def test_kquant_q6k_known_answer(orc):
    # d = 0.25; scales[i] = i - 8; ql bytes = 0x53, qh bytes = 0b11100100
    # (bit pairs 0, 1, 2, 3 for g = 0..3) -> q = (nibble | g << 4) - 32.
    blk = np.zeros(210, np.uint8)
    blk[0:128] = 0x53
    blk[128:192] = 0b11100100
    blk[192:208] = (np.arange(16) - 8).astype(np.int8).view(np.uint8)
    blk[208:210] = np.array([0.25], np.float16).view(np.uint8)
    w = orc.dequantize(blk, "q6_k", 1, 256)[0]
    for h in range(2):
        for g in range(4):
            nib = 3 if g < 2 else 5
            q = (nib | (g << 4)) - 32
            for l in (0, 15, 16, 31):
                sc = (8 * h + l // 16 + 2 * g) - 8
                assert w[128 * h + 32 * g + l] == np.float32(0.25) * sc * q
