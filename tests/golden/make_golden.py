"""Writes reference_kats.json: the known-answer cases of the reference's own
tests for this path, with the inputs each test feeds and the expected values
each test asserts (evaluated here in float32 from the formulas the tests state,
since the reference is Rust and cannot run in this environment).

Sources (crates/lux3d-core/tests/...):
  trellis2_blocks.rs:43-73    rope_tables_match_reference_formula      tol 1e-6
  trellis2_blocks.rs:78-111   rope_apply_matches_complex_product...    tol 1e-5 (+ norm 1e-4)
  trellis2_blocks.rs:115-123  cubic_token_coords_are_row_major_ij...   exact
  trellis2_blocks.rs:126-153  qk_rms_norm_matches_reference            tol 1e-6
  trellis2_blocks.rs:157-171  timestep_embedding_matches_reference     tol 1e-5
  trellis2_blocks.rs:204-225  ada_ln_modulation_chunks_in_reference... exact
  trellis2_sparse.rs:68-78    coord_map_builds_and_looks_up            exact
  trellis2_sparse.rs:80-96    kernel_offset_deltas_cover_the_3x3x3...  exact
Run: python tests/golden/make_golden.py
"""
import json
from pathlib import Path

import numpy as np

f32 = np.float32


def rope_tables():
    coords = [[1, 0, 0], [0, 1, 0]]
    freq2 = f32(1.0) / np.power(f32(10000.0), f32(0.5), dtype=f32)
    cos, sin = [], []
    for c in coords:
        ang = [f32(c[0]) * f32(1), f32(c[0]) * freq2, f32(c[1]) * f32(1), f32(c[1]) * freq2,
               f32(c[2]) * f32(1), f32(c[2]) * freq2]
        cos.append([float(np.cos(f32(a))) for a in ang])
        sin.append([float(np.sin(f32(a))) for a in ang])
    return {"source": "crates/lux3d-core/tests/trellis2_blocks.rs:43-73", "head_dim": 12,
            "coords": coords, "cos": cos, "sin": sin, "tol": 1e-6}


def rope_apply():
    x = [1.0, 0.0, 2.0, 3.0, 5.0, 0.0, 7.0, 1.0, 0.0, 2.0, 4.0, 4.0]
    freq2 = f32(1.0) / np.power(f32(10000.0), f32(0.5), dtype=f32)
    phases = [(f32(1), f32(1)), (freq2, freq2)]
    out = []
    for p in range(6):
        c, s = (np.cos(phases[p][0]), np.sin(phases[p][1])) if p < 2 else (f32(1), f32(0))
        re, im = f32(x[2 * p]), f32(x[2 * p + 1])
        out += [float(re * c - im * s), float(re * s + im * c)]
    return {"source": "crates/lux3d-core/tests/trellis2_blocks.rs:78-111", "head_dim": 12,
            "coords": [[1, 0, 0]], "x": x, "expected": out, "tol": 1e-5, "norm_tol": 1e-4}


def cubic_coords():
    return {"source": "crates/lux3d-core/tests/trellis2_blocks.rs:115-123", "resolution": 3,
            "len": 81, "index_x1_y2_z0": 1 * 9 + 2 * 3 + 0, "coord_at_index": [1, 2, 0],
            "last": [2, 2, 2]}


def qk_rms_norm():
    return {"source": "crates/lux3d-core/tests/trellis2_blocks.rs:126-153",
            "x": [3.0, 4.0, 0.0, 0.0],
            "cases": [{"gamma": 1.0, "expected": [0.6 * 2.0, 0.8 * 2.0, 0.0, 0.0]},
                      {"gamma": 2.0, "expected": [2.4, 3.2, 0.0, 0.0]}], "tol": 1e-6}


def timestep():
    freq1 = f32(np.exp(-np.log(10000.0) / 2.0))
    t = f32(500.0)
    exp = [np.cos(t), np.cos(t * freq1), np.sin(t), np.sin(t * freq1)]
    return {"source": "crates/lux3d-core/tests/trellis2_blocks.rs:157-171", "t": 500.0, "dim": 4,
            "expected": [float(v) for v in exp], "tol": 1e-5}


def ada_chunks():
    return {"source": "crates/lux3d-core/tests/trellis2_blocks.rs:204-225",
            "mod_vec": [float(v) for v in range(1, 13)],
            "expected": [[1, 2], [3, 4], [5, 6], [7, 8], [9, 10], [11, 12]]}


def coord_map():
    return {"source": "crates/lux3d-core/tests/trellis2_sparse.rs:68-78",
            "coords": [[0, 0, 0], [1, 0, 3], [7, 2, 5]],
            "lookups": [[[1, 0, 3], 1], [[7, 2, 5], 2], [[9, 9, 9], None]]}


def offsets():
    return {"source": "crates/lux3d-core/tests/trellis2_sparse.rs:80-96",
            "cases": [[0, [-1, -1, -1]], [13, [0, 0, 0]], [26, [1, 1, 1]], [5, [-1, 0, 1]]]}


def main():
    out = {"rope_tables": rope_tables(), "rope_apply": rope_apply(), "cubic_coords": cubic_coords(),
           "qk_rms_norm": qk_rms_norm(), "timestep": timestep(), "ada_chunks": ada_chunks(),
           "coord_map": coord_map(), "offsets": offsets()}
    path = Path(__file__).with_name("reference_kats.json")
    path.write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", path)


if __name__ == "__main__":
    main()
