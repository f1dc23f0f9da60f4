#!/usr/bin/env python3
"""Generate tests/golden/golden.npz from the reference shaders.

Runs the reference's own GLSL shaders, compiled as C++ by oracle/build_ref.py
(oracle/_ref/libvkref.so), on seeded synthetic blocks and on hand-built edge
blocks, and stores inputs and outputs.  The fixtures pin the C oracle
(oracle/oracle.c) and, through it, the CUDA kernels on machines where the
reference tree is absent (the GPU box).

Usage: python tests/golden/gen_golden.py   (needs oracle/_ref built here)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import pyoracle as po  # noqa: E402
from vkflame_b200 import synth as S  # noqa: E402


def edge_blocks(qtype: int) -> np.ndarray:
    """Hand-built blocks: all-zero codes, all-max codes, alternating codes,
    fp16 scales at the edges (0, smallest subnormal, largest normal below
    overflow of the products, negative)."""
    bb, qk = S.BLOCK_BYTES[qtype], S.BLOCK_VALUES[qtype]
    scales = np.array([0.0, 6e-8, 6.1e-5, 1.0, -0.5, 3.0e2], np.float16).view(np.uint8).reshape(-1, 2)
    fills = [0x00, 0xFF, 0x5A, 0x81]
    out = []
    for si in range(len(scales)):
        for f in fills:
            b = np.full(bb, f, np.uint8)
            if qtype in (S.Q4_0, S.Q5_0, S.Q8_0):
                b[0:2] = scales[si]
            elif qtype in (S.Q4_1, S.Q8_1):
                b[0:2] = scales[si]
                b[2:4] = scales[(si + 1) % len(scales)]
            elif qtype in (S.Q4_K, S.Q5_K):
                b[0:2] = scales[si]
                b[2:4] = scales[(si + 2) % len(scales)]
            elif qtype == S.Q6_K:
                b[208:210] = scales[si]
            out.append(b)
    return np.stack(out)


def main() -> int:
    if not po.ref_available():
        print("oracle/_ref/libvkref.so missing: run `python oracle/build_ref.py` first", file=sys.stderr)
        return 1
    data = {}
    for q in range(8):
        name = S.NAMES[q]
        # Seeded blocks: 3 rows x 512 values (several blocks per row).
        raw = S.quant_matrix(q, 3, 512, seed=100 + q).ravel()
        nb = raw.size // S.BLOCK_BYTES[q]
        data[f"dq_{name}_in"] = raw
        data[f"dq_{name}_out"] = po.ref_dequant(q, raw, nb)
        edge = edge_blocks(q).ravel()
        nbe = edge.size // S.BLOCK_BYTES[q]
        data[f"dqe_{name}_in"] = edge
        data[f"dqe_{name}_out"] = po.ref_dequant(q, edge, nbe)

    rng = np.random.default_rng(7)
    # linear_int8.glsl: fp16 A quantised in-shader, K not a multiple of 4 to
    # exercise its tail loop (linear_int8.glsl:84-90).
    M, N, K = 5, 19, 70
    a = (rng.standard_normal((M, K)) * 2).astype(np.float16)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    ws = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    data["i8_a"], data["i8_w"], data["i8_ws"] = a, w, ws
    for act in range(4):
        data[f"i8_out_act{act}"] = po.ref_linear_int8(a, w, ws, 0.03, act)
    # Small-magnitude case whose fp16 output equals the int32 accumulator exactly
    # (|acc| <= 2048, w_scale = 1, act_scale = 1): pins the accumulator itself.
    a2 = rng.integers(-3, 4, (4, 48)).astype(np.float16)
    w2 = rng.integers(-3, 4, (6, 48), dtype=np.int8)
    data["i8x_a"], data["i8x_w"] = a2, w2
    data["i8x_out"] = po.ref_linear_int8(a2, w2, np.ones(6, np.float32), 1.0, 0)

    # linear_fp16.glsl: A [MxK] x B [KxN].
    a3 = rng.standard_normal((3, 40)).astype(np.float16)
    b3 = rng.standard_normal((40, 24)).astype(np.float16)
    data["f16_a"], data["f16_b"] = a3, b3
    for act in range(4):
        data[f"f16_out_act{act}"] = po.ref_linear_fp16(a3, b3, act)

    # The non-matmul kernels of the hipLaunchKernel table.  Inputs include
    # zeros, negatives, large magnitudes and values where the ops saturate.
    ew = np.concatenate([np.array([0.0, -0.0, 1.0, -1.0, 3.0, -3.0, 20.0, -20.0, 88.0, -88.0, 1e-30, 0.5],
                                  np.float32), (rng.standard_normal(500) * 4).astype(np.float32)])
    data["ew_in"] = ew
    for op in range(15):
        data[f"ew_out_op{op}"] = po.ref_elementwise(op, np.abs(ew) if op in (8, 10) else ew)
    data["sc_out"] = po.ref_scale(ew, 0.37, -1.25)
    bb = (rng.standard_normal(24) * 2).astype(np.float32)
    bb[3] = 0.0  # division by zero gives 0 (binop_f32.glsl:27)
    data["bin_b"] = bb
    for op in range(4):
        data[f"bin_out_op{op}"] = po.ref_binop(op, ew[:480], bb)  # src1 broadcast: i % 24
    ne0, ne1, n_dims, n_seqs = 128, 3, 96, 2
    rx = rng.standard_normal(ne0 * ne1 * n_seqs).astype(np.float32)
    rp = np.array([7, 1234], np.int32)
    data["rope_in"], data["rope_pos"] = rx, rp
    data["rope_out"] = po.ref_rope_neox(rx, rp, ne0, ne1, n_dims, n_seqs, 10000.0 ** (-2.0 / n_dims), 1.0)
    emb = rng.standard_normal((50, 40)).astype(np.float16)
    eidx = np.array([0, 49, 7, -1, 50, 3, 3], np.int32)
    data["emb_w"], data["emb_idx"] = emb, eidx
    data["emb_out"] = po.ref_embedding(emb, eidx)

    out = Path(__file__).resolve().parent / "golden.npz"
    np.savez_compressed(out, **data)
    print(f"wrote {out} ({out.stat().st_size} bytes, {len(data)} arrays)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
