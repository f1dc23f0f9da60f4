"""Seeded synthetic ggml block tensors with the benchmark configs' distributions.

No model weights or datasets are used anywhere: every input is generated here
from ``numpy.random.default_rng(seed)``.  The value distributions are the ones
the benchmark configs specify (fp16 scales uniform in a range, quants uniform
over their full code range, fp16 activations N(0,1)).

A quantised matrix is returned as a ``uint8`` array of shape
``(N, row_bytes)``: ``N`` output rows, each holding ``K / QK`` consecutive
blocks in ggml's byte layout (see ``include/ggml_blocks.h``).
"""
from __future__ import annotations

import numpy as np

Q4_0, Q4_1, Q8_0, Q5_0, Q4_K, Q5_K, Q6_K, Q8_1 = range(8)
NAMES = {Q4_0: "q4_0", Q4_1: "q4_1", Q8_0: "q8_0", Q5_0: "q5_0", Q4_K: "q4_K",
         Q5_K: "q5_K", Q6_K: "q6_K", Q8_1: "q8_1"}
BLOCK_VALUES = {Q4_0: 32, Q4_1: 32, Q8_0: 32, Q5_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_1: 32}
BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q8_0: 34, Q5_0: 22, Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_1: 36}


def row_bytes(qtype: int, K: int) -> int:
    assert K % BLOCK_VALUES[qtype] == 0, (qtype, K)
    return K // BLOCK_VALUES[qtype] * BLOCK_BYTES[qtype]


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(v.astype(np.float16)).view(np.uint8).reshape(*v.shape, 2)


def _scale(rng, shape, lo, hi):
    return rng.uniform(lo, hi, size=shape).astype(np.float32)


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack 8 six-bit (scale, min) pairs per super-block into 12 bytes, the
    inverse of get_scale_min_k4 (kernels/dequant_q4_k.glsl:16-24)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 0xF) | ((mn[..., 4:8] & 0xF) << 4)
    return out


def quant_matrix(qtype: int, N: int, K: int, seed: int = 0, d_range=None) -> np.ndarray:
    """Random ggml blocks for an N x K weight (N rows of K/QK blocks)."""
    rng = np.random.default_rng(seed)
    qk, bb = BLOCK_VALUES[qtype], BLOCK_BYTES[qtype]
    nb = K // qk
    assert nb * qk == K
    blk = np.empty((N, nb, bb), np.uint8)
    if qtype == Q4_0:
        lo, hi = d_range or (1e-3, 2e-2)
        blk[..., 0:2] = _f16_bytes(_scale(rng, (N, nb), lo, hi))
        blk[..., 2:18] = rng.integers(0, 256, (N, nb, 16), dtype=np.uint8)
    elif qtype == Q4_1:
        lo, hi = d_range or (1e-3, 2e-2)
        blk[..., 0:2] = _f16_bytes(_scale(rng, (N, nb), lo, hi))
        blk[..., 2:4] = _f16_bytes(-_scale(rng, (N, nb), lo, hi) * 8)
        blk[..., 4:20] = rng.integers(0, 256, (N, nb, 16), dtype=np.uint8)
    elif qtype == Q5_0:
        lo, hi = d_range or (1e-3, 2e-2)
        blk[..., 0:2] = _f16_bytes(_scale(rng, (N, nb), lo, hi))
        blk[..., 2:22] = rng.integers(0, 256, (N, nb, 20), dtype=np.uint8)
    elif qtype in (Q8_0, Q8_1):
        lo, hi = d_range or (1e-3, 1e-2)
        d = _scale(rng, (N, nb), lo, hi)
        q = rng.integers(-127, 128, (N, nb, 32), dtype=np.int8)
        blk[..., 0:2] = _f16_bytes(d)
        if qtype == Q8_0:
            blk[..., 2:34] = q.view(np.uint8)
        else:
            s = d.astype(np.float16).astype(np.float32) * q.astype(np.int32).sum(-1).astype(np.float32)
            blk[..., 2:4] = _f16_bytes(s)
            blk[..., 4:36] = q.view(np.uint8)
    elif qtype in (Q4_K, Q5_K):
        lo, hi = d_range or (1e-3, 1e-2)
        blk[..., 0:2] = _f16_bytes(_scale(rng, (N, nb), lo, hi))
        blk[..., 2:4] = _f16_bytes(_scale(rng, (N, nb), lo, hi))
        sc = rng.integers(0, 64, (N, nb, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, (N, nb, 8), dtype=np.uint8)
        blk[..., 4:16] = pack_scale_min_k4(sc, mn)
        blk[..., 16:] = rng.integers(0, 256, (N, nb, bb - 16), dtype=np.uint8)
    elif qtype == Q6_K:
        lo, hi = d_range or (1e-3, 1e-2)
        blk[..., 0:192] = rng.integers(0, 256, (N, nb, 192), dtype=np.uint8)
        blk[..., 192:208] = rng.integers(-128, 128, (N, nb, 16), dtype=np.int8).view(np.uint8)
        blk[..., 208:210] = _f16_bytes(_scale(rng, (N, nb), lo, hi))
    else:
        raise ValueError(qtype)
    return blk.reshape(N, nb * bb)


def normal_f16(shape, seed: int = 0) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32).astype(np.float16)


def normal_f32(shape, seed: int = 0) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
