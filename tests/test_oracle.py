"""The CPU oracle against the golden vectors made by the reference shaders.

The golden vectors come from the reference's own GLSL run as C++
(tests/golden/gen_golden.py); these tests pin oracle/oracle.c to them bit for
bit, so the oracle can stand in for the reference on the GPU box.
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from vkflame_b200 import synth as S


@pytest.mark.parametrize("q", range(8))
@pytest.mark.parametrize("kind", ["dq", "dqe"])
def test_dequant_matches_reference_shader(golden, q, kind):
    name = S.NAMES[q]
    raw = golden[f"{kind}_{name}_in"]
    exp = golden[f"{kind}_{name}_out"]
    nb = raw.size // S.BLOCK_BYTES[q]
    got = po.dequant(q, raw, nb)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("act", range(4))
def test_linear_int8_shader(golden, act):
    got = po.linear_int8_shader(golden["i8_a"], golden["i8_w"], golden["i8_ws"], 0.03, act)
    assert np.array_equal(got.view(np.uint16), golden[f"i8_out_act{act}"].view(np.uint16))


def test_int8_accumulator_pinned(golden):
    """Small case whose fp16 output is the exact int32 accumulator."""
    a, w = golden["i8x_a"], golden["i8x_w"]
    acc, _ = po.linear_int8(a.astype(np.int8), w, np.ones(a.shape[0], np.float32),
                            np.ones(w.shape[0], np.float32))
    assert np.array_equal(acc.astype(np.float16), golden["i8x_out"])
    assert np.abs(acc).max() <= 2048


@pytest.mark.parametrize("act", range(4))
def test_linear_fp16_shader(golden, act):
    got = po.linear_fp16_shader(golden["f16_a"], golden["f16_b"], act)
    assert np.array_equal(got.view(np.uint16), golden[f"f16_out_act{act}"].view(np.uint16))


def test_q8_1_roundtrip():
    x = S.normal_f32((4, 256), seed=3)
    q = po.quantize_q8_1(x)
    y = po.dequant(S.Q8_1, q, 4 * 8).reshape(4, 256)
    amax = np.abs(x.reshape(4, 8, 32)).max(-1, keepdims=True)
    err = np.abs((y - x).reshape(4, 8, 32))
    # half a quantisation step, plus the fp16 rounding of d times |q| <= 127
    assert (err <= amax / 127 * 0.57).all()


@pytest.mark.parametrize("q", [S.Q4_0, S.Q8_0, S.Q4_K, S.Q5_K, S.Q6_K])
def test_quant_linear_against_fp64(q):
    M, N, K = 3, 16, 512
    w = S.quant_matrix(q, N, K, seed=5)
    x = S.normal_f16((M, K), seed=6)
    y = po.quant_linear(q, w, x, M, N, K)
    wf = po.dequant(q, w, N * K // S.BLOCK_VALUES[q]).reshape(N, K).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T
    assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-5


@pytest.mark.skipif(not po.ref_available(), reason="reference harness not built here")
@pytest.mark.parametrize("q", range(8))
def test_dequant_random_against_live_shader(q):
    w = S.quant_matrix(q, 5, 1024, seed=77 + q).ravel()
    nb = w.size // S.BLOCK_BYTES[q]
    assert np.array_equal(po.dequant(q, w, nb).view(np.uint32), po.ref_dequant(q, w, nb).view(np.uint32))


# ---- the non-matmul kernels of the hipLaunchKernel table -------------------
# The oracle uses the same C library functions (expf, tanhf, ...) as the
# shader-as-C++ harness and the same operation order, so it matches the
# golden vectors bit for bit.

@pytest.mark.parametrize("op", range(15))
def test_elementwise_matches_reference_shader(golden, op):
    x = golden["ew_in"]
    x = np.abs(x) if op in (8, 10) else x
    got = po.elementwise(op, x)
    assert np.array_equal(got.view(np.uint32), golden[f"ew_out_op{op}"].view(np.uint32))


def test_scale_matches_reference_shader(golden):
    got = po.scale(golden["ew_in"], 0.37, -1.25)
    assert np.array_equal(got.view(np.uint32), golden["sc_out"].view(np.uint32))


@pytest.mark.parametrize("op", range(4))
def test_binop_matches_reference_shader(golden, op):
    got = po.binop(op, golden["ew_in"][:480], golden["bin_b"])
    assert np.array_equal(got.view(np.uint32), golden[f"bin_out_op{op}"].view(np.uint32))


def test_rope_neox_matches_reference_shader(golden):
    ne0, ne1, n_dims, n_seqs = 128, 3, 96, 2
    got = po.rope_neox(golden["rope_in"], golden["rope_pos"], ne0, ne1, n_dims, n_seqs, 10000.0 ** (-2.0 / n_dims), 1.0)
    assert np.array_equal(got.view(np.uint32), golden["rope_out"].view(np.uint32))


def test_embedding_matches_reference_shader(golden):
    got = po.embedding(golden["emb_w"], golden["emb_idx"])
    assert np.array_equal(got.view(np.uint16), golden["emb_out"].view(np.uint16))
    assert (got[3] == 0).all() and (got[4] == 0).all()  # indices -1 and V


def test_row_ops_against_fp64():
    """rms_norm*.glsl and softmax_online.glsl reduce with subgroup operations
    the harness cannot run; the restatement is checked against fp64 math."""
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((5, 300)) * 3).astype(np.float32)
    ref = x.astype(np.float64) / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6)
    assert np.abs(po.rms_norm_f32(x, 1e-6) - ref).max() < 1e-5 * np.abs(ref).max()
    e = np.exp(x.astype(np.float64) - x.max(1, keepdims=True))
    assert np.abs(po.softmax(x) - e / e.sum(1, keepdims=True)).max() < 1e-6
    x16, g16 = x.astype(np.float16), rng.standard_normal(300).astype(np.float16)
    r16 = x16.astype(np.float64) / np.sqrt((x16.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * g16
    assert np.abs(po.rms_norm_f16(x16, g16, 1e-6).astype(np.float64) - r16).max() < 2e-3 * np.abs(r16).max()


@pytest.mark.skipif(not po.ref_available(), reason="reference harness not built here")
def test_ops_random_against_live_shaders():
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(3000) * 5).astype(np.float32)
    for op in range(15):
        xi = np.abs(x) if op in (8, 10) else x
        assert np.array_equal(po.elementwise(op, xi).view(np.uint32), po.ref_elementwise(op, xi).view(np.uint32)), op
    b = rng.standard_normal(100).astype(np.float32)
    for op in range(4):
        assert np.array_equal(po.binop(op, x, b).view(np.uint32), po.ref_binop(op, x, b).view(np.uint32))
