"""Fused dequant + GEMV (vkflame_quant_linear, M <= 8) against fp64.

The reference's value of every weight is the oracle's dequantised fp32
(bit-exact with the reference shaders); the product is computed in float64
and the kernel output must be within the north-star tolerance (max relative
error 2e-3, normwise) of it.  The CUDA path keeps the weights exact, so the
observed error is fp32-accumulation level; the tests also assert that
tighter 1e-4 bound to catch decode mistakes that hide under 2e-3.
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests import gpu_util as G
from vkflame_b200 import synth as S

pytestmark = pytest.mark.gpu

FORMATS = [S.Q4_0, S.Q8_0, S.Q4_K, S.Q5_K, S.Q6_K]


@pytest.fixture(scope="module")
def rt():
    from vkflame_b200 import rt
    rt.lib()
    return rt


def ref_fp64(q, w, x, N, K):
    wf = po.dequant(q, w, N * K // S.BLOCK_VALUES[q]).reshape(N, K).astype(np.float64)
    return x.astype(np.float64) @ wf.T


def run(rt, q, w, x, N, K, y_f16=False, ldy=None, xtype=0, ldx=None, x_offset=0):
    M = x.shape[0]
    ldy = ldy or N
    wd = G.dev(w)
    if xtype == rt.X_Q8_1:
        xd = G.dev(x)
        ldx = ldx or K // 32
        xptr = xd.data_ptr()
    else:
        ldx = ldx or x.shape[1]
        xd = G.dev(np.concatenate([np.zeros(x_offset, np.uint8), x.view(np.uint8).ravel()]))
        xptr = xd.data_ptr() + x_offset
    esz = 2 if y_f16 else 4
    yd = G.empty(M * ldy * esz)
    rt.quant_linear(wd.data_ptr(), q, xptr, xtype, yd.data_ptr(), rt.Y_F16 if y_f16 else rt.Y_F32, M, N, K, ldx, ldy)
    y = G.host(yd, np.float16 if y_f16 else np.float32, (M, ldy))
    rt.check_kernel_errors()
    return y[:, :N].astype(np.float64), y


@pytest.mark.parametrize("q", FORMATS)
@pytest.mark.parametrize("M", [1, 2, 3, 8])
def test_gemv_small(rt, q, M):
    N, K = 200, 1024  # N not a multiple of the 128-row tile
    w = S.quant_matrix(q, N, K, seed=q * 10 + M)
    x = S.normal_f16((M, K), seed=M)
    y, _ = run(rt, q, w, x, N, K)
    err = G.normwise_err(y, ref_fp64(q, w, x, N, K))
    assert err < 1e-4 < G.REL_TOL, err


@pytest.mark.parametrize("q", [S.Q4_0, S.Q8_0])
def test_gemv_ragged_k(rt, q):
    """K not a multiple of the 256-value step: a tail step of 32-value blocks."""
    N, K = 130, 32 * 13
    w = S.quant_matrix(q, N, K, seed=3)
    x = S.normal_f16((2, K), seed=4)
    y, _ = run(rt, q, w, x, N, K)
    assert G.normwise_err(y, ref_fp64(q, w, x, N, K)) < 1e-4


@pytest.mark.parametrize("q", FORMATS)
def test_gemv_f16_out_and_strides(rt, q):
    N, K, M = 384, 512, 4
    w = S.quant_matrix(q, N, K, seed=21)
    xf = S.normal_f16((M, K + 24), seed=22)  # ldx > K (16-byte aligned rows)
    y, full = run(rt, q, w, xf, N, K, y_f16=True, ldy=N + 8, ldx=K + 24)
    ref = ref_fp64(q, w, xf[:, :K], N, K)
    assert G.normwise_err(y, ref) < 1e-3  # fp16 output rounding
    assert (full[:, N:].view(np.uint16) == 0xFFFF).all(), "wrote outside the ldy padding"


def test_gemv_unaligned_activations(rt):
    """X at an address that is not 16-byte aligned takes the staged path."""
    q, N, K = S.Q4_K, 256, 512
    w = S.quant_matrix(q, N, K, seed=5)
    x = S.normal_f16((3, K), seed=6)
    y, _ = run(rt, q, w, x, N, K, x_offset=2)
    assert G.normwise_err(y, ref_fp64(q, w, x, N, K)) < 1e-4


@pytest.mark.parametrize("q", [S.Q4_K, S.Q8_0, S.Q6_K])
def test_gemv_q8_1_activations(rt, q):
    """The ggml mul_mat pattern: activations arrive as Q8_1 blocks."""
    N, K, M = 256, 1024, 2
    w = S.quant_matrix(q, N, K, seed=7)
    xq = po.quantize_q8_1(S.normal_f32((M, K), seed=8))
    xf = po.dequant(S.Q8_1, xq, M * K // 32).reshape(M, K)
    y, _ = run(rt, q, w, xq, N, K, xtype=rt.X_Q8_1)
    # activations are widened to fp16 (one rounding of d*q) before the product
    assert G.normwise_err(y, ref_fp64(q, w, xf, N, K)) < 1e-3


@pytest.mark.parametrize("q,K,N", [(S.Q4_K, 5120, 13824), (S.Q4_K, 13824, 5120), (S.Q4_K, 5120, 1024),
                                   (S.Q6_K, 13824, 5120), (S.Q8_0, 4096, 4096), (S.Q4_0, 4096, 4096)])
def test_gemv_full_size(rt, q, K, N):
    """Benchmark shapes: the stream-K split crosses many tiles here."""
    w = S.quant_matrix(q, N, K, seed=1)
    x = S.normal_f16((1, K), seed=2)
    y, _ = run(rt, q, w, x, N, K)
    assert G.normwise_err(y, ref_fp64(q, w, x, N, K)) < 1e-4


def test_gemv_deterministic(rt):
    q, N, K = S.Q4_K, 1024, 5120
    w = S.quant_matrix(q, N, K, seed=12)
    x = S.normal_f16((1, K), seed=13)
    y1, _ = run(rt, q, w, x, N, K)
    y2, _ = run(rt, q, w, x, N, K)
    assert np.array_equal(y1, y2)


def test_quant_linear_rejects_bad_shapes(rt):
    buf = G.empty(1 << 16)
    p = buf.data_ptr()
    with pytest.raises(rt.VkflameError):
        rt.quant_linear(p, S.Q4_K, p, 0, p, 0, 1, 16, 100, 100, 16)  # K % 256 != 0
    with pytest.raises(rt.VkflameError):
        rt.quant_linear(p, 42, p, 0, p, 0, 1, 16, 256, 256, 16)
