"""Tensor-core GEMM paths (tcgen05): linear_int8, vkflame_dispatch_linear, and
quantised prefill (vkflame_quant_linear with M > 8).

int8: the int32 accumulators are bit-exact with the oracle's restatement of
kernels/linear_int8.glsl:54-90, and so is the fp16 output without an
activation (same fp32 operation order, no contraction).  fp16 paths: max
relative error (normwise) <= 2e-3 against fp64.
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests import gpu_util as G
from vkflame_b200 import synth as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from vkflame_b200 import rt
    rt.lib()
    return rt


def int8_case(M, N, K, seed):
    rng = np.random.default_rng(seed)
    x = rng.integers(-127, 128, (M, K), dtype=np.int8)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sx = rng.uniform(1e-3, 1e-2, M).astype(np.float32)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    return x, w, sx, sw, bias


def run_int8(rt, x, w, sx, sw, bias, act=0):
    M, K = x.shape
    N = w.shape[0]
    xd, wd, sxd, swd, bd = (G.dev(a) for a in (x, w, sx, sw, bias))
    yd = G.empty(M * N * 2)
    ad = G.empty(M * N * 4)
    rt.linear_int8(xd.data_ptr(), wd.data_ptr(), sxd.data_ptr(), swd.data_ptr(), bd.data_ptr(), yd.data_ptr(),
                   ad.data_ptr(), M, N, K, act)
    rt.check_kernel_errors()
    return G.host(ad, np.int32, (M, N)), G.host(yd, np.float16, (M, N))


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (256, 512, 1024), (37, 100, 72), (1, 300, 4096), (130, 260, 528)])
def test_linear_int8_bit_exact(rt, M, N, K):
    x, w, sx, sw, bias = int8_case(M, N, K, seed=M + N + K)
    acc, y = run_int8(rt, x, w, sx, sw, bias)
    ref_acc, ref_y = po.linear_int8(x, w, sx, sw, bias)
    assert np.array_equal(acc, ref_acc)
    assert np.array_equal(y.view(np.uint16), ref_y.view(np.uint16))


@pytest.mark.parametrize("act", [1, 2, 3])
def test_linear_int8_activations(rt, act):
    x, w, sx, sw, bias = int8_case(64, 256, 512, seed=act)
    sw *= 20  # outputs of order 1 so the activations are not trivially linear
    acc, y = run_int8(rt, x, w, sx, sw, bias, act)
    ref_acc, ref_y = po.linear_int8(x, w, sx, sw, bias, act=act)
    assert np.array_equal(acc, ref_acc)
    # expf on the GPU and in libm may differ in the last ulp before fp16 rounding
    assert G.normwise_err(y, ref_y) < 2e-3


def test_linear_int8_config2_rows(rt):
    """Config 2 size (M=512, K=4096, N=11008); 24 sampled rows checked bit-exactly."""
    M, N, K = 512, 11008, 4096
    x, w, sx, sw, bias = int8_case(M, N, K, seed=2)
    acc, y = run_int8(rt, x, w, sx, sw, bias)
    rows = np.random.default_rng(0).choice(M, 24, replace=False)
    ref_acc, ref_y = po.linear_int8(x[rows], w, sx[rows], sw, bias)
    assert np.array_equal(acc[rows], ref_acc)
    assert np.array_equal(y[rows].view(np.uint16), ref_y.view(np.uint16))


def f16(a):
    return np.ascontiguousarray(a, np.float16)


@pytest.mark.parametrize("transA,transB", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("dtype", [1, 4])  # FP16 (fp16 out), FP16_FP32OUT
def test_dispatch_linear_f16(rt, transA, transB, dtype):
    M, N, K = 200, 300, 264
    rng = np.random.default_rng(5)
    a = rng.standard_normal((M, K)).astype(np.float16)
    b = rng.standard_normal((K, N)).astype(np.float16)
    c = rng.standard_normal((M, N)).astype(np.float16 if dtype == 1 else np.float32)
    ad = G.dev(f16(a.T) if transA else a)
    bd = G.dev(f16(b.T) if transB else b)
    dd = G.dev(c.copy())
    rt.dispatch_linear(ad.data_ptr(), bd.data_ptr(), dd.data_ptr(), dd.data_ptr(), M, N, K, dtype, transA, transB,
                       alpha=0.5, beta=2.0)
    got = G.host(dd, c.dtype, (M, N))
    ref = 0.5 * (a.astype(np.float64) @ b.astype(np.float64)) + 2.0 * c.astype(np.float64)
    assert G.normwise_err(got, ref) < 2e-3


def test_dispatch_linear_int8(rt):
    M, N, K = 64, 96, 128
    rng = np.random.default_rng(6)
    a = rng.integers(-5, 6, (M, K), dtype=np.int8)
    b = rng.integers(-5, 6, (K, N), dtype=np.int8)
    ad, bd = G.dev(a), G.dev(b)
    dd = G.empty(M * N * 2)
    rt.dispatch_linear(ad.data_ptr(), bd.data_ptr(), 0, dd.data_ptr(), M, N, K, 2, 0, 0)
    got = G.host(dd, np.float16, (M, N))
    ref = a.astype(np.int64) @ b.astype(np.int64)
    assert np.array_equal(got.astype(np.int64), ref)  # |acc| <= 3200: exact in fp16


@pytest.mark.parametrize("q", [S.Q4_0, S.Q8_0, S.Q4_K, S.Q5_K, S.Q6_K])
@pytest.mark.parametrize("M", [32, 77])
def test_quant_linear_prefill(rt, q, M):
    N, K = 384, 1024
    w = S.quant_matrix(q, N, K, seed=40 + q)
    x = S.normal_f16((M, K), seed=M)
    wd, xd = G.dev(w), G.dev(x)
    yd = G.empty(M * N * 4)
    rt.quant_linear(wd.data_ptr(), q, xd.data_ptr(), rt.X_F16, yd.data_ptr(), rt.Y_F32, M, N, K, K, N)
    y = G.host(yd, np.float32, (M, N))
    wf = po.dequant(q, w, N * K // S.BLOCK_VALUES[q]).reshape(N, K).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T
    # weights are widened to fp16 (one rounding each) before the fp32-accumulated product
    assert G.normwise_err(y, ref) < 1e-3


def test_quant_linear_prefill_q8_1(rt):
    """Config 4 pattern (Q8_0 weights x on-device Q8_1 activations), reduced size."""
    M, N, K = 128, 512, 2048
    w = S.quant_matrix(S.Q8_0, N, K, seed=9)
    xf = S.normal_f32((M, K), seed=10)
    xd = G.dev(xf)
    xq = G.empty(M * K // 32 * 36)
    rt.quantize_q8_1(xd.data_ptr(), xq.data_ptr(), M, K, K)
    wd = G.dev(w)
    yd = G.empty(M * N * 4)
    rt.quant_linear(wd.data_ptr(), S.Q8_0, xq.data_ptr(), rt.X_Q8_1, yd.data_ptr(), rt.Y_F32, M, N, K, K // 32, N)
    y = G.host(yd, np.float32, (M, N))
    xq_h = G.host(xq, np.uint8)
    assert np.array_equal(xq_h, po.quantize_q8_1(xf).ravel())
    xdq = po.dequant(S.Q8_1, xq_h, M * K // 32).reshape(M, K).astype(np.float64)
    wf = po.dequant(S.Q8_0, w, N * K // 32).reshape(N, K).astype(np.float64)
    assert G.normwise_err(y, xdq @ wf.T) < 2e-3


@pytest.mark.gpu
@pytest.mark.parametrize("q,M,N,K,f16,ldy", [
    (S.Q4_K, 300, 200, 2048, True, 256),    # two activation tiles of 256 (second ragged), ragged weight tile
    (S.Q8_0, 9, 130, 512, False, 130),      # smallest prefill M, one-row second weight tile
    (S.Q5_K, 64, 256, 5120, False, 264),    # 14B K, padded output rows
    (S.Q4_0, 129, 384, 4096, True, 384),    # 129 -> activation tiles of 256
    (S.Q4_K, 96, 1000, 1280, True, 1000),   # 128-wide activation tile, odd N
    # Q6_K: 210-byte super-blocks, rows fetched one bulk copy each from the
    # 16-byte boundary below them (row starts at every even offset mod 16)
    (S.Q6_K, 300, 200, 2048, True, 256),    # ragged tiles, padded output rows
    (S.Q6_K, 512, 640, 13824, False, 640),  # ffn_down K (row pitch 11340 = 12 mod 16)
    (S.Q6_K, 40, 1000, 5120, True, 1000),   # attn_v / head K (pitch 4200 = 8 mod 16), odd N
])
def test_quant_linear_prefill_fused_shapes(rt, q, M, N, K, f16, ldy):
    """Fused-dequant tcgen05 prefill (packed W bytes -> fp16 tiles in shared
    memory): ragged M and N, fp16 and fp32 outputs, output stride > N; the
    bytes between N and ldy must stay untouched."""
    w = S.quant_matrix(q, N, K, seed=50 + q + M)
    x = S.normal_f16((M, K), seed=M + 1)
    wd, xd = G.dev(w), G.dev(x)
    es = 2 if f16 else 4
    yd = G.empty(M * ldy * es)
    rt.quant_linear(wd.data_ptr(), q, xd.data_ptr(), rt.X_F16, yd.data_ptr(), rt.Y_F16 if f16 else rt.Y_F32,
                    M, N, K, K, ldy)
    yfull = G.host(yd, np.float16 if f16 else np.float32, (M, ldy))
    wf = po.dequant(q, w, N * K // S.BLOCK_VALUES[q]).reshape(N, K).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T
    assert G.normwise_err(yfull[:, :N].astype(np.float64), ref) < G.REL_TOL
    if ldy > N:
        pad = G.host(yd, np.uint8, (M, ldy * es))[:, N * es:]
        assert (pad == 0xFF).all()
    rt.check_kernel_errors()


@pytest.mark.gpu
def test_quant_linear_prefill_config4_size(rt):
    """Config 4 at full size (M=512, K=5120, N=13824, Q8_0 x Q8_1): sampled
    output rows against the fp64 product of the dequantised operands."""
    M, N, K = 512, 13824, 5120
    w = S.quant_matrix(S.Q8_0, N, K, seed=77)
    xf = S.normal_f32((M, K), seed=78)
    xd, wd = G.dev(xf), G.dev(w)
    xq = G.empty(M * K // 32 * 36)
    rt.quantize_q8_1(xd.data_ptr(), xq.data_ptr(), M, K, K)
    yd = G.empty(M * N * 4)
    rt.quant_linear(wd.data_ptr(), S.Q8_0, xq.data_ptr(), rt.X_Q8_1, yd.data_ptr(), rt.Y_F32, M, N, K, K // 32, N)
    y = G.host(yd, np.float32, (M, N))
    rows = np.array([0, 1, 127, 128, 255, 256, 300, 511])
    xq_h = G.host(xq, np.uint8).reshape(M, K // 32 * 36)
    xdq = po.dequant(S.Q8_1, np.ascontiguousarray(xq_h[rows]).ravel(), len(rows) * K // 32).reshape(len(rows), K)
    wf = po.dequant(S.Q8_0, w, N * K // 32).reshape(N, K).astype(np.float64)
    ref = xdq.astype(np.float64) @ wf.T
    assert G.normwise_err(y[rows], ref) < G.REL_TOL
    rt.check_kernel_errors()


@pytest.mark.gpu
@pytest.mark.parametrize("q,M,N,K", [(S.Q4_K, 512, 5120, 5120), (S.Q6_K, 256, 640, 13824)])
def test_quant_linear_prefill_fresh_streams(rt, q, M, N, K):
    """Stream-K tiles on streams the library has not seen: each call on a new
    non-blocking stream makes the library create that stream's scratch and
    flag arenas, whose zeroing must be ordered before the GEMM's first flag
    store on that stream.  Every result equals, byte for byte, the same call
    on a stream whose arenas already exist (the partial sums of a split tile
    are added in a fixed order)."""
    import torch
    from cuda.bindings import runtime as cr
    w = S.quant_matrix(q, N, K, seed=90 + q)
    x = S.normal_f16((M, K), seed=91)
    wd, xd = G.dev(w), G.dev(x)

    def run(stream):
        yd = torch.empty(M * N, dtype=torch.float16, device="cuda")
        rt.quant_linear_ex(wd.data_ptr(), q, xd.data_ptr(), rt.X_F16, yd.data_ptr(), rt.Y_F16, M, N, K, K, N,
                           rt.FLAG_STATIC_WEIGHTS, stream)
        torch.cuda.synchronize()
        return yd.cpu().numpy()

    warm = torch.cuda.Stream()
    run(warm.cuda_stream)
    ref = run(warm.cuda_stream)
    streams = []
    try:
        for _ in range(6):
            err, s = cr.cudaStreamCreateWithFlags(cr.cudaStreamNonBlocking)
            assert err == cr.cudaError_t.cudaSuccess
            streams.append(s)
            assert np.array_equal(run(int(s)).view(np.uint16), ref.view(np.uint16))
        rt.check_kernel_errors()
    finally:
        torch.cuda.synchronize()
        for s in streams:
            cr.cudaStreamDestroy(s)
