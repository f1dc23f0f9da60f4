"""The non-matmul kernels of ggml's hipLaunchKernel name table (ggml_ops.cu):
through their C entry points (vkflame_dispatch_*, the reference's dispatch.h
names) and through hipLaunchKernel with ggml kernel names and the
reference's argument positions.  Checked against the oracle (which matches
the reference shaders bit for bit on the golden vectors).  The tolerances are
those of fp32 transcendental functions from two libraries (CUDA's and the C
library's): a few ulp, written per test."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po
from tests import gpu_util as G

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from vkflame_b200 import rt as _rt
    _rt.lib()
    return _rt


def f32dev(a):
    return G.dev(np.ascontiguousarray(a, np.float32))


def close(got, ref, rtol=2e-6, atol=1e-6):
    got, ref = np.asarray(got, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
    fin = np.isfinite(ref)
    if not np.array_equal(np.isfinite(got), fin) or not np.array_equal(got[~fin], ref[~fin]):
        return False, float("nan")  # infinities and NaNs must match in place (log(0) = -inf)
    d = np.abs(got[fin] - ref[fin])
    ok = d <= atol + rtol * np.abs(ref[fin])
    return bool(ok.all()), float(d.max()) if d.size else 0.0


@pytest.mark.parametrize("op", range(15))
def test_elementwise(rt, golden, op):
    lib = rt.lib()
    x = golden["ew_in"]
    x = np.abs(x) if op in (8, 10) else x
    x = np.concatenate([x, np.random.default_rng(op).standard_normal(100003).astype(np.float32)])
    x = np.abs(x) if op in (8, 10) else x
    xd, yd = f32dev(x), G.empty(x.size * 4)
    lib.vkflame_dispatch_elementwise_f32.argtypes = [C.c_void_p] * 3 + [C.c_uint32] * 2
    assert lib.vkflame_dispatch_elementwise_f32(None, xd.data_ptr(), yd.data_ptr(), x.size, op) == 0
    got = G.host(yd, np.float32)
    ok, err = close(got, po.elementwise(op, x), rtol=4e-6, atol=2e-7)
    assert ok, err


def test_elementwise_in_place_and_unaligned(rt):
    lib = rt.lib()
    x = np.random.default_rng(1).standard_normal(1001).astype(np.float32)
    d = f32dev(np.concatenate([[0.0], x]).astype(np.float32))  # data at +4 bytes: not 16-byte aligned
    lib.vkflame_dispatch_elementwise_f32.argtypes = [C.c_void_p] * 3 + [C.c_uint32] * 2
    assert lib.vkflame_dispatch_elementwise_f32(None, d.data_ptr() + 4, d.data_ptr() + 4, x.size, 0) == 0
    ok, err = close(G.host(d, np.float32)[1:], po.elementwise(0, x), rtol=4e-6)
    assert ok, err


def test_scale_binop(rt, golden):
    lib = rt.lib()
    x = golden["ew_in"]
    xd, yd = f32dev(x), G.empty(x.size * 4)
    lib.vkflame_dispatch_scale_f32.argtypes = [C.c_void_p] * 3 + [C.c_uint32, C.c_float, C.c_float]
    assert lib.vkflame_dispatch_scale_f32(None, xd.data_ptr(), yd.data_ptr(), x.size, 0.37, -1.25) == 0
    assert np.array_equal(G.host(yd, np.float32).view(np.uint32), golden["sc_out"].view(np.uint32))
    lib.vkflame_dispatch_binop_f32.argtypes = [C.c_void_p] * 4 + [C.c_uint32] * 3
    bd = f32dev(golden["bin_b"])
    for op in range(4):
        assert lib.vkflame_dispatch_binop_f32(None, xd.data_ptr(), bd.data_ptr(), yd.data_ptr(), 480, 24, op) == 0
        got = G.host(yd, np.float32)[:480]
        if op == 3:  # CUDA's division rounds correctly, as the C library's does
            assert np.array_equal(got.view(np.uint32), golden["bin_out_op3"].view(np.uint32))
        else:
            assert np.array_equal(got.view(np.uint32), golden[f"bin_out_op{op}"].view(np.uint32))


def test_rms_norms_softmax(rt):
    lib = rt.lib()
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((37, 5120)) * 3).astype(np.float32)
    xd, yd = f32dev(x), G.empty(x.size * 4)
    lib.vkflame_dispatch_rms_norm_f32.argtypes = [C.c_void_p] * 3 + [C.c_uint32] * 2 + [C.c_float]
    assert lib.vkflame_dispatch_rms_norm_f32(None, xd.data_ptr(), yd.data_ptr(), 37, 5120, 1e-6) == 0
    ok, err = close(G.host(yd, np.float32), po.rms_norm_f32(x, 1e-6), rtol=1e-5, atol=1e-6)
    assert ok, err
    lib.vkflame_dispatch_softmax.argtypes = [C.c_void_p] * 3 + [C.c_int] * 2
    assert lib.vkflame_dispatch_softmax(None, xd.data_ptr(), yd.data_ptr(), 37, 5120) == 0
    got = G.host(yd, np.float32).reshape(37, 5120)
    ok, err = close(got, po.softmax(x), rtol=2e-5, atol=1e-9)
    assert ok, err
    assert np.abs(got.sum(1) - 1).max() < 1e-4
    x16, g16 = x[:, :4096].astype(np.float16).copy(), rng.standard_normal(4096).astype(np.float16)
    xd16, gd16, yd16 = G.dev(x16), G.dev(g16), G.empty(x16.size * 2)
    lib.vkflame_dispatch_rms_norm.argtypes = [C.c_void_p] * 4 + [C.c_int] * 2 + [C.c_float]
    assert lib.vkflame_dispatch_rms_norm(None, xd16.data_ptr(), gd16.data_ptr(), yd16.data_ptr(), 37, 4096, 1e-6) == 0
    got = G.host(yd16, np.float16).reshape(37, 4096).astype(np.float64)
    ref = po.rms_norm_f16(x16, g16, 1e-6).astype(np.float64)
    assert np.abs(got - ref).max() <= 2 ** -10 * np.abs(ref).max()  # at most an fp16 rounding apart


def test_rope_neox_every_row_and_pair(rt, golden):
    """Every row of every sequence and every pair (the reference's dispatch
    grid reached only part of them)."""
    lib = rt.lib()
    ne0, ne1, n_dims, n_seqs = 128, 3, 96, 2
    xd, pd, yd = f32dev(golden["rope_in"]), G.dev(golden["rope_pos"]), G.empty(golden["rope_in"].size * 4)
    lib.vkflame_dispatch_rope_neox.argtypes = [C.c_void_p] * 4 + [C.c_uint32] * 4 + [C.c_float] * 2 + [C.c_uint32] * 2
    ts = 10000.0 ** (-2.0 / n_dims)
    assert lib.vkflame_dispatch_rope_neox(None, xd.data_ptr(), pd.data_ptr(), yd.data_ptr(), ne0, ne1, n_dims, n_seqs,
                                          ts, 1.0, 0, 0) == 0
    ok, err = close(G.host(yd, np.float32), golden["rope_out"], rtol=0, atol=2e-3)  # theta up to ~1234 rad
    assert ok, err


def test_embedding_and_get_rows(rt, golden):
    lib = rt.lib()
    w, idx = golden["emb_w"], golden["emb_idx"]
    wd, idd, od = G.dev(w), G.dev(idx), G.empty(idx.size * w.shape[1] * 4)
    lib.vkflame_dispatch_embedding.argtypes = [C.c_void_p] * 4 + [C.c_int] * 3
    assert lib.vkflame_dispatch_embedding(None, wd.data_ptr(), idd.data_ptr(), od.data_ptr(), 50, 40, idx.size) == 0
    got = G.host(od, np.uint16)[:idx.size * 40].reshape(idx.size, 40)
    assert np.array_equal(got, golden["emb_out"].view(np.uint16))
    lib.vkflame_get_rows.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p] + [C.c_int] * 3 + [C.c_void_p]
    w32 = w.astype(np.float32)
    assert lib.vkflame_get_rows(f32dev(w32).data_ptr(), 1, idd.data_ptr(), od.data_ptr(), 50, 40, idx.size, None) == 0
    assert np.array_equal(G.host(od, np.float32).reshape(idx.size, 40), po.embedding(w32, idx))


# ---- through hipLaunchKernel with ggml names ---------------------------------

from tests.test_gpu_shims import hip  # noqa: E402,F401  (the libamdhip64 fixture)


def _launch(hip, name, grid, block, args):
    from tests import test_gpu_shims as T
    fn = T.register(hip, name)
    return T.launch(hip, fn, grid, block, args)


@pytest.mark.parametrize("name,op", [("silu_f32", 0), ("gelu_quick_f32", 4), ("gelu_f32", 1), ("relu_f32", 2),
                                     ("tanh_f32", 3), ("sigmoid_f32", 6), ("sqr_f32", 7), ("sqrt_f32", 8),
                                     ("neg_f32", 5), ("abs_f32", 11)])
def test_hip_launch_unary(hip, name, op):
    from tests.test_gpu_shims import Dev
    x = np.random.default_rng(op).standard_normal(4099).astype(np.float32)
    x = np.abs(x) if op in (8, 10) else x
    xd, yd = Dev(hip, x), Dev(hip, nbytes=x.nbytes)
    assert _launch(hip, f"void {name}(const float*, float*, int)", (17, 1, 1), (256, 1, 1),
                   [xd.ptr, yd.ptr, (C.c_int, x.size)]) == 0
    ok, err = close(yd.get(np.float32), po.elementwise(op, x), rtol=4e-6, atol=2e-7)
    assert ok, (name, err)


def test_hip_launch_scale_rms_norm_softmax_binop_rope_get_rows(hip):
    from tests.test_gpu_shims import Dev
    rng = np.random.default_rng(5)
    x = rng.standard_normal((6, 512)).astype(np.float32)
    xd, yd = Dev(hip, x), Dev(hip, nbytes=x.nbytes)
    # scale_f32(x, dst, float scale, float bias, int64 n)
    assert _launch(hip, "scale_f32", (12, 1, 1), (256, 1, 1),
                   [xd.ptr, yd.ptr, (C.c_float, 0.5), (C.c_float, 2.0), (C.c_int64, x.size)]) == 0
    assert np.array_equal(yd.get(np.float32).reshape(6, 512), po.scale(x, 0.5, 2.0).reshape(6, 512))
    # rms_norm_f32(x, dst, ncols, s_row, s_chan, s_sample, eps): rows = grid.x
    assert _launch(hip, "rms_norm_f32<256>", (6, 1, 1), (256, 1, 1),
                   [xd.ptr, yd.ptr, (C.c_int, 512), (C.c_int, 512), (C.c_int, 0), (C.c_int, 0), (C.c_float, 1e-5)]) == 0
    ok, err = close(yd.get(np.float32).reshape(6, 512), po.rms_norm_f32(x, 1e-5), rtol=1e-5)
    assert ok, err
    # soft_max_f32(x, mask, dst, ncols, ...): rows = grid.y
    assert _launch(hip, "soft_max_f32", (1, 6, 1), (256, 1, 1), [xd.ptr, 0, yd.ptr, (C.c_int, 512)]) == 0
    ok, err = close(yd.get(np.float32).reshape(6, 512), po.softmax(x), rtol=2e-5, atol=1e-9)
    assert ok, err
    # k_bin_bcast mul: (src0, src1, dst): n = grid.x * block.x
    b = rng.standard_normal((6, 512)).astype(np.float32)
    bd = Dev(hip, b)
    assert _launch(hip, "k_bin_bcast<op_mul>", (12, 1, 1), (256, 1, 1), [xd.ptr, bd.ptr, yd.ptr]) == 0
    assert np.array_equal(yd.get(np.float32), po.binop(1, x, b).ravel())
    # a grid that over-covers (16 x 256 > 3072 values) is clamped to the
    # sources' allocations: nothing is written past 3072 values
    big = Dev(hip, np.full(x.size + 1024, 7.0, np.float32))
    assert _launch(hip, "k_bin_bcast<op_add>", (16, 1, 1), (256, 1, 1), [xd.ptr, bd.ptr, big.ptr]) == 0
    got = big.get(np.float32)
    assert np.array_equal(got[:x.size], po.binop(0, x, b).ravel()) and (got[x.size:] == 7.0).all()
    # rope_neox(x, dst, ne0, ne1, s1, s2, n_dims, pos, freq_scale, ..., theta_scale at 13); seqs = grid.y
    ne0, ne1 = 64, 4
    rx = rng.standard_normal((2, ne1, ne0)).astype(np.float32)
    pos = np.array([3, 11], np.int32)
    rxd, rpd, ryd = Dev(hip, rx), Dev(hip, pos), Dev(hip, nbytes=rx.nbytes)
    ts = 10000.0 ** (-2.0 / 64)
    args = [rxd.ptr, ryd.ptr, (C.c_int, ne0), (C.c_int, ne1), (C.c_int, 0), (C.c_int, 0), (C.c_int, 64), rpd.ptr,
            (C.c_float, 1.0), (C.c_int, 0), (C.c_float, 0.0), (C.c_float, 1.0), (C.c_float, 0.0), (C.c_float, ts)]
    assert _launch(hip, "rope_neox<true>", (ne1, 2, 1), (64, 1, 1), args) == 0
    ok, err = close(ryd.get(np.float32), po.rope_neox(rx, pos, ne0, ne1, 64, 2, ts, 1.0), rtol=0, atol=2e-5)
    assert ok, err
    # get_rows_f32(table, int32 idx, fp32 dst, dim): vocab and rows from the allocation sizes
    tab = rng.standard_normal((30, 16)).astype(np.float32)
    idx = np.array([4, 29, 0, 31], np.int32)
    td, idd, od = Dev(hip, tab), Dev(hip, idx), Dev(hip, nbytes=4 * 16 * 4)
    assert _launch(hip, "k_get_rows_float<float, float>", (4, 1, 1), (16, 1, 1), [td.ptr, idd.ptr, od.ptr,
                                                                                (C.c_int, 16)]) == 0
    assert np.array_equal(od.get(np.float32).reshape(4, 16), po.embedding(tab, idx))
