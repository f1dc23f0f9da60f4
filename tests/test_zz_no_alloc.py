"""The allocation-free decode GEMV entry point, vkflame_quant_linear_noalloc.

It exists for callers that may not allocate device memory (allocator
callbacks, processes that reserve all device memory up front, runtimes that
forbid allocation after start-up): it keeps its scratch in a fixed array
inside the library instead of allocating per-stream arenas.  These tests call
it through the C ABI and compare it with the regular entry point,
vkflame_quant_linear, on the same inputs, twice in a row (the shared scratch
keeps the previous call's contents, which must not leak into the next).

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from tests import gpu_util as G
from vkflame_b200 import synth as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from vkflame_b200 import rt
    rt.lib()
    return rt


@pytest.mark.parametrize("q,K,N,M", [(S.Q4_K, 5120, 13824, 1), (S.Q6_K, 2048, 1000, 3), (S.Q8_0, 1024, 200, 8)])
def test_noalloc_matches_regular_entry_point(rt, q, K, N, M):
    lib = rt.lib()
    for call in range(2):  # two calls in a row on the shared scratch
        w = S.quant_matrix(q, N, K, seed=100 * call + q)
        x = S.normal_f16((M, K), seed=call + 7)
        wd, xd = G.dev(w), G.dev(x)
        y_ref = G.empty(M * N * 4)
        y_new = G.empty(M * N * 4)
        rt.quant_linear(wd.data_ptr(), q, xd.data_ptr(), rt.X_F16, y_ref.data_ptr(), rt.Y_F32, M, N, K, K, N)
        rc = lib.vkflame_quant_linear_noalloc(wd.data_ptr(), q, xd.data_ptr(), y_new.data_ptr(), rt.Y_F32, M, N, K,
                                              K, N, None)
        assert rc == 0, rt.STATUS.get(rc, rc)
        ref = G.host(y_ref, np.float32, (M, N)).astype(np.float64)
        got = G.host(y_new, np.float32, (M, N)).astype(np.float64)
        rt.check_kernel_errors()
        assert G.normwise_err(got, ref) < 1e-4
        assert np.array_equal(got, ref)  # same kernel and schedule: identical bits


def test_noalloc_rejects_sizes_beyond_its_scratch(rt):
    lib = rt.lib()
    buf = G.empty(1 << 20)
    p = buf.data_ptr()
    assert lib.vkflame_quant_linear_noalloc(p, S.Q4_K, p, p, rt.Y_F32, 9, 16, 256, 256, 16, None) != 0  # M > 8
    assert lib.vkflame_quant_linear_noalloc(p, S.Q4_K, p, p, rt.Y_F32, 1, 300000, 256, 256, 300000, None) != 0
    assert lib.vkflame_quant_linear_noalloc(p, S.Q4_K, p, p, rt.Y_F32, 8, 16, 13824, 13824, 16, None) != 0
