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


_FRESH = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from vkflame_b200 import rt, synth as S
lib = rt.load()  # no vkflame_init: this process touches nothing but the allocation-free entry point first
q, N, K, M = S.Q4_K, 4096, 5120, 1
ws = [torch.from_numpy(S.quant_matrix(q, N, K, seed=s).reshape(-1).copy()).cuda() for s in (1, 2)]
xs = [torch.from_numpy(S.normal_f16((M, K), seed=s).view(np.uint8).reshape(-1).copy()).cuda() for s in (3, 4)]
ys = [torch.zeros(M * N, dtype=torch.float32, device="cuda") for _ in range(3)]
torch.cuda.synchronize()
def call(w, x, y):
    return lib.vkflame_quant_linear_noalloc(w.data_ptr(), q, x.data_ptr(), y.data_ptr(), rt.Y_F32, M, N, K, K, N, None)
assert call(ws[0], xs[0], ys[0]) == 0   # first call: looks up the scratch address, loads the kernel
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
assert call(ws[1], xs[1], ys[1]) == 0
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
assert free1 == free0, (free0, free1)
assert lib.vkflame_check_kernel_errors() == 0
torch.cuda.synchronize()
assert torch.cuda.mem_get_info()[0] == free0  # checking errors allocated nothing either
rt.quant_linear(ws[1].data_ptr(), q, xs[1].data_ptr(), rt.X_F16, ys[2].data_ptr(), rt.Y_F32, M, N, K, K, N)
torch.cuda.synchronize()
assert torch.equal(ys[1], ys[2])
print("NOALLOC_FRESH_OK")
"""


def test_noalloc_first_in_a_fresh_process_allocates_nothing():
    """In a new process whose first vkflame call is the allocation-free entry
    point, a second call leaves the device's free memory unchanged (after the
    first call has loaded the module), the error check allocates nothing, and
    the result equals the regular entry point's bit for bit."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, "-c", _FRESH, str(root)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "NOALLOC_FRESH_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
