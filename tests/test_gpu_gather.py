"""Column-sharded decode GEMV fused with the all-gather
(vkflame_quant_linear_gather), on 2 GPUs: two ranks (one process each, NCCL
only for the handle exchange) run a 2-linear chain whose second linear reads
the first's gathered output ({fp16 pair, epoch} words), for several steps
(both buffer parities; each call site's run count advanced by its kernel).  Checks: every rank's
gathered buffers are identical bit for bit, and equal the unsharded product
within the fp tolerance (fp64 reference from the oracle's dequant)."""
from __future__ import annotations

import os
import tempfile

import numpy as np
import pytest

from oracle import pyoracle as po
from tests import gpu_util as G
from vkflame_b200 import synth as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from vkflame_b200 import rt as _rt
    _rt.lib()
    return _rt

KA, NA, KB, NB = 1024, 512, 512, 256   # linear A: Q4_K 1024 -> 512; linear B: Q8_0 512 -> 256 (X = A's output)
STEPS = 3


def _worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    from vkflame_b200 import rt, shard
    from vkflame_b200.gather import GatherGroup, unpack
    rt.lib()
    wa = S.quant_matrix(S.Q4_K, NA, KA, seed=5)
    wb = S.quant_matrix(S.Q8_0, NB, KB, seed=6)
    x = S.normal_f16((1, KA), seed=7)
    a0, a1 = shard.row_range(NA, world, rank)
    b0, b1 = shard.row_range(NB, world, rank)
    wad = torch.from_numpy(np.ascontiguousarray(shard.shard_bytes(wa, NA, world, rank)).view(np.uint8).ravel()).cuda()
    wbd = torch.from_numpy(np.ascontiguousarray(shard.shard_bytes(wb, NB, world, rank)).view(np.uint8).ravel()).cuda()
    xd = torch.from_numpy(x.view(np.uint16).astype(np.int16)).cuda().view(torch.float16)
    # Load both kernels on this rank before the ranks wait on one another
    # (lazy module loading of a first launch can delay one rank by more than
    # the kernels' bounded waits): the same calls at world size 1, locally.
    lg = GatherGroup(None, 1, 0)
    la, lb = lg.buffer(NA), lg.buffer(NB)
    rt.quant_linear_gather(wad.data_ptr(), S.Q4_K, xd.data_ptr(), rt.Y_F16, 1, a1 - a0, KA, KA, a1 - a0, 0,
                           lg.op(la), 0)
    rt.quant_linear_gather(wbd.data_ptr(), S.Q8_0, xd.data_ptr(), rt.Y_F16, 1, b1 - b0, KB, KA, b1 - b0, 0,
                           lg.op(lb), 0)
    torch.cuda.synchronize()
    rt.check_kernel_errors()
    gg = GatherGroup(dist, world, rank)
    ya = gg.buffer(NA)
    yb = gg.buffer(NB)
    ga = gg.op(ya)                    # X: the replicated input row
    gb = gg.op(yb, x=ya)              # X: A's gathered output
    torch.cuda.synchronize()
    dist.barrier()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(STEPS):
            rt.quant_linear_gather(wad.data_ptr(), S.Q4_K, xd.data_ptr(), rt.Y_F16, 1, a1 - a0, KA, KA, NA,
                                   rt.FLAG_STATIC_WEIGHTS, ga, s.cuda_stream)
            rt.quant_linear_gather(wbd.data_ptr(), S.Q8_0, ya.tensor.data_ptr(), rt.Y_F16, 1, b1 - b0, KB, NA, NB,
                                   rt.FLAG_STATIC_WEIGHTS, gb, s.cuda_stream)
    torch.cuda.synchronize()
    rt.check_kernel_errors()
    assert [int(e.item()) for e in gg.epochs] == [STEPS, STEPS]
    ya_h = unpack(ya.tensor.cpu().numpy(), STEPS)
    yb_h = unpack(yb.tensor.cpu().numpy(), STEPS)
    np.save(os.path.join(outdir, f"ya{rank}.npy"), ya_h)
    np.save(os.path.join(outdir, f"yb{rank}.npy"), yb_h)
    dist.barrier()
    gg.close()
    dist.destroy_process_group()


def test_quant_linear_gather_two_ranks():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, 29555, d), nprocs=world, join=True)
        ya = [np.load(os.path.join(d, f"ya{r}.npy")) for r in range(world)]
        yb = [np.load(os.path.join(d, f"yb{r}.npy")) for r in range(world)]
    assert all(np.array_equal(ya[0].view(np.uint16), t.view(np.uint16)) for t in ya)
    assert all(np.array_equal(yb[0].view(np.uint16), t.view(np.uint16)) for t in yb)
    wa = po.dequant(S.Q4_K, S.quant_matrix(S.Q4_K, NA, KA, seed=5), NA * KA // 256).reshape(NA, KA)
    wb = po.dequant(S.Q8_0, S.quant_matrix(S.Q8_0, NB, KB, seed=6), NB * KB // 32).reshape(NB, KB)
    x = S.normal_f16((1, KA), seed=7).astype(np.float64)
    ref_a = x @ wa.astype(np.float64).T
    assert G.normwise_err(ya[0].astype(np.float64), ref_a) < G.REL_TOL
    ref_b = ya[0].astype(np.float64)[:, :KB] @ wb.astype(np.float64).T
    assert G.normwise_err(yb[0].astype(np.float64), ref_b) < G.REL_TOL


def test_quant_linear_gather_world1_matches_gemv_bitwise(rt):
    """World size 1 (no peers): the gathered words hold exactly the plain
    GEMV's fp16 outputs, over two runs (both buffer parities), with the
    second linear reading the first's gathered output."""
    import torch
    from vkflame_b200.gather import GatherGroup, unpack
    wa = G.dev(S.quant_matrix(S.Q4_K, NA, KA, seed=5))
    wb = G.dev(S.quant_matrix(S.Q6_K, NB, KB, seed=8))
    x = G.dev(S.normal_f16((1, KA), seed=7))
    gg = GatherGroup(None, 1, 0)
    ya, yb = gg.buffer(NA), gg.buffer(NB)
    ga, gb = gg.op(ya), gg.op(yb, x=ya)
    for step in (1, 2):
        rt.quant_linear_gather(wa.data_ptr(), S.Q4_K, x.data_ptr(), rt.Y_F16, 1, NA, KA, KA, NA, 0, ga)
        rt.quant_linear_gather(wb.data_ptr(), S.Q6_K, ya.tensor.data_ptr(), rt.Y_F16, 1, NB, KB, NA, NB, 0, gb)
        torch.cuda.synchronize()
        rt.check_kernel_errors()
        a = unpack(ya.tensor.cpu().numpy(), step)
        b = unpack(yb.tensor.cpu().numpy(), step)
        ref_a = G.empty(NA * 2)
        rt.quant_linear_ex(wa.data_ptr(), S.Q4_K, x.data_ptr(), rt.X_F16, ref_a.data_ptr(), rt.Y_F16, 1, NA, KA, KA,
                           NA, 0)
        xa = torch.from_numpy(a.view(np.int16).copy()).cuda()
        ref_b = G.empty(NB * 2)
        rt.quant_linear_ex(wb.data_ptr(), S.Q6_K, xa.data_ptr(), rt.X_F16, ref_b.data_ptr(), rt.Y_F16, 1, NB, KB, NA,
                           NB, 0)
        assert np.array_equal(a.view(np.uint16).ravel(), G.host(ref_a, np.uint16))
        assert np.array_equal(b.view(np.uint16).ravel(), G.host(ref_b, np.uint16))


def test_quant_linear_gather_rejects_bad_args(rt):
    from vkflame_b200.gather import GatherGroup
    w = G.dev(S.quant_matrix(S.Q4_K, 64, 512, seed=1))
    x = G.dev(S.normal_f16((2, 512), seed=2))
    gg = GatherGroup(None, 1, 0)
    y = gg.buffer(64)
    g = gg.op(y)
    bad = [dict(M=2), dict(ytype=rt.Y_F32), dict(N=63), dict(X=x.data_ptr() + 2)]
    for b in bad:
        a = dict(W=w.data_ptr(), wtype=S.Q4_K, X=x.data_ptr(), ytype=rt.Y_F16, M=1, N=64, K=512, ldx=512, ldy=64)
        a.update(b)
        with pytest.raises(rt.VkflameError):
            rt.quant_linear_gather(a["W"], a["wtype"], a["X"], a["ytype"], a["M"], a["N"], a["K"], a["ldx"], a["ldy"],
                                   0, g)
