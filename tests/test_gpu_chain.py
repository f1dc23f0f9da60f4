"""The persistent per-token decode kernel (vkflame_chain_*): a chain of
quantised linears, each reading an earlier one's gathered output, run as one
cooperative launch.  Checks, over several runs (both buffer parities): every
gathered output is within the fp tolerance of the fp64 product of the
oracle's dequantised weights and the chain's own (unpacked) input, and agrees
with the per-linear decode GEMV (vkflame_quant_linear_ex) on the same input
to fp32 summation-order level; the run count advances once per run; the
plain-output form (world size 1) matches too; and on 2 GPUs the sharded
chain's gathered buffers are identical on both ranks."""
from __future__ import annotations

import os
import tempfile

import numpy as np
import pytest

from oracle import pyoracle as po
from tests import gpu_util as G
from vkflame_b200 import synth as S

pytestmark = pytest.mark.gpu

# (format, K, N, source of X: -1 = the plain input row, else an earlier link)
# Rows over 4400 bytes (links 5 and 6) are cut into K-ranges (items of
# several row copies); link 1's 100-row shards at 2 ranks end in a partial
# 16-row block.
LINKS = [(S.Q4_K, 1024, 768, -1),   # 0: reads the input (K 1024)
         (S.Q6_K, 1024, 200, -1),   # 1: same input, another format
         (S.Q4_K, 512, 1024, 0),    # 2: reads link 0's output (first 512 values)
         (S.Q6_K, 1024, 512, 2),    # 3: reads link 2
         (S.Q5_K, 512, 8192, 3),    # 4: reads link 3
         (S.Q6_K, 5632, 512, 4),    # 5: reads link 4 (Q6_K rows of 4620 bytes)
         (S.Q4_K, 8192, 256, 4)]    # 6: reads link 4 (Q4_K rows of 4608 bytes)
RUNS = 3


def _drange(q):
    """Block scales small enough that the chain's values stay finite in fp16
    (with the benchmark's U[1e-3, 1e-2] each link grows them ~100x)."""
    return (2e-5, 1e-4)


@pytest.fixture(scope="module")
def rt():
    from vkflame_b200 import rt as _rt
    _rt.lib()
    return _rt


def _weights():
    return [S.quant_matrix(q, N, K, seed=40 + i, d_range=_drange(q)) for i, (q, K, N, _) in enumerate(LINKS)]


def _dq(q, w, N, K):
    return po.dequant(q, w, N * K // 256).reshape(N, K).astype(np.float64)


def test_chain_world1_matches_fp64_and_gemv(rt):
    import torch
    from vkflame_b200.gather import GatherGroup, unpack
    ws = _weights()
    x = S.normal_f16((1, 1024), seed=9)
    wd = [G.dev(w) for w in ws]
    xd = G.dev(x)
    gg = GatherGroup(None, 1, 0)
    outs = [gg.buffer(N) for _, _, N, _ in LINKS]
    links = [gg.chain_linear(wd[i].data_ptr(), q, K, N, outs[i], x_src=src, x_plain=xd.data_ptr() if src < 0 else 0)
             for i, (q, K, N, src) in enumerate(LINKS)]
    ch = rt.Chain(links, 1, 0)
    try:
        for run in range(1, RUNS + 1):
            ch.run(0)
            torch.cuda.synchronize()
            assert ch.status() == [0, 0, 0, 0], ch.status()
            rt.check_kernel_errors()
            assert ch.epoch() == run
            ys = [unpack(o.tensor.cpu().numpy(), run) for o in outs]
            for i, (q, K, N, src) in enumerate(LINKS):
                assert np.isfinite(ys[i]).all(), (run, i)
                xin = x if src < 0 else ys[src][:, :K]
                ref = xin.astype(np.float64) @ _dq(q, ws[i], N, K).T
                got = ys[i].astype(np.float64)
                assert G.normwise_err(got, ref) < G.REL_TOL, (run, i)
                # the per-linear GEMV on the same input
                xg = G.dev(np.ascontiguousarray(xin.astype(np.float16)))
                yg = G.empty(N * 2)
                rt.quant_linear_ex(wd[i].data_ptr(), q, xg.data_ptr(), rt.X_F16, yg.data_ptr(), rt.Y_F16, 1, N, K, K,
                                   N, 0)
                gem = G.host(yg, np.float16).astype(np.float64)
                assert G.normwise_err(got.ravel(), gem) < 1e-3, (run, i)
    finally:
        ch.close()


def test_chain_world1_plain_outputs(rt):
    """Independent links with plain fp16 outputs (the weight-streaming form)."""
    import torch
    from vkflame_b200.gather import GatherGroup
    q_k_n = [(S.Q4_K, 1024, 512), (S.Q6_K, 1024, 1536), (S.Q5_K, 1024, 96)]
    ws = [S.quant_matrix(q, N, K, seed=70 + i) for i, (q, K, N) in enumerate(q_k_n)]
    x = S.normal_f16((1, 1024), seed=3)
    wd, xd = [G.dev(w) for w in ws], G.dev(x)
    ys = [G.empty(N * 2) for _, _, N in q_k_n]
    gg = GatherGroup(None, 1, 0)
    links = [gg.chain_linear(wd[i].data_ptr(), q, K, N, None, x_plain=xd.data_ptr(), y_plain=ys[i].data_ptr())
             for i, (q, K, N) in enumerate(q_k_n)]
    ch = rt.Chain(links)
    try:
        for _ in range(2):
            ch.run(0)
            torch.cuda.synchronize()
            rt.check_kernel_errors()
            for i, (q, K, N) in enumerate(q_k_n):
                ref = x.astype(np.float64) @ _dq(q, ws[i], N, K).T
                assert G.normwise_err(G.host(ys[i], np.float16).astype(np.float64), ref.ravel()) < G.REL_TOL
    finally:
        ch.close()


def test_chain_rejects_bad_links(rt):
    from vkflame_b200.gather import GatherGroup
    w = G.dev(S.quant_matrix(S.Q4_K, 64, 512, seed=1))
    x = G.dev(S.normal_f16((1, 512), seed=2))
    gg = GatherGroup(None, 1, 0)
    out = gg.buffer(64)
    ok = gg.chain_linear(w.data_ptr(), S.Q4_K, 512, 64, out, x_plain=x.data_ptr())
    bad = [dict(wtype=S.Q8_0), dict(K=500), dict(x_src=0), dict(x_plain=x.data_ptr() + 2)]
    for b in bad:
        c = gg.chain_linear(w.data_ptr(), S.Q4_K, 512, 64, out, x_plain=x.data_ptr())
        for k, v in b.items():
            setattr(c, k, v)
        with pytest.raises(rt.VkflameError):
            rt.Chain([c])
    rt.Chain([ok]).close()


def _worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    from vkflame_b200 import rt, shard
    from vkflame_b200.gather import GatherGroup, unpack
    rt.lib()
    ws = _weights()
    x = S.normal_f16((1, 1024), seed=9)
    xd = G.dev(x)
    gg = GatherGroup(dist, world, rank)
    outs = [gg.buffer(N) for _, _, N, _ in LINKS]
    wd, links = [], []
    for i, (q, K, N, src) in enumerate(LINKS):
        wd.append(G.dev(np.ascontiguousarray(shard.shard_bytes(ws[i], N, world, rank))))
        links.append(gg.chain_linear(wd[-1].data_ptr(), q, K, N // world, outs[i], x_src=src,
                                     x_plain=xd.data_ptr() if src < 0 else 0))
    ch = rt.Chain(links, world, rank)
    torch.cuda.synchronize()
    dist.barrier()
    s = torch.cuda.Stream()
    for _ in range(RUNS):
        ch.run(s.cuda_stream)
    torch.cuda.synchronize()
    assert ch.status() == [0, 0, 0, 0], ch.status()
    rt.check_kernel_errors()
    assert ch.epoch() == RUNS
    for i, o in enumerate(outs):
        np.save(os.path.join(outdir, f"y{i}_{rank}.npy"), unpack(o.tensor.cpu().numpy(), RUNS))
    dist.barrier()
    ch.close()
    gg.close()
    dist.destroy_process_group()


def test_chain_two_ranks():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, 29571, d), nprocs=world, join=True)
        ys = [[np.load(os.path.join(d, f"y{i}_{r}.npy")) for r in range(world)] for i in range(len(LINKS))]
    ws = _weights()
    x = S.normal_f16((1, 1024), seed=9)
    for i, (q, K, N, src) in enumerate(LINKS):
        assert all(np.array_equal(ys[i][0].view(np.uint16), t.view(np.uint16)) for t in ys[i])
        xin = x if src < 0 else ys[src][0][:, :K]
        ref = xin.astype(np.float64) @ _dq(q, ws[i], N, K).T
        assert G.normwise_err(ys[i][0].astype(np.float64), ref) < G.REL_TOL
