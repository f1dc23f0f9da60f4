"""Column sharding of the stack over ranks (the multi-GPU path of the
benchmark), run as world-size-2 gloo process groups on the CPU: each rank
computes its row slice of a quantised linear with the CPU reference, the
slices are all-gathered, and the joined result must equal the unsharded
computation bit for bit (the per-row arithmetic does not depend on the
split)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from vkflame_b200 import shard
from vkflame_b200 import synth as S


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, N, K, M, out):
    import torch
    import torch.distributed as dist
    from oracle import pyoracle as po
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = S.quant_matrix(q, N, K, seed=11)
        x = S.normal_f16((M, K), seed=12)
        ws = shard.shard_bytes(w, N, world, rank)
        n = N // world
        y = po.quant_linear(q, ws, x, M, n, K, xtype=0, ytype=0, threads=1)  # fp32 [M, n]
        gathered = torch.empty((world * M, n), dtype=torch.float32)  # concatenated form (gloo)
        dist.all_gather_into_tensor(gathered, torch.from_numpy(np.ascontiguousarray(y, np.float32)))
        if rank == 0:
            out.put(shard.join_gathered(gathered.numpy().reshape(world, M, n)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("q,N,K,M", [(S.Q4_K, 256, 512, 1), (S.Q6_K, 128, 256, 3)])
def test_sharded_gather_equals_unsharded(q, N, K, M):
    from oracle import pyoracle as po
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, N, K, M, out)) for r in range(world)]
    for p in procs:
        p.start()
    got = out.get(timeout=60)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w = S.quant_matrix(q, N, K, seed=11)
    x = S.normal_f16((M, K), seed=12)
    ref = po.quant_linear(q, w, x, M, N, K, xtype=0, ytype=0, threads=1)
    assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(ref, np.float32).view(np.uint32))


def test_row_ranges_cover_stack_shapes():
    # every linear of the 14B stack divides over 1, 2, 4 and 8 ranks
    for N in (5120, 1024, 5120 + 1024, 2 * 13824, 152064):
        for world in (1, 2, 4, 8):
            ranges = [shard.row_range(N, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    with pytest.raises(ValueError):
        shard.row_range(1000, 3, 0)


def test_join_gathered_layout():
    g = np.arange(2 * 3 * 4).reshape(2, 3, 4)
    j = shard.join_gathered(g)
    assert j.shape == (3, 8)
    assert (j[:, :4] == g[0]).all() and (j[:, 4:] == g[1]).all()


def test_gathered_word_layout_unpack():
    """{fp16 pair, epoch} words: buffer epoch & 1 of step `epoch`, values in
    column order; a word of another step is rejected."""
    from vkflame_b200.gather import unpack
    y = np.arange(8, dtype=np.float16).reshape(1, 8) * np.float16(0.5)
    words = np.zeros((2, 1, 4, 2), np.int32)
    words[1, 0, :, 0] = y.view(np.int32).reshape(-1)
    words[1, 0, :, 1] = 3
    assert np.array_equal(unpack(words, 3).view(np.uint16), y.view(np.uint16))
    words[1, 0, 2, 1] = 1
    with pytest.raises(ValueError):
        unpack(words, 3)


def _gather_group_main(rank, world, port, out):
    """Host side of the NVLink gather set-up on gloo (CPU tensors, fake IPC):
    handle exchange order, one mapping per peer allocation, word offsets of
    each rank's slice, parity strides, per-call-site counters."""
    import torch
    import torch.distributed as dist
    from vkflame_b200 import gather, rt
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    opened = []
    # fake IPC: a handle names (rank, allocation base); "opening" maps rank
    # q's allocation to 10**12 * (q + 1) + its base in this process
    rt.ipc_handle = lambda ptr: (f"{rank}:{ptr}".encode().ljust(64, b"\0"), 0)

    def fake_open(h):
        q, base = h.rstrip(b"\0").decode().split(":")
        opened.append(h)
        return 10**12 * (int(q) + 1) + int(base)
    rt.ipc_open = fake_open
    rt.ipc_close = lambda base: None
    try:
        gg = gather.GatherGroup(dist, world, rank, device="cpu")
        ya, yb = gg.buffer(1024), gg.buffer(256)
        ga, gb = gg.op(ya), gg.op(yb, x=ya)
        out.put((rank, [ya.ptrs, yb.ptrs], [ya.tensor.data_ptr(), yb.tensor.data_ptr()],
                 [list(ga.y_rank)[:world], list(gb.y_rank)[:world]], ga.stride, gb.stride,
                 ga.x_gathered, gb.x_gathered, gb.x_stride, ga.epoch != gb.epoch, len(opened)))
    finally:
        dist.destroy_process_group()


def test_gather_group_host_logic_two_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_group_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = out.get(timeout=60)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, (_, ptrs, own, yr, sa, sb, xa, xb, xsb, distinct, nopen) in res.items():
        peer = 1 - rank
        for i, (n_full) in enumerate((1024, 256)):
            assert ptrs[i][rank] == own[i]                                   # own buffer, unmapped
            assert ptrs[i][peer] == 10**12 * (peer + 1) + res[peer][2][i]    # the peer's buffer, mapped
            r0 = shard.row_range(n_full, world, rank)[0]
            assert yr[i] == [p + (r0 // 2) * 8 for p in ptrs[i]]             # this rank's first word everywhere
        assert (sa, sb) == (1024 // 2 * 8, 256 // 2 * 8)                    # buffer 0 -> buffer 1, one row
        assert (xa, xb, xsb) == (0, 1, 1024 // 2 * 8)
        assert distinct                                                      # one run counter per call site
        assert nopen == 2                                                    # each peer allocation opened once
