"""GGUF container: write and read back (metadata of every value kind,
tensor table, alignment of the data section and of every tensor), the
link plan of the GGUF-driven stack, and rejection of damaged files."""
import numpy as np
import pytest

from tests import gguf_model
from vkflame_b200 import gguf, stack
from vkflame_b200 import synth as S


def test_roundtrip(tmp_path):
    p = tmp_path / "m.gguf"
    tensors = gguf_model.make(p, layers=2)
    g = gguf.read(p)
    try:
        assert g.version == 3
        assert g.metadata["general.architecture"] == "qwen2"
        assert g.metadata["qwen2.block_count"] == 2
        assert abs(g.metadata["qwen2.rope.freq_base"] - 1e6) < 1
        assert g.metadata["tokenizer.ggml.tokens"] == ["<a>", "<b>"]
        assert g.data_offset % 32 == 0
        assert [t[0] for t in tensors] == list(g.tensors)
        for name, dims, gt, data in tensors:
            info = g.tensors[name]
            assert info.dims == tuple(dims) and info.ggml_type == gt and info.offset % 32 == 0
            assert np.array_equal(g.tensor_bytes(name), np.ascontiguousarray(data).view(np.uint8).ravel())
        kind, K, N, rows = g.weight("blk.1.ffn_down.weight")
        assert (kind, K, N, rows.shape) == (S.Q6_K, 1280, 512, (512, 1280 // 256 * 210))
    finally:
        g.close()


def test_alignment_option(tmp_path):
    p = tmp_path / "a.gguf"
    w = S.quant_matrix(S.Q4_K, 3, 256, seed=1)
    gguf.write(p, {"general.architecture": "llama"}, [("x", (256, 3), gguf.GGML_Q4_K, w),
                                                     ("y", (256, 3), gguf.GGML_Q4_K, w)], alignment=64)
    g = gguf.read(p)
    assert g.metadata["general.alignment"] == 64 and g.data_offset % 64 == 0
    assert g.tensors["y"].offset == 448  # 432 bytes rounded up to 64
    assert np.array_equal(g.tensor_bytes("y"), w.ravel())
    g.close()


def test_stack_plan(tmp_path):
    p = tmp_path / "m.gguf"
    gguf_model.make(p, layers=3, hidden=512, heads=4, kv_heads=2, head_dim=128, ffn=1280, vocab=2048)
    g = gguf.read(p)
    links = stack.plan(g)
    g.close()
    names = [l[0] for l in links]
    assert names[:5] == ["0.qk", "0.v", "0.o", "0.gate_up", "0.down"] and names[-1] == "head"
    assert len(links) == 3 * 5 + 1
    qk = links[0]
    assert qk[1:4] == (S.Q4_K, 512, 512 + 256) and qk[5] is None
    assert links[5][5] == "0.down" and links[-1][5] == "2.down"
    assert links[3][1:4] == (S.Q4_K, 512, 2 * 1280) and links[4][1:4] == (S.Q6_K, 1280, 512)


def test_rejects_damaged_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(ValueError):
        gguf.read(p)
    q = tmp_path / "trunc.gguf"
    gguf_model.make(q, layers=1)
    data = q.read_bytes()
    q.write_bytes(data[:len(data) // 2])
    with pytest.raises(ValueError):
        gguf.read(q)
