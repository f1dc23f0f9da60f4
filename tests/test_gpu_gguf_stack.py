"""The GGUF-driven linear stack (vkflame_b200/stack.py) on a small synthetic
Qwen2-layout model file: two decode steps through the per-token chain
kernel; every link's gathered output within the fp tolerance of the fp64
product of the oracle's dequantised weights (read back from the file) and
the link's actual input."""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests import gguf_model
from tests import gpu_util as G

pytestmark = pytest.mark.gpu


def test_gguf_stack_two_steps(tmp_path):
    from vkflame_b200 import gguf, rt
    from vkflame_b200.stack import GGUFStack
    rt.lib()
    p = tmp_path / "m.gguf"
    gguf_model.make(p, layers=2, d_range=(1e-5, 5e-5))  # values stay finite through 11 chained links
    st = GGUFStack(p)
    try:
        hidden = st.x.shape[1]
        for step in range(2):
            x = np.random.default_rng(step).standard_normal(hidden).astype(np.float16)
            st.step(x)
            import torch
            torch.cuda.synchronize()
            assert st.chain.status() == [0, 0, 0, 0], st.chain.status()
            rt.check_kernel_errors()
            outs = {name: st.output(name) for name, *_ in st.links}
            for name, kind, K, N, tensors, src in st.links:
                xin = x.reshape(1, -1) if src is None else outs[src][:, :K]
                w = np.concatenate([po.dequant(kind, st.file.weight(t)[3], st.file.weight(t)[2] * K // 256)
                                    .reshape(-1, K) for t in tensors])
                ref = xin.astype(np.float64) @ w.astype(np.float64).T
                assert np.isfinite(outs[name]).all(), (step, name)
                assert G.normwise_err(outs[name].astype(np.float64), ref) < G.REL_TOL, (step, name)
        assert outs["head"].shape == (1, 2048)
    finally:
        st.close()
