"""Dequant kernels (vkflame_dispatch_dequant) against the reference shaders.

Bit-exact: the golden vectors were produced by the reference's own GLSL
(tests/golden/gen_golden.py); larger random cases are checked against the C
oracle, which the CPU suite pins to the same golden vectors.
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


@pytest.mark.parametrize("q", range(8))
@pytest.mark.parametrize("kind", ["dq", "dqe"])
def test_dequant_golden(rt, golden, q, kind):
    name = S.NAMES[q]
    raw = golden[f"{kind}_{name}_in"]
    exp = golden[f"{kind}_{name}_out"]
    nb = raw.size // S.BLOCK_BYTES[q]
    src = G.dev(raw)
    dst = G.empty(exp.size * 4)
    rt.dequant(src.data_ptr(), dst.data_ptr(), nb, q)
    got = G.host(dst, np.float32)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("q", range(8))
@pytest.mark.parametrize("nb_extra", [0, 3])
def test_dequant_random_vs_oracle(rt, q, nb_extra):
    qk = S.BLOCK_VALUES[q]
    raw = S.quant_matrix(q, 37, 1024, seed=q).ravel()
    nb = raw.size // S.BLOCK_BYTES[q] - nb_extra  # ragged block counts
    exp = po.dequant(q, raw, nb)
    src = G.dev(raw)
    dst = G.empty(nb * qk * 4 + 64)
    rt.dequant(src.data_ptr(), dst.data_ptr(), nb, q)
    got = G.host(dst, np.float32)
    assert np.array_equal(got[: nb * qk].view(np.uint32), exp.view(np.uint32))
    assert (got[nb * qk:].view(np.uint32) == 0xFFFFFFFF).all(), "wrote past the end"


@pytest.mark.parametrize("q", [S.Q4_0, S.Q8_0, S.Q4_K, S.Q6_K])
def test_dequant_suballocation_offsets(rt, q):
    """Pointers inside a larger allocation (the reference only resolved block
    bases, shim/hip_runtime_shim.cpp:875-881): src at +2 bytes, dst at +4."""
    raw = S.quant_matrix(q, 4, 512, seed=9).ravel()
    nb = raw.size // S.BLOCK_BYTES[q]
    buf = G.dev(np.concatenate([np.zeros(2, np.uint8), raw]))
    dst = G.empty(nb * S.BLOCK_VALUES[q] * 4 + 4)
    rt.dequant(buf.data_ptr() + 2, dst.data_ptr() + 4, nb, q)
    got = G.host(dst, np.uint8)[4:].view(np.float32)
    assert np.array_equal(got.view(np.uint32), po.dequant(q, raw, nb).view(np.uint32))


def test_dequant_rejects_bad_args(rt):
    src = G.empty(64)
    with pytest.raises(rt.VkflameError):
        rt.dequant(src.data_ptr(), src.data_ptr(), 1, 99)
    with pytest.raises(rt.VkflameError):
        rt.dequant(0, src.data_ptr(), 1, S.Q4_0)


def test_quantize_q8_1_bit_exact(rt):
    x = S.normal_f32((7, 512), seed=11)
    x[0, :32] = 0.0  # all-zero block: d = 0, q = 0
    x[1, 5] = 1e6    # one outlier block
    exp = po.quantize_q8_1(x)
    xd = G.dev(x)
    yd = G.empty(exp.size)
    rt.quantize_q8_1(xd.data_ptr(), yd.data_ptr(), 7, 512, 512)
    assert np.array_equal(G.host(yd, np.uint8), exp.ravel())


def test_quantize_q8_1_ties_and_config4_size(rt):
    """Quotients exactly on and next to half-integers (where a reciprocal
    product could round differently from the IEEE division), several scale
    regimes, and the config 4 activation size: bit-exact with the oracle."""
    M, K = 512, 5120
    x = S.normal_f32((M, K), seed=21)
    # row 0: amax 127 -> d = 1 exactly; values k + 0.5 are ties for roundf
    x[0, :] = np.resize(np.arange(-126.5, 127.0, 1.0, dtype=np.float32), K)
    x[0, ::32] = 127.0
    # row 1: amax 254 -> d = 2; values 2k + 1 are ties
    x[1, :] = np.resize(np.arange(-253.0, 254.0, 2.0, dtype=np.float32), K)
    x[1, ::32] = 254.0
    # row 2: ties one ulp either side
    t = np.resize(np.arange(-120.5, 121.0, 1.0, dtype=np.float32), K)
    x[2, :] = np.where(np.arange(K) % 2 == 0, np.nextafter(t, np.float32(np.inf)), np.nextafter(t, np.float32(-np.inf)))
    x[2, ::32] = 127.0
    x[3:8] *= np.float32(1e-3)
    x[8:12] *= np.float32(3e4)
    exp = po.quantize_q8_1(x)
    xd = G.dev(x)
    yd = G.empty(exp.size)
    rt.quantize_q8_1(xd.data_ptr(), yd.data_ptr(), M, K, K)
    assert np.array_equal(G.host(yd, np.uint8), exp.ravel())
