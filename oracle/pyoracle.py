"""ctypes front-end of the CPU oracle (test infrastructure only).

Loads ``oracle/_build/liboracle.so`` (the C restatement, oracle.c) and, when
it has been built here, ``oracle/_ref/libvkref.so`` (the reference shaders
compiled as C++ by build_ref.py).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import this module.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = HERE / "_build" / "liboracle.so"
_REF = HERE / "_ref" / "libvkref.so"

_lib = None
_ref = None

BLOCK_VALUES = {0: 32, 1: 32, 2: 32, 3: 32, 4: 256, 5: 256, 6: 256, 7: 32}
BLOCK_BYTES = {0: 18, 1: 20, 2: 34, 3: 22, 4: 144, 5: 176, 6: 210, 7: 36}
SHADER = {0: "dequant_q4_0", 1: "dequant_q4_1", 2: "dequant_q8_0", 3: "dequant_q5_0",
          4: "dequant_q4_k", 5: "dequant_q5_k", 6: "dequant_q6_k", 7: "dequant_q8_1"}


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not _LIB.exists():
            raise RuntimeError(f"oracle library missing: {_LIB} (run `make -C oracle`)")
        _lib = C.CDLL(str(_LIB))
        _lib.oracle_dequant.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64]
        _lib.oracle_quantize_q8_1.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        _lib.oracle_linear_int8_shader.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                                   C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
        _lib.oracle_linear_int8.argtypes = [C.c_void_p] * 5 + [C.c_int] * 4 + [C.c_void_p, C.c_void_p, C.c_int]
        _lib.oracle_linear_fp16_shader.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                                   C.c_int, C.c_void_p]
        _lib.oracle_quant_linear.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                             C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
        _lib.oracle_activation.argtypes = [C.c_int, C.c_float]
        _lib.oracle_activation.restype = C.c_float
    return _lib


def ref_available() -> bool:
    return _REF.exists()


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        if not _REF.exists():
            raise RuntimeError(f"reference shader harness missing: {_REF} (run oracle/build_ref.py)")
        _ref = C.CDLL(str(_REF))
    return _ref


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def dequant(qtype: int, raw: np.ndarray, nb: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw).view(np.uint8)
    out = np.empty(nb * BLOCK_VALUES[qtype], np.float32)
    rc = lib().oracle_dequant(qtype, _p(raw), _p(out), nb)
    assert rc == 0
    return out


def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    out = np.empty(n // 32 * 36, np.uint8)
    lib().oracle_quantize_q8_1(_p(x), _p(out), n)
    return out.reshape(*x.shape[:-1], x.shape[-1] // 32 * 36)


def linear_int8(x, w, sx, sw, bias=None, act=0, want_acc=True, threads=0):
    x = np.ascontiguousarray(x, np.int8)
    w = np.ascontiguousarray(w, np.int8)
    M, K = x.shape
    N = w.shape[0]
    sx = np.ascontiguousarray(sx, np.float32)
    sw = np.ascontiguousarray(sw, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float16)
    acc = np.empty((M, N), np.int32) if want_acc else None
    out = np.empty((M, N), np.float16)
    lib().oracle_linear_int8(_p(x), _p(w), _p(sx), _p(sw), None if b is None else _p(b), act, M, N, K,
                             None if acc is None else _p(acc), _p(out), threads)
    return acc, out


def linear_int8_shader(a_f16, w, w_scale, act_scale, act=0):
    a = np.ascontiguousarray(a_f16, np.float16)
    w = np.ascontiguousarray(w, np.int8)
    M, K = a.shape
    N = w.shape[0]
    out = np.empty((M, N), np.float16)
    lib().oracle_linear_int8_shader(_p(a), _p(w), _p(np.ascontiguousarray(w_scale, np.float32)),
                                    act_scale, act, M, N, K, _p(out))
    return out


def linear_fp16_shader(a, b, act=0):
    a = np.ascontiguousarray(a, np.float16)
    b = np.ascontiguousarray(b, np.float16)
    M, K = a.shape
    N = b.shape[1]
    out = np.empty((M, N), np.float16)
    lib().oracle_linear_fp16_shader(_p(a), _p(b), act, M, N, K, _p(out))
    return out


def quant_linear(wtype, w, x, M, N, K, xtype=0, ytype=0, threads=0):
    """The reference's mul_mat sequence on CPU (see oracle.h)."""
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x)
    y = np.empty((M, N), np.float32 if ytype == 0 else np.float16)
    rc = lib().oracle_quant_linear(wtype, _p(w), xtype, _p(x), ytype, _p(y), M, N, K, threads)
    assert rc == 0, rc
    return y


def activation(act: int, x: float) -> float:
    return lib().oracle_activation(act, x)


# ---- reference shaders run through the shader-as-C++ harness -------------

def _pad4(raw: np.ndarray) -> np.ndarray:
    """The shaders read their source as 32-bit words: pad to a multiple of 4 bytes."""
    raw = np.ascontiguousarray(raw).view(np.uint8).ravel()
    pad = (-raw.size) % 4
    return np.concatenate([raw, np.zeros(pad + 4, np.uint8)]) if pad or True else raw


def ref_dequant(qtype: int, raw: np.ndarray, nb: int) -> np.ndarray:
    """Run the reference's dequant shader; grid per runtime/dispatch.cpp:488-494."""
    src = _pad4(raw)
    dst = np.zeros(nb * BLOCK_VALUES[qtype], np.float32)
    binds = (C.c_void_p * 2)(_p(src), _p(dst))
    pc = np.array([nb], np.uint32)
    small = qtype in (0, 1, 3)
    gx = (nb + 7) // 8 if small else nb
    getattr(ref(), "vkref_" + SHADER[qtype])(binds, C.c_void_p(_p(pc)), gx, 1, 1)
    return dst


def ref_linear_int8(a_f16, w, w_scale, act_scale, act=0):
    """Run kernels/linear_int8.glsl (grid per runtime/dispatch.cpp:320-323)."""
    a = np.ascontiguousarray(a_f16, np.float16)
    w = np.ascontiguousarray(w, np.int8)
    M, K = a.shape
    N = w.shape[0]
    ws = np.ascontiguousarray(w_scale, np.float32)
    bias = np.zeros(N, np.float32)
    out = np.zeros((M, N), np.float16)
    binds = (C.c_void_p * 5)(_p(a), _p(w), _p(bias), _p(ws), _p(out))
    pc = np.zeros(5, np.uint32)
    pc[0], pc[1], pc[2] = M, N, K
    pc[3] = np.array([act_scale], np.float32).view(np.uint32)[0]
    pc[4] = act
    ref().vkref_linear_int8(binds, C.c_void_p(_p(pc)), (N + 15) // 16, (M + 15) // 16, 1)
    return out


def ref_linear_fp16(a, b, act=0, fp32out_shader=False):
    a = np.ascontiguousarray(a, np.float16)
    b = np.ascontiguousarray(b, np.float16)
    M, K = a.shape
    N = b.shape[1]
    out = np.zeros((M, N), np.float16)
    c = np.zeros(1, np.float16)
    binds = (C.c_void_p * 4)(_p(a), _p(b), _p(c), _p(out))
    pc = np.array([M, N, K, act], np.uint32)
    fn = ref().vkref_linear_fp16_fp32out if fp32out_shader else ref().vkref_linear_fp16
    fn(binds, C.c_void_p(_p(pc)), (N + 15) // 16, (M + 15) // 16, 1)
    return out


# ---- the non-matmul kernels of the hipLaunchKernel table -------------------

def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def _sig(name, args, res=None):
    fn = getattr(lib(), name)
    fn.argtypes = args
    fn.restype = res
    return fn


def elementwise(op: int, x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    _sig("oracle_elementwise", [C.c_int, C.c_void_p, C.c_void_p, C.c_int64])(op, _p(x), _p(y), x.size)
    return y


def scale(x, s, b):
    x = _f32(x)
    y = np.empty_like(x)
    _sig("oracle_scale", [C.c_void_p, C.c_void_p, C.c_int64, C.c_float, C.c_float])(_p(x), _p(y), x.size, s, b)
    return y


def binop(op, a, b):
    a, b = _f32(a), _f32(b)
    y = np.empty_like(a)
    _sig("oracle_binop", [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64])(
        op, _p(a), _p(b), _p(y), a.size, b.size)
    return y


def rms_norm_f32(x, eps):
    x = _f32(x)
    y = np.empty_like(x)
    M, N = x.shape
    _sig("oracle_rms_norm_f32", [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float])(_p(x), _p(y), M, N, eps)
    return y


def rms_norm_f16(x, g, eps):
    x = np.ascontiguousarray(x, np.float16)
    g = np.ascontiguousarray(g, np.float16)
    y = np.empty_like(x)
    M, N = x.shape
    _sig("oracle_rms_norm_f16", [C.c_void_p] * 3 + [C.c_int, C.c_int, C.c_float])(_p(x), _p(g), _p(y), M, N, eps)
    return y


def softmax(x):
    x = _f32(x)
    y = np.empty_like(x)
    M, N = x.shape
    _sig("oracle_softmax", [C.c_void_p, C.c_void_p, C.c_int, C.c_int])(_p(x), _p(y), M, N)
    return y


def rope_neox(x, pos, ne0, ne1, n_dims, n_seqs, theta_scale, freq_scale):
    x = _f32(x)
    pos = np.ascontiguousarray(pos, np.int32)
    y = np.empty_like(x)
    _sig("oracle_rope_neox", [C.c_void_p, C.c_void_p, C.c_void_p] + [C.c_int] * 4 + [C.c_float] * 2)(
        _p(x), _p(pos), _p(y), ne0, ne1, n_dims, n_seqs, theta_scale, freq_scale)
    return y


def embedding(w, idx):
    w = np.ascontiguousarray(w)
    idx = np.ascontiguousarray(idx, np.int32)
    V, D = w.shape
    out = np.empty((idx.size, D), w.dtype)
    _sig("oracle_embedding", [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p] + [C.c_int] * 3)(
        _p(w), w.itemsize, _p(idx), _p(out), V, D, idx.size)
    return out


def _u32(*vals):
    """Push-constant words: ints as uint32, floats as their fp32 bits."""
    out = np.zeros(max(4, len(vals)), np.uint32)
    for i, v in enumerate(vals):
        out[i] = np.array([v], np.float32).view(np.uint32)[0] if isinstance(v, float) else v
    return out


def ref_elementwise(op, x):
    """kernels/elementwise_f32.glsl (grid per runtime/dispatch.cpp:519-521)."""
    x = _f32(x).ravel()
    y = np.zeros_like(x)
    pc = _u32(x.size, op)
    ref().vkref_elementwise_f32((C.c_void_p * 2)(_p(x), _p(y)), C.c_void_p(_p(pc)), (x.size + 255) // 256, 1, 1)
    return y


def ref_scale(x, s, b):
    x = _f32(x).ravel()
    y = np.zeros_like(x)
    pc = _u32(x.size, float(s), float(b))
    ref().vkref_scale_f32((C.c_void_p * 2)(_p(x), _p(y)), C.c_void_p(_p(pc)), (x.size + 255) // 256, 1, 1)
    return y


def ref_binop(op, a, b):
    a, b = _f32(a).ravel(), _f32(b).ravel()
    y = np.zeros_like(a)
    pc = _u32(a.size, op, b.size, 0)
    ref().vkref_binop_f32((C.c_void_p * 3)(_p(a), _p(b), _p(y)), C.c_void_p(_p(pc)), (a.size + 255) // 256, 1, 1)
    return y


def ref_rope_neox(x, pos, ne0, ne1, n_dims, n_seqs, theta_scale, freq_scale):
    """kernels/rope_neox.glsl over the grid its own header states (rows in x,
    64-pair groups in y), which covers every row and pair."""
    x = _f32(x).ravel()
    pos = np.ascontiguousarray(pos, np.int32)
    y = np.zeros_like(x)
    pc = _u32(ne0, ne1, n_dims, n_seqs, float(theta_scale), float(freq_scale), 0, 0)
    ref().vkref_rope_neox((C.c_void_p * 3)(_p(x), _p(pos), _p(y)), C.c_void_p(_p(pc)), ne1 * n_seqs,
                          (ne0 // 2 + 63) // 64, 1)
    return y


def ref_embedding(w16, idx):
    w = np.ascontiguousarray(w16, np.float16)
    idx = np.ascontiguousarray(idx, np.int32)
    V, D = w.shape
    out = np.zeros((idx.size, D), np.float16)
    pc = _u32(V, D, idx.size)
    ref().vkref_embedding((C.c_void_p * 3)(_p(w), _p(idx), _p(out)), C.c_void_p(_p(pc)),
                          (idx.size * D + 255) // 256, 1, 1)
    return out
