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
