"""ctypes bindings of libvkflame_rt.so (include/vkflame_rt.h).

Every wrapper takes raw device pointers (ints) and raises VkflameError on a
non-zero status.  Streams are cudaStream_t values (0 = legacy default).
"""
from __future__ import annotations

import ctypes as C

from . import LIBS

VKF_OK = 0
STATUS = {0: "VKF_OK", 1: "VKF_ERR_INVALID", 2: "VKF_ERR_NOMEM", 3: "VKF_ERR_BADPTR",
          4: "VKF_ERR_UNSUPPORTED", 5: "VKF_ERR_CUDA", 6: "VKF_ERR_NO_DEVICE", 7: "VKF_ERR_TIMEOUT"}

Q4_0, Q4_1, Q8_0, Q5_0, Q4_K, Q5_K, Q6_K, Q8_1 = range(8)
X_F16, X_Q8_1 = 0, 1
Y_F32, Y_F16 = 0, 1
DTYPE_FP32, DTYPE_FP16, DTYPE_INT8, DTYPE_BF16, DTYPE_FP16_FP32OUT = range(5)
ACT_NONE, ACT_SILU, ACT_RELU, ACT_GELU_ERF = range(4)


class VkflameError(RuntimeError):
    def __init__(self, status: int, what: str):
        super().__init__(f"{what}: {STATUS.get(status, status)}")
        self.status = status


_SIGS = {
    "vkflame_init": ([], C.c_int),
    "vkflame_get_context": ([], C.c_void_p),
    "vkflame_shutdown": ([], None),
    "vkflame_print_info": ([], None),
    "vkflame_alloc": ([C.c_size_t], C.c_void_p),
    "vkflame_free": ([C.c_void_p], C.c_int),
    "vkflame_memcpy_h2d": ([C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t], C.c_int),
    "vkflame_memcpy_d2h": ([C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t], C.c_int),
    "vkflame_memcpy_d2d": ([C.c_void_p, C.c_void_p, C.c_size_t], C.c_int),
    "vkflame_memset": ([C.c_void_p, C.c_int, C.c_size_t], C.c_int),
    "vkflame_ptr_lookup": ([C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)], C.c_int),
    "vkflame_register_alloc": ([C.c_void_p, C.c_size_t], C.c_int),
    "vkflame_unregister_alloc": ([C.c_void_p], C.c_int),
    "vkflame_dispatch_linear": ([C.c_void_p] * 5 + [C.c_int] * 7 + [C.c_void_p] * 3, C.c_int),
    "vkflame_dispatch_dequant": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_int], C.c_int),
    "vkflame_dispatch_dequant_async": ([C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_void_p], C.c_int),
    "vkflame_quant_linear": ([C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                              C.c_int, C.c_int, C.c_int, C.c_int64, C.c_int64, C.c_void_p], C.c_int),
    "vkflame_quant_linear_ex": ([C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                 C.c_int, C.c_int, C.c_int, C.c_int64, C.c_int64, C.c_uint, C.c_void_p], C.c_int),
    "vkflame_quant_linear_noalloc": ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_int64, C.c_int64, C.c_void_p], C.c_int),
    "vkflame_quantize_q8_1": ([C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int64, C.c_void_p], C.c_int),
    "vkflame_linear_int8": ([C.c_void_p] * 7 + [C.c_int] * 4 + [C.c_void_p], C.c_int),
    "vkflame_quant_linear_gather": ([C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_int64, C.c_int64, C.c_uint, C.c_void_p, C.c_void_p], C.c_int),
    "vkflame_chain_create": ([C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint, C.POINTER(C.c_void_p)], C.c_int),
    "vkflame_chain_run": ([C.c_void_p, C.c_void_p], C.c_int),
    "vkflame_chain_epoch": ([C.c_void_p, C.POINTER(C.c_int)], C.c_int),
    "vkflame_chain_trace": ([C.c_void_p, C.c_void_p], C.c_int),
    "vkflame_chain_status": ([C.c_void_p, C.c_void_p], C.c_int),
    "vkflame_chain_destroy": ([C.c_void_p], C.c_int),
    "vkflame_set_stream": ([C.c_void_p], C.c_int),
    "vkflame_get_stream": ([], C.c_void_p),
    "vkflame_dispatch_elementwise_f32": ([C.c_void_p] * 3 + [C.c_uint32] * 2, C.c_int),
    "vkflame_dispatch_scale_f32": ([C.c_void_p] * 3 + [C.c_uint32, C.c_float, C.c_float], C.c_int),
    "vkflame_dispatch_binop_f32": ([C.c_void_p] * 4 + [C.c_uint32] * 3, C.c_int),
    "vkflame_dispatch_rms_norm_f32": ([C.c_void_p] * 3 + [C.c_uint32] * 2 + [C.c_float], C.c_int),
    "vkflame_dispatch_rms_norm": ([C.c_void_p] * 4 + [C.c_int] * 2 + [C.c_float], C.c_int),
    "vkflame_dispatch_softmax": ([C.c_void_p] * 3 + [C.c_int] * 2, C.c_int),
    "vkflame_dispatch_rope_neox": ([C.c_void_p] * 4 + [C.c_uint32] * 4 + [C.c_float] * 2 + [C.c_uint32] * 2,
                                   C.c_int),
    "vkflame_dispatch_embedding": ([C.c_void_p] * 4 + [C.c_int] * 3, C.c_int),
    "vkflame_get_rows": ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p] + [C.c_int] * 3 + [C.c_void_p], C.c_int),
    "vkflame_ipc_handle": ([C.c_void_p, C.c_void_p, C.POINTER(C.c_uint64)], C.c_int),
    "vkflame_ipc_open": ([C.c_void_p, C.POINTER(C.c_void_p)], C.c_int),
    "vkflame_ipc_close": ([C.c_void_p], C.c_int),
    "vkflame_get_last_error": ([], C.c_int),
    "vkflame_status_string": ([C.c_int], C.c_char_p),
    "vkflame_check_kernel_errors": ([], C.c_int),
    "vkflame_kernel_launch_count": ([], C.c_uint64),
}


def declared_symbols() -> list[str]:
    return list(_SIGS)


def load(path=None) -> C.CDLL:
    import os
    from pathlib import Path
    p = Path(path or os.environ.get("VKFLAME_RT_LIB") or LIBS["rt"])
    if not p.exists():
        raise ImportError(f"[vkflame_b200] {p} not built (run __graft_entry__.build())")
    lib = C.CDLL(str(p), mode=C.RTLD_GLOBAL)
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.argtypes = args
        fn.restype = res
    return lib


_lib = None


def lib() -> C.CDLL:
    """The runtime library, initialised on a B200; raises otherwise."""
    global _lib
    if _lib is None:
        l = load()
        rc = l.vkflame_init()
        if rc != VKF_OK:
            raise VkflameError(rc, "vkflame_init (needs an sm_100 GPU)")
        _lib = l
    return _lib


def _check(rc: int, what: str) -> None:
    if rc != VKF_OK:
        raise VkflameError(rc, what)


def dequant(src: int, dst: int, n_blocks: int, qtype: int, stream: int = 0) -> None:
    _check(lib().vkflame_dispatch_dequant_async(src, dst, n_blocks, qtype, stream), "dequant")


def quant_linear(W: int, wtype: int, X: int, xtype: int, Y: int, ytype: int, M: int, N: int, K: int,
                 ldx: int, ldy: int, stream: int = 0) -> None:
    _check(lib().vkflame_quant_linear(W, wtype, X, xtype, Y, ytype, M, N, K, ldx, ldy, stream), "quant_linear")


FLAG_STATIC_WEIGHTS = 1


def quant_linear_ex(W: int, wtype: int, X: int, xtype: int, Y: int, ytype: int, M: int, N: int, K: int,
                    ldx: int, ldy: int, flags: int = 0, stream: int = 0) -> None:
    _check(lib().vkflame_quant_linear_ex(W, wtype, X, xtype, Y, ytype, M, N, K, ldx, ldy, flags, stream),
           "quant_linear_ex")


def quantize_q8_1(x: int, y: int, M: int, K: int, ldx: int, stream: int = 0) -> None:
    _check(lib().vkflame_quantize_q8_1(x, y, M, K, ldx, stream), "quantize_q8_1")


def linear_int8(X: int, W: int, sx: int, sw: int, bias: int, Y: int, acc: int, M: int, N: int, K: int,
                act: int = 0, stream: int = 0) -> None:
    _check(lib().vkflame_linear_int8(X, W, sx, sw, bias, Y, acc, M, N, K, act, stream), "linear_int8")


def dispatch_linear(A: int, B: int, C_: int, D: int, M: int, N: int, K: int, dtype: int, transA: int = 0,
                    transB: int = 0, act: int = 0, alpha=None, beta=None, stream: int = 0) -> None:
    a = C.byref(C.c_float(alpha)) if alpha is not None else None
    b = C.byref(C.c_float(beta)) if beta is not None else None
    _check(lib().vkflame_dispatch_linear(None, A, B, C_, D, M, N, K, dtype, transA, transB, act, a, b, stream),
           "dispatch_linear")


MAX_RANKS = 8


class Gather(C.Structure):
    """vkf_gather_t (include/vkflame_rt.h)."""
    _fields_ = [("world", C.c_int), ("rank", C.c_int), ("y_rank", C.c_void_p * MAX_RANKS),
                ("stride", C.c_int64), ("epoch", C.c_void_p), ("done", C.c_void_p),
                ("x_gathered", C.c_int), ("x_stride", C.c_int64)]


def quant_linear_gather(W: int, wtype: int, X: int, ytype: int, M: int, N: int, K: int, ldx: int, ldy: int,
                        flags: int, g: Gather, stream: int = 0) -> None:
    _check(lib().vkflame_quant_linear_gather(W, wtype, X, ytype, M, N, K, ldx, ldy, flags, C.byref(g), stream),
           "quant_linear_gather")


class ChainLinear(C.Structure):
    """vkf_chain_linear_t (include/vkflame_rt.h)."""
    _fields_ = [("W", C.c_void_p), ("wtype", C.c_int), ("K", C.c_int), ("N", C.c_int), ("x_src", C.c_int),
                ("x_plain", C.c_void_p), ("y_rank", C.c_void_p * MAX_RANKS), ("y_stride", C.c_int64),
                ("y_plain", C.c_void_p)]


CHAIN_TRACE = 1


class Chain:
    """A token's decode linears as one persistent kernel (vkflame_chain_*)."""

    def __init__(self, linears: list, world: int = 1, rank: int = 0, flags: int = 0):
        arr = (ChainLinear * len(linears))(*linears)
        h = C.c_void_p()
        _check(lib().vkflame_chain_create(arr, len(linears), world, rank, flags, C.byref(h)), "chain_create")
        self.handle, self.n = h.value, len(linears)

    def run(self, stream: int = 0) -> None:
        _check(lib().vkflame_chain_run(self.handle, stream), "chain_run")

    def epoch(self) -> int:
        e = C.c_int()
        _check(lib().vkflame_chain_epoch(self.handle, C.byref(e)), "chain_epoch")
        return e.value

    def trace(self):
        import numpy as np
        t = np.zeros((self.n, 2), np.uint64)
        _check(lib().vkflame_chain_trace(self.handle, t.ctypes.data), "chain_trace")
        return t

    def status(self) -> list:
        """First wait that gave up: [role, linear, item, CTA] (zeros: none)."""
        import numpy as np
        f = np.zeros(4, np.int32)
        _check(lib().vkflame_chain_status(self.handle, f.ctypes.data), "chain_status")
        return [int(v) for v in f]

    def close(self) -> None:
        if self.handle:
            _check(lib().vkflame_chain_destroy(self.handle), "chain_destroy")
            self.handle = None


def ipc_handle(ptr: int) -> tuple[bytes, int]:
    h = (C.c_uint8 * 64)()
    off = C.c_uint64()
    _check(lib().vkflame_ipc_handle(ptr, h, C.byref(off)), "ipc_handle")
    return bytes(h), off.value


def ipc_open(handle: bytes) -> int:
    h = (C.c_uint8 * 64).from_buffer_copy(handle)
    base = C.c_void_p()
    _check(lib().vkflame_ipc_open(h, C.byref(base)), "ipc_open")
    return base.value


def ipc_close(base: int) -> None:
    _check(lib().vkflame_ipc_close(base), "ipc_close")


def check_kernel_errors() -> None:
    _check(lib().vkflame_check_kernel_errors(), "kernel error bits")


def launch_count() -> int:
    return lib().vkflame_kernel_launch_count()
