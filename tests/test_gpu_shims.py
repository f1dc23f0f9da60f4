"""The drop-in shim libraries, called through their C ABI as an application
would: libamdhip64 (memory, streams, events, device queries, the
hipLaunchKernel name table), libhipblas (column-major GEMMs with transposes,
leading dimensions, alpha/beta) and libhipblaslt (row-major matmul with the
int8 bias/scale epilogue of config 2)."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po
from vkflame_b200 import LIBS
from vkflame_b200 import synth as S

pytestmark = pytest.mark.gpu

OP_N, OP_T = 111, 112
H2D, D2H, D2D = 1, 2, 3


class Dim3(C.Structure):
    _fields_ = [("x", C.c_uint), ("y", C.c_uint), ("z", C.c_uint)]


@pytest.fixture(scope="module")
def hip():
    from vkflame_b200 import rt
    rt.lib()
    lib = C.CDLL(str(LIBS["hip"]))
    lib.hipMalloc.argtypes = [C.POINTER(C.c_void_p), C.c_size_t]
    lib.hipFree.argtypes = [C.c_void_p]
    lib.hipMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    lib.hipMemset.argtypes = [C.c_void_p, C.c_int, C.c_size_t]
    lib.hipLaunchKernel.argtypes = [C.c_void_p, Dim3, Dim3, C.POINTER(C.c_void_p), C.c_size_t, C.c_void_p]
    lib.__hipRegisterFunction.argtypes = [C.c_void_p, C.c_void_p, C.c_char_p, C.c_char_p, C.c_int] + [C.c_void_p] * 5
    lib.hipEventElapsedTime.argtypes = [C.POINTER(C.c_float), C.c_void_p, C.c_void_p]
    lib.hipEventRecord.argtypes = [C.c_void_p, C.c_void_p]
    lib.hipEventSynchronize.argtypes = [C.c_void_p]
    lib.hipStreamSynchronize.argtypes = [C.c_void_p]
    lib.hipGetErrorString.restype = C.c_char_p
    return lib


class Dev:
    """A device buffer from hipMalloc."""

    def __init__(self, hip, data=None, nbytes=None):
        self.hip = hip
        self.nbytes = nbytes if nbytes is not None else data.nbytes
        p = C.c_void_p()
        assert hip.hipMalloc(C.byref(p), self.nbytes) == 0
        self.ptr = p.value
        if data is not None:
            d = np.ascontiguousarray(data)
            assert hip.hipMemcpy(self.ptr, d.ctypes.data, d.nbytes, H2D) == 0

    def get(self, dtype, shape=None, offset=0, nbytes=None):
        n = nbytes if nbytes is not None else self.nbytes - offset
        out = np.empty(n, np.uint8)
        assert self.hip.hipMemcpy(out.ctypes.data, self.ptr + offset, n, D2H) == 0
        out = out.view(dtype)
        return out.reshape(shape) if shape is not None else out

    def __del__(self):
        self.hip.hipFree(self.ptr)


def test_hip_memory_roundtrip_and_suballocation(hip):
    a = np.arange(1 << 20, dtype=np.uint8) * 7
    d = Dev(hip, a)
    assert np.array_equal(d.get(np.uint8), a)
    # pointers inside an allocation (the reference only resolved bases)
    assert hip.hipMemset(d.ptr + 1000, 0xAB, 24) == 0
    got = d.get(np.uint8)
    assert (got[1000:1024] == 0xAB).all() and got[999] == a[999] and got[1024] == a[1024]
    assert hip.hipFree(C.c_void_p(12345)) != 0  # not an allocation


class DeviceProp(C.Structure):
    """hipDeviceProp_t as declared by the shim header."""
    _fields_ = [("name", C.c_char * 256), ("totalGlobalMem", C.c_size_t), ("sharedMemPerBlock", C.c_size_t),
                ("regsPerBlock", C.c_int), ("warpSize", C.c_int), ("memPitch", C.c_size_t),
                ("maxThreadsPerBlock", C.c_int), ("maxThreadsDim", C.c_int * 3), ("maxGridSize", C.c_int * 3),
                ("clockRate", C.c_int), ("totalConstMem", C.c_size_t), ("major", C.c_int), ("minor", C.c_int),
                ("textureAlignment", C.c_size_t), ("deviceOverlap", C.c_int), ("multiProcessorCount", C.c_int),
                ("kernelExecTimeoutEnabled", C.c_int), ("integrated", C.c_int), ("canMapHostMemory", C.c_int),
                ("computeMode", C.c_int), ("gcnArch", C.c_int), ("gcnArchName", C.c_char * 256),
                ("isMultiGpuBoard", C.c_int), ("clockInstructionRate", C.c_int), ("cooperativeLaunch", C.c_int),
                ("cooperativeMultiDeviceLaunch", C.c_int), ("maxSharedMemoryPerMultiProcessor", C.c_int),
                ("isLargeBar", C.c_int)]


def test_hip_device_queries(hip, monkeypatch):
    monkeypatch.delenv("VKFLAME_GFX_ARCH", raising=False)
    monkeypatch.delenv("HSA_OVERRIDE_GFX_VERSION", raising=False)
    n = C.c_int()
    assert hip.hipGetDeviceCount(C.byref(n)) == 0 and n.value >= 1
    prop = DeviceProp()
    assert hip.hipGetDeviceProperties(C.byref(prop), 0) == 0
    assert prop.totalGlobalMem > 100e9 and prop.multiProcessorCount >= 100 and prop.warpSize == 32
    assert prop.gcnArchName == b"gfx1201" and (prop.major, prop.minor) == (12, 0)
    v = C.c_int()
    assert hip.hipDeviceGetAttribute(C.byref(v), 13, 0) == 0 and v.value == prop.multiProcessorCount
    assert hip.hipDeviceGetAttribute(C.byref(v), 10, 0) == 0 and v.value == 32


def test_hip_streams_events(hip):
    s, e0, e1 = C.c_void_p(), C.c_void_p(), C.c_void_p()
    assert hip.hipStreamCreate(C.byref(s)) == 0
    assert hip.hipEventCreateWithFlags(C.byref(e0), 0) == 0 and hip.hipEventCreateWithFlags(C.byref(e1), 0) == 0
    d = Dev(hip, nbytes=256 << 20)
    assert hip.hipEventRecord(e0, s) == 0
    for _ in range(4):
        assert hip.hipMemsetAsync(C.c_void_p(d.ptr), 1, C.c_size_t(d.nbytes), s) == 0
    assert hip.hipEventRecord(e1, s) == 0
    assert hip.hipEventSynchronize(e1) == 0
    ms = C.c_float()
    assert hip.hipEventElapsedTime(C.byref(ms), e0, e1) == 0 and ms.value > 0  # the reference returned 0
    assert hip.hipStreamSynchronize(s) == 0
    hip.hipEventDestroy(e0)
    hip.hipEventDestroy(e1)
    hip.hipStreamDestroy(s)


_stub_keep = []


def register(hip, name):
    stub = C.create_string_buffer(8)  # any unique host address stands in for a kernel stub
    _stub_keep.append(stub)
    hip.__hipRegisterFunction(None, C.addressof(stub), name.encode(), name.encode(), -1, None, None, None, None, None)
    return C.addressof(stub)


def launch(hip, fn, grid, block, args):
    holders = []
    for a in args:
        if isinstance(a, tuple):
            v = a[0](a[1])
        else:
            v = C.c_void_p(a)
        holders.append(v)
    argv = (C.c_void_p * len(holders))(*[C.addressof(h) for h in holders])
    return hip.hipLaunchKernel(C.c_void_p(fn), Dim3(*grid), Dim3(*block), argv, 0, None)


def test_hip_launch_dequant_q4_K(hip):
    raw = S.quant_matrix(S.Q4_K, 4, 1024, seed=1).ravel()
    nb = raw.size // 144
    src, dst = Dev(hip, raw), Dev(hip, nbytes=nb * 256 * 4)
    fn = register(hip, "void dequantize_block_q4_K<float>(void const*, float*)")
    assert launch(hip, fn, (nb, 1, 1), (32, 1, 1), [src.ptr, dst.ptr]) == 0
    got = dst.get(np.float32)
    assert np.array_equal(got.view(np.uint32), po.dequant(S.Q4_K, raw, nb).view(np.uint32))


def test_hip_launch_dequant_q8_0_int64_count(hip):
    raw = S.quant_matrix(S.Q8_0, 2, 512, seed=2).ravel()
    nb = raw.size // 34
    src, dst = Dev(hip, raw), Dev(hip, nbytes=nb * 32 * 4)
    fn = register(hip, "dequantize_block_q8_0<float>")
    assert launch(hip, fn, (nb, 1, 1), (256, 1, 1), [src.ptr, dst.ptr, (C.c_int64, nb * 32)]) == 0
    assert np.array_equal(dst.get(np.float32).view(np.uint32), po.dequant(S.Q8_0, raw, nb).view(np.uint32))


@pytest.mark.parametrize("q,name", [(S.Q4_0, "dequantize_block_q4_0<float>"), (S.Q4_1, "dequantize_block_q4_1"),
                                    (S.Q5_0, "dequantize_block_q5_0<float>")])
def test_hip_launch_dequant_nb32_convention(hip, q, name):
    """q4_0 / q4_1 / q5_0: (vx, y, int nb32), nb32 = the count of 32-value
    blocks (shim/hip_runtime_shim.cpp:896-920); the launch grid is ignored."""
    raw = S.quant_matrix(q, 3, 512, seed=20 + q).ravel()
    nb = raw.size // S.BLOCK_BYTES[q]
    src, dst = Dev(hip, raw), Dev(hip, nbytes=nb * 32 * 4)
    fn = register(hip, name)
    assert launch(hip, fn, ((nb + 7) // 8, 1, 1), (32, 1, 1), [src.ptr, dst.ptr, (C.c_int, nb)]) == 0
    assert np.array_equal(dst.get(np.float32).view(np.uint32), po.dequant(q, raw, nb).view(np.uint32))


@pytest.mark.parametrize("q,name", [(S.Q5_K, "dequantize_block_q5_K<__half>"), (S.Q6_K, "dequantize_block_q6_K")])
def test_hip_launch_dequant_k_quants_grid_count(hip, q, name):
    """K-quants: (vx, y), one super-block per grid.x."""
    raw = S.quant_matrix(q, 2, 1024, seed=30 + q).ravel()
    nb = raw.size // S.BLOCK_BYTES[q]
    src, dst = Dev(hip, raw), Dev(hip, nbytes=nb * 256 * 4)
    fn = register(hip, name)
    assert launch(hip, fn, (nb, 1, 1), (64, 1, 1), [src.ptr, dst.ptr]) == 0
    assert np.array_equal(dst.get(np.float32).view(np.uint32), po.dequant(q, raw, nb).view(np.uint32))


@pytest.mark.parametrize("M", [1, 40])
@pytest.mark.parametrize("q,name", [(S.Q8_0, "mul_mat_q8_0_q8_1"), (S.Q6_K, "mul_mat_q6_K_q8_1"),
                                    (S.Q4_0, "mul_mat_q4_0_q8_1"), (S.Q4_1, "mul_mat_q4_1_q8_1"),
                                    (S.Q5_0, "mul_mat_q5_0_q8_1"), (S.Q5_K, "mul_mat_q5_K_q8_1")])
def test_hip_launch_mul_mat_formats(hip, q, name, M):
    """Every weight format of the mul_mat branch (shim/hip_runtime_shim.cpp:
    1102-1166), Q4_1 and Q5_0 included (dequant + tensor-core GEMM)."""
    N, K = 192, 1024
    w = S.quant_matrix(q, N, K, seed=50 + q)
    xq = po.quantize_q8_1(S.normal_f32((M, K), seed=51))
    wd, xd, yd = Dev(hip, w), Dev(hip, xq), Dev(hip, nbytes=M * N * 4)
    fn = register(hip, name)
    args = [wd.ptr, xd.ptr, yd.ptr, (C.c_int, K), (C.c_int, N), (C.c_int, K), (C.c_int, M), (C.c_int, N)]
    assert launch(hip, fn, (1, 1, 1), (32, 1, 1), args) == 0
    y = yd.get(np.float32, (M, N)).astype(np.float64)
    wf = po.dequant(q, w, N * K // S.BLOCK_VALUES[q]).reshape(N, K).astype(np.float64)
    xf = po.dequant(S.Q8_1, xq, M * K // 32).reshape(M, K).astype(np.float64)
    ref = xf @ wf.T
    assert np.abs(y - ref).max() / np.abs(ref).max() < 2e-3


def test_hip_launch_mul_mat_f16(hip):
    """The fp16 mul_mat branch: (A = activations M x K, B = weights N x K,
    dst fp16 M x N), K = args[3], N = args[4], M = args[6]
    (shim/hip_runtime_shim.cpp:1174-1188, vkflame_dispatch_linear TN)."""
    M, N, K = 24, 200, 320
    rng = np.random.default_rng(8)
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = rng.standard_normal((N, K)).astype(np.float16)
    xd, wd, yd = Dev(hip, x), Dev(hip, w), Dev(hip, nbytes=M * N * 2)
    fn = register(hip, "mul_mat_f16")
    args = [xd.ptr, wd.ptr, yd.ptr, (C.c_int, K), (C.c_int, N), (C.c_int, K), (C.c_int, M)]
    assert launch(hip, fn, (1, 1, 1), (32, 1, 1), args) == 0
    got = yd.get(np.float16, (M, N)).astype(np.float64)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-3


@pytest.mark.parametrize("M", [1, 40])
def test_hip_launch_mul_mat_q4_K_q8_1(hip, M):
    """ggml's quantised mul_mat: weights Q4_K, activations Q8_1, fp32 output."""
    N, K = 256, 1024
    w = S.quant_matrix(S.Q4_K, N, K, seed=3)
    xq = po.quantize_q8_1(S.normal_f32((M, K), seed=4))
    wd, xd, yd = Dev(hip, w), Dev(hip, xq), Dev(hip, nbytes=M * N * 4)
    fn = register(hip, "mul_mat_q4_K_q8_1")
    args = [wd.ptr, xd.ptr, yd.ptr, (C.c_int, K), (C.c_int, N), (C.c_int, K), (C.c_int, M), (C.c_int, N)]
    assert launch(hip, fn, (1, 1, 1), (32, 1, 1), args) == 0
    y = yd.get(np.float32, (M, N)).astype(np.float64)
    wf = po.dequant(S.Q4_K, w, N * K // 256).reshape(N, K).astype(np.float64)
    xf = po.dequant(S.Q8_1, xq, M * K // 32).reshape(M, K).astype(np.float64)
    ref = xf @ wf.T
    assert np.abs(y - ref).max() / np.abs(ref).max() < 2e-3


def test_hip_launch_unknown_kernel_is_skipped(hip):
    fn = register(hip, "k_silu_f32")
    assert launch(hip, fn, (1, 1, 1), (32, 1, 1), [0, 0, (C.c_int, 0)]) == 0


# ---------------------------------------------------------------- hipBLAS --

@pytest.fixture(scope="module")
def blas(hip):
    lib = C.CDLL(str(LIBS["hipblas"]))
    h = C.c_void_p()
    assert lib.hipblasCreate(C.byref(h)) == 0
    lib.handle = h
    return lib


def colmajor(a):
    return np.asfortranarray(a)


@pytest.mark.parametrize("tA,tB", [(OP_N, OP_N), (OP_T, OP_N), (OP_N, OP_T), (OP_T, OP_T)])
def test_hipblas_hgemm_all_layouts(hip, blas, tA, tB):
    m, n, k = 96, 80, 144
    lda, ldb, ldc = (m if tA == OP_N else k) + 8, (k if tB == OP_N else n) + 8, m + 8
    rng = np.random.default_rng(1)
    opA = rng.standard_normal((m, k)).astype(np.float16)
    opB = rng.standard_normal((k, n)).astype(np.float16)
    c0 = rng.standard_normal((m, n)).astype(np.float16)
    A = opA if tA == OP_N else opA.T
    B = opB if tB == OP_N else opB.T
    def store(mat, ld):  # column-major with leading dimension ld
        buf = np.zeros((mat.shape[1], ld), np.float16)
        buf[:, :mat.shape[0]] = mat.T
        return buf
    Ad, Bd, Cd = Dev(hip, store(A, lda)), Dev(hip, store(B, ldb)), Dev(hip, store(c0, ldc))
    alpha, beta = np.float16(0.5).view(np.uint16), np.float16(-1.0).view(np.uint16)
    a_ = C.c_uint16(int(alpha))
    b_ = C.c_uint16(int(beta))
    rc = blas.hipblasHgemm(blas.handle, tA, tB, m, n, k, C.byref(a_), C.c_void_p(Ad.ptr), lda, C.c_void_p(Bd.ptr), ldb,
                           C.byref(b_), C.c_void_p(Cd.ptr), ldc)
    assert rc == 0
    got = Cd.get(np.float16, (n, ldc))[:, :m].T.astype(np.float64)
    ref = 0.5 * opA.astype(np.float64) @ opB.astype(np.float64) - c0.astype(np.float64)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-3


@pytest.mark.parametrize("m,n,k", [(80, 200, 64), (20000, 64, 128), (64, 20000, 128)])
def test_hipblas_hgemm_both_operands_staged(hip, blas, m, n, k):
    """op(A) = A and op(B) = B^T: both operands are copied K-major into the
    stream's scratch; n > m and m > n (the large cases exceed the arena's
    minimum size, so an overlap or overrun of the two regions shows)."""
    rng = np.random.default_rng(m + n)
    A = rng.standard_normal((m, k)).astype(np.float16)  # op N: m x k, column-major (lda = m)
    B = rng.standard_normal((n, k)).astype(np.float16)  # op T: stored n x k column-major (ldb = n)
    Ad, Bd, Cd = Dev(hip, colmajor(A).T.copy()), Dev(hip, colmajor(B).T.copy()), Dev(hip, nbytes=m * n * 2)
    one, zero = C.c_uint16(int(np.float16(1).view(np.uint16))), C.c_uint16(0)
    rc = blas.hipblasHgemm(blas.handle, OP_N, OP_T, m, n, k, C.byref(one), C.c_void_p(Ad.ptr), m, C.c_void_p(Bd.ptr),
                           n, C.byref(zero), C.c_void_p(Cd.ptr), m)
    assert rc == 0
    got = Cd.get(np.float16, (n, m)).T.astype(np.float64)
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-3


def test_hipblas_k_zero_scales_c(hip, blas):
    """k = 0 is a valid hipBLAS call: C = beta * C."""
    m, n = 33, 17
    c0 = np.random.default_rng(9).standard_normal((n, m)).astype(np.float32)
    Cd = Dev(hip, c0)
    one, half = C.c_float(1.0), C.c_float(0.5)
    assert blas.hipblasSgemm(blas.handle, OP_N, OP_N, m, n, 0, C.byref(one), None, m, None, 1, C.byref(half),
                             C.c_void_p(Cd.ptr), m) == 0
    assert np.array_equal(Cd.get(np.float32, (n, m)), c0 * np.float32(0.5))


def test_hipblas_sgemm_fp32_accuracy(hip, blas):
    """hipblasSgemm at fp32 accuracy (three tf32 products), with alpha, beta."""
    m, n, k = 200, 136, 1000
    rng = np.random.default_rng(12)
    A = rng.standard_normal((m, k)).astype(np.float32)  # op N
    B = rng.standard_normal((k, n)).astype(np.float32)  # op N
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    Ad, Bd, Cd = Dev(hip, colmajor(A).T.copy()), Dev(hip, colmajor(B).T.copy()), Dev(hip, colmajor(c0).T.copy())
    al, be = C.c_float(0.75), C.c_float(-0.5)
    assert blas.hipblasSgemm(blas.handle, OP_N, OP_N, m, n, k, C.byref(al), C.c_void_p(Ad.ptr), m, C.c_void_p(Bd.ptr),
                             k, C.byref(be), C.c_void_p(Cd.ptr), m) == 0
    got = Cd.get(np.float32, (n, m)).T.astype(np.float64)
    ref = 0.75 * A.astype(np.float64) @ B.astype(np.float64) - 0.5 * c0.astype(np.float64)
    # fp32 class: a k = 1000 fp32 dot product is good to ~1e-6 of its scale;
    # one tf32 product would be ~1e-3
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-5


def test_hipblas_batched_pointer_arrays(hip, blas):
    """Sgemm/HgemmBatched with device arrays of device pointers."""
    m, n, k, batch = 64, 40, 96, 3
    rng = np.random.default_rng(13)
    for half in (False, True):
        dt = np.float16 if half else np.float32
        As = [rng.standard_normal((k, m)).astype(dt) for _ in range(batch)]  # op T: stored k x m col-major
        Bs = [rng.standard_normal((k, n)).astype(dt) for _ in range(batch)]
        Ad = [Dev(hip, a.T.copy()) for a in As]
        Bd = [Dev(hip, b.T.copy()) for b in Bs]
        Cd = [Dev(hip, nbytes=m * n * np.dtype(dt).itemsize) for _ in range(batch)]
        arrs = [Dev(hip, np.array([d.ptr for d in L], np.uint64)) for L in (Ad, Bd, Cd)]
        if half:
            one, zero = C.c_uint16(int(np.float16(1).view(np.uint16))), C.c_uint16(0)
            fn = blas.hipblasHgemmBatched
        else:
            one, zero = C.c_float(1.0), C.c_float(0.0)
            fn = blas.hipblasSgemmBatched
        assert fn(blas.handle, OP_T, OP_N, m, n, k, C.byref(one), C.c_void_p(arrs[0].ptr), k, C.c_void_p(arrs[1].ptr), k,
                  C.byref(zero), C.c_void_p(arrs[2].ptr), m, batch) == 0
        for i in range(batch):
            got = Cd[i].get(dt, (n, m)).T.astype(np.float64)
            ref = As[i].T.astype(np.float64) @ Bs[i].astype(np.float64)
            assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-3


def test_hipblas_sgemm_tf32(hip, blas):
    m, n, k = 128, 64, 256
    rng = np.random.default_rng(2)
    A = rng.standard_normal((k, m)).astype(np.float32)  # op T: stored k x m column-major
    B = rng.standard_normal((k, n)).astype(np.float32)
    Ad, Bd, Cd = Dev(hip, colmajor(A).T.copy()), Dev(hip, colmajor(B).T.copy()), Dev(hip, nbytes=m * n * 4)
    one, zero = C.c_float(1.0), C.c_float(0.0)
    assert blas.hipblasSgemm(blas.handle, OP_T, OP_N, m, n, k, C.byref(one), C.c_void_p(Ad.ptr), k, C.c_void_p(Bd.ptr),
                             k, C.byref(zero), C.c_void_p(Cd.ptr), m) == 0
    got = Cd.get(np.float32, (n, m)).T.astype(np.float64)
    ref = A.T.astype(np.float64) @ B.astype(np.float64)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-5  # three tf32 products: fp32 accuracy


def test_hipblas_gemmex_int8_int32(hip, blas):
    m, n, k = 64, 96, 128
    rng = np.random.default_rng(3)
    A = rng.integers(-127, 128, (k, m), dtype=np.int8)  # op T
    B = rng.integers(-127, 128, (k, n), dtype=np.int8)
    Ad, Bd, Cd = Dev(hip, A.T.copy()), Dev(hip, B.T.copy()), Dev(hip, nbytes=m * n * 4)
    one, zero = C.c_float(1.0), C.c_float(0.0)
    rc = blas.hipblasGemmEx(blas.handle, OP_T, OP_N, m, n, k, C.byref(one), C.c_void_p(Ad.ptr), 4, k,
                            C.c_void_p(Bd.ptr), 4, k, C.byref(zero), C.c_void_p(Cd.ptr), 10, m, 0, 0)
    assert rc == 0
    got = Cd.get(np.int32, (n, m)).T
    assert np.array_equal(got, A.T.astype(np.int64) @ B.astype(np.int64))


def test_hipblas_strided_batched_ex_f16_to_f32(hip, blas):
    m, n, k, batch = 64, 48, 96, 3
    rng = np.random.default_rng(4)
    A = rng.standard_normal((batch, m, k)).astype(np.float16)  # op T storage: k x m col-major == m x k row-major
    B = rng.standard_normal((batch, n, k)).astype(np.float16)  # op N: k x n col-major == n x k row-major
    Ad, Bd, Cd = Dev(hip, A), Dev(hip, B), Dev(hip, nbytes=batch * m * n * 4)
    one, zero = C.c_float(1.0), C.c_float(0.0)
    rc = blas.hipblasGemmStridedBatchedEx(blas.handle, OP_T, OP_N, m, n, k, C.byref(one), C.c_void_p(Ad.ptr), 2, k,
                                          C.c_longlong(m * k), C.c_void_p(Bd.ptr), 2, k, C.c_longlong(n * k),
                                          C.byref(zero), C.c_void_p(Cd.ptr), 0, m, C.c_longlong(m * n), batch, 0, 0)
    assert rc == 0
    got = Cd.get(np.float32, (batch, n, m))
    for b in range(batch):
        ref = A[b].astype(np.float64) @ B[b].astype(np.float64).T
        assert np.abs(got[b].T - ref).max() / np.abs(ref).max() < 2e-3


# -------------------------------------------------------------- hipBLASLt --

def lt_set(lib, desc, attr, value, ctype):
    v = ctype(value)
    assert lib.hipblasLtMatmulDescSetAttribute(desc, attr, C.byref(v), C.sizeof(v)) == 0


def test_hipblaslt_int8_bias_scales_config2_pattern(hip):
    """Config 2 through hipblasLtMatmul: int8 X (M x K) x int8 W (N x K, TRANSB=T),
    per-row / per-channel scales, fp16 bias (BIAS epilogue); bit-exact with the
    linear_int8 oracle."""
    lt = C.CDLL(str(LIBS["hipblaslt"]))
    M, N, K = 256, 640, 512
    rng = np.random.default_rng(5)
    x = rng.integers(-127, 128, (M, K), dtype=np.int8)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sx = rng.uniform(1e-3, 1e-2, M).astype(np.float32)
    sw = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    Xd, Wd, sxd, swd, bd, Yd = Dev(hip, x), Dev(hip, w), Dev(hip, sx), Dev(hip, sw), Dev(hip, bias), Dev(hip, nbytes=M * N * 2)
    h, desc, la, lb, ld = (C.c_void_p() for _ in range(5))
    assert lt.hipblasLtCreate(C.byref(h)) == 0
    assert lt.hipblasLtMatmulDescCreate(C.byref(desc), 0, 0) == 0
    lt.hipblasLtMatrixLayoutCreate.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.c_uint64, C.c_uint64, C.c_int64]
    assert lt.hipblasLtMatrixLayoutCreate(C.byref(la), 2, M, K, K) == 0
    assert lt.hipblasLtMatrixLayoutCreate(C.byref(lb), 2, N, K, K) == 0
    assert lt.hipblasLtMatrixLayoutCreate(C.byref(ld), 0, M, N, N) == 0
    lt_set(lt, desc, 1, OP_T, C.c_int)           # TRANSB
    lt_set(lt, desc, 5, 2, C.c_int)              # EPILOGUE_BIAS
    lt_set(lt, desc, 6, bd.ptr, C.c_void_p)      # BIAS_POINTER
    lt_set(lt, desc, 7, sxd.ptr, C.c_void_p)     # A_SCALE_POINTER (per row)
    lt_set(lt, desc, 8, swd.ptr, C.c_void_p)     # B_SCALE_POINTER (per channel)
    one, zero = C.c_float(1.0), C.c_float(0.0)
    rc = lt.hipblasLtMatmul(h, desc, C.byref(one), C.c_void_p(Xd.ptr), la, C.c_void_p(Wd.ptr), lb, C.byref(zero),
                            None, None, C.c_void_p(Yd.ptr), ld, None, None, C.c_size_t(0), None)
    assert rc == 0
    y = Yd.get(np.float16, (M, N))
    _, ref = po.linear_int8(x, w, sx, sw, bias)
    assert np.array_equal(y.view(np.uint16), ref.view(np.uint16))


def test_hipblaslt_f16_relu(hip):
    lt = C.CDLL(str(LIBS["hipblaslt"]))
    M, N, K = 128, 192, 256
    rng = np.random.default_rng(6)
    a = rng.standard_normal((M, K)).astype(np.float16)
    b = rng.standard_normal((K, N)).astype(np.float16)  # TRANSB = N: K x N row-major
    Ad, Bd, Dd = Dev(hip, a), Dev(hip, b), Dev(hip, nbytes=M * N * 2)
    h, desc, la, lb, ld = (C.c_void_p() for _ in range(5))
    lt.hipblasLtCreate(C.byref(h))
    lt.hipblasLtMatmulDescCreate(C.byref(desc), 0, 0)
    lt.hipblasLtMatrixLayoutCreate.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.c_uint64, C.c_uint64, C.c_int64]
    lt.hipblasLtMatrixLayoutCreate(C.byref(la), 0, M, K, K)
    lt.hipblasLtMatrixLayoutCreate(C.byref(lb), 0, K, N, N)
    lt.hipblasLtMatrixLayoutCreate(C.byref(ld), 0, M, N, N)
    lt_set(lt, desc, 5, 1, C.c_int)  # RELU
    rc = lt.hipblasLtMatmul(h, desc, None, C.c_void_p(Ad.ptr), la, C.c_void_p(Bd.ptr), lb, None, None, None,
                            C.c_void_p(Dd.ptr), ld, None, None, C.c_size_t(0), None)
    assert rc == 0
    got = Dd.get(np.float16, (M, N)).astype(np.float64)
    ref = np.maximum(a.astype(np.float64) @ b.astype(np.float64), 0)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 2e-3
