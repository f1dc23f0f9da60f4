// hipblaslt_shim.cpp — libhipblaslt.so.0: the hipBLASLt drop-in over the B200
// tensor-core GEMMs (include/vkflame_hipblaslt.h).
//
// Replaces shim/hipblaslt_shim.cpp of the reference, whose hipblasLtMatmul
// dropped the bias and scale pointers, the transposes, alpha/beta, the
// leading dimensions and the batch attributes (shim/hipblaslt_shim.cpp:
// 121-128, 163-167, 254-262, 418-423).  int8 inputs run the kind::i8 kernel
// with the linear_int8 epilogue fp16(act((acc * a_scale[m]) * b_scale[n] +
// bias[n])); f16 / f32 inputs the kind::f16 / kind::tf32 kernels.

#include "../../include/vkflame_hipblaslt.h"

#include <cuda_runtime.h>

#include <cstring>

#include "shim_api.h"

namespace {

constexpr int OP_N = 111, OP_T = 112, OP_C = 113;

struct Handle {
    int pad = 0;
};
struct Layout {
    uint64_t rows = 0, cols = 0;
    int64_t ld = 0;  // 0: the column count (row-major, packed)
    int type = HIPBLASLT_R_32F;
    int batch_count = 1;
    int64_t stride = 0;  // elements between batch entries
};
struct Desc {
    int transA = OP_N, transB = OP_N;
    int compute_type = 0, scale_type = 0;
    int epilogue = HIPBLASLT_EPILOGUE_DEFAULT;
    const void *bias = nullptr, *a_scale = nullptr, *b_scale = nullptr;
};
struct Pref {
    uint64_t max_workspace = 0;
};
struct HeuristicResult {
    int algo_id;
};

int blas_type(int t) {
    switch (t) {
    case HIPBLASLT_R_16F: return vkf::BT_F16;
    case HIPBLASLT_R_32F: return vkf::BT_F32;
    case HIPBLASLT_R_8I: return vkf::BT_I8;
    case HIPBLASLT_R_32I: return vkf::BT_I32;
    default: return -1;
    }
}
int esize(int t) { return t == HIPBLASLT_R_16F || t == HIPBLASLT_R_16B ? 2 : t == HIPBLASLT_R_8I ? 1 : 4; }
int64_t ld_of(const Layout *l) { return l->ld ? l->ld : (int64_t)l->cols; }
bool trans(int op) { return op == OP_T || op == OP_C; }

hipblasStatus_t status_of(int vkf) {
    switch (vkf) {
    case VKF_OK: return 0;
    case VKF_ERR_INVALID:
    case VKF_ERR_BADPTR: return 3;
    case VKF_ERR_UNSUPPORTED: return 8;
    case VKF_ERR_NOMEM: return 2;
    default: return 6;
    }
}

}  // namespace

extern "C" {

hipblasStatus_t hipblasLtCreate(void **lightHandle) {
    if (!lightHandle) return 3;
    if (vkflame_init() != VKF_OK) return 4;
    *lightHandle = new Handle;
    return 0;
}

hipblasStatus_t hipblasLtDestroy(void *lightHandle) {
    delete static_cast<Handle *>(lightHandle);
    return 0;
}

hipblasStatus_t hipblasLtMatrixLayoutCreate(void **matLayout, int type, uint64_t rows, uint64_t cols, int64_t ld) {
    if (!matLayout) return 3;
    auto *l = new Layout;
    l->type = type;
    l->rows = rows;
    l->cols = cols;
    l->ld = ld;
    *matLayout = l;
    return 0;
}

hipblasStatus_t hipblasLtMatrixLayoutDestroy(void *matLayout) {
    delete static_cast<Layout *>(matLayout);
    return 0;
}

hipblasStatus_t hipblasLtMatrixLayoutSetAttribute(void *matLayout, int attr, const void *buf, size_t) {
    if (!matLayout || !buf) return 3;
    auto *l = static_cast<Layout *>(matLayout);
    switch (attr) {
    case HIPBLASLT_MATRIX_LAYOUT_ROWS: l->rows = *(const uint64_t *)buf; break;
    case HIPBLASLT_MATRIX_LAYOUT_COLS: l->cols = *(const uint64_t *)buf; break;
    case HIPBLASLT_MATRIX_LAYOUT_LD: l->ld = *(const int64_t *)buf; break;
    case HIPBLASLT_MATRIX_LAYOUT_TYPE: l->type = *(const int *)buf; break;
    case HIPBLASLT_MATRIX_LAYOUT_BATCH_COUNT: l->batch_count = *(const int *)buf; break;
    case HIPBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET: l->stride = *(const int64_t *)buf; break;
    default: break;
    }
    return 0;
}

hipblasStatus_t hipblasLtMatrixLayoutGetAttribute(void *matLayout, int attr, void *buf, size_t, size_t *sizeWritten) {
    if (!matLayout || !buf) return 3;
    auto *l = static_cast<Layout *>(matLayout);
    size_t w = 8;
    switch (attr) {
    case HIPBLASLT_MATRIX_LAYOUT_ROWS: *(uint64_t *)buf = l->rows; break;
    case HIPBLASLT_MATRIX_LAYOUT_COLS: *(uint64_t *)buf = l->cols; break;
    case HIPBLASLT_MATRIX_LAYOUT_LD: *(int64_t *)buf = ld_of(l); break;
    case HIPBLASLT_MATRIX_LAYOUT_TYPE: *(int *)buf = l->type; w = 4; break;
    case HIPBLASLT_MATRIX_LAYOUT_BATCH_COUNT: *(int *)buf = l->batch_count; w = 4; break;
    case HIPBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET: *(int64_t *)buf = l->stride; break;
    default: w = 0; break;
    }
    if (sizeWritten) *sizeWritten = w;
    return 0;
}

hipblasStatus_t hipblasLtMatmulDescCreate(void **matmulDesc, int computeType, int scaleType) {
    if (!matmulDesc) return 3;
    auto *d = new Desc;
    d->compute_type = computeType;
    d->scale_type = scaleType;
    *matmulDesc = d;
    return 0;
}

hipblasStatus_t hipblasLtMatmulDescDestroy(void *matmulDesc) {
    delete static_cast<Desc *>(matmulDesc);
    return 0;
}

hipblasStatus_t hipblasLtMatmulDescSetAttribute(void *matmulDesc, int attr, const void *buf, size_t) {
    if (!matmulDesc || !buf) return 3;
    auto *d = static_cast<Desc *>(matmulDesc);
    switch (attr) {
    case HIPBLASLT_MATMUL_DESC_TRANSA: d->transA = *(const int *)buf; break;
    case HIPBLASLT_MATMUL_DESC_TRANSB: d->transB = *(const int *)buf; break;
    case HIPBLASLT_MATMUL_DESC_COMPUTE_TYPE: d->compute_type = *(const int *)buf; break;
    case HIPBLASLT_MATMUL_DESC_SCALE_TYPE: d->scale_type = *(const int *)buf; break;
    case HIPBLASLT_MATMUL_DESC_EPILOGUE: d->epilogue = *(const int *)buf; break;
    case HIPBLASLT_MATMUL_DESC_BIAS_POINTER: d->bias = *(const void *const *)buf; break;
    case HIPBLASLT_MATMUL_DESC_A_SCALE_POINTER: d->a_scale = *(const void *const *)buf; break;
    case HIPBLASLT_MATMUL_DESC_B_SCALE_POINTER: d->b_scale = *(const void *const *)buf; break;
    default: break;
    }
    return 0;
}

hipblasStatus_t hipblasLtMatmulDescGetAttribute(void *matmulDesc, int attr, void *buf, size_t, size_t *sizeWritten) {
    if (!matmulDesc || !buf) return 3;
    auto *d = static_cast<Desc *>(matmulDesc);
    size_t w = 4;
    switch (attr) {
    case HIPBLASLT_MATMUL_DESC_TRANSA: *(int *)buf = d->transA; break;
    case HIPBLASLT_MATMUL_DESC_TRANSB: *(int *)buf = d->transB; break;
    case HIPBLASLT_MATMUL_DESC_COMPUTE_TYPE: *(int *)buf = d->compute_type; break;
    case HIPBLASLT_MATMUL_DESC_SCALE_TYPE: *(int *)buf = d->scale_type; break;
    case HIPBLASLT_MATMUL_DESC_EPILOGUE: *(int *)buf = d->epilogue; break;
    case HIPBLASLT_MATMUL_DESC_BIAS_POINTER: *(const void **)buf = d->bias; w = sizeof(void *); break;
    case HIPBLASLT_MATMUL_DESC_A_SCALE_POINTER: *(const void **)buf = d->a_scale; w = sizeof(void *); break;
    case HIPBLASLT_MATMUL_DESC_B_SCALE_POINTER: *(const void **)buf = d->b_scale; w = sizeof(void *); break;
    default: w = 0; break;
    }
    if (sizeWritten) *sizeWritten = w;
    return 0;
}

hipblasStatus_t hipblasLtMatmulPreferenceCreate(void **pref) {
    if (!pref) return 3;
    *pref = new Pref;
    return 0;
}

hipblasStatus_t hipblasLtMatmulPreferenceDestroy(void *pref) {
    delete static_cast<Pref *>(pref);
    return 0;
}

hipblasStatus_t hipblasLtMatmulPreferenceSetAttribute(void *pref, int attr, const void *buf, size_t) {
    if (!pref || !buf) return 3;
    if (attr == HIPBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES) static_cast<Pref *>(pref)->max_workspace = *(const uint64_t *)buf;
    return 0;
}

hipblasStatus_t hipblasLtMatmulAlgoGetHeuristic(void *, void *, void *, void *, void *, void *, void *,
                                                int requestedAlgoCount, void *heuristicResultsArray,
                                                int *returnAlgoCount) {
    if (returnAlgoCount) *returnAlgoCount = requestedAlgoCount > 0 ? 1 : 0;
    if (heuristicResultsArray && requestedAlgoCount > 0)
        static_cast<HeuristicResult *>(heuristicResultsArray)->algo_id = 0;
    return 0;
}

hipblasStatus_t hipblasLtMatmul(void *lightHandle, void *matmulDesc, const void *alpha, const void *A, void *Adesc,
                                const void *B, void *Bdesc, const void *beta, const void *C, void *Cdesc, void *D,
                                void *Ddesc, const void *algo, void *workspace, size_t workspaceSizeInBytes,
                                hipStream_t stream) {
    (void)algo;
    (void)workspace;
    (void)workspaceSizeInBytes;
    if (!lightHandle || !matmulDesc || !Adesc || !Bdesc || !Ddesc || !A || !B || !D) return 3;
    const auto *desc = static_cast<const Desc *>(matmulDesc);
    const auto *la = static_cast<const Layout *>(Adesc), *lb = static_cast<const Layout *>(Bdesc);
    const auto *ld = static_cast<const Layout *>(Ddesc);
    const auto *lc = Cdesc ? static_cast<const Layout *>(Cdesc) : ld;
    const bool ta = trans(desc->transA), tb = trans(desc->transB);
    const int64_t M = ta ? la->cols : la->rows, K = ta ? la->rows : la->cols;
    const int64_t K2 = tb ? lb->cols : lb->rows, N = tb ? lb->rows : lb->cols;
    if (K != K2 || (int64_t)ld->rows != M || (int64_t)ld->cols != N) return 3;
    const int at = blas_type(la->type), bt = blas_type(lb->type), dt = blas_type(ld->type);
    if (at < 0 || bt < 0 || dt < 0) return 8;
    int act = 0;
    switch (desc->epilogue) {
    case HIPBLASLT_EPILOGUE_RELU: act = VKF_ACT_RELU; break;
    case HIPBLASLT_EPILOGUE_GELU: act = VKF_ACT_GELU_ERF; break;
    case HIPBLASLT_EPILOGUE_SILU: act = VKF_ACT_SILU; break;
    default: act = 0; break;
    }
    const float al = alpha ? *(const float *)alpha : 1.0f, be = beta ? *(const float *)beta : 0.0f;
    const int batches = ld->batch_count > 0 ? ld->batch_count : 1;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t lda = ld_of(la), ldb = ld_of(lb), ldd = ld_of(ld), ldc = ld_of(lc);
    for (int i = 0; i < batches; ++i) {
        const char *a = (const char *)A + (la->batch_count > 1 ? i * la->stride * esize(la->type) : 0);
        const char *b = (const char *)B + (lb->batch_count > 1 ? i * lb->stride * esize(lb->type) : 0);
        char *d = (char *)D + i * ld->stride * esize(ld->type);
        if (be != 0.0f && C && C != D) {
            // beta * C is read from D: bring C there first.
            const char *c = (const char *)C + i * lc->stride * esize(lc->type);
            if (cudaMemcpy2DAsync(d, ldd * esize(ld->type), c, ldc * esize(lc->type), N * esize(ld->type), M,
                                  cudaMemcpyDeviceToDevice, st) != cudaSuccess)
                return 6;
        }
        // Row-major D = op(A) op(B) is the column-major D^T = op(B)^T op(A)^T.
        const int rc = vkf::blas_gemm_ex(tb, ta, (int)N, (int)M, (int)K, al, b, bt, ldb, a, at, lda, be, d, dt, ldd,
                                         (const float *)desc->a_scale, (const float *)desc->b_scale, desc->bias, act,
                                         st);
        if (rc) return status_of(rc);
    }
    return 0;
}

}  // extern "C"
