// noalloc.cu — an allocation-free variant of the decode GEMV entry point.
//
// vkflame_quant_linear keeps its stream-K scratch (partial row-block sums and
// arrival counters) in per-stream arenas it allocates with cudaMalloc on first
// use.  Some callers cannot allow that: code running inside a custom
// allocator's callback, a host process whose device memory is fully
// pre-reserved, or a runtime that forbids allocation after start-up.  For
// them vkflame_quant_linear_noalloc uses a fixed scratch that lives in this
// library's own device globals instead: the arrays below, placed in every
// GPU's memory when the library's module is loaded there and kept until the
// process exits.

#include "rt_internal.h"

#include <mutex>

namespace vkf {

int gemv_launch_raw(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy,
                    int M, int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap,
                    int sms, unsigned *err, int plan_only);

namespace noalloc {

// Partial sums: two 128-float slots per CTA, for up to NOALLOC_MAX_CTAS CTAs
// (the GEMV runs one CTA per SM).  Counters: one per 16-row block,
// so N <= NOALLOC_MAX_ROWS.  512 KiB + 64 KiB + 4 bytes in total.
constexpr int NOALLOC_MAX_CTAS = 512;
constexpr int NOALLOC_MAX_ROWS = 262144;
constexpr size_t WS_FLOATS = (size_t)NOALLOC_MAX_CTAS * 2 * 128;
constexpr size_t CNT_INTS = NOALLOC_MAX_ROWS / 16;

static __device__ __align__(256) float g_ws[WS_FLOATS];
static __device__ __align__(256) int g_cnt[CNT_INTS];
static __device__ __align__(256) unsigned g_err;

// In host code g_ws / g_cnt / g_err name host-side stand-ins, not device
// addresses: their device addresses are looked up once per device with that
// device current (cudaGetSymbolAddress) and cached here.
struct Addrs {
    bool ready = false;
    float *ws = nullptr;
    int *cnt = nullptr;
    unsigned *err = nullptr;
    int sms = 0;
};
constexpr int MAX_DEVICES = 64;
static Addrs g_addrs[MAX_DEVICES];
static std::mutex g_mu;

static int setup(int dev, Addrs **out) {
    std::lock_guard<std::mutex> lk(g_mu);
    Addrs &a = g_addrs[dev];
    if (!a.ready) {
        if (cudaGetSymbolAddress((void **)&a.ws, g_ws) != cudaSuccess ||
            cudaGetSymbolAddress((void **)&a.cnt, g_cnt) != cudaSuccess ||
            cudaGetSymbolAddress((void **)&a.err, g_err) != cudaSuccess ||
            cudaDeviceGetAttribute(&a.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return VKF_ERR_CUDA;
        }
        a.ready = true;
    }
    *out = &a;
    return VKF_OK;
}

}  // namespace noalloc

// Error bits the allocation-free kernels set on the current device (a bounded
// wait gave up), read and cleared; 0 when the entry point was never used
// there.  Called by vkflame_check_kernel_errors after it synchronised.
int noalloc_take_errors(unsigned *bits) {
    *bits = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= noalloc::MAX_DEVICES) return VKF_ERR_NO_DEVICE;
    noalloc::Addrs *ad = nullptr;
    {
        std::lock_guard<std::mutex> lk(noalloc::g_mu);
        if (!noalloc::g_addrs[dev].ready) return VKF_OK;
        ad = &noalloc::g_addrs[dev];
    }
    if (cudaMemcpy(bits, ad->err, sizeof(unsigned), cudaMemcpyDeviceToHost) != cudaSuccess) return VKF_ERR_CUDA;
    if (*bits && cudaMemset(ad->err, 0, sizeof(unsigned)) != cudaSuccess) return VKF_ERR_CUDA;
    return VKF_OK;
}
}  // namespace vkf

using namespace vkf;

extern "C" int vkflame_quant_linear_noalloc(const void *W, int wtype, const void *X, void *Y, int ytype, int M,
                                            int N, int K, int64_t ldx, int64_t ldy, void *stream) {
    if (wtype != VKF_DEQUANT_Q4_0 && wtype != VKF_DEQUANT_Q8_0 && wtype != VKF_DEQUANT_Q4_K &&
        wtype != VKF_DEQUANT_Q5_K && wtype != VKF_DEQUANT_Q6_K)
        return set_status(VKF_ERR_UNSUPPORTED);
    if (ytype != VKF_Y_F32 && ytype != VKF_Y_F16) return set_status(VKF_ERR_INVALID);
    // Size limits of the fixed scratch, and the cases that would need staging
    // memory (more than 8 batch rows, activations too large to stay resident,
    // activation rows not 16-byte aligned), are rejected rather than served.
    if (M < 1 || M > 8 || N < 1 || N > noalloc::NOALLOC_MAX_ROWS || K <= 0) return set_status(VKF_ERR_INVALID);
    const int qk = vkf_qtype_block_values(wtype);
    if (K % qk || K % 32 || ldx < K || ldy < N) return set_status(VKF_ERR_INVALID);
    if ((size_t)M * ((size_t)K * 2 + 160 + (size_t)K / 8) > (size_t)80 * 1024) return set_status(VKF_ERR_UNSUPPORTED);
    if (((uintptr_t)X & 15) || (ldx * 2) % 16) return set_status(VKF_ERR_BADPTR);
    const uintptr_t wa = (uintptr_t)W;
    if ((wtype == VKF_DEQUANT_Q4_K || wtype == VKF_DEQUANT_Q5_K) ? (wa & 3) : (wa & 1)) return set_status(VKF_ERR_BADPTR);
    if ((uintptr_t)Y & (ytype == VKF_Y_F16 ? 1 : 3)) return set_status(VKF_ERR_BADPTR);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= noalloc::MAX_DEVICES) return set_status(VKF_ERR_NO_DEVICE);
    noalloc::Addrs *ad = nullptr;
    int rc = noalloc::setup(dev, &ad);
    if (rc) return set_status(rc);
    if (2 * ad->sms > noalloc::NOALLOC_MAX_CTAS) return set_status(VKF_ERR_UNSUPPORTED);
    cudaStream_t st = (cudaStream_t)stream;
    // Plan first, so that a request the kernel cannot serve is refused before
    // anything is queued on the stream.
    rc = gemv_launch_raw(wtype, W, X, ldx * 2, Y, ytype == VKF_Y_F16, ldy, M, N, K, st, ad->ws, noalloc::WS_FLOATS,
                         ad->cnt, noalloc::CNT_INTS, ad->sms, ad->err, 1);
    if (rc) return set_status(rc);
    // The arrival counters must start at zero; a completed call leaves them
    // zero, but an interrupted one may not, so clear the ones this call uses.
    const size_t ncnt = (size_t)(N + 15) / 16;
    if (cudaMemsetAsync(ad->cnt, 0, ncnt * sizeof(int), st) != cudaSuccess) return set_status(VKF_ERR_CUDA);
    rc = gemv_launch_raw(wtype, W, X, ldx * 2, Y, ytype == VKF_Y_F16, ldy, M, N, K, st, ad->ws, noalloc::WS_FLOATS,
                         ad->cnt, noalloc::CNT_INTS, ad->sms, ad->err, 0);
    return set_status(rc);
}
