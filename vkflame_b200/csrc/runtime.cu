// runtime.cu — device bring-up, allocation table, scratch arenas, status
// reporting.  Replaces runtime/device.cpp (Vulkan instance/device/queues,
// device.cpp:131-370), runtime/buffer.cpp (VkBuffer allocation, staging arena,
// buffer.cpp:235-579) and runtime/pipeline.cpp (SPIR-V pipelines) of the
// reference: on CUDA none of that machinery exists, so what remains is
// device validation, a range-aware allocation table and per-stream scratch.

#include "rt_internal.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <shared_mutex>
#include <utility>
#include <vector>

namespace vkf {

static thread_local int t_last_status = VKF_OK;
static std::atomic<uint64_t> g_launches{0};

int set_status(int status) {
    t_last_status = status;
    return status;
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool debug_enabled() {
    static int enabled = -1;
    if (enabled < 0) {
        const char *e = getenv("VKFLAME_DEBUG");
        enabled = (e && e[0] && e[0] != '0') ? 1 : 0;
    }
    return enabled == 1;
}

void log(const char *fmt, ...) {
    if (!debug_enabled()) return;
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "[vkflame] ");
    vfprintf(stderr, fmt, ap);
    va_end(ap);
}

int check_launch() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        log("kernel launch failed: %s\n", cudaGetErrorString(e));
        return VKF_ERR_CUDA;
    }
    count_launch();
    return VKF_OK;
}

// ---- per-device state ------------------------------------------------------

static std::mutex g_dev_mu;
static std::vector<DeviceState *> g_devs;

DeviceState *existing_device_state() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    return dev < (int)g_devs.size() ? g_devs[dev] : nullptr;
}

DeviceState *device_state() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if (dev < (int)g_devs.size() && g_devs[dev]) return g_devs[dev];
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return nullptr;
    auto *st = new DeviceState;
    st->device = dev;
    st->sm_count = prop.multiProcessorCount;
    st->cc_major = prop.major;
    st->cc_minor = prop.minor;
    st->smem_optin = prop.sharedMemPerBlockOptin;
    if (cudaMalloc(&st->d_error, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(st->d_error, 0, sizeof(unsigned)) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {  // zeroed before any kernel on any stream uses it
        delete st;
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (dev >= (int)g_devs.size()) g_devs.resize(dev + 1, nullptr);
    if (g_devs[dev]) {  // lost a race with another thread
        cudaFree(st->d_error);
        delete st;
        return g_devs[dev];
    }
    g_devs[dev] = st;
    return st;
}

// ---- per-stream scratch ----------------------------------------------------

struct Arena {
    void *ptr = nullptr;
    size_t size = 0;
};
static std::mutex g_scratch_mu;
static std::map<std::pair<int, cudaStream_t>, Arena> g_scratch, g_counters;

static void *arena_get(std::map<std::pair<int, cudaStream_t>, Arena> &tab, cudaStream_t stream, size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    Arena &a = tab[{dev, stream}];
    if (a.size >= bytes) return a.ptr;
    size_t want = bytes < (size_t(4) << 20) ? (size_t(4) << 20) : bytes;
    want = (want + 0xFFFFF) & ~size_t(0xFFFFF);
    if (a.ptr) {
        cudaStreamSynchronize(stream);
        cudaFree(a.ptr);
        a.ptr = nullptr;
        a.size = 0;
    }
    void *p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) return nullptr;
    // Zeroed on the stream that uses it: a plain cudaMemset runs on the
    // legacy default stream, which does not order itself before work on a
    // non-blocking stream, so a kernel could set a flag the late memset
    // then clears.
    if (cudaMemsetAsync(p, 0, want, stream) != cudaSuccess) {
        cudaFree(p);
        return nullptr;
    }
    a.ptr = p;
    a.size = want;
    log("arena for stream %p on device %d: %zu bytes\n", (void *)stream, dev, want);
    return p;
}

void *stream_scratch(cudaStream_t stream, size_t bytes) { return arena_get(g_scratch, stream, bytes); }

int *stream_counters(cudaStream_t stream, size_t count) {
    return (int *)arena_get(g_counters, stream, count * sizeof(int));
}

// ---- allocation table ------------------------------------------------------

static std::shared_mutex g_alloc_mu;
static std::map<uintptr_t, size_t> g_allocs;  // base -> size

static bool table_lookup(uintptr_t p, uintptr_t *base, size_t *size) {
    std::shared_lock<std::shared_mutex> lk(g_alloc_mu);
    auto it = g_allocs.upper_bound(p);
    if (it == g_allocs.begin()) return false;
    --it;
    if (p < it->first + it->second || (it->second == 0 && p == it->first)) {
        *base = it->first;
        *size = it->second;
        return true;
    }
    return false;
}

int validate_device_range(const void *p, size_t bytes) {
    if (!p) return bytes == 0 ? VKF_OK : VKF_ERR_BADPTR;
    uintptr_t base = 0;
    size_t size = 0;
    uintptr_t u = (uintptr_t)p;
    if (table_lookup(u, &base, &size)) return (u + bytes <= base + size) ? VKF_OK : VKF_ERR_BADPTR;
    // Not ours (e.g. a torch or NCCL buffer): accept device-accessible memory.
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return VKF_ERR_BADPTR;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) return VKF_OK;
    return VKF_ERR_BADPTR;
}

}  // namespace vkf

using namespace vkf;

extern "C" {

int vkflame_init(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return set_status(VKF_ERR_NO_DEVICE);
    }
    DeviceState *st = device_state();
    if (!st) return set_status(VKF_ERR_CUDA);
    if (st->cc_major != 10) {
        log("device %d is sm_%d%d; this build targets sm_100a\n", st->device, st->cc_major, st->cc_minor);
        return set_status(VKF_ERR_NO_DEVICE);
    }
    return set_status(VKF_OK);
}

void *vkflame_get_context(void) {
    static int ctx_token = 0;
    return device_state() ? (void *)&ctx_token : nullptr;
}

void vkflame_shutdown(void) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    for (auto *tab : {&g_scratch, &g_counters})
    for (auto &kv : *tab) {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(kv.first.first);
        cudaStreamSynchronize(kv.first.second);
        cudaFree(kv.second.ptr);
        cudaSetDevice(cur);
    }
    g_scratch.clear();
    g_counters.clear();
}

void vkflame_print_info(void) {
    DeviceState *st = device_state();
    if (!st) {
        printf("[vkflame] no CUDA device\n");
        return;
    }
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, st->device);
    printf("[vkflame] device %d: %s, sm_%d%d, %d SMs, %.1f GB, smem/block opt-in %zu B\n", st->device, prop.name,
           prop.major, prop.minor, prop.multiProcessorCount, prop.totalGlobalMem / 1e9, st->smem_optin);
}

void *vkflame_alloc(size_t size) {
    void *p = nullptr;
    if (size == 0) size = 1;
    if (cudaMalloc(&p, size) != cudaSuccess) {
        cudaGetLastError();
        set_status(VKF_ERR_NOMEM);
        return nullptr;
    }
    vkflame_register_alloc(p, size);
    set_status(VKF_OK);
    return p;
}

int vkflame_register_alloc(void *base, size_t size) {
    if (!base) return set_status(VKF_ERR_INVALID);
    std::unique_lock<std::shared_mutex> lk(g_alloc_mu);
    g_allocs[(uintptr_t)base] = size;
    return set_status(VKF_OK);
}

int vkflame_unregister_alloc(void *base) {
    std::unique_lock<std::shared_mutex> lk(g_alloc_mu);
    auto it = g_allocs.find((uintptr_t)base);
    if (it == g_allocs.end()) return set_status(VKF_ERR_BADPTR);
    g_allocs.erase(it);
    return set_status(VKF_OK);
}

int vkflame_free(void *ptr) {
    if (!ptr) return set_status(VKF_OK);
    if (vkflame_unregister_alloc(ptr) != VKF_OK) return set_status(VKF_ERR_BADPTR);
    return set_status(cudaFree(ptr) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
}

int vkflame_ptr_lookup(const void *ptr, void **base, size_t *size) {
    uintptr_t b = 0;
    size_t s = 0;
    if (!table_lookup((uintptr_t)ptr, &b, &s)) return set_status(VKF_ERR_BADPTR);
    if (base) *base = (void *)b;
    if (size) *size = s;
    return set_status(VKF_OK);
}

int vkflame_memcpy_h2d(void *dst, const void *src, size_t size, size_t offset) {
    char *d = (char *)dst + offset;
    if (validate_device_range(d, size) != VKF_OK) return set_status(VKF_ERR_BADPTR);
    return set_status(cudaMemcpy(d, src, size, cudaMemcpyHostToDevice) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
}

int vkflame_memcpy_d2h(void *dst, const void *src, size_t size, size_t offset) {
    const char *s = (const char *)src + offset;
    if (validate_device_range(s, size) != VKF_OK) return set_status(VKF_ERR_BADPTR);
    return set_status(cudaMemcpy(dst, s, size, cudaMemcpyDeviceToHost) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
}

int vkflame_memcpy_d2d(void *dst, const void *src, size_t size) {
    if (validate_device_range(dst, size) != VKF_OK || validate_device_range(src, size) != VKF_OK)
        return set_status(VKF_ERR_BADPTR);
    return set_status(cudaMemcpy(dst, src, size, cudaMemcpyDeviceToDevice) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
}

int vkflame_memset(void *dst, int value, size_t size) {
    if (validate_device_range(dst, size) != VKF_OK) return set_status(VKF_ERR_BADPTR);
    return set_status(cudaMemset(dst, value, size) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
}

int vkflame_get_last_error(void) { return t_last_status; }

const char *vkflame_status_string(int status) {
    switch (status) {
    case VKF_OK: return "VKF_OK";
    case VKF_ERR_INVALID: return "VKF_ERR_INVALID";
    case VKF_ERR_NOMEM: return "VKF_ERR_NOMEM";
    case VKF_ERR_BADPTR: return "VKF_ERR_BADPTR";
    case VKF_ERR_UNSUPPORTED: return "VKF_ERR_UNSUPPORTED";
    case VKF_ERR_CUDA: return "VKF_ERR_CUDA";
    case VKF_ERR_NO_DEVICE: return "VKF_ERR_NO_DEVICE";
    case VKF_ERR_TIMEOUT: return "VKF_ERR_TIMEOUT";
    default: return "VKF_ERR_UNKNOWN";
    }
}

int vkflame_check_kernel_errors(void) {
    // Looks only at state that exists already, so a process that uses just the
    // allocation-free entry point allocates nothing here either.
    if (cudaDeviceSynchronize() != cudaSuccess) return set_status(VKF_ERR_CUDA);
    unsigned bits = 0;
    int rc = noalloc_take_errors(&bits);
    if (rc) return set_status(rc);
    DeviceState *st = existing_device_state();
    if (st) {
        unsigned b = 0;
        if (cudaMemcpy(&b, st->d_error, sizeof(b), cudaMemcpyDeviceToHost) != cudaSuccess)
            return set_status(VKF_ERR_CUDA);
        if (b && cudaMemset(st->d_error, 0, sizeof(unsigned)) != cudaSuccess) return set_status(VKF_ERR_CUDA);
        bits |= b;
    }
    return set_status(bits ? VKF_ERR_TIMEOUT : VKF_OK);
}

uint64_t vkflame_kernel_launch_count(void) { return g_launches.load(); }

}  // extern "C"

// ---- CUDA IPC of device buffers (multi-GPU gathered outputs and counters) ----

extern "C" int vkflame_ipc_handle(const void *dev_ptr, void *handle64, uint64_t *offset) {
    if (!dev_ptr || !handle64 || !offset) return vkf::set_status(VKF_ERR_INVALID);
    // cuMemGetAddressRange through the runtime's driver entry point (the
    // library does not link libcuda directly).
    using RangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
    static RangeFn range = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        return (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
                q == cudaDriverEntryPointSuccess)
                   ? reinterpret_cast<RangeFn>(p)
                   : nullptr;
    }();
    CUdeviceptr base = 0;
    size_t size = 0;
    if (!range || range(&base, &size, (CUdeviceptr)dev_ptr) != CUDA_SUCCESS) return vkf::set_status(VKF_ERR_BADPTR);
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, (void *)base) != cudaSuccess) return vkf::set_status(VKF_ERR_CUDA);
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle64, &h, sizeof(h));
    *offset = (uint64_t)((CUdeviceptr)dev_ptr - base);
    return vkf::set_status(VKF_OK);
}

extern "C" int vkflame_ipc_open(const void *handle64, void **base) {
    if (!handle64 || !base) return vkf::set_status(VKF_ERR_INVALID);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    if (cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return vkf::set_status(VKF_ERR_CUDA);
    return vkf::set_status(VKF_OK);
}

extern "C" int vkflame_ipc_close(void *base) {
    return vkf::set_status(cudaIpcCloseMemHandle(base) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
}
