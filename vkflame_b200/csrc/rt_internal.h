// rt_internal.h — shared host-side state of libvkflame_rt (not installed).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/vkflame_rt.h"

namespace vkf {

// Records status as the calling thread's last error and returns it.
int set_status(int status);

// Per-device state, created on first use with that device current.
struct DeviceState {
    int device = -1;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    size_t smem_optin = 0;
    unsigned *d_error = nullptr;  // kernels OR a VKF_KERR_* bit here when a bounded wait gives up
};
DeviceState *device_state();  // current device; nullptr if CUDA has no device

// Scratch memory for one stream on the current device (grows on demand,
// zero-filled when (re)allocated).  Calls on one stream are ordered, so a
// per-stream arena is never used by two kernels at once.  Growing waits for
// the stream first.  Returns nullptr on allocation failure.
void *stream_scratch(cudaStream_t stream, size_t bytes);
// Arrival counters for one stream on the current device: a separate, zeroed
// allocation that kernels leave zeroed again when they finish (so nothing
// else may write it).  Returns nullptr on allocation failure.
int *stream_counters(cudaStream_t stream, size_t count);

// Checks the launch just made; maps failures to VKF_ERR_CUDA.
int check_launch();
void count_launch(uint64_t n = 1);

// Host-side validation of a device pointer range [p, p+bytes).
int validate_device_range(const void *p, size_t bytes);

bool debug_enabled();
void log(const char *fmt, ...);

}  // namespace vkf

// Kernel error bits written to DeviceState::d_error.
#define VKF_KERR_WAIT_TIMEOUT 1u
#define VKF_KERR_BAD_COPY 2u
