// rt_internal.h — shared host-side state of libvkflame_rt (not installed).
#pragma once

#include <cuda.h>
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
DeviceState *existing_device_state();  // same, but never creates it (nullptr if not yet created)
// Reads and clears the allocation-free entry point's kernel error bits on the
// current device (noalloc.cu); *bits = 0 if it never ran there.
int noalloc_take_errors(unsigned *bits);

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

// Tensor maps (false if the shape or alignment is not encodable):
// K-major operand of esize-byte elements [rows x cols], row stride ld
// elements, box = 128 bytes of K x box_rows, 128-byte swizzle (the tcgen05
// operand layout);
bool make_kmajor_map(CUtensorMap *m, const void *base, int esize, int64_t rows, int64_t cols, int64_t ld,
                     int box_rows);
// row-major fp16 (esize 2) or fp32 (4) matrix [rows x cols], row stride ld
// elements, box = box_rows x box_cols, no swizzle (tile stores);
bool make_rowmajor_map(CUtensorMap *m, const void *base, int esize, int64_t rows, int64_t cols, int64_t ld,
                       int box_cols, int box_rows);
// byte matrix [rows x row_bytes] (16-byte multiple) as 8-byte elements, box
// = box_rows x box_bytes, no swizzle.
bool make_byte_matrix_map(CUtensorMap *m, const void *base, int64_t rows, int64_t row_bytes, int box_bytes,
                          int box_rows);

}  // namespace vkf

// Kernel error bits written to DeviceState::d_error.
#define VKF_KERR_WAIT_TIMEOUT 1u
#define VKF_KERR_BAD_COPY 2u
