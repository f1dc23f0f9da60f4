/*
 * vkflame_hip.h — exports of libamdhip64.so.6 (the HIP runtime drop-in).
 *
 * Names, signatures, error codes and the hipDeviceProp_t layout of the
 * reference shim (shim/hip_runtime_shim.cpp:18-78 types, :335-1404 exports),
 * implemented over the CUDA runtime of a B200: hipMalloc returns real device
 * pointers (the reference returned VkDeviceAddress values, :352-353), streams
 * are cudaStream_t, events cudaEvent_t with real timing (the reference's
 * hipEventElapsedTime returned 0, :747-752), device count / peer access are
 * the machine's (the reference reported 1 device and no peers, :642-649,
 * :718-723).  hipLaunchKernel keeps the reference's name -> kernel table for
 * ggml kernels (:896-1205): quantised mul_mat -> fused dequant GEMV/GEMM,
 * f16 mul_mat -> tensor-core GEMM, dequantize_* -> the bit-exact dequant
 * kernels; other kernel names are logged and skipped, as in the reference.
 * Device identity for HIP callers keeps the reference's gfx-arch fields
 * (VKFLAME_GFX_ARCH / HSA_OVERRIDE_GFX_VERSION, default gfx1201) with the
 * B200's real memory size, SM count, shared memory and clocks.
 */
#ifndef VKFLAME_HIP_H
#define VKFLAME_HIP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int hipError_t;
typedef void *hipStream_t;
typedef void *hipEvent_t;
typedef void *hipModule_t;
typedef void *hipFunction_t;

#define hipSuccess 0
#define hipErrorInvalidValue 1
#define hipErrorMemoryAllocation 2
#define hipErrorInvalidDevicePointer 3
#define hipErrorUnknown 999

#define hipMemcpyHostToHost 0
#define hipMemcpyHostToDevice 1
#define hipMemcpyDeviceToHost 2
#define hipMemcpyDeviceToDevice 3
#define hipMemcpyDefault 4

#define hipDeviceAttributeWarpSize 10
#define hipDeviceAttributeMaxSharedMemoryPerBlock 11
#define hipDeviceAttributeMaxThreadsPerBlock 12
#define hipDeviceAttributeMultiprocessorCount 13
#define hipDeviceAttributeClockRate 14
#define hipDeviceAttributeMemoryClockRate 15
#define hipDeviceAttributeMemoryBusWidth 16
#define hipDeviceAttributeComputeCapabilityMajor 75
#define hipDeviceAttributeComputeCapabilityMinor 76
#define hipDeviceAttributeGcnArch 90

/* shim/hip_runtime_shim.cpp:49-78 */
typedef struct hipDeviceProp_t {
    char name[256];
    size_t totalGlobalMem;
    size_t sharedMemPerBlock;
    int regsPerBlock;
    int warpSize;
    size_t memPitch;
    int maxThreadsPerBlock;
    int maxThreadsDim[3];
    int maxGridSize[3];
    int clockRate;
    size_t totalConstMem;
    int major;
    int minor;
    size_t textureAlignment;
    int deviceOverlap;
    int multiProcessorCount;
    int kernelExecTimeoutEnabled;
    int integrated;
    int canMapHostMemory;
    int computeMode;
    int gcnArch;
    char gcnArchName[256];
    int isMultiGpuBoard;
    int clockInstructionRate;
    int cooperativeLaunch;
    int cooperativeMultiDeviceLaunch;
    int maxSharedMemoryPerMultiProcessor;
    int isLargeBar;
} hipDeviceProp_t;

typedef struct vkf_dim3 { unsigned x, y, z; } vkf_dim3; /* HIP's dim3, passed by value */
typedef struct vkf_uint3 { unsigned x, y, z; } vkf_uint3;

/* shim/hip_runtime_shim.cpp:1343-1355 */
typedef struct hipFuncAttributes {
    size_t sharedSizeBytes;
    size_t constSizeBytes;
    size_t localSizeBytes;
    int maxThreadsPerBlock;
    int numRegs;
    int ptxVersion;
    int binaryVersion;
    int cacheModeCA;
    int maxDynamicSharedSizeBytes;
    int preferredShmemCarveout;
} hipFuncAttributes;

/* memory, shim/hip_runtime_shim.cpp:335-469, 775-828 */
hipError_t hipMalloc(void **devPtr, size_t size);
hipError_t hipFree(void *devPtr);
hipError_t hipMallocManaged(void **devPtr, size_t size, unsigned int flags);
hipError_t hipMemcpy(void *dst, const void *src, size_t count, int kind);
hipError_t hipMemcpyAsync(void *dst, const void *src, size_t count, int kind, hipStream_t stream);
hipError_t hipMemset(void *devPtr, int value, size_t count);
hipError_t hipMemsetAsync(void *devPtr, int value, size_t count, hipStream_t stream);
hipError_t hipHostMalloc(void **ptr, size_t size, unsigned int flags);
hipError_t hipHostFree(void *ptr);
hipError_t hipHostRegister(void *ptr, size_t size, unsigned int flags);
hipError_t hipHostUnregister(void *ptr);
hipError_t hipMemGetInfo(size_t *free_out, size_t *total_out);
hipError_t hipMemAdvise(const void *ptr, size_t count, int advice, int dev);
hipError_t hipMemcpy2DAsync(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t height,
                            int kind, hipStream_t stream);
hipError_t hipMemcpyPeerAsync(void *dst, int dstDev, const void *src, int srcDev, size_t count, hipStream_t stream);
hipError_t hipPointerGetAttributes(void *attributes, const void *ptr);
hipError_t hipDrvPointerGetAttributes(unsigned int numAttributes, int *attributes, void **data, const void *ptr);

/* synchronisation, streams, events, graphs: :473-496, 726-772 */
hipError_t hipDeviceSynchronize(void);
hipError_t hipStreamCreate(hipStream_t *stream);
hipError_t hipStreamCreateWithFlags(hipStream_t *stream, unsigned int flags);
hipError_t hipStreamDestroy(hipStream_t stream);
hipError_t hipStreamSynchronize(hipStream_t stream);
hipError_t hipStreamWaitEvent(hipStream_t stream, hipEvent_t event, unsigned int flags);
hipError_t hipEventCreateWithFlags(hipEvent_t *event, unsigned int flags);
hipError_t hipEventDestroy(hipEvent_t event);
hipError_t hipEventRecord(hipEvent_t event, hipStream_t stream);
hipError_t hipEventSynchronize(hipEvent_t event);
hipError_t hipEventElapsedTime(float *ms, hipEvent_t start, hipEvent_t stop);
hipError_t hipStreamBeginCapture(hipStream_t stream, int mode);
hipError_t hipStreamEndCapture(hipStream_t stream, void **graph);
hipError_t hipGraphDestroy(void *graph);

/* device queries and control: :500-725 */
hipError_t hipSetDevice(int device);
hipError_t hipGetDevice(int *device);
hipError_t hipGetDeviceCount(int *count);
hipError_t hipGetDeviceProperties(hipDeviceProp_t *prop, int device);
hipError_t hipGetDevicePropertiesR0600(void *prop, int device);
hipError_t hipDeviceGetAttribute(int *value, int attr, int device);
hipError_t hipDriverGetVersion(int *driverVersion);
hipError_t hipDeviceReset(void);
hipError_t hipDeviceCanAccessPeer(int *canAccessPeer, int dev, int peer);
hipError_t hipDeviceEnablePeerAccess(int peerDevice, unsigned int flags);
hipError_t hipDeviceDisablePeerAccess(int peerDevice);

/* errors: :621-640 (last error per thread) */
const char *hipGetErrorString(hipError_t error);
hipError_t hipGetLastError(void);
hipError_t hipPeekAtLastError(void);

/* kernel launch and registration: :833-1336 */
hipError_t hipLaunchKernel(const void *func, vkf_dim3 gridDim, vkf_dim3 blockDim, void **args, size_t sharedMem,
                           hipStream_t stream);
void **__hipRegisterFatBinary(const void *data);
void __hipUnregisterFatBinary(void **modules);
void __hipRegisterFunction(void **modules, const void *hostFn, char *deviceFn, const char *deviceName,
                           int threadLimit, vkf_uint3 *tid, vkf_uint3 *bid, vkf_dim3 *blockDim, vkf_dim3 *gridDim,
                           int *wSize);
hipError_t __hipPushCallConfiguration(vkf_dim3 gridDim, vkf_dim3 blockDim, size_t sharedMem, hipStream_t stream);
hipError_t __hipPopCallConfiguration(vkf_dim3 *gridDim, vkf_dim3 *blockDim, size_t *sharedMem, hipStream_t *stream);
hipError_t hipOccupancyMaxActiveBlocksPerMultiprocessor(int *numBlocks, const void *func, int blockSize,
                                                        size_t dynSharedMemPerBlk);
hipError_t hipModuleLoad(hipModule_t *module, const char *fname);
hipError_t hipModuleLoadData(hipModule_t *module, const void *image);
hipError_t hipModuleLoadDataEx(hipModule_t *module, const void *image, unsigned int numOptions, int *options,
                               void **optionValues);
hipError_t hipModuleUnload(hipModule_t module);
hipError_t hipModuleGetFunction(hipFunction_t *func, hipModule_t mod, const char *name);
hipError_t hipModuleLaunchKernel(hipFunction_t f, uint32_t gridX, uint32_t gridY, uint32_t gridZ, uint32_t blockX,
                                 uint32_t blockY, uint32_t blockZ, uint32_t sharedMem, hipStream_t stream,
                                 void **kernelParams, void **extra);
hipError_t hipExtModuleLaunchKernel(hipFunction_t f, uint32_t globalX, uint32_t globalY, uint32_t globalZ,
                                    uint32_t blockX, uint32_t blockY, uint32_t blockZ, uint32_t sharedMem,
                                    hipStream_t stream, void **kernelParams, void **extra, hipEvent_t startEvent,
                                    hipEvent_t stopEvent, uint32_t flags);
hipError_t hipFuncGetAttributes(hipFuncAttributes *attr, const void *func);
hipError_t hipFuncSetAttribute(const void *func, int attr, int value);
hipError_t hipFuncSetCacheConfig(const void *func, int cacheConfig);
hipError_t hiprtcCreateProgram(void **prog, const char *src, const char *name, int numHeaders, const char **headers,
                               const char **includeNames);

#ifdef __cplusplus
}
#endif
#endif
