/* vkflame_rocblas.h — librocblas.so.4: the single symbol ggml-hip imports
 * (shim/rocblas_shim.cpp:1-11). */
#ifndef VKFLAME_ROCBLAS_H
#define VKFLAME_ROCBLAS_H
#ifdef __cplusplus
extern "C" {
#endif
int rocblas_initialize(void);
#ifdef __cplusplus
}
#endif
#endif
