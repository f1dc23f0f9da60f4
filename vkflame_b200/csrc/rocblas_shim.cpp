// rocblas_shim.cpp — librocblas.so.4: rocblas_initialize, the one rocBLAS
// symbol ggml-hip links against (shim/rocblas_shim.cpp of the reference).
#include "../../include/vkflame_rocblas.h"

extern "C" int rocblas_initialize(void) { return 0; }
