// k_matmul_tc.cu - placeholder until the tcgen05 3xTF32 GEMM lands.
#include <cuda_runtime.h>
#include <cstdint>
#include "mcu_kernels.h"

extern "C" int mcu_matmul_tc_supported(void) { return 0; }
extern "C" size_t mcu_matmul_tc_scratch_bytes(int64_t, int64_t, int64_t) { return 0; }
extern "C" int mcu_launch_matmul_tc(float*, const float*, const float*, int64_t, int64_t, int64_t, void*, int*,
                                    cudaStream_t) {
    return (int)cudaErrorNotSupported;
}
