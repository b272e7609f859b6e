// q8_gemm_tc.cu -- tcgen05 / TMEM int8-weight GEMM (fp16 activations).
#include <cuda_runtime.h>

#include "kernels.h"

namespace b200q8 {

bool gemm_tc_supports(const LinearArgs&) { return false; }

cudaError_t launch_q8_gemm_tc(const LinearArgs&, int, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace b200q8
