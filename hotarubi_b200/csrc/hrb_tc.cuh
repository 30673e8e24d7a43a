// Tensor-core (tcgen05) GEMM path: declarations shared with capi.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "hrb_kernels.cuh"

namespace hrb {

// Whether the tensor-core kernel serves this GEMM (shape and format limits).
bool tc_supported(const DenseJob& job);

// Launches the tensor-core GEMM over `n` host-side jobs (one or more
// kernels).  Returns the number of kernels launched, or -1 on a launch error.
int launch_tc(const DenseJob* jobs, uint32_t n, int sm_count, cudaStream_t stream);

}  // namespace hrb
