// Test infrastructure only: force-included (g++ -include) when compiling the
// reference's own model sources for the CPU/FP32 oracle build. Nothing in the
// product links or loads this.
//
// The reference hard-codes CUDA and BF16 (src/models/ModelBase.cpp:118-129,
// :317, :352, :359, :379, :392-393, :846). Its sources are compiled where they
// lie, unmodified; this header is included first so that every LibTorch and
// CUDA header is already expanded, and only then renames the two tokens the
// reference uses for device and dtype. The headers' include guards keep the
// macros out of LibTorch itself.
#pragma once
#include <torch/torch.h>
#include <cuda_runtime.h>

// ModelBase.cpp:317 asks the GPU for free memory to size MaxSequenceLength.
// On the CPU build there is no GPU: report 64 GiB free so the reference keeps
// max_position_embeddings from config.json (ModelBase.cpp:326-328).
static inline cudaError_t ylm_oracle_cpu_mem_info(size_t *free_b, size_t *total_b)
{
    *free_b = (size_t)64 << 30;
    *total_b = (size_t)64 << 30;
    return cudaSuccess;
}

#define cudaMemGetInfo ylm_oracle_cpu_mem_info
#define kCUDA kCPU
#define kBFloat16 kFloat
