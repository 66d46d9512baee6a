// Test infrastructure only: force-included (g++ -include) when compiling the
// reference's own model sources for the "LibTorch CUDA FP16" oracle build.
//
// The reference reinterprets every weight as BF16 and keeps KV, RoPE tables and
// embeddings in BF16 (src/models/ModelBase.cpp:118-122, :352, :359, :392-393,
// :846). This variant keeps its CUDA device and renames only the dtype token so
// the same code path runs in FP16, the storage type this engine uses. LibTorch
// headers are expanded first; their include guards keep the macro out of them.
#pragma once
#include <torch/torch.h>
#include <cuda_runtime.h>

#define kBFloat16 kHalf
