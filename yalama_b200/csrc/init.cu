// Weight initialisation and dtype conversion on the device.
//
// fill_normal reproduces, element for element, the counter-based N(0, std)
// generator of yalama_b200/synth.py (SplitMix64 finaliser of Steele, Lea and
// Flood, OOPSLA 2014, on counters 2i and 2i+1 of the stream keyed by
// mix(seed) ^ fnv1a64(tensor name), then Box-Muller in double precision and
// one rounding to FP16), so a random-init engine holds the same weights as a
// snapshot written by synth.write_snapshot with the same seed.
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <cuda_bf16.h>
#include <algorithm>

namespace ylm {

__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(__half *dst, int64_t rows, int64_t cols, int64_t ld, uint64_t key, int64_t row0,
                                   int64_t col0, int64_t full_cols, double stdv)
{
    const uint64_t golden = 0x9E3779B97F4A7C15ull;
    const int64_t n = rows * cols;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x)
    {
        const int64_t r = t / cols, c = t % cols;
        const uint64_t i = (uint64_t)((row0 + r) * full_cols + col0 + c);
        const uint64_t z1 = mix64(key + (2ull * i) * golden);
        const uint64_t z2 = mix64(key + (2ull * i + 1ull) * golden);
        const double u1 = ((double)(z1 >> 11) + 1.0) * 0x1.0p-53;
        const double u2 = (double)(z2 >> 11) * 0x1.0p-53;
        const double v = sqrt(-2.0 * log(u1)) * cos(2.0 * 3.141592653589793 * u2);
        dst[r * ld + c] = __double2half(stdv * v);
    }
}

cudaError_t fill_normal_launch(__half *dst, int64_t rows, int64_t cols, int64_t ld, uint64_t key, int64_t row0,
                               int64_t col0, int64_t full_cols, double stdv, cudaStream_t s)
{
    const int64_t n = rows * cols;
    if (n <= 0)
        return cudaSuccess;
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 32);
    fill_normal_kernel<<<blocks, 256, 0, s>>>(dst, rows, cols, ld, key, row0, col0, full_cols, stdv);
    return cudaGetLastError();
}

__global__ void fill_const_kernel(__half *dst, int64_t n, float v)
{
    const __half h = __float2half_rn(v);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x)
        dst[t] = h;
}

cudaError_t fill_const_launch(__half *dst, int64_t n, float v, cudaStream_t s)
{
    if (n <= 0)
        return cudaSuccess;
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 32);
    fill_const_kernel<<<blocks, 256, 0, s>>>(dst, n, v);
    return cudaGetLastError();
}

// A dense band [nr][nc] of BF16 (src_dtype 1) or F32 (2) values -> FP16 rows
// of `dst` with row stride `ld`, rounded to nearest even (as __float2half_rn
// on the host). Grid: x over column blocks, y over rows (nr <= 65535).
__global__ void convert_rows_kernel(const void *src, int src_dtype, int64_t nc, __half *dst, int64_t ld)
{
    const int64_t r = blockIdx.y;
    __half *d = dst + r * ld;
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < nc; c += (int64_t)gridDim.x * blockDim.x)
    {
        const int64_t t = r * nc + c;
        const float f = src_dtype == 1 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(src)[t])
                                       : reinterpret_cast<const float *>(src)[t];
        d[c] = __float2half_rn(f);
    }
}

cudaError_t convert_rows_launch(const void *src, int src_dtype, int64_t nr, int64_t nc, __half *dst, int64_t ld,
                                cudaStream_t s)
{
    if (nr <= 0 || nc <= 0)
        return cudaSuccess;
    if (nr > 65535 || (src_dtype != 1 && src_dtype != 2))
        return cudaErrorInvalidValue;
    const unsigned bx = (unsigned)std::min<int64_t>((nc + 255) / 256, 16);
    convert_rows_kernel<<<dim3(bx, (unsigned)nr), 256, 0, s>>>(src, src_dtype, nc, dst, ld);
    return cudaGetLastError();
}

cudaError_t kernels_prepare()
{
    cudaError_t e = gemv_prepare();
    if (e == cudaSuccess)
        e = attn_prepare();
    if (e == cudaSuccess)
        e = attn_prefill_prepare();
    if (e == cudaSuccess)
        e = attn_prefill_tc_prepare();
    if (e == cudaSuccess)
        e = sample_prepare();
    if (e == cudaSuccess)
        e = gemm_tc_prepare();
    return e;
}

} // namespace ylm
