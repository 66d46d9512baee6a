// Prefill (T prompt tokens at once) building blocks.
//
// The reference's prefill runs the same per-layer ops as decode over [1, T, H]
// (src/models/ModelBase.cpp:396-471), with RoPE at positions 0..T-1 (:539-543),
// a bulk KV write (:557-563) and causal SDPA with an additive -65504 mask
// (:620-636). Here: row-wise embedding gather and RMSNorm, a GEMM with fused
// bias / residual / SwiGLU epilogues, a per-(token, head) kernel for q/k-norm,
// RoPE and the KV write, and causal attention that reads K/V straight from the
// cache with the mask implicit. FP16 storage, FP32 accumulation, the
// reference's rounding after every op.
#include "ylm_common.cuh"
#include "ylm_kernels.h"

namespace ylm {

// ------------------------------------------------------------------ embedding
__global__ void embed_rows_kernel(const int64_t *ids, int T, const __half *emb, int64_t vocab, int H, __half *x,
                                  int *err)
{
    const int t = blockIdx.x;
    int64_t id = ids[t];
    if (id < 0 || id >= vocab)
    {
        if (threadIdx.x == 0 && err)
            atomicExch(err, YLM_DEV_ERR_BAD_TOKEN);
        id = 0;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(emb + id * (int64_t)H);
    uint4 *dst = reinterpret_cast<uint4 *>(x + (int64_t)t * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x)
        dst[i] = src[i];
}

cudaError_t embed_rows_launch(const int64_t *ids, int T, const __half *emb, int64_t vocab, int H, __half *x, int *err,
                              cudaStream_t s)
{
    if (T <= 0)
        return cudaSuccess;
    embed_rows_kernel<<<T, 256, 0, s>>>(ids, T, emb, vocab, H, x, err);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ residual add
// ModelBase.cpp:426, 437 (x = x + y, rounded to FP16), used after the
// tensor-parallel all-reduce of the O and down projections.
__global__ void resid_add_kernel(__half *x, const __half *y, int64_t n)
{
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = f2h(h2f(x[i]) + h2f(y[i]));
}

cudaError_t resid_add_rows_launch(__half *x, const __half *y, int64_t n, cudaStream_t s)
{
    if (n <= 0)
        return cudaSuccess;
    const int blocks = (int)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
    resid_add_kernel<<<blocks, 256, 0, s>>>(x, y, n);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ RMSNorm rows
// ModelBase.cpp:724-736 with FP16 rounding after each op.
__global__ void rmsnorm_rows_kernel(const __half *x, const __half *w, float eps, int H, __half *y)
{
    __shared__ float red[32];
    const int t = blockIdx.x;
    const __half *xr = x + (int64_t)t * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x)
    {
        const float f = h2f(xr[i]);
        ss += rh(f * f);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++)
        tot += red[i];
    const float mean = rh(tot * (1.0f / (float)H));
    const float d = rh(rsqrtf(mean + eps));
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        y[(int64_t)t * H + i] = f2h(rh(h2f(xr[i]) * d) * h2f(w[i]));
}

cudaError_t rmsnorm_rows_launch(const __half *x, const __half *w, float eps, int T, int H, __half *y, cudaStream_t s)
{
    if (T <= 0)
        return cudaSuccess;
    rmsnorm_rows_kernel<<<T, 256, 0, s>>>(x, w, eps, H, y);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ GEMM (CUDA cores)
// C[T, N] = A[T, K] W[N, K]^T. 64x64 output tile per CTA, 16x16 threads with a
// 4x4 register tile each, K staged 32 at a time in shared memory (transposed
// so the inner loop reads contiguous rows).
constexpr int GM_BM = 64, GM_BN = 64, GM_BK = 32;

__global__ void __launch_bounds__(256) gemm_simt_kernel(const __half *A, int lda, const __half *W, int T, int N, int K,
                                                        int epi, const __half *bias, __half *C, int ldc)
{
    __shared__ float As[GM_BK][GM_BM + 4];
    __shared__ float Ws[GM_BK][GM_BN + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * GM_BM, n0 = blockIdx.x * GM_BN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += GM_BK)
    {
        for (int i = threadIdx.x; i < GM_BM * GM_BK; i += 256)
        {
            const int r = i / GM_BK, kk = i % GM_BK;
            const int m = m0 + r, k = k0 + kk;
            As[kk][r] = (m < T && k < K) ? h2f(A[(int64_t)m * lda + k]) : 0.f;
            const int n = n0 + r;
            Ws[kk][r] = (n < N && k < K) ? h2f(W[(int64_t)n * K + k]) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < GM_BK; kk++)
        {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
            {
                a[i] = As[kk][ty * 4 + i];
                b[i] = Ws[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        const int m = m0 + ty * 4 + i;
        if (m >= T)
            continue;
#pragma unroll
        for (int j = 0; j < 4; j++)
        {
            const int n = n0 + tx * 4 + j;
            if (n >= N)
                continue;
            if (epi == GEMM_STORE)
            {
                float y = acc[i][j];
                if (bias)
                    y = rh(y) + h2f(bias[n]);
                C[(int64_t)m * ldc + n] = f2h(y);
            }
            else if (epi == GEMM_RESID)
            {
                __half *c = C + (int64_t)m * ldc + n;
                *c = f2h(h2f(*c) + rh(acc[i][j]));
            }
            else if ((j & 1) == 0 && n + 1 < N)
            {
                // SwiGLU over interleaved (gate, up) columns; tx*4 is even
                const float g = rh(acc[i][j]);
                const float u = rh(acc[i][j + 1]);
                const float sg = rh(g / (1.0f + expf(-g)));
                C[(int64_t)m * ldc + (n >> 1)] = f2h(sg * u);
            }
        }
    }
}

cudaError_t gemm_launch(const __half *A, int lda, const __half *W, int T, int N, int K, int epi, const __half *bias,
                        __half *C, int ldc, cudaStream_t s)
{
    if (T <= 0)
        return cudaSuccess;
    dim3 grid((N + GM_BN - 1) / GM_BN, (T + GM_BM - 1) / GM_BM);
    gemm_simt_kernel<<<grid, 256, 0, s>>>(A, lda, W, T, N, K, epi, bias, C, ldc);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ q/k-norm, RoPE, KV write
// grid (T, hq + 2*hkv), one warp per (token, head). Positions pos0 + t.
__global__ void qkv_post_prefill_kernel(const QkvPostArgs a)
{
    const int t = blockIdx.x, h = blockIdx.y, lane = threadIdx.x;
    const int width = (a.hq + 2 * a.hkv) * YLM_HEAD_DIM;
    const __half *src = a.qkv + (int64_t)t * width + (int64_t)h * YLM_HEAD_DIM;
    const int pos = a.pos0 + t;
    if (h >= a.hq + a.hkv)
    {
        const int g = h - a.hq - a.hkv;
        __half *dst = a.v_cache + ((int64_t)g * a.cap + pos) * YLM_HEAD_DIM;
        for (int d = lane; d < YLM_HEAD_DIM; d += 32)
            dst[d] = src[d];
        return;
    }
    const bool is_q = h < a.hq;
    float x[4];
    for (int e = 0; e < 4; e++)
        x[e] = h2f(src[lane * 4 + e]);
    const __half *nw = is_q ? a.q_norm : a.k_norm;
    if (nw)
    {
        float ss = 0.f;
        for (int e = 0; e < 4; e++)
            ss += rh(x[e] * x[e]);
        ss = warp_sum(ss);
        const float mean = rh(ss * (1.0f / YLM_HEAD_DIM));
        const float dn = rh(rsqrtf(mean + a.eps));
        for (int e = 0; e < 4; e++)
            x[e] = rh(rh(x[e] * dn) * h2f(nw[lane * 4 + e]));
    }
    float px[4];
    for (int e = 0; e < 4; e++)
        px[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const __half *cr = a.rope_cos + (int64_t)pos * 64, *sr = a.rope_sin + (int64_t)pos * 64;
    __half *dst = is_q ? a.q_out + (int64_t)t * a.hq * YLM_HEAD_DIM + (int64_t)h * YLM_HEAD_DIM
                       : a.k_cache + ((int64_t)(h - a.hq) * a.cap + pos) * YLM_HEAD_DIM;
    for (int e = 0; e < 4; e++)
    {
        const int d = lane * 4 + e;
        const float rot = d < 64 ? -px[e] : px[e];
        dst[d] = f2h(rh(rh(x[e] * h2f(cr[d & 63])) + rh(rot * h2f(sr[d & 63]))));
    }
}

cudaError_t qkv_post_prefill_launch(const QkvPostArgs &a, cudaStream_t s)
{
    if (a.T <= 0)
        return cudaSuccess;
    qkv_post_prefill_kernel<<<dim3(a.T, a.hq + 2 * a.hkv), 32, 0, s>>>(a);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ causal attention
// grid (ceil(T/32), hq), 4 warps, each warp 8 query rows. Keys in tiles of 32
// from the KV cache (slots [0, T)); lane j scores key j of the tile.
constexpr int AP_ROWS = 32, AP_KT = 32, AP_RPW = AP_ROWS / 4;

__global__ void __launch_bounds__(128) attn_prefill_kernel(const __half *q, const __half *kc, const __half *vc, int cap,
                                                           int hq, int hkv, int T, __half *out)
{
    __shared__ float Kt[YLM_HEAD_DIM][AP_KT]; // transposed: Kt[d][key]
    __shared__ float Vt[AP_KT][YLM_HEAD_DIM];
    __shared__ float Qs[AP_ROWS][YLM_HEAD_DIM];
    const int h = blockIdx.y, g = h / (hq / hkv);
    const int r0 = blockIdx.x * AP_ROWS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float scale = 0.08838834764831845f * 1.4426950408889634f;
    for (int i = threadIdx.x; i < AP_ROWS * YLM_HEAD_DIM; i += 128)
    {
        const int r = i / YLM_HEAD_DIM, d = i % YLM_HEAD_DIM;
        Qs[r][d] = (r0 + r < T) ? h2f(q[(int64_t)(r0 + r) * hq * YLM_HEAD_DIM + h * YLM_HEAD_DIM + d]) * scale : 0.f;
    }
    float m[AP_RPW], l[AP_RPW], o[AP_RPW][4];
    for (int i = 0; i < AP_RPW; i++)
    {
        m[i] = -INFINITY;
        l[i] = 0.f;
        for (int e = 0; e < 4; e++)
            o[i][e] = 0.f;
    }
    const int last_row = min(T, r0 + AP_ROWS) - 1;
    const __half *kbase = kc + (int64_t)g * cap * YLM_HEAD_DIM;
    const __half *vbase = vc + (int64_t)g * cap * YLM_HEAD_DIM;
    for (int k0 = 0; k0 <= last_row; k0 += AP_KT)
    {
        __syncthreads();
        for (int i = threadIdx.x; i < AP_KT * YLM_HEAD_DIM; i += 128)
        {
            const int j = i % AP_KT, d = i / AP_KT;
            Kt[d][j] = (k0 + j < T) ? h2f(kbase[(int64_t)(k0 + j) * YLM_HEAD_DIM + d]) : 0.f;
            const int jv = i / YLM_HEAD_DIM, dv = i % YLM_HEAD_DIM;
            Vt[jv][dv] = (k0 + jv < T) ? h2f(vbase[(int64_t)(k0 + jv) * YLM_HEAD_DIM + dv]) : 0.f;
        }
        __syncthreads();
        for (int i = 0; i < AP_RPW; i++)
        {
            const int row = r0 + warp * AP_RPW + i;
            if (row >= T || k0 > row)
                continue; // warp-uniform
            float sc = 0.f;
            for (int d = 0; d < YLM_HEAD_DIM; d++)
                sc = fmaf(Qs[warp * AP_RPW + i][d], Kt[d][lane], sc);
            const int key = k0 + lane;
            if (key > row)
                sc = -INFINITY;
            const float mt = warp_max(sc);
            const float mn = fmaxf(m[i], mt);
            const float c = exp2f(m[i] - mn);
            const float p = exp2f(sc - mn);
            l[i] = l[i] * c + warp_sum(p);
            for (int e = 0; e < 4; e++)
                o[i][e] *= c;
            for (int j = 0; j < AP_KT; j++)
            {
                const float pj = __shfl_sync(0xffffffffu, p, j);
                for (int e = 0; e < 4; e++)
                    o[i][e] = fmaf(pj, Vt[j][lane * 4 + e], o[i][e]);
            }
            m[i] = mn;
        }
    }
    for (int i = 0; i < AP_RPW; i++)
    {
        const int row = r0 + warp * AP_RPW + i;
        if (row >= T)
            continue;
        for (int e = 0; e < 4; e++)
            out[(int64_t)row * hq * YLM_HEAD_DIM + h * YLM_HEAD_DIM + lane * 4 + e] = f2h(o[i][e] / l[i]);
    }
}

cudaError_t attn_prefill_launch(const __half *q, const __half *k_cache, const __half *v_cache, int cap, int hq,
                                int hkv, int T, __half *out, cudaStream_t s)
{
    if (T <= 0)
        return cudaSuccess;
    attn_prefill_kernel<<<dim3((T + AP_ROWS - 1) / AP_ROWS, hq), 128, 0, s>>>(q, k_cache, v_cache, cap, hq, hkv, T, out);
    return cudaGetLastError();
}

} // namespace ylm
