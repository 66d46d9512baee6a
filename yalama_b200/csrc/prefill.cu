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
// ModelBase.cpp:724-736 with FP16 rounding after each op. One CTA per row;
// each thread holds its 16-byte chunks of the row in registers, so the row is
// read from memory once (RN_CHUNKS x 8 halves x RN_THREADS covers H <= 8192).
constexpr int RN_THREADS = 128, RN_CHUNKS = 8;

__global__ void __launch_bounds__(RN_THREADS) rmsnorm_rows_kernel(const __half *x, const __half *w, float eps, int H,
                                                                 __half *y)
{
    __shared__ float red[RN_THREADS / 32];
    const int t = blockIdx.x, nv = H >> 3;
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + (int64_t)t * H);
    uint4 v[RN_CHUNKS];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < RN_CHUNKS; c++)
    {
        const int i = threadIdx.x + c * RN_THREADS;
        if (i < nv)
        {
            v[c] = xr[i];
            const __half *h = reinterpret_cast<const __half *>(&v[c]);
#pragma unroll
            for (int e = 0; e < 8; e++)
            {
                const float f = h2f(h[e]);
                ss += rh(f * f);
            }
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < RN_THREADS / 32; i++)
        tot += red[i];
    const float mean = rh(tot * (1.0f / (float)H));
    const float d = rh(rsqrtf(mean + eps));
    const uint4 *wr = reinterpret_cast<const uint4 *>(w);
    uint4 *yr = reinterpret_cast<uint4 *>(y + (int64_t)t * H);
#pragma unroll
    for (int c = 0; c < RN_CHUNKS; c++)
    {
        const int i = threadIdx.x + c * RN_THREADS;
        if (i < nv)
        {
            const uint4 wv = wr[i];
            const __half *h = reinterpret_cast<const __half *>(&v[c]);
            const __half *wh = reinterpret_cast<const __half *>(&wv);
            uint4 o;
            __half *oh = reinterpret_cast<__half *>(&o);
#pragma unroll
            for (int e = 0; e < 8; e++)
                oh[e] = f2h(rh(h2f(h[e]) * d) * h2f(wh[e]));
            yr[i] = o;
        }
    }
}

// Rows whose width is not a multiple of 8 halves or above the register budget.
__global__ void rmsnorm_rows_scalar_kernel(const __half *x, const __half *w, float eps, int H, __half *y)
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
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                           reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    if (aligned && H % 8 == 0 && H <= 8 * RN_THREADS * RN_CHUNKS)
        rmsnorm_rows_kernel<<<T, RN_THREADS, 0, s>>>(x, w, eps, H, y);
    else
        rmsnorm_rows_scalar_kernel<<<T, 256, 0, s>>>(x, w, eps, H, y);
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
// grid (T, ceil((hq + 2*hkv) / QP_WARPS)), one warp per (token, head); lane l
// holds head dims 4l..4l+3 (8-byte loads and stores). Positions pos0 + t.
constexpr int QP_WARPS = 4;

__device__ __forceinline__ void ld4h(const __half *p, float x[4])
{
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const __half *h = reinterpret_cast<const __half *>(&u);
#pragma unroll
    for (int e = 0; e < 4; e++)
        x[e] = h2f(h[e]);
}

__global__ void __launch_bounds__(QP_WARPS * 32) qkv_post_prefill_kernel(const QkvPostArgs a)
{
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x, h = blockIdx.y * QP_WARPS + (threadIdx.x >> 5);
    if (h >= a.hq + 2 * a.hkv)
        return;
    const int width = (a.hq + 2 * a.hkv) * YLM_HEAD_DIM;
    const __half *src = a.qkv + (int64_t)t * width + (int64_t)h * YLM_HEAD_DIM;
    const int pos = a.pos0 + t;
    if (h >= a.hq + a.hkv)
    {
        const int g = h - a.hq - a.hkv;
        __half *dst = a.v_cache + ((int64_t)g * a.cap + pos) * YLM_HEAD_DIM;
        reinterpret_cast<uint2 *>(dst)[lane] = reinterpret_cast<const uint2 *>(src)[lane];
        return;
    }
    const bool is_q = h < a.hq;
    float x[4];
    ld4h(src + lane * 4, x);
    const __half *nw = is_q ? a.q_norm : a.k_norm;
    if (nw)
    {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++)
            ss += rh(x[e] * x[e]);
        ss = warp_sum(ss);
        const float mean = rh(ss * (1.0f / YLM_HEAD_DIM));
        const float dn = rh(rsqrtf(mean + a.eps));
        float wv[4];
        ld4h(nw + lane * 4, wv);
#pragma unroll
        for (int e = 0; e < 4; e++)
            x[e] = rh(rh(x[e] * dn) * wv[e]);
    }
    float px[4];
#pragma unroll
    for (int e = 0; e < 4; e++)
        px[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    float cv[4], sv[4];
    ld4h(a.rope_cos + (int64_t)pos * 64 + (lane & 15) * 4, cv);
    ld4h(a.rope_sin + (int64_t)pos * 64 + (lane & 15) * 4, sv);
    __half *dst = is_q ? a.q_out + (int64_t)t * a.hq * YLM_HEAD_DIM + (int64_t)h * YLM_HEAD_DIM
                       : a.k_cache + ((int64_t)(h - a.hq) * a.cap + pos) * YLM_HEAD_DIM;
    uint2 o;
    __half *oh = reinterpret_cast<__half *>(&o);
#pragma unroll
    for (int e = 0; e < 4; e++)
    {
        const float rot = lane < 16 ? -px[e] : px[e];
        oh[e] = f2h(rh(rh(x[e] * cv[e]) + rh(rot * sv[e])));
    }
    reinterpret_cast<uint2 *>(dst)[lane] = o;
}

cudaError_t qkv_post_prefill_launch(const QkvPostArgs &a, cudaStream_t s)
{
    if (a.T <= 0)
        return cudaSuccess;
    const int heads = a.hq + 2 * a.hkv;
    qkv_post_prefill_kernel<<<dim3(a.T, (heads + QP_WARPS - 1) / QP_WARPS), QP_WARPS * 32, 0, s>>>(a);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ causal attention
// Flash attention on the tensor cores (mma.sync m16n8k16, FP16 inputs, FP32
// accumulation). Replaces the prefill SDPA of ModelBase.cpp:671-693 with the
// additive causal mask of :620-636 (implicit here) and without ExpandKV
// (:695-707): query head h reads KV head h / (hq / hkv) straight from the cache.
//
// grid (ceil(T / 64), hq), 4 warps; warp w owns query rows r0 + 16 w .. + 15.
// K and V tiles of 64 keys go through shared memory with cp.async, double
// buffered; rows are 256 bytes and their 16-byte chunks are XOR-swizzled by
// row & 7, so every ldmatrix phase reads eight distinct bank groups. The
// scores stay in registers: the m16n8 accumulator of S = Q K^T is the A
// fragment of P V after rounding P to FP16 (online softmax in FP32, base 2).
// Rows past the prompt are zero-filled in shared memory (never read from the
// cache), so a masked key never feeds a NaN into P V.
constexpr int FA_BQ = 64, FA_BK = 64, FA_THREADS = 128;
constexpr int FA_ROWB = YLM_HEAD_DIM * 2; // bytes per K / V / Q row

// byte offset of 16-byte chunk `chunk` of row `row` in a [rows][128] FP16 tile
__device__ __forceinline__ uint32_t fa_swz(int row, int chunk)
{
    return (uint32_t)(row * FA_ROWB + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void fa_cp16(uint32_t dst, const void *src, bool valid)
{
    // src-size 0 writes 16 zero bytes and reads nothing
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void fa_ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void fa_ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void fa_mma(float *d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t fa_pack(float lo, float hi)
{
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__global__ void __launch_bounds__(FA_THREADS) attn_prefill_kernel(const __half *q, const __half *kc, const __half *vc,
                                                                  int cap, int hq, int hkv, int T, __half *out)
{
    extern __shared__ __align__(128) uint8_t fa_smem[];
    // [Q 64 rows][K 2 x 64 rows][V 2 x 64 rows], each row 256 bytes
    const uint32_t s_q = (uint32_t)__cvta_generic_to_shared(fa_smem);
    const uint32_t s_k = s_q + FA_BQ * FA_ROWB;
    const uint32_t s_v = s_k + 2 * FA_BK * FA_ROWB;
    const int h = blockIdx.y, g = h / (hq / hkv);
    const int r0 = blockIdx.x * FA_BQ;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t qstride = (int64_t)hq * YLM_HEAD_DIM;
    const __half *kbase = kc + (int64_t)g * cap * YLM_HEAD_DIM;
    const __half *vbase = vc + (int64_t)g * cap * YLM_HEAD_DIM;

    // Q tile: 16 chunks of 16 bytes per row
    for (int i = tid; i < FA_BQ * 16; i += FA_THREADS)
    {
        const int r = i >> 4, c = i & 15;
        const bool ok = r0 + r < T;
        fa_cp16(s_q + fa_swz(r, c), q + (ok ? (int64_t)(r0 + r) * qstride + h * YLM_HEAD_DIM + c * 8 : 0), ok);
    }
    const int last_row = min(T, r0 + FA_BQ) - 1;
    const int ntiles = last_row / FA_BK + 1; // key tiles 0 .. the one holding the block's last row
    auto load_kv = [&](int j, int buf) {
        const int k0 = j * FA_BK;
        for (int i = tid; i < FA_BK * 16; i += FA_THREADS)
        {
            const int r = i >> 4, c = i & 15;
            const bool ok = k0 + r < T;
            const int64_t off = ok ? (int64_t)(k0 + r) * YLM_HEAD_DIM + c * 8 : 0;
            fa_cp16(s_k + buf * FA_BK * FA_ROWB + fa_swz(r, c), kbase + off, ok);
            fa_cp16(s_v + buf * FA_BK * FA_ROWB + fa_swz(r, c), vbase + off, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_kv(0, 0); // (the Q copies join this group)

    const int g4 = lane >> 2, c4 = lane & 3; // accumulator row / column pair of this lane
    const int qr = warp * 16;                 // this warp's first row in the tile
    const int row_a = r0 + qr + g4, row_b = row_a + 8;
    const float sl2 = 0.08838834764831845f * 1.4426950408889634f; // 1/sqrt(128) * log2(e)
    uint32_t qf[8][4];                                             // Q A-fragments, 8 steps of 16 dims
    float o[16][4];                                                // O accumulators, 16 tiles of 8 dims
#pragma unroll
    for (int j = 0; j < 16; j++)
        o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

    for (int j = 0; j < ntiles; j++)
    {
        const int buf = j & 1;
        if (j + 1 < ntiles)
        {
            load_kv(j + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        }
        else
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        if (j == 0)
        {
            // x4 matrices: (rows 0-7, dims 0-7), (rows 8-15, dims 0-7), (rows 0-7, dims 8-15), (rows 8-15, dims 8-15)
            const int mrow = qr + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int kk = 0; kk < 8; kk++)
                fa_ldsm_x4(s_q + fa_swz(mrow, kk * 2 + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
        }
        const uint32_t kb = s_k + buf * FA_BK * FA_ROWB, vb = s_v + buf * FA_BK * FA_ROWB;
        // S = Q K^T: 8 tiles of 8 keys
        float sc[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++)
            sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++)
        {
#pragma unroll
            for (int n = 0; n < 8; n += 2)
            {
                // matrices: (keys 8n.., dims 16kk..), (8n.., 16kk+8..), (8n+8.., 16kk..), (8n+8.., 16kk+8..)
                const int krow = n * 8 + (lane & 7) + (lane >> 4) * 8;
                const int kch = kk * 2 + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                fa_ldsm_x4(kb + fa_swz(krow, kch), b0, b1, b2, b3);
                fa_mma(sc[n], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
                fa_mma(sc[n + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
            }
        }
        // scale, causal mask, online softmax (rows row_a and row_b, 4 lanes per row)
        const int k0 = j * FA_BK;
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int n = 0; n < 8; n++)
        {
            const int key = k0 + n * 8 + c4 * 2;
            sc[n][0] = key <= row_a ? sc[n][0] * sl2 : -INFINITY;
            sc[n][1] = key + 1 <= row_a ? sc[n][1] * sl2 : -INFINITY;
            sc[n][2] = key <= row_b ? sc[n][2] * sl2 : -INFINITY;
            sc[n][3] = key + 1 <= row_b ? sc[n][3] * sl2 : -INFINITY;
            mx_a = fmaxf(mx_a, fmaxf(sc[n][0], sc[n][1]));
            mx_b = fmaxf(mx_b, fmaxf(sc[n][2], sc[n][3]));
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        // each tile holds key k0 <= every row of this block, so the maxima are finite
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float cr_a = exp2f(m_a - mn_a), cr_b = exp2f(m_b - mn_b);
        m_a = mn_a;
        m_b = mn_b;
        float sum_a = 0.f, sum_b = 0.f;
        uint32_t pf[4][4]; // P A-fragments, 4 steps of 16 keys
#pragma unroll
        for (int n = 0; n < 8; n++)
        {
            const float p0 = exp2f(sc[n][0] - mn_a), p1 = exp2f(sc[n][1] - mn_a);
            const float p2 = exp2f(sc[n][2] - mn_b), p3 = exp2f(sc[n][3] - mn_b);
            sum_a += p0 + p1;
            sum_b += p2 + p3;
            pf[n >> 1][(n & 1) * 2 + 0] = fa_pack(p0, p1);
            pf[n >> 1][(n & 1) * 2 + 1] = fa_pack(p2, p3);
        }
        l_a = l_a * cr_a + sum_a;
        l_b = l_b * cr_b + sum_b;
#pragma unroll
        for (int d = 0; d < 16; d++)
        {
            o[d][0] *= cr_a;
            o[d][1] *= cr_a;
            o[d][2] *= cr_b;
            o[d][3] *= cr_b;
        }
        // O += P V: 4 steps of 16 keys x 16 tiles of 8 dims
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
        {
#pragma unroll
            for (int d = 0; d < 16; d += 2)
            {
                // transposed: (keys 16kk.., dims 8d..), (16kk+8.., 8d..), (16kk.., 8d+8..), (16kk+8.., 8d+8..)
                const int vrow = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int vch = d + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                fa_ldsm_x4_t(vb + fa_swz(vrow, vch), b0, b1, b2, b3);
                fa_mma(o[d], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b0, b1);
                fa_mma(o[d + 1], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b2, b3);
            }
        }
        __syncthreads(); // this buffer is refilled by the next iteration's loads
    }
    // row sums over the 4 lanes of each row, then O / l
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    const float inv_a = 1.f / l_a, inv_b = 1.f / l_b;
#pragma unroll
    for (int d = 0; d < 16; d++)
    {
        const int col = h * YLM_HEAD_DIM + d * 8 + c4 * 2;
        if (row_a < T)
            *reinterpret_cast<__half2 *>(out + (int64_t)row_a * qstride + col) =
                __floats2half2_rn(o[d][0] * inv_a, o[d][1] * inv_a);
        if (row_b < T)
            *reinterpret_cast<__half2 *>(out + (int64_t)row_b * qstride + col) =
                __floats2half2_rn(o[d][2] * inv_b, o[d][3] * inv_b);
    }
}

static size_t fa_smem_bytes() { return (size_t)(FA_BQ + 4 * FA_BK) * FA_ROWB; }

cudaError_t attn_prefill_prepare()
{
    return cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)fa_smem_bytes());
}

cudaError_t attn_prefill_launch(const __half *q, const __half *k_cache, const __half *v_cache, int cap, int hq,
                                int hkv, int T, __half *out, cudaStream_t s)
{
    if (T <= 0)
        return cudaSuccess;
    if (T > cap || hq % hkv)
        return cudaErrorInvalidValue;
    attn_prefill_kernel<<<dim3((T + FA_BQ - 1) / FA_BQ, hq), FA_THREADS, fa_smem_bytes(), s>>>(q, k_cache, v_cache,
                                                                                              cap, hq, hkv, T, out);
    return cudaGetLastError();
}

} // namespace ylm
