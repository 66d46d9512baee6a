// Kernel parameter blocks and launchers shared by the engine and the kernels.
// Host-side declarations only; no torch types anywhere.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#define YLM_HEAD_DIM 128

// Device-side error words (written with atomicExch, read by the host after a step).
#define YLM_DEV_ERR_NONE 0
#define YLM_DEV_ERR_TIMEOUT_FULL 1
#define YLM_DEV_ERR_TIMEOUT_EMPTY 2
#define YLM_DEV_ERR_TIMEOUT_DRAIN 3
#define YLM_DEV_ERR_BAD_TOKEN 4
#define YLM_DEV_ERR_BAD_STATE 5
#define YLM_DEV_ERR_TIMEOUT_PEER 6

namespace ylm {

// Per-engine device-resident step state. The decode graph reads the token,
// slot and RoPE position from here, so one captured graph serves every step.
struct StepState
{
    int64_t token;        // input token of the decode step
    int64_t next_token;   // sampler output
    int64_t sample_calls; // sampler calls so far (Philox counter)
    int32_t slot;         // KV slot written this step
    int32_t rope_pos;     // RoPE position of this step's token
    int32_t err;          // device error word (YLM_DEV_ERR_*)
    int32_t greedy;       // 1: argmax; 0: top-k + temperature
    int32_t top_k;        // 1..64
    float inv_temp;       // 1/temperature (FP32)
    float u_override;     // >= 0: uniform draw to use instead of Philox (tests)
    int32_t advance;      // 1: after sampling, token=next, slot++, rope_pos++
    uint64_t seed;        // Philox key
    float u_used;         // the uniform the last top-k draw used
    int32_t pad;
};

// ------------------------------------------------------------------ GEMV
enum GemvPro
{
    PRO_VEC = 0,          // input vector as is
    PRO_RMSNORM = 1,      // RMSNorm(x) * w of the residual stream
    PRO_EMBED_RMSNORM = 2 // x = embedding[state.token]; CTA 0 writes x to resid_out
};
enum GemvEpi
{
    EPI_STORE = 0, // out[row] = fp16(y) (+ bias, rounded again)
    EPI_RESID = 1, // resid[row] = fp16(resid[row] + fp16(y))
    EPI_SWIGLU = 2 // rows (2p, 2p+1) = (gate_p, up_p): out[p] = fp16(fp16(silu(g)) * u)
};

struct GemvPlan
{
    const __half *w;
    int N, K;    // rows, columns of W
    int rb;      // rows per CTA (a contiguous range of W)
    int grid;    // CTAs
    int n_kc;    // 2048-column chunks per row
    int k_pad;   // n_kc * 2048
    int pair;    // 1: SwiGLU row pairs
    size_t smem; // dynamic shared memory bytes
};

struct GemvArgs
{
    const __half *w = nullptr;      // set from the plan
    const __half *x = nullptr;      // input vector (PRO_VEC) or residual stream (PRO_RMSNORM)
    const __half *norm_w = nullptr; // RMSNorm weight [K]
    float eps = 0.f;
    const __half *emb = nullptr;    // PRO_EMBED_RMSNORM: embedding [V, K]
    int64_t vocab = 0;
    const StepState *state = nullptr;
    __half *resid_out = nullptr;    // PRO_EMBED_RMSNORM: x written here by CTA 0
    __half *out = nullptr;
    const __half *bias = nullptr;
    __half *resid = nullptr;
    int *err = nullptr;
};

bool gemv_make_plan(GemvPlan *plan, const __half *w, int N, int K, int pair, int num_sms);
cudaError_t gemv_launch(const GemvPlan &plan, int pro, int epi, const GemvArgs &a, cudaStream_t s, bool pdl);
cudaError_t gemv_prepare();

// ------------------------------------------------------------------ decode attention
struct AttnArgs
{
    const __half *qkv;    // [ (hq + 2 hkv) * 128 ]: q heads, k heads, v heads
    const __half *q_norm; // [128] or null (Qwen3 q/k RMSNorm)
    const __half *k_norm;
    float eps;
    const __half *rope_cos; // [max_pos][64]
    const __half *rope_sin;
    int max_pos;
    __half *k_cache; // this layer, [hkv][cap][128]
    __half *v_cache;
    int cap;
    int hq, hkv;
    int splits;
    float *partial; // [hq][splits][2 + 128]
    int *counters;  // [hkv], zero between launches
    __half *out;    // [hq * 128]
    const StepState *state;
    int *err;
};
size_t attn_partial_floats(int hq, int splits);
int attn_default_splits(int hkv, int num_sms);
cudaError_t attn_decode_launch(const AttnArgs &a, cudaStream_t s, bool pdl);
cudaError_t attn_prepare();
// Process-wide: launch the split-K kernel (global partials, tickets) even where
// cluster launches are available; whether later launches use it.
void attn_force_split_kernel(bool on);
bool attn_uses_split_kernel();

// ------------------------------------------------------------------ sampler
struct SampleArgs
{
    const __half *logits;
    int64_t vocab;
    const uint32_t *mask_bits; // V bits, 1 = masked special id; null = none
    StepState *state;
    uint64_t *cand;   // [parts][64]
    int *cand_count;  // [parts]
    int *counter;     // zero between launches
    int parts;
    int64_t *dbg_ids; // [64] final top-k ids in sampling order (or null)
    float *dbg_probs; // [64]
    int *err;
};
int sample_parts(int64_t vocab, int num_sms);
cudaError_t sample_launch(const SampleArgs &a, cudaStream_t s, bool pdl);
cudaError_t sample_prepare();

// ------------------------------------------------------------------ persistent GEMV segments
// The projections between two attention launches of a decode step run as one
// persistent launch of one CTA per SM (decode_step.cu).
struct DsPhase
{
    int pro;         // GemvPro
    int epi;         // GemvEpi
    const __half *w; // [N, K] row-major
    int N, K;
    const __half *x;    // PRO_VEC / RMSNorm input written by an earlier launch (plain FP16), or null
    const uint32_t *xt; // input written tagged by phase `src` of the same launch, or null
    int src;
    const __half *norm_w; // RMSNorm weight [K]
    __half *out;          // EPI_STORE output (read by a later launch)
    uint32_t *out_t;      // EPI_SWIGLU output, tagged
    const __half *bias;   // EPI_STORE bias or null
    uint32_t *resid_t;    // EPI_RESID target, the tagged residual stream; PRO_EMBED_RMSNORM: each
                          // CTA writes its rows of the embedding row here
    int mbox;             // tensor parallel EPI_RESID: 0 none, 1 / 2 the mailbox set the partial
                          // rows are all-reduced through (see DsArgs::mb)
    int greedy_pick;      // EPI_STORE of the logits: also pick the argmax (DsArgs::pick_*)
};
#define DS_MAX_SEG_PHASES 4
struct DsArgs
{
    DsPhase ph[DS_MAX_SEG_PHASES]; // this launch's phases (kernel parameters: constant bank)
    int nph;                       // phases in the step (tags)
    int p0, p1;                    // this launch runs the step's phases [p0, p1); ph[i - p0] is phase i
    int last;          // 1: the step's last segment (advances *gen)
    float eps;
    const __half *emb;
    int64_t vocab;
    const StepState *state;
    const uint32_t *xt; // tagged residual stream [hidden]
    int hidden;         // each CTA keeps its rows of it (split like an N = hidden projection);
                        // a CTA's rows must not exceed the block size
    unsigned *gen;      // decode steps completed
    int *err;
    unsigned long long wait_ns; // bound of every wait (YLM_DEV_ERR_TIMEOUT_PEER after it)
    // greedy sampling fused into the lm_head epilogue (a phase with greedy_pick):
    // each CTA's best key goes to pick_cand[CTA], the last CTA to finish
    // (pick_counter, zero between launches) writes the token into pick_state
    StepState *pick_state;
    unsigned long long *pick_cand;
    int *pick_counter;
    // tensor parallelism: pick_mb[q] = rank q's pick mailbox ([tp][4] tagged
    // words, slot r written by rank r), mapped into this process; a device
    // array of tp pointers (null without tensor parallelism)
    uint32_t *const *pick_mb;
    // tensor parallelism: rank `rank` of `tp`; mb[s][q] is mailbox set s + 1 of
    // rank q ([tp][hidden] tagged words, slot r written by rank r), mapped
    // into this process (peer memory over NVLink for q != rank)
    int tp, rank;
    uint32_t *mb[2][8];
    // exchange timing (tensor parallel, may be null): [0] += ns from block 0
    // thread 0's first partial store to the arrival of every rank's partial of
    // its row, [1] += 1, per exchange
    unsigned long long *xstat;
    int tab_bytes;  // shared-memory layout: phase table, work area, residual rows
    int work_bytes; // GEMV input vector, partials, RMSNorm scratch
    int kpad_max;   // largest input vector (halves, multiple of the task width)
    int part_max;   // largest per-CTA task count of a phase
};
int ds_threads();
int ds_task_cols();
int ds_tab_bytes(); // shared-memory bytes of a launch's phase table
// Shared-memory opt-in and the resulting CTAs per SM.
cudaError_t ds_prepare(size_t smem, int *blocks_per_sm);
cudaError_t ds_launch(const DsArgs &a, size_t smem, int grid, cudaStream_t s);

// Shared-memory opt-in of every kernel on the current device (idempotent).
cudaError_t kernels_prepare();
// kernels_prepare() once per device, thread-safe (the kernel-level entry points).
cudaError_t prepare_device();

// Message returned by ylm_last_error() on the calling thread (kernel-level entry points).
void set_last_error(const char *msg);

// ------------------------------------------------------------------ prefill (T tokens)
cudaError_t embed_rows_launch(const int64_t *ids, int T, const __half *emb, int64_t vocab, int H, __half *x, int *err,
                              cudaStream_t s);
cudaError_t rmsnorm_rows_launch(const __half *x, const __half *w, float eps, int T, int H, __half *y, cudaStream_t s);

enum GemmEpi
{
    GEMM_STORE = 0,
    GEMM_RESID = 1,
    GEMM_SWIGLU = 2
};
// C[T, N] = A[T, K] x W[N, K]^T with epilogue; A row stride lda, C row stride ldc.
cudaError_t gemm_launch(const __half *A, int lda, const __half *W, int T, int N, int K, int epi, const __half *bias,
                        __half *C, int ldc, cudaStream_t s);

// Tensor-core (tcgen05) GEMM with the same epilogues. Operand maps: A [T, K]
// (row stride lda) and W [N, K], both FP16 K-major, built once per buffer.
bool tc_make_a_map(CUtensorMap *map, const __half *A, int T, int K, int lda);
bool tc_make_w_map(CUtensorMap *map, const __half *W, int N, int K);
cudaError_t gemm_tc_launch(const CUtensorMap &amap, const CUtensorMap &wmap, int T, int N, int K, int epi,
                           const __half *bias, __half *C, int ldc, int *err, cudaStream_t s);
cudaError_t gemm_tc_prepare();

struct QkvPostArgs
{
    const __half *qkv; // [T][(hq + 2 hkv) * 128]
    const __half *q_norm, *k_norm;
    float eps;
    const __half *rope_cos, *rope_sin;
    __half *q_out; // [T][hq * 128]
    __half *k_cache, *v_cache;
    int cap, hq, hkv, T, pos0;
};
cudaError_t qkv_post_prefill_launch(const QkvPostArgs &a, cudaStream_t s);
// x[i] = fp16(x[i] + y[i]) (residual add after a tensor-parallel all-reduce)
cudaError_t resid_add_rows_launch(__half *x, const __half *y, int64_t n, cudaStream_t s);
// causal attention over KV slots [0, T): q [T][hq*128] -> out [T][hq*128]
cudaError_t attn_prefill_prepare();
// The same on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
cudaError_t attn_prefill_tc_prepare();
cudaError_t attn_prefill_tc_launch(const __half *q, const __half *k_cache, const __half *v_cache, int cap, int hq,
                                   int hkv, int T, __half *out, int *err, cudaStream_t s);
cudaError_t attn_prefill_launch(const __half *q, const __half *k_cache, const __half *v_cache, int cap, int hq,
                                int hkv, int T, __half *out, cudaStream_t s);

// ------------------------------------------------------------------ init
// dst[r * ld + c] = N(0, std) element ((row0 + r) * full_cols + col0 + c) of stream `key`
cudaError_t fill_normal_launch(__half *dst, int64_t rows, int64_t cols, int64_t ld, uint64_t key, int64_t row0,
                               int64_t col0, int64_t full_cols, double stdv, cudaStream_t s);
cudaError_t fill_const_launch(__half *dst, int64_t n, float v, cudaStream_t s);
// Dense [nr][nc] BF16 (1) / F32 (2) -> FP16 rows of dst (stride ld), nr <= 65535.
cudaError_t convert_rows_launch(const void *src, int src_dtype, int64_t nr, int64_t nc, __half *dst, int64_t ld,
                                cudaStream_t s);

} // namespace ylm
