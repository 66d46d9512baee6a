/*
 * yalama_b200 — C ABI of the B200-native batch-1 decode engine.
 *
 * The engine replaces the LibTorch token loop of the reference runtime
 * (Yaz-X/yalama): ModelBase::Infer with its per-layer forward and ChatSession::
 * Sample. Every entry point returns an int status (ylm_status); no C++
 * exception crosses this boundary and no torch type appears in it. One engine
 * serves one GPU (one tensor-parallel rank); a handle is not thread-safe, the
 * caller serialises calls the way ChatSession's inferMutex does
 * (src/ChatSession.cpp:19, 85-93).
 *
 * Paths cited as file:line refer to the reference project's tree.
 */
#ifndef YALAMA_B200_H
#define YALAMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 0..5 are GenerationError (include/enums/GenerationError.h:1-8)
 * in the same order; the rest replace the exceptions the reference throws. */
typedef enum ylm_status {
    YLM_OK = 0,
    YLM_SEQUENCE_LENGTH_EXCEEDED = 1,
    YLM_KV_CACHE_EXCEEDED = 2, /* ModelBase::EnsureKVCapacity, src/models/ModelBase.cpp:853-866 */
    YLM_INVALID_PROMPT = 3,
    YLM_CANCELED = 4,
    YLM_GPU_QUEUE_TIMED_OUT = 5,
    YLM_INVALID_ARG = 16,
    YLM_NOT_READY = 17,   /* Infer before BeginInfer: ModelBase.cpp:401-402 throws */
    YLM_LOAD_ERROR = 18,  /* bad model folder / shards: ModelBase.cpp:25-73, Model.cpp:29-30 */
    YLM_CUDA_ERROR = 19,
    YLM_DEVICE_TIMEOUT = 20, /* a bounded device-side wait expired; the step was abandoned */
    YLM_COMM_ERROR = 21,     /* NCCL failure or peer timeout (tensor parallel) */
    YLM_UNSUPPORTED = 22     /* shape outside what the kernels handle (head_dim != 128, ...) */
} ylm_status;

/* ModelType (include/enums/ModelType.h:1-7) */
typedef enum ylm_model_type {
    YLM_MODEL_LLAMA = 1,
    YLM_MODEL_MISTRAL = 2,
    YLM_MODEL_QWEN2_5 = 3, /* q/k/v biases: src/models/Qwen2_5Model.cpp:16-47 */
    YLM_MODEL_QWEN3 = 4    /* per-head q/k RMSNorm: src/models/Qwen3Model.cpp:8-33 */
} ylm_model_type;

/* The ConfigManager model fields read from HF config.json
 * (src/ConfigManager.cpp:410-471, include/ConfigManager.h:16-33). */
typedef struct ylm_model_config {
    int32_t model_type;
    int32_t num_layers;
    int32_t hidden_size;
    int32_t num_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t intermediate_size;
    int32_t tie_word_embeddings; /* no lm_head.weight: ModelBase.cpp:148-155 falls back to the embedding */
    int64_t vocab_size;
    float rms_eps;
    float rope_theta;
    float rope_factor;      /* llama3 rope_scaling fields, ConfigManager.cpp:443-463 */
    float rope_low_freq;
    float rope_high_freq;
    int32_t rope_orig_max_pos;
    int32_t max_position_embeddings;
    int32_t eos_ids[8];     /* ConfigManager::EosIds */
    int32_t n_eos;
} ylm_model_config;

/* Engine options: the ConfigManager runtime flags that reach the token loop,
 * plus the engine's own. */
typedef struct ylm_engine_options {
    int32_t device;
    int32_t kv_cache_gb;      /* ConfigManager::KVCacheSizeInGB (default 2) */
    int32_t kv_cache_enabled; /* ConfigManager::IsKVCacheEnabled (default 1) */
    int32_t rope_compat;      /* 1 (default): a decode token written to slot s is rotated at s-1,
                                 as ModelBase.cpp:577-581 does; 0: rotated at s */
    int32_t rope_scaling;     /* 1: apply llama3 frequency scaling (the reference parses it,
                                 ConfigManager.cpp:448-463, but BuildRopeCache ignores it) */
    int32_t use_cuda_graph;   /* 1 (default): one graph launch per decode step */
    int32_t use_pdl;          /* programmatic dependent launch: 1 between all decode kernels,
                                 2 only into the projections, 0 (default) off */
    int32_t tp_rank;
    int32_t tp_size;          /* tensor-parallel ranks (1, 2, 4, 8); one engine per rank */
    const void *nccl_id;      /* 128-byte NCCL unique id from ylm_nccl_unique_id on rank 0 */
    uint64_t init_seed;       /* snapshot_dir == NULL: seeded N(0, init_std) weights, norms 1.0 */
    double init_std;
    int32_t zero_kv_on_begin; /* 1 (default): BeginInfer zeroes the cache like ModelBase.cpp:302-309 */
    int32_t prefill_tensor_cores; /* 1 (default): tcgen05 GEMMs for prefill; 0: CUDA-core GEMMs */
    int32_t decode_persistent;    /* 1 (default): the projections between two attention launches of a
                                     decode step run as one persistent kernel; with tensor parallelism
                                     its O and down epilogues all-reduce over NVLink peer memory;
                                     0: the per-op graph */
    int32_t wait_limit_us;        /* bound of every device-side wait of the persistent path (a
                                     producer phase's tagged output, a peer's partials), in
                                     microseconds; 0 (default): 2 s. A wait that expires records an
                                     error, the step's remaining waits give up at once and the call
                                     returns YLM_DEVICE_TIMEOUT; the engine stays usable. */
} ylm_engine_options;

/* ChatSession::Sample parameters (src/ChatSession.cpp:560-593). */
typedef struct ylm_sampling {
    int32_t greedy;            /* ConfigManager::IsGreedy */
    int32_t top_k;             /* ConfigManager::TopK, 1..64 */
    float temperature;         /* ConfigManager::Temp */
    uint64_t seed;             /* Philox key of the engine's draws */
    const int64_t *masked_ids; /* special ids forced to -1e9 before top-k (ChatSession.cpp:41-61, 573-576) */
    int32_t n_masked;
} ylm_sampling;

typedef struct ylm_engine ylm_engine;

/* ---- library ------------------------------------------------------------ */
const char *ylm_status_string(int status);
/* Message of the last failure on the calling thread ("" if none). */
const char *ylm_last_error(void);
int ylm_options_default(ylm_engine_options *opt);
/* Parse an HF config.json (ConfigManager::Load model section,
 * src/ConfigManager.cpp:389-471). */
int ylm_config_from_json(const char *config_json_path, ylm_model_config *cfg);
/* Resolve an HF hub root (refs/main -> snapshots/<hash>, ConfigManager.cpp:320-342)
 * into the snapshot directory. */
int ylm_resolve_snapshot(const char *hf_root, char *out, int32_t out_len);
/* NCCL unique id for a tensor-parallel group (call on rank 0, share the 128 bytes). */
int ylm_nccl_unique_id(void *out128);

/* ---- engine lifecycle: Model::Init (src/models/Model.cpp:10-34) ---------- */
/* snapshot_dir: folder with *.safetensors (ModelBase::Load, ModelBase.cpp:19-237);
 * NULL: random-init weights from opt->init_seed. cfg: model shape. */
int ylm_create(const char *snapshot_dir, const ylm_model_config *cfg, const ylm_engine_options *opt,
               ylm_engine **out);
int ylm_destroy(ylm_engine *e);

/* ---- token loop ----------------------------------------------------------- */
/* Model::BeginInfer (Model.cpp:36-41 -> ModelBase.cpp:296-310). */
int ylm_begin_infer(ylm_engine *e);
/* Model::Infer (Model.cpp:43-48 -> ModelBase.cpp:396-471). ids/n_ids and
 * eos_per_prompt/n_eos are in/out: left-trimmed in place to the maximum
 * sequence length (ModelBase.cpp:473-505). The first call after BeginInfer
 * (or every call with the KV cache disabled) is a prefill; later calls take one
 * token. The last-row logits stay on the device (ylm_logits*). */
int ylm_infer(ylm_engine *e, int64_t *ids, int32_t *n_ids, int32_t *eos_per_prompt, int32_t *n_eos);
/* Copy the last-row logits to host memory: FP16 (as_float32 = 0) or FP32.
 * Tensor parallel: a greedy decode step (ylm_decode, ylm_generate,
 * ylm_time_decode) exchanges each rank's best candidate instead of gathering
 * the logits, so after one this call, ylm_logits_device and ylm_sample first
 * gather them with one NCCL all-gather: like every engine call with tp_size > 1,
 * every rank makes it, in the same order. */
int ylm_logits(ylm_engine *e, void *host_out, int32_t as_float32);
/* Device pointer of the last-row FP16 logits [vocab] (gathered first, as above). */
int ylm_logits_device(ylm_engine *e, const void **dev_ptr, int64_t *vocab);
/* Sampling parameters used by ylm_sample / ylm_decode / ylm_generate. */
int ylm_set_sampling(ylm_engine *e, const ylm_sampling *s);
/* ChatSession::Sample (ChatSession.cpp:560-593) on the current logits;
 * greedy = IsGreedy || first generated token (ChatSession.cpp:140). */
int ylm_sample(ylm_engine *e, int32_t greedy, int64_t *next_id);
/* One decode step and its sample in one graph launch: Infer({id}) + Sample. */
int ylm_decode(ylm_engine *e, int64_t id, int32_t greedy, int64_t *next_id);
/* The token loop of ChatSession::Generate (ChatSession.cpp:113-230) on token
 * ids: BeginInfer, prefill, then decode until an EOS id, max_new tokens, the
 * maximum sequence length or an error. The first token is greedy. out_ids gets
 * the generated ids without the EOS. Times are wall-clock per the reference's
 * definition: first token (prefill + sample) and the sum over later tokens. */
int ylm_generate(ylm_engine *e, const int64_t *prompt, int32_t n_prompt, int32_t max_new, const int64_t *eos_ids,
                 int32_t n_eos, int64_t *out_ids, int32_t *n_out, double *first_token_ms, double *decode_ms);
/* Uniform in (0,1) for the next top-k draw instead of the Philox stream (< 0: Philox). */
int ylm_set_draw(ylm_engine *e, float u);
/* The last top-k draw: candidate ids in sampling order, their FP16 probabilities, K, and u. */
int ylm_last_topk(ylm_engine *e, int64_t *ids, float *probs, int32_t *k, float *u);
/* KV capacity in tokens (ModelBase.cpp:345-357), _LastKVCacheTokenIndex, MaxSequenceLength. */
int ylm_info(ylm_engine *e, int32_t *kv_capacity, int32_t *last_kv_index, int32_t *max_seq_len);
/* Device time of the last prefill (CUDA events around its kernels), in ms. */
int ylm_last_prefill_ms(ylm_engine *e, double *ms);
/* Time of one decode graph launch averaged over `iters` back-to-back launches
 * (CUDA events on the engine stream; state advanced on the device). */
int ylm_time_decode(ylm_engine *e, int32_t iters, double *ms_per_step);
/* Which decode path the engine runs: *persistent = 1 when each decode step's
 * projections run as persistent GEMV segments, 0 for the per-op graph. No counterpart in
 * the reference (engine introspection for tests and benchmarks). */
int ylm_decode_path(ylm_engine *e, int32_t *persistent);
/* Time `iters` back-to-back launches of one persistent GEMV segment (the
 * projections of layer `layer`: O, gate-up, down and the next layer's QKV, or
 * the lm_head for the last) with CUDA events on the engine stream; writes the
 * segment's weight bytes. Overwrites the decode workspace (call between
 * requests). YLM_UNSUPPORTED on the per-op path and with tensor parallelism.
 * No counterpart in the reference (benchmark support). */
int ylm_time_segment(ylm_engine *e, int32_t layer, int32_t iters, double *ms_per_launch, double *weight_bytes);

/* Tensor-parallel exchange timing of the persistent path: *wait_ms = the
 * device time (%globaltimer) that block 0 spent in the all-reduce exchanges
 * fused into the O and down epilogues, from its first partial store until
 * every rank's partial of its row had arrived, summed since the last reset;
 * *exchanges = their number; *steps = decode steps since the last reset.
 * reset != 0 clears the three afterwards. Zeros without tensor parallelism.
 * No counterpart in the reference (it runs on one GPU). */
int ylm_exchange_stats(ylm_engine *e, int32_t reset, double *wait_ms, double *exchanges, double *steps);
/* Time one decode step's collectives alone: 2 x num_layers NCCL all-reduces
 * of [hidden] FP16 back to back in a CUDA graph on the engine's communicator,
 * averaged over `iters` replays. Every rank must call it together.
 * YLM_UNSUPPORTED without tensor parallelism. Benchmark support; no
 * counterpart in the reference. */
int ylm_time_allreduce(ylm_engine *e, int32_t iters, double *ms_per_step);

/* Test support for the bounded device waits (no counterpart in the reference):
 * layer >= 0 makes the persistent path write that layer's SwiGLU activation
 * (the gate-up projection's tagged output) into a scratch buffer instead, so
 * the down projection polls words that nothing writes and its wait expires
 * after wait_limit_us; -1 restores the step. YLM_UNSUPPORTED on the per-op
 * path. */
int ylm_debug_drop_output(ylm_engine *e, int32_t layer);

/* Decode-attention kernel for all later launches in this process (and CUDA
 * graphs captured afterwards): 0 (default) one thread-block cluster per KV
 * head where the device can launch clusters, else the split-K kernel; 1 the
 * split-K kernel (global partials and per-KV-head tickets) everywhere. For
 * tests and diagnostics; no counterpart in the reference. */
int ylm_set_attention_path(int32_t split_kernel);

/* ---- kernel-level entry points (device pointers; stream = cudaStream_t or NULL) */
/* y[n] = W[n,k] x[k], FP16 in and out, FP32 accumulation (the decode GEMV). */
int ylm_k_gemv(const void *w, int32_t n, int32_t k, const void *x, void *y, void *stream);
/* C[t,n] = A[t,k] W[n,k]^T, FP16 (the prefill GEMM): tensor_cores = 1 the
 * tcgen05 kernel, 0 the CUDA-core kernel. */
int ylm_k_gemm(const void *a, const void *w, int32_t t, int32_t n, int32_t k, void *c, int32_t tensor_cores,
               void *stream);
/* Causal attention of a T-token prompt for one layer (the prefill SDPA with its
 * causal mask, src/models/ModelBase.cpp:620-636 and :671-693, without the GQA
 * ExpandKV copy of :695-707): q [t][hq*128] (RoPE applied), K/V already in the
 * cache at slots [0, t) of [hkv][cap][128]; out [t][hq*128]. FP16 inputs, FP32
 * accumulation. tensor_cores = 1: tcgen05 with TMEM accumulators (the engine's
 * prefill); 0: mma.sync. */
int ylm_k_prefill_attention(const void *q, const void *k_cache, const void *v_cache, int32_t cap, int32_t hq,
                            int32_t hkv, int32_t t, void *out, int32_t tensor_cores, void *stream);
/* One decode-attention step for one layer: q/k-norm (optional), RoPE at rope_pos,
 * append k/v at `slot`, attention over slots [0, slot]. qkv: [(hq+2hkv)*128];
 * rope tables [max_pos][64]; caches [hkv][cap][128]; out [hq*128]. */
int ylm_k_decode_attention(const void *qkv, const void *q_norm, const void *k_norm, float eps, const void *rope_cos,
                           const void *rope_sin, int32_t max_pos, void *k_cache, void *v_cache, int32_t cap,
                           int32_t hq, int32_t hkv, int32_t slot, int32_t rope_pos, void *out, void *stream);
/* The same decode-attention step with no device allocation, for callers that
 * cannot allocate device memory (their memory is owned by their own pool, or an
 * allocation's synchronisation is not acceptable where they call from). It has
 * no counterpart in the reference. Scratch lives in one 2 MiB array that the
 * library reserves on every GPU that loads it, for the life of the process.
 * The cluster kernel needs only a 256-byte step state there; the split-K
 * kernel (no cluster launch, or ylm_set_attention_path(1)) also keeps its
 * partials (hq x splits x 130 floats) and KV-head tickets there, and shapes
 * whose partials do not fit return YLM_UNSUPPORTED (only past ~4000 query
 * heads). Calls share that array: calls that overlap on the GPU race, so
 * serialise them. The first call on a device looks the array up (with that
 * device current) and should come before any stream capture. */
int ylm_k_decode_attention_noalloc(const void *qkv, const void *q_norm, const void *k_norm, float eps,
                                   const void *rope_cos, const void *rope_sin, int32_t max_pos, void *k_cache,
                                   void *v_cache, int32_t cap, int32_t hq, int32_t hkv, int32_t slot,
                                   int32_t rope_pos, void *out, void *stream);
/* Sample from FP16 logits on the device (greedy or top-k with uniform u). The
 * chosen id and, for top-k, the candidates and probabilities go to host memory. */
int ylm_k_sample(const void *logits, int64_t vocab, int32_t greedy, int32_t top_k, float temperature,
                 const uint32_t *mask_bits_dev, float u, int64_t *out_id, int64_t *topk_ids, float *topk_probs,
                 void *stream);

#ifdef __cplusplus
}
#endif

#endif /* YALAMA_B200_H */
