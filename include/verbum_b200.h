/*
 * verbum_b200.h -- C ABI of the B200 (sm_100a) decode engine for the
 * Qwen3-0.6B architecture.
 *
 * This is the seam that replaces the reference's CUDA backend
 * (verbum.cpp core/include/verbum/cuda_backend.h:7-43 and the CUDA half of
 * verbum::Model, core/src/model.cpp:367-497).  Plain C: no CUDA or torch types
 * in any signature; device pointers are `void*`/typed pointers, streams are
 * `void*` (a cudaStream_t, NULL = the legacy default stream).  Every call
 * returns a vb_status; on failure vb_last_error() holds the message, worded
 * like the reference's std::runtime_error texts where one exists.
 *
 * Nothing here aborts the process.  The reference's CUDA_CHECK calls abort()
 * (kernels/cuda_ops.cu:9-16); this library returns VB_ERR_CUDA instead.
 */
#ifndef VERBUM_B200_H
#define VERBUM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VB_API __attribute__((visibility("default")))
#else
#define VB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int vb_status;

enum {
    VB_OK = 0,
    VB_ERR_ARG = -1,         /* bad argument / shape                       */
    VB_ERR_CUDA = -2,        /* a CUDA runtime call failed                 */
    VB_ERR_NO_CACHE = -3,    /* "call reset_cache() first"   model.cpp:288  */
    VB_ERR_CACHE_FULL = -4,  /* "kv cache is full"      generate.cpp:30-32  */
    VB_ERR_ROPE = -5,        /* "position is outside the rope table" nn.cpp:82-84 */
    VB_ERR_TOKEN = -6,       /* "token id out of range for the embedding table" nn.cpp:113-115 */
    VB_ERR_STATE = -7,       /* call order violated                        */
    VB_ERR_TIMEOUT = -8,     /* a bounded device wait gave up              */
    VB_ERR_UNSUPPORTED = -9  /* shape outside what the kernels handle      */
};

/* Message of the last failed call on this thread. */
VB_API const char* vb_last_error(void);
/* "sm_100a" build tag + version string. */
VB_API const char* vb_version(void);
/* Test hook for the failure paths (no reference counterpart; the reference's
 * CUDA_CHECK aborts, kernels/cuda_ops.cu:9-16): arms one launch of a kernel to
 * wait for something nothing will produce, so that one of its bounded waits
 * (2 s of %globaltimer) runs out.  site 1: the next clustered decode step
 * (vb_engine_step / decode on path 2) -- one CTA waits for an exchange word no
 * CTA writes; site 2: the next tensor-core GEMM launched outside a stream
 * capture (vb_matmul_nt_tc with M <= 64) -- its first CTA never fills its first
 * stage.  The kernel records the timeout, lets its own copies and MMAs land,
 * releases its tensor memory and returns; the call returns VB_ERR_TIMEOUT and
 * the engine stays usable.  0 disarms.  Nothing faults, traps or hangs. */
VB_API vb_status vb_debug_arm_fault(int site);

/* ------------------------------------------------------------------------ */
/* Device and memory: replaces cuda_backend.h:12-21                          */
/* ------------------------------------------------------------------------ */

/* cuda_available(): number of visible devices (0 when none). */
VB_API int vb_device_count(void);
/* cuda_device_name(): copies the name of device `dev` into buf. */
VB_API vb_status vb_device_name(int dev, char* buf, size_t len);
/* cuda_free_memory() */
VB_API vb_status vb_free_memory(int dev, size_t* free_bytes);
/* cuda_alloc / cuda_free / cuda_upload / cuda_download / cuda_zero / cuda_sync */
VB_API vb_status vb_alloc(void** ptr, size_t bytes);
VB_API vb_status vb_free(void* ptr);
VB_API vb_status vb_upload(void* dst, const void* host, size_t bytes, void* stream);
VB_API vb_status vb_download(void* host, const void* src, size_t bytes, void* stream);
VB_API vb_status vb_zero(void* dst, size_t bytes, void* stream);
VB_API vb_status vb_sync(void* stream);

/* ------------------------------------------------------------------------ */
/* Kernel entry points (device pointers, caller-owned memory)                */
/* ------------------------------------------------------------------------ */

/* C[M,N] = A[M,K] . W[N,K]^T in f32.
 * Replaces cuda_matmul_nt (cuda_backend.h:23-24, kernels/cuda_ops.cu:237-244)
 * and the CPU matmul_nt (core/src/ops.cpp:42-70).  M==1 runs the streaming
 * GEMV; M>1 the batched kernel.  K must be a multiple of 4, pointers 16-byte
 * aligned. */
VB_API vb_status vb_matmul_nt_f32(const float* A, const float* W, float* C, int M, int N,
                           int K, void* stream);

/* C[M,N] = (A[M,K] . float(Wq[N,K])^T) * scales[N]: weight-only INT8 GEMV/GEMM
 * with the dequantisation fused into the dot product.
 * Replaces matmul_nt_q8 (core/src/quant.cpp:43-70); the reference has no GPU
 * version (core/src/model.cpp:374-377).  K must be a multiple of 16. */
VB_API vb_status vb_matmul_nt_q8(const float* A, const int8_t* Wq, const float* scales,
                          float* C, int M, int N, int K, void* stream);

/* C[M][N] = A[M][K] . W[N][K]^T on the tensor cores (tcgen05, bf16 operands,
 * f32 accumulation): the batched form of matmul_nt / matmul_nt_q8 (ops.cpp:42-70,
 * quant.cpp:43-70) for M >= 1 activation rows (64-row tiles; split-K when
 * M <= 64) and K % 64 == 0.  W is
 * f32 (w_int8 = 0; used as a bf16 hi+lo pair) or INT8 with per-row scales
 * applied after the sum (w_int8 = 1); A is split into bf16 hi+lo.  Synchronous
 * on `stream`; scratch comes from a per-device buffer grown on demand. */
VB_API vb_status vb_matmul_nt_tc(const float* A, const void* W, const float* scales, float* C, int M, int N,
                                 int K, int w_int8, void* stream);

/* Per-row symmetric absmax INT8 quantisation, bit-exact with quantize_rows
 * (core/src/quant.cpp:9-41): scale = amax>0 ? amax/127 : 1, q = clamp(
 * round-half-even(w * (1/scale)), -127, 127). */
VB_API vb_status vb_quantize_rows(const float* W, int64_t rows, int64_t cols, int8_t* q,
                           float* scales, void* stream);

/* out = x * (1/sqrt(mean(x^2)+eps)) * w per row.  Replaces cuda_rmsnorm
 * (cuda_backend.h:26-27) with the CPU rmsnorm's double accumulation
 * (core/src/nn.cpp:8-42).  x may equal out. */
VB_API vb_status vb_rmsnorm(const float* x, const float* w, float* out, int rows, int dim,
                     float eps, void* stream);

/* Split-half RoPE in place on x[heads, D] at position pos using host-built
 * tables [max_pos, D].  Replaces cuda_rope (cuda_backend.h:29-30) /
 * apply_rope (core/src/nn.cpp:76-101). */
VB_API vb_status vb_rope(float* x, const float* cos_tab, const float* sin_tab, int pos,
                  int heads, int D, void* stream);

/* gate = silu(gate) * up.  Replaces cuda_silu_mul (cuda_backend.h:32);
 * silu as core/src/model.cpp:15-18 with accurate expf. */
VB_API vb_status vb_silu_mul(float* gate, const float* up, int n, void* stream);

/* a += b.  Replaces cuda_add (cuda_backend.h:34). */
VB_API vb_status vb_add(float* a, const float* b, int n, void* stream);

/* Copies knew/vnew (width floats) into row `pos` of caches laid out
 * [max_seq, width].  Replaces cuda_cache_append (cuda_backend.h:40-42). */
VB_API vb_status vb_cache_append(float* kcache, float* vcache, const float* knew,
                          const float* vnew, int pos, int width, void* stream);

/* Single-query GQA decode attention over a contiguous cache [n, KVH*D]
 * (the reference's layout, core/include/verbum/generate.h:19-30).
 * q [H, D] already normed and roped; out [H, D].  Replaces cuda_attn_decode
 * (cuda_backend.h:36-38), whose one-block-per-head kernel cannot launch past
 * n of about 12288; this split-K kernel has no length limit.  Scratch for the
 * split partials is allocated by the library on first use per device and
 * reused (not thread-safe across concurrent calls). D must be 128. */
VB_API vb_status vb_attn_decode(const float* q, const float* kcache, const float* vcache,
                         float* out, int H, int KVH, int D, int n, void* stream);

/* Same computation as vb_attn_decode, for callers that must not allocate
 * device memory (a host framework that owns all device memory through its own
 * budgeted pool, a plugin whose enqueue path may not allocate, a serving loop
 * that cannot afford cudaMalloc's implicit synchronisation).  No counterpart
 * in the reference.  The split partials live in a 1 MiB array compiled into
 * the library (held by every GPU that loads it until the process exits).  The
 * split count is capped at what that array holds (H * splits * 132 floats,
 * plus 512 B: 124 splits for 16 heads), so every context length runs, with
 * longer splits past about 16k positions; only a head count too large for one
 * split (H > 1984) returns VB_ERR_UNSUPPORTED.  The first call on a device (and
 * the first after the device's context was replaced, e.g. by cudaDeviceReset)
 * looks up the array's device address, so make that call before any stream
 * capture.  All calls share the array: calls that overlap on the GPU
 * (different streams, or devices sharing nothing but this array's name) race
 * and must be serialised by the caller.  Nothing in it needs clearing between
 * calls.  Calls no cudaMalloc, cudaFree or allocating routine. */
VB_API vb_status vb_attn_decode_noalloc(const float* q, const float* kcache,
                                        const float* vcache, float* out, int H, int KVH,
                                        int D, int n, void* stream);

/* Batched/strided decode attention for B independent sequences.
 * q [B, H, D]; element (b, pos, kvh, d) of K/V is at
 *   base + b*stride_b + pos*stride_pos + kvh*stride_h + d   (floats);
 * lens[b] (device int array) is each sequence's cache length (>=1, <= n_max).
 * workspace: vb_attn_workspace_bytes(B, H, n_max) bytes of device memory,
 * 16-byte aligned.
 * out [B, H, D].  No reference counterpart beyond generate.cpp:73-105 applied
 * per sequence. */
VB_API size_t vb_attn_workspace_bytes(int B, int H, int n_max);
/* Causal attention of a prompt chunk (prefill), the decode attention of
 * generate.cpp:73-105 applied at every position p0 + c (c < C) of B sequences:
 * q and out [B*C][H*D] (row b*C + c); element (b, kvh, pos, d) of K/V at
 * base + b*stride_b + kvh*stride_h + pos*D (floats), positions 0 .. p0 + C - 1
 * filled.  H == 2*KVH, D == 128.  p0 == 0 runs on the tensor cores (bf16 hi/lo
 * operands, scratch from the per-device buffer, synchronous on `stream`);
 * p0 > 0 on the CUDA cores (no scratch, asynchronous). */
VB_API vb_status vb_attn_prefill(const float* q, const float* k, const float* v, float* out,
                                 int B, int C, int p0, int H, int KVH, int D,
                                 int64_t stride_b, int64_t stride_h, void* stream);
VB_API vb_status vb_attn_decode_batched(const float* q, const float* k, const float* v,
                                 float* out, const int* lens, int B, int H, int KVH,
                                 int D, int n_max, int64_t stride_b,
                                 int64_t stride_pos, int64_t stride_h,
                                 void* workspace, void* stream);

/* Greedy pick over rows of logits [rows, n]: lowest index among maxima, the
 * strict-'>' scan of Sampler::sample (core/src/generate.cpp:199-206).
 * out_idx: device int[rows]. */
VB_API vb_status vb_argmax_rows(const float* logits, int rows, int64_t n, int* out_idx,
                         void* stream);

/* ------------------------------------------------------------------------ */
/* Synthetic weights (host): seeded N(0, std) f32 fill, identical for a given  */
/* (seed, offset) whatever the thread count.                                 */
/* ------------------------------------------------------------------------ */
VB_API void vb_synth_normal(float* out, uint64_t n, uint64_t seed, float std);

/* ------------------------------------------------------------------------ */
/* Engine: the decode loop of verbum::Model (core/include/verbum/model.h:47-116)
 * with weights, KV cache and scratch resident in HBM.                        */
/* ------------------------------------------------------------------------ */

typedef struct {
    int hidden;          /* hidden_size                         */
    int layers;          /* num_hidden_layers                   */
    int heads;           /* num_attention_heads                 */
    int kv_heads;        /* num_key_value_heads                 */
    int head_dim;        /* head_dim (must be 128)              */
    int ffn;             /* intermediate_size                   */
    int vocab;           /* vocab_size                          */
    int rope_positions;  /* min(max_position_embeddings, 4096), model.cpp:136-138 */
    float eps;           /* rms_norm_eps                        */
    float theta;         /* rope_theta                          */
} vb_config;

/* Host pointers to one layer's f32 weights in HF layout [out, in]
 * (the tensors model.cpp:145-157 loads). */
typedef struct {
    const float* input_norm;  /* [hidden]           */
    const float* post_norm;   /* [hidden]           */
    const float* wq;          /* [H*D, hidden]      */
    const float* wk;          /* [KVH*D, hidden]    */
    const float* wv;          /* [KVH*D, hidden]    */
    const float* wo;          /* [hidden, H*D]      */
    const float* q_norm;      /* [D]                */
    const float* k_norm;      /* [D]                */
    const float* wg;          /* [ffn, hidden]      */
    const float* wu;          /* [ffn, hidden]      */
    const float* wd;          /* [hidden, ffn]      */
} vb_layer_host;

/* The same tensors as bf16 bit patterns (the dtype of released checkpoints;
 * the reference widens them on the host, safetensors.cpp:239-264). */
typedef struct {
    const uint16_t *input_norm, *post_norm, *wq, *wk, *wv, *wo, *q_norm, *k_norm, *wg, *wu, *wd;
} vb_layer_host_bf16;

typedef struct vb_engine vb_engine;

/* Creates an engine on `device` (Model::to_cuda, model.cpp:367-443, minus the
 * upload, which the two calls below do). */
VB_API vb_status vb_engine_create(const vb_config* cfg, int device, vb_engine** out);
VB_API vb_status vb_engine_destroy(vb_engine* e);
/* Uploads the tied embedding / lm_head [vocab, hidden] and final norm. */
VB_API vb_status vb_engine_set_globals(vb_engine* e, const float* embed, const float* final_norm);
/* Uploads one layer's f32 weights (model.cpp:407-421). */
VB_API vb_status vb_engine_set_layer(vb_engine* e, int layer, const vb_layer_host* w);
/* bf16 uploads: half the host-to-device bytes, widened to f32 on the device
 * (exactly: bf16 is the top half of an f32, as bf16_to_f32 in
 * safetensors.cpp:59-66), giving the same device weights as the f32 calls. */
VB_API vb_status vb_engine_set_globals_bf16(vb_engine* e, const uint16_t* embed, const uint16_t* final_norm);
VB_API vb_status vb_engine_set_layer_bf16(vb_engine* e, int layer, const vb_layer_host_bf16* w);
/* One layer already quantized on the host (the reference's QuantLayer,
 * quant.h:29-36, as Model::quantize leaves it, model.cpp:313-338): int8 rows
 * [rows][cols] and one f32 scale per row for each projection, plus the f32
 * norms.  The first call switches the engine to INT8 weights (the f32
 * projection memory is released); every layer must then come through this
 * call.  The device holds exactly these bytes, so the weights are the
 * reference's own quantized values.  Replaces the refusal of quantized
 * weights at model.cpp:374-377. */
typedef struct {
    const float *input_norm, *post_norm, *q_norm, *k_norm;
    const int8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *sq, *sk, *sv, *so, *sg, *su, *sd;
} vb_layer_host_q8;
VB_API vb_status vb_engine_set_layer_q8(vb_engine* e, int layer, const vb_layer_host_q8* w);
/* Model::quantize (model.cpp:313-338) on the device: the 7 projections of
 * every layer become INT8 + per-row scales bit-exactly as quantize_rows, and
 * the f32 copies are freed.  Embedding, lm_head and norms stay f32. */
VB_API vb_status vb_engine_quantize(vb_engine* e);
VB_API int vb_engine_is_quantized(const vb_engine* e);
/* Opt-in, no reference counterpart (the reference keeps the tied lm_head in
 * f32, model.cpp:313-338): quantize_rows of the embedding rows becomes the
 * lm_head (matmul_nt_q8); the embedding lookup keeps the f32 table.  Cuts the
 * lm_head's 622 MB per token to 156 MB; logits then differ from the
 * reference's by the quantisation of the lm_head (not a parity mode).  Applies
 * to the engine's steps and to batches made from it. */
VB_API vb_status vb_engine_quantize_lm_head(vb_engine* e);
VB_API int vb_engine_lm_head_int8(const vb_engine* e);
/* Model::weight_bytes (model.cpp:340-365). */
VB_API size_t vb_engine_weight_bytes(const vb_engine* e);
/* Model::reset_cache (model.cpp:277-282): (re)allocates the device KV cache
 * for max_seq positions and sets the length to 0. */
VB_API vb_status vb_engine_reset_cache(vb_engine* e, int max_seq);
VB_API int vb_engine_cache_len(const vb_engine* e);
/* Model::step (model.cpp:284-311 / step_cuda 446-497): one token in, logits
 * [vocab] f32 out to HOST memory. */
VB_API vb_status vb_engine_step(vb_engine* e, int token, float* logits_host);
/* Greedy decode of n tokens entirely on the device: token t+1 is the argmax of
 * step t's logits (Sampler greedy, generate.cpp:199-206) fed back without a
 * host round trip.  tokens_host[i] receives the token chosen after step i
 * (so tokens_host[n-1] is the next token to feed).  logits_host, if not NULL,
 * receives the last step's logits. */
VB_API vb_status vb_engine_decode(vb_engine* e, int first_token, int n, int* tokens_host,
                           float* logits_host);
/* Prefill: feeds tokens_host[0..n) one position at a time (the token-by-token
 * prefill of tools/generate.cpp:75-77) with no host synchronisation between
 * tokens; logits_host, if not NULL, receives the last token's logits. */
VB_API vb_status vb_engine_prefill(vb_engine* e, const int* tokens_host, int n,
                                   float* logits_host);
/* Kernel launches in one captured step (graph nodes), 0 before the first step. */
VB_API int vb_engine_graph_nodes(const vb_engine* e);
/* Copies layer `layer`'s K (which=0) or V cache rows [0, len) into host
 * memory as [len, KVH*D] (the reference KVCache layout). */
VB_API vb_status vb_engine_read_kv(const vb_engine* e, int layer, int which, float* host);
/* Selects the bs1 step implementation: 1 = one kernel per op in a CUDA graph,
 * 2 = persistent kernel on KV-head thread-block clusters exchanging tagged
 * data words (no barriers), -1 = automatic (the default: the faster of the two
 * for the weight format as measured on B200 -- 2 for INT8 weights, 1 for f32).
 * Path 2 needs hidden 1024, GQA group 2 and head_dim 128; where those are not
 * met the step falls back to 1. */
VB_API vb_status vb_engine_set_path(vb_engine* e, int path);
/* The path the next step runs (1 or 2; the automatic choice if not fixed). */
VB_API int vb_engine_path(const vb_engine* e);
/* The stream the engine runs on (a cudaStream_t). */
VB_API void* vb_engine_stream(vb_engine* e);
/* Phase tracing of the clustered step (path 2; no reference counterpart, the
 * reference times whole steps with steady_clock, tools/bench.cpp:63-69): when
 * on, each CTA c of the next steps records %globaltimer nanoseconds in words
 * [c*2048, c*2048+2048): word 0 = start, then 12 stamps per layer (phase ends)
 * and from word 400 a 40-word clock64 profile per layer.  Only libraries built
 * with VB_STEP_TRACE=1 record anything; others return 0 words.  read_trace
 * copies up to cap words of the last step and returns how many it copied. */
VB_API vb_status vb_engine_set_trace(vb_engine* e, int on);
VB_API int vb_engine_read_trace(vb_engine* e, uint64_t* out, int cap);

/* ------------------------------------------------------------------------ */
/* Sampling: Sampler / SamplerConfig (generate.h:49-67, generate.cpp:197-252)  */
/* on the device.  The host keeps the reference's generator                 */
/* (std::mt19937_64(seed), one std::uniform_real_distribution<double> draw   */
/* per non-greedy sample); the device sorts the logits, applies temperature, */
/* top_k (0 disables) and top_p (1 disables) and picks.  temperature <= 0 or */
/* top_k == 1 is the greedy argmax, as in the reference.                    */
/* ------------------------------------------------------------------------ */
typedef struct vb_sampler vb_sampler;
VB_API vb_status vb_sampler_create(float temperature, int top_k, float top_p, uint64_t seed,
                                   vb_sampler** out);
VB_API vb_status vb_sampler_destroy(vb_sampler* s);
/* One Sampler::sample of device logits [vocab]; synchronous on `stream`. */
VB_API vb_status vb_sampler_sample(vb_sampler* s, const float* logits, int64_t vocab, void* stream,
                                   int* token);
/* n decode steps from first_token with each next token drawn by the sampler on
 * the device (the generate loop of tools/generate.cpp:63-90 without a host
 * round trip per token); the n picks go to tokens_host if not NULL. */
VB_API vb_status vb_engine_decode_sampled(vb_engine* e, vb_sampler* s, int first_token, int n,
                                          int* tokens_host);

/* ------------------------------------------------------------------------ */
/* Batched independent-sequence decode (no reference counterpart; the
 * reference is batch-1 only).  B sequences share the engine's weights; each
 * has its own KV cache and position.                                        */
/* ------------------------------------------------------------------------ */
typedef struct vb_batch vb_batch;
VB_API vb_status vb_batch_create(vb_engine* e, int batch, int max_seq, vb_batch** out);
VB_API vb_status vb_batch_destroy(vb_batch* b);
/* One step for all B sequences: tokens_host [B] in; logits_host [B, vocab]
 * and/or next_host [B] (greedy picks) out, either may be NULL. */
VB_API vb_status vb_batch_step(vb_batch* b, const int* tokens_host, float* logits_host,
                        int* next_host);
/* n greedy steps on the device from the tokens fed last (or tokens_host if not
 * NULL); next tokens after the last step go to next_host [B] if not NULL. */
VB_API vb_status vb_batch_decode(vb_batch* b, const int* tokens_host, int n, int* next_host);
/* Prefill P positions for all B sequences: tokens_host is [P][B]
 * (position-major); next_host [B] (may be NULL) gets the greedy pick after
 * the last position. */
VB_API vb_status vb_batch_prefill(vb_batch* b, const int* tokens_host, int P, int* next_host);
VB_API int vb_batch_graph_nodes(const vb_batch* b);
VB_API int vb_batch_cache_len(const vb_batch* b);
VB_API vb_status vb_batch_reset(vb_batch* b);
/* Model::embed_text (model.cpp:191-233) on the device: the n ids' layers
 * through the batched prefill path (a temporary one-sequence batch), the final
 * RMSNorm of every position, the mean over positions and L2 normalisation into
 * out_host [hidden].  f32 projections only, like the reference. */
VB_API vb_status vb_engine_embed_text(vb_engine* e, const int* ids, int n, float* out_host);
/* Roll every sequence back to len cached positions (0 <= len <= cache length):
 * the next step writes position len.  Cached entries past len are left in
 * place and overwritten before they are read again. */
VB_API vb_status vb_batch_truncate(vb_batch* b, int len);

#ifdef __cplusplus
}
#endif
#endif /* VERBUM_B200_H */
