// vb_kernels.cuh -- internal launchers shared by the C ABI and the engines.
#pragma once

#include "vb_common.cuh"

namespace vb {

// Split-K decode attention: one partial per (sequence, head, split) is
// kAttnPart floats -- m, l, two pad words, then the 128 accumulators (16-byte
// aligned for vector loads) -- and a split covers at least kAttnMinSplit
// positions.
constexpr int kAttnPart = 132;
constexpr int kAttnMinSplit = 64;

// GEMV prologue: the input vector is used as is, or RMS-normalised with a
// weight vector first (the rmsnorm that precedes every projection).
enum GemvPro : int { kProNone = 0, kProRms = 1, kProMerge = 2 };
// GEMV epilogue.
enum GemvEpi : int {
    kEpiStore = 0,     // y[j] = dot_j
    kEpiResidual = 1,  // y[j] += dot_j                        (o_proj / down_proj + residual)
    kEpiSwiGLU = 2,    // rows interleaved gate/up: y[j] = silu(dot_2j) * dot_2j+1
    kEpiArgmax = 3,    // y[j] = dot_j and per-CTA (max, argmax) partials
    kEpiQkNorm = 4,    // tensor-core GEMM of the q|k|v rows (one head per 128-row tile): the
                       // per-head q/k norm + RoPE, q out, k and v appended to the cache
};

struct GemvArgs {
    const float* x;        // [K] input (or embedding row base when x_tok != null)
    const int* x_tok;      // optional: x = x + (*x_tok) * K  (embedding lookup fused)
    const float* norm_w;   // [K] rmsnorm weight (kProRms)
    float eps;
    const void* W;         // [N, K] f32 or int8
    const float* scales;   // [N] (int8 only)
    float* y;              // output
    int N, K;
    float* part_val;       // [gridDim] (kEpiArgmax)
    int* part_idx;         // [gridDim]
    int* err;              // optional: device error word (bounded waits)
    const void* l2_ahead;  // optional (prefetching GEMV): bytes a later kernel reads,
    size_t l2_ahead_bytes; //   pulled into L2 by this kernel's CTAs (a 1/grid share each)
    // optional (prefetching GEMV): the cached K and V rows [0, *kv_pos) of
    // kv_heads heads (head h at kv_k / kv_v + h * kv_stride_h floats, D = 128),
    // pulled into L2 for the attention that follows
    const float* kv_k;
    const float* kv_v;
    const int* kv_pos;
    int kv_heads;
    int64_t kv_stride_h;
    // kProMerge (prefetching GEMV): x is the batch-1 attention output merged
    // from the split attention's partials ([head][split] records of
    // kAttnPart floats: M, L, -, -, 128 weighted sums), K = heads * 128
    const float* attn_parts;
    int attn_splits;
    unsigned pf_xs_off;  // prefetching GEMV: byte offset of x in its dynamic shared memory (set by the launcher)
};

// Batch-1 GEMV with its weights prefetched into shared memory before it waits
// for the previous kernel (vb_gemv_pf.cu): one CTA per SM, each a contiguous
// slice of at most kPfSliceBytes of W; larger matrices run as several launches
// (gemv_pf_parts).  Store, residual and SwiGLU epilogues; RMSNorm prologue.
// The budget fills an SM's shared memory, so one such CTA runs per SM: with
// 96 KB slices (two per SM, the next kernel's prefetching while this one
// computes) the per-op step measured slower (f32 1001 against 1101 tok/s).
constexpr size_t kPfSliceBytes = 200 * 1024;
constexpr int kPfCtas = 148;
int gemv_pf_parts(int N, int K, bool q8, int epi);  // 0: does not fit
vb_status launch_gemv_pf(const GemvArgs& a, bool q8, int pro, int epi, cudaStream_t s);

// Launch config chosen so every SM streams weights even for 1024-row outputs.
vb_status launch_gemv(const GemvArgs& a, bool q8, int pro, int epi, cudaStream_t s,
                      int* grid_out = nullptr);
int gemv_grid(int N, bool q8, int epi);

// Final reduction of argmax partials: out_idx[0] = argmax, optional value.
vb_status launch_argmax_parts(const float* part_val, const int* part_idx, int parts,
                              int* out_idx, cudaStream_t s);

vb_status launch_quantize_rows(const float* W, int64_t rows, int64_t cols, int8_t* q,
                               float* scales, cudaStream_t s);
vb_status launch_rmsnorm_rows(const float* x, const float* w, float* out, int rows,
                              int dim, float eps, cudaStream_t s,
                              void* hi = nullptr, void* lo = nullptr);

// Per-head q/k RMSNorm + RoPE for B sequences, writing rotated q to q_out
// [B, H, D] and k / v rows into the caches at each sequence's position.
struct QkNormArgs {
    const float* qkv;       // [B, (H + 2*KVH) * D]  (q | k | v)
    int rows_per_seq;       // > 0: row b belongs to sequence b / rows_per_seq (a prompt chunk)
    void* q_hi;             // optional bf16 hi/lo copies of the q rows [B][H*D]
    void* q_lo;
    void* k_hi;             // and of the k rows [(seq*KVH + h) * kbf_rows + pos][D]
    void* k_lo;
    int kbf_rows;
    const float* parts;     // or, when set: split-K partials [splits][B][(H + 2*KVH) * D]
    int splits;             //   summed in split order,
    const float* scales;    //   times these INT8 row scales when set
    const float* q_norm;    // [D]
    const float* k_norm;    // [D]
    const float* cos_tab;   // [rope_positions, D]
    const float* sin_tab;
    const int* pos;         // [B] device positions (write row)
    float* q_out;           // [B, H, D] (null: only the bf16 copies)
    float* kc;              // cache base
    float* vc;
    int64_t stride_b, stride_pos, stride_h;  // cache strides (floats)
    int B, H, KVH, D, rope_positions;
    float eps;
    int* err;               // device error word (may be null)
};
vb_status launch_qk_norm_rope_append(const QkNormArgs& a, cudaStream_t s);

// x[b] += sum_s parts[s][b] (x scales), then out[b] = RMSNorm(x[b]) . w and its
// bf16 split (hi, lo) -- the split-K reduce of a residual projection fused
// with the next RMSNorm.  One block per row.
vb_status launch_reduce_residual_norm(float* x, const float* parts, int splits, const float* scales,
                                      const float* w, float* out, void* hi, void* lo, int rows, int dim,
                                      float eps, cudaStream_t s);

// Split-K decode attention.  lens[b] = number of valid cache rows.
struct AttnArgs {
    const float* q;        // [B, H, D]
    const float* k;        // cache base
    const float* v;
    float* out;            // [B, H, D]
    const int* lens;       // [B] (device)
    const int* pos;        // alternative to lens: lens[b] = pos[b] + 1 (may be null)
    int B, H, KVH, D, n_max;
    int64_t stride_b, stride_pos, stride_h;
    int splits;            // splits per (b, kvh)
    float* ws;             // partials
    void* out_hi;          // optional bf16 split of out (tensor-core GEMM operand)
    void* out_lo;
    // fuse_qk: q is not read from `q` but normed and rotated by each CTA from
    // qk's source (the q|k|v GEMV row or GEMM partials), and the CTA whose
    // range holds position pos[b] also computes k, v, appends them to the cache
    // and uses them for that position (generate.cpp:52-71 inside the attention)
    int fuse_qk;
    QkNormArgs qk;
    // positions (pos / lens) and the cached rows before them were written
    // before this launch's predecessor started (a decode step's graph): the
    // kernel may read them, and request the rows, before griddepcontrol.wait
    int pos_stable;
    // the split partials are left in ws for the consumer to merge (the
    // batch-1 o projection's prologue); no merge launch, out is not written
    int no_merge;
};
int attn_splits_for(int B, int KVH, int n_max);
size_t attn_ws_bytes(int B, int H, int splits);
vb_status launch_attention(const AttnArgs& a, cudaStream_t s);

// Causal attention of a prompt chunk (vb_prefill.cu): q / out [B*C][H*D]
// (row b*C + c = position p0 + c of sequence b), keys 0 .. p0 + c of the
// cache (already holding the chunk's rows).  H == 2 * KVH, D == 128.
struct PrefillAttnArgs {
    const float* q;
    const float* k;        // cache base of the layer: + b*stride_b + g*stride_h + pos*D
    const float* v;
    int64_t stride_b;
    int64_t stride_h;
    int B, C, p0, H, KVH, D;
    float* out;
    void* out_hi;          // optional bf16 split of out
    void* out_lo;
    int* err;              // device error word (tensor-core form; may be null)
};
vb_status launch_prefill_attention(const PrefillAttnArgs& a, cudaStream_t s);
size_t prefill_attention_smem();
// Tensor-core form for a prompt from position 0 (a.p0 == 0, a.C = prompt
// length, q given as f32 [B*C][H*D]): bf16 hi/lo copies of q, K and V^T go to
// `scratch` (prompt_attention_tc_bytes), the split output to a.out_hi/out_lo
// (and f32 to a.out when set).
size_t prompt_attention_tc_bytes(int B, int P, int H, int KVH);
struct PromptCopies {  // where the bf16 copies sit in that scratch
    void *q_hi, *q_lo, *k_hi, *k_lo, *vt_hi, *vt_lo;
};
PromptCopies prompt_attention_copies(void* scratch, int B, int P, int H, int KVH);
// qk_ready: the q and K copies are already in the scratch (written by the
// q/k-norm kernel); only V^T is built here.
vb_status launch_prompt_attention_tc(const PrefillAttnArgs& a, const float* q, void* scratch, cudaStream_t s,
                                     bool qk_ready = false);

vb_status launch_embed(const float* E, const int* tokens, int B, int dim, int vocab,
                       float* out, int* err, cudaStream_t s);
vb_status launch_argmax_rows(const float* logits, int rows, int64_t n, int* out_idx,
                             cudaStream_t s);
vb_status launch_rope(float* x, const float* cos_tab, const float* sin_tab, int pos,
                      int heads, int D, cudaStream_t s);
vb_status launch_silu_mul(float* gate, const float* up, int n, cudaStream_t s);
vb_status launch_add(float* a, const float* b, int n, cudaStream_t s);
vb_status launch_cache_append(float* kc, float* vc, const float* kn, const float* vn,
                              int pos, int width, cudaStream_t s);
// pos[b] += 1; tokens[b] = next[b]
vb_status launch_advance(int* pos, int* tokens, const int* next, int B, cudaStream_t s);
// Per-row argmax of a decode step's logits [rows][n] over all SMs: each CTA
// folds its slice into keys[row] (atomicMax of a (value, lowest index) key);
// keys must be zero before.  launch_advance_keys then turns the keys into
// next[] (argmax_rows_kernel's result: lowest index on ties, NaN never
// picked, 0 for a row without a pick), tokens = next, pos += 1, and zeroes
// the keys for the next step.
vb_status launch_argmax_rows_keys(const float* logits, int rows, int64_t n, unsigned long long* keys,
                                  cudaStream_t s);
vb_status launch_advance_keys(int* pos, int* tokens, int* next, unsigned long long* keys, int B, cudaStream_t s);

// Batched (M <= 64) GEMM, C = A . W^T with split-K partials and a fused
// reduction epilogue.
struct GemmArgs {
    const float* A;        // [M, K]
    const void* W;         // [N, K] f32 or int8
    const float* scales;   // [N] int8 only
    float* C;              // output (layout depends on epi)
    int M, N, K;
    int ldc;               // row stride of C in floats
    float* ws;             // split-K partial workspace
    size_t ws_floats;
    void* out_hi;          // kEpiSwiGLU: optional bf16 split of the output
    void* out_lo;
};
size_t gemm_ws_floats(int M, int N, int K, bool q8);
vb_status launch_gemm(const GemmArgs& a, bool q8, int epi, cudaStream_t s);
// Sums `splits` partials P[s][M][N] (a.ws) in fixed order, applies the INT8
// row scales (q8) and the epilogue into a.C.
vb_status launch_gemm_reduce(const GemmArgs& a, int splits, bool q8, int epi, cudaStream_t s);

// Tensor-core projection (vb_tcgemm.cu): partial sums of A . W^T over K
// splits into ws [splits][M][N], from bf16 operands: W_hi (+ W_lo for f32
// weights, null for INT8), A_hi + A_lo ([64][K], rows >= M zero).
// The K splits are summed in fixed order, the INT8 row scales applied (when
// `scales` is set) and the epilogue written into C: kEpiStore C[m][n] = v,
// kEpiResidual C[m][n] += v, kEpiSwiGLU (rows interleaved gate/up)
// C[m][n/2] = silu(v_n) * v_n+1, also written as a bf16 split to
// out_hi/out_lo when set (the next GEMM's operand).
struct TcGemmArgs {
    const void* w_hi;
    const void* w_lo;
    const void* a_hi;
    const void* a_lo;
    int M, N, K;
    float* ws;             // split partials
    size_t ws_floats;
    const float* scales;
    float* C;
    int ldc;
    int epi;
    void* out_hi;
    void* out_lo;
    bool partials_only;    // leave the split partials in ws for a fused consumer
    int* err;
    const QkNormArgs* qk;  // kEpiQkNorm: norms, rope table, positions, q out, cache (parts / qkv unused)
};
// split-K factor of a tensor-core GEMM (pair: f32 weights as a bf16 pair)
int tc_gemm_splits(int N, int K, bool pair);
// True when a GEMM of M <= 64 rows can take the kEpiQkNorm epilogue: its
// split-K partials summed inside a thread-block cluster (at most 8 splits), no
// workspace round trip and no q/k-norm launch.
bool tc_gemm_cluster_reduce(int M, int N, int K, bool pair);
size_t tc_gemm_ws_floats(int M, int N, int K);
int tc_gemm_tiles(int N);
vb_status launch_tc_gemm(const TcGemmArgs& a, cudaStream_t s);
// A [M][lda] -> bf16 hi/lo [rows][K]: rows = max(M, 64) zero-padded (pad64, the
// decode GEMM's 64-row operand) or exactly M.
vb_status launch_split_bf16(const float* A, int M, int K, int lda, void* hi, void* lo, cudaStream_t s,
                            bool pad64 = true);
vb_status launch_weights_bf16(const void* W, bool q8, size_t count, void* hi, void* lo, cudaStream_t s);

}  // namespace vb
