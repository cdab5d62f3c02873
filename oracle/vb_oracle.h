/*
 * vb_oracle.h -- CPU oracle for the Qwen3 per-token decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * engine's CPU arithmetic (verbum.cpp, core/src/{nn,ops,quant,generate,model}.cpp),
 * kept operation-for-operation identical so that its outputs are bit-identical
 * to the reference's own CPU path: same accumulation order, same float/double
 * widths, no FMA contraction (built with -ffp-contract=off), the same libm
 * calls (expf, sqrtf, lrintf, pow/cos/sin in double).  Rows, heads and output
 * elements are spread over OpenMP threads, but every individual dot product /
 * reduction runs sequentially exactly as in the reference, so threading does
 * not change a single bit.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may call
 * into this library, and only as the checker.  The CUDA engine never links it.
 *
 * Parity is pinned two ways (see tests/test_oracle_*.py):
 *   - against the reference's committed golden vectors (tests/reference_nn.json,
 *     reference_attn.json, reference_block.json, converted to tests/golden/),
 *     and the known answers of tests/test_quant.cpp:42-66;
 *   - bit-for-bit against the reference itself, compiled from its own sources
 *     into oracle/_ref/ by oracle/Makefile.
 */
#ifndef VB_ORACLE_H
#define VB_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- primitive ops (each cites the reference function it restates) ---- */

/* nn.cpp:8-42  rmsnorm: double sum of squares, float scale, out = x*scale*w */
void or_rmsnorm(const float* x, const float* w, float eps, float* out,
                int64_t rows, int64_t dim);

/* nn.cpp:44-74  build_rope_table: inv_freq in double, duplicated halves.
 * cos_tab/sin_tab are [max_pos, head_dim]. Returns 0, or -1 if head_dim odd. */
int or_build_rope_table(int head_dim, int max_pos, float theta,
                        float* cos_tab, float* sin_tab);

/* nn.cpp:76-101  apply_rope (split-half) in place on x [heads, head_dim]. */
int or_apply_rope(float* x, int64_t heads, int head_dim, int pos, int max_pos,
                  const float* cos_tab, const float* sin_tab);

/* ops.cpp:42-70  matmul_nt: C[M,N] = A[M,K] . B[N,K]^T, sequential f32 sum. */
void or_matmul_nt(const float* A, const float* B, float* C,
                  int64_t M, int64_t N, int64_t K);

/* quant.cpp:9-41  quantize_rows: per-row symmetric absmax int8. */
void or_quantize_rows(const float* W, int64_t rows, int64_t cols,
                      int8_t* q, float* scales);

/* quant.cpp:43-70  matmul_nt_q8: acc = sum a*float(q); C = acc*scale[j]. */
void or_matmul_nt_q8(const float* A, const int8_t* Bq, const float* scales,
                     float* C, int64_t M, int64_t N, int64_t K);

/* quant.cpp:72-82  dequantize. */
void or_dequantize(const int8_t* q, const float* scales, int64_t rows,
                   int64_t cols, float* out);

/* generate.cpp:73-105  single-query GQA attention over a contiguous cache.
 * q [H, D] (already normed + roped); k/v cache rows at stride row_stride
 * floats, head kvh at offset kvh*D; n = number of cached positions;
 * ctx [H, D] is overwritten. */
void or_attention_decode(const float* q, const float* kcache,
                         const float* vcache, int64_t row_stride, int H,
                         int KVH, int D, int n, float* ctx);

/* model.cpp:15-18 silu, applied as gate = silu(gate) * up (model.cpp:44-46). */
void or_silu_mul(float* gate, const float* up, int64_t n);

/* generate.cpp:199-206  greedy pick: strict '>' scan from index 0. */
int or_argmax(const float* logits, int64_t vocab);

/* Seeded N(0, std) fill (the synthetic-weight generator; identical output for
 * a given (seed, n) whatever the thread count). */
void or_synth_normal(float* out, uint64_t n, uint64_t seed, float stdv);

/* generate.cpp:197-252  Sampler(cfg).sample() called n times with one
 * generator: row i of logits [n][vocab] gives out[i].  The generator is
 * std::mt19937_64(seed) (the published MT19937-64 recurrence and seeding) and
 * each non-greedy call draws one uniform double in [0, 1) the way
 * std::uniform_real_distribution<double> does with libstdc++ (one 64-bit
 * output scaled by 2^-64, clamped below 1).  Candidates are ordered by value,
 * ties by index (the reference's partial_sort leaves tie order unspecified). */
int or_sample_seq(float temperature, int top_k, float top_p, uint64_t seed,
                  const float* logits, int64_t vocab, int n, int* out);

/* ---- whole-model decode step (model.cpp:235-311, generate.cpp:24-108) ---- */

typedef struct {
    int hidden, layers, heads, kv_heads, head_dim, ffn, vocab;
    int rope_positions;      /* min(max_position_embeddings, 4096), model.cpp:136-138 */
    float eps, theta;
} or_config;

/* Per-layer weight pointers, HF [out,in] row-major f32. The oracle does not copy
 * them; the caller keeps them alive for the model's lifetime. */
typedef struct {
    const float* input_norm;  /* [hidden] */
    const float* post_norm;   /* [hidden] */
    const float* wq;          /* [H*D, hidden] */
    const float* wk;          /* [KVH*D, hidden] */
    const float* wv;          /* [KVH*D, hidden] */
    const float* wo;          /* [hidden, H*D] */
    const float* q_norm;      /* [D] */
    const float* k_norm;      /* [D] */
    const float* wg;          /* [ffn, hidden] */
    const float* wu;          /* [ffn, hidden] */
    const float* wd;          /* [hidden, ffn] */
} or_layer_weights;

typedef struct or_model or_model;

/* Error codes; or_last_error() returns the reference's message text. */
enum {
    OR_OK = 0,
    OR_ERR_NO_CACHE = -1,      /* "call reset_cache() first"            model.cpp:288 */
    OR_ERR_CACHE_FULL = -2,    /* "kv cache is full"                    generate.cpp:30-32 */
    OR_ERR_ROPE = -3,          /* "position is outside the rope table"  nn.cpp:82-84 */
    OR_ERR_TOKEN = -4,         /* "token id out of range for the embedding table" nn.cpp:113-115 */
    OR_ERR_ARG = -5,
    OR_ERR_OOM = -6
};
const char* or_last_error(void);

or_model* or_model_create(const or_config* cfg, const float* embed,
                          const float* final_norm,
                          const or_layer_weights* layers);
void or_model_free(or_model* m);
/* model.cpp:313-338: quantize the 7 projections of every layer. */
int or_model_quantize(or_model* m);
/* Opt-in INT8 tied lm_head: quantize_rows of the embedding, matmul_nt_q8. */
int or_model_quantize_lm_head(or_model* m);
int or_model_is_quantized(const or_model* m);
/* which: 0 q,1 k,2 v,3 o,4 gate,5 up,6 down. Pointers stay owned by m. */
int or_model_quant_tensor(const or_model* m, int layer, int which,
                          const int8_t** q, const float** scales,
                          int64_t* rows, int64_t* cols);
/* model.cpp:277-282 */
int or_model_reset_cache(or_model* m, int max_seq);
/* model.cpp:284-311: logits [vocab] f32. */
int or_model_step(or_model* m, int token, float* logits);
/* Feeds tokens[0..n) from the current position, layer by layer over all n
 * positions: bit-identical to n or_model_step calls; logits (if not NULL)
 * receives the last position's [vocab]. */
int or_model_prefill(or_model* m, const int* tokens, int n, float* logits);
int or_model_cache_len(const or_model* m);
/* model.cpp:340-365 */
size_t or_model_weight_bytes(const or_model* m);
/* direct access to a layer's cache [max_seq, KVH*D] (k if which==0, else v) */
const float* or_model_kv(const or_model* m, int layer, int which);

/* threads used by OpenMP regions (0 = library default) */
void or_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
