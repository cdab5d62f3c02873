/*
 * vb_oracle.c -- CPU oracle for the Qwen3 decode path (TEST INFRASTRUCTURE).
 *
 * Restates the reference engine's CPU arithmetic (verbum.cpp) in C, operation
 * for operation; see vb_oracle.h for the contract and how it is pinned.
 * Build flags matter for bit-exactness: -O2 -ffp-contract=off, no -ffast-math,
 * x86-64 baseline ISA (no FMA), exactly as the reference compiles.
 */
#include "vb_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static __thread char g_err[256];
static void set_err(const char* msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
}
const char* or_last_error(void) { return g_err; }

void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* nn.cpp:8-42 */
void or_rmsnorm(const float* x, const float* w, float eps, float* out,
                int64_t rows, int64_t dim) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * dim;
        float* orow = out + r * dim;
        double sumsq = 0.0;
        for (int64_t i = 0; i < dim; i++) sumsq += (double)xr[i] * (double)xr[i];
        const float scale = 1.0f / sqrtf((float)(sumsq / (double)dim) + eps);
        for (int64_t i = 0; i < dim; i++) orow[i] = xr[i] * scale * w[i];
    }
}

/* nn.cpp:44-74 */
int or_build_rope_table(int head_dim, int max_pos, float theta,
                        float* cos_tab, float* sin_tab) {
    if (head_dim % 2 != 0) return -1;
    const int half = head_dim / 2;
    for (int pos = 0; pos < max_pos; pos++) {
        for (int i = 0; i < half; i++) {
            const double inv_freq =
                1.0 / pow((double)theta, (double)(2 * i) / (double)head_dim);
            const double angle = (double)pos * inv_freq;
            const float c = (float)cos(angle);
            const float s = (float)sin(angle);
            const size_t base = (size_t)pos * head_dim;
            cos_tab[base + i] = c;
            cos_tab[base + i + half] = c;
            sin_tab[base + i] = s;
            sin_tab[base + i + half] = s;
        }
    }
    return 0;
}

/* nn.cpp:76-101 */
int or_apply_rope(float* x, int64_t heads, int head_dim, int pos, int max_pos,
                  const float* cos_tab, const float* sin_tab) {
    if (pos < 0 || pos >= max_pos) {
        set_err("position is outside the rope table");
        return OR_ERR_ROPE;
    }
    const int half = head_dim / 2;
    const float* c = cos_tab + (size_t)pos * head_dim;
    const float* s = sin_tab + (size_t)pos * head_dim;
    for (int64_t h = 0; h < heads; h++) {
        float* row = x + h * head_dim;
        for (int i = 0; i < half; i++) {
            const float a = row[i];
            const float b = row[i + half];
            row[i] = a * c[i] - b * s[i];
            row[i + half] = b * c[i + half] + a * s[i + half];
        }
    }
    return 0;
}

/* ops.cpp:42-70; rows are independent so they may run on separate threads. */
void or_matmul_nt(const float* A, const float* B, float* C, int64_t M, int64_t N,
                  int64_t K) {
    for (int64_t i = 0; i < M; i++) {
        const float* arow = A + i * K;
#pragma omp parallel for schedule(static) if (N * K > (1 << 18))
        for (int64_t j = 0; j < N; j++) {
            const float* brow = B + j * K;
            float sum = 0.0f;
            for (int64_t k = 0; k < K; k++) sum += arow[k] * brow[k];
            C[i * N + j] = sum;
        }
    }
}

/* quant.cpp:9-41 */
void or_quantize_rows(const float* W, int64_t rows, int64_t cols, int8_t* q,
                      float* scales) {
#pragma omp parallel for schedule(static) if (rows * cols > (1 << 18))
    for (int64_t r = 0; r < rows; r++) {
        const float* row = W + r * cols;
        float amax = 0.0f;
        for (int64_t c = 0; c < cols; c++) {
            const float a = fabsf(row[c]);
            if (amax < a) amax = a; /* std::max(amax, a) */
        }
        const float scale = (amax > 0.0f) ? amax / 127.0f : 1.0f;
        scales[r] = scale;
        const float inv = 1.0f / scale;
        for (int64_t c = 0; c < cols; c++) {
            int v = (int)lrintf(row[c] * inv);
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            q[r * cols + c] = (int8_t)v;
        }
    }
}

/* quant.cpp:43-70 */
void or_matmul_nt_q8(const float* A, const int8_t* Bq, const float* scales,
                     float* C, int64_t M, int64_t N, int64_t K) {
    for (int64_t i = 0; i < M; i++) {
        const float* arow = A + i * K;
#pragma omp parallel for schedule(static) if (N * K > (1 << 18))
        for (int64_t j = 0; j < N; j++) {
            const int8_t* brow = Bq + j * K;
            float acc = 0.0f;
            for (int64_t k = 0; k < K; k++) acc += arow[k] * (float)brow[k];
            C[i * N + j] = acc * scales[j];
        }
    }
}

/* quant.cpp:72-82 */
void or_dequantize(const int8_t* q, const float* scales, int64_t rows,
                   int64_t cols, float* out) {
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++)
            out[r * cols + c] = (float)q[r * cols + c] * scales[r];
}

/* generate.cpp:73-105.  Heads are independent; each head's loops run in the
 * reference's order. */
void or_attention_decode(const float* q, const float* kcache,
                         const float* vcache, int64_t row_stride, int H,
                         int KVH, int D, int n, float* ctx) {
    const int group = H / KVH;
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    memset(ctx, 0, sizeof(float) * (size_t)H * D);
#pragma omp parallel if ((int64_t)n * H * D > (1 << 16))
    {
        float* scores = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
#pragma omp for schedule(static)
        for (int h = 0; h < H; h++) {
            const int kvh = h / group;
            const float* qh = q + (size_t)h * D;
            float m = -INFINITY;
            for (int j = 0; j < n; j++) {
                const float* kj = kcache + (size_t)j * row_stride + (size_t)kvh * D;
                float dot = 0.0f;
                for (int d = 0; d < D; d++) dot += qh[d] * kj[d];
                scores[j] = dot * inv_sqrt_d;
                m = (m < scores[j]) ? scores[j] : m; /* std::max(m, s) */
            }
            double sum = 0.0;
            for (int j = 0; j < n; j++) {
                scores[j] = expf(scores[j] - m);
                sum += scores[j];
            }
            const float inv = (float)(1.0 / sum);
            float* c = ctx + (size_t)h * D;
            for (int j = 0; j < n; j++) {
                const float p = scores[j] * inv;
                const float* vj = vcache + (size_t)j * row_stride + (size_t)kvh * D;
                for (int d = 0; d < D; d++) c[d] += p * vj[d];
            }
        }
        free(scores);
    }
}

/* model.cpp:15-18 and 44-46 */
void or_silu_mul(float* gate, const float* up, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const float g = gate[i];
        gate[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

/* generate.cpp:199-206 */
int or_argmax(const float* logits, int64_t vocab) {
    int best = 0;
    for (int64_t i = 1; i < vocab; i++)
        if (logits[i] > logits[best]) best = (int)i;
    return best;
}

/* ------------------------------------------------------------------------ */
/* sampling (generate.cpp:197-252)                                          */
/* ------------------------------------------------------------------------ */

/* MT19937-64 (Matsumoto & Nishimura), the std::mt19937_64 parameters. */
typedef struct {
    uint64_t mt[312];
    int idx;
} or_mt64;

static void or_mt64_seed(or_mt64* g, uint64_t seed) {
    g->mt[0] = seed;
    for (int i = 1; i < 312; i++)
        g->mt[i] = 6364136223846793005ULL * (g->mt[i - 1] ^ (g->mt[i - 1] >> 62)) + (uint64_t)i;
    g->idx = 312;
}

static uint64_t or_mt64_next(or_mt64* g) {
    const uint64_t upper = 0xFFFFFFFF80000000ULL, lower = 0x7FFFFFFFULL;
    if (g->idx >= 312) {
        for (int i = 0; i < 312; i++) {
            const uint64_t y = (g->mt[i] & upper) | (g->mt[(i + 1) % 312] & lower);
            uint64_t v = g->mt[(i + 156) % 312] ^ (y >> 1);
            if (y & 1ULL) v ^= 0xB5026F5AA96619E9ULL;
            g->mt[i] = v;
        }
        g->idx = 0;
    }
    uint64_t x = g->mt[g->idx++];
    x ^= (x >> 29) & 0x5555555555555555ULL;
    x ^= (x << 17) & 0x71D67FFFEDA60000ULL;
    x ^= (x << 37) & 0xFFF7EEE000000000ULL;
    x ^= x >> 43;
    return x;
}

static double or_uniform01(or_mt64* g) {
    double r = (double)or_mt64_next(g) / 18446744073709551616.0;
    if (r >= 1.0) r = nextafter(1.0, 0.0);
    return r;
}

typedef struct {
    float v;
    int i;
} or_cand;

static int or_cand_cmp(const void* a, const void* b) {
    const or_cand* x = (const or_cand*)a;
    const or_cand* y = (const or_cand*)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

int or_sample_seq(float temperature, int top_k, float top_p, uint64_t seed, const float* logits, int64_t vocab,
                  int n, int* out) {
    or_mt64 g;
    or_mt64_seed(&g, seed);
    or_cand* c = (or_cand*)malloc(sizeof(or_cand) * (size_t)vocab);
    float* p = (float*)malloc(sizeof(float) * (size_t)vocab);
    if (!c || !p) {
        free(c);
        free(p);
        return -1;
    }
    for (int s = 0; s < n; s++) {
        const float* lg = logits + (size_t)s * vocab;
        if (temperature <= 0.0f || top_k == 1) {
            out[s] = or_argmax(lg, vocab);
            continue;
        }
        for (int64_t i = 0; i < vocab; i++) {
            c[i].v = lg[i];
            c[i].i = (int)i;
        }
        qsort(c, (size_t)vocab, sizeof(or_cand), or_cand_cmp);
        int64_t keep = vocab;
        if (top_k > 0 && top_k < keep) keep = top_k;
        const float m = c[0].v;
        double sum = 0.0;
        for (int64_t i = 0; i < keep; i++) {
            const float d = c[i].v - m;
            const float q = d / temperature;
            p[i] = expf(q);
            sum += p[i];
        }
        for (int64_t i = 0; i < keep; i++) p[i] = (float)(p[i] / sum);
        if (top_p < 1.0f) {
            double cum = 0.0;
            int64_t cut = keep;
            for (int64_t i = 0; i < keep; i++) {
                cum += p[i];
                if (cum >= top_p) {
                    cut = i + 1;
                    break;
                }
            }
            keep = cut;
            double renorm = 0.0;
            for (int64_t i = 0; i < keep; i++) renorm += p[i];
            for (int64_t i = 0; i < keep; i++) p[i] = (float)(p[i] / renorm);
        }
        const double r = or_uniform01(&g);
        double cum = 0.0;
        int pick = c[keep - 1].i;
        for (int64_t i = 0; i < keep; i++) {
            cum += p[i];
            if (r <= cum) {
                pick = c[i].i;
                break;
            }
        }
        out[s] = pick;
    }
    free(c);
    free(p);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* whole model                                                              */
/* ------------------------------------------------------------------------ */

typedef struct {
    int8_t* q;
    float* s;
    int64_t rows, cols;
} qt;

struct or_model {
    or_config c;
    const float* embed;
    const float* final_norm;
    or_layer_weights* L;
    int quantized;
    qt* Q; /* [layers*7] */
    int8_t* lm_q; /* opt-in INT8 tied lm_head (quantize_rows of embed), or NULL */
    float* lm_s;
    float* rope_cos;
    float* rope_sin;
    /* caches */
    int max_seq, len;
    float** kc;
    float** vc;
    /* scratch */
    float *x, *normed, *attn_out, *ffn_out, *q, *k, *v, *ctx, *gate, *up, *next;
};

static void* xcalloc(size_t n, size_t sz) {
    void* p = calloc(n ? n : 1, sz);
    return p;
}

or_model* or_model_create(const or_config* cfg, const float* embed,
                          const float* final_norm,
                          const or_layer_weights* layers) {
    if (!cfg || !embed || !final_norm || !layers) return NULL;
    if (cfg->heads % cfg->kv_heads != 0 || cfg->head_dim % 2 != 0) return NULL;
    or_model* m = (or_model*)xcalloc(1, sizeof(or_model));
    m->c = *cfg;
    m->embed = embed;
    m->final_norm = final_norm;
    m->L = (or_layer_weights*)xcalloc((size_t)cfg->layers, sizeof(or_layer_weights));
    memcpy(m->L, layers, sizeof(or_layer_weights) * (size_t)cfg->layers);
    m->rope_cos = (float*)xcalloc((size_t)cfg->rope_positions * cfg->head_dim, sizeof(float));
    m->rope_sin = (float*)xcalloc((size_t)cfg->rope_positions * cfg->head_dim, sizeof(float));
    or_build_rope_table(cfg->head_dim, cfg->rope_positions, cfg->theta, m->rope_cos,
                        m->rope_sin);
    const size_t hd = (size_t)cfg->hidden, qd = (size_t)cfg->heads * cfg->head_dim,
                 kd = (size_t)cfg->kv_heads * cfg->head_dim, fd = (size_t)cfg->ffn;
    m->x = (float*)xcalloc(hd, 4);
    m->next = (float*)xcalloc(hd, 4);
    m->normed = (float*)xcalloc(hd, 4);
    m->attn_out = (float*)xcalloc(hd, 4);
    m->ffn_out = (float*)xcalloc(hd, 4);
    m->q = (float*)xcalloc(qd, 4);
    m->k = (float*)xcalloc(kd, 4);
    m->v = (float*)xcalloc(kd, 4);
    m->ctx = (float*)xcalloc(qd, 4);
    m->gate = (float*)xcalloc(fd, 4);
    m->up = (float*)xcalloc(fd, 4);
    return m;
}

static void free_caches(or_model* m) {
    if (m->kc) {
        for (int l = 0; l < m->c.layers; l++) {
            free(m->kc[l]);
            free(m->vc[l]);
        }
        free(m->kc);
        free(m->vc);
    }
    m->kc = m->vc = NULL;
}

void or_model_free(or_model* m) {
    if (!m) return;
    free_caches(m);
    if (m->Q) {
        for (int i = 0; i < m->c.layers * 7; i++) {
            free(m->Q[i].q);
            free(m->Q[i].s);
        }
        free(m->Q);
    }
    free(m->lm_q);
    free(m->lm_s);
    free(m->L);
    free(m->rope_cos);
    free(m->rope_sin);
    free(m->x); free(m->next); free(m->normed); free(m->attn_out); free(m->ffn_out);
    free(m->q); free(m->k); free(m->v); free(m->ctx); free(m->gate); free(m->up);
    free(m);
}

static const float* proj_ptr(const or_layer_weights* L, int which) {
    switch (which) {
        case 0: return L->wq; case 1: return L->wk; case 2: return L->wv;
        case 3: return L->wo; case 4: return L->wg; case 5: return L->wu;
        default: return L->wd;
    }
}

static void proj_shape(const or_config* c, int which, int64_t* rows, int64_t* cols) {
    const int64_t qd = (int64_t)c->heads * c->head_dim, kd = (int64_t)c->kv_heads * c->head_dim;
    switch (which) {
        case 0: *rows = qd; *cols = c->hidden; break;
        case 1: case 2: *rows = kd; *cols = c->hidden; break;
        case 3: *rows = c->hidden; *cols = qd; break;
        case 4: case 5: *rows = c->ffn; *cols = c->hidden; break;
        default: *rows = c->hidden; *cols = c->ffn; break;
    }
}

/* model.cpp:313-338 */
int or_model_quantize(or_model* m) {
    if (m->quantized) return 0;
    m->Q = (qt*)xcalloc((size_t)m->c.layers * 7, sizeof(qt));
    for (int l = 0; l < m->c.layers; l++) {
        for (int w = 0; w < 7; w++) {
            qt* t = &m->Q[l * 7 + w];
            proj_shape(&m->c, w, &t->rows, &t->cols);
            t->q = (int8_t*)xcalloc((size_t)(t->rows * t->cols), 1);
            t->s = (float*)xcalloc((size_t)t->rows, 4);
            if (!t->q || !t->s) { set_err("out of memory"); return OR_ERR_OOM; }
            or_quantize_rows(proj_ptr(&m->L[l], w), t->rows, t->cols, t->q, t->s);
        }
    }
    m->quantized = 1;
    return 0;
}

int or_model_is_quantized(const or_model* m) { return m->quantized; }

int or_model_quant_tensor(const or_model* m, int layer, int which,
                          const int8_t** q, const float** scales, int64_t* rows,
                          int64_t* cols) {
    if (!m->quantized || layer < 0 || layer >= m->c.layers || which < 0 || which > 6)
        return OR_ERR_ARG;
    const qt* t = &m->Q[layer * 7 + which];
    *q = t->q; *scales = t->s; *rows = t->rows; *cols = t->cols;
    return 0;
}

/* model.cpp:277-282, generate.cpp:14-22 */
int or_model_reset_cache(or_model* m, int max_seq) {
    if (max_seq <= 0) return OR_ERR_ARG;
    free_caches(m);
    const size_t n = (size_t)max_seq * m->c.kv_heads * m->c.head_dim;
    m->kc = (float**)xcalloc((size_t)m->c.layers, sizeof(float*));
    m->vc = (float**)xcalloc((size_t)m->c.layers, sizeof(float*));
    for (int l = 0; l < m->c.layers; l++) {
        m->kc[l] = (float*)xcalloc(n, 4);
        m->vc[l] = (float*)xcalloc(n, 4);
        if (!m->kc[l] || !m->vc[l]) { set_err("out of memory"); return OR_ERR_OOM; }
    }
    m->max_seq = max_seq;
    m->len = 0;
    return 0;
}

int or_model_cache_len(const or_model* m) { return m->len; }

const float* or_model_kv(const or_model* m, int layer, int which) {
    if (!m->kc || layer < 0 || layer >= m->c.layers) return NULL;
    return which == 0 ? m->kc[layer] : m->vc[layer];
}

static void proj(const or_model* m, int l, int which, const float* x, float* y) {
    int64_t rows, cols;
    proj_shape(&m->c, which, &rows, &cols);
    if (m->quantized) {
        const qt* t = &m->Q[l * 7 + which];
        or_matmul_nt_q8(x, t->q, t->s, y, 1, rows, cols);
    } else {
        or_matmul_nt(x, proj_ptr(&m->L[l], which), y, 1, rows, cols);
    }
}

/* generate.cpp:24-108 (f32) and 110-195 (int8); the cache-full and rope
 * checks run before anything is written, so an error leaves the model as it
 * was. */
static int attention_step(or_model* m, int l, const float* x, float* out, int pos) {
    const or_config* c = &m->c;
    const int H = c->heads, KVH = c->kv_heads, D = c->head_dim;
    const or_layer_weights* L = &m->L[l];
    proj(m, l, 0, x, m->q);
    proj(m, l, 1, x, m->k);
    proj(m, l, 2, x, m->v);
    /* per-head q/k rmsnorm (generate.cpp:52-64): in place is equivalent to the
     * reference's tmp copies since each head only reads itself */
    or_rmsnorm(m->q, L->q_norm, c->eps, m->q, H, D);
    int rc = or_apply_rope(m->q, H, D, pos, c->rope_positions, m->rope_cos, m->rope_sin);
    if (rc) return rc;
    or_rmsnorm(m->k, L->k_norm, c->eps, m->k, KVH, D);
    rc = or_apply_rope(m->k, KVH, D, pos, c->rope_positions, m->rope_cos, m->rope_sin);
    if (rc) return rc;
    const size_t w = (size_t)KVH * D;
    memcpy(m->kc[l] + (size_t)pos * w, m->k, w * 4);
    memcpy(m->vc[l] + (size_t)pos * w, m->v, w * 4);
    or_attention_decode(m->q, m->kc[l], m->vc[l], (int64_t)w, H, KVH, D, pos + 1, m->ctx);
    proj(m, l, 3, m->ctx, out);
    return 0;
}

/* model.cpp:284-311 with layer_step (235-254) / layer_step_q (256-275) */
int or_model_step(or_model* m, int token, float* logits) {
    const or_config* c = &m->c;
    if (!m->kc) { set_err("call reset_cache() first"); return OR_ERR_NO_CACHE; }
    if (token < 0 || token >= c->vocab) {
        set_err("token id out of range for the embedding table");
        return OR_ERR_TOKEN;
    }
    if (m->len >= m->max_seq) { set_err("kv cache is full"); return OR_ERR_CACHE_FULL; }
    if (m->len >= c->rope_positions) {
        set_err("position is outside the rope table");
        return OR_ERR_ROPE;
    }
    const int64_t hd = c->hidden;
    const int pos = m->len;
    memcpy(m->x, m->embed + (size_t)token * hd, (size_t)hd * 4);
    for (int l = 0; l < c->layers; l++) {
        const or_layer_weights* L = &m->L[l];
        or_rmsnorm(m->x, L->input_norm, c->eps, m->normed, 1, hd);
        int rc = attention_step(m, l, m->normed, m->attn_out, pos);
        if (rc) return rc;
        for (int64_t i = 0; i < hd; i++) m->next[i] = m->x[i] + m->attn_out[i];
        or_rmsnorm(m->next, L->post_norm, c->eps, m->normed, 1, hd);
        proj(m, l, 4, m->normed, m->gate);
        proj(m, l, 5, m->normed, m->up);
        or_silu_mul(m->gate, m->up, c->ffn);
        proj(m, l, 6, m->gate, m->ffn_out);
        for (int64_t i = 0; i < hd; i++) m->next[i] += m->ffn_out[i];
        memcpy(m->x, m->next, (size_t)hd * 4);
    }
    m->len++;
    or_rmsnorm(m->x, m->final_norm, c->eps, m->normed, 1, hd);
    if (m->lm_q)
        or_matmul_nt_q8(m->normed, m->lm_q, m->lm_s, logits, 1, c->vocab, hd);
    else
        or_matmul_nt(m->normed, m->embed, logits, 1, c->vocab, hd);
    return 0;
}

/* ---- prefill: many positions, layer by layer -----------------------------
 * The reference feeds a prompt one position at a time through Model::step
 * (tools/generate.cpp:75-77).  Position p's layer-l values depend only on its
 * own layer-l input and on the K/V rows of positions <= p, so running every
 * position through layer l before layer l+1 computes the very same numbers --
 * each dot product, norm and softmax below is the per-position operation of
 * or_model_step in the same order -- while every weight row is read once per
 * block of positions instead of once per position.  or_model_prefill is
 * therefore bit-identical to n calls of or_model_step (tested), only faster. */

/* Y[p][j] = sum_k X[p][k] * W[j][k] (sequential in k, as ops.cpp:42-70) for a
 * block of positions at a time: the block's accumulators are independent, so
 * they vectorise without reordering any one sum. */
#define OR_PB 32   /* positions per block (independent accumulators) */
/* 4 independent float lanes; each lane's product and sum round exactly as the
 * scalar statement acc += x * w (no contraction: -ffp-contract=off) */
typedef float or_v4 __attribute__((vector_size(16)));
#define OR_RB 128  /* weight rows per block */

/* Tasks are (row block, position block) pairs; a thread takes consecutive
 * position blocks of one row block, so the row block stays in its cache
 * while the transposed activations stream past. */
#define OR_ROWS_BODY(WTYPE, CONV, FINISH)                                                        \
    const int64_t nrb = (N + OR_RB - 1) / OR_RB, npb = (P + OR_PB - 1) / OR_PB;                 \
    /* XT[pb][k][u] = X[pb * OR_PB + u][k]: one position block is contiguous */                 \
    _Pragma("omp parallel for schedule(static)")                                                 \
    for (int64_t pb = 0; pb < npb; pb++)                                                        \
        for (int64_t k = 0; k < K; k++)                                                         \
            for (int u = 0; u < OR_PB; u++) {                                                   \
                const int64_t p = pb * OR_PB + u;                                               \
                XT[(pb * K + k) * OR_PB + u] = p < P ? X[p * K + k] : 0.0f;                     \
            }                                                                                   \
    _Pragma("omp parallel for collapse(2) schedule(static)")                                     \
    for (int64_t rb = 0; rb < nrb; rb++)                                                        \
        for (int64_t pb = 0; pb < npb; pb++) {                                                  \
            const int64_t p0 = pb * OR_PB, nb = (P - p0 < OR_PB) ? P - p0 : OR_PB;              \
            const int64_t j1 = (rb + 1) * OR_RB < N ? (rb + 1) * OR_RB : N;                     \
            for (int64_t j = rb * OR_RB; j < j1; j++) {                                         \
                const WTYPE* w = W + j * K;                                                     \
                float acc[OR_PB] = {0};                                                         \
                if (nb == OR_PB) {                                                              \
                    or_v4 a[8];                                                                 \
                    for (int i = 0; i < 8; i++) a[i] = (or_v4){0.0f, 0.0f, 0.0f, 0.0f};         \
                    const float* xt = XT + pb * K * OR_PB;                                      \
                    for (int64_t k = 0; k < K; k++, xt += OR_PB) {                              \
                        const float wk = CONV(w[k]);                                            \
                        const or_v4 wv = {wk, wk, wk, wk};                                      \
                        for (int i = 0; i < 8; i++) {                                           \
                            or_v4 xv;                                                           \
                            memcpy(&xv, xt + 4 * i, 16);                                        \
                            a[i] += xv * wv;                                                    \
                        }                                                                       \
                    }                                                                           \
                    memcpy(acc, a, sizeof a);                                                   \
                } else {                                                                        \
                    for (int64_t k = 0; k < K; k++) {                                           \
                        const float wk = CONV(w[k]);                                            \
                        const float* xt = XT + (pb * K + k) * OR_PB;                            \
                        for (int64_t u = 0; u < nb; u++) acc[u] += xt[u] * wk;                  \
                    }                                                                           \
                }                                                                               \
                for (int64_t u = 0; u < nb; u++) Y[(p0 + u) * N + j] = FINISH(acc[u]);          \
            }                                                                                   \
        }

#define OR_ID(v) (v)
#define OR_I2F(v) ((float)(v))

/* Y[p][j] = sum_k X[p][k] * W[j][k], sequential in k as ops.cpp:42-70; the
 * OR_PB accumulators of a block are independent, so they vectorise without
 * reordering any one sum. */
static void rows_matmul_nt(const float* X, int64_t P, const float* W, int64_t N, int64_t K, float* Y,
                           float* XT) {
    OR_ROWS_BODY(float, OR_ID, OR_ID)
}

/* The INT8 twin (quant.cpp:43-70): acc += x[k] * float(q[j][k]), then
 * acc * scale[j]. */
static void rows_matmul_nt_q8(const float* X, int64_t P, const int8_t* W, const float* scales, int64_t N,
                              int64_t K, float* Y, float* XT) {
#define OR_SCALE(a) ((a) * scales[j])
    OR_ROWS_BODY(int8_t, OR_I2F, OR_SCALE)
#undef OR_SCALE
}

static void rows_proj(const or_model* m, int l, int which, const float* X, int64_t P, float* Y, float* XT) {
    int64_t rows, cols;
    proj_shape(&m->c, which, &rows, &cols);
    if (m->quantized) {
        const qt* t = &m->Q[l * 7 + which];
        rows_matmul_nt_q8(X, P, t->q, t->s, rows, cols, Y, XT);
    } else {
        rows_matmul_nt(X, P, proj_ptr(&m->L[l], which), rows, cols, Y, XT);
    }
}

/* One head of or_attention_decode (generate.cpp:73-105) for one query, with
 * the keys of its KV head transposed (KT[d][j], row length ldk) so four
 * positions' dot products run in four vector lanes, each lane summing over d
 * in order; the P.V sum runs four dims per lane, each over j in order. */
static void attention_head(const float* qh, const float* KT, int64_t ldk, const float* vcache,
                           int64_t row_stride, int kvh, int D, int n, float* scores, float* c) {
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    float m = -INFINITY;
    int j = 0;
    for (; j + 4 <= n; j += 4) {
        or_v4 dot = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int d = 0; d < D; d++) {
            or_v4 kv;
            memcpy(&kv, KT + (size_t)d * ldk + j, 16);
            const or_v4 qv = {qh[d], qh[d], qh[d], qh[d]};
            dot += qv * kv;
        }
        for (int u = 0; u < 4; u++) {
            scores[j + u] = dot[u] * inv_sqrt_d;
            m = (m < scores[j + u]) ? scores[j + u] : m;
        }
    }
    for (; j < n; j++) {
        float dot = 0.0f;
        for (int d = 0; d < D; d++) dot += qh[d] * KT[(size_t)d * ldk + j];
        scores[j] = dot * inv_sqrt_d;
        m = (m < scores[j]) ? scores[j] : m;
    }
    double sum = 0.0;
    for (j = 0; j < n; j++) {
        scores[j] = expf(scores[j] - m);
        sum += scores[j];
    }
    const float inv = (float)(1.0 / sum);
    or_v4 acc[32];
    for (int i = 0; i < D / 4; i++) acc[i] = (or_v4){0.0f, 0.0f, 0.0f, 0.0f};
    for (j = 0; j < n; j++) {
        const float pj = scores[j] * inv;
        const or_v4 pv = {pj, pj, pj, pj};
        const float* vj = vcache + (size_t)j * row_stride + (size_t)kvh * D;
        for (int i = 0; i < D / 4; i++) {
            or_v4 vv;
            memcpy(&vv, vj + 4 * i, 16);
            acc[i] += pv * vv;
        }
    }
    memcpy(c, acc, sizeof(float) * (size_t)D);
}

int or_model_prefill(or_model* m, const int* tokens, int n, float* logits) {
    const or_config* c = &m->c;
    if (!m->kc) { set_err("call reset_cache() first"); return OR_ERR_NO_CACHE; }
    if (n <= 0) return 0;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c->vocab) {
            set_err("token id out of range for the embedding table");
            return OR_ERR_TOKEN;
        }
    if (m->len + n > m->max_seq) { set_err("kv cache is full"); return OR_ERR_CACHE_FULL; }
    if (m->len + n > c->rope_positions) {
        set_err("position is outside the rope table");
        return OR_ERR_ROPE;
    }
    const int64_t P = n, hd = c->hidden, H = c->heads, KVH = c->kv_heads, D = c->head_dim;
    const int64_t qd = H * D, kd = KVH * D, fd = c->ffn;
    const int64_t widest = (fd > qd ? fd : qd) > hd ? (fd > qd ? fd : qd) : hd;
    float* X = (float*)malloc(sizeof(float) * P * hd);
    float* X2 = (float*)malloc(sizeof(float) * P * hd);
    float* NR = (float*)malloc(sizeof(float) * P * hd);
    float* T = (float*)malloc(sizeof(float) * P * hd);
    float* Qb = (float*)malloc(sizeof(float) * P * qd);
    float* Kb = (float*)malloc(sizeof(float) * P * kd);
    float* Vb = (float*)malloc(sizeof(float) * P * kd);
    float* CX = (float*)malloc(sizeof(float) * P * qd);
    float* G = (float*)malloc(sizeof(float) * P * fd);
    float* U = (float*)malloc(sizeof(float) * P * fd);
    float* XT = (float*)malloc(sizeof(float) * (P + OR_PB) * widest);
    float* KTa = (float*)malloc(sizeof(float) * (size_t)(m->len + P) * kd);
    int rc = 0;
    if (!X || !X2 || !NR || !T || !Qb || !Kb || !Vb || !CX || !G || !U || !XT || !KTa) {
        set_err("out of memory");
        rc = OR_ERR_OOM;
        goto done;
    }
    const int p0 = m->len;
    for (int64_t p = 0; p < P; p++) memcpy(X + p * hd, m->embed + (size_t)tokens[p] * hd, (size_t)hd * 4);
    for (int l = 0; l < c->layers; l++) {
        const or_layer_weights* L = &m->L[l];
        or_rmsnorm(X, L->input_norm, c->eps, NR, P, hd);
        rows_proj(m, l, 0, NR, P, Qb, XT);
        rows_proj(m, l, 1, NR, P, Kb, XT);
        rows_proj(m, l, 2, NR, P, Vb, XT);
        for (int64_t p = 0; p < P; p++) {
            float* q = Qb + p * qd;
            float* k = Kb + p * kd;
            or_rmsnorm(q, L->q_norm, c->eps, q, H, D);
            or_apply_rope(q, H, (int)D, p0 + (int)p, c->rope_positions, m->rope_cos, m->rope_sin);
            or_rmsnorm(k, L->k_norm, c->eps, k, KVH, D);
            or_apply_rope(k, KVH, (int)D, p0 + (int)p, c->rope_positions, m->rope_cos, m->rope_sin);
            memcpy(m->kc[l] + (size_t)(p0 + p) * kd, k, (size_t)kd * 4);
            memcpy(m->vc[l] + (size_t)(p0 + p) * kd, Vb + p * kd, (size_t)kd * 4);
        }
        const int group = (int)(H / KVH);
        const int64_t nk = p0 + P;
        /* keys transposed per KV head: KTa[kvh][d][j] */
#pragma omp parallel for schedule(static)
        for (int64_t hk = 0; hk < KVH; hk++)
            for (int64_t j = 0; j < nk; j++)
                for (int64_t d = 0; d < D; d++)
                    KTa[(hk * D + d) * nk + j] = m->kc[l][(size_t)j * kd + hk * D + d];
#pragma omp parallel
        {
            float* scores = (float*)malloc(sizeof(float) * (size_t)nk);
#pragma omp for schedule(dynamic, 1)
            for (int64_t t = P * H - 1; t >= 0; t--) { /* longest rows first */
                const int64_t p = t / H, h = t % H, hk = h / group;
                attention_head(Qb + p * qd + h * D, KTa + hk * D * nk, nk, m->vc[l], kd, (int)hk, (int)D,
                               p0 + (int)p + 1, scores, CX + p * qd + h * D);
            }
            free(scores);
        }
        rows_proj(m, l, 3, CX, P, T, XT);
        for (int64_t i = 0; i < P * hd; i++) X2[i] = X[i] + T[i];
        or_rmsnorm(X2, L->post_norm, c->eps, NR, P, hd);
        rows_proj(m, l, 4, NR, P, G, XT);
        rows_proj(m, l, 5, NR, P, U, XT);
        for (int64_t p = 0; p < P; p++) or_silu_mul(G + p * fd, U + p * fd, fd);
        rows_proj(m, l, 6, G, P, T, XT);
        for (int64_t i = 0; i < P * hd; i++) X[i] = X2[i] + T[i];
    }
    m->len += n;
    memcpy(m->x, X + (P - 1) * hd, (size_t)hd * 4);
    if (logits) {
        or_rmsnorm(m->x, m->final_norm, c->eps, m->normed, 1, hd);
        if (m->lm_q)
            or_matmul_nt_q8(m->normed, m->lm_q, m->lm_s, logits, 1, c->vocab, hd);
        else
            or_matmul_nt(m->normed, m->embed, logits, 1, c->vocab, hd);
    }
done:
    free(X); free(X2); free(NR); free(T); free(Qb); free(Kb); free(Vb); free(CX); free(G); free(U); free(XT);
    free(KTa);
    return rc;
}

/* Opt-in (no reference counterpart: the reference keeps the tied lm_head in
 * f32, model.cpp:313-338): the lm_head product with the embedding rows
 * quantised by quantize_rows and multiplied as matmul_nt_q8. */
int or_model_quantize_lm_head(or_model* m) {
    if (m->lm_q) return 0;
    const int64_t V = m->c.vocab, hd = m->c.hidden;
    m->lm_q = (int8_t*)malloc((size_t)V * hd);
    m->lm_s = (float*)malloc(sizeof(float) * (size_t)V);
    if (!m->lm_q || !m->lm_s) return -1;
    or_quantize_rows(m->embed, V, hd, m->lm_q, m->lm_s);
    return 0;
}

/* model.cpp:340-365 (tied embeddings: lm_head_ is empty) */
size_t or_model_weight_bytes(const or_model* m) {
    const or_config* c = &m->c;
    size_t total = (size_t)c->vocab * c->hidden * 4 + (size_t)c->hidden * 4;
    for (int l = 0; l < c->layers; l++) {
        total += (size_t)(2 * c->hidden + 2 * c->head_dim) * 4;
        for (int w = 0; w < 7; w++) {
            int64_t r, cc;
            proj_shape(c, w, &r, &cc);
            total += m->quantized ? (size_t)(r * cc) + (size_t)r * 4 : (size_t)(r * cc) * 4;
        }
    }
    return total;
}

/* ---- synthetic weights ---------------------------------------------------
 * The seeded N(0, std) generator every benchmark and test model is drawn from,
 * restated here so the reference arm of the benchmark can produce the same
 * weights without loading the engine library: element pair p takes the
 * SplitMix64 finaliser (Steele, Lea & Flood, OOPSLA 2014) of
 * seed + (p + 1) * golden-gamma as two 24-bit uniforms in (0, 1), turned into
 * two normals by the Box-Muller transform in double.  Pairs are independent,
 * so the result does not depend on the thread count. */
static uint64_t or_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void or_synth_normal(float* out, uint64_t n, uint64_t seed, float stdv) {
    const double two_pi = 6.283185307179586476925286766559;
    const int64_t pairs = (int64_t)((n + 1) / 2);
#pragma omp parallel for schedule(static) if (pairs > (1 << 16))
    for (int64_t p = 0; p < pairs; p++) {
        const uint64_t z = or_mix64(seed + ((uint64_t)p + 1) * 0x9E3779B97F4A7C15ull);
        const double u1 = ((double)(z >> 40) + 0.5) * (1.0 / 16777216.0);
        const double u2 = ((double)(z & 0xFFFFFFull) + 0.5) * (1.0 / 16777216.0);
        const double r = sqrt(-2.0 * log(u1));
        const double a = two_pi * u2;
        const uint64_t i = 2 * (uint64_t)p;
        out[i] = (float)(r * cos(a) * stdv);
        if (i + 1 < n) out[i + 1] = (float)(r * sin(a) * stdv);
    }
}
