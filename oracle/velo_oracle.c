/*
 * velo_oracle.c -- CPU oracle (TEST INFRASTRUCTURE ONLY, see velo_oracle.h).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no fast-math) so that
 * every float operation is one IEEE operation in source order, as in the
 * Rust reference (which LLVM compiles without contraction).  libm supplies
 * expf/powf/sinf/cosf/sqrtf exactly as Rust's f32 methods do on Linux.
 */
#include "velo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* ------------------------------------------------------------------ */
/* quant.rs                                                            */
/* ------------------------------------------------------------------ */

/* quant.rs:18-34 -- note the subnormal branch scales mant by 2^-24. */
float vo_f16_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t)(bits >> 15)) << 31;
    uint32_t exp = (bits >> 10) & 0x1F;
    uint32_t mant = bits & 0x3FF;
    float out;
    if (exp == 0) {
        float v = (float)mant * (1.0f / (float)(1u << 24));
        return sign ? -v : v;
    } else if (exp == 31) {
        uint32_t b = sign | 0x7F800000u | (mant << 13);
        memcpy(&out, &b, 4);
        return out;
    } else {
        uint32_t b = sign | ((exp + 112) << 23) | (mant << 13);
        memcpy(&out, &b, 4);
        return out;
    }
}

/* IEEE binary16 encode, round to nearest even (inputs for fp16 tensors). */
uint16_t vo_f32_to_f16(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    uint32_t sign = (b >> 16) & 0x8000u;
    uint32_t absb = b & 0x7FFFFFFFu;
    if (absb >= 0x7F800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (absb > 0x7F800000u ? 0x200u : 0));
    }
    if (absb >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* overflow */
    if (absb < 0x38800000u) { /* subnormal or zero in f16 */
        /* value = absb as float; f16 subnormal unit = 2^-24 */
        float a;
        memcpy(&a, &absb, 4);
        float scaled = a * 16777216.0f; /* exact: multiply by 2^24 */
        float r = rintf(scaled);        /* ties to even */
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t exp = ((absb >> 23) - 127 + 15);
    uint32_t mant = absb & 0x7FFFFFu;
    uint32_t half = (exp << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half += 1;
    return (uint16_t)(sign | half);
}

/* quant.rs:44-73: block = f16 d + 16 bytes; element 2i = d*(lo-8),
 * element 2i+1 = d*(hi-8) (interleaved, NOT the upstream ggml order). */
void vo_dequant_q4_0_row(const uint8_t *data, float *out, size_t n) {
    size_t nb = n / 32;
    for (size_t b = 0; b < nb; ++b) {
        const uint8_t *blk = data + b * 18;
        float delta = vo_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int i = 0; i < 16; ++i) {
            uint8_t byte = blk[2 + i];
            int lo = (int)(byte & 0x0F) - 8;
            int hi = (int)((byte >> 4) & 0x0F) - 8;
            out[b * 32 + 2 * i] = delta * (float)lo;
            out[b * 32 + 2 * i + 1] = delta * (float)hi;
        }
    }
}

size_t vo_row_bytes(int dtype, size_t cols) {
    switch (dtype) {
    case VO_F32: return cols * 4;
    case VO_F16: return cols * 2;
    case VO_Q4_0: return cols / 32 * 18;
    default: return 0;
    }
}

/* quant.rs:181-191 */
void vo_dequant_row(int dtype, const uint8_t *data, float *out, size_t n) {
    switch (dtype) {
    case VO_F32:
        for (size_t i = 0; i < n; ++i) memcpy(&out[i], data + 4 * i, 4);
        break;
    case VO_F16:
        for (size_t i = 0; i < n; ++i)
            out[i] = vo_f16_to_f32((uint16_t)(data[2 * i] | (data[2 * i + 1] << 8)));
        break;
    case VO_Q4_0:
        vo_dequant_q4_0_row(data, out, n);
        break;
    default:
        for (size_t i = 0; i < n; ++i) out[i] = 0.0f;
    }
}

/* q4_0 quantiser (own method; the reference only dequantises).  Per block of
 * 32: m = the element of largest magnitude (first on ties), d = m / -8 so the
 * extreme maps to nibble 0, q = clamp((int)(x/d + 8.5), 0, 15); d stored as
 * f16.  Nibbles are written in the reference's interleaved order. */
void vo_quantize_q4_0_row(const float *x, size_t n, uint8_t *out) {
    size_t nb = n / 32;
    for (size_t b = 0; b < nb; ++b) {
        const float *xb = x + b * 32;
        float amax = 0.0f, m = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(xb[j]);
            if (a > amax) { amax = a; m = xb[j]; }
        }
        float d = m / -8.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = vo_f32_to_f16(d);
        uint8_t *blk = out + b * 18;
        blk[0] = (uint8_t)(dh & 0xFF);
        blk[1] = (uint8_t)(dh >> 8);
        for (int i = 0; i < 16; ++i) {
            int q0 = (int)(xb[2 * i] * id + 8.5f);
            int q1 = (int)(xb[2 * i + 1] * id + 8.5f);
            if (q0 < 0) q0 = 0;
            if (q0 > 15) q0 = 15;
            if (q1 < 0) q1 = 0;
            if (q1 > 15) q1 = 15;
            blk[2 + i] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

/* ------------------------------------------------------------------ */
/* llama_cpu.rs math primitives                                        */
/* ------------------------------------------------------------------ */

/* llama_cpu.rs:55-60: x = (x / rms) * w, rms = sqrt(sum(x^2)/n + eps) */
void vo_rms_norm(float *x, const float *w, size_t n, float eps) {
    float ss = 0.0f;
    for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float rms = sqrtf(ss / (float)n + eps);
    for (size_t i = 0; i < n; ++i) x[i] = (x[i] / rms) * w[i];
}

/* llama_cpu.rs:94 */
float vo_silu(float x) { return x * (1.0f / (1.0f + expf(-x))); }

/* llama_cpu.rs:113-132 (NeoX half-split rotation) */
static void apply_rope(float *x, size_t pos, size_t n_heads, size_t head_dim,
                       size_t half, float freq_base) {
    for (size_t h = 0; h < n_heads; ++h) {
        size_t off = h * head_dim;
        for (size_t i = 0; i < half; ++i) {
            float theta = (float)pos / powf(freq_base, 2.0f * (float)i / (float)head_dim);
            float s = sinf(theta), c = cosf(theta);
            float x0 = x[off + i];
            float x1 = x[off + i + half];
            x[off + i] = x0 * c - x1 * s;
            x[off + i + half] = x0 * s + x1 * c;
        }
    }
}

/* llama_cpu.rs:99-111 */
void vo_rope(float *q, float *k, size_t pos, size_t n_heads, size_t n_kv_heads,
             size_t head_dim, float freq_base) {
    size_t half = head_dim / 2;
    apply_rope(q, pos, n_heads, head_dim, half, freq_base);
    apply_rope(k, pos, n_kv_heads, head_dim, half, freq_base);
}

/* llama_cpu.rs:135-146 */
void vo_softmax(float *x, size_t n) {
    float mx = -INFINITY;
    for (size_t i = 0; i < n; ++i) mx = fmaxf(mx, x[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

/* llama_cpu.rs:75-90: out[r] += dot(dequant(row r), x) */
static void matvec_rows(float *out, const uint8_t *data, int dtype, const float *x,
                        size_t r0, size_t r1, size_t cols) {
    size_t rb = vo_row_bytes(dtype, cols);
    float *row = (float *)malloc(cols * sizeof(float));
    for (size_t r = r0; r < r1; ++r) {
        vo_dequant_row(dtype, data + r * rb, row, cols);
        float dot = 0.0f;
        for (size_t c = 0; c < cols; ++c) dot += row[c] * x[c];
        out[r] += dot;
    }
    free(row);
}

/* Rows of a matvec may be split over threads (vo_set_threads, default 1):
 * each row is still one sequential dot product, so the result is the same
 * bits as one thread.  Only the tests raise it, to check large shapes. */
static int g_threads = 1;
void vo_set_threads(int n) { g_threads = n < 1 ? 1 : n > 256 ? 256 : n; }

typedef struct {
    float *out;
    const uint8_t *data;
    int dtype;
    const float *x;
    size_t r0, r1, cols;
} matvec_job;

static void *matvec_job_run(void *arg) {
    matvec_job *j = (matvec_job *)arg;
    matvec_rows(j->out, j->data, j->dtype, j->x, j->r0, j->r1, j->cols);
    return NULL;
}

void vo_matvec_quant(float *out, const uint8_t *data, int dtype, const float *x,
                     size_t rows, size_t cols) {
    int nt = g_threads;
    if (nt <= 1 || rows * cols < ((size_t)1 << 20) || rows < (size_t)nt) {
        matvec_rows(out, data, dtype, x, 0, rows, cols);
        return;
    }
    pthread_t th[256];
    matvec_job jobs[256];
    int joined[256];
    for (int t = 0; t < nt; ++t) {
        jobs[t] = (matvec_job){out, data, dtype, x, rows * t / nt, rows * (t + 1) / nt, cols};
        joined[t] = 0;
        if (t == 0) continue;
        if (pthread_create(&th[t], NULL, matvec_job_run, &jobs[t]) == 0)
            joined[t] = 1;
        else
            matvec_job_run(&jobs[t]); /* no thread: do its rows here */
    }
    matvec_job_run(&jobs[0]);
    for (int t = 1; t < nt; ++t)
        if (joined[t]) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------ */
/* model (llama_cpu.rs:168-419)                                        */
/* ------------------------------------------------------------------ */

struct vo_model {
    vo_meta meta;
    const uint8_t **t; /* tensor pointers */
    int *dt;
    size_t n_tensors;
    float *k, *v;      /* KvCache [layer][n_ctx][n_kv*hd] */
    float *tk, *tv;    /* tree scratch [layer][n_nodes_cap][n_kv*hd] */
    size_t tree_cap;
    size_t pos;
};

enum { T_EMBD = 0, T_ONORM = 1, T_OUT = 2, T_LAYER0 = 3 };
enum { L_ANORM = 0, L_WQ, L_WK, L_WV, L_WO, L_FNORM, L_W1, L_W2, L_W3, L_N };

vo_model *vo_model_new(const vo_meta *meta, const void *const *tensors,
                       const int *dtypes) {
    vo_model *m = (vo_model *)calloc(1, sizeof(vo_model));
    m->meta = *meta;
    m->n_tensors = 3 + (size_t)L_N * meta->n_layer;
    m->t = (const uint8_t **)calloc(m->n_tensors, sizeof(void *));
    m->dt = (int *)calloc(m->n_tensors, sizeof(int));
    for (size_t i = 0; i < m->n_tensors; ++i) {
        m->t[i] = (const uint8_t *)tensors[i];
        m->dt[i] = dtypes[i];
    }
    size_t stride = (size_t)meta->n_head_kv * meta->head_dim;
    size_t per_layer = (size_t)meta->n_ctx * stride;
    m->k = (float *)calloc(per_layer * meta->n_layer, sizeof(float));
    m->v = (float *)calloc(per_layer * meta->n_layer, sizeof(float));
    return m;
}

void vo_model_free(vo_model *m) {
    if (!m) return;
    free(m->t);
    free(m->dt);
    free(m->k);
    free(m->v);
    free(m->tk);
    free(m->tv);
    free(m);
}

size_t vo_model_kv_pos(const vo_model *m) { return m->pos; }
void vo_model_set_kv_pos(vo_model *m, size_t pos) { m->pos = pos; }

static const uint8_t *T(const vo_model *m, size_t i) { return m->t[i]; }
static int DT(const vo_model *m, size_t i) { return m->dt[i]; }
static size_t LT(size_t l, int which) { return T_LAYER0 + (size_t)L_N * l + (size_t)which; }

/* The source of the keys/values one token attends to. */
typedef struct {
    size_t n_prefix;          /* cached positions [0, n_prefix) */
    const int32_t *path;      /* tree nodes appended after the prefix */
    size_t path_len;
} kv_view;

/* One token through the network (llama_cpu.rs:191-358).  `store` writes the
 * token's K/V either into the cache at `pos` (tree_node < 0) or into the tree
 * scratch row `tree_node`; `view` lists what the token attends to. */
static int forward_token(vo_model *m, uint32_t token, size_t pos, long tree_node,
                         const kv_view *view, float *logits) {
    const vo_meta *mt = &m->meta;
    size_t n_embd = mt->n_embd, n_head = mt->n_head, n_kv = mt->n_head_kv;
    size_t hd = mt->head_dim, n_ff = mt->n_ff, n_vocab = mt->n_vocab;
    size_t kv_stride = n_kv * hd;
    if (token >= n_vocab) return 1;

    float *x = (float *)calloc(n_embd, sizeof(float));
    float *xb = (float *)calloc(n_embd, sizeof(float));
    float *q = (float *)calloc(n_head * hd, sizeof(float));
    float *kk = (float *)calloc(kv_stride, sizeof(float));
    float *vv = (float *)calloc(kv_stride, sizeof(float));
    float *att = (float *)calloc(n_head * hd, sizeof(float));
    float *xo = (float *)calloc(n_embd, sizeof(float));
    float *gate = (float *)calloc(n_ff, sizeof(float));
    float *up = (float *)calloc(n_ff, sizeof(float));
    size_t n_seq = view->n_prefix + view->path_len;
    float *scores = (float *)calloc(n_seq ? n_seq : 1, sizeof(float));
    float *normw = (float *)calloc(n_embd, sizeof(float));

    /* embedding row (llama_cpu.rs:207-212) */
    size_t erb = vo_row_bytes(DT(m, T_EMBD), n_embd);
    vo_dequant_row(DT(m, T_EMBD), T(m, T_EMBD) + (size_t)token * erb, x, n_embd);

    for (size_t l = 0; l < mt->n_layer; ++l) {
        vo_dequant_row(DT(m, LT(l, L_ANORM)), T(m, LT(l, L_ANORM)), normw, n_embd);
        memcpy(xb, x, n_embd * sizeof(float));
        vo_rms_norm(xb, normw, n_embd, mt->norm_eps);

        memset(q, 0, n_head * hd * sizeof(float));
        memset(kk, 0, kv_stride * sizeof(float));
        memset(vv, 0, kv_stride * sizeof(float));
        vo_matvec_quant(q, T(m, LT(l, L_WQ)), DT(m, LT(l, L_WQ)), xb, n_head * hd, n_embd);
        vo_matvec_quant(kk, T(m, LT(l, L_WK)), DT(m, LT(l, L_WK)), xb, kv_stride, n_embd);
        vo_matvec_quant(vv, T(m, LT(l, L_WV)), DT(m, LT(l, L_WV)), xb, kv_stride, n_embd);

        vo_rope(q, kk, pos, n_head, n_kv, hd, mt->rope_freq_base);

        /* store KV (llama_cpu.rs:252) */
        float *kdst, *vdst;
        if (tree_node < 0) {
            kdst = m->k + ((size_t)l * mt->n_ctx + pos) * kv_stride;
            vdst = m->v + ((size_t)l * mt->n_ctx + pos) * kv_stride;
        } else {
            kdst = m->tk + ((size_t)l * m->tree_cap + (size_t)tree_node) * kv_stride;
            vdst = m->tv + ((size_t)l * m->tree_cap + (size_t)tree_node) * kv_stride;
        }
        memcpy(kdst, kk, kv_stride * sizeof(float));
        memcpy(vdst, vv, kv_stride * sizeof(float));

        /* GQA attention (llama_cpu.rs:255-284) */
        memset(att, 0, n_head * hd * sizeof(float));
        for (size_t h = 0; h < n_head; ++h) {
            size_t kvh = h * n_kv / n_head;
            const float *qh = q + h * hd;
            for (size_t t = 0; t < n_seq; ++t) {
                const float *kt;
                if (t < view->n_prefix)
                    kt = m->k + ((size_t)l * mt->n_ctx + t) * kv_stride + kvh * hd;
                else
                    kt = m->tk + ((size_t)l * m->tree_cap +
                                  (size_t)view->path[t - view->n_prefix]) * kv_stride + kvh * hd;
                float dot = 0.0f;
                for (size_t d = 0; d < hd; ++d) dot += qh[d] * kt[d];
                scores[t] = dot / sqrtf((float)hd);
            }
            vo_softmax(scores, n_seq);
            float *oh = att + h * hd;
            for (size_t t = 0; t < n_seq; ++t) {
                const float *vt;
                if (t < view->n_prefix)
                    vt = m->v + ((size_t)l * mt->n_ctx + t) * kv_stride + kvh * hd;
                else
                    vt = m->tv + ((size_t)l * m->tree_cap +
                                  (size_t)view->path[t - view->n_prefix]) * kv_stride + kvh * hd;
                float s = scores[t];
                for (size_t d = 0; d < hd; ++d) oh[d] += s * vt[d];
            }
        }

        /* wo + residual (llama_cpu.rs:287-297) */
        memset(xo, 0, n_embd * sizeof(float));
        vo_matvec_quant(xo, T(m, LT(l, L_WO)), DT(m, LT(l, L_WO)), att, n_embd, n_head * hd);
        for (size_t i = 0; i < n_embd; ++i) x[i] += xo[i];

        /* FFN (llama_cpu.rs:300-335) */
        vo_dequant_row(DT(m, LT(l, L_FNORM)), T(m, LT(l, L_FNORM)), normw, n_embd);
        memcpy(xb, x, n_embd * sizeof(float));
        vo_rms_norm(xb, normw, n_embd, mt->norm_eps);
        memset(gate, 0, n_ff * sizeof(float));
        memset(up, 0, n_ff * sizeof(float));
        vo_matvec_quant(gate, T(m, LT(l, L_W1)), DT(m, LT(l, L_W1)), xb, n_ff, n_embd);
        vo_matvec_quant(up, T(m, LT(l, L_W3)), DT(m, LT(l, L_W3)), xb, n_ff, n_embd);
        for (size_t i = 0; i < n_ff; ++i) gate[i] = vo_silu(gate[i]) * up[i];
        memset(xo, 0, n_embd * sizeof(float));
        vo_matvec_quant(xo, T(m, LT(l, L_W2)), DT(m, LT(l, L_W2)), gate, n_embd, n_ff);
        for (size_t i = 0; i < n_embd; ++i) x[i] += xo[i];
    }

    /* output head (llama_cpu.rs:339-355), tied fallback to token_embd */
    vo_dequant_row(DT(m, T_ONORM), T(m, T_ONORM), normw, n_embd);
    vo_rms_norm(x, normw, n_embd, mt->norm_eps);
    size_t head = T(m, T_OUT) ? T_OUT : T_EMBD;
    memset(logits, 0, n_vocab * sizeof(float));
    vo_matvec_quant(logits, T(m, head), DT(m, head), x, n_vocab, n_embd);

    free(x); free(xb); free(q); free(kk); free(vv); free(att); free(xo);
    free(gate); free(up); free(scores); free(normw);
    return 0;
}

int vo_forward_one(vo_model *m, uint32_t token, size_t pos, float *logits) {
    if (pos >= m->meta.n_ctx) return 1;
    kv_view view = {pos + 1, NULL, 0};
    return forward_token(m, token, pos, -1, &view, logits);
}

int vo_forward_sequence(vo_model *m, const uint32_t *tokens, size_t n,
                        float *last_logits) {
    size_t start = m->pos;
    for (size_t i = 0; i < n; ++i) {
        int rc = vo_forward_one(m, tokens[i], start + i, last_logits);
        if (rc) return rc;
    }
    m->pos += n;
    return 0;
}

int vo_verify_tree(vo_model *m, const uint32_t *tokens, const int32_t *parents,
                   size_t n_nodes, size_t n_cached, float *logits) {
    const vo_meta *mt = &m->meta;
    if (n_nodes == 0 || parents[0] != -1) return 1;
    for (size_t n = 1; n < n_nodes; ++n)
        if (parents[n] < 0 || (size_t)parents[n] >= n) return 1;
    size_t kv_stride = (size_t)mt->n_head_kv * mt->head_dim;
    if (m->tree_cap < n_nodes) {
        free(m->tk);
        free(m->tv);
        m->tree_cap = n_nodes;
        m->tk = (float *)calloc(m->tree_cap * mt->n_layer * kv_stride, sizeof(float));
        m->tv = (float *)calloc(m->tree_cap * mt->n_layer * kv_stride, sizeof(float));
    }
    int32_t *path = (int32_t *)malloc(n_nodes * sizeof(int32_t));
    for (size_t n = 0; n < n_nodes; ++n) {
        size_t depth = 0;
        for (int32_t c = (int32_t)n; c >= 0; c = parents[c]) ++depth;
        /* path root..n */
        size_t i = depth;
        for (int32_t c = (int32_t)n; c >= 0; c = parents[c]) path[--i] = c;
        size_t pos = n_cached + depth - 1;
        if (pos >= mt->n_ctx) { free(path); return 1; }
        kv_view view = {n_cached, path, depth};
        int rc = forward_token(m, tokens[n], pos, (long)n, &view,
                               logits + n * (size_t)mt->n_vocab);
        if (rc) { free(path); return rc; }
    }
    free(path);
    return 0;
}

int vo_commit_path(vo_model *m, const int32_t *path, size_t len, size_t n_cached) {
    const vo_meta *mt = &m->meta;
    size_t kv_stride = (size_t)mt->n_head_kv * mt->head_dim;
    if (n_cached + len > mt->n_ctx) return 1;
    for (size_t l = 0; l < mt->n_layer; ++l)
        for (size_t i = 0; i < len; ++i) {
            size_t node = (size_t)path[i];
            memcpy(m->k + ((size_t)l * mt->n_ctx + n_cached + i) * kv_stride,
                   m->tk + ((size_t)l * m->tree_cap + node) * kv_stride,
                   kv_stride * sizeof(float));
            memcpy(m->v + ((size_t)l * mt->n_ctx + n_cached + i) * kv_stride,
                   m->tv + ((size_t)l * m->tree_cap + node) * kv_stride,
                   kv_stride * sizeof(float));
        }
    m->pos = n_cached + len;
    return 0;
}

/* Test setup: place n cached rows (positions pos0..) of one layer in the
 * KvCache, as a prefill would have left them. */
int vo_write_kv(vo_model *m, int which, size_t layer, size_t pos0, size_t n, const float *src) {
    const vo_meta *mt = &m->meta;
    size_t kv_stride = (size_t)mt->n_head_kv * mt->head_dim;
    if (layer >= mt->n_layer || pos0 + n > mt->n_ctx) return 1;
    float *dst = (which == 0 ? m->k : m->v) + ((size_t)layer * mt->n_ctx + pos0) * kv_stride;
    memcpy(dst, src, n * kv_stride * sizeof(float));
    return 0;
}

int vo_read_kv(const vo_model *m, int which, size_t layer, size_t n, float *out) {
    const vo_meta *mt = &m->meta;
    size_t kv_stride = (size_t)mt->n_head_kv * mt->head_dim;
    if (layer >= mt->n_layer || n > mt->n_ctx) return 1;
    const float *src = (which == 0 ? m->k : m->v) + (size_t)layer * mt->n_ctx * kv_stride;
    memcpy(out, src, n * kv_stride * sizeof(float));
    return 0;
}

/* ------------------------------------------------------------------ */
/* sampling.rs:39-58 GreedySampler                                     */
/* ------------------------------------------------------------------ */
uint32_t vo_greedy(const float *logits, size_t n, const uint8_t *mask,
                   float *confidence) {
    float max_logit = -INFINITY;
    uint32_t max_token = 0;
    for (size_t i = 0; i < n; ++i) {
        if (mask && !mask[i]) continue;
        if (logits[i] >= max_logit) { /* last maximal index wins; NaN skipped */
            max_logit = logits[i];
            max_token = (uint32_t)i;
        }
    }
    if (confidence) *confidence = max_logit;
    return max_token;
}

/* ------------------------------------------------------------------ */
/* speculative.rs:97-129 SpeculativeTree::find_best_path               */
/* ------------------------------------------------------------------ */
size_t vo_find_best_path(const int32_t *parents, const uint32_t *tokens,
                         const uint32_t *expected, size_t n, int32_t *path_out,
                         uint32_t *bonus) {
    if (n == 0) return 0;
    uint8_t *valid = (uint8_t *)calloc(n, 1);
    valid[0] = 1;
    for (size_t i = 1; i < n; ++i) {
        int32_t p = parents[i];
        if (p >= 0 && (size_t)p < n && valid[p] && tokens[i] == expected[p]) valid[i] = 1;
    }
    size_t max_len = 0, best = 0;
    for (size_t i = 0; i < n; ++i) {
        if (!valid[i]) continue;
        size_t len = 0;
        for (int32_t c = (int32_t)i; c >= 0; c = parents[c]) ++len;
        if (len >= max_len) { max_len = len; best = i; }
    }
    size_t k = max_len;
    for (int32_t c = (int32_t)best; c >= 0; c = parents[c]) path_out[--k] = c;
    if (bonus) *bonus = expected[best];
    free(valid);
    return max_len;
}

/* ------------------------------------------------------------------ */
/* Acceptance spec (no reference implementation; Leviathan et al.     */
/* 2023, Chen et al. 2023).  The arithmetic order below IS the spec   */
/* that the CUDA kernel implements; every operation is one IEEE-754   */
/* binary32 operation with round-to-nearest-even.                     */
/* ------------------------------------------------------------------ */

/* Exponential: Cody & Waite (1980) two-constant argument reduction
 * x = k ln2 + r, |r| <= ln2/2, then the degree-6 Taylor polynomial of e^r in
 * Horner form, scaled by 2^k built from the exponent bits.  Constants:
 *   LN2_HI = 45426/65536 = 0.693145751953125 (15 significant bits, so k*LN2_HI
 *            is exact for |k| < 512), LN2_LO = ln2 - LN2_HI rounded to float,
 *   ROUND  = 1.5*2^23: fma(y, log2e, ROUND) rounds y*log2(e) to an integer k
 *            held in the low mantissa bits; (bits(t) << 23) + bits(1.0f) is
 *            then the bit pattern of 2^k.
 * The input is clamped below at -87 so 2^k stays a normal float (NaN maps to
 * -87); the domain is y <= 88 (every use has y <= 0 up to one rounding).
 * Max relative error vs e^y is below 3e-7 (tests check it). */
#define SPEC_LOG2E 1.44269504088896341f
#define SPEC_LN2_HI 0.693145751953125f
#define SPEC_LN2_LO 1.42860682030941723e-6f
#define SPEC_ROUND 12582912.0f

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float vo_spec_exp(float y) {
    y = fmaxf(y, -87.0f);
    float t = fmaf(y, SPEC_LOG2E, SPEC_ROUND);
    float kf = t + (-SPEC_ROUND);
    float r = fmaf(kf, -SPEC_LN2_HI, y);
    r = fmaf(kf, -SPEC_LN2_LO, r);
    float p = fmaf(1.38888888888888889e-3f, r, 8.33333333333333333e-3f); /* 1/720, 1/120 */
    p = fmaf(p, r, 4.16666666666666667e-2f); /* 1/24 */
    p = fmaf(p, r, 1.66666666666666667e-1f); /* 1/6  */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return p * u2f((f2u(t) << 23) + 0x3F800000u);
}

/* Vocabulary enumeration of the spec: tiles of 1024 elements; in tile t,
 * lane l (0..31) owns e = 1024t + 128i + 4l + c for i = 0..7, c = 0..3
 * (the order a warp reads with 16-byte loads).  Elements >= V are absent. */
#define SPEC_TILE 1024
static inline int spec_elem(int t, int l, int i, int c) {
    return SPEC_TILE * t + 128 * i + 4 * l + c;
}

/* warp butterfly: for off in 16,8,4,2,1: v[l] = v[l] + v[l ^ off]; v[0] */
static float butterfly32(const float *lane) {
    float v[32], nv[32];
    memcpy(v, lane, sizeof(v));
    for (int off = 16; off >= 1; off >>= 1) {
        for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
        memcpy(v, nv, sizeof(v));
    }
    return v[0];
}

/* lane value = (acc0 + acc1) + (acc2 + acc3), acc_c = sequential over i */
static float lane_combine(const float *acc) {
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

/* Tile statistics: m_t = rn(max x * inv_t); z_t = butterfly of lane sums of
 * E(fma(x, inv_t, -m_t)). */
static void tile_stats(const float *row, int V, float inv_t, int t, float *mt,
                       float *zt) {
    float mx = -INFINITY;
    for (int l = 0; l < 32; ++l)
        for (int i = 0; i < 8; ++i)
            for (int c = 0; c < 4; ++c) {
                int e = spec_elem(t, l, i, c);
                if (e < V) mx = fmaxf(mx, row[e]);
            }
    float m = mx * inv_t;
    float lanes[32];
    for (int l = 0; l < 32; ++l) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int i = 0; i < 8; ++i)
            for (int c = 0; c < 4; ++c) {
                int e = spec_elem(t, l, i, c);
                if (e < V) acc[c] = acc[c] + vo_spec_exp(fmaf(row[e], inv_t, -m));
            }
        lanes[l] = lane_combine(acc);
    }
    *mt = m;
    *zt = butterfly32(lanes);
}

/* Row statistics: M = max_t m_t; Z = fma-chain over tiles in order of
 * z_t * E(m_t - M). */
void vo_row_stats(const float *row, int V, float inv_t, float *M, float *Z) {
    int nt = (V + SPEC_TILE - 1) / SPEC_TILE;
    float *m = (float *)malloc(sizeof(float) * nt);
    float *z = (float *)malloc(sizeof(float) * nt);
    float mm = -INFINITY;
    for (int t = 0; t < nt; ++t) {
        tile_stats(row, V, inv_t, t, &m[t], &z[t]);
        mm = fmaxf(mm, m[t]);
    }
    float zz = 0.0f;
    for (int t = 0; t < nt; ++t) zz = fmaf(z[t], vo_spec_exp(m[t] - mm), zz);
    *M = mm;
    *Z = zz;
    free(m);
    free(z);
}

/* weight of element e for the sampling pass */
typedef struct {
    const float *trow, *drow; /* drow NULL => weight = P */
    float inv_t, Mt, Rt, Md, Rd;
} wctx;

static inline float spec_weight(const wctx *w, int e) {
    float P = vo_spec_exp(fmaf(w->trow[e], w->inv_t, -w->Mt)) * w->Rt;
    if (!w->drow) return P;
    float Q = vo_spec_exp(fmaf(w->drow[e], w->inv_t, -w->Md)) * w->Rd;
    return P > Q ? P - Q : 0.0f;
}

/* Sequential selection rule used at every level: the first child whose
 * running sum exceeds tau (and whose weight is positive); fallback to the
 * last positive child with tau' = its weight. Returns -1 if all are zero. */
static int select_level(const float *wts, int n, float tau, float *tau_out) {
    float acc = 0.0f;
    int last = -1;
    for (int i = 0; i < n; ++i) {
        float nxt = acc + wts[i];
        if (wts[i] > 0.0f) {
            last = i;
            if (nxt > tau) {
                *tau_out = tau - acc;
                return i;
            }
        }
        acc = nxt;
    }
    if (last >= 0) *tau_out = wts[last];
    return last;
}

/* Inverse-CDF draw from the spec weights; returns the token. */
static int spec_sample(const wctx *w, int V, float u, int *zero_total) {
    int nt = (V + SPEC_TILE - 1) / SPEC_TILE;
    float *lane_w = (float *)malloc(sizeof(float) * nt * 32);
    float *tile_w = (float *)malloc(sizeof(float) * nt);
    float total = 0.0f;
    for (int t = 0; t < nt; ++t) {
        for (int l = 0; l < 32; ++l) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int i = 0; i < 8; ++i)
                for (int c = 0; c < 4; ++c) {
                    int e = spec_elem(t, l, i, c);
                    if (e < V) acc[c] = acc[c] + spec_weight(w, e);
                }
            lane_w[t * 32 + l] = lane_combine(acc);
        }
        tile_w[t] = butterfly32(&lane_w[t * 32]);
        total = total + tile_w[t];
    }
    int tok = 0;
    *zero_total = !(total > 0.0f);
    if (!*zero_total) {
        float tau = u * total, tau1 = 0.0f, tau2 = 0.0f, tau3 = 0.0f;
        int ts = select_level(tile_w, nt, tau, &tau1);
        int ls = select_level(&lane_w[ts * 32], 32, tau1, &tau2);
        float ew[32];
        int eidx[32];
        int n = 0;
        for (int i = 0; i < 8; ++i)
            for (int c = 0; c < 4; ++c) {
                int e = spec_elem(ts, ls, i, c);
                ew[n] = e < V ? spec_weight(w, e) : 0.0f;
                eidx[n] = e;
                ++n;
            }
        int es = select_level(ew, 32, tau2, &tau3);
        tok = eidx[es];
    }
    free(lane_w);
    free(tile_w);
    return tok;
}

static void accept_one(const float *tgt, const float *drf, const uint32_t *tok,
                       const float *u, int k, int V, float temperature,
                       int32_t *acc_len, uint32_t *bonus) {
    size_t Vs = (size_t)V;
    if (temperature == 0.0f) {
        /* greedy: sampling.rs:39-58 per row, prefix rule speculative.rs:441-467 */
        int r = k;
        for (int i = 0; i < k; ++i) {
            uint32_t g = vo_greedy(tgt + (size_t)i * Vs, Vs, NULL, NULL);
            if (tok[i] != g) { r = i; break; }
        }
        *acc_len = r;
        *bonus = vo_greedy(tgt + (size_t)r * Vs, Vs, NULL, NULL);
        return;
    }
    float inv_t = 1.0f / temperature;
    float *Mt = (float *)malloc(sizeof(float) * (k + 1));
    float *Rt = (float *)malloc(sizeof(float) * (k + 1));
    float *Md = (float *)malloc(sizeof(float) * (k + 1));
    float *Rd = (float *)malloc(sizeof(float) * (k + 1));
    for (int i = 0; i <= k; ++i) {
        float Z;
        vo_row_stats(tgt + (size_t)i * Vs, V, inv_t, &Mt[i], &Z);
        Rt[i] = 1.0f / Z;
    }
    for (int i = 0; i < k; ++i) {
        float Z;
        vo_row_stats(drf + (size_t)i * Vs, V, inv_t, &Md[i], &Z);
        Rd[i] = 1.0f / Z;
    }
    int r = k;
    for (int i = 0; i < k; ++i) {
        uint32_t x = tok[i];
        float p = vo_spec_exp(fmaf(tgt[(size_t)i * Vs + x], inv_t, -Mt[i])) * Rt[i];
        float q = vo_spec_exp(fmaf(drf[(size_t)i * Vs + x], inv_t, -Md[i])) * Rd[i];
        if (!(u[i] * q <= p)) { r = i; break; }
    }
    wctx w;
    w.inv_t = inv_t;
    w.trow = tgt + (size_t)r * Vs;
    w.Mt = Mt[r];
    w.Rt = Rt[r];
    w.drow = r < k ? drf + (size_t)r * Vs : NULL;
    w.Md = r < k ? Md[r] : 0.0f;
    w.Rd = r < k ? Rd[r] : 0.0f;
    int zero;
    int t = spec_sample(&w, V, u[k], &zero);
    if (zero) { /* residual mass vanished: draw from p of the same row */
        w.drow = NULL;
        t = spec_sample(&w, V, u[k], &zero);
    }
    *acc_len = r;
    *bonus = (uint32_t)t;
    free(Mt); free(Rt); free(Md); free(Rd);
}

typedef struct {
    const float *tgt, *drf; const uint32_t *tok; const float *u;
    int B, k, V; float temperature; int32_t *acc_len; uint32_t *bonus;
    int next; pthread_mutex_t mu;
} accept_job;

static void *accept_worker(void *arg) {
    accept_job *j = (accept_job *)arg;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        int b = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (b >= j->B) break;
        size_t V = (size_t)j->V, k = (size_t)j->k;
        accept_one(j->tgt + (size_t)b * (k + 1) * V,
                   j->drf ? j->drf + (size_t)b * k * V : NULL, j->tok + (size_t)b * k,
                   j->u + (size_t)b * (k + 1), j->k, j->V, j->temperature,
                   &j->acc_len[b], &j->bonus[b]);
    }
    return NULL;
}

int vo_accept(const float *tgt, const float *drf, const uint32_t *tok,
              const float *u, int B, int k, int V, float temperature,
              int32_t *acc_len, uint32_t *bonus, int n_threads) {
    if (B < 0 || k < 0 || V <= 0 || !(temperature >= 0.0f)) return 1;
    for (long b = 0; b < (long)B * k; ++b)
        if (tok[b] >= (uint32_t)V) return 1;
    if (n_threads <= 0) n_threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (n_threads < 1) n_threads = 1;
    if (n_threads > B) n_threads = B > 0 ? B : 1;
    accept_job j = {tgt, drf, tok, u, B, k, V, temperature, acc_len, bonus, 0,
                    PTHREAD_MUTEX_INITIALIZER};
    pthread_t th[256];
    if (n_threads > 256) n_threads = 256;
    for (int i = 1; i < n_threads; ++i) pthread_create(&th[i], NULL, accept_worker, &j);
    accept_worker(&j);
    for (int i = 1; i < n_threads; ++i) pthread_join(th[i], NULL);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Rejection sampling over a draft tree.  No reference implementation  */
/* (velo-core verifies trees greedily, speculative.rs:97-129); the     */
/* method is multi-candidate speculative sampling (SpecInfer, Miao et  */
/* al. 2024, Algorithm 2): walk from the root; at node n test its      */
/* children in index order against the target distribution p_n and    */
/* the draft distribution q_n the children were drawn from; after each */
/* rejected child replace p by norm(max(0, p - q)); move to the first  */
/* accepted child; at a node where no child is accepted (or a leaf)    */
/* draw the bonus token from the current distribution.  For chains it  */
/* is the acceptance rule above, bit for bit.                           */
/* Arithmetic (the spec the CUDA kernel implements):                    */
/*   P0(x) = E(fma(t_x, 1/T, -Mt)) * Rt, Q(x) = E(fma(d_x, 1/T, -Md)) * Rd */
/*   W_1 = P0 > Q ? P0 - Q : 0;  W_{j+1} = P_j > Q ? P_j - Q : 0 with    */
/*   P_j = W_j * R_j, R_j = 1 / total_j, total_j = the spec's ordered sum */
/*   of W_j over the vocabulary (tiles, lanes, butterfly as above).     */
/*   Child c (parent n) at level j is accepted iff u[c-1] * Q(x_c) <= P_j */
/*   (P_0 = P0).  A level whose total is 0 falls back to level 0 (p).   */
/*   The draw uses u[N-1] and the weights of the final level.           */
/* ------------------------------------------------------------------ */
#define TREE_MAX_LEVEL 64
typedef struct {
    const float *trow, *drow;
    float inv_t, Mt, Rt, Md, Rd;
    int level;
    float R[TREE_MAX_LEVEL + 1];
} tree_w;

/* W_level of element e (level 0: P0) */
static inline float tree_weight(const tree_w *w, int e) {
    float P = vo_spec_exp(fmaf(w->trow[e], w->inv_t, -w->Mt)) * w->Rt;
    if (w->level == 0) return P;
    float Q = vo_spec_exp(fmaf(w->drow[e], w->inv_t, -w->Md)) * w->Rd;
    float W = 0.0f;
    for (int j = 1; j <= w->level; ++j) {
        W = P > Q ? P - Q : 0.0f;
        if (j < w->level) P = W * w->R[j];
    }
    return W;
}

/* lane / tile weights and their ordered total for the current level */
static float tree_weigh(const tree_w *w, int V, float *lane_w, float *tile_w) {
    int nt = (V + SPEC_TILE - 1) / SPEC_TILE;
    float total = 0.0f;
    for (int t = 0; t < nt; ++t) {
        for (int l = 0; l < 32; ++l) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int i = 0; i < 8; ++i)
                for (int c = 0; c < 4; ++c) {
                    int e = spec_elem(t, l, i, c);
                    if (e < V) acc[c] = acc[c] + tree_weight(w, e);
                }
            lane_w[t * 32 + l] = lane_combine(acc);
        }
        tile_w[t] = butterfly32(&lane_w[t * 32]);
        total = total + tile_w[t];
    }
    return total;
}

static void accept_tree_one(const float *tgt, const float *drf, const uint32_t *tok,
                            const int32_t *par, const float *u, int N, int V,
                            float temperature, int32_t *path, int32_t *plen,
                            uint32_t *bonus) {
    size_t Vs = (size_t)V;
    int nt = (V + SPEC_TILE - 1) / SPEC_TILE;
    float *lane_w = (float *)malloc(sizeof(float) * nt * 32);
    float *tile_w = (float *)malloc(sizeof(float) * nt);
    for (int n = 0; n < N; ++n) path[n] = -1;
    int cur = 0, len = 0;
    path[len++] = 0;
    tree_w w;
    memset(&w, 0, sizeof(w));
    w.inv_t = 1.0f / temperature;
    for (;;) {
        float Z;
        w.trow = tgt + (size_t)cur * Vs;
        vo_row_stats(w.trow, V, w.inv_t, &w.Mt, &Z);
        w.Rt = 1.0f / Z;
        int has_child = 0;
        for (int c = cur + 1; c < N; ++c) has_child |= par[c] == cur;
        w.drow = NULL;
        if (has_child) {
            w.drow = drf + (size_t)cur * Vs;
            vo_row_stats(w.drow, V, w.inv_t, &w.Md, &Z);
            w.Rd = 1.0f / Z;
        }
        w.level = 0;
        int accepted = -1;
        for (int c = cur + 1; c < N && accepted < 0; ++c) {
            if (par[c] != cur) continue;
            uint32_t x = tok[c];
            float P;
            if (w.level == 0) {
                P = tree_weight(&w, (int)x);
            } else {
                P = tree_weight(&w, (int)x) * w.R[w.level];
            }
            float Q = vo_spec_exp(fmaf(w.drow[x], w.inv_t, -w.Md)) * w.Rd;
            if (u[c - 1] * Q <= P) {
                accepted = c;
                break;
            }
            if (w.level == TREE_MAX_LEVEL) continue; /* cannot happen: <= 63 children */
            w.level += 1;
            float total = tree_weigh(&w, V, lane_w, tile_w);
            if (!(total > 0.0f))
                w.level = 0; /* residual mass vanished: back to p */
            else
                w.R[w.level] = 1.0f / total;
        }
        if (accepted >= 0) {
            path[len++] = accepted;
            cur = accepted;
            continue;
        }
        /* draw from the final level's weights */
        float total = tree_weigh(&w, V, lane_w, tile_w);
        int token = 0;
        if (total > 0.0f) {
            float tau = u[N - 1] * total, tau1 = 0.0f, tau2 = 0.0f, tau3 = 0.0f;
            int ts = select_level(tile_w, nt, tau, &tau1);
            int ls = select_level(&lane_w[ts * 32], 32, tau1, &tau2);
            float ew[32];
            int eidx[32], n = 0;
            for (int i = 0; i < 8; ++i)
                for (int c = 0; c < 4; ++c) {
                    int e = spec_elem(ts, ls, i, c);
                    ew[n] = e < V ? tree_weight(&w, e) : 0.0f;
                    eidx[n] = e;
                    ++n;
                }
            int es = select_level(ew, 32, tau2, &tau3);
            token = eidx[es];
        }
        *bonus = (uint32_t)token;
        break;
    }
    *plen = len;
    free(lane_w);
    free(tile_w);
}

int vo_accept_tree(const float *tgt, const float *drf, const uint32_t *tok,
                   const int32_t *parents, const float *u, int B, int N, int V,
                   float temperature, int32_t *path, int32_t *path_len, uint32_t *bonus) {
    if (B < 0 || N < 1 || N > TREE_MAX_LEVEL || V <= 0 || !(temperature > 0.0f)) return 1;
    for (long b = 0; b < B; ++b) {
        if (parents[b * N] != -1) return 1;
        for (int n = 1; n < N; ++n) {
            int p = parents[b * N + n];
            if (p < 0 || p >= n || tok[b * N + n] >= (uint32_t)V) return 1;
        }
    }
    size_t Vs = (size_t)V, Ns = (size_t)N;
    for (long b = 0; b < B; ++b)
        accept_tree_one(tgt + (size_t)b * Ns * Vs, drf + (size_t)b * (Ns - 1) * Vs,
                        tok + (size_t)b * Ns, parents + (size_t)b * Ns, u + (size_t)b * Ns, N, V,
                        temperature, path + (size_t)b * Ns, &path_len[b], &bonus[b]);
    return 0;
}

/* ------------------------------------------------------------------ */
/* paged_attention.rs:92-211 PagedAttentionBlockManager (FIFO)         */
/* ------------------------------------------------------------------ */
size_t vo_pages_for_tokens(size_t tokens, size_t block_size) {
    return (tokens + block_size - 1) / block_size; /* div_ceil, :150-152 */
}

typedef struct { uint64_t handle; uint32_t *pages; size_t n; } vo_mapping;
struct vo_allocator {
    size_t block_size, total;
    uint32_t *ring; size_t head, count; /* FIFO of free page ids */
    vo_mapping *maps; size_t n_maps;
};

vo_allocator *vo_allocator_new(size_t block_size, size_t total_pages) {
    if (block_size == 0) return NULL; /* InvalidBlockSize, :103-106 */
    vo_allocator *a = (vo_allocator *)calloc(1, sizeof(*a));
    a->block_size = block_size;
    a->total = total_pages;
    a->ring = (uint32_t *)malloc(sizeof(uint32_t) * (total_pages ? total_pages : 1));
    for (size_t i = 0; i < total_pages; ++i) a->ring[i] = (uint32_t)i;
    a->count = total_pages;
    return a;
}

void vo_allocator_free(vo_allocator *a) {
    if (!a) return;
    for (size_t i = 0; i < a->n_maps; ++i) free(a->maps[i].pages);
    free(a->maps);
    free(a->ring);
    free(a);
}

int vo_allocator_allocate(vo_allocator *a, uint64_t handle, size_t token_len,
                          uint32_t *pages_out, size_t *n_pages,
                          size_t *requested, size_t *available) {
    size_t req = vo_pages_for_tokens(token_len, a->block_size);
    if (req > a->count) { /* OutOfPages, :163-169 */
        *requested = req;
        *available = a->count;
        return 1;
    }
    uint32_t *pages = (uint32_t *)malloc(sizeof(uint32_t) * (req ? req : 1));
    for (size_t i = 0; i < req; ++i) {
        pages[i] = a->ring[a->head];
        a->head = (a->head + 1) % a->total;
        a->count--;
        if (pages_out) pages_out[i] = pages[i];
    }
    *n_pages = req;
    /* BTreeMap insert replaces an existing mapping (pages of the old one are
     * not returned to the pool, as in the reference). */
    for (size_t i = 0; i < a->n_maps; ++i)
        if (a->maps[i].handle == handle) {
            free(a->maps[i].pages);
            a->maps[i].pages = pages;
            a->maps[i].n = req;
            return 0;
        }
    a->maps = (vo_mapping *)realloc(a->maps, sizeof(vo_mapping) * (a->n_maps + 1));
    a->maps[a->n_maps].handle = handle;
    a->maps[a->n_maps].pages = pages;
    a->maps[a->n_maps].n = req;
    a->n_maps++;
    return 0;
}

int vo_allocator_release(vo_allocator *a, uint64_t handle) {
    for (size_t i = 0; i < a->n_maps; ++i)
        if (a->maps[i].handle == handle) {
            for (size_t j = 0; j < a->maps[i].n; ++j) { /* push_back, :194-196 */
                a->ring[(a->head + a->count) % a->total] = a->maps[i].pages[j];
                a->count++;
            }
            free(a->maps[i].pages);
            a->maps[i] = a->maps[a->n_maps - 1];
            a->n_maps--;
            return 0;
        }
    return 1; /* UnknownHandle */
}

size_t vo_allocator_free_pages(const vo_allocator *a) { return a->count; }

/* ------------------------------------------------------------------ */
/* Paged tree attention (kernels.metal:512-599 semantics)             */
/* ------------------------------------------------------------------ */
static float kv_elem(int kv_dtype, const void *pool, const uint16_t *scale,
                     size_t page, size_t h, size_t slot, size_t d, size_t n_kv,
                     size_t hd, size_t page_size) {
    size_t row = (page * n_kv + h) * page_size + slot;
    if (kv_dtype == VO_KV_F16)
        return vo_f16_to_f32(((const uint16_t *)pool)[row * hd + d]);
    /* INT8: value * fp16 per-token-per-head scale (kernels.metal:707-711) */
    return (float)((const int8_t *)pool)[row * hd + d] * vo_f16_to_f32(scale[row]);
}

void vo_tree_attention(const float *q, int kv_dtype, const void *k_pool,
                       const void *v_pool, const uint16_t *k_scale,
                       const uint16_t *v_scale, const uint32_t *page_table,
                       size_t n_cached, const uint16_t *k_nodes,
                       const uint16_t *v_nodes, const int32_t *parents,
                       size_t n_nodes, size_t n_head, size_t n_kv, size_t hd,
                       size_t page_size, float *out) {
    size_t group = n_head / n_kv;
    double scale = 1.0 / sqrt((double)hd);
    int32_t *path = (int32_t *)malloc(sizeof(int32_t) * (n_nodes ? n_nodes : 1));
    double *s = (double *)malloc(sizeof(double) * (n_cached + n_nodes + 1));
    double *acc = (double *)malloc(sizeof(double) * hd);
    for (size_t n = 0; n < n_nodes; ++n) {
        size_t depth = 0;
        for (int32_t c = (int32_t)n; c >= 0; c = parents[c]) ++depth;
        size_t i = depth;
        for (int32_t c = (int32_t)n; c >= 0; c = parents[c]) path[--i] = c;
        for (size_t h = 0; h < n_head; ++h) {
            size_t kvh = h / group; /* GQA grouping, kernels.metal:534 */
            const float *qh = q + (n * n_head + h) * hd;
            size_t L = n_cached + depth;
            double mx = -INFINITY;
            for (size_t t = 0; t < L; ++t) {
                double dot = 0.0;
                for (size_t d = 0; d < hd; ++d) {
                    float kv;
                    if (t < n_cached)
                        kv = kv_elem(kv_dtype, k_pool, k_scale, page_table[t / page_size],
                                     kvh, t % page_size, d, n_kv, hd, page_size);
                    else
                        kv = vo_f16_to_f32(k_nodes[((size_t)path[t - n_cached] * n_kv + kvh) * hd + d]);
                    dot += (double)qh[d] * (double)kv;
                }
                s[t] = dot * scale;
                if (s[t] > mx) mx = s[t];
            }
            double z = 0.0;
            for (size_t t = 0; t < L; ++t) { s[t] = exp(s[t] - mx); z += s[t]; }
            for (size_t d = 0; d < hd; ++d) acc[d] = 0.0;
            for (size_t t = 0; t < L; ++t) {
                for (size_t d = 0; d < hd; ++d) {
                    float vv;
                    if (t < n_cached)
                        vv = kv_elem(kv_dtype, v_pool, v_scale, page_table[t / page_size],
                                     kvh, t % page_size, d, n_kv, hd, page_size);
                    else
                        vv = vo_f16_to_f32(v_nodes[((size_t)path[t - n_cached] * n_kv + kvh) * hd + d]);
                    acc[d] += s[t] * (double)vv;
                }
            }
            for (size_t d = 0; d < hd; ++d) out[(n * n_head + h) * hd + d] = (float)(acc[d] / z);
        }
    }
    free(path);
    free(s);
    free(acc);
}

/* kernels.metal:783-801 with an fp16 scale: scale = max/127, q = (int8)(x*inv) */
void vo_quantize_kv_int8(const float *x, size_t hd, int8_t *q, uint16_t *scale) {
    float mx = 0.0f;
    for (size_t d = 0; d < hd; ++d) mx = fmaxf(mx, fabsf(x[d]));
    float sc = mx / 127.0f;
    float inv = mx > 0.0f ? 127.0f / mx : 0.0f;
    for (size_t d = 0; d < hd; ++d) q[d] = (int8_t)(x[d] * inv); /* truncation */
    *scale = vo_f32_to_f16(sc);
}

int vo_kv_commit(int kv_dtype, void *pool, uint16_t *scale,
                 const uint32_t *page_table, size_t n_bound, size_t n_cached,
                 const uint16_t *node_kv, const int32_t *path, size_t len,
                 size_t n_kv, size_t hd, size_t page_size) {
    if (len && (n_cached + len - 1) / page_size >= n_bound) return 5;
    float *tmp = (float *)malloc(sizeof(float) * hd);
    for (size_t i = 0; i < len; ++i) {
        size_t pos = n_cached + i;
        size_t page = page_table[pos / page_size], slot = pos % page_size;
        for (size_t h = 0; h < n_kv; ++h) {
            const uint16_t *src = node_kv + ((size_t)path[i] * n_kv + h) * hd;
            size_t row = (page * n_kv + h) * page_size + slot;
            if (kv_dtype == VO_KV_F16) {
                memcpy((uint16_t *)pool + row * hd, src, hd * 2);
            } else {
                for (size_t d = 0; d < hd; ++d) tmp[d] = vo_f16_to_f32(src[d]);
                vo_quantize_kv_int8(tmp, hd, (int8_t *)pool + row * hd, &scale[row]);
            }
        }
    }
    free(tmp);
    return 0;
}

/* ------------------------------------------------------------------ */
/* sharding.rs:112-126 get_shard_strategy                              */
/* ------------------------------------------------------------------ */
int vo_shard_strategy(const char *name) {
    if (strstr(name, "attention.wq") || strstr(name, "attention.wk") || strstr(name, "attention.wv"))
        return 1;
    if (strstr(name, "attention.wo")) return 2;
    if (strstr(name, "feed_forward.w1") || strstr(name, "feed_forward.w3")) return 1;
    if (strstr(name, "feed_forward.w2")) return 2;
    if (strcmp(name, "output.weight") == 0) return 1;
    return 0;
}

/* sharding.rs:28-110 shard_weight.  The reference's shape is GGUF order
 * [cols, rows]: Column divides shape[last] = rows and takes rows
 * [rank*rows/tp, (rank+1)*rows/tp); Row divides shape[0] = cols, requires the
 * shard width to be a multiple of the quant block, and takes the same byte
 * slice of every row. */
int vo_shard_weight(int dtype, const uint8_t *data, size_t rows, size_t cols, int strategy,
                    int tp, int rank, uint8_t *out, size_t *rows_out, size_t *cols_out) {
    size_t rb = vo_row_bytes(dtype, cols);
    if (tp <= 1 || strategy == 0) {
        memcpy(out, data, rb * rows);
        *rows_out = rows;
        *cols_out = cols;
        return 0;
    }
    if (strategy == 1) {
        if (rows % (size_t)tp) return 1;
        size_t sr = rows / (size_t)tp;
        memcpy(out, data + (size_t)rank * sr * rb, sr * rb);
        *rows_out = sr;
        *cols_out = cols;
        return 0;
    }
    if (cols % (size_t)tp) return 1;
    size_t sc = cols / (size_t)tp, block = dtype == VO_Q4_0 ? 32 : 1;
    if (sc % block) return 1;
    size_t srb = rb / (size_t)tp;
    for (size_t r = 0; r < rows; ++r) memcpy(out + r * srb, data + r * rb + (size_t)rank * srb, srb);
    *rows_out = rows;
    *cols_out = sc;
    return 0;
}
