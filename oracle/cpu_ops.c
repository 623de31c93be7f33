/*
 * oracle/cpu_ops.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * CPU restatement of the Infer-LLM reference CPU backend for the F32 Qwen3 path
 * (the checker for the B200 kernels). See cpu_ops.h for the contract. Build with
 * -ffp-contract=off: the reference's float expressions are evaluated as separate
 * IEEE multiplies and adds, and so is every expression here.
 */
#include "cpu_ops.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_THREADS(nt) ((nt) > 1 ? (nt) : 1)

/* cpu_backend.cpp:406-422: one task per output element, float sum in k order. */
void orc_mul_mat(const float *w, const float *x, float *out,
                 int64_t K, int64_t N, int64_t M, int nthreads) {
    const int64_t total = N * M;
#pragma omp parallel for num_threads(ORC_THREADS(nthreads)) schedule(static)
    for (int64_t i = 0; i < total; ++i) {
        const int64_t token = i / N;
        const int64_t row = i % N;
        const float *xr = x + token * K;
        const float *wr = w + row * K;
        float sum = 0.0f;
        for (int64_t k = 0; k < K; ++k) sum += xr[k] * wr[k];
        out[i] = sum;
    }
}

/* cpu_backend.cpp:361-380: the square is a float product, accumulated in a
 * double; scale = float(1 / sqrt(double mean + eps)); y = (x * scale) * gamma. */
void orc_rms_norm(const float *x, const float *gamma, float *out,
                  int64_t D, int64_t rows, float eps, int nthreads) {
#pragma omp parallel for num_threads(ORC_THREADS(nthreads)) schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * D;
        float *yr = out + r * D;
        double sum = 0.0;
        for (int64_t i = 0; i < D; ++i) {
            const float sq = xr[i] * xr[i];
            sum += sq;
        }
        const float scale = (float)(1.0f / sqrt(sum / (double)D + (double)eps));
        for (int64_t i = 0; i < D; ++i) yr[i] = xr[i] * scale * gamma[i];
    }
}

/* graph.cpp:119-131. powf (the float overload std::pow(float, float) resolves
 * to), the reciprocal in float, widened to double for the position product. */
void orc_rope_theta_table(float theta_base, uint32_t head_dim, uint32_t n_ctx, float *out) {
    const uint32_t half = head_dim / 2;
    double *freq = (double *)malloc(sizeof(double) * (half ? half : 1));
    for (uint32_t i = 0; i < half; ++i) {
        const float expo = 2.0f * (float)i / (float)head_dim;
        freq[i] = (double)(1.0f / powf(theta_base, expo));
    }
    for (uint32_t pos = 0; pos < n_ctx; ++pos) {
        float *row = out + (size_t)pos * half;
        for (uint32_t i = 0; i < half; ++i) row[i] = (float)((double)pos * freq[i]);
    }
    free(freq);
}

/* cpu_backend.cpp:468-521: sinf/cosf per (token, pair) then the half-split
 * rotation (x_j, x_{j+D/2}). */
void orc_rope(const float *x, const int32_t *pos, const float *table, float *out,
              int64_t D, int64_t H, int64_t T, int nthreads) {
    const int64_t half = D / 2;
    float *sinc = (float *)malloc(sizeof(float) * (size_t)(T * half + 1));
    float *cosc = (float *)malloc(sizeof(float) * (size_t)(T * half + 1));
    for (int64_t t = 0; t < T; ++t) {
        const float *row = table + (int64_t)pos[t] * half;
        for (int64_t j = 0; j < half; ++j) {
            sinc[t * half + j] = sinf(row[j]);
            cosc[t * half + j] = cosf(row[j]);
        }
    }
#pragma omp parallel for num_threads(ORC_THREADS(nthreads)) schedule(static)
    for (int64_t i = 0; i < H * T; ++i) {
        const int64_t t = i / H;
        const float *src = x + i * D;
        float *dst = out + i * D;
        const float *s = sinc + t * half;
        const float *c = cosc + t * half;
        for (int64_t j = 0; j < half; ++j) {
            const float x0 = src[j];
            const float x1 = src[half + j];
            const float a = x0 * c[j];
            const float b = x1 * s[j];
            const float e = x0 * s[j];
            const float f = x1 * c[j];
            dst[j] = a - b;
            dst[half + j] = e + f;
        }
    }
    free(sinc);
    free(cosc);
}

/* cpu_backend.cpp:555-632: one task per (query token, query head). */
void orc_flash_attn(const float *q, const float *k, const float *v, float *out,
                    int64_t D, int64_t Hq, int64_t Hkv, int64_t Tq, int64_t Tkv,
                    int64_t n_past, int nthreads) {
    const int64_t group = Hq / Hkv;
    const float scale = 1.0f / sqrtf((float)D);
#pragma omp parallel num_threads(ORC_THREADS(nthreads))
    {
        float *scores = (float *)malloc(sizeof(float) * (size_t)(Tkv > 0 ? Tkv : 1));
#pragma omp for schedule(static)
        for (int64_t i = 0; i < Hq * Tq; ++i) {
            const int64_t qt = i / Hq;
            const int64_t qh = i % Hq;
            const int64_t kvh = qh / group;
            const float *qs = q + i * D;
            float *dst = out + i * D;
            for (int64_t j = 0; j < Tkv; ++j) {
                if (j > n_past + qt) {
                    scores[j] = -INFINITY;
                    continue;
                }
                const float *ks = k + (j * Hkv + kvh) * D;
                float dot = 0.0f;
                for (int64_t d = 0; d < D; ++d) dot += qs[d] * ks[d];
                scores[j] = dot * scale;
            }
            /* std::max_element: the first maximum */
            float mx = Tkv > 0 ? scores[0] : 0.0f;
            for (int64_t j = 1; j < Tkv; ++j)
                if (mx < scores[j]) mx = scores[j];
            float sum = 0.0f;
            for (int64_t j = 0; j < Tkv; ++j) {
                scores[j] = expf(scores[j] - mx);
                sum += scores[j];
            }
            for (int64_t j = 0; j < Tkv; ++j) scores[j] /= sum;
            for (int64_t d = 0; d < D; ++d) dst[d] = 0.0f;
            for (int64_t j = 0; j < Tkv; ++j) {
                const float *vs = v + (j * Hkv + kvh) * D;
                const float wgt = scores[j];
                for (int64_t d = 0; d < D; ++d) {
                    const float p = wgt * vs[d];
                    dst[d] += p;
                }
            }
        }
        free(scores);
    }
}

void orc_silu(const float *x, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] / (1.0f + expf(-x[i]));
}

void orc_mul(const float *a, const float *b, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] * b[i];
}

void orc_add(const float *a, const float *b, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

int orc_get_rows(const float *table, const int32_t *ids, float *out,
                 int64_t D, int64_t n, int64_t n_rows) {
    int rc = 0;
    for (int64_t t = 0; t < n; ++t) {
        if (ids[t] < 0 || ids[t] >= n_rows) {
            rc = -1;
            continue;
        }
        memcpy(out + t * D, table + (int64_t)ids[t] * D, sizeof(float) * (size_t)D);
    }
    return rc;
}

int32_t orc_argmax(const float *logits, int64_t n) {
    float best = -INFINITY;
    int32_t id = -1;
    for (int64_t i = 0; i < n; ++i) {
        const float s = logits[i];
        if (isnan(s) || s == INFINITY) return -1;
        if (s > best) {
            best = s;
            id = (int32_t)i;
        }
    }
    return id;
}

/* ------------------------------------------------------------------------ */

struct orc_qwen3 {
    orc_qwen3_config c;
    const float *tok, *onorm, *out;
    orc_qwen3_layer *layers;
    float *kv;      /* per layer: K [cap][Hkv][D] then V [cap][Hkv][D] */
    float *theta;   /* [n_ctx_train][D/2] */
    int64_t n_past;
};

orc_qwen3 *orc_qwen3_create(const orc_qwen3_config *cfg, const float *token_embd,
                            const float *output_norm, const float *output,
                            const orc_qwen3_layer *layers) {
    orc_qwen3 *m = (orc_qwen3 *)calloc(1, sizeof(orc_qwen3));
    if (!m) return NULL;
    m->c = *cfg;
    m->tok = token_embd;
    m->onorm = output_norm;
    m->out = output ? output : token_embd; /* tied LM head, model.cpp:203-206 */
    m->layers = (orc_qwen3_layer *)malloc(sizeof(orc_qwen3_layer) * (size_t)cfg->n_layer);
    memcpy(m->layers, layers, sizeof(orc_qwen3_layer) * (size_t)cfg->n_layer);
    const size_t per_layer = (size_t)cfg->kv_capacity * cfg->n_head_kv * cfg->head_dim * 2;
    m->kv = (float *)calloc(per_layer * (size_t)cfg->n_layer, sizeof(float));
    m->theta = (float *)malloc(sizeof(float) * (size_t)cfg->n_ctx_train * (cfg->head_dim / 2));
    if (!m->layers || !m->kv || !m->theta) {
        orc_qwen3_destroy(m);
        return NULL;
    }
    orc_rope_theta_table(cfg->rope_theta, (uint32_t)cfg->head_dim, (uint32_t)cfg->n_ctx_train, m->theta);
    return m;
}

void orc_qwen3_destroy(orc_qwen3 *m) {
    if (!m) return;
    free(m->layers);
    free(m->kv);
    free(m->theta);
    free(m);
}

void orc_qwen3_reset(orc_qwen3 *m) { m->n_past = 0; }
int64_t orc_qwen3_n_past(const orc_qwen3 *m) { return m->n_past; }

int orc_qwen3_eval(orc_qwen3 *m, const int32_t *ids, int64_t n, float *logits,
                   int all_rows, int nt) {
    const orc_qwen3_config *c = &m->c;
    const int64_t H = c->n_embd, D = c->head_dim, Hq = c->n_head, Hkv = c->n_head_kv;
    const int64_t F = c->n_ff, V = c->n_vocab, cap = c->kv_capacity;
    const int64_t qd = Hq * D, kd = Hkv * D;
    const int64_t n_past = m->n_past;
    if (n <= 0 || n_past + n > cap || n_past + n > c->n_ctx_train) return -1;
    for (int64_t t = 0; t < n; ++t)
        if (ids[t] < 0 || ids[t] >= V) return -1;

    float *x = (float *)malloc(sizeof(float) * n * H);      /* residual stream */
    float *cur = (float *)malloc(sizeof(float) * n * H);
    float *q = (float *)malloc(sizeof(float) * n * qd);
    float *k = (float *)malloc(sizeof(float) * n * kd);
    float *v = (float *)malloc(sizeof(float) * n * kd);
    float *qn = (float *)malloc(sizeof(float) * n * qd);
    float *kn = (float *)malloc(sizeof(float) * n * kd);
    float *attn = (float *)malloc(sizeof(float) * n * qd);
    float *o = (float *)malloc(sizeof(float) * n * H);
    float *g = (float *)malloc(sizeof(float) * n * F);
    float *u = (float *)malloc(sizeof(float) * n * F);
    float *s = (float *)malloc(sizeof(float) * n * F);
    int32_t *pos = (int32_t *)malloc(sizeof(int32_t) * n);
    for (int64_t t = 0; t < n; ++t) pos[t] = (int32_t)(n_past + t);

    orc_get_rows(m->tok, ids, x, H, n, V);
    const size_t per_layer = (size_t)cap * kd * 2;
    for (int32_t l = 0; l < c->n_layer; ++l) {
        const orc_qwen3_layer *w = &m->layers[l];
        float *kc = m->kv + per_layer * l;
        float *vc = kc + (size_t)cap * kd;
        orc_rms_norm(x, w->attn_norm, cur, H, n, c->rms_eps, nt);
        orc_mul_mat(w->wq, cur, q, H, qd, n, nt);
        orc_mul_mat(w->wk, cur, k, H, kd, n, nt);
        orc_mul_mat(w->wv, cur, v, H, kd, n, nt);
        orc_rms_norm(q, w->q_norm, qn, D, Hq * n, c->rms_eps, nt);
        orc_rms_norm(k, w->k_norm, kn, D, Hkv * n, c->rms_eps, nt);
        orc_rope(qn, pos, m->theta, q, D, Hq, n, nt);                 /* q <- q_rope */
        orc_rope(kn, pos, m->theta, kc + n_past * kd, D, Hkv, n, nt); /* cache write */
        memcpy(vc + n_past * kd, v, sizeof(float) * n * kd);
        orc_flash_attn(q, kc, vc, attn, D, Hq, Hkv, n, n_past + n, n_past, nt);
        orc_mul_mat(w->wo, attn, o, qd, H, n, nt);
        orc_add(o, x, x, n * H);                                       /* ffn_inp */
        orc_rms_norm(x, w->ffn_norm, cur, H, n, c->rms_eps, nt);
        orc_mul_mat(w->ffn_gate, cur, g, H, F, n, nt);
        orc_mul_mat(w->ffn_up, cur, u, H, F, n, nt);
        orc_silu(g, s, n * F);
        orc_mul(u, s, g, n * F);                                       /* g <- ffn_inter */
        orc_mul_mat(w->ffn_down, g, o, F, H, n, nt);
        orc_add(o, x, x, n * H);
    }
    orc_rms_norm(x, m->onorm, cur, H, n, c->rms_eps, nt);
    if (all_rows)
        orc_mul_mat(m->out, cur, logits, H, V, n, nt);
    else
        orc_mul_mat(m->out, cur + (n - 1) * H, logits, H, V, 1, nt);
    m->n_past = n_past + n;

    free(x); free(cur); free(q); free(k); free(v); free(qn); free(kn);
    free(attn); free(o); free(g); free(u); free(s); free(pos);
    return 0;
}
