/*
 * af_oracle.c — CPU restatement of the reference decode path, for TESTS ONLY.
 *
 * This is test infrastructure: only tests/, the smoke check and bench.py's
 * cpu_baseline leg load liboracle.so, and only as the checker.  The product
 * path (llm_core_b200) never calls it and has no CPU fallback.
 *
 * Every function restates the algorithm of songqiuyu/llm_core ("AxonForge")
 * at the cited file:line (paths relative to the reference project root).
 * Parity pin: tests/test_oracle.py checks this file against the reference
 * compiled in place (oracle/_ref/libaxref.so, built by oracle/ref.mk) and
 * against the committed fixtures in tests/golden/ produced from that library by
 * tests/golden/make_golden.py.
 *
 * Numerics: plain fp32 with the reference's expression order inside each dot
 * product row; summation order differs from the AVX2 kernels (8-lane partial
 * sums), so agreement is to ~1e-6 relative, not bit-exact.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK_K 256
#define Q4K_BYTES 144
#define Q6K_BYTES 210
#define GGML_F32 0
#define GGML_Q4_K 12
#define GGML_Q6_K 14

/* f16 -> f32 bit conversion: llama_model.cpp:102-120. */
float afo_f16_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u, exponent = (h >> 10) & 0x1Fu, mantissa = h & 0x3FFu, bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign << 31;
        } else {
            int e = 1;
            while (!(mantissa & 0x400)) { mantissa <<= 1; e--; }
            mantissa &= 0x3FF;
            bits = (sign << 31) | ((uint32_t)(e + 127 - 15) << 23) | (mantissa << 13);
        }
    } else if (exponent == 31) {
        bits = (sign << 31) | 0x7F800000u | (mantissa << 13);
    } else {
        bits = (sign << 31) | ((exponent + 127 - 15) << 23) | (mantissa << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* 6-bit (scale, min) pair j of the 12 packed bytes: llama_model.cpp:464-473,
 * gemv_q4k_avx2.cpp:34-43. */
static void q4k_get_scale_min(int j, const uint8_t* sc, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = sc[j] & 0x3F;
        *m = sc[j + 4] & 0x3F;
    } else {
        *d = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
        *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

/* Dequantise one Q4_K row of `cols` values: emb_lookup Q4_K branch,
 * llama_model.cpp:905-930. */
void afo_q4k_row_to_f32(float* out, const uint8_t* row, int cols) {
    const int nb = cols / QK_K;
    for (int b = 0; b < nb; b++) {
        const uint8_t* block = row + (size_t)b * Q4K_BYTES;
        uint16_t db, mb;
        memcpy(&db, block, 2);
        memcpy(&mb, block + 2, 2);
        const float d = afo_f16_to_f32(db), dmin = afo_f16_to_f32(mb);
        const uint8_t* scales = block + 4;
        const uint8_t* qs = block + 16;
        float* ob = out + (size_t)b * QK_K;
        for (int chunk = 0; chunk < 4; chunk++) {
            uint8_t sc1, m1, sc2, m2;
            q4k_get_scale_min(chunk * 2 + 0, scales, &sc1, &m1);
            q4k_get_scale_min(chunk * 2 + 1, scales, &sc2, &m2);
            const float d1 = d * sc1, mf1 = dmin * m1, d2 = d * sc2, mf2 = dmin * m2;
            const uint8_t* q = qs + chunk * 32;
            float* oc = ob + chunk * 64;
            for (int l = 0; l < 32; l++) {
                oc[l] = d1 * (q[l] & 0xF) - mf1;
                oc[l + 32] = d2 * (q[l] >> 4) - mf2;
            }
        }
    }
}

/* Dot of one Q4_K row with f32 x: q4k_dot_row, llama_model.cpp:476-504. */
float afo_q4k_dot_row(const uint8_t* row, const float* x, int cols) {
    float acc = 0.f;
    const int nb = cols / QK_K;
    for (int b = 0; b < nb; b++) {
        const uint8_t* block = row + (size_t)b * Q4K_BYTES;
        uint16_t db, mb;
        memcpy(&db, block, 2);
        memcpy(&mb, block + 2, 2);
        const float d = afo_f16_to_f32(db), dmin = afo_f16_to_f32(mb);
        const uint8_t* scales = block + 4;
        const uint8_t* qs = block + 16;
        const float* xb = x + (size_t)b * QK_K;
        for (int chunk = 0; chunk < 4; chunk++) {
            uint8_t sc1, m1, sc2, m2;
            q4k_get_scale_min(chunk * 2 + 0, scales, &sc1, &m1);
            q4k_get_scale_min(chunk * 2 + 1, scales, &sc2, &m2);
            const float d1 = d * sc1, mf1 = dmin * m1, d2 = d * sc2, mf2 = dmin * m2;
            const uint8_t* q = qs + chunk * 32;
            const float* xi = xb + chunk * 64;
            for (int l = 0; l < 32; l++) {
                acc += (d1 * (q[l] & 0xF) - mf1) * xi[l];
                acc += (d2 * (q[l] >> 4) - mf2) * xi[l + 32];
            }
        }
    }
    return acc;
}

/* Dequantise one Q6_K row: q6k_row_to_f32, llama_model.cpp:560-592. */
void afo_q6k_row_to_f32(float* out, const uint8_t* row, int cols) {
    const int nb = cols / QK_K;
    for (int b = 0; b < nb; b++) {
        const uint8_t* block = row + (size_t)b * Q6K_BYTES;
        uint16_t db;
        memcpy(&db, block + 208, 2);
        const float d = afo_f16_to_f32(db);
        const uint8_t* ql = block;
        const uint8_t* qh = block + 128;
        const int8_t* sc = (const int8_t*)(block + 192);
        float* y = out + (size_t)b * QK_K;
        for (int n = 0; n < 2; n++) {
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int q1 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l + 0] = d * sc[is + 0] * q1;
                y[l + 32] = d * sc[is + 2] * q2;
                y[l + 64] = d * sc[is + 4] * q3;
                y[l + 96] = d * sc[is + 6] * q4;
            }
            ql += 64;
            qh += 32;
            sc += 8;
            y += 128;
        }
    }
}

/* Dot of one Q6_K row with f32 x: q6k_dot_row, llama_model.cpp:595-629. */
float afo_q6k_dot_row(const uint8_t* row, const float* x, int cols) {
    float acc = 0.f;
    const int nb = cols / QK_K;
    for (int b = 0; b < nb; b++) {
        const uint8_t* block = row + (size_t)b * Q6K_BYTES;
        uint16_t db;
        memcpy(&db, block + 208, 2);
        const float d = afo_f16_to_f32(db);
        const uint8_t* ql = block;
        const uint8_t* qh = block + 128;
        const int8_t* sc = (const int8_t*)(block + 192);
        const float* xp = x + (size_t)b * QK_K;
        for (int n = 0; n < 2; n++) {
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int q1 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                acc += (d * sc[is + 0] * q1) * xp[l + 0];
                acc += (d * sc[is + 2] * q2) * xp[l + 32];
                acc += (d * sc[is + 4] * q3) * xp[l + 64];
                acc += (d * sc[is + 6] * q4) * xp[l + 96];
            }
            ql += 64;
            qh += 32;
            sc += 8;
            xp += 128;
        }
    }
    return acc;
}

static size_t row_bytes_of(int type, int cols) {
    if (type == GGML_Q4_K) return (size_t)(cols / QK_K) * Q4K_BYTES;
    if (type == GGML_Q6_K) return (size_t)(cols / QK_K) * Q6K_BYTES;
    return (size_t)cols * 4;
}

static int g_threads = 1;

/* Number of host threads afo_gemv splits its rows over (default 1). */
void afo_set_threads(int n) { g_threads = n < 1 ? 1 : n; }

typedef struct {
    float* y;
    const uint8_t* W;
    const float* x;
    int type, cols, r0, r1;
    size_t rb;
} gemv_job;

static void* gemv_rows(void* arg) {
    const gemv_job* j = (const gemv_job*)arg;
    for (int o = j->r0; o < j->r1; o++) {
        const uint8_t* row = j->W + (size_t)o * j->rb;
        if (j->type == GGML_Q4_K) {
            j->y[o] = afo_q4k_dot_row(row, j->x, j->cols);
        } else if (j->type == GGML_Q6_K) {
            j->y[o] = afo_q6k_dot_row(row, j->x, j->cols);
        } else {
            const float* r = (const float*)row;
            float acc = 0.f;
            for (int i = 0; i < j->cols; i++) acc += r[i] * j->x[i];
            j->y[o] = acc;
        }
    }
    return NULL;
}

/* y[0:rows] = W·x for a Q4_K / Q6_K / F32 matrix: gemv_wt dtype dispatch,
 * llama_model.cpp:670-730 (F32-activation path).  Rows are split over
 * afo_set_threads() threads like ThreadPool::parallel_for (thread_pool.hpp:61-83). */
void afo_gemv(float* y, const void* W, int type, const float* x, int rows, int cols) {
    const size_t rb = row_bytes_of(type, cols);
    int nt = g_threads;
    if (nt > 64) nt = 64;
    if (rows < 64) nt = 1;
    gemv_job jobs[64];
    pthread_t th[64];
    const int chunk = (rows + nt - 1) / nt;
    for (int t = 0; t < nt; t++) {
        const int r0 = t * chunk, r1 = r0 + chunk < rows ? r0 + chunk : rows;
        gemv_job j = {y, (const uint8_t*)W, x, type, cols, r0 < rows ? r0 : rows, r1, rb};
        jobs[t] = j;
    }
    for (int t = 1; t < nt; t++) pthread_create(&th[t], NULL, gemv_rows, &jobs[t]);
    gemv_rows(&jobs[0]);
    for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
}

/* F32 -> Q8_0 blocks (32 int8 + f32 d): quantize_q8_avx2,
 * src/backend/cpu_x86/kernels/quant_q8_avx2.cpp:33-84.  d = amax/127;
 * q = x·(127/amax) rounded to nearest, ties to even (the default rounding of
 * _mm256_cvtps_epi32, here lrintf), saturated to int8 like the packs. */
void afo_quantize_q8(float* d_out, int8_t* q_out, const float* x, int k) {
    for (int i = 0; i < k / 32; i++) {
        const float* s = x + (size_t)32 * i;
        float amax = 0.f;
        for (int j = 0; j < 32; j++) {
            const float a = fabsf(s[j]);
            if (a > amax) amax = a;
        }
        const float id = amax > 0.f ? 127.f / amax : 0.f;
        d_out[i] = amax / 127.f;
        for (int j = 0; j < 32; j++) {
            long v = lrintf(s[j] * id);
            q_out[(size_t)32 * i + j] = (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v));
        }
    }
}

/* Q4_K row · Q8_0 input, the production decode GEMV's arithmetic
 * (gemv_q4k_r8_avx2.cpp:196-220): per 32-value sub-block j with Q8 block
 * scale dq, (d·sc_j·dq)·Σ q·q8 − (dmin·m_j·dq)·Σ q8, integer sums exact. */
static float q4k_q8_dot_row(const uint8_t* row, const float* xd, const int8_t* xq, int cols) {
    float acc = 0.f;
    for (int b = 0; b < cols / QK_K; b++) {
        const uint8_t* block = row + (size_t)b * Q4K_BYTES;
        uint16_t db, mb;
        memcpy(&db, block, 2);
        memcpy(&mb, block + 2, 2);
        const float d = afo_f16_to_f32(db), dmin = afo_f16_to_f32(mb);
        const uint8_t* qs = block + 16;
        for (int chunk = 0; chunk < 4; chunk++) {
            for (int half = 0; half < 2; half++) {
                const int j = 2 * chunk + half, blk = 8 * b + j;
                uint8_t sc, m;
                q4k_get_scale_min(j, block + 4, &sc, &m);
                const int8_t* q8 = xq + (size_t)32 * blk;
                int dot = 0, sum = 0;
                for (int l = 0; l < 32; l++) {
                    const int q = half ? (qs[32 * chunk + l] >> 4) : (qs[32 * chunk + l] & 0xF);
                    dot += q * q8[l];
                    sum += q8[l];
                }
                acc += (d * sc * xd[blk]) * (float)dot;
                acc -= (dmin * m * xd[blk]) * (float)sum;
            }
        }
    }
    return acc;
}

/* Q6_K row · Q8_0 input: gemv_q6k_q8_avx2.cpp:103 — per 16-value group g,
 * d·sc_g·dq·(Σ q6·q8 − 32·Σ q8), q6 the unsigned 6-bit value. */
static float q6k_q8_dot_row(const uint8_t* row, const float* xd, const int8_t* xq, int cols) {
    float acc = 0.f;
    for (int b = 0; b < cols / QK_K; b++) {
        const uint8_t* block = row + (size_t)b * Q6K_BYTES;
        uint16_t db;
        memcpy(&db, block + 208, 2);
        const float d = afo_f16_to_f32(db);
        const int8_t* sc = (const int8_t*)(block + 192);
        int q6[QK_K];
        for (int n = 0; n < 2; n++) {
            const uint8_t* ql = block + 64 * n;
            const uint8_t* qh = block + 128 + 32 * n;
            for (int l = 0; l < 32; l++) {
                q6[128 * n + l] = (ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4);
                q6[128 * n + l + 32] = (ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4);
                q6[128 * n + l + 64] = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
                q6[128 * n + l + 96] = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
            }
        }
        for (int g = 0; g < 16; g++) {
            const int blk = 8 * b + g / 2;
            const int8_t* q8 = xq + (size_t)QK_K * b + 16 * g;
            int dot = 0, sum = 0;
            for (int l = 0; l < 16; l++) {
                dot += q6[16 * g + l] * q8[l];
                sum += q8[l];
            }
            acc += (d * sc[g] * xd[blk]) * (float)(dot - 32 * sum);
        }
    }
    return acc;
}

/* y = W · Q8_0(x): the reference's production decode GEMV gemv_wt_q8
 * (src/models/llama_model.cpp:767-831) with x quantised as above. */
void afo_gemv_q8(float* y, const void* W, int type, const float* x, int rows, int cols) {
    const size_t rb = row_bytes_of(type, cols);
    float* xd = (float*)malloc(sizeof(float) * (size_t)(cols / 32));
    int8_t* xq = (int8_t*)malloc((size_t)cols);
    afo_quantize_q8(xd, xq, x, cols);
    for (int r = 0; r < rows; r++) {
        const uint8_t* row = (const uint8_t*)W + (size_t)r * rb;
        y[r] = type == GGML_Q6_K ? q6k_q8_dot_row(row, xd, xq, cols) : q4k_q8_dot_row(row, xd, xq, cols);
    }
    free(xd);
    free(xq);
}

/* One sampling step on `lg` (modified in place): the repetition penalty of
 * llama_generate's decode loop (llama_model.cpp:1586-1598: for each window id
 * in order, v/pen if v > 0 else v·pen), then sample() (llama_model.cpp:
 * 1466-1498): greedy first maximum at temperature <= 0; otherwise the k
 * largest of lg/T in descending order (ties: lower index first), p_i =
 * exp(s_i − s_0) normalised in order, the nucleus cut at the first cumulative
 * p >= top_p and renormalised, and the first i whose cumulative p exceeds r
 * (r: the uniform draw of the reference's rng). */
typedef struct {
    float v;
    int i;
} afo_scored;

static int scored_desc(const void* a, const void* b) {
    const afo_scored* x = (const afo_scored*)a;
    const afo_scored* y = (const afo_scored*)b;
    if (x->v != y->v) return x->v > y->v ? -1 : 1;
    return x->i - y->i;
}

int afo_sample(float* lg, int V, const int32_t* win, int n_win, float pen, int top_k, float top_p, float temp,
               float r) {
    if (pen != 1.0f)
        for (int i = 0; i < n_win; i++) {
            const int id = win[i];
            if (id < 0 || id >= V) continue;
            lg[id] = lg[id] > 0.f ? lg[id] / pen : lg[id] * pen;
        }
    if (temp <= 0.f) {
        int best = 0;
        for (int i = 1; i < V; i++)
            if (lg[i] > lg[best]) best = i;
        return best;
    }
    int k = (top_k > 0 && top_k < V) ? top_k : V;
    afo_scored* sc = (afo_scored*)malloc(sizeof(afo_scored) * (size_t)V);
    for (int i = 0; i < V; i++) {
        sc[i].v = lg[i] / temp;
        sc[i].i = i;
    }
    qsort(sc, (size_t)V, sizeof(afo_scored), scored_desc);
    float* p = (float*)malloc(sizeof(float) * (size_t)k);
    const float mx = sc[0].v;
    float sum = 0.f;
    for (int i = 0; i < k; i++) {
        p[i] = expf(sc[i].v - mx);
        sum += p[i];
    }
    for (int i = 0; i < k; i++) p[i] /= sum;
    if (top_p < 1.0f) {
        float cum = 0.f;
        int cut = k;
        for (int i = 0; i < k; i++) {
            cum += p[i];
            if (cum >= top_p) {
                cut = i + 1;
                break;
            }
        }
        sum = 0.f;
        for (int i = 0; i < cut; i++) sum += p[i];
        for (int i = 0; i < cut; i++) p[i] /= sum;
        k = cut;
    }
    float cum = 0.f;
    int pick = sc[k - 1].i;
    for (int i = 0; i < k; i++) {
        cum += p[i];
        if (r < cum) {
            pick = sc[i].i;
            break;
        }
    }
    free(p);
    free(sc);
    return pick;
}

/* RMSNorm with separate output: rms_norm_out, llama_model.cpp:393-419. */
void afo_rms_norm(float* dst, const float* src, const float* w, int n, float eps) {
    float ss = 0.f;
    for (int i = 0; i < n; i++) ss += src[i] * src[i];
    ss = 1.f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; i++) dst[i] = w[i] * (src[i] * ss);
}

/* RoPE tables: RopeCache::build, llama_model.cpp:1024-1043.  cos/sin [n_pos][hd/2]. */
void afo_rope_tables(float* cos_t, float* sin_t, int head_dim, float theta, int n_pos) {
    const int half = head_dim / 2;
    for (int p = 0; p < n_pos; p++) {
        for (int i = 0; i < half; i++) {
            const float freq = 1.f / powf(theta, (float)(2 * i) / (float)head_dim);
            const float angle = (float)p * freq;
            cos_t[(size_t)p * half + i] = cosf(angle);
            sin_t[(size_t)p * half + i] = sinf(angle);
        }
    }
}

/* Half-split ("NeoX") rotation of n_heads heads: apply_rope,
 * llama_model.cpp:1046-1060 (also rope_and_store_k, 1063-1080). */
void afo_rope(float* dst, const float* src, int n_heads, int head_dim, const float* cos_row,
              const float* sin_row) {
    const int half = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        const float* s = src + h * head_dim;
        float* d = dst + h * head_dim;
        for (int i = 0; i < half; i++) {
            const float x0 = s[i], x1 = s[i + half];
            d[i] = x0 * cos_row[i] - x1 * sin_row[i];
            d[i + half] = x0 * sin_row[i] + x1 * cos_row[i];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Whole-model single-token forward: llama_forward_token, llama_model.cpp:1207-1333 */

typedef struct {
    int n_layer, n_embd, n_head, n_kv_head, ffn, vocab, n_ctx;
    float eps, theta;
    int qk_norm_order; /* 0 none, 1 before RoPE (qwen3), 2 after RoPE (hunyuan) */
} afo_cfg;

typedef struct {
    const float *attn_norm, *ffn_norm, *bq, *bk, *bv, *q_norm, *k_norm;
    const void *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    int tq, tk, tv, to, tg, tu, td;
} afo_layer;

typedef struct {
    afo_cfg c;
    int head_dim, kv_dim;
    const void* tok_embd;
    int tok_type;
    const float* out_norm;
    const void* output;
    int out_type;
    afo_layer* layers;
    float *kv_k, *kv_v, *cos_t, *sin_t;
    float *x, *xb, *q, *k, *v, *att, *ao, *gate, *up, *ffo, *logits;
} afo_model;

void* afo_create(const afo_cfg* c) {
    afo_model* m = (afo_model*)calloc(1, sizeof(afo_model));
    m->c = *c;
    m->head_dim = c->n_embd / c->n_head;
    m->kv_dim = c->n_kv_head * m->head_dim;
    m->layers = (afo_layer*)calloc((size_t)c->n_layer, sizeof(afo_layer));
    const size_t kvn = (size_t)c->n_layer * c->n_ctx * m->kv_dim;
    m->kv_k = (float*)calloc(kvn, 4);
    m->kv_v = (float*)calloc(kvn, 4);
    m->cos_t = (float*)malloc((size_t)c->n_ctx * (m->head_dim / 2) * 4);
    m->sin_t = (float*)malloc((size_t)c->n_ctx * (m->head_dim / 2) * 4);
    afo_rope_tables(m->cos_t, m->sin_t, m->head_dim, c->theta, c->n_ctx);
    m->x = (float*)calloc(c->n_embd, 4);
    m->xb = (float*)calloc(c->n_embd, 4);
    m->q = (float*)calloc(c->n_embd, 4);
    m->k = (float*)calloc(m->kv_dim, 4);
    m->v = (float*)calloc(m->kv_dim, 4);
    m->att = (float*)calloc(c->n_ctx, 4);
    m->ao = (float*)calloc(c->n_embd, 4);
    m->gate = (float*)calloc(c->ffn, 4);
    m->up = (float*)calloc(c->ffn, 4);
    m->ffo = (float*)calloc(c->n_embd, 4);
    m->logits = (float*)calloc(c->vocab, 4);
    return m;
}

void afo_destroy(void* h) {
    afo_model* m = (afo_model*)h;
    if (!m) return;
    free(m->layers); free(m->kv_k); free(m->kv_v); free(m->cos_t); free(m->sin_t);
    free(m->x); free(m->xb); free(m->q); free(m->k); free(m->v); free(m->att); free(m->ao);
    free(m->gate); free(m->up); free(m->ffo); free(m->logits);
    free(m);
}

/* `output` may be NULL: the LM head then falls back to token_embd
 * (make_wt_opt, llama_model.cpp:979). */
void afo_set_global(void* h, const void* tok_embd, int tok_type, const float* out_norm,
                    const void* output, int out_type) {
    afo_model* m = (afo_model*)h;
    m->tok_embd = tok_embd;
    m->tok_type = tok_type;
    m->out_norm = out_norm;
    m->output = output ? output : tok_embd;
    m->out_type = output ? out_type : tok_type;
}

void afo_set_layer(void* h, int l, const afo_layer* lw) { ((afo_model*)h)->layers[l] = *lw; }

static void add_bias(float* y, const float* b, int n) {
    if (!b) return;
    for (int i = 0; i < n; i++) y[i] += b[i];
}

static void rms_norm_heads(float* x, const float* w, int n_heads, int hd, float eps) {
    if (!w) return;
    for (int h = 0; h < n_heads; h++) afo_rms_norm(x + (size_t)h * hd, x + (size_t)h * hd, w, hd, eps);
}

/* Embedding lookup: emb_lookup, llama_model.cpp:882-934 (Q4_K / Q6_K / F32). */
static void emb_row(float* out, const void* W, int type, int row, int cols) {
    const uint8_t* base = (const uint8_t*)W + (size_t)row * row_bytes_of(type, cols);
    if (type == GGML_Q4_K) afo_q4k_row_to_f32(out, base, cols);
    else if (type == GGML_Q6_K) afo_q6k_row_to_f32(out, base, cols);
    else memcpy(out, base, (size_t)cols * 4);
}

/* One new token's attention for one layer, llama_model.cpp:1236-1272: the
 * optional per-head Q/K RMSNorm before RoPE (qwen3, order 1) or after it
 * (hunyuan, order 2) (:1236-1247, rms_norm_heads_inplace :421-441), half-split
 * RoPE of q and k (apply_rope / rope_and_store_k :1046-1080), K and V stored
 * at row pos of the fp32 caches [n_ctx][KVH*HD], then GQA attention over
 * positions 0..pos: scores * 1/sqrt(HD), max-subtracted softmax (:445-451),
 * weighted V sum (:1253-1272).  q and k are rotated in place; att is scratch
 * of pos + 1 floats. */
void afo_attention_decode(float* ao, float* q, float* k, const float* v, float* kc, float* vc, const float* cr,
                          const float* sr, const float* q_norm, const float* k_norm, int pos, int H, int KVH,
                          int HD, int qk_norm_order, float eps, float* att) {
    const int KVD = KVH * HD;
    const float scale = 1.f / sqrtf((float)HD);
    if (qk_norm_order == 1) {
        rms_norm_heads(q, q_norm, H, HD, eps);
        rms_norm_heads(k, k_norm, KVH, HD, eps);
    }
    afo_rope(q, q, H, HD, cr, sr);
    if (qk_norm_order == 2) {
        afo_rope(k, k, KVH, HD, cr, sr);
        rms_norm_heads(q, q_norm, H, HD, eps);
        rms_norm_heads(k, k_norm, KVH, HD, eps);
        memcpy(kc + (size_t)pos * KVD, k, (size_t)KVD * 4);
    } else {
        afo_rope(kc + (size_t)pos * KVD, k, KVH, HD, cr, sr);
    }
    memcpy(vc + (size_t)pos * KVD, v, (size_t)KVD * 4);
    const int seq = pos + 1, group = H / KVH;
    memset(ao, 0, (size_t)H * HD * 4);
    for (int hh = 0; hh < H; hh++) {
        const int kvh = hh / group;
        const float* qh = q + hh * HD;
        for (int t = 0; t < seq; t++) {
            const float* kt = kc + (size_t)t * KVD + kvh * HD;
            float s = 0.f;
            for (int i = 0; i < HD; i++) s += qh[i] * kt[i];
            att[t] = s * scale;
        }
        float mx = att[0], sum = 0.f;
        for (int t = 1; t < seq; t++) if (att[t] > mx) mx = att[t];
        for (int t = 0; t < seq; t++) { att[t] = expf(att[t] - mx); sum += att[t]; }
        for (int t = 0; t < seq; t++) att[t] /= sum;
        float* oh = ao + hh * HD;
        for (int t = 0; t < seq; t++) {
            const float* vt = vc + (size_t)t * KVD + kvh * HD;
            for (int i = 0; i < HD; i++) oh[i] += att[t] * vt[i];
        }
    }
}

int afo_forward_token(void* h, int token, int pos, float* logits_out) {
    afo_model* m = (afo_model*)h;
    const afo_cfg* c = &m->c;
    const int E = c->n_embd, H = c->n_head, KVH = c->n_kv_head, HD = m->head_dim, FD = c->ffn;
    const int KVD = m->kv_dim;
    if (pos < 0 || pos >= c->n_ctx || token < 0 || token >= c->vocab) return -1;
    const float* cr = m->cos_t + (size_t)pos * (HD / 2);
    const float* sr = m->sin_t + (size_t)pos * (HD / 2);
    emb_row(m->x, m->tok_embd, m->tok_type, token, E);
    for (int l = 0; l < c->n_layer; l++) {
        const afo_layer* lw = &m->layers[l];
        float* kc = m->kv_k + (size_t)l * c->n_ctx * KVD;
        float* vc = m->kv_v + (size_t)l * c->n_ctx * KVD;
        afo_rms_norm(m->xb, m->x, lw->attn_norm, E, c->eps);
        afo_gemv(m->q, lw->wq, lw->tq, m->xb, H * HD, E);
        afo_gemv(m->k, lw->wk, lw->tk, m->xb, KVD, E);
        afo_gemv(m->v, lw->wv, lw->tv, m->xb, KVD, E);
        add_bias(m->q, lw->bq, H * HD);
        add_bias(m->k, lw->bk, KVD);
        add_bias(m->v, lw->bv, KVD);
        afo_attention_decode(m->ao, m->q, m->k, m->v, kc, vc, cr, sr, lw->q_norm, lw->k_norm, pos, H, KVH, HD,
                             c->qk_norm_order, c->eps, m->att);
        afo_gemv(m->xb, lw->wo, lw->to, m->ao, E, E);
        for (int i = 0; i < E; i++) m->x[i] += m->xb[i];
        afo_rms_norm(m->xb, m->x, lw->ffn_norm, E, c->eps);
        afo_gemv(m->gate, lw->wg, lw->tg, m->xb, FD, E);
        afo_gemv(m->up, lw->wu, lw->tu, m->xb, FD, E);
        /* SwiGLU: silu(g)*u, llama_model.cpp:313-315 / 344-368. */
        for (int i = 0; i < FD; i++) {
            const float g = m->gate[i];
            m->gate[i] = (g / (1.f + expf(-g))) * m->up[i];
        }
        afo_gemv(m->ffo, lw->wd, lw->td, m->gate, E, FD);
        for (int i = 0; i < E; i++) m->x[i] += m->ffo[i];
    }
    afo_rms_norm(m->xb, m->x, m->out_norm, E, c->eps);
    afo_gemv(m->logits, m->output, m->out_type, m->xb, c->vocab, E);
    if (logits_out) memcpy(logits_out, m->logits, (size_t)c->vocab * 4);
    return 0;
}

/* Greedy argmax, first maximum: sample() at temperature 0, llama_model.cpp:1466-1471. */
int afo_argmax(const float* v, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (v[i] > v[best]) best = i;
    return best;
}

/* Residual stream after the last forward, before the final RMSNorm (the
 * reference normalises it in place, rms_norm_avx2(s.x) at llama_model.cpp:1328;
 * here the normalised copy goes to a scratch buffer instead). */
void afo_hidden(void* h, float* out) {
    afo_model* m = (afo_model*)h;
    memcpy(out, m->x, (size_t)m->c.n_embd * 4);
}

/* Rows [0, n_pos) of layer l's K (which_v = 0) or V cache. */
void afo_kv(void* h, int l, int which_v, int n_pos, float* out) {
    afo_model* m = (afo_model*)h;
    const float* base = (which_v ? m->kv_v : m->kv_k) + (size_t)l * m->c.n_ctx * m->kv_dim;
    memcpy(out, base, (size_t)n_pos * m->kv_dim * 4);
}
