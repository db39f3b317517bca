/*
 * orc_model.c -- oracle for the W4A16 projections, verify attention, the
 * verify forward and the chained MTP draft.  TEST INFRASTRUCTURE ONLY.
 *
 * Rounding points follow the CUDA path: activations that feed a GEMM are
 * rounded to fp16 (RMSNorm output, attention output, SwiGLU output), K/V
 * are stored in fp16, GEMM and softmax accumulate in fp32.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------ synthetic weights */
float orc_synth_value(uint32_t seed, uint32_t tid, uint64_t e) {
    uint32_t ctr[4] = {(uint32_t)e, (uint32_t)(e >> 32), tid, 0u}, key[2] = {seed, 0x5EEDF00Du}, o[4];
    orc_philox4x32_10(ctr, key, o);
    const double inv24 = 1.0 / 16777216.0;
    double s = (double)(o[0] >> 8) * inv24 + (double)(o[1] >> 8) * inv24 + (double)(o[2] >> 8) * inv24 +
               (double)(o[3] >> 8) * inv24;
    return (float)((s - 2.0) * 0.034641016151377546); /* sqrt(3) * 0.02 */
}

/* One row of K values to int4 with group-128 fp16 scales: s = fp16(amax / 7)
 * (1 when amax = 0), q = clamp(round(w / s), -8, 7), u4 = q + 8, low nibble
 * = even k. */
static void quantize_row(const float* w, int K, uint8_t* packed, uint16_t* scales) {
    const int G = (K + 127) / 128; /* the last group may hold fewer than 128 columns */
    for (int g = 0; g < G; ++g) {
        const float* wg = w + (size_t)g * 128;
        const int gl = (K - g * 128) < 128 ? (K - g * 128) : 128;
        float amax = 0.0f;
        for (int t = 0; t < gl; ++t) {
            float a = fabsf(wg[t]);
            if (a > amax) amax = a;
        }
        uint16_t s16 = orc_f32_to_f16(amax / 7.0f);
        if (amax == 0.0f) s16 = orc_f32_to_f16(1.0f);
        scales[g] = s16;
        float sf = orc_f16_to_f32(s16);
        uint8_t* dst = packed + g * 64;
        for (int t = 0; t < gl; t += 2) {
            int q0 = (int)roundf(wg[t] / sf), q1 = (int)roundf(wg[t + 1] / sf);
            q0 = q0 < -8 ? -8 : (q0 > 7 ? 7 : q0);
            q1 = q1 < -8 ? -8 : (q1 > 7 ? 7 : q1);
            dst[t / 2] = (uint8_t)((q0 + 8) | ((q1 + 8) << 4));
        }
    }
}

void orc_w4_quantize(const float* w, int n, int K, uint8_t* packed, uint16_t* scales) {
    const int G = (K + 127) / 128;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; ++r) quantize_row(w + (size_t)r * K, K, packed + (size_t)r * (K / 2), scales + (size_t)r * G);
}

void orc_synth_w4(uint32_t seed, uint32_t tid, int N, int K, int n0, int n, uint8_t* packed, uint16_t* scales) {
    (void)N;
    const int G = (K + 127) / 128;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; ++r) {
        const int row = n0 + r;
        float* w = (float*)malloc(sizeof(float) * (size_t)G * 128);
        for (int t = 0; t < K; ++t) w[t] = orc_synth_value(seed, tid, (uint64_t)row * K + t);
        quantize_row(w, K, packed + (size_t)r * (K / 2), scales + (size_t)r * G);
        free(w);
    }
}

void orc_synth_f16(uint32_t seed, uint32_t tid, uint64_t e0, size_t n, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16(orc_synth_value(seed, tid, e0 + i));
}

void orc_w4_dequant(const uint8_t* packed, const uint16_t* scales, int N, int K, float* out) {
    const int G = (K + 127) / 128;
    for (int n = 0; n < N; ++n)
        for (int k = 0; k < K; ++k) {
            uint8_t byte = packed[(size_t)n * (K / 2) + k / 2];
            int u = (k & 1) ? (byte >> 4) : (byte & 15);
            float s = orc_f16_to_f32(scales[(size_t)n * G + k / 128]);
            out[(size_t)n * K + k] = orc_f16_to_f32(orc_f32_to_f16((float)(u - 8) * s));
        }
}

void orc_w4a16_gemm(const uint16_t* X, int M, const uint8_t* packed, const uint16_t* scales, int N, int K, float* Y,
                    int ldy, int mode) {
    const int G = (K + 127) / 128;
    float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
    orc_f16_to_f32_n(X, xf, (size_t)M * K);
#pragma omp parallel
    {
        float* wrow = (float*)malloc(sizeof(float) * K);
#pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            const uint8_t* pr = packed + (size_t)n * (K / 2);
            for (int k = 0; k < K; ++k) {
                int u = (k & 1) ? (pr[k / 2] >> 4) : (pr[k / 2] & 15);
                float s = orc_f16_to_f32(scales[(size_t)n * G + k / 128]);
                wrow[k] = orc_f16_to_f32(orc_f32_to_f16((float)(u - 8) * s));
            }
            for (int m = 0; m < M; ++m) {
                const float* xr = xf + (size_t)m * K;
                float acc = 0.0f;
                for (int k = 0; k < K; ++k) acc += xr[k] * wrow[k];
                float* y = Y + (size_t)m * ldy + n;
                if (mode) *y += acc;
                else *y = acc;
            }
        }
        free(wrow);
    }
    free(xf);
}

/* lib.rs:21-36 (sum of squares, mean, 1/sqrt(mean+eps), times weight) */
void orc_rmsnorm_f16(const float* x, const float* w, int n, float eps, uint16_t* out) {
    float ss = 0.0f;
    for (int i = 0; i < n; ++i) ss += x[i] * x[i];
    float r = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; ++i) out[i] = orc_f32_to_f16(x[i] * r * (w ? w[i] : 1.0f));
}

void orc_rope_tables(int max_pos, int head_dim, float theta, float* cos_t, float* sin_t) {
    int half = head_dim / 2;
    for (int p = 0; p < max_pos; ++p)
        for (int d = 0; d < half; ++d) {
            double inv = pow((double)theta, -2.0 * d / (double)head_dim);
            double ang = (double)p * inv;
            cos_t[(size_t)p * half + d] = (float)cos(ang);
            sin_t[(size_t)p * half + d] = (float)sin(ang);
        }
}

/* lib.rs:621-663 rotate-half on one head vector */
static void rope_apply(float* v, int hd, const float* c, const float* s) {
    int half = hd / 2;
    for (int d = 0; d < half; ++d) {
        float a = v[d], b = v[d + half];
        v[d] = a * c[d] - b * s[d];
        v[d + half] = b * c[d] + a * s[d];
    }
}

/* -------------------------------------------------------- attention */
void orc_attention(const uint16_t* q, const orc_kv_pool* kv, int layer, const int32_t* tables, int max_blocks,
                   const int32_t* ctx_len, const uint64_t* mask, int B, int R, int Hq, uint16_t* out) {
    const int hd = kv->head_dim, Hkv = kv->n_kv_heads, bs = kv->block_size, G = Hq / Hkv;
    const float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < Hkv; ++h) {
            int L = ctx_len[b] + R;
            float* sc = (float*)malloc(sizeof(float) * L);
            float* qf = (float*)malloc(sizeof(float) * hd);
            float* acc = (float*)malloc(sizeof(float) * hd);
            for (int r = 0; r < R; ++r)
                for (int g = 0; g < G; ++g) {
                    int qh = h * G + g; /* lib.rs:841-842 */
                    const uint16_t* qr = q + ((size_t)(b * R + r) * Hq + qh) * hd;
                    for (int d = 0; d < hd; ++d) qf[d] = orc_f16_to_f32(qr[d]);
                    float mx = -INFINITY;
                    for (int t = 0; t < L; ++t) {
                        int vis = t < ctx_len[b] || ((mask[r] >> (t - ctx_len[b])) & 1ull);
                        if (!vis) { sc[t] = -INFINITY; continue; }
                        int blk = tables[(size_t)b * max_blocks + t / bs];
                        const uint16_t* kr = kv->pool + orc_kv_offset(kv, layer, blk, 0, h, t % bs);
                        float dot = 0.0f;
                        for (int d = 0; d < hd; ++d) dot += qf[d] * orc_f16_to_f32(kr[d]);
                        sc[t] = dot * scale;
                        if (sc[t] > mx) mx = sc[t];
                    }
                    float sum = 0.0f;
                    for (int d = 0; d < hd; ++d) acc[d] = 0.0f;
                    for (int t = 0; t < L; ++t) {
                        if (sc[t] == -INFINITY) continue;
                        float w = expf(sc[t] - mx);
                        sum += w;
                        int blk = tables[(size_t)b * max_blocks + t / bs];
                        const uint16_t* vr = kv->pool + orc_kv_offset(kv, layer, blk, 1, h, t % bs);
                        for (int d = 0; d < hd; ++d) acc[d] += w * orc_f16_to_f32(vr[d]);
                    }
                    uint16_t* o = out + ((size_t)(b * R + r) * Hq + qh) * hd;
                    for (int d = 0; d < hd; ++d) o[d] = orc_f32_to_f16(acc[d] / sum);
                }
            free(sc);
            free(qf);
            free(acc);
        }
}

/* paged_attention.cpp:16-111: un-normalised exp(q.k/sqrt(H))/seq_len weights */
void orc_compat_paged_attention(const float* q, const float* k_pool, const float* v_pool, const int32_t* table_off,
                                const int32_t* tables, const int32_t* seq_lens, float* o, int M, int H, int bs) {
    for (int m = 0; m < M; ++m) {
        int seq_len = seq_lens[m];
        int nb = table_off[m + 1] - table_off[m];
        if (seq_len == 0 || nb == 0) continue;
        float att_scale = 1.0f / sqrtf((float)H);
        float inv_len = 1.0f / (float)(seq_len > 1 ? seq_len : 1);
        int done = 0;
        const float* qp = q + (size_t)m * H;
        float* op = o + (size_t)m * H;
        for (int b = 0; b < nb; ++b) {
            int phys = tables[table_off[m] + b];
            int tib = bs < seq_len - done ? bs : seq_len - done;
            size_t base = (size_t)phys * bs * H;
            for (int t = 0; t < tib; ++t) {
                const float* kp = k_pool + base + (size_t)t * H;
                const float* vp = v_pool + base + (size_t)t * H;
                float s = 0.0f;
                for (int i = 0; i < H; ++i) s += qp[i] * kp[i];
                s *= att_scale;
                float w = expf(s) * inv_len;
                for (int j = 0; j < H; ++j) op[j] += w * vp[j];
            }
            done += tib;
        }
    }
}

/* lib.rs:1638-1712 */
void orc_flashdecoding_chunk(const float* q, const float* k, const float* v, int len, int hd, float scale,
                             float* part_o, float* part_max, float* part_sum) {
    float mx = -INFINITY;
    for (int t = 0; t < len; ++t) {
        float s = 0.0f;
        for (int d = 0; d < hd; ++d) s += q[d] * k[(size_t)t * hd + d];
        s *= scale;
        if (s > mx) mx = s;
    }
    float sum = 0.0f;
    for (int d = 0; d < hd; ++d) part_o[d] = 0.0f;
    for (int t = 0; t < len; ++t) {
        float s = 0.0f;
        for (int d = 0; d < hd; ++d) s += q[d] * k[(size_t)t * hd + d];
        s *= scale;
        float w = expf(s - mx);
        sum += w;
        for (int d = 0; d < hd; ++d) part_o[d] += w * v[(size_t)t * hd + d];
    }
    *part_max = mx;
    *part_sum = sum;
}

/* lib.rs:1721-1783 */
void orc_flashdecoding_reduce(const float* part_o, const float* part_max, const float* part_sum, int chunks, int hd,
                              float* out) {
    float g = -INFINITY;
    for (int c = 0; c < chunks; ++c)
        if (part_max[c] > g) g = part_max[c];
    for (int d = 0; d < hd; ++d) out[d] = 0.0f;
    float gs = 0.0f;
    for (int c = 0; c < chunks; ++c) {
        float r = expf(part_max[c] - g);
        gs += part_sum[c] * r;
        for (int d = 0; d < hd; ++d) out[d] += part_o[(size_t)c * hd + d] * r;
    }
    float inv = 1.0f / gs;
    for (int d = 0; d < hd; ++d) out[d] *= inv;
}

/* ------------------------------------------------------------- model */
static size_t w_rows(const orc_model_cfg* c, int which) {
    switch (which) {
        case ORC_T_Q: return (size_t)c->n_q_heads * c->head_dim;
        case ORC_T_K:
        case ORC_T_V: return (size_t)c->n_kv_heads * c->head_dim;
        case ORC_T_O: return (size_t)c->hidden;
        case ORC_T_GATE:
        case ORC_T_UP: return (size_t)c->ffn;
        default: return (size_t)c->hidden;
    }
}
static size_t w_cols(const orc_model_cfg* c, int which) {
    switch (which) {
        case ORC_T_O: return (size_t)c->n_q_heads * c->head_dim;
        case ORC_T_DOWN: return (size_t)c->ffn;
        default: return (size_t)c->hidden;
    }
}

orc_model* orc_model_create(const orc_model_cfg* cfg, uint32_t seed, int n_layers_present, int rope_max_pos) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->cfg = *cfg;
    if (n_layers_present < 0 || n_layers_present > cfg->layers) n_layers_present = cfg->layers;
    m->n_layers_present = n_layers_present;
    const int H = cfg->hidden, V = cfg->vocab;
    m->emb = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)V * H);
    orc_synth_f16(seed, ORC_T_EMB, 0, (size_t)V * H, m->emb);
    for (int w = 0; w < 7; ++w) {
        size_t N = w_rows(cfg, w), K = w_cols(cfg, w);
        m->w_packed[w] = (uint8_t*)malloc((size_t)n_layers_present * N * K / 2);
        m->w_scales[w] = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n_layers_present * N * ((K + 127) / 128));
        for (int l = 0; l < n_layers_present; ++l)
            orc_synth_w4(seed, orc_layer_tensor(l, w), (int)N, (int)K, 0, (int)N, m->w_packed[w] + (size_t)l * N * K / 2,
                         m->w_scales[w] + (size_t)l * N * ((K + 127) / 128));
    }
    m->lm_packed = (uint8_t*)malloc((size_t)V * H / 2);
    m->lm_scales = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)V * (H / 128));
    orc_synth_w4(seed, ORC_T_LM, V, H, 0, V, m->lm_packed, m->lm_scales);
    m->mtp_packed = (uint8_t*)malloc((size_t)cfg->n_mtp_heads * H * H / 2);
    m->mtp_scales = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)cfg->n_mtp_heads * H * (H / 128));
    for (int i = 0; i < cfg->n_mtp_heads; ++i)
        orc_synth_w4(seed, ORC_T_MTP0 + i, H, H, 0, H, m->mtp_packed + (size_t)i * H * H / 2,
                     m->mtp_scales + (size_t)i * H * (H / 128));
    m->rope_max_pos = rope_max_pos;
    int half = cfg->head_dim / 2;
    m->rope_cos = (float*)malloc(sizeof(float) * (size_t)rope_max_pos * half);
    m->rope_sin = (float*)malloc(sizeof(float) * (size_t)rope_max_pos * half);
    orc_rope_tables(rope_max_pos, cfg->head_dim, cfg->rope_theta, m->rope_cos, m->rope_sin);
    return m;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    free(m->emb);
    for (int w = 0; w < 7; ++w) { free(m->w_packed[w]); free(m->w_scales[w]); }
    free(m->lm_packed); free(m->lm_scales); free(m->mtp_packed); free(m->mtp_scales);
    free(m->rope_cos); free(m->rope_sin);
    free(m);
}

static const uint8_t* lw(const orc_model* m, int which, int l) {
    size_t N = w_rows(&m->cfg, which), K = w_cols(&m->cfg, which);
    return m->w_packed[which] + (size_t)l * N * K / 2;
}
static const uint16_t* ls(const orc_model* m, int which, int l) {
    size_t N = w_rows(&m->cfg, which), K = w_cols(&m->cfg, which);
    return m->w_scales[which] + (size_t)l * N * ((K + 127) / 128);
}

void orc_forward(const orc_model* m, orc_kv_pool* kv, const int32_t* tables, int max_blocks, const int32_t* ctx_len,
                 const int32_t* tokens, const int32_t* pos, const int32_t* slot, const uint64_t* mask, int B, int R,
                 int n_layers, float* logits, float* hidden_out) {
    const orc_model_cfg* c = &m->cfg;
    const int H = c->hidden, Hq = c->n_q_heads, Hkv = c->n_kv_heads, hd = c->head_dim, F = c->ffn, V = c->vocab;
    const int M = B * R, qd = Hq * hd, kd = Hkv * hd, half = hd / 2, bs = c->block_size;
    if (n_layers < 0 || n_layers > m->n_layers_present) n_layers = m->n_layers_present;
    float* x = (float*)malloc(sizeof(float) * (size_t)M * H);
    uint16_t* xn = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M * (F > H ? F : H));
    float* q = (float*)malloc(sizeof(float) * (size_t)M * qd);
    float* kk = (float*)malloc(sizeof(float) * (size_t)M * kd);
    float* vv = (float*)malloc(sizeof(float) * (size_t)M * kd);
    uint16_t* q16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M * qd);
    uint16_t* att = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)M * qd);
    float* g = (float*)malloc(sizeof(float) * (size_t)M * F);
    float* u = (float*)malloc(sizeof(float) * (size_t)M * F);
    for (int r = 0; r < M; ++r)
        for (int i = 0; i < H; ++i) x[(size_t)r * H + i] = orc_f16_to_f32(m->emb[(size_t)tokens[r] * H + i]);
    for (int l = 0; l < n_layers; ++l) {
        for (int r = 0; r < M; ++r) orc_rmsnorm_f16(x + (size_t)r * H, NULL, H, c->rms_eps, xn + (size_t)r * H);
        orc_w4a16_gemm(xn, M, lw(m, ORC_T_Q, l), ls(m, ORC_T_Q, l), qd, H, q, qd, 0);
        orc_w4a16_gemm(xn, M, lw(m, ORC_T_K, l), ls(m, ORC_T_K, l), kd, H, kk, kd, 0);
        orc_w4a16_gemm(xn, M, lw(m, ORC_T_V, l), ls(m, ORC_T_V, l), kd, H, vv, kd, 0);
        for (int r = 0; r < M; ++r) {
            const float* cs = m->rope_cos + (size_t)pos[r] * half;
            const float* sn = m->rope_sin + (size_t)pos[r] * half;
            for (int hh = 0; hh < Hq; ++hh) rope_apply(q + (size_t)r * qd + hh * hd, hd, cs, sn);
            for (int hh = 0; hh < Hkv; ++hh) rope_apply(kk + (size_t)r * kd + hh * hd, hd, cs, sn);
            int b = r / R, s = slot[r];
            int blk = tables[(size_t)b * max_blocks + s / bs];
            for (int hh = 0; hh < Hkv; ++hh) {
                uint16_t* kdst = kv->pool + orc_kv_offset(kv, l, blk, 0, hh, s % bs);
                uint16_t* vdst = kv->pool + orc_kv_offset(kv, l, blk, 1, hh, s % bs);
                for (int d = 0; d < hd; ++d) {
                    kdst[d] = orc_f32_to_f16(kk[(size_t)r * kd + hh * hd + d]);
                    vdst[d] = orc_f32_to_f16(vv[(size_t)r * kd + hh * hd + d]);
                }
            }
        }
        orc_f32_to_f16_n(q, q16, (size_t)M * qd);
        orc_attention(q16, kv, l, tables, max_blocks, ctx_len, mask, B, R, Hq, att);
        orc_w4a16_gemm(att, M, lw(m, ORC_T_O, l), ls(m, ORC_T_O, l), H, qd, x, H, 1);
        for (int r = 0; r < M; ++r) orc_rmsnorm_f16(x + (size_t)r * H, NULL, H, c->rms_eps, xn + (size_t)r * H);
        orc_w4a16_gemm(xn, M, lw(m, ORC_T_GATE, l), ls(m, ORC_T_GATE, l), F, H, g, F, 0);
        orc_w4a16_gemm(xn, M, lw(m, ORC_T_UP, l), ls(m, ORC_T_UP, l), F, H, u, F, 0);
        for (size_t i = 0; i < (size_t)M * F; ++i) {
            float gv = g[i];
            xn[i] = orc_f32_to_f16(gv / (1.0f + expf(-gv)) * u[i]);
        }
        orc_w4a16_gemm(xn, M, lw(m, ORC_T_DOWN, l), ls(m, ORC_T_DOWN, l), H, F, x, H, 1);
    }
    if (hidden_out) memcpy(hidden_out, x, sizeof(float) * (size_t)M * H);
    if (logits) {
        for (int r = 0; r < M; ++r) orc_rmsnorm_f16(x + (size_t)r * H, NULL, H, c->rms_eps, xn + (size_t)r * H);
        orc_w4a16_gemm(xn, M, m->lm_packed, m->lm_scales, V, H, logits, V, 0);
    }
    free(x); free(xn); free(q); free(kk); free(vv); free(q16); free(att); free(g); free(u);
}

void orc_draft_chain(const orc_model* m, const float* h0, int B, int k, float temperature, float top_p, uint64_t seed,
                     uint32_t step, float* draft_logits, int32_t* drafts, float* hid_out) {
    const orc_model_cfg* c = &m->cfg;
    const int H = c->hidden, V = c->vocab;
    float* h = (float*)malloc(sizeof(float) * (size_t)B * H);
    float* hn = (float*)malloc(sizeof(float) * (size_t)B * H);
    uint16_t* x16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)B * H);
    float* lg = (float*)malloc(sizeof(float) * (size_t)B * V);
    int32_t* tok = (int32_t*)malloc(sizeof(int32_t) * B);
    memcpy(h, h0, sizeof(float) * (size_t)B * H);
    for (int i = 0; i < k; ++i) {
        int head = i < c->n_mtp_heads ? i : c->n_mtp_heads - 1;
        for (int b = 0; b < B; ++b) orc_rmsnorm_f16(h + (size_t)b * H, NULL, H, c->rms_eps, x16 + (size_t)b * H);
        orc_w4a16_gemm(x16, B, m->mtp_packed + (size_t)head * H * H / 2, m->mtp_scales + (size_t)head * H * (H / 128),
                       H, H, hn, H, 0);
        memcpy(h, hn, sizeof(float) * (size_t)B * H);
        if (hid_out)
            for (int b = 0; b < B; ++b) memcpy(hid_out + ((size_t)b * k + i) * H, h + (size_t)b * H, sizeof(float) * H);
        for (int b = 0; b < B; ++b) orc_rmsnorm_f16(h + (size_t)b * H, NULL, H, c->rms_eps, x16 + (size_t)b * H);
        orc_w4a16_gemm(x16, B, m->lm_packed, m->lm_scales, V, H, lg, V, 0);
        /* rows of this draft position: sample with stream (b, i) */
        for (int b = 0; b < B; ++b) {
            memcpy(draft_logits + ((size_t)b * k + i) * V, lg + (size_t)b * V, sizeof(float) * V);
        }
        for (int b = 0; b < B; ++b) {
            const float* z = lg + (size_t)b * V;
            if (!(temperature > 0.0f)) { tok[b] = orc_argmax(z, V); continue; }
            orc_row_stats st;
            float cc = (float)(1.4426950408889634 / (double)temperature);
            uint64_t tp = (top_p < 1.0f) ? (uint64_t)llround((double)top_p * 4294967296.0) : (1ull << 32);
            orc_row_stats_compute(z, V, cc, tp, &st);
            tok[b] = orc_draw_row(z, V, cc, &st, seed, step, (uint32_t)b, (uint32_t)i, ORC_U_GUMBEL_DRAFT, NULL, 0);
        }
        for (int b = 0; b < B; ++b) drafts[(size_t)b * k + i] = tok[b];
    }
    free(h); free(hn); free(x16); free(lg); free(tok);
}
