/*
 * orc_sample.c -- oracle for the acceptance / sampling part of the hot path.
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Deterministic arithmetic: every quantity that decides a token is an integer
 * (fixed-point probability masses and their exact sums), so the CUDA kernels
 * and this file agree bit for bit given the same logits.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

/* ------------------------------------------------------------ fp16 */
uint16_t orc_f32_to_f16(float f) {
    _Float16 h = (_Float16)f;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}
float orc_f16_to_f32(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}
void orc_f32_to_f16_n(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_f32_to_f16(src[i]);
}
void orc_f16_to_f32_n(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_f16_to_f32(src[i]);
}

/* ---------------------------------------------------------- Philox */
void orc_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; ++r) {
        if (r) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

uint32_t orc_uniform_u32(uint64_t seed, uint32_t step, uint32_t b, uint32_t i, uint32_t purpose) {
    uint32_t ctr[4] = {b, i, purpose, step}, key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)}, o[4];
    orc_philox4x32_10(ctr, key, o);
    return o[0];
}
uint64_t orc_uniform_u64(uint64_t seed, uint32_t step, uint32_t b, uint32_t i, uint32_t purpose) {
    uint32_t ctr[4] = {b, i, purpose, step}, key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)}, o[4];
    orc_philox4x32_10(ctr, key, o);
    return ((uint64_t)o[0] << 32) | o[1];
}

/* ------------------------------------------------ deterministic exp2 */
/* 1/k! for k = 0..7 and ln 2, as exact fp32 hex literals (shared with the
 * CUDA implementation so both evaluate the identical polynomial). */
static const float kExpTaylor[8] = {0x1p+0f, 0x1p+0f, 0x1p-1f, 0x1.555556p-3f,
                                    0x1.555556p-5f, 0x1.111112p-7f, 0x1.6c16c2p-10f, 0x1.a01a02p-13f};
static const float kLn2f = 0x1.62e43p-1f;

static float pow2_int(int e) { /* exact 2^e for -126 <= e <= 127 */
    uint32_t b = (uint32_t)(e + 127) << 23;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

uint32_t orc_exp2_fx31(float t) {
    if (!(t <= 0.0f)) t = 0.0f;
    if (t < -40.0f) return 0;
    float n = rintf(t);
    float f = t - n;
    float x = f * kLn2f;
    float p = kExpTaylor[7];
    p = fmaf(p, x, kExpTaylor[6]);
    p = fmaf(p, x, kExpTaylor[5]);
    p = fmaf(p, x, kExpTaylor[4]);
    p = fmaf(p, x, kExpTaylor[3]);
    p = fmaf(p, x, kExpTaylor[2]);
    p = fmaf(p, x, kExpTaylor[1]);
    p = fmaf(p, x, kExpTaylor[0]);
    int e = (int)n + 31;
    if (e < 0) return 0;
    float v = p * pow2_int(e);
    return (uint32_t)v;
}

uint32_t orc_logit_key(float z) {
    uint32_t b;
    memcpy(&b, &z, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

/* ------------------------------------------------------ row statistics */
static float row_max(const float* z, int V) {
    float m = -INFINITY;
    for (int j = 0; j < V; ++j)
        if (z[j] > m) m = z[j];
    return m;
}

static inline uint32_t mass_of(float zj, float m, float c) { return orc_exp2_fx31((zj - m) * c); }

void orc_row_stats_compute(const float* z, int V, float c, uint64_t top_p_q32, orc_row_stats* st) {
    float m = row_max(z, V);
    uint64_t S = 0;
    for (int j = 0; j < V; ++j) S += mass_of(z[j], m, c);
    st->max = m;
    st->sum = S;
    if (top_p_q32 >= (1ull << 32)) {
        st->tau = 0;
        st->nuc = S;
        return;
    }
    uint64_t thr = (uint64_t)(((u128)S * top_p_q32) >> 32);
    if (thr < 1) thr = 1;
    uint32_t prefix = 0;
    uint64_t G = 0, last_bin = 0;
    uint64_t* H = (uint64_t*)calloc(256, sizeof(uint64_t));
    for (int d = 3; d >= 0; --d) {
        int shift = 8 * d;
        memset(H, 0, 256 * sizeof(uint64_t));
        for (int j = 0; j < V; ++j) {
            uint32_t key = orc_logit_key(z[j]);
            if (d < 3 && (key >> (shift + 8)) != (prefix >> (shift + 8))) continue;
            H[(key >> shift) & 255u] += mass_of(z[j], m, c);
        }
        uint64_t cum = G;
        int chosen = 0;
        for (int dg = 255; dg >= 0; --dg) {
            if (cum + H[dg] >= thr) { chosen = dg; break; }
            cum += H[dg];
        }
        G = cum;
        last_bin = H[chosen];
        prefix |= (uint32_t)chosen << shift;
    }
    free(H);
    st->tau = prefix;
    st->nuc = G + last_bin;
}

uint32_t orc_row_mass(const float* z, const orc_row_stats* st, float c, int x) {
    if (orc_logit_key(z[x]) < st->tau) return 0;
    return mass_of(z[x], st->max, c);
}

static inline uint64_t mulhi64(uint64_t a, uint64_t b) { return (uint64_t)(((u128)a * b) >> 64); }

/* ---------------------------------------------------- draws
 * A token is drawn with probability proportional to its integer weight w_j
 * (the row mass E_j, or the residual max(0, E_p S_q - E_q S_p)) as the
 * arg-max of the race key w_j / (-log2 U_j) (U_j from Philox per element,
 * ctr = {b, i, (j / 4) << 4 | purpose, step}, word j % 4): -log2 U is
 * exponential, and the smallest of exponentials scaled by 1 / w_j falls on j
 * with probability w_j / sum(w) (the exponential race, equivalent to the
 * Gumbel-max trick).  Ties go to the lower index.
 * log2 by the atanh series ln x = 2 atanh((x - 1) / (x + 1)) on the mantissa
 * in [sqrt(1/2), sqrt(2)), five terms; -log2 U above one half through the
 * complement w = 1 - U, ln(1 / (1 - w)) = 2 atanh(w / (2 - w)), eight terms.
 * Every operation is a single round-to-nearest fp32 operation (the file is
 * compiled with -ffp-contract=off; fmaf is the fused multiply-add), the same
 * sequence as the CUDA kernels, so draws agree bit for bit. */
static float from_bits(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}
static uint32_t to_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}
static float atanh_series5(float s) {
    float s2 = s * s;
    float p = 0x1.c71c72p-4f;          /* 1/9 */
    p = fmaf(p, s2, 0x1.24924ap-3f);   /* 1/7 */
    p = fmaf(p, s2, 0x1.99999ap-3f);   /* 1/5 */
    p = fmaf(p, s2, 0x1.555556p-2f);   /* 1/3 */
    return fmaf(p, s2, 1.0f);
}
float orc_det_log2(float x) {
    uint32_t bits = to_bits(x);
    int e = (int)((bits >> 23) & 255u) - 127;
    float m = from_bits((bits & 0x7FFFFFu) | 0x3F800000u);
    if (m > 0x1.6a09e6p+0f) {
        m = m * 0.5f;
        e += 1;
    }
    float s = (m - 1.0f) / (m + 1.0f);
    return fmaf(s * atanh_series5(s), 0x1.715476p+1f, (float)e);
}
float orc_neg_log2_uniform(uint32_t x) {
    if (x < 0x80000000u) return -orc_det_log2(((float)x + 0.5f) * 0x1p-32f);
    uint32_t y = (uint32_t)(0x100000000ull - (uint64_t)x);
    float w = ((float)y - 0.5f) * 0x1p-32f;
    float s = w / (2.0f - w);
    float s2 = s * s;
    float p = 0x1.111112p-4f;
    p = fmaf(p, s2, 0x1.3b13b2p-4f);
    p = fmaf(p, s2, 0x1.745d18p-4f);
    p = fmaf(p, s2, 0x1.c71c72p-4f);
    p = fmaf(p, s2, 0x1.24924ap-3f);
    p = fmaf(p, s2, 0x1.99999ap-3f);
    p = fmaf(p, s2, 0x1.555556p-2f);
    p = fmaf(p, s2, 1.0f);
    return (s * p) * 0x1.715476p+1f;
}
static float u128_to_f32(u128 w) {
    uint64_t hi = (uint64_t)(w >> 64);
    if (!hi) return (float)(uint64_t)w;
    int sh = 64 - __builtin_clzll(hi);
    return (float)(uint64_t)(w >> sh) * from_bits((uint32_t)(127 + sh) << 23);
}
uint32_t orc_gumbel_uniform(uint64_t seed, uint32_t step, uint32_t b, uint32_t i, uint32_t purpose, uint32_t j) {
    uint32_t ctr[4] = {b, i, ((j >> 2) << 4) | purpose, step}, key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)},
             o[4];
    orc_philox4x32_10(ctr, key, o);
    return o[j & 3];
}
float orc_race_key(float w, uint32_t u) { return w / orc_neg_log2_uniform(u); }

int orc_draw_row(const float* z, int V, float c, const orc_row_stats* st, uint64_t seed, uint32_t step, uint32_t b,
                 uint32_t i, uint32_t purpose, const int32_t* excl, int n_excl) {
    int best = -1;
    float bs = 0.0f;
    for (int j = 0; j < V; ++j) {
        uint32_t e = orc_row_mass(z, st, c, j);
        if (!e) continue;
        int ex = 0;
        for (int t = 0; t < n_excl; ++t) ex |= excl[t] == j;
        if (ex) continue;
        float sc = orc_race_key((float)e, orc_gumbel_uniform(seed, step, b, i, purpose, (uint32_t)j));
        if (best < 0 || sc > bs) {
            bs = sc;
            best = j;
        }
    }
    return best;
}

int orc_argmax(const float* z, int V) {
    int best = -1;
    float bv = -INFINITY;
    for (int j = 0; j < V; ++j) {
        if (z[j] > bv || (best < 0 && z[j] == bv)) { bv = z[j]; best = j; }
    }
    return best;
}

void orc_top2(const float* z, int V, float* top1, float* top2) {
    float a = -INFINITY, b = -INFINITY;
    for (int j = 0; j < V; ++j) {
        float v = z[j];
        if (v > a) { b = a; a = v; }
        else if (v > b) b = v;
    }
    *top1 = a;
    *top2 = b;
}

void orc_topk(const float* z, int V, int k, int* out) {
    for (int t = 0; t < k; ++t) out[t] = -1;
    for (int j = 0; j < V; ++j) {
        float v = z[j];
        int pos = k;
        while (pos > 0 && (out[pos - 1] < 0 || v > z[out[pos - 1]])) --pos;
        if (pos >= k) continue;
        for (int t = k - 1; t > pos; --t) out[t] = out[t - 1];
        out[pos] = j;
    }
}

/* ------------------------------------------------------- acceptance */
static float temp_coeff(float temperature) { return (float)(1.4426950408889634 / (double)temperature); }
static uint64_t top_p_q32(float top_p) {
    if (!(top_p < 1.0f)) return 1ull << 32;
    if (top_p <= 0.0f) return 0;
    return (uint64_t)llround((double)top_p * 4294967296.0);
}

/* Residual draw from max(0, P - Q) (integer cross-multiplied masses); from P
 * when the residual is zero everywhere. */
static int draw_residual(const float* zp, const orc_row_stats* sp, const float* zq, const orc_row_stats* sq, int V,
                         float c, uint64_t seed, uint32_t step, uint32_t b, uint32_t i) {
    int best = -1;
    float bs = 0.0f;
    for (int j = 0; j < V; ++j) {
        u128 a = (u128)orc_row_mass(zp, sp, c, j) * sq->nuc;
        u128 q = (u128)orc_row_mass(zq, sq, c, j) * sp->nuc;
        if (a <= q) continue;
        float sc = orc_race_key(u128_to_f32(a - q), orc_gumbel_uniform(seed, step, b, i, ORC_U_GUMBEL_RESAMPLE,
                                                                         (uint32_t)j));
        if (best < 0 || sc > bs) {
            bs = sc;
            best = j;
        }
    }
    if (best < 0) best = orc_draw_row(zp, V, c, sp, seed, step, b, i, ORC_U_GUMBEL_RESAMPLE, NULL, 0);
    return best;
}

void orc_accept_chain(const float* target, const float* draft, const int32_t* drafts, int B, int k, int V,
                      float temperature, float top_p, uint64_t seed, uint32_t step, int32_t* accepted_len,
                      int32_t* out_tokens) {
    const int greedy = !(temperature > 0.0f);
    const float c = greedy ? 0.0f : temp_coeff(temperature);
    const uint64_t tp = top_p_q32(top_p);
#pragma omp parallel for schedule(dynamic)
    for (int b = 0; b < B; ++b) {
        const float* P = target + (size_t)b * (k + 1) * V;
        const float* Q = draft + (size_t)b * k * V;
        const int32_t* D = drafts + (size_t)b * k;
        int32_t* out = out_tokens + (size_t)b * (k + 1);
        int a = 0, tok;
        if (greedy) {
            while (a < k && orc_argmax(P + (size_t)a * V, V) == D[a]) ++a;
            tok = orc_argmax(P + (size_t)a * V, V);
        } else {
            orc_row_stats sp, sq;
            for (;;) {
                if (a == k) {
                    orc_row_stats_compute(P + (size_t)k * V, V, c, tp, &sp);
                    tok = orc_draw_row(P + (size_t)k * V, V, c, &sp, seed, step, (uint32_t)b, (uint32_t)k,
                                       ORC_U_GUMBEL_RESAMPLE, NULL, 0);
                    break;
                }
                const float* zp = P + (size_t)a * V;
                const float* zq = Q + (size_t)a * V;
                orc_row_stats_compute(zp, V, c, tp, &sp);
                orc_row_stats_compute(zq, V, c, tp, &sq);
                int x = D[a];
                uint64_t ep = (x >= 0 && x < V) ? orc_row_mass(zp, &sp, c, x) : 0;
                uint64_t eq = (x >= 0 && x < V) ? orc_row_mass(zq, &sq, c, x) : 0;
                uint32_t u = orc_uniform_u32(seed, step, b, a, ORC_U_ACCEPT);
                u128 lhs = (u128)u * eq * sp.nuc;
                u128 rhs = ((u128)ep * sq.nuc) << 32;
                if (lhs < rhs) { ++a; continue; }
                tok = draw_residual(zp, &sp, zq, &sq, V, c, seed, step, (uint32_t)b, (uint32_t)a);
                break;
            }
        }
        for (int i = 0; i < a; ++i) out[i] = D[i];
        out[a] = tok;
        for (int i = a + 1; i <= k; ++i) out[i] = -1;
        accepted_len[b] = a;
    }
}

void orc_accept_tree(const float* target, const int32_t* node_tokens, const int32_t* parent, int B, int R, int V,
                     float temperature, float top_p, uint64_t seed, uint32_t step, int32_t* accepted_len,
                     int32_t* path_nodes, int32_t* out_tokens) {
    const int greedy = !(temperature > 0.0f);
    const float c = greedy ? 0.0f : temp_coeff(temperature);
    const uint64_t tp = top_p_q32(top_p);
#pragma omp parallel for schedule(dynamic)
    for (int b = 0; b < B; ++b) {
        const float* P = target + (size_t)b * R * V;
        const int32_t* tok = node_tokens + (size_t)b * R;
        int32_t* path = path_nodes + (size_t)b * R;
        int32_t* out = out_tokens + (size_t)b * R;
        int cur = 0, a = 0, emit = -1;
        for (int i = 0; i < R; ++i) { path[i] = -1; out[i] = -1; }
        for (;;) {
            const float* z = P + (size_t)cur * V;
            int next = -1;
            if (greedy) {
                int best = orc_argmax(z, V);
                for (int ch = cur + 1; ch < R; ++ch)
                    if (parent[ch] == cur && tok[ch] == best) { next = ch; break; }
                if (next < 0) { emit = best; break; }
            } else {
                orc_row_stats st;
                orc_row_stats_compute(z, V, c, tp, &st);
                uint64_t remaining = st.nuc;
                /* removed tokens of rejected siblings */
                int removed[64];
                int n_removed = 0;
                for (int ch = cur + 1; ch < R && next < 0; ++ch) {
                    if (parent[ch] != cur) continue;
                    int x = tok[ch];
                    uint64_t e = (x >= 0 && x < V) ? orc_row_mass(z, &st, c, x) : 0;
                    int dup = 0;
                    for (int t = 0; t < n_removed; ++t) dup |= removed[t] == x;
                    if (dup) e = 0;
                    uint32_t u = orc_uniform_u32(seed, step, b, (uint32_t)ch, ORC_U_ACCEPT);
                    if ((u128)u * remaining < ((u128)e << 32)) { next = ch; break; }
                    if (!dup && n_removed < 64) removed[n_removed++] = x;
                    remaining -= e;
                }
                if (next < 0) {
                    /* P without the rejected children's tokens; all of P when they cover it */
                    emit = orc_draw_row(z, V, c, &st, seed, step, (uint32_t)b, (uint32_t)cur, ORC_U_GUMBEL_RESAMPLE,
                                        removed, remaining ? n_removed : 0);
                    break;
                }
            }
            path[a] = next;
            out[a] = tok[next];
            ++a;
            cur = next;
        }
        out[a] = emit;
        accepted_len[b] = a;
    }
}

void orc_sample_rows(const float* logits, int rows, int k, int V, float temperature, float top_p, uint64_t seed,
                     uint32_t step, int32_t* out) {
    const int greedy = !(temperature > 0.0f);
    const float c = greedy ? 0.0f : temp_coeff(temperature);
    const uint64_t tp = top_p_q32(top_p);
#pragma omp parallel for schedule(dynamic)
    for (int r = 0; r < rows; ++r) {
        const float* z = logits + (size_t)r * V;
        if (greedy) { out[r] = orc_argmax(z, V); continue; }
        orc_row_stats st;
        orc_row_stats_compute(z, V, c, tp, &st);
        out[r] = orc_draw_row(z, V, c, &st, seed, step, (uint32_t)(r / k), (uint32_t)(r % k), ORC_U_GUMBEL_DRAFT,
                              NULL, 0);
    }
}

/* ---------------------------------------------- reference compatibility */
int orc_compat_argmax(const float* z, int V, int vl, int default_idx) {
    /* lane l scans indices l, l+vl, ... with strict '>' from -inf, initial index = l */
    float lane_max[64];
    int lane_idx[64];
    if (vl > 64) vl = 64;
    for (int l = 0; l < vl; ++l) { lane_max[l] = -INFINITY; lane_idx[l] = l; }
    for (int j = 0; j < V; ++j) {
        int l = j % vl;
        if (z[j] > lane_max[l]) { lane_max[l] = z[j]; lane_idx[l] = j; }
    }
    float g = -INFINITY;
    for (int l = 0; l < vl; ++l) g = fmaxf(g, lane_max[l]);
    for (int l = 0; l < vl; ++l)
        if (lane_max[l] == g) return lane_idx[l];
    return default_idx;
}

void orc_compat_verify(const float* logits, const int32_t* drafts, const int32_t* lens, int V, int max_draft,
                       int B, int vl, int32_t* accepted, int32_t* replacement) {
    for (int b = 0; b < B; ++b) {
        int d = lens[b];
        if (d <= 0) { accepted[b] = 0; replacement[b] = -1; continue; }
        if (d > 8) d = 8; /* best_tokens[8] in the reference */
        int best[8];
        for (int i = 0; i < d; ++i)
            best[i] = orc_compat_argmax(logits + ((size_t)b * max_draft + i) * V, V, vl, -1);
        int cnt = 0, any_mismatch = 0;
        for (int i = 0; i < d; ++i) {
            if (best[i] == drafts[(size_t)b * max_draft + i]) ++cnt;
            else any_mismatch = 1;
        }
        accepted[b] = cnt;
        replacement[b] = any_mismatch ? best[cnt] : -1;
    }
}

void orc_compat_mtp_predict(const float* h, const float* W, float* out, int H, int V, int K) {
#pragma omp parallel for
    for (int kk = 0; kk < K; ++kk) {
        for (int j = 0; j < V; ++j) {
            float acc = 0.0f;
            for (int d = 0; d < H; ++d) acc += h[d] * W[((size_t)kk * H + d) * V + j];
            out[(size_t)kk * V + j] = acc;
        }
    }
}

void orc_compat_mtp_sample(const float* logits, int32_t* out, int V, int K, int vl) {
    for (int kk = 0; kk < K; ++kk) out[kk] = orc_compat_argmax(logits + (size_t)kk * V, V, vl, 0);
}
