/*
 * oracle.h -- CPU restatement of the speculative-decoding hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * implementation in sme-llm-edge_b200/csrc.  Only tests/, the smoke() entry
 * of __graft_entry__.py and the cpu_baseline / --impl reference legs of
 * bench.py may load it.  The product path never calls into it.
 *
 * Reference anchors (paths inside the Soumyadeeps006/sme-llm-edge tree):
 *   - greedy verify, count-matches rule and SVE lane tie rule:
 *       src/sme_kernel/rust_sme/src/lib.rs:696-779
 *   - MTP head GEMV / per-head argmax: lib.rs:1792-1886
 *   - RMSNorm / softmax: lib.rs:21-55 ; RoPE rotate-half: lib.rs:621-663
 *   - SwiGLU: lib.rs:393-457, server/main.cpp:246-249,325-344
 *   - split-KV chunk / combine math: lib.rs:1638-1783 ; GQA head map lib.rs:841-842
 *   - reference paged attention formula: server/paged_attention.cpp:16-111
 *   - int4 packing (offset binary, low nibble = even k): server/sve_packing.cpp:8-30
 *   - block allocator / tables: server/paged_kv_cache.cpp:50-228
 *   - verify-forward shape: server/main.cpp:252-370
 * New math with no reference counterpart (parity unpinned against the
 * reference, pinned against published algorithms and known-answer tests):
 *   - Philox4x32-10 counter RNG (Salmon et al., SC'11)
 *   - rejection-sampling acceptance min(1,p/q) with residual max(0,p-q)
 *     (Leviathan et al. 2023; Chen et al. 2023)
 *   - temperature + top-p nucleus, tree ancestor mask (SpecInfer, Miao et al. 2023)
 *   - int4 group-128 fp16-scale weights
 */
#ifndef SPECDEC_ORACLE_H
#define SPECDEC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- common */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_f16_n(const float* src, uint16_t* dst, size_t n);
void orc_f16_to_f32_n(const uint16_t* src, float* dst, size_t n);

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as
 * easy as 1, 2, 3", SC 2011). */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);

/* floor(2^t * 2^31) for t <= 0 (t > 0 and NaN treated as 0), computed with a
 * fixed sequence of IEEE operations so that host and device agree bit for bit:
 * n = rint(t), f = t - n, 2^f = e^(f ln2) by a degree-7 Taylor polynomial in
 * Horner form with fused multiply-adds, then an exact power-of-two scaling. */
uint32_t orc_exp2_fx31(float t);

/* Order-preserving map of an fp32 logit onto uint32 (larger logit -> larger key). */
uint32_t orc_logit_key(float z);

/* ------------------------------------------------------- sampling / accept */
/* Per-row statistics of softmax(z / T) restricted to the top-p nucleus.
 *   c     = log2(e) / T, rounded to fp32 by the caller
 *   top_p = top-p in Q32 fixed point (2^32 means 1.0 / nucleus disabled)
 * E_j   = orc_exp2_fx31((z_j - max) * c)
 * sum   = sum_j E_j (exact integer)
 * tau   = largest key such that sum_{key_j >= tau} E_j >= max(1, sum*top_p>>32)
 * nuc   = sum_{key_j >= tau} E_j ; nucleus = { j : key_j >= tau } */
typedef struct {
    float max;
    uint32_t tau;
    uint64_t sum;
    uint64_t nuc;
} orc_row_stats;

void orc_row_stats_compute(const float* z, int V, float c, uint64_t top_p_q32, orc_row_stats* st);
/* E of token x under the row statistics (0 outside the nucleus). */
uint32_t orc_row_mass(const float* z, const orc_row_stats* st, float c, int x);
/* Draw (exponential race) from the nucleus distribution (weights E_j) of row z with
 * the element uniforms of draw (seed, step, b, i, purpose), the tokens
 * excl[0 .. n_excl) left out; -1 when no token has weight.  See
 * orc_sample.c for the arithmetic. */
int orc_draw_row(const float* z, int V, float c, const orc_row_stats* st, uint64_t seed, uint32_t step, uint32_t b,
                 uint32_t i, uint32_t purpose, const int32_t* excl, int n_excl);
/* The pieces: log2 by the atanh series, -log2 of a Philox uniform, the
 * uniform of element j of a draw, and a candidate's race key w / (-log2 U). */
float orc_det_log2(float x);
float orc_neg_log2_uniform(uint32_t x);
uint32_t orc_gumbel_uniform(uint64_t seed, uint32_t step, uint32_t b, uint32_t i, uint32_t purpose, uint32_t j);
float orc_race_key(float w, uint32_t u);
/* Lowest index of the maximum (NaN never wins); -1 if V == 0. */
int orc_argmax(const float* z, int V);
/* Maximum and the second maximum (value of the best other index). */
void orc_top2(const float* z, int V, float* top1, float* top2);
/* Top-k indices, descending value, ascending index on ties. */
void orc_topk(const float* z, int V, int k, int* out);

/* Uniform streams.  ctr = {b, i, purpose, step}, key = {seed_lo, seed_hi}.
 * purpose 1 = accept test; the draws use one uniform per element:
 * 3 = draft sampling, 4 = residual / bonus / tree draw (orc_gumbel_uniform). */
enum { ORC_U_ACCEPT = 1, ORC_U_GUMBEL_DRAFT = 3, ORC_U_GUMBEL_RESAMPLE = 4 };
uint32_t orc_uniform_u32(uint64_t seed, uint32_t step, uint32_t b, uint32_t i, uint32_t purpose);
uint64_t orc_uniform_u64(uint64_t seed, uint32_t step, uint32_t b, uint32_t i, uint32_t purpose);

/* Chain acceptance (standard speculative sampling).
 *   target [B, k+1, V] fp32 logits, draft [B, k, V] fp32 logits,
 *   drafts [B, k] int32.  temperature == 0 selects greedy acceptance.
 * Outputs accepted_len[B] and out_tokens[B, k+1] (accepted drafts, then the
 * corrected / bonus token, then -1 padding). */
void orc_accept_chain(const float* target, const float* draft, const int32_t* drafts, int B, int k, int V,
                      float temperature, float top_p, uint64_t seed, uint32_t step, int32_t* accepted_len,
                      int32_t* out_tokens);

/* Tree acceptance.  Nodes 0..R-1 in BFS order, node 0 = root (the pending
 * token), parent[0] = -1, node_tokens[B, R].  target [B, R, V].  Candidates of
 * a node are its children in index order and are deterministic (top-b of an
 * MTP head), so each is tested as a point-mass draft: accept child c with
 * probability P(c) / (1 - sum of P over already rejected siblings); after all
 * children are rejected the token is drawn from P with the rejected tokens
 * removed.  Greedy when temperature == 0.
 * Outputs accepted_len[B] (path length excluding root), path_nodes[B, R]
 * (node indices of the accepted path, root excluded), out_tokens[B, R]
 * (path tokens then the emitted token, -1 padded). */
void orc_accept_tree(const float* target, const int32_t* node_tokens, const int32_t* parent, int B, int R, int V,
                     float temperature, float top_p, uint64_t seed, uint32_t step, int32_t* accepted_len,
                     int32_t* path_nodes, int32_t* out_tokens);

/* Draft-token sampling from draft logits rows [rows, V] (purpose 3 draw,
 * b = row / k, i = row % k).  temperature == 0 -> argmax. */
void orc_sample_rows(const float* logits, int rows, int k, int V, float temperature, float top_p, uint64_t seed,
                     uint32_t step, int32_t* out);

/* ------------------------------------------------ reference compatibility */
/* Argmax as sve2_speculative_verify_f32 / rust_sme_mtp_sample_f32 compute it
 * for an SVE vector of `vl` fp32 lanes: strict '>' per lane keeps the earliest
 * index of each lane, the winner is the lowest lane whose lane maximum equals
 * the global maximum (lib.rs:717-749, 1853-1883). */
int orc_compat_argmax(const float* z, int V, int vl, int default_idx);
/* sve2_speculative_verify_f32 (lib.rs:696-779): count of matching positions,
 * replacement = best[count] when any position mismatches, else -1. */
void orc_compat_verify(const float* logits, const int32_t* drafts, const int32_t* lens, int V, int max_draft,
                       int B, int vl, int32_t* accepted, int32_t* replacement);
/* rust_sme_mtp_predict_f32 (lib.rs:1792-1831): logits[k,j] = sum_d h[d] W[k,d,j]. */
void orc_compat_mtp_predict(const float* h, const float* W, float* out, int H, int V, int K);
/* rust_sme_mtp_sample_f32 (lib.rs:1840-1886). */
void orc_compat_mtp_sample(const float* logits, int32_t* out, int V, int K, int vl);
/* compute_paged_attention (server/paged_attention.cpp:16-111), flattened
 * tables: request m owns tables[table_off[m] .. table_off[m+1]). Adds into o. */
void orc_compat_paged_attention(const float* q, const float* k_pool, const float* v_pool, const int32_t* table_off,
                                const int32_t* tables, const int32_t* seq_lens, float* o, int M, int H, int bs);
/* rust_sme_flashdecoding_chunk_f32 / rust_sve2_flashdecoding_reduce_f32. */
void orc_flashdecoding_chunk(const float* q, const float* k, const float* v, int len, int hd, float scale,
                             float* part_o, float* part_max, float* part_sum);
void orc_flashdecoding_reduce(const float* part_o, const float* part_max, const float* part_sum, int chunks, int hd,
                              float* out);

/* ---------------------------------------------------------- model pieces */
typedef struct {
    int hidden, layers, n_q_heads, n_kv_heads, head_dim, ffn, vocab;
    int n_mtp_heads;
    int block_size;
    float rms_eps;
    float rope_theta;
} orc_model_cfg;

/* Tensor ids for the synthetic weight generator. */
enum {
    ORC_T_Q = 0, ORC_T_K = 1, ORC_T_V = 2, ORC_T_O = 3, ORC_T_GATE = 4, ORC_T_UP = 5, ORC_T_DOWN = 6,
    ORC_T_EMB = 0x10000, ORC_T_LM = 0x10001, ORC_T_MTP0 = 0x10010
};
static inline uint32_t orc_layer_tensor(int layer, int which) { return (uint32_t)(layer * 16 + which); }

/* Synthetic N(0, 0.02) draw for element e of tensor `tid`: Irwin-Hall sum of
 * four 24-bit Philox uniforms, centred and scaled to unit variance, times 0.02.
 * Exact in binary64 so host and device draw identical values. */
float orc_synth_value(uint32_t seed, uint32_t tid, uint64_t e);
/* Quantise rows [n0, n0+n) of an [N, K] tensor to int4 with group-128 fp16
 * scales: s = fp16(amax/7), q = clamp(round(w/s), -8, 7), u4 = q + 8.
 * packed is [n, K/2] (low nibble = even k), scales [n, K/128]. */
void orc_synth_w4(uint32_t seed, uint32_t tid, int N, int K, int n0, int n, uint8_t* packed, uint16_t* scales);
void orc_synth_f16(uint32_t seed, uint32_t tid, uint64_t e0, size_t n, uint16_t* out);
/* The same quantiser over given rows w [n, K] (K even): packed [n, K/2],
 * scales [n, K/128]. */
void orc_w4_quantize(const float* w, int n, int K, uint8_t* packed, uint16_t* scales);
/* Dequantise int4 rows to fp16-rounded fp32 values. */
void orc_w4_dequant(const uint8_t* packed, const uint16_t* scales, int N, int K, float* out);
/* Y[m,n] (op)= sum_k X[m,k] * Wdq[n,k]; X fp16 [M,K]; accumulate in fp32.
 * mode 0: store, 1: add into Y. */
void orc_w4a16_gemm(const uint16_t* X, int M, const uint8_t* packed, const uint16_t* scales, int N, int K, float* Y,
                    int ldy, int mode);
void orc_rmsnorm_f16(const float* x, const float* w, int n, float eps, uint16_t* out);
void orc_rope_tables(int max_pos, int head_dim, float theta, float* cos_t, float* sin_t);

/* Paged fp16 KV cache: pool[L][num_blocks][2][Hkv][bs][hd]. */
typedef struct {
    int layers, num_blocks, n_kv_heads, block_size, head_dim;
    uint16_t* pool;
} orc_kv_pool;
static inline size_t orc_kv_offset(const orc_kv_pool* p, int layer, int blk, int kv, int h, int slot) {
    return ((((size_t)layer * p->num_blocks + blk) * 2 + kv) * p->n_kv_heads + h) * ((size_t)p->block_size * p->head_dim)
           + (size_t)slot * p->head_dim;
}

/* Verify attention for R new rows per sequence.
 * q [B*R, Hq, hd] fp16; output [B*R, Hq, hd] fp16.
 * Sequence b attends over slots 0..ctx_len[b]-1 (always visible) and the new
 * slots ctx_len[b]+j, j < R, visible to row r iff bit j of mask[r] is set
 * (chain: mask[r] = (2^(r+1))-1).  Exact softmax with max subtraction. */
void orc_attention(const uint16_t* q, const orc_kv_pool* kv, int layer, const int32_t* tables, int max_blocks,
                   const int32_t* ctx_len, const uint64_t* mask, int B, int R, int Hq, uint16_t* out);

/* Whole-model weights (logical, untiled). */
typedef struct {
    orc_model_cfg cfg;
    uint16_t* emb;                       /* [V, H] fp16 */
    uint8_t* w_packed[7];                /* per layer, concatenated over layers */
    uint16_t* w_scales[7];
    uint8_t* lm_packed; uint16_t* lm_scales;
    uint8_t* mtp_packed; uint16_t* mtp_scales; /* [n_mtp, H, H] */
    float* rope_cos; float* rope_sin; int rope_max_pos;
    int n_layers_present;                /* layers actually generated (CPU baseline samples fewer) */
} orc_model;

orc_model* orc_model_create(const orc_model_cfg* cfg, uint32_t seed, int n_layers_present, int rope_max_pos);
void orc_model_free(orc_model* m);

/* Verify forward of R rows per sequence (chain or tree).
 * tokens/pos/slot are [B*R]; rows of sequence b are b*R .. b*R+R-1.
 * Writes K/V of every row into its slot, then attends with `mask`.
 * Outputs logits [B*R, V] fp32 (may be NULL) and final hidden (pre final
 * norm) [B*R, H] fp32 (may be NULL).  n_layers < 0 means all. */
void orc_forward(const orc_model* m, orc_kv_pool* kv, const int32_t* tables, int max_blocks, const int32_t* ctx_len,
                 const int32_t* tokens, const int32_t* pos, const int32_t* slot, const uint64_t* mask, int B, int R,
                 int n_layers, float* logits, float* hidden_out);

/* Chained MTP drafting: h_{i+1} = W_head[min(i,n_mtp-1)] . rmsnorm(h_i),
 * logits_i = W_lm . rmsnorm(h_{i+1}).  h0 [B, H] fp32.
 * Outputs draft_logits [B, k, V] and sampled drafts [B, k]; hid_out [B,k,H] optional. */
void orc_draft_chain(const orc_model* m, const float* h0, int B, int k, float temperature, float top_p, uint64_t seed,
                     uint32_t step, float* draft_logits, int32_t* drafts, float* hid_out);

/* ---------------------------------------------- block manager (reference) */
/* Restatement of PagedKVCache's table logic (paged_kv_cache.cpp:50-228):
 * lowest-free-index allocation with reference counts, append with OOM stop,
 * free, prefix share, tail-block free / evict. */
typedef struct orc_blockmgr orc_blockmgr;
orc_blockmgr* orc_bm_create(int num_blocks, int block_size, int max_reqs, int max_blocks_per_req);
void orc_bm_free(orc_blockmgr* bm);
int orc_bm_append(orc_blockmgr* bm, int req, int n_tokens);          /* returns last block written or -1 */
void orc_bm_free_request(orc_blockmgr* bm, int req);
void orc_bm_share_prefix(orc_blockmgr* bm, int new_req, int src_req, int shared_len);
void orc_bm_free_tail_blocks(orc_blockmgr* bm, int req, int n_blocks);   /* free_merged_blocks */
int orc_bm_evict_tokens(orc_blockmgr* bm, int req, int n_tokens);       /* evict_least_important_blocks */
void orc_bm_truncate(orc_blockmgr* bm, int req, int new_len);           /* token-granular rollback */
float orc_bm_utilization(const orc_blockmgr* bm);
int orc_bm_table(const orc_blockmgr* bm, int req, int32_t* blocks, int cap, int32_t* len); /* returns n blocks */
int orc_bm_refcount(const orc_blockmgr* bm, int blk);

/* Tree shape helper: BFS tree with per-level branching, truncated to max_nodes
 * (root included).  Fills parent, depth, child rank and ancestor masks. */
int orc_tree_build(const int* branching, int levels, int max_nodes, int32_t* parent, int32_t* depth, int32_t* rank,
                   uint64_t* anc_mask);

#ifdef __cplusplus
}
#endif
#endif
