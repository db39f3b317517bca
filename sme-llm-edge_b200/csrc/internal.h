// internal.h -- declarations shared between the translation units of the
// library (not part of the C ABI).  Every .cu file that defines or calls one
// of these includes this header, so a signature or struct layout that drifts
// between files is a compile error instead of a silent mismatch.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "specdec.h"

namespace specdec {

// ---------------------------------------------------------------- W4A16 GEMM
struct GemmPlan {
    int MT;       // token tile
    int m_tiles;  // token tiles
    int QN;       // 128-row weight units per CTA (1 or 2)
    int n_tiles;  // weight tiles of 128 * QN rows
    int KG;       // 128-wide k steps
    int S;        // CTAs per tile (cluster size, split of the k range)
    int grid;     // CTAs launched
};
GemmPlan plan_gemm(int M, int N, int K);
int make_x_tmap(CUtensorMap* map, const void* X, int M, int K, int ldx, int MT);
// pdl: launch as a programmatic dependent of the previous kernel in the stream
// (its weight stream starts before that kernel has finished; only for weights
// that no kernel in flight writes).
int gemm_launch(const CUtensorMap& map, const GemmPlan& p, const void* w_tiled, int M, int N, float* Y, int ldy,
                int mode, void* ws, cudaStream_t s, bool pdl = false);
// Fused gate/up GEMM with the SwiGLU epilogue: h[m, f] = fp16(silu(g) * u)
// for f < F, from weights whose 256-row tile t holds gate rows 128t .. 128t+127
// then the up rows of the same features (zero rows past F): swiglu_units(F)
// 128-row units.
int swiglu_units(int F);
GemmPlan plan_gemm_swiglu(int M, int F, int K);
int gemm_launch_swiglu(const CUtensorMap& map, const GemmPlan& p, const void* w_gu, int M, int F, __half* h, int ldh,
                       cudaStream_t s, bool pdl = false);
// Fused QKV projection + RoPE + KV-cache write: the epilogue of the one-unit
// tiles (each tile = 128 / hd whole heads of [q | k | v]) applies rotate-half
// RoPE (pairs d, d + hd/2, cos/sin tables [pos][hd/2]) to q and k, writes q as
// fp16 [M, Hq*hd] and k / v as fp16 into the paged slots of kv_layer
// ([num_blocks][2][Hkv][16][hd]); no fp32 output.  hd must divide 128.
struct RopeArgs {
    const int32_t* pos;     // [M] positions
    const int32_t* slot;    // [M] KV slot (token index within the sequence)
    const int32_t* tables;  // [B, max_blocks]
    int max_blocks, R;      // R = rows per sequence
    const float* cos_t;     // [max_pos][hd/2]
    const float* sin_t;
    int Hq, Hkv, hd;
    __half* kv_layer;
    __half* q16;
};
GemmPlan plan_gemm_qkv(int M, int N, int K);
int gemm_launch_qkv_rope(const CUtensorMap& map, const GemmPlan& p, const void* w_qkv, int M, int N, const RopeArgs& ra,
                         cudaStream_t s, bool pdl = false);
size_t gemm_workspace_bound(int max_m, int max_n, int max_k);

// W4A16 contraction for few token rows (gemv_w4a16.cu): mode 0 store / 1 add,
// 1 <= M <= kGemvMaxRows.  plan_gemm_uses_gemv() is the crossover the planner
// applies (measured against the tcgen05 tiles: up to 16 rows).
constexpr int kGemvMaxRows = 64;
struct GemvPlan {
    int NT;      // tiles of 8 token rows
    int KG;      // 128-wide k units
    int blocks;  // 128-row unit blocks
    int S;       // CTAs per unit block (cluster split of the k range)
    int grid;
};
GemvPlan plan_gemv(int M, int N, int K);
bool plan_gemm_uses_gemv(int M, int N, int K);
int gemv_launch(const __half* X, int ldx, int K, const GemvPlan& p, const void* w_tiled, int M, int N, float* Y,
                int ldy, int mode, cudaStream_t s, bool pdl = false);
size_t w4_tiled_bytes(int N, int K);

// ---------------------------------------------------------------- attention
size_t attention_workspace(int B, int R, int Hq, int Hkv, int HD, int max_ctx);
int launch_attention(const __half* q, const __half* kv_layer, int num_blocks, int Hkv, int HD, const int32_t* tables,
                     int max_blocks, const int32_t* ctx_len, const uint64_t* mask, int B, int R, int Hq, __half* out,
                     void* ws, size_t ws_bytes, int max_ctx, cudaStream_t s);

// ---------------------------------------------------------------- sampling / acceptance
constexpr size_t kAcceptStatsBytes = 32;  // one logits row's statistics in the acceptance scratch
int launch_topk(const float* logits, int rows, int V, int k, int32_t* out, cudaStream_t s);
float temp_coeff(float temperature);
uint64_t top_p_q32(float top_p);
int launch_accept_chain_dev(const float* target, const float* draft, const int32_t* drafts, int B, int k, int V,
                            float temperature, float top_p, uint64_t seed, const uint32_t* step_dev,
                            int32_t* accepted_len, int32_t* out_tokens, void* ws, bool draft_stats_ready,
                            cudaStream_t s);
int launch_accept_tree_dev(const float* target, const int32_t* node_tokens, const int32_t* parent, int B, int R, int V,
                           float temperature, float top_p, uint64_t seed, const uint32_t* step_dev,
                           int32_t* accepted_len, int32_t* path, int32_t* out_tokens, cudaStream_t s);
int launch_sample_rows_dev(const float* logits, int rows, int k, int V, float temperature, float top_p, uint64_t seed,
                           const uint32_t* step_dev, int32_t* out, void* stats, cudaStream_t s);

// ---------------------------------------------------------------- paged KV block manager
struct KVState {
    int num_blocks, block_size, max_reqs, max_bpr;
    int32_t* tables;   // [max_reqs, max_bpr], -1 padded
    int32_t* nblk;     // [max_reqs], -1 = no table
    int32_t* len;      // [max_reqs]
    int32_t* ref;      // [num_blocks]
    int32_t* ctx;      // [max_reqs] length before the last batch append
    int32_t* scratch;  // [max(num_blocks, max_reqs) * 4]
    int32_t* status;   // [1] ENOMEM flag of the last batch append
};
KVState& kv_state(specdec_kv* kv);
// requests r0 .. r0 + n - 1 each append `tokens` tokens
int kv_append_uniform(specdec_kv* kv, int n, int tokens, cudaStream_t s, int r0 = 0);
int kv_truncate_dev(specdec_kv* kv, const int32_t* new_len_dev, int n, cudaStream_t s);

// ------------------------------------------------------------ .sme weights
// Rows of a source weight on the device: int8 with the writer's per-row
// factor (value = q / rs) or fp32; fold = optional per-column multiplier
// (an RMSNorm weight folded into the following projection).
struct W4Source {
    const int8_t* q8;
    const float* rs;
    const float* f32;
    const float* fold;
    int K;
};
// Source rows -> tiled W4 units (KG = ceil(K / 128) units per 128 rows).
// layout 0: source row r is row row0 + r; 1 / 2: gate / up half of the fused
// SwiGLU weight (row0 = 0).
int w4_convert_launch(const W4Source& src, int rows, int row0, int layout, uint8_t* tiled, int KG, cudaStream_t s);
int w4_fill_zero_launch(uint8_t* tiled, size_t units, cudaStream_t s);
int f16_rows_launch(const W4Source& src, int rows, __half* out, cudaStream_t s);
// The tensor of a role of a .sme file ("embed", "norm", "lm_head", "q", "k",
// "v", "o", "gate", "up", "down", "attn_norm", "ffn_norm", "mtp",
// "mtp_norm") for layer / head `layer`; false when the file has none.
bool sme_role_view(const specdec_sme* f, const char* role, int layer, specdec_sme_tensor* out);
// Copies a file tensor to the device through `stage` in row chunks and
// converts it: into tiled W4 rows (row0 / layout as w4_convert_launch, fold =
// device f32 [K] or null) or, with f16 non-null, into fp16 rows.
int sme_upload_convert(const specdec_sme_tensor& t, const float* fold, uint8_t* tiled, int KG, int row0, int layout,
                       __half* f16, uint8_t* stage, size_t stage_bytes, cudaStream_t s);

}  // namespace specdec
