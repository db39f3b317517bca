/*
 * specdec.h -- C ABI of libspecdec_sm100.so, the B200 (sm_100a) speculative-
 * decoding hot path of the sme-llm-edge server.
 *
 * Two groups of entry points:
 *
 *  1. The reference's FFI symbols, with the reference's exact signatures and
 *     host-pointer semantics, so the unchanged reference C++ operator classes
 *     (server/speculative_decoder.cpp, server/mtp_heads.cpp,
 *     server/paged_kv_cache.cpp) link against this library instead of the Rust
 *     SVE2/SME library (src/sme_kernel/rust_sme/src/lib.rs).  They stage their
 *     inputs to the GPU, run a CUDA kernel and copy results back.  They return
 *     void like the reference; failures leave the reference's default outputs
 *     and are reported through specdec_last_error().
 *
 *  2. Device-resident entry points (specdec_*): device pointers, an explicit
 *     cudaStream_t (passed as void*), int status return.  These are the fast
 *     path used by the step engine.
 *
 * No torch types appear here; plain pointers and sizes only.
 */
#ifndef SPECDEC_H
#define SPECDEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------- status */
enum {
    SPECDEC_OK = 0,
    SPECDEC_EINVAL = 1,   /* bad argument / shape */
    SPECDEC_ENOMEM = 2,   /* device memory or KV block pool exhausted */
    SPECDEC_ECUDA = 3,    /* CUDA runtime / launch error */
    SPECDEC_ETIMEOUT = 4, /* a bounded device-side wait gave up */
    SPECDEC_ENOTSUP = 5,  /* feature not available on this device */
    SPECDEC_EFORMAT = 6,  /* malformed or truncated .sme model file */
    SPECDEC_EIO = 7       /* model file cannot be opened or mapped */
};
/* Last error message of the calling thread ("" if none). */
const char* specdec_last_error(void);
int specdec_abi_version(void);
/* Failure-path self-test: launches one thread that waits on an mbarrier phase
 * no thread completes, with the bounded wait every TMA / tensor-core kernel of
 * the library uses (about 2 s of wall time).  The wait gives up, the kernel
 * records SPECDEC_ETIMEOUT in the device status word and returns; the call
 * reads the word back on `stream` and returns SPECDEC_ETIMEOUT (message
 * "device-side wait gave up at site 90").  The status word is cleared and the
 * context stays usable.  No fault, trap or unbounded wait is involved. */
int specdec_selftest_wait_timeout(void* stream);

/* ===================================================================== */
/* 1. Reference FFI symbols (host pointers).                               */
/* ===================================================================== */

/* Replaces sve2_speculative_verify_f32, src/sme_kernel/rust_sme/src/lib.rs:696-779
 * (declared by the reference at server/speculative_decoder.cpp:5-16).
 * logits [batch, max_draft_length, vocab]; drafts [batch, max_draft_length];
 * accepted = number of positions i < len[b] whose argmax equals the draft
 * (count, not prefix); replacement = argmax at index `accepted` when any
 * position mismatches, else -1.  Argmax ties follow the reference's 128-bit
 * SVE lane rule (4 fp32 lanes). */
void sve2_speculative_verify_f32(const float* logits_ptr, const int32_t* draft_tokens_ptr,
                                 const int32_t* draft_lengths_ptr, uint32_t vocab_size, uint32_t max_draft_length,
                                 uint32_t batch_size, int32_t* accepted_counts_ptr, int32_t* replacement_tokens_ptr);

/* Replaces rust_sme_mtp_predict_f32, lib.rs:1792-1831 (declared at
 * server/mtp_heads.h:6-13): logits[k, j] = sum_d h[d] * W[k, d, j].
 * The fp32 weights [K, H, V] stay resident on the current device between
 * calls, keyed by host pointer, size and a sampled content fingerprint: a
 * call with the same weights copies only the hidden state in and the logits
 * out.  A caller that edits the weights in place (other than by loading a new
 * checkpoint into the buffer) calls specdec_compat_release_weights first. */
void rust_sme_mtp_predict_f32(const float* hidden_state_ptr, const float* weights_ptr, float* logits_out_ptr,
                              uint32_t hidden_dim, uint32_t vocab_size, uint32_t k_heads);
/* Drops the MTP weights resident on the current device; *uploads (may be
 * NULL) receives the number of weight uploads made so far on that device.
 * No reference counterpart (the Rust kernels read host memory directly). */
int specdec_compat_release_weights(uint64_t* uploads);
/* Number of MTP weight uploads made so far on the current device. */
int specdec_compat_weight_uploads(uint64_t* uploads);

/* Replaces rust_sme_mtp_sample_f32, lib.rs:1840-1886 (server/mtp_heads.h:15-20):
 * per-head argmax with the SVE lane tie rule, default 0. */
void rust_sme_mtp_sample_f32(const float* logits_ptr, int32_t* draft_tokens_out, uint32_t vocab_size,
                             uint32_t k_heads);

/* Replaces sme_sm_prefetch_kv_blocks, lib.rs:670-689 (server/paged_kv_cache.cpp:6-8).
 * A no-op: on the GPU the attention kernel stages KV blocks with bulk async
 * copies, so a host-side prefetch hint has nothing to do. */
void sme_sm_prefetch_kv_blocks(const int8_t** k_ptrs, const int8_t** v_ptrs, uint32_t num_blocks);

/* Replaces rust_sme_flashdecoding_chunk_f32 / rust_sve2_flashdecoding_reduce_f32
 * (lib.rs:1638-1783; declared by server/flash_decoding_tracker.cpp). */
void rust_sme_flashdecoding_chunk_f32(const float* q_ptr, const float* k_chunk_ptr, const float* v_chunk_ptr,
                                      uint32_t chunk_len, uint32_t head_dim, float softmax_scale,
                                      float* partial_o_out, float* partial_max_out, float* partial_sum_exp_out);
void rust_sve2_flashdecoding_reduce_f32(const float* partial_o_ptr, const float* partial_max_ptr,
                                        const float* partial_sum_exp_ptr, uint32_t num_chunks, uint32_t head_dim,
                                        float* final_o_out);

/* C-ABI form of compute_paged_attention (server/paged_attention.h:10-19,
 * server/paged_attention.cpp:16-111), host pointers.  The std::vector
 * arguments are flattened: request m owns tables[table_off[m] .. table_off[m+1]).
 * Adds exp(q.k/sqrt(hidden))/seq_len * v into o, exactly the reference formula
 * (no max subtraction, no normalisation).  Returns a status. */
int specdec_paged_attention_compat_f32(const float* q, const float* k_pool, const float* v_pool, size_t pool_floats,
                                       const int32_t* table_off, const int32_t* tables, const int32_t* seq_lens,
                                       float* o, int M, int hidden_dim, int block_size);

/* ===================================================================== */
/* 2. Device-resident kernels (device pointers, stream as void*).          */
/* ===================================================================== */

/* Sampling parameters.  temperature <= 0 selects greedy decisions; top_p >= 1
 * disables the nucleus.  Uniforms come from Philox4x32-10 with
 * counter {b, i, purpose, step} and key {seed_lo, seed_hi}. */
typedef struct {
    float temperature;
    float top_p;
    uint64_t seed;
    uint32_t step;
} specdec_sampling;

/* Bytes of device scratch the acceptance / sampling kernels need for `rows`
 * logits rows. */
size_t specdec_accept_workspace_bytes(int rows);

/* Chain acceptance (speculative sampling, min(1,p/q) test, residual
 * max(0,p-q) draw, bonus token).  Replaces the reference's greedy verify
 * (lib.rs:696-779) with the standard algorithm; temperature <= 0 gives
 * greedy longest-prefix acceptance.
 *   target [B, k+1, V] fp32, draft [B, k, V] fp32 (unused when greedy),
 *   drafts [B, k] int32 -> accepted_len [B], out_tokens [B, k+1]. */
int specdec_accept_chain(const float* target, const float* draft, const int32_t* drafts, int B, int k, int V,
                         const specdec_sampling* sp, int32_t* accepted_len, int32_t* out_tokens, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Same chain acceptance as specdec_accept_chain, for callers that may not
 * allocate device memory when they accept drafts (a serving loop that reserves
 * its whole memory budget up front, or a host program that owns the GPU
 * allocator).  No counterpart exists in the reference.  The row statistics
 * live in a fixed array compiled into the library: 8192 rows of 32 bytes
 * (256 KB on every GPU that loads the library, held until exit).  Where that
 * array is used -- sampling with top_p < 1, or more than 16 drafts -- B*(k+1)
 * + B*k must not exceed 8192 (B*(k+1) when greedy); larger calls fail with
 * SPECDEC_EINVAL.  Greedy and top_p = 1 acceptance with at most 16 drafts
 * needs no row scratch and takes any batch.  The first call on a device looks up the array's
 * address with that device current and should come before any stream
 * capture.  All calls share the array: calls whose kernels overlap on the
 * GPU race.  No cudaMalloc, cudaFree or allocating library routine is used. */
int specdec_accept_chain_noalloc(const float* target, const float* draft, const int32_t* drafts, int B, int k, int V,
                                 const specdec_sampling* sp, int32_t* accepted_len, int32_t* out_tokens,
                                 void* stream);

/* Tree acceptance over R BFS-ordered nodes (node 0 = root / pending token).
 * target [B, R, V]; node_tokens [B, R]; parent [R] (device).  Outputs
 * accepted_len [B], path_nodes [B, R], out_tokens [B, R]. */
int specdec_accept_tree(const float* target, const int32_t* node_tokens, const int32_t* parent, int B, int R, int V,
                        const specdec_sampling* sp, int32_t* accepted_len, int32_t* path_nodes, int32_t* out_tokens,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Draft-token sampling of logits rows [rows, V]; row r uses stream (r/k, r%k). */
int specdec_sample_rows(const float* logits, int rows, int k, int V, const specdec_sampling* sp, int32_t* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Vocabulary-sharded chain acceptance (the 8-way variant of the acceptance
 * micro-benchmark; replaces verify_drafts_sve2, speculative_decoder.cpp:53-77,
 * when the lm_head is split by vocabulary across GPUs).  Rank w of W holds
 * vocabulary columns [v0, v0 + Vs) of every logits row, ranks in vocabulary
 * order: target shard [B][k+1][Vs], draft shard [B][k][Vs] (row-major, fp32).
 * The caller runs the steps in order and combines across ranks between them
 * (NCCL or any collective); every decision then equals specdec_accept_chain's
 * on the whole rows.  rows_p = B*(k+1) target rows, rows_q = B*k draft rows.
 *  1. specdec_shard_row_max on both shards; all-gather max/arg [W][rows];
 *     specdec_shard_merge_max -> per-row max and arg-max (global index).
 *     Greedy (temperature 0): go to 5 with parg only.
 *  2. specdec_shard_row_mass -> per-row integer mass sums; all-reduce (sum).
 *  3. top_p < 1: for digit 3, 2, 1, 0: specdec_shard_digit_hist (rows x 256
 *     u64); all-reduce (sum); specdec_shard_select_digit -> prefix, G, last.
 *     Then tau = prefix and nuc = G + last; with top_p = 1: tau = 0, nuc = sum.
 *  2'-3'. Instead of 2-3 when top_p < 1 and W <= 8 (one shard pass, two
 *     collectives): specdec_shard_mass_hist -> per row {sum, listed mass,
 *     NaN count, overflow count, 256-bin histogram of t = (z - max) * c over
 *     the listed elements t >= -14} (rows x 260 u64) and this shard's listed
 *     (key, mass) pairs; all-reduce the stats (sum); specdec_shard_cross -> G
 *     and this shard's candidates in the bin where the mass from the top
 *     reaches the threshold (rows x 33 (key, mass) pairs, the last holding the
 *     count); all-gather them [W]; specdec_shard_union_select -> tau, nuc and
 *     ok per row.  ok is 0 for rows with a NaN exponent, a list past `cap`, a
 *     nucleus reaching below t = -14 or more than 32 candidates on a rank:
 *     when any row is not ok (the same answer on every rank), run 2-3 (and
 *     4-7 again).  The flags can be read after 4-7 are queued, so the host
 *     never waits in the middle.
 *  4. specdec_shard_point_mass -> ep, eq [B*k]; all-reduce (sum).
 *  5. specdec_shard_accept_test -> accepted [B] (identical on every rank).
 *     Greedy: the emitted token is parg[b*(k+1) + accepted[b]].
 *  6. specdec_shard_draw_winners -> [B][4] int32, this shard's Gumbel-max
 *     winners of the residual / bonus draw; all-gather [W][B][4].
 *  7. specdec_shard_draw_merge -> the emitted token per sequence (identical on
 *     every rank).
 * The per-row steps (row_max, row_mass, digit_hist) take the target rows
 * (z, rows) and the draft rows (z2, rows2; NULL, 0 when greedy) in one call;
 * their per-row inputs and outputs list the target rows first.  Unsigned
 * 64-bit values may travel as signed 64-bit: every sum stays below 2^63.
 * Shard widths up to 262144; k >= 1. */
int specdec_shard_row_max(const float* z, int rows, const float* z2, int rows2, int Vs, int v0, float* out_max,
                          int32_t* out_arg, void* stream);
int specdec_shard_merge_max(const float* gmax, const int32_t* garg, int W, int rows, float* out_max, int32_t* out_arg,
                            void* stream);
int specdec_shard_row_mass(const float* z, int rows, const float* z2, int rows2, int Vs, const float* gmax,
                           float temperature, uint64_t* out_sum, void* stream);
int specdec_shard_digit_hist(const float* z, int rows, const float* z2, int rows2, int Vs, const float* gmax,
                             float temperature, const uint32_t* prefix, int digit, uint64_t* out_hist, void* stream);
int specdec_shard_select_digit(const uint64_t* hist, int rows, int digit, const uint64_t* gsum, float top_p,
                               uint32_t* prefix, uint64_t* G, uint64_t* last, void* stream);
int specdec_shard_mass_hist(const float* z, int rows, const float* z2, int rows2, int Vs, const float* gmax,
                            float temperature, int cap, void* list, int32_t* list_n, uint64_t* out_stats,
                            void* stream);
int specdec_shard_cross(const uint64_t* stats, int rows, float top_p, const float* gmax, float temperature,
                        const void* list, int cap, const int32_t* list_n, uint64_t* out_G, void* out_cand,
                        void* stream);
int specdec_shard_union_select(const void* gcand, int W, int rows, const uint64_t* stats, const uint64_t* G,
                               float top_p, uint32_t* out_tau, uint64_t* out_nuc, int32_t* out_ok, void* stream);
int specdec_shard_point_mass(const float* target, const float* draft, const int32_t* drafts, int B, int k, int Vs,
                             int v0, float temperature, const float* pmax, const uint32_t* ptau, const float* qmax,
                             const uint32_t* qtau, uint64_t* ep, uint64_t* eq, void* stream);
/* step_dev (may be NULL): a device step counter read instead of sp->step,
 * so that a captured sequence of the steps serves every decoding step. */
int specdec_shard_accept_test(const int32_t* drafts, int B, int k, const specdec_sampling* sp, const int32_t* parg,
                              const uint64_t* pnuc, const uint64_t* qnuc, const uint64_t* ep, const uint64_t* eq,
                              int32_t* accepted, const uint32_t* step_dev, void* stream);
int specdec_shard_draw_winners(const float* target, const float* draft, int B, int k, int Vs, int v0,
                               const specdec_sampling* sp, const int32_t* accepted, const float* pmax,
                               const uint32_t* ptau, const float* qmax, const uint32_t* qtau, const uint64_t* pnuc,
                               const uint64_t* qnuc, int32_t* out_win, const uint32_t* step_dev, void* stream);
int specdec_shard_draw_merge(const int32_t* gwin, int W, int B, int k, const int32_t* accepted, int32_t* tok_out,
                             void* stream);

/* Reference-semantics greedy verify on device pointers (see
 * sve2_speculative_verify_f32 above). */
int specdec_compat_verify(const float* logits, const int32_t* drafts, const int32_t* lens, int V, int max_draft,
                          int B, int32_t* accepted, int32_t* replacement, void* stream);

/* W4A16 weights in the device tiled layout: for every 128-row x 128-column
 * unit, 8192 bytes of nibbles then 128 fp16 group scales (8448 bytes). */
size_t specdec_w4_tiled_bytes(int N, int K);
/* Converts reference-format int4 (packed [N, K/2], low nibble = even k,
 * u4 = q + 8, server/sve_packing.cpp:8-30) plus fp16 group-128 scales
 * [N, K/128] (device pointers) into the tiled layout. */
int specdec_w4_tile(const uint8_t* packed, const uint16_t* scales, int N, int K, void* tiled, void* stream);
int specdec_w4_untile(const void* tiled, int N, int K, uint8_t* packed, uint16_t* scales, void* stream);
/* Y[m, n] = sum_k X[m, k] * W[n, k] (mode 0 store, 1 add).  X fp16 [M, K]
 * (row stride ldx elements, 16-byte aligned), Y fp32 with row stride ldy.
 * Replaces compute_sme_gemm_i4_f32 (server/sme_gemm.cpp:249-285) and the W8
 * GEMV of the model forward (gemv_s8_f32_batched, server/sme_gemm.cpp:41-66)
 * for int4 group-128 weights.  From 17 token rows up, the int4 weights are
 * dequantised in registers and multiplied on the tcgen05 tensor cores with
 * TMEM accumulators; below, the call runs specdec_w4a16_gemv (the measured
 * crossover between the two).  Partial tiles
 * of k-ranges split across the CTAs of a cluster are summed on chip in a
 * fixed order, so the result is deterministic; the workspace
 * (specdec_w4a16_workspace_bytes, 0) is kept for the interface and may be
 * NULL. */
size_t specdec_w4a16_workspace_bytes(int M, int N, int K);
int specdec_w4a16_gemm(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K, float* Y, int ldy,
                       int mode, void* workspace, size_t workspace_bytes, void* stream);
/* The same contraction for 0 <= M <= 64 token rows (decode at small batch,
 * batch-1 steps): each CTA streams 128-row weight units by bulk copy,
 * dequantises them into tensor-core fragments in registers, a cluster splits
 * the k range and reduces in rank order through distributed shared memory.
 * Same results as specdec_w4a16_gemm within fp32 summation order.  Replaces
 * rust_sme_mtp_predict_f32's contraction (lib.rs:1792-1831) for W4A16 heads. */
int specdec_w4a16_gemv(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K, float* Y, int ldy,
                       int mode, void* stream);
/* The launch plan for a shape: out[0] token tile, out[1] 128-row weight
 * units per CTA (1 or 2), out[2] CTAs splitting the k range of a tile (1, 2,
 * 4, 8), out[3] CTAs launched.  units = 0: the plan specdec_w4a16_gemm picks;
 * 1 or 2: the best plan with that many units per CTA (2 is the plan of
 * specdec_w4a16_gemm_swiglu). */
int specdec_w4a16_plan(int M, int N, int K, int units, int32_t* out);
/* specdec_w4a16_gemm with the units per CTA (qn 1 / 2) and the k split
 * (1, 2, 4, 8; <= ceil(K / 128)) fixed by the caller instead of the planner:
 * for validating and timing every path.  Same result up to the order of the
 * k-range sums. */
int specdec_w4a16_gemm_with_plan(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K, float* Y,
                                 int ldy, int mode, int qn, int split, void* stream);
/* Gate/up projection fused with SwiGLU (server/main.cpp:246-249, 338-340):
 * h[m, f] = fp16(silu(g) * u), g = X . gate[f], u = X . up[f], for f < F,
 * h fp16 [M, F] with row stride ldh.  w_gu_tiled holds 256 * ceil(F / 128)
 * rows in the tiled layout: rows 256t .. 256t+127 are gate rows 128t ..
 * 128t+127 and the next 128 the up rows of the same features (rows past F
 * zero: nibbles 8, scale 0).  One launch; g and u never leave the chip. */
int specdec_w4a16_gemm_swiglu(const uint16_t* X, int M, int ldx, const void* w_gu_tiled, int F, int K, uint16_t* h,
                              int ldh, void* stream);
/* Same contraction on the CUDA cores (used to cross-check the tensor path). */
int specdec_w4a16_gemm_simt(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K, float* Y, int ldy,
                            int mode, void* stream);

/* Verify attention over a paged fp16 KV pool [num_blocks, 2, Hkv, 16, hd]
 * (one layer).  q/out [B*R, Hq, hd] fp16.  Row r of sequence b sees slots
 * 0..ctx_len[b]-1 and new slot ctx_len[b]+j iff bit j of mask[r].
 * tables [B, max_blocks] int32.  The workspace is zero-filled by the call. */
size_t specdec_attention_workspace_bytes(int B, int R, int n_q_heads, int n_kv_heads, int head_dim, int max_blocks);
int specdec_attention(const uint16_t* q, const uint16_t* kv_layer, int num_blocks, int n_kv_heads, int head_dim,
                      const int32_t* tables, int max_blocks, const int32_t* ctx_len, const uint64_t* mask, int B,
                      int R, int n_q_heads, uint16_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* ===================================================================== */
/* 3. Paged KV block manager (device resident).  Mirrors PagedKVCache      */
/*    (server/paged_kv_cache.h:28-63): lowest-free-index allocation with   */
/*    reference counts; tables live in device memory.                     */
/* ===================================================================== */
typedef struct specdec_kv specdec_kv;
int specdec_kv_create(int num_blocks, int block_size, int max_reqs, int max_blocks_per_req, specdec_kv** out);
int specdec_kv_destroy(specdec_kv* kv);
/* Appends n_tokens[i] tokens to request reqs[i] for i < n, in order
 * (PagedKVCache::append_tokens).  last_block[i] receives the reference's
 * return value. Host arrays. */
int specdec_kv_append(specdec_kv* kv, const int32_t* reqs, const int32_t* n_tokens, int n, int32_t* last_block,
                      void* stream);
int specdec_kv_free_request(specdec_kv* kv, int req, void* stream);
int specdec_kv_share_prefix(specdec_kv* kv, int new_req, int src_req, int shared_len, void* stream);
int specdec_kv_free_merged_blocks(specdec_kv* kv, int req, int n_blocks, void* stream);
int specdec_kv_evict_tokens(specdec_kv* kv, int req, int n_tokens, int* evicted, void* stream);
/* Token-granular rollback: new lengths (host array, -1 = unchanged); tail
 * blocks past the new length are released. */
int specdec_kv_truncate(specdec_kv* kv, const int32_t* new_len, int n, void* stream);
float specdec_kv_utilization(specdec_kv* kv, void* stream);
/* Copies tables [max_reqs, max_blocks_per_req] (-1 padded), lengths and
 * reference counts to host buffers (any may be NULL). */
int specdec_kv_read(specdec_kv* kv, int32_t* tables, int32_t* lens, int32_t* refcounts, void* stream);
/* Device pointers to the table state (for kernels that read block tables). */
int32_t* specdec_kv_tables_dev(specdec_kv* kv);
int32_t* specdec_kv_lens_dev(specdec_kv* kv);

/* Prefix index of admitted prompts: RadixKVCache (server/radix_kv_cache.h:
 * 16-38, .cpp:39-98) with its per-token semantics -- insert adds one
 * reference to every position of the path and records the request as the
 * source of the positions it creates; match returns the positions matched
 * from the root and the source of the deepest one ((0, -1) for none);
 * release removes one reference along the request's remembered path and
 * drops subtrees left without references.  Host memory, thread-safe. */
typedef struct specdec_radix specdec_radix;
int specdec_radix_create(specdec_radix** out);
int specdec_radix_destroy(specdec_radix* r);
int specdec_radix_match(specdec_radix* r, const int32_t* tokens, int n, int32_t* matched, int32_t* source);
int specdec_radix_insert(specdec_radix* r, int32_t request_id, const int32_t* tokens, int n);
int specdec_radix_release(specdec_radix* r, int32_t request_id);
/* Nodes (edges) held and token positions they cover. */
int specdec_radix_stats(specdec_radix* r, int64_t* nodes, int64_t* positions);

/* ===================================================================== */
/* 4. Step engine: the whole speculative step on device.                  */
/* ===================================================================== */
typedef struct {
    int hidden, layers, n_q_heads, n_kv_heads, head_dim, ffn, vocab;
    int n_mtp_heads;
    int block_size;     /* 16 */
    float rms_eps;      /* 1e-5 */
    float rope_theta;   /* 10000 */
} specdec_model_config;

typedef struct {
    int batch;          /* sequences held by this engine (one GPU) */
    int draft_len;      /* chain draft length k (tree: ignored) */
    int tree_nodes;     /* 0 = chain; else nodes of the draft tree incl. root */
    int tree_branching[8];
    int tree_levels;
    int max_ctx;        /* maximum tokens per sequence */
    int num_blocks;     /* KV pool blocks (0 = derive from batch * max_ctx) */
    int use_graph;      /* capture the step in a CUDA graph */
    specdec_sampling sampling;
} specdec_run_config;

typedef struct specdec_engine specdec_engine;
typedef struct specdec_sme specdec_sme;
int specdec_engine_create(const specdec_model_config* mc, const specdec_run_config* rc, int device,
                          specdec_engine** out);
int specdec_engine_destroy(specdec_engine* e);
/* Synthesises all weights on the device (bit-identical to the oracle's
 * host-side generator for the same seed). */
int specdec_engine_init_weights(specdec_engine* e, uint32_t seed);
/* Loads the weights of a `.sme` model file (section 5 below) into the
 * engine, whose model config must equal specdec_sme_model_config(f).
 * Projections are requantised to int4 group-128 on the device (the
 * converter of specdec_w4_convert), q/k/v fused, gate/up interleaved; each
 * RMSNorm weight is folded into the columns of the projections it feeds
 * (attn_norm -> q, k, v; ffn_norm -> gate, up; norm -> lm_head;
 * mtp.<i>.norm -> mtp.<i>.proj).  embed_tokens becomes fp16 rows.  A missing
 * lm_head is tied to embed_tokens; missing MTP heads (the reference format
 * has none) are synthesised from missing_seed like specdec_engine_init_weights. */
int specdec_engine_load_sme(specdec_engine* e, const specdec_sme* f, uint32_t missing_seed);
/* Chunked prefill of host prompts [batch, prompt_len] (all but the last
 * token enter the KV; the last becomes the pending token). */
int specdec_engine_prefill(specdec_engine* e, const int32_t* prompts, int prompt_len);
/* Starts sequence slot `seq` on a new request (ids are the caller's): the
 * slot's previous request is retired first.  With a prefix index, the
 * longest indexed prefix of the prompt whose source request still holds a
 * slot is shared block by block (the source's whole 16-token blocks, at most
 * prompt_len - 2 tokens so the last KV token is recomputed for the draft
 * state; PagedKVCache::share_prefix, paged_kv_cache.cpp:136-154, with
 * reference counts), only the remaining prompt tokens are prefilled (64-row
 * chunks of this sequence alone), and the prompt's KV tokens are inserted
 * into the index under request_id.  shared_tokens (may be NULL) receives the
 * number of shared tokens.  Synchronises the engine stream. */
int specdec_engine_admit(specdec_engine* e, int seq, int32_t request_id, const int32_t* prompt, int prompt_len,
                         specdec_radix* cache, int32_t* shared_tokens);
/* Releases slot `seq`: its KV blocks (shared blocks survive while another
 * slot holds them) and, with an index, its prefix references. */
int specdec_engine_retire(specdec_engine* e, int seq, specdec_radix* cache);
/* The first half of specdec_engine_admit, for chunked admission: retires the
 * slot, shares the indexed prefix of the prompt's K/V tokens whose source
 * request holds a slot (whole blocks, at most prompt_len - 2 tokens) and
 * records request_id for the slot.  *shared_tokens receives the number of
 * shared tokens: feed the rest of the prompt from there with
 * specdec_engine_prefill_chunk (the reference scheduler's match_prefix,
 * share_prefix and advance_offset, server/continuous_scheduler.cpp:77-86),
 * and insert the prompt's K/V tokens into the index when the prompt is
 * complete (as mark_completed does, :399-409). */
int specdec_engine_share_prefix(specdec_engine* e, int seq, int32_t request_id, const int32_t* prompt,
                                int prompt_len, specdec_radix* cache, int32_t* shared_tokens);
/* One chunk of slot `seq`'s prompt, for a scheduler that interleaves prompt
 * chunks with decode steps (ChunkedPrefillState::get_next_chunk,
 * server/chunked_prefill.cpp:4-24, consumed in
 * server/continuous_scheduler.cpp:160-176 and server/main.cpp:385-398).
 * The n tokens follow the K/V the slot already holds (none after
 * specdec_engine_retire); they run through the forward in 64-row chunks and
 * their K/V is appended, except that with final_chunk set the last token
 * becomes the pending token instead.  The draft state h0 becomes the hidden
 * state of the last token processed.  Fed in 64-token chunks from a retired
 * slot, the slot ends bit-identical to specdec_engine_admit of the whole
 * prompt.  Keep the slot inactive (specdec_engine_set_active) while its
 * prompt is incomplete: steps leave an inactive slot's K/V, pending token
 * and h0 as they were.  request_id >= 0 records the slot's request (the
 * source rule of prefix sharing); insert the prompt into a prefix index when
 * it is complete.  EINVAL when the prompt would exceed max_ctx or the final
 * chunk leaves no K/V token.  Synchronises the engine stream. */
int specdec_engine_prefill_chunk(specdec_engine* e, int seq, int32_t request_id, const int32_t* tokens, int n,
                                 int final_chunk);
/* Synthetic state: every sequence gets ctx_len[b] tokens of seeded random
 * fp16 K/V, a random pending token and a random draft hidden state. */
int specdec_engine_seed_state(specdec_engine* e, const int32_t* ctx_len, uint32_t seed);
/* One speculative step on device: draft -> verify forward -> acceptance ->
 * KV commit / rollback.  No host synchronisation. */
int specdec_engine_step(specdec_engine* e);
/* Same step with the host boundary: copies per-sequence control inputs
 * (step counter) from host, runs the step, copies accepted lengths and
 * emitted tokens back (out_len [batch], out_tokens [batch, rows]). */
int specdec_engine_step_host(specdec_engine* e, int32_t* out_len, int32_t* out_tokens);
/* Per-sequence active flags used by the next specdec_engine_step_host
 * (inactive sequences keep their state; their reserved slots roll back). */
int specdec_engine_set_active(specdec_engine* e, const int32_t* active);
/* The step's four stages as separate calls on the engine stream (no host
 * synchronisation), in this order; together they queue exactly what
 * specdec_engine_step does (eagerly, without its CUDA graph):
 *   draft             MTP heads -> draft logits -> drafted tokens ("drafts";
 *                     the tree engine's top-k candidates); uploads the active
 *                     flags set by specdec_engine_set_active;
 *   verify_forward    reserves R K/V slots per sequence, builds the verify
 *                     rows and runs the target forward ("logits");
 *   accept            acceptance -> "accepted", "out_tokens";
 *   kv_commit_rollback keeps the accepted rows' K/V, sets the next pending
 *                     token and draft state, rolls the rest back.
 * Between stages the drafts or logits may be read or replaced
 * (specdec_engine_read / _write).  Under sampling (temperature > 0) the
 * acceptance tests drafts against the MTP heads' draft distribution, so
 * replaced drafts belong under greedy decoding, where acceptance is the
 * longest prefix equal to the verify logits' arg-max. */
int specdec_engine_draft(specdec_engine* e);
int specdec_engine_verify_forward(specdec_engine* e);
int specdec_engine_accept(specdec_engine* e);
int specdec_engine_kv_commit_rollback(specdec_engine* e);
void* specdec_engine_stream(specdec_engine* e);
/* Read back state / intermediate buffers ("logits", "draft_logits", "drafts",
 * "accepted", "out_tokens", "pending", "h0", "hidden", "lens", "tables", "kv",
 * "step", "emitted", "mask": the 64 per-row visibility masks of the new
 * rows, ...) and overwrite state ("h0", "pending", "drafts",
 * "kv").  Both synchronise the engine stream. */
int specdec_engine_read(specdec_engine* e, const char* what, void* host, size_t bytes);
int specdec_engine_write(specdec_engine* e, const char* what, const void* host, size_t bytes);
int specdec_engine_info(specdec_engine* e, const char* what, int64_t* value);
/* Runs `steps` eager steps with an event after every kernel and writes the
 * mean device ms per step of: [0] verify GEMMs, [1] verify attention,
 * [2] draft GEMMs, [3] sampling / acceptance, [4] other kernels, [5] whole
 * step, [6] verify GEMM launches per step.  ms_out holds 7 floats. */
int specdec_engine_profile(specdec_engine* e, int steps, float* ms_out);
/* Runs one step through a second CUDA graph of the step that stamps the
 * global timer around the verify forward (embedding, every layer, the
 * lm_head) and returns that forward's device time in ms.  The first call
 * captures that graph (after one eager step).  Synchronises the engine
 * stream. */
int specdec_engine_step_verify_timed(specdec_engine* e, float* verify_ms);

/* ===================================================================== */
/* 5. `.sme` model files (model/README.md:9-36, written by                 */
/*    convert_model.py:26-67, read by load_sme_model, server/main.cpp:     */
/*    112-228).  Host-only: no call in this section touches the GPU        */
/*    except specdec_w4_convert.                                           */
/* ===================================================================== */
/* Maps the file read-only and parses it with every field bounds-checked
 * (SPECDEC_EFORMAT on a short or malformed file, SPECDEC_EIO when it cannot
 * be opened).  Offsets advance by the element count of each tensor as in
 * main.cpp:207-221; a repeated tensor name replaces the earlier tensor. */
int specdec_sme_open(const char* path, specdec_sme** out);
/* Same over a caller-owned buffer (kept alive until specdec_sme_close). */
int specdec_sme_open_buffer(const void* data, size_t bytes, specdec_sme** out);
int specdec_sme_close(specdec_sme* f);
/* The config JSON text, and a top-level number under `key` (the text after
 * "key" and its colon, as main.cpp:129-135 extract_int; EINVAL if absent). */
int specdec_sme_config_json(const specdec_sme* f, const char** json, size_t* len);
int specdec_sme_config_number(const specdec_sme* f, const char* key, double* value);
/* Vocabulary: token text (not NUL-terminated) by id, and id by text with
 * unknown words mapping to 1 (tokenize_word, main.cpp:230-233). */
int specdec_sme_vocab_size(const specdec_sme* f, uint32_t* n);
int specdec_sme_token(const specdec_sme* f, uint32_t id, const char** text, uint32_t* len);
int specdec_sme_token_id(const specdec_sme* f, const char* text, uint32_t len, int32_t* id);
/* Tensor views into the mapping (host pointers, no alignment guarantee). */
typedef struct {
    const char* name;
    uint32_t n_dims;
    const uint32_t* dims;
    uint64_t elements;       /* product of dims */
    int quantized;           /* 1: int8 data + f32 row factors rs = 127 / max|w| */
    uint32_t data_bytes;     /* data size as written in the file */
    const void* scales;      /* f32 [dims[0]] when quantized, else NULL */
    const void* data;        /* int8 or f32 [elements] */
} specdec_sme_tensor;
int specdec_sme_tensor_count(const specdec_sme* f, uint32_t* n);
int specdec_sme_tensor_at(const specdec_sme* f, uint32_t index, specdec_sme_tensor* out);
int specdec_sme_find(const specdec_sme* f, const char* name, specdec_sme_tensor* out);
/* Engine model config of the file: hidden_dim, num_layers, num_heads and
 * vocab_size from the JSON (hidden / vocab default to embed_tokens' shape);
 * head_dim = JSON head_dim or hidden / num_heads; n_kv_heads = JSON
 * num_kv_heads / num_key_value_heads or rows(layers.0.k_proj) / head_dim;
 * ffn = rows(layers.0.gate_proj); n_mtp_heads = the mtp.<i>.proj tensors
 * present, else JSON num_mtp_heads, else 3; rms_eps = JSON rms_norm_eps or
 * 1e-5 (main.cpp:272); rope_theta = JSON rope_theta or 10000.  Tensors are
 * found under the reference's names (embed_tokens, layers.<l>.q_proj ...
 * attn_norm, ffn_norm, norm, lm_head) or the Hugging Face names
 * (model.layers.<l>.self_attn.q_proj.weight ...). */
int specdec_sme_model_config(const specdec_sme* f, specdec_model_config* mc);
/* Device converter: rows [rows, K] of int8 (row factors row_scales, value =
 * q / rs) or f32 (src_f32 = 1), times fold[k] when fold is non-NULL, to
 * int4 group-128 (s = fp16(amax / 7), 1 when amax = 0; q = clamp(round(v /
 * s), -8, 7)) written into the tiled weight of N rows: rows row0 .. (layout
 * 0), or the gate (1) / up (2) half of a fused SwiGLU weight.  K % 8 == 0.
 * Device pointers. */
int specdec_w4_convert(const void* src, int src_f32, const float* row_scales, const float* fold, int rows, int K,
                       void* tiled, int N, int row0, int layout, void* stream);

#ifdef __cplusplus
}
#endif
#endif
