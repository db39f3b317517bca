// ref_shim.cpp -- glue that lets the reference's own C++ operator classes run on
// x86 as a checker (TEST INFRASTRUCTURE ONLY).
//
// The reference C++ (server/paged_attention.cpp, server/paged_kv_cache.cpp,
// server/speculative_decoder.cpp, server/mtp_heads.cpp) is compiled unmodified
// by oracle/build_ref.sh.  Those files call into the Rust SVE2/SME library
// (src/sme_kernel/rust_sme/src/lib.rs), which cannot be built here (no Rust
// toolchain, aarch64-only intrinsics).  This file provides those C symbols by
// forwarding to the oracle's C restatements, and exposes plain C entry points
// that Python (ctypes) uses to drive the reference classes.
#include <cstdint>
#include <cstring>
#include <vector>

#include "chunked_prefill.h"
#include "mtp_heads.h"
#include "paged_attention.h"
#include "paged_kv_cache.h"
#include "radix_kv_cache.h"
#include "speculative_decoder.h"

extern "C" {
#include "oracle.h"
}

// ---- Rust kernel symbols the reference C++ links against ------------------
extern "C" void sve2_speculative_verify_f32(const float* logits, const int32_t* drafts, const int32_t* lens,
                                            uint32_t vocab, uint32_t max_draft, uint32_t batch, int32_t* accepted,
                                            int32_t* replacement) {
    orc_compat_verify(logits, drafts, lens, (int)vocab, (int)max_draft, (int)batch, 4, accepted, replacement);
}

extern "C" void rust_sme_mtp_predict_f32(const float* h, const float* w, float* out, uint32_t hidden, uint32_t vocab,
                                         uint32_t k) {
    orc_compat_mtp_predict(h, w, out, (int)hidden, (int)vocab, (int)k);
}

extern "C" void rust_sme_mtp_sample_f32(const float* logits, int32_t* out, uint32_t vocab, uint32_t k) {
    orc_compat_mtp_sample(logits, out, (int)vocab, (int)k, 4);
}

extern "C" void sme_sm_prefetch_kv_blocks(const int8_t**, const int8_t**, uint32_t) {}

// ---- ctypes entry points ----------------------------------------------------
extern "C" void ref_paged_attention(const float* q, const float* k_pool, const float* v_pool, size_t pool_floats,
                                    const int32_t* table_off, const int32_t* tables, const int32_t* seq_lens,
                                    float* o, int M, int hidden, int bs) {
    std::vector<float> vq(q, q + (size_t)M * hidden);
    std::vector<float> vk(k_pool, k_pool + pool_floats), vv(v_pool, v_pool + pool_floats);
    std::vector<std::vector<int>> tabs(M);
    for (int m = 0; m < M; ++m) tabs[m].assign(tables + table_off[m], tables + table_off[m + 1]);
    std::vector<int> lens(seq_lens, seq_lens + M);
    std::vector<float> vo(o, o + (size_t)M * hidden);
    compute_paged_attention(vq, vk, vv, tabs, lens, vo, hidden, bs);
    std::memcpy(o, vo.data(), sizeof(float) * vo.size());
}

extern "C" void* ref_kv_create(int num_blocks, int block_size, int hidden) {
    return new PagedKVCache(num_blocks, block_size, hidden);
}
extern "C" void ref_kv_destroy(void* h) { delete static_cast<PagedKVCache*>(h); }
extern "C" int ref_kv_append(void* h, int req, int n_tokens, int hidden) {
    std::vector<float> k((size_t)n_tokens * hidden, 0.5f), v((size_t)n_tokens * hidden, -0.5f);
    return static_cast<PagedKVCache*>(h)->append_tokens(req, k, v);
}
extern "C" void ref_kv_free_request(void* h, int req) { static_cast<PagedKVCache*>(h)->free_request(req); }
extern "C" void ref_kv_share_prefix(void* h, int new_req, int src, int len) {
    static_cast<PagedKVCache*>(h)->share_prefix(new_req, src, len);
}
extern "C" void ref_kv_free_merged(void* h, int req, int n) { static_cast<PagedKVCache*>(h)->free_merged_blocks(req, n); }
extern "C" int ref_kv_evict(void* h, int req, int n) {
    return static_cast<PagedKVCache*>(h)->evict_least_important_blocks(req, n) ? 1 : 0;
}
extern "C" float ref_kv_utilization(void* h) { return static_cast<PagedKVCache*>(h)->get_utilization(); }
// Returns the number of blocks of `req` (0 if unknown); copies up to cap entries.
extern "C" int ref_kv_table(void* h, int req, int32_t* out, int cap, int32_t* len) {
    std::vector<std::vector<int>> tabs;
    std::vector<int> lens;
    static_cast<PagedKVCache*>(h)->get_cache_for_batch({req}, tabs, lens);
    int n = (int)tabs[0].size();
    for (int i = 0; i < n && i < cap; ++i) out[i] = tabs[0][i];
    *len = lens[0];
    return n;
}

extern "C" void ref_verify(const float* logits, size_t n_logits, const int32_t* drafts, size_t n_drafts,
                           const int32_t* lens, int batch, int vocab, int max_draft, int32_t* accepted,
                           int32_t* replacement) {
    SpeculativeDecoder dec(max_draft);
    std::vector<float> vl(logits, logits + n_logits);
    std::vector<int> vd(drafts, drafts + n_drafts), vlen(lens, lens + batch), acc, rep;
    dec.verify_drafts_sve2(vl, vd, vlen, vocab, batch, acc, rep);
    for (int b = 0; b < batch; ++b) { accepted[b] = acc[b]; replacement[b] = rep[b]; }
}

extern "C" void ref_mtp_generate(const float* weights, const float* hidden_state, int k, int hidden, int vocab,
                                 int32_t* out) {
    MTPHeads heads((uint32_t)k, (uint32_t)hidden, (uint32_t)vocab);
    heads.load_weights(weights);
    std::vector<int32_t> d = heads.generate_drafts(hidden_state);
    for (int i = 0; i < k; ++i) out[i] = d[i];
}

// RadixKVCache (server/radix_kv_cache.cpp), driven op by op.
extern "C" void* ref_radix_create() { return new RadixKVCache(); }
extern "C" void ref_radix_destroy(void* h) { delete static_cast<RadixKVCache*>(h); }
extern "C" void ref_radix_insert(void* h, int req, const int32_t* t, int n) {
    static_cast<RadixKVCache*>(h)->insert_prefix(req, std::vector<int>(t, t + n));
}
extern "C" void ref_radix_release(void* h, int req) { static_cast<RadixKVCache*>(h)->release_prefix(req); }
extern "C" void ref_radix_match(void* h, const int32_t* t, int n, int32_t* matched, int32_t* source) {
    auto r = static_cast<RadixKVCache*>(h)->match_prefix(std::vector<int>(t, t + n));
    *matched = r.first;
    *source = r.second;
}

// ChunkedPrefillState (server/chunked_prefill.cpp), driven call by call: up
// to `cap` calls of get_next_chunk, with reset() after call `reset_after`
// (-1: never), each recorded as (chunk length, first token or -1,
// get_remaining_tokens(), is_prefill_complete) in out4[4 * call].  Returns
// the number of calls made (the last one returned an empty chunk, or cap).
extern "C" int ref_chunked_prefill(const int32_t* t, int n, int chunk, int reset_after, int32_t* out4, int cap) {
    ChunkedPrefillState st(std::vector<int>(t, t + n), chunk);
    int calls = 0;
    while (calls < cap) {
        const std::vector<int> c = st.get_next_chunk();
        out4[4 * calls + 0] = (int32_t)c.size();
        out4[4 * calls + 1] = c.empty() ? -1 : c[0];
        out4[4 * calls + 2] = st.get_remaining_tokens();
        out4[4 * calls + 3] = st.is_prefill_complete ? 1 : 0;
        if (calls == reset_after) st.reset();
        ++calls;
        if (c.empty()) break;
    }
    return calls;
}
