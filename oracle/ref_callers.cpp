// ref_callers.cpp -- the reference's own C++ callers of the kernel FFI, linked
// against libspecdec_sm100.so (TEST INFRASTRUCTURE ONLY: the proof of the
// drop-in boundary, built by oracle/build_ref.sh into oracle/_ref/).
//
// The reference's unmodified server/speculative_decoder.cpp, server/mtp_heads.cpp,
// server/paged_kv_cache.cpp and server/flash_decoding_tracker.cpp are linked
// with this file against libspecdec_sm100.so and nothing else that defines
// their extern "C" kernel symbols (sve2_speculative_verify_f32,
// rust_sme_mtp_predict_f32 / rust_sme_mtp_sample_f32,
// sme_sm_prefetch_kv_blocks, rust_sme_flashdecoding_chunk_f32 /
// rust_sve2_flashdecoding_reduce_f32); the link uses --no-undefined, so every
// one of them resolves to the CUDA library.  The functions below only build the
// reference's classes and call their public methods, the way
// server/continuous_scheduler.cpp and server/main.cpp do, and expose the
// results to a test through plain C entry points.
#include <dlfcn.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "flash_decoding_tracker.h"  // includes the reference's paged_kv_cache.h
#include "mtp_heads.h"
#include "speculative_decoder.h"

extern "C" {
void sve2_speculative_verify_f32(const float*, const int32_t*, const int32_t*, uint32_t, uint32_t, uint32_t, int32_t*,
                                 int32_t*);
void rust_sme_flashdecoding_chunk_f32(const float*, const float*, const float*, uint32_t, uint32_t, float, float*,
                                      float*, float*);
void rust_sve2_flashdecoding_reduce_f32(const float*, const float*, const float*, uint32_t, uint32_t, float*);
void sme_sm_prefetch_kv_blocks(const int8_t**, const int8_t**, uint32_t);
}

// SpeculativeDecoder(max_draft).verify_drafts_sve2 on host vectors
// (continuous_scheduler.cpp:340-397 packs drafts and calls it this way).
extern "C" void refc_verify(const float* logits, size_t n_logits, const int32_t* drafts, size_t n_drafts,
                            const int32_t* lens, int B, int V, int max_draft, int32_t* acc, int32_t* rep) {
    SpeculativeDecoder dec(max_draft);
    std::vector<float> lg(logits, logits + n_logits);
    std::vector<int> dr(drafts, drafts + n_drafts), ln(lens, lens + B), a, r;
    dec.verify_drafts_sve2(lg, dr, ln, V, B, a, r);
    for (int b = 0; b < B; ++b) {
        acc[b] = a[b];
        rep[b] = r[b];
    }
}

// MTPHeads(K, H, V): load_weights, then generate_drafts for each of n hidden
// states in turn (continuous_scheduler.cpp:326-338 calls it once per request).
extern "C" void refc_mtp_generate(const float* w, const float* hidden, int n, int K, int H, int V, int32_t* out) {
    MTPHeads heads((uint32_t)K, (uint32_t)H, (uint32_t)V);
    heads.load_weights(w);
    for (int i = 0; i < n; ++i) {
        std::vector<int32_t> d = heads.generate_drafts(hidden + (size_t)i * H);
        for (int j = 0; j < K; ++j) out[(size_t)i * K + j] = d[j];
    }
}

// FlashDecodingTracker::execute_flash_decoding (its chunk / reduce calls run
// on the GPU) and PagedKVCache::prefetch_kv_blocks (a no-op on the GPU).
extern "C" void refc_flash_decoding(const float* q, int head_dim, float scale, float* out) {
    PagedKVCache cache(64, 16, head_dim);
    const std::vector<float> kv((size_t)20 * head_dim, 0.5f);
    cache.append_tokens(0, kv, kv);
    cache.prefetch_kv_blocks(std::vector<int>{0, 1});
    FlashDecodingTracker fd(&cache);
    fd.execute_flash_decoding(0, q, (uint32_t)head_dim, scale, out);
}

// Path of the shared object that defines the FFI symbol `name` as this
// library was linked (dladdr of the address the reference objects call).
extern "C" const char* refc_symbol_origin(const char* name) {
    static Dl_info info;
    const void* addr = nullptr;
    const std::string n(name ? name : "");
    if (n == "sve2_speculative_verify_f32") addr = (const void*)&sve2_speculative_verify_f32;
    else if (n == "rust_sme_mtp_predict_f32") addr = (const void*)&rust_sme_mtp_predict_f32;
    else if (n == "rust_sme_mtp_sample_f32") addr = (const void*)&rust_sme_mtp_sample_f32;
    else if (n == "rust_sme_flashdecoding_chunk_f32") addr = (const void*)&rust_sme_flashdecoding_chunk_f32;
    else if (n == "rust_sve2_flashdecoding_reduce_f32") addr = (const void*)&rust_sve2_flashdecoding_reduce_f32;
    else if (n == "sme_sm_prefetch_kv_blocks") addr = (const void*)&sme_sm_prefetch_kv_blocks;
    if (!addr || !dladdr(addr, &info) || !info.dli_fname) return "";
    return info.dli_fname;
}
