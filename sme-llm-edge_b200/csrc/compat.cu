// compat.cu -- the reference's kernel FFI symbols, implemented on the GPU.
//
// server/speculative_decoder.cpp, server/mtp_heads.cpp,
// server/paged_kv_cache.cpp and server/flash_decoding_tracker.cpp declare these
// extern "C" functions (normally provided by src/sme_kernel/rust_sme/src/lib.rs)
// and keep working unchanged when linked against this library.  Arguments are
// host pointers with the reference's layouts; each call stages its inputs to
// the current device, runs a kernel and copies the outputs back.  The
// functions return void like the reference; on failure the outputs hold the
// reference wrapper's defaults and specdec_last_error() says why.
//
// Staging is per device: one stream and grow-only device buffers, reused by
// every call (a call allocates only when its inputs outgrow the buffers), and
// the MTP heads' fp32 weights stay resident on the device between calls,
// keyed by host pointer, size and a content fingerprint, so that
// MTPHeads::generate_drafts (server/mtp_heads.cpp:53-79) uploads only the
// hidden state once its weights are cached.
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace specdec {

// logits[k, j] = sum_d h[d] * W[k, d, j] summed in d order (lib.rs:1792-1831).
__global__ void mtp_predict_kernel(const float* __restrict__ h, const float* __restrict__ W, float* __restrict__ out,
                                   int H, int V) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int k = blockIdx.y;
    if (j >= V) return;
    const float* w = W + (size_t)k * H * V + j;
    float acc = 0.f;
    for (int d = 0; d < H; ++d) acc = __fadd_rn(acc, __fmul_rn(h[d], w[(size_t)d * V]));
    out[(size_t)k * V + j] = acc;
}

// compute_paged_attention (paged_attention.cpp:16-111): weight
// exp(q.k / sqrt(H)) / seq_len, no max subtraction, accumulated into o.
__global__ void compat_paged_attention_kernel(const float* __restrict__ q, const float* __restrict__ kp,
                                              const float* __restrict__ vp, const int32_t* __restrict__ off,
                                              const int32_t* __restrict__ tables, const int32_t* __restrict__ lens,
                                              float* __restrict__ o, int H, int bs) {
    __shared__ float red[32];
    const int m = blockIdx.x;
    const int seq = lens[m];
    const int nb = off[m + 1] - off[m];
    if (seq == 0 || nb == 0) return;
    const float scale = 1.0f / sqrtf((float)H);
    const float inv_len = 1.0f / (float)(seq > 1 ? seq : 1);
    const float* qr = q + (size_t)m * H;
    float* orow = o + (size_t)m * H;
    int done = 0;
    for (int b = 0; b < nb; ++b) {
        const int phys = tables[off[m] + b];
        const int tib = min(bs, seq - done);
        for (int t = 0; t < tib; ++t) {
            const float* kr = kp + ((size_t)phys * bs + t) * H;
            const float* vr = vp + ((size_t)phys * bs + t) * H;
            float part = 0.f;
            for (int i = threadIdx.x; i < H; i += blockDim.x) part = __fadd_rn(part, __fmul_rn(qr[i], kr[i]));
            const float s = block_sum<float>(part, red);
            const float w = __fmul_rn(expf(__fmul_rn(s, scale)), inv_len);
            for (int i = threadIdx.x; i < H; i += blockDim.x) orow[i] = __fadd_rn(orow[i], __fmul_rn(w, vr[i]));
            __syncthreads();
        }
        done += tib > 0 ? tib : 0;
    }
}

// rust_sme_flashdecoding_chunk_f32 (lib.rs:1638-1712), one CTA.
__global__ void fd_chunk_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                int len, int hd, float scale, float* __restrict__ po, float* __restrict__ pm,
                                float* __restrict__ ps) {
    __shared__ float red[32];
    __shared__ float s_max;
    float mx = -INFINITY;
    for (int t = 0; t < len; ++t) {
        float part = 0.f;
        for (int d = threadIdx.x; d < hd; d += blockDim.x) part = __fadd_rn(part, __fmul_rn(q[d], k[(size_t)t * hd + d]));
        const float s = __fmul_rn(block_sum<float>(part, red), scale);
        mx = fmaxf(mx, s);
        __syncthreads();
    }
    if (threadIdx.x == 0) s_max = mx;
    __syncthreads();
    float sum = 0.f;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) po[d] = 0.f;
    for (int t = 0; t < len; ++t) {
        float part = 0.f;
        for (int d = threadIdx.x; d < hd; d += blockDim.x) part = __fadd_rn(part, __fmul_rn(q[d], k[(size_t)t * hd + d]));
        const float s = __fmul_rn(block_sum<float>(part, red), scale);
        const float w = expf(s - s_max);
        sum += w;
        for (int d = threadIdx.x; d < hd; d += blockDim.x) po[d] += w * v[(size_t)t * hd + d];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *pm = s_max;
        *ps = sum;
    }
}

// rust_sve2_flashdecoding_reduce_f32 (lib.rs:1721-1783).
__global__ void fd_reduce_kernel(const float* __restrict__ po, const float* __restrict__ pm,
                                 const float* __restrict__ ps, int chunks, int hd, float* __restrict__ out) {
    float g = -INFINITY;
    for (int c = 0; c < chunks; ++c) g = fmaxf(g, pm[c]);
    float gs = 0.f;
    for (int c = 0; c < chunks; ++c) gs += ps[c] * expf(pm[c] - g);
    const float inv = 1.0f / gs;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.f;
        for (int c = 0; c < chunks; ++c) acc += po[(size_t)c * hd + d] * expf(pm[c] - g);
        out[d] = acc * inv;
    }
}

// Kernels shared with sampling.cu
__global__ void compat_argmax_kernel(const float* __restrict__ logits, const int32_t* __restrict__ lens, int V,
                                     int max_draft, int32_t* __restrict__ best);

// Per-device staging for the host-pointer entry points.  Calls on one device
// serialise on its mutex; every copy and kernel of a call is ordered on the
// device's own stream, which the call synchronises before it returns.
enum { kStageIn = 0, kStageAux, kStageAux2, kStageOut, kStageOut2, kStageOff, kStageTab, kStageLen, kStageBufs };
struct CompatStage {
    std::mutex mu;
    cudaStream_t stream = nullptr;
    void* buf[kStageBufs] = {nullptr};
    size_t cap[kStageBufs] = {0};
    // MTP heads weights resident on the device
    const float* w_host = nullptr;
    size_t w_floats = 0;
    uint64_t w_print = 0;
    float* w_dev = nullptr;
    uint64_t w_uploads = 0;
};
static std::mutex g_stage_mu;
static CompatStage* g_stage[64] = {nullptr};

static CompatStage* compat_stage() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_stage_mu);
    if (!g_stage[dev]) {
        CompatStage* st = new CompatStage();
        if (cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking) != cudaSuccess) {
            delete st;
            return nullptr;
        }
        g_stage[dev] = st;
    }
    return g_stage[dev];
}

// Device buffer i of at least `bytes` (grown, never shrunk).
static void* stage_buf(CompatStage* st, int i, size_t bytes) {
    if (bytes == 0) bytes = 1;
    if (st->cap[i] < bytes) {
        if (st->buf[i]) cudaFree(st->buf[i]);
        st->buf[i] = nullptr;
        st->cap[i] = 0;
        if (cudaMalloc(&st->buf[i], bytes) != cudaSuccess) {
            cudaGetLastError();
            st->buf[i] = nullptr;
            return nullptr;
        }
        st->cap[i] = bytes;
    }
    return st->buf[i];
}

// FNV-1a over 64K evenly spaced floats and the first and last 1024 of the
// weights: a cheap content check (a few hundred KB read per call) that sees a
// new checkpoint loaded into the same buffer.  An in-place edit that changes
// only elements the sample misses is not seen; such callers release the
// resident copy with specdec_compat_release_weights().
static uint64_t weights_print(const float* w, size_t n) {
    uint64_t h = 1469598103934665603ull ^ (uint64_t)n;
    auto mix = [&](size_t i) {
        uint32_t v;
        std::memcpy(&v, w + i, 4);
        h = (h ^ v) * 1099511628211ull;
    };
    const size_t edge = n < 1024 ? n : 1024;
    for (size_t i = 0; i < edge; ++i) mix(i);
    for (size_t i = n - edge; i < n; ++i) mix(i);
    const size_t samples = 65536, stride = n > samples ? n / samples : 1;
    for (size_t i = 0; i < n; i += stride) mix(i);
    return h;
}

}  // namespace specdec

using namespace specdec;

extern "C" void sve2_speculative_verify_f32(const float* logits_ptr, const int32_t* draft_tokens_ptr,
                                            const int32_t* draft_lengths_ptr, uint32_t vocab_size,
                                            uint32_t max_draft_length, uint32_t batch_size,
                                            int32_t* accepted_counts_ptr, int32_t* replacement_tokens_ptr) {
    const size_t B = batch_size, D = max_draft_length, V = vocab_size;
    for (size_t b = 0; b < B; ++b) {
        accepted_counts_ptr[b] = 0;
        replacement_tokens_ptr[b] = -1;
    }
    if (!B || !D || !V || !logits_ptr || !draft_tokens_ptr || !draft_lengths_ptr) return;
    CompatStage* st = compat_stage();
    if (!st) {
        set_error("sve2_speculative_verify_f32: no CUDA device");
        return;
    }
    std::lock_guard<std::mutex> lk(st->mu);
    float* dl = static_cast<float*>(stage_buf(st, kStageIn, 4 * B * D * V));
    int32_t* dd = static_cast<int32_t*>(stage_buf(st, kStageAux, 4 * B * D));
    int32_t* dn = static_cast<int32_t*>(stage_buf(st, kStageAux2, 4 * B));
    int32_t* dout = static_cast<int32_t*>(stage_buf(st, kStageOut, 8 * B));
    if (!dl || !dd || !dn || !dout) {
        set_error("sve2_speculative_verify_f32: device allocation failed");
        return;
    }
    cudaStream_t s = st->stream;
    if (cudaMemcpyAsync(dl, logits_ptr, 4 * B * D * V, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(dd, draft_tokens_ptr, 4 * B * D, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(dn, draft_lengths_ptr, 4 * B, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        set_error("sve2_speculative_verify_f32: copy to device failed");
        return;
    }
    if (specdec_compat_verify(dl, dd, dn, (int)V, (int)D, (int)B, dout, dout + B, s)) return;
    std::vector<int32_t> h(2 * B);
    if (cudaMemcpyAsync(h.data(), dout, 8 * B, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        set_error("sve2_speculative_verify_f32: copy to host failed");
        return;
    }
    std::memcpy(accepted_counts_ptr, h.data(), 4 * B);
    std::memcpy(replacement_tokens_ptr, h.data() + B, 4 * B);
}

extern "C" void rust_sme_mtp_predict_f32(const float* hidden_state_ptr, const float* weights_ptr,
                                         float* logits_out_ptr, uint32_t hidden_dim, uint32_t vocab_size,
                                         uint32_t k_heads) {
    const size_t H = hidden_dim, V = vocab_size, K = k_heads;
    if (!H || !V || !K || !hidden_state_ptr || !weights_ptr || !logits_out_ptr) return;
    CompatStage* st = compat_stage();
    if (!st) {
        set_error("rust_sme_mtp_predict_f32: no CUDA device");
        return;
    }
    std::lock_guard<std::mutex> lk(st->mu);
    cudaStream_t s = st->stream;
    const size_t wn = K * H * V;
    const uint64_t print = weights_print(weights_ptr, wn);
    if (st->w_host != weights_ptr || st->w_floats != wn || st->w_print != print || !st->w_dev) {
        if (st->w_dev && st->w_floats != wn) {
            cudaFree(st->w_dev);
            st->w_dev = nullptr;
        }
        st->w_host = nullptr;
        if (!st->w_dev && cudaMalloc(&st->w_dev, 4 * wn) != cudaSuccess) {
            cudaGetLastError();
            st->w_dev = nullptr;
            set_error("rust_sme_mtp_predict_f32: device allocation failed");
            return;
        }
        if (cudaMemcpyAsync(st->w_dev, weights_ptr, 4 * wn, cudaMemcpyHostToDevice, s) != cudaSuccess) {
            set_error("rust_sme_mtp_predict_f32: copy to device failed");
            return;
        }
        st->w_host = weights_ptr;
        st->w_floats = wn;
        st->w_print = print;
        ++st->w_uploads;
    }
    float* dh = static_cast<float*>(stage_buf(st, kStageAux, 4 * H));
    float* dout = static_cast<float*>(stage_buf(st, kStageOut, 4 * K * V));
    if (!dh || !dout) {
        set_error("rust_sme_mtp_predict_f32: device allocation failed");
        return;
    }
    if (cudaMemcpyAsync(dh, hidden_state_ptr, 4 * H, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        set_error("rust_sme_mtp_predict_f32: copy to device failed");
        return;
    }
    mtp_predict_kernel<<<dim3((unsigned)((V + 255) / 256), (unsigned)K), 256, 0, s>>>(dh, st->w_dev, dout, (int)H,
                                                                                    (int)V);
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpyAsync(logits_out_ptr, dout, 4 * K * V, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        set_error("rust_sme_mtp_predict_f32: kernel or copy failed");
}

extern "C" void rust_sme_mtp_sample_f32(const float* logits_ptr, int32_t* draft_tokens_out, uint32_t vocab_size,
                                        uint32_t k_heads) {
    const size_t V = vocab_size, K = k_heads;
    if (!V || !K || !logits_ptr || !draft_tokens_out) return;
    CompatStage* st = compat_stage();
    if (!st) {
        set_error("rust_sme_mtp_sample_f32: no CUDA device");
        return;
    }
    std::lock_guard<std::mutex> lk(st->mu);
    cudaStream_t s = st->stream;
    float* dl = static_cast<float*>(stage_buf(st, kStageIn, 4 * K * V));
    int32_t* dout = static_cast<int32_t*>(stage_buf(st, kStageOut2, 4 * K));
    if (!dl || !dout) {
        set_error("rust_sme_mtp_sample_f32: device allocation failed");
        return;
    }
    if (cudaMemcpyAsync(dl, logits_ptr, 4 * K * V, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        set_error("rust_sme_mtp_sample_f32: copy to device failed");
        return;
    }
    // each head is one row of a [K, 1, V] "draft" tensor with no length limit
    compat_argmax_kernel<<<(unsigned)K, 256, 0, s>>>(dl, nullptr, (int)V, 1, dout);
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpyAsync(draft_tokens_out, dout, 4 * K, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        set_error("rust_sme_mtp_sample_f32: kernel or copy failed");
}

extern "C" void sme_sm_prefetch_kv_blocks(const int8_t** k_ptrs, const int8_t** v_ptrs, uint32_t num_blocks) {
    (void)k_ptrs;
    (void)v_ptrs;
    (void)num_blocks;
}

extern "C" void rust_sme_flashdecoding_chunk_f32(const float* q_ptr, const float* k_chunk_ptr,
                                                 const float* v_chunk_ptr, uint32_t chunk_len, uint32_t head_dim,
                                                 float softmax_scale, float* partial_o_out, float* partial_max_out,
                                                 float* partial_sum_exp_out) {
    const size_t L = chunk_len, D = head_dim;
    if (!D || !q_ptr || !k_chunk_ptr || !v_chunk_ptr || !partial_o_out || !partial_max_out || !partial_sum_exp_out)
        return;
    CompatStage* st = compat_stage();
    if (!st) {
        set_error("rust_sme_flashdecoding_chunk_f32: no CUDA device");
        return;
    }
    std::lock_guard<std::mutex> lk(st->mu);
    cudaStream_t s = st->stream;
    float* dq = static_cast<float*>(stage_buf(st, kStageAux, 4 * D));
    float* dk = static_cast<float*>(stage_buf(st, kStageIn, 4 * L * D));
    float* dv = static_cast<float*>(stage_buf(st, kStageAux2, 4 * L * D));
    float* dout = static_cast<float*>(stage_buf(st, kStageOut, 4 * (D + 2)));
    if (!dq || !dk || !dv || !dout) {
        set_error("rust_sme_flashdecoding_chunk_f32: device allocation failed");
        return;
    }
    bool ok = cudaMemcpyAsync(dq, q_ptr, 4 * D, cudaMemcpyHostToDevice, s) == cudaSuccess;
    if (L) {
        ok = ok && cudaMemcpyAsync(dk, k_chunk_ptr, 4 * L * D, cudaMemcpyHostToDevice, s) == cudaSuccess;
        ok = ok && cudaMemcpyAsync(dv, v_chunk_ptr, 4 * L * D, cudaMemcpyHostToDevice, s) == cudaSuccess;
    }
    if (ok) {
        fd_chunk_kernel<<<1, 128, 0, s>>>(dq, dk, dv, (int)L, (int)D, softmax_scale, dout, dout + D, dout + D + 1);
        ok = cudaGetLastError() == cudaSuccess;
    }
    std::vector<float> h(D + 2);
    if (!ok || cudaMemcpyAsync(h.data(), dout, 4 * (D + 2), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        set_error("rust_sme_flashdecoding_chunk_f32: kernel or copy failed");
        return;
    }
    std::memcpy(partial_o_out, h.data(), 4 * D);
    *partial_max_out = h[D];
    *partial_sum_exp_out = h[D + 1];
}

extern "C" void rust_sve2_flashdecoding_reduce_f32(const float* partial_o_ptr, const float* partial_max_ptr,
                                                   const float* partial_sum_exp_ptr, uint32_t num_chunks,
                                                   uint32_t head_dim, float* final_o_out) {
    const size_t Cn = num_chunks, D = head_dim;
    if (!D || !partial_o_ptr || !partial_max_ptr || !partial_sum_exp_ptr || !final_o_out) return;
    CompatStage* st = compat_stage();
    if (!st) {
        set_error("rust_sve2_flashdecoding_reduce_f32: no CUDA device");
        return;
    }
    std::lock_guard<std::mutex> lk(st->mu);
    cudaStream_t s = st->stream;
    float* dpo = static_cast<float*>(stage_buf(st, kStageIn, 4 * Cn * D));
    float* dpm = static_cast<float*>(stage_buf(st, kStageAux, 4 * Cn));
    float* dps = static_cast<float*>(stage_buf(st, kStageAux2, 4 * Cn));
    float* dout = static_cast<float*>(stage_buf(st, kStageOut, 4 * D));
    if (!dpo || !dpm || !dps || !dout) {
        set_error("rust_sve2_flashdecoding_reduce_f32: device allocation failed");
        return;
    }
    bool ok = true;
    if (Cn) {
        ok = cudaMemcpyAsync(dpo, partial_o_ptr, 4 * Cn * D, cudaMemcpyHostToDevice, s) == cudaSuccess &&
             cudaMemcpyAsync(dpm, partial_max_ptr, 4 * Cn, cudaMemcpyHostToDevice, s) == cudaSuccess &&
             cudaMemcpyAsync(dps, partial_sum_exp_ptr, 4 * Cn, cudaMemcpyHostToDevice, s) == cudaSuccess;
    }
    if (ok) {
        fd_reduce_kernel<<<1, 128, 0, s>>>(dpo, dpm, dps, (int)Cn, (int)D, dout);
        ok = cudaGetLastError() == cudaSuccess;
    }
    if (!ok || cudaMemcpyAsync(final_o_out, dout, 4 * D, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        set_error("rust_sve2_flashdecoding_reduce_f32: kernel or copy failed");
}

// Drops the MTP weights kept resident on the current device (the next
// rust_sme_mtp_predict_f32 uploads them again) and reports how many uploads
// the cache has made so far.
extern "C" int specdec_compat_release_weights(uint64_t* uploads) {
    CompatStage* st = compat_stage();
    SD_CHECK(st, SPECDEC_ECUDA, "compat_release_weights: no CUDA device");
    std::lock_guard<std::mutex> lk(st->mu);
    if (uploads) *uploads = st->w_uploads;
    if (st->w_dev) cudaFree(st->w_dev);
    st->w_dev = nullptr;
    st->w_host = nullptr;
    st->w_floats = 0;
    st->w_print = 0;
    return SPECDEC_OK;
}

extern "C" int specdec_compat_weight_uploads(uint64_t* uploads) {
    SD_CHECK(uploads, SPECDEC_EINVAL, "compat_weight_uploads: null");
    CompatStage* st = compat_stage();
    SD_CHECK(st, SPECDEC_ECUDA, "compat_weight_uploads: no CUDA device");
    std::lock_guard<std::mutex> lk(st->mu);
    *uploads = st->w_uploads;
    return SPECDEC_OK;
}

extern "C" int specdec_paged_attention_compat_f32(const float* q, const float* k_pool, const float* v_pool,
                                                  size_t pool_floats, const int32_t* table_off, const int32_t* tables,
                                                  const int32_t* seq_lens, float* o, int M, int hidden_dim,
                                                  int block_size) {
    SD_CHECK(q && k_pool && v_pool && table_off && tables && seq_lens && o && M >= 0 && hidden_dim > 0 &&
                 block_size > 0,
             SPECDEC_EINVAL, "paged_attention_compat: bad argument");
    if (M == 0) return SPECDEC_OK;
    const size_t H = hidden_dim;
    const size_t ntab = (size_t)table_off[M];
    for (int m = 0; m < M; ++m) {
        SD_CHECK(table_off[m + 1] >= table_off[m], SPECDEC_EINVAL, "paged_attention_compat: bad table offsets");
        const int seq = seq_lens[m];
        const int nb = table_off[m + 1] - table_off[m];
        if (seq == 0 || nb == 0) continue;
        int done = 0;
        for (int b = 0; b < nb && done < seq; ++b) {
            const int phys = tables[table_off[m] + b];
            const int tib = std::min(block_size, seq - done);
            SD_CHECK(phys >= 0 && ((size_t)phys * block_size + tib) * H <= pool_floats, SPECDEC_EINVAL,
                     "paged_attention_compat: block index outside the pool");
            done += tib;
        }
    }
    CompatStage* st = compat_stage();
    SD_CHECK(st, SPECDEC_ECUDA, "paged_attention_compat: no CUDA device");
    std::lock_guard<std::mutex> lk(st->mu);
    cudaStream_t s = st->stream;
    float* dq = static_cast<float*>(stage_buf(st, kStageAux, 4 * M * H));
    float* dk = static_cast<float*>(stage_buf(st, kStageIn, 4 * pool_floats));
    float* dv = static_cast<float*>(stage_buf(st, kStageAux2, 4 * pool_floats));
    int32_t* doff = static_cast<int32_t*>(stage_buf(st, kStageOff, 4 * (M + 1)));
    int32_t* dt = static_cast<int32_t*>(stage_buf(st, kStageTab, 4 * (ntab ? ntab : 1)));
    int32_t* dl = static_cast<int32_t*>(stage_buf(st, kStageLen, 4 * M));
    float* dout = static_cast<float*>(stage_buf(st, kStageOut, 4 * M * H));
    SD_CHECK(dq && dk && dv && doff && dt && dl && dout, SPECDEC_ENOMEM,
             "paged_attention_compat: device allocation failed");
    SD_CUDA(cudaMemcpyAsync(dq, q, 4 * M * H, cudaMemcpyHostToDevice, s));
    SD_CUDA(cudaMemcpyAsync(dk, k_pool, 4 * pool_floats, cudaMemcpyHostToDevice, s));
    SD_CUDA(cudaMemcpyAsync(dv, v_pool, 4 * pool_floats, cudaMemcpyHostToDevice, s));
    SD_CUDA(cudaMemcpyAsync(doff, table_off, 4 * (M + 1), cudaMemcpyHostToDevice, s));
    if (ntab) SD_CUDA(cudaMemcpyAsync(dt, tables, 4 * ntab, cudaMemcpyHostToDevice, s));
    SD_CUDA(cudaMemcpyAsync(dl, seq_lens, 4 * M, cudaMemcpyHostToDevice, s));
    SD_CUDA(cudaMemcpyAsync(dout, o, 4 * M * H, cudaMemcpyHostToDevice, s));
    compat_paged_attention_kernel<<<M, 128, 0, s>>>(dq, dk, dv, doff, dt, dl, dout, (int)H, block_size);
    SD_LAUNCH_CHECK("compat_paged_attention_kernel");
    SD_CUDA(cudaMemcpyAsync(o, dout, 4 * M * H, cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaStreamSynchronize(s));
    return SPECDEC_OK;
}
