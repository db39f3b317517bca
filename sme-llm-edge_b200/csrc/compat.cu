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
#include <cstring>
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

// RAII device buffer for the staging paths.
struct DevBuf {
    void* p = nullptr;
    cudaError_t err = cudaSuccess;
    explicit DevBuf(size_t bytes) { err = cudaMalloc(&p, bytes ? bytes : 1); }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    template <typename T>
    T* as() const {
        return reinterpret_cast<T*>(p);
    }
};

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
    DevBuf dl(4 * B * D * V), dd(4 * B * D), dn(4 * B), da(4 * B), dr(4 * B);
    if (dl.err || dd.err || dn.err || da.err || dr.err) {
        set_error("sve2_speculative_verify_f32: device allocation failed");
        return;
    }
    if (cudaMemcpy(dl.p, logits_ptr, 4 * B * D * V, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dd.p, draft_tokens_ptr, 4 * B * D, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dn.p, draft_lengths_ptr, 4 * B, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_error("sve2_speculative_verify_f32: copy to device failed");
        return;
    }
    int rc = specdec_compat_verify(dl.as<float>(), dd.as<int32_t>(), dn.as<int32_t>(), (int)V, (int)D, (int)B,
                                   da.as<int32_t>(), dr.as<int32_t>(), nullptr);
    if (rc) return;
    std::vector<int32_t> a(B), r(B);
    if (cudaMemcpy(a.data(), da.p, 4 * B, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(r.data(), dr.p, 4 * B, cudaMemcpyDeviceToHost) != cudaSuccess) {
        set_error("sve2_speculative_verify_f32: copy to host failed");
        return;
    }
    std::memcpy(accepted_counts_ptr, a.data(), 4 * B);
    std::memcpy(replacement_tokens_ptr, r.data(), 4 * B);
}

extern "C" void rust_sme_mtp_predict_f32(const float* hidden_state_ptr, const float* weights_ptr,
                                         float* logits_out_ptr, uint32_t hidden_dim, uint32_t vocab_size,
                                         uint32_t k_heads) {
    const size_t H = hidden_dim, V = vocab_size, K = k_heads;
    if (!H || !V || !K || !hidden_state_ptr || !weights_ptr || !logits_out_ptr) return;
    DevBuf dh(4 * H), dw(4 * K * H * V), dout(4 * K * V);
    if (dh.err || dw.err || dout.err) {
        set_error("rust_sme_mtp_predict_f32: device allocation failed");
        return;
    }
    if (cudaMemcpy(dh.p, hidden_state_ptr, 4 * H, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dw.p, weights_ptr, 4 * K * H * V, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_error("rust_sme_mtp_predict_f32: copy to device failed");
        return;
    }
    mtp_predict_kernel<<<dim3((unsigned)((V + 255) / 256), (unsigned)K), 256>>>(dh.as<float>(), dw.as<float>(),
                                                                               dout.as<float>(), (int)H, (int)V);
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpy(logits_out_ptr, dout.p, 4 * K * V, cudaMemcpyDeviceToHost) != cudaSuccess)
        set_error("rust_sme_mtp_predict_f32: kernel or copy failed");
}

extern "C" void rust_sme_mtp_sample_f32(const float* logits_ptr, int32_t* draft_tokens_out, uint32_t vocab_size,
                                        uint32_t k_heads) {
    const size_t V = vocab_size, K = k_heads;
    if (!V || !K || !logits_ptr || !draft_tokens_out) return;
    DevBuf dl(4 * K * V), dout(4 * K);
    if (dl.err || dout.err) {
        set_error("rust_sme_mtp_sample_f32: device allocation failed");
        return;
    }
    if (cudaMemcpy(dl.p, logits_ptr, 4 * K * V, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_error("rust_sme_mtp_sample_f32: copy to device failed");
        return;
    }
    // each head is one row of a [K, 1, V] "draft" tensor with no length limit
    compat_argmax_kernel<<<(unsigned)K, 256>>>(dl.as<float>(), nullptr, (int)V, 1, dout.as<int32_t>());
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpy(draft_tokens_out, dout.p, 4 * K, cudaMemcpyDeviceToHost) != cudaSuccess)
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
    DevBuf dq(4 * D), dk(4 * L * D), dv(4 * L * D), dout(4 * (D + 2));
    if (dq.err || dk.err || dv.err || dout.err) {
        set_error("rust_sme_flashdecoding_chunk_f32: device allocation failed");
        return;
    }
    cudaMemcpy(dq.p, q_ptr, 4 * D, cudaMemcpyHostToDevice);
    if (L) {
        cudaMemcpy(dk.p, k_chunk_ptr, 4 * L * D, cudaMemcpyHostToDevice);
        cudaMemcpy(dv.p, v_chunk_ptr, 4 * L * D, cudaMemcpyHostToDevice);
    }
    fd_chunk_kernel<<<1, 128>>>(dq.as<float>(), dk.as<float>(), dv.as<float>(), (int)L, (int)D, softmax_scale,
                                dout.as<float>(), dout.as<float>() + D, dout.as<float>() + D + 1);
    std::vector<float> h(D + 2);
    if (cudaGetLastError() != cudaSuccess || cudaMemcpy(h.data(), dout.p, 4 * (D + 2), cudaMemcpyDeviceToHost)) {
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
    const size_t C = num_chunks, D = head_dim;
    if (!D || !partial_o_ptr || !partial_max_ptr || !partial_sum_exp_ptr || !final_o_out) return;
    DevBuf dpo(4 * C * D), dpm(4 * C), dps(4 * C), dout(4 * D);
    if (dpo.err || dpm.err || dps.err || dout.err) {
        set_error("rust_sve2_flashdecoding_reduce_f32: device allocation failed");
        return;
    }
    if (C) {
        cudaMemcpy(dpo.p, partial_o_ptr, 4 * C * D, cudaMemcpyHostToDevice);
        cudaMemcpy(dpm.p, partial_max_ptr, 4 * C, cudaMemcpyHostToDevice);
        cudaMemcpy(dps.p, partial_sum_exp_ptr, 4 * C, cudaMemcpyHostToDevice);
    }
    fd_reduce_kernel<<<1, 128>>>(dpo.as<float>(), dpm.as<float>(), dps.as<float>(), (int)C, (int)D, dout.as<float>());
    if (cudaGetLastError() != cudaSuccess || cudaMemcpy(final_o_out, dout.p, 4 * D, cudaMemcpyDeviceToHost))
        set_error("rust_sve2_flashdecoding_reduce_f32: kernel or copy failed");
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
    DevBuf dq(4 * M * H), dk(4 * pool_floats), dv(4 * pool_floats), doff(4 * (M + 1)), dt(4 * (ntab ? ntab : 1)),
        dl(4 * M), dout(4 * M * H);
    SD_CHECK(!(dq.err || dk.err || dv.err || doff.err || dt.err || dl.err || dout.err), SPECDEC_ENOMEM,
             "paged_attention_compat: device allocation failed");
    SD_CUDA(cudaMemcpy(dq.p, q, 4 * M * H, cudaMemcpyHostToDevice));
    SD_CUDA(cudaMemcpy(dk.p, k_pool, 4 * pool_floats, cudaMemcpyHostToDevice));
    SD_CUDA(cudaMemcpy(dv.p, v_pool, 4 * pool_floats, cudaMemcpyHostToDevice));
    SD_CUDA(cudaMemcpy(doff.p, table_off, 4 * (M + 1), cudaMemcpyHostToDevice));
    if (ntab) SD_CUDA(cudaMemcpy(dt.p, tables, 4 * ntab, cudaMemcpyHostToDevice));
    SD_CUDA(cudaMemcpy(dl.p, seq_lens, 4 * M, cudaMemcpyHostToDevice));
    SD_CUDA(cudaMemcpy(dout.p, o, 4 * M * H, cudaMemcpyHostToDevice));
    compat_paged_attention_kernel<<<M, 128>>>(dq.as<float>(), dk.as<float>(), dv.as<float>(), doff.as<int32_t>(),
                                              dt.as<int32_t>(), dl.as<int32_t>(), dout.as<float>(), (int)H, block_size);
    SD_LAUNCH_CHECK("compat_paged_attention_kernel");
    SD_CUDA(cudaMemcpy(o, dout.p, 4 * M * H, cudaMemcpyDeviceToHost));
    return SPECDEC_OK;
}
