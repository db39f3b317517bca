// kvcache.cu -- device-resident paged-KV block manager.
//
// Same table semantics as PagedKVCache (server/paged_kv_cache.cpp):
//   append_tokens          :50-102 fill the tail block, then take the lowest-
//                                  index free block (68-77); OOM stops (78-81)
//   free_request           :123-134
//   share_prefix           :136-154
//   free_merged_blocks     :178-194
//   evict_least_important  :207-228
//   get_utilization        :197-204
// A batch append in request order is computed in one pass: with no frees in
// between, sequential lowest-free allocation hands out the n lowest free
// indices in ascending order, so a prefix sum over the requests' needs and a
// compaction of the free list reproduce it exactly.
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace specdec {

constexpr int kKVThreads = 1024;

// Block-wide exclusive scan of ints (blockDim.x == kKVThreads).
__device__ int block_excl_scan(int v, int* sh, int* total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
    }
    __syncthreads();
    if (lane == 31) sh[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int w = sh[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        sh[lane] = w;
    }
    __syncthreads();
    const int before = wid ? sh[wid - 1] : 0;
    *total = sh[31];
    __syncthreads();
    return before + x - v;
}

// Batch append (one CTA).  reqs/ntok: n entries (device).  uniform_n >= 0
// means every request in [r0, r0 + n) appends uniform_n tokens.
__global__ void __launch_bounds__(kKVThreads) kv_append_kernel(KVState s, const int32_t* __restrict__ reqs,
                                                               const int32_t* __restrict__ ntok, int n, int uniform_n,
                                                               int r0, int32_t* __restrict__ last_block) {
    __shared__ int sh[32];
    int32_t* need = s.scratch;                       // [n] blocks granted
    int32_t* got_off = s.scratch + s.max_reqs;       // [n] offset into the free list
    int32_t* base_nb = s.scratch + 2 * s.max_reqs;   // [n] table length before the grant
    int32_t* freelist = s.scratch + 3 * s.max_reqs;  // [num_blocks]
    // 1) free-block count and ascending free list
    const int per = (s.num_blocks + blockDim.x - 1) / blockDim.x;
    const int lo = threadIdx.x * per, hi = min(s.num_blocks, lo + per);
    int cnt = 0;
    for (int b = lo; b < hi; ++b) cnt += s.ref[b] == 0;
    int total_free;
    int off = block_excl_scan(cnt, sh, &total_free);
    for (int b = lo; b < hi; ++b)
        if (s.ref[b] == 0) freelist[off++] = b;
    // 2) needs, sequentially (request order matters), by thread 0
    if (threadIdx.x == 0) {
        int avail = total_free, used = 0;
        s.status[0] = 0;
        for (int i = 0; i < n; ++i) {
            const int r = uniform_n >= 0 ? r0 + i : reqs[i];
            const int t = uniform_n >= 0 ? uniform_n : ntok[i];
            if (s.nblk[r] < 0) {
                s.nblk[r] = 0;
                s.len[r] = 0;
            }
            s.ctx[r] = s.len[r];
            const int L = s.len[r], nb = s.nblk[r], bs = s.block_size;
            base_nb[i] = nb;
            got_off[i] = used;
            if (t <= 0) {
                need[i] = 0;
                if (last_block) last_block[i] = -1;
                continue;
            }
            const int want = max(0, (L + t + bs - 1) / bs - nb);
            const int got = min(min(want, avail), s.max_bpr - nb);
            need[i] = got;
            used += got;
            avail -= got;
            const int cap = (nb + got) * bs - L;
            const int added = min(t, cap);
            if (added < t) s.status[0] = SPECDEC_ENOMEM;
            s.len[r] = L + added;
            s.nblk[r] = nb + got;  // a request may appear more than once in a batch
            if (last_block) last_block[i] = added > 0 ? -2 - ((L + added - 1) / bs) : -1;  // resolved below
        }
    }
    __syncthreads();
    // 3) hand out the lowest free indices in request order
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int r = uniform_n >= 0 ? r0 + i : reqs[i];
        for (int j = 0; j < need[i]; ++j) {
            const int blk = freelist[got_off[i] + j];
            s.tables[(size_t)r * s.max_bpr + base_nb[i] + j] = blk;
            s.ref[blk] = 1;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int r = uniform_n >= 0 ? r0 + i : reqs[i];
        if (last_block && last_block[i] <= -2) last_block[i] = s.tables[(size_t)r * s.max_bpr + (-2 - last_block[i])];
    }
}

__global__ void kv_free_request_kernel(KVState s, int req) {
    if (threadIdx.x || blockIdx.x) return;
    if (s.nblk[req] < 0) return;
    for (int i = 0; i < s.nblk[req]; ++i) {
        const int p = s.tables[(size_t)req * s.max_bpr + i];
        if (p >= 0 && p < s.num_blocks) s.ref[p]--;
        s.tables[(size_t)req * s.max_bpr + i] = -1;
    }
    s.nblk[req] = -1;
    s.len[req] = 0;
}

__global__ void kv_share_prefix_kernel(KVState s, int new_req, int src, int shared_len) {
    if (threadIdx.x || blockIdx.x) return;
    if (s.nblk[src] < 0) return;
    const int want = (shared_len + s.block_size - 1) / s.block_size;
    int n = 0;
    // the reference overwrites any existing table of new_req without releasing it
    for (int i = 0; i < want && i < s.nblk[src] && i < s.max_bpr; ++i) {
        const int p = s.tables[(size_t)src * s.max_bpr + i];
        s.tables[(size_t)new_req * s.max_bpr + n++] = p;
        s.ref[p]++;
    }
    for (int i = n; i < s.max_bpr; ++i) s.tables[(size_t)new_req * s.max_bpr + i] = -1;
    s.nblk[new_req] = n;
    s.len[new_req] = shared_len;
}

// mode 0: free_merged_blocks(req, n blocks); mode 1: evict n tokens.
__global__ void kv_tail_free_kernel(KVState s, int req, int n, int mode, int32_t* result) {
    if (threadIdx.x || blockIdx.x) return;
    if (s.nblk[req] < 0 || n <= 0) {
        if (result) *result = 0;
        return;
    }
    int freed = 0;
    while (s.nblk[req] > 0 && freed < n) {
        const int idx = --s.nblk[req];
        const int p = s.tables[(size_t)req * s.max_bpr + idx];
        if (p >= 0 && p < s.num_blocks) s.ref[p]--;
        s.tables[(size_t)req * s.max_bpr + idx] = -1;
        freed += mode == 0 ? 1 : s.block_size;
    }
    const int drop = mode == 0 ? n * s.block_size : freed;
    s.len[req] = max(0, s.len[req] - drop);
    if (result) *result = 1;
}

// Token-granular rollback: one thread per request.
__global__ void kv_truncate_kernel(KVState s, const int32_t* __restrict__ new_len, int n) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    int nl = new_len[r];
    if (nl < 0 || s.nblk[r] < 0) return;
    if (nl > s.len[r]) return;
    const int keep = (nl + s.block_size - 1) / s.block_size;
    while (s.nblk[r] > keep) {
        const int idx = --s.nblk[r];
        const int p = s.tables[(size_t)r * s.max_bpr + idx];
        if (p >= 0 && p < s.num_blocks) atomicSub(&s.ref[p], 1);
        s.tables[(size_t)r * s.max_bpr + idx] = -1;
    }
    s.len[r] = nl;
}

__global__ void kv_used_kernel(KVState s, int32_t* out) {
    __shared__ int sh[32];
    int c = 0;
    for (int b = threadIdx.x; b < s.num_blocks; b += blockDim.x) c += s.ref[b] > 0;
    int tot;
    (void)block_excl_scan(c, sh, &tot);
    if (threadIdx.x == 0) *out = tot;
}

}  // namespace specdec

using namespace specdec;

struct specdec_kv {
    KVState s;
    int32_t* h_tmp = nullptr;  // pinned staging
    int32_t* d_tmp = nullptr;  // device staging [3 * max_reqs + 8]
};

namespace specdec {
KVState& kv_state(specdec_kv* kv) { return kv->s; }
int kv_append_uniform(specdec_kv* kv, int n, int tokens, cudaStream_t s, int r0) {
    kv_append_kernel<<<1, kKVThreads, 0, s>>>(kv->s, nullptr, nullptr, n, tokens, r0, nullptr);
    SD_LAUNCH_CHECK("kv_append_kernel");
    return SPECDEC_OK;
}
int kv_truncate_dev(specdec_kv* kv, const int32_t* new_len_dev, int n, cudaStream_t s) {
    kv_truncate_kernel<<<(n + 127) / 128, 128, 0, s>>>(kv->s, new_len_dev, n);
    SD_LAUNCH_CHECK("kv_truncate_kernel");
    return SPECDEC_OK;
}
}  // namespace specdec

extern "C" int specdec_kv_create(int num_blocks, int block_size, int max_reqs, int max_blocks_per_req,
                                 specdec_kv** out) {
    SD_CHECK(out && num_blocks > 0 && block_size > 0 && max_reqs > 0 && max_blocks_per_req > 0, SPECDEC_EINVAL,
             "kv_create: bad argument");
    specdec_kv* kv = new specdec_kv();
    KVState& s = kv->s;
    s.num_blocks = num_blocks;
    s.block_size = block_size;
    s.max_reqs = max_reqs;
    s.max_bpr = max_blocks_per_req;
    const size_t scratch = (size_t)3 * max_reqs + num_blocks + 32;
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = cudaMalloc(&s.tables, sizeof(int32_t) * (size_t)max_reqs * max_blocks_per_req);
    if (e == cudaSuccess) e = cudaMalloc(&s.nblk, sizeof(int32_t) * max_reqs);
    if (e == cudaSuccess) e = cudaMalloc(&s.len, sizeof(int32_t) * max_reqs);
    if (e == cudaSuccess) e = cudaMalloc(&s.ctx, sizeof(int32_t) * max_reqs);
    if (e == cudaSuccess) e = cudaMalloc(&s.ref, sizeof(int32_t) * num_blocks);
    if (e == cudaSuccess) e = cudaMalloc(&s.scratch, sizeof(int32_t) * scratch);
    if (e == cudaSuccess) e = cudaMalloc(&s.status, sizeof(int32_t) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&kv->d_tmp, sizeof(int32_t) * (3 * (size_t)max_reqs + 8));
    if (e == cudaSuccess) e = cudaMallocHost(&kv->h_tmp, sizeof(int32_t) * (3 * (size_t)max_reqs + 8));
    if (e == cudaSuccess) e = cudaMemset(s.tables, 0xff, sizeof(int32_t) * (size_t)max_reqs * max_blocks_per_req);
    if (e == cudaSuccess) e = cudaMemset(s.nblk, 0xff, sizeof(int32_t) * max_reqs);
    if (e == cudaSuccess) e = cudaMemset(s.len, 0, sizeof(int32_t) * max_reqs);
    if (e == cudaSuccess) e = cudaMemset(s.ctx, 0, sizeof(int32_t) * max_reqs);
    if (e == cudaSuccess) e = cudaMemset(s.ref, 0, sizeof(int32_t) * num_blocks);
    if (e == cudaSuccess) e = cudaMemset(s.status, 0, sizeof(int32_t) * 4);
    if (e != cudaSuccess) {
        specdec_kv_destroy(kv);
        return cuda_status(e, "kv_create");
    }
    *out = kv;
    return SPECDEC_OK;
}

extern "C" int specdec_kv_destroy(specdec_kv* kv) {
    if (!kv) return SPECDEC_OK;
    KVState& s = kv->s;
    cudaFree(s.tables);
    cudaFree(s.nblk);
    cudaFree(s.len);
    cudaFree(s.ctx);
    cudaFree(s.ref);
    cudaFree(s.scratch);
    cudaFree(s.status);
    cudaFree(kv->d_tmp);
    cudaFreeHost(kv->h_tmp);
    delete kv;
    return SPECDEC_OK;
}

extern "C" int specdec_kv_append(specdec_kv* kv, const int32_t* reqs, const int32_t* n_tokens, int n,
                                 int32_t* last_block, void* stream) {
    SD_CHECK(kv && reqs && n_tokens && n >= 0 && n <= kv->s.max_reqs, SPECDEC_EINVAL, "kv_append: bad argument");
    for (int i = 0; i < n; ++i)
        SD_CHECK(reqs[i] >= 0 && reqs[i] < kv->s.max_reqs, SPECDEC_EINVAL, "kv_append: request id out of range");
    if (n == 0) return SPECDEC_OK;
    cudaStream_t s = as_stream(stream);
    int32_t* h = kv->h_tmp;
    for (int i = 0; i < n; ++i) {
        h[i] = reqs[i];
        h[n + i] = n_tokens[i];
    }
    SD_CUDA(cudaMemcpyAsync(kv->d_tmp, h, sizeof(int32_t) * 2 * n, cudaMemcpyHostToDevice, s));
    int32_t* d_out = kv->d_tmp + 2 * n;
    kv_append_kernel<<<1, kKVThreads, 0, s>>>(kv->s, kv->d_tmp, kv->d_tmp + n, n, -1, 0, d_out);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(h, d_out, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e, "kv_append");
    if (last_block)
        for (int i = 0; i < n; ++i) last_block[i] = h[i];
    int st = 0;
    SD_CUDA(cudaMemcpy(&st, kv->s.status, sizeof(int), cudaMemcpyDeviceToHost));
    if (st) {
        set_error("kv_append: KV block pool exhausted (append stopped, as PagedKVCache does)");
        return SPECDEC_ENOMEM;
    }
    return SPECDEC_OK;
}

extern "C" int specdec_kv_free_request(specdec_kv* kv, int req, void* stream) {
    SD_CHECK(kv && req >= 0 && req < kv->s.max_reqs, SPECDEC_EINVAL, "kv_free_request: bad argument");
    kv_free_request_kernel<<<1, 1, 0, as_stream(stream)>>>(kv->s, req);
    SD_LAUNCH_CHECK("kv_free_request_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_kv_share_prefix(specdec_kv* kv, int new_req, int src_req, int shared_len, void* stream) {
    SD_CHECK(kv && new_req >= 0 && new_req < kv->s.max_reqs && src_req >= 0 && src_req < kv->s.max_reqs,
             SPECDEC_EINVAL, "kv_share_prefix: bad argument");
    kv_share_prefix_kernel<<<1, 1, 0, as_stream(stream)>>>(kv->s, new_req, src_req, shared_len);
    SD_LAUNCH_CHECK("kv_share_prefix_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_kv_free_merged_blocks(specdec_kv* kv, int req, int n_blocks, void* stream) {
    SD_CHECK(kv && req >= 0 && req < kv->s.max_reqs, SPECDEC_EINVAL, "kv_free_merged_blocks: bad argument");
    kv_tail_free_kernel<<<1, 1, 0, as_stream(stream)>>>(kv->s, req, n_blocks, 0, nullptr);
    SD_LAUNCH_CHECK("kv_tail_free_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_kv_evict_tokens(specdec_kv* kv, int req, int n_tokens, int* evicted, void* stream) {
    SD_CHECK(kv && req >= 0 && req < kv->s.max_reqs, SPECDEC_EINVAL, "kv_evict_tokens: bad argument");
    cudaStream_t s = as_stream(stream);
    kv_tail_free_kernel<<<1, 1, 0, s>>>(kv->s, req, n_tokens, 1, kv->d_tmp);
    SD_LAUNCH_CHECK("kv_tail_free_kernel");
    if (evicted) {
        SD_CUDA(cudaMemcpyAsync(kv->h_tmp, kv->d_tmp, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
        SD_CUDA(cudaStreamSynchronize(s));
        *evicted = kv->h_tmp[0];
    }
    return SPECDEC_OK;
}

extern "C" int specdec_kv_truncate(specdec_kv* kv, const int32_t* new_len, int n, void* stream) {
    SD_CHECK(kv && new_len && n >= 0 && n <= kv->s.max_reqs, SPECDEC_EINVAL, "kv_truncate: bad argument");
    if (n == 0) return SPECDEC_OK;
    cudaStream_t s = as_stream(stream);
    for (int i = 0; i < n; ++i) kv->h_tmp[i] = new_len[i];
    SD_CUDA(cudaMemcpyAsync(kv->d_tmp, kv->h_tmp, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s));
    int rc = kv_truncate_dev(kv, kv->d_tmp, n, s);
    if (rc) return rc;
    SD_CUDA(cudaStreamSynchronize(s));
    return SPECDEC_OK;
}

extern "C" float specdec_kv_utilization(specdec_kv* kv, void* stream) {
    if (!kv) return -1.0f;
    cudaStream_t s = as_stream(stream);
    kv_used_kernel<<<1, kKVThreads, 0, s>>>(kv->s, kv->d_tmp);
    if (cudaGetLastError() != cudaSuccess) return -1.0f;
    if (cudaMemcpyAsync(kv->h_tmp, kv->d_tmp, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess) return -1.0f;
    if (cudaStreamSynchronize(s) != cudaSuccess) return -1.0f;
    return (float)kv->h_tmp[0] / (float)kv->s.num_blocks;
}

extern "C" int specdec_kv_read(specdec_kv* kv, int32_t* tables, int32_t* lens, int32_t* refcounts, void* stream) {
    SD_CHECK(kv, SPECDEC_EINVAL, "kv_read: null");
    cudaStream_t s = as_stream(stream);
    const KVState& st = kv->s;
    if (tables)
        SD_CUDA(cudaMemcpyAsync(tables, st.tables, sizeof(int32_t) * (size_t)st.max_reqs * st.max_bpr,
                                cudaMemcpyDeviceToHost, s));
    if (lens) SD_CUDA(cudaMemcpyAsync(lens, st.len, sizeof(int32_t) * st.max_reqs, cudaMemcpyDeviceToHost, s));
    if (refcounts)
        SD_CUDA(cudaMemcpyAsync(refcounts, st.ref, sizeof(int32_t) * st.num_blocks, cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaStreamSynchronize(s));
    return SPECDEC_OK;
}

extern "C" int32_t* specdec_kv_tables_dev(specdec_kv* kv) { return kv ? kv->s.tables : nullptr; }
extern "C" int32_t* specdec_kv_lens_dev(specdec_kv* kv) { return kv ? kv->s.len : nullptr; }
