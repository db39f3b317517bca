// attention.cu -- split-KV verify attention over paged fp16 KV (sm_100a).
//
// One CTA per (sequence, KV head, split).  All G = Hq/Hkv query heads of the
// KV head and all R new rows of the sequence are processed together, so every
// KV byte is read from HBM once per step.  KV blocks (16 tokens) are walked
// through the block table and staged into shared memory with 16-byte async
// copies (double buffered); scores and P.V run on the tensor cores
// (m16n8k16, fp16 in, fp32 accumulate) with an online base-2 softmax.
// Masking: a context slot (< ctx_len) is visible to every row; new slot
// ctx_len + j is visible to row r iff bit j of mask[r] is set (chain: causal,
// tree: ancestor-or-self).  Splits are merged by the last CTA to finish
// (atomic ticket, no waiting), with the log-sum-exp combine of
// rust_sve2_flashdecoding_reduce_f32 (lib.rs:1721-1783).
// GQA head map q_head = kv_head * G + g as in lib.rs:841-842.
#include "common.cuh"
#include "internal.h"

namespace specdec {

struct AttnArgs {
    const __half* q;
    const __half* kv;
    int num_blocks, Hkv, Hq, G;
    const int32_t* tables;
    int max_blocks;
    const int32_t* ctx_len;
    const uint64_t* mask;
    int B, R, QR;
    __half* out;
    float* part_o;   // [B, Hkv, S, QRP, HD]
    float* part_ml;  // [B, Hkv, S, QRP, 2]
    int* tickets;    // [B * Hkv]
    int S, QRP;
    float scale_log2;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int HD>
struct AttnCfg {
    static constexpr int LD = HD + 8;           // padded smem row (halves): conflict-free ldmatrix
    static constexpr int BLK_HALVES = 2 * 16 * LD;  // K then V of one 16-token block
};

// MT m-tiles x KG key groups; blockDim = MT * KG * 32.
template <int HD>
__global__ void __launch_bounds__(512) attn_kernel(AttnArgs a, int MT, int KG) {
    using Cfg = AttnCfg<HD>;
    constexpr int LD = Cfg::LD;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half* sQ = reinterpret_cast<__half*>(smem_raw);
    const int QRP = MT * 16;
    __half* sKV = sQ + (size_t)QRP * LD;  // [2 stages][KG blocks][K|V][16][LD]
    float* sMerge = reinterpret_cast<float*>(sKV);  // reused after the main loop

    const int nthreads = blockDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = warp % MT, kg = warp / MT;
    const int split = blockIdx.x % a.S;
    const int bh = blockIdx.x / a.S;
    const int b = bh / a.Hkv, h = bh % a.Hkv;

    const int ctx = a.ctx_len[b];
    const int L = ctx + a.R;
    const int nb = (L + 15) / 16;
    const int per = (nb + a.S - 1) / a.S;
    const int blo = split * per, bhi = min(nb, blo + per);
    const int nchunks = bhi > blo ? (bhi - blo + KG - 1) / KG : 0;

    // ---- Q tile: query vector qi = r * G + g  ->  q[(b*R + r), h*G + g, :]
    for (int idx = threadIdx.x; idx < QRP * (HD / 8); idx += nthreads) {
        const int qi = idx / (HD / 8), c8 = idx % (HD / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (qi < a.QR) {
            const int r = qi / a.G, g = qi % a.G;
            const __half* src = a.q + (((size_t)(b * a.R + r) * a.Hq) + h * a.G + g) * HD + c8 * 8;
            v = *reinterpret_cast<const uint4*>(src);
        }
        *reinterpret_cast<uint4*>(sQ + (size_t)qi * LD + c8 * 8) = v;
    }

    auto load_chunk = [&](int c, int stage) {
        for (int idx = threadIdx.x; idx < KG * 2 * 16 * (HD / 8); idx += nthreads) {
            const int c8 = idx % (HD / 8);
            const int t = (idx / (HD / 8)) % 16;
            const int kv = (idx / (HD / 8 * 16)) % 2;
            const int j = idx / (HD / 8 * 16 * 2);
            const int blk = blo + c * KG + j;
            if (blk >= bhi) continue;
            const int phys = a.tables[(size_t)b * a.max_blocks + blk];
            const __half* src = a.kv + ((((size_t)phys * 2 + kv) * a.Hkv + h) * 16 + t) * HD + c8 * 8;
            __half* dst = sKV + ((size_t)(stage * KG + j) * 2 + kv) * 16 * LD + t * LD + c8 * 8;
            cp_async16(dst, src);
        }
        cp_async_commit();
    };

    if (nchunks > 0) load_chunk(0, 0);
    __syncthreads();

    // Q fragments (A operand) for this warp's m-tile.
    uint32_t qf[HD / 16][4];
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
        const int row = mt * 16 + (lane % 8) + 8 * ((lane / 8) % 2);
        const int col = ks * 16 + 8 * (lane / 16);
        ldmatrix_x4(qf[ks], sQ + (size_t)row * LD + col);
    }

    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    const int qrow0 = mt * 16 + lane / 4;
    uint64_t rmask[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        const int qi = qrow0 + 8 * hr;
        rmask[hr] = qi < a.QR ? a.mask[qi / a.G] : ~0ull;
    }

    for (int c = 0; c < nchunks; ++c) {
        const int stage = c & 1;
        if (c + 1 < nchunks) {
            load_chunk(c + 1, stage ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int blk = blo + c * KG + kg;
        if (blk < bhi) {
            const __half* sK = sKV + ((size_t)(stage * KG + kg) * 2 + 0) * 16 * LD;
            const __half* sV = sKV + ((size_t)(stage * KG + kg) * 2 + 1) * 16 * LD;
            float s[2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                uint32_t kb[4];
                const int key = (lane % 8) + 8 * (lane / 16);
                const int col = ks * 16 + 8 * ((lane / 8) % 2);
                ldmatrix_x4(kb, sK + (size_t)key * LD + col);
                mma16816(s[0], qf[ks], kb[0], kb[1]);
                mma16816(s[1], qf[ks], kb[2], kb[3]);
            }
            // scale + mask
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int hr = e >> 1;
                    const int t = blk * 16 + n * 8 + (lane % 4) * 2 + (e & 1);
                    bool vis = t < L && (t < ctx || ((rmask[hr] >> (t - ctx)) & 1ull));
                    s[n][e] = vis ? s[n][e] * a.scale_log2 : -INFINITY;
                }
            // online softmax (rows lane/4 and lane/4 + 8)
            float alpha[2];
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                float mx = fmaxf(fmaxf(s[0][2 * hr], s[0][2 * hr + 1]), fmaxf(s[1][2 * hr], s[1][2 * hr + 1]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float mnew = fmaxf(m_r[hr], mx);
                const float muse = mnew == -INFINITY ? 0.f : mnew;
                alpha[hr] = exp2f(m_r[hr] - muse);
                m_r[hr] = mnew;
#pragma unroll
                for (int n = 0; n < 2; ++n) {
                    s[n][2 * hr] = exp2f(s[n][2 * hr] - muse);
                    s[n][2 * hr + 1] = exp2f(s[n][2 * hr + 1] - muse);
                }
                l_r[hr] = l_r[hr] * alpha[hr] + s[0][2 * hr] + s[0][2 * hr + 1] + s[1][2 * hr] + s[1][2 * hr + 1];
            }
#pragma unroll
            for (int i = 0; i < HD / 8; ++i) {
                o[i][0] *= alpha[0];
                o[i][1] *= alpha[0];
                o[i][2] *= alpha[1];
                o[i][3] *= alpha[1];
            }
            uint32_t pa[4];
            pa[0] = pack_half2(s[0][0], s[0][1]);
            pa[1] = pack_half2(s[0][2], s[0][3]);
            pa[2] = pack_half2(s[1][0], s[1][1]);
            pa[3] = pack_half2(s[1][2], s[1][3]);
#pragma unroll
            for (int np = 0; np < HD / 16; ++np) {
                uint32_t vb[4];
                const int key = (lane % 8) + 8 * ((lane / 8) % 2);
                const int col = np * 16 + 8 * (lane / 16);
                ldmatrix_x4_trans(vb, sV + (size_t)key * LD + col);
                mma16816(o[2 * np], pa, vb[0], vb[1]);
                mma16816(o[2 * np + 1], pa, vb[2], vb[3]);
            }
        }
        __syncthreads();
    }
    // quad-reduce the row sums
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 1);
        l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 2);
    }

    // ---- merge key groups through shared memory: [KG][QRP][HD] O, [KG][QRP][2] m,l
    float* mO = sMerge;
    float* mML = sMerge + (size_t)KG * QRP * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = mt * 16 + lane / 4 + 8 * (e >> 1);
            const int col = i * 8 + (lane % 4) * 2 + (e & 1);
            mO[((size_t)kg * QRP + row) * HD + col] = o[i][e];
        }
    if ((lane % 4) == 0) {
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int row = mt * 16 + lane / 4 + 8 * hr;
            mML[((size_t)kg * QRP + row) * 2 + 0] = m_r[hr];
            mML[((size_t)kg * QRP + row) * 2 + 1] = l_r[hr];
        }
    }
    __syncthreads();

    // combined (m, l) per row, then O
    const bool single = a.S == 1;
    float* pO = a.part_o + ((size_t)bh * a.S + split) * QRP * HD;
    float* pML = a.part_ml + ((size_t)bh * a.S + split) * QRP * 2;
    for (int idx = threadIdx.x; idx < QRP * HD; idx += nthreads) {
        const int row = idx / HD, col = idx % HD;
        float M = -INFINITY;
        for (int g = 0; g < KG; ++g) M = fmaxf(M, mML[((size_t)g * QRP + row) * 2]);
        const float Muse = M == -INFINITY ? 0.f : M;
        float acc = 0.f, l = 0.f;
        for (int g = 0; g < KG; ++g) {
            const float w = exp2f(mML[((size_t)g * QRP + row) * 2] - Muse);
            acc += mO[((size_t)g * QRP + row) * HD + col] * w;
            l += mML[((size_t)g * QRP + row) * 2 + 1] * w;
        }
        if (single) {
            if (row < a.QR) {
                const int r = row / a.G, g = row % a.G;
                a.out[(((size_t)(b * a.R + r) * a.Hq) + h * a.G + g) * HD + col] =
                    __float2half_rn(l > 0.f ? acc / l : 0.f);
            }
        } else {
            pO[(size_t)row * HD + col] = acc;
            if (col == 0) {
                pML[row * 2 + 0] = M;
                pML[row * 2 + 1] = l;
            }
        }
    }
    if (single) return;

    // ---- last CTA of (b, h) merges the splits
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int t = atomicAdd(&a.tickets[bh], 1);
        s_last = (t == a.S - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* allO = a.part_o + (size_t)bh * a.S * QRP * HD;
    const float* allML = a.part_ml + (size_t)bh * a.S * QRP * 2;
    for (int idx = threadIdx.x; idx < a.QR * HD; idx += nthreads) {
        const int row = idx / HD, col = idx % HD;
        float M = -INFINITY;
        for (int sp = 0; sp < a.S; ++sp) M = fmaxf(M, __ldcg(allML + ((size_t)sp * QRP + row) * 2));
        const float Muse = M == -INFINITY ? 0.f : M;
        float acc = 0.f, l = 0.f;
        for (int sp = 0; sp < a.S; ++sp) {
            const float w = exp2f(__ldcg(allML + ((size_t)sp * QRP + row) * 2) - Muse);
            acc += __ldcg(allO + ((size_t)sp * QRP + row) * HD + col) * w;
            l += __ldcg(allML + ((size_t)sp * QRP + row) * 2 + 1) * w;
        }
        const int r = row / a.G, g = row % a.G;
        a.out[(((size_t)(b * a.R + r) * a.Hq) + h * a.G + g) * HD + col] = __float2half_rn(l > 0.f ? acc / l : 0.f);
    }
    if (threadIdx.x == 0) a.tickets[bh] = 0;
}

struct AttnPlan {
    int MT, KG, S, QRP, threads;
    size_t smem;
};

static AttnPlan plan_attention(int B, int R, int G, int Hkv, int HD, int max_ctx) {
    AttnPlan p;
    const int QR = R * G;
    p.MT = (QR + 15) / 16;
    p.KG = p.MT >= 8 ? 1 : (8 / p.MT);
    if (p.MT * p.KG > 16) p.KG = 1;
    p.QRP = p.MT * 16;
    p.threads = p.MT * p.KG * 32;
    const int LD = HD + 8;
    const size_t q_bytes = (size_t)p.QRP * LD * 2;
    const size_t kv_bytes = (size_t)2 * p.KG * 2 * 16 * LD * 2;
    const size_t merge_bytes = (size_t)p.KG * p.QRP * (HD + 2) * 4;
    p.smem = q_bytes + (kv_bytes > merge_bytes ? kv_bytes : merge_bytes);
    const int nb = (max_ctx + R + 15) / 16;
    int pairs = B * Hkv;
    int want = (4 * 148 + pairs - 1) / pairs;
    int maxs = nb / (2 * p.KG);
    if (maxs < 1) maxs = 1;
    p.S = want < 1 ? 1 : (want > maxs ? maxs : want);
    if (p.S > 64) p.S = 64;
    return p;
}

}  // namespace specdec

using namespace specdec;

namespace specdec {
// Workspace: split tickets first (fixed offset, so plans with different row
// counts sharing one workspace never overlap each other's tickets), then the
// partial O and (m, l) of every split.
static size_t ticket_bytes(size_t pairs) { return (pairs * 4 + 255) / 256 * 256; }
size_t attention_workspace(int B, int R, int Hq, int Hkv, int HD, int max_ctx) {
    AttnPlan p = plan_attention(B, R, Hq / Hkv, Hkv, HD, max_ctx);
    const size_t pairs = (size_t)B * Hkv;
    return ticket_bytes(pairs) + pairs * p.S * p.QRP * HD * 4 + pairs * p.S * p.QRP * 2 * 4;
}

int launch_attention(const __half* q, const __half* kv_layer, int num_blocks, int Hkv, int HD, const int32_t* tables,
                     int max_blocks, const int32_t* ctx_len, const uint64_t* mask, int B, int R, int Hq, __half* out,
                     void* ws, size_t ws_bytes, int max_ctx, cudaStream_t s) {
    SD_CHECK(HD == 64 || HD == 128, SPECDEC_EINVAL, "attention: head_dim must be 64 or 128");
    SD_CHECK(Hkv > 0 && Hq % Hkv == 0 && R >= 1 && R <= 64, SPECDEC_EINVAL, "attention: bad head / row counts");
    AttnPlan p = plan_attention(B, R, Hq / Hkv, Hkv, HD, max_ctx);
    SD_CHECK(p.MT <= 16, SPECDEC_EINVAL, "attention: R * G must be <= 256");
    SD_CHECK(ws && ws_bytes >= attention_workspace(B, R, Hq, Hkv, HD, max_ctx), SPECDEC_EINVAL,
             "attention: workspace too small");
    AttnArgs a;
    a.q = q;
    a.kv = kv_layer;
    a.num_blocks = num_blocks;
    a.Hkv = Hkv;
    a.Hq = Hq;
    a.G = Hq / Hkv;
    a.tables = tables;
    a.max_blocks = max_blocks;
    a.ctx_len = ctx_len;
    a.mask = mask;
    a.B = B;
    a.R = R;
    a.QR = R * a.G;
    a.out = out;
    const size_t pairs = (size_t)B * Hkv;
    char* w = reinterpret_cast<char*>(ws);
    a.tickets = reinterpret_cast<int*>(w);
    a.part_o = reinterpret_cast<float*>(w + ticket_bytes(pairs));
    a.part_ml = reinterpret_cast<float*>(w + ticket_bytes(pairs) + pairs * p.S * p.QRP * HD * 4);
    a.S = p.S;
    a.QRP = p.QRP;
    a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)HD));
    const unsigned grid = (unsigned)(pairs * p.S);
    // opt in once to the largest dynamic shared memory the device allows next
    // to the kernel's static shared memory
    static bool attr128 = false, attr64 = false;
    auto opt_in = [](const void* fn) -> cudaError_t {
        int dev = 0, optin = 0;
        cudaFuncAttributes fa;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, fn);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
        return e;
    };
    if (HD == 128) {
        if (!attr128) {
            SD_CUDA(opt_in(reinterpret_cast<const void*>(attn_kernel<128>)));
            attr128 = true;
        }
        attn_kernel<128><<<grid, p.threads, p.smem, s>>>(a, p.MT, p.KG);
    } else {
        if (!attr64) {
            SD_CUDA(opt_in(reinterpret_cast<const void*>(attn_kernel<64>)));
            attr64 = true;
        }
        attn_kernel<64><<<grid, p.threads, p.smem, s>>>(a, p.MT, p.KG);
    }
    SD_LAUNCH_CHECK("attn_kernel");
    return SPECDEC_OK;
}
}  // namespace specdec

extern "C" size_t specdec_attention_workspace_bytes(int B, int R, int n_q_heads, int n_kv_heads, int head_dim,
                                                    int max_blocks) {
    if (B <= 0 || R <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads) return 0;
    return attention_workspace(B, R, n_q_heads, n_kv_heads, head_dim, max_blocks * 16);
}

extern "C" int specdec_attention(const uint16_t* q, const uint16_t* kv_layer, int num_blocks, int n_kv_heads,
                                 int head_dim, const int32_t* tables, int max_blocks, const int32_t* ctx_len,
                                 const uint64_t* mask, int B, int R, int n_q_heads, uint16_t* out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    SD_CHECK(q && kv_layer && tables && ctx_len && mask && out, SPECDEC_EINVAL, "attention: null argument");
    if (B <= 0) return SPECDEC_OK;
    SD_CHECK(n_kv_heads > 0 && n_q_heads % n_kv_heads == 0, SPECDEC_EINVAL, "attention: bad head counts");
    const size_t need = attention_workspace(B, R, n_q_heads, n_kv_heads, head_dim, max_blocks * 16);
    SD_CHECK(workspace && workspace_bytes >= need, SPECDEC_EINVAL, "attention: workspace too small");
    cudaStream_t s = as_stream(stream);
    // split tickets live at the tail of the workspace; the kernel leaves them zeroed
    SD_CUDA(cudaMemsetAsync(workspace, 0, need, s));
    return launch_attention(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(kv_layer), num_blocks,
                            n_kv_heads, head_dim, tables, max_blocks, ctx_len, mask, B, R, n_q_heads,
                            reinterpret_cast<__half*>(out), workspace, workspace_bytes, max_blocks * 16, s);
}
