// engine.cu -- the speculative step on one B200: MTP drafting, verify forward
// over the paged KV, acceptance, KV commit / rollback.  Everything stays on the
// device; the step is captured once into a CUDA graph and replayed.
//
// Verify forward (shape of run_batched_inference_step, server/main.cpp:252-370):
//   x = emb[token]; per layer: xn = rmsnorm(x); qkv = W4(xn); RoPE(q, k)
//   (lib.rs:621-663); K/V -> paged slots; a = attention; x += W4_o(a);
//   xn = rmsnorm(x); h = silu(W4_gate xn) * W4_up xn (lib.rs:393-457); x += W4_down(h)
//   logits = W4_lm(rmsnorm(x)).
// Drafting (MTP heads, mtp_heads.cpp:53-79 reworked for W4A16 hidden->hidden
// heads sharing the lm_head): h_{i+1} = W4_head[min(i, n-1)](rmsnorm(h_i)),
// draft logits_i = W4_lm(rmsnorm(h_{i+1})), drafts sampled from them.
#include <cuda.h>

#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace specdec {

// -------------------------------------------------------- synthetic data
__device__ __forceinline__ float synth_value(uint32_t seed, uint32_t tid, uint64_t e) {
    uint32_t o[4];
    philox4x32_10((uint32_t)e, (uint32_t)(e >> 32), tid, 0u, seed, 0x5EEDF00Du, o);
    const double inv24 = 1.0 / 16777216.0;
    double s = __dadd_rn(__dadd_rn(__dadd_rn(__dmul_rn((double)(o[0] >> 8), inv24), __dmul_rn((double)(o[1] >> 8), inv24)),
                                   __dmul_rn((double)(o[2] >> 8), inv24)),
                         __dmul_rn((double)(o[3] >> 8), inv24));
    return __double2float_rn(__dmul_rn(__dsub_rn(s, 2.0), 0x1.1bc779ef0d4e8p-5));  // sqrt(3) * 0.02
}

// Row segments of a fused weight matrix: rows [end[i-1], end[i]) come from
// tensor tid[i] (row index relative to the segment start), e.g. QKV = [q|k|v].
// inter > 0 instead interleaves two tensors of inter rows in 128-row blocks
// (row n: tensor tid[(n / 128) % 2], row (n / 256) * 128 + n % 128; zero rows
// past inter), the gate/up layout of the fused SwiGLU GEMM.
struct RowSegs {
    int n;
    int end[3];
    uint32_t tid[3];
    int inter;
};

// One thread per (row n, group g): same quantiser as the oracle generator
// (s = fp16(amax / 7), q = clamp(round(w / s), -8, 7)), written straight into
// the tiled layout used by the GEMM.
__global__ void synth_w4_tiled_kernel(uint32_t seed, RowSegs segs, int N, int K, int KG, int units_n,
                                      uint8_t* __restrict__ tiled) {
    const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= (size_t)units_n * 128 * KG) return;
    const int n = (int)(id / KG), g = (int)(id % KG);
    uint8_t* unit = tiled + ((size_t)(n / 128) * KG + g) * 8448;
    const int r = n % 128;
    const int gl = min(128, K - g * 128);
    if (n >= N || gl <= 0) {
        for (int kc = 0; kc < 16; ++kc) *reinterpret_cast<uint32_t*>(unit + ((kc * 128 + r) << 2)) = 0x88888888u;
        *reinterpret_cast<uint16_t*>(unit + 8192 + r * 2) = 0;
        return;
    }
    uint32_t tid;
    int row;
    if (segs.inter > 0) {
        tid = segs.tid[(n >> 7) & 1];
        row = (n >> 8) * 128 + (n & 127);
        if (row >= segs.inter) {
            for (int kc = 0; kc < 16; ++kc) *reinterpret_cast<uint32_t*>(unit + ((kc * 128 + r) << 2)) = 0x88888888u;
            *reinterpret_cast<uint16_t*>(unit + 8192 + r * 2) = 0;
            return;
        }
    } else {
        int si = 0;
        while (si + 1 < segs.n && n >= segs.end[si]) ++si;
        tid = segs.tid[si];
        row = n - (si ? segs.end[si - 1] : 0);
    }
    float amax = 0.f;
    for (int t = 0; t < gl; ++t)
        amax = fmaxf(amax, fabsf(synth_value(seed, tid, (uint64_t)row * K + (uint64_t)g * 128 + t)));
    __half s16 = __float2half_rn(__fdiv_rn(amax, 7.0f));
    if (amax == 0.f) s16 = __float2half_rn(1.0f);
    const float sf = __half2float(s16);
    *reinterpret_cast<__half*>(unit + 8192 + r * 2) = s16;
    for (int kc = 0; kc < 16; ++kc) {
        uint32_t word = 0;
        for (int i = 0; i < 8; ++i) {
            const int t = kc * 8 + i;
            uint32_t u = 8;
            if (t < gl) {
                const float w = synth_value(seed, tid, (uint64_t)row * K + (uint64_t)g * 128 + t);
                int q = (int)roundf(__fdiv_rn(w, sf));
                q = q < -8 ? -8 : (q > 7 ? 7 : q);
                u = (uint32_t)(q + 8);
            }
            const int j = i >> 1;
            word |= u << ((i & 1) ? (4 * j + 16) : (4 * j));
        }
        *reinterpret_cast<uint32_t*>(unit + ((kc * 128 + r) << 2)) = word;
    }
}

__global__ void synth_f16_kernel(uint32_t seed, uint32_t tid, size_t n, float scale, __half* __restrict__ out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(synth_value(seed, tid, i) * scale);
}
__global__ void synth_f32_kernel(uint32_t seed, uint32_t tid, size_t n, float scale, float* __restrict__ out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = synth_value(seed, tid, i) * scale;
}
__global__ void synth_tokens_kernel(uint32_t seed, int n, int V, int32_t* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t o[4];
    philox4x32_10((uint32_t)i, 0u, 0x70CE7u, 0u, seed, 0x5EEDF00Du, o);
    out[i] = (int32_t)(((uint64_t)o[0] * (uint32_t)V) >> 32);
}

// ------------------------------------------------------- forward pieces
__global__ void embed_kernel(const int32_t* __restrict__ tokens, const __half* __restrict__ emb, int H, int V,
                             float* __restrict__ x) {
    const int m = blockIdx.x;
    int t = tokens[m];
    t = t < 0 ? 0 : (t >= V ? V - 1 : t);
    const __half* e = emb + (size_t)t * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) x[(size_t)m * H + i] = __half2float(e[i]);
}

// out = fp16(x * 1/sqrt(mean(x^2) + eps)) (unit norm weights), lib.rs:21-36.
// One block per row; the row is read from HBM once (float4) into shared
// memory, summed in a fixed order, and written from there.
constexpr int kNormThreads = 256;
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x, int ldx, int H, float eps,
                                                              __half* __restrict__ out, int ldo) {
    extern __shared__ float row_s[];  // [H]
    __shared__ float red[32];
    pdl_trigger();  // a following GEMM may start streaming its weights
    const float* xr = x + (size_t)blockIdx.x * ldx;
    float ss = 0.f;
    const bool vec = (H & 3) == 0 && (ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (vec) {
        for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
            const float4 v = reinterpret_cast<const float4*>(xr)[i];
            reinterpret_cast<float4*>(row_s)[i] = v;
            ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
            ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
            ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
            ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
        }
    } else {
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            const float v = xr[i];
            row_s[i] = v;
            ss = __fadd_rn(ss, __fmul_rn(v, v));
        }
    }
    ss = block_sum<float>(ss, red);  // ends with a barrier: row_s is complete
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)H), eps));
    __half* o = out + (size_t)blockIdx.x * ldo;
    if (vec && (ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0) {
        for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
            const float4 v = reinterpret_cast<const float4*>(row_s)[i];
            __half2 a = __floats2half2_rn(__fmul_rn(v.x, r), __fmul_rn(v.y, r));
            __half2 b = __floats2half2_rn(__fmul_rn(v.z, r), __fmul_rn(v.w, r));
            uint2 w;
            w.x = *reinterpret_cast<uint32_t*>(&a);
            w.y = *reinterpret_cast<uint32_t*>(&b);
            reinterpret_cast<uint2*>(o)[i] = w;
        }
    } else {
        for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = __float2half_rn(__fmul_rn(row_s[i], r));
    }
}
// The same RMSNorm with each thread's float4s of the row held in registers and
// no shared memory beyond the 16-byte reduction, so its CTAs fit beside a
// running GEMM CTA (which leaves ~12K registers and a few KB of shared memory
// on its SM).  Launched as a programmatic dependent, its CTAs become resident
// while the kernel that writes x is still running and wait on
// griddepcontrol.wait, so no launch latency sits between the two.
constexpr int kNormRowThreads = 128;
template <int VPT>  // float4s per thread: H <= 4 * kNormRowThreads * VPT
__global__ void __launch_bounds__(kNormRowThreads) rmsnorm_reg_kernel(const float* __restrict__ x, int ldx, int H,
                                                                      float eps, __half* __restrict__ out, int ldo) {
    __shared__ float red[kNormRowThreads / 32];
    pdl_trigger();  // a following GEMM may start streaming its weights
    pdl_wait();     // x is written by the kernel before this one
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)blockIdx.x * ldx);
    const int n4 = H / 4;
    float4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int j = threadIdx.x + i * kNormRowThreads;
        v[i] = j < n4 ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        ss = __fadd_rn(ss, __fmul_rn(v[i].x, v[i].x));
        ss = __fadd_rn(ss, __fmul_rn(v[i].y, v[i].y));
        ss = __fadd_rn(ss, __fmul_rn(v[i].z, v[i].z));
        ss = __fadd_rn(ss, __fmul_rn(v[i].w, v[i].w));
    }
    ss = block_sum<float>(ss, red);
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)H), eps));
    uint2* o = reinterpret_cast<uint2*>(out + (size_t)blockIdx.x * ldo);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int j = threadIdx.x + i * kNormRowThreads;
        if (j < n4) {
            __half2 a = __floats2half2_rn(__fmul_rn(v[i].x, r), __fmul_rn(v[i].y, r));
            __half2 b = __floats2half2_rn(__fmul_rn(v[i].z, r), __fmul_rn(v[i].w, r));
            uint2 w;
            w.x = *reinterpret_cast<uint32_t*>(&a);
            w.y = *reinterpret_cast<uint32_t*>(&b);
            o[j] = w;
        }
    }
}

template <int VPT>
static cudaError_t launch_rmsnorm_reg(const float* x, int ldx, int rows, int H, float eps, __half* out, int ldo,
                                      cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)rows);
    cfg.blockDim = dim3(kNormRowThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rmsnorm_reg_kernel<VPT>, x, ldx, H, eps, out, ldo);
}

static void launch_rmsnorm(const float* x, int ldx, int rows, int H, float eps, __half* out, int ldo, cudaStream_t s) {
    const bool vec = (H & 3) == 0 && (ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldo & 3) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 7) == 0;
    const int per = 4 * kNormRowThreads;  // row elements per float4 per thread
    if (vec && H <= 16 * per) {
        // a launch error is reported by the caller's launch check
        if (H <= 4 * per) (void)launch_rmsnorm_reg<4>(x, ldx, rows, H, eps, out, ldo, s);
        else if (H <= 8 * per) (void)launch_rmsnorm_reg<8>(x, ldx, rows, H, eps, out, ldo, s);
        else if (H <= 12 * per) (void)launch_rmsnorm_reg<12>(x, ldx, rows, H, eps, out, ldo, s);
        else (void)launch_rmsnorm_reg<16>(x, ldx, rows, H, eps, out, ldo, s);
        return;
    }
    const size_t smem = (size_t)H * sizeof(float);
    static size_t opted = 48 * 1024;
    if (smem > opted) {  // rows wider than 12288 need the opt-in
        cudaFuncSetAttribute(rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        opted = smem;
    }
    rmsnorm_kernel<<<rows, kNormThreads, smem, s>>>(x, ldx, H, eps, out, ldo);
}

// RoPE on q and k (rotate-half pairs d, d + hd/2, as rust_sme_rope_f32,
// src/sme_kernel/rust_sme/src/lib.rs:621-666), K/V into their paged slots,
// q to fp16 (head dims that do not divide 128; otherwise the QKV GEMM's
// epilogue does this).  qkv rows are [q (Hq*hd) | k (Hkv*hd) | v (Hkv*hd)].  A thread
// handles two adjacent dims (d, d+1) of a head: float2 loads, half2 stores.
__global__ void rope_kv_kernel(const float* __restrict__ qkv, int ldq, const int32_t* __restrict__ pos,
                               const int32_t* __restrict__ slot, const int32_t* __restrict__ tables, int max_blocks,
                               int R, const float* __restrict__ cos_t, const float* __restrict__ sin_t, int Hq,
                               int Hkv, int hd, __half* __restrict__ kv_layer, __half* __restrict__ q16) {
    const int m = blockIdx.x;
    const int b = m / R;
    const int half = hd / 2, hp = hd / 4;  // pairs of dims per rotated half
    const float* row = qkv + (size_t)m * ldq;
    const float* cs = cos_t + (size_t)pos[m] * half;
    const float* sn = sin_t + (size_t)pos[m] * half;
    const int s = slot[m];
    const int blk = tables[(size_t)b * max_blocks + s / 16];
    const int off = s % 16;
    const int nrot = (Hq + Hkv) * hp;
    for (int i = threadIdx.x; i < nrot + Hkv * (hd / 2); i += blockDim.x) {
        if (i < nrot) {
            const int h = i / hp, d = (i % hp) * 2;
            const float2 a = *reinterpret_cast<const float2*>(row + h * hd + d);
            const float2 c = *reinterpret_cast<const float2*>(row + h * hd + d + half);
            const float2 cv = *reinterpret_cast<const float2*>(cs + d);
            const float2 sv = *reinterpret_cast<const float2*>(sn + d);
            const __half2 lo = __floats2half2_rn(__fsub_rn(__fmul_rn(a.x, cv.x), __fmul_rn(c.x, sv.x)),
                                                 __fsub_rn(__fmul_rn(a.y, cv.y), __fmul_rn(c.y, sv.y)));
            const __half2 hi = __floats2half2_rn(__fadd_rn(__fmul_rn(c.x, cv.x), __fmul_rn(a.x, sv.x)),
                                                 __fadd_rn(__fmul_rn(c.y, cv.y), __fmul_rn(a.y, sv.y)));
            __half* dst = h < Hq ? q16 + (size_t)m * Hq * hd + h * hd
                                 : kv_layer + ((((size_t)blk * 2 + 0) * Hkv + (h - Hq)) * 16 + off) * hd;
            *reinterpret_cast<__half2*>(dst + d) = lo;
            *reinterpret_cast<__half2*>(dst + d + half) = hi;
        } else {
            const int j = (i - nrot) * 2;
            const int vh = j / hd, d = j % hd;
            const float2 v = *reinterpret_cast<const float2*>(row + (Hq + Hkv) * hd + j);
            __half* dst = kv_layer + ((((size_t)blk * 2 + 1) * Hkv + vh) * 16 + off) * hd;
            *reinterpret_cast<__half2*>(dst + d) = __floats2half2_rn(v.x, v.y);
        }
    }
}

// Global timer (ns) into out[i]: brackets the verify forward in the timed graph.
__global__ void stamp_kernel(unsigned long long* out, int i) {
    if (threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        out[i] = t;
    }
}

// Chain verify rows: [pending, d_0 .. d_{k-1}] at positions ctx .. ctx + k.
__global__ void build_chain_rows_kernel(const int32_t* __restrict__ pending, const int32_t* __restrict__ drafts,
                                        const int32_t* __restrict__ ctx, int B, int k, int32_t* tokens, int32_t* pos,
                                        int32_t* slot) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int R = k + 1;
    if (i >= B * R) return;
    const int b = i / R, r = i % R;
    tokens[i] = r == 0 ? pending[b] : drafts[(size_t)b * k + r - 1];
    pos[i] = ctx[b] + r;
    slot[i] = ctx[b] + r;
}

// Tree verify rows: node 0 = pending, node n at depth d takes candidate
// rank(n) of the level-d top-k list; RoPE position ctx + depth, slot ctx + n.
__global__ void build_tree_rows_kernel(const int32_t* __restrict__ pending, const int32_t* __restrict__ topk, int topk_w,
                                       int levels, const int32_t* __restrict__ depth, const int32_t* __restrict__ rank,
                                       const int32_t* __restrict__ ctx, int B, int R, int32_t* tokens,
                                       int32_t* node_tokens, int32_t* pos, int32_t* slot) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * R) return;
    const int b = i / R, n = i % R;
    int t = pending[b];
    if (n > 0) t = topk[((size_t)b * levels + (depth[n] - 1)) * topk_w + rank[n]];
    tokens[i] = t;
    node_tokens[i] = t;
    pos[i] = ctx[b] + depth[n];
    slot[i] = ctx[b] + n;
}

// Chain commit: new length, next pending token, next draft hidden state.
__global__ void commit_chain_kernel(const int32_t* __restrict__ acc, const int32_t* __restrict__ out_tokens, int R,
                                    const int32_t* __restrict__ ctx, const int32_t* __restrict__ active,
                                    const float* __restrict__ x, int H, int32_t* __restrict__ new_len,
                                    int32_t* __restrict__ pending, float* __restrict__ h0,
                                    unsigned long long* emitted, uint32_t* step) {
    const int b = blockIdx.x;
    const bool on = !active || active[b];
    const int a = acc[b];
    if (on) {
        for (int i = threadIdx.x; i < H; i += blockDim.x) h0[(size_t)b * H + i] = x[((size_t)b * R + a) * H + i];
    }
    if (threadIdx.x == 0) {
        if (on) {
            new_len[b] = ctx[b] + a + 1;
            pending[b] = out_tokens[(size_t)b * R + a];
            atomicAdd(emitted, (unsigned long long)(a + 1));
        } else {
            new_len[b] = ctx[b];  // inactive: roll the reserved slots back
        }
        if (b == 0) atomicAdd(step, 1u);
    }
}

// Tree commit: move the accepted path's K/V (slots ctx + path[t-1]) to
// ctx + t for all layers, then as the chain commit.  grid (B, L).
__global__ void tree_compact_kernel(const int32_t* __restrict__ acc, const int32_t* __restrict__ path, int R,
                                    const int32_t* __restrict__ ctx, const int32_t* __restrict__ tables,
                                    int max_blocks, __half* __restrict__ kv, size_t layer_stride, int Hkv, int hd) {
    extern __shared__ __half sbuf[];
    const int b = blockIdx.x, l = blockIdx.y;
    const int a = acc[b];
    if (a <= 0) return;
    __half* kvl = kv + layer_stride * l;
    const int per = 2 * Hkv * hd;
    for (int i = threadIdx.x; i < a * per; i += blockDim.x) {
        const int t = i / per, rem = i % per;
        const int kvsel = rem / (Hkv * hd), h = (rem / hd) % Hkv, d = rem % hd;
        const int s = ctx[b] + path[(size_t)b * R + t];
        const int blk = tables[(size_t)b * max_blocks + s / 16];
        sbuf[i] = kvl[((((size_t)blk * 2 + kvsel) * Hkv + h) * 16 + s % 16) * hd + d];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < a * per; i += blockDim.x) {
        const int t = i / per, rem = i % per;
        const int kvsel = rem / (Hkv * hd), h = (rem / hd) % Hkv, d = rem % hd;
        const int s = ctx[b] + t + 1;
        const int blk = tables[(size_t)b * max_blocks + s / 16];
        kvl[((((size_t)blk * 2 + kvsel) * Hkv + h) * 16 + s % 16) * hd + d] = sbuf[i];
    }
}

__global__ void commit_tree_kernel(const int32_t* __restrict__ acc, const int32_t* __restrict__ path,
                                   const int32_t* __restrict__ out_tokens, int R, const int32_t* __restrict__ ctx,
                                   const float* __restrict__ x, int H, int32_t* __restrict__ new_len,
                                   int32_t* __restrict__ pending, float* __restrict__ h0, unsigned long long* emitted,
                                   uint32_t* step) {
    const int b = blockIdx.x;
    const int a = acc[b];
    const int last = a > 0 ? path[(size_t)b * R + a - 1] : 0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) h0[(size_t)b * H + i] = x[((size_t)b * R + last) * H + i];
    if (threadIdx.x == 0) {
        new_len[b] = ctx[b] + a + 1;
        pending[b] = out_tokens[(size_t)b * R + a];
        atomicAdd(emitted, (unsigned long long)(a + 1));
        if (b == 0) atomicAdd(step, 1u);
    }
}

__global__ void prefill_rows_kernel(const int32_t* __restrict__ prompts, int P, int c0, int Rp,
                                    const int32_t* __restrict__ ctx, int B, int32_t* tokens, int32_t* pos,
                                    int32_t* slot) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * Rp) return;
    const int b = i / Rp, r = i % Rp;
    tokens[i] = prompts[(size_t)b * P + c0 + r];
    pos[i] = ctx[b] + r;
    slot[i] = ctx[b] + r;
}

// Per sequence b: h0 = the hidden state of its last prefill row (Rp rows per
// sequence in x; none when Rp = 0) and, unless pending is null, the pending
// token = the prompt's last token.
__global__ void prefill_finish_kernel(const int32_t* __restrict__ prompts, int P, const float* __restrict__ x, int Rp,
                                      int H, int32_t* __restrict__ pending, float* __restrict__ h0) {
    const int b = blockIdx.x;
    if (Rp > 0)
        for (int i = threadIdx.x; i < H; i += blockDim.x) h0[(size_t)b * H + i] = x[((size_t)b * Rp + Rp - 1) * H + i];
    if (threadIdx.x == 0 && pending) pending[b] = prompts[(size_t)b * P + P - 1];
}

// Seeded random fp16 K/V for slots [0, ctx_len[b]) of every layer.
__global__ void seed_kv_kernel(uint32_t seed, const int32_t* __restrict__ ctx, const int32_t* __restrict__ tables,
                               int max_blocks, int B, int L, int Hkv, int hd, __half* __restrict__ kv,
                               size_t layer_stride) {
    const int b = blockIdx.x, l = blockIdx.y;
    const int n = ctx[b];
    __half* kvl = kv + layer_stride * l;
    const size_t per_tok = (size_t)2 * Hkv * hd;
    for (size_t i = threadIdx.x; i < (size_t)n * per_tok; i += blockDim.x) {
        const int t = (int)(i / per_tok);
        const int rem = (int)(i % per_tok);
        const int kvsel = rem / (Hkv * hd), h = (rem / hd) % Hkv, d = rem % hd;
        const int blk = tables[(size_t)b * max_blocks + t / 16];
        uint32_t o[4];
        philox4x32_10((uint32_t)i, (uint32_t)b, 0x4B560000u + (uint32_t)l, 0u, seed, 0x5EEDF00Du, o);
        const float v = (float)(int)(o[0] >> 8) * (1.0f / 8388608.0f) - 1.0f;
        kvl[((((size_t)blk * 2 + kvsel) * Hkv + h) * 16 + t % 16) * hd + d] = __float2half_rn(v);
    }
}

}  // namespace specdec

using namespace specdec;

// ============================================================== engine
struct WeightSet {
    uint8_t* qkv = nullptr;
    uint8_t* o = nullptr;
    uint8_t* gu = nullptr;
    uint8_t* down = nullptr;
};

struct specdec_engine {
    specdec_model_config mc{};
    specdec_run_config rc{};
    int device = 0;
    cudaStream_t stream = nullptr;
    bool tree = false;
    int B = 0, R = 0, k = 0, M = 0, Mdraft = 0, Mmax = 0, NQKV = 0, qd = 0, max_blocks = 0, num_blocks = 0;
    int topk_w = 0;
    size_t sz_qkv = 0, sz_o = 0, sz_gu = 0, sz_down = 0, sz_lm = 0, sz_head = 0;
    std::vector<void*> allocs;
    uint8_t* weights = nullptr;
    std::vector<WeightSet> layers;
    uint8_t* lm = nullptr;
    std::vector<uint8_t*> heads;
    __half* emb = nullptr;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    int rope_max = 0;
    __half* kv = nullptr;
    size_t layer_stride = 0;  // halves per layer of the KV pool
    specdec_kv* kvm = nullptr;
    // activations
    float* x = nullptr;
    __half* xn = nullptr;
    float* qkv = nullptr;
    __half* q16 = nullptr;
    __half* att = nullptr;
    __half* hmid = nullptr;
    float* logits = nullptr;
    float* dlogits = nullptr;
    float* dh = nullptr;      // [B, k, H] draft hidden chain
    __half* dxn = nullptr;    // [B * k, H]
    float* h0 = nullptr;      // [B, H]
    // state
    int32_t* pending = nullptr;
    int32_t* drafts = nullptr;
    int32_t* tokens = nullptr;
    int32_t* pos = nullptr;
    int32_t* slot = nullptr;
    uint64_t* mask = nullptr;
    int32_t* acc = nullptr;
    int32_t* out_tokens = nullptr;
    int32_t* path = nullptr;
    int32_t* node_tokens = nullptr;
    int32_t* topk = nullptr;
    int32_t* parent = nullptr;
    int32_t* depth = nullptr;
    int32_t* rank = nullptr;
    int32_t* new_len = nullptr;
    int32_t* active = nullptr;
    uint32_t* step = nullptr;
    unsigned long long* emitted = nullptr;
    // workspaces
    void* gemm_ws = nullptr;
    size_t gemm_ws_bytes = 0;
    void* attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    void* acc_ws = nullptr;
    // host staging (pinned)
    int32_t* h_ctrl = nullptr;
    int32_t* h_out = nullptr;
    // graph
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t gexec = nullptr;
    int kernels_per_step = 0;
    std::vector<int> host_parent;
    std::vector<int32_t> slot_request;  // request id admitted into each slot (-1: none)
    // profiler: an event after every launch; the interval since the previous
    // event is that launch's device time (one stream, in-order execution)
    bool prof_on = false;
    int gemm_cat = 0;
    // verify interval (embedding through the lm_head): a second graph of the
    // same step with a global-timer stamp kernel on each side of the forward
    bool stamp_on = false;
    unsigned long long* stamps = nullptr;
    cudaGraph_t graph_timed = nullptr;
    cudaGraphExec_t gexec_timed = nullptr;
    std::vector<cudaEvent_t> prof_pool;
    std::vector<int> prof_cat;
    size_t prof_used = 0;
};

enum { CAT_GEMM_VERIFY = 0, CAT_ATTENTION = 1, CAT_GEMM_DRAFT = 2, CAT_ACCEPT = 3, CAT_OTHER = 4, CAT_N = 5 };

static void prof_mark(specdec_engine* e, int cat) {
    if (!e->prof_on) return;
    if (e->prof_used == e->prof_pool.size()) {
        cudaEvent_t ev;
        cudaEventCreate(&ev);
        e->prof_pool.push_back(ev);
    }
    cudaEventRecord(e->prof_pool[e->prof_used], e->stream);
    e->prof_cat.push_back(cat);
    ++e->prof_used;
}

namespace {

template <typename T>
int dalloc(specdec_engine* e, T** p, size_t count) {
    void* q = nullptr;
    if (count == 0) count = 1;
    cudaError_t r = cudaMalloc(&q, sizeof(T) * count);
    if (r != cudaSuccess) return cuda_status(r, "engine cudaMalloc");
    e->allocs.push_back(q);
    *p = reinterpret_cast<T*>(q);
    return SPECDEC_OK;
}

int gemm(specdec_engine* e, const __half* X, int M, int K, const uint8_t* w, int N, float* Y, int ldy, int mode) {
    if (plan_gemm_uses_gemv(M, N, K)) {  // few token rows: draft heads, batch-1 steps
        ++e->kernels_per_step;
        int rc = gemv_launch(X, K, K, plan_gemv(M, N, K), w, M, N, Y, ldy, mode, e->stream, /*pdl=*/true);
        prof_mark(e, e->gemm_cat);
        return rc;
    }
    GemmPlan p = plan_gemm(M, N, K);
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, K, p.MT);
    if (rc) return rc;
    ++e->kernels_per_step;
    rc = gemm_launch(map, p, w, M, N, Y, ldy, mode, e->gemm_ws, e->stream, /*pdl=*/true);
    prof_mark(e, e->gemm_cat);
    return rc;
}

// QKV projection + RoPE + K/V into their paged slots in one launch
int gemm_qkv_rope(specdec_engine* e, const __half* X, int M, int K, const uint8_t* w, int N, const RopeArgs& ra) {
    GemmPlan p = plan_gemm_qkv(M, N, K);
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, K, p.MT);
    if (rc) return rc;
    ++e->kernels_per_step;
    rc = gemm_launch_qkv_rope(map, p, w, M, N, ra, e->stream, /*pdl=*/true);
    prof_mark(e, e->gemm_cat);
    return rc;
}

// gate/up projection + SwiGLU in one launch: h fp16 [M, F]
int gemm_swiglu(specdec_engine* e, const __half* X, int M, int K, const uint8_t* w_gu, int F, __half* h) {
    GemmPlan p = plan_gemm_swiglu(M, F, K);
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, K, p.MT);
    if (rc) return rc;
    ++e->kernels_per_step;
    rc = gemm_launch_swiglu(map, p, w_gu, M, F, h, F, e->stream, /*pdl=*/true);
    prof_mark(e, e->gemm_cat);
    return rc;
}

#define ENG_TRY(x)              \
    do {                        \
        int _rc = (x);          \
        if (_rc) return _rc;    \
    } while (0)
// one kernel launched: count it, check the launch, close its profiler interval
#define ENG_LAUNCH_CAT(name, cat)        \
    do {                                 \
        ++e->kernels_per_step;           \
        SD_LAUNCH_CHECK(name);           \
        prof_mark(e, cat);               \
    } while (0)
#define ENG_LAUNCH(name) ENG_LAUNCH_CAT(name, CAT_OTHER)

// Verify forward over Rrows rows per sequence for sequences b0 .. b0 + nseq - 1
// (all of them by default): Rrows * nseq rows in total.
int forward(specdec_engine* e, int Rrows, bool want_logits, int b0 = 0, int nseq = -1) {
    const auto& c = e->mc;
    const int B = nseq < 0 ? e->B : nseq, M = B * Rrows, H = c.hidden, F = c.ffn, hd = c.head_dim;
    cudaStream_t s = e->stream;
    KVState& kvs = kv_state(e->kvm);
    const int32_t* tables = kvs.tables + (size_t)b0 * e->max_blocks;
    const int32_t* ctx = kvs.ctx + b0;
    e->gemm_cat = CAT_GEMM_VERIFY;
    embed_kernel<<<M, 256, 0, s>>>(e->tokens, e->emb, H, c.vocab, e->x);
    ENG_LAUNCH("embed_kernel");
    for (int l = 0; l < c.layers; ++l) {
        const WeightSet& w = e->layers[l];
        __half* kv_l = e->kv + e->layer_stride * l;
        launch_rmsnorm(e->x, H, M, H, c.rms_eps, e->xn, H, s);
        ENG_LAUNCH("rmsnorm_kernel");
        if (128 % hd == 0) {  // whole heads per 128-row unit: RoPE and the KV write in the GEMM epilogue
            RopeArgs ra;
            ra.pos = e->pos;
            ra.slot = e->slot;
            ra.tables = tables;
            ra.max_blocks = e->max_blocks;
            ra.R = Rrows;
            ra.cos_t = e->rope_cos;
            ra.sin_t = e->rope_sin;
            ra.Hq = c.n_q_heads;
            ra.Hkv = c.n_kv_heads;
            ra.hd = hd;
            ra.kv_layer = kv_l;
            ra.q16 = e->q16;
            ENG_TRY(gemm_qkv_rope(e, e->xn, M, H, w.qkv, e->NQKV, ra));
        } else {
            ENG_TRY(gemm(e, e->xn, M, H, w.qkv, e->NQKV, e->qkv, e->NQKV, 0));
            rope_kv_kernel<<<M, 256, 0, s>>>(e->qkv, e->NQKV, e->pos, e->slot, tables, e->max_blocks, Rrows,
                                             e->rope_cos, e->rope_sin, c.n_q_heads, c.n_kv_heads, hd, kv_l, e->q16);
            ENG_LAUNCH("rope_kv_kernel");
        }
        ++e->kernels_per_step;
        ENG_TRY(launch_attention(e->q16, kv_l, e->num_blocks, c.n_kv_heads, hd, tables, e->max_blocks, ctx,
                                 e->mask, B, Rrows, c.n_q_heads, e->att, e->attn_ws, e->attn_ws_bytes,
                                 e->rc.max_ctx, s));
        prof_mark(e, CAT_ATTENTION);
        ENG_TRY(gemm(e, e->att, M, e->qd, w.o, H, e->x, H, 1));
        launch_rmsnorm(e->x, H, M, H, c.rms_eps, e->xn, H, s);
        ENG_LAUNCH("rmsnorm_kernel");
        ENG_TRY(gemm_swiglu(e, e->xn, M, H, w.gu, F, e->hmid));
        ENG_TRY(gemm(e, e->hmid, M, F, w.down, H, e->x, H, 1));
    }
    if (want_logits) {
        launch_rmsnorm(e->x, H, M, H, c.rms_eps, e->xn, H, s);
        ENG_LAUNCH("rmsnorm_kernel");
        ENG_TRY(gemm(e, e->xn, M, H, e->lm, c.vocab, e->logits, c.vocab, 0));
    }
    return SPECDEC_OK;
}

// MTP hidden chain h_1..h_levels from h0, then one lm_head GEMM over all of them.
int draft_hidden_and_logits(specdec_engine* e, int levels) {
    const auto& c = e->mc;
    const int B = e->B, H = c.hidden;
    cudaStream_t s = e->stream;
    e->gemm_cat = CAT_GEMM_DRAFT;
    for (int i = 0; i < levels; ++i) {
        const int head = i < c.n_mtp_heads ? i : c.n_mtp_heads - 1;
        const float* src = i == 0 ? e->h0 : e->dh + (size_t)(i - 1) * H;
        const int lds = i == 0 ? H : levels * H;
        launch_rmsnorm(src, lds, B, H, c.rms_eps, e->dxn, H, s);
        ENG_LAUNCH("rmsnorm_kernel");
        ENG_TRY(gemm(e, e->dxn, B, H, e->heads[head], H, e->dh + (size_t)i * H, levels * H, 0));
    }
    launch_rmsnorm(e->dh, H, B * levels, H, c.rms_eps, e->dxn, H, s);
    ENG_LAUNCH("rmsnorm_kernel");
    ENG_TRY(gemm(e, e->dxn, B * levels, H, e->lm, c.vocab, e->dlogits, c.vocab, 0));
    return SPECDEC_OK;
}

// The four stages of a speculative step, queued on the engine stream.
// draft: MTP heads -> draft logits -> drafted tokens (chain: sampled, with
// their row statistics kept for the acceptance; tree: top-k candidates).
int record_draft(specdec_engine* e) {
    const int B = e->B, V = e->mc.vocab;
    cudaStream_t s = e->stream;
    const auto& sp = e->rc.sampling;
    prof_mark(e, CAT_OTHER);  // step start
    if (!e->tree) {
        const int k = e->k;
        ENG_TRY(draft_hidden_and_logits(e, k));
        ++e->kernels_per_step;
        // the draft rows' statistics go where the acceptance reads them: after the B*(k+1) target rows
        ENG_TRY(launch_sample_rows_dev(e->dlogits, B * k, k, V, sp.temperature, sp.top_p, sp.seed, e->step, e->drafts,
                                       static_cast<char*>(e->acc_ws) + (size_t)B * (k + 1) * kAcceptStatsBytes, s));
    } else {
        const int levels = e->rc.tree_levels;
        ENG_TRY(draft_hidden_and_logits(e, levels));
        ++e->kernels_per_step;
        ENG_TRY(launch_topk(e->dlogits, B * levels, V, e->topk_w, e->topk, s));
    }
    prof_mark(e, CAT_ACCEPT);
    ++e->kernels_per_step;
    return SPECDEC_OK;
}

// verify: reserve the R new K/V slots per sequence, build the verify rows
// (pending token + drafts, or the tree's nodes) and run the target forward
// with logits for every row.
int record_verify(specdec_engine* e) {
    const int B = e->B, R = e->R;
    cudaStream_t s = e->stream;
    KVState& kvs = kv_state(e->kvm);
    ENG_TRY(kv_append_uniform(e->kvm, B, R, s));
    prof_mark(e, CAT_OTHER);
    if (!e->tree) {
        build_chain_rows_kernel<<<(B * R + 127) / 128, 128, 0, s>>>(e->pending, e->drafts, kvs.ctx, B, e->k, e->tokens,
                                                                   e->pos, e->slot);
        ENG_LAUNCH("build_chain_rows_kernel");
    } else {
        build_tree_rows_kernel<<<(B * R + 127) / 128, 128, 0, s>>>(e->pending, e->topk, e->topk_w, e->rc.tree_levels,
                                                                  e->depth, e->rank, kvs.ctx, B, R, e->tokens,
                                                                  e->node_tokens, e->pos, e->slot);
        ENG_LAUNCH("build_tree_rows_kernel");
    }
    if (e->stamp_on) stamp_kernel<<<1, 32, 0, s>>>(e->stamps, 0);
    ENG_TRY(forward(e, R, true));
    if (e->stamp_on) stamp_kernel<<<1, 32, 0, s>>>(e->stamps, 1);
    e->kernels_per_step += e->tree ? 1 : 2;
    return SPECDEC_OK;
}

// accept: the acceptance over the verify logits -> accepted lengths and
// emitted tokens (and the tree's accepted path).
int record_accept(specdec_engine* e) {
    const int B = e->B, R = e->R, V = e->mc.vocab;
    cudaStream_t s = e->stream;
    const auto& sp = e->rc.sampling;
    if (!e->tree) {
        ENG_TRY(launch_accept_chain_dev(e->logits, e->dlogits, e->drafts, B, e->k, V, sp.temperature, sp.top_p,
                                        sp.seed, e->step, e->acc, e->out_tokens, e->acc_ws, true, s));
    } else {
        ENG_TRY(launch_accept_tree_dev(e->logits, e->node_tokens, e->parent, B, R, V, sp.temperature, sp.top_p,
                                       sp.seed, e->step, e->acc, e->path, e->out_tokens, s));
    }
    prof_mark(e, CAT_ACCEPT);
    return SPECDEC_OK;
}

// commit: keep the accepted rows' K/V (the tree moves its accepted path's
// K/V into place), set the next pending token and draft state, advance the
// step counter, and roll the unaccepted reserved slots back.
int record_commit(specdec_engine* e) {
    const auto& c = e->mc;
    const int B = e->B, R = e->R;
    cudaStream_t s = e->stream;
    KVState& kvs = kv_state(e->kvm);
    if (!e->tree) {
        commit_chain_kernel<<<B, 256, 0, s>>>(e->acc, e->out_tokens, R, kvs.ctx, e->active, e->x, c.hidden, e->new_len,
                                              e->pending, e->h0, e->emitted, e->step);
        ENG_LAUNCH("commit_chain_kernel");
    } else {
        const int levels = e->rc.tree_levels;
        const int per = 2 * c.n_kv_heads * c.head_dim;
        const size_t sm = sizeof(__half) * (size_t)levels * per;
        tree_compact_kernel<<<dim3(B, c.layers), 256, sm, s>>>(e->acc, e->path, R, kvs.ctx, kvs.tables, e->max_blocks,
                                                               e->kv, e->layer_stride, c.n_kv_heads, c.head_dim);
        ENG_LAUNCH("tree_compact_kernel");
        commit_tree_kernel<<<B, 256, 0, s>>>(e->acc, e->path, e->out_tokens, R, kvs.ctx, e->x, c.hidden, e->new_len,
                                             e->pending, e->h0, e->emitted, e->step);
        ENG_LAUNCH("commit_tree_kernel");
    }
    ++e->kernels_per_step;
    ENG_TRY(kv_truncate_dev(e->kvm, e->new_len, B, s));
    prof_mark(e, CAT_OTHER);
    return SPECDEC_OK;
}

int record_step(specdec_engine* e) {
    e->kernels_per_step = 0;
    ENG_TRY(record_draft(e));
    ENG_TRY(record_verify(e));
    ENG_TRY(record_accept(e));
    return record_commit(e);
}

int synth_tiled(cudaStream_t s, uint32_t seed, RowSegs segs, int N, int K, uint8_t* dst) {
    const int KG = (K + 127) / 128, units_n = ((N + 255) / 256) * 2;
    const size_t threads = (size_t)units_n * 128 * KG;
    synth_w4_tiled_kernel<<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(seed, segs, N, K, KG, units_n, dst);
    SD_LAUNCH_CHECK("synth_w4_tiled_kernel");
    return SPECDEC_OK;
}

RowSegs one(uint32_t tid, int N) {
    RowSegs r;
    r.n = 1;
    r.inter = 0;
    r.end[0] = N;
    r.tid[0] = tid;
    return r;
}

}  // namespace

extern "C" int specdec_engine_destroy(specdec_engine* e) {
    if (!e) return SPECDEC_OK;
    for (cudaEvent_t ev : e->prof_pool) cudaEventDestroy(ev);
    if (e->gexec_timed) cudaGraphExecDestroy(e->gexec_timed);
    if (e->graph_timed) cudaGraphDestroy(e->graph_timed);
    if (e->gexec) cudaGraphExecDestroy(e->gexec);
    if (e->graph) cudaGraphDestroy(e->graph);
    if (e->kvm) specdec_kv_destroy(e->kvm);
    for (void* p : e->allocs) cudaFree(p);
    if (e->h_ctrl) cudaFreeHost(e->h_ctrl);
    if (e->h_out) cudaFreeHost(e->h_out);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return SPECDEC_OK;
}

extern "C" int specdec_engine_create(const specdec_model_config* mc, const specdec_run_config* rc, int device,
                                     specdec_engine** out) {
    SD_CHECK(mc && rc && out, SPECDEC_EINVAL, "engine_create: null argument");
    SD_CHECK(mc->hidden % 128 == 0 && mc->head_dim % 16 == 0 && mc->n_q_heads % mc->n_kv_heads == 0 &&
                 mc->block_size == 16 && mc->layers > 0 && mc->vocab > 0 && mc->n_mtp_heads > 0 && mc->ffn % 8 == 0,
             SPECDEC_EINVAL, "engine_create: unsupported model shape");
    SD_CHECK(rc->batch > 0 && rc->max_ctx > 0, SPECDEC_EINVAL, "engine_create: bad run config");
    SD_CUDA(cudaSetDevice(device));
    specdec_engine* e = new specdec_engine();
    e->mc = *mc;
    e->rc = *rc;
    e->device = device;
    int rcode = SPECDEC_OK;
    auto fail = [&](int code) {
        specdec_engine_destroy(e);
        return code;
    };
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(SPECDEC_ECUDA);
    const int H = mc->hidden, F = mc->ffn, V = mc->vocab, hd = mc->head_dim, Hkv = mc->n_kv_heads;
    e->tree = rc->tree_nodes > 0;
    e->B = rc->batch;
    e->slot_request.assign(rc->batch, -1);
    if (e->tree) {
        SD_CHECK(rc->tree_nodes <= 64 && rc->tree_levels >= 1 && rc->tree_levels <= 8, SPECDEC_EINVAL,
                 "engine_create: tree must have <= 64 nodes and 1..8 levels");
        // BFS tree with per-level branching, truncated to tree_nodes (root included)
        std::vector<int> parent(1, -1), depth(1, 0), rank(1, 0);
        int lvl_begin = 0, lvl_end = 1, wmax = 1;
        for (int L = 0; L < rc->tree_levels && (int)parent.size() < rc->tree_nodes; ++L) {
            wmax = std::max(wmax, rc->tree_branching[L]);
            for (int p = lvl_begin; p < lvl_end && (int)parent.size() < rc->tree_nodes; ++p)
                for (int cc = 0; cc < rc->tree_branching[L] && (int)parent.size() < rc->tree_nodes; ++cc) {
                    parent.push_back(p);
                    depth.push_back(depth[p] + 1);
                    rank.push_back(cc);
                }
            lvl_begin = lvl_end;
            lvl_end = (int)parent.size();
        }
        e->R = (int)parent.size();
        e->k = rc->tree_levels;
        e->topk_w = wmax;
        e->host_parent = parent;
        std::vector<uint64_t> anc(e->R);
        for (int n = 0; n < e->R; ++n) anc[n] = (n ? anc[parent[n]] : 0ull) | (1ull << n);
        if ((rcode = dalloc(e, &e->parent, e->R)) || (rcode = dalloc(e, &e->depth, e->R)) ||
            (rcode = dalloc(e, &e->rank, e->R)) || (rcode = dalloc(e, &e->mask, 64)))
            return fail(rcode);
        cudaMemcpy(e->parent, parent.data(), 4 * e->R, cudaMemcpyHostToDevice);
        cudaMemcpy(e->depth, depth.data(), 4 * e->R, cudaMemcpyHostToDevice);
        cudaMemcpy(e->rank, rank.data(), 4 * e->R, cudaMemcpyHostToDevice);
        cudaMemcpy(e->mask, anc.data(), 8 * e->R, cudaMemcpyHostToDevice);
    } else {
        SD_CHECK(rc->draft_len >= 1 && rc->draft_len <= 63, SPECDEC_EINVAL, "engine_create: draft_len must be 1..63");
        e->k = rc->draft_len;
        e->R = e->k + 1;
        if ((rcode = dalloc(e, &e->mask, 64))) return fail(rcode);
    }
    // chain / prefill masks: row r sees new slots 0..r (prefill chunks reuse it with up to 64 rows)
    {
        std::vector<uint64_t> chain(64);
        for (int r = 0; r < 64; ++r) chain[r] = (r == 63) ? ~0ull : ((1ull << (r + 1)) - 1);
        if (!e->tree) cudaMemcpy(e->mask, chain.data(), 8 * 64, cudaMemcpyHostToDevice);
    }
    e->M = e->B * e->R;
    e->Mdraft = e->B * e->k;
    const int Mprefill = e->B * 64;
    e->Mmax = std::max(std::max(e->M, e->Mdraft), Mprefill);
    e->qd = mc->n_q_heads * hd;
    e->NQKV = (mc->n_q_heads + 2 * Hkv) * hd;
    e->max_blocks = (rc->max_ctx + 64 + 15) / 16 + 1;
    e->num_blocks = rc->num_blocks > 0 ? rc->num_blocks : e->B * e->max_blocks;
    // weights
    e->sz_qkv = w4_tiled_bytes(e->NQKV, H);
    e->sz_o = w4_tiled_bytes(H, e->qd);
    e->sz_gu = w4_tiled_bytes(128 * swiglu_units(F), H);
    e->sz_down = w4_tiled_bytes(H, F);
    e->sz_lm = w4_tiled_bytes(V, H);
    e->sz_head = w4_tiled_bytes(H, H);
    const size_t per_layer = e->sz_qkv + e->sz_o + e->sz_gu + e->sz_down;
    const size_t wbytes = per_layer * mc->layers + e->sz_lm + e->sz_head * mc->n_mtp_heads;
    if ((rcode = dalloc(e, &e->weights, wbytes))) return fail(rcode);
    uint8_t* wp = e->weights;
    e->layers.resize(mc->layers);
    for (int l = 0; l < mc->layers; ++l) {
        e->layers[l].qkv = wp; wp += e->sz_qkv;
        e->layers[l].o = wp; wp += e->sz_o;
        e->layers[l].gu = wp; wp += e->sz_gu;
        e->layers[l].down = wp; wp += e->sz_down;
    }
    e->lm = wp; wp += e->sz_lm;
    for (int i = 0; i < mc->n_mtp_heads; ++i) { e->heads.push_back(wp); wp += e->sz_head; }
    if ((rcode = dalloc(e, &e->emb, (size_t)V * H))) return fail(rcode);
    // RoPE tables (host double precision, as the oracle)
    e->rope_max = rc->max_ctx + 80;
    {
        const int half = hd / 2;
        std::vector<float> cs((size_t)e->rope_max * half), sn((size_t)e->rope_max * half);
        for (int p = 0; p < e->rope_max; ++p)
            for (int d = 0; d < half; ++d) {
                const double inv = std::pow((double)mc->rope_theta, -2.0 * d / (double)hd);
                const double ang = (double)p * inv;
                cs[(size_t)p * half + d] = (float)std::cos(ang);
                sn[(size_t)p * half + d] = (float)std::sin(ang);
            }
        if ((rcode = dalloc(e, &e->rope_cos, cs.size())) || (rcode = dalloc(e, &e->rope_sin, sn.size())))
            return fail(rcode);
        cudaMemcpy(e->rope_cos, cs.data(), 4 * cs.size(), cudaMemcpyHostToDevice);
        cudaMemcpy(e->rope_sin, sn.data(), 4 * sn.size(), cudaMemcpyHostToDevice);
    }
    // KV pool and block manager
    e->layer_stride = (size_t)e->num_blocks * 2 * Hkv * 16 * hd;
    if ((rcode = dalloc(e, &e->kv, e->layer_stride * mc->layers))) return fail(rcode);
    // zeroed: attention reads whole 16-slot blocks and multiplies the masked
    // slots' V by a zero probability, which stale NaN / Inf bits would defeat
    if (cudaMemset(e->kv, 0, sizeof(__half) * e->layer_stride * mc->layers) != cudaSuccess) return fail(SPECDEC_ECUDA);
    if ((rcode = specdec_kv_create(e->num_blocks, 16, e->B, e->max_blocks, &e->kvm))) return fail(rcode);
    // activations
    const int Mx = e->Mmax;
    if ((rcode = dalloc(e, &e->x, (size_t)Mx * H)) || (rcode = dalloc(e, &e->xn, (size_t)Mx * H)) ||
        (rcode = dalloc(e, &e->qkv, (size_t)Mx * e->NQKV)) || (rcode = dalloc(e, &e->q16, (size_t)Mx * e->qd)) ||
        (rcode = dalloc(e, &e->att, (size_t)Mx * e->qd)) ||
        (rcode = dalloc(e, &e->hmid, (size_t)Mx * F)) || (rcode = dalloc(e, &e->logits, (size_t)e->M * V)) ||
        (rcode = dalloc(e, &e->dlogits, (size_t)e->Mdraft * V)) || (rcode = dalloc(e, &e->dh, (size_t)e->Mdraft * H)) ||
        (rcode = dalloc(e, &e->dxn, (size_t)std::max(e->Mdraft, e->B) * H)) ||
        (rcode = dalloc(e, &e->h0, (size_t)e->B * H)))
        return fail(rcode);
    if ((rcode = dalloc(e, &e->pending, e->B)) || (rcode = dalloc(e, &e->drafts, (size_t)e->B * e->k)) ||
        (rcode = dalloc(e, &e->tokens, Mx)) || (rcode = dalloc(e, &e->pos, Mx)) || (rcode = dalloc(e, &e->slot, Mx)) ||
        (rcode = dalloc(e, &e->acc, e->B)) || (rcode = dalloc(e, &e->out_tokens, (size_t)e->B * e->R)) ||
        (rcode = dalloc(e, &e->path, (size_t)e->B * e->R)) || (rcode = dalloc(e, &e->node_tokens, (size_t)e->B * e->R)) ||
        (rcode = dalloc(e, &e->topk, (size_t)e->B * e->k * std::max(1, e->topk_w))) ||
        (rcode = dalloc(e, &e->new_len, e->B)) || (rcode = dalloc(e, &e->active, e->B)) ||
        (rcode = dalloc(e, &e->step, 1)) || (rcode = dalloc(e, &e->emitted, 1)) ||
        (rcode = dalloc(e, &e->stamps, 2)))
        return fail(rcode);
    cudaMemset(e->step, 0, 4);
    cudaMemset(e->emitted, 0, 8);
    cudaMemset(e->h0, 0, sizeof(float) * e->B * H);
    cudaMemset(e->pending, 0, 4 * e->B);
    {
        std::vector<int32_t> on(e->B, 1);
        cudaMemcpy(e->active, on.data(), 4 * e->B, cudaMemcpyHostToDevice);
    }
    // workspaces
    const int maxN = std::max(std::max(V, 128 * swiglu_units(F)), std::max(e->NQKV, H));
    e->gemm_ws_bytes = gemm_workspace_bound(Mx, maxN, std::max(H, F));
    if ((rcode = dalloc(e, reinterpret_cast<char**>(&e->gemm_ws), e->gemm_ws_bytes))) return fail(rcode);
    cudaMemset(e->gemm_ws, 0, e->gemm_ws_bytes);
    e->attn_ws_bytes = std::max(attention_workspace(e->B, e->R, mc->n_q_heads, Hkv, hd, rc->max_ctx),
                                attention_workspace(e->B, 64, mc->n_q_heads, Hkv, hd, rc->max_ctx));
    if ((rcode = dalloc(e, reinterpret_cast<char**>(&e->attn_ws), e->attn_ws_bytes))) return fail(rcode);
    cudaMemset(e->attn_ws, 0, e->attn_ws_bytes);
    if ((rcode = dalloc(e, reinterpret_cast<char**>(&e->acc_ws), (size_t)e->B * (2 * e->R + 1) * kAcceptStatsBytes))) return fail(rcode);
    if (cudaMallocHost(&e->h_ctrl, sizeof(int32_t) * (e->B + 8)) != cudaSuccess) return fail(SPECDEC_ENOMEM);
    for (int b = 0; b < e->B; ++b) e->h_ctrl[b] = 1;  // every sequence starts active
    if (cudaMallocHost(&e->h_out, sizeof(int32_t) * (e->B * (e->R + 1) + 8)) != cudaSuccess) return fail(SPECDEC_ENOMEM);
    if (cudaDeviceSynchronize() != cudaSuccess) return fail(cuda_status(cudaGetLastError(), "engine_create"));
    *out = e;
    return SPECDEC_OK;
}

extern "C" int specdec_engine_init_weights(specdec_engine* e, uint32_t seed) {
    SD_CHECK(e, SPECDEC_EINVAL, "engine_init_weights: null");
    const auto& c = e->mc;
    cudaStream_t s = e->stream;
    const int H = c.hidden, F = c.ffn, V = c.vocab, hd = c.head_dim;
    auto synth = [&](RowSegs segs, int N, int K, uint8_t* dst) { return synth_tiled(s, seed, segs, N, K, dst); };
    const int qd = c.n_q_heads * hd, kd = c.n_kv_heads * hd;
    int rc;
    // tensor ids: layer l, which (q 0, k 1, v 2, o 3, gate 4, up 5, down 6) -> l * 16 + which
    for (int l = 0; l < c.layers; ++l) {
        const uint32_t base = (uint32_t)l * 16u;
        RowSegs qkv;
        qkv.n = 3;
        qkv.inter = 0;
        qkv.end[0] = qd;
        qkv.end[1] = qd + kd;
        qkv.end[2] = qd + 2 * kd;
        qkv.tid[0] = base + 0;
        qkv.tid[1] = base + 1;
        qkv.tid[2] = base + 2;
        RowSegs gu;
        gu.n = 2;
        gu.end[0] = 0;
        gu.end[1] = 0;
        gu.inter = F;
        gu.tid[0] = base + 4;
        gu.tid[1] = base + 5;
        if ((rc = synth(qkv, e->NQKV, H, e->layers[l].qkv))) return rc;
        if ((rc = synth(one(base + 3, H), H, qd, e->layers[l].o))) return rc;
        if ((rc = synth(gu, 128 * swiglu_units(F), H, e->layers[l].gu))) return rc;
        if ((rc = synth(one(base + 6, H), H, F, e->layers[l].down))) return rc;
    }
    if ((rc = synth(one(0x10001u, V), V, H, e->lm))) return rc;
    for (int i = 0; i < c.n_mtp_heads; ++i)
        if ((rc = synth(one(0x10010u + (uint32_t)i, H), H, H, e->heads[i]))) return rc;
    synth_f16_kernel<<<1184, 256, 0, s>>>(seed, 0x10000u, (size_t)V * H, 1.0f, e->emb);
    SD_LAUNCH_CHECK("synth_f16_kernel");
    SD_CUDA(cudaStreamSynchronize(s));
    return SPECDEC_OK;
}

extern "C" int specdec_engine_load_sme(specdec_engine* e, const specdec_sme* f, uint32_t missing_seed) {
    SD_CHECK(e && f, SPECDEC_EINVAL, "engine_load_sme: null argument");
    specdec_model_config fc{};
    int rc = specdec_sme_model_config(f, &fc);
    if (rc) return rc;
    const auto& c = e->mc;
    SD_CHECK(fc.hidden == c.hidden && fc.layers == c.layers && fc.n_q_heads == c.n_q_heads &&
                 fc.n_kv_heads == c.n_kv_heads && fc.head_dim == c.head_dim && fc.ffn == c.ffn && fc.vocab == c.vocab,
             SPECDEC_EINVAL, "engine_load_sme: the file's model config differs from the engine's");
    cudaStream_t s = e->stream;
    const int H = c.hidden, F = c.ffn, V = c.vocab, hd = c.head_dim;
    const int qd = c.n_q_heads * hd, kd = c.n_kv_heads * hd;
    // staging for row chunks plus one fold vector, released on every return
    // (after the stream has drained)
    struct Scratch {
        cudaStream_t stream = nullptr;
        uint8_t* stage = nullptr;
        float* fold = nullptr;
        ~Scratch() {
            cudaStreamSynchronize(stream);
            if (stage) cudaFree(stage);
            if (fold) cudaFree(fold);
        }
    } sc;
    sc.stream = s;
    const size_t stage_bytes = (size_t)64 << 20;
    SD_CUDA(cudaMalloc(&sc.stage, stage_bytes));
    SD_CUDA(cudaMalloc(&sc.fold, sizeof(float) * (size_t)H));
    auto view = [&](const char* role, int l, uint32_t rows, uint32_t cols, specdec_sme_tensor* v) -> int {
        SD_CHECK(sme_role_view(f, role, l, v), SPECDEC_EFORMAT,
                 std::string("sme: no ") + role + " tensor for layer/head " + std::to_string(l));
        SD_CHECK(v->n_dims == 2 && v->dims[0] == rows && v->dims[1] == cols, SPECDEC_EFORMAT,
                 std::string("sme: ") + v->name + " has the wrong shape");
        return SPECDEC_OK;
    };
    // RMSNorm weight of a role -> the device fold vector (null when absent).
    // One buffer: each copy is stream-ordered after the conversions that read
    // the previous vector.
    auto fold = [&](const char* role, int l, const float** out) -> int {
        specdec_sme_tensor v;
        *out = nullptr;
        if (!sme_role_view(f, role, l, &v)) return SPECDEC_OK;
        SD_CHECK(v.n_dims == 1 && v.dims[0] == (uint32_t)H && !v.quantized, SPECDEC_EFORMAT,
                 std::string("sme: ") + v.name + " must be f32 [hidden]");
        SD_CUDA(cudaMemcpyAsync(sc.fold, v.data, sizeof(float) * H, cudaMemcpyHostToDevice, s));
        *out = sc.fold;
        return SPECDEC_OK;
    };
    auto conv = [&](const specdec_sme_tensor& v, const float* fv, uint8_t* dst, int row0, int layout) {
        return sme_upload_convert(v, fv, dst, ((int)v.dims[1] + 127) / 128, row0, layout, nullptr, sc.stage,
                                  stage_bytes, s);
    };
    const size_t per_layer = e->sz_qkv + e->sz_o + e->sz_gu + e->sz_down;
    const size_t wbytes = per_layer * c.layers + e->sz_lm + e->sz_head * c.n_mtp_heads;
    if ((rc = w4_fill_zero_launch(e->weights, wbytes / 8448, s))) return rc;
    specdec_sme_tensor v;
    const float* fv = nullptr;
    for (int l = 0; l < c.layers; ++l) {
        const WeightSet& w = e->layers[l];
        if ((rc = fold("attn_norm", l, &fv))) return rc;
        if ((rc = view("q", l, qd, H, &v)) || (rc = conv(v, fv, w.qkv, 0, 0))) return rc;
        if ((rc = view("k", l, kd, H, &v)) || (rc = conv(v, fv, w.qkv, qd, 0))) return rc;
        if ((rc = view("v", l, kd, H, &v)) || (rc = conv(v, fv, w.qkv, qd + kd, 0))) return rc;
        if ((rc = view("o", l, H, qd, &v)) || (rc = conv(v, nullptr, w.o, 0, 0))) return rc;
        if ((rc = fold("ffn_norm", l, &fv))) return rc;
        if ((rc = view("gate", l, F, H, &v)) || (rc = conv(v, fv, w.gu, 0, 1))) return rc;
        if ((rc = view("up", l, F, H, &v)) || (rc = conv(v, fv, w.gu, 0, 2))) return rc;
        if ((rc = view("down", l, H, F, &v)) || (rc = conv(v, nullptr, w.down, 0, 0))) return rc;
    }
    if ((rc = fold("norm", 0, &fv))) return rc;
    const char* lm_role = sme_role_view(f, "lm_head", 0, &v) ? "lm_head" : "embed";  // embed: tied output embedding
    if ((rc = view(lm_role, 0, V, H, &v)) || (rc = conv(v, fv, e->lm, 0, 0))) return rc;
    for (int i = 0; i < c.n_mtp_heads; ++i) {
        if (sme_role_view(f, "mtp", i, &v)) {
            if ((rc = fold("mtp_norm", i, &fv))) return rc;
            if ((rc = view("mtp", i, H, H, &v)) || (rc = conv(v, fv, e->heads[i], 0, 0))) return rc;
        } else if ((rc = synth_tiled(s, missing_seed, one(0x10010u + (uint32_t)i, H), H, H, e->heads[i]))) {
            return rc;
        }
    }
    if ((rc = view("embed", 0, V, H, &v))) return rc;
    if ((rc = sme_upload_convert(v, nullptr, nullptr, 0, 0, 0, e->emb, sc.stage, stage_bytes, s))) return rc;
    SD_CUDA(cudaStreamSynchronize(s));
    return SPECDEC_OK;
}

extern "C" int specdec_engine_prefill(specdec_engine* e, const int32_t* prompts, int P) {
    SD_CHECK(e && prompts && P >= 2 && P <= e->rc.max_ctx, SPECDEC_EINVAL, "engine_prefill: bad argument");
    cudaStream_t s = e->stream;
    const int B = e->B, H = e->mc.hidden;
    int32_t* d_prompts = nullptr;
    SD_CUDA(cudaMallocAsync(&d_prompts, sizeof(int32_t) * (size_t)B * P, s));
    SD_CUDA(cudaMemcpyAsync(d_prompts, prompts, sizeof(int32_t) * (size_t)B * P, cudaMemcpyHostToDevice, s));
    // chain mask for the chunk rows
    std::vector<uint64_t> chain(64);
    for (int r = 0; r < 64; ++r) chain[r] = (r == 63) ? ~0ull : ((1ull << (r + 1)) - 1);
    uint64_t* saved_mask = nullptr;
    if (e->tree) {
        SD_CUDA(cudaMallocAsync(&saved_mask, 8 * 64, s));
        SD_CUDA(cudaMemcpyAsync(saved_mask, e->mask, 8 * 64, cudaMemcpyDeviceToDevice, s));
    }
    SD_CUDA(cudaMemcpyAsync(e->mask, chain.data(), 8 * 64, cudaMemcpyHostToDevice, s));
    KVState& kvs = kv_state(e->kvm);
    int rc = SPECDEC_OK;
    const int n_tok = P - 1;  // the last prompt token becomes the pending token
    int last_rp = 0;
    for (int c0 = 0; c0 < n_tok && !rc; c0 += 64) {
        const int Rp = std::min(64, n_tok - c0);
        rc = kv_append_uniform(e->kvm, B, Rp, s);
        if (rc) break;
        prefill_rows_kernel<<<(B * Rp + 127) / 128, 128, 0, s>>>(d_prompts, P, c0, Rp, kvs.ctx, B, e->tokens, e->pos,
                                                                e->slot);
        if (cudaGetLastError() != cudaSuccess) {
            rc = SPECDEC_ECUDA;
            break;
        }
        rc = forward(e, Rp, false);
        last_rp = Rp;
    }
    if (!rc) {
        prefill_finish_kernel<<<B, 256, 0, s>>>(d_prompts, P, e->x, last_rp, H, e->pending, e->h0);
        if (cudaGetLastError() != cudaSuccess) rc = SPECDEC_ECUDA;
    }
    if (e->tree) {
        cudaMemcpyAsync(e->mask, saved_mask, 8 * 64, cudaMemcpyDeviceToDevice, s);
        cudaFreeAsync(saved_mask, s);
    }
    cudaFreeAsync(d_prompts, s);
    SD_CUDA(cudaStreamSynchronize(s));
    if (rc) return rc;
    int st = 0;
    SD_CUDA(cudaMemcpy(&st, kvs.status, sizeof(int), cudaMemcpyDeviceToHost));
    SD_CHECK(!st, SPECDEC_ENOMEM, "engine_prefill: KV block pool exhausted");
    return check_device_status(s);
}

extern "C" int specdec_engine_retire(specdec_engine* e, int seq, specdec_radix* cache) {
    SD_CHECK(e && seq >= 0 && seq < e->B, SPECDEC_EINVAL, "engine_retire: bad argument");
    if (cache && e->slot_request[seq] >= 0) {
        const int rc = specdec_radix_release(cache, e->slot_request[seq]);
        if (rc) return rc;
    }
    e->slot_request[seq] = -1;
    return specdec_kv_free_request(e->kvm, seq, e->stream);
}

namespace {
// Prompt tokens [c_begin, c_end) of slot seq (d_tok[0, T) on the device)
// through the forward in chunks of at most 64 rows under the chain mask, each
// chunk's K/V appended after the slot's context; then h0[seq] = the hidden
// state of the last row processed (when there was one) and, for the final
// chunk of a prompt, pending[seq] = d_tok[T - 1].  A tree engine's node mask
// is saved and put back.  Queued on the engine stream; the caller syncs.
int prefill_slot(specdec_engine* e, int seq, const int32_t* d_tok, int T, int c_begin, int c_end, bool final_chunk) {
    cudaStream_t s = e->stream;
    const int H = e->mc.hidden;
    std::vector<uint64_t> chain(64);
    for (int r = 0; r < 64; ++r) chain[r] = (r == 63) ? ~0ull : ((1ull << (r + 1)) - 1);
    uint64_t* saved_mask = nullptr;
    if (e->tree) {
        SD_CUDA(cudaMallocAsync(&saved_mask, 8 * 64, s));
        SD_CUDA(cudaMemcpyAsync(saved_mask, e->mask, 8 * 64, cudaMemcpyDeviceToDevice, s));
    }
    SD_CUDA(cudaMemcpyAsync(e->mask, chain.data(), 8 * 64, cudaMemcpyHostToDevice, s));
    KVState& kvs = kv_state(e->kvm);
    int rc = SPECDEC_OK, last_rp = 0;
    for (int c0 = c_begin; c0 < c_end && !rc; c0 += 64) {
        const int Rp = std::min(64, c_end - c0);
        if ((rc = kv_append_uniform(e->kvm, 1, Rp, s, seq))) break;
        prefill_rows_kernel<<<(Rp + 127) / 128, 128, 0, s>>>(d_tok, T, c0, Rp, kvs.ctx + seq, 1, e->tokens, e->pos,
                                                            e->slot);
        if (cudaGetLastError() != cudaSuccess) {
            rc = SPECDEC_ECUDA;
            break;
        }
        rc = forward(e, Rp, false, seq, 1);
        last_rp = Rp;
    }
    if (!rc && (last_rp > 0 || final_chunk)) {
        prefill_finish_kernel<<<1, 256, 0, s>>>(d_tok, T, e->x, last_rp, H, final_chunk ? e->pending + seq : nullptr,
                                                e->h0 + (size_t)seq * H);
        if (cudaGetLastError() != cudaSuccess) rc = SPECDEC_ECUDA;
    }
    if (e->tree) {
        cudaMemcpyAsync(e->mask, saved_mask, 8 * 64, cudaMemcpyDeviceToDevice, s);
        cudaFreeAsync(saved_mask, s);
    }
    return rc;
}
}  // namespace

extern "C" int specdec_engine_share_prefix(specdec_engine* e, int seq, int32_t request_id, const int32_t* prompt,
                                           int P, specdec_radix* cache, int32_t* shared_tokens) {
    SD_CHECK(e && prompt && seq >= 0 && seq < e->B && P >= 2 && P <= e->rc.max_ctx, SPECDEC_EINVAL,
             "engine_share_prefix: bad argument");
    int rc = specdec_engine_retire(e, seq, cache);
    if (rc) return rc;
    // longest indexed prefix of the prompt's KV tokens whose source still holds a slot
    int shared = 0;
    if (cache) {
        int32_t m = 0, src = -1;
        if ((rc = specdec_radix_match(cache, prompt, P - 1, &m, &src))) return rc;
        int src_slot = -1;
        for (int b = 0; b < e->B && src >= 0; ++b)
            if (b != seq && e->slot_request[b] == src) src_slot = b;
        if (src_slot >= 0) {
            shared = std::min<int>(m, P - 2) / 16 * 16;  // whole blocks; the last KV token is recomputed
            if (shared > 0 && (rc = specdec_kv_share_prefix(e->kvm, seq, src_slot, shared, e->stream))) return rc;
        }
    }
    e->slot_request[seq] = request_id;
    if (shared_tokens) *shared_tokens = shared;
    return SPECDEC_OK;
}

extern "C" int specdec_engine_admit(specdec_engine* e, int seq, int32_t request_id, const int32_t* prompt, int P,
                                    specdec_radix* cache, int32_t* shared_tokens) {
    SD_CHECK(e && prompt && seq >= 0 && seq < e->B && P >= 2 && P <= e->rc.max_ctx, SPECDEC_EINVAL,
             "engine_admit: bad argument");
    cudaStream_t s = e->stream;
    int32_t shared = 0;
    int rc = specdec_engine_share_prefix(e, seq, request_id, prompt, P, cache, &shared);
    if (rc) return rc;
    e->slot_request[seq] = -1;  // a source only once its prompt is in
    int32_t* d_prompt = nullptr;
    SD_CUDA(cudaMallocAsync(&d_prompt, sizeof(int32_t) * (size_t)P, s));
    SD_CUDA(cudaMemcpyAsync(d_prompt, prompt, sizeof(int32_t) * (size_t)P, cudaMemcpyHostToDevice, s));
    KVState& kvs = kv_state(e->kvm);
    // the last prompt token becomes the pending token
    rc = prefill_slot(e, seq, d_prompt, P, shared, P - 1, true);
    cudaFreeAsync(d_prompt, s);
    SD_CUDA(cudaStreamSynchronize(s));
    if (rc) return rc;
    int st = 0;
    SD_CUDA(cudaMemcpy(&st, kvs.status, sizeof(int), cudaMemcpyDeviceToHost));
    SD_CHECK(!st, SPECDEC_ENOMEM, "engine_admit: KV block pool exhausted");
    if ((rc = check_device_status(s))) return rc;
    if (cache && (rc = specdec_radix_insert(cache, request_id, prompt, P - 1))) return rc;
    e->slot_request[seq] = request_id;
    if (shared_tokens) *shared_tokens = shared;
    return SPECDEC_OK;
}

extern "C" int specdec_engine_prefill_chunk(specdec_engine* e, int seq, int32_t request_id, const int32_t* tokens,
                                            int n, int final_chunk) {
    SD_CHECK(e && tokens && seq >= 0 && seq < e->B && n >= 1, SPECDEC_EINVAL, "engine_prefill_chunk: bad argument");
    cudaStream_t s = e->stream;
    KVState& kvs = kv_state(e->kvm);
    int32_t len = 0, nblk = 0;
    SD_CUDA(cudaMemcpyAsync(&len, kvs.len + seq, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaMemcpyAsync(&nblk, kvs.nblk + seq, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaStreamSynchronize(s));
    const int have = nblk < 0 ? 0 : len;  // K/V tokens the slot holds (a retired slot: none)
    const int n_kv = final_chunk ? n - 1 : n;
    SD_CHECK(have + n <= e->rc.max_ctx, SPECDEC_EINVAL, "engine_prefill_chunk: prompt longer than max_ctx");
    SD_CHECK(have + n_kv >= 1, SPECDEC_EINVAL, "engine_prefill_chunk: a prompt needs a token before the pending one");
    int32_t* d_tok = nullptr;
    SD_CUDA(cudaMallocAsync(&d_tok, sizeof(int32_t) * (size_t)n, s));
    SD_CUDA(cudaMemcpyAsync(d_tok, tokens, sizeof(int32_t) * (size_t)n, cudaMemcpyHostToDevice, s));
    int rc = prefill_slot(e, seq, d_tok, n, 0, n_kv, final_chunk != 0);
    cudaFreeAsync(d_tok, s);
    SD_CUDA(cudaStreamSynchronize(s));
    if (rc) return rc;
    int st = 0;
    SD_CUDA(cudaMemcpy(&st, kvs.status, sizeof(int), cudaMemcpyDeviceToHost));
    SD_CHECK(!st, SPECDEC_ENOMEM, "engine_prefill_chunk: KV block pool exhausted");
    if ((rc = check_device_status(s))) return rc;
    if (request_id >= 0) e->slot_request[seq] = request_id;
    return SPECDEC_OK;
}

extern "C" int specdec_engine_seed_state(specdec_engine* e, const int32_t* ctx_len, uint32_t seed) {
    SD_CHECK(e && ctx_len, SPECDEC_EINVAL, "engine_seed_state: bad argument");
    cudaStream_t s = e->stream;
    const int B = e->B, H = e->mc.hidden;
    for (int b = 0; b < B; ++b)
        SD_CHECK(ctx_len[b] >= 1 && ctx_len[b] <= e->rc.max_ctx, SPECDEC_EINVAL, "engine_seed_state: bad ctx_len");
    std::vector<int32_t> reqs(B);
    for (int b = 0; b < B; ++b) reqs[b] = b;
    int rc = specdec_kv_append(e->kvm, reqs.data(), ctx_len, B, nullptr, s);
    if (rc) return rc;
    KVState& kvs = kv_state(e->kvm);
    // after the append, ctx = 0 and len = ctx_len; fill slots [0, len)
    seed_kv_kernel<<<dim3(B, e->mc.layers), 256, 0, s>>>(seed, kvs.len, kvs.tables, e->max_blocks, B, e->mc.layers,
                                                         e->mc.n_kv_heads, e->mc.head_dim, e->kv, e->layer_stride);
    SD_LAUNCH_CHECK("seed_kv_kernel");
    synth_tokens_kernel<<<(B + 127) / 128, 128, 0, s>>>(seed, B, e->mc.vocab, e->pending);
    SD_LAUNCH_CHECK("synth_tokens_kernel");
    synth_f32_kernel<<<(B * H + 255) / 256, 256, 0, s>>>(seed, 0x40000u, (size_t)B * H, 50.0f, e->h0);
    SD_LAUNCH_CHECK("synth_f32_kernel");
    SD_CUDA(cudaStreamSynchronize(s));
    return SPECDEC_OK;
}

extern "C" int specdec_engine_step(specdec_engine* e) {
    SD_CHECK(e, SPECDEC_EINVAL, "engine_step: null");
    cudaStream_t s = e->stream;
    if (!e->rc.use_graph) return record_step(e);
    if (!e->gexec) {
        // first call: run eagerly once (sets kernel attributes), then capture
        int rc = record_step(e);
        if (rc) return rc;
        SD_CUDA(cudaStreamSynchronize(s));
        SD_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        rc = record_step(e);
        cudaGraph_t g = nullptr;
        cudaError_t ce = cudaStreamEndCapture(s, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return cuda_status(ce, "engine_step capture");
        e->graph = g;
        SD_CUDA(cudaGraphInstantiate(&e->gexec, g, 0));
        return SPECDEC_OK;  // the eager run above was this call's step
    }
    SD_CUDA(cudaGraphLaunch(e->gexec, s));
    return SPECDEC_OK;
}

extern "C" int specdec_engine_step_host(specdec_engine* e, int32_t* out_len, int32_t* out_tokens) {
    SD_CHECK(e, SPECDEC_EINVAL, "engine_step_host: null");
    cudaStream_t s = e->stream;
    const int B = e->B, R = e->R;
    // per-step control input: the active flags of every sequence
    SD_CUDA(cudaMemcpyAsync(e->active, e->h_ctrl, sizeof(int32_t) * B, cudaMemcpyHostToDevice, s));
    int rc = specdec_engine_step(e);
    if (rc) return rc;
    SD_CUDA(cudaMemcpyAsync(e->h_out, e->acc, sizeof(int32_t) * B, cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaMemcpyAsync(e->h_out + B, e->out_tokens, sizeof(int32_t) * B * R, cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaStreamSynchronize(s));
    if (out_len) std::memcpy(out_len, e->h_out, sizeof(int32_t) * B);
    if (out_tokens) std::memcpy(out_tokens, e->h_out + B, sizeof(int32_t) * B * R);
    return SPECDEC_OK;
}

// The step's stages one call at a time (eager launches on the engine stream,
// no host synchronisation): draft, verify forward, accept, K/V commit /
// rollback.  Called in that order they queue exactly what specdec_engine_step
// does; between them a caller may read or replace the drafts
// (specdec_engine_read / _write) or the verify logits.
extern "C" int specdec_engine_draft(specdec_engine* e) {
    SD_CHECK(e, SPECDEC_EINVAL, "engine_draft: null");
    // per-step control input, as specdec_engine_step_host
    SD_CUDA(cudaMemcpyAsync(e->active, e->h_ctrl, sizeof(int32_t) * e->B, cudaMemcpyHostToDevice, e->stream));
    e->kernels_per_step = 0;
    return record_draft(e);
}

extern "C" int specdec_engine_verify_forward(specdec_engine* e) {
    SD_CHECK(e, SPECDEC_EINVAL, "engine_verify_forward: null");
    return record_verify(e);
}

extern "C" int specdec_engine_accept(specdec_engine* e) {
    SD_CHECK(e, SPECDEC_EINVAL, "engine_accept: null");
    return record_accept(e);
}

extern "C" int specdec_engine_kv_commit_rollback(specdec_engine* e) {
    SD_CHECK(e, SPECDEC_EINVAL, "engine_kv_commit_rollback: null");
    return record_commit(e);
}

extern "C" int specdec_engine_set_active(specdec_engine* e, const int32_t* active) {
    SD_CHECK(e && active, SPECDEC_EINVAL, "engine_set_active: bad argument");
    // a copy of the previous flags queued by a step or a draft stage reads this
    // pinned buffer when the stream reaches it: let it finish first
    SD_CUDA(cudaStreamSynchronize(e->stream));
    std::memcpy(e->h_ctrl, active, sizeof(int32_t) * e->B);
    return SPECDEC_OK;
}

extern "C" void* specdec_engine_stream(specdec_engine* e) { return e ? (void*)e->stream : nullptr; }

namespace {
struct View {
    const void* ptr;
    size_t bytes;
};
View engine_view(specdec_engine* e, const char* what) {
    const auto& c = e->mc;
    const std::string w(what ? what : "");
    const size_t B = e->B, R = e->R, k = e->k, H = c.hidden, V = c.vocab;
    KVState& kvs = kv_state(e->kvm);
    if (w == "logits") return {e->logits, 4 * B * R * V};
    if (w == "draft_logits") return {e->dlogits, 4 * B * k * V};
    if (w == "drafts") return {e->drafts, 4 * B * k};
    if (w == "tokens") return {e->tokens, 4 * B * R};
    if (w == "node_tokens") return {e->node_tokens, 4 * B * R};
    if (w == "accepted") return {e->acc, 4 * B};
    if (w == "out_tokens") return {e->out_tokens, 4 * B * R};
    if (w == "path") return {e->path, 4 * B * R};
    if (w == "pending") return {e->pending, 4 * B};
    if (w == "h0") return {e->h0, 4 * B * H};
    if (w == "hidden") return {e->x, 4 * B * R * H};
    if (w == "lens") return {kvs.len, 4 * B};
    if (w == "ctx") return {kvs.ctx, 4 * B};
    if (w == "tables") return {kvs.tables, 4 * B * (size_t)e->max_blocks};
    if (w == "refcounts") return {kvs.ref, 4 * (size_t)e->num_blocks};
    if (w == "kv") return {e->kv, 2 * e->layer_stride * (size_t)c.layers};
    if (w == "step") return {e->step, 4};
    if (w == "mask") return {e->mask, 8 * 64};
    if (w == "emitted") return {e->emitted, 8};
    if (w == "emb") return {e->emb, 2 * V * H};
    if (w == "w_lm") return {e->lm, e->sz_lm};
    // per-layer / per-head weights: "w_qkv<l>", "w_o<l>", "w_gu<l>", "w_down<l>", "w_head<i>"
    for (const char* pre : {"w_qkv", "w_o", "w_gu", "w_down", "w_head"}) {
        const size_t n = std::strlen(pre);
        if (w.compare(0, n, pre) != 0 || w.size() == n || w.size() > n + 4 ||
            w.find_first_not_of("0123456789", n) != std::string::npos)
            continue;
        const int i = std::atoi(w.c_str() + n);
        if (w == std::string(pre) + std::to_string(i)) {
            if (pre[2] == 'h') return i < (int)e->heads.size() ? View{e->heads[i], e->sz_head} : View{nullptr, 0};
            if (i >= c.layers) return {nullptr, 0};
            const WeightSet& ws = e->layers[i];
            if (pre[2] == 'q') return {ws.qkv, e->sz_qkv};
            if (pre[2] == 'o') return {ws.o, e->sz_o};
            if (pre[2] == 'g') return {ws.gu, e->sz_gu};
            return {ws.down, e->sz_down};
        }
    }
    return {nullptr, 0};
}
}  // namespace

extern "C" int specdec_engine_read(specdec_engine* e, const char* what, void* host, size_t bytes) {
    SD_CHECK(e && host, SPECDEC_EINVAL, "engine_read: bad argument");
    View v = engine_view(e, what);
    SD_CHECK(v.ptr, SPECDEC_EINVAL, std::string("engine_read: unknown buffer ") + (what ? what : ""));
    SD_CHECK(bytes <= v.bytes, SPECDEC_EINVAL, "engine_read: too many bytes");
    SD_CUDA(cudaStreamSynchronize(e->stream));
    SD_CUDA(cudaMemcpy(host, v.ptr, bytes, cudaMemcpyDeviceToHost));
    return SPECDEC_OK;
}

extern "C" int specdec_engine_write(specdec_engine* e, const char* what, const void* host, size_t bytes) {
    SD_CHECK(e && host, SPECDEC_EINVAL, "engine_write: bad argument");
    const std::string w(what ? what : "");
    SD_CHECK(w == "h0" || w == "pending" || w == "kv" || w == "drafts", SPECDEC_EINVAL,
             "engine_write: only h0, pending, drafts and kv are writable");
    View v = engine_view(e, what);
    SD_CHECK(bytes <= v.bytes, SPECDEC_EINVAL, "engine_write: too many bytes");
    SD_CUDA(cudaStreamSynchronize(e->stream));
    SD_CUDA(cudaMemcpy(const_cast<void*>(v.ptr), host, bytes, cudaMemcpyHostToDevice));
    return SPECDEC_OK;
}

// Runs `steps` eager steps with an event after every launch and returns the
// device time per step of each kernel category (ms): [0] verify GEMMs,
// [1] attention, [2] draft GEMMs, [3] sampling / acceptance, [4] the rest,
// [5] whole step.  Also returns the verify GEMM launch count per step in [6].
extern "C" int specdec_engine_profile(specdec_engine* e, int steps, float* ms_out) {
    SD_CHECK(e && ms_out && steps > 0, SPECDEC_EINVAL, "engine_profile: bad argument");
    SD_CUDA(cudaStreamSynchronize(e->stream));
    double acc[CAT_N + 2] = {0};
    for (int it = 0; it < steps; ++it) {
        e->prof_on = true;
        e->prof_used = 0;
        e->prof_cat.clear();
        int rc = record_step(e);
        e->prof_on = false;
        if (rc) return rc;
        SD_CUDA(cudaStreamSynchronize(e->stream));
        int ngemm = 0;
        for (size_t i = 1; i < e->prof_used; ++i) {
            float ms = 0.f;
            SD_CUDA(cudaEventElapsedTime(&ms, e->prof_pool[i - 1], e->prof_pool[i]));
            acc[e->prof_cat[i]] += ms;
            ngemm += e->prof_cat[i] == CAT_GEMM_VERIFY;
        }
        float total = 0.f;
        SD_CUDA(cudaEventElapsedTime(&total, e->prof_pool[0], e->prof_pool[e->prof_used - 1]));
        acc[CAT_N] += total;
        acc[CAT_N + 1] += ngemm;
    }
    for (int i = 0; i < CAT_N + 2; ++i) ms_out[i] = (float)(acc[i] / steps);
    return SPECDEC_OK;
}

// One step through a second graph of the same step that stamps the global
// timer (ns) right before the verify forward's first kernel and right after
// its last (the lm_head), and the verify forward's device time (ms) between the
// stamps.  The stamp kernels are launched normally, so each waits for the
// kernel before it to finish and the next one starts only after it.
extern "C" int specdec_engine_step_verify_timed(specdec_engine* e, float* verify_ms) {
    SD_CHECK(e && verify_ms, SPECDEC_EINVAL, "engine_step_verify_timed: bad argument");
    cudaStream_t s = e->stream;
    if (!e->gexec_timed) {
        // an eager step first (kernel attributes), then the capture
        e->stamp_on = true;
        int rc = record_step(e);
        if (!rc) {
            SD_CUDA(cudaStreamSynchronize(s));
            SD_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
            rc = record_step(e);
            cudaGraph_t g = nullptr;
            cudaError_t ce = cudaStreamEndCapture(s, &g);
            e->stamp_on = false;
            if (rc) {
                if (g) cudaGraphDestroy(g);
                return rc;
            }
            if (ce != cudaSuccess) return cuda_status(ce, "engine_step_verify_timed capture");
            e->graph_timed = g;
            SD_CUDA(cudaGraphInstantiate(&e->gexec_timed, g, 0));
        }
        e->stamp_on = false;
        if (rc) return rc;
        // the eager run above was this call's step
    } else {
        SD_CUDA(cudaGraphLaunch(e->gexec_timed, s));
    }
    unsigned long long t[2] = {0, 0};
    SD_CUDA(cudaMemcpyAsync(t, e->stamps, sizeof(t), cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaStreamSynchronize(s));
    *verify_ms = (float)((double)(t[1] - t[0]) * 1e-6);
    return SPECDEC_OK;
}

extern "C" int specdec_engine_info(specdec_engine* e, const char* what, int64_t* value) {
    SD_CHECK(e && value, SPECDEC_EINVAL, "engine_info: bad argument");
    const std::string w(what ? what : "");
    if (w == "rows") *value = e->R;
    else if (w == "draft_len") *value = e->k;
    else if (w == "max_blocks") *value = e->max_blocks;
    else if (w == "num_blocks") *value = e->num_blocks;
    else if (w == "kernels_per_step") *value = e->kernels_per_step;
    else if (w == "weight_bytes") {
        const auto& c = e->mc;
        *value = (int64_t)((e->sz_qkv + e->sz_o + e->sz_gu + e->sz_down) * c.layers + e->sz_lm);
    } else if (w == "head_bytes") *value = (int64_t)e->sz_head;
    else if (w == "kv_layer_stride") *value = (int64_t)e->layer_stride;
    else if (w == "status") {
        int st = 0;
        SD_CUDA(cudaMemcpy(&st, kv_state(e->kvm).status, sizeof(int), cudaMemcpyDeviceToHost));
        int dev = check_device_status(e->stream);
        *value = st ? st : dev;
    } else {
        set_error("engine_info: unknown key " + w);
        return SPECDEC_EINVAL;
    }
    return SPECDEC_OK;
}
