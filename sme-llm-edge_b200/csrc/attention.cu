// attention.cu -- split-KV verify attention over paged fp16 KV (sm_100a).
//
// One CTA per (sequence, KV head, split).  All G = Hq/Hkv query heads of the
// KV head and all R new rows of the sequence are processed together, so every
// KV byte is read from HBM once per step.
//
// The path is HBM-bound, so the kernel is built around keeping enough bytes in
// flight: warp 0 streams the split's KV blocks (16 tokens; K then V, each as
// 64-column halves with 128-byte swizzle) through an ST-deep ring, one TMA
// tensor load per block, block numbers read from a copy of the block-table
// slice in shared memory.  Consumer warps (m-tile mt, key group kg) take blocks
// j = kg, kg + KG, ...: scores and P.V on the tensor cores (m16n8k16, fp16 in,
// fp32 accumulate, swizzle-aware ldmatrix) with an online base-2 softmax, then
// release the stage.  Key groups are merged in shared memory; the S splits of
// one (sequence, KV head) form a thread-block cluster and are merged through
// distributed shared memory with the log-sum-exp combine of
// rust_sve2_flashdecoding_reduce_f32 (lib.rs:1721-1783) -- no global
// workspace, no second kernel.
// Masking: a context slot (< ctx_len) is visible to every row; new slot
// ctx_len + j is visible to row r iff bit j of mask[r] is set (chain: causal,
// tree: ancestor-or-self).  GQA head map q_head = kv_head * G + g as in
// lib.rs:841-842.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace specdec {

constexpr int kAttnMaxWarps = 17;  // producer + up to 16 consumers
// Variant for <= 4 consumer warps (decode / verify rows): launch-bounded for
// three resident CTAs per SM, each thread keeping the HD=128 O tile in registers.
constexpr int kAttnSmallWarps = 5;
constexpr int kBox = 2048;         // 16 tokens x 64 columns fp16, 128-byte rows, 128B swizzle

struct AttnArgs {
    const __half* q;
    int Hkv, Hq, G, num_blocks;
    const int32_t* tables;
    int max_blocks;
    const int32_t* ctx_len;
    const uint64_t* mask;
    int B, R, QR;
    int MT, KG, S, ST, max_per;
    __half* out;
    float scale_log2;
    DeviceStatus* status;
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t r[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
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
// Shared address of (token row, column col) of a swizzled [16][HD] K or V
// block: 64-column boxes of 16 x 128-byte rows; the 16-byte chunk index of a
// row is XORed with the row index mod 8.
__device__ __forceinline__ uint32_t sw_addr(uint32_t blk, int row, int col) {
    return blk + (uint32_t)((col >> 6) * kBox + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4));
}

// Bytes of dynamic shared memory laid out by the kernel (host mirror below).
__host__ __device__ constexpr size_t attn_ring_bytes(int HD, int ST) { return (size_t)ST * 2 * (HD / 64) * kBox; }

template <int HD, int MAXW>
__global__ void __launch_bounds__(MAXW * 32, MAXW == kAttnSmallWarps ? 3 : 1)
    attn_kernel(const __grid_constant__ CUtensorMap kv_map, AttnArgs a) {
    constexpr int NBOX = HD / 64;
    constexpr int BLK = 2 * NBOX * kBox;  // K then V of one 16-token block
    constexpr int LD = HD + 8;            // padded Q row (halves): conflict-free ldmatrix
    extern __shared__ unsigned char smem_raw[];
    unsigned char* ring =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int ST = a.ST, MT = a.MT, KG = a.KG, QRP = MT * 16;
    __half* sQ = reinterpret_cast<__half*>(ring + (size_t)ST * BLK);
    int* tbl = reinterpret_cast<int*>(sQ + (size_t)QRP * LD);
    uint64_t* full = reinterpret_cast<uint64_t*>(tbl + ((a.max_per + 3) & ~3));
    uint64_t* empty = full + ST;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + ST);

    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31;
    const int S = a.S;
    const int split = S > 1 ? (int)cluster_rank() : 0;
    const int pair = blockIdx.x / S;
    const int b = pair / a.Hkv, h = pair % a.Hkv;
    const int ctx = a.ctx_len[b];
    const int L = ctx + a.R;
    const int nb = min((L + 15) / 16, a.max_blocks);  // a table never reads past its row
    const int per = (nb + S - 1) / S;
    const int blo = min(nb, split * per), bhi = min(nb, blo + per);
    const int n = min(bhi - blo, a.max_per);  // the table slice fits its shared-memory copy

    // ---- Q tile (query vector qi = r * G + g -> q[(b*R + r), h*G + g, :]), table slice, barriers
    for (int idx = threadIdx.x; idx < QRP * (HD / 8); idx += blockDim.x) {
        const int qi = idx / (HD / 8), c8 = idx % (HD / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (qi < a.QR) {
            const int r = qi / a.G, g = qi % a.G;
            v = *reinterpret_cast<const uint4*>(a.q + (((size_t)(b * a.R + r) * a.Hq) + h * a.G + g) * HD + c8 * 8);
        }
        *reinterpret_cast<uint4*>(sQ + (size_t)qi * LD + c8 * 8) = v;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) tbl[i] = a.tables[(size_t)b * a.max_blocks + blo + i];
    if (threadIdx.x == 0) {
        for (int i = 0; i < ST; ++i) {
            mbar_init(s_addr(&full[i]), 1);
            mbar_init(s_addr(&empty[i]), MT);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int ncons = MT * KG;
    const int cw = warp - 1, mt = cw % MT, kg = cw / MT;
    const bool consumer = warp >= 1 && cw < ncons;
    float o[HD / 8][4];
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    if (warp == 0) {
        // ------------------------------------------------ KV producer
        bool ok = true;
        int j = 0;
        for (; j < n; ++j) {
            const int s = j % ST;
            if (j >= ST) ok = mbar_wait(s_addr(&empty[s]), ((j / ST) - 1) & 1);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) break;
            if (lane == 0) {
                int phys = tbl[j];
                if (phys < 0 || phys >= a.num_blocks) phys = 0;  // a malformed table reads block 0, never out of range
                const uint32_t fb = s_addr(&full[s]);
                mbar_expect_tx(fb, BLK);
                // the whole block (K and V, all column halves) in one request
                tma_load_5d(s_addr(ring + (size_t)s * BLK), &kv_map, 0, h * 16, 0, 0, phys, fb);
            }
            __syncwarp();
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            record_timeout(a.status, 11);
        }
        // the loads issued have landed before the ring is reused or the CTA exits
        if (j > 0) (void)mbar_wait(s_addr(&full[(j - 1) % ST]), ((j - 1) / ST) & 1);
    } else if (consumer) {
        // ------------------------------------------------ scores, softmax, P.V
        // Q fragments are re-read from shared memory per k-slice (registers go to O)
        const uint32_t q_lane = s_addr(sQ + (size_t)(mt * 16 + (lane % 8) + 8 * ((lane / 8) % 2)) * LD + 8 * (lane / 16));
        const int qrow0 = mt * 16 + lane / 4;
        uint64_t rmask[2];
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int qi = qrow0 + 8 * hr;
            rmask[hr] = qi < a.QR ? a.mask[qi / a.G] : ~0ull;
        }
        bool ok = true;
        for (int j = kg; j < n; j += KG) {
            const int s = j % ST;
            ok = __all_sync(0xffffffffu, mbar_wait(s_addr(&full[s]), (j / ST) & 1));
            if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) break;
            const uint32_t sK = s_addr(ring + (size_t)s * BLK);
            const uint32_t sV = sK + NBOX * kBox;
            const int blk = blo + j;
            float sc[2][4];
#pragma unroll
            for (int nn = 0; nn < 2; ++nn) sc[nn][0] = sc[nn][1] = sc[nn][2] = sc[nn][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                uint32_t kb[4], qf[4];
                ldmatrix_x4(qf, q_lane + ks * 32);
                const int key = (lane % 8) + 8 * (lane / 16);
                const int col = ks * 16 + 8 * ((lane / 8) % 2);
                ldmatrix_x4(kb, sw_addr(sK, key, col));
                mma16816(sc[0], qf, kb[0], kb[1]);
                mma16816(sc[1], qf, kb[2], kb[3]);
            }
            // scale + mask
#pragma unroll
            for (int nn = 0; nn < 2; ++nn)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int hr = e >> 1;
                    const int t = blk * 16 + nn * 8 + (lane % 4) * 2 + (e & 1);
                    const bool vis = t < L && (t < ctx || ((rmask[hr] >> (t - ctx)) & 1ull));
                    sc[nn][e] = vis ? sc[nn][e] * a.scale_log2 : -INFINITY;
                }
            // online softmax (rows lane/4 and lane/4 + 8)
            float alpha[2];
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                float mx = fmaxf(fmaxf(sc[0][2 * hr], sc[0][2 * hr + 1]), fmaxf(sc[1][2 * hr], sc[1][2 * hr + 1]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float mnew = fmaxf(m_r[hr], mx);
                const float muse = mnew == -INFINITY ? 0.f : mnew;
                alpha[hr] = exp2f(m_r[hr] - muse);
                m_r[hr] = mnew;
#pragma unroll
                for (int nn = 0; nn < 2; ++nn) {
                    sc[nn][2 * hr] = exp2f(sc[nn][2 * hr] - muse);
                    sc[nn][2 * hr + 1] = exp2f(sc[nn][2 * hr + 1] - muse);
                }
                l_r[hr] = l_r[hr] * alpha[hr] + sc[0][2 * hr] + sc[0][2 * hr + 1] + sc[1][2 * hr] + sc[1][2 * hr + 1];
            }
#pragma unroll
            for (int i = 0; i < HD / 8; ++i) {
                o[i][0] *= alpha[0];
                o[i][1] *= alpha[0];
                o[i][2] *= alpha[1];
                o[i][3] *= alpha[1];
            }
            uint32_t pa[4];
            pa[0] = pack_half2(sc[0][0], sc[0][1]);
            pa[1] = pack_half2(sc[0][2], sc[0][3]);
            pa[2] = pack_half2(sc[1][0], sc[1][1]);
            pa[3] = pack_half2(sc[1][2], sc[1][3]);
#pragma unroll
            for (int np = 0; np < HD / 16; ++np) {
                uint32_t vb[4];
                const int key = (lane % 8) + 8 * ((lane / 8) % 2);
                const int col = np * 16 + 8 * (lane / 16);
                ldmatrix_x4_trans(vb, sw_addr(sV, key, col));
                mma16816(o[2 * np], pa, vb[0], vb[1]);
                mma16816(o[2 * np + 1], pa, vb[2], vb[3]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(s_addr(&empty[s]));
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            record_timeout(a.status, 12);
        }
        // quad-reduce the row sums
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 1);
            l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 2);
        }
    }
    __syncthreads();  // the ring and the Q tile are free from here on

    // ---- this CTA's partial: pO [QRP][HD] (relative to pM), pM / pL [QRP]
    float* base = reinterpret_cast<float*>(ring);
    float* mO = base;                                 // KG > 1: [KG][QRP][HD]
    float* mML = mO + (size_t)KG * QRP * HD;          //         [KG][QRP][2]
    float* pO = KG > 1 ? mML + (size_t)KG * QRP * 2 : base;
    float* pML = pO + (size_t)QRP * HD;               // [QRP][2] = (m, l)
    if (consumer) {
        float* dO = KG > 1 ? mO + (size_t)kg * QRP * HD : pO;
        float* dML = KG > 1 ? mML + (size_t)kg * QRP * 2 : pML;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = mt * 16 + lane / 4 + 8 * (e >> 1);
                const int col = i * 8 + (lane % 4) * 2 + (e & 1);
                dO[(size_t)row * HD + col] = o[i][e];
            }
        if ((lane % 4) == 0) {
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int row = mt * 16 + lane / 4 + 8 * hr;
                dML[row * 2 + 0] = m_r[hr];
                dML[row * 2 + 1] = l_r[hr];
            }
        }
    }
    __syncthreads();
    if (KG > 1) {
        for (int idx = threadIdx.x; idx < QRP * HD; idx += blockDim.x) {
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
            pO[idx] = acc;
            if (col == 0) {
                pML[row * 2 + 0] = M;
                pML[row * 2 + 1] = l;
            }
        }
        __syncthreads();
    }

    // ---- output: one CTA writes directly; a cluster of S splits merges through DSMEM
    if (S == 1) {
        for (int idx = threadIdx.x; idx < a.QR * HD; idx += blockDim.x) {
            const int row = idx / HD, col = idx % HD;
            const float l = pML[row * 2 + 1];
            const int r = row / a.G, g = row % a.G;
            a.out[(((size_t)(b * a.R + r) * a.Hq) + h * a.G + g) * HD + col] =
                __float2half_rn(l > 0.f ? pO[idx] / l : 0.f);
        }
    } else {
        cluster_sync_all();
        const int r0 = split * a.QR / S, r1 = (split + 1) * a.QR / S;
        for (int idx = threadIdx.x; idx < (r1 - r0) * HD; idx += blockDim.x) {
            const int row = r0 + idx / HD, col = idx % HD;
            const uint32_t aM = s_addr(pML + row * 2), aO = s_addr(pO + (size_t)row * HD + col);
            // every remote load is issued before any is used: one DSMEM round trip
            float pm[8], pl[8], po[8];
#pragma unroll
            for (int p = 0; p < 8; ++p)
                if (p < S) {
                    pm[p] = ld_dsmem_f32(aM, (uint32_t)p);
                    pl[p] = ld_dsmem_f32(aM + 4, (uint32_t)p);
                    po[p] = ld_dsmem_f32(aO, (uint32_t)p);
                }
            float M = -INFINITY;
#pragma unroll
            for (int p = 0; p < 8; ++p)
                if (p < S) M = fmaxf(M, pm[p]);
            const float Muse = M == -INFINITY ? 0.f : M;
            float acc = 0.f, l = 0.f;
#pragma unroll
            for (int p = 0; p < 8; ++p)  // rank order: deterministic
                if (p < S) {
                    const float w = exp2f(pm[p] - Muse);
                    acc += po[p] * w;
                    l += pl[p] * w;
                }
            const int r = row / a.G, g = row % a.G;
            a.out[(((size_t)(b * a.R + r) * a.Hq) + h * a.G + g) * HD + col] = __float2half_rn(l > 0.f ? acc / l : 0.f);
        }
        cluster_sync_all();  // peers keep their partials until every rank has read them
    }
}

// ------------------------------------------------------------ host side
struct AttnPlan {
    int MT, KG, QRP, threads, S, ST, max_per;
    size_t smem;
};

static size_t attn_smem_bytes(int HD, int MT, int ST, int max_per) {
    const int QRP = MT * 16;
    return 1024 + attn_ring_bytes(HD, ST) + (size_t)QRP * (HD + 8) * 2 + (size_t)((max_per + 3) & ~3) * 4 +
           (size_t)ST * 16 + 16;
}
// the merge area (partials of the key groups, then of the CTA) fits in the ring + Q tile
static bool attn_merge_fits(int HD, int MT, int KG, int ST) {
    const size_t QRP = (size_t)MT * 16;
    const size_t need = (KG > 1 ? (size_t)(KG + 1) : 1) * QRP * (HD + 2) * 4;
    return need <= attn_ring_bytes(HD, ST) + QRP * (HD + 8) * 2;
}

static const void* attn_fn(int HD, int threads) {
    const bool small = threads <= kAttnSmallWarps * 32;
    if (HD == 128)
        return small ? reinterpret_cast<const void*>(attn_kernel<128, kAttnSmallWarps>)
                     : reinterpret_cast<const void*>(attn_kernel<128, kAttnMaxWarps>);
    return small ? reinterpret_cast<const void*>(attn_kernel<64, kAttnSmallWarps>)
                 : reinterpret_cast<const void*>(attn_kernel<64, kAttnMaxWarps>);
}

static int attn_optin(int HD, int threads) {
    static bool done[4] = {false, false, false, false};
    const int i = (HD == 128 ? 2 : 0) + (threads <= kAttnSmallWarps * 32 ? 1 : 0);
    if (!done[i]) {
        int dev = 0, optin = 0;
        SD_CUDA(cudaGetDevice(&dev));
        SD_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        SD_CUDA(cudaFuncSetAttribute(attn_fn(HD, threads), cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
        done[i] = true;
    }
    return SPECDEC_OK;
}

// Clusters of S CTAs the device runs at once for this configuration (cached).
static int attn_clusters(int HD, int threads, size_t smem, int S) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, size_t, int>, int> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto key = std::make_tuple(HD, threads, smem, S);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (attn_optin(HD, threads) == SPECDEC_OK) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(S * 148));
        cfg.blockDim = dim3((unsigned)threads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)S;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, attn_fn(HD, threads), &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
    }
    if (n <= 0) n = 148 / S > 0 ? 148 / S : 1;
    cache[key] = n;
    return n;
}

static AttnPlan plan_attention(int B, int R, int G, int Hkv, int HD, int max_ctx) {
    AttnPlan p;
    const int QR = R * G;
    p.MT = (QR + 15) / 16;
    p.KG = p.MT >= 4 ? 1 : 4 / p.MT;
    p.QRP = p.MT * 16;
    p.threads = 32 * (1 + p.MT * p.KG);
    const int nb_max = (max_ctx + R + 15) / 16;
    // Ring depth: most KV bytes in flight per SM (stages x resident CTAs)
    // among the depths whose merge area fits; ties go to the deeper ring.
    int dev = 0, smem_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (smem_sm <= 0) smem_sm = 228 * 1024;
    p.ST = 0;
    int best = -1;
    for (int st = 8; st >= 3; --st) {
        if (!attn_merge_fits(HD, p.MT, p.KG, st)) continue;
        const size_t sm = attn_smem_bytes(HD, p.MT, st, nb_max) + 1024;  // + per-CTA reserve
        const int ctas = (int)(smem_sm / sm) < 1 ? 1 : (int)(smem_sm / sm);
        if (ctas * st > best) {
            best = ctas * st;
            p.ST = st;
        }
    }
    if (p.ST == 0) p.ST = 8;
    // Split count: minimise waves x (blocks per CTA + a fixed cost per CTA).
    // The fixed cost (prologue, ring fill, cluster merge, co-scheduling the
    // cluster) was measured at about 48 blocks' worth of streaming time: with
    // enough pairs to fill the device, one CTA per pair wins.
    const int pairs = B * Hkv;
    p.S = 1;
    long long best_cost = -1;
    for (int S = 1; S <= 8 && S <= nb_max; ++S) {
        const int per = (nb_max + S - 1) / S;
        const size_t sm = attn_smem_bytes(HD, p.MT, p.ST, per);
        const int clusters = attn_clusters(HD, p.threads, sm, S);
        const long long waves = (pairs + clusters - 1) / clusters;
        const long long cost = waves * (per + 48);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            p.S = S;
        }
    }
    p.max_per = (nb_max + p.S - 1) / p.S;
    p.smem = attn_smem_bytes(HD, p.MT, p.ST, p.max_per);
    return p;
}

static PFN_cuTensorMapEncodeTiled_v12000 attn_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// The layer's pool [num_blocks][K|V][Hkv][16][HD] as a 5-D fp16 tensor
// (innermost first): 64 columns, token row h*16 + t (all heads), column half,
// K|V, block.  One box {64, 16, HD/64, 2, 1} is a whole 16-token block of one
// head, landing in shared memory as [K|V][half][token][64] with 128-byte
// swizzle -- the same layout as separate 16 x 64 boxes, in one request.
static int make_kv_tmap(CUtensorMap* map, const __half* kv, int num_blocks, int Hkv, int HD) {
    auto enc = attn_encode();
    SD_CHECK(enc, SPECDEC_ENOTSUP, "cuTensorMapEncodeTiled unavailable");
    SD_CHECK((reinterpret_cast<uintptr_t>(kv) & 15) == 0, SPECDEC_EINVAL, "attention: KV pool must be 16-byte aligned");
    const cuuint64_t row = (cuuint64_t)HD * 2, head_block = row * 16 * Hkv;
    cuuint64_t dims[5] = {64, (cuuint64_t)Hkv * 16, (cuuint64_t)(HD / 64), 2, (cuuint64_t)num_blocks};
    cuuint64_t strides[4] = {row, 128, head_block, 2 * head_block};
    cuuint32_t box[5] = {64, 16, (cuuint32_t)(HD / 64), 2, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<__half*>(kv), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SD_CHECK(r == CUDA_SUCCESS, SPECDEC_EINVAL, "attention: cuTensorMapEncodeTiled failed");
    return SPECDEC_OK;
}

// The kernel needs no global workspace (splits are merged on chip).
size_t attention_workspace(int, int, int, int, int, int) { return 0; }

int launch_attention(const __half* q, const __half* kv_layer, int num_blocks, int Hkv, int HD, const int32_t* tables,
                     int max_blocks, const int32_t* ctx_len, const uint64_t* mask, int B, int R, int Hq, __half* out,
                     void* ws, size_t ws_bytes, int max_ctx, cudaStream_t s) {
    (void)ws;
    (void)ws_bytes;
    SD_CHECK(HD == 64 || HD == 128, SPECDEC_EINVAL, "attention: head_dim must be 64 or 128");
    SD_CHECK(Hkv > 0 && Hq % Hkv == 0 && R >= 1 && R <= 64, SPECDEC_EINVAL, "attention: bad head / row counts");
    SD_CHECK(num_blocks > 0 && max_blocks > 0, SPECDEC_EINVAL, "attention: empty block pool or table");
    AttnPlan p = plan_attention(B, R, Hq / Hkv, Hkv, HD, max_ctx);
    SD_CHECK(p.MT <= 16, SPECDEC_EINVAL, "attention: R * G must be <= 256");
    SD_CHECK(attn_merge_fits(HD, p.MT, p.KG, p.ST), SPECDEC_EINVAL, "attention: merge area does not fit");
    int rc = attn_optin(HD, p.threads);
    if (rc) return rc;
    CUtensorMap map;
    rc = make_kv_tmap(&map, kv_layer, num_blocks, Hkv, HD);
    if (rc) return rc;
    AttnArgs a;
    a.q = q;
    a.Hkv = Hkv;
    a.Hq = Hq;
    a.G = Hq / Hkv;
    a.num_blocks = num_blocks;
    a.tables = tables;
    a.max_blocks = max_blocks;
    a.ctx_len = ctx_len;
    a.mask = mask;
    a.B = B;
    a.R = R;
    a.QR = R * a.G;
    a.MT = p.MT;
    a.KG = p.KG;
    a.S = p.S;
    a.ST = p.ST;
    a.max_per = p.max_per;
    a.out = out;
    a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)HD));
    a.status = device_status_ptr();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(B * Hkv * p.S));
    cfg.blockDim = dim3((unsigned)p.threads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)p.S;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const bool small = p.threads <= kAttnSmallWarps * 32;
    if (HD == 128) {
        if (small) SD_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel<128, kAttnSmallWarps>, map, a));
        else SD_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel<128, kAttnMaxWarps>, map, a));
    } else {
        if (small) SD_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel<64, kAttnSmallWarps>, map, a));
        else SD_CUDA(cudaLaunchKernelEx(&cfg, attn_kernel<64, kAttnMaxWarps>, map, a));
    }
    return SPECDEC_OK;
}
}  // namespace specdec

using namespace specdec;

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
    SD_CHECK(need == 0 || (workspace && workspace_bytes >= need), SPECDEC_EINVAL, "attention: workspace too small");
    return launch_attention(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(kv_layer), num_blocks,
                            n_kv_heads, head_dim, tables, max_blocks, ctx_len, mask, B, R, n_q_heads,
                            reinterpret_cast<__half*>(out), workspace, workspace_bytes, max_blocks * 16, as_stream(stream));
}
