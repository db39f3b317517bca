// gemv_w4a16.cu -- the W4A16 contraction for few token rows (M <= 64): decode
// steps at batch 1, the MTP draft heads (one row per sequence), the tiny
// model.  The weights are streamed once from HBM and every output column
// needs only M dot products, so the work is a bandwidth-bound matrix-vector
// product; the 128-row tcgen05 tiles of gemm_w4a16.cu spend most of their
// time in per-tile setup (TMEM allocation, accumulator drain) at these sizes.
//
// Y[m, n] (op)= sum_k X[m, k] * deq(W)[n, k], the operands and the tiled weight
// layout of gemm_w4a16.cu (units of 128 rows x 128 k: words [kc][row], nibble
// j = k_2j, nibble j + 4 = k_2j+1, then 128 fp16 group scales), and the same
// dequantised values: fp16((u - 8) * scale), one rounding.  Reference shapes:
// gemv_s8_f32_batched (server/sme_gemm.cpp:41-66) and rust_sme_mtp_predict_f32
// (src/sme_kernel/rust_sme/src/lib.rs:1792-1831), re-formulated for int4
// group-128 weights and fp16 activations.
//
// Work decomposition: a CTA owns one 128-row unit block and a contiguous range
// of its k units; a cluster of S CTAs (S = 1, 2, 4 or 8) splits the k range of
// one unit block and sums its S partial tiles through distributed shared memory
// in rank order (deterministic, no global workspace).  S is chosen so that the
// grid covers two CTAs per SM.
//
// CTA = 9 warps:
//   warp 8     producer: one 8448-byte cp.async.bulk per unit into a ring of
//              RS slots (8, 6 or 4 by token tile) -- the first RS issued
//              before griddepcontrol.wait
//              (weights are never written by a kernel of the step) -- and the
//              unit's activation slice (MP tokens x 128 k fp16, two 64-column
//              TMA boxes with 128-byte swizzle, rows past M filled with zeros)
//              after it;
//   warps 0-7  warp w owns weight rows 16w .. 16w+15 of every unit: it
//              dequantises them straight from the unit's words into the
//              registers of m16n8k16 A fragments (a nibble pair of a word is
//              exactly one fragment register; k is permuted within each k16
//              step so that a lane's four k are contiguous: one word per row
//              and one 8-byte activation load per fragment) and multiplies
//              them with the activation fragments read from the swizzled
//              slice, fp32 accumulators in registers (MP / 8 tiles of 8 tokens).
// Epilogue: accumulators to shared memory as [token][128 rows]; CTA rank r of
// the cluster sums token rows [r * MP / S, (r + 1) * MP / S) over the S
// partial tiles and writes them (store, or add for mode 1).
// Every mbarrier wait is bounded: a CTA whose wait gives up records
// SPECDEC_ETIMEOUT in the device status word, skips its output and still meets
// the cluster barriers.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace specdec {

constexpr int kGvUnitBytes = 8448;
constexpr int kGvMathWarps = 8;
constexpr int kGvThreads = 32 * (kGvMathWarps + 1);
constexpr int kGvMaxSplit = 8;

// Unit slots in flight per CTA: as many as ~100 KB of shared memory holds
// (two CTAs per SM), so that an SM keeps ~200 KB of weights in flight.
template <int MP>
struct GvSmem {
    static constexpr int kXBox = 64 * 2 * MP;       // one 64-column box: MP rows of 128 bytes
    static constexpr int kXSlot = 2 * kXBox;        // a unit's 128 columns
    static constexpr int kRing = MP <= 16 ? 8 : (MP <= 32 ? 6 : 4);
    static constexpr int kX = 0;                    // X ring first: 1024-byte aligned boxes
    static constexpr int kW = kX + kRing * kXSlot;
    static constexpr int kBars = kW + kRing * kGvUnitBytes;
    static constexpr int kBytes = kBars + 2 * kRing * 8 + 16;
    static constexpr int kLaunch = 1024 + kBytes;   // + alignment slack
    // the epilogue's fp32 [MP][128] tile reuses the rings
    static_assert(MP * 128 * 4 <= kBars, "partial tile must fit in the rings");
    static_assert(kBytes + 1024 <= 113 * 1024, "two CTAs per SM");
};

struct GemvArgs {
    const uint8_t* w;
    int M, N, KG, S;
    float* Y;
    int ldy, mode;
    int pdl;
    DeviceStatus* status;
};

__device__ __forceinline__ void mma_f16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// the nibble pair in bits 0-3 / 16-19 of a (shifted) unit word -> fp16x2
// fp16((u - 8) * s): fp16 1024 + u in each half, exact u - 8, one rounding of
// the product
__device__ __forceinline__ uint32_t deq_pair(uint32_t w, __half2 s2) {
    const uint32_t t = (w & 0x000F000Fu) | 0x64006400u;
    __half2 h = *reinterpret_cast<const __half2*>(&t);
    h = __hmul2(__hsub2(h, __float2half2_rn(1032.0f)), s2);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int NT>  // tiles of 8 tokens: MP = 8 * NT >= M
__global__ void __launch_bounds__(kGvThreads, 2)
    w4a16_gemv_kernel(const __grid_constant__ CUtensorMap tmap_x, GemvArgs args) {
    constexpr int MP = 8 * NT;
    using L = GvSmem<MP>;
    constexpr int kGvRing = L::kRing;
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    unsigned char* sX = base + L::kX;
    unsigned char* sW = base + L::kW;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L::kBars);
    uint64_t* empty = full + kGvRing;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kGvRing);

    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31;
    const int S = args.S;
    const int blk = blockIdx.x / S;
    const int rank = S > 1 ? (int)cluster_rank() : 0;
    const int k0 = (int)(((long long)rank * args.KG) / S);
    const int k1 = (int)(((long long)(rank + 1) * args.KG) / S);
    const int n_items = k1 - k0;  // >= 1 (S <= KG)

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGvRing; ++i) {
            mbar_init(s_addr(&full[i]), 1);
            mbar_init(s_addr(&empty[i]), kGvMathWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    __syncthreads();
    pdl_trigger();  // the next kernel may start its prologue

    if (warp == kGvMathWarps) {
        // ------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t tx = (uint32_t)(kGvUnitBytes + L::kXSlot);
            auto issue_w = [&](int it) {
                const int s = it % kGvRing;
                mbar_expect_tx(s_addr(&full[s]), tx);  // the unit and its activation slice
                bulk_g2s(s_addr(sW + s * kGvUnitBytes),
                         args.w + ((size_t)blk * args.KG + (k0 + it)) * kGvUnitBytes, kGvUnitBytes,
                         s_addr(&full[s]));
            };
            auto issue_x = [&](int it) {
                const int s = it % kGvRing;
#pragma unroll
                for (int p = 0; p < 2; ++p)
                    tma_load_2d(s_addr(sX + s * L::kXSlot + p * L::kXBox), &tmap_x, (k0 + it) * 128 + p * 64, 0,
                                s_addr(&full[s]));
            };
            const int first = n_items < kGvRing ? n_items : kGvRing;
            for (int it = 0; it < first; ++it) issue_w(it);
            if (args.pdl) pdl_wait();  // X is written by the kernel before this one
            for (int it = 0; it < first; ++it) issue_x(it);
            bool ok = true;
            int it = first;
            for (; it < n_items; ++it) {
                ok = mbar_wait(s_addr(&empty[it % kGvRing]), ((it / kGvRing) - 1) & 1);
                if (!ok || *abort_flag) break;
                issue_w(it);
                issue_x(it);
            }
            if (!ok) {
                *abort_flag = 1;
                record_timeout(args.status, 11);
            }
            // drain: every copy issued has landed before the CTA reuses or frees shared memory
            if (it > 0) (void)mbar_wait(s_addr(&full[(it - 1) % kGvRing]), ((it - 1) / kGvRing) & 1);
        }
        __syncwarp();
    }

    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
    const int g = lane >> 2, c = lane & 3;
    const int r = warp * 16 + g;  // this lane's rows r and r + 8 of the unit
    const int cw = c >> 1;                  // the word of a k16 step this lane reads
    const uint32_t sh = 8u * (uint32_t)(c & 1);  // its nibble pairs 2(c&1), 2(c&1)+1
    if (warp < kGvMathWarps) {
        // ------------------------------------------------ dequant + MMA
        bool ok = true;
        for (int it = 0; it < n_items; ++it) {
            const int s = it % kGvRing;
            ok = __all_sync(0xffffffffu, mbar_wait(s_addr(&full[s]), (it / kGvRing) & 1) && !*abort_flag);
            if (!ok) break;
            const unsigned char* unit = sW + s * kGvUnitBytes;
            const uint32_t* words = reinterpret_cast<const uint32_t*>(unit);
            const __half2 s_lo = __half2half2(*reinterpret_cast<const __half*>(unit + 8192 + r * 2));
            const __half2 s_hi = __half2half2(*reinterpret_cast<const __half*>(unit + 8192 + (r + 8) * 2));
            const unsigned char* xs = sX + s * L::kXSlot;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                // k16 step ks = words 2ks, 2ks + 1.  The contraction does not
                // depend on the order of k, so lane (g, c) takes physical k
                // 4c .. 4c + 3 of the step for its fragment slots (2c, 2c+1)
                // and (2c+8, 2c+9): nibble pairs 2(c&1), 2(c&1)+1 of word
                // 2ks + c/2 -- one word per row -- and 8 contiguous bytes of X.
                const uint32_t w0 = words[(2 * ks + cw) * 128 + r] >> sh;
                const uint32_t w1 = words[(2 * ks + cw) * 128 + r + 8] >> sh;
                uint32_t a[4];
                a[0] = deq_pair(w0, s_lo);
                a[1] = deq_pair(w1, s_hi);
                a[2] = deq_pair(w0 >> 4, s_lo);
                a[3] = deq_pair(w1 >> 4, s_hi);
                const unsigned char* box = xs + (ks >> 2) * L::kXBox;
                const int chunk = 2 * (ks & 3) + cw;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const int n = 8 * t + g;  // token row of the box
                    const uint2 b = *reinterpret_cast<const uint2*>(box + n * 128 + (((chunk ^ (n & 7)) << 4) + 8 * (c & 1)));
                    mma_f16_16816(acc[t], a, b.x, b.y);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(s_addr(&empty[s]));
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            record_timeout(args.status, 12);
        }
    }

    // ---------------------------------------------------- epilogue
    // all copies have landed and every slot is consumed: the rings become the
    // fp32 partial tile [MP tokens][128 rows]
    __syncthreads();
    float* part = reinterpret_cast<float*>(base);
    if (warp < kGvMathWarps) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int m = 8 * t + 2 * c;
            part[m * 128 + r] = acc[t][0];
            part[(m + 1) * 128 + r] = acc[t][1];
            part[m * 128 + r + 8] = acc[t][2];
            part[(m + 1) * 128 + r + 8] = acc[t][3];
        }
    }
    __syncthreads();
    if (S > 1) cluster_sync_all();  // every CTA's partial tile is in place
    const int rows = MP / S, m0 = rank * rows;  // S divides MP
    if (args.pdl) pdl_wait();  // Y may still be read or written by earlier kernels
    if (!*abort_flag) {
        for (int idx = threadIdx.x; idx < rows * 32; idx += blockDim.x) {
            const int m = m0 + (idx >> 5), col = (idx & 31) * 4;
            const int n = blk * 128 + col;
            const uint32_t la = s_addr(part + m * 128 + col);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (S > 1) {
                float4 pv[kGvMaxSplit];
#pragma unroll
                for (int q = 0; q < kGvMaxSplit; ++q)
                    if (q < S) pv[q] = ld_dsmem_f4(la, (uint32_t)q);
#pragma unroll
                for (int q = 0; q < kGvMaxSplit; ++q)
                    if (q < S) {
                        v.x += pv[q].x;
                        v.y += pv[q].y;
                        v.z += pv[q].z;
                        v.w += pv[q].w;
                    }
            } else {
                v = *reinterpret_cast<const float4*>(part + m * 128 + col);
            }
            if (m >= args.M) continue;
            float* y = args.Y + (size_t)m * args.ldy + n;
            const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (n + j < args.N) y[j] = args.mode ? y[j] + vv[j] : vv[j];
        }
    }
    if (S > 1) cluster_sync_all();  // peers have finished reading this CTA's partial tile
}

// ------------------------------------------------------------ host side
static int gemv_num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// The planner's crossover between this kernel and the tcgen05 tiles, from
// graph-replay timings on a B200 (K = 4096): at N = 4096 this kernel takes
// 8.3 / 10.1 / 12.8 / 19.6 us at M = 8 / 16 / 32 / 64 against 10.2 / 10.4 /
// 10.9 / 11.6 for the tiles; at N = 128256, 93.6 / 114 / 172 / 306 against
// 139 / 140 / 142 / 146.  Above 16 rows the tiles win.
constexpr int kGemvRouteRows = 16;
bool plan_gemm_uses_gemv(int M, int N, int K) {
    (void)N;
    (void)K;
    return M >= 1 && M <= kGemvRouteRows;
}

int gemv_tiles(int M) { return M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8)); }

GemvPlan plan_gemv(int M, int N, int K) {
    GemvPlan p;
    p.NT = gemv_tiles(M);
    p.KG = (K + 127) / 128;
    p.blocks = (N + 127) / 128;
    // the smallest split that gives two CTAs per SM, within KG and the cluster limit
    const int want = 2 * gemv_num_sms();
    p.S = 1;
    while (p.S < kGvMaxSplit && p.S * 2 <= p.KG && p.blocks * p.S < want) p.S *= 2;
    p.grid = p.blocks * p.S;
    return p;
}

template <int NT>
static int launch_gemv_nt(const CUtensorMap& map, const GemvArgs& a, int grid, cudaStream_t s) {
    constexpr size_t smem = GvSmem<8 * NT>::kLaunch;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(w4a16_gemv_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess) {
            cudaGetLastError();
            set_error("w4a16_gemv: cannot opt in to the shared memory the kernel needs");
            return SPECDEC_ECUDA;
        }
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = (unsigned)a.S;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = a.pdl ? 2 : 1;
    SD_CUDA(cudaLaunchKernelEx(&cfg, w4a16_gemv_kernel<NT>, map, a));
    return SPECDEC_OK;
}

int gemv_launch(const __half* X, int ldx, int K, const GemvPlan& p, const void* w_tiled, int M, int N, float* Y,
                int ldy, int mode, cudaStream_t s, bool pdl) {
    SD_CHECK(M >= 1 && M <= kGemvMaxRows && (mode == 0 || mode == 1) && p.KG == (K + 127) / 128, SPECDEC_EINVAL,
             "w4a16_gemv: 1 <= M <= 64 rows, mode 0 or 1");
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, ldx, 8 * p.NT);
    if (rc) return rc;
    GemvArgs a;
    a.w = reinterpret_cast<const uint8_t*>(w_tiled);
    a.M = M;
    a.N = N;
    a.KG = p.KG;
    a.S = p.S;
    a.Y = Y;
    a.ldy = ldy;
    a.mode = mode;
    a.pdl = pdl ? 1 : 0;
    a.status = device_status_ptr();
    switch (p.NT) {
        case 1: return launch_gemv_nt<1>(map, a, p.grid, s);
        case 2: return launch_gemv_nt<2>(map, a, p.grid, s);
        case 4: return launch_gemv_nt<4>(map, a, p.grid, s);
        case 8: return launch_gemv_nt<8>(map, a, p.grid, s);
        default: break;
    }
    set_error("w4a16_gemv: unsupported token tile");
    return SPECDEC_EINVAL;
}

}  // namespace specdec

using namespace specdec;

extern "C" int specdec_w4a16_gemv(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K, float* Y,
                                  int ldy, int mode, void* stream) {
    SD_CHECK(X && w_tiled && Y && M >= 0 && M <= kGemvMaxRows && N > 0 && K > 0 && ldx >= K && ldy >= N &&
                 (mode == 0 || mode == 1),
             SPECDEC_EINVAL, "w4a16_gemv: bad argument (0 <= M <= 64, mode 0 or 1)");
    if (M == 0) return SPECDEC_OK;
    const GemvPlan p = plan_gemv(M, N, K);
    return gemv_launch(reinterpret_cast<const __half*>(X), ldx, K, p, w_tiled, M, N, Y, ldy, mode, as_stream(stream),
                       false);
}
