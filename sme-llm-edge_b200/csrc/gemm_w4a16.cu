// gemm_w4a16.cu -- W4A16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Y[m, n] (op)= sum_k X[m, k] * deq(W)[n, k]
//   X  fp16 activations [M, K] (row stride ldx), loaded by TMA (128B swizzle)
//   W  int4 weights, group-128 fp16 scales, pre-tiled: unit (n128, k128) =
//      8192 bytes of nibbles (word [kc][row] holds k = kc*8 .. kc*8+7 of one
//      row, nibble j = k_2j, nibble j+4 = k_2j+1) followed by 128 fp16 scales.
//      Units are stored [n128][k128] so one unit is one 8448-byte bulk copy.
//   deq(w) = fp16((u4 - 8) * scale)   (offset-binary nibbles as written by the
//            reference packer, server/sve_packing.cpp:8-30)
//
// CTA = 15 warps, warp-specialised:
//   warp 0      bulk-copy producer of the int4 units (runs 4 k-steps ahead)
//   warp 14     TMA producer of the activation tiles
//   warp 1      TMEM allocator and the single-thread tcgen05.mma issuer
//   warps 2-5   epilogue: tcgen05.ld of the accumulators, fp32 store / add
//   warps 6-13  dequant: int4 -> fp16 in registers, stored in the K-major
//               128B-swizzled UMMA layout
// MMA: M = 128 weight rows (two per CTA tile of 256), N = token tile MT,
// K = 16 per instruction, accumulators fp32 in TMEM (2 x MT columns).
// Work is split "stream-K" style over (tile, k128) items so every SM gets the
// same number of k-steps; tiles shared by two CTAs are combined with fp32
// atomics.  Every mbarrier wait is bounded: on timeout the CTA records
// SPECDEC_ETIMEOUT in the device status word and unwinds.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace specdec {

constexpr int kUnitBytes = 8448;   // 8192 nibble bytes + 128 fp16 scales
constexpr int kRawStageBytes = 2 * kUnitBytes;
constexpr int kGemmThreads = 480;
constexpr int kASlotBytes = 32768;  // 256 rows x 64 k fp16
constexpr int kSmemBudget = 227 * 1024;

// int4 prefetch depth (k128 items): deeper for small token tiles, whose
// A/B slots are cheap and whose step is bound by the weight stream.
__host__ __device__ constexpr int raw_stages_for(int MT) { return MT <= 64 ? 6 : 4; }
__host__ __device__ constexpr int ab_stages_for(int MT) {
    return (kSmemBudget - raw_stages_for(MT) * kRawStageBytes - 2048 - 1024) / (kASlotBytes + MT * 128) > 4
               ? 4
               : (kSmemBudget - raw_stages_for(MT) * kRawStageBytes - 2048 - 1024) / (kASlotBytes + MT * 128);
}
__host__ __device__ constexpr int tmem_cols_for(int MT) {
    return 2 * MT <= 32 ? 32 : (2 * MT <= 64 ? 64 : (2 * MT <= 128 ? 128 : (2 * MT <= 256 ? 256 : 512)));
}
template <int MT>
__host__ __device__ constexpr size_t gemm_smem_bytes() {
    return 1024 /*align slack*/ + (size_t)ab_stages_for(MT) * (kASlotBytes + MT * 128) +
           (size_t)raw_stages_for(MT) * kRawStageBytes + 2048;
}

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t s_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait that lets the thread sleep (up to hint_ns) until the phase completes,
// so waiting warps do not take issue slots from the working ones.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t a, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: ~2 s of wall time at most.  The first probe is a plain
// try_wait; after that the thread sleeps in the barrier between probes.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity) {
    if (mbar_try(a, parity)) return true;
    const uint64_t t0 = gtimer();
    for (;;) {
        if (mbar_try_sleep(a, parity, 20000u)) return true;
        if (gtimer() - t0 > 2000000000ull) return false;
    }
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(mbar)
                 : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
        : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_ld_x16(uint32_t taddr, uint32_t v[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// K-major, 128-byte swizzled shared-memory matrix descriptor: rows of 128 B,
// 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;               // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset between 8-row groups
    d |= (uint64_t)1 << 46;               // descriptor version for sm_100
    d |= (uint64_t)2 << 61;               // SWIZZLE_128B
    return d;
}
// kind::f16 instruction descriptor: D fp32, A = B = fp16, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct GemmArgs {
    const uint8_t* w;
    int M, N, KG, m_tiles, n_tiles, total;
    float* Y;
    int ldy, mode;
    float* part;   // [grid][2 slots][2 halves][MT][128] partial tiles
    int* tickets;  // [m_tiles * n_tiles], zero between launches
    DeviceStatus* status;
};

// CTA whose stream-K item range [c*total/grid, (c+1)*total/grid) holds item i.
__device__ __forceinline__ int item_owner(long long i, int total, int grid) {
    int c = (int)((i * grid) / total);
    while (c + 1 < grid && ((long long)(c + 1) * total) / grid <= i) ++c;
    while (c > 0 && ((long long)c * total) / grid > i) --c;
    return c;
}

__device__ __forceinline__ void record_timeout(DeviceStatus* st, int where) {
    if (st) {
        atomicExch(&st->code, SPECDEC_ETIMEOUT);
        atomicExch(&st->where, where);
    }
}

template <int MT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, GemmArgs args) {
    constexpr int AB = ab_stages_for(MT);
    constexpr int RS = raw_stages_for(MT);
    constexpr int BSLOT = MT * 128;
    constexpr int TMEM_COLS = tmem_cols_for(MT);
    constexpr uint32_t IDESC = idesc_f16(128, MT);

    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    unsigned char* sA = base;                                   // AB x 32 KB
    unsigned char* sB = sA + AB * kASlotBytes;                  // AB x MT*128
    unsigned char* sRaw = sB + AB * BSLOT;                      // 4 x 16896
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRaw + RS * kRawStageBytes);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = bars + RS;
    uint64_t* a_full = bars + 2 * RS;
    uint64_t* b_full = a_full + AB;
    uint64_t* ab_empty = b_full + AB;
    uint64_t* acc_full = ab_empty + AB;
    uint64_t* acc_empty = acc_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g0 = (int)(((long long)blockIdx.x * args.total) / gridDim.x);
    const int g1 = (int)(((long long)(blockIdx.x + 1) * args.total) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int i = 0; i < RS; ++i) {
            mbar_init(s_addr(&raw_full[i]), 1);
            mbar_init(s_addr(&raw_empty[i]), 8);
        }
        for (int i = 0; i < AB; ++i) {
            mbar_init(s_addr(&a_full[i]), 8);
            mbar_init(s_addr(&b_full[i]), 1);
            mbar_init(s_addr(&ab_empty[i]), 1);
        }
        mbar_init(s_addr(acc_full), 1);
        mbar_init(s_addr(acc_empty), 4);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_addr(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int KG = args.KG;

    if (warp == 0) {
        // ------------------------------------------------ producer
        if (lane == 0 && g0 < g1) {
            int r_it = 0, ab_it = 0;
            // int4 units only: runs up to RS items ahead of the dequant warps
            bool ok = true;
            for (int g = g0; g < g1 && ok; ++g) {
                const int tile = g / KG, kg = g % KG;
                const int n_tile = tile / args.m_tiles;
                const int rs = r_it % RS;
                if (r_it >= RS) ok = mbar_wait(s_addr(&raw_empty[rs]), ((r_it / RS) - 1) & 1);
                if (!ok || *abort_flag) break;
                const uint32_t rf = s_addr(&raw_full[rs]);
                mbar_expect_tx(rf, kRawStageBytes);
                for (int u = 0; u < 2; ++u) {
                    const uint8_t* src = args.w + ((size_t)(n_tile * 2 + u) * KG + kg) * kUnitBytes;
                    bulk_g2s(s_addr(sRaw + rs * kRawStageBytes + u * kUnitBytes), src, kUnitBytes, rf);
                }
                ++r_it;
            }
            if (!ok) {
                *abort_flag = 1;
                record_timeout(args.status, 1);
            }
            // drain: every copy issued above completes on its barrier before the CTA exits
            if (r_it > 0) (void)mbar_wait(s_addr(&raw_full[(r_it - 1) % RS]), ((r_it - 1) / RS) & 1);
        }
    } else if (warp == 14) {
        // ------------------------------------------------ activation (B operand) producer
        if (lane == 0 && g0 < g1) {
            int ab_it = 0;
            bool ok = true;
            for (int g = g0; g < g1 && ok; ++g) {
                const int tile = g / KG, kg = g % KG;
                const int m_tile = tile % args.m_tiles;
                for (int hk = 0; hk < 2; ++hk) {
                    const int s = ab_it % AB;
                    if (ab_it >= AB) ok = mbar_wait(s_addr(&ab_empty[s]), ((ab_it / AB) - 1) & 1);
                    if (!ok || *abort_flag) {
                        ok = false;
                        break;
                    }
                    const uint32_t bf = s_addr(&b_full[s]);
                    mbar_expect_tx(bf, BSLOT);
                    tma_load_2d(s_addr(sB + s * BSLOT), &tmap_x, kg * 128 + hk * 64, m_tile * MT, bf);
                    ++ab_it;
                }
            }
            if (!ok) {
                *abort_flag = 1;
                record_timeout(args.status, 5);
            }
            if (ab_it > 0) (void)mbar_wait(s_addr(&b_full[(ab_it - 1) % AB]), ((ab_it - 1) / AB) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0 && g0 < g1) {
            int ab_it = 0, t_it = 0;
            bool ok = true;
            for (int g = g0; g < g1 && ok; ++g) {
                const int kg = g % KG;
                const bool first = (g == g0) || (kg == 0);
                const bool last = (g == g1 - 1) || (kg == KG - 1);
                if (first) {
                    ok = mbar_wait(s_addr(acc_empty), (t_it & 1) ^ 1);
                    if (!ok) break;
                    tc_fence_after();
                }
                for (int hk = 0; hk < 2 && ok; ++hk) {
                    const int s = ab_it % AB;
                    const uint32_t par = (ab_it / AB) & 1;
                    ok = mbar_wait(s_addr(&a_full[s]), par) && mbar_wait(s_addr(&b_full[s]), par);
                    if (!ok || *abort_flag) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = s_addr(sA + s * kASlotBytes);
                    const uint32_t b0 = s_addr(sB + s * BSLOT);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t bd = sw128_desc(b0 + ks * 32);
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const uint64_t ad = sw128_desc(a0 + q * 16384 + ks * 32);
                            const uint32_t acc = (first && hk == 0 && ks == 0) ? 0u : 1u;
                            tc_mma_f16(tmem + (uint32_t)(q * MT), ad, bd, IDESC, acc);
                        }
                    }
                    tc_commit(s_addr(&ab_empty[s]));
                    ++ab_it;
                }
                if (ok && last) {
                    tc_commit(s_addr(acc_full));
                    ++t_it;
                }
            }
            if (!ok) {
                *abort_flag = 1;
                record_timeout(args.status, 2);
            }
        }
    } else if (warp < 6) {
        // ------------------------------------------------ epilogue
        // A tile whose k-range is split over several CTAs (at stream-K range
        // boundaries) is finished by the last of them to arrive (atomic
        // ticket, no waiting): the others park their partial sums in the
        // workspace, the last one adds all parts in CTA order and writes Y.
        const int quad = warp & 3;
        const int et = threadIdx.x - 64;  // 0..127
        int* s_ticket = reinterpret_cast<int*>(tmem_slot + 2);
        const size_t slot_floats = (size_t)2 * MT * 128;
        int t_it = 0;
        for (int g = g0; g < g1; ++g) {
            const int kg = g % KG;
            const bool last = (g == g1 - 1) || (kg == KG - 1);
            if (!last) continue;
            const int tile = g / KG;
            const int n_tile = tile / args.m_tiles, m_tile = tile % args.m_tiles;
            const int c_lo = item_owner((long long)tile * KG, args.total, gridDim.x);
            const int c_hi = item_owner((long long)tile * KG + KG - 1, args.total, gridDim.x);
            const int my_slot = (g0 / KG == tile) ? 0 : 1;
            if (!mbar_wait(s_addr(acc_full), t_it & 1) || *abort_flag) {
                *abort_flag = 1;
                record_timeout(args.status, 3);
                break;
            }
            tc_fence_after();
            bool finisher = true;
            if (c_hi > c_lo) {
                // park this CTA's part, then take a ticket
                float* mine = args.part + ((size_t)blockIdx.x * 2 + my_slot) * slot_floats;
#pragma unroll 1
                for (int q = 0; q < 2; ++q)
#pragma unroll 1
                    for (int c = 0; c < MT / 16; ++c) {
                        uint32_t v[16];
                        tc_ld_x16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(q * MT + c * 16), v);
                        tc_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            __stcg(mine + ((size_t)q * MT + c * 16 + j) * 128 + quad * 32 + lane, __uint_as_float(v[j]));
                    }
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (et == 0) *s_ticket = atomicAdd(&args.tickets[tile], 1);
                asm volatile("bar.sync 1, 128;" ::: "memory");
                finisher = (*s_ticket == c_hi - c_lo);
                if (finisher) __threadfence();
            }
            if (finisher) {
#pragma unroll 1
                for (int q = 0; q < 2; ++q) {
                    const int n = n_tile * 256 + q * 128 + quad * 32 + lane;
#pragma unroll 1
                    for (int c = 0; c < MT / 16; ++c) {
                        uint32_t v[16];
                        tc_ld_x16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(q * MT + c * 16), v);
                        tc_wait_ld();
                        float acc[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) acc[j] = 0.f;
                        // parts in CTA order (deterministic sum); the first part of
                        // CTA p is its slot 0, a later tile of p its slot 1
                        const size_t off = ((size_t)q * MT + c * 16) * 128 + quad * 32 + lane;
                        for (int p = c_lo; p <= c_hi; ++p) {
                            if (p == (int)blockIdx.x) {
#pragma unroll
                                for (int j = 0; j < 16; ++j) acc[j] += __uint_as_float(v[j]);
                            } else {
                                const int ps = ((((long long)p * args.total) / gridDim.x) / KG == tile) ? 0 : 1;
                                const float* src = args.part + ((size_t)p * 2 + ps) * slot_floats + off;
#pragma unroll
                                for (int j = 0; j < 16; ++j) acc[j] += __ldcg(src + (size_t)j * 128);
                            }
                        }
                        if (n < args.N) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const int m = m_tile * MT + c * 16 + j;
                                if (m < args.M) {
                                    float* y = args.Y + (size_t)m * args.ldy + n;
                                    if (args.mode) *y += acc[j];
                                    else *y = acc[j];
                                }
                            }
                        }
                    }
                }
                if (c_hi > c_lo && et == 0) args.tickets[tile] = 0;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_addr(acc_empty));
            ++t_it;
        }
    } else {
        // ------------------------------------------------ dequant
        const int dt = threadIdx.x - 192;  // 0..255
        int r_it = 0, ab_it = 0;
        bool ok = true;
        for (int g = g0; g < g1 && ok; ++g) {
            const int rs = r_it % RS;
            ok = mbar_wait(s_addr(&raw_full[rs]), (r_it / RS) & 1);
            if (!ok || *abort_flag) {
                ok = false;
                break;
            }
            const unsigned char* raw = sRaw + rs * kRawStageBytes;
            // this thread's row r and its two units' group scales are fixed for the item
            const int r = dt & 127;
            const __half2 s2u0 = __half2half2(*reinterpret_cast<const __half*>(raw + 8192 + r * 2));
            const __half2 s2u1 = __half2half2(*reinterpret_cast<const __half*>(raw + kUnitBytes + 8192 + r * 2));
            const __half2 bias = __float2half2_rn(1032.0f);
            for (int hk = 0; hk < 2; ++hk) {
                const int s = ab_it % AB;
                if (ab_it >= AB) ok = mbar_wait(s_addr(&ab_empty[s]), ((ab_it / AB) - 1) & 1);
                if (!ok || *abort_flag) {
                    ok = false;
                    break;
                }
                unsigned char* a_slot = sA + s * kASlotBytes;
                uint32_t wv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {  // all loads first: 8 independent shared loads in flight
                    const int u = i >> 2, kcl = 2 * (i & 3) + (dt >> 7);
                    wv[i] = *reinterpret_cast<const uint32_t*>(raw + u * kUnitBytes + (((hk * 8 + kcl) * 128 + r) << 2));
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int u = i >> 2, kcl = 2 * (i & 3) + (dt >> 7);
                    const __half2 s2 = u ? s2u1 : s2u0;
                    uint32_t outw[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t t = ((wv[i] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
                        __half2 hv = *reinterpret_cast<const __half2*>(&t);
                        hv = __hmul2(__hsub2(hv, bias), s2);  // exact (u - 8), then one rounding of (u - 8) * s
                        outw[j] = *reinterpret_cast<uint32_t*>(&hv);
                    }
                    unsigned char* dst = a_slot + u * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + ((kcl ^ (r & 7)) << 4);
                    *reinterpret_cast<uint4*>(dst) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_addr(&a_full[s]));
                ++ab_it;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(s_addr(&raw_empty[rs]));
            ++r_it;
        }
        if (!ok) {
            *abort_flag = 1;
            record_timeout(args.status, 4);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// CUDA-core reference contraction on the same tiled weights (cross-check path).
__global__ void w4a16_simt_kernel(const __half* __restrict__ X, int M, int ldx, const uint8_t* __restrict__ w,
                                  int N, int K, int KG, float* __restrict__ Y, int ldy, int mode) {
    const int r = threadIdx.x;  // 128 rows of one unit row-block
    const int n = blockIdx.x * 128 + r;
    const int m = blockIdx.y;
    if (m >= M) return;
    float acc = 0.f;
    for (int kg = 0; kg < KG; ++kg) {
        const uint8_t* unit = w + ((size_t)blockIdx.x * KG + kg) * kUnitBytes;
        const float s = __half2float(*reinterpret_cast<const __half*>(unit + 8192 + r * 2));
        for (int kc = 0; kc < 16; ++kc) {
            const uint32_t wd = *reinterpret_cast<const uint32_t*>(unit + ((kc * 128 + r) << 2));
            const int k0 = kg * 128 + kc * 8;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int k = k0 + 2 * j + e;
                    const int u = (wd >> (4 * j + 16 * e)) & 15;
                    const float wv = __half2float(__float2half_rn((float)(u - 8) * s));
                    if (k < K) acc += __half2float(X[(size_t)m * ldx + k]) * wv;
                }
            }
        }
    }
    if (n < N) {
        float* y = Y + (size_t)m * ldy + n;
        if (mode) *y += acc;
        else *y = acc;
    }
}

// Reference packed int4 [N, K/2] + scales [N, ceil(K/128)] -> tiled units.
__global__ void w4_tile_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales, int N, int K,
                               int KG, int units_n, uint8_t* __restrict__ tiled) {
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t total = (size_t)units_n * KG * 16 * 128;
    if (tid >= total) return;
    const int r = tid % 128;
    const int kc = (tid / 128) % 16;
    const int kg = (tid / 2048) % KG;
    const int un = (int)(tid / ((size_t)2048 * KG));
    const int n = un * 128 + r;
    const int G = (K + 127) / 128;
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int k = kg * 128 + kc * 8 + i;
        uint32_t u = 8;
        if (n < N && k < K) {
            const uint8_t byte = packed[(size_t)n * (K / 2) + k / 2];
            u = (k & 1) ? (byte >> 4) : (byte & 15);
        }
        const int j = i >> 1;
        word |= u << ((i & 1) ? (4 * j + 16) : (4 * j));
    }
    uint8_t* unit = tiled + ((size_t)un * KG + kg) * kUnitBytes;
    *reinterpret_cast<uint32_t*>(unit + ((kc * 128 + r) << 2)) = word;
    if (kc == 0) {
        const uint16_t s = (n < N && kg < G) ? scales[(size_t)n * G + kg] : (uint16_t)0;
        *reinterpret_cast<uint16_t*>(unit + 8192 + r * 2) = s;
    }
}

__global__ void w4_untile_kernel(const uint8_t* __restrict__ tiled, int N, int K, int KG, uint8_t* __restrict__ packed,
                                 uint16_t* __restrict__ scales) {
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // one byte of packed
    const size_t total = (size_t)N * (K / 2);
    const int G = (K + 127) / 128;
    if (tid < (size_t)N * G) {
        const int n = tid / G, g = tid % G;
        const uint8_t* unit = tiled + ((size_t)(n / 128) * KG + g) * kUnitBytes;
        scales[tid] = *reinterpret_cast<const uint16_t*>(unit + 8192 + (n % 128) * 2);
    }
    if (tid >= total) return;
    const int n = tid / (K / 2), kb = (int)(tid % (K / 2));
    uint8_t out = 0;
    for (int e = 0; e < 2; ++e) {
        const int k = kb * 2 + e;
        const int kg = k / 128, kc = (k % 128) / 8, i = k % 8, j = i >> 1;
        const uint8_t* unit = tiled + ((size_t)(n / 128) * KG + kg) * kUnitBytes;
        const uint32_t w = *reinterpret_cast<const uint32_t*>(unit + ((kc * 128 + (n % 128)) << 2));
        const uint32_t u = (w >> ((i & 1) ? (4 * j + 16) : (4 * j))) & 15;
        out |= (uint8_t)(u << (4 * e));
    }
    packed[tid] = out;
}

// ------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

int make_x_tmap(CUtensorMap* map, const void* X, int M, int K, int ldx, int MT) {
    auto enc = get_encode();
    SD_CHECK(enc, SPECDEC_ENOTSUP, "cuTensorMapEncodeTiled unavailable");
    SD_CHECK((reinterpret_cast<uintptr_t>(X) & 15) == 0 && (ldx % 8) == 0, SPECDEC_EINVAL,
             "w4a16_gemm: X must be 16-byte aligned with a row stride that is a multiple of 8 elements");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)MT};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(X), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SD_CHECK(r == CUDA_SUCCESS, SPECDEC_EINVAL, "cuTensorMapEncodeTiled failed");
    return SPECDEC_OK;
}

int pick_mt(int M) {
    static const int opts[] = {16, 32, 64, 128, 160, 256};
    if (M <= 256) {
        for (int o : opts)
            if (o >= M) return o;
    }
    const int t160 = (M + 159) / 160 * 160, t256 = (M + 255) / 256 * 256;
    return t160 < t256 ? 160 : 256;
}

static int g_num_sms = 0;
static int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

template <int MT>
static int launch_tc(const CUtensorMap& map, const GemmArgs& a, int grid, cudaStream_t s) {
    constexpr size_t smem = gemm_smem_bytes<MT>();
    static bool attr = false;
    if (!attr) {
        SD_CUDA(cudaFuncSetAttribute(w4a16_tc_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr = true;
    }
    w4a16_tc_kernel<MT><<<grid, kGemmThreads, smem, s>>>(map, a);
    SD_LAUNCH_CHECK("w4a16_tc_kernel");
    return SPECDEC_OK;
}

struct GemmPlan {
    int MT, m_tiles, n_tiles, KG, total, grid;
    bool split;  // some tile is shared by several CTAs
};

GemmPlan plan_gemm(int M, int N, int K) {
    GemmPlan p;
    p.MT = pick_mt(M);
    p.m_tiles = (M + p.MT - 1) / p.MT;
    p.n_tiles = (N + 255) / 256;
    p.KG = (K + 127) / 128;
    p.total = p.m_tiles * p.n_tiles * p.KG;
    const int tiles = p.m_tiles * p.n_tiles;
    p.grid = num_sms();
    if (p.grid > p.total) p.grid = p.total;
    p.split = false;
    for (int c = 0; c < p.grid && !p.split; ++c) {
        const long long g0 = (long long)c * p.total / p.grid, g1 = (long long)(c + 1) * p.total / p.grid;
        if (g0 % p.KG || g1 % p.KG) p.split = true;
    }
    (void)tiles;
    return p;
}

// Workspace of one launch: per-tile tickets at a fixed offset (the front, so
// that launches with different token tiles sharing one workspace never
// overlap each other's tickets), then the parked partial tiles.  The tickets
// must be zero before the first launch; every launch leaves them zero.
constexpr size_t kTicketBytes = 1 << 18;  // 65536 tiles
size_t gemm_workspace_bytes(const GemmPlan& p) {
    return kTicketBytes + (size_t)p.grid * 2 * 2 * p.MT * 128 * sizeof(float);
}
size_t gemm_workspace_bound(int max_m, int max_n, int max_k) {
    (void)max_m;
    (void)max_n;
    (void)max_k;
    // the partial area depends only on the grid and the token tile (<= 256)
    return kTicketBytes + (size_t)num_sms() * 2 * 2 * 256 * 128 * sizeof(float);
}

// Launch with a prebuilt tensor map (built for this plan's MT).
int gemm_launch(const CUtensorMap& map, const GemmPlan& p, const void* w_tiled, int M, int N, float* Y, int ldy,
                int mode, void* ws, cudaStream_t s) {
    GemmArgs a;
    a.w = reinterpret_cast<const uint8_t*>(w_tiled);
    a.M = M;
    a.N = N;
    a.KG = p.KG;
    a.m_tiles = p.m_tiles;
    a.n_tiles = p.n_tiles;
    a.total = p.total;
    a.Y = Y;
    a.ldy = ldy;
    a.mode = mode;
    if ((size_t)p.m_tiles * p.n_tiles * sizeof(int) > kTicketBytes) {
        set_error("w4a16_gemm: too many output tiles for the ticket area");
        return SPECDEC_EINVAL;
    }
    a.tickets = reinterpret_cast<int*>(ws);
    a.part = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kTicketBytes);
    a.status = device_status_ptr();
    switch (p.MT) {
        case 16: return launch_tc<16>(map, a, p.grid, s);
        case 32: return launch_tc<32>(map, a, p.grid, s);
        case 64: return launch_tc<64>(map, a, p.grid, s);
        case 128: return launch_tc<128>(map, a, p.grid, s);
        case 160: return launch_tc<160>(map, a, p.grid, s);
        case 256: return launch_tc<256>(map, a, p.grid, s);
        default: break;
    }
    set_error("w4a16_gemm: unsupported token tile");
    return SPECDEC_EINVAL;
}

size_t w4_tiled_bytes(int N, int K) {
    const size_t units_n = (size_t)((N + 255) / 256) * 2;
    return units_n * ((K + 127) / 128) * kUnitBytes;
}

}  // namespace specdec

using namespace specdec;

extern "C" size_t specdec_w4_tiled_bytes(int N, int K) { return (N > 0 && K > 0) ? w4_tiled_bytes(N, K) : 0; }

extern "C" int specdec_w4_tile(const uint8_t* packed, const uint16_t* scales, int N, int K, void* tiled, void* stream) {
    SD_CHECK(packed && scales && tiled && N > 0 && K > 0 && (K % 2) == 0, SPECDEC_EINVAL, "w4_tile: bad argument");
    const int KG = (K + 127) / 128, units_n = ((N + 255) / 256) * 2;
    const size_t total = (size_t)units_n * KG * 2048;
    w4_tile_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(
        packed, scales, N, K, KG, units_n, reinterpret_cast<uint8_t*>(tiled));
    SD_LAUNCH_CHECK("w4_tile_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_w4_untile(const void* tiled, int N, int K, uint8_t* packed, uint16_t* scales, void* stream) {
    SD_CHECK(packed && scales && tiled && N > 0 && K > 0 && (K % 2) == 0, SPECDEC_EINVAL, "w4_untile: bad argument");
    const int KG = (K + 127) / 128;
    size_t total = (size_t)N * (K / 2);
    const size_t ns = (size_t)N * ((K + 127) / 128);
    if (ns > total) total = ns;
    w4_untile_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const uint8_t*>(tiled), N, K, KG, packed, scales);
    SD_LAUNCH_CHECK("w4_untile_kernel");
    return SPECDEC_OK;
}

extern "C" size_t specdec_w4a16_workspace_bytes(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return gemm_workspace_bytes(plan_gemm(M, N, K));
}

extern "C" int specdec_w4a16_gemm(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K, float* Y,
                                  int ldy, int mode, void* workspace, size_t workspace_bytes, void* stream) {
    SD_CHECK(X && w_tiled && Y && M >= 0 && N > 0 && K > 0 && ldx >= K && ldy >= N && (mode == 0 || mode == 1),
             SPECDEC_EINVAL, "w4a16_gemm: bad argument");
    if (M == 0) return SPECDEC_OK;
    cudaStream_t s = as_stream(stream);
    GemmPlan p = plan_gemm(M, N, K);
    const size_t need = gemm_workspace_bytes(p);
    SD_CHECK(workspace && workspace_bytes >= need, SPECDEC_EINVAL, "w4a16_gemm: workspace too small");
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, ldx, p.MT);
    if (rc) return rc;
    // tickets must start at zero; clear them (the kernel leaves them zero again)
    SD_CUDA(cudaMemsetAsync(workspace, 0, (size_t)p.m_tiles * p.n_tiles * sizeof(int), s));
    return gemm_launch(map, p, w_tiled, M, N, Y, ldy, mode, workspace, s);
}

extern "C" int specdec_w4a16_gemm_simt(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K, float* Y,
                                       int ldy, int mode, void* stream) {
    SD_CHECK(X && w_tiled && Y && M >= 0 && N > 0 && K > 0 && ldx >= K && ldy >= N, SPECDEC_EINVAL,
             "w4a16_gemm_simt: bad argument");
    if (M == 0) return SPECDEC_OK;
    const int KG = (K + 127) / 128;
    const int units = ((N + 255) / 256) * 2;
    dim3 grid(units, M);
    w4a16_simt_kernel<<<grid, 128, 0, as_stream(stream)>>>(reinterpret_cast<const __half*>(X), M, ldx,
                                                           reinterpret_cast<const uint8_t*>(w_tiled), N, K, KG, Y,
                                                           ldy, mode);
    SD_LAUNCH_CHECK("w4a16_simt_kernel");
    return SPECDEC_OK;
}
