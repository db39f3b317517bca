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
// Work decomposition: one output tile = 256 weight rows x MT tokens.  A
// cluster of S CTAs (1 <= S <= 8) owns one tile and splits its K range; the
// S partial accumulators are summed on chip through distributed shared memory
// (each CTA reduces 1/S of the tile's columns from all S CTAs in rank order,
// so the result is deterministic) and written once.  S is chosen per shape so
// the grid fills the 148 SMs with little wave quantisation.
//
// CTA = 15 warps, warp-specialised:
//   warp 0      bulk-copy producer of the int4 units (RS k-steps ahead)
//   warp 14     TMA producer of the activation tiles (BS half-steps ahead)
//   warp 1      TMEM allocator and the single-thread tcgen05.mma issuer
//   warps 2-5   epilogue: tcgen05.ld of the accumulators
//   warps 6-13  dequant: int4 -> fp16 in registers, written straight into
//               tensor memory with tcgen05.st (one TMEM lane = one weight row)
// MMA: M = 128 weight rows (two per tile), N = MT, K = 16 per instruction,
// A (the dequantised weights) read from TMEM, B (the activations) from shared
// memory, fp32 accumulators in TMEM.  Keeping A out of shared memory matters:
// with A staged there, the dequant stores plus the MMA's A reads doubled the
// shared-memory traffic of a k-step and made it, not the tensor pipe, the
// limit.  TMEM columns: [0, 2*MT) accumulators, then AS stages of 64 columns
// (two units x 64 k fp16, two fp16 per 32-bit column).
// Every mbarrier wait is bounded: on timeout the CTA records SPECDEC_ETIMEOUT
// in the device status word, skips its output and still meets its cluster
// barriers.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace specdec {

constexpr int kUnitBytes = 8448;  // 8192 nibble bytes + 128 fp16 scales
constexpr int kRawStageBytes = 2 * kUnitBytes;
constexpr int kGemmThreads = 480;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kMaxSplit = 8;
constexpr int kTmemCols = 512;
constexpr int kAStageCols = 64;  // one half k-step of A: 2 units x 64 k fp16
constexpr int kMaxTokenTile = 160;

// Ring depths per token tile.  A lives in the TMEM columns the accumulators
// leave free; raw int4 units and activation tiles share the shared memory.
__host__ __device__ constexpr int a_stages_for(int MT) {
    return (kTmemCols - 2 * MT) / kAStageCols > 4 ? 4 : (kTmemCols - 2 * MT) / kAStageCols;
}
__host__ __device__ constexpr int raw_stages_for(int MT) { return MT <= 32 ? 8 : (MT <= 64 ? 6 : 4); }
__host__ __device__ constexpr int b_stages_for(int MT) {
    return (kSmemBudget - 3072 - raw_stages_for(MT) * kRawStageBytes) / (MT * 128) > 8
               ? 8
               : (kSmemBudget - 3072 - raw_stages_for(MT) * kRawStageBytes) / (MT * 128);
}
template <int MT>
__host__ __device__ constexpr size_t gemm_smem_bytes() {
    return 1024 /*align slack*/ + (size_t)b_stages_for(MT) * MT * 128 + (size_t)raw_stages_for(MT) * kRawStageBytes +
           2048;
}
// the split-K reduction reuses the B and raw rings for one 128-row half (MT x 128 fp32)
template <int MT>
__host__ __device__ constexpr bool reduce_fits() {
    return (size_t)b_stages_for(MT) * MT * 128 + (size_t)raw_stages_for(MT) * kRawStageBytes >= (size_t)MT * 128 * 4;
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
// D (TMEM) (+)= A (TMEM, K-major, lane = row) x B (shared memory descriptor)
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 consecutive columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tc_st_x32(uint32_t taddr, const uint32_t v[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_ld_x16(uint32_t taddr, uint32_t v[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local_addr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}

// K-major, 128-byte swizzled shared-memory matrix descriptor: rows of 128 B,
// 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset between 8-row groups
    d |= (uint64_t)1 << 46;            // descriptor version for sm_100
    d |= (uint64_t)2 << 61;            // SWIZZLE_128B
    return d;
}
// kind::f16 instruction descriptor: D fp32, A = B = fp16, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct GemmArgs {
    const uint8_t* w;
    int M, N, KG, m_tiles, S;
    float* Y;
    int ldy, mode;
    DeviceStatus* status;
};

__device__ __forceinline__ void record_timeout(DeviceStatus* st, int where) {
    if (st) {
        atomicExch(&st->code, SPECDEC_ETIMEOUT);
        atomicExch(&st->where, where);
    }
}

template <int MT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, GemmArgs args) {
    constexpr int AS = a_stages_for(MT);
    constexpr int BS = b_stages_for(MT);
    constexpr int RS = raw_stages_for(MT);
    constexpr int BSLOT = MT * 128;
    constexpr uint32_t A_COL0 = 2 * MT;  // first TMEM column of the A stages
    constexpr uint32_t IDESC = idesc_f16(128, MT);
    static_assert(AS >= 2 && A_COL0 + AS * kAStageCols <= kTmemCols, "TMEM plan");

    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    unsigned char* sB = base;               // BS x MT*128 (1024-byte aligned slots)
    unsigned char* sRaw = sB + BS * BSLOT;  // RS x 16896
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRaw + RS * kRawStageBytes);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + RS;
    uint64_t* a_full = raw_empty + RS;
    uint64_t* a_empty = a_full + AS;
    uint64_t* b_full = a_empty + AS;
    uint64_t* b_empty = b_full + BS;
    uint64_t* acc_full = b_empty + BS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = args.S;
    const int tile = blockIdx.x / S;
    const int rank = S > 1 ? (int)cluster_rank() : 0;
    const int n_tile = tile / args.m_tiles, m_tile = tile % args.m_tiles;
    const int k0 = (int)(((long long)rank * args.KG) / S);
    const int k1 = (int)(((long long)(rank + 1) * args.KG) / S);
    const int n_items = k1 - k0;  // >= 1 (S <= KG)
    const int n_halves = 2 * n_items;

    if (threadIdx.x == 0) {
        for (int i = 0; i < RS; ++i) {
            mbar_init(s_addr(&raw_full[i]), 1);
            mbar_init(s_addr(&raw_empty[i]), 8);
        }
        for (int i = 0; i < AS; ++i) {
            mbar_init(s_addr(&a_full[i]), 8);
            mbar_init(s_addr(&a_empty[i]), 1);
        }
        for (int i = 0; i < BS; ++i) {
            mbar_init(s_addr(&b_full[i]), 1);
            mbar_init(s_addr(&b_empty[i]), 1);
        }
        mbar_init(s_addr(acc_full), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_addr(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ int4 unit producer
        if (lane == 0) {
            bool ok = true;
            int it = 0;
            for (; it < n_items; ++it) {
                const int rs = it % RS;
                if (it >= RS) ok = mbar_wait(s_addr(&raw_empty[rs]), ((it / RS) - 1) & 1);
                if (!ok || *abort_flag) break;
                const uint32_t rf = s_addr(&raw_full[rs]);
                mbar_expect_tx(rf, kRawStageBytes);
                for (int u = 0; u < 2; ++u) {
                    const uint8_t* src = args.w + ((size_t)(n_tile * 2 + u) * args.KG + (k0 + it)) * kUnitBytes;
                    bulk_g2s(s_addr(sRaw + rs * kRawStageBytes + u * kUnitBytes), src, kUnitBytes, rf);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                record_timeout(args.status, 1);
            }
            // drain: the copies issued above complete before the CTA exits
            if (it > 0) (void)mbar_wait(s_addr(&raw_full[(it - 1) % RS]), ((it - 1) / RS) & 1);
        }
    } else if (warp == 14) {
        // ------------------------------------------------ activation (B operand) producer
        if (lane == 0) {
            bool ok = true;
            int j = 0;
            for (; j < n_halves; ++j) {
                const int s = j % BS;
                if (j >= BS) ok = mbar_wait(s_addr(&b_empty[s]), ((j / BS) - 1) & 1);
                if (!ok || *abort_flag) break;
                const uint32_t bf = s_addr(&b_full[s]);
                mbar_expect_tx(bf, BSLOT);
                tma_load_2d(s_addr(sB + s * BSLOT), &tmap_x, (k0 + (j >> 1)) * 128 + (j & 1) * 64, m_tile * MT, bf);
            }
            if (!ok) {
                *abort_flag = 1;
                record_timeout(args.status, 5);
            }
            if (j > 0) (void)mbar_wait(s_addr(&b_full[(j - 1) % BS]), ((j - 1) / BS) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            bool ok = true;
            for (int j = 0; j < n_halves && ok; ++j) {
                const int sa = j % AS, sb = j % BS;
                ok = mbar_wait(s_addr(&a_full[sa]), (j / AS) & 1) && mbar_wait(s_addr(&b_full[sb]), (j / BS) & 1);
                if (!ok || *abort_flag) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = tmem + A_COL0 + (uint32_t)(sa * kAStageCols);
                const uint32_t b0 = s_addr(sB + sb * BSLOT);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t bd = sw128_desc(b0 + ks * 32);
#pragma unroll
                    for (int q = 0; q < 2; ++q)  // unit q: A columns q*32 + ks*8 .. +8 (k16 = 8 columns)
                        tc_mma_f16_ts(tmem + (uint32_t)(q * MT), a0 + (uint32_t)(q * 32 + ks * 8), bd, IDESC,
                                      (j > 0 || ks > 0) ? 1u : 0u);
                }
                tc_commit(s_addr(&a_empty[sa]));
                tc_commit(s_addr(&b_empty[sb]));
            }
            if (ok) tc_commit(s_addr(acc_full));
            else {
                *abort_flag = 1;
                record_timeout(args.status, 2);
            }
        }
    } else if (warp >= 6) {
        // ------------------------------------------------ dequant
        // A warp may only touch TMEM lanes 32*(warp%4) .. +31, so warps 6-9
        // cover the four lane quarters of unit 0 and warps 10-13 those of
        // unit 1.  Thread = one weight row r of its unit.
        const int q = (warp - 6) >> 2;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t t_row = tmem + ((uint32_t)(quarter * 32) << 16) + A_COL0 + (uint32_t)(q * 32);
        const __half2 bias = __float2half2_rn(1032.0f);
        bool ok = true;
        for (int it = 0; it < n_items && ok; ++it) {
            const int rs = it % RS;
            ok = mbar_wait(s_addr(&raw_full[rs]), (it / RS) & 1);
            // warp-uniform decision: the tcgen05.st below is a .sync.aligned warp instruction
            ok = __all_sync(0xffffffffu, ok && !*abort_flag);
            if (!ok) break;
            const unsigned char* unit = sRaw + rs * kRawStageBytes + q * kUnitBytes;
            const __half2 s2 = __half2half2(*reinterpret_cast<const __half*>(unit + 8192 + r * 2));
            for (int hk = 0; hk < 2; ++hk) {
                const int j = 2 * it + hk;
                const int s = j % AS;
                if (j >= AS) ok = mbar_wait(s_addr(&a_empty[s]), ((j / AS) - 1) & 1);
                ok = __all_sync(0xffffffffu, ok && !*abort_flag);
                if (!ok) break;
                uint32_t wv[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)  // word (kc, r): k = kc*8 .. kc*8+7 of row r; lanes read consecutive words
                    wv[i] = *reinterpret_cast<const uint32_t*>(unit + (((hk * 8 + i) * 128 + r) << 2));
                uint32_t outw[32];  // column i*4+jj = fp16 pair (k = 8i+2jj, 8i+2jj+1) of this half
#pragma unroll
                for (int i = 0; i < 8; ++i) {
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const uint32_t t = ((wv[i] >> (4 * jj)) & 0x000F000Fu) | 0x64006400u;
                        __half2 hv = *reinterpret_cast<const __half2*>(&t);
                        hv = __hmul2(__hsub2(hv, bias), s2);  // exact (u - 8), then one rounding of (u - 8) * s
                        outw[i * 4 + jj] = *reinterpret_cast<uint32_t*>(&hv);
                    }
                }
                tc_st_x32(t_row + (uint32_t)(s * kAStageCols), outw);
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_addr(&a_full[s]));
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(s_addr(&raw_empty[rs]));
        }
        if (!ok) {
            *abort_flag = 1;
            record_timeout(args.status, 4);
        }
    }

    // ---------------------------------------------------- epilogue (all threads)
    const bool epi_warp = warp >= 2 && warp < 6;
    const int quad = warp & 3;
    bool acc_ok = true;
    if (epi_warp) {
        acc_ok = mbar_wait(s_addr(acc_full), 0) && !*abort_flag;
        if (!acc_ok) {
            *abort_flag = 1;
            record_timeout(args.status, 3);
        }
        tc_fence_after();
    }
    if (S == 1) {
        if (epi_warp && acc_ok) {
#pragma unroll 1
            for (int q = 0; q < 2; ++q) {
                const int n = n_tile * 256 + q * 128 + quad * 32 + lane;
#pragma unroll 1
                for (int c = 0; c < MT / 16; ++c) {
                    uint32_t v[16];
                    tc_ld_x16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(q * MT + c * 16), v);
                    tc_wait_ld();
                    if (n < args.N) {
#pragma unroll
                        for (int jj = 0; jj < 16; ++jj) {
                            const int m = m_tile * MT + c * 16 + jj;
                            if (m < args.M) {
                                float* y = args.Y + (size_t)m * args.ldy + n;
                                if (args.mode) *y += __uint_as_float(v[jj]);
                                else *y = __uint_as_float(v[jj]);
                            }
                        }
                    }
                }
            }
        }
    } else if constexpr (reduce_fits<MT>()) {
        // split-K: park this CTA's half-tile in its own shared memory (the A/B
        // rings are idle once the accumulator is final), then every CTA sums a
        // column slice over all S CTAs of the cluster through DSMEM.
        float* red = reinterpret_cast<float*>(base);  // [MT][128]
        const int cols = 128 / S;                     // S divides 128 (1, 2, 4, 8)
        const int vec_per_row = cols / 4;
        for (int q = 0; q < 2; ++q) {
            if (epi_warp && acc_ok) {
#pragma unroll 1
                for (int c = 0; c < MT / 16; ++c) {
                    uint32_t v[16];
                    tc_ld_x16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(q * MT + c * 16), v);
                    tc_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) red[(c * 16 + jj) * 128 + quad * 32 + lane] = __uint_as_float(v[jj]);
                }
            }
            __syncthreads();
            cluster_sync_all();
            const bool cluster_ok = !*abort_flag;
            if (cluster_ok) {
                for (int idx = threadIdx.x; idx < MT * vec_per_row; idx += blockDim.x) {
                    const int mr = idx / vec_per_row;
                    const int cl = rank * cols + (idx % vec_per_row) * 4;
                    const uint32_t la = s_addr(red + mr * 128 + cl);
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int p = 0; p < S; ++p) {
                        const float4 v = ld_dsmem_f4(la, (uint32_t)p);
                        acc.x += v.x;
                        acc.y += v.y;
                        acc.z += v.z;
                        acc.w += v.w;
                    }
                    const int m = m_tile * MT + mr;
                    const int n = n_tile * 256 + q * 128 + cl;
                    if (m < args.M) {
                        float* y = args.Y + (size_t)m * args.ldy + n;
                        const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (n + e < args.N) {
                                if (args.mode) y[e] += vals[e];
                                else y[e] = vals[e];
                            }
                        }
                    }
                }
            }
            cluster_sync_all();  // peers are done reading before the next half overwrites `red`
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
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

// Token tile: the smallest that holds M; above 160 tokens, the one of 128 / 160
// that pads M least (160 on a tie: fewer passes over the weights).
int pick_mt(int M) {
    static const int opts[] = {16, 32, 64, 128, kMaxTokenTile};
    if (M <= kMaxTokenTile) {
        for (int o : opts)
            if (o >= M) return o;
    }
    const int t160 = (M + 159) / 160 * 160, t128 = (M + 127) / 128 * 128;
    return t128 < t160 ? 128 : 160;
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

struct GemmPlan {
    int MT, m_tiles, n_tiles, KG, S, grid;
};

// Split factor S (CTAs per tile, a power of two <= 8 and <= KG) minimising
// waves * (k-steps per CTA + setup), plus a penalty for the on-chip reduction.
GemmPlan plan_gemm(int M, int N, int K) {
    GemmPlan p;
    p.MT = pick_mt(M);
    p.m_tiles = (M + p.MT - 1) / p.MT;
    p.n_tiles = (N + 255) / 256;
    p.KG = (K + 127) / 128;
    const int tiles = p.m_tiles * p.n_tiles;
    const int sms = num_sms();
    double best = 1e30;
    p.S = 1;
    for (int S = 1; S <= kMaxSplit && S <= p.KG; S *= 2) {
        const double waves = (double)((tiles * S + sms - 1) / sms);
        const double items = (double)((p.KG + S - 1) / S);
        const double cost = waves * (items + 1.0) + (S > 1 ? 1.5 : 0.0);
        if (cost < best - 1e-9) {
            best = cost;
            p.S = S;
        }
    }
    p.grid = tiles * p.S;
    return p;
}

template <int MT>
static int launch_tc(const CUtensorMap& map, const GemmArgs& a, int grid, cudaStream_t s) {
    constexpr size_t smem = gemm_smem_bytes<MT>();
    static_assert(smem <= (size_t)kSmemBudget, "shared memory plan exceeds the opt-in limit");
    static_assert(reduce_fits<MT>(), "split-K reduction buffer does not fit in the rings");
    // one CTA per SM: every CTA allocates all 512 TMEM columns, so two CTAs of
    // one cluster must never share an SM
    static_assert(smem > (size_t)kSmemBudget / 2, "shared memory plan must force one CTA per SM");
    static bool attr = false;
    if (!attr) {
        SD_CUDA(cudaFuncSetAttribute(w4a16_tc_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = (unsigned)a.S;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    SD_CUDA(cudaLaunchKernelEx(&cfg, w4a16_tc_kernel<MT>, map, a));
    return SPECDEC_OK;
}

// The kernel needs no global workspace (split tiles are reduced on chip); the
// workspace arguments of the C ABI are kept and may be NULL / 0.
size_t gemm_workspace_bytes(const GemmPlan&) { return 0; }
size_t gemm_workspace_bound(int, int, int) { return 0; }

int gemm_launch(const CUtensorMap& map, const GemmPlan& p, const void* w_tiled, int M, int N, float* Y, int ldy,
                int mode, void* ws, cudaStream_t s) {
    (void)ws;
    GemmArgs a;
    a.w = reinterpret_cast<const uint8_t*>(w_tiled);
    a.M = M;
    a.N = N;
    a.KG = p.KG;
    a.m_tiles = p.m_tiles;
    a.S = p.S;
    a.Y = Y;
    a.ldy = ldy;
    a.mode = mode;
    a.status = device_status_ptr();
    switch (p.MT) {
        case 16: return launch_tc<16>(map, a, p.grid, s);
        case 32: return launch_tc<32>(map, a, p.grid, s);
        case 64: return launch_tc<64>(map, a, p.grid, s);
        case 128: return launch_tc<128>(map, a, p.grid, s);
        case 160: return launch_tc<160>(map, a, p.grid, s);
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
    (void)workspace;
    (void)workspace_bytes;
    SD_CHECK(X && w_tiled && Y && M >= 0 && N > 0 && K > 0 && ldx >= K && ldy >= N && (mode == 0 || mode == 1),
             SPECDEC_EINVAL, "w4a16_gemm: bad argument");
    if (M == 0) return SPECDEC_OK;
    GemmPlan p = plan_gemm(M, N, K);
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, ldx, p.MT);
    if (rc) return rc;
    return gemm_launch(map, p, w_tiled, M, N, Y, ldy, mode, nullptr, as_stream(stream));
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
