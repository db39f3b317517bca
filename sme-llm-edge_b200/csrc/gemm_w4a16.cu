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
// Work decomposition: one output tile = QN x 128 weight rows x MT tokens
// (QN = 2, or QN = 1 for weight matrices with too few 256-row tiles to fill
// the SMs).  A cluster of S CTAs (1 <= S <= 8) owns one tile and splits its K
// range; the S partial accumulators are summed on chip through distributed
// shared memory (each CTA reduces 1/S of the tile's token rows from all S CTAs
// in rank order, so the result is deterministic) and written once.  QN and S
// are chosen per shape from a cost model of waves, k-steps and reduction.
//
// CTA = 19 warps, warp-specialised:
//   warp 0      bulk-copy producer of the int4 units (RS k-steps ahead)
//   warp 18     TMA producer of the activation tiles (SB half-steps ahead)
//   warp 1      TMEM allocator and the single-thread tcgen05.mma issuer
//   warps 2-17  dequant: int4 -> fp16 in registers, written straight into
//               tensor memory with tcgen05.st (one TMEM lane = one weight row);
//               then the epilogue: tcgen05.ld of the accumulators into shared
//               memory, TMA stores out
// MMA: M = 128 weight rows (QN per tile), N = MT, K = 16 per instruction,
// A (the dequantised weights) read from TMEM, B (the activations) from shared
// memory, fp32 accumulators in TMEM.  Keeping A out of shared memory matters:
// with A staged there, the dequant stores plus the MMA's A reads doubled the
// shared-memory traffic of a k-step and made it, not the tensor pipe, the
// limit.  TMEM columns: [0, QN*MT) accumulators, then ST stages of 64 columns
// (QN units x 128/QN k fp16, two fp16 per 32-bit column).
// Every mbarrier wait is bounded: on timeout the CTA records SPECDEC_ETIMEOUT
// in the device status word, skips its output and still meets its cluster
// barriers.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "internal.h"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace specdec {

constexpr int kUnitBytes = 8448;  // 8192 nibble bytes + 128 fp16 scales
constexpr int kGemmThreads = 608;  // 19 warps
constexpr int kDeqWarps = 16;      // warps 2..17
constexpr int kBWarp = 18;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kMaxSplit = 8;
constexpr int kTmemCols = 512;
constexpr int kAStageCols = 64;  // one A stage: QN units x 128/QN k fp16
constexpr int kMaxTokenTile = 160;

// A CTA owns QN 128-row weight units (QN = 2: 256-row tiles; QN = 1: 128-row
// tiles, twice as many, for weight matrices too small to fill the SMs
// otherwise).  One pipeline stage covers KS = 128 / QN k of every unit: 64
// TMEM columns of A and an MT x KS activation tile.  Ring depths, in stages
// unless noted:
//   ST  A stages in TMEM (after the QN*MT accumulator columns)
//   SB  activation tiles in shared memory, a multiple of ST: a tile comes from
//       L2 with about twice the latency of one stage's MMAs, so its ring runs
//       further ahead than the TMEM one where shared memory allows
//   RS  raw int4 k-steps (QN 8448-byte units each) in shared memory; deep
//       enough to hide HBM latency, and what the smem budget leaves
__host__ __device__ constexpr int stages_for(int MT, int QN) {
    return (kTmemCols - QN * MT) / kAStageCols > 4 ? 4 : (kTmemCols - QN * MT) / kAStageCols;
}
__host__ __device__ constexpr int bslot_bytes(int MT, int QN) { return MT * 256 / QN; }
__host__ __device__ constexpr int bstages_for(int MT, int QN) {
    return (QN == 1 && MT > 64) ? stages_for(MT, QN) : 2 * stages_for(MT, QN);
}
__host__ __device__ constexpr int rstages_for(int MT, int QN) {
    return QN == 1 ? (MT > 128 ? 6 : 8) : (MT > 128 ? 6 : (MT > 64 ? 5 : 8));
}
constexpr int kEarlyRaw = 2;  // <= every rstages_for
template <int MT, int QN>
__host__ __device__ constexpr size_t gemm_smem_bytes() {
    return 1024 /*align slack*/ + (size_t)bstages_for(MT, QN) * bslot_bytes(MT, QN) +
           (size_t)rstages_for(MT, QN) * QN * kUnitBytes + 2048;
}
// Requested at launch: at least half the opt-in budget, so that two CTAs
// never share an SM (each allocates all 512 TMEM columns).
template <int MT, int QN>
__host__ __device__ constexpr size_t gemm_launch_smem() {
    return gemm_smem_bytes<MT, QN>() > (size_t)kSmemBudget / 2 + 1024 ? gemm_smem_bytes<MT, QN>()
                                                                       : (size_t)kSmemBudget / 2 + 1024;
}
// the epilogue reuses the B and raw rings: QN MT x 128 fp32 tiles
template <int MT, int QN>
__host__ __device__ constexpr bool reduce_fits() {
    return (size_t)bstages_for(MT, QN) * bslot_bytes(MT, QN) + (size_t)rstages_for(MT, QN) * QN * kUnitBytes >=
           (size_t)QN * MT * 128 * 4;
}

struct GemmArgs {
    const uint8_t* w;
    int M, N, KG, m_tiles, S;
    float* Y;
    int ldy, mode;  // mode 0 store, 1 add, 2 SwiGLU (h = silu(gate) * up into H, below), 3 QKV + RoPE (rope)
    __half* H;      // mode 2: fp16 [M, F] with row stride ldy; weight tile t = [gate rows 128t.. | up rows 128t..]
    int F;          // mode 2: columns of H
    int tma_out;  // tmap_y is valid: the output leaves by TMA (box {128, MT / S}; fp16 over H in mode 2)
    int pdl;      // launched as a programmatic dependent: only the weights may be read before pdl_wait()
    DeviceStatus* status;
    RopeArgs rope;  // mode 3
};

template <int MT, int QN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                    GemmArgs args) {
    static_assert(QN == 1 || QN == 2, "one or two 128-row units per CTA");
    constexpr int ST = stages_for(MT, QN);
    constexpr int SB = bstages_for(MT, QN);
    constexpr int RS = rstages_for(MT, QN);
    constexpr int KS = 128 / QN;               // k per stage and unit
    constexpr int BSLOT = bslot_bytes(MT, QN);  // KS / 64 swizzled panels of MT x 64 fp16
    constexpr int PANEL = MT * 128;
    constexpr int RAWB = QN * kUnitBytes;      // one raw k-step
    constexpr uint32_t A_COL0 = QN * MT;       // first TMEM column of the A stages
    constexpr uint32_t IDESC = idesc_f16(128, MT);
    static_assert(ST >= 2 && A_COL0 + ST * kAStageCols <= kTmemCols, "TMEM plan");
    static_assert(SB % ST == 0, "B ring rounds cover whole A rings");
    static_assert(2 * (RS + ST + SB) + 1 <= 240, "barrier area");

    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    unsigned char* sB = base;               // SB x BSLOT (1024-byte aligned slots)
    unsigned char* sRaw = sB + SB * BSLOT;  // RS x RAWB
    uint64_t* bars = reinterpret_cast<uint64_t*>(sRaw + RS * RAWB);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + RS;
    uint64_t* a_full = raw_empty + RS;  // ST: the 16 dequant warps' columns are in TMEM
    uint64_t* a_empty = a_full + ST;    // ST: MMA commit, the stage's MMAs have read them
    uint64_t* b_full = a_empty + ST;    // SB: activation tile landed (TMA bytes)
    uint64_t* b_empty = b_full + SB;    // SB: MMA commit
    uint64_t* acc_full = b_empty + SB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    // warp index and TMEM base through a shuffle from lane 0: provably
    // warp-uniform, so the tcgen05 / bulk-copy operands derived from them sit
    // in uniform registers.  The role loops below run on whole warps for the
    // same reason; one lane issues.
    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31;
    const int S = args.S;
    const int tile = blockIdx.x / S;
    const int rank = S > 1 ? (int)cluster_rank() : 0;
    const int n_tile = tile / args.m_tiles, m_tile = tile % args.m_tiles;
    const int k0 = (int)(((long long)rank * args.KG) / S);
    const int k1 = (int)(((long long)(rank + 1) * args.KG) / S);
    const int n_items = k1 - k0;  // >= 1 (S <= KG)
    const int n_stages = QN * n_items;
    // int4 k-step it (the QN 128-row units of the tile) -> raw ring slot it % RS
    auto issue_raw = [&](int it) {
        const uint32_t rf = s_addr(&raw_full[it % RS]);
        mbar_expect_tx(rf, RAWB);
        for (int u = 0; u < QN; ++u) {
            const uint8_t* src = args.w + ((size_t)(n_tile * QN + u) * args.KG + (k0 + it)) * kUnitBytes;
            bulk_g2s(s_addr(sRaw + (it % RS) * RAWB + u * kUnitBytes), src, kUnitBytes, rf);
        }
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < RS; ++i) {
            mbar_init(s_addr(&raw_full[i]), 1);
            mbar_init(s_addr(&raw_empty[i]), kDeqWarps);
        }
        for (int i = 0; i < ST; ++i) {
            mbar_init(s_addr(&a_full[i]), kDeqWarps);
            mbar_init(s_addr(&a_empty[i]), 1);
        }
        for (int i = 0; i < SB; ++i) {
            mbar_init(s_addr(&b_full[i]), 1);
            mbar_init(s_addr(&b_empty[i]), 1);
        }
        mbar_init(s_addr(acc_full), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_async_smem();
        // the first kEarlyRaw int4 k-steps start streaming now, ahead of the
        // TMEM allocation and the block-wide barrier (issuing more here delays
        // that barrier by more than it gains)
        for (int it = 0; it < kEarlyRaw && it < n_items; ++it) issue_raw(it);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_addr(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = __shfl_sync(0xffffffffu, *tmem_slot, 0);

    pdl_trigger();  // the next kernel may start its prologue
    if (warp == 0) {
        // ------------------------------------------------ int4 unit producer
        // (weights: read before pdl_wait -- they are written once, before any step)
        // k-steps 0 .. kEarlyRaw-1 were issued before the block-wide barrier
        bool ok = true;
        int it = kEarlyRaw < n_items ? kEarlyRaw : n_items;
        for (; it < n_items; ++it) {
            if (it >= RS) ok = mbar_wait(s_addr(&raw_empty[it % RS]), ((it / RS) - 1) & 1);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) break;
            if (lane == 0) issue_raw(it);
            __syncwarp();
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            record_timeout(args.status, 1);
        }
        // drain: the copies issued above complete before the CTA exits
        if (it > 0) (void)mbar_wait(s_addr(&raw_full[(it - 1) % RS]), ((it - 1) / RS) & 1);
    } else if (warp == kBWarp) {
        // ------------------------------------------------ activation (B operand) producer
        if (args.pdl) pdl_wait();  // X is written by the kernel before this one
        // Rounds of SB stages with the slot index unrolled, so every
        // shared-memory address below is a fixed offset from a loop-invariant
        // base.
        bool ok = true, stop = false;
        int j = 0;
        for (int j0 = 0; j0 < n_stages && !stop; j0 += SB) {
#pragma unroll
            for (int sb = 0; sb < SB; ++sb) {
                j = j0 + sb;
                if (j >= n_stages) break;
                if (j0 > 0) ok = mbar_wait(s_addr(&b_empty[sb]), ((j0 / SB) - 1) & 1);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) {
                    stop = true;
                    break;
                }
                if (lane == 0) {
                    const uint32_t bf = s_addr(&b_full[sb]);
                    mbar_expect_tx(bf, BSLOT);
#pragma unroll
                    for (int pn = 0; pn < KS / 64; ++pn)
                        tma_load_2d(s_addr(sB + sb * BSLOT + pn * PANEL), &tmap_x, k0 * 128 + j * KS + pn * 64,
                                    m_tile * MT, bf);
                }
                __syncwarp();
                ++j;
            }
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            record_timeout(args.status, 5);
        }
        // j = stages issued; drain the last one
        if (j > 0) (void)mbar_wait(s_addr(&b_full[(j - 1) % SB]), ((j - 1) / SB) & 1);
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        // One thread runs the loop: a stage's 8 MMAs are queued behind the
        // previous stage's, so the time from one commit to the next stage's
        // first MMA is idle tensor pipe and is kept to one barrier probe.  The
        // descriptors are precomputed offsets of one base: an MMA whose
        // operands are recomputed in the issue loop costs several times the
        // tensor-pipe time of the instruction itself.
        if (lane == 0) {
            const uint64_t bdesc0 = sw128_desc(s_addr(sB));
            const uint32_t a_base = tmem + A_COL0;
            bool ok = true;
            // rounds of SB stages: B slot u, A stage u % ST (both constants)
            for (int j0 = 0; j0 < n_stages && ok; j0 += SB) {
                const uint32_t bpar = (uint32_t)(j0 / SB) & 1u;
                const int a_uses = j0 / ST;  // uses of every A stage before this round
#pragma unroll
                for (int u = 0; u < SB; ++u) {
                    const int j = j0 + u;
                    if (j >= n_stages) break;
                    const int s = u % ST;
                    if (!mbar_wait(s_addr(&a_full[s]), (uint32_t)(a_uses + u / ST) & 1u) ||
                        !mbar_wait(s_addr(&b_full[u]), bpar)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int ks = 0; ks < KS / 16; ++ks) {
                        // B: slot u, panel ks / 4, k16 slice ks % 4 (32 bytes into each 128-byte swizzled row)
                        const uint64_t bd = bdesc0 + (uint64_t)((u * BSLOT + (ks >> 2) * PANEL + (ks & 3) * 32) >> 4);
#pragma unroll
                        for (int q = 0; q < QN; ++q)  // unit q: A columns q*KS/2 + ks*8 .. +8 (k16 = 8 columns)
                            tc_mma_f16_ts(tmem + (uint32_t)(q * MT),
                                          a_base + (uint32_t)(s * kAStageCols + q * (KS / 2) + ks * 8), bd, IDESC,
                                          (j > 0 || ks > 0) ? 1u : 0u);
                    }
                    tc_commit(s_addr(&a_empty[s]));
                    tc_commit(s_addr(&b_empty[u]));
                }
            }
            if (ok) tc_commit(s_addr(acc_full));
            else {  // a stage never filled: a producer failed (and flagged it) or timed out
                *abort_flag = 1;
                record_timeout(args.status, 2);
            }
        }
        __syncwarp();
    } else if (warp >= 2 && warp < 2 + kDeqWarps) {
        // ------------------------------------------------ dequant
        // A warp may only touch TMEM lanes 32*(warp%4) .. +31.  The four warps
        // of one lane quarter split a stage as (unit q, 32-k slice kh): the
        // thread = weight row r of unit q, 32 k (4 words, 16 TMEM columns).
        const int dw = warp - 2;
        const int q = (dw >> 2) % QN;
        const int kh = (dw >> 2) / QN;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t t_row =
            tmem + ((uint32_t)(quarter * 32) << 16) + A_COL0 + (uint32_t)(q * (KS / 2) + kh * 16);
        const __half2 bias = __float2half2_rn(1032.0f);
        bool ok = true;
        // Rounds of ST k-steps = QN*ST stages, so the stage of the round's
        // stage h is the constant h % ST.
        for (int it0 = 0; it0 < n_items && ok; it0 += ST) {
#pragma unroll
            for (int u = 0; u < ST; ++u) {
                const int it = it0 + u;
                if (it >= n_items) break;
                const int rs = it % RS;
                ok = mbar_wait(s_addr(&raw_full[rs]), (it / RS) & 1);
                // warp-uniform decision: the tcgen05.st below is a .sync.aligned warp instruction
                ok = __all_sync(0xffffffffu, ok && !*abort_flag);
                if (!ok) break;
                const unsigned char* unit = sRaw + rs * RAWB + q * kUnitBytes;
                const __half2 s2 = __half2half2(*reinterpret_cast<const __half*>(unit + 8192 + r * 2));
#pragma unroll
                for (int hk = 0; hk < QN; ++hk) {
                    const int s = (QN * u + hk) % ST;
                    const int j = QN * it + hk;
                    if (j >= ST) ok = mbar_wait(s_addr(&a_empty[s]), ((j / ST) - 1) & 1);
                    ok = __all_sync(0xffffffffu, ok && !*abort_flag);
                    if (!ok) break;
                    uint32_t wv[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i)  // word (kc, r): k = kc*8 .. kc*8+7 of row r; lanes read consecutive words
                        wv[i] = *reinterpret_cast<const uint32_t*>(
                            unit + (((hk * (KS / 8) + kh * 4 + i) * 128 + r) << 2));
                    uint32_t outw[16];  // column i*4+jj = fp16 pair (k = 8i+2jj, 8i+2jj+1) of this k-quarter
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            const uint32_t t = ((wv[i] >> (4 * jj)) & 0x000F000Fu) | 0x64006400u;
                            __half2 hv = *reinterpret_cast<const __half2*>(&t);
                            hv = __hmul2(__hsub2(hv, bias), s2);  // exact (u - 8), then one rounding of (u - 8) * s
                            outw[i * 4 + jj] = *reinterpret_cast<uint32_t*>(&hv);
                        }
                    }
                    tc_st_x16(t_row + (uint32_t)(s * kAStageCols), outw);
                    tc_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_addr(&a_full[s]));
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(s_addr(&raw_empty[rs]));
            }
        }
        if (!ok) {
            *abort_flag = 1;
            record_timeout(args.status, 4);
        }
    }

    // ---------------------------------------------------- epilogue (all threads)
    // Warps 2-17 (four per TMEM lane quarter) drain the accumulators into
    // shared memory as [token][weight row] fp32 (the rings are idle now).  The
    // tile then leaves by one TMA store per unit (a TMA reduce-add for mode 1)
    // when Y's rows are 16-byte aligned, else by coalesced plain stores.
    const bool epi_warp = warp >= 2 && warp < 2 + kDeqWarps;
    const int quad = warp & 3;       // TMEM lane quarter = weight rows quad*32 .. +31
    const int eg = (warp - 2) >> 2;  // column chunks c = eg, eg + 4, ...
    if (epi_warp) {
        const bool acc_ok = __all_sync(0xffffffffu, mbar_wait(s_addr(acc_full), 0));
        if (!acc_ok && lane == 0) {
            *abort_flag = 1;
            record_timeout(args.status, 3);
        }
        tc_fence_after();
    }
    __syncthreads();
    const bool acc_ok = !*abort_flag;
    // half q of the accumulator -> dst[token][128]: a warp's 16-column
    // chunks c = eg, eg + 4, ... are all loaded before one wait
    auto drain = [&](int q, float* dst) {
        constexpr int kChunks = MT / 16, kGroups = kDeqWarps / 4, kPer = (kChunks + kGroups - 1) / kGroups;
        uint32_t v[kPer][16];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int c = eg + i * kGroups;
            if (c < kChunks) tc_ld_x16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(q * MT + c * 16), v[i]);
        }
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int c = eg + i * kGroups;
            if (c < kChunks) {
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) dst[(c * 16 + jj) * 128 + quad * 32 + lane] = __uint_as_float(v[i][jj]);
            }
        }
    };
    // The QN units of this CTA's accumulator are parked in shared memory as
    // [unit][token][128].  The CTA's share of the output is token rows
    // [r0, r0 + MT/S) of every unit: with S > 1 it sums those rows over the S
    // CTAs of the cluster through DSMEM, in rank order, in place (each CTA
    // overwrites only its own rows, which no peer reads), then writes them.
    float* stage = reinterpret_cast<float*>(base);  // [QN][MT][128]
    const int rows = MT / S, r0 = rank * rows;       // S divides MT (16 | MT, S <= 8)
    // Mode 2 without a k split: the gate and up rows of a feature share a
    // TMEM lane (unit 0 at columns 0.., unit 1 at MT..), so each thread forms
    // h = fp16(silu(g) * u) from its two loads and writes the fp16 [MT][128]
    // box directly -- no fp32 staging of g and u in shared memory.
    const bool swiglu_direct = QN == 2 && args.mode == 2 && S == 1;
    if (epi_warp && acc_ok) {
        if (swiglu_direct) {
            constexpr int kChunks = MT / 16, kGroups = kDeqWarps / 4;
            __half* h = reinterpret_cast<__half*>(stage);
            const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
            for (int c = eg; c < kChunks; c += kGroups) {
                uint32_t g[16], u[16];
                tc_ld_x16(trow + (uint32_t)(c * 16), g);
                tc_ld_x16(trow + (uint32_t)(MT + c * 16), u);
                tc_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    // fast exp and divide (one MUFU op each): within a few fp32 ulp,
                    // well inside the fp16 rounding of h
                    const float gv = __uint_as_float(g[jj]);
                    const float hv = __fmul_rn(__fdividef(gv, __fadd_rn(1.0f, __expf(-gv))), __uint_as_float(u[jj]));
                    h[(c * 16 + jj) * 128 + quad * 32 + lane] = __float2half_rn(hv);
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < QN; ++q) drain(q, stage + q * MT * 128);
        }
    }
    if constexpr (reduce_fits<MT, QN>()) {
        if (S > 1) {
            __syncthreads();
            cluster_sync_all();  // every CTA's partial tile is parked
            if (!*abort_flag) {
                const int nvec = QN * rows * 32;  // float4 columns of (unit, row)
                for (int idx = threadIdx.x; idx < nvec; idx += blockDim.x) {
                    const int q = idx / (rows * 32), rem = idx - q * rows * 32;
                    float* p = stage + (size_t)q * MT * 128 + (r0 + (rem >> 5)) * 128 + (rem & 31) * 4;
                    const uint32_t la = s_addr(p);
                    float4 v[kMaxSplit];  // all S remote loads in flight before the sum
#pragma unroll
                    for (int pr = 0; pr < kMaxSplit; ++pr)
                        if (pr < S) v[pr] = ld_dsmem_f4(la, (uint32_t)pr);
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int pr = 0; pr < kMaxSplit; ++pr)
                        if (pr < S) {
                            acc.x += v[pr].x;
                            acc.y += v[pr].y;
                            acc.z += v[pr].z;
                            acc.w += v[pr].w;
                        }
                    *reinterpret_cast<float4*>(p) = acc;
                }
            }
        }
    }
    // Mode 2 (SwiGLU): half 0 holds gate rows 128 * n_tile .. +127 and half 1
    // the up rows of the same features, so this CTA's token rows give
    // h[m][128 * n_tile + c] = fp16(silu(g) * u) (main.cpp:246-249, 338-340).
    // Every thread keeps its results in registers until all have read the
    // fp32 rows, then the CTA overwrites the start of its own half-0 rows
    // (no peer reads them) with a dense fp16 [rows][128] box.
    __half* hbox = reinterpret_cast<__half*>(stage + r0 * 128);
    if (QN == 2 && args.mode == 2 && !swiglu_direct) {
        constexpr int kItems = (MT * 16 + kGemmThreads - 1) / kGemmThreads;  // (row, 8 features) per thread
        const int nitems = rows * 16;
        uint4 hv[kItems];
        __syncthreads();
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            const int idx = threadIdx.x + it * kGemmThreads;
            if (idx < nitems) {
                const float* gp = stage + (r0 + (idx >> 4)) * 128 + (idx & 15) * 8;
                const float* up = gp + MT * 128;
                float g[8], u[8];
                *reinterpret_cast<float4*>(g) = *reinterpret_cast<const float4*>(gp);
                *reinterpret_cast<float4*>(g + 4) = *reinterpret_cast<const float4*>(gp + 4);
                *reinterpret_cast<float4*>(u) = *reinterpret_cast<const float4*>(up);
                *reinterpret_cast<float4*>(u + 4) = *reinterpret_cast<const float4*>(up + 4);
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    // fast exp and divide (one MUFU op each): within a few fp32 ulp,
                    // well inside the fp16 rounding of h
                    const float a = __fmul_rn(__fdividef(g[2 * j], __fadd_rn(1.0f, __expf(-g[2 * j]))), u[2 * j]);
                    const float b = __fmul_rn(__fdividef(g[2 * j + 1], __fadd_rn(1.0f, __expf(-g[2 * j + 1]))),
                                              u[2 * j + 1]);
                    __half2 h2 = __floats2half2_rn(a, b);
                    w[j] = *reinterpret_cast<uint32_t*>(&h2);
                }
                hv[it] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < kItems; ++it) {
            const int idx = threadIdx.x + it * kGemmThreads;
            if (idx < nitems) *reinterpret_cast<uint4*>(hbox + (idx >> 4) * 128 + (idx & 15) * 8) = hv[it];
        }
    }
    fence_async_smem();  // the generic-proxy writes above, before the TMA reads them
    if (args.pdl) pdl_wait();  // Y may still be read or written by earlier kernels
    __syncthreads();
    if (QN == 1 && args.mode == 3) {
        // Mode 3 (QKV + RoPE + KV write; rotate-half RoPE as rust_sme_rope_f32,
        // src/sme_kernel/rust_sme/src/lib.rs:621-666): this
        // CTA's token rows of the tile's 128 / hd heads.  An item = dims
        // (d, d+1) and (d + hd/2, d + hd/2 + 1) of one head of one token, the
        // same arithmetic as the standalone RoPE pass.
        const RopeArgs& ra = args.rope;
        const int hd = ra.hd, halfd = hd / 2;
        const int per_head = halfd / 2, per_tok = 128 / hd * per_head;  // = 32
        if (acc_ok && !*abort_flag) {
            for (int idx = threadIdx.x; idx < rows * per_tok; idx += blockDim.x) {
                const int rr = idx / per_tok, w = idx - rr * per_tok;
                const int m = m_tile * MT + r0 + rr;
                if (m >= args.M) continue;
                const int hu = w / per_head, d = (w - hu * per_head) * 2;
                const int h = n_tile * (128 / hd) + hu;  // head in [q | k | v]
                if (h >= ra.Hq + 2 * ra.Hkv) continue;
                const float* row = stage + (size_t)(r0 + rr) * 128 + hu * hd;
                const float2 a = *reinterpret_cast<const float2*>(row + d);
                const float2 c = *reinterpret_cast<const float2*>(row + d + halfd);
                __half* dst;
                if (h < ra.Hq) {
                    dst = ra.q16 + (size_t)m * ra.Hq * hd + (size_t)h * hd;
                } else {
                    const int b = m / ra.R, sl = ra.slot[m];
                    const int blk = ra.tables[(size_t)b * ra.max_blocks + sl / 16];
                    const int kvsel = h < ra.Hq + ra.Hkv ? 0 : 1, kh = h - ra.Hq - kvsel * ra.Hkv;
                    dst = ra.kv_layer + ((((size_t)blk * 2 + kvsel) * ra.Hkv + kh) * 16 + sl % 16) * hd;
                }
                if (h < ra.Hq + ra.Hkv) {
                    const float* cs = ra.cos_t + (size_t)ra.pos[m] * halfd;
                    const float* sn = ra.sin_t + (size_t)ra.pos[m] * halfd;
                    const float2 cv = *reinterpret_cast<const float2*>(cs + d);
                    const float2 sv = *reinterpret_cast<const float2*>(sn + d);
                    *reinterpret_cast<__half2*>(dst + d) =
                        __floats2half2_rn(__fsub_rn(__fmul_rn(a.x, cv.x), __fmul_rn(c.x, sv.x)),
                                          __fsub_rn(__fmul_rn(a.y, cv.y), __fmul_rn(c.y, sv.y)));
                    *reinterpret_cast<__half2*>(dst + d + halfd) =
                        __floats2half2_rn(__fadd_rn(__fmul_rn(c.x, cv.x), __fmul_rn(a.x, sv.x)),
                                          __fadd_rn(__fmul_rn(c.y, cv.y), __fmul_rn(a.y, sv.y)));
                } else {
                    *reinterpret_cast<__half2*>(dst + d) = __floats2half2_rn(a.x, a.y);
                    *reinterpret_cast<__half2*>(dst + d + halfd) = __floats2half2_rn(c.x, c.y);
                }
            }
        }
    } else if (QN == 2 && args.mode == 2) {
        if (acc_ok && !*abort_flag && m_tile * MT + r0 < args.M) {
            if (args.tma_out) {
                if (threadIdx.x == 0) {
                    tma_out_2d(&tmap_y, s_addr(hbox), n_tile * 128, m_tile * MT + r0, 0);
                    bulk_commit();
                    bulk_wait_read();
                }
            } else {
                for (int idx = threadIdx.x; idx < rows * 128; idx += blockDim.x) {
                    const int m = m_tile * MT + r0 + (idx >> 7), f = n_tile * 128 + (idx & 127);
                    if (m < args.M && f < args.F) args.H[(size_t)m * args.ldy + f] = hbox[idx];
                }
            }
        }
    } else if (acc_ok && !*abort_flag && m_tile * MT + r0 < args.M) {
        if (args.tma_out) {
            if (threadIdx.x == 0) {
                for (int q = 0; q < QN; ++q)  // a unit wholly past N has nothing to write
                    if ((n_tile * QN + q) * 128 < args.N)
                        tma_out_2d(&tmap_y, s_addr(stage + (size_t)q * MT * 128 + r0 * 128), (n_tile * QN + q) * 128,
                                   m_tile * MT + r0, args.mode);
                bulk_commit();
                bulk_wait_read();
            }
        } else {
            for (int idx = threadIdx.x; idx < QN * rows * 128; idx += blockDim.x) {
                const int q = idx / (rows * 128), rem = idx - q * rows * 128;
                const int r = r0 + rem / 128, c = rem & 127;
                const int m = m_tile * MT + r, n = (n_tile * QN + q) * 128 + c;
                if (m < args.M && n < args.N) {
                    float* y = args.Y + (size_t)m * args.ldy + n;
                    const float v = stage[(size_t)q * MT * 128 + r * 128 + c];
                    if (args.mode) *y += v;
                    else *y = v;
                }
            }
        }
    }
    if (S > 1) cluster_sync_all();  // peers have finished reading this CTA's parked tile

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

// Output map: fp32 Y [M][ldy], box {128, MT / S} (one CTA's token rows of a
// half tile).  Returns 0 when Y cannot be written by TMA.
static int make_y_tmap(CUtensorMap* map, float* Y, int M, int N, int ldy, int MT, int S) {
    auto enc = get_encode();
    if (!enc || (reinterpret_cast<uintptr_t>(Y) & 15) != 0 || (ldy % 4) != 0) return 0;
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)ldy * 4};
    cuuint32_t box[2] = {128, (cuuint32_t)(MT / S)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, Y, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 1 : 0;
}

// fp16 h [M, F] of the SwiGLU epilogue (box {128 features, MT / S tokens}).
static int make_h_tmap(CUtensorMap* map, __half* h, int M, int F, int ldh, int MT, int S) {
    auto enc = get_encode();
    if (!enc || (reinterpret_cast<uintptr_t>(h) & 15) != 0 || (ldh % 8) != 0) return 0;
    cuuint64_t dims[2] = {(cuuint64_t)F, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)ldh * 2};
    cuuint32_t box[2] = {128, (cuuint32_t)(MT / S)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, h, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 1 : 0;
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

template <int MT, int QN>
static bool set_smem_attr() {
    constexpr size_t smem = gemm_launch_smem<MT, QN>();
    static_assert(smem <= (size_t)kSmemBudget, "shared memory plan exceeds the opt-in limit");
    static_assert(reduce_fits<MT, QN>(), "split-K reduction buffer does not fit in the rings");
    // one CTA per SM: every CTA allocates all 512 TMEM columns, so two CTAs of
    // one cluster must never share an SM
    static_assert(smem > (size_t)kSmemBudget / 2, "shared memory plan must force one CTA per SM");
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(w4a16_tc_kernel<MT, QN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        attr = true;
    }
    return true;
}

// How many clusters of S CTAs the device runs at once.  Clusters must fit
// inside one GPC, so for S = 8 this is fewer than SMs / 8; planning with
// SMs / S would turn a one-wave grid into two waves.
template <int MT, int QN>
static int max_active_clusters(int S) {
    static int cache[4] = {0, 0, 0, 0};
    const int idx = S == 1 ? 0 : (S == 2 ? 1 : (S == 4 ? 2 : 3));
    if (!cache[idx]) {
        int n = 0;
        if (S == 1) {
            n = num_sms();
        } else if (set_smem_attr<MT, QN>()) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)(S * num_sms()));
            cfg.blockDim = dim3(kGemmThreads);
            cfg.dynamicSmemBytes = gemm_launch_smem<MT, QN>();
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = (unsigned)S;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&n, w4a16_tc_kernel<MT, QN>, &cfg) != cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
        }
        cache[idx] = n > 0 ? n : num_sms() / S;
    }
    return cache[idx];
}

template <int QN>
static int clusters_for_qn(int MT, int S) {
    switch (MT) {
        case 16: return max_active_clusters<16, QN>(S);
        case 32: return max_active_clusters<32, QN>(S);
        case 64: return max_active_clusters<64, QN>(S);
        case 128: return max_active_clusters<128, QN>(S);
        default: return max_active_clusters<160, QN>(S);
    }
}
static int clusters_for(int MT, int QN, int S) { return QN == 1 ? clusters_for_qn<1>(MT, S) : clusters_for_qn<2>(MT, S); }

// Estimated time (us) of one plan: waves of co-scheduled clusters, each CTA
// running ceil(KG / S) k-steps of QN units (8 MMAs of N = MT per unit and
// k-step, at the power-capped tensor rate) plus its fixed setup and epilogue,
// and the DSMEM reduction of split tiles (its data grows with QN).  Fitted to
// timelines measured on B200.
static double plan_cost(int MT, int QN, int S, int tiles, int KG) {
    const int per_wave = clusters_for(MT, QN, S);
    const double waves = (double)((tiles + per_wave - 1) / per_wave);
    const double t8 = 0.28 + 0.0018 * MT;  // us per 8 MMAs (one unit, one k-step)
    const double main = (double)((KG + S - 1) / S) * QN * t8;
    return waves * (main + 5.0) + (S > 1 ? 0.8 + 2.1 * QN : 0.0);
}

// Units per CTA QN (from qn_mask: bit 0 allows 1, bit 1 allows 2) and split
// factor S (CTAs per tile, a power of two <= 8 and <= KG) of least cost.
static GemmPlan plan_gemm_qn(int M, int N, int K, int qn_mask) {
    GemmPlan p;
    p.MT = pick_mt(M);
    p.m_tiles = (M + p.MT - 1) / p.MT;
    p.KG = (K + 127) / 128;
    double best = 1e30;
    p.QN = 2;
    p.S = 1;
    for (int QN = 2; QN >= 1; --QN) {
        if (!(qn_mask & QN)) continue;
        const int tiles = p.m_tiles * ((N + 128 * QN - 1) / (128 * QN));
        for (int S = 1; S <= kMaxSplit && S <= p.KG; S *= 2) {
            const double cost = plan_cost(p.MT, QN, S, tiles, p.KG);
            if (cost < best - 1e-9) {
                best = cost;
                p.QN = QN;
                p.S = S;
            }
        }
    }
    p.n_tiles = (N + 128 * p.QN - 1) / (128 * p.QN);
    p.grid = p.m_tiles * p.n_tiles * p.S;
    return p;
}

GemmPlan plan_gemm(int M, int N, int K) { return plan_gemm_qn(M, N, K, 3); }

// A plan with QN and S fixed by the caller (validation of every path).
static GemmPlan plan_fixed(int M, int N, int K, int QN, int S) {
    GemmPlan p;
    p.MT = pick_mt(M);
    p.m_tiles = (M + p.MT - 1) / p.MT;
    p.KG = (K + 127) / 128;
    p.QN = QN;
    p.S = S;
    p.n_tiles = (N + 128 * QN - 1) / (128 * QN);
    p.grid = p.m_tiles * p.n_tiles * S;
    return p;
}

template <int MT, int QN>
static int launch_tc(const CUtensorMap& map, const CUtensorMap& map_y, const GemmArgs& a, int grid, cudaStream_t s) {
    constexpr size_t smem = gemm_launch_smem<MT, QN>();
    if (!set_smem_attr<MT, QN>()) {
        set_error("w4a16_gemm: cannot opt in to the shared memory the kernel needs");
        return SPECDEC_ECUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kGemmThreads);
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
    SD_CUDA(cudaLaunchKernelEx(&cfg, w4a16_tc_kernel<MT, QN>, map, map_y, a));
    return SPECDEC_OK;
}

// The kernel needs no global workspace (split tiles are reduced on chip); the
// workspace arguments of the C ABI are kept and may be NULL / 0.
size_t gemm_workspace_bytes(const GemmPlan&) { return 0; }
size_t gemm_workspace_bound(int, int, int) { return 0; }

template <int QN>
static int launch_mt_qn(const CUtensorMap& map, const CUtensorMap& map_y, const GemmArgs& a, const GemmPlan& p,
                        cudaStream_t s) {
    switch (p.MT) {
        case 16: return launch_tc<16, QN>(map, map_y, a, p.grid, s);
        case 32: return launch_tc<32, QN>(map, map_y, a, p.grid, s);
        case 64: return launch_tc<64, QN>(map, map_y, a, p.grid, s);
        case 128: return launch_tc<128, QN>(map, map_y, a, p.grid, s);
        case 160: return launch_tc<160, QN>(map, map_y, a, p.grid, s);
        default: break;
    }
    set_error("w4a16_gemm: unsupported token tile");
    return SPECDEC_EINVAL;
}

static int launch_mt(const CUtensorMap& map, const CUtensorMap& map_y, const GemmArgs& a, const GemmPlan& p,
                     cudaStream_t s) {
    if (p.QN == 1) return launch_mt_qn<1>(map, map_y, a, p, s);
    if (p.QN == 2) return launch_mt_qn<2>(map, map_y, a, p, s);
    set_error("w4a16_gemm: unsupported token tile");
    return SPECDEC_EINVAL;
}

static GemmArgs gemm_args(const GemmPlan& p, const void* w_tiled, int M, int N, int ldy, int mode, bool pdl) {
    GemmArgs a;
    a.w = reinterpret_cast<const uint8_t*>(w_tiled);
    a.M = M;
    a.N = N;
    a.KG = p.KG;
    a.m_tiles = p.m_tiles;
    a.S = p.S;
    a.Y = nullptr;
    a.ldy = ldy;
    a.mode = mode;
    a.H = nullptr;
    a.F = 0;
    a.tma_out = 0;
    a.pdl = pdl ? 1 : 0;
    a.status = device_status_ptr();
    memset(&a.rope, 0, sizeof(a.rope));
    return a;
}

int gemm_launch(const CUtensorMap& map, const GemmPlan& p, const void* w_tiled, int M, int N, float* Y, int ldy,
                int mode, void* ws, cudaStream_t s, bool pdl) {
    (void)ws;
    GemmArgs a = gemm_args(p, w_tiled, M, N, ldy, mode, pdl);
    a.Y = Y;
    // Y leaves by TMA when its rows are 16-byte aligned; otherwise plain stores.
    CUtensorMap map_y;
    a.tma_out = make_y_tmap(&map_y, Y, M, N, ldy, p.MT, p.S);
    if (!a.tma_out) memset(&map_y, 0, sizeof(map_y));
    return launch_mt(map, map_y, a, p, s);
}

int swiglu_units(int F) { return 2 * ((F + 127) / 128); }

// the QKV + RoPE epilogue keeps whole heads in one-unit tiles
GemmPlan plan_gemm_qkv(int M, int N, int K) { return plan_gemm_qn(M, N, K, 1); }

int gemm_launch_qkv_rope(const CUtensorMap& map, const GemmPlan& p, const void* w_qkv, int M, int N, const RopeArgs& ra,
                         cudaStream_t s, bool pdl) {
    if (p.QN != 1 || ra.hd <= 0 || 128 % ra.hd != 0 || ra.hd % 4 != 0 || N != (ra.Hq + 2 * ra.Hkv) * ra.hd) {
        set_error("w4a16_gemm_qkv_rope: the plan must use one-unit tiles of whole heads");
        return SPECDEC_EINVAL;
    }
    GemmArgs a = gemm_args(p, w_qkv, M, N, 0, 3, pdl);
    a.rope = ra;
    CUtensorMap unused;
    memset(&unused, 0, sizeof(unused));
    return launch_mt(map, unused, a, p, s);
}

// the SwiGLU epilogue pairs gate and up units: two units per CTA
GemmPlan plan_gemm_swiglu(int M, int F, int K) { return plan_gemm_qn(M, 128 * swiglu_units(F), K, 2); }

int gemm_launch_swiglu(const CUtensorMap& map, const GemmPlan& p, const void* w_gu, int M, int F, __half* h, int ldh,
                       cudaStream_t s, bool pdl) {
    if (p.QN != 2) {
        set_error("w4a16_gemm_swiglu: the plan must pair gate and up units");
        return SPECDEC_EINVAL;
    }
    GemmArgs a = gemm_args(p, w_gu, M, 128 * swiglu_units(F), ldh, 2, pdl);
    a.H = h;
    a.F = F;
    CUtensorMap map_h;
    a.tma_out = make_h_tmap(&map_h, h, M, F, ldh, p.MT, p.S);
    if (!a.tma_out) memset(&map_h, 0, sizeof(map_h));
    return launch_mt(map, map_h, a, p, s);
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
    if (plan_gemm_uses_gemv(M, N, K))  // few token rows: the bandwidth-shaped kernel
        return gemv_launch(reinterpret_cast<const __half*>(X), ldx, K, plan_gemv(M, N, K), w_tiled, M, N, Y, ldy,
                           mode, as_stream(stream), false);
    GemmPlan p = plan_gemm(M, N, K);
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, ldx, p.MT);
    if (rc) return rc;
    return gemm_launch(map, p, w_tiled, M, N, Y, ldy, mode, nullptr, as_stream(stream), false);
}

extern "C" int specdec_w4a16_plan(int M, int N, int K, int units, int32_t* out) {
    SD_CHECK(out && M > 0 && N > 0 && K > 0 && units >= 0 && units <= 2, SPECDEC_EINVAL, "w4a16_plan: bad argument");
    const GemmPlan p = plan_gemm_qn(M, N, K, units == 0 ? 3 : units);
    out[0] = p.MT;
    out[1] = p.QN;
    out[2] = p.S;
    out[3] = p.grid;
    return SPECDEC_OK;
}

extern "C" int specdec_w4a16_gemm_with_plan(const uint16_t* X, int M, int ldx, const void* w_tiled, int N, int K,
                                            float* Y, int ldy, int mode, int qn, int split, void* stream) {
    SD_CHECK(X && w_tiled && Y && M >= 0 && N > 0 && K > 0 && ldx >= K && ldy >= N && (mode == 0 || mode == 1) &&
                 (qn == 1 || qn == 2) && (split == 1 || split == 2 || split == 4 || split == 8) &&
                 split <= (K + 127) / 128,
             SPECDEC_EINVAL, "w4a16_gemm_with_plan: bad argument");
    if (M == 0) return SPECDEC_OK;
    const GemmPlan p = plan_fixed(M, N, K, qn, split);
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, ldx, p.MT);
    if (rc) return rc;
    return gemm_launch(map, p, w_tiled, M, N, Y, ldy, mode, nullptr, as_stream(stream), false);
}

extern "C" int specdec_w4a16_gemm_swiglu(const uint16_t* X, int M, int ldx, const void* w_gu_tiled, int F, int K,
                                         uint16_t* h, int ldh, void* stream) {
    SD_CHECK(X && w_gu_tiled && h && M >= 0 && F > 0 && K > 0 && ldx >= K && ldh >= F, SPECDEC_EINVAL,
             "w4a16_gemm_swiglu: bad argument");
    if (M == 0) return SPECDEC_OK;
    GemmPlan p = plan_gemm_swiglu(M, F, K);
    CUtensorMap map;
    int rc = make_x_tmap(&map, X, M, K, ldx, p.MT);
    if (rc) return rc;
    return gemm_launch_swiglu(map, p, w_gu_tiled, M, F, reinterpret_cast<__half*>(h), ldh, as_stream(stream), false);
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
