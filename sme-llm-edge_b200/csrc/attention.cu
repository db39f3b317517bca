// attention.cu -- split-KV verify attention over paged fp16 KV (sm_100a).
//
// One CTA per (sequence, KV head, split, 128-row query tile).  All G = Hq/Hkv
// query heads of the KV head and all R new rows of the sequence are processed
// together (query row r * G + g), so every KV byte is read from HBM once per
// step; R * G rows beyond 128 take further tiles.
//
// The path is HBM-bound, so the kernel is built around keeping enough bytes in
// flight: producer warps stream the split's KV blocks (16 tokens; K and V, each
// as 64-column halves with 128-byte swizzle) through rings of shared memory,
// one TMA tensor load per block, block numbers read from a copy of the
// block-table slice in shared memory.  Scores S = Q.K^T and O = P.V accumulate
// in tensor memory (tcgen05.mma, fp16 in, fp32 accumulate) and the CUDA cores
// run an online base-2 softmax (see the kernel's comment below).  The S splits
// of one (sequence, KV head, tile) form a thread-block cluster and are merged
// through distributed shared memory with the log-sum-exp combine of
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
#include "tcgen05.cuh"

namespace specdec {

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

// ------------------------------------------------------------ tcgen05 variant
// 128 query rows per CTA (a further tile per 128 rows beyond).  The query tile is the M = 128 side of every MMA,
// so the scores S = Q.K^T and the output O = P.V accumulate in TMEM and the
// CUDA cores only run the softmax.  A group = four 16-token blocks = 64 keys.
//   warps 0-7  softmax: warp w serves the query rows of TMEM lane quarter
//              w % 4 and keys [32 * (w / 4), +32) of every group, one thread
//              per row: scale, mask, row max (the two halves of a row swap
//              theirs through shared memory), P = exp2(s - m) in fp16 into
//              TMEM, running sum.  O is rescaled only when a row's max grows
//              by more than 2^8, so P stays below 256 and most groups never
//              touch O.
//   warp 8     V producer, warp 9 K producer: one TMA load per block and
//              64-column half into a ring of GS groups each (K laid out
//              [half][slot * 4 + block][16][64] so that a group is one 64-row
//              K-major operand per half; V [slot * 4 + block][half][16][64]).
//              A K slot is released by its group's Q.K^T and a V slot by its
//              P.V, so the next K loads start while the softmax still runs.
//   warp 10    TMEM allocator and MMA issuer: polls and issues whichever of
//              the next Q.K^T (its K landed and S is free) and the next P.V
//              (its P was written and its V landed) is ready.
// A warp's SM sub-partition is its index mod 4 and TMEM lane quarter q belongs
// to sub-partition q; up to 32 query rows (chain verify) only warps 0 and 4
// compute, and the K producer and the MMA issuer sit on sub-partitions 1 and
// 2, away from them: a single issuing thread slows down markedly when a busy
// warp shares its sub-partition.
// Two CTAs share an SM (one per sequence x KV head leaves most SMs with two),
// so each allocates only 256 TMEM columns: O [0, HD), S (one 64-column
// buffer, released by the softmax right after it is read) at 128, P (2 x 32)
// at 192.  The K / V streams start before the CTA loads its query tile and
// allocates TMEM.
// The query tile holds QROWS rows in shared memory: 128, or 32 when the tile
// has at most 32 rows (chain verify).  The M = 128 MMAs then read rows 32-127
// from the memory after the tile (the rings): those rows' S, P and O lanes are
// never read, and the 24 KB saved (HD = 128) deepen both rings to three
// groups, which the V stream needs: a V slot refills only after the P.V of the
// group before last, and its HBM latency under load exceeds two groups.
__host__ __device__ constexpr int tc_group_slots(int QROWS) { return QROWS == 32 ? 3 : 2; }
constexpr int kTcTmemCols = 256;
constexpr int kTcSoftWarps = 8;
constexpr int kTcVLoadWarp = 8, kTcKLoadWarp = 9, kTcMmaWarp = 10;
constexpr int kTcThreads = 32 * (kTcMmaWarp + 1);
constexpr uint32_t kTmemO = 0, kTmemS = 128, kTmemP = 192;

// 2^x on the special-function unit (2 ulp); the result is rounded to fp16 next.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Bit c = key key0 + c is visible: it exists (c < nkeys, key < L) and is a
// context key (key < ctx) or a new key whose bit is set in the row's mask.
__device__ __forceinline__ uint64_t group_visibility(int key0, int ctx, int L, int nkeys, uint64_t rmask) {
    auto low_bits = [](int k) -> uint64_t {  // bits [0, k), k clamped to [0, 64]
        return k <= 0 ? 0ull : (k >= 64 ? ~0ull : ((1ull << k) - 1ull));
    };
    const int d = key0 - ctx;  // new-key index of bit 0 (negative: the group starts in the context)
    uint64_t fresh = 0ull;     // bit c = mask bit d + c
    if (d >= 0) fresh = d < 64 ? (rmask >> d) : 0ull;
    else fresh = -d < 64 ? (rmask << (-d)) : 0ull;
    return (low_bits(ctx - key0) | fresh) & low_bits(L - key0) & low_bits(nkeys);
}

__host__ __device__ constexpr size_t attn_tc_smem_bytes(int HD, int QROWS, int max_per) {
    return 1024 + (size_t)(HD / 64) * QROWS * 128 /* Q */ +
           (size_t)4 * tc_group_slots(QROWS) * 2 * (HD / 64) * kBox /* K + V */ + (size_t)((max_per + 3) & ~3) * 4 +
           2 * 2 * 128 * 4 /* row max / sum exchange */ + (size_t)(4 * tc_group_slots(QROWS) + 12) * 8 + 16;
}

template <int HD, int QROWS>
__global__ void __launch_bounds__(kTcThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, AttnArgs a) {
    constexpr int NBOX = HD / 64;
    constexpr int GS = tc_group_slots(QROWS);  // groups of four blocks in flight per ring
    constexpr int ST = 4 * GS;                 // blocks per ring
    constexpr int QPANEL = QROWS * 128;        // one 64-column half of the query tile
    // the MMAs read 128 query rows: the rows past a 32-row tile lie in the rings
    static_assert(QROWS == 128 || (HD / 64) * QPANEL + (size_t)2 * ST * (HD / 64) * kBox >= (HD / 64) * 16384,
                  "rows past the query tile stay inside the CTA's shared memory");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sQ = base;                             // [NBOX][QROWS][128 B], swizzled K-major
    unsigned char* sK = sQ + NBOX * QPANEL;               // [NBOX][ST][16][128 B]
    unsigned char* sV = sK + (size_t)NBOX * ST * kBox;    // [ST][NBOX][16][128 B]
    int* tbl = reinterpret_cast<int*>(sV + (size_t)ST * NBOX * kBox);
    float* xch = reinterpret_cast<float*>(tbl + ((a.max_per + 3) & ~3));  // [2 phases][2 halves][128 lanes]
    uint64_t* k_full = reinterpret_cast<uint64_t*>(xch + 2 * 2 * 128);
    uint64_t* k_empty = k_full + GS;
    uint64_t* v_full = k_empty + GS;
    uint64_t* v_empty = v_full + GS;
    uint64_t* s_full = v_empty + GS;  // Q.K^T of a group landed in S
    uint64_t* s_free = s_full + 1;    // the softmax read S (8 warps)
    uint64_t* p_full = s_free + 1;    // [2] softmax wrote P[g%2] (8 warps)
    uint64_t* pv_done = p_full + 2;   // [2] P.V of a group finished
    uint64_t* o_final = pv_done + 2;
    uint64_t* xbar = o_final + 1;     // [4] the two softmax warps of a lane quarter posted their values
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    pdl_trigger();  // a following GEMM may start streaming its weights
    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31;
    const int S = a.S;
    const int split = S > 1 ? (int)cluster_rank() : 0;
    // cluster = (pair, 128-row tile of the query rows); a.MT = number of row tiles
    const int pair = (blockIdx.x / S) / a.MT, mtile = (blockIdx.x / S) % a.MT;
    const int b = pair / a.Hkv, kvh = pair % a.Hkv;
    const int row0 = mtile * 128;                      // first query row of this tile
    const int QR = min(128, a.QR - row0);              // rows of this tile
    const int ctx = a.ctx_len[b];
    const int L = ctx + a.R;
    const int nb = min((L + 15) / 16, a.max_blocks);
    const int per = (nb + S - 1) / S;
    const int blo = min(nb, split * per), bhi = min(nb, blo + per);
    const int n = min(bhi - blo, a.max_per);
    const int ngroups = (n + 3) / 4;

    // block table slice and barriers first: the producers start streaming K and
    // V right after the first block-wide barrier
    for (int i = threadIdx.x; i < n; i += blockDim.x) tbl[i] = a.tables[(size_t)b * a.max_blocks + blo + i];
    if (threadIdx.x == 0) {
        for (int i = 0; i < GS; ++i) {
            mbar_init(s_addr(&k_full[i]), 1);
            mbar_init(s_addr(&k_empty[i]), 1);
            mbar_init(s_addr(&v_full[i]), 1);
            mbar_init(s_addr(&v_empty[i]), 1);
        }
        mbar_init(s_addr(s_full), 1);
        mbar_init(s_addr(s_free), kTcSoftWarps);
        for (int i = 0; i < 2; ++i) {
            mbar_init(s_addr(&p_full[i]), kTcSoftWarps);
            mbar_init(s_addr(&pv_done[i]), 1);
        }
        mbar_init(s_addr(o_final), 1);
        for (int i = 0; i < 4; ++i) mbar_init(s_addr(&xbar[i]), 2);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int quarter = warp & 3;
    const int half = (warp >> 2) & 1;                  // softmax warps: key half of every group
    const int qi = quarter * 32 + lane;                // softmax warps: this thread's query row (TMEM lane)
    const bool soft = warp < kTcSoftWarps;
    const bool rows_here = soft && quarter * 32 < QR;  // warp holds at least one real row
    float m_used = -INFINITY, l_sum = 0.f;             // l_sum: this half's keys
    uint32_t tmem = 0;
    // Exchange k of a value with the other key half of the row (same lane, the
    // quarter's other softmax warp): each posts into buffer k % 2 and arrives;
    // the barrier's phase k completes when both have.  A buffer is rewritten
    // two exchanges later, after the partner's arrival for the exchange in
    // between, i.e. after it has read.  Bounded: false on timeout.
    auto exchange = [&](int k, float& v) -> bool {
        float* xb = xch + (k & 1) * 256;
        xb[half * 128 + qi] = v;
        __syncwarp();
        if (lane == 0) mbar_arrive(s_addr(&xbar[quarter]));
        const bool ok = __all_sync(0xffffffffu, mbar_wait(s_addr(&xbar[quarter]), (uint32_t)k & 1u));
        if (ok) v = xb[(half ^ 1) * 128 + qi];
        return ok;
    };

    if (warp == kTcKLoadWarp || warp == kTcVLoadWarp) {
        // ------------------------------------------------ K / V producer, one group per wait
        const bool is_k = warp == kTcKLoadWarp;
        uint64_t* fullb = is_k ? k_full : v_full;
        uint64_t* emptyb = is_k ? k_empty : v_empty;
        bool ok = true;
        int g = 0;
        for (; g < ngroups; ++g) {
            const int slot = g % GS;
            if (g >= GS) ok = mbar_wait(s_addr(&emptyb[slot]), ((g / GS) - 1) & 1);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) break;
            if (lane == 0) {
                const int nbg = min(4, n - 4 * g);
                const uint32_t fb = s_addr(&fullb[slot]);
                mbar_expect_tx(fb, (uint32_t)(nbg * NBOX * kBox));
                for (int i = 0; i < nbg; ++i) {
                    int phys = tbl[4 * g + i];
                    if (phys < 0 || phys >= a.num_blocks) phys = 0;  // a malformed table reads block 0, never out of range
                    const int s = slot * 4 + i;
                    if (is_k) {
#pragma unroll
                        for (int hb = 0; hb < NBOX; ++hb)
                            tma_load_5d(s_addr(sK + ((size_t)hb * ST + s) * kBox), &kmap, 0, kvh * 16, hb, 0, phys, fb);
                    } else {
                        tma_load_5d(s_addr(sV + (size_t)s * NBOX * kBox), &vmap, 0, kvh * 16, 0, 1, phys, fb);
                    }
                }
            }
            __syncwarp();
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            record_timeout(a.status, 13);
        }
        // the loads issued above land before the CTA exits
        if (g > 0) (void)mbar_wait(s_addr(&fullb[(g - 1) % GS]), ((g - 1) / GS) & 1);
    } else {
        // ------------------------------------------------ query tile and TMEM (warps 0-7 and 10)
        if (soft) {
            // rows row0 + qi = r * G + g (zero past QR), in the 128B-swizzled K-major layout
            for (int idx = threadIdx.x; idx < QROWS * (HD / 8); idx += 32 * kTcSoftWarps) {
                const int r_i = idx / (HD / 8), c8 = idx % (HD / 8);
                uint4 v = make_uint4(0, 0, 0, 0);
                if (r_i < QR) {
                    const int r = (row0 + r_i) / a.G, g = (row0 + r_i) % a.G;
                    v = *reinterpret_cast<const uint4*>(a.q + (((size_t)(b * a.R + r) * a.Hq) + kvh * a.G + g) * HD +
                                                        c8 * 8);
                }
                *reinterpret_cast<uint4*>(sQ + (c8 >> 3) * QPANEL + r_i * 128 + (((c8 & 7) ^ (r_i & 7)) << 4)) = v;
            }
            fence_async_smem();  // Q is read by the tensor cores (async proxy)
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_addr(tmem_slot)),
                         "r"(kTcTmemCols));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
        tc_fence_before();
        asm volatile("bar.sync 1, %0;" ::"r"(32 * (kTcSoftWarps + 1)) : "memory");  // warps 0-7 and 10
        tc_fence_after();
        tmem = __shfl_sync(0xffffffffu, *tmem_slot, 0);

        if (warp == kTcMmaWarp) {
            // ------------------------------------------------ MMA issuer
            // Polls with test_wait: a try_wait on a barrier that is not ready
            // may suspend the thread while the other operation is ready.
            const uint32_t qb = s_addr(sQ), kb = s_addr(sK), vb = s_addr(sV);
            bool ok = true, timed_out = false;
            int gq = 0, gp = 0;
            uint64_t t_idle = 0;
            while (gp < ngroups) {
                bool progressed = false;
                if (gq < ngroups && gq <= gp + 1) {
                    const bool ready = mbar_test(s_addr(&k_full[gq % GS]), (gq / GS) & 1) &&
                                       (gq == 0 || mbar_test(s_addr(s_free), (gq - 1) & 1));
                    if (__all_sync(0xffffffffu, ready)) {
                        tc_fence_after();
                        if (lane == 0) {
                            const int nbg = min(4, n - 4 * gq);
                            const int st0 = (gq % GS) * 4;
                            const uint32_t idesc = idesc_f16(128, 16 * nbg);
#pragma unroll
                            for (int kk = 0; kk < HD / 16; ++kk)
                                tc_mma_f16_ss(tmem + kTmemS,
                                              sw128_desc(qb + (uint32_t)((kk >> 2) * QPANEL + (kk & 3) * 32)),
                                              sw128_desc(kb + (uint32_t)(((kk >> 2) * ST + st0) * kBox + (kk & 3) * 32)),
                                              idesc, kk > 0 ? 1u : 0u);
                            tc_commit(s_addr(s_full));
                            tc_commit(s_addr(&k_empty[gq % GS]));
                        }
                        __syncwarp();
                        ++gq;
                        progressed = true;
                    }
                }
                if (gp < gq) {
                    const bool ready = mbar_test(s_addr(&p_full[gp & 1]), (gp >> 1) & 1) &&
                                       mbar_test(s_addr(&v_full[gp % GS]), (gp / GS) & 1);
                    if (__all_sync(0xffffffffu, ready)) {
                        tc_fence_after();
                        if (lane == 0) {
                            const int nbg = min(4, n - 4 * gp);
                            for (int i = 0; i < nbg; ++i) {
                                const int s = (gp % GS) * 4 + i;
                                tc_mma_f16_ts(tmem + kTmemO, tmem + kTmemP + (uint32_t)((gp & 1) * 32 + i * 8),
                                              sw128_mn_desc(vb + (uint32_t)(s * NBOX * kBox), kBox, 1024),
                                              idesc_f16_bmn(128, HD), (gp > 0 || i > 0) ? 1u : 0u);
                            }
                            tc_commit(s_addr(&pv_done[gp & 1]));
                            tc_commit(s_addr(&v_empty[gp % GS]));
                        }
                        __syncwarp();
                        ++gp;
                        progressed = true;
                    }
                }
                if (progressed) {
                    t_idle = 0;
                } else {
                    // bounded: give up after ~2 s without progress
                    const uint64_t now = gtimer();
                    if (t_idle == 0) t_idle = now;
                    timed_out = __any_sync(0xffffffffu, now - t_idle > 2000000000ull);
                    if (timed_out || __any_sync(0xffffffffu, *abort_flag != 0)) {
                        ok = false;
                        break;
                    }
                }
            }
            if (lane == 0) {
                if (ok) tc_commit(s_addr(o_final));
                else {
                    *abort_flag = 1;
                    if (timed_out) record_timeout(a.status, 14);
                    mbar_arrive(s_addr(o_final));  // release the softmax warps' final wait
                }
            }
        } else {
            // ------------------------------------------------ softmax, one thread per (query row, key half)
            const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
            const uint64_t rmask = qi < QR ? a.mask[(row0 + qi) / a.G] : ~0ull;
            bool ok = true;
            for (int g = 0; g < ngroups; ++g) {
                ok = __all_sync(0xffffffffu, mbar_wait(s_addr(s_full), g & 1));
                if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) break;
                tc_fence_after();
                if (!rows_here) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_addr(s_free));
                } else {
                    uint32_t sv[32];
                    tc_ld_x32(t_lane + kTmemS + (uint32_t)(half * 32), sv);
                    tc_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_addr(s_free));  // S may be overwritten by the next Q.K^T
                    const int nkeys = 16 * min(4, n - 4 * g);
                    const int key0 = (blo + 4 * g) * 16;
                    // visibility of the group's 64 keys as one word: context keys,
                    // then the new keys this row may see, cut at L and at the group end
                    const uint32_t vis = (uint32_t)(group_visibility(key0, ctx, L, nkeys, rmask) >> (32 * half));
                    float mx = -INFINITY;
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const float x = ((vis >> c) & 1u) ? __uint_as_float(sv[c]) * a.scale_log2 : -INFINITY;
                        sv[c] = __float_as_uint(x);
                        mx = fmaxf(mx, x);
                    }
                    // the row max over both key halves
                    float mo = mx;
                    ok = exchange(g, mo);
                    if (!ok) break;
                    mx = fmaxf(mx, mo);
                    const bool grow = mx > m_used + 8.0f;  // also when the row had no visible key yet
                    const float m_new = grow ? mx : m_used;
                    const float alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - m_new);
                    const float muse = m_new == -INFINITY ? 0.f : m_new;
                    uint32_t pw[16];
                    float sum = 0.f;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const __half2 h = __floats2half2_rn(ex2_approx(__uint_as_float(sv[2 * j]) - muse),
                                                            ex2_approx(__uint_as_float(sv[2 * j + 1]) - muse));
                        sum += __low2float(h) + __high2float(h);
                        pw[j] = *reinterpret_cast<const uint32_t*>(&h);
                    }
                    // P[g%2] was last read by P.V of group g-2
                    if (g >= 2) ok = mbar_wait(s_addr(&pv_done[g & 1]), ((g - 2) >> 1) & 1);
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) break;
                    tc_fence_after();
                    tc_st_x16(t_lane + kTmemP + (uint32_t)((g & 1) * 32 + half * 16), pw);
                    // O holds groups < g; rescale this half's O columns once P.V of group g-1 has landed
                    if (g > 0 && __any_sync(0xffffffffu, grow && m_used != -INFINITY)) {
                        ok = __all_sync(0xffffffffu, mbar_wait(s_addr(&pv_done[(g - 1) & 1]), ((g - 1) >> 1) & 1));
                        if (!ok) break;
                        tc_fence_after();
#pragma unroll
                        for (int c0 = half * (HD / 2); c0 < (half + 1) * (HD / 2); c0 += 32) {
                            uint32_t ov[32];
                            tc_ld_x32(t_lane + kTmemO + (uint32_t)c0, ov);
                            tc_wait_ld();
#pragma unroll
                            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                            tc_st_x32(t_lane + kTmemO + (uint32_t)c0, ov);
                        }
                    }
                    l_sum = l_sum * alpha + sum;
                    m_used = m_new;
                    tc_wait_st();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_addr(&p_full[g & 1]));
            }
            if (!ok && lane == 0) {
                *abort_flag = 1;
                record_timeout(a.status, 15);
            }
            // every MMA has finished (and read its shared-memory operands) after this
            (void)__all_sync(0xffffffffu, mbar_wait(s_addr(o_final), 0));
            tc_fence_after();
            // the row's sum over both key halves
            if (rows_here && ok) {
                float lo = l_sum;
                if (exchange(ngroups, lo)) l_sum += lo;
                else if (lane == 0) {
                    *abort_flag = 1;
                    record_timeout(a.status, 16);
                }
            }
        }
    }
    __syncthreads();  // the Q tile and the rings are free from here on

    // ---- output: this CTA's O rows (each softmax warp half of the columns);
    // one CTA writes, a cluster merges through DSMEM
    float* pO = reinterpret_cast<float*>(base);  // [128][HD]
    float* pML = pO + 128 * HD;                  // [128][2] = (m, l)
    const bool valid = !*abort_flag;
    if (rows_here && valid) {
#pragma unroll 1
        for (int c0 = half * (HD / 2); c0 < (half + 1) * (HD / 2); c0 += 32) {
            uint32_t ov[32];
            tc_ld_x32(tmem + ((uint32_t)(quarter * 32) << 16) + kTmemO + (uint32_t)c0, ov);
            tc_wait_ld();
            if (qi < QR) {
                if (S == 1) {
                    const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
                    const int r = (row0 + qi) / a.G, g = (row0 + qi) % a.G;
                    __half* dst = a.out + (((size_t)(b * a.R + r) * a.Hq) + kvh * a.G + g) * HD + c0;
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        uint4 w;
                        uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const float x0 = n > 0 ? __uint_as_float(ov[e + 2 * k]) * inv : 0.f;
                            const float x1 = n > 0 ? __uint_as_float(ov[e + 2 * k + 1]) * inv : 0.f;
                            const __half2 h = __floats2half2_rn(x0, x1);
                            wp[k] = *reinterpret_cast<const uint32_t*>(&h);
                        }
                        *reinterpret_cast<uint4*>(dst + e) = w;
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) pO[(size_t)qi * HD + c0 + e] = n > 0 ? __uint_as_float(ov[e]) : 0.f;
                }
            }
        }
        if (S > 1 && half == 0 && qi < QR) {
            pML[qi * 2 + 0] = m_used;
            pML[qi * 2 + 1] = l_sum;
        }
    }
    if (S > 1) {
        __syncthreads();
        cluster_sync_all();
        const int r0 = split * QR / S, r1 = (split + 1) * QR / S;
        if (valid) {
            for (int idx = threadIdx.x; idx < (r1 - r0) * HD; idx += blockDim.x) {
                const int row = r0 + idx / HD, col = idx % HD;
                const uint32_t aM = s_addr(pML + row * 2), aO = s_addr(pO + (size_t)row * HD + col);
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
                const int r = (row0 + row) / a.G, g = (row0 + row) % a.G;
                a.out[(((size_t)(b * a.R + r) * a.Hq) + kvh * a.G + g) * HD + col] =
                    __float2half_rn(l > 0.f ? acc / l : 0.f);
            }
        }
        cluster_sync_all();  // peers keep their partials until every rank has read them
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols));
    }
}

// ------------------------------------------------------------ host side
struct AttnPlan {
    int MT, KG, QRP, threads, S, ST, max_per;
    size_t smem;
};

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
// `halves` / `kvs` = how many column halves / K|V planes one box spans.
static int make_kv_tmap(CUtensorMap* map, const __half* kv, int num_blocks, int Hkv, int HD, int halves = -1,
                        int kvs = 2) {
    if (halves < 0) halves = HD / 64;
    auto enc = attn_encode();
    SD_CHECK(enc, SPECDEC_ENOTSUP, "cuTensorMapEncodeTiled unavailable");
    SD_CHECK((reinterpret_cast<uintptr_t>(kv) & 15) == 0, SPECDEC_EINVAL, "attention: KV pool must be 16-byte aligned");
    const cuuint64_t row = (cuuint64_t)HD * 2, head_block = row * 16 * Hkv;
    cuuint64_t dims[5] = {64, (cuuint64_t)Hkv * 16, (cuuint64_t)(HD / 64), 2, (cuuint64_t)num_blocks};
    cuuint64_t strides[4] = {row, 128, head_block, 2 * head_block};
    cuuint32_t box[5] = {64, 16, (cuuint32_t)halves, (cuuint32_t)kvs, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<__half*>(kv), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SD_CHECK(r == CUDA_SUCCESS, SPECDEC_EINVAL, "attention: cuTensorMapEncodeTiled failed");
    return SPECDEC_OK;
}

// The kernel needs no global workspace (splits are merged on chip).
size_t attention_workspace(int, int, int, int, int, int) { return 0; }

static const void* attn_tc_fn(int HD, int QROWS) {
    if (HD == 128)
        return QROWS == 32 ? reinterpret_cast<const void*>(attn_tc_kernel<128, 32>)
                           : reinterpret_cast<const void*>(attn_tc_kernel<128, 128>);
    return QROWS == 32 ? reinterpret_cast<const void*>(attn_tc_kernel<64, 32>)
                       : reinterpret_cast<const void*>(attn_tc_kernel<64, 128>);
}

// tcgen05 variant: split count from the same cost model as the legacy kernel.
static AttnPlan plan_attention_tc(int B, int R, int Hkv, int HD, int max_ctx, int QROWS) {
    AttnPlan p;
    p.MT = 8;
    p.KG = 1;
    p.QRP = QROWS;
    p.threads = kTcThreads;
    p.ST = 4 * tc_group_slots(QROWS);
    const int nb_max = (max_ctx + R + 15) / 16;
    const int pairs = B * Hkv;
    static bool opted[4] = {false, false, false, false};
    const int vi = (HD == 128 ? 2 : 0) + (QROWS == 32 ? 1 : 0);
    if (!opted[vi]) {
        int dev = 0, optin = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaFuncSetAttribute(attn_tc_fn(HD, QROWS), cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
        opted[vi] = true;
    }
    p.S = 1;
    long long best_cost = -1;
    for (int S = 1; S <= 8 && S <= nb_max; ++S) {
        const int per = (nb_max + S - 1) / S;
        const size_t sm = attn_tc_smem_bytes(HD, QROWS, per);
        int clusters = 0;
        {
            static std::mutex mu;
            static std::map<std::tuple<int, size_t, int>, int> cache;
            std::lock_guard<std::mutex> lk(mu);
            auto key = std::make_tuple(HD * 1000 + QROWS, sm, S);
            auto it = cache.find(key);
            if (it != cache.end()) {
                clusters = it->second;
            } else {
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3((unsigned)(S * 148));
                cfg.blockDim = dim3(kTcThreads);
                cfg.dynamicSmemBytes = sm;
                cudaLaunchAttribute at[1];
                at[0].id = cudaLaunchAttributeClusterDimension;
                at[0].val.clusterDim.x = (unsigned)S;
                at[0].val.clusterDim.y = 1;
                at[0].val.clusterDim.z = 1;
                cfg.attrs = at;
                cfg.numAttrs = 1;
                if (cudaOccupancyMaxActiveClusters(&clusters, attn_tc_fn(HD, QROWS), &cfg) != cudaSuccess) {
                    cudaGetLastError();
                    clusters = 0;
                }
                if (clusters <= 0) clusters = 148 / S > 0 ? 148 / S : 1;
                cache[key] = clusters;
            }
        }
        const long long waves = (pairs + clusters - 1) / clusters;
        const long long cost = waves * (per + 48);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            p.S = S;
        }
    }
    p.max_per = (nb_max + p.S - 1) / p.S;
    p.smem = attn_tc_smem_bytes(HD, QROWS, p.max_per);
    return p;
}

int launch_attention(const __half* q, const __half* kv_layer, int num_blocks, int Hkv, int HD, const int32_t* tables,
                     int max_blocks, const int32_t* ctx_len, const uint64_t* mask, int B, int R, int Hq, __half* out,
                     void* ws, size_t ws_bytes, int max_ctx, cudaStream_t s) {
    (void)ws;
    (void)ws_bytes;
    SD_CHECK(HD == 64 || HD == 128, SPECDEC_EINVAL, "attention: head_dim must be 64 or 128");
    SD_CHECK(Hkv > 0 && Hq % Hkv == 0 && R >= 1 && R <= 64, SPECDEC_EINVAL, "attention: bad head / row counts");
    SD_CHECK(num_blocks > 0 && max_blocks > 0, SPECDEC_EINVAL, "attention: empty block pool or table");
    // the tcgen05 kernel, one CTA (cluster) per 128 query rows
    const int mtiles = (R * (Hq / Hkv) + 127) / 128;
    const int qrows = R * (Hq / Hkv) <= 32 ? 32 : 128;  // query rows the tile stores
    AttnPlan p = plan_attention_tc(B * mtiles, R, Hkv, HD, max_ctx, qrows);
    CUtensorMap kmap, vmap;
    int rc = make_kv_tmap(&kmap, kv_layer, num_blocks, Hkv, HD, 1, 1);
    if (!rc) rc = make_kv_tmap(&vmap, kv_layer, num_blocks, Hkv, HD, HD / 64, 1);
    if (rc) return rc;
    AttnArgs a = {};
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
    a.MT = mtiles;
    a.KG = p.KG;
    a.S = p.S;
    a.ST = p.ST;
    a.max_per = p.max_per;
    a.out = out;
    a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)HD));
    a.status = device_status_ptr();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(B * Hkv * mtiles * p.S));
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
    if (HD == 128 && qrows == 32) SD_CUDA(cudaLaunchKernelEx(&cfg, attn_tc_kernel<128, 32>, kmap, vmap, a));
    else if (HD == 128) SD_CUDA(cudaLaunchKernelEx(&cfg, attn_tc_kernel<128, 128>, kmap, vmap, a));
    else if (qrows == 32) SD_CUDA(cudaLaunchKernelEx(&cfg, attn_tc_kernel<64, 32>, kmap, vmap, a));
    else SD_CUDA(cudaLaunchKernelEx(&cfg, attn_tc_kernel<64, 128>, kmap, vmap, a));
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
