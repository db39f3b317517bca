// sampling.cu -- fused acceptance / sampling kernels (sm_100a).
//
// Row statistics, rejection-sampling acceptance (min(1, p/q) test, residual
// max(0, p - q) redraw, bonus token), tree acceptance, draft sampling, top-k,
// and the reference-compatible greedy verify (lib.rs:696-779).
//
// Every decision is taken on exact integers: a token's probability mass is
// E_j = floor(2^((z_j - max) * log2(e) / T) * 2^31) (deterministic exp2), sums
// are integer, the min(1, p/q) test and the residual are integer
// cross-multiplications, so the result does not depend on reduction order.
// Draws (draft tokens, the residual / bonus token, the tree's fallback) are
// arg-maxes of per-element race keys (gumbel.cuh), merged as (key desc, index
// asc), which is order-independent as well.
#include <cfloat>
#include <climits>
#include <mutex>

#include "common.cuh"
#include "gumbel.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace specdec {

struct DevRowStats {
    float max;
    uint32_t tau;
    uint64_t sum;
    uint64_t nuc;
    int32_t argmax;
    int32_t pad;
};
static_assert(sizeof(DevRowStats) == kAcceptStatsBytes, "row stats layout");

constexpr int kRowThreads = 1024;
// The top-p histograms of a row keep one per warp of 16-bit mass halves: a warp
// sees at most 8192 elements of a row (32 warps), which bounds V.
constexpr int kMaxVocab = 262144;

struct RowSmem {
    uint64_t hist[256];
    uint64_t red64[32];
    float redf[32];
    int redi[32];
    DevRowStats st;
};

__device__ __forceinline__ uint32_t mass_of(float z, float m, float c) {
    return exp2_fx31(__fmul_rn(__fsub_rn(z, m), c));
}

// (value desc, index asc) arg-max reduction; NaN never wins.
__device__ __forceinline__ void argmax_merge(float& v, int& i, float v2, int i2) {
    if (i2 < 0) return;
    if (i < 0 || v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

__device__ void cta_argmax(const float* __restrict__ z, int V, RowSmem& sm, float* out_max, int* out_idx) {
    float bv = -INFINITY;
    int bi = -1;
    // each thread visits its indices in increasing order: strict > keeps the first of equal values
    auto upd = [&](float v, int j) {
        if (v > bv || (bi < 0 && v == bv)) {
            bv = v;
            bi = j;
        }
    };
    if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(z) & 15) == 0) {
        // four float4 loads in flight per thread; indices still visited in increasing order
        const float4* z4 = reinterpret_cast<const float4*>(z);
        const int n4 = V / 4, bd = blockDim.x;
        int q = threadIdx.x;
        for (; q + 3 * bd < n4; q += 4 * bd) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = z4[q + u * bd];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = 4 * (q + u * bd);
                upd(v[u].x, j);
                upd(v[u].y, j + 1);
                upd(v[u].z, j + 2);
                upd(v[u].w, j + 3);
            }
        }
        for (; q < n4; q += bd) {
            const float4 v = z4[q];
            upd(v.x, 4 * q);
            upd(v.y, 4 * q + 1);
            upd(v.z, 4 * q + 2);
            upd(v.w, 4 * q + 3);
        }
    } else {
        for (int j = threadIdx.x; j < V; j += blockDim.x) upd(z[j], j);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, v2, i2);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) {
        sm.redf[wid] = bv;
        sm.redi[wid] = bi;
    }
    __syncthreads();
    if (wid == 0) {
        bv = lane < nw ? sm.redf[lane] : -INFINITY;
        bi = lane < nw ? sm.redi[lane] : -1;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(bv, bi, v2, i2);
        }
        if (lane == 0) {
            sm.redf[0] = bv;
            sm.redi[0] = bi;
        }
    }
    __syncthreads();
    *out_max = sm.redf[0];
    *out_idx = sm.redi[0];
    __syncthreads();
}

// Row maximum only (NaN never wins; -inf for an empty or all-NaN row): one
// max per element, four float4 loads in flight per thread.  *finite (if
// given) tells whether every value is finite (sum of v * 0 stays a zero).
__device__ float cta_max(const float* __restrict__ z, int V, RowSmem& sm, bool* finite = nullptr) {
    float bv = -INFINITY, nz = 0.0f;
    if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(z) & 15) == 0) {
        const float4* z4 = reinterpret_cast<const float4*>(z);
        const int n4 = V / 4, bd = blockDim.x;
        int q = threadIdx.x;
        // eight float4 loads in flight per thread: the row comes from HBM
        for (; q + 7 * bd < n4; q += 8 * bd) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = z4[q + u * bd];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                bv = fmaxf(bv, fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w)));
                if (finite) nz = __fmaf_rn(v[u].x, 0.0f, __fmaf_rn(v[u].y, 0.0f, __fmaf_rn(v[u].z, 0.0f, __fmaf_rn(v[u].w, 0.0f, nz))));
            }
        }
        for (; q < n4; q += bd) {
            const float4 v = z4[q];
            bv = fmaxf(bv, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
            if (finite) nz = __fmaf_rn(v.x, 0.0f, __fmaf_rn(v.y, 0.0f, __fmaf_rn(v.z, 0.0f, __fmaf_rn(v.w, 0.0f, nz))));
        }
    } else {
        for (int j = threadIdx.x; j < V; j += blockDim.x) {
            const float v = z[j];
            bv = fmaxf(bv, v);
            if (finite) nz = __fmaf_rn(v, 0.0f, nz);
        }
    }
    if (finite) *finite = __syncthreads_and(nz == 0.0f);
    bv = warp_max(bv);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) sm.redf[wid] = bv;
    __syncthreads();
    float r = lane < nw ? sm.redf[lane] : -INFINITY;
    r = warp_max(r);
    __syncthreads();
    return r;
}

// Calls f(z_j) for every element of the row z[0, V) once, in no particular
// order: four float4 loads in flight per thread when z is 16-byte aligned and
// V a multiple of 4, else one element per thread and iteration.
template <class F>
__device__ __forceinline__ void for_each_row_value(const float* __restrict__ z, int V, F f) {
    if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(z) & 15) == 0) {
        const float4* z4 = reinterpret_cast<const float4*>(z);
        const int n4 = V / 4, bd = blockDim.x;
        int q = threadIdx.x;
        for (; q + 3 * bd < n4; q += 4 * bd) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = z4[q + u * bd];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                f(v[u].x);
                f(v[u].y);
                f(v[u].z);
                f(v[u].w);
            }
        }
        for (; q < n4; q += bd) {
            const float4 v = z4[q];
            f(v.x);
            f(v.y);
            f(v.z);
            f(v.w);
        }
    } else {
        for (int j = threadIdx.x; j < V; j += blockDim.x) f(z[j]);
    }
}

// Per-warp mass histograms for the top-p radix select: warp w owns
// whist[w][0][256] (the low 16 bits of each mass) and whist[w][1][256] (the
// high bits), updated by 32-bit shared-memory atomics from every lane (only
// lanes of the same warp contend).  A warp sees at most 8192 elements of a row
// (V <= 262144 over 32 warps), so the halves stay below 2^29 and 2^28 and the
// merge recombines them exactly.
__device__ __forceinline__ void hist_add_lane(uint32_t* Hw, uint32_t bin, uint32_t e) {
    if (e & 0xFFFFu) atomicAdd(&Hw[bin], e & 0xFFFFu);
    if (e >> 16) atomicAdd(&Hw[256 + bin], e >> 16);
}

// The per-warp histograms summed into sm.hist, then cleared for the next pass.
__device__ __forceinline__ void merge_warp_hists(uint32_t* whist, RowSmem& sm) {
    const int nw = blockDim.x >> 5;
    __syncthreads();
    for (int b = threadIdx.x; b < 256; b += blockDim.x) {
        uint64_t t = 0;
        for (int w = 0; w < nw; ++w) t += ((uint64_t)whist[w * 512 + 256 + b] << 16) + whist[w * 512 + b];
        sm.hist[b] = t;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nw * 512; i += blockDim.x) whist[i] = 0;
    __syncthreads();
}

// Warp 0 picks the highest digit whose cumulative mass (from the top) reaches thr.
__device__ void select_digit(RowSmem& sm, uint64_t thr, uint64_t* G, uint32_t* digit, uint64_t* last_bin) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        uint64_t local = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) local += sm.hist[255 - 8 * lane - i];
        uint64_t incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const uint64_t g0 = *G;
        const unsigned hit = __ballot_sync(0xffffffffu, g0 + incl >= thr);
        const int f = hit ? (__ffs(hit) - 1) : 31;
        if (lane == f) {
            uint64_t cum = g0 + incl - local;
            int chosen = 255 - 8 * f - 7;
            for (int i = 0; i < 8; ++i) {
                const int bin = 255 - 8 * f - i;
                if (cum + sm.hist[bin] >= thr) {
                    chosen = bin;
                    break;
                }
                cum += sm.hist[bin];
            }
            sm.red64[0] = cum;
            sm.red64[1] = sm.hist[chosen];
            sm.redi[0] = chosen;
        }
    }
    __syncthreads();
    *G = sm.red64[0];
    *last_bin = sm.red64[1];
    *digit = (uint32_t)sm.redi[0];
    __syncthreads();
}

// Integer mass sum over z[0, n) (no nucleus): four float4 loads in flight per
// thread when z is 16-byte aligned and n a multiple of 4.
__device__ uint64_t cta_mass_sum(const float* __restrict__ z, int n, float m, float c, RowSmem& sm) {
    uint64_t s = 0;
    if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(z) & 15) == 0) {
        const float4* z4 = reinterpret_cast<const float4*>(z);
        const int n4 = n / 4, bd = blockDim.x;
        int q = threadIdx.x;
        for (; q + 3 * bd < n4; q += 4 * bd) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = z4[q + u * bd];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                s += (uint64_t)mass_of(v[u].x, m, c) + mass_of(v[u].y, m, c) + mass_of(v[u].z, m, c) +
                     mass_of(v[u].w, m, c);
        }
        for (; q < n4; q += bd) {
            const float4 v = z4[q];
            s += (uint64_t)mass_of(v.x, m, c) + mass_of(v.y, m, c) + mass_of(v.z, m, c) + mass_of(v.w, m, c);
        }
    } else {
        for (int j = threadIdx.x; j < n; j += blockDim.x) s += mass_of(z[j], m, c);
    }
    return block_sum<uint64_t>(s, sm.red64);
}

// Full row statistics (max, argmax, mass sum, top-p threshold, nucleus mass).
//
// The top-p threshold tau is the largest logit key with
// sum_{key >= tau} E >= thr, thr = max(1, floor(S * top_p)).  Two passes over
// the row in the common case: the arg-max pass, then one pass that sums the
// masses and lists the elements whose exponent t = (z - max) * c is at least
// kTList (mass >= 2^kTList of the maximum's) as (key, mass) pairs.  When the
// list holds all of them (at most kNucleusList) and its mass reaches thr, the
// threshold lies among the listed elements -- every element with a larger key
// has a larger t and is listed too -- and a 4-digit radix select over the
// list (8 bits per digit, mass-weighted) finds it.  Otherwise (flat rows whose
// nucleus reaches below kTList, NaN logits) the radix select runs over the
// whole row: the first digit from a row pass into per-warp histograms (the
// 16-bit halves of each mass, only lanes of one warp contend), the second from
// another row pass that also lists the elements of the selected top digit, the
// last two from that list (or the row again when it overflowed).
// whist (only needed when tp < 2^32) holds the per-warp histograms
// ([warps][2][256] u32) and then the list.
constexpr int kNucleusList = 8192;
constexpr float kTList = -14.0f;
constexpr size_t kWarpHistWords = (size_t)(kRowThreads / 32) * 512;
constexpr size_t kWarpHistBytes = kWarpHistWords * sizeof(uint32_t) + (size_t)kNucleusList * sizeof(uint2) + 16;

// Mass-weighted radix select of tau over list[0, n) (every element with a key
// above tau is in the list): returns tau and the mass of the keys >= tau.
// Per-warp 32-bit histograms as in the row passes (the listed keys share their
// leading digits, so one shared histogram would serialise on a few bins).
__device__ void list_topp_select(const uint2* list, int n, uint64_t thr, RowSmem& sm, uint32_t* whist,
                                 uint32_t* tau, uint64_t* nuc) {
    uint32_t* Hw = whist + (threadIdx.x >> 5) * 512;
    for (int i = threadIdx.x; i < (int)(blockDim.x >> 5) * 512; i += blockDim.x) whist[i] = 0;
    __syncthreads();
    uint64_t G = 0, last = 0;
    uint32_t prefix = 0, dg = 0;
    for (int d = 3; d >= 0; --d) {
        const int shift = 8 * d;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint2 en = list[i];
            if (d == 3 || (en.x >> (shift + 8)) == (prefix >> (shift + 8))) hist_add_lane(Hw, (en.x >> shift) & 255u, en.y);
        }
        merge_warp_hists(whist, sm);
        select_digit(sm, thr, &G, &dg, &last);
        prefix |= dg << shift;
    }
    *tau = prefix;
    *nuc = G + last;
}

// The radix select over the whole row (see above); s = the row's mass sum.
__device__ void row_topp_select(const float* __restrict__ z, int V, float m, float c, uint64_t thr, RowSmem& sm,
                                uint32_t* whist, uint32_t* tau, uint64_t* nuc) {
    uint32_t* Hw = whist + (threadIdx.x >> 5) * 512;
    uint2* list = reinterpret_cast<uint2*>(whist + kWarpHistWords);
    int* list_n = reinterpret_cast<int*>(list + kNucleusList);
    for (int i = threadIdx.x; i < (int)(blockDim.x >> 5) * 512; i += blockDim.x) whist[i] = 0;
    if (threadIdx.x == 0) *list_n = 0;
    __syncthreads();
    for_each_row_value(z, V, [&](float zj) { hist_add_lane(Hw, logit_key(zj) >> 24, mass_of(zj, m, c)); });
    merge_warp_hists(whist, sm);
    uint64_t G = 0, last = 0;
    uint32_t prefix = 0, dg = 0;
    select_digit(sm, thr, &G, &dg, &last);
    prefix = dg << 24;
    for (int d = 2; d >= 0; --d) {
        const int shift = 8 * d;
        const uint32_t want = prefix >> (shift + 8);
        if (d == 2) {
            for_each_row_value(z, V, [&](float zj) {
                const uint32_t key = logit_key(zj);
                if ((key >> (shift + 8)) == want) {
                    const uint32_t e = mass_of(zj, m, c);
                    hist_add_lane(Hw, (key >> shift) & 255u, e);
                    const int at = atomicAdd(list_n, 1);
                    if (at < kNucleusList) list[at] = make_uint2(key, e);
                }
            });
        } else if (*list_n <= kNucleusList) {
            const int n = *list_n;
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const uint2 en = list[i];
                if ((en.x >> (shift + 8)) == want) hist_add_lane(Hw, (en.x >> shift) & 255u, en.y);
            }
        } else {
            for_each_row_value(z, V, [&](float zj) {
                const uint32_t key = logit_key(zj);
                if ((key >> (shift + 8)) == want) hist_add_lane(Hw, (key >> shift) & 255u, mass_of(zj, m, c));
            });
        }
        merge_warp_hists(whist, sm);
        select_digit(sm, thr, &G, &dg, &last);
        prefix |= dg << shift;
    }
    *tau = prefix;
    *nuc = G + last;
}

// need_mass: the sampling statistics (max, mass sum, top-p threshold and
// nucleus mass; argmax = -1); else the greedy statistics (max and argmax).
__device__ void cta_row_stats(const float* __restrict__ z, int V, float c, uint64_t tp, bool need_mass, RowSmem& sm,
                              DevRowStats* st, uint32_t* whist = nullptr) {
    float m;
    int am = -1;
    if (need_mass) {
        m = cta_max(z, V, sm);
    } else {
        cta_argmax(z, V, sm, &m, &am);
    }
    DevRowStats r;
    r.max = m;
    r.argmax = am;
    r.pad = 0;
    r.tau = 0;
    r.sum = 0;
    r.nuc = 0;
    if (need_mass) {
        const bool nucleus = tp < (1ull << 32);
        uint64_t s = 0;
        if (!nucleus) {
            s = cta_mass_sum(z, V, m, c, sm);
            r.sum = s;
            r.nuc = s;
        } else {
            uint2* list = reinterpret_cast<uint2*>(whist + kWarpHistWords);
            int* list_n = reinterpret_cast<int*>(list + kNucleusList);
            int* nan_seen = list_n + 1;  // a NaN exponent: NaN logits, or an infinite maximum
            if (threadIdx.x == 0) {
                *list_n = 0;
                *nan_seen = 0;
            }
            __syncthreads();
            uint64_t ls = 0;
            // the masses of a group of values first (independent, branch-free),
            // then the rare listing
            auto group = [&](const float* v, int nv) {
                float t[16];
                uint32_t e[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    if (u < nv) {
                        t[u] = __fmul_rn(__fsub_rn(v[u], m), c);
                        e[u] = exp2_fx31_neg(t[u]);  // t <= 0 or -inf; a NaN exponent: general path below
                        s += e[u];
                    }
                }
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    if (u < nv && !(t[u] < kTList)) {  // NaN exponents come here too
                        if (t[u] != t[u]) *nan_seen = 1;
                        ls += e[u];
                        const int at = atomicAdd(list_n, 1);
                        if (at < kNucleusList) list[at] = make_uint2(logit_key(v[u]), e[u]);
                    }
                }
            };
            if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(z) & 15) == 0) {
                const float4* z4 = reinterpret_cast<const float4*>(z);
                const int n4 = V / 4, bd = blockDim.x;
                int q = threadIdx.x;
                for (; q + 3 * bd < n4; q += 4 * bd) {
                    float v[16];
#pragma unroll
                    for (int u = 0; u < 4; ++u) *reinterpret_cast<float4*>(&v[4 * u]) = z4[q + u * bd];
                    group(v, 16);
                }
                for (; q < n4; q += bd) {
                    float v[16];
                    *reinterpret_cast<float4*>(&v[0]) = z4[q];
                    group(v, 4);
                }
            } else {
                for (int j = threadIdx.x; j < V; j += blockDim.x) {
                    float v[16];
                    v[0] = z[j];
                    group(v, 1);
                }
            }
            s = block_sum<uint64_t>(s, sm.red64);
            ls = block_sum<uint64_t>(ls, sm.red64);
            const int n = *list_n;
            const bool nan_row = *nan_seen != 0;
            __syncthreads();
            if (nan_row) {
                // exp2_fx31's handling of a NaN exponent (the pass above used the
                // finite-only form) and the keys' order decide: the general path.
                // -inf logits under a finite maximum stay on the list path: their
                // exponent is -inf, their mass 0 in both forms.
                s = cta_mass_sum(z, V, m, c, sm);
            }
            uint64_t thr = (uint64_t)(((u128)s * tp) >> 32);
            if (thr < 1) thr = 1;
            if (!nan_row && n <= kNucleusList && ls >= thr) {
                list_topp_select(list, n, thr, sm, whist, &r.tau, &r.nuc);
            } else {
                row_topp_select(z, V, m, c, thr, sm, whist, &r.tau, &r.nuc);
            }
            r.sum = s;
        }
    }
    *st = r;
}

__device__ __forceinline__ uint32_t nucleus_mass(const float* z, const DevRowStats& st, float c, int x) {
    const float zx = z[x];
    if (logit_key(zx) < st.tau) return 0u;
    return mass_of(zx, st.max, c);
}

// ------------------------------------------------------ Gumbel-max draws
// The CTA's best (score, index) of the per-thread candidates (every thread gets it).
__device__ void cta_best(float bs, int bj, RowSmem& sm, float* out_s, int* out_j) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float s2 = __shfl_xor_sync(0xffffffffu, bs, o);
        const int j2 = __shfl_xor_sync(0xffffffffu, bj, o);
        gumbel_merge(bs, bj, s2, j2);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) {
        sm.redf[wid] = bs;
        sm.redi[wid] = bj;
    }
    __syncthreads();
    if (wid == 0) {
        bs = lane < nw ? sm.redf[lane] : -INFINITY;
        bj = lane < nw ? sm.redi[lane] : -1;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float s2 = __shfl_xor_sync(0xffffffffu, bs, o);
            const int j2 = __shfl_xor_sync(0xffffffffu, bj, o);
            gumbel_merge(bs, bj, s2, j2);
        }
        if (lane == 0) {
            sm.redf[0] = bs;
            sm.redi[0] = bj;
        }
    }
    __syncthreads();
    *out_s = sm.redf[0];
    *out_j = sm.redi[0];
    __syncthreads();
}

// Visits the elements j of [L, H) in groups of four aligned on the element
// index (the draw's uniforms come four per Philox block): f(g, v[4], in[4])
// with the four values of group g (v = z[4g + e]) and which of them lie in
// [L, H).  One float4 load per group when z is 16-byte aligned and L, H are
// multiples of 4; element loads otherwise.
template <class F>
__device__ __forceinline__ void for_each_group(const float* __restrict__ z, int L, int H, F f) {
    const int g0 = L >> 2, g1 = (H + 3) >> 2;
    const bool vec = ((reinterpret_cast<uintptr_t>(z) & 15) == 0) && ((L & 3) == 0) && ((H & 3) == 0);
    for (int g = g0 + (int)threadIdx.x; g < g1; g += blockDim.x) {
        float v[4];
        bool in[4];
        if (vec) {
            const float4 q = reinterpret_cast<const float4*>(z)[g];
            v[0] = q.x;
            v[1] = q.y;
            v[2] = q.z;
            v[3] = q.w;
#pragma unroll
            for (int e = 0; e < 4; ++e) in[e] = true;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * g + e;
                in[e] = j >= L && j < H;
                v[e] = in[e] ? z[j] : 0.f;
            }
        }
        f(g, v, in);
    }
}

// Draw from the masses of row z over [L, H): candidates are the elements with
// key >= tau and mass E_j > 0, minus excl[0, nex); race key E_j / (-log2 U_j)
// with the uniforms of draw (seed, step, b, i, purpose) by element index (the
// oracle's orc_draw_row).  *sum (if given) receives the candidates' mass total.
__device__ void cta_gumbel_mass(const float* __restrict__ z, int L, int H, float m, float c, uint32_t tau,
                                const int* excl, int nex, uint64_t seed, uint32_t step, uint32_t b, uint32_t i,
                                uint32_t purpose, RowSmem& sm, float* out_s, int* out_j, uint64_t* sum = nullptr) {
    float bs = -INFINITY;
    int bj = -1;
    uint64_t tot = 0;
    for_each_group(z, L, H, [&](int g, const float* v, const bool* in) {
        uint32_t e4[4];
        bool any = false;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = 4 * g + e;
            uint32_t me = (in[e] && logit_key(v[e]) >= tau) ? mass_of(v[e], m, c) : 0u;
            for (int t = 0; t < nex; ++t)
                if (excl[t] == j) me = 0u;
            e4[e] = me;
            tot += me;
            any |= me != 0u;
        }
        if (!any) return;
        uint32_t o[4];
        gumbel_uniforms(seed, step, b, i, purpose, (uint32_t)g, o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (!e4[e]) continue;
            const float wf = __uint2float_rn(e4[e]);
            if (race_may_beat(wf, o[e], bs)) gumbel_merge(bs, bj, race_key(wf, o[e]), 4 * g + e);
        }
    });
    if (sum) *sum = block_sum<uint64_t>(tot, sm.red64);
    cta_best(bs, bj, sm, out_s, out_j);
}

// Draw from the residual max(0, E_p N_q - E_q N_p) of target row zp and draft
// row zq over [L, H) (nucleus masses at their row statistics; N = nucleus
// totals); race key residual / (-log2 U_j) (the oracle's draw_residual).  Index -1
// when the residual is zero everywhere in [L, H).
__device__ void cta_gumbel_resid(const float* __restrict__ zp, float pm, uint32_t pt, uint64_t Np,
                                 const float* __restrict__ zq, float qm, uint32_t qt, uint64_t Nq, int L, int H,
                                 float c, uint64_t seed, uint32_t step, uint32_t b, uint32_t i, RowSmem& sm,
                                 float* out_s, int* out_j) {
    float bs = -INFINITY;
    int bj = -1;
    const bool vec = ((reinterpret_cast<uintptr_t>(zq) & 15) == 0);
    for_each_group(zp, L, H, [&](int g, const float* vp, const bool* in) {
        float vq[4];
        if (vec && in[0] && in[3]) {
            const float4 q = reinterpret_cast<const float4*>(zq)[g];
            vq[0] = q.x;
            vq[1] = q.y;
            vq[2] = q.z;
            vq[3] = q.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) vq[e] = in[e] ? zq[4 * g + e] : 0.f;
        }
        u128 r4[4];
        bool any = false;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            r4[e] = 0;
            if (!in[e]) continue;
            const uint32_t ep = logit_key(vp[e]) >= pt ? mass_of(vp[e], pm, c) : 0u;
            const uint32_t eq = logit_key(vq[e]) >= qt ? mass_of(vq[e], qm, c) : 0u;
            const u128 x = (u128)ep * Nq, y = (u128)eq * Np;
            if (x > y) {
                r4[e] = x - y;
                any = true;
            }
        }
        if (!any) return;
        uint32_t o[4];
        gumbel_uniforms(seed, step, b, i, U_GUMBEL_RESAMPLE, (uint32_t)g, o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (!r4[e]) continue;
            const float wf = u128_to_f32(r4[e]);
            if (race_may_beat(wf, o[e], bs)) gumbel_merge(bs, bj, race_key(wf, o[e]), 4 * g + e);
        }
    });
    cta_best(bs, bj, sm, out_s, out_j);
}

// --------------------------------------------------------------- kernels
struct RowSet {
    const float* base;  // rows of length V, row r at base + r * V
    int rows;
};

__global__ void __launch_bounds__(kRowThreads) row_stats_kernel(RowSet a, RowSet b, int V, float c, uint64_t tp,
                                                                bool need_mass_a, bool need_mass_b,
                                                                DevRowStats* out) {
    __shared__ RowSmem sm;
    extern __shared__ uint32_t whist_dyn[];  // kWarpHistBytes when tp < 2^32
    const int r = blockIdx.x;
    const bool in_a = r < a.rows;
    const float* z = in_a ? a.base + (size_t)r * V : b.base + (size_t)(r - a.rows) * V;
    DevRowStats st;
    cta_row_stats(z, V, c, tp, in_a ? need_mass_a : need_mass_b, sm, &st, whist_dyn);
    if (threadIdx.x == 0) out[r] = st;
}

// One CTA per sequence: sequential min(1, p/q) tests over the draft positions,
// then the residual (or bonus) draw on the first rejected (or last) row.
__global__ void __launch_bounds__(kRowThreads) accept_chain_kernel(const float* __restrict__ target,
                                                                   const float* __restrict__ draft,
                                                                   const int32_t* __restrict__ drafts, int k, int V,
                                                                   float c, bool greedy, uint64_t seed, const uint32_t* step_dev, uint32_t step_host,
                                                                   const DevRowStats* __restrict__ stats, int B,
                                                                   int32_t* __restrict__ accepted_len,
                                                                   int32_t* __restrict__ out_tokens) {
    __shared__ RowSmem sm;
    const uint32_t step = step_dev ? *step_dev : step_host;
    const int b = blockIdx.x;
    const DevRowStats* sp = stats + (size_t)b * (k + 1);
    const DevRowStats* sq = stats + (size_t)B * (k + 1) + (size_t)b * k;
    const float* P = target + (size_t)b * (k + 1) * V;
    const float* Q = draft + (size_t)b * k * V;
    const int32_t* D = drafts + (size_t)b * k;
    if (threadIdx.x == 0) {
        int a = 0;
        if (greedy) {
            while (a < k && sp[a].argmax == D[a]) ++a;
        } else {
            while (a < k) {
                const int x = D[a];
                uint64_t ep = 0, eq = 0;
                if (x >= 0 && x < V) {
                    ep = nucleus_mass(P + (size_t)a * V, sp[a], c, x);
                    eq = nucleus_mass(Q + (size_t)a * V, sq[a], c, x);
                }
                const uint32_t u = uniform_u32(seed, step, (uint32_t)b, (uint32_t)a, U_ACCEPT);
                const u128 lhs = (u128)u * eq * sp[a].nuc;
                const u128 rhs = ((u128)ep * sq[a].nuc) << 32;
                if (!(lhs < rhs)) break;
                ++a;
            }
        }
        sm.redi[0] = a;
    }
    __syncthreads();
    const int a = sm.redi[0];
    __syncthreads();
    int tok;
    if (greedy) {
        tok = sp[a].argmax;
    } else {
        // the residual max(0, p - q) on the first rejected position, the bonus
        // token from p_k, and p itself where the residual is zero everywhere
        const float* zp = P + (size_t)a * V;
        const DevRowStats stp = sp[a];
        float sc;
        tok = -1;
        if (a < k) {
            const DevRowStats stq = sq[a];
            cta_gumbel_resid(zp, stp.max, stp.tau, stp.nuc, Q + (size_t)a * V, stq.max, stq.tau, stq.nuc, 0, V, c, seed,
                             step, (uint32_t)b, (uint32_t)a, sm, &sc, &tok);
        }
        if (tok < 0)
            cta_gumbel_mass(zp, 0, V, stp.max, c, stp.tau, nullptr, 0, seed, step, (uint32_t)b, (uint32_t)a,
                            U_GUMBEL_RESAMPLE, sm, &sc, &tok);
    }
    if (threadIdx.x == 0) {
        int32_t* out = out_tokens + (size_t)b * (k + 1);
        for (int i = 0; i < a; ++i) out[i] = D[i];
        out[a] = tok;
        for (int i = a + 1; i <= k; ++i) out[i] = -1;
        accepted_len[b] = a;
    }
}

// ------------------------------------------- chain acceptance, one cluster per sequence
// For greedy acceptance and for sampling without a nucleus (top_p = 1): the
// S CTAs of a cluster split every logits row of their sequence into S
// contiguous vocabulary slices (CTA r: [r*Vs, (r+1)*Vs), Vs a multiple of 4).
// Row arg-max and mass sums are per-slice partials merged in rank order
// through distributed shared memory; the final draw takes every slice's
// Gumbel-max winner and merges them (score desc, index asc).  All masses are
// integers and the scores are per element, so every total, and with it every
// decision, is the one the single-CTA kernels above take.
constexpr int kAcceptClusterMaxK = 16;
constexpr int kAcceptClusterRows = 2 * kAcceptClusterMaxK + 1;
constexpr int kAcceptClusterMax = 8;

struct AcceptXchg {
    float pmax[kAcceptClusterRows];      // this CTA's slice partials, read by its peers
    int parg[kAcceptClusterRows];
    uint64_t psum[kAcceptClusterRows];
    DevRowStats st[kAcceptClusterRows];  // merged statistics (identical in every CTA)
    float gs[2];                         // this CTA's draw winner (score, index): residual, then p
    int gj[2];
    int a;
};

__global__ void __launch_bounds__(kRowThreads) accept_chain_cluster_kernel(
    const float* __restrict__ target, const float* __restrict__ draft, const int32_t* __restrict__ drafts, int k,
    int V, float c, bool greedy, uint64_t seed, const uint32_t* step_dev, uint32_t step_host,
    const DevRowStats* __restrict__ qstats, int S, int32_t* __restrict__ accepted_len,
    int32_t* __restrict__ out_tokens) {
    __shared__ RowSmem sm;
    __shared__ AcceptXchg xs;
    const uint32_t step = step_dev ? *step_dev : step_host;
    const int rank = (int)cluster_rank();
    const int b = blockIdx.x / S;
    const int Vs = ((V + S - 1) / S + 3) & ~3;
    const int L = min(V, rank * Vs), H = min(V, L + Vs);
    const float* P = target + (size_t)b * (k + 1) * V;
    const float* Q = draft + (size_t)b * k * V;
    const int32_t* D = drafts + (size_t)b * k;
    // rows 0..k: the target rows; k+1..2k: the draft rows, when their statistics are not given
    const bool own_q = !greedy && qstats == nullptr;
    const int nrows = (k + 1) + (own_q ? k : 0);
    auto row = [&](int i) { return i <= k ? P + (size_t)i * V : Q + (size_t)(i - k - 1) * V; };

    for (int i = 0; i < nrows; ++i) {
        float m;
        int am;
        cta_argmax(row(i) + L, H - L, sm, &m, &am);
        if (threadIdx.x == 0) {
            xs.pmax[i] = m;
            xs.parg[i] = am < 0 ? -1 : am + L;
        }
    }
    cluster_sync_all();
    if (threadIdx.x < nrows) {
        const int i = threadIdx.x;
        float v = -INFINITY;
        int idx = -1;
        for (int r = 0; r < S; ++r)
            argmax_merge(v, idx, ld_dsmem_f32(s_addr(&xs.pmax[i]), (uint32_t)r),
                         (int)ld_dsmem_u32(s_addr(&xs.parg[i]), (uint32_t)r));
        DevRowStats st;
        st.max = v;
        st.argmax = idx;
        st.tau = 0;
        st.sum = 0;
        st.nuc = 0;
        st.pad = 0;
        xs.st[i] = st;
    }
    __syncthreads();
    if (!greedy) {
        for (int i = 0; i < nrows; ++i) {
            const uint64_t part = cta_mass_sum(row(i) + L, H - L, xs.st[i].max, c, sm);
            if (threadIdx.x == 0) xs.psum[i] = part;
        }
        cluster_sync_all();
        if (threadIdx.x < nrows) {
            uint64_t t = 0;
            for (int r = 0; r < S; ++r) t += ld_dsmem_u64(s_addr(&xs.psum[threadIdx.x]), (uint32_t)r);
            xs.st[threadIdx.x].sum = t;
            xs.st[threadIdx.x].nuc = t;
        }
        __syncthreads();
    }
    // the sequential min(1, p/q) tests (as accept_chain_kernel), taken identically in every CTA
    if (threadIdx.x == 0) {
        int a = 0;
        if (greedy) {
            while (a < k && xs.st[a].argmax == D[a]) ++a;
        } else {
            while (a < k) {
                const int x = D[a];
                const DevRowStats sp = xs.st[a];
                const DevRowStats sq = own_q ? xs.st[k + 1 + a] : qstats[(size_t)b * k + a];
                uint64_t ep = 0, eq = 0;
                if (x >= 0 && x < V) {
                    ep = mass_of(P[(size_t)a * V + x], sp.max, c);
                    eq = mass_of(Q[(size_t)a * V + x], sq.max, c);
                }
                const uint32_t u = uniform_u32(seed, step, (uint32_t)b, (uint32_t)a, U_ACCEPT);
                const u128 lhs = (u128)u * eq * sp.nuc;
                const u128 rhs = ((u128)ep * sq.nuc) << 32;
                if (!(lhs < rhs)) break;
                ++a;
            }
        }
        xs.a = a;
    }
    __syncthreads();
    const int a = xs.a;
    int tok = -1;
    if (greedy) {
        tok = xs.st[a].argmax;
    } else {
        // every CTA draws over its slice; the slices' winners are merged in
        // rank order (score desc, index asc) identically in every CTA
        const float* zp = P + (size_t)a * V;
        const DevRowStats stp = xs.st[a];
        auto merged = [&](int slot) {
            float bs = -INFINITY;
            int bj = -1;
            for (int r = 0; r < S; ++r)
                gumbel_merge(bs, bj, ld_dsmem_f32(s_addr(&xs.gs[slot]), (uint32_t)r),
                             (int)ld_dsmem_u32(s_addr(&xs.gj[slot]), (uint32_t)r));
            return bj;
        };
        float sc;
        int j;
        if (a < k) {
            const DevRowStats stq = own_q ? xs.st[k + 1 + a] : qstats[(size_t)b * k + a];
            cta_gumbel_resid(zp, stp.max, 0u, stp.nuc, Q + (size_t)a * V, stq.max, 0u, stq.nuc, L, H, c, seed, step,
                             (uint32_t)b, (uint32_t)a, sm, &sc, &j);
            if (threadIdx.x == 0) {
                xs.gs[0] = sc;
                xs.gj[0] = j;
            }
            cluster_sync_all();
            tok = merged(0);
        }
        if (tok < 0) {  // the bonus row, or p and q agree
            cta_gumbel_mass(zp, L, H, stp.max, c, 0u, nullptr, 0, seed, step, (uint32_t)b, (uint32_t)a,
                            U_GUMBEL_RESAMPLE, sm, &sc, &j);
            if (threadIdx.x == 0) {
                xs.gs[1] = sc;
                xs.gj[1] = j;
            }
            cluster_sync_all();
            tok = merged(1);
        }
    }
    if (rank == 0 && threadIdx.x == 0) {
        int32_t* out = out_tokens + (size_t)b * (k + 1);
        for (int i = 0; i < a; ++i) out[i] = D[i];
        out[a] = tok;
        for (int i = a + 1; i <= k; ++i) out[i] = -1;
        accepted_len[b] = a;
    }
    cluster_sync_all();  // no CTA leaves while a peer may still read its shared memory
}

// Tree acceptance, one CTA per sequence; statistics of the visited rows are
// computed on demand (a path visits at most depth+1 of the R rows).
__global__ void __launch_bounds__(kRowThreads) accept_tree_kernel(const float* __restrict__ target,
                                                                  const int32_t* __restrict__ node_tokens,
                                                                  const int32_t* __restrict__ parent, int R, int V,
                                                                  float c, uint64_t tp, bool greedy, uint64_t seed,
                                                                  const uint32_t* step_dev, uint32_t step_host,
                                                                  int32_t* __restrict__ accepted_len,
                                                                  int32_t* __restrict__ path_nodes,
                                                                  int32_t* __restrict__ out_tokens) {
    __shared__ RowSmem sm;
    extern __shared__ uint32_t whist_dyn[];  // kWarpHistBytes when tp < 2^32
    __shared__ int s_removed[64];
    __shared__ int s_nremoved, s_next;
    __shared__ uint64_t s_remaining;
    const uint32_t step = step_dev ? *step_dev : step_host;
    const int b = blockIdx.x;
    const float* P = target + (size_t)b * R * V;
    const int32_t* tok = node_tokens + (size_t)b * R;
    int32_t* path = path_nodes + (size_t)b * R;
    int32_t* out = out_tokens + (size_t)b * R;
    for (int i = threadIdx.x; i < R; i += blockDim.x) {
        path[i] = -1;
        out[i] = -1;
    }
    int cur = 0, a = 0, emit = -1;
    for (;;) {
        const float* z = P + (size_t)cur * V;
        DevRowStats st;
        cta_row_stats(z, V, c, tp, !greedy, sm, &st, whist_dyn);
        if (threadIdx.x == 0) {
            int next = -1;
            s_nremoved = 0;
            if (greedy) {
                for (int ch = cur + 1; ch < R; ++ch)
                    if (parent[ch] == cur && tok[ch] == st.argmax) {
                        next = ch;
                        break;
                    }
            } else {
                uint64_t remaining = st.nuc;
                for (int ch = cur + 1; ch < R && next < 0; ++ch) {
                    if (parent[ch] != cur) continue;
                    const int x = tok[ch];
                    uint64_t e = (x >= 0 && x < V) ? nucleus_mass(z, st, c, x) : 0;
                    bool dup = false;
                    for (int t = 0; t < s_nremoved; ++t) dup |= s_removed[t] == x;
                    if (dup) e = 0;
                    const uint32_t u = uniform_u32(seed, step, (uint32_t)b, (uint32_t)ch, U_ACCEPT);
                    if ((u128)u * remaining < ((u128)e << 32)) {
                        next = ch;
                        break;
                    }
                    if (!dup && s_nremoved < 64) s_removed[s_nremoved++] = x;
                    remaining -= e;
                }
                s_remaining = remaining;
            }
            s_next = next;
        }
        __syncthreads();
        const int next = s_next;
        if (next < 0) {
            if (greedy) {
                emit = st.argmax;
            } else {
                // p without the rejected children's tokens (all of p when they cover its mass)
                const int nrem = s_remaining ? s_nremoved : 0;
                float sc;
                cta_gumbel_mass(z, 0, V, st.max, c, st.tau, s_removed, nrem, seed, step, (uint32_t)b, (uint32_t)cur,
                                U_GUMBEL_RESAMPLE, sm, &sc, &emit);
            }
            break;
        }
        if (threadIdx.x == 0) {
            path[a] = next;
            out[a] = tok[next];
        }
        ++a;
        cur = next;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        out[a] = emit;
        accepted_len[b] = a;
    }
}

// Draft sampling: one CTA per row.  Without a nucleus the row's mass total
// comes out of the draw's pass itself, so a row is read twice: arg-max, then
// masses and scores.  When `stats` is given, the row's statistics are kept
// there for the acceptance.
__global__ void __launch_bounds__(kRowThreads) sample_rows_kernel(const float* __restrict__ logits, int k, int V,
                                                                  float c, uint64_t tp, bool greedy, uint64_t seed,
                                                                  const uint32_t* step_dev, uint32_t step_host,
                                                                  int32_t* __restrict__ out,
                                                                  DevRowStats* __restrict__ stats) {
    __shared__ RowSmem sm;
    extern __shared__ uint32_t whist_dyn[];  // kWarpHistBytes when tp < 2^32
    const uint32_t step = step_dev ? *step_dev : step_host;
    const int r = blockIdx.x;
    const float* z = logits + (size_t)r * V;
    DevRowStats st;
    int tok;
    float sc;
    if (!greedy && tp >= (1ull << 32)) {
        st.max = cta_max(z, V, sm);
        st.argmax = -1;
        st.tau = 0;
        st.pad = 0;
        uint64_t total = 0;  // the mass total comes out of the draw's pass
        cta_gumbel_mass(z, 0, V, st.max, c, 0u, nullptr, 0, seed, step, (uint32_t)(r / k), (uint32_t)(r % k),
                        U_GUMBEL_DRAFT, sm, &sc, &tok, &total);
        st.sum = st.nuc = total;  // <= V * 2^31 < 2^64
    } else {
        cta_row_stats(z, V, c, tp, !greedy, sm, &st, whist_dyn);
        tok = st.argmax;
        if (!greedy)
            cta_gumbel_mass(z, 0, V, st.max, c, st.tau, nullptr, 0, seed, step, (uint32_t)(r / k),
                            (uint32_t)(r % k), U_GUMBEL_DRAFT, sm, &sc, &tok);
    }
    if (threadIdx.x == 0) {
        out[r] = tok;
        if (stats) stats[r] = st;
    }
}

// Top-k (descending value, ascending index) per row: k rounds of arg-max with
// the already chosen indices excluded.
__global__ void __launch_bounds__(kRowThreads) topk_kernel(const float* __restrict__ logits, int V, int k,
                                                           int32_t* __restrict__ out) {
    __shared__ RowSmem sm;
    __shared__ int chosen[16];
    const int r = blockIdx.x;
    const float* z = logits + (size_t)r * V;
    for (int t = 0; t < k; ++t) {
        float bv = -INFINITY;
        int bi = -1;
        for (int j = threadIdx.x; j < V; j += blockDim.x) {
            bool ex = false;
            for (int u = 0; u < t; ++u) ex |= chosen[u] == j;
            if (ex) continue;
            const float v = z[j];
            if (bi < 0 || v > bv) {
                bv = v;
                bi = j;
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_merge(bv, bi, v2, i2);
        }
        const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
        __syncthreads();
        if (lane == 0) {
            sm.redf[wid] = bv;
            sm.redi[wid] = bi;
        }
        __syncthreads();
        if (wid == 0) {
            bv = lane < nw ? sm.redf[lane] : -INFINITY;
            bi = lane < nw ? sm.redi[lane] : -1;
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
                int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
                argmax_merge(bv, bi, v2, i2);
            }
            if (lane == 0) {
                chosen[t] = bi;
                out[(size_t)r * k + t] = bi;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------- reference-compatible verify
// Arg-max as a 4-lane (128-bit SVE) scan computes it: per lane strict '>' keeps
// the earliest index, the lowest lane holding the global max wins.
__device__ __forceinline__ bool compat_better(float v, int i, float bv, int bi) {
    if (bi < 0) return true;
    if (v > bv) return true;
    if (v < bv) return false;
    const int l = i & 3, bl = bi & 3;
    return l < bl || (l == bl && i < bi);
}

__global__ void compat_argmax_kernel(const float* __restrict__ logits, const int32_t* __restrict__ lens, int V,
                                     int max_draft, int32_t* __restrict__ best) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const int b = blockIdx.x / max_draft, i = blockIdx.x % max_draft;
    const int d = lens ? min(lens[b], 8) : max_draft;
    if (i >= d) {
        if (threadIdx.x == 0) best[blockIdx.x] = 0;
        return;
    }
    const float* z = logits + (size_t)blockIdx.x * V;
    float bv = -INFINITY;
    int bi = -1;
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float v = z[j];
        if (v != v) continue;  // NaN never compares greater
        if (compat_better(v, j, bv, bi)) {
            bv = v;
            bi = j;
        }
    }
    for (int o = 16; o; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (i2 >= 0 && compat_better(v2, i2, bv, bi)) {
            bv = v2;
            bi = i2;
        }
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) {
        sv[wid] = bv;
        si[wid] = bi;
    }
    __syncthreads();
    if (wid == 0) {
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : -1;
        for (int o = 16; o; o >>= 1) {
            float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (i2 >= 0 && compat_better(v2, i2, bv, bi)) {
                bv = v2;
                bi = i2;
            }
        }
        if (lane == 0) best[blockIdx.x] = bi < 0 ? 0 : bi;
    }
}

__global__ void compat_count_kernel(const int32_t* __restrict__ best, const int32_t* __restrict__ drafts,
                                    const int32_t* __restrict__ lens, int max_draft, int B, int32_t* accepted,
                                    int32_t* replacement) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int d = lens[b];
    if (d <= 0) {
        accepted[b] = 0;
        replacement[b] = -1;
        return;
    }
    d = min(d, min(8, max_draft));
    int cnt = 0;
    bool mism = false;
    for (int i = 0; i < d; ++i) {
        if (best[(size_t)b * max_draft + i] == drafts[(size_t)b * max_draft + i]) ++cnt;
        else mism = true;
    }
    accepted[b] = cnt;
    replacement[b] = mism ? best[(size_t)b * max_draft + cnt] : -1;
}

// -------------------------------------- vocabulary-sharded chain acceptance
// Each rank holds columns [v0, v0 + Vs) of every logits row: target shard
// [B][k+1][Vs], draft shard [B][k][Vs].  The kernels below compute shard
// partials; the caller sums or gathers them across ranks between the steps
// (maxima and arg-maxima merged in rank order, integer mass sums and
// histograms summed, residual totals gathered), so every decision is the one
// the single-GPU acceptance takes on the whole rows.

// (1) row max / arg-max of the shard (global index, -1 for a row of NaN)
// Rows r < rows1 are rows of z1, the rest rows of z2 (one launch for the
// target and draft shards); per-row outputs follow that order.
__device__ __forceinline__ const float* shard_row(const float* z1, int rows1, const float* z2, int Vs, int r) {
    return r < rows1 ? z1 + (size_t)r * Vs : z2 + (size_t)(r - rows1) * Vs;
}

__global__ void __launch_bounds__(kRowThreads) shard_row_max_kernel(const float* __restrict__ z1, int rows1,
                                                                    const float* __restrict__ z2, int Vs, int v0,
                                                                    float* __restrict__ out_max,
                                                                    int32_t* __restrict__ out_arg) {
    __shared__ RowSmem sm;
    float m;
    int am;
    cta_argmax(shard_row(z1, rows1, z2, Vs, blockIdx.x), Vs, sm, &m, &am);
    if (threadIdx.x == 0) {
        out_max[blockIdx.x] = m;
        out_arg[blockIdx.x] = am < 0 ? -1 : am + v0;
    }
}

// (2) the W ranks' partials ([W][rows]) merged in rank order
__global__ void shard_merge_max_kernel(const float* __restrict__ gmax, const int32_t* __restrict__ garg, int W,
                                       int rows, float* __restrict__ out_max, int32_t* __restrict__ out_arg) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float v = -INFINITY;
    int idx = -1;
    for (int w = 0; w < W; ++w) argmax_merge(v, idx, gmax[(size_t)w * rows + r], garg[(size_t)w * rows + r]);
    out_max[r] = v;
    out_arg[r] = idx;
}

// (3) integer mass sum of the shard row at the global row max
__global__ void __launch_bounds__(kRowThreads) shard_row_mass_kernel(const float* __restrict__ z1, int rows1,
                                                                     const float* __restrict__ z2, int Vs,
                                                                     const float* __restrict__ gmax, float c,
                                                                     unsigned long long* __restrict__ out_sum) {
    __shared__ RowSmem sm;
    const uint64_t s = cta_mass_sum(shard_row(z1, rows1, z2, Vs, blockIdx.x), Vs, gmax[blockIdx.x], c, sm);
    if (threadIdx.x == 0) out_sum[blockIdx.x] = s;
}

// (4) mass-weighted histogram of key digit d (3 = top byte) over the shard
// elements whose higher digits equal prefix's
__global__ void __launch_bounds__(kRowThreads) shard_digit_hist_kernel(const float* __restrict__ z1, int rows1,
                                                                       const float* __restrict__ z2, int Vs,
                                                                       const float* __restrict__ gmax, float c,
                                                                       const uint32_t* __restrict__ prefix, int d,
                                                                       unsigned long long* __restrict__ out_hist) {
    __shared__ RowSmem sm;
    extern __shared__ uint32_t whist_dyn[];  // kWarpHistWords words
    const float* zr = shard_row(z1, rows1, z2, Vs, blockIdx.x);
    const float m = gmax[blockIdx.x];
    uint32_t* Hw = whist_dyn + (threadIdx.x >> 5) * 512;
    for (int i = threadIdx.x; i < (int)(blockDim.x >> 5) * 512; i += blockDim.x) whist_dyn[i] = 0;
    __syncthreads();
    const int shift = 8 * d;
    const uint32_t want = d == 3 ? 0u : prefix[blockIdx.x] >> (shift + 8);
    for_each_row_value(zr, Vs, [&](float zj) {
        const uint32_t key = logit_key(zj);
        if (d == 3 || (key >> (shift + 8)) == want) hist_add_lane(Hw, (key >> shift) & 255u, mass_of(zj, m, c));
    });
    merge_warp_hists(whist_dyn, sm);
    for (int b = threadIdx.x; b < 256; b += blockDim.x) out_hist[(size_t)blockIdx.x * 256 + b] = sm.hist[b];
}

// (5) per row (one warp): the digit of the summed histogram where the mass
// from the top reaches thr = max(1, floor(sum * tp / 2^32)), as select_digit;
// G carries the mass above, last the chosen bin's, prefix the digits so far
__global__ void shard_select_digit_kernel(const unsigned long long* __restrict__ hist, int rows, int d,
                                          const unsigned long long* __restrict__ gsum, uint64_t tp,
                                          uint32_t* __restrict__ prefix, unsigned long long* __restrict__ G,
                                          unsigned long long* __restrict__ last) {
    const int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;  // whole warps
    uint64_t thr = (uint64_t)(((u128)gsum[r] * tp) >> 32);
    if (thr < 1) thr = 1;
    const unsigned long long* h = hist + (size_t)r * 256;
    uint64_t local = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) local += h[255 - 8 * lane - i];
    uint64_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const uint64_t g0 = d == 3 ? 0ull : G[r];
    const unsigned hit = __ballot_sync(0xffffffffu, g0 + incl >= thr);
    const int f = hit ? (__ffs(hit) - 1) : 31;
    if (lane == f) {
        uint64_t cum = g0 + incl - local;
        int chosen = 255 - 8 * f - 7;
        for (int i = 0; i < 8; ++i) {
            const int bin = 255 - 8 * f - i;
            if (cum + h[bin] >= thr) {
                chosen = bin;
                break;
            }
            cum += h[bin];
        }
        G[r] = cum;
        last[r] = h[chosen];
        prefix[r] = (d == 3 ? 0u : prefix[r]) | ((uint32_t)chosen << (8 * d));
    }
}

// ---- top-p over the listed high-mass elements (the fast form of steps 2-3)
// (2') per shard row: the integer mass sum S, the mass of the elements with
// t = (z - gmax) * c >= kTList and their 256-bin t histogram (bin =
// floor((t - kTList) * 256 / -kTList), monotone in the key), a count of
// non-finite exponents and of list overflow; the listed (key, mass) pairs go
// to list[row][0, cap).  Layout of out_stats[row]: {S, listed mass, odd,
// overflow, hist[256]} (kShardStatCols u64), summed over ranks.
constexpr int kShardStatCols = 4 + 256;
constexpr int kShardCand = 32;  // candidates per rank and row in the crossing bin
__device__ __forceinline__ int shard_tbin(float t) {
    const int b = (int)__fmul_rn(__fsub_rn(t, kTList), 256.0f / -kTList);
    return b < 255 ? b : 255;
}
__device__ __forceinline__ float key_value(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

__global__ void __launch_bounds__(kRowThreads) shard_mass_hist_kernel(const float* __restrict__ z1, int rows1,
                                                                      const float* __restrict__ z2, int Vs,
                                                                      const float* __restrict__ gmax, float c,
                                                                      int cap, uint2* __restrict__ list,
                                                                      int32_t* __restrict__ list_n,
                                                                      unsigned long long* __restrict__ out_stats) {
    __shared__ RowSmem sm;
    // the t histogram as 16-bit halves of each mass: with at most `cap`
    // (<= 2^16) listed elements a bin stays below 2^32; a row whose list
    // overflowed is not read (step 3' falls back)
    __shared__ uint32_t hlo[256], hhi[256];
    __shared__ int s_n, s_odd;
    const float* zr = shard_row(z1, rows1, z2, Vs, blockIdx.x);
    const float m = gmax[blockIdx.x];
    uint2* lrow = list + (size_t)blockIdx.x * cap;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hlo[i] = hhi[i] = 0;
    if (threadIdx.x == 0) {
        s_n = 0;
        s_odd = 0;
    }
    __syncthreads();
    uint64_t s = 0, ls = 0;
    bool odd = false;
    for_each_row_value(zr, Vs, [&](float zj) {
        const float t = __fmul_rn(__fsub_rn(zj, m), c);
        odd |= t != t;
        const uint32_t e = exp2_fx31_neg(t);
        s += e;
        if (t >= kTList) {
            ls += e;
            const int at = atomicAdd(&s_n, 1);
            if (at < cap) {
                lrow[at] = make_uint2(logit_key(zj), e);
                const int b = shard_tbin(t);
                atomicAdd(&hlo[b], e & 0xFFFFu);
                atomicAdd(&hhi[b], e >> 16);
            }
        }
    });
    if (odd) s_odd = 1;
    s = block_sum<uint64_t>(s, sm.red64);
    ls = block_sum<uint64_t>(ls, sm.red64);
    __syncthreads();
    unsigned long long* o = out_stats + (size_t)blockIdx.x * kShardStatCols;
    if (threadIdx.x == 0) {
        o[0] = s;
        o[1] = ls;
        o[2] = s_odd;
        o[3] = s_n > cap ? 1ull : 0ull;
        list_n[blockIdx.x] = min(s_n, cap);
    }
    for (int b = threadIdx.x; b < 256; b += blockDim.x) o[4 + b] = ((unsigned long long)hhi[b] << 16) + hlo[b];
}

// (3') per row (one warp), on the rank-summed stats: thr = max(1, floor(S *
// top_p)); the row takes the listed path when no exponent was NaN, no rank's
// list overflowed and the listed mass reaches thr.  Then the t bin where the
// mass from the top reaches thr, G = the mass of the bins above it, and this
// rank's listed elements of that bin (at most kShardCand, else the row falls
// back) as candidates: out_cand[row] = {kShardCand (key, mass) pairs, count}
// (count = kShardCand + 1 for a fallback row).
__global__ void shard_cross_kernel(const unsigned long long* __restrict__ stats, int rows, uint64_t tp,
                                   const float* __restrict__ gmax, float c, const uint2* __restrict__ list, int cap,
                                   const int32_t* __restrict__ list_n, unsigned long long* __restrict__ out_G,
                                   uint2* __restrict__ out_cand) {
    const int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;  // whole warps
    const unsigned long long* st = stats + (size_t)r * kShardStatCols;
    uint2* cand = out_cand + (size_t)r * (kShardCand + 1);
    uint64_t thr = (uint64_t)(((u128)st[0] * tp) >> 32);
    if (thr < 1) thr = 1;
    if (st[2] != 0 || st[3] != 0 || st[1] < thr) {
        if (lane == 0) {
            out_G[r] = 0;
            cand[kShardCand] = make_uint2(kShardCand + 1, 0);
        }
        return;
    }
    const unsigned long long* h = st + 4;
    uint64_t local = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) local += h[255 - 8 * lane - i];
    uint64_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, incl >= thr);
    const int f = hit ? (__ffs(hit) - 1) : 31;
    int chosen = 0;
    uint64_t G = 0;
    if (lane == f) {
        uint64_t cum = incl - local;
        chosen = 255 - 8 * f - 7;
        for (int i = 0; i < 8; ++i) {
            const int bin = 255 - 8 * f - i;
            if (cum + h[bin] >= thr) {
                chosen = bin;
                break;
            }
            cum += h[bin];
        }
        G = cum;
    }
    chosen = __shfl_sync(0xffffffffu, chosen, f);
    G = __shfl_sync(0xffffffffu, G, f);
    // this rank's listed elements in the chosen bin (the list is complete: no overflow)
    const float m = gmax[r];
    const uint2* lrow = list + (size_t)r * cap;
    int n = 0;
    const int ln = list_n[r];
    for (int i0 = 0; i0 < ln; i0 += 32) {
        const int i = i0 + lane;
        bool in = false;
        uint2 en = make_uint2(0, 0);
        if (i < ln) {
            en = lrow[i];
            in = en.y != 0u && shard_tbin(__fmul_rn(__fsub_rn(key_value(en.x), m), c)) == chosen;
        }
        const unsigned msk = __ballot_sync(0xffffffffu, in);
        const int at = n + __popc(msk & ((1u << lane) - 1u));
        if (in && at < kShardCand) cand[at] = en;
        n += __popc(msk);
    }
    if (lane == 0) {
        out_G[r] = G;
        cand[kShardCand] = make_uint2((uint32_t)min(n, kShardCand + 1), 0);
    }
}

// (4') per row (one CTA): the radix select over the W ranks' gathered
// candidates ([W][rows][kShardCand + 1]) above G, as list_topp_select; a row
// any rank marked for fallback gets ok = 0.
__global__ void __launch_bounds__(256) shard_union_select_kernel(const uint2* __restrict__ gcand, int W, int rows,
                                                                 const unsigned long long* __restrict__ stats,
                                                                 const unsigned long long* __restrict__ gG,
                                                                 uint64_t tp, uint32_t* __restrict__ out_tau,
                                                                 unsigned long long* __restrict__ out_nuc,
                                                                 int32_t* __restrict__ out_ok) {
    __shared__ RowSmem sm;
    __shared__ uint32_t whist[8 * 512];
    __shared__ uint2 cands[256];
    __shared__ int s_n, s_bad;
    const int r = blockIdx.x;
    if (threadIdx.x == 0) {
        s_n = 0;
        s_bad = 0;
    }
    __syncthreads();
    for (int w = 0; w < W; ++w) {
        const uint2* cw = gcand + ((size_t)w * rows + r) * (kShardCand + 1);
        const int cnt = (int)cw[kShardCand].x;
        if (cnt > kShardCand) {
            if (threadIdx.x == 0) s_bad = 1;
            continue;
        }
        for (int i = threadIdx.x; i < cnt; i += blockDim.x) cands[atomicAdd(&s_n, 1)] = cw[i];
    }
    __syncthreads();
    if (s_bad) {
        if (threadIdx.x == 0) out_ok[r] = 0;
        return;
    }
    uint64_t thr = (uint64_t)(((u128)stats[(size_t)r * kShardStatCols] * tp) >> 32);
    if (thr < 1) thr = 1;
    const int n = s_n;
    uint32_t* Hw = whist + (threadIdx.x >> 5) * 512;
    for (int i = threadIdx.x; i < 8 * 512; i += blockDim.x) whist[i] = 0;
    __syncthreads();
    uint64_t G = gG[r], last = 0;
    uint32_t prefix = 0, dg = 0;
    for (int d = 3; d >= 0; --d) {
        const int shift = 8 * d;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint2 en = cands[i];
            if (d == 3 || (en.x >> (shift + 8)) == (prefix >> (shift + 8))) hist_add_lane(Hw, (en.x >> shift) & 255u, en.y);
        }
        merge_warp_hists(whist, sm);
        select_digit(sm, thr, &G, &dg, &last);
        prefix |= dg << shift;
    }
    if (threadIdx.x == 0) {
        out_tau[r] = prefix;
        out_nuc[r] = G + last;
        out_ok[r] = 1;
    }
}

// (6) the nucleus masses of the drafted tokens in the shard that owns them (0 elsewhere)
__global__ void shard_point_mass_kernel(const float* __restrict__ target, const float* __restrict__ draft,
                                        const int32_t* __restrict__ drafts, int B, int k, int Vs, int v0, float c,
                                        const float* __restrict__ pmax, const uint32_t* __restrict__ ptau,
                                        const float* __restrict__ qmax, const uint32_t* __restrict__ qtau,
                                        unsigned long long* __restrict__ ep, unsigned long long* __restrict__ eq) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= B * k) return;
    const int b = t / k, i = t - b * k, x = drafts[t];
    uint64_t a = 0, q = 0;
    if (x >= v0 && x < v0 + Vs) {
        const int prow = b * (k + 1) + i, qrow = t;
        const float zp = target[(size_t)prow * Vs + (x - v0)], zq = draft[(size_t)qrow * Vs + (x - v0)];
        a = logit_key(zp) < ptau[prow] ? 0u : mass_of(zp, pmax[prow], c);
        q = logit_key(zq) < qtau[qrow] ? 0u : mass_of(zq, qmax[qrow], c);
    }
    ep[t] = a;
    eq[t] = q;
}

// (7) the sequential min(1, p/q) tests (as accept_chain_kernel), one thread per sequence
__global__ void shard_accept_test_kernel(const int32_t* __restrict__ drafts, int B, int k, bool greedy, uint64_t seed,
                                         const uint32_t* __restrict__ step_dev, uint32_t step_host,
                                         const int32_t* __restrict__ parg,
                                         const unsigned long long* __restrict__ pnuc,
                                         const unsigned long long* __restrict__ qnuc,
                                         const unsigned long long* __restrict__ ep,
                                         const unsigned long long* __restrict__ eq, int32_t* __restrict__ a_out) {
    const uint32_t step = step_dev ? *step_dev : step_host;
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int32_t* D = drafts + (size_t)b * k;
    int a = 0;
    if (greedy) {
        while (a < k && parg[b * (k + 1) + a] == D[a]) ++a;
    } else {
        while (a < k) {
            const uint32_t u = uniform_u32(seed, step, (uint32_t)b, (uint32_t)a, U_ACCEPT);
            const u128 lhs = (u128)u * eq[b * k + a] * pnuc[b * (k + 1) + a];
            const u128 rhs = ((u128)ep[b * k + a] * qnuc[b * k + a]) << 32;
            if (!(lhs < rhs)) break;
            ++a;
        }
    }
    a_out[b] = a;
}

struct ShardRows {
    const float* target;
    const float* draft;
    int k, Vs, v0;
    float c;
    const float* pmax;
    const uint32_t* ptau;
    const float* qmax;
    const uint32_t* qtau;
    const unsigned long long* pnuc;
    const unsigned long long* qnuc;
};

// (8) per sequence b with a = a_in[b]: this shard's Gumbel-max winners of the
// draw on target row a, over the residual max(0, p - q) (a < k) and over the
// nucleus of p, as out[b] = {residual score bits, index, p score bits, index}
// (global indices; -1 when the shard has no candidate).  The element uniforms
// are those of the global index, so the winners merged over the shards are
// the draw on the whole row.
__global__ void __launch_bounds__(kRowThreads) shard_draw_winners_kernel(ShardRows sr, const int32_t* __restrict__ a_in,
                                                                         uint64_t seed,
                                                                         const uint32_t* __restrict__ step_dev,
                                                                         uint32_t step_host, int32_t* __restrict__ out) {
    const uint32_t step = step_dev ? *step_dev : step_host;
    __shared__ RowSmem sm;
    const int b = blockIdx.x, a = a_in[b], k = sr.k;
    const int prow = b * (k + 1) + a;
    // rows addressed by global vocabulary index: element j of the shard at [j - v0]
    const float* zp = sr.target + (size_t)prow * sr.Vs - sr.v0;
    const int L = sr.v0, H = sr.v0 + sr.Vs;
    float rs = -INFINITY, ps = -INFINITY;
    int rj = -1, pj = -1;
    if (a < k) {
        const int qrow = b * k + a;
        const float* zq = sr.draft + (size_t)qrow * sr.Vs - sr.v0;
        cta_gumbel_resid(zp, sr.pmax[prow], sr.ptau[prow], sr.pnuc[prow], zq, sr.qmax[qrow], sr.qtau[qrow],
                         sr.qnuc[qrow], L, H, sr.c, seed, step, (uint32_t)b, (uint32_t)a, sm, &rs, &rj);
    }
    cta_gumbel_mass(zp, L, H, sr.pmax[prow], sr.c, sr.ptau[prow], nullptr, 0, seed, step, (uint32_t)b, (uint32_t)a,
                    U_GUMBEL_RESAMPLE, sm, &ps, &pj);
    if (threadIdx.x == 0) {
        out[(size_t)b * 4 + 0] = __float_as_int(rs);
        out[(size_t)b * 4 + 1] = rj;
        out[(size_t)b * 4 + 2] = __float_as_int(ps);
        out[(size_t)b * 4 + 3] = pj;
    }
}

// (9) per sequence: the gathered winners ([W][B][4]) merged in rank order
// (score desc, index asc): the residual's when a < k and it has a candidate
// anywhere, else p's.
__global__ void shard_draw_merge_kernel(const int32_t* __restrict__ gwin, int W, int B, int k,
                                        const int32_t* __restrict__ a_in, int32_t* __restrict__ tok_out) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    float rs = -INFINITY, ps = -INFINITY;
    int rj = -1, pj = -1;
    for (int w = 0; w < W; ++w) {
        const int32_t* g = gwin + ((size_t)w * B + b) * 4;
        gumbel_merge(rs, rj, __int_as_float(g[0]), g[1]);
        gumbel_merge(ps, pj, __int_as_float(g[2]), g[3]);
    }
    tok_out[b] = (a_in[b] < k && rj >= 0) ? rj : pj;
}

// ------------------------------------------------------------ host side
float temp_coeff(float temperature) { return (float)(1.4426950408889634 / (double)temperature); }
uint64_t top_p_q32(float top_p) {
    if (!(top_p < 1.0f)) return 1ull << 32;
    if (top_p <= 0.0f) return 0;
    return (uint64_t)llround((double)top_p * 4294967296.0);
}

int launch_topk(const float* logits, int rows, int V, int k, int32_t* out, cudaStream_t s) {
    SD_CHECK(k >= 1 && k <= 16, SPECDEC_EINVAL, "topk: k must be in [1,16]");
    topk_kernel<<<rows, kRowThreads, 0, s>>>(logits, V, k, out);
    SD_LAUNCH_CHECK("topk_kernel");
    return SPECDEC_OK;
}

// Dynamic shared memory of the row-statistics kernels: the per-warp top-p
// histograms, needed only when the rows need mass sums and a nucleus.  They
// exceed the 48 KB default, so the kernels opt in once per device.
static std::mutex g_hist_mu;
static bool g_hist_opted[64] = {};

static int hist_smem(bool need_mass, uint64_t tp, size_t* bytes) {
    *bytes = 0;
    if (!need_mass || tp >= (1ull << 32)) return SPECDEC_OK;
    int dev = 0;
    SD_CUDA(cudaGetDevice(&dev));
    SD_CHECK(dev >= 0 && dev < 64, SPECDEC_EINVAL, "sampling: device index out of range");
    std::lock_guard<std::mutex> lk(g_hist_mu);  // first calls from several host threads
    if (!g_hist_opted[dev]) {
        const int sz = (int)kWarpHistBytes;
        SD_CUDA(cudaFuncSetAttribute(row_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sz));
        SD_CUDA(cudaFuncSetAttribute(accept_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sz));
        SD_CUDA(cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sz));
        g_hist_opted[dev] = true;
    }
    *bytes = kWarpHistBytes;
    return SPECDEC_OK;
}

// Whether the chain acceptance takes the row-statistics path (which uses the
// per-row scratch) rather than the sliced cluster kernel (which needs none).
static bool accept_uses_row_stats(bool greedy, uint64_t tp, int k) {
    return !((greedy || tp >= (1ull << 32)) && k <= kAcceptClusterMaxK);
}

// Cluster size of the sliced chain acceptance: the largest power of two
// <= 8 whose B * S CTAs fit one wave on the device's SMs.
static int accept_cluster_size(int B) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) (void)cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int S = kAcceptClusterMax;
    while (S > 1 && (long long)B * S > sms) S >>= 1;
    return S;
}

// Chain acceptance: the sliced cluster kernel for greedy decisions and
// sampling without a nucleus (k <= 16), else row statistics into `st`
// (B*(k+1) target rows, then B*k draft rows) and one CTA per sequence.
// With draft_stats_ready the draft rows' statistics are already in st (the
// draft sampler wrote them), and are not recomputed.
static int launch_accept_chain_impl(const float* target, const float* draft, const int32_t* drafts, int B, int k,
                                    int V, float temperature, float top_p, uint64_t seed, const uint32_t* step_dev,
                                    uint32_t step_host, DevRowStats* st, bool draft_stats_ready,
                                    int32_t* accepted_len, int32_t* out_tokens, cudaStream_t s) {
    const bool greedy = !(temperature > 0.0f);
    const float c = greedy ? 0.0f : temp_coeff(temperature);
    const uint64_t tp = top_p_q32(top_p);
    const float* dq = greedy ? target : draft;
    if (!accept_uses_row_stats(greedy, tp, k)) {
        const int S = accept_cluster_size(B);
        const DevRowStats* qstats = (!greedy && draft_stats_ready) ? st + (size_t)B * (k + 1) : nullptr;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(B * S));
        cfg.blockDim = dim3(kRowThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)S;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        SD_CUDA(cudaLaunchKernelEx(&cfg, accept_chain_cluster_kernel, target, dq, drafts, k, V, c, greedy, seed,
                                   step_dev, step_host, qstats, S, accepted_len, out_tokens));
        return SPECDEC_OK;
    }
    SD_CHECK(st, SPECDEC_EINVAL, "accept_chain: row statistics scratch required");
    const long long rows_ll = (long long)B * (k + 1) + (greedy ? 0 : (long long)B * k);
    SD_CHECK(rows_ll <= INT_MAX, SPECDEC_EINVAL, "accept_chain: too many logits rows");
    const int rows = (int)rows_ll;
    RowSet a{target, B * (k + 1)}, bq{dq, greedy ? 0 : B * k};
    size_t hs = 0;
    int rc = hist_smem(!greedy, tp, &hs);
    if (rc) return rc;
    row_stats_kernel<<<(unsigned)rows, kRowThreads, hs, s>>>(a, bq, V, c, tp, !greedy, true, st);
    SD_LAUNCH_CHECK("row_stats_kernel");
    accept_chain_kernel<<<B, kRowThreads, 0, s>>>(target, dq, drafts, k, V, c, greedy, seed, step_dev, step_host, st,
                                                  B, accepted_len, out_tokens);
    SD_LAUNCH_CHECK("accept_chain_kernel");
    return SPECDEC_OK;
}

int launch_accept_chain_dev(const float* target, const float* draft, const int32_t* drafts, int B, int k, int V,
                            float temperature, float top_p, uint64_t seed, const uint32_t* step_dev,
                            int32_t* accepted_len, int32_t* out_tokens, void* ws, bool draft_stats_ready,
                            cudaStream_t s) {
    SD_CHECK(V <= kMaxVocab, SPECDEC_EINVAL, "launch_accept_chain_dev: vocabulary above 262144");
    return launch_accept_chain_impl(target, draft, drafts, B, k, V, temperature, top_p, seed, step_dev, 0u,
                                    reinterpret_cast<DevRowStats*>(ws), draft_stats_ready, accepted_len, out_tokens, s);
}

int launch_accept_tree_dev(const float* target, const int32_t* node_tokens, const int32_t* parent, int B, int R, int V,
                           float temperature, float top_p, uint64_t seed, const uint32_t* step_dev,
                           int32_t* accepted_len, int32_t* path, int32_t* out_tokens, cudaStream_t s) {
    SD_CHECK(V <= kMaxVocab, SPECDEC_EINVAL, "launch_accept_tree_dev: vocabulary above 262144");
    const bool greedy = !(temperature > 0.0f);
    size_t hs = 0;
    int rc = hist_smem(!greedy, top_p_q32(top_p), &hs);
    if (rc) return rc;
    accept_tree_kernel<<<B, kRowThreads, hs, s>>>(target, node_tokens, parent, R, V, greedy ? 0.0f : temp_coeff(temperature),
                                                 top_p_q32(top_p), greedy, seed, step_dev, 0u, accepted_len, path,
                                                 out_tokens);
    SD_LAUNCH_CHECK("accept_tree_kernel");
    return SPECDEC_OK;
}

int launch_sample_rows_dev(const float* logits, int rows, int k, int V, float temperature, float top_p, uint64_t seed,
                           const uint32_t* step_dev, int32_t* out, void* stats, cudaStream_t s) {
    SD_CHECK(V <= kMaxVocab, SPECDEC_EINVAL, "launch_sample_rows_dev: vocabulary above 262144");
    const bool greedy = !(temperature > 0.0f);
    size_t hs = 0;
    int rc = hist_smem(!greedy, top_p_q32(top_p), &hs);
    if (rc) return rc;
    sample_rows_kernel<<<rows, kRowThreads, hs, s>>>(logits, k, V, greedy ? 0.0f : temp_coeff(temperature),
                                                    top_p_q32(top_p), greedy, seed, step_dev, 0u, out,
                                                    reinterpret_cast<DevRowStats*>(stats));
    SD_LAUNCH_CHECK("sample_rows_kernel");
    return SPECDEC_OK;
}

}  // namespace specdec

using namespace specdec;

extern "C" size_t specdec_accept_workspace_bytes(int rows) { return (size_t)(rows > 0 ? rows : 0) * sizeof(DevRowStats); }

extern "C" int specdec_accept_chain(const float* target, const float* draft, const int32_t* drafts, int B, int k,
                                    int V, const specdec_sampling* sp, int32_t* accepted_len, int32_t* out_tokens,
                                    void* workspace, size_t workspace_bytes, void* stream) {
    SD_CHECK(V <= kMaxVocab, SPECDEC_EINVAL, "specdec_accept_chain: vocabulary above 262144");
    SD_CHECK(sp && target && drafts && accepted_len && out_tokens, SPECDEC_EINVAL, "accept_chain: null argument");
    SD_CHECK(B >= 0 && k >= 0 && V > 0, SPECDEC_EINVAL, "accept_chain: bad shape");
    if (B == 0) return SPECDEC_OK;
    const bool greedy = !(sp->temperature > 0.0f);
    SD_CHECK(greedy || draft, SPECDEC_EINVAL, "accept_chain: draft logits required when sampling");
    const long long ws_rows = (long long)B * (2 * (long long)k + 1);
    SD_CHECK(ws_rows <= INT_MAX, SPECDEC_EINVAL, "accept_chain: too many logits rows");
    SD_CHECK(workspace && workspace_bytes >= specdec_accept_workspace_bytes((int)ws_rows), SPECDEC_EINVAL,
             "accept_chain: workspace too small");
    return launch_accept_chain_impl(target, draft, drafts, B, k, V, sp->temperature, sp->top_p, sp->seed, nullptr,
                                    sp->step, reinterpret_cast<DevRowStats*>(workspace), false, accepted_len,
                                    out_tokens, as_stream(stream));
}

// ---------------------------------------------------------------------------
// Chain acceptance without any allocation.
//
// Some callers cannot allocate device memory at the point where they accept
// drafts: a serving loop that reserves its whole device-memory budget at
// start-up and must not grow it per step, or a host program that owns the
// GPU allocator and forbids plug-ins from calling it.  For them this variant
// keeps the per-row statistics in a fixed array compiled into the library
// (kStaticAcceptRows rows of 32 bytes, 256 KB on every GPU that loads the
// library, held until the process exits) instead of a caller workspace.
//
// The array's device address is looked up once per device, on the first call
// made with that device current (cudaGetSymbolAddress); that first call should
// come before any stream capture.  Every call shares the array: two calls
// whose kernels overlap on the GPU (different streams, no ordering between
// them) race on it.  Nothing in it needs to start at zero: the statistics
// kernel overwrites every row it later reads.
namespace specdec {
constexpr int kStaticAcceptRows = 8192;
static __device__ __align__(256) DevRowStats g_static_accept_rows[kStaticAcceptRows];

static std::mutex g_static_accept_mu;
static DevRowStats* g_static_accept_ptr[64] = {};

// Device address of the fixed scratch for the current device (looked up once).
static int static_accept_rows(DevRowStats** out) {
    int dev = 0;
    SD_CUDA(cudaGetDevice(&dev));
    SD_CHECK(dev >= 0 && dev < 64, SPECDEC_EINVAL, "accept_chain_noalloc: device index out of range");
    std::lock_guard<std::mutex> lk(g_static_accept_mu);
    if (!g_static_accept_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_accept_rows);
        if (e != cudaSuccess) return cuda_status(e, "accept_chain_noalloc: cudaGetSymbolAddress");
        g_static_accept_ptr[dev] = reinterpret_cast<DevRowStats*>(p);
    }
    *out = g_static_accept_ptr[dev];
    return SPECDEC_OK;
}
}  // namespace specdec

extern "C" int specdec_accept_chain_noalloc(const float* target, const float* draft, const int32_t* drafts, int B,
                                            int k, int V, const specdec_sampling* sp, int32_t* accepted_len,
                                            int32_t* out_tokens, void* stream) {
    SD_CHECK(V <= kMaxVocab, SPECDEC_EINVAL, "specdec_accept_chain_noalloc: vocabulary above 262144");
    SD_CHECK(sp && target && drafts && accepted_len && out_tokens, SPECDEC_EINVAL,
             "accept_chain_noalloc: null argument");
    SD_CHECK(B >= 0 && k >= 0 && V > 0, SPECDEC_EINVAL, "accept_chain_noalloc: bad shape");
    if (B == 0) return SPECDEC_OK;
    const bool greedy = !(sp->temperature > 0.0f);
    SD_CHECK(greedy || draft, SPECDEC_EINVAL, "accept_chain_noalloc: draft logits required when sampling");
    const long long rows = (long long)B * (k + 1) + (greedy ? 0 : (long long)B * k);
    // the limit binds only where the fixed scratch is used: the row-statistics
    // path (top_p < 1 sampling, or more than 16 drafts)
    if (accept_uses_row_stats(greedy, top_p_q32(sp->top_p), k) && rows > kStaticAcceptRows) {
        set_error("accept_chain_noalloc: batch*(k+1) + batch*k logits rows (" + std::to_string(rows) +
                  ") exceed the fixed scratch of " + std::to_string(kStaticAcceptRows) +
                  " rows; use specdec_accept_chain with a caller workspace");
        return SPECDEC_EINVAL;
    }
    DevRowStats* st = nullptr;
    int rc = static_accept_rows(&st);
    if (rc) return rc;
    return launch_accept_chain_impl(target, draft, drafts, B, k, V, sp->temperature, sp->top_p, sp->seed, nullptr,
                                    sp->step, st, false, accepted_len, out_tokens, as_stream(stream));
}

extern "C" int specdec_accept_tree(const float* target, const int32_t* node_tokens, const int32_t* parent, int B,
                                   int R, int V, const specdec_sampling* sp, int32_t* accepted_len,
                                   int32_t* path_nodes, int32_t* out_tokens, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    SD_CHECK(V <= kMaxVocab, SPECDEC_EINVAL, "specdec_accept_tree: vocabulary above 262144");
    (void)workspace;
    (void)workspace_bytes;
    SD_CHECK(sp && target && node_tokens && parent && accepted_len && path_nodes && out_tokens, SPECDEC_EINVAL,
             "accept_tree: null argument");
    SD_CHECK(R >= 1 && R <= 64 && V > 0 && B >= 0, SPECDEC_EINVAL, "accept_tree: bad shape (R must be 1..64)");
    if (B == 0) return SPECDEC_OK;
    const bool greedy = !(sp->temperature > 0.0f);
    const float c = greedy ? 0.0f : temp_coeff(sp->temperature);
    size_t hs = 0;
    int rc = hist_smem(!greedy, top_p_q32(sp->top_p), &hs);
    if (rc) return rc;
    accept_tree_kernel<<<B, kRowThreads, hs, as_stream(stream)>>>(target, node_tokens, parent, R, V, c,
                                                                 top_p_q32(sp->top_p), greedy, sp->seed, nullptr,
                                                                 sp->step, accepted_len, path_nodes, out_tokens);
    SD_LAUNCH_CHECK("accept_tree_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_sample_rows(const float* logits, int rows, int k, int V, const specdec_sampling* sp,
                                   int32_t* out, void* workspace, size_t workspace_bytes, void* stream) {
    SD_CHECK(V <= kMaxVocab, SPECDEC_EINVAL, "specdec_sample_rows: vocabulary above 262144");
    (void)workspace;
    (void)workspace_bytes;
    SD_CHECK(sp && logits && out && rows >= 0 && k >= 1 && V > 0, SPECDEC_EINVAL, "sample_rows: bad argument");
    if (rows == 0) return SPECDEC_OK;
    const bool greedy = !(sp->temperature > 0.0f);
    size_t hs = 0;
    int rc = hist_smem(!greedy, top_p_q32(sp->top_p), &hs);
    if (rc) return rc;
    sample_rows_kernel<<<rows, kRowThreads, hs, as_stream(stream)>>>(
        logits, k, V, greedy ? 0.0f : temp_coeff(sp->temperature), top_p_q32(sp->top_p), greedy, sp->seed, nullptr, sp->step,
        out, nullptr);
    SD_LAUNCH_CHECK("sample_rows_kernel");
    return SPECDEC_OK;
}

// ---------------------------------------------------------------------------
// Vocabulary-sharded chain acceptance: the shard steps (see include/specdec.h).
// Threads per shard row: narrow shards (many ranks) get smaller CTAs, so that
// several rows share an SM instead of one 1024-thread CTA per row idling in
// its reductions.
static int shard_threads(int Vs) {
    int t = 256;
    while (t < kRowThreads && t * 64 < Vs) t *= 2;
    return t;
}

static int shard_check(int rows, int Vs, const char* what) {
    if (rows < 0 || Vs <= 0 || Vs > kMaxVocab) {
        set_error(std::string(what) + ": bad shape (shard width must be 1 .. 262144)");
        return SPECDEC_EINVAL;
    }
    return SPECDEC_OK;
}

extern "C" int specdec_shard_row_max(const float* z, int rows, const float* z2, int rows2, int Vs, int v0,
                                     float* out_max, int32_t* out_arg, void* stream) {
    if (int rc = shard_check(rows, Vs, "shard_row_max")) return rc;
    SD_CHECK(z && out_max && out_arg && rows2 >= 0 && (rows2 == 0 || z2), SPECDEC_EINVAL,
             "shard_row_max: null argument");
    if (rows + rows2 == 0) return SPECDEC_OK;
    shard_row_max_kernel<<<rows + rows2, shard_threads(Vs), 0, as_stream(stream)>>>(z, rows, z2, Vs, v0, out_max, out_arg);
    SD_LAUNCH_CHECK("shard_row_max_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_merge_max(const float* gmax, const int32_t* garg, int W, int rows, float* out_max,
                                       int32_t* out_arg, void* stream) {
    SD_CHECK(gmax && garg && out_max && out_arg && W >= 1 && rows >= 0, SPECDEC_EINVAL, "shard_merge_max: bad argument");
    if (rows == 0) return SPECDEC_OK;
    shard_merge_max_kernel<<<(rows + 255) / 256, 256, 0, as_stream(stream)>>>(gmax, garg, W, rows, out_max, out_arg);
    SD_LAUNCH_CHECK("shard_merge_max_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_row_mass(const float* z, int rows, const float* z2, int rows2, int Vs,
                                      const float* gmax, float temperature, uint64_t* out_sum, void* stream) {
    if (int rc = shard_check(rows, Vs, "shard_row_mass")) return rc;
    SD_CHECK(z && gmax && out_sum && temperature > 0.0f && rows2 >= 0 && (rows2 == 0 || z2), SPECDEC_EINVAL,
             "shard_row_mass: bad argument");
    if (rows + rows2 == 0) return SPECDEC_OK;
    shard_row_mass_kernel<<<rows + rows2, shard_threads(Vs), 0, as_stream(stream)>>>(
        z, rows, z2, Vs, gmax, temp_coeff(temperature), reinterpret_cast<unsigned long long*>(out_sum));
    SD_LAUNCH_CHECK("shard_row_mass_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_digit_hist(const float* z, int rows, const float* z2, int rows2, int Vs,
                                        const float* gmax, float temperature, const uint32_t* prefix, int digit,
                                        uint64_t* out_hist, void* stream) {
    if (int rc = shard_check(rows, Vs, "shard_digit_hist")) return rc;
    SD_CHECK(z && gmax && out_hist && temperature > 0.0f && digit >= 0 && digit <= 3 && (digit == 3 || prefix) &&
                 rows2 >= 0 && (rows2 == 0 || z2),
             SPECDEC_EINVAL, "shard_digit_hist: bad argument");
    if (rows + rows2 == 0) return SPECDEC_OK;
    const size_t hs = kWarpHistWords * sizeof(uint32_t);
    SD_CUDA(cudaFuncSetAttribute(shard_digit_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hs));
    shard_digit_hist_kernel<<<rows + rows2, kRowThreads, hs, as_stream(stream)>>>(
        z, rows, z2, Vs, gmax, temp_coeff(temperature), prefix, digit, reinterpret_cast<unsigned long long*>(out_hist));
    SD_LAUNCH_CHECK("shard_digit_hist_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_mass_hist(const float* z, int rows, const float* z2, int rows2, int Vs, const float* gmax,
                                       float temperature, int cap, void* list, int32_t* list_n, uint64_t* out_stats,
                                       void* stream) {
    if (int rc = shard_check(rows, Vs, "shard_mass_hist")) return rc;
    SD_CHECK(z && gmax && list && list_n && out_stats && temperature > 0.0f && cap > 0 && rows2 >= 0 &&
                 (rows2 == 0 || z2),
             SPECDEC_EINVAL, "shard_mass_hist: bad argument");
    if (rows + rows2 == 0) return SPECDEC_OK;
    SD_CHECK(cap <= 65536, SPECDEC_EINVAL, "shard_mass_hist: cap above 65536");
    shard_mass_hist_kernel<<<rows + rows2, shard_threads(Vs), 0, as_stream(stream)>>>(
        z, rows, z2, Vs, gmax, temp_coeff(temperature), cap, static_cast<uint2*>(list), list_n,
        reinterpret_cast<unsigned long long*>(out_stats));
    SD_LAUNCH_CHECK("shard_mass_hist_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_cross(const uint64_t* stats, int rows, float top_p, const float* gmax, float temperature,
                                   const void* list, int cap, const int32_t* list_n, uint64_t* out_G, void* out_cand,
                                   void* stream) {
    SD_CHECK(stats && gmax && list && list_n && out_G && out_cand && rows >= 0 && cap > 0 && temperature > 0.0f &&
                 top_p > 0.0f && top_p < 1.0f,
             SPECDEC_EINVAL, "shard_cross: bad argument");
    if (rows == 0) return SPECDEC_OK;
    shard_cross_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const unsigned long long*>(stats), rows, top_p_q32(top_p), gmax, temp_coeff(temperature),
        static_cast<const uint2*>(list), cap, list_n, reinterpret_cast<unsigned long long*>(out_G),
        static_cast<uint2*>(out_cand));
    SD_LAUNCH_CHECK("shard_cross_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_union_select(const void* gcand, int W, int rows, const uint64_t* stats,
                                          const uint64_t* G, float top_p, uint32_t* out_tau, uint64_t* out_nuc,
                                          int32_t* out_ok, void* stream) {
    SD_CHECK(gcand && stats && G && out_tau && out_nuc && out_ok && rows >= 0 && W >= 1 && W * kShardCand <= 256 &&
                 top_p > 0.0f && top_p < 1.0f,
             SPECDEC_EINVAL, "shard_union_select: bad argument (at most 8 ranks)");
    if (rows == 0) return SPECDEC_OK;
    shard_union_select_kernel<<<(unsigned)rows, 256, 0, as_stream(stream)>>>(
        static_cast<const uint2*>(gcand), W, rows, reinterpret_cast<const unsigned long long*>(stats),
        reinterpret_cast<const unsigned long long*>(G), top_p_q32(top_p), out_tau,
        reinterpret_cast<unsigned long long*>(out_nuc), out_ok);
    SD_LAUNCH_CHECK("shard_union_select_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_select_digit(const uint64_t* hist, int rows, int digit, const uint64_t* gsum, float top_p,
                                          uint32_t* prefix, uint64_t* G, uint64_t* last, void* stream) {
    SD_CHECK(hist && gsum && prefix && G && last && rows >= 0 && digit >= 0 && digit <= 3, SPECDEC_EINVAL,
             "shard_select_digit: bad argument");
    if (rows == 0) return SPECDEC_OK;
    shard_select_digit_kernel<<<(rows + 7) / 8, 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const unsigned long long*>(hist), rows, digit,
        reinterpret_cast<const unsigned long long*>(gsum), top_p_q32(top_p), prefix,
        reinterpret_cast<unsigned long long*>(G), reinterpret_cast<unsigned long long*>(last));
    SD_LAUNCH_CHECK("shard_select_digit_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_point_mass(const float* target, const float* draft, const int32_t* drafts, int B, int k,
                                        int Vs, int v0, float temperature, const float* pmax, const uint32_t* ptau,
                                        const float* qmax, const uint32_t* qtau, uint64_t* ep, uint64_t* eq,
                                        void* stream) {
    if (int rc = shard_check(B, Vs, "shard_point_mass")) return rc;
    SD_CHECK(target && draft && drafts && pmax && ptau && qmax && qtau && ep && eq && k >= 1 && temperature > 0.0f,
             SPECDEC_EINVAL, "shard_point_mass: bad argument");
    SD_CHECK((long long)B * k <= INT_MAX - 255, SPECDEC_EINVAL, "shard_point_mass: too many draft rows");
    if (B == 0) return SPECDEC_OK;
    shard_point_mass_kernel<<<(B * k + 255) / 256, 256, 0, as_stream(stream)>>>(
        target, draft, drafts, B, k, Vs, v0, temp_coeff(temperature), pmax, ptau, qmax, qtau,
        reinterpret_cast<unsigned long long*>(ep), reinterpret_cast<unsigned long long*>(eq));
    SD_LAUNCH_CHECK("shard_point_mass_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_accept_test(const int32_t* drafts, int B, int k, const specdec_sampling* sp,
                                         const int32_t* parg, const uint64_t* pnuc, const uint64_t* qnuc,
                                         const uint64_t* ep, const uint64_t* eq, int32_t* accepted,
                                         const uint32_t* step_dev, void* stream) {
    SD_CHECK(drafts && sp && parg && accepted && B >= 0 && k >= 1, SPECDEC_EINVAL, "shard_accept_test: bad argument");
    const bool greedy = !(sp->temperature > 0.0f);
    SD_CHECK(greedy || (pnuc && qnuc && ep && eq), SPECDEC_EINVAL, "shard_accept_test: statistics required");
    if (B == 0) return SPECDEC_OK;
    shard_accept_test_kernel<<<(B + 127) / 128, 128, 0, as_stream(stream)>>>(
        drafts, B, k, greedy, sp->seed, step_dev, sp->step, parg, reinterpret_cast<const unsigned long long*>(pnuc),
        reinterpret_cast<const unsigned long long*>(qnuc), reinterpret_cast<const unsigned long long*>(ep),
        reinterpret_cast<const unsigned long long*>(eq), accepted);
    SD_LAUNCH_CHECK("shard_accept_test_kernel");
    return SPECDEC_OK;
}

static ShardRows shard_rows(const float* target, const float* draft, int k, int Vs, int v0, float temperature,
                            const float* pmax, const uint32_t* ptau, const float* qmax, const uint32_t* qtau,
                            const uint64_t* pnuc, const uint64_t* qnuc) {
    ShardRows sr;
    sr.target = target;
    sr.draft = draft;
    sr.k = k;
    sr.Vs = Vs;
    sr.v0 = v0;
    sr.c = temp_coeff(temperature);
    sr.pmax = pmax;
    sr.ptau = ptau;
    sr.qmax = qmax;
    sr.qtau = qtau;
    sr.pnuc = reinterpret_cast<const unsigned long long*>(pnuc);
    sr.qnuc = reinterpret_cast<const unsigned long long*>(qnuc);
    return sr;
}

extern "C" int specdec_shard_draw_winners(const float* target, const float* draft, int B, int k, int Vs, int v0,
                                         const specdec_sampling* sp, const int32_t* accepted, const float* pmax,
                                         const uint32_t* ptau, const float* qmax, const uint32_t* qtau,
                                         const uint64_t* pnuc, const uint64_t* qnuc, int32_t* out_win,
                                         const uint32_t* step_dev, void* stream) {
    if (int rc = shard_check(B, Vs, "shard_draw_winners")) return rc;
    SD_CHECK(target && draft && sp && accepted && pmax && ptau && qmax && qtau && pnuc && qnuc && out_win && k >= 1 &&
                 v0 >= 0 && sp->temperature > 0.0f,
             SPECDEC_EINVAL, "shard_draw_winners: bad argument");
    if (B == 0) return SPECDEC_OK;
    shard_draw_winners_kernel<<<B, shard_threads(Vs), 0, as_stream(stream)>>>(
        shard_rows(target, draft, k, Vs, v0, sp->temperature, pmax, ptau, qmax, qtau, pnuc, qnuc), accepted, sp->seed,
        step_dev, sp->step, out_win);
    SD_LAUNCH_CHECK("shard_draw_winners_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_shard_draw_merge(const int32_t* gwin, int W, int B, int k, const int32_t* accepted,
                                        int32_t* tok_out, void* stream) {
    SD_CHECK(gwin && accepted && tok_out && W >= 1 && B >= 0 && k >= 0, SPECDEC_EINVAL,
             "shard_draw_merge: bad argument");
    if (B == 0) return SPECDEC_OK;
    shard_draw_merge_kernel<<<(B + 127) / 128, 128, 0, as_stream(stream)>>>(gwin, W, B, k, accepted, tok_out);
    SD_LAUNCH_CHECK("shard_draw_merge_kernel");
    return SPECDEC_OK;
}

extern "C" int specdec_compat_verify(const float* logits, const int32_t* drafts, const int32_t* lens, int V,
                                     int max_draft, int B, int32_t* accepted, int32_t* replacement, void* stream) {
    SD_CHECK(logits && drafts && lens && accepted && replacement, SPECDEC_EINVAL, "compat_verify: null argument");
    SD_CHECK(V > 0 && max_draft > 0 && B >= 0, SPECDEC_EINVAL, "compat_verify: bad shape");
    if (B == 0) return SPECDEC_OK;
    cudaStream_t s = as_stream(stream);
    int32_t* best = nullptr;
    SD_CUDA(cudaMallocAsync(&best, sizeof(int32_t) * (size_t)B * max_draft, s));
    compat_argmax_kernel<<<B * max_draft, 256, 0, s>>>(logits, lens, V, max_draft, best);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
        compat_count_kernel<<<(B + 127) / 128, 128, 0, s>>>(best, drafts, lens, max_draft, B, accepted, replacement);
        e = cudaGetLastError();
    }
    cudaFreeAsync(best, s);
    if (e != cudaSuccess) return cuda_status(e, "compat_verify");
    return SPECDEC_OK;
}
