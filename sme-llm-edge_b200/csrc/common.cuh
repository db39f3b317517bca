// common.cuh -- shared device helpers for libspecdec_sm100 (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "specdec.h"

namespace specdec {

// ------------------------------------------------------------ host errors
void set_error(const std::string& msg);
int cuda_status(cudaError_t e, const char* what);
#define SD_CUDA(call)                                                   \
    do {                                                                \
        cudaError_t _e = (call);                                        \
        if (_e != cudaSuccess) return ::specdec::cuda_status(_e, #call); \
    } while (0)
#define SD_CHECK(cond, code, msg)          \
    do {                                   \
        if (!(cond)) {                     \
            ::specdec::set_error(msg);     \
            return (code);                 \
        }                                  \
    } while (0)
#define SD_LAUNCH_CHECK(what)                                                          \
    do {                                                                               \
        cudaError_t _e = cudaGetLastError();                                           \
        if (_e != cudaSuccess) return ::specdec::cuda_status(_e, what);                \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Device-side error word (bounded waits that give up record here).
struct DeviceStatus {
    int code;
    int where;
};
DeviceStatus* device_status_ptr();  // per-device, allocated on first use
int check_device_status(cudaStream_t s);

// --------------------------------------------------------- device helpers
typedef unsigned __int128 u128;

__device__ __forceinline__ void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                              uint32_t k1, uint32_t out[4]) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

// Uniform streams: ctr = {b, i, purpose, step}, key = seed.  The accept tests
// use one uniform per test; the draws one per element (gumbel.cuh, purposes 3
// and 4 with the element group in the counter's third word).
enum { U_ACCEPT = 1 };

__device__ __forceinline__ uint32_t uniform_u32(uint64_t seed, uint32_t step, uint32_t b, uint32_t i, uint32_t purpose) {
    uint32_t o[4];
    philox4x32_10(b, i, purpose, step, (uint32_t)seed, (uint32_t)(seed >> 32), o);
    return o[0];
}

// floor(2^t * 2^31), t <= 0: rint range reduction, degree-7 Taylor polynomial
// of e^(f ln 2) in Horner form with fused multiply-adds, exact 2^e scaling.
// The identical operation sequence runs in the host oracle.
__device__ __forceinline__ uint32_t exp2_fx31(float t) {
    if (!(t <= 0.0f)) t = 0.0f;
    if (t < -40.0f) return 0u;
    const float n = rintf(t);
    const float f = __fsub_rn(t, n);
    const float x = __fmul_rn(f, 0x1.62e43p-1f);  // ln 2
    float p = 0x1.a01a02p-13f;                         // 1/7!
    p = __fmaf_rn(p, x, 0x1.6c16c2p-10f);              // 1/6!
    p = __fmaf_rn(p, x, 0x1.111112p-7f);               // 1/5!
    p = __fmaf_rn(p, x, 0x1.555556p-5f);               // 1/4!
    p = __fmaf_rn(p, x, 0x1.555556p-3f);               // 1/3!
    p = __fmaf_rn(p, x, 0x1p-1f);                      // 1/2!
    p = __fmaf_rn(p, x, 0x1p+0f);
    p = __fmaf_rn(p, x, 0x1p+0f);
    const int e = (int)n + 31;
    if (e < 0) return 0u;
    const float v = __fmul_rn(p, __int_as_float((e + 127) << 23));
    return (uint32_t)v;
}

// exp2_fx31 for t <= 0 or t = -inf (no NaN), without branches and with
// the rounding of t done by the 1.5 * 2^23 addition (round to nearest even,
// the mode of rintf) instead of conversion instructions: identical results.
// t is clamped at -40 (below -31.5 the exponent e = n + 31 is negative and
// p * 2^e < 1 truncates to 0, the value exp2_fx31 returns there).
__device__ __forceinline__ uint32_t exp2_fx31_neg(float t) {
    t = fmaxf(t, -40.0f);
    const float big = __fadd_rn(t, 0x1.8p23f);
    const float n = __fsub_rn(big, 0x1.8p23f);
    const int ni = __float_as_int(big) - 0x4B400000;
    const float f = __fsub_rn(t, n);
    const float x = __fmul_rn(f, 0x1.62e43p-1f);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, x, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, x, 0x1.111112p-7f);
    p = __fmaf_rn(p, x, 0x1.555556p-5f);
    p = __fmaf_rn(p, x, 0x1.555556p-3f);
    p = __fmaf_rn(p, x, 0x1p-1f);
    p = __fmaf_rn(p, x, 0x1p+0f);
    p = __fmaf_rn(p, x, 0x1p+0f);
    return (uint32_t)__fmul_rn(p, __int_as_float((ni + 31 + 127) << 23));  // ni + 31 >= -9
}

__device__ __forceinline__ uint32_t logit_key(float z) {
    uint32_t b = __float_as_uint(z);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ uint64_t mulhi64(uint64_t a, uint64_t b) { return __umul64hi(a, b); }

// ---------------------------------------------------------- reductions
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ u128 shfl_xor_u128(u128 v, int o) {
    uint64_t lo = (uint64_t)v, hi = (uint64_t)(v >> 64);
    lo = __shfl_xor_sync(0xffffffffu, lo, o);
    hi = __shfl_xor_sync(0xffffffffu, hi, o);
    return ((u128)hi << 64) | lo;
}
__device__ __forceinline__ u128 warp_sum_u128(u128 v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += shfl_xor_u128(v, o);
    return v;
}

// Block-wide sum; `scratch` holds >= 32 entries of T.  All threads get the result.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    T r = (lane < nw) ? scratch[lane] : (T)0;
    r = warp_sum(r);
    return r;
}
__device__ __forceinline__ u128 block_sum_u128(u128 v, u128* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_u128(v);
    __syncthreads();
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    u128 r = (lane < nw) ? scratch[lane] : (u128)0;
    r = warp_sum_u128(r);
    return r;
}
__device__ __forceinline__ float block_max(float v, float* scratch) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    float r = (lane < nw) ? scratch[lane] : -INFINITY;
    return warp_max(r);
}

// Bounded spin limit for device-side waits (mbarrier polls).
constexpr uint32_t kSpinLimit = 1u << 26;

}  // namespace specdec
