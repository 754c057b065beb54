// il_common.cuh -- device helpers shared by the IndexedLinear kernels.
//
// Bucketing restates aiwn/layers/indexed_linear.py:175-177 (IndexedLinear._eager)
// operation by operation in fp32 so that bins are bit-identical to the
// reference on every input:
//   bk = ((x + 1) / bw).long().clamp(0, K-1)
//   hi = (bk + 1).clamp(max=K-1)
//   fr = ((x - (-1 + bk.float()*bw)) / bw).clamp(0, 1)
// Every operation is written with an explicit round-to-nearest intrinsic
// (__fadd_rn, __fmul_rn, __fdiv_rn) so that the compiler cannot contract a
// multiply and an add into one FMA, which would change the rounding.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace il {

constexpr int kF32 = 0;
constexpr int kBF16 = 1;

// Scalar parameters of the bucketing.  `pow2` is set when bw is an exact
// power of two (every K that is a power of two): then a division by bw is
// the exact multiplication by inv = 1/bw and both round identically.
struct BinCfg {
    float bw;
    float inv;
    int K;
    int pow2;
};

__device__ __forceinline__ float bf16_round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float div_bw(float v, const BinCfg& c) {
    return c.pow2 ? __fmul_rn(v, c.inv) : __fdiv_rn(v, c.bw);
}

// trunc toward zero to int64 then clamp(0, K-1).  An fp32 value outside the
// int64 range (|q| >= 2^63) or NaN converts to INT64_MIN on the x86 CPUs the
// reference's .long() runs on, which the clamp maps to bin 0.
__device__ __forceinline__ int lo_from_q(float q, int K) {
    if (!(fabsf(q) < 9.2233720368547758e18f)) return 0;
    float t = fminf(fmaxf(truncf(q), 0.0f), (float)(K - 1));
    return (int)t;
}

struct Bin {
    int lo;        // low bin, hi = min(lo + 1, K - 1)
    float fr;      // clamp(fr_pre, 0, 1), NaN propagated like torch.clamp
    float fr_pre;  // unclamped fraction (the gradient mask needs it)
    float x;       // exact fp32 value of the input element
};

__device__ __forceinline__ Bin bin_from_q(float xv, float q, const BinCfg& c) {
    Bin b;
    b.lo = lo_from_q(q, c.K);
    float c0 = __fadd_rn(__fmul_rn((float)b.lo, c.bw), -1.0f);
    b.fr_pre = div_bw(__fsub_rn(xv, c0), c);
    float f = fminf(fmaxf(b.fr_pre, 0.0f), 1.0f);
    b.fr = (b.fr_pre != b.fr_pre) ? b.fr_pre : f;
    b.x = xv;
    return b;
}

__device__ __forceinline__ Bin bin_f32(float xv, const BinCfg& c) {
    float q = div_bw(__fadd_rn(xv, 1.0f), c);
    return bin_from_q(xv, q, c);
}

// bf16 x: (x + 1) and the quotient by bw are each rounded to bf16, as ATen
// evaluates reduced-precision elementwise ops (compute in fp32, round the
// result); fr uses the exact fp32 value of x (bf16 - fp32 promotes).
__device__ __forceinline__ Bin bin_bf16(float xv, const BinCfg& c) {
    float s = bf16_round(__fadd_rn(xv, 1.0f));
    float q = bf16_round(div_bw(s, c));
    return bin_from_q(xv, q, c);
}

template <int DT>
__device__ __forceinline__ float load_x(const void* x, int64_t idx) {
    if constexpr (DT == kBF16) {
        return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[idx]);
    } else {
        return reinterpret_cast<const float*>(x)[idx];
    }
}

template <int DT>
__device__ __forceinline__ Bin bin_of(float xv, const BinCfg& c) {
    if constexpr (DT == kBF16) return bin_bf16(xv, c);
    else return bin_f32(xv, c);
}

// Gradient mask of torch.clamp: the gradient passes where min <= v <= max
// (false for NaN).
__device__ __forceinline__ bool clamp_passes(float fr_pre) {
    return fr_pre >= 0.0f && fr_pre <= 1.0f;
}

template <int DT>
__device__ __forceinline__ void store_gx(void* gx, int64_t idx, float v) {
    if constexpr (DT == kBF16) {
        reinterpret_cast<__nv_bfloat16*>(gx)[idx] = __float2bfloat16_rn(v);
    } else {
        reinterpret_cast<float*>(gx)[idx] = v;
    }
}

// Device-side error word: kernels whose bounded waits give up set it, the
// host reads it back with il_check_device_status().  The library is a single
// translation unit (il_capi.cu includes every kernel header), so this is the
// one definition.
__device__ unsigned int g_il_error = 0;

constexpr unsigned int kErrTimeout = 1u;

__device__ __forceinline__ void report_error(unsigned int code) { atomicOr(&g_il_error, code); }

}  // namespace il
