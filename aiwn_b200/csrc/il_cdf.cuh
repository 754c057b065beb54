// il_cdf.cuh -- the GaussianCDFNorm prologue of IndexedLinearV2
// (aiwn/layers/indexed_linear_v2.py:19-37, used at :80-88):
//
//   z  = LayerNorm(x) = (x - mean) * rstd * gamma + beta     (over in_d, eps)
//   xn = 2 * (0.5 * (1 + erf(z / sqrt(2)))) - 1              in [-1, 1]
//
// computed in the reference's fp32 operation order (the scalar sqrt(2) is the
// fp32 value 1.41421354; u and 2u - 1 are rounded separately, so xn carries
// the reference's quantisation near 0).  erf is CUDA's erff.
//
//   * fwd_token_cdf_kernel: the one-token-per-lane forward with the prologue
//     fused into it -- a lane loads its token's x row (in_d <= 32) into
//     registers once, takes its mean and variance, maps every value to xn and
//     buckets it.  The CTAs of j-range 0 write xn, mean and rstd, which the
//     backward needs.
//   * cdf_prologue_kernel: the same map as a standalone pass, for shapes the
//     fused kernel does not cover; the forward then runs on xn.
//   * cdf_backward_kernel: autograd's backward of the prologue given the
//     gradient with respect to xn: dx, dgamma, dbeta.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "il_common.cuh"
#include "il_fast.cuh"
#include "il_fwd_token.cuh"
#include "il_sm100.cuh"

namespace il {

constexpr float kSqrt2F = 1.41421354f;  // fp32 value of math.sqrt(2.0)

struct CdfArgs {
    const float* gamma;
    const float* beta;
    float eps;
    float* xn;    // [N, IN], may be null in the fused forward
    float* mean;  // [N]
    float* rstd;  // [N]
};

__device__ __forceinline__ float cdf_map(float xv, float mean, float rstd, float g, float b) {
    const float z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv, mean), rstd), g), b);
    const float e = erff(__fdiv_rn(z, kSqrt2F));
    const float u = __fmul_rn(0.5f, __fadd_rn(1.0f, e));
    return __fsub_rn(__fmul_rn(u, 2.0f), 1.0f);
}

// mean and 1/sqrt(var + eps) of n values (biased variance, two passes)
template <int MAXN>
__device__ __forceinline__ void row_stats(const float (&v)[MAXN], int n, float eps, float& mean, float& rstd) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < MAXN; ++k)
        if (k < n) s = __fadd_rn(s, v[k]);
    mean = __fdiv_rn(s, (float)n);
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < MAXN; ++k)
        if (k < n) {
            const float d = __fsub_rn(v[k], mean);
            q = __fadd_rn(q, __fmul_rn(d, d));
        }
    rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, (float)n), eps)));
}

// ---------------------------------------------------------------------------
// fused forward (fp32 x, in_d <= kCdfMaxIn): fwd_token_kernel with the prologue
// ---------------------------------------------------------------------------
constexpr int kCdfMaxIn = 32;
constexpr int kCdfThreads = 512;

template <int C>
__global__ void __launch_bounds__(kCdfThreads, 1)
    fwd_token_cdf_kernel(const __grid_constant__ CUtensorMap tmap, const FwdArgs p, const CdfArgs q) {
    extern __shared__ unsigned char smem[];
    const int IN = p.IN;
    const int j0 = blockIdx.y * p.JR;
    const uint32_t table_s = (smem_addr(smem) + 127u) & ~127u;
    // the slices load as in fwd_token_kernel: blocks of kTokXB columns, one
    // mbarrier each, kTokAhead blocks in flight, waited for in the first pass
    const int nbar = (IN + kTokXB - 1) / kTokXB;
    const uint32_t bar0 = table_s + (uint32_t)(IN * p.slice_bytes);
    const uint32_t row_bytes = (uint32_t)p.RS * 4;
    const uint32_t box_bytes = (uint32_t)(p.KB * p.RS * 4);
    auto issue_block = [&](int g) {
        const uint32_t bar = bar0 + 8u * (uint32_t)g;
        const int s1 = min(IN, (g + 1) * kTokXB);
        mbar_arrive_expect_tx(bar, (uint32_t)((s1 - g * kTokXB) * p.nbox) * box_bytes);
        for (int s = g * kTokXB; s < s1; ++s)
            for (int b = 0; b < p.nbox; ++b)
                tma_load_3d(table_s + s * p.slice_bytes + b * box_bytes, &tmap, bar, j0, s, b * p.KB);
    };

    if (threadIdx.x == 0) {
        prefetch_tensormap(&tmap);
        for (int g = 0; g < nbar; ++g) mbar_init(bar0 + 8u * (uint32_t)g, 1);
        fence_mbar_init();
        for (int g = 0; g < min(nbar, kTokAhead); ++g) issue_block(g);
    }

    const int r0 = blockIdx.x * p.ntiles;  // this CTA's token range (ntiles = its length)
    const int r1 = min(p.N, r0 + p.ntiles);
    const float* x = reinterpret_cast<const float*>(p.x);
    const bool writer = blockIdx.y == 0;
    // gamma, beta staged after the mbarriers (bytes [gb, gb + 8*kCdfMaxIn))
    const uint32_t gb_addr = bar0 + 8u * (uint32_t)nbar;
    float* gb_s = reinterpret_cast<float*>(smem + (gb_addr - smem_addr(smem)));
    for (int k = threadIdx.x; k < IN; k += kCdfThreads) {
        gb_s[k] = q.gamma[k];
        gb_s[kCdfMaxIn + k] = q.beta[k];
    }
    __syncthreads();  // gamma, beta staged; the mbarriers are initialised
    // Every thread makes at least one pass (r0 < r1), so it waits for every
    // block of slices before it exits, and thread 0 issues every block.
    bool first = true;
    for (int n = r0 + (int)threadIdx.x; n - (int)threadIdx.x < r1; n += kCdfThreads) {
        const bool ok = n < r1;
        float v[kCdfMaxIn];
        if (p.xvec) {  // rows of 4-aligned floats: 16-byte loads
#pragma unroll
            for (int k = 0; k < kCdfMaxIn; k += 4) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                if (ok && k < IN) t = __ldg(reinterpret_cast<const float4*>(x + (int64_t)n * IN + k));
                v[k] = t.x;
                v[k + 1] = t.y;
                v[k + 2] = t.z;
                v[k + 3] = t.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < kCdfMaxIn; ++k) v[k] = (ok && k < IN) ? __ldg(x + (int64_t)n * IN + k) : 0.0f;
        }
        float mean, rstd;
        row_stats(v, IN, q.eps, mean, rstd);
#pragma unroll
        for (int k = 0; k < kCdfMaxIn; ++k)
            if (k < IN) v[k] = cdf_map(v[k], mean, rstd, gb_s[k], gb_s[kCdfMaxIn + k]);
        if (writer && ok) {
            q.mean[n] = mean;
            q.rstd[n] = rstd;
            if (q.xn) {
                if (p.xvec) {
#pragma unroll
                    for (int k = 0; k < kCdfMaxIn; k += 4)
                        if (k < IN)
                            *reinterpret_cast<float4*>(q.xn + (int64_t)n * IN + k) =
                                make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
                } else {
#pragma unroll
                    for (int k = 0; k < kCdfMaxIn; ++k)
                        if (k < IN) q.xn[(int64_t)n * IN + k] = v[k];
                }
            }
        }
        float4 acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < kCdfMaxIn; ++s) {
            if (s >= IN) break;
            if (first && s % kTokXB == 0) {
                const int g = s / kTokXB;
                mbar_wait_bounded(bar0 + 8u * (uint32_t)g, 0);
                if (threadIdx.x == 0 && g + kTokAhead < nbar) issue_block(g + kTokAhead);
                // row K = row K-1 (the top bin's hi row), written by every
                // thread before its own first read; TMA never writes row K
                for (int t = s; t < min(IN, s + kTokXB); ++t) {
                    const uint32_t sl = table_s + (uint32_t)(t * p.slice_bytes) + (uint32_t)(p.K - 1) * row_bytes;
#pragma unroll
                    for (int c = 0; c < C; ++c) sts_v4(sl + row_bytes + c * 16, lds_v4(sl + c * 16));
                }
            }
            int lo;
            float wa, wc;
            gather_weights<kF32>(v[s], p.cfg, lo, wa, wc);
            const uint32_t row = table_s + (uint32_t)(s * p.slice_bytes) + (uint32_t)lo * row_bytes;
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const float4 tl = lds_v4(row + c * 16);
                const float4 th = lds_v4(row + row_bytes + c * 16);
                acc[c].x = fmaf(wa, tl.x, acc[c].x);
                acc[c].y = fmaf(wa, tl.y, acc[c].y);
                acc[c].z = fmaf(wa, tl.z, acc[c].z);
                acc[c].w = fmaf(wa, tl.w, acc[c].w);
                acc[c].x = fmaf(wc, th.x, acc[c].x);
                acc[c].y = fmaf(wc, th.y, acc[c].y);
                acc[c].z = fmaf(wc, th.z, acc[c].z);
                acc[c].w = fmaf(wc, th.w, acc[c].w);
            }
        }
        first = false;
        if (ok) {
            float4* o = reinterpret_cast<float4*>(p.out + (int64_t)n * p.OUT + j0);
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + j0) + c);
                o[c] = make_float4(acc[c].x + b.x, acc[c].y + b.y, acc[c].z + b.z, acc[c].w + b.w);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// standalone prologue and the prologue's backward (any in_d, fp32)
// ---------------------------------------------------------------------------
constexpr int kCdfRowThreads = 256;

// one thread per token: two passes over its row for the statistics, one for xn
__global__ void __launch_bounds__(kCdfRowThreads) cdf_prologue_kernel(const float* x, CdfArgs q, int N, int IN) {
    const int n = blockIdx.x * kCdfRowThreads + threadIdx.x;
    if (n >= N) return;
    const float* r = x + (int64_t)n * IN;
    float s = 0.f;
    for (int k = 0; k < IN; ++k) s = __fadd_rn(s, r[k]);
    const float mean = __fdiv_rn(s, (float)IN);
    float qq = 0.f;
    for (int k = 0; k < IN; ++k) {
        const float d = __fsub_rn(r[k], mean);
        qq = __fadd_rn(qq, __fmul_rn(d, d));
    }
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(qq, (float)IN), q.eps)));
    q.mean[n] = mean;
    q.rstd[n] = rstd;
    for (int k = 0; k < IN; ++k) q.xn[(int64_t)n * IN + k] = cdf_map(r[k], mean, rstd, q.gamma[k], q.beta[k]);
}

// The prologue for in_d <= MAXIN with the row in registers and 16-byte loads
// and stores when rows are 4-aligned.  With CDF = false it is a plain
// LayerNorm: xn receives the affine output (x - mean) * rstd * gamma + beta.
template <int MAXIN, bool CDF = true>
__global__ void __launch_bounds__(kCdfRowThreads)
    cdf_prologue_small_kernel(const float* x, CdfArgs q, int N, int IN, int vec) {
    const int n = blockIdx.x * kCdfRowThreads + threadIdx.x;
    if (n >= N) return;
    const float* r = x + (int64_t)n * IN;
    float v[MAXIN];
    if (vec) {
#pragma unroll
        for (int k = 0; k < MAXIN; k += 4) {
            float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < IN) t = __ldg(reinterpret_cast<const float4*>(r + k));
            v[k] = t.x, v[k + 1] = t.y, v[k + 2] = t.z, v[k + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int k = 0; k < MAXIN; ++k) v[k] = k < IN ? __ldg(r + k) : 0.f;
    }
    float mean, rstd;
    row_stats(v, IN, q.eps, mean, rstd);
    q.mean[n] = mean;
    q.rstd[n] = rstd;
#pragma unroll
    for (int k = 0; k < MAXIN; ++k)
        if (k < IN) {
            if constexpr (CDF)
                v[k] = cdf_map(v[k], mean, rstd, __ldg(q.gamma + k), __ldg(q.beta + k));
            else
                v[k] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[k], mean), rstd), __ldg(q.gamma + k)),
                                 __ldg(q.beta + k));
        }
    float* o = q.xn + (int64_t)n * IN;
    if (vec) {
#pragma unroll
        for (int k = 0; k < MAXIN; k += 4)
            if (k < IN) *reinterpret_cast<float4*>(o + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
    } else {
#pragma unroll
        for (int k = 0; k < MAXIN; ++k)
            if (k < IN) o[k] = v[k];
    }
}

// Autograd's backward of the prologue, one thread per token, given gxn = dL/dxn:
//   s = z / sqrt(2):  dz = (gxn * 2/sqrt(pi) * exp(-s^2)) / sqrt(2)
//   dgamma += dz * xhat,  dbeta += dz,  dxhat = dz * gamma
//   dx = rstd * (dxhat - mean(dxhat) - xhat * mean(dxhat * xhat))
// dgamma / dbeta are summed per block in shared memory, then added to the
// (zeroed) outputs with one atomic per column and block.
__global__ void __launch_bounds__(kCdfRowThreads)
    cdf_backward_kernel(const float* gxn, const float* x, const float* gamma, const float* beta, const float* mean,
                        const float* rstd, float* dx, float* dgamma, float* dbeta, int N, int IN) {
    extern __shared__ float sacc[];  // [2 * IN]: dgamma, dbeta partial sums of this block
    for (int k = threadIdx.x; k < 2 * IN; k += kCdfRowThreads) sacc[k] = 0.f;
    __syncthreads();
    const int n = blockIdx.x * kCdfRowThreads + threadIdx.x;
    if (n < N) {
        const float* r = x + (int64_t)n * IN;
        const float* g = gxn + (int64_t)n * IN;
        const float m = mean[n], rs = rstd[n];
        float s1 = 0.f, s2 = 0.f;
        for (int k = 0; k < IN; ++k) {
            const float xh = __fmul_rn(__fsub_rn(r[k], m), rs);
            const float z = __fadd_rn(__fmul_rn(xh, gamma[k]), beta[k]);
            const float sv = __fdiv_rn(z, kSqrt2F);
            const float dz = __fdiv_rn(__fmul_rn(__fmul_rn(g[k], 1.12837916709551257f), expf(-__fmul_rn(sv, sv))),
                                       kSqrt2F);
            const float dxh = __fmul_rn(dz, gamma[k]);
            s1 += dxh;
            s2 += dxh * xh;
            if (dgamma) atomicAdd(&sacc[k], dz * xh);
            if (dbeta) atomicAdd(&sacc[IN + k], dz);
        }
        if (dx) {
            const float a1 = s1 / (float)IN, a2 = s2 / (float)IN;
            for (int k = 0; k < IN; ++k) {
                const float xh = __fmul_rn(__fsub_rn(r[k], m), rs);
                const float z = __fadd_rn(__fmul_rn(xh, gamma[k]), beta[k]);
                const float sv = __fdiv_rn(z, kSqrt2F);
                const float dz =
                    __fdiv_rn(__fmul_rn(__fmul_rn(g[k], 1.12837916709551257f), expf(-__fmul_rn(sv, sv))), kSqrt2F);
                const float dxh = __fmul_rn(dz, gamma[k]);
                dx[(int64_t)n * IN + k] = rs * (dxh - a1 - xh * a2);
            }
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < IN; k += kCdfRowThreads) {
        if (dgamma) atomicAdd(dgamma + k, sacc[k]);
        if (dbeta) atomicAdd(dbeta + k, sacc[IN + k]);
    }
}

// The same backward for in_d <= kCdfMaxIn with the rows in registers: one
// pass per token (16-byte loads when rows are 4-aligned), a grid-stride loop
// over tokens, dgamma / dbeta partial sums in registers, reduced over the warp
// by shuffles and over the block with one shared atomic per warp and column.
// With CDF = false it is a plain LayerNorm's backward: gxn is the gradient of
// the affine output itself (beta is not read).
template <int MAXIN, bool CDF = true>
__global__ void __launch_bounds__(kCdfRowThreads)
    cdf_backward_small_kernel(const float* gxn, const float* x, const float* gamma, const float* beta,
                              const float* mean, const float* rstd, float* dx, float* dgamma, float* dbeta, int N,
                              int IN, int vec) {
    __shared__ float sacc[2 * MAXIN];
    __shared__ float sgb[2 * MAXIN];
    for (int k = threadIdx.x; k < 2 * MAXIN; k += kCdfRowThreads) sacc[k] = 0.f;
    for (int k = threadIdx.x; k < IN; k += kCdfRowThreads) {
        sgb[k] = gamma[k];
        sgb[MAXIN + k] = CDF ? beta[k] : 0.f;
    }
    __syncthreads();
    float ag[MAXIN], ab[MAXIN];
#pragma unroll
    for (int k = 0; k < MAXIN; ++k) ag[k] = ab[k] = 0.f;
    for (int n = blockIdx.x * kCdfRowThreads + threadIdx.x; n < N; n += gridDim.x * kCdfRowThreads) {
        float xv[MAXIN], gv[MAXIN];
        const float* r = x + (int64_t)n * IN;
        const float* g = gxn + (int64_t)n * IN;
        if (vec) {
#pragma unroll
            for (int k = 0; k < MAXIN; k += 4) {
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
                if (k < IN) {
                    a = __ldg(reinterpret_cast<const float4*>(r + k));
                    b = __ldg(reinterpret_cast<const float4*>(g + k));
                }
                xv[k] = a.x, xv[k + 1] = a.y, xv[k + 2] = a.z, xv[k + 3] = a.w;
                gv[k] = b.x, gv[k + 1] = b.y, gv[k + 2] = b.z, gv[k + 3] = b.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < MAXIN; ++k) {
                xv[k] = k < IN ? __ldg(r + k) : 0.f;
                gv[k] = k < IN ? __ldg(g + k) : 0.f;
            }
        }
        const float m = mean[n], rs = rstd[n];
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int k = 0; k < MAXIN; ++k) {
            if (k < IN) {
                const float xh = __fmul_rn(__fsub_rn(xv[k], m), rs);
                float dz = gv[k];
                if constexpr (CDF) {
                    const float z = __fadd_rn(__fmul_rn(xh, sgb[k]), sgb[MAXIN + k]);
                    const float sv = __fdiv_rn(z, kSqrt2F);
                    dz = __fdiv_rn(__fmul_rn(__fmul_rn(gv[k], 1.12837916709551257f), expf(-__fmul_rn(sv, sv))),
                                   kSqrt2F);
                }
                const float dxh = __fmul_rn(dz, sgb[k]);
                s1 += dxh;
                s2 += dxh * xh;
                ag[k] += dz * xh;
                ab[k] += dz;
                xv[k] = xh;   // keep xhat
                gv[k] = dxh;  // keep dxhat
            }
        }
        if (dx) {
            const float a1 = s1 / (float)IN, a2 = s2 / (float)IN;
            float* o = dx + (int64_t)n * IN;
            if (vec) {
#pragma unroll
                for (int k = 0; k < MAXIN; k += 4)
                    if (k < IN)
                        *reinterpret_cast<float4*>(o + k) =
                            make_float4(rs * (gv[k] - a1 - xv[k] * a2), rs * (gv[k + 1] - a1 - xv[k + 1] * a2),
                                        rs * (gv[k + 2] - a1 - xv[k + 2] * a2), rs * (gv[k + 3] - a1 - xv[k + 3] * a2));
            } else {
#pragma unroll
                for (int k = 0; k < MAXIN; ++k)
                    if (k < IN) o[k] = rs * (gv[k] - a1 - xv[k] * a2);
            }
        }
    }
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < MAXIN; ++k) {
        if (k >= IN) break;
        float a = ag[k], b = ab[k];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            a += __shfl_xor_sync(0xffffffffu, a, o);
            b += __shfl_xor_sync(0xffffffffu, b, o);
        }
        if (lane == 0) {
            atomicAdd(&sacc[k], a);
            atomicAdd(&sacc[MAXIN + k], b);
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < IN; k += kCdfRowThreads) {
        if (dgamma) atomicAdd(dgamma + k, sacc[k]);
        if (dbeta) atomicAdd(dbeta + k, sacc[MAXIN + k]);
    }
}

// ---------------------------------------------------------------------------
// host side of the fused forward
// ---------------------------------------------------------------------------
template <int C>
inline int launch_token_cdf(const CUtensorMap& map, const FwdArgs& a, const CdfArgs& q, const FwdPlan& pl, int sms,
                            cudaStream_t s) {
    auto kern = fwd_token_cdf_kernel<C>;
    // slices + base alignment + mbarriers + gamma, beta
    const int smem = a.IN * pl.slice_bytes + 128 + 8 * ceil_div(a.IN, kTokXB) + 2 * kCdfMaxIn * 4;
    if (smem > kSmemBudget) return kNotApplicable;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return 4;
    const int jranges = ceil_div(a.OUT, pl.JR);
    const int max_ranges = std::max(1, sms / jranges);
    const int per = std::max(32, round_up(ceil_div(a.N, max_ranges), 32));
    FwdArgs b = a;
    b.ntiles = per;
    kern<<<dim3((unsigned)ceil_div(a.N, per), (unsigned)jranges, 1), kCdfThreads, smem, s>>>(map, b, q);
    return 0;
}

// fp32 x, in_d <= 32 and a token-forward plan; kNotApplicable otherwise
inline int token_cdf_forward(const float* x, const CdfArgs& q, const float* table, const float* bias, float* out,
                             int64_t N, int64_t IN, int64_t OUT, const BinCfg& c, int sms, cudaStream_t s) {
    if (IN > kCdfMaxIn) return kNotApplicable;
    FwdPlan pl;
    if (!plan_token_forward(N, c.K, (int)IN, (int)OUT, sms, pl)) return kNotApplicable;
    if (pl.C > 5) return kNotApplicable;  // register budget of the fused kernel
    // with several j-ranges every CTA of a token would redo the prologue: the
    // standalone pass plus the plain forward is faster then
    if (pl.JR != (int)OUT) return kNotApplicable;
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, pl.RS, pl.KB)) return kNotApplicable;
    FwdArgs a;
    a.x = x;
    a.bias = bias;
    a.out = out;
    a.N = (int)N;
    a.IN = (int)IN;
    a.OUT = (int)OUT;
    a.K = c.K;
    a.JR = pl.JR;
    a.RS = pl.RS;
    a.xvec = (IN % 4 == 0) && (((uintptr_t)x | (uintptr_t)q.xn) % 16 == 0);
    a.IG = pl.IG;
    a.KB = pl.KB;
    a.nbox = pl.nbox;
    a.slice_bytes = pl.slice_bytes;
    a.ntiles = 0;
    a.cfg = c;
    switch (pl.C) {
        case 5: return launch_token_cdf<5>(map, a, q, pl, sms, s);
        case 4: return launch_token_cdf<4>(map, a, q, pl, sms, s);
        case 2: return launch_token_cdf<2>(map, a, q, pl, sms, s);
        default: return launch_token_cdf<1>(map, a, q, pl, sms, s);
    }
}

}  // namespace il
