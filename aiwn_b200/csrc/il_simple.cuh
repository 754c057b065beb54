// il_simple.cuh -- general-shape IndexedLinear kernels.
//
// These handle every shape the fast kernels do not (OUT not a multiple of 4,
// misaligned pointers, very large sizes).  One thread per output element,
// 64-bit indexing, table rows read through the read-only cache.  They follow
// the reference's eager arithmetic (aiwn/layers/indexed_linear.py:173-182 and
// autograd's backward of it) in the same operation order.
#pragma once
#include "il_common.cuh"

namespace il {

// out[n, j] = sum_i ((T[lo,i,j]*(1-fr) + T[hi,i,j]*fr) * x[n,i]) + bias[j]
template <int DT>
__global__ void __launch_bounds__(256) fwd_simple_kernel(const void* __restrict__ x,
                                                         const float* __restrict__ table,
                                                         const float* __restrict__ bias,
                                                         float* __restrict__ out, int64_t N,
                                                         int64_t IN, int64_t OUT, BinCfg c) {
    const int64_t total = N * OUT;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = e / OUT, j = e - n * OUT;
        float acc = 0.0f;
        for (int64_t i = 0; i < IN; ++i) {
            Bin b = bin_of<DT>(load_x<DT>(x, n * IN + i), c);
            const int hi = min(b.lo + 1, c.K - 1);
            const float tlo = __ldg(table + ((int64_t)b.lo * IN + i) * OUT + j);
            const float thi = __ldg(table + ((int64_t)hi * IN + i) * OUT + j);
            const float w = __fadd_rn(__fmul_rn(tlo, __fsub_rn(1.0f, b.fr)), __fmul_rn(thi, b.fr));
            acc = __fadd_rn(acc, __fmul_rn(w, b.x));
        }
        out[e] = __fadd_rn(acc, __ldg(bias + j));
    }
}

// gx[n, i] = sum_j go*L + [0<=fr_pre<=1] * (sum_j (go*x)*thi - sum_j (go*x)*tlo) / bw
// (bf16 x: the two terms are rounded to bf16 separately and summed in bf16,
// as autograd accumulates the two contributions to a bf16 leaf)
template <int DT>
__global__ void __launch_bounds__(256) dx_simple_kernel(const float* __restrict__ go,
                                                        const void* __restrict__ x,
                                                        const float* __restrict__ table,
                                                        void* __restrict__ gx, int64_t N,
                                                        int64_t IN, int64_t OUT, BinCfg c) {
    const int64_t total = N * IN;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = e / IN, i = e - n * IN;
        Bin b = bin_of<DT>(load_x<DT>(x, e), c);
        const int hi = min(b.lo + 1, c.K - 1);
        const float* tlo = table + ((int64_t)b.lo * IN + i) * OUT;
        const float* thi = table + ((int64_t)hi * IN + i) * OUT;
        const float* g = go + n * OUT;
        const float omf = __fsub_rn(1.0f, b.fr);
        float t1 = 0.0f, shi = 0.0f, slo = 0.0f;
        for (int64_t j = 0; j < OUT; ++j) {
            const float gj = __ldg(g + j), lo_v = __ldg(tlo + j), hi_v = __ldg(thi + j);
            const float L = __fadd_rn(__fmul_rn(lo_v, omf), __fmul_rn(hi_v, b.fr));
            t1 = __fadd_rn(t1, __fmul_rn(gj, L));
            const float gxj = __fmul_rn(gj, b.x);
            shi = __fadd_rn(shi, __fmul_rn(gxj, hi_v));
            slo = __fadd_rn(slo, __fmul_rn(gxj, lo_v));
        }
        const float gfr = __fsub_rn(shi, slo);
        const float t2 = clamp_passes(b.fr_pre) ? __fdiv_rn(gfr, c.bw) : 0.0f;
        if constexpr (DT == kBF16) {
            store_gx<DT>(gx, e, __fadd_rn(bf16_round(t1), bf16_round(t2)));
        } else {
            store_gx<DT>(gx, e, __fadd_rn(t1, t2));
        }
    }
}

// gt[lo,i,j] += (go*x)*(1-fr);  gt[hi,i,j] += (go*x)*fr   (gt zeroed first)
template <int DT>
__global__ void __launch_bounds__(256) dtable_simple_kernel(const float* __restrict__ go,
                                                            const void* __restrict__ x,
                                                            float* __restrict__ gt, int64_t N,
                                                            int64_t IN, int64_t OUT, BinCfg c) {
    const int64_t total = N * IN * OUT;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = e % OUT;
        const int64_t ni = e / OUT;
        const int64_t n = ni / IN, i = ni - n * IN;
        Bin b = bin_of<DT>(load_x<DT>(x, ni), c);
        const int hi = min(b.lo + 1, c.K - 1);
        const float gxj = __fmul_rn(__ldg(go + n * OUT + j), b.x);
        atomicAdd(gt + ((int64_t)b.lo * IN + i) * OUT + j, __fmul_rn(gxj, __fsub_rn(1.0f, b.fr)));
        atomicAdd(gt + ((int64_t)hi * IN + i) * OUT + j, __fmul_rn(gxj, b.fr));
    }
}

// gb[j] = sum_n go[n, j]: each block reduces a stripe of rows for 32 columns
// (gb zeroed first).
__global__ void __launch_bounds__(256) dbias_simple_kernel(const float* __restrict__ go,
                                                           float* __restrict__ gb, int64_t N,
                                                           int64_t OUT, int64_t rows_per_block) {
    __shared__ float part[8][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t j = blockIdx.x * 32 + lane;
    const int64_t r0 = blockIdx.y * rows_per_block;
    const int64_t r1 = min(N, r0 + rows_per_block);
    float acc = 0.0f;
    if (j < OUT)
        for (int64_t n = r0 + w; n < r1; n += 8) acc += __ldg(go + n * OUT + j);
    part[w][lane] = acc;
    __syncthreads();
    if (w == 0) {
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) s += part[k][lane];
        if (j < OUT) atomicAdd(gb + j, s);
    }
}

template <int DT>
__global__ void __launch_bounds__(256) bins_kernel(const void* __restrict__ x, int64_t total,
                                                   BinCfg c, int32_t* __restrict__ lo,
                                                   int32_t* __restrict__ hi,
                                                   float* __restrict__ fr) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        Bin b = bin_of<DT>(load_x<DT>(x, e), c);
        if (lo) lo[e] = b.lo;
        if (hi) hi[e] = min(b.lo + 1, c.K - 1);
        if (fr) fr[e] = b.fr;
    }
}

// Bin-occupancy histogram: counts[k] += number of x elements whose bin lo is
// k (the bincount of aiwn/experiments/bucket_analysis.py:44-47 and of
// transformer_validation.py:105-108).  Per-CTA counters in shared memory
// (dynamic, K entries), one 64-bit atomic per bin and CTA at the end.
template <int DT>
__global__ void __launch_bounds__(256) bin_counts_kernel(const void* __restrict__ x, int64_t total, BinCfg c,
                                                         unsigned long long* __restrict__ counts) {
    extern __shared__ unsigned int hist[];
    for (int k = threadIdx.x; k < c.K; k += blockDim.x) hist[k] = 0u;
    __syncthreads();
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(&hist[bin_of<DT>(load_x<DT>(x, e), c).lo], 1u);
    __syncthreads();
    for (int k = threadIdx.x; k < c.K; k += blockDim.x)
        if (hist[k]) atomicAdd(counts + k, (unsigned long long)hist[k]);
}

// torch.optim.Adam (single-tensor order) in fp32:
//   m = m + (g - m)*(1-b1);  v = v*b2 + ((1-b2)*g)*g
//   p = p - step_size * m / (sqrt(v)/bc2_sqrt + eps)
__global__ void __launch_bounds__(256) adam_kernel(float* __restrict__ p,
                                                   const float* __restrict__ g,
                                                   float* __restrict__ m, float* __restrict__ v,
                                                   int64_t n, float b1, float b2, float eps,
                                                   float step_size, float bc2_sqrt) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n;
         k += (int64_t)gridDim.x * blockDim.x) {
        const float gk = g[k];
        float mk = m[k], vk = v[k];
        mk = __fadd_rn(mk, __fmul_rn(__fsub_rn(gk, mk), __fsub_rn(1.0f, b1)));
        vk = __fadd_rn(__fmul_rn(vk, b2), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, b2), gk), gk));
        const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vk), bc2_sqrt), eps);
        p[k] = __fsub_rn(p[k], __fmul_rn(step_size, __fdiv_rn(mk, denom)));
        m[k] = mk;
        v[k] = vk;
    }
}

}  // namespace il
