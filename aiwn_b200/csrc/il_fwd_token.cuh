// il_fwd_token.cuh -- IndexedLinear forward with one token per lane.
//
//   out[n, j0:j0+JR] = bias + sum_i  x(1-fr) T[lo,i,j0:j0+JR] + x fr T[lo+1,i,j0:j0+JR]
//
// (aiwn/layers/indexed_linear.py:173-182; bins bit-exact as in
// gather_weights).  A CTA owns one j-range of JR = 4*C output columns and
// keeps the slices T[:, i, j0:j0+JR] of ALL input columns resident in shared
// memory (TMA tensor copies, one extra row K = row K-1 per slice so that row
// lo+1 always exists).  Each lane then handles one token on its own: it
// computes the bins of its token's x values and reads the 2*C 16-byte chunks
// of rows lo and lo+1 with 128-bit shared loads, accumulating JR outputs in
// registers.  Nothing is exchanged between lanes or CTAs; the price is that
// the OUT/JR CTAs of a token range each bin the token's x values.
//
// Shared-memory gathers from 32 random rows per warp instruction need ~7.4
// wavefronts for 32 chunks (4 when conflict-free): that, not HBM, bounds the
// kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "il_common.cuh"
#include "il_fast.cuh"
#include "il_sm100.cuh"

namespace il {

constexpr int kTokXB = 4;     // input columns per x block (prefetched one block ahead)
constexpr int kTokAhead = 2;  // blocks of table slices in flight during the first pass

// threads per CTA (one token each): more warps hide latency where the
// per-token state is small
__host__ __device__ constexpr int tok_threads(int C) { return C <= 2 ? 1024 : 512; }

// Each CTA owns the contiguous token range [blockIdx.x * p.ntiles, ...) of
// p.ntiles tokens (here `ntiles` is the range length) and walks it in steps of
// one token per thread, so that the work per SM is balanced to the token.
//
// With CNT the kernel also adds the bin-occupancy histogram of x into
// p.counts (the bincount of aiwn/experiments/bucket_analysis.py:44-47 and
// transformer_validation.py:105-108): CTA (range, j-range y) counts input
// columns i with i % gridDim.y == y, so every (token, column) is counted once
// and the counting is spread over all CTAs, into K shared-memory counters
// flushed with one 64-bit atomic per non-empty bin.
template <int DT, int C, bool CNT>
__global__ void __launch_bounds__(tok_threads(C), 1)
    fwd_token_kernel(const __grid_constant__ CUtensorMap tmap, const FwdArgs p) {
    constexpr int kTokThreads = tok_threads(C);
    extern __shared__ unsigned char smem[];
    const int IN = p.IN;
    const int j0 = blockIdx.y * p.JR;
    const uint32_t table_s = (smem_addr(smem) + 127u) & ~127u;
    // One mbarrier per block of kTokXB input columns.  Thread 0 keeps
    // kTokAhead blocks in flight and issues block g + kTokAhead once block g
    // has landed, so that the blocks arrive one after another and the first
    // pass over the tokens works on block g while the next ones load.
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

    // bin counters (CNT) after the mbarriers
    unsigned int* scnt = reinterpret_cast<unsigned int*>(smem + (bar0 + 8u * (uint32_t)nbar - smem_addr(smem)));
    if constexpr (CNT)
        for (int k = threadIdx.x; k < p.K; k += kTokThreads) scnt[k] = 0u;
    if (threadIdx.x == 0) {
        prefetch_tensormap(&tmap);
        for (int g = 0; g < nbar; ++g) mbar_init(bar0 + 8u * (uint32_t)g, 1);
        fence_mbar_init();
        for (int g = 0; g < min(nbar, kTokAhead); ++g) issue_block(g);
    }
    __syncthreads();  // the mbarriers are initialised

    const int r0 = blockIdx.x * p.ntiles;
    const int r1 = min(p.N, r0 + p.ntiles);
    // x values of block (token n, columns [sb, sb+kTokXB))
    static_assert(kTokXB == 4, "vector x loads read 4 elements");
    auto load_block = [&](int n, int sb, float (&dst)[kTokXB]) {
        const bool ok = n < r1;
        const int64_t at = (int64_t)n * IN + sb;
        if (p.xvec) {  // one 16-byte (fp32) or 8-byte (bf16) load
            if constexpr (DT == kBF16) {
                uint2 v = ok ? __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p.x) + at))
                             : make_uint2(0u, 0u);
                dst[0] = __uint_as_float(v.x << 16);
                dst[1] = __uint_as_float(v.x & 0xffff0000u);
                dst[2] = __uint_as_float(v.y << 16);
                dst[3] = __uint_as_float(v.y & 0xffff0000u);
            } else {
                const float4 v = ok ? __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + at))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                dst[0] = v.x;
                dst[1] = v.y;
                dst[2] = v.z;
                dst[3] = v.w;
            }
        } else {
#pragma unroll
            for (int q = 0; q < kTokXB; ++q) dst[q] = (ok && sb + q < IN) ? load_x<DT>(p.x, at + q) : 0.0f;
        }
    };
    float xpre[kTokXB];
    load_block(r0 + (int)threadIdx.x, 0, xpre);

    // Every thread makes at least one pass (r0 < r1), so it waits for every
    // block of slices before it exits, and thread 0 issues every block.
    bool first = true;
    for (int n = r0 + (int)threadIdx.x; n - (int)threadIdx.x < r1; n += kTokThreads) {
        float4 acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sb = 0; sb < IN; sb += kTokXB) {
            if (first) {
                const int g = sb / kTokXB;
                mbar_wait_bounded(bar0 + 8u * (uint32_t)g, 0);
                if (threadIdx.x == 0 && g + kTokAhead < nbar) issue_block(g + kTokAhead);
                // row K of these slices = row K-1 (the top bin's hi row).  Each
                // thread writes it before its own first read; all write the
                // same values, and TMA never writes row K.
                for (int s = sb; s < min(IN, sb + kTokXB); ++s) {
                    const uint32_t sl = table_s + (uint32_t)(s * p.slice_bytes) + (uint32_t)(p.K - 1) * row_bytes;
#pragma unroll
                    for (int c = 0; c < C; ++c) sts_v4(sl + row_bytes + c * 16, lds_v4(sl + c * 16));
                }
            }
            float xv[kTokXB];
#pragma unroll
            for (int q = 0; q < kTokXB; ++q) xv[q] = xpre[q];
            if (sb + kTokXB < IN) load_block(n, sb + kTokXB, xpre);
            else load_block(n + kTokThreads, 0, xpre);
#pragma unroll
            for (int q = 0; q < kTokXB; ++q) {
                if (sb + q >= IN) break;
                int lo;
                float wa, wc;
                gather_weights<DT>(xv[q], p.cfg, lo, wa, wc);
                if constexpr (CNT)
                    if (n < r1 && (sb + q) % (int)gridDim.y == (int)blockIdx.y) atomicAdd(scnt + lo, 1u);
                const uint32_t row = table_s + (uint32_t)((sb + q) * p.slice_bytes) + (uint32_t)lo * row_bytes;
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
        }
        first = false;
        if (n < r1) {
            float4* o = reinterpret_cast<float4*>(p.out + (int64_t)n * p.OUT + j0);
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + j0) + c);
                o[c] = make_float4(acc[c].x + b.x, acc[c].y + b.y, acc[c].z + b.z, acc[c].w + b.w);
            }
        }
    }
    if constexpr (CNT) {
        __syncthreads();
        for (int k = threadIdx.x; k < p.K; k += kTokThreads)
            if (scnt[k]) atomicAdd(p.counts + k, (unsigned long long)scnt[k]);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr int kTokChunks[] = {8, 5, 4, 2, 1};

// j-range width: the widest whose slices of every input column fit one CTA's
// shared memory, narrowed while the token ranges alone would leave SMs idle
// (a narrower j-range gives more CTAs per token range)
inline bool plan_token_forward(int64_t N, int K, int IN, int OUT, int sms, FwdPlan& pl, bool counts = false) {
    if (OUT % 4 != 0) return false;
    const int chunks = OUT / 4;
    bool found = false;
    for (int C : kTokChunks) {
        if (chunks % C != 0) continue;
        const int JR = 4 * C;
        const int RS = (C % 2 == 0) ? JR + 4 : JR;
        const int nb = ceil_div(K, 256);
        const int m = 32 / std::gcd(RS, 32);  // keeps every box 128-byte aligned
        const int KB = round_up(ceil_div(K, nb), m);
        if (KB > 256) continue;
        const int slice = round_up(std::max(KB * nb, K + 1) * RS * 4, 128);
        const int64_t smem = (int64_t)IN * slice + 128 + 8 * ceil_div(IN, kTokXB) +  // + alignment + mbarriers
                             (counts ? 4 * (int64_t)K : 0);                          // + bin counters
        if (smem > kSmemBudget) continue;
        pl = {C, 1, JR, IN, KB, nb, slice, (int)smem};
        pl.RS = RS;
        found = true;
        const int64_t ranges = (N + tok_threads(C) - 1) / tok_threads(C);
        if (ranges * (chunks / C) >= sms) break;  // enough CTAs at this width
    }
    return found;
}

template <int DT, int C>
inline int launch_token_fwd(const CUtensorMap& map, const FwdArgs& a, const FwdPlan& pl, int sms,
                            cudaStream_t s) {
    auto kern = a.counts ? fwd_token_kernel<DT, C, true> : fwd_token_kernel<DT, C, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess)
        return 4;
    const int jranges = ceil_div(a.OUT, pl.JR);
    const int T = tok_threads(C);
    // contiguous token ranges, one per CTA, a multiple of 32 tokens each
    const int max_ranges = std::max(1, sms / jranges);
    int per = round_up(ceil_div(a.N, max_ranges), 32);
    per = std::max(per, 32);
    FwdArgs b = a;
    b.ntiles = per;
    const int ranges = ceil_div(a.N, per);
    kern<<<dim3((unsigned)ranges, (unsigned)jranges, 1), T, pl.smem, s>>>(map, b);
    (void)T;
    return 0;
}

template <int DT>
inline int launch_token_fwd_c(const CUtensorMap& map, const FwdArgs& a, const FwdPlan& pl, int sms,
                              cudaStream_t s) {
    switch (pl.C) {
        case 8: return launch_token_fwd<DT, 8>(map, a, pl, sms, s);
        case 5: return launch_token_fwd<DT, 5>(map, a, pl, sms, s);
        case 4: return launch_token_fwd<DT, 4>(map, a, pl, sms, s);
        case 2: return launch_token_fwd<DT, 2>(map, a, pl, sms, s);
        default: return launch_token_fwd<DT, 1>(map, a, pl, sms, s);
    }
}

// kNotApplicable when the table slices of all input columns do not fit one CTA
inline int token_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out,
                         int64_t N, int64_t IN, int64_t OUT, const BinCfg& c, int sms, cudaStream_t s,
                         unsigned long long* counts = nullptr) {
    FwdPlan pl;
    if (!plan_token_forward(N, c.K, (int)IN, (int)OUT, sms, pl, counts != nullptr)) return kNotApplicable;
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, pl.RS, pl.KB)) return kNotApplicable;
    FwdArgs a;
    a.counts = counts;
    a.x = x;
    a.bias = bias;
    a.out = out;
    a.N = (int)N;
    a.IN = (int)IN;
    a.OUT = (int)OUT;
    a.K = c.K;
    a.JR = pl.JR;
    a.RS = pl.RS;
    a.xvec = (IN % 4 == 0) && ((uintptr_t)x % (x_dtype == kBF16 ? 8 : 16) == 0);
    a.IG = pl.IG;
    a.KB = pl.KB;
    a.nbox = pl.nbox;
    a.slice_bytes = pl.slice_bytes;
    a.ntiles = 0;  // set per launch: tokens per CTA range
    a.cfg = c;
    return x_dtype == kBF16 ? launch_token_fwd_c<kBF16>(map, a, pl, sms, s)
                            : launch_token_fwd_c<kF32>(map, a, pl, sms, s);
}


// ---------------------------------------------------------------------------
// streamed variant for tables too large to keep resident (e.g. 1024 x 1024
// columns at K=64, 256 MB)
// ---------------------------------------------------------------------------
//
// A CTA owns one tile of kStrThreads tokens (one per thread) and one j-range
// of JR = 4*C output columns, and streams the table through shared memory in
// chunks of CB input columns: one TMA box {RS floats, CB columns, K rows} per
// chunk, two buffers, so that chunk c+1 lands while chunk c is used.  A box
// lays rows out as [K][CB][RS]; row k of column s is (k*CB + s)*RS floats in,
// and with RS/4 and CB both odd consecutive rows of a column start in
// different bank groups.  hi = min(lo+1, K-1) is read from the box directly
// (no extra row).  Each thread keeps its token's JR accumulators in registers
// for the whole stream.
constexpr int kStrThreads = 512;
constexpr int kStrMaxCB = 15;  // input columns per chunk, at most (odd)

struct StrArgs {
    const void* x;
    const float* bias;
    float* out;
    int N, IN, OUT, K;
    int JR, RS;      // j-range width and shared-memory row stride (floats)
    int CB;          // input columns per chunk (odd)
    int nchunks;
    int box_bytes;   // bytes of one chunk (K * CB * RS * 4)
    int buf_stride;  // shared-memory bytes between the two buffers
    BinCfg cfg;
};

template <int DT, int C>
__global__ void __launch_bounds__(kStrThreads, 1)
    fwd_stream_kernel(const __grid_constant__ CUtensorMap tmap, const StrArgs p) {
    extern __shared__ unsigned char smem[];
    const int IN = p.IN, K = p.K, CB = p.CB;
    const int j0 = blockIdx.y * p.JR;
    const int n = blockIdx.x * kStrThreads + (int)threadIdx.x;
    const bool tok = n < p.N;
    const uint32_t buf0 = (smem_addr(smem) + 127u) & ~127u;
    const uint32_t bar0 = buf0 + 2u * (uint32_t)p.buf_stride;  // two mbarriers, 8 bytes each
    const uint32_t row_bytes = (uint32_t)(CB * p.RS * 4);      // between rows k and k+1 of a column
    const uint32_t col_bytes = (uint32_t)(p.RS * 4);

    if (threadIdx.x == 0) {
        prefetch_tensormap(&tmap);
        mbar_init(bar0, 1);
        mbar_init(bar0 + 8, 1);
        fence_mbar_init();
        for (int c = 0; c < 2 && c < p.nchunks; ++c) {
            mbar_arrive_expect_tx(bar0 + 8u * c, (uint32_t)p.box_bytes);
            tma_load_3d(buf0 + (uint32_t)(c * p.buf_stride), &tmap, bar0 + 8u * c, j0, c * CB, 0);
        }
    }
    __syncthreads();

    float4 acc[C];
#pragma unroll
    for (int c = 0; c < C; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int64_t xrow = (int64_t)(tok ? n : 0) * IN;

    for (int ch = 0; ch < p.nchunks; ++ch) {
        const int b = ch & 1;
        const uint32_t buf = buf0 + (uint32_t)(b * p.buf_stride);
        mbar_wait_bounded(bar0 + 8u * b, (uint32_t)((ch >> 1) & 1));
        const int i0 = ch * CB;
        const int ncol = min(CB, IN - i0);
        float xs[kStrMaxCB];  // this chunk's x values of the token, loaded together
#pragma unroll
        for (int s = 0; s < kStrMaxCB; ++s) xs[s] = (tok && s < ncol) ? load_x<DT>(p.x, xrow + i0 + s) : 0.0f;
#pragma unroll
        for (int s = 0; s < kStrMaxCB; ++s) {
            if (s >= ncol) break;
            const float xv = xs[s];
            int lo;
            float wa, wc;
            gather_weights<DT>(xv, p.cfg, lo, wa, wc);
            const uint32_t rlo = buf + (uint32_t)lo * row_bytes + (uint32_t)s * col_bytes;
            const uint32_t rhi = rlo + (lo < K - 1 ? row_bytes : 0u);
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const float4 tl = lds_v4(rlo + c * 16);
                const float4 th = lds_v4(rhi + c * 16);
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
        __syncthreads();  // every thread is done with this buffer
        if (threadIdx.x == 0 && ch + 2 < p.nchunks) {
            fence_proxy_async_smem();  // generic reads of the buffer before the async-proxy refill
            mbar_arrive_expect_tx(bar0 + 8u * b, (uint32_t)p.box_bytes);
            tma_load_3d(buf, &tmap, bar0 + 8u * b, j0, (ch + 2) * CB, 0);
        }
    }
    if (tok) {
        float4* o = reinterpret_cast<float4*>(p.out + (int64_t)n * p.OUT + j0);
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const float4 bb = __ldg(reinterpret_cast<const float4*>(p.bias + j0) + c);
            o[c] = make_float4(acc[c].x + bb.x, acc[c].y + bb.y, acc[c].z + bb.z, acc[c].w + bb.w);
        }
    }
}

constexpr int kStrChunks[] = {8, 4, 2, 1};

struct StrPlan {
    int C = 0, JR = 0, RS = 0, CB = 0, nchunks = 0, box_bytes = 0, buf_stride = 0, smem = 0;
};

// widest j-range (C <= 8) whose two chunk buffers of at least 3 columns fit;
// the TMA box needs K <= 256 rows and CB <= 256 columns
inline bool plan_stream_forward(int K, int IN, int OUT, StrPlan& pl) {
    if (OUT % 4 != 0 || K > 256 || K < 2) return false;
    const int chunks = OUT / 4;
    for (int C : kStrChunks) {
        if (chunks % C != 0) continue;
        const int JR = 4 * C;
        const int RS = (C % 2 == 0) ? JR + 4 : JR;  // RS/4 odd
        const int col = K * RS * 4;                 // bytes of one column's rows
        int CB = (kSmemBudget - 128 - 32) / 2 / col;
        CB = std::min(CB, std::min(kStrMaxCB, IN));
        if (CB % 2 == 0) --CB;  // odd: rows of a column spread over the bank groups
        if (CB < 1) continue;
        const int box = K * CB * RS * 4;
        const int stride = round_up(box, 128);
        pl = {C, JR, RS, CB, ceil_div(IN, CB), box, stride, 2 * stride + 128 + 32};
        return true;
    }
    return false;
}

template <int DT, int C>
inline int launch_stream_fwd(const CUtensorMap& map, const StrArgs& a, const StrPlan& pl, cudaStream_t s) {
    auto kern = fwd_stream_kernel<DT, C>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess)
        return 4;
    kern<<<dim3((unsigned)ceil_div(a.N, kStrThreads), (unsigned)(a.OUT / pl.JR), 1), kStrThreads, pl.smem, s>>>(map,
                                                                                                             a);
    return 0;
}

template <int DT>
inline int launch_stream_fwd_c(const CUtensorMap& map, const StrArgs& a, const StrPlan& pl, cudaStream_t s) {
    switch (pl.C) {
        case 8: return launch_stream_fwd<DT, 8>(map, a, pl, s);
        case 4: return launch_stream_fwd<DT, 4>(map, a, pl, s);
        case 2: return launch_stream_fwd<DT, 2>(map, a, pl, s);
        default: return launch_stream_fwd<DT, 1>(map, a, pl, s);
    }
}

// kNotApplicable when the shape has no streaming plan
inline int stream_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out,
                          int64_t N, int64_t IN, int64_t OUT, const BinCfg& c, cudaStream_t s) {
    StrPlan pl;
    if (!plan_stream_forward(c.K, (int)IN, (int)OUT, pl)) return kNotApplicable;
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, pl.RS, c.K, pl.CB)) return kNotApplicable;
    StrArgs a;
    a.x = x;
    a.bias = bias;
    a.out = out;
    a.N = (int)N;
    a.IN = (int)IN;
    a.OUT = (int)OUT;
    a.K = c.K;
    a.JR = pl.JR;
    a.RS = pl.RS;
    a.CB = pl.CB;
    a.nchunks = pl.nchunks;
    a.box_bytes = pl.box_bytes;
    a.buf_stride = pl.buf_stride;
    a.cfg = c;
    return x_dtype == kBF16 ? launch_stream_fwd_c<kBF16>(map, a, pl, s) : launch_stream_fwd_c<kF32>(map, a, pl, s);
}

}  // namespace il
