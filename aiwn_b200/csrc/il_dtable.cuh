// il_dtable.cuh -- table gradient (and bias gradient) without atomics on the
// hot path.
//
//   gt[k,i,:] = sum_{n: lo=k} x(1-fr) go[n,:]  +  sum_{n: hi=k} x fr go[n,:]
//
// is the scatter-add that autograd performs for the reference's gathers
// table[bk, ie] and table[hi, ie] (aiwn/layers/indexed_linear.py:179-180).
// Scattering it with atomics is bound by the atomic rate of the memory
// system; instead each CTA owns one input column i and a range of tokens and
// turns the scatter into register accumulation:
//
//   per tile of TT tokens
//     1. bucket every token (bit-exact bins), count tokens per bin
//     2. exclusive scan of the bin counts, scatter of (token, weights, bin)
//        into bin order (the order inside a bin follows shared-memory
//        atomics, so the fp32 sums are not bitwise reproducible run to run;
//        they agree with the reference to ~1e-6 relative)
//     3. the sorted entries are cut into equal slices, one per lane group
//        (C lanes, one 16-byte chunk of a row each).  A group walks its
//        slice in order with two register accumulators: x(1-fr)*go for row
//        `bin` and x*fr*go for row bin+1 (row K-1 for the top bin).  When the
//        bin changes both are added into the CTA's gt slice in shared memory:
//        plainly for bins inside the slice, with shared-memory atomics for
//        the first and last bin (a neighbour group may hold part of them).
//        go rows are read straight from global memory (L2), each row once
//        per (token, column), with kDtDepth rows in flight per group.
//   at the end the CTA adds its gt slice to global memory (vector reds).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "il_common.cuh"
#include "il_sm100.cuh"

namespace il {

struct DtArgs {
    const float* go;
    const void* x;
    float* gt;
    float* gb;
    int N, IN, OUT, K;
    int TT;          // tokens per tile (multiple of 32, <= kDtThreads)
    int tok_per_cta; // tokens of one CTA's range (multiple of TT)
    int want_gb;
    BinCfg cfg;
};

constexpr int kDtThreads = 512;

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// block-wide exclusive scan of cnt[0..n) into out[0..n], out[n] = total, by
// a block of NT threads (uses `tmp` of NT/32 <= 32 ints)
template <int NT = kDtThreads>
__device__ __forceinline__ void block_exclusive_scan(const uint32_t* cnt, uint32_t* out, int n,
                                                     uint32_t* tmp) {
    static_assert(NT % 32 == 0 && NT <= 1024, "whole warps, at most 32 of them");
    const int per = (n + NT - 1) / NT;  // items per thread
    const int b = threadIdx.x * per;
    uint32_t local = 0;
    for (int q = 0; q < per; ++q)
        if (b + q < n) local += cnt[b + q];
    // warp scan of `local`
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t v = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    if (lane == 31) tmp[warp] = v;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < NT / 32 ? tmp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        if (lane < NT / 32) tmp[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    uint32_t run = (warp > 0 ? tmp[warp - 1] : 0) + v - local;
    for (int q = 0; q < per; ++q) {
        if (b + q < n) {
            out[b + q] = run;
            run += cnt[b + q];
        }
    }
    if (threadIdx.x == NT - 1) out[n] = tmp[NT / 32 - 1];
}

template <int C>
struct DtGroup {
    static_assert(C >= 1 && C <= 32, "a row is covered by one group of at most 32 lanes");
    static constexpr int G = C;                              // lanes per group (one chunk each)
    static constexpr int GPW = 32 / C;                       // groups per warp
    static constexpr int NG = GPW * (kDtThreads / 32);       // groups per CTA
};

// sorted entry: token (offset in the tile), x(1-fr), x*fr, bin
struct __align__(16) DtEntry {
    uint32_t tok;
    float wa, wc;
    uint32_t bin;
};

constexpr int kDtDepth = 6;  // entries whose go rows are in flight per group

__device__ __forceinline__ void flush_row(float* gts, int OUT, int row, int gl, float4 a, bool shared) {
    float* d = gts + (size_t)row * OUT + 4 * gl;
    if (shared) {
        atomicAdd(d + 0, a.x);
        atomicAdd(d + 1, a.y);
        atomicAdd(d + 2, a.z);
        atomicAdd(d + 3, a.w);
    } else {
        float4 o = *reinterpret_cast<float4*>(d);
        o.x += a.x;
        o.y += a.y;
        o.z += a.z;
        o.w += a.w;
        *reinterpret_cast<float4*>(d) = o;
    }
}

template <int DT, int C>
__global__ void __launch_bounds__(kDtThreads, 1) dtable_kernel(const DtArgs p) {
    constexpr int GPW = DtGroup<C>::GPW, NG = DtGroup<C>::NG;
    extern __shared__ unsigned char smem[];
    const int i = blockIdx.y;
    const int K = p.K, OUT = p.OUT, TT = p.TT;
    const int r0 = blockIdx.x * p.tok_per_cta;
    const int r1 = min(p.N, r0 + p.tok_per_cta);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = lane / C, gl = lane - gw * C;      // group in warp, lane in group
    const bool glive = gw < GPW;                      // lanes past the last full group idle
    const int grp = warp * GPW + gw;

    // shared memory layout (from a 128-byte aligned base)
    const uint32_t base = (smem_addr(smem) + 127u) & ~127u;
    unsigned char* gen = smem + (base - smem_addr(smem));
    DtEntry* ent = reinterpret_cast<DtEntry*>(gen);                   // sorted entries [TT]
    DtEntry* tke = ent + TT;                                          // per token [TT]
    float* gts = reinterpret_cast<float*>(tke + TT);                  // gt slice [K][OUT]
    uint32_t* cnt = reinterpret_cast<uint32_t*>(gts + (size_t)K * OUT);  // [K+1]
    uint32_t* sb = cnt + (K + 1);                                     // bin starts [K+1]
    uint32_t* tmp = sb + (K + 1);                                     // scan scratch [32]

    for (int e = threadIdx.x; e < K * OUT; e += kDtThreads) gts[e] = 0.f;
    for (int e = threadIdx.x; e < K + 1; e += kDtThreads) cnt[e] = 0;
    __syncthreads();

    const int ntile = r1 > r0 ? (r1 - r0 + TT - 1) / TT : 0;
    for (int t = 0; t < ntile; ++t) {
        const int t0 = r0 + t * TT;
        const int nt = min(TT, r1 - t0);
        // 1. bins and weights of the tile's tokens; counts per bin
        for (int tk = threadIdx.x; tk < nt; tk += kDtThreads) {
            const Bin b = bin_of<DT>(load_x<DT>(p.x, (int64_t)(t0 + tk) * p.IN + i), p.cfg);
            DtEntry e;
            e.tok = (uint32_t)tk;
            e.wa = __fmul_rn(b.x, __fsub_rn(1.0f, b.fr));
            e.wc = __fmul_rn(b.x, b.fr);
            e.bin = (uint32_t)b.lo;
            tke[tk] = e;
            atomicAdd(&cnt[b.lo], 1u);
        }
        __syncthreads();
        // 2. bin starts (exclusive scan), then scatter into bin order
        block_exclusive_scan(cnt, sb, K, tmp);
        __syncthreads();
        for (int e = threadIdx.x; e < K + 1; e += kDtThreads) cnt[e] = 0;
        __syncthreads();
        for (int tk = threadIdx.x; tk < nt; tk += kDtThreads) {
            const DtEntry e = tke[tk];
            const uint32_t pos = sb[e.bin] + atomicAdd(&cnt[e.bin], 1u);
            ent[pos] = e;
        }
        __syncthreads();
        // 3. each group walks an equal slice of the sorted entries; row `bin`
        //    gets x(1-fr) go, row bin+1 (K-1 for the top bin) gets x fr go
        const int per = (nt + NG - 1) / NG;
        const int e0 = glive ? min(nt, grp * per) : nt;
        const int e1 = min(nt, e0 + per);
        if (e0 < e1) {
            const int bfirst = (int)ent[e0].bin, blast = (int)ent[e1 - 1].bin;
            const float* gob = p.go + (int64_t)t0 * OUT + 4 * gl;
            float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
            int cur = bfirst;
            // prefetch the first kDtDepth entries' go chunks
            DtEntry en[kDtDepth];
            float4 gv[kDtDepth];
#pragma unroll
            for (int d = 0; d < kDtDepth; ++d) {
                if (e0 + d < e1) {
                    en[d] = ent[e0 + d];
                    gv[d] = __ldg(reinterpret_cast<const float4*>(gob + (size_t)en[d].tok * OUT));
                }
            }
            for (int e = e0; e < e1; e += kDtDepth) {
#pragma unroll
                for (int d = 0; d < kDtDepth; ++d) {
                    if (e + d >= e1) break;
                    const DtEntry c = en[d];
                    const float4 g = gv[d];
                    // refill this slot with the entry kDtDepth ahead
                    const int nx = e + d + kDtDepth;
                    if (nx < e1) {
                        en[d] = ent[nx];
                        gv[d] = __ldg(reinterpret_cast<const float4*>(gob + (size_t)en[d].tok * OUT));
                    }
                    if ((int)c.bin != cur) {
                        // rows next to either end of the slice can also receive
                        // a neighbour group's part of a split bin
                        const int rh = min(cur + 1, K - 1);
                        flush_row(gts, OUT, cur, gl, lo, cur <= bfirst + 1 || cur >= blast);
                        flush_row(gts, OUT, rh, gl, hi, rh <= bfirst + 1 || rh >= blast);
                        lo = make_float4(0.f, 0.f, 0.f, 0.f);
                        hi = lo;
                        cur = (int)c.bin;
                    }
                    lo.x = fmaf(c.wa, g.x, lo.x);
                    lo.y = fmaf(c.wa, g.y, lo.y);
                    lo.z = fmaf(c.wa, g.z, lo.z);
                    lo.w = fmaf(c.wa, g.w, lo.w);
                    hi.x = fmaf(c.wc, g.x, hi.x);
                    hi.y = fmaf(c.wc, g.y, hi.y);
                    hi.z = fmaf(c.wc, g.z, hi.z);
                    hi.w = fmaf(c.wc, g.w, hi.w);
                }
            }
            // the last bin of the slice may continue in the next group's slice
            flush_row(gts, OUT, cur, gl, lo, true);
            flush_row(gts, OUT, min(cur + 1, K - 1), gl, hi, true);
        }
        for (int e = threadIdx.x; e < K + 1; e += kDtThreads) cnt[e] = 0;
        __syncthreads();
    }
    // 4. add this CTA's slice to the global table gradient
    for (int e = threadIdx.x; e < K * (OUT / 4); e += kDtThreads) {
        const int k = e / (OUT / 4), c4 = e - k * (OUT / 4);
        const float4 v = *reinterpret_cast<const float4*>(gts + (size_t)k * OUT + 4 * c4);
        red_global_add_v4(p.gt + ((int64_t)k * p.IN + i) * OUT + 4 * c4, v);
    }
}

}  // namespace il
