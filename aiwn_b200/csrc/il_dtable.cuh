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
//     2. exclusive scan of the bin counts, scatter of (token, weights) into
//        bin order (the order inside a bin follows shared-memory atomics, so
//        the fp32 sums are not bitwise reproducible run to run; they agree
//        with the reference to ~1e-6 relative)
//     3. the "visit sequence" lists, row by row, the tokens contributing to
//        row k: bin k's tokens (weight x(1-fr)) then bin k-1's (weight x fr).
//        It is cut into equal pieces, one per lane group; a group walks its
//        piece, accumulates go[token, 4jc:4jc+4] * weight in registers and
//        adds the finished row into the CTA's gt slice in shared memory
//        (plain read-modify-write: interior rows of a piece belong to that
//        group alone; the first and last row of a piece may be shared with a
//        neighbour group and use shared-memory atomics).
//   at the end the CTA adds its gt slice to global memory (vector reds).
//
// The top bin's hi contribution (lo = K-1, hi = K-1) is collected as a
// virtual row K and folded into row K-1.  go tiles are double-buffered with
// bulk copies so that loading tile t+1 overlaps the work on tile t.
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

constexpr int kDtThreads = 1024;

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// block-wide exclusive scan of cnt[0..n) into out[0..n], out[n] = total
// (n <= kDtThreads * 4; uses `tmp` of kDtThreads/32 ints)
__device__ __forceinline__ void block_exclusive_scan(const uint32_t* cnt, uint32_t* out, int n,
                                                     uint32_t* tmp) {
    const int per = (n + kDtThreads - 1) / kDtThreads;  // items per thread
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
        uint32_t w = lane < kDtThreads / 32 ? tmp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        if (lane < kDtThreads / 32) tmp[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    uint32_t run = (warp > 0 ? tmp[warp - 1] : 0) + v - local;
    for (int q = 0; q < per; ++q) {
        if (b + q < n) {
            out[b + q] = run;
            run += cnt[b + q];
        }
    }
    if (threadIdx.x == kDtThreads - 1) out[n] = tmp[kDtThreads / 32 - 1];
}

template <int C>
struct DtGroup {
    static_assert(C >= 1 && C <= 32, "a row is covered by one group of at most 32 lanes");
    static constexpr int G = C;                              // lanes per row group (one chunk each)
    static constexpr int GPW = 32 / C;                       // groups per warp
    static constexpr int NG = GPW * (kDtThreads / 32);       // groups per CTA
};

// per sorted entry: token (as bits), x(1-fr), x*fr
struct __align__(16) DtEntry {
    uint32_t tok;
    float wa, wc;
    uint32_t pad;
};

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
    const uint32_t go_bytes = (uint32_t)(TT * OUT * 4);
    const uint32_t go_s0 = base, go_s1 = base + go_bytes;        // go tiles (double buffer)
    DtEntry* ent = reinterpret_cast<DtEntry*>(gen + 2 * go_bytes);    // sorted entries [TT]
    DtEntry* tke = ent + TT;                                          // per token [TT] (tok = bin)
    float* gts = reinterpret_cast<float*>(tke + TT);                  // gt slice [(K+1)][OUT]
    uint32_t* cnt = reinterpret_cast<uint32_t*>(gts + (size_t)(K + 1) * OUT);  // [K+1]
    uint32_t* sb = cnt + (K + 1);                                     // bin starts [K+1]
    uint32_t* tmp = sb + (K + 1);                                     // scan scratch [32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uintptr_t>(tmp + 32 + 1) & ~uintptr_t(7));
    const uint32_t bar0 = smem_addr(bars), bar1 = bar0 + 8;

    for (int e = threadIdx.x; e < (K + 1) * OUT; e += kDtThreads) gts[e] = 0.f;
    for (int e = threadIdx.x; e < K + 1; e += kDtThreads) cnt[e] = 0;
    const int ntile = r1 > r0 ? (r1 - r0 + TT - 1) / TT : 0;
    if (threadIdx.x == 0) {
        mbar_init(bar0, 1);
        mbar_init(bar1, 1);
        fence_mbar_init();
        fence_proxy_async_smem();
        if (ntile > 0) {
            const int nt = min(TT, r1 - r0);
            mbar_arrive_expect_tx(bar0, (uint32_t)(nt * OUT * 4));
            bulk_load(go_s0, p.go + (int64_t)r0 * OUT, (uint32_t)(nt * OUT * 4), bar0);
        }
    }
    __syncthreads();

    float4 bsum = make_float4(0.f, 0.f, 0.f, 0.f);  // bias gradient (column i == 0 CTAs)
    for (int t = 0; t < ntile; ++t) {
        const int t0 = r0 + t * TT;
        const int nt = min(TT, r1 - t0);
        const uint32_t go_s = (t & 1) ? go_s1 : go_s0;
        const float* gos = reinterpret_cast<const float*>(gen + (go_s - base));
        // prefetch the next tile into the other buffer (its last readers
        // finished before the __syncthreads that closed tile t-1)
        if (threadIdx.x == 0 && t + 1 < ntile) {
            const int t1 = t0 + TT;
            const int n1 = min(TT, r1 - t1);
            const uint32_t bn = (t & 1) ? bar0 : bar1;
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(bn, (uint32_t)(n1 * OUT * 4));
            bulk_load((t & 1) ? go_s0 : go_s1, p.go + (int64_t)t1 * OUT, (uint32_t)(n1 * OUT * 4), bn);
        }
        // 1. bins and weights of the tile's tokens; counts per bin
        if (threadIdx.x < nt) {
            const Bin b = bin_of<DT>(load_x<DT>(p.x, (int64_t)(t0 + threadIdx.x) * p.IN + i), p.cfg);
            DtEntry e;
            e.tok = (uint32_t)b.lo;
            e.wa = __fmul_rn(b.x, __fsub_rn(1.0f, b.fr));
            e.wc = __fmul_rn(b.x, b.fr);
            e.pad = 0;
            tke[threadIdx.x] = e;
            atomicAdd(&cnt[b.lo], 1u);
        }
        __syncthreads();
        // 2. bin starts (exclusive scan, sb[K] = nt), then scatter into bin order
        block_exclusive_scan(cnt, sb, K, tmp);
        __syncthreads();
        for (int e = threadIdx.x; e < K + 1; e += kDtThreads) cnt[e] = 0;
        __syncthreads();
        if (threadIdx.x < nt) {
            DtEntry e = tke[threadIdx.x];
            const uint32_t lo = e.tok;
            const uint32_t pos = sb[lo] + atomicAdd(&cnt[lo], 1u);
            e.tok = (uint32_t)threadIdx.x;
            ent[pos] = e;
        }
        // go tile t has landed (waited by everyone before reading it)
        mbar_wait_bounded((t & 1) ? bar1 : bar0, (uint32_t)((t >> 1) & 1));
        __syncthreads();
        // 3. walk the visit sequence: rows 0..K (row K = top bin's hi part).
        //    V(k) = S(k) + S(k-1) visits precede row k (S = bin starts); 2*nt visits
        const int total = 2 * nt;
        const int per = (total + NG - 1) / NG;
        const int v0 = glive ? min(total, grp * per) : total;
        const int v1 = min(total, v0 + per);
        if (v0 < v1) {
            int k = 0;
            {  // largest k in [0, K] with V(k) <= v0
                int lo_k = 0, hi_k = K;
                while (lo_k < hi_k) {
                    const int mid = (lo_k + hi_k + 1) >> 1;
                    if (sb[mid] + sb[mid - 1] <= (uint32_t)v0) lo_k = mid;
                    else hi_k = mid - 1;
                }
                k = lo_k;
            }
            // registers describing row k
            uint32_t sbk = sb[k], sbp = k > 0 ? sb[k - 1] : 0u;
            uint32_t sbn = k < K ? sb[k + 1] : sbk;
            uint32_t vk = sbk + sbp;
            uint32_t vsplit = vk + (k < K ? sbn - sbk : 0u);   // end of the lo part
            uint32_t vnext = k < K ? sbn + sbk : (uint32_t)total;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            bool first = true, any = false;
            for (uint32_t v = (uint32_t)v0; v < (uint32_t)v1; ++v) {
                while (v >= vnext) {  // row k is complete
                    if (any) {
                        float* d = gts + (size_t)(k == K ? K - 1 : k) * OUT + 4 * gl;
                        // rows another group may also add to: the first row of
                        // this piece and rows K-1 / K (top bin)
                        if (first || k >= K - 1) {
                            atomicAdd(d + 0, acc.x);
                            atomicAdd(d + 1, acc.y);
                            atomicAdd(d + 2, acc.z);
                            atomicAdd(d + 3, acc.w);
                        } else {
                            float4 o = *reinterpret_cast<float4*>(d);
                            o.x += acc.x;
                            o.y += acc.y;
                            o.z += acc.z;
                            o.w += acc.w;
                            *reinterpret_cast<float4*>(d) = o;
                        }
                    }
                    acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    first = false;
                    any = false;
                    ++k;
                    sbp = sbk;
                    sbk = sbn;
                    sbn = k < K ? sb[k + 1] : sbk;
                    vk = vnext;
                    vsplit = vk + (k < K ? sbn - sbk : 0u);
                    vnext = k < K ? sbn + sbk : (uint32_t)total;
                }
                const bool lopart = v < vsplit;
                const uint32_t e = lopart ? v - vk + sbk : v - vsplit + sbp;
                const DtEntry en = ent[e];
                const float w = lopart ? en.wa : en.wc;
                const float4 g = *reinterpret_cast<const float4*>(gos + (size_t)en.tok * OUT + 4 * gl);
                acc.x = fmaf(w, g.x, acc.x);
                acc.y = fmaf(w, g.y, acc.y);
                acc.z = fmaf(w, g.z, acc.z);
                acc.w = fmaf(w, g.w, acc.w);
                any = true;
            }
            if (any) {  // last row of the piece (possibly shared with the next group)
                float* d = gts + (size_t)(k == K ? K - 1 : k) * OUT + 4 * gl;
                atomicAdd(d + 0, acc.x);
                atomicAdd(d + 1, acc.y);
                atomicAdd(d + 2, acc.z);
                atomicAdd(d + 3, acc.w);
            }
        }
        // bias gradient: CTAs of column 0 add up the tile's go rows
        if (p.want_gb && i == 0 && glive) {
            for (int tk = grp; tk < nt; tk += NG) {
                const float4 g = *reinterpret_cast<const float4*>(gos + (size_t)tk * OUT + 4 * gl);
                bsum.x += g.x;
                bsum.y += g.y;
                bsum.z += g.z;
                bsum.w += g.w;
            }
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
    if (p.want_gb && i == 0 && glive) {
        float* d = p.gb + 4 * gl;
        atomicAdd(d + 0, bsum.x);
        atomicAdd(d + 1, bsum.y);
        atomicAdd(d + 2, bsum.z);
        atomicAdd(d + 3, bsum.w);
    }
}

}  // namespace il
