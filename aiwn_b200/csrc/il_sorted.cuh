// il_sorted.cuh -- backward of IndexedLinear by bin-sorted walks.
//
//   dx[n,i]  = sum_j go[n,j] * ((1-fr-s) T[lo,i,j] + (fr+s) T[hi,i,j])
//   gt[k,i,:] = sum_{n: lo=k} x(1-fr) go[n,:] + sum_{n: hi=k} x fr go[n,:]
//   gb[:]     = sum_n go[n,:]
//
// (s = x/bw where torch.clamp passes the gradient of fr, else 0) are the
// gradients autograd produces for the reference's eager forward
// (aiwn/layers/indexed_linear.py:173-182): the scatter-add into gt is the
// backward of the gathers table[bk, ie] / table[hi, ie].
//
// A CTA owns G consecutive input columns (G = 4 when in_d allows, else 1)
// and a range of tokens.  Per tile of up to kSrtMaxTile tokens it loads the
// tile's x values of its G columns once (one 16-byte load per token for G=4
// fp32) into a shared-memory tile xd[G][token], then for each column c:
//   1. bins every token (bit-exact, bw = 2^-e) and takes a rank inside its
//      bin from a shared-memory counter,
//   2. scans the bin counts into bin starts,
//   3. writes each token's weights x(1-fr), x fr, 1-fr-s and its packed
//      (bin, token) word as one 16-byte entry at its sorted position (the
//      fourth weight, fr+s, is 1 minus the third),
//   4. cuts the sorted entries into equal slices, one per lane group (C
//      lanes, one 16-byte chunk of a go row each).  A group walks its slice
//      in bin order with
//        - rows T[bin] and T[bin+1] of the column in registers (re-read from
//          the column's table slice in shared memory when the bin changes),
//        - two register accumulators, for gt rows bin and bin+1, added into
//          gt with red.global.add.v4 only when the bin changes,
//        - dx of each entry as a sum over the group's lanes, stored into
//          xd[c][token] (x of column c is no longer needed by then),
//      reading entries kSrtDepth ahead from shared memory and their go rows
//      from global memory (L2).
// After the G columns, xd holds dx of the tile: one 16-byte store per token
// writes its G columns of gx.  Each gt row receives one reduction per (lane
// group, tile) that touches it instead of one per token: at 131072 tokens,
// 20 columns and K=512 about 1 M vector reductions instead of 26 M.
//
// The order inside a bin follows shared-memory atomics, so the fp32 sums of
// gt are not bitwise reproducible from run to run; dx is (each entry's dot
// products do not depend on the order).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "il_common.cuh"
#include "il_fast.cuh"
#include "il_sm100.cuh"

namespace il {

constexpr int kSrtThreads = 1024;
constexpr int kSrtPer = 8;                            // tokens per thread per tile
constexpr int kSrtMaxTile = kSrtThreads * kSrtPer;    // 8192
constexpr int kSrtG = 4;                              // input columns per CTA when in_d % 4 == 0
constexpr int kSrtTokBits = 14;                       // tile-local token bits of an entry
constexpr uint32_t kSrtTokMask = (1u << kSrtTokBits) - 1u;
constexpr int kSrtDepth = 3;                          // go rows in flight per lane group
constexpr int kSrtCtasPerSm = 1;                      // co-resident CTAs the plan sizes for
// dynamic shared memory per CTA when kSrtCtasPerSm share an SM's 228 KB
constexpr int kSrtSmemBudget = kSrtCtasPerSm == 1 ? kSmemBudget : (228 * 1024) / kSrtCtasPerSm - 1024 - 256;
static_assert(kSrtMaxTile <= (1 << kSrtTokBits), "tile-local token index must fit the entry");

struct SrtArgs {
    const float* go;
    const void* x;
    const float* table;
    void* gx;
    float* gt;
    float* gb;
    int N, IN, OUT, K;
    int G;            // input columns per CTA (1 or kSrtG)
    int TT;           // tokens per tile (multiple of 32, <= kSrtMaxTile)
    int tok_per_cta;  // tokens of one CTA's range
    int want_gx, want_gb;  // gt is always written (the kernel is chosen for it)
    int gx_atomic;         // several j-ranges: dx partial sums are added (gx zeroed, fp32)
    BinCfg cfg;
};

// add a finished gradient row chunk: element offset row * IN*OUT + lane_off
// (lane_off = i*OUT + j-range start + 4*lane; the plan keeps K*IN*OUT < 2^31)
__device__ __forceinline__ void srt_flush(float* gt, int row, int rs, int lane_off, float4 v) {
    red_global_add_v4(gt + (uint32_t)(row * rs + lane_off), v);
}

// Walk of one lane group over its sorted entries [e0, e1) of column c of a
// tile.  The trip count `steps` (a multiple of kSrtDepth) is the same for
// every lane of the warp, since the dx sums use shuffles; steps past e1 use
// the all-zero entry TT (token 0 of the tile, a valid go row), so the common
// path has no branch except the one taken when the bin changes.
template <int C, int G, bool GX>
__device__ __forceinline__ void srt_walk(const SrtArgs& p, uint32_t slice_s, uint32_t ew_s, uint32_t xd_s, int c,
                                         int t0, int e0, int e1, int steps, int gl, int i) {
    const int OUT = p.OUT, IN = p.IN, K = p.K, TT = p.TT;
    const float* gob = p.go + (int64_t)t0 * OUT + blockIdx.z * 4 * C + 4 * gl;  // j-range blockIdx.z
    const uint32_t row_bytes = (uint32_t)C * 16;         // slice rows hold the j-range
    const int rs = IN * OUT;                             // gt row stride (elements)
    const int lane_off = i * OUT + (int)blockIdx.z * 4 * C + 4 * gl;
    const uint32_t tcol = slice_s + 16u * (uint32_t)gl;  // this lane's chunk of table row 0
    // entries' packed words (their fourth word) kSrtDepth ahead, with their go rows
    uint32_t rn[kSrtDepth];
    float4 rg[kSrtDepth];
#pragma unroll
    for (int d = 0; d < kSrtDepth; ++d) {
        rn[d] = lds_u32(ew_s + 16u * (uint32_t)(e0 + d < e1 ? e0 + d : TT) + 12u);
        rg[d] = __ldg(reinterpret_cast<const float4*>(gob + (rn[d] & kSrtTokMask) * OUT));
    }
    int cur = -1;
    float4 tlo = make_float4(0.f, 0.f, 0.f, 0.f), thi = tlo, acl = tlo, ach = tlo;
    // power-of-two groups of at least 4 lanes: the dx partials of an
    // iteration's entries are reduced together after it (wpart, wtok, wok)
    constexpr bool kWarpDx = GX && C >= 4 && (C & (C - 1)) == 0;
    float wpart[kSrtDepth];
    uint32_t wtok[kSrtDepth];
    bool wok[kSrtDepth];
    for (int b = 0; b < steps; b += kSrtDepth) {
#pragma unroll
        for (int d = 0; d < kSrtDepth; ++d) {
            const int e = e0 + b + d;
            const bool valid = e < e1;
            const float4 w = lds_v4(ew_s + 16u * (uint32_t)(valid ? e : TT));
            const float4 g = rg[d];
            const int en = e + kSrtDepth;
            rn[d] = lds_u32(ew_s + 16u * (uint32_t)(en < e1 ? en : TT) + 12u);
            rg[d] = __ldg(reinterpret_cast<const float4*>(gob + (rn[d] & kSrtTokMask) * OUT));
            const uint32_t ent = __float_as_uint(w.w);
            const int bin = valid ? (int)(ent >> kSrtTokBits) : cur;
            if (bin != cur) {
                if (cur >= 0) {
                    // row cur is complete; row cur+1 continues as the new low
                    // row when the next bin is cur+1
                    srt_flush(p.gt, cur, rs, lane_off, acl);
                    if (bin == cur + 1) {
                        acl = ach;
                    } else {
                        srt_flush(p.gt, cur + 1, rs, lane_off, ach);
                        acl = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    ach = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                // rows bin and bin+1; on a step to the next bin the old high row is the new low row
                tlo = (cur >= 0 && bin == cur + 1) ? thi : lds_v4(tcol + (uint32_t)bin * row_bytes);
                thi = bin + 1 < K ? lds_v4(tcol + (uint32_t)(bin + 1) * row_bytes) : tlo;  // hi = min(lo+1, K-1)
                cur = bin;
            }
            acl.x = fmaf(w.x, g.x, acl.x);
            acl.y = fmaf(w.x, g.y, acl.y);
            acl.z = fmaf(w.x, g.z, acl.z);
            acl.w = fmaf(w.x, g.w, acl.w);
            ach.x = fmaf(w.y, g.x, ach.x);
            ach.y = fmaf(w.y, g.y, ach.y);
            ach.z = fmaf(w.y, g.z, ach.z);
            ach.w = fmaf(w.y, g.w, ach.w);
            if constexpr (GX) {
                const float dl = g.x * tlo.x + g.y * tlo.y + g.z * tlo.z + g.w * tlo.w;
                const float dh = g.x * thi.x + g.y * thi.y + g.z * thi.z + g.w * thi.w;
                float part = w.z * dl + (1.0f - w.z) * dh;
                if constexpr (kWarpDx) {
                    wpart[d] = part;
                    wtok[d] = ent & kSrtTokMask;
                    wok[d] = valid;
                } else {
                    // sum over the group's C lanes into its lane 0
#pragma unroll
                    for (int off = 1; off < C; off <<= 1) {
                        const float o = __shfl_down_sync(0xffffffffu, part, off);
                        if (gl + off < C) part += o;
                    }
                    if (valid && gl == 0)
                        sts_u32(xd_s + 4u * (uint32_t)(c * TT + (ent & kSrtTokMask)), __float_as_uint(part));
                }
            }
        }
        if constexpr (kWarpDx) {
            // the up to four partials of this iteration summed over the group's
            // C lanes at once: the group's halves swap at distance C/2 (two
            // values each), its quarters at C/4 (one value), then a butterfly
            // over C/8 .. 1; lane k*C/4 of the group ends with entry k's sum.
            // log2(C) + 1 shuffles for the iteration against 3 log2(C).
            static_assert(kSrtDepth <= 4, "four values per reduction");
            constexpr int H = C / 2, Q = C / 4;
            const float a0 = wpart[0], a1 = kSrtDepth > 1 ? wpart[1 % kSrtDepth] : 0.0f;
            const float a2 = kSrtDepth > 2 ? wpart[2 % kSrtDepth] : 0.0f, a3 = kSrtDepth > 3 ? wpart[3 % kSrtDepth] : 0.0f;
            const bool hh = (gl & H) != 0, hq = (gl & Q) != 0;
            float k0 = hh ? a2 : a0, k1 = hh ? a3 : a1;
            k0 += __shfl_xor_sync(0xffffffffu, hh ? a0 : a2, H);
            k1 += __shfl_xor_sync(0xffffffffu, hh ? a1 : a3, H);
            float r = hq ? k1 : k0;
            r += __shfl_xor_sync(0xffffffffu, hq ? k0 : k1, Q);
#pragma unroll
            for (int off = Q / 2; off >= 1; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
            const int k = gl / Q;
#pragma unroll
            for (int d = 0; d < kSrtDepth; ++d)
                if (k == d && (gl % Q) == 0 && wok[d]) sts_u32(xd_s + 4u * (uint32_t)(c * TT + wtok[d]), __float_as_uint(r));
        }
    }
    if (cur >= 0) {
        // the top bin's hi row is row K-1 itself
        if (cur == K - 1) {
            acl.x += ach.x;
            acl.y += ach.y;
            acl.z += ach.z;
            acl.w += ach.w;
            srt_flush(p.gt, cur, rs, lane_off, acl);
        } else {
            srt_flush(p.gt, cur, rs, lane_off, acl);
            srt_flush(p.gt, cur + 1, rs, lane_off, ach);
        }
    }
}

// x of G consecutive columns of token n (row-major x, in_d % G == 0 when G > 1)
template <int DT, int G>
__device__ __forceinline__ void load_x_cols(const void* x, int64_t off, float (&v)[G]) {
    if constexpr (G == 4 && DT == kF32) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + off));
        v[0] = q.x;
        v[1] = q.y;
        v[2] = q.z;
        v[3] = q.w;
    } else if constexpr (G == 4 && DT == kBF16) {
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(x) + off));
        v[0] = __uint_as_float(q.x << 16);
        v[1] = __uint_as_float(q.x & 0xffff0000u);
        v[2] = __uint_as_float(q.y << 16);
        v[3] = __uint_as_float(q.y & 0xffff0000u);
    } else {
#pragma unroll
        for (int c = 0; c < G; ++c) v[c] = load_x<DT>(x, off + c);
    }
}

// dx of G consecutive columns of token n into gx (or added into it)
template <int DT, int G>
__device__ __forceinline__ void store_gx_cols(void* gx, int64_t off, const float (&v)[G], bool atomic) {
    if constexpr (DT == kF32) {
        float* g = reinterpret_cast<float*>(gx) + off;
        if constexpr (G == 4) {
            if (atomic) red_global_add_v4(g, make_float4(v[0], v[1], v[2], v[3]));
            else *reinterpret_cast<float4*>(g) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int c = 0; c < G; ++c) {
                if (atomic) atomicAdd(g + c, v[c]);
                else g[c] = v[c];
            }
        }
    } else {
        if constexpr (G == 4) {
            const uint32_t a = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[0])) |
                               ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[1])) << 16);
            const uint32_t b = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2])) |
                               ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[3])) << 16);
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(gx) + off) = make_uint2(a, b);
        } else {
#pragma unroll
            for (int c = 0; c < G; ++c) store_gx<DT>(gx, off + c, v[c]);
        }
    }
}

template <int DT, int C, int G>
__global__ void __launch_bounds__(kSrtThreads, kSrtCtasPerSm)
    bwd_sorted_kernel(const __grid_constant__ CUtensorMap tmap, const SrtArgs p) {
    static_assert(C >= 1 && C <= 32, "one go row per lane group of at most 32 lanes");
    static_assert(G == 1 || G == kSrtG, "one column or a group of kSrtG");
    constexpr int GPW = 32 / C;                       // lane groups per warp
    constexpr int NG = GPW * (kSrtThreads / 32);      // lane groups per CTA
    extern __shared__ unsigned char smem[];
    const int i0 = blockIdx.y * G;                    // the CTA's first input column
    const int K = p.K, OUT = p.OUT, IN = p.IN, TT = p.TT;
    const int r0 = blockIdx.x * p.tok_per_cta;
    const int r1 = min(p.N, r0 + p.tok_per_cta);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = lane / C, gl = lane - gw * C;      // group in warp, lane in group
    const bool glive = gw < GPW;                      // lanes past the last full group idle
    const int grp = warp * GPW + gw;

    // shared memory (from a 128-byte aligned base):
    //   slice [K][4C] f32 (the j-range of T[:, i, :], by TMA) | ew [TT+1] float4 (entry TT all zero) |
    //   xd [G][TT] f32 (x, then dx, of the tile) | cnt [K+1] | start [K+1] | tmp [32] | gbs [4C] | mbarrier
    const uint32_t base = (smem_addr(smem) + 127u) & ~127u;
    float* slice = reinterpret_cast<float*>(smem + (base - smem_addr(smem)));
    float4* ew = reinterpret_cast<float4*>(slice + (size_t)K * 4 * C);
    float* xd = reinterpret_cast<float*>(ew + TT + 1);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(xd + (size_t)TT * G);
    uint32_t* start = cnt + (K + 1);
    uint32_t* tmp = start + (K + 1);
    float* gbs = reinterpret_cast<float*>(tmp + 32);
    const uint32_t slice_s = base;
    const uint32_t ew_s = slice_s + (uint32_t)(K * C * 16);
    const uint32_t xd_s = ew_s + 16u * (uint32_t)(TT + 1);
    const uint32_t cnt_s = xd_s + 4u * (uint32_t)(TT * G);
    const uint32_t bar = (smem_addr(gbs + 4 * C) + 7u) & ~7u;
    const int j0 = blockIdx.z * 4 * C;
    const uint32_t slice_bytes = (uint32_t)(K * C * 16);
    const int KB = K < 256 ? K : 256;  // table rows per TMA box

    for (int e = threadIdx.x; e < K + 1; e += kSrtThreads) cnt[e] = 0;
    for (int e = threadIdx.x; e < 4 * C; e += kSrtThreads) gbs[e] = 0.f;
    if (threadIdx.x == 0) {
        sts_v4(ew_s + 16u * (uint32_t)TT, make_float4(0.f, 0.f, 0.f, 0.f));
        mbar_init(bar, 1);
        fence_mbar_init();
        prefetch_tensormap(&tmap);
    }
    uint32_t parity = 0;

    const int ntile = r1 > r0 ? (r1 - r0 + TT - 1) / TT : 0;
    for (int t = 0; t < ntile; ++t) {
        const int t0 = r0 + t * TT;
        const int nt = min(TT, r1 - t0);
        __syncthreads();  // the previous tile's dx has left xd
        for (int c = 0; c < G; ++c) {
            const int i = i0 + c;
            // the column's table slice T[:, i, j-range] by TMA (the previous
            // column's walk, the slice's last reader, ended at a barrier); it
            // lands while the entries are binned and sorted
            if (threadIdx.x == 0) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(bar, slice_bytes);
                for (int b = 0; b * KB < K; ++b)
                    tma_load_3d(slice_s + (uint32_t)(b * KB * C * 16), &tmap, bar, j0, i, b * KB);
            }
            if (c == 0) {
                // 0. x of the G columns of every token of the tile
                for (int tl = threadIdx.x; tl < nt; tl += kSrtThreads) {
                    float v[G];
                    load_x_cols<DT, G>(p.x, (int64_t)(t0 + tl) * IN + i0, v);
#pragma unroll
                    for (int q = 0; q < G; ++q) xd[q * TT + tl] = v[q];
                }
            }
            __syncthreads();  // x in xd; counters zero
            // 1. bins and ranks inside the bins
            uint32_t br[kSrtPer];
#pragma unroll
            for (int m = 0; m < kSrtPer; ++m) {
                const int tl = threadIdx.x + m * kSrtThreads;
                br[m] = 0;
                if (tl < nt) {
                    int lo;
                    float fr, frp;
                    bwd_bin<DT>(xd[c * TT + tl], p.cfg, lo, fr, frp);
                    br[m] = ((uint32_t)lo << 16) | atom_add_shared_u32(cnt_s + 4u * (uint32_t)lo, 1u);
                }
            }
            __syncthreads();
            // 2. bin starts
            block_exclusive_scan<kSrtThreads>(cnt, start, K, tmp);
            __syncthreads();
            // 3. entries into bin order: weights and the packed (bin, token) word
#pragma unroll
            for (int m = 0; m < kSrtPer; ++m) {
                const int tl = threadIdx.x + m * kSrtThreads;
                if (tl < nt) {
                    const float xv = xd[c * TT + tl];
                    int lo;
                    float fr, frp;
                    bwd_bin<DT>(xv, p.cfg, lo, fr, frp);
                    const float omf = __fsub_rn(1.0f, fr);
                    const float sl = clamp_passes(frp) ? __fmul_rn(xv, p.cfg.inv) : 0.0f;
                    const uint32_t pos = start[lo] + (br[m] & 0xffffu);
                    sts_v4(ew_s + 16u * pos,
                           make_float4(omf == 0.0f ? 0.0f : __fmul_rn(xv, omf), fr == 0.0f ? 0.0f : __fmul_rn(xv, fr),
                                       omf - sl, __uint_as_float(((uint32_t)lo << kSrtTokBits) | (uint32_t)tl)));
                }
            }
            for (int e = threadIdx.x; e < K + 1; e += kSrtThreads) cnt[e] = 0;  // last read by the scan
            __syncthreads();  // entries sorted; x of column c read for the last time
            mbar_wait_bounded(bar, parity);  // the slice has landed
            parity ^= 1u;
            // 4. walk: every group takes `per` consecutive entries.  `per` is
            // odd, so the 16-byte entries the groups of a warp read at one
            // step (per entries apart) fall into different bank groups
            const int per = ((nt + NG - 1) / NG) | 1;
            const int e0 = glive ? min(nt, grp * per) : nt;
            const int e1 = glive ? min(nt, e0 + per) : nt;
            const int steps = (per + kSrtDepth - 1) / kSrtDepth * kSrtDepth;
            if (p.want_gx) srt_walk<C, G, true>(p, slice_s, ew_s, xd_s, c, t0, e0, e1, steps, gl, i);
            else srt_walk<C, G, false>(p, slice_s, ew_s, xd_s, c, t0, e0, e1, steps, gl, i);
            __syncthreads();  // the next column rewrites the slice and the entries
        }
        // 5. dx of the tile's G columns
        if (p.want_gx) {
            for (int tl = threadIdx.x; tl < nt; tl += kSrtThreads) {
                float v[G];
#pragma unroll
                for (int c = 0; c < G; ++c) v[c] = xd[c * TT + tl];
                store_gx_cols<DT, G>(p.gx, (int64_t)(t0 + tl) * IN + i0, v, p.gx_atomic != 0);
            }
        }
    }
    if (p.want_gb) {
        // bias gradient of the j-range: the IN/G CTAs of a token range split
        // it into IN/G parts.  Warp w sums chunk w % C of every (32 * warps
        // per chunk)-th row from lane l's starting row, several loads in
        // flight, then reduces over its lanes by shuffles; lane 0 adds the
        // chunk into the CTA's sums (32/C-way contention only).
        const int parts = IN / G;
        const int q = (r1 - r0 + parts - 1) / parts;
        const int a0 = min(r1, r0 + (int)blockIdx.y * q), a1 = min(r1, a0 + q);
        constexpr int kWarpsPerChunk = (kSrtThreads / 32) / C;
        static_assert(kWarpsPerChunk >= 1, "every 4-column chunk of a j-range needs a warp for the bias gradient");
        const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
        if (w < kWarpsPerChunk * C) {
            const int c = w % C, wr = w / C;
            const float* gj = p.go + (int64_t)a0 * OUT + j0 + 4 * c;
            const int nrows = a1 - a0;
            constexpr int kStep = 32 * kWarpsPerChunk;
            float4 bsum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
            for (int row = wr * 32 + l; row < nrows; row += kStep) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(gj + (int64_t)row * OUT));
                bsum.x += v.x;
                bsum.y += v.y;
                bsum.z += v.z;
                bsum.w += v.w;
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                bsum.x += __shfl_xor_sync(0xffffffffu, bsum.x, o);
                bsum.y += __shfl_xor_sync(0xffffffffu, bsum.y, o);
                bsum.z += __shfl_xor_sync(0xffffffffu, bsum.z, o);
                bsum.w += __shfl_xor_sync(0xffffffffu, bsum.w, o);
            }
            if (l == 0) {
                atomicAdd(gbs + 4 * c + 0, bsum.x);
                atomicAdd(gbs + 4 * c + 1, bsum.y);
                atomicAdd(gbs + 4 * c + 2, bsum.z);
                atomicAdd(gbs + 4 * c + 3, bsum.w);
            }
        }
        __syncthreads();
        if (a1 > a0)
            for (int e = threadIdx.x; e < 4 * C; e += kSrtThreads) atomicAdd(p.gb + j0 + e, gbs[e]);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct SrtPlan {
    int C = 0, G = 1, TT = 0, R = 0, tok_per_cta = 0, smem = 0, jranges = 1;
};

constexpr int kSrtChunks[] = {32, 20, 16, 12, 10, 8, 5, 4, 2, 1};

// j-ranges of 4*C output columns: one range when OUT/4 is an instantiated C,
// else equal ranges of the widest power-of-two C <= 32 dividing OUT/4
inline bool plan_sorted(int64_t N, int K, int IN, int OUT, int sms, int G, SrtPlan& pl) {
    if (OUT % 4 != 0 || K < 1 || K > 65535 || IN > 65535) return false;
    if ((int64_t)K * IN * OUT >= ((int64_t)1 << 31)) return false;  // 32-bit gt offsets
    int C = OUT / 4, jranges = 1;
    if (C > 32) {
        int c = 32;
        while (c > 1 && (OUT / 4) % c != 0) c >>= 1;
        jranges = (OUT / 4) / c;
        C = c;
    }
    bool inst = false;
    for (int c : kSrtChunks) inst |= (c == C);
    if (!inst) return false;
    // bytes that do not scale with the tile: alignment, table slice, zero
    // entry, bin counters and starts, scan scratch, bias partials
    const int64_t fixed = 128 + (int64_t)K * C * 16 + 16 + (int64_t)(2 * K + 2) * 4 + 32 * 4 + C * 16 + 16;
    const int64_t per_tok = 16 + 4 * G;  // entry (weights + packed word) + x/dx of the G columns
    int64_t ttmax = (kSrtSmemBudget - fixed) / per_tok;
    ttmax = std::min<int64_t>(ttmax, kSrtMaxTile) / 32 * 32;
    // a tile must give the rows some reuse: below 2 entries per bin the
    // gather kernel's direct reductions are as good
    if (ttmax < 512 || ttmax < 2 * (int64_t)K) return false;
    int R = std::max(1, sms * kSrtCtasPerSm / ((IN / G) * jranges));
    R = (int)std::min<int64_t>(R, (N + 511) / 512);
    R = std::max(R, 1);
    const int64_t S = (N + R - 1) / R;
    const int64_t ntile = (S + ttmax - 1) / ttmax;
    const int64_t tt = std::min<int64_t>(ttmax, ((S + ntile - 1) / ntile + 31) / 32 * 32);
    const int64_t per = ((S + tt - 1) / tt) * tt;  // tiles of one CTA tile its range exactly
    R = (int)((N + per - 1) / per);
    if (per > INT32_MAX / 2) return false;
    pl = {C, G, (int)tt, R, (int)per, (int)(fixed + per_tok * tt), jranges};
    return true;
}

template <int DT, int C>
inline int launch_sorted(const CUtensorMap& map, const SrtArgs& a, const SrtPlan& pl, cudaStream_t s) {
    auto kern = pl.G == kSrtG ? bwd_sorted_kernel<DT, C, kSrtG> : bwd_sorted_kernel<DT, C, 1>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess)
        return 4;
    kern<<<dim3((unsigned)pl.R, (unsigned)(a.IN / pl.G), (unsigned)pl.jranges), kSrtThreads, pl.smem, s>>>(map, a);
    return 0;
}

template <int DT>
inline int launch_sorted_c(const CUtensorMap& map, const SrtArgs& a, const SrtPlan& pl, cudaStream_t s) {
    switch (pl.C) {
        case 32: return launch_sorted<DT, 32>(map, a, pl, s);
        case 20: return launch_sorted<DT, 20>(map, a, pl, s);
        case 16: return launch_sorted<DT, 16>(map, a, pl, s);
        case 12: return launch_sorted<DT, 12>(map, a, pl, s);
        case 10: return launch_sorted<DT, 10>(map, a, pl, s);
        case 8: return launch_sorted<DT, 8>(map, a, pl, s);
        case 5: return launch_sorted<DT, 5>(map, a, pl, s);
        case 4: return launch_sorted<DT, 4>(map, a, pl, s);
        case 2: return launch_sorted<DT, 2>(map, a, pl, s);
        default: return launch_sorted<DT, 1>(map, a, pl, s);
    }
}

inline bool sorted_backward_ok(const float* go, const void* x, int x_dtype, const float* table, const void* gx,
                               const float* gt, const float* gb, int64_t N, int64_t IN, int64_t OUT,
                               int64_t K, const BinCfg& c) {
    if (!c.pow2 || gt == nullptr) return false;  // bins written for bw = 2^-e; gt is what it is for
    if (N > ((int64_t)1 << 30) || IN > 65535 || K > 65535) return false;
    if (((uintptr_t)go | (uintptr_t)table | (uintptr_t)gt) & 15) return false;
    if (x_dtype == kBF16 ? (((uintptr_t)x | (uintptr_t)gx) & 1) : (((uintptr_t)x | (uintptr_t)gx) & 3))
        return false;
    (void)gb;
    return true;
}

// gt and gb must already be zero.  Returns kNotApplicable when the shape has
// no plan (the caller then takes the gather kernel or the general kernels).
inline int sorted_backward(const float* go, const void* x, int x_dtype, const float* table, void* gx, float* gt,
                           float* gb, int64_t N, int64_t IN, int64_t OUT, const BinCfg& c, int sms,
                           cudaStream_t s) {
    // G = kSrtG columns per CTA (one 16-byte load of x and one 16-byte store
    // of dx per token and CTA instead of four strided 4-byte ones) when in_d
    // allows it (in_d % 4 == 0, 16-byte aligned rows, 8-byte for bf16) and the
    // CTA's tokens fit one tile of at least 2048: the G columns run one after
    // another, so small batches keep one column per CTA for parallelism, and
    // several tiles would reload every column's slice per tile.
    const int xalign = x_dtype == kBF16 ? 8 : 16;
    const bool g4ok = IN % kSrtG == 0 && ((uintptr_t)x % xalign) == 0 && (gx == nullptr || ((uintptr_t)gx % xalign) == 0);
    SrtPlan pl;
    bool planned = false;
    if (g4ok && plan_sorted(N, c.K, (int)IN, (int)OUT, sms, kSrtG, pl))
        planned = pl.tok_per_cta <= pl.TT && pl.tok_per_cta >= 2048;
    if (!planned && !plan_sorted(N, c.K, (int)IN, (int)OUT, sms, 1, pl)) return kNotApplicable;
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, 4 * pl.C, c.K < 256 ? c.K : 256)) return kNotApplicable;
    // with several j-ranges each adds its part of dx: fp32 gx only, zeroed first
    const bool gx_atomic = pl.jranges > 1 && gx != nullptr;
    if (gx_atomic) {
        if (x_dtype != kF32) return kNotApplicable;
        if (cudaMemsetAsync(gx, 0, (size_t)(N * IN) * sizeof(float), s) != cudaSuccess) return 4;
    }
    SrtArgs a;
    a.go = go;
    a.x = x;
    a.table = table;
    a.gx = gx;
    a.gt = gt;
    a.gb = gb;
    a.N = (int)N;
    a.IN = (int)IN;
    a.OUT = (int)OUT;
    a.K = c.K;
    a.G = pl.G;
    a.TT = pl.TT;
    a.tok_per_cta = pl.tok_per_cta;
    a.want_gx = gx != nullptr;
    a.want_gb = gb != nullptr;
    a.gx_atomic = gx_atomic ? 1 : 0;
    a.cfg = c;
    return x_dtype == kBF16 ? launch_sorted_c<kBF16>(map, a, pl, s) : launch_sorted_c<kF32>(map, a, pl, s);
}

}  // namespace il
