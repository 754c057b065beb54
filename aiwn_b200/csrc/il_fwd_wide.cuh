// il_fwd_wide.cuh -- forward for wide rows over few bins: out_d a multiple of
// 128 and K <= 128, e.g. IndexedLinear(1024, 1024, K=64) with its 256 MB table.
//
// The math is aiwn/layers/indexed_linear.py:173-182 (the same as the other
// forwards): out[n, j] = bias[j] + sum_i x(1-fr) T[lo, i, j] + x fr T[hi, i, j].
//
// Layout.  A CTA owns one j-range of 128 output columns and MW*W tokens; each
// of its W consumer warps owns MW of those tokens and keeps their 128 x MW
// accumulators in registers (lane l: columns j0+4l .. j0+4l+3 of every token).
// A warp works on ONE token at a time, so the 32 lanes of a table-row read
// cover one contiguous 512-byte row of the slice: every quarter-warp reads an
// aligned 128-byte line, which is conflict-free whatever the row -- the gather
// kernels' per-lane random rows cost ~8.7 wavefronts per 128-bit load against
// 4 here.  The row and the two weights of each (token, column) are computed
// once per warp into shared memory and read back as a broadcast.
//
// The table streams through kWideStages shared-memory stages of CB input
// columns each (one TMA box {128 floats, CB columns, K rows}, laid out
// [K][CB][128]); a producer warp refills a stage once every consumer warp has
// released it (per-stage full/empty mbarriers, bounded waits).
#pragma once
#include "il_fast.cuh"
#include "il_sm100.cuh"

namespace il {

constexpr int kWideJ = 128;   // output columns per CTA (32 lanes x 4)
constexpr int kWideEB = 8;    // input columns per block of (row, weight) entries
constexpr int kWideStages = 3;
constexpr int kWideStageMax = 64 * 1024;
constexpr int kWideMW = 16;   // tokens per consumer warp (their accumulators stay in registers)
// consumer warps per CTA, at most (with the producer warp: 512 threads for MW = 16,
// so that 128 registers per thread fit; 288 for MW = 32)
__host__ __device__ constexpr int wide_max_warps(int mw) { return mw >= 32 ? 8 : 15; }
// one warp's entry block: kWideEB columns of MW + 1 entries (16 bytes each; the
// padding entry staggers the columns over the bank groups, so that the eight
// lanes of a quarter-warp, one column each, store without conflicts)
__host__ __device__ constexpr int wide_entry_bytes(int mw) { return (mw + 1) * kWideEB * 16; }

struct WideArgs {
    const void* x;
    const float* bias;
    float* out;
    int N, IN, OUT, K;
    int nchunks;      // IN / CB
    int warps;        // consumer warps; tokens per CTA = MW * warps
    int stage_bytes;  // K * CB * 512
    BinCfg cfg;
};

template <int DT, int CB, int MW>
__global__ void __launch_bounds__(32 * (wide_max_warps(MW) + 1), 1)
    fwd_wide_kernel(const __grid_constant__ CUtensorMap tmap, const WideArgs p) {
    constexpr int kEntryBytes = wide_entry_bytes(MW);
    extern __shared__ unsigned char smem[];
    static_assert(kWideEB % CB == 0, "entry blocks hold whole chunks");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int W = p.warps;
    const uint32_t sbase = smem_addr(smem);
    const uint32_t pad = ((sbase + 1023u) & ~1023u) - sbase;
    unsigned char* const stages = smem + pad;
    unsigned char* const entries = stages + kWideStages * p.stage_bytes;
    const uint32_t full = smem_addr(entries + W * kEntryBytes);
    const uint32_t empty = full + 8u * kWideStages;
    const int j0 = blockIdx.y * kWideJ;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWideStages; ++s) {
            mbar_init(full + 8u * s, 1);
            mbar_init(empty + 8u * s, (uint32_t)W);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == W) {
        // producer: stage ch % S receives chunk ch once chunk ch - S is released
        if (lane == 0) {
            prefetch_tensormap(&tmap);
            for (int ch = 0; ch < p.nchunks; ++ch) {
                const int st = ch % kWideStages;
                if (ch >= kWideStages) {
                    mbar_wait_bounded(empty + 8u * st, (uint32_t)((ch / kWideStages - 1) & 1));
                    fence_proxy_async_smem();  // the consumers' reads before the async-proxy refill
                }
                mbar_arrive_expect_tx(full + 8u * st, (uint32_t)p.stage_bytes);
                tma_load_3d(smem_addr(stages + st * p.stage_bytes), &tmap, full + 8u * st, j0, ch * CB, 0);
            }
        }
        return;
    }

    const int IN = p.IN, K = p.K;
    const int tok0 = (int)blockIdx.x * (MW * W) + warp * MW;
    unsigned char* const ent = entries + warp * kEntryBytes;
    constexpr uint32_t kRow = 512u;               // one row of one column in a stage
    constexpr uint32_t kRowK = (uint32_t)CB * kRow;  // rows k and k+1 of a column
    float4 acc[MW];
#pragma unroll
    for (int m = 0; m < MW; ++m) acc[m] = make_float4(0.f, 0.f, 0.f, 0.f);

    // entry (column c0 + e, token m) at ent + (e * (MW + 1) + m) * 16:
    // {byte offset of row lo, byte offset of row hi, x(1-fr), x fr}.
    // Lane (eq, es) computes tokens eq, eq+4, .. of column c0 + es; the x
    // values of the next block load while this block's chunks are used.
    const int es = lane & 7, eq = lane >> 3;
    constexpr int kPasses = MW / 4;
    float xnext[kPasses];
    auto load_block_x = [&](int c0) {
        const int col = c0 + es;
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
            const int n = tok0 + pass * 4 + eq;
            xnext[pass] = (n < p.N && col < IN) ? load_x<DT>(p.x, (int64_t)n * IN + col) : 0.0f;
        }
    };
    load_block_x(0);
    for (int c0 = 0; c0 < IN; c0 += kWideEB) {
        const int col = c0 + es;
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
            const int m = pass * 4 + eq;
            const int n = tok0 + m;
            const bool ok = n < p.N && col < IN;
            int lo;
            float wa, wc;
            gather_weights<DT>(xnext[pass], p.cfg, lo, wa, wc);
            const uint32_t olo = (uint32_t)lo * kRowK + (uint32_t)(es % CB) * kRow;
            const uint32_t ohi = olo + (lo < K - 1 ? kRowK : 0u);  // hi = min(lo+1, K-1)
            *reinterpret_cast<float4*>(ent + (es * (MW + 1) + m) * 16) =
                make_float4(__uint_as_float(olo), __uint_as_float(ohi), ok ? wa : 0.0f, ok ? wc : 0.0f);
        }
        if (c0 + kWideEB < IN) load_block_x(c0 + kWideEB);
        __syncwarp();
#pragma unroll 1
        for (int cc = 0; cc < kWideEB / CB; ++cc) {
            const int ch = c0 / CB + cc;
            if (ch >= p.nchunks) break;
            const int st = ch % kWideStages;
            mbar_wait_bounded(full + 8u * st, (uint32_t)((ch / kWideStages) & 1));
            const unsigned char* const buf = stages + st * p.stage_bytes + 16 * lane;
#pragma unroll 1
            for (int s = 0; s < CB; ++s) {
                const float4* const e = reinterpret_cast<const float4*>(ent + (cc * CB + s) * (MW + 1) * 16);
#pragma unroll
                for (int m = 0; m < MW; ++m) {
                    const float4 w = e[m];
                    const float4 tl = *reinterpret_cast<const float4*>(buf + __float_as_uint(w.x));
                    const float4 th = *reinterpret_cast<const float4*>(buf + __float_as_uint(w.y));
                    acc[m].x = fmaf(w.z, tl.x, acc[m].x);
                    acc[m].y = fmaf(w.z, tl.y, acc[m].y);
                    acc[m].z = fmaf(w.z, tl.z, acc[m].z);
                    acc[m].w = fmaf(w.z, tl.w, acc[m].w);
                    acc[m].x = fmaf(w.w, th.x, acc[m].x);
                    acc[m].y = fmaf(w.w, th.y, acc[m].y);
                    acc[m].z = fmaf(w.w, th.z, acc[m].z);
                    acc[m].w = fmaf(w.w, th.w, acc[m].w);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8u * st);
        }
        __syncwarp();  // the entry block is rewritten next
    }

    const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + j0) + lane);
#pragma unroll
    for (int m = 0; m < MW; ++m) {
        const int n = tok0 + m;
        if (n < p.N)
            *reinterpret_cast<float4*>(p.out + (int64_t)n * p.OUT + j0 + 4 * lane) =
                make_float4(acc[m].x + b.x, acc[m].y + b.y, acc[m].z + b.z, acc[m].w + b.w);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct WidePlan {
    int CB = 0, warps = 0, stage_bytes = 0, smem = 0;
};

// CB: the most input columns (1, 2, 4 or 8, dividing in_d) whose stage fits
// 64 KB; W: consumer warps minimising (waves of CTAs) x W, the larger W on ties
inline bool plan_wide_forward(int64_t N, int K, int IN, int OUT, int sms, WidePlan& pl) {
    if (OUT % kWideJ != 0 || K < 1 || K > 128 || IN < 1) return false;
    int CB = 8;
    while (CB > 1 && (CB * K * 512 > kWideStageMax || IN % CB != 0)) CB >>= 1;
    if (CB * K * 512 > kWideStageMax) return false;
    const int64_t jr = OUT / kWideJ;
    constexpr int kMax = wide_max_warps(kWideMW);
    int best_w = 0;
    int64_t best = 0;
    for (int w = kMax; w >= 4; --w) {
        const int64_t ctas = (N + kWideMW * w - 1) / (kWideMW * w) * jr;
        const int64_t cost = (ctas + sms - 1) / sms * w;
        if (best_w == 0 || cost < best) {
            best = cost;
            best_w = w;
        }
    }
    pl.CB = CB;
    pl.warps = best_w;
    pl.stage_bytes = CB * K * 512;
    pl.smem = 1024 + kWideStages * pl.stage_bytes + best_w * wide_entry_bytes(kWideMW) + 16 * kWideStages;
    return pl.smem <= kSmemBudget + 1024;
}

template <int DT, int CB>
inline int launch_wide_fwd(const CUtensorMap& map, const WideArgs& a, const WidePlan& pl, cudaStream_t s) {
    auto kern = fwd_wide_kernel<DT, CB, kWideMW>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess) return 4;
    const dim3 grid((unsigned)ceil_div(a.N, kWideMW * pl.warps), (unsigned)(a.OUT / kWideJ), 1);
    kern<<<grid, 32 * (pl.warps + 1), pl.smem, s>>>(map, a);
    return 0;
}

template <int DT>
inline int launch_wide_fwd_cb(const CUtensorMap& map, const WideArgs& a, const WidePlan& pl, cudaStream_t s) {
    switch (pl.CB) {
        case 8: return launch_wide_fwd<DT, 8>(map, a, pl, s);
        case 4: return launch_wide_fwd<DT, 4>(map, a, pl, s);
        case 2: return launch_wide_fwd<DT, 2>(map, a, pl, s);
        default: return launch_wide_fwd<DT, 1>(map, a, pl, s);
    }
}

// kNotApplicable when the shape has no plan
inline int wide_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out, int64_t N,
                        int64_t IN, int64_t OUT, const BinCfg& c, int sms, cudaStream_t s) {
    WidePlan pl;
    if (!plan_wide_forward(N, c.K, (int)IN, (int)OUT, sms, pl)) return kNotApplicable;
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, kWideJ, c.K, pl.CB)) return kNotApplicable;
    WideArgs a;
    a.x = x;
    a.bias = bias;
    a.out = out;
    a.N = (int)N;
    a.IN = (int)IN;
    a.OUT = (int)OUT;
    a.K = c.K;
    a.nchunks = (int)IN / pl.CB;
    a.warps = pl.warps;
    a.stage_bytes = pl.stage_bytes;
    a.cfg = c;
    return x_dtype == kBF16 ? launch_wide_fwd_cb<kBF16>(map, a, pl, s) : launch_wide_fwd_cb<kF32>(map, a, pl, s);
}

}  // namespace il
