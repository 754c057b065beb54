// il_fwd_wide.cuh -- forward for wide rows over few bins: out_d a multiple of
// 64 and K <= 128, e.g. IndexedLinear(1024, 1024, K=64) with its 256 MB table.
//
// The math is aiwn/layers/indexed_linear.py:173-182 (the same as the other
// forwards): out[n, j] = bias[j] + sum_i x(1-fr) T[lo, i, j] + x fr T[hi, i, j].
//
// Layout.  A CTA owns one j-range of JW = 128 (or 64) output columns and MW*W
// tokens; each of its W consumer warps owns MW of those tokens and keeps their
// accumulators in registers (lane l: columns j0+4(l%(JW/4)) .. +3).  A warp
// works on ONE token at a time (JW = 128) or two (JW = 64, one per half-warp),
// so the lanes of a table-row read cover contiguous 512- (256-) byte rows of
// the slice: every quarter-warp reads one aligned 128-byte line, which is
// conflict-free whatever the row -- the gather kernels' per-lane random rows
// cost ~8.7 wavefronts per 128-bit load against 4 here.  The row and the two
// weights of each (token, column) are computed once per warp into shared
// memory and read back as a broadcast.
//
// The table streams through kWideStages shared-memory stages of CB input
// columns each (one TMA box {JW floats, CB columns, K rows}, laid out
// [K][CB][JW]); a producer warp refills a stage once every consumer warp has
// released it (per-stage full/empty mbarriers, bounded waits).
#pragma once
#include "il_fast.cuh"
#include "il_sm100.cuh"

namespace il {

constexpr int kWideEB = 8;    // input columns per block of (row, weight) entries
constexpr int kWideStages = 3;
// tokens per consumer warp: 16 accumulators of float4 per lane either way
__host__ __device__ constexpr int wide_mw(int jw) { return jw >= 128 ? 16 : 32; }
// bytes per stage, at most (the 64-wide kernel's entry blocks are twice as large)
__host__ __device__ constexpr int wide_stage_max(int jw) { return jw >= 128 ? 64 * 1024 : 32 * 1024; }
// consumer warps per CTA, at most (with the producer warp: 512 threads, so
// that 128 registers per thread fit)
__host__ __device__ constexpr int wide_max_warps(int mw) { return mw >= 64 ? 8 : 15; }
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
    int stage_bytes;  // K * CB * JW * 4
    BinCfg cfg;
};

template <int DT, int CB, int JW>
__global__ void __launch_bounds__(32 * (wide_max_warps(wide_mw(JW)) + 1), 1)
    fwd_wide_kernel(const __grid_constant__ CUtensorMap tmap, const WideArgs p) {
    constexpr int MW = wide_mw(JW);
    constexpr int LPT = JW / 4;         // lanes per token
    constexpr int TPS = 32 / LPT;       // tokens per warp step
    constexpr int NACC = MW / TPS;      // accumulators per lane
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
    const int j0 = blockIdx.y * JW;

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
    constexpr uint32_t kRow = (uint32_t)JW * 4u;      // one row of one column in a stage
    constexpr uint32_t kRowK = (uint32_t)CB * kRow;  // rows k and k+1 of a column
    const int ts = lane / LPT, cl = lane % LPT;     // token of the step, chunk of the row
    float4 acc[NACC];
#pragma unroll
    for (int q = 0; q < NACC; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);

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
            const unsigned char* const buf = stages + st * p.stage_bytes + 16 * cl;
#pragma unroll 1
            for (int s = 0; s < CB; ++s) {
                const float4* const e = reinterpret_cast<const float4*>(ent + (cc * CB + s) * (MW + 1) * 16);
#pragma unroll
                for (int q = 0; q < NACC; ++q) {
                    const float4 w = e[q * TPS + ts];
                    const float4 tl = *reinterpret_cast<const float4*>(buf + __float_as_uint(w.x));
                    const float4 th = *reinterpret_cast<const float4*>(buf + __float_as_uint(w.y));
                    acc[q].x = fmaf(w.z, tl.x, acc[q].x);
                    acc[q].y = fmaf(w.z, tl.y, acc[q].y);
                    acc[q].z = fmaf(w.z, tl.z, acc[q].z);
                    acc[q].w = fmaf(w.z, tl.w, acc[q].w);
                    acc[q].x = fmaf(w.w, th.x, acc[q].x);
                    acc[q].y = fmaf(w.w, th.y, acc[q].y);
                    acc[q].z = fmaf(w.w, th.z, acc[q].z);
                    acc[q].w = fmaf(w.w, th.w, acc[q].w);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8u * st);
        }
        __syncwarp();  // the entry block is rewritten next
    }

    const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + j0) + cl);
#pragma unroll
    for (int q = 0; q < NACC; ++q) {
        const int n = tok0 + q * TPS + ts;
        if (n < p.N)
            *reinterpret_cast<float4*>(p.out + (int64_t)n * p.OUT + j0 + 4 * cl) =
                make_float4(acc[q].x + b.x, acc[q].y + b.y, acc[q].z + b.z, acc[q].w + b.w);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct WidePlan {
    int JW = 0, CB = 0, warps = 0, stage_bytes = 0, smem = 0;
};

// the warp-per-token forward's j-range width for out_d, 0 when it has none
inline int wide_jw(int64_t OUT) { return OUT % 128 == 0 ? 128 : (OUT % 64 == 0 ? 64 : 0); }

// JW: 128 when out_d % 128 == 0, else 64 when out_d % 64 == 0.  CB: the most
// input columns (1, 2, 4 or 8, dividing in_d) whose stage fits the stage
// limit; W: consumer warps minimising (waves of CTAs) x W, the larger W on ties
inline bool plan_wide_forward(int64_t N, int K, int IN, int OUT, int sms, WidePlan& pl) {
    const int JW = wide_jw(OUT);
    if (JW == 0 || K < 1 || K > 128 || IN < 1) return false;
    const int row = JW * 4, smax = wide_stage_max(JW), MW = wide_mw(JW);
    int CB = 8;
    while (CB > 1 && (CB * K * row > smax || IN % CB != 0)) CB >>= 1;
    if (CB * K * row > smax) return false;
    const int64_t jr = OUT / JW;
    const int kMax = wide_max_warps(MW);
    int best_w = 0;
    int64_t best = 0;
    for (int w = kMax; w >= 4; --w) {
        const int64_t ctas = (N + MW * w - 1) / (MW * w) * jr;
        const int64_t cost = (ctas + sms - 1) / sms * w;
        if (best_w == 0 || cost < best) {
            best = cost;
            best_w = w;
        }
    }
    pl.JW = JW;
    pl.CB = CB;
    pl.warps = best_w;
    pl.stage_bytes = CB * K * row;
    pl.smem = 1024 + kWideStages * pl.stage_bytes + best_w * wide_entry_bytes(MW) + 16 * kWideStages;
    return pl.smem <= kSmemBudget + 1024;
}

template <int DT, int CB, int JW>
inline int launch_wide_fwd(const CUtensorMap& map, const WideArgs& a, const WidePlan& pl, cudaStream_t s) {
    auto kern = fwd_wide_kernel<DT, CB, JW>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess) return 4;
    const dim3 grid((unsigned)ceil_div(a.N, wide_mw(JW) * pl.warps), (unsigned)(a.OUT / JW), 1);
    kern<<<grid, 32 * (pl.warps + 1), pl.smem, s>>>(map, a);
    return 0;
}

template <int DT, int JW>
inline int launch_wide_fwd_cb(const CUtensorMap& map, const WideArgs& a, const WidePlan& pl, cudaStream_t s) {
    switch (pl.CB) {
        case 8: return launch_wide_fwd<DT, 8, JW>(map, a, pl, s);
        case 4: return launch_wide_fwd<DT, 4, JW>(map, a, pl, s);
        case 2: return launch_wide_fwd<DT, 2, JW>(map, a, pl, s);
        default: return launch_wide_fwd<DT, 1, JW>(map, a, pl, s);
    }
}

template <int DT>
inline int launch_wide_fwd_jw(const CUtensorMap& map, const WideArgs& a, const WidePlan& pl, cudaStream_t s) {
    return pl.JW == 128 ? launch_wide_fwd_cb<DT, 128>(map, a, pl, s) : launch_wide_fwd_cb<DT, 64>(map, a, pl, s);
}

// kNotApplicable when the shape has no plan
inline int wide_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out, int64_t N,
                        int64_t IN, int64_t OUT, const BinCfg& c, int sms, cudaStream_t s) {
    WidePlan pl;
    if (!plan_wide_forward(N, c.K, (int)IN, (int)OUT, sms, pl)) return kNotApplicable;
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, pl.JW, c.K, pl.CB)) return kNotApplicable;
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
    return x_dtype == kBF16 ? launch_wide_fwd_jw<kBF16>(map, a, pl, s) : launch_wide_fwd_jw<kF32>(map, a, pl, s);
}

}  // namespace il
