// il_fast.cuh -- shape-specialised IndexedLinear kernels for B200 (sm_100a).
//
// Data layout and work split (forward):
//   * table [K, IN, OUT] fp32 stays in HBM in the reference's layout.  A CTA
//     keeps the slices T[:, i, j0:j0+JR] of its input columns i resident in
//     shared memory, loaded once per CTA with TMA tensor copies; every slice
//     is K rows of JR floats, so rows lo and lo+1 of one slice are adjacent.
//   * Input columns are split across the CTAs of a thread-block cluster
//     (rank r owns i in [r*IG, (r+1)*IG)) so that large tables fit: each CTA
//     computes a partial sum over its columns and the partials of a token
//     are added across the cluster through distributed shared memory, in a
//     fixed rank order (deterministic).
//   * Output columns beyond one CTA's shared memory are split into j-ranges
//     over grid.y (independent CTAs, no reduction).
//   * Lanes are mapped to (token, 16-byte chunk of the lo|hi row pair): a
//     token's run of 2*JR floats (row lo followed by row lo+1) is read with
//     128-bit loads, 8 consecutive chunks per shared-memory wavefront.
//
// Bucketing is bit-exact with aiwn/layers/indexed_linear.py:175-177 (see
// il_common.cuh); the lerp-and-accumulate reorders the reference's fp32 sum
// (IL:181-182) and agrees with it to ~1e-7 relative.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <numeric>

#include "il_common.cuh"
#include "il_sm100.cuh"
#include "il_dtable.cuh"

namespace il {

// ---------------------------------------------------------------------------
// lane -> (token, chunk) mapping for runs of R = 2*C chunks
// ---------------------------------------------------------------------------
template <int C>
struct RunMap {
    static constexpr int R = 2 * C;                         // chunks per token run
    static constexpr int P = R >= 32 ? 1 : 32 / R;          // tokens per warp
    static constexpr int U = R >= 32 ? (R + 31) / 32 : 1;   // chunk slots per lane
    static constexpr int Q = R < 32 ? R / 8 : 0;            // full 8-chunk groups per token
    static constexpr int RR = R < 32 ? R % 8 : 0;           // leftover chunks per token

    // (t, c) of `lane` in slot u, false if the lane is idle in that slot
    __device__ __forceinline__ static bool map(int lane, int u, int& t, int& c) {
        if constexpr (R >= 32) {
            t = 0;
            c = lane + 32 * u;
            return c < R;
        } else if constexpr (Q == 0) {
            t = lane / R;
            c = lane % R;
            return t < P;
        } else {
            constexpr int kMain = P * 8 * Q;
            if (lane < kMain) {
                t = lane / (8 * Q);
                c = lane % (8 * Q);
                return true;
            }
            const int m = lane - kMain;
            t = RR > 0 ? m / (RR > 0 ? RR : 1) : 0;
            c = 8 * Q + (RR > 0 ? m % (RR > 0 ? RR : 1) : 0);
            return RR > 0 && m < P * RR;
        }
    }
    // lane and slot holding chunk c of token t
    __device__ __forceinline__ static void where(int t, int c, int& lane, int& u) {
        if constexpr (R >= 32) {
            lane = c & 31;
            u = c >> 5;
        } else if constexpr (Q == 0) {
            lane = t * R + c;
            u = 0;
        } else {
            u = 0;
            if (c < 8 * Q) lane = t * 8 * Q + c;
            else lane = P * 8 * Q + t * (RR > 0 ? RR : 1) + (c - 8 * Q);
        }
    }
};

// Bucket of one input element for the gather: the low row `lo` and the
// weights wa = x*(1-fr) of row lo and wc = x*fr of row lo+1.  Every table
// slice in shared memory carries one extra row K, a copy of row K-1, so the
// reference's hi = min(lo+1, K-1) is always row lo+1.  Bins are bit-exact
// with aiwn/layers/indexed_linear.py:175-177 for bw = 2^-e (every K that is a
// power of two): divisions by bw are then exact scalings, and
//   (x+1)/bw == fma(x, 1/bw, 1/bw),   -1 + lo*bw == fma(lo, bw, -1)
// round identically to the reference's separate operations.
template <int DT>
__device__ __forceinline__ void gather_weights(float xv, const BinCfg& c, int& lo, float& wa,
                                               float& wc) {
    float q;
    if constexpr (DT == kBF16) {
        q = bf16_round(__fmul_rn(bf16_round(__fadd_rn(xv, 1.0f)), c.inv));
    } else {
        q = __fmaf_rn(xv, c.inv, c.inv);
    }
    float t = fminf(fmaxf(truncf(q), 0.0f), (float)(c.K - 1));
    if (!(fabsf(q) < 9.2233720368547758e18f)) t = 0.0f;  // x86 .long() of NaN / |q| >= 2^63
    const float fr = __saturatef(__fmul_rn(__fsub_rn(xv, __fmaf_rn(t, c.bw, -1.0f)), c.inv));
    const float omf = __fsub_rn(1.0f, fr);
    // a zero weight stays exactly zero (as tlo*0 does in the reference) even for x = +-inf
    wa = omf == 0.0f ? 0.0f : __fmul_rn(xv, omf);
    wc = fr == 0.0f ? 0.0f : __fmul_rn(xv, fr);
    lo = (int)t;
}

// ---------------------------------------------------------------------------
// forward kernel
// ---------------------------------------------------------------------------
struct FwdArgs {
    const void* x;
    const float* bias;
    float* out;
    int N, IN, OUT, K;
    int JR;           // j-range width (floats) = 4*C
    int RS;           // row stride of a table slice in shared memory (floats, >= JR)
    int xvec;         // x rows can be read 4 elements at a time (aligned, IN % 4 == 0)
    int IG;           // input columns per CTA of a cluster
    int KB;           // rows per TMA box
    int nbox;         // boxes per slice
    int slice_bytes;  // shared-memory stride between slices
    int ntiles;       // token tiles
    BinCfg cfg;
    unsigned long long* counts = nullptr;  // token kernel: bin-occupancy histogram [K] added into (or none)
};

#ifndef IL_FWD_THREADS
#define IL_FWD_THREADS 1024
#endif
constexpr int kFwdThreads = IL_FWD_THREADS;
constexpr int kWarps = kFwdThreads / 32;
#ifndef IL_FWD_SLOTS
#define IL_FWD_SLOTS 2
#endif
#ifndef IL_FWD_XB
#define IL_FWD_XB 8
#endif
constexpr int kSlots = IL_FWD_SLOTS;  // token slots per lane
constexpr int kXB = IL_FWD_XB;        // input columns handled per weights pass

template <int C>
__host__ __device__ constexpr int fwd_tile_tokens() {
    return RunMap<C>::P * kWarps * kSlots;
}

// Partial sums of a tile are exchanged inside the cluster with st.async into
// the owner CTA's receive buffer [CS producers][TT/CS tokens][C] float4:
// `full` (owner side, 1 arrival + bytes) completes when every producer's
// partials arrived; `empty` (producer side, CS arrivals) completes when every
// owner has consumed the producer's previous tile.
template <int DT, int C, int CS>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_cluster_kernel(const __grid_constant__ CUtensorMap tmap, const FwdArgs p) {
    using M = RunMap<C>;
    constexpr int TT = fwd_tile_tokens<C>();
    constexpr int TTQ = TT / CS;
    static_assert(TT % CS == 0, "tile must split evenly over the cluster");
    extern __shared__ unsigned char smem[];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rank = CS > 1 ? (int)cluster_ctarank() : 0;
    const int i0 = rank * p.IG;
    const int ig = max(0, min(p.IG, p.IN - i0));
    const int j0 = blockIdx.y * p.JR;
    // layout from a 128-byte aligned base: IG table slices | receive buffer | 3 mbarriers
    const uint32_t table_s = (smem_addr(smem) + 127u) & ~127u;
    const uint32_t recv_s = table_s + (uint32_t)(p.IG * p.slice_bytes);
    const uint32_t bar_tma = recv_s + (uint32_t)(CS > 1 ? TT * C * 16 : 0);
    const uint32_t bar_full = bar_tma + 8, bar_empty = bar_tma + 16;

    if (threadIdx.x == 0) {
        prefetch_tensormap(&tmap);
        mbar_init(bar_tma, 1);
        mbar_init(bar_full, 1);
        mbar_init(bar_empty, CS);
        fence_mbar_init();
        if (ig > 0) {
            mbar_arrive_expect_tx(bar_tma, (uint32_t)(ig * p.nbox * p.KB * p.JR * 4));
            for (int s = 0; s < ig; ++s)
                for (int b = 0; b < p.nbox; ++b)
                    tma_load_3d(table_s + s * p.slice_bytes + b * p.KB * p.JR * 4, &tmap, bar_tma,
                                j0, i0 + s, b * p.KB);
        }
    }
    if constexpr (CS > 1) cluster_sync();  // every mbarrier of the cluster is initialised
    else __syncthreads();
    if (ig > 0) mbar_wait_bounded(bar_tma, 0);
    // row K of every slice = row K-1 (the reference's hi for the top bin)
    for (int e = threadIdx.x; e < ig * (p.JR / 4); e += kFwdThreads) {
        const int s = e / (p.JR / 4), c4 = e - s * (p.JR / 4);
        const uint32_t sl = table_s + (uint32_t)(s * p.slice_bytes);
        sts_v4(sl + (uint32_t)(p.K * p.JR * 4 + c4 * 16), lds_v4(sl + (uint32_t)((p.K - 1) * p.JR * 4 + c4 * 16)));
    }
    __syncthreads();

    int tl[M::U], ch[M::U];
    bool act[M::U];
#pragma unroll
    for (int u = 0; u < M::U; ++u) act[u] = M::map(lane, u, tl[u], ch[u]);
    const uint32_t row_stride = (uint32_t)p.JR * 4;
    uint32_t coff[M::U];  // byte offset of this lane's chunk inside its row
    bool hs[M::U];        // chunk belongs to row lo+1
#pragma unroll
    for (int u = 0; u < M::U; ++u) {
        hs[u] = ch[u] >= C;
        coff[u] = (uint32_t)((ch[u] - (hs[u] ? C : 0)) * 16);
    }
    const int cid = CS > 1 ? (int)cluster_id_x() : (int)blockIdx.x;
    const int ncl = CS > 1 ? (int)nclusters_x() : (int)gridDim.x;

    constexpr int XB = M::P >= 8 ? 2 : kXB;                // columns per weights pass
    constexpr int kSpr = 16 / M::P;                        // steps per weight register
    constexpr int kNR = (kSlots * XB + kSpr - 1) / kSpr;   // weight registers per block
    const int pj = lane >> 1, pv = lane & 1;               // pair of this lane, lo/hi view
    const int pt = pj % M::P, pst = pj / M::P;             // its token, step in register
    // x values of the pairs this lane computes weights for, block (t, sb)
    auto load_block_x = [&](int t, int sb_, float (&dst)[kNR]) {
        const int nq_ = min(XB, ig - sb_);
#pragma unroll
        for (int r = 0; r < kNR; ++r) {
            const int st = r * kSpr + pst;
            const int q = st / kSlots, sl = st - q * kSlots;
            const int n = t * TT + sl * (M::P * kWarps) + warp * M::P + pt;
            const bool ok = t < p.ntiles && pj < kSpr * M::P && q < nq_ && n < p.N;
            dst[r] = ok ? load_x<DT>(p.x, (int64_t)n * p.IN + i0 + sb_ + q) : 0.0f;
        }
    };
    float xpre[kNR];
    load_block_x(cid, 0, xpre);

    int k = 0;
    for (int tile = cid; tile < p.ntiles; tile += ncl, ++k) {
        float4 acc[kSlots][M::U];
        int tok[kSlots];
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
            tok[sl] = sl * (M::P * kWarps) + warp * M::P + tl[0];
#pragma unroll
            for (int u = 0; u < M::U; ++u) acc[sl][u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        // Weights of the warp's (token, column) pairs, two lanes per pair:
        // lane 2j holds (byte offset of row lo, x(1-fr)), lane 2j+1 holds
        // (byte offset of row lo+1, x fr) of pair j.  Pair j of register r
        // is step st = r*kSpr + j/P (st = q*kSlots + slot) of token j%P.
        // The x values of the next block (possibly of the next tile) are
        // loaded before this block's gather, so their latency is hidden.
        for (int sb = 0; sb < ig; sb += XB) {
            const int nq = min(XB, ig - sb);
            float xv[kNR];
#pragma unroll
            for (int r = 0; r < kNR; ++r) xv[r] = xpre[r];
            {  // prefetch the following block
                int nsb = sb + XB, ntile = tile;
                if (nsb >= ig) {
                    nsb = 0;
                    ntile = tile + ncl;
                }
                load_block_x(ntile, nsb, xpre);
            }
            uint32_t woff[kNR];
            float ww[kNR];
#pragma unroll
            for (int r = 0; r < kNR; ++r) {
                int lo;
                float wa, wc;
                gather_weights<DT>(xv[r], p.cfg, lo, wa, wc);
                woff[r] = (uint32_t)(lo + pv) * row_stride;
                ww[r] = pv ? wc : wa;
            }
#pragma unroll
            for (int q = 0; q < XB; ++q) {
                if (q >= nq) break;
                const uint32_t slice = table_s + (uint32_t)((sb + q) * p.slice_bytes);
#pragma unroll
                for (int sl = 0; sl < kSlots; ++sl) {
                    const int st = q * kSlots + sl;
                    const int r = st / kSpr;  // compile-time after unrolling
                    const int jb = (st - r * kSpr) * M::P + tl[0];
#pragma unroll
                    for (int u = 0; u < M::U; ++u) {
                        const int src = 2 * jb + (hs[u] ? 1 : 0);
                        const uint32_t off = __shfl_sync(0xffffffffu, woff[r], src);
                        const float w = __shfl_sync(0xffffffffu, ww[r], src);
                        if (!act[u]) continue;
                        const float4 v = lds_v4(slice + off + coff[u]);
                        acc[sl][u].x = fmaf(w, v.x, acc[sl][u].x);
                        acc[sl][u].y = fmaf(w, v.y, acc[sl][u].y);
                        acc[sl][u].z = fmaf(w, v.z, acc[sl][u].z);
                        acc[sl][u].w = fmaf(w, v.w, acc[sl][u].w);
                    }
                }
            }
        }
        // fold the hi-row partial of each output chunk into the lane of its lo-row chunk
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
#pragma unroll
            for (int u = 0; u < M::U; ++u) {
                int src_lane = 0, src_u = 0;
                const bool dst = act[u] && ch[u] < C;
                if (dst) M::where(tl[u], ch[u] + C, src_lane, src_u);
                float4 got = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int v = 0; v < M::U; ++v) {
                    float4 s4;
                    s4.x = __shfl_sync(0xffffffffu, acc[sl][v].x, src_lane);
                    s4.y = __shfl_sync(0xffffffffu, acc[sl][v].y, src_lane);
                    s4.z = __shfl_sync(0xffffffffu, acc[sl][v].z, src_lane);
                    s4.w = __shfl_sync(0xffffffffu, acc[sl][v].w, src_lane);
                    if (v == src_u) got = s4;
                }
                if (dst) {
                    acc[sl][u].x += got.x;
                    acc[sl][u].y += got.y;
                    acc[sl][u].z += got.z;
                    acc[sl][u].w += got.w;
                }
            }
        }
        if constexpr (CS == 1) {
#pragma unroll
            for (int sl = 0; sl < kSlots; ++sl) {
                const int n = tile * TT + tok[sl];
#pragma unroll
                for (int u = 0; u < M::U; ++u) {
                    const int jc = ch[u];
                    if (act[u] && jc < C && n < p.N) {
                        const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + j0) + jc);
                        float4 o = acc[sl][u];
                        o.x += b.x;
                        o.y += b.y;
                        o.z += b.z;
                        o.w += b.w;
                        *reinterpret_cast<float4*>(p.out + (int64_t)n * p.OUT + j0 + 4 * jc) = o;
                    }
                }
            }
        } else {
            // 1) send this CTA's partials of every token to the token's owner
            if (k > 0) mbar_wait_cluster_bounded(bar_empty, (uint32_t)((k - 1) & 1));
#pragma unroll
            for (int sl = 0; sl < kSlots; ++sl) {
#pragma unroll
                for (int u = 0; u < M::U; ++u) {
                    if (act[u] && ch[u] < C) {
                        const int t = tok[sl];
                        const int owner = t / TTQ, tq = t - owner * TTQ;
                        const uint32_t dst = recv_s + (uint32_t)(((rank * TTQ + tq) * C + ch[u]) * 16);
                        st_async_v4(map_to_rank(dst, owner), acc[sl][u], map_to_rank(bar_full, owner));
                    }
                }
            }
            // 2) add up the CS partials of the tokens this CTA owns
            if (threadIdx.x == 0) mbar_arrive_expect_tx_local(bar_full, (uint32_t)(CS * TTQ * C * 16));
            const bool reducer = threadIdx.x < TTQ * C;
            if (reducer) mbar_wait_cluster_bounded(bar_full, (uint32_t)(k & 1));
            for (int e = threadIdx.x; e < TTQ * C; e += kFwdThreads) {
                const int tq = e / C, jc = e - tq * C;
                float4 s = lds_v4(recv_s + (uint32_t)((tq * C + jc) * 16));
#pragma unroll
                for (int r = 1; r < CS; ++r) {
                    const float4 v = lds_v4(recv_s + (uint32_t)(((r * TTQ + tq) * C + jc) * 16));
                    s.x += v.x;
                    s.y += v.y;
                    s.z += v.z;
                    s.w += v.w;
                }
                const int n = tile * TT + rank * TTQ + tq;
                if (n < p.N) {
                    const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + j0) + jc);
                    s.x += b.x;
                    s.y += b.y;
                    s.z += b.z;
                    s.w += b.w;
                    *reinterpret_cast<float4*>(p.out + (int64_t)n * p.OUT + j0 + 4 * jc) = s;
                }
            }
            // 3) the receive buffer may be refilled once every reader is done
            //    (named barrier 1 over the reducer warps only)
            constexpr int kRedRounded = ((TTQ * C + 31) / 32) * 32;
            constexpr int kRedThreads = kRedRounded < kFwdThreads ? kRedRounded : kFwdThreads;
            if (threadIdx.x < kRedThreads) {
                asm volatile("bar.sync 1, %0;" ::"n"(kRedThreads) : "memory");
                if (threadIdx.x < CS) mbar_arrive_remote(map_to_rank(bar_empty, (uint32_t)threadIdx.x));
            }
        }
    }
    if constexpr (CS > 1) cluster_sync();  // no CTA exits while cluster traffic targets it
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        cudaGetLastError();
    });
    return fn;
}

// 3-D map of table [K][IN][OUT] fp32 with box {JR, COLS, KB} (shared-memory
// layout of one box: [KB rows][COLS input columns][JR floats])
inline bool make_table_map(CUtensorMap* m, const float* table, int K, int IN, int OUT, int JR, int KB,
                           int COLS = 1) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)OUT, (cuuint64_t)IN, (cuuint64_t)K};
    const cuuint64_t strides[2] = {(cuuint64_t)OUT * 4, (cuuint64_t)IN * OUT * 4};
    const cuuint32_t box[3] = {(cuuint32_t)JR, (cuuint32_t)COLS, (cuuint32_t)KB};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(table), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kSmemBudget = 227 * 1024 - 1024;  // dynamic shared memory per CTA (static part aside)

struct FwdPlan {
    int C = 0, CS = 0, JR = 0, IG = 0, KB = 0, nbox = 0, slice_bytes = 0, smem = 0, RS = 0;
};

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

inline int round_up(int a, int b) { return ceil_div(a, b) * b; }

// the j-range widths (in float4 chunks) the forward is compiled for
constexpr int kFwdChunks[] = {20, 16, 10, 8, 5, 4, 2, 1};

inline int tokens_per_tile(int C) {
    const int R = 2 * C;
    return (R >= 32 ? 1 : 32 / R) * kWarps * kSlots;
}

// min_cs > 1 asks for clusters of at least min_cs CTAs (fewer input columns
// each), which spreads a small batch over more SMs
inline bool plan_forward(int K, int IN, int OUT, FwdPlan& pl, int min_cs = 1) {
    const int chunks = OUT / 4;
    for (int C : kFwdChunks) {
        if (chunks % C != 0) continue;  // j-ranges tile OUT exactly
        const int JR = 4 * C;
        const int nb = ceil_div(K, 256);
        const int m = 32 / std::gcd(JR, 32);  // keeps every box 128-byte aligned
        const int KB = round_up(ceil_div(K, nb), m);
        if (KB > 256) continue;
        // nb*KB rows from TMA (zero-filled past K) plus row K, rounded to 128 bytes
        const int slice = round_up(std::max(KB * nb, K + 1) * JR * 4, 128);
        for (int CS : {1, 2, 4, 8}) {
            if (CS < min_cs) continue;
            const int IG = ceil_div(IN, CS);
            if (CS > 1 && (IG - 1) * CS >= IN) continue;  // every rank gets at least one column
            const int TT = tokens_per_tile(C);
            const int xch = CS > 1 ? TT * C * 16 : 0;
            const int smem = IG * slice + xch + 128 + 32;  // + base alignment + mbarriers
            if (smem <= kSmemBudget) {
                pl = {C, CS, JR, IG, KB, nb, slice, smem};
                return true;
            }
        }
    }
    return false;
}

// argument conditions shared by the shape-specialised forwards
inline bool fast_forward_args_ok(const void* x, int x_dtype, const float* table, const float* bias,
                                 const float* out, int64_t N, int64_t IN, int64_t OUT, int64_t K,
                                 const BinCfg& c) {
    if (!c.pow2) return false;  // the gather's bucketing is written for bw = 2^-e
    if (OUT % 4 != 0 || N > (int64_t)1 << 30 || IN > 65535 || K > 65535) return false;
    if (N * IN > ((int64_t)1 << 40)) return false;
    if (((uintptr_t)table | (uintptr_t)bias | (uintptr_t)out) & 15) return false;
    if (x_dtype == kBF16 ? ((uintptr_t)x & 1) : ((uintptr_t)x & 3)) return false;
    return true;
}

inline bool fast_forward_ok(const void* x, int x_dtype, const float* table, const float* bias,
                            const float* out, int64_t N, int64_t IN, int64_t OUT, int64_t K,
                            const BinCfg& c) {
    if (!fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, K, c)) return false;
    FwdPlan pl;
    return plan_forward((int)K, (int)IN, (int)OUT, pl);
}

template <int DT, int C, int CS>
inline int launch_fwd(const CUtensorMap& map, const FwdArgs& a, const FwdPlan& pl, int num_sms,
                      cudaStream_t s) {
    auto kern = fwd_cluster_kernel<DT, C, CS>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess)
        return 4;
    if (CS > 1 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0) != cudaSuccess)
        return 4;
    const int jranges = ceil_div(a.OUT, pl.JR);
    int clusters = max(1, (num_sms / CS) / jranges);
    cudaLaunchConfig_t cfg = {};
    if (CS > 1) {
        // only as many clusters as can be co-resident (clusters occupy whole GPCs' SMs)
        static int cached[9] = {0};
        if (!cached[CS]) {
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3((unsigned)(CS * clusters), 1, 1);
            q.blockDim = dim3(kFwdThreads, 1, 1);
            q.dynamicSmemBytes = (size_t)pl.smem;
            cudaLaunchAttribute qa[1];
            qa[0].id = cudaLaunchAttributeClusterDimension;
            qa[0].val.clusterDim.x = CS;
            qa[0].val.clusterDim.y = 1;
            qa[0].val.clusterDim.z = 1;
            q.attrs = qa;
            q.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n < 1) {
                cudaGetLastError();
                n = num_sms / CS;
            }
            cached[CS] = n;
        }
        clusters = max(1, std::min(clusters, cached[CS] / jranges));
    }
    clusters = min(clusters, a.ntiles);
    cfg.gridDim = dim3((unsigned)(clusters * CS), (unsigned)jranges, 1);
    cfg.blockDim = dim3(kFwdThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)pl.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, map, a) == cudaSuccess ? 0 : 4;
}

template <int DT, int C>
inline int launch_fwd_cs(const CUtensorMap& map, const FwdArgs& a, const FwdPlan& pl, int sms,
                         cudaStream_t s) {
    switch (pl.CS) {
        case 1: return launch_fwd<DT, C, 1>(map, a, pl, sms, s);
        case 2: return launch_fwd<DT, C, 2>(map, a, pl, sms, s);
        case 4: return launch_fwd<DT, C, 4>(map, a, pl, sms, s);
        default: return launch_fwd<DT, C, 8>(map, a, pl, sms, s);
    }
}

template <int DT>
inline int launch_fwd_c(const CUtensorMap& map, const FwdArgs& a, const FwdPlan& pl, int sms,
                        cudaStream_t s) {
    switch (pl.C) {
        case 20: return launch_fwd_cs<DT, 20>(map, a, pl, sms, s);
        case 16: return launch_fwd_cs<DT, 16>(map, a, pl, sms, s);
        case 10: return launch_fwd_cs<DT, 10>(map, a, pl, sms, s);
        case 8: return launch_fwd_cs<DT, 8>(map, a, pl, sms, s);
        case 5: return launch_fwd_cs<DT, 5>(map, a, pl, sms, s);
        case 4: return launch_fwd_cs<DT, 4>(map, a, pl, sms, s);
        case 2: return launch_fwd_cs<DT, 2>(map, a, pl, sms, s);
        default: return launch_fwd_cs<DT, 1>(map, a, pl, sms, s);
    }
}

// returns kNotApplicable when the shape has no plan or the tensor map cannot
// be encoded (the caller then uses the general kernel)
constexpr int kNotApplicable = -1;

inline int fast_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out,
                        int64_t N, int64_t IN, int64_t OUT, const BinCfg& c, int num_sms,
                        cudaStream_t s) {
    FwdPlan pl;
    if (!plan_forward(c.K, (int)IN, (int)OUT, pl)) return kNotApplicable;
    {
        // too few token tiles to keep half the SMs busy: larger clusters, fewer
        // columns per CTA (64x64, K=16 at 2 K tokens: 14.2 us with pairs, 9.4
        // with clusters of 4, 11.1 with 8, whose 32 tiles take two rounds)
        const int64_t tiles = ceil_div((int)N, tokens_per_tile(pl.C));
        const int64_t jr = ceil_div((int)OUT, pl.JR);
        int cs = pl.CS;
        while (cs < 8 && 2 * tiles * jr * cs < num_sms) cs *= 2;
        FwdPlan wide;
        if (cs > pl.CS && plan_forward(c.K, (int)IN, (int)OUT, wide, cs) && wide.C == pl.C) pl = wide;
    }
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, pl.JR, pl.KB)) return kNotApplicable;
    FwdArgs a;
    a.x = x;
    a.bias = bias;
    a.out = out;
    a.N = (int)N;
    a.IN = (int)IN;
    a.OUT = (int)OUT;
    a.K = c.K;
    a.JR = pl.JR;
    a.RS = pl.JR;
    a.xvec = 0;
    a.IG = pl.IG;
    a.KB = pl.KB;
    a.nbox = pl.nbox;
    a.slice_bytes = pl.slice_bytes;
    a.ntiles = ceil_div((int)N, tokens_per_tile(pl.C));
    a.cfg = c;
    return x_dtype == kBF16 ? launch_fwd_c<kBF16>(map, a, pl, num_sms, s)
                            : launch_fwd_c<kF32>(map, a, pl, num_sms, s);
}

// ---------------------------------------------------------------------------
// backward kernel: dx, dtable and dbias in one pass over (go, x)
// ---------------------------------------------------------------------------
//
// CTA = (token range, group of IG input columns).  The group's table slices
// T[:, i, :] (full rows) are resident in shared memory.  A token is handled
// by a group of G = next_pow2(C) lanes; lane jc owns output chunk jc (4
// floats of go) and reads chunk jc of both rows lo and lo+1, so that
//   dx[n,i] = sum_jc [ (1-fr-s) * <go_jc, T[lo]_jc> + (fr+s) * <go_jc, T[lo+1]_jc> ]
//             (s = x/bw where the clamp on fr passes the gradient, else 0)
// is a sum over the group's lanes, done for 8 columns at a time with a
// transposed butterfly (7 shuffles for 8 sums in an 8-lane group).
//   dtable: red.global.add.v4 of x*(1-fr)*go_jc into gt[lo, i, jc] and of
//           x*fr*go_jc into gt[lo+1, i, jc] (gt zeroed beforehand).
//   dbias:  CTAs of the first column group add up go over their tokens.
// exact bins for bw = 2^-e (see gather_weights): lo, clamped fr and the
// unclamped fr that decides whether the clamp passes the gradient
template <int DT>
__device__ __forceinline__ void bwd_bin(float xv, const BinCfg& c, int& lo, float& fr, float& frp) {
    float q;
    if constexpr (DT == kBF16) {
        q = bf16_round(__fmul_rn(bf16_round(__fadd_rn(xv, 1.0f)), c.inv));
    } else {
        q = __fmaf_rn(xv, c.inv, c.inv);
    }
    float t = fminf(fmaxf(truncf(q), 0.0f), (float)(c.K - 1));
    if (!(fabsf(q) < 9.2233720368547758e18f)) t = 0.0f;
    frp = __fmul_rn(__fsub_rn(xv, __fmaf_rn(t, c.bw, -1.0f)), c.inv);
    const float f = fminf(fmaxf(frp, 0.0f), 1.0f);
    fr = (frp != frp) ? frp : f;
    lo = (int)t;
}

template <int C>
struct PairMap {
    static constexpr int G = C >= 32 ? 32 : (C > 16 ? 32 : (C > 8 ? 16 : (C > 4 ? 8 : (C > 2 ? 4 : (C > 1 ? 2 : 1)))));
    static constexpr int P = 32 / G;                 // tokens per warp
    static constexpr int U = (C + 31) / 32;          // chunks per lane
};

struct BwdArgs {
    const float* go;
    const void* x;
    void* gx;
    float* gt;
    float* gb;
    int N, IN, OUT, K;
    int IG;           // input columns per CTA
    int KB, nbox;     // TMA boxes per slice
    int slice_bytes;
    int ntiles;
    int want_gx, want_gt, want_gb;
    BinCfg cfg;
};

constexpr int kBwdThreads = 1024;
constexpr int kBwdV = 8;  // columns reduced per butterfly

// transposed butterfly over the G lanes of a group: on return lane holds the
// group sums of values [idx, idx + cnt) in v[0..cnt)
template <int G>
__device__ __forceinline__ void group_reduce8(float (&v)[kBwdV], int lane, int& idx, int& cnt,
                                              bool& writer) {
    idx = 0;
    cnt = kBwdV;
    writer = true;
#pragma unroll
    for (int h = G / 2; h >= 1; h >>= 1) {
        const bool bit = (lane & h) != 0;
        if (cnt >= 2) {
            const int half = cnt / 2;
#pragma unroll
            for (int k = 0; k < kBwdV / 2; ++k) {
                if (k < half) {
                    const float send = bit ? v[k] : v[half + k];
                    const float keep = bit ? v[half + k] : v[k];
                    v[k] = keep + __shfl_xor_sync(0xffffffffu, send, h);
                }
            }
            if (bit) idx += half;
            cnt = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], h);
            if (bit) writer = false;
        }
    }
}

template <int DT, int C>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_fused_kernel(const __grid_constant__ CUtensorMap tmap, const BwdArgs p) {
    using M = PairMap<C>;
    constexpr int G = M::G, P = M::P, U = M::U;
    constexpr int TT = P * (kBwdThreads / 32);
    extern __shared__ unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = blockIdx.y;  // column group
    const int i0 = g * p.IG;
    const int ig = max(0, min(p.IG, p.IN - i0));
    const int OUT = p.OUT;
    const uint32_t table_s = (smem_addr(smem) + 127u) & ~127u;
    const uint32_t bar_s = table_s + (uint32_t)(p.IG * p.slice_bytes);
    float* red_s = reinterpret_cast<float*>(smem + (bar_s + 16 - smem_addr(smem)));  // dbias partials

    if (threadIdx.x == 0) {
        prefetch_tensormap(&tmap);
        mbar_init(bar_s, 1);
        fence_mbar_init();
        if (ig > 0 && (p.want_gx || p.want_gt)) {
            mbar_arrive_expect_tx(bar_s, (uint32_t)(ig * p.nbox * p.KB * OUT * 4));
            for (int s = 0; s < ig; ++s)
                for (int b = 0; b < p.nbox; ++b)
                    tma_load_3d(table_s + s * p.slice_bytes + b * p.KB * OUT * 4, &tmap, bar_s, 0,
                                i0 + s, b * p.KB);
        }
    }
    __syncthreads();
    if (ig > 0 && (p.want_gx || p.want_gt)) {
        mbar_wait_bounded(bar_s, 0);
        // row K of every slice = row K-1 (the reference's hi for the top bin)
        for (int e = threadIdx.x; e < ig * C; e += kBwdThreads) {
            const int s = e / C, c4 = e - s * C;
            const uint32_t sl = table_s + (uint32_t)(s * p.slice_bytes);
            sts_v4(sl + (uint32_t)(p.K * OUT * 4 + c4 * 16), lds_v4(sl + (uint32_t)((p.K - 1) * OUT * 4 + c4 * 16)));
        }
        __syncthreads();
    }

    const int tg = lane / G, gl = lane % G;  // token in warp, lane in group
    const int row_stride = OUT * 4;
    const bool do_gb = p.want_gb && g == 0;
    float4 bsum[U];
#pragma unroll
    for (int u = 0; u < U; ++u) bsum[u] = make_float4(0.f, 0.f, 0.f, 0.f);

    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
        const int n = tile * TT + warp * P + tg;
        const bool tok = n < p.N;
        float4 gv[U];
        bool cact[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int jc = gl + G * u;
            cact[u] = tok && jc < C;
            gv[u] = cact[u] ? __ldg(reinterpret_cast<const float4*>(p.go + (int64_t)n * OUT) + jc)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
            if (do_gb) {
                bsum[u].x += gv[u].x;
                bsum[u].y += gv[u].y;
                bsum[u].z += gv[u].z;
                bsum[u].w += gv[u].w;
            }
        }
        if (!(p.want_gx || p.want_gt)) continue;
        const int64_t xrow = (int64_t)(tok ? n : 0) * p.IN + i0;
        for (int sb = 0; sb < ig; sb += kBwdV) {
            // weights of the warp's (token, column) pairs, one lane per pair:
            // pair j = s*P + token (s < kBwdV), held by lane j % 32 in register j / 32
            constexpr int kNR = (kBwdV * P + 31) / 32;
            uint32_t woff[kNR];
            float w0[kNR], w1[kNR], wa_[kNR], wc_[kNR];
#pragma unroll
            for (int r = 0; r < kNR; ++r) {
                const int j = r * 32 + lane;
                const int s = j / P, tt = j - s * P;
                const int nn = tile * TT + warp * P + tt;
                const bool ok = s < kBwdV && sb + s < ig && nn < p.N;
                const float xv = ok ? load_x<DT>(p.x, (int64_t)nn * p.IN + i0 + sb + s) : 0.0f;
                int lo;
                float fr, frp;
                bwd_bin<DT>(xv, p.cfg, lo, fr, frp);
                const float omf = __fsub_rn(1.0f, fr);
                const float sl = clamp_passes(frp) ? __fmul_rn(xv, p.cfg.inv) : 0.0f;
                woff[r] = (uint32_t)lo * row_stride;
                w0[r] = omf - sl;
                w1[r] = fr + sl;
                wa_[r] = omf == 0.0f ? 0.0f : __fmul_rn(xv, omf);
                wc_[r] = fr == 0.0f ? 0.0f : __fmul_rn(xv, fr);
            }
            float part[kBwdV];
#pragma unroll
            for (int k = 0; k < kBwdV; ++k) {
                part[k] = 0.f;
                const int j = k * P + tg;
                const int r = (k * P) / 32;  // all P pairs of step k share one register
                const uint32_t off = __shfl_sync(0xffffffffu, woff[r], j & 31);
                const float a0 = __shfl_sync(0xffffffffu, w0[r], j & 31);
                const float a1 = __shfl_sync(0xffffffffu, w1[r], j & 31);
                float wa = 0.f, wc = 0.f;
                if (p.want_gt) {
                    wa = __shfl_sync(0xffffffffu, wa_[r], j & 31);
                    wc = __shfl_sync(0xffffffffu, wc_[r], j & 31);
                }
                if (!tok || sb + k >= ig) continue;
                const uint32_t base = table_s + (uint32_t)((sb + k) * p.slice_bytes) + off;
                const int i = i0 + sb + k;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (!cact[u]) continue;
                    const int jc = gl + G * u;
                    if (p.want_gx) {
                        const float4 tl = lds_v4(base + jc * 16);
                        const float4 th = lds_v4(base + row_stride + jc * 16);
                        const float dl = gv[u].x * tl.x + gv[u].y * tl.y + gv[u].z * tl.z + gv[u].w * tl.w;
                        const float dh = gv[u].x * th.x + gv[u].y * th.y + gv[u].z * th.z + gv[u].w * th.w;
                        part[k] += a0 * dl + a1 * dh;
                    }
                    if (p.want_gt) {
                        const int lo = (int)(off / row_stride);
                        const int hi = min(lo + 1, p.K - 1);
                        float* rl = p.gt + ((int64_t)lo * p.IN + i) * OUT + 4 * jc;
                        float* rh = p.gt + ((int64_t)hi * p.IN + i) * OUT + 4 * jc;
                        red_global_add_v4(rl, make_float4(wa * gv[u].x, wa * gv[u].y, wa * gv[u].z, wa * gv[u].w));
                        red_global_add_v4(rh, make_float4(wc * gv[u].x, wc * gv[u].y, wc * gv[u].z, wc * gv[u].w));
                    }
                }
            }
            if (p.want_gx) {
                int idx, cnt;
                bool writer;
                group_reduce8<G>(part, lane, idx, cnt, writer);
                if (writer && tok) {
#pragma unroll
                    for (int k = 0; k < kBwdV; ++k) {
                        const int s = sb + idx + k;
                        if (k < cnt && s < ig) store_gx<DT>(p.gx, xrow + s, part[k]);
                    }
                }
            }
        }
    }
    if (do_gb) {
        // add over the P tokens of the warp, then over warps, then one red per column chunk
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int h = G; h < 32; h <<= 1) {
                bsum[u].x += __shfl_xor_sync(0xffffffffu, bsum[u].x, h);
                bsum[u].y += __shfl_xor_sync(0xffffffffu, bsum[u].y, h);
                bsum[u].z += __shfl_xor_sync(0xffffffffu, bsum[u].z, h);
                bsum[u].w += __shfl_xor_sync(0xffffffffu, bsum[u].w, h);
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < OUT; e += kBwdThreads) red_s[e] = 0.f;
        __syncthreads();
        if (tg == 0) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int jc = gl + G * u;
                if (jc < C) {
                    atomicAdd(red_s + 4 * jc + 0, bsum[u].x);
                    atomicAdd(red_s + 4 * jc + 1, bsum[u].y);
                    atomicAdd(red_s + 4 * jc + 2, bsum[u].z);
                    atomicAdd(red_s + 4 * jc + 3, bsum[u].w);
                }
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < OUT; e += kBwdThreads) atomicAdd(p.gb + e, red_s[e]);
    }
}

struct BwdPlan {
    int C = 0, IG = 0, ngroups = 0, KB = 0, nbox = 0, slice_bytes = 0, smem = 0;
};

constexpr int kBwdChunks[] = {20, 16, 10, 8, 5, 4, 2, 1};

inline bool plan_backward(int K, int IN, int OUT, BwdPlan& pl) {
    if (OUT % 4 != 0) return false;
    const int C = OUT / 4;
    bool inst = false;
    for (int c : kBwdChunks) inst |= (c == C);
    if (!inst) return false;
    const int nb = ceil_div(K, 256);
    const int m = 32 / std::gcd(OUT, 32);
    const int KB = round_up(ceil_div(K, nb), m);
    if (KB > 256) return false;
    const int slice = round_up(std::max(KB * nb, K + 1) * OUT * 4, 128);  // + row K
    const int fixed = 128 + 16 + OUT * 4 + 16;
    int IG = (kSmemBudget - fixed) / slice;
    if (IG < 1) return false;
    IG = std::min(IG, IN);
    const int ngroups = ceil_div(IN, IG);
    IG = ceil_div(IN, ngroups);
    pl = {C, IG, ngroups, KB, nb, slice, IG * slice + fixed};
    return true;
}

inline int64_t fast_backward_workspace(int64_t, int64_t, int64_t, int64_t, int) { return 0; }

inline bool fast_backward_ok(const float* go, const void* x, int x_dtype, const float* table,
                             const void* gx, const float* gt, const float* gb, int64_t N, int64_t IN,
                             int64_t OUT, int64_t K, const BinCfg& c) {
    if (!c.pow2) return false;  // the gathers' bucketing is written for bw = 2^-e
    if (N > ((int64_t)1 << 30) || IN > 65535 || K > 65535) return false;
    if (((uintptr_t)go | (uintptr_t)table | (uintptr_t)gt | (uintptr_t)gb) & 15) return false;
    if (x_dtype == kBF16 ? (((uintptr_t)x | (uintptr_t)gx) & 1) : (((uintptr_t)x | (uintptr_t)gx) & 3))
        return false;
    BwdPlan pl;
    return plan_backward((int)K, (int)IN, (int)OUT, pl);
}

template <int DT, int C>
inline int launch_bwd(const CUtensorMap& map, const BwdArgs& a, const BwdPlan& pl, int sms,
                      cudaStream_t s) {
    auto kern = bwd_fused_kernel<DT, C>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess)
        return 4;
    const int per = std::max(1, sms / pl.ngroups);
    dim3 grid((unsigned)std::min(per, a.ntiles), (unsigned)pl.ngroups, 1);
    kern<<<grid, kBwdThreads, pl.smem, s>>>(map, a);
    return 0;
}

template <int DT>
inline int launch_bwd_c(const CUtensorMap& map, const BwdArgs& a, const BwdPlan& pl, int sms,
                        cudaStream_t s) {
    switch (pl.C) {
        case 20: return launch_bwd<DT, 20>(map, a, pl, sms, s);
        case 16: return launch_bwd<DT, 16>(map, a, pl, sms, s);
        case 10: return launch_bwd<DT, 10>(map, a, pl, sms, s);
        case 8: return launch_bwd<DT, 8>(map, a, pl, sms, s);
        case 5: return launch_bwd<DT, 5>(map, a, pl, sms, s);
        case 4: return launch_bwd<DT, 4>(map, a, pl, sms, s);
        case 2: return launch_bwd<DT, 2>(map, a, pl, sms, s);
        default: return launch_bwd<DT, 1>(map, a, pl, sms, s);
    }
}

inline int bwd_tokens_per_tile(int C) {
    int G = 1;
    while (G < C && G < 32) G <<= 1;
    return (32 / G) * (kBwdThreads / 32);
}

struct DtPlan {
    int C = 0, TT = 0, R = 0, tok_per_cta = 0, smem = 0;
};

constexpr int kDtChunks[] = {20, 16, 10, 8, 5, 4, 2, 1};

inline bool plan_dtable(int N, int K, int IN, int OUT, int sms, DtPlan& pl) {
    if (OUT % 4 != 0 || OUT / 4 > 32 || K > 65535) return false;
    const int C = OUT / 4;
    bool inst = false;
    for (int c : kDtChunks) inst |= (c == C);
    if (!inst) return false;
    // bytes that do not scale with the tile: alignment, gt slice, bin counters,
    // scan scratch (+ padding)
    const int64_t fixed = 128 + (int64_t)K * OUT * 4 + (int64_t)(2 * K + 2) * 4 + 33 * 4 + 16;
    const int64_t per_tok = 2 * 16;  // per-token and sorted entries
    int64_t tt = (kSmemBudget - fixed) / per_tok;
    tt = std::min<int64_t>(tt, 4096) / 32 * 32;
    if (tt < 32) return false;
    int R = std::max(1, sms / IN);
    R = std::min(R, ceil_div(N, (int)tt));
    const int per = ceil_div(ceil_div(N, R), (int)tt) * (int)tt;
    R = ceil_div(N, per);
    pl = {C, (int)tt, R, per, (int)(fixed + per_tok * tt)};
    // sorting pays off only when a tile gives each row many contributions
    // (>= 64 per tile on average: K <= 64 at 4096 tokens).  Measured on B200:
    // at K=512 (4 per row per 1024 tokens) the vector reductions of the gather
    // kernel win (120 us vs 181 us for sort + separate dx), at K=128 they tie
    // or win, at K=16 the two are equal.
    return tt >= 64 * (int64_t)K;
}

template <int DT, int C>
inline int launch_dtable(const DtArgs& a, const DtPlan& pl, cudaStream_t s) {
    auto kern = dtable_kernel<DT, C>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem) != cudaSuccess)
        return 4;
    kern<<<dim3((unsigned)pl.R, (unsigned)a.IN, 1), kDtThreads, pl.smem, s>>>(a);
    return 0;
}

template <int DT>
inline int launch_dtable_c(const DtArgs& a, const DtPlan& pl, cudaStream_t s) {
    switch (pl.C) {
        case 20: return launch_dtable<DT, 20>(a, pl, s);
        case 16: return launch_dtable<DT, 16>(a, pl, s);
        case 10: return launch_dtable<DT, 10>(a, pl, s);
        case 8: return launch_dtable<DT, 8>(a, pl, s);
        case 5: return launch_dtable<DT, 5>(a, pl, s);
        case 4: return launch_dtable<DT, 4>(a, pl, s);
        case 2: return launch_dtable<DT, 2>(a, pl, s);
        default: return launch_dtable<DT, 1>(a, pl, s);
    }
}

// gt and gb must already be zero.  dx comes from the gather kernel, gt and gb
// from the sort-and-accumulate kernel when the shapes allow it; otherwise the
// gather kernel also scatters gt with vector reductions.
inline int fast_backward(const float* go, const void* x, int x_dtype, const float* table, void* gx,
                         float* gt, float* gb, int64_t N, int64_t IN, int64_t OUT, const BinCfg& c,
                         void*, int sms, cudaStream_t s, int* kernels) {
    *kernels = 0;
    BwdPlan pl;
    if (!plan_backward(c.K, (int)IN, (int)OUT, pl)) return kNotApplicable;
    DtPlan dp;
    const bool dt_ok = gt != nullptr && plan_dtable((int)N, c.K, (int)IN, (int)OUT, sms, dp);
    int rc = 0;
    if (gx || gb || (!dt_ok && gt)) {
        CUtensorMap map;
        if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, (int)OUT, pl.KB)) return kNotApplicable;
        BwdArgs a;
        a.go = go;
        a.x = x;
        a.gx = gx;
        a.gt = gt;
        a.gb = gb;
        a.N = (int)N;
        a.IN = (int)IN;
        a.OUT = (int)OUT;
        a.K = c.K;
        a.IG = pl.IG;
        a.KB = pl.KB;
        a.nbox = pl.nbox;
        a.slice_bytes = pl.slice_bytes;
        a.ntiles = ceil_div((int)N, bwd_tokens_per_tile(pl.C));
        a.want_gx = gx != nullptr;
        a.want_gt = !dt_ok && gt != nullptr;
        a.want_gb = gb != nullptr;
        a.cfg = c;
        rc = x_dtype == kBF16 ? launch_bwd_c<kBF16>(map, a, pl, sms, s) : launch_bwd_c<kF32>(map, a, pl, sms, s);
        if (rc) return rc;
        *kernels = 1;
        if (!dt_ok) return 0;
        if (cudaGetLastError() != cudaSuccess) return 4;
    }
    DtArgs d;
    d.go = go;
    d.x = x;
    d.gt = gt;
    d.gb = gb;
    d.N = (int)N;
    d.IN = (int)IN;
    d.OUT = (int)OUT;
    d.K = c.K;
    d.TT = dp.TT;
    d.tok_per_cta = dp.tok_per_cta;
    d.want_gb = 0;
    d.cfg = c;
    *kernels += 1;
    return x_dtype == kBF16 ? launch_dtable_c<kBF16>(d, dp, s) : launch_dtable_c<kF32>(d, dp, s);
}

}  // namespace il
