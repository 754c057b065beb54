// il_tc.cuh -- IndexedLinear forward as a dense matrix product on the 5th-
// generation tensor cores (tcgen05, accumulator in tensor memory).
//
// The forward of aiwn/layers/indexed_linear.py:173-182,
//   out[n,j] = sum_i x(1-fr) T[lo,i,j] + x fr T[hi,i,j] + b[j],
// is the product of the "hat basis" matrix A[n, (i,k)] (for every input i
// two non-zeros: x(1-fr) at k = lo and x fr at k = hi = min(lo+1, K-1)) with
// the table viewed as B[(i,k), j] = T[k,i,j]: a GEMM of M = tokens, N = out_d,
// reduction in_d*K, of which a fraction 2/K is non-zero.  Dense MMAs do K/2
// times the useful multiply-adds, so this form can only pay at small K.
//
// fp32 parity with kind::tf32 operands (10 explicit mantissa bits) uses the
// 3xTF32 split: a = a_hi + a_lo with a_hi = a truncated to tf32 and a_lo the
// exact fp32 remainder (the MMA truncates it in turn), likewise b, and
// D += a_hi b_hi + a_lo b_hi + a_hi b_lo in fp32 (the dropped a_lo b_lo and the
// truncations are ~2^-21 relative).
//
// One CTA of 9 warps per tile of 128 tokens.  Warps 0-7 build operands: two
// threads own token row m, each half of every chunk.  Warp 8 (one thread)
// issues the TMA loads of table rows and the MMAs.  The reduction runs in
// chunks of 32 (i,k) indices through S = 3 (or 2) shared-memory stages with
// full/empty mbarriers: the builders write chunk c -- A rows from the token's
// bins, B from table rows (both split into hi/lo) -- in the canonical K-major
// layout without swizzle (core matrices of 8 rows x 16 bytes, [16-byte K
// group][row][4 values]) and arrive on the stage's full barrier; the issuer
// multiplies it and commits to the stage's empty barrier, which the builders
// wait on before reusing the stage S chunks later.  The table rows of a chunk arrive by TMA into a ring
// of kTcRaw raw stages, issued that many chunks ahead, and the tile's x
// (in_d <= 64) is loaded into shared memory once, so building a chunk never
// waits on global memory.
// The accumulator (128 lanes x out_d fp32 columns) lives in tensor memory and
// is read back with tcgen05.ld, bias added, stored.  Tokens with a non-finite
// weight (x = +-inf or NaN) take the plain formula in the epilogue, since the
// hi/lo split of an infinity is not defined.  Every mbarrier wait is bounded;
// tensor memory is released on every path.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "il_common.cuh"
#include "il_fast.cuh"
#include "il_sm100.cuh"

namespace il {

constexpr int kTcThreads = 256;  // two threads per token row (128 rows = 128 TMEM lanes)
constexpr int kTcM = 128;        // MMA M
constexpr int kTcKC = 32;        // reduction indices per chunk (4 MMAs of K = 8)

struct TcArgs {
    const void* x;
    const float* table;
    const float* bias;
    float* out;
    int N, IN, OUT, K;
    int nchunk;      // IN*K / kTcKC
    int stage_bytes; // A hi, A lo, B hi, B lo of one chunk
    int stages;      // operand stages in flight (2 or 3)
    BinCfg cfg;
};

__device__ __forceinline__ float tf32_trunc(float v) { return __uint_as_float(__float_as_uint(v) & 0xffffe000u); }

// tcgen05 shared-memory matrix descriptor, K-major, no swizzle: start address,
// leading byte offset (next core matrix along K), stride byte offset (next
// 8-row group), descriptor version 1 (bits 46-47)
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr & 0x3ffffu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// instruction descriptor of kind::tf32: D fp32, A and B tf32, both K-major, M x N
__host__ __device__ constexpr uint32_t tc_idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_tf32(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 accumulator columns of this thread's TMEM lane
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int q = 0; q < 16; ++q) v[q] = __uint_as_float(r[q]);
}

// the two hat-basis weights of x for bins lo and hi = min(lo+1, K-1); a zero
// fraction gives an exact zero weight (no 0 * inf)
template <int DT>
__device__ __forceinline__ void tc_weights(float xv, const BinCfg& c, int& lo, float& wlo, float& whi) {
    int l;
    float fr, frp;
    bwd_bin<DT>(xv, c, l, fr, frp);
    const float omf = __fsub_rn(1.0f, fr);
    lo = l;
    wlo = omf == 0.0f ? 0.0f : __fmul_rn(xv, omf);
    whi = fr == 0.0f ? 0.0f : __fmul_rn(xv, fr);
}

constexpr int kTcRaw = 4;        // raw table-row stages in flight (TMA)
constexpr int kTcXPitch = kTcM + 1;  // floats per input column of the shared x tile
constexpr int kTcMaxIn = 64;     // in_d whose x tile the CTA keeps in shared memory
constexpr int kTcMaxStages = 3;  // operand stages (fewer when shared memory is short)

// thread 0: the raw table rows of chunk c -- T[k0 .. k0+31, i, :] for K >= 32,
// T[0..15, i, :] and T[0..15, i+1, :] for K = 16 -- into raw stage c % kTcRaw
__device__ __forceinline__ void tc_issue_raw(const CUtensorMap* map, const TcArgs& p, int c, uint32_t raw0,
                                             uint32_t rawbar0, uint32_t raw_bytes) {
    if (c >= p.nchunk) return;
    const int st = c % kTcRaw;
    const uint32_t dst = raw0 + (uint32_t)st * raw_bytes, bar = rawbar0 + 8u * (uint32_t)st;
    const int q0 = c * kTcKC;
    // (the builders' reads of this stage are ordered before by the mbarrier they arrived on)
    mbar_arrive_expect_tx(bar, raw_bytes);
    if (p.K >= kTcKC) {
        tma_load_3d(dst, map, bar, 0, q0 / p.K, q0 % p.K);
    } else {
        const uint32_t half_bytes = raw_bytes / 2;
        tma_load_3d(dst, map, bar, 0, q0 / p.K, 0);
        tma_load_3d(dst + half_bytes, map, bar, 0, q0 / p.K + 1, 0);
    }
}

// byte offset of A element (row m, index 16*half + kk of the chunk) in a stage
__device__ __forceinline__ uint32_t tc_a_off(int kk, int half, int m) {
    return (uint32_t)((4 * half + (kk >> 2)) * kTcM + m) * 16u + (uint32_t)(kk & 3) * 4u;
}

template <int DT>
__global__ void __launch_bounds__(kTcThreads + 32, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmap, const TcArgs p) {
    extern __shared__ unsigned char smem[];
    __shared__ uint64_t s_full[kTcMaxStages], s_empty[kTcMaxStages], s_raw[kTcRaw];
    __shared__ uint32_t s_tmem;
    __shared__ int s_bad[kTcM];
    const int tid = threadIdx.x, warp = tid >> 5;
    const bool builder = tid < kTcThreads;  // warps 0-7 build operands; warp 8 issues TMA and MMAs
    const int m = tid & (kTcM - 1), half = (tid / kTcM) & 1;  // token row, and which 16 of a chunk's 32 indices
    const int t0 = blockIdx.x * kTcM;
    const int n = t0 + m;
    const bool live = builder && n < p.N;
    const int K = p.K, IN = p.IN, OUT = p.OUT, S = p.stages;
    const uint32_t base = (smem_addr(smem) + 1023u) & ~1023u;
    // operand stage layout: A_hi [8][128][4] | A_lo | B_hi [8][OUT][4] | B_lo;
    // after the S operand stages, kTcRaw raw stages of [32 rows][OUT] fp32, then x
    const uint32_t a_bytes = kTcM * kTcKC * 4, b_bytes = (uint32_t)OUT * kTcKC * 4;
    const uint32_t raw0 = base + (uint32_t)S * (uint32_t)p.stage_bytes, raw_bytes = b_bytes;
    float* xs = reinterpret_cast<float*>(smem + (raw0 + (uint32_t)kTcRaw * raw_bytes - smem_addr(smem)));
    const uint32_t full0 = smem_addr(&s_full[0]), empty0 = smem_addr(&s_empty[0]), raw_bar0 = smem_addr(&s_raw[0]);
    const uint32_t tcols = OUT <= 32 ? 32 : (OUT <= 64 ? 64 : (OUT <= 128 ? 128 : 256));
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid < kTcM) s_bad[tid] = 0;
    if (tid == 0) {
        for (int b = 0; b < S; ++b) {
            mbar_init(full0 + 8u * b, kTcThreads);  // every builder arrives
            mbar_init(empty0 + 8u * b, 1);          // the commit of the stage's MMAs
        }
        for (int b = 0; b < kTcRaw; ++b) mbar_init(raw_bar0 + 8u * b, 1);
        fence_mbar_init();
    }
    if (builder) {
        // A_hi and A_lo of every stage start at zero
        for (int st = 0; st < S; ++st)
            for (uint32_t off = 16u * (uint32_t)tid; off < 2u * a_bytes; off += 16u * kTcThreads)
                sts_v4(base + (uint32_t)st * (uint32_t)p.stage_bytes + off, make_float4(0.f, 0.f, 0.f, 0.f));
        // the tile's x, transposed: xs[i][row] (coalesced global reads, a padded
        // pitch so that the transposing writes spread over the banks)
        for (int e = tid; e < kTcM * IN; e += kTcThreads) {
            const int row = e / IN, col = e - row * IN;
            xs[col * kTcXPitch + row] = t0 + row < p.N ? load_x<DT>(p.x, (int64_t)t0 * IN + e) : 0.0f;
        }
    }
    tc_fence_before();
    __syncthreads();  // barriers, tensor memory, zeros and x in place
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;
    if (!builder) {
        // ---- issuer: one thread of warp 8 ----
        if (tid == kTcThreads) {
            prefetch_tensormap(&tmap);
            for (int c = 0; c < kTcRaw; ++c) tc_issue_raw(&tmap, p, c, raw0, raw_bar0, raw_bytes);
            const uint32_t idesc = tc_idesc_tf32(kTcM, OUT);
            // descriptors of stage 0's operands; a stage or K step moves only the
            // start-address field (16-byte units, low bits of the descriptor)
            const uint64_t ah0 = tc_desc(base, kTcM * 16, 128), al0 = tc_desc(base + a_bytes, kTcM * 16, 128);
            const uint64_t bh0 = tc_desc(base + 2 * a_bytes, (uint32_t)OUT * 16, 128);
            const uint64_t bl0 = tc_desc(base + 2 * a_bytes + b_bytes, (uint32_t)OUT * 16, 128);
            const uint64_t astep = (2u * kTcM * 16) >> 4, bstep = (2u * (uint32_t)OUT * 16) >> 4;
            for (int c = 0; c < p.nchunk; ++c) {
                const int st = c % S;
                const uint64_t so = ((uint64_t)st * (uint64_t)p.stage_bytes) >> 4;
                ok &= mbar_wait_bounded(full0 + 8u * st, (uint32_t)((c / S) & 1));  // stage built
                tc_fence_after();
#pragma unroll
                for (int s = 0; s < kTcKC / 8; ++s) {
                    // K = 8 per MMA: two 16-byte K groups
                    const uint64_t ah = ah0 + so + s * astep, al = al0 + so + s * astep;
                    const uint64_t bh = bh0 + so + s * bstep, bl = bl0 + so + s * bstep;
                    tc_mma_tf32(tmem, ah, bh, idesc, (c > 0 || s > 0) ? 1u : 0u);
                    tc_mma_tf32(tmem, al, bh, idesc, 1u);
                    tc_mma_tf32(tmem, ah, bl, idesc, 1u);
                }
                tc_commit(empty0 + 8u * st);
                // the builders converted chunk c's raw rows before arriving: refill that raw stage
                tc_issue_raw(&tmap, p, c + kTcRaw, raw0, raw_bar0, raw_bytes);
            }
        }
    } else {
        // ---- builders: warps 0-7 ----
        bool bad = false;  // a non-finite weight: the epilogue recomputes this row
        int pa[kTcMaxStages], pb[kTcMaxStages];  // this thread's non-zero indices in each stage
#pragma unroll
        for (int st = 0; st < kTcMaxStages; ++st) pa[st] = pb[st] = -1;
        for (int c = 0; c < p.nchunk; ++c) {
            const int st = c % S;
            const uint32_t sa = base + (uint32_t)st * (uint32_t)p.stage_bytes;
            if (c >= S) ok &= mbar_wait_bounded(empty0 + 8u * st, (uint32_t)((c / S - 1) & 1));  // chunk c-S read it
            const int q0 = c * kTcKC;
            // A: row m, indices q0 + 16*half .. +15, all in one input column.
            // The stages were zeroed once; a chunk only clears the (at most
            // two) values this thread wrote into the stage S chunks ago and
            // writes its new ones, so the zeros of the hat basis cost nothing.
            int qa = -1, qb = -1;
#pragma unroll
            for (int t = 0; t < kTcMaxStages; ++t)
                if (t == st) {
                    qa = pa[t];
                    qb = pb[t];
                }
            if (qa >= 0) {
                sts_u32(sa + tc_a_off(qa, half, m), 0u);
                sts_u32(sa + a_bytes + tc_a_off(qa, half, m), 0u);
            }
            if (qb >= 0) {
                sts_u32(sa + tc_a_off(qb, half, m), 0u);
                sts_u32(sa + a_bytes + tc_a_off(qb, half, m), 0u);
            }
            int lo;
            float wl, wh;
            const float xv = xs[((q0 + 16 * half) / K) * kTcXPitch + m];
            tc_weights<DT>(xv, p.cfg, lo, wl, wh);
            bad |= !(isfinite(wl) && isfinite(wh));
            const int k0 = (q0 + 16 * half) % K;  // bin of the thread's first index
            const int dl = lo - k0;
            const bool top = lo == K - 1;          // hi = lo: one value, wl + wh
            const float vl = top ? wl + wh : wl;
            qa = (dl >= 0 && dl < 16) ? dl : -1;
            qb = (!top && dl + 1 >= 0 && dl + 1 < 16) ? dl + 1 : -1;
#pragma unroll
            for (int t = 0; t < kTcMaxStages; ++t)
                if (t == st) {
                    pa[t] = qa;
                    pb[t] = qb;
                }
            if (qa >= 0) {
                const float h = tf32_trunc(vl);
                sts_u32(sa + tc_a_off(qa, half, m), __float_as_uint(h));
                sts_u32(sa + a_bytes + tc_a_off(qa, half, m), __float_as_uint(vl - h));
            }
            if (qb >= 0) {
                const float h = tf32_trunc(wh);
                sts_u32(sa + tc_a_off(qb, half, m), __float_as_uint(h));
                sts_u32(sa + a_bytes + tc_a_off(qb, half, m), __float_as_uint(wh - h));
            }
            // B: [8 groups][OUT][4] from the raw rows [32][OUT] (row 4g+e, column j)
            const int rs = c % kTcRaw;
            ok &= mbar_wait_bounded(raw_bar0 + 8u * rs, (uint32_t)((c / kTcRaw) & 1));
            const uint32_t raw = raw0 + (uint32_t)rs * raw_bytes;
            for (int pidx = tid; pidx < 8 * OUT; pidx += kTcThreads) {
                const int g = pidx / OUT, j = pidx - g * OUT;
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    v[e] = __uint_as_float(lds_u32(raw + (uint32_t)((4 * g + e) * OUT + j) * 4u));
                const float4 h = make_float4(tf32_trunc(v[0]), tf32_trunc(v[1]), tf32_trunc(v[2]), tf32_trunc(v[3]));
                const float4 l = make_float4(v[0] - h.x, v[1] - h.y, v[2] - h.z, v[3] - h.w);
                const uint32_t off = (uint32_t)(g * OUT + j) * 16u;
                sts_v4(sa + 2 * a_bytes + off, h);
                sts_v4(sa + 2 * a_bytes + b_bytes + off, l);
            }
            fence_proxy_async_smem();  // this thread's operand writes, visible to the tensor core
            mbar_arrive(full0 + 8u * st);
        }
        // every chunk multiplied (a commit covers all earlier MMAs of the issuer)
        const int last = p.nchunk - 1;
        ok &= mbar_wait_bounded(empty0 + 8u * (last % S), (uint32_t)((last / S) & 1));
        tc_fence_after();
        // a row is bad when either of its two threads met a non-finite weight
        if (bad) s_bad[m] = 1;
        asm volatile("bar.sync 1, %0;" ::"r"(kTcThreads) : "memory");  // builders only
        bad = s_bad[m] != 0;
        // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its threads' rows);
        // the two halves take alternate blocks of 16 columns
        const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        for (int b = half; b < OUT / 16; b += 2) {
            const int j0 = 16 * b;
            float v[16];
            tc_ld16(trow + (uint32_t)j0, v);
            if (live && ok && !bad) {
                float* o = p.out + (int64_t)n * OUT + j0;
#pragma unroll
                for (int q = 0; q < 16; q += 4)
                    *reinterpret_cast<float4*>(o + q) = make_float4(v[q] + __ldg(p.bias + j0 + q),
                                                                    v[q + 1] + __ldg(p.bias + j0 + q + 1),
                                                                    v[q + 2] + __ldg(p.bias + j0 + q + 2),
                                                                    v[q + 3] + __ldg(p.bias + j0 + q + 3));
            }
        }
        if (live && ok && bad && half == 0) {
            // the plain formula, in the operation order of the general kernel
            for (int j = 0; j < OUT; ++j) {
                float acc = 0.0f;
                for (int i = 0; i < IN; ++i) {
                    const float xv = load_x<DT>(p.x, (int64_t)n * IN + i);
                    const Bin bb = bin_of<DT>(xv, p.cfg);
                    const int hi = min(bb.lo + 1, K - 1);
                    const float w = __fadd_rn(__fmul_rn(__ldg(p.table + ((int64_t)bb.lo * IN + i) * OUT + j),
                                                        __fsub_rn(1.0f, bb.fr)),
                                              __fmul_rn(__ldg(p.table + ((int64_t)hi * IN + i) * OUT + j), bb.fr));
                    acc = __fadd_rn(acc, __fmul_rn(w, xv));
                }
                p.out[(int64_t)n * OUT + j] = __fadd_rn(acc, __ldg(p.bias + j));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols) : "memory");
    }
}

// host side ---------------------------------------------------------------

// shapes the tensor-core forward takes: out_d a multiple of 16 up to 256 (MMA
// N), K a power of two >= 16 (at most two input columns per chunk), in_d*K a
// multiple of the chunk, in_d <= 64 (the x tile in shared memory)
inline bool tc_forward_ok(int64_t N, int64_t IN, int64_t OUT, int64_t K, const BinCfg& c) {
    if (!c.pow2 || K < 16 || (K & (K - 1)) || OUT % 16 || OUT < 16 || OUT > 256) return false;
    if ((IN * K) % kTcKC || N < 1 || N > ((int64_t)1 << 31) - kTcM || IN > kTcMaxIn) return false;
    return true;
}

inline int tc_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out, int64_t N,
                      int64_t IN, int64_t OUT, const BinCfg& c, cudaStream_t s) {
    if (!tc_forward_ok(N, IN, OUT, c.K, c)) return kNotApplicable;
    if (((uintptr_t)out | (uintptr_t)table) & 15) return kNotApplicable;
    TcArgs a;
    a.x = x;
    a.table = table;
    a.bias = bias;
    a.out = out;
    a.N = (int)N;
    a.IN = (int)IN;
    a.OUT = (int)OUT;
    a.K = c.K;
    a.nchunk = (int)(IN * c.K / kTcKC);
    a.stage_bytes = (int)(2 * kTcM * kTcKC * 4 + 2 * OUT * kTcKC * 4);
    a.cfg = c;
    // operand stages, the raw ring, the x tile, 1 KB alignment slack
    const int fixed = kTcRaw * (int)OUT * kTcKC * 4 + (int)IN * kTcXPitch * 4 + 1024;
    a.stages = kTcMaxStages;
    while (a.stages > 2 && a.stages * a.stage_bytes + fixed > kSmemBudget) --a.stages;
    const int smem = a.stages * a.stage_bytes + fixed;
    if (smem > kSmemBudget) return kNotApplicable;
    CUtensorMap map;
    if (!make_table_map(&map, table, c.K, (int)IN, (int)OUT, (int)OUT, std::min(c.K, kTcKC))) return kNotApplicable;
    auto kern = x_dtype == kBF16 ? fwd_tc_kernel<kBF16> : fwd_tc_kernel<kF32>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 4;
    const unsigned grid = (unsigned)((N + kTcM - 1) / kTcM);
    kern<<<grid, kTcThreads + 32, smem, s>>>(map, a);
    return 0;
}

}  // namespace il
