// il_allreduce.cuh -- in-place all-reduce (sum) of an fp32 buffer over the
// GPUs of one NVLink/NVSwitch node, by plain peer loads and stores.
//
// This is the exchange step of token-parallel training: every rank holds the
// gradient of the replicated table and bias ([dtable | dbias], the outputs of
// aiwn/layers/indexed_linear.py:131-151 for its own tokens) and all ranks need
// their sum.  The reference trains on one device and has no such step.
//
// Every rank's buffer and scratch region live in memory that all ranks have
// mapped (symmetric memory), so a kernel on one GPU can store into every
// peer's scratch and load from every peer's buffer over NVLink.  The buffer
// is cut into one chunk per rank; rank r reduces chunk r.  Two kernels:
//
// * allreduce_ll_kernel (buffers up to kArLLMaxElems): each 64-bit word a
//   rank stores into a peer's staging area carries one fp32 value and the
//   call's flag, and a 64-bit store arrives whole, so a word whose flag
//   matches holds this call's value: no fences and no barriers.  Every
//   thread owns pairs j of every chunk and
//     1. pushes pair j of chunk p of its buffer to rank p's stage1 (every p),
//     2. polls its stage1 for pair j of its own chunk from every rank, sums
//        in rank order (every rank ends with the same bits), stores the sum
//        into its buffer and pushes it to every rank's stage2,
//     3. polls its stage2 for pair j of every other chunk and stores it into
//        its buffer.
//   A call costs two NVLink one-way trips plus the stores (twice the data,
//   flags included).  Flags are the call's number (a counter in the scratch
//   region, advanced by the last block of each call), never reset; staging words
//   of one call cannot be overwritten by the next before they are read,
//   because no rank starts phase 1 of call k+1 before every rank's phase 2 of
//   call k reached it.
// * allreduce_kernel (larger buffers, bandwidth-bound): two shots with
//   per-block flag barriers: A (every rank's buffer complete), 1 (peer loads
//   sum chunk r, peer stores deliver it to every rank), B (every chunk has
//   arrived everywhere before the kernel ends).
//
// Each rank must make the same sequence of calls with the same sizes.  Waits
// are bounded by the global timer: past the limit the thread reports
// kErrAllreduceTimeout in the device error word and stops, so the host sees
// a status instead of a hung GPU.  No TMA, no bulk copies and no multicast
// touch peer memory: loads and stores are plain (L1-bypassing) accesses.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "il_common.cuh"

namespace il {

constexpr int kArThreads = 256;
constexpr int kArMaxBlocks = 1184;  // 8 per SM: enough loads in flight for NVLink on large buffers
constexpr int kArMaxRanks = 16;
constexpr unsigned int kErrAllreduceTimeout = 2u;

// words of a rank's flag region: [2 phases][kArMaxBlocks][kArMaxRanks] flags
// written by peers, then [kArMaxBlocks] generation counters of its own blocks
// (shared by both kernels: a block index's counter advances once per call)
constexpr int64_t kArFlagWords = 2 * kArMaxBlocks * kArMaxRanks + kArMaxBlocks + 2;
// the flag-in-word kernel's call counter and finished-block counter follow
constexpr int64_t kArCallWord = 2 * kArMaxBlocks * kArMaxRanks + kArMaxBlocks;
// buffers of at most this many elements take the flag-in-word kernel
constexpr int64_t kArLLMaxElems = (int64_t)1 << 21;

// pairs of fp32 values per rank's chunk in the flag-in-word kernel
inline int64_t ar_ll_pairs(int64_t n, int world) { return (n + 2 * world - 1) / (2 * world); }

// bytes of a rank's scratch region: the flag words, then (small buffers) the
// staging areas stage1 and stage2, each [world][pairs] of 16-byte words
inline int64_t ar_scratch_bytes(int64_t n, int world) {
    int64_t b = kArFlagWords * 4;
    b = (b + 255) / 256 * 256;
    if (n <= kArLLMaxElems) b += 2 * (int64_t)world * ar_ll_pairs(n, world) * 16;
    return b;
}
inline int64_t ar_stage_offset() { return (kArFlagWords * 4 + 255) / 256 * 256; }

struct ArLLArgs {
    float* buf;                      // this rank's buffer
    uint2* stage[kArMaxRanks];       // every rank's stage1 (stage2 follows at + world*pairs), as mapped here
    uint32_t* ctr;                   // this rank's [call counter, finished blocks]
    int64_t n, pairs;
    int rank, world;
    float scale;
    unsigned long long timeout_ns;
};

struct ArArgs {
    float* bufs[kArMaxRanks];      // every rank's buffer, as mapped on this GPU
    uint32_t* flags[kArMaxRanks];  // every rank's flag region, as mapped on this GPU
    int64_t n;               // fp32 elements of the buffer
    int64_t chunk4;          // float4 elements per rank's chunk
    int rank, world;
    float scale;             // result = scale * sum (1/world averages)
    unsigned long long timeout_ns;
};

__device__ __forceinline__ void st_relaxed_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Cross-rank barrier of block blockIdx.x in phase `ph` with value v.  Thread
// p < world signals rank p and waits for rank p's signal.  `publish`: this
// block stored into peer memory since the last barrier, so a release fence
// orders those stores (made block-wide by the bar.sync before it) ahead of
// the flag.  After the flag is seen, an acquire fence orders the block's
// later loads after the peer's stores.  Phase A publishes nothing: the
// buffer was written by earlier kernels on this GPU, complete in this GPU's
// L2, which is where peers' loads are served from.  Returns false (for the
// whole block) when a wait ran out.
__device__ __forceinline__ bool ar_barrier(const ArArgs& a, int ph, uint32_t v, bool publish) {
    __syncthreads();  // the block's earlier loads and stores come first
    int late = 0;
    if (threadIdx.x < a.world) {
        const int p = threadIdx.x;
        const int64_t slot = ((int64_t)ph * kArMaxBlocks + blockIdx.x) * kArMaxRanks;
        if (publish) fence_acq_rel_sys();
        st_relaxed_sys_u32(a.flags[p] + slot + a.rank, v);
        const uint32_t* mine = a.flags[a.rank] + slot + p;
        unsigned long long t0 = 0;
        for (uint32_t it = 0; (int32_t)(ld_relaxed_sys_u32(mine) - v) < 0; ++it) {
            // the timer is read once in a while; the first reads start the clock
            if ((it & 255u) == 0) {
                const unsigned long long t = global_timer_ns();
                if (t0 == 0) {
                    t0 = t;
                } else if (t - t0 > a.timeout_ns) {
                    late = 1;
                    report_error(kErrAllreduceTimeout);
                    break;
                }
            }
        }
        fence_acq_rel_sys();
    }
    return __syncthreads_or(late) == 0;
}

__device__ __forceinline__ float4 ld_cg_v4(const float* p) {
    return __ldcg(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ void st_cg_v4(float* p, float4 v) { __stcg(reinterpret_cast<float4*>(p), v); }

template <int W>
__device__ __forceinline__ void ar_chunk(const ArArgs& a, int64_t lo4, int64_t hi4) {
    const int world = W > 0 ? W : a.world;
    for (int64_t i = lo4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < hi4;
         i += (int64_t)gridDim.x * blockDim.x) {
        float4 v[W > 0 ? W : kArMaxRanks];
        // every peer's load in flight before the first add
#pragma unroll
        for (int p = 0; p < (W > 0 ? W : kArMaxRanks); ++p)
            if (W > 0 || p < world) v[p] = ld_cg_v4(a.bufs[p] + 4 * i);
        float4 s = v[0];
#pragma unroll
        for (int p = 1; p < (W > 0 ? W : kArMaxRanks); ++p) {
            if (W > 0 || p < world) {
                s.x += v[p].x;
                s.y += v[p].y;
                s.z += v[p].z;
                s.w += v[p].w;
            }
        }
        s.x *= a.scale;
        s.y *= a.scale;
        s.z *= a.scale;
        s.w *= a.scale;
#pragma unroll
        for (int p = 0; p < (W > 0 ? W : kArMaxRanks); ++p)
            if (W > 0 || p < world) st_cg_v4(a.bufs[p] + 4 * i, s);
    }
}

template <int W>
__global__ void __launch_bounds__(kArThreads) allreduce_kernel(const ArArgs a) {
    __shared__ uint32_t s_v;
    uint32_t* gen = a.flags[a.rank] + 2 * kArMaxBlocks * kArMaxRanks + blockIdx.x;
    if (threadIdx.x == 0) s_v = *gen + 1u;
    __syncthreads();
    const uint32_t v = s_v;
    if (!ar_barrier(a, 0, v, false)) return;
    const int64_t n4 = a.n / 4;
    const int64_t lo4 = (int64_t)a.rank * a.chunk4;
    const int64_t hi4 = lo4 + a.chunk4 < n4 ? lo4 + a.chunk4 : n4;
    if (lo4 < hi4) ar_chunk<W>(a, lo4, hi4);
    // the n % 4 tail elements: the last rank, block 0
    if (a.rank == a.world - 1 && blockIdx.x == 0 && threadIdx.x < (int)(a.n - 4 * n4)) {
        const int64_t e = 4 * n4 + threadIdx.x;
        float s = __ldcg(a.bufs[0] + e);
        for (int p = 1; p < a.world; ++p) s += __ldcg(a.bufs[p] + e);
        s *= a.scale;
        for (int p = 0; p < a.world; ++p) __stcg(a.bufs[p] + e, s);
    }
    if (!ar_barrier(a, 1, v, true)) return;
    if (threadIdx.x == 0) *gen = v;
}

__device__ __forceinline__ void st_relaxed_sys_v2u64(uint2* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void ld_relaxed_sys_v2u64(const uint2* p, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ unsigned long long ll_word(float d, uint32_t v) {
    return ((unsigned long long)v << 32) | (unsigned long long)__float_as_uint(d);
}

// Polls a 16-byte staging word until both halves carry flag v; false on timeout.
__device__ __forceinline__ bool ll_wait(const uint2* p, uint32_t v, unsigned long long timeout_ns, float& d0,
                                        float& d1) {
    unsigned long long a, b, t0 = 0;
    for (uint32_t it = 0;; ++it) {
        ld_relaxed_sys_v2u64(p, a, b);
        if ((uint32_t)(a >> 32) == v && (uint32_t)(b >> 32) == v) break;
        if ((it & 255u) == 0) {
            const unsigned long long t = global_timer_ns();
            if (t0 == 0) {
                t0 = t;
            } else if (t - t0 > timeout_ns) {
                report_error(kErrAllreduceTimeout);
                return false;
            }
        }
    }
    d0 = __uint_as_float((uint32_t)a);
    d1 = __uint_as_float((uint32_t)b);
    return true;
}

template <int W>
__global__ void __launch_bounds__(kArThreads) allreduce_ll_kernel(const ArLLArgs a) {
    constexpr int WM = W > 0 ? W : kArMaxRanks;
    const int world = W > 0 ? W : a.world;
    __shared__ uint32_t s_v;
    if (threadIdx.x == 0) s_v = a.ctr[0] + 1u;  // advanced only after every block of the last call
    __syncthreads();
    const uint32_t v = s_v;
    const int64_t P = a.pairs, n = a.n;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t j0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int me = a.rank;
    bool ok = true;
    // 1. pair j of chunk p goes to rank p's stage1, slot [me][j]
    for (int64_t j = j0; j < P; j += stride) {
#pragma unroll
        for (int p = 0; p < WM; ++p) {
            if ((W == 0 && p >= world) || p == me) continue;
            const int64_t e = 2 * (p * P + j);
            const float d0 = e < n ? __ldcg(a.buf + e) : 0.0f;
            const float d1 = e + 1 < n ? __ldcg(a.buf + e + 1) : 0.0f;
            st_relaxed_sys_v2u64(a.stage[p] + 2 * (me * P + j), ll_word(d0, v), ll_word(d1, v));
        }
    }
    // 2. this rank's chunk: every rank's pair j, summed in rank order
    for (int64_t j = j0; j < P && ok; j += stride) {
        const int64_t e = 2 * (me * P + j);
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int p = 0; p < WM; ++p) {
            if (W == 0 && p >= world) continue;
            float d0, d1;
            if (p == me) {
                d0 = e < n ? __ldcg(a.buf + e) : 0.0f;
                d1 = e + 1 < n ? __ldcg(a.buf + e + 1) : 0.0f;
            } else if (!ll_wait(a.stage[me] + 2 * (p * P + j), v, a.timeout_ns, d0, d1)) {
                ok = false;
                break;
            }
            s0 = p == 0 ? d0 : s0 + d0;
            s1 = p == 0 ? d1 : s1 + d1;
        }
        if (!ok) break;
        s0 *= a.scale;
        s1 *= a.scale;
        if (e < n) a.buf[e] = s0;
        if (e + 1 < n) a.buf[e + 1] = s1;
#pragma unroll
        for (int p = 0; p < WM; ++p) {
            if ((W == 0 && p >= world) || p == me) continue;
            st_relaxed_sys_v2u64(a.stage[p] + 2 * ((int64_t)world * P + me * P + j), ll_word(s0, v), ll_word(s1, v));
        }
    }
    // 3. every other rank's reduced chunk, from this rank's stage2
    for (int64_t j = j0; j < P && ok; j += stride) {
#pragma unroll
        for (int p = 0; p < WM; ++p) {
            if ((W == 0 && p >= world) || p == me) continue;
            float d0, d1;
            if (!ll_wait(a.stage[me] + 2 * ((int64_t)world * P + p * P + j), v, a.timeout_ns, d0, d1)) {
                ok = false;
                break;
            }
            const int64_t e = 2 * (p * P + j);
            if (e < n) a.buf[e] = d0;
            if (e + 1 < n) a.buf[e + 1] = d1;
        }
    }
    // the last block to finish advances the call counter (the next launch on
    // this stream starts after every block of this one has exited)
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.ctr + 1, 1u) == gridDim.x - 1) {
        a.ctr[1] = 0;
        a.ctr[0] = v;
    }
}

// Flag-in-word kernel with one warp per (group of 32 pairs, rank): a block of
// kArThreads threads holds 8 / W groups, warp w serves rank w % W of group
// w / W, so every push is a coalesced 512-byte store by one warp and a
// call of n elements runs n / 2 * W / 32 warps (8 ranks, 819 KB: 400 blocks
// against 51 for the thread-per-pair kernel).  Same staging layout, flags and
// call counter as allreduce_ll_kernel; the sum of pair j is taken in rank
// order by every warp of its group from shared memory (identical bits on
// every rank), then each warp pushes it to its rank.
template <int W>
__global__ void __launch_bounds__(kArThreads) allreduce_ll_warp_kernel(const ArLLArgs a) {
    static_assert(W == 2 || W == 4 || W == 8, "ranks per warp group");
    constexpr int kGroups = (kArThreads / 32) / W;
    __shared__ uint32_t s_v;
    __shared__ float2 sv[kGroups][W][32];
    if (threadIdx.x == 0) s_v = a.ctr[0] + 1u;  // advanced only after every block of the last call
    __syncthreads();
    const uint32_t v = s_v;
    const int64_t P = a.pairs, n = a.n;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = warp / W, p = warp % W;
    const int me = a.rank;
    bool ok = true;
    // every block makes the same number of passes, so its barriers line up
    const int64_t gstride = (int64_t)gridDim.x * kGroups * 32;
    const int64_t passes = (P + gstride - 1) / gstride;
    for (int64_t pass = 0; pass < passes; ++pass) {
        const int64_t j = pass * gstride + ((int64_t)blockIdx.x * kGroups + g) * 32 + lane;
        const bool have = j < P;
        // 1. pair j of chunk p of this rank's buffer to rank p's stage1, slot [me][j]
        if (p != me && have) {
            const int64_t e = 2 * (p * P + j);
            const float d0 = e < n ? __ldcg(a.buf + e) : 0.0f;
            const float d1 = e + 1 < n ? __ldcg(a.buf + e + 1) : 0.0f;
            st_relaxed_sys_v2u64(a.stage[p] + 2 * (me * P + j), ll_word(d0, v), ll_word(d1, v));
        }
        // 2. rank p's pair j of this rank's chunk, into shared memory
        const int64_t e = 2 * (me * P + j);
        float d0 = 0.0f, d1 = 0.0f;
        if (have) {
            if (p == me) {
                d0 = e < n ? __ldcg(a.buf + e) : 0.0f;
                d1 = e + 1 < n ? __ldcg(a.buf + e + 1) : 0.0f;
            } else if (ok && !ll_wait(a.stage[me] + 2 * (p * P + j), v, a.timeout_ns, d0, d1)) {
                ok = false;
            }
        }
        sv[g][p][lane] = make_float2(d0, d1);
        if (__syncthreads_or(!ok)) {
            ok = false;
            break;
        }
        float s0 = sv[g][0][lane].x, s1 = sv[g][0][lane].y;
#pragma unroll
        for (int q = 1; q < W; ++q) {
            s0 += sv[g][q][lane].x;
            s1 += sv[g][q][lane].y;
        }
        s0 *= a.scale;
        s1 *= a.scale;
        if (have) {
            if (p == me) {
                if (e < n) a.buf[e] = s0;
                if (e + 1 < n) a.buf[e + 1] = s1;
            } else {
                st_relaxed_sys_v2u64(a.stage[p] + 2 * ((int64_t)W * P + me * P + j), ll_word(s0, v), ll_word(s1, v));
            }
        }
        // 3. rank p's reduced pair j of chunk p, from this rank's stage2
        if (have && p != me) {
            float r0, r1;
            if (ll_wait(a.stage[me] + 2 * ((int64_t)W * P + p * P + j), v, a.timeout_ns, r0, r1)) {
                const int64_t ep = 2 * (p * P + j);
                if (ep < n) a.buf[ep] = r0;
                if (ep + 1 < n) a.buf[ep + 1] = r1;
            } else {
                ok = false;
            }
        }
        // sv is rewritten by the next pass
        if (__syncthreads_or(!ok)) break;
    }
    // the last block to finish advances the call counter
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.ctr + 1, 1u) == gridDim.x - 1) {
        a.ctr[1] = 0;
        a.ctr[0] = v;
    }
}

// ---- variant for callers that cannot allocate: scratch in a static array ----
//
// One process drives every rank's GPU and launches all ranks of a call.  The
// scratch is each device's own copy of a file-scope array, touched only by
// that device: a device's static data is not mapped into its peers, so every
// cross-device access goes to the callers' buffers (their allocations are,
// with peer access enabled).  Rank p sums every rank's buffer into its
// scratch (peer loads, ranks added in rank order, so every rank ends with
// the same bits); after every rank has done so -- the host orders the
// devices' streams with events, no device waits on another -- it copies the
// scratch into its buffer.
struct NaArgs {
    const float* bufs[kArMaxRanks];  // every rank's buffer (the callers' allocations)
    float* scratch;                  // this device's copy of the static array
    int64_t n;
    int world;
    float scale;
};

__global__ void __launch_bounds__(kArThreads) allreduce_noalloc_sum_kernel(const NaArgs a) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t n4 = a.n / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 s = __ldcg(reinterpret_cast<const float4*>(a.bufs[0]) + i);
        for (int q = 1; q < a.world; ++q) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(a.bufs[q]) + i);
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        s.x *= a.scale;
        s.y *= a.scale;
        s.z *= a.scale;
        s.w *= a.scale;
        reinterpret_cast<float4*>(a.scratch)[i] = s;
    }
    const int64_t e = 4 * n4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // the n % 4 tail
    if (e < a.n && blockIdx.x == 0) {
        float s = __ldcg(a.bufs[0] + e);
        for (int q = 1; q < a.world; ++q) s += __ldcg(a.bufs[q] + e);
        a.scratch[e] = s * a.scale;
    }
}

__global__ void __launch_bounds__(kArThreads) allreduce_noalloc_copy_kernel(float* buf, const float* scratch,
                                                                             int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t n4 = n / 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride)
        reinterpret_cast<float4*>(buf)[i] = reinterpret_cast<const float4*>(scratch)[i];
    const int64_t e = 4 * n4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < n && blockIdx.x == 0) buf[e] = scratch[e];
}

struct ArPlan {
    int blocks = 1;
    int64_t chunk4 = 0;
};

// One float4 per thread and pass; at most 4 blocks per SM, so that every block
// of the grid is resident at once (block b waits for block b of the peers).
inline ArPlan plan_allreduce(int64_t n, int world, int sms) {
    ArPlan pl;
    const int64_t n4 = n / 4;
    pl.chunk4 = (n4 + world - 1) / world;
    int64_t b = (pl.chunk4 + kArThreads - 1) / kArThreads;
    const int64_t cap = std::min<int64_t>(kArMaxBlocks, (int64_t)sms * 4);
    if (b < 1) b = 1;
    if (b > cap) b = cap;
    pl.blocks = (int)b;
    return pl;
}

// flag-in-word kernel: one pair per thread and pass, at most 4 blocks per SM
// (corresponding threads of all ranks must be resident together)
inline int ll_blocks(int64_t pairs, int sms) {
    int64_t b = (pairs + kArThreads - 1) / kArThreads;
    const int64_t cap = std::min<int64_t>(kArMaxBlocks, (int64_t)sms * 4);
    return (int)std::max<int64_t>(1, std::min(b, cap));
}

// the warp-per-rank kernel (2, 4 or 8 ranks): pairs * world / 256 blocks, same cap
inline bool ll_warp_ok(int world) { return world == 2 || world == 4 || world == 8; }
// the default: 4 and 8 ranks.  At 8 ranks inside the training step (C3, the
// 819 KB gradient after the backward) the exchange cost 14 us against 19.7
// with one thread per pair; at 2 ranks the thread kernel measured a little
// faster (7.9 against 8.2 us per call).
inline bool ll_warp_default(int world) { return world == 4 || world == 8; }
inline int ll_warp_blocks(int64_t pairs, int world, int sms) {
    int64_t b = (pairs * world + kArThreads - 1) / kArThreads;
    const int64_t cap = std::min<int64_t>(kArMaxBlocks, (int64_t)sms * 4);
    return (int)std::max<int64_t>(1, std::min(b, cap));
}

inline int launch_allreduce_ll_warp(const ArLLArgs& a, int blocks, cudaStream_t s) {
    const dim3 g((unsigned)blocks), t(kArThreads);
    switch (a.world) {
        case 2: allreduce_ll_warp_kernel<2><<<g, t, 0, s>>>(a); break;
        case 4: allreduce_ll_warp_kernel<4><<<g, t, 0, s>>>(a); break;
        default: allreduce_ll_warp_kernel<8><<<g, t, 0, s>>>(a); break;
    }
    return 0;
}

inline int launch_allreduce_ll(const ArLLArgs& a, int blocks, cudaStream_t s) {
    const dim3 g((unsigned)blocks), t(kArThreads);
    switch (a.world) {
        case 2: allreduce_ll_kernel<2><<<g, t, 0, s>>>(a); break;
        case 4: allreduce_ll_kernel<4><<<g, t, 0, s>>>(a); break;
        case 8: allreduce_ll_kernel<8><<<g, t, 0, s>>>(a); break;
        default: allreduce_ll_kernel<0><<<g, t, 0, s>>>(a); break;
    }
    return 0;
}

inline int launch_allreduce(const ArArgs& a, const ArPlan& pl, cudaStream_t s) {
    const dim3 g((unsigned)pl.blocks), t(kArThreads);
    switch (a.world) {
        case 2: allreduce_kernel<2><<<g, t, 0, s>>>(a); break;
        case 4: allreduce_kernel<4><<<g, t, 0, s>>>(a); break;
        case 8: allreduce_kernel<8><<<g, t, 0, s>>>(a); break;
        default: allreduce_kernel<0><<<g, t, 0, s>>>(a); break;
    }
    return 0;
}

}  // namespace il
