// il_attn.cuh -- causal self-attention for the narrow heads of IndexedGPT.
//
// IndexedGPT's blocks attend over d_idx / n_head = 4 features per head at the
// reference's config 5 (transformer_validation.py:254-269).  Library kernels
// for attention pad such heads to 32 or more features; here one CTA owns one
// (batch, head), a group of S lanes one query row, and K and V of the head sit in
// shared memory, with S = 1, 2 or 4 lanes sharing a query (or key):
//
//   forward:  o_i = sum_{j<=i} softmax_j(q_i.k_j * scale) * keep_ij / (1-p) * v_j
//             (online softmax over j), plus lse_i = log sum_j exp(s_ij)
//   backward: Dsum_i = dO_i . o_i;  P_ij = exp(s_ij - lse_i);
//             dS_ij = P_ij (keep_ij / (1-p) * dO_i.v_j - Dsum_i)
//             dq_i = scale * sum_{j<=i} dS_ij k_j           (thread per query)
//             dk_j = scale * sum_{i>=j} dS_ij q_i,
//             dv_j = sum_{i>=j} P_ij keep_ij / (1-p) dO_i   (thread per key)
//   so every backward lane group runs i+1 + T-i iterations.
//
// q, k, v, o, dq, dk, dv are [B, T, H*D] (the projections' own layout: no
// head transposes).  Dropout keeps element (b, h, i, j) when a 32-bit hash
// (MurmurHash3's finaliser) of the score row's key plus j reaches p * 2^32;
// the row key mixes the device-resident 64-bit seed with the row index, so
// the backward regenerates the same mask from the same seed.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace il {

constexpr int kAttnMaxT = 1024;
// the 16-feature backward keeps more state per thread: at most 512 positions
__host__ __device__ constexpr int attn_max_t(int D) { return D >= 16 ? 512 : kAttnMaxT; }

// MurmurHash3's 32-bit finaliser (Appleby, public domain)
__device__ __forceinline__ uint32_t fmix32(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85EBCA6Bu;
    h ^= h >> 13;
    h *= 0xC2B2AE35u;
    h ^= h >> 16;
    return h;
}

// the key of score row (b*H + h)*T + i under a 64-bit seed
__device__ __forceinline__ uint32_t attn_row_key(uint64_t seed, uint64_t row) {
    const uint32_t mixed = (uint32_t)(seed >> 32) + (uint32_t)row * 0x9E3779B9u + (uint32_t)(row >> 32);
    return fmix32((uint32_t)seed ^ fmix32(mixed));
}

// element (row, j) is kept when fmix32(row key + j * 0x85EBCA77) >= p * 2^32
__device__ __forceinline__ bool attn_keep(uint32_t row_key, int j, uint32_t thr) {
    return fmix32(row_key + (uint32_t)j * 0x85EBCA77u) >= thr;
}

template <int D>
__device__ __forceinline__ void attn_load_row(const float* s, float (&r)[D]) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int d = 0; d < D; d += 4) {
            const float4 t = *reinterpret_cast<const float4*>(s + d);
            r[d] = t.x, r[d + 1] = t.y, r[d + 2] = t.z, r[d + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int d = 0; d < D; ++d) r[d] = s[d];
    }
}

template <int D>
__device__ __forceinline__ float attn_dot(const float (&a)[D], const float (&b)[D]) {
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) s = fmaf(a[d], b[d], s);
    return s;
}

// S lanes share one query (forward, dq) or one key (dk, dv): lane r of a
// group takes every S-th key or query from r on, and the group's partial
// results are combined by shuffles.  Block = T*S threads.
// lanes of this thread's warp that exist (the last warp of a block of T*S
// threads may be partial; groups of S never straddle its end)
__device__ __forceinline__ unsigned warp_lanes() {
    const int n = min(32, (int)blockDim.x - ((int)threadIdx.x & ~31));
    return n == 32 ? 0xffffffffu : ((1u << n) - 1u);
}

template <int S>
__device__ __forceinline__ float group_sum(float v, unsigned lanes) {
#pragma unroll
    for (int o = 1; o < S; o <<= 1) v += __shfl_xor_sync(lanes, v, o);
    return v;
}

template <int S>
__device__ __forceinline__ float group_max(float v, unsigned lanes) {
#pragma unroll
    for (int o = 1; o < S; o <<= 1) v = fmaxf(v, __shfl_xor_sync(lanes, v, o));
    return v;
}

// grid (H, B), block T*S threads; dynamic shared memory 2*T*D floats
template <int D, int S>
__global__ void __launch_bounds__(kAttnMaxT)
    attn_fwd_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                    float* __restrict__ o, float* __restrict__ lse, int T, int H, float scale, uint32_t thr,
                    float inv_keep, const uint64_t* __restrict__ seedp) {
    extern __shared__ float sm[];
    float* ks = sm;
    float* vs = sm + T * D;
    const int h = blockIdx.x, b = blockIdx.y;
    const int i = (int)threadIdx.x / S, r = (int)threadIdx.x % S;
    const int HD = H * D;
    const int64_t base = (int64_t)b * T * HD + (int64_t)h * D;
    for (int e = threadIdx.x; e < T * D; e += blockDim.x) {
        const int t = e / D, d = e - t * D;
        ks[e] = k[base + (int64_t)t * HD + d];
        vs[e] = v[base + (int64_t)t * HD + d];
    }
    __syncthreads();
    const uint64_t seed = thr ? *seedp : 0ull;
    float qi[D], acc[D];
#pragma unroll
    for (int d = 0; d < D; ++d) {
        qi[d] = q[base + (int64_t)i * HD + d];
        acc[d] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const uint32_t rk = thr ? attn_row_key(seed, (uint64_t)(b * H + h) * (uint64_t)T + (uint64_t)i) : 0u;
    for (int j = r; j <= i; j += S) {
        float kj[D], vj[D];
        attn_load_row<D>(ks + j * D, kj);
        const float s = attn_dot<D>(qi, kj) * scale;
        if (s > m) {  // rescale the running sums to the new maximum
            const float c = expf(m - s);
            l *= c;
#pragma unroll
            for (int d = 0; d < D; ++d) acc[d] *= c;
            m = s;
        }
        const float e = expf(s - m);
        l += e;
        if (thr == 0u || attn_keep(rk, j, thr)) {
            attn_load_row<D>(vs + j * D, vj);
#pragma unroll
            for (int d = 0; d < D; ++d) acc[d] = fmaf(e, vj[d], acc[d]);
        }
    }
    // combine the group's running sums at the group's maximum (lane 0 always
    // saw key 0, so the maximum is finite; lanes without keys add zero)
    const unsigned lanes = warp_lanes();
    const float mg = group_max<S>(m, lanes);
    const float c = m == -INFINITY ? 0.f : expf(m - mg);
    l = group_sum<S>(l * c, lanes);
#pragma unroll
    for (int d = 0; d < D; ++d) acc[d] = group_sum<S>(acc[d] * c, lanes);
    if (r == 0) {
        const float rr = inv_keep / l;
#pragma unroll
        for (int d = 0; d < D; ++d) o[base + (int64_t)i * HD + d] = acc[d] * rr;
        lse[(int64_t)(b * H + h) * T + i] = mg + logf(l);
    }
}

// grid (H, B), block T*S threads; dynamic shared memory (4*T*D + 2*T) floats
template <int D, int S>
__global__ void __launch_bounds__(attn_max_t(D))
    attn_bwd_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                    const float* __restrict__ o, const float* __restrict__ dout, const float* __restrict__ lse,
                    float* __restrict__ dq, float* __restrict__ dk, float* __restrict__ dv, int T, int H,
                    float scale, uint32_t thr, float inv_keep, const uint64_t* __restrict__ seedp) {
    extern __shared__ float sm[];
    float* qs = sm;
    float* ks = qs + T * D;
    float* vs = ks + T * D;
    float* dos = vs + T * D;
    float* ls = dos + T * D;
    float* dsum = ls + T;
    uint32_t* rks = reinterpret_cast<uint32_t*>(dsum + T);  // row keys of the dropout mask
    const int h = blockIdx.x, b = blockIdx.y;
    const int t0 = (int)threadIdx.x / S, r = (int)threadIdx.x % S;
    const int HD = H * D;
    const int64_t base = (int64_t)b * T * HD + (int64_t)h * D;
    for (int e = threadIdx.x; e < T * D; e += blockDim.x) {
        const int t = e / D, d = e - t * D;
        const int64_t at = base + (int64_t)t * HD + d;
        qs[e] = q[at];
        ks[e] = k[at];
        vs[e] = v[at];
        dos[e] = dout[at];
    }
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) {
            const int64_t at = base + (int64_t)t * HD + d;
            s = fmaf(dout[at], o[at], s);
        }
        dsum[t] = s;
        ls[t] = lse[(int64_t)(b * H + h) * T + t];
        rks[t] = thr ? attn_row_key(*seedp, (uint64_t)(b * H + h) * (uint64_t)T + (uint64_t)t) : 0u;
    }
    __syncthreads();
    // dq: this group's query i = t0, keys j <= i (every S-th from r)
    {
        const int i = t0;
        float qi[D], doi[D], g[D];
        attn_load_row<D>(qs + i * D, qi);
        attn_load_row<D>(dos + i * D, doi);
#pragma unroll
        for (int d = 0; d < D; ++d) g[d] = 0.f;
        const float li = ls[i], di = dsum[i];
        const uint32_t rk = rks[i];
        for (int j = r; j <= i; j += S) {
            float kj[D], vj[D];
            attn_load_row<D>(ks + j * D, kj);
            attn_load_row<D>(vs + j * D, vj);
            const float p = expf(attn_dot<D>(qi, kj) * scale - li);
            const bool keep = thr == 0u || attn_keep(rk, j, thr);
            const float dp = keep ? attn_dot<D>(doi, vj) * inv_keep : 0.f;
            const float ds = p * (dp - di);
#pragma unroll
            for (int d = 0; d < D; ++d) g[d] = fmaf(ds, kj[d], g[d]);
        }
#pragma unroll
        for (int d = 0; d < D; ++d) g[d] = group_sum<S>(g[d], warp_lanes());
        if (r == 0) {
#pragma unroll
            for (int d = 0; d < D; ++d) dq[base + (int64_t)i * HD + d] = g[d] * scale;
        }
    }
    // dk, dv: this group's key j = t0, queries i >= j (every S-th from j + r)
    {
        const int j = t0;
        float kj[D], vj[D], gk[D], gv[D];
        attn_load_row<D>(ks + j * D, kj);
        attn_load_row<D>(vs + j * D, vj);
#pragma unroll
        for (int d = 0; d < D; ++d) gk[d] = gv[d] = 0.f;
        for (int i = j + r; i < T; i += S) {
            float qi[D], doi[D];
            attn_load_row<D>(qs + i * D, qi);
            attn_load_row<D>(dos + i * D, doi);
            const float p = expf(attn_dot<D>(qi, kj) * scale - ls[i]);
            const bool keep = thr == 0u || attn_keep(rks[i], j, thr);
            const float z = keep ? p * inv_keep : 0.f;
            const float dp = keep ? attn_dot<D>(doi, vj) * inv_keep : 0.f;
            const float ds = p * (dp - dsum[i]);
#pragma unroll
            for (int d = 0; d < D; ++d) {
                gv[d] = fmaf(z, doi[d], gv[d]);
                gk[d] = fmaf(ds, qi[d], gk[d]);
            }
        }
        const unsigned lanes = warp_lanes();
#pragma unroll
        for (int d = 0; d < D; ++d) {
            gk[d] = group_sum<S>(gk[d], lanes);
            gv[d] = group_sum<S>(gv[d], lanes);
        }
        if (r == 0) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                dk[base + (int64_t)j * HD + d] = gk[d] * scale;
                dv[base + (int64_t)j * HD + d] = gv[d];
            }
        }
    }
}

// lanes per query (or key): as many as a CTA of at most `cap` threads allows, up to 4
inline int attn_lanes(int T, int cap) { return T * 4 <= cap ? 4 : (T * 2 <= cap ? 2 : 1); }

// keep[b, h, i, j] (1 = kept) of the dropout mask, for the tests
__global__ void attn_mask_kernel(uint8_t* keep, int64_t n, int T, uint32_t thr, const uint64_t* seedp) {
    const uint64_t seed = *seedp;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
        keep[e] = attn_keep(attn_row_key(seed, (uint64_t)(e / T)), (int)(e % T), thr) ? 1 : 0;
}

inline int64_t attn_fwd_smem(int T, int D) { return (int64_t)2 * T * D * 4; }
inline int64_t attn_bwd_smem(int T, int D) { return ((int64_t)4 * T * D + 3 * T) * 4; }

}  // namespace il
