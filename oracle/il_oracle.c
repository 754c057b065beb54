/*
 * il_oracle.c -- CPU restatement of the reference IndexedLinear eager path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle: the parity tests,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg use it as the
 * checker.  Nothing in the aiwn_b200 package links, loads or calls it.
 *
 * It restates, operation by operation and in fp32, what the reference
 * computes on its `--device cpu` path:
 *
 *   bins      aiwn/layers/indexed_linear.py:175-177  (IndexedLinear._eager)
 *               bk = ((x + 1) / bw).long().clamp(0, K-1)
 *               hi = (bk + 1).clamp(max=K-1)
 *               fr = ((x - (-1 + bk.float()*bw)) / bw).clamp(0, 1)
 *   forward   aiwn/layers/indexed_linear.py:178-182
 *               out = ((T[bk,i]*(1-fr) + T[hi,i]*fr) * x).sum(1) + bias
 *   backward  PyTorch autograd of the forward above (the reference has no
 *             hand-written backward on this path):
 *               gx  = sum_j go*L  +  [0<=fr_pre<=1] * (sum_j (go*x)*thi
 *                                                    - sum_j (go*x)*tlo) / bw
 *               gt  = index_put(accumulate) of (go*x)*(1-fr) at bk and of
 *                     (go*x)*fr at hi  (two index backwards, then summed)
 *               gb  = go.sum(0)
 *
 * Numeric conventions pinned against the reference (tests/golden/):
 *   - bw is the Python double 2/K converted once to fp32; every division is
 *     an IEEE fp32 division by that value (ATen's CPU scalar division).
 *   - bf16 x: (x + 1) is rounded to bf16, then the quotient by bw is rounded
 *     to bf16 again, before truncation (ATen computes reduced-float ops in
 *     fp32 and rounds each result).  fr is computed in fp32 from the exact
 *     fp32 value of x.  The output is fp32 (type promotion against the fp32
 *     table and bias).  gx is the bf16 sum of the two separately rounded
 *     gradient contributions, as autograd accumulates them.
 *   - .long() of an fp32 value outside the int64 range, or of NaN, yields
 *     INT64_MIN on x86 (cvttss2si), which the clamp turns into bin 0.
 *   - clamp propagates NaN; its gradient passes where min <= v <= max.
 *
 * Build: oracle/Makefile  (gcc -O2 -ffp-contract=off: no FMA contraction,
 * every fp32 operation rounds exactly once, as ATen's elementwise ops do).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <pthread.h>
#include <unistd.h>

#define DT_F32 0
#define DT_BF16 1

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* round-to-nearest-even fp32 -> bf16 (NaN kept quiet) */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float bf16_round(float f) { return bf16_to_f32(f32_to_bf16(f)); }

static inline float load_x(const void* x, int dt, int64_t idx) {
    if (dt == DT_BF16) return bf16_to_f32(((const uint16_t*)x)[idx]);
    return ((const float*)x)[idx];
}

/* trunc-to-int64 then clamp(0, K-1), with x86's out-of-range result */
static inline int32_t lo_from_quotient(float q, int64_t K) {
    if (!(fabsf(q) < 9223372036854775808.0f)) return 0; /* NaN / |q|>=2^63 */
    int64_t t = (int64_t)q; /* C truncation toward zero */
    if (t < 0) return 0;
    if (t > K - 1) return (int32_t)(K - 1);
    return (int32_t)t;
}

static inline float clamp01_nan(float v) {
    if (v != v) return v;
    if (v < 0.0f) return 0.0f;
    if (v > 1.0f) return 1.0f;
    return v;
}

/* One (n,i) element: lo, hi, fr, the unclamped fr and the exact fp32 x. */
typedef struct {
    int32_t lo, hi;
    float fr, fr_pre, xv;
} bin_t;

static inline bin_t bin_of(const void* x, int dt, int64_t idx, int64_t K, float bwf) {
    bin_t b;
    float xv = load_x(x, dt, idx);
    float q;
    if (dt == DT_BF16) {
        float s = bf16_round(xv + 1.0f);
        q = bf16_round(s / bwf);
    } else {
        q = (xv + 1.0f) / bwf;
    }
    b.lo = lo_from_quotient(q, K);
    b.hi = (b.lo + 1 > K - 1) ? (int32_t)(K - 1) : b.lo + 1;
    float c = (float)b.lo * bwf;
    c = c + (-1.0f);
    float num = xv - c;
    b.fr_pre = num / bwf;
    b.fr = clamp01_nan(b.fr_pre);
    b.xv = xv;
    return b;
}

void il_oracle_bins(const void* x, int x_dtype, int64_t N, int64_t IN, int64_t K,
                    double bw, int32_t* lo, int32_t* hi, float* fr) {
    float bwf = (float)bw;
    for (int64_t e = 0; e < N * IN; ++e) {
        bin_t b = bin_of(x, x_dtype, e, K, bwf);
        if (lo) lo[e] = b.lo;
        if (hi) hi[e] = b.hi;
        if (fr) fr[e] = b.fr;
    }
}

static int pick_threads(int nthreads) {
    if (nthreads <= 0) {
        long c = sysconf(_SC_NPROCESSORS_ONLN);
        nthreads = c > 0 ? (int)c : 1;
    }
    return nthreads > 256 ? 256 : nthreads;
}

/* static-schedule parallel for over [0, n): body(lo, hi, arg) */
typedef void (*range_fn)(int64_t lo, int64_t hi, void* arg);
typedef struct {
    range_fn fn;
    void* arg;
    int64_t lo, hi;
} range_task;

static void* range_thread(void* p) {
    range_task* t = (range_task*)p;
    t->fn(t->lo, t->hi, t->arg);
    return NULL;
}

static void parallel_for(int64_t n, int nthreads, range_fn fn, void* arg) {
    int nt = pick_threads(nthreads);
    if (nt > n) nt = (int)(n > 0 ? n : 1);
    if (nt <= 1) {
        fn(0, n, arg);
        return;
    }
    pthread_t th[256];
    range_task task[256];
    int64_t chunk = (n + nt - 1) / nt;
    int started = 0;
    for (int t = 0; t < nt; ++t) {
        task[t].fn = fn;
        task[t].arg = arg;
        task[t].lo = t * chunk < n ? t * chunk : n;
        task[t].hi = (t + 1) * chunk < n ? (t + 1) * chunk : n;
        if (pthread_create(&th[t], NULL, range_thread, &task[t]) != 0) {
            range_thread(&task[t]);
            th[t] = 0;
        } else {
            ++started;
        }
    }
    for (int t = 0; t < nt; ++t)
        if (th[t]) pthread_join(th[t], NULL);
    (void)started;
}

/* ---- forward ---------------------------------------------------------- */
typedef struct {
    const void* x;
    int dt;
    const float *table, *bias;
    float* out;
    int64_t IN, OUT, K;
    float bwf;
} fwd_args;

static void fwd_range(int64_t n0, int64_t n1, void* p) {
    fwd_args* a = (fwd_args*)p;
    const int64_t IN = a->IN, OUT = a->OUT;
    for (int64_t n = n0; n < n1; ++n) {
        float* o = a->out + n * OUT;
        for (int64_t j = 0; j < OUT; ++j) o[j] = 0.0f;
        for (int64_t i = 0; i < IN; ++i) {
            bin_t b = bin_of(a->x, a->dt, n * IN + i, a->K, a->bwf);
            const float* tlo = a->table + ((int64_t)b.lo * IN + i) * OUT;
            const float* thi = a->table + ((int64_t)b.hi * IN + i) * OUT;
            float omf = 1.0f - b.fr;
            for (int64_t j = 0; j < OUT; ++j) {
                float L = tlo[j] * omf;
                float R = thi[j] * b.fr;
                float w = L + R;
                o[j] += w * b.xv;
            }
        }
        for (int64_t j = 0; j < OUT; ++j) o[j] = o[j] + a->bias[j];
    }
}

/* out[N,OUT] (fp32) = ((T[lo,i]*(1-fr) + T[hi,i]*fr) * x).sum(i) + bias */
void il_oracle_forward(const void* x, int x_dtype, const float* table, const float* bias,
                       float* out, int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw,
                       int nthreads) {
    fwd_args a = {x, x_dtype, table, bias, out, IN, OUT, K, (float)bw};
    parallel_for(N, nthreads, fwd_range, &a);
}

/* ---- backward ---------------------------------------------------------- */
typedef struct {
    const float* go;
    const void* x;
    int dt;
    const float* table;
    void* gx;
    float *glo, *ghi;
    int64_t N, IN, OUT, K;
    float bwf;
} bwd_args;

static void gx_range(int64_t n0, int64_t n1, void* p) {
    bwd_args* a = (bwd_args*)p;
    const int64_t IN = a->IN, OUT = a->OUT;
    for (int64_t n = n0; n < n1; ++n) {
        const float* g = a->go + n * OUT;
        for (int64_t i = 0; i < IN; ++i) {
            bin_t b = bin_of(a->x, a->dt, n * IN + i, a->K, a->bwf);
            const float* tlo = a->table + ((int64_t)b.lo * IN + i) * OUT;
            const float* thi = a->table + ((int64_t)b.hi * IN + i) * OUT;
            float omf = 1.0f - b.fr;
            float t1 = 0.0f, shi = 0.0f, slo = 0.0f;
            for (int64_t j = 0; j < OUT; ++j) {
                float L = tlo[j] * omf + thi[j] * b.fr;
                t1 += g[j] * L;
                float gxj = g[j] * b.xv;
                shi += gxj * thi[j];
                slo += gxj * tlo[j];
            }
            float gfr = shi + (-slo);
            int pass = (b.fr_pre >= 0.0f) && (b.fr_pre <= 1.0f);
            float t2 = pass ? gfr / a->bwf : 0.0f;
            int64_t e = n * IN + i;
            if (a->dt == DT_BF16) {
                float s = bf16_round(t1) + bf16_round(t2);
                ((uint16_t*)a->gx)[e] = f32_to_bf16(s);
            } else {
                ((float*)a->gx)[e] = t1 + t2;
            }
        }
    }
}

/* each worker owns whole input columns i, so the n-order accumulation
   into glo / ghi is sequential and deterministic */
static void gt_range(int64_t i0, int64_t i1, void* p) {
    bwd_args* a = (bwd_args*)p;
    const int64_t IN = a->IN, OUT = a->OUT;
    for (int64_t i = i0; i < i1; ++i) {
        for (int64_t n = 0; n < a->N; ++n) {
            bin_t b = bin_of(a->x, a->dt, n * IN + i, a->K, a->bwf);
            const float* g = a->go + n * OUT;
            float omf = 1.0f - b.fr;
            float* dlo = a->glo + ((int64_t)b.lo * IN + i) * OUT;
            float* dhi = a->ghi + ((int64_t)b.hi * IN + i) * OUT;
            for (int64_t j = 0; j < OUT; ++j) {
                float gxj = g[j] * b.xv;
                dlo[j] += gxj * omf;
                dhi[j] += gxj * b.fr;
            }
        }
    }
}

/*
 * Backward of the eager forward.  gx has x's dtype (fp32 or raw bf16),
 * gt[K,IN,OUT] and gb[OUT] are fp32.  Any of gx/gt/gb may be NULL.
 * Returns 0, or -1 when the temporary index-backward buffers cannot be
 * allocated.
 */
int il_oracle_backward(const float* go, const void* x, int x_dtype, const float* table,
                       void* gx, float* gt, float* gb, int64_t N, int64_t IN, int64_t OUT,
                       int64_t K, double bw, int nthreads) {
    bwd_args a = {go, x, x_dtype, table, gx, NULL, NULL, N, IN, OUT, K, (float)bw};
    if (gx) parallel_for(N, nthreads, gx_range, &a);
    if (gt) {
        /* two separate index backwards (lo and hi), each accumulated in n
           order, then summed -- as autograd does for table[bk], table[hi] */
        int64_t tsz = K * IN * OUT;
        a.glo = (float*)calloc((size_t)tsz, sizeof(float));
        a.ghi = (float*)calloc((size_t)tsz, sizeof(float));
        if (!a.glo || !a.ghi) {
            free(a.glo);
            free(a.ghi);
            return -1;
        }
        parallel_for(IN, nthreads, gt_range, &a);
        for (int64_t e = 0; e < tsz; ++e) gt[e] = a.glo[e] + a.ghi[e];
        free(a.glo);
        free(a.ghi);
    }
    if (gb) {
        for (int64_t j = 0; j < OUT; ++j) gb[j] = 0.0f;
        for (int64_t n = 0; n < N; ++n)
            for (int64_t j = 0; j < OUT; ++j) gb[j] += go[n * OUT + j];
    }
    return 0;
}

/* Adam step (torch.optim.Adam defaults, no weight decay, no amsgrad),
   in fp32 with torch's single-tensor update order:
     m = b1*m + (1-b1)*g ;  v = b2*v + (1-b2)*g*g
     p -= lr/(1-b1^t) * m / (sqrt(v)/sqrt(1-b2^t) + eps)               */
void il_oracle_adam(float* p, const float* g, float* m, float* v, int64_t n, double lr,
                    double beta1, double beta2, double eps, int64_t step) {
    double bc1 = 1.0 - pow(beta1, (double)step);
    double bc2 = 1.0 - pow(beta2, (double)step);
    float step_size = (float)(lr / bc1);
    float bc2_sqrt = (float)sqrt(bc2);
    float b1 = (float)beta1, b2 = (float)beta2, e = (float)eps;
    for (int64_t k = 0; k < n; ++k) {
        float gk = g[k];
        m[k] = m[k] + (gk - m[k]) * (1.0f - b1);
        v[k] = v[k] * b2 + ((1.0f - b2) * gk) * gk;
        float denom = sqrtf(v[k]) / bc2_sqrt + e;
        p[k] = p[k] - step_size * (m[k] / denom);
    }
}
