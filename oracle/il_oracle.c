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
 * GaussianCDFNorm prologue of IndexedLinearV2 (aiwn/layers/indexed_linear_v2.py:19-37):
 *   z = LayerNorm(x) (biased variance, eps), e = erf(z / sqrt 2),
 *   u = 0.5 * (1 + e), xn = u * 2 - 1, each fp32 operation rounded once; the
 *   row mean and variance are accumulated in double (closest to ATen's
 *   vectorised moments; the restatement stays within 2.4e-7 of the
 *   reference).  erf is the C library's erff.  Its backward is autograd's:
 *   ds = g * 2/sqrt(pi) * exp(-s^2) with s = z / sqrt 2, dz = ds / sqrt 2,
 *   then ATen's LayerNorm backward.
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


/* ---- GaussianCDFNorm prologue (IndexedLinearV2) --------------------------- */

static const float kSqrt2f = 1.41421354f; /* fp32 value of math.sqrt(2.0) */

static void row_moments(const float* r, int64_t IN, float eps, float* mean, float* rstd) {
    double s = 0.0, q = 0.0;
    for (int64_t k = 0; k < IN; ++k) s += r[k];
    const double m = s / (double)IN;
    for (int64_t k = 0; k < IN; ++k) q += ((double)r[k] - m) * ((double)r[k] - m);
    *mean = (float)m;
    const float var = (float)(q / (double)IN);
    *rstd = 1.0f / sqrtf(var + eps);
}

/* xn [N, IN], mean [N], rstd [N]  (aiwn/layers/indexed_linear_v2.py:33-36) */
void il_oracle_cdf_forward(const float* x, const float* gamma, const float* beta, double eps, int64_t N,
                           int64_t IN, float* xn, float* mean, float* rstd) {
    const float epsf = (float)eps;
    for (int64_t n = 0; n < N; ++n) {
        const float* r = x + n * IN;
        float m, rs;
        row_moments(r, IN, epsf, &m, &rs);
        if (mean) mean[n] = m;
        if (rstd) rstd[n] = rs;
        for (int64_t k = 0; k < IN; ++k) {
            const float z = ((r[k] - m) * rs) * gamma[k] + beta[k];
            const float e = erff(z / kSqrt2f);
            const float u = 0.5f * (1.0f + e);
            xn[n * IN + k] = u * 2.0f - 1.0f;
        }
    }
}

/* dx [N, IN], dgamma [IN], dbeta [IN] given g = dL/dxn (any output may be NULL) */
int il_oracle_cdf_backward(const float* g, const float* x, const float* gamma, const float* beta, double eps,
                           int64_t N, int64_t IN, float* dx, float* dgamma, float* dbeta) {
    const float epsf = (float)eps;
    double* ag = (double*)calloc((size_t)(2 * IN), sizeof(double));
    float* dz = (float*)malloc((size_t)IN * sizeof(float));
    if (!ag || !dz) {
        free(ag);
        free(dz);
        return 1;
    }
    for (int64_t n = 0; n < N; ++n) {
        const float* r = x + n * IN;
        float m, rs;
        row_moments(r, IN, epsf, &m, &rs);
        double sdy_g_x = 0.0, sdy_g = 0.0;
        for (int64_t k = 0; k < IN; ++k) {
            const float xh = (r[k] - m) * rs;
            const float z = xh * gamma[k] + beta[k];
            const float sv = z / kSqrt2f;
            const float ds = (g[n * IN + k] * 1.12837916709551257f) * expf(-(sv * sv));
            dz[k] = ds / kSqrt2f;
            ag[k] += (double)dz[k] * (double)xh;
            ag[IN + k] += (double)dz[k];
            sdy_g_x += (double)dz[k] * (double)gamma[k] * (double)r[k];
            sdy_g += (double)dz[k] * (double)gamma[k];
        }
        if (dx) {
            /* ATen's CPU LayerNorm backward: dx = a*dy*gamma + b*x + c */
            const double a = rs;
            const double b = (sdy_g * m - sdy_g_x) * a * a * a / (double)IN;
            const double c = -b * m - sdy_g * a / (double)IN;
            for (int64_t k = 0; k < IN; ++k)
                dx[n * IN + k] = (float)(a * (double)dz[k] * (double)gamma[k] + b * (double)r[k] + c);
        }
    }
    for (int64_t k = 0; k < IN; ++k) {
        if (dgamma) dgamma[k] = (float)ag[k];
        if (dbeta) dbeta[k] = (float)ag[IN + k];
    }
    free(ag);
    free(dz);
    return 0;
}
