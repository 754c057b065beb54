/*
 * aiwn_il.h -- C ABI of the B200 (sm_100a) IndexedLinear kernels.
 *
 * Drop-in boundary for the reference's GPU path of IndexedLinear
 * (capbrady92-svg/AIWN).  Every entry point takes plain device pointers,
 * int64 sizes, an explicit dtype code and a cudaStream_t (passed as void*),
 * and returns an il_status (0 = success).  No entry point allocates device
 * memory: outputs and workspaces are provided by the caller.  All kernels
 * are enqueued on `stream`; nothing synchronises the host.
 *
 * Shapes (row-major, contiguous):
 *   x      [N, IN]        fp32 or bf16           (IL_F32 / IL_BF16)
 *   table  [K, IN, OUT]   fp32
 *   bias   [OUT]          fp32
 *   out    [N, OUT]       fp32   (fp32 also for bf16 x, as the reference's
 *                                 eager path promotes against the fp32 table)
 *   go     [N, OUT]       fp32
 *   gx     [N, IN]        same dtype as x
 *   gt     [K, IN, OUT]   fp32
 *   gb     [OUT]          fp32
 * bw is the bucket width the reference passes as a Python float (2/K); it
 * is used as the fp32 value (float)bw, exactly as the reference's tensors do.
 *
 * Reference interfaces replaced (paths inside the reference repository):
 *   il_forward        aiwn/layers/indexed_linear.py:101-113 (_Fn.forward:
 *                     Triton _fwd, IL:23-39, then `out + bias`) and
 *                     aiwn/layers/indexed_linear_cuda.cu:192-221
 *                     (pybind `forward(x, table, bias, bw)`, cu:274-276)
 *   il_backward       aiwn/layers/indexed_linear.py:115-151 (_Fn.backward:
 *                     Triton _bwd_x IL:41-60 for gx, one-hot einsum
 *                     IL:131-149 for gt, go.sum(0) IL:151 for gb) and
 *                     aiwn/layers/indexed_linear_cuda.cu:224-267
 *                     (pybind `backward(go, x, table, bw)`, cu:277-279)
 *   il_bins           the bucketing of aiwn/layers/indexed_linear.py:175-177
 *                     (exposed on its own for the bit-exact bin tests)
 *   il_adam_step      torch.optim.Adam as used for the table and bias in the
 *                     reference's training loops (aiwn/training/regression.py:75,
 *                     transformer_validation.py:391)
 * Semantics follow the reference's eager path (IndexedLinear._eager,
 * aiwn/layers/indexed_linear.py:173-182, and autograd's backward of it),
 * which clamps the low bin at 0 and masks the gradient's slope term where
 * the interpolation fraction was clamped; the reference's Triton and CUDA
 * kernels do neither.
 */
#ifndef AIWN_IL_H
#define AIWN_IL_H

#include <stdint.h>

#if defined(__GNUC__)
#define IL_API __attribute__((visibility("default")))
#else
#define IL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    IL_OK = 0,
    IL_ERR_SHAPE = 1,       /* a size is negative, zero where it must not be, or too large */
    IL_ERR_DTYPE = 2,       /* unknown dtype code */
    IL_ERR_ALIGN = 3,       /* a pointer is not aligned as the kernels require */
    IL_ERR_LAUNCH = 4,      /* a CUDA launch or API call failed (cudaGetLastError) */
    IL_ERR_WORKSPACE = 5,   /* workspace missing or smaller than il_workspace_bytes() */
    IL_ERR_NULL = 6,        /* a required pointer is NULL */
    IL_ERR_DEVICE = 7,      /* no usable sm_100 device, or the kernel image does not match */
    IL_ERR_TIMEOUT = 8,     /* a kernel's bounded wait gave up (reported by il_check_device_status) */
    IL_ERR_VALUE = 9        /* an invalid scalar argument (e.g. bw <= 0, K < 2) */
} il_status;

typedef enum { IL_F32 = 0, IL_BF16 = 1 } il_dtype;

/* Human-readable text of a status code (static storage). */
IL_API const char* il_status_string(int status);

/* Library version, e.g. "aiwn_il 0.1.0 sm_100a". */
IL_API const char* il_version(void);

/*
 * Forward: out = sum_i x[n,i] * lerp(T[lo,i,:], T[hi,i,:], fr) + bias.
 * Replaces aiwn/layers/indexed_linear.py:101-113 and
 * aiwn/layers/indexed_linear_cuda.cu:192-221.
 */
IL_API int il_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out,
               int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw, void* stream);

/*
 * il_forward that also adds the bin-occupancy histogram of x into counts[K]
 * (uint64, K <= 16384; the bins of il_bins): the forward kernel that keeps
 * every input column's table slice resident counts while it bins, other
 * shapes run the forward and then il_bin_counts.  Replaces the forward of a
 * layer tracked by the reference's BucketTracker (transformer_validation.py:
 * 92-123: a forward hook copying the input to the host for torch.bincount).
 */
IL_API int il_forward_counts(const void* x, int x_dtype, const float* table, const float* bias, float* out,
                             int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw, uint64_t* counts,
                             void* stream);

/*
 * Bytes of device workspace il_backward needs for these sizes (0 if none).
 */
IL_API int64_t il_workspace_bytes(int64_t N, int64_t IN, int64_t OUT, int64_t K, int x_dtype);

/*
 * Backward.  Any of gx / gt / gb may be NULL to skip that gradient.
 * gt and gb are overwritten (not accumulated into).
 * Replaces aiwn/layers/indexed_linear.py:115-151 and
 * aiwn/layers/indexed_linear_cuda.cu:224-267.
 */
IL_API int il_backward(const float* go, const void* x, int x_dtype, const float* table, void* gx,
                float* gt, float* gb, int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw,
                void* workspace, int64_t workspace_bytes, void* stream);

/*
 * il_backward with gt and gb added into instead of overwritten: the caller
 * zeroes them once, then one call per chunk of a batch sums the chunks'
 * gradients in place (gx is still written, not accumulated).  The reference
 * has no counterpart (autograd returns fresh gradients); it serves chunked
 * passes over a batch, such as the host-buffer pipeline, without an extra
 * add per chunk.
 */
IL_API int il_backward_accumulate(const float* go, const void* x, int x_dtype, const float* table, void* gx,
                           float* gt, float* gb, int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw,
                           void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Bins of every x element: lo (int32), hi (int32), fr (fp32); any output may
 * be NULL.  Bit-exact with aiwn/layers/indexed_linear.py:175-177.
 */
IL_API int il_bins(const void* x, int x_dtype, int64_t N, int64_t IN, int64_t K, double bw, int32_t* lo,
            int32_t* hi, float* fr, void* stream);

/*
 * Bin-occupancy histogram: counts[k] += the number of elements of x[N, IN]
 * whose bin lo is k (k < K <= 16384), with the bit-exact bins of il_bins.
 * Accumulates, so repeated calls add up.  Replaces the bincount of
 * aiwn/experiments/bucket_analysis.py:44-47 and transformer_validation.py:105-108.
 */
IL_API int il_bin_counts(const void* x, int x_dtype, int64_t N, int64_t IN, int64_t K, double bw,
                  uint64_t* counts, void* stream);

/*
 * One fused Adam step over `n` fp32 parameters (torch.optim.Adam semantics,
 * no weight decay, no amsgrad):  m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2;
 * p -= lr/(1-b1^step) * m / (sqrt(v)/sqrt(1-b2^step) + eps).
 */
IL_API int il_adam_step(float* p, const float* g, float* m, float* v, int64_t n, double lr, double beta1,
                 double beta2, double eps, int64_t step, void* stream);

/*
 * IndexedLinearV2 forward: the GaussianCDFNorm prologue
 *   xn = 2 * (0.5 * (1 + erf(LayerNorm(x; gamma, beta, eps) / sqrt 2))) - 1
 * feeding the IndexedLinear forward, out = IndexedLinear(xn).  x is fp32
 * [N, IN]; gamma, beta [IN].  Also writes xn [N, IN] and the per-token mean
 * and rstd = 1/sqrt(var + eps) [N], which il_cdf_backward and il_backward (on
 * xn) need.  For IN <= 32 the prologue runs inside the forward kernel.
 * Replaces aiwn/layers/indexed_linear_v2.py:19-37 and :80-88.
 */
IL_API int il_cdf_forward(const float* x, const float* gamma, const float* beta, double eps, const float* table,
                   const float* bias, float* xn, float* mean, float* rstd, float* out, int64_t N, int64_t IN,
                   int64_t OUT, int64_t K, double bw, void* stream);

/*
 * LayerNorm over the last dimension for in_d = IN <= 32 (fp32, biased
 * variance, elementwise affine): y = (x - mean) * rstd * gamma + beta with
 * rstd = 1/sqrt(var + eps); also writes mean and rstd [N] for the backward.
 * Replaces torch.nn.LayerNorm(d_idx) in the reference's IndexedGPT blocks
 * (transformer_validation.py:297-298, 329), whose d_idx is 16 at config 5.
 */
IL_API int il_layernorm_forward(const float* x, const float* gamma, const float* beta, double eps, float* y,
                         float* mean, float* rstd, int64_t N, int64_t IN, void* stream);

/*
 * Backward of il_layernorm_forward given gy = dL/dy: writes dx [N, IN] and
 * overwrites dgamma, dbeta [IN] (any of the three may be NULL).  IN <= 32.
 */
IL_API int il_layernorm_backward(const float* gy, const float* x, const float* gamma, const float* mean,
                          const float* rstd, float* dx, float* dgamma, float* dbeta, int64_t N, int64_t IN,
                          void* stream);

/*
 * Causal self-attention of the IndexedGPT blocks (transformer_validation.py:
 * 254-269: softmax(mask(q k^T * scale)) with dropout p, times v) for heads of
 * D = 2, 4, 8 or 16 features, T <= 1024 positions (512 for D = 16).  q, k, v, o are fp32
 * [B, T, H*D] (head h in columns h*D..h*D+D-1); lse [B, H, T] receives the
 * log-sum-exp of each query's scores for the backward.  With p > 0, *seed
 * (device memory) selects the dropout mask; the backward must get the same
 * seed.  Element (b, h, i, j) is kept when fmix32(rk + j * 0x85EBCA77) >= p *
 * 2^32, with fmix32 MurmurHash3's 32-bit finaliser and the row key
 * rk = fmix32(lo32(seed) ^ fmix32(hi32(seed) + lo32(row) * 0x9E3779B9 + hi32(row))),
 * row = (b*H + h)*T + i.
 */
IL_API int il_attention_forward(const float* q, const float* k, const float* v, float* o, float* lse, int64_t B,
                         int64_t T, int64_t H, int64_t D, double scale, double p, const uint64_t* seed,
                         void* stream);

/* Backward of il_attention_forward given dout = dL/do: writes dq, dk, dv. */
IL_API int il_attention_backward(const float* q, const float* k, const float* v, const float* o,
                          const float* dout, const float* lse, float* dq, float* dk, float* dv, int64_t B,
                          int64_t T, int64_t H, int64_t D, double scale, double p, const uint64_t* seed,
                          void* stream);

/* The dropout mask of il_attention_forward as keep[B, H, T, T] (1 = kept), for tests. */
IL_API int il_attention_dropout_mask(uint8_t* keep, int64_t B, int64_t T, int64_t H, double p,
                              const uint64_t* seed, void* stream);

/*
 * Backward of the GaussianCDFNorm prologue: given gxn = dL/dxn (from
 * il_backward run on xn), writes dx [N, IN] and overwrites dgamma, dbeta [IN].
 * Any of dx / dgamma / dbeta may be NULL.  IN <= 16384.  PyTorch autograd's
 * backward of aiwn/layers/indexed_linear_v2.py:33-36.
 */
IL_API int il_cdf_backward(const float* gxn, const float* x, const float* gamma, const float* beta,
                    const float* mean, const float* rstd, float* dx, float* dgamma, float* dbeta, int64_t N,
                    int64_t IN, void* stream);

/*
 * In-place all-reduce (sum, times `scale`) of an fp32 buffer of n elements
 * across the `world` GPUs of one NVLink/NVSwitch node, one process (rank) per
 * GPU.  bufs[p] and scratch[p] (HOST arrays of `world` device addresses) are
 * rank p's buffer and scratch region as mapped in this process (peer-
 * accessible memory, e.g. torch symmetric memory); bufs[rank] and
 * scratch[rank] are this rank's own.  Every address is 256-byte aligned;
 * each scratch region holds il_allreduce_scratch_bytes(n, world) bytes,
 * zeroed on every rank (and all ranks past a host barrier) before the first
 * call.  Every rank makes the same sequence of calls with the same n.  One
 * kernel, enqueued on `stream`: up to 2^21 elements, every value travels
 * with its call's flag in one 64-bit word (pushed to the reducing rank, then
 * the sums pushed back), so no fence or barrier is needed; larger buffers
 * take a two-shot kernel (peer loads reduce, peer stores deliver) with
 * per-block flag barriers.  Waits are bounded by timeout_s; on expiry
 * il_check_device_status reports IL_ERR_TIMEOUT.  world <= 16.  The
 * reference has no multi-GPU path; this is the gradient exchange of
 * token-parallel training, summing the table and bias gradients of
 * aiwn/layers/indexed_linear.py:131-151 over the ranks' tokens.
 */
IL_API int64_t il_allreduce_scratch_bytes(int64_t n, int world);
IL_API int il_allreduce_sum(float* const* bufs, void* const* scratch, int64_t n, int rank, int world,
                            double scale, double timeout_s, void* stream);

/*
 * il_allreduce_sum for callers that cannot allocate device memory: no
 * counterpart in the reference.  Meant for code that drives all the GPUs of
 * a node from one process but may not call cudaMalloc itself -- for example
 * a plugin inside a host framework whose memory pool owns every byte of the
 * device, or code running where an allocation would stall or fail -- and so
 * cannot provide the scratch region il_allreduce_sum needs.  One call sums
 * bufs[0..world-1] in place (times scale): bufs[p] is a 16-byte aligned
 * device pointer on device p (host array), streams[p] a stream of device p;
 * the call enqueues every device's work itself and orders the devices'
 * streams with events (no kernel waits on another).  Each device builds the
 * sum in a static array compiled into the library (1 MiB, held by every GPU
 * that loads it until the process exits), then copies it into its buffer;
 * hence n <= 2^18 elements and world <= 8 (devices 0..world-1), IL_ERR_SHAPE
 * beyond.  The first call that uses a device looks up that device's copy,
 * creates its two events and enables peer access between the call's devices
 * (no allocation of device memory), so make it before any stream capture.
 * All calls share the static arrays, so calls whose kernels overlap on the
 * GPUs race: order them (the same streams, or synchronise between calls).
 */
IL_API int il_allreduce_sum_noalloc(float* const* bufs, int64_t n, int world, double scale,
                                    void* const* streams);

/*
 * Number of kernels this library has launched in the process so far
 * (host-side counter, all devices and threads).  Lets a caller count the
 * library's launches inside a timed region.
 */
IL_API int64_t il_kernel_launches(void);

/*
 * Reads (and clears) the device-side error word that kernels set when a
 * bounded wait gives up; returns IL_OK or IL_ERR_TIMEOUT.  Synchronises
 * `stream`.
 */
IL_API int il_check_device_status(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AIWN_IL_H */
