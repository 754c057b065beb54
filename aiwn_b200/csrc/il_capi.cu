// il_capi.cu -- the extern "C" entry points declared in include/aiwn_il.h.
//
// Argument checking, kernel selection and launch.  All kernels are compiled
// into this one translation unit (they are included below), so the library
// needs no relocatable device code.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "../../include/aiwn_il.h"
#include "il_common.cuh"
#include "il_simple.cuh"
#include "il_fast.cuh"
#include "il_sorted.cuh"
#include "il_fwd_token.cuh"
#include "il_cdf.cuh"
#include "il_attn.cuh"
#include "il_allreduce.cuh"
#include "il_tc.cuh"
#include "il_fwd_wide.cuh"

namespace {

constexpr int kMaxDevices = 64;
int g_dev_ok[kMaxDevices];  // 0 = unchecked, 1 = sm_100, -1 = other
int g_num_sms[kMaxDevices];
std::mutex g_dev_mu;

int check_device(int* num_sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return IL_ERR_DEVICE;
    }
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_dev_ok[dev] == 0) {
        int major = 0, minor = 0, sms = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (cudaGetLastError() != cudaSuccess) return IL_ERR_DEVICE;
        // the fatbin holds sm_100a code only
        g_dev_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
        g_num_sms[dev] = sms > 0 ? sms : 1;
    }
    if (num_sms) *num_sms = g_num_sms[dev];
    return g_dev_ok[dev] == 1 ? IL_OK : IL_ERR_DEVICE;
}

il::BinCfg make_cfg(double bw, int64_t K) {
    il::BinCfg c;
    c.bw = (float)bw;
    c.K = (int)K;
    int e = 0;
    const float m = frexpf(c.bw, &e);
    c.pow2 = (m == 0.5f) ? 1 : 0;  // bw == 2^(e-1) exactly
    c.inv = c.pow2 ? ldexpf(1.0f, 1 - e) : 1.0f / c.bw;
    return c;
}

int check_common(const void* x, int x_dtype, int64_t N, int64_t IN, int64_t K, double bw) {
    if (x_dtype != IL_F32 && x_dtype != IL_BF16) return IL_ERR_DTYPE;
    if (N < 0 || IN < 1 || K < 2 || K > (1 << 24)) return IL_ERR_SHAPE;
    const float bwf = (float)bw;
    if (!(bwf > 0.0f) || isinf(bwf)) return IL_ERR_VALUE;
    if (N > 0 && !x) return IL_ERR_NULL;
    return IL_OK;
}

// Kernel families.  AIWN_IL_FORWARD=token|cluster and AIWN_IL_BACKWARD=sorted|gather
// restrict il_forward / il_backward to the named family (shapes it cannot take
// fall through to the general kernels).  Unset, or any other value, selects
// automatically: forward with one token per lane when every input column's
// table slice fits one CTA, else one token per lane with the table streamed
// through shared memory (K <= 256), else the cluster kernel; backward by the bin-sorted
// walk whenever the table gradient is wanted and the shape has a plan, else the
// gather kernel.  The families compute the same results; the switches let the
// tests cover each of them.
enum KernelChoice { kAny = 0, kOnlyPreferred = 1, kOnlyOther = 2 };

KernelChoice kernel_choice(const char* var, const char* preferred, const char* other) {
    const char* v = getenv(var);
    if (!v) return kAny;
    if (strcmp(v, preferred) == 0) return kOnlyPreferred;
    if (strcmp(v, other) == 0) return kOnlyOther;
    return kAny;
}

std::atomic<int64_t> g_launches{0};

// every kernel launch of the library is followed by this check
inline int launch_status(int kernels = 1) {
    g_launches.fetch_add(kernels, std::memory_order_relaxed);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? IL_OK : IL_ERR_LAUNCH;
}

inline unsigned grid_for(int64_t work, int threads, int num_sms) {
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)num_sms * 32;
    if (blocks > cap) blocks = cap;
    return (unsigned)(blocks < 1 ? 1 : blocks);
}

// kernel selection of the forward (arguments already checked)
int forward_dispatch(const void* x, int x_dtype, const float* table, const float* bias, float* out, int64_t N,
                     int64_t IN, int64_t OUT, const il::BinCfg& c, int sms, cudaStream_t s) {
    // AIWN_IL_FORWARD=tc: the tensor-core (hat-basis GEMM) forward where it applies
    const char* fv = getenv("AIWN_IL_FORWARD");
    if (fv && strcmp(fv, "tc") == 0 && il::tc_forward_ok(N, IN, OUT, c.K, c)) {
        const int rc = il::tc_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    // AIWN_IL_FORWARD=wide: the warp-per-token forward wherever it applies
    if (fv && strcmp(fv, "wide") == 0 && il::fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        const int rc = il::wide_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    const KernelChoice path = kernel_choice("AIWN_IL_FORWARD", "token", "cluster");
    // Rows of a multiple of 128 (or 64) outputs over at most 128 bins, with
    // tokens for at least one CTA of 4 warps per SM: the warp-per-token
    // forward reads each table row as conflict-free 128-byte lines and beat
    // the cluster and token kernels from 8 K tokens up (16384 x 64 -> 128,
    // K=64: 46 against 97 us; 65536 x 16 -> 128, K=128: 48 against 99 us;
    // 32768 x 128 -> 1024, K=32: 1.25 against 4.14 ms; 64-wide rows: 131072 x
    // 64 -> 64, K=16: 168 against 221 us; 32768 x 64 -> 64, K=64: 51 against
    // 90 us; 131072 x 20 -> 64, K=128: 60 against 113 us), while with fewer
    // tokens its few CTAs lost (2048 x 64 -> 128, K=16: 30 against 17 us;
    // 8192 x 64 -> 64, K=16: 31 against 24 us).
    if (path == kAny && il::wide_jw(OUT) > 0 && c.K <= 128 && (N / 64) * (OUT / il::wide_jw(OUT)) >= sms &&
        il::fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        const int rc = il::wide_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    // Rows of a multiple of 32 outputs over few bins (K <= 64): the cluster
    // kernel's lanes read consecutive chunks of one table row, and it beat the
    // token kernel's per-lane gathers at 32x32 (K=64), 64x64 and 128x128
    // (K=16) for N = 2 K .. 131 K tokens (e.g. 64x64, K=16: 13.8 against
    // 23.7 us at 2 K tokens, 218 against 275 us at 131 K).  With more bins the
    // token kernel stays ahead (20x64, K=512: 126 against 224 us; 32x64,
    // K=128: 205 against 228 us at 131 K).  Tables without a token plan keep
    // the streamed kernel.
    if (path == kAny && OUT % 32 == 0 && c.K <= 64 &&
        il::fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        il::FwdPlan pl;
        if (il::plan_token_forward(N, c.K, (int)IN, (int)OUT, sms, pl) &&
            il::fast_forward_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
            const int rc = il::fast_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s);
            if (rc != il::kNotApplicable) {
                if (rc) {
                    cudaGetLastError();
                    return IL_ERR_LAUNCH;
                }
                return launch_status();
            }
        }
    }
    if (path != kOnlyOther && il::fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        const int rc = il::token_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    if (path == kAny && il::fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        // tables too large to keep resident, rows of a multiple of 128 outputs
        // over at most 128 bins: one warp per token streams the table
        const int rc = il::wide_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    if (path != kOnlyOther && il::fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        // tables too large to keep resident: stream column chunks through shared memory
        const int rc = il::stream_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    if (path != kOnlyPreferred && il::fast_forward_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        const int rc = il::fast_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    const unsigned g = grid_for(N * OUT, 256, sms);
    if (x_dtype == IL_BF16)
        il::fwd_simple_kernel<il::kBF16><<<g, 256, 0, s>>>(x, table, bias, out, N, IN, OUT, c);
    else
        il::fwd_simple_kernel<il::kF32><<<g, 256, 0, s>>>(x, table, bias, out, N, IN, OUT, c);
    return launch_status();
}

// zeroes a[0..na) and b[0..nb) (either may be NULL) with one memset when b
// directly follows a in memory, as the library's own callers allocate them
int zero_pair(float* a, int64_t na, float* b, int64_t nb, cudaStream_t s) {
    if (a && b && b == a + na)
        return cudaMemsetAsync(a, 0, (size_t)(na + nb) * sizeof(float), s) == cudaSuccess ? IL_OK : IL_ERR_LAUNCH;
    if (a && cudaMemsetAsync(a, 0, (size_t)na * sizeof(float), s) != cudaSuccess) return IL_ERR_LAUNCH;
    if (b && cudaMemsetAsync(b, 0, (size_t)nb * sizeof(float), s) != cudaSuccess) return IL_ERR_LAUNCH;
    return IL_OK;
}

// shape, dropout and seed checks shared by the attention entry points
int attn_check(int64_t B, int64_t T, int64_t H, int64_t D, double p, const uint64_t* seed, bool bwd) {
    if (B < 1 || B > 65535 || H < 1 || H > 65535 || T < 1 || T > il::kAttnMaxT) return IL_ERR_SHAPE;
    if (D != 2 && D != 4 && D != 8 && D != 16) return IL_ERR_SHAPE;
    if (T > il::attn_max_t((int)D)) return IL_ERR_SHAPE;
    if ((bwd ? il::attn_bwd_smem((int)T, (int)D) : il::attn_fwd_smem((int)T, (int)D)) > 227 * 1024)
        return IL_ERR_SHAPE;
    if (!(p >= 0.0 && p < 1.0)) return IL_ERR_VALUE;
    if (p > 0.0 && !seed) return IL_ERR_NULL;
    return IL_OK;
}

uint32_t attn_threshold(double p) {
    const double t = p * 4294967296.0;
    return p <= 0.0 ? 0u : (t >= 4294967295.0 ? 4294967295u : (uint32_t)t);
}

template <typename Kern, typename... Args>
int attn_launch(Kern kern, int64_t smem, int64_t B, int64_t T, int64_t H, cudaStream_t s, Args... args) {
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                                cudaSuccess)
        return IL_ERR_LAUNCH;
    kern<<<dim3((unsigned)H, (unsigned)B, 1), (unsigned)T, (size_t)smem, s>>>(args...);
    return launch_status();
}

// ---- all-reduce without allocation (il_allreduce_sum_noalloc) -------------
//
// The sum is built in this file-scope array: every GPU that loads the library
// holds one copy (kNoAllocMaxElems floats, 1 MiB) until the process exits, and
// only that GPU touches it.  In host code the name is only a stand-in for the
// device copies; their addresses come from cudaGetSymbolAddress with each
// device current, once per device, on the first call that uses the device,
// which also enables peer access between the call's devices and creates the
// two events per device that order the devices' streams.  Nothing in the
// array has to start at zero: every call overwrites the elements it reads.
constexpr int64_t kNoAllocMaxElems = (int64_t)1 << 18;  // fp32 elements per buffer
constexpr int kNoAllocMaxRanks = 8;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxElems];

struct NoAllocDev {
    float* scratch = nullptr;               // this device's copy (set-up done when non-null)
    cudaEvent_t entered = nullptr, summed = nullptr;
    bool peer[kMaxDevices] = {};
};
NoAllocDev g_noalloc[kMaxDevices];
std::mutex g_noalloc_mu;

// addresses of the devices' copies, events, peer access between devices 0..world-1
int noalloc_setup(int world) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    for (int p = 0; p < world; ++p) {
        NoAllocDev& d = g_noalloc[p];
        if (cudaSetDevice(p) != cudaSuccess) {
            cudaGetLastError();
            return IL_ERR_DEVICE;
        }
        if (!d.scratch) {
            void* ptr = nullptr;
            if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) {
                cudaGetLastError();
                return IL_ERR_DEVICE;
            }
            if (cudaEventCreateWithFlags(&d.entered, cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&d.summed, cudaEventDisableTiming) != cudaSuccess) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            d.scratch = static_cast<float*>(ptr);
        }
        for (int q = 0; q < world; ++q) {
            if (q == p || d.peer[q]) continue;
            int can = 0;
            if (cudaDeviceCanAccessPeer(&can, p, q) != cudaSuccess || !can) {
                cudaGetLastError();
                return IL_ERR_DEVICE;
            }
            const cudaError_t e = cudaDeviceEnablePeerAccess(q, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
                cudaGetLastError();
                return IL_ERR_DEVICE;
            }
            cudaGetLastError();  // clears cudaErrorPeerAccessAlreadyEnabled
            d.peer[q] = true;
        }
    }
    return IL_OK;
}

// every stream of the call waits for every other device's event (recorded
// just before); the host orders the devices, no kernel waits on another
int noalloc_cross_wait(int world, void* const* streams, bool summed) {
    for (int p = 0; p < world; ++p) {
        if (cudaSetDevice(p) != cudaSuccess) return IL_ERR_DEVICE;
        if (cudaEventRecord(summed ? g_noalloc[p].summed : g_noalloc[p].entered, (cudaStream_t)streams[p]) !=
            cudaSuccess)
            return IL_ERR_LAUNCH;
    }
    for (int p = 0; p < world; ++p) {
        if (cudaSetDevice(p) != cudaSuccess) return IL_ERR_DEVICE;
        for (int q = 0; q < world; ++q)
            if (q != p && cudaStreamWaitEvent((cudaStream_t)streams[p],
                                              summed ? g_noalloc[q].summed : g_noalloc[q].entered, 0) != cudaSuccess)
                return IL_ERR_LAUNCH;
    }
    return IL_OK;
}

}  // namespace

extern "C" {

const char* il_status_string(int s) {
    switch (s) {
        case IL_OK: return "ok";
        case IL_ERR_SHAPE: return "invalid shape";
        case IL_ERR_DTYPE: return "invalid dtype";
        case IL_ERR_ALIGN: return "misaligned pointer";
        case IL_ERR_LAUNCH: return "CUDA launch or API error";
        case IL_ERR_WORKSPACE: return "workspace missing or too small";
        case IL_ERR_NULL: return "required pointer is NULL";
        case IL_ERR_DEVICE: return "no sm_100 (B200) device current";
        case IL_ERR_TIMEOUT: return "a device-side bounded wait gave up";
        case IL_ERR_VALUE: return "invalid scalar argument";
        default: return "unknown status";
    }
}

const char* il_version(void) { return "aiwn_il 0.1.0 sm_100a"; }

int il_forward(const void* x, int x_dtype, const float* table, const float* bias, float* out,
               int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw, void* stream) {
    int st = check_common(x, x_dtype, N, IN, K, bw);
    if (st) return st;
    if (OUT < 1) return IL_ERR_SHAPE;
    if (N == 0) return IL_OK;
    if (!table || !bias || !out) return IL_ERR_NULL;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const il::BinCfg c = make_cfg(bw, K);
    return forward_dispatch(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s);
}

int il_forward_counts(const void* x, int x_dtype, const float* table, const float* bias, float* out, int64_t N,
                      int64_t IN, int64_t OUT, int64_t K, double bw, uint64_t* counts, void* stream) {
    int st = check_common(x, x_dtype, N, IN, K, bw);
    if (st) return st;
    if (OUT < 1 || K > 16384) return IL_ERR_SHAPE;
    if (N == 0) return IL_OK;
    if (!table || !bias || !out || !counts) return IL_ERR_NULL;
    if ((uintptr_t)counts & 7) return IL_ERR_ALIGN;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const il::BinCfg c = make_cfg(bw, K);
    auto* cnt = reinterpret_cast<unsigned long long*>(counts);
    // the token forward counts while it bins; other shapes take the forward and a counting pass
    if (kernel_choice("AIWN_IL_FORWARD", "token", "cluster") != kOnlyOther &&
        il::fast_forward_args_ok(x, x_dtype, table, bias, out, N, IN, OUT, c.K, c)) {
        const int rc = il::token_forward(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s, cnt);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    if ((st = forward_dispatch(x, x_dtype, table, bias, out, N, IN, OUT, c, sms, s))) return st;
    return il_bin_counts(x, x_dtype, N, IN, K, bw, counts, stream);
}

int il_cdf_forward(const float* x, const float* gamma, const float* beta, double eps, const float* table,
                   const float* bias, float* xn, float* mean, float* rstd, float* out, int64_t N, int64_t IN,
                   int64_t OUT, int64_t K, double bw, void* stream) {
    int st = check_common(x, IL_F32, N, IN, K, bw);
    if (st) return st;
    if (OUT < 1) return IL_ERR_SHAPE;
    if (!(eps >= 0.0)) return IL_ERR_VALUE;
    if (N == 0) return IL_OK;
    if (!gamma || !beta || !table || !bias || !xn || !mean || !rstd || !out) return IL_ERR_NULL;
    if (N > INT32_MAX) return IL_ERR_SHAPE;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const il::BinCfg c = make_cfg(bw, K);
    const il::CdfArgs q{gamma, beta, (float)eps, xn, mean, rstd};
    const KernelChoice path = kernel_choice("AIWN_IL_FORWARD", "token", "cluster");
    if (path != kOnlyOther && il::fast_forward_args_ok(x, IL_F32, table, bias, out, N, IN, OUT, K, c)) {
        const int rc = il::token_cdf_forward(x, q, table, bias, out, N, IN, OUT, c, sms, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    // prologue as its own pass, then the forward on xn
    const unsigned blocks = (unsigned)((N + il::kCdfRowThreads - 1) / il::kCdfRowThreads);
    const int vec = (IN % 4 == 0) && ((((uintptr_t)x | (uintptr_t)xn) & 15) == 0);
    if (IN <= 8)
        il::cdf_prologue_small_kernel<8><<<blocks, il::kCdfRowThreads, 0, s>>>(x, q, (int)N, (int)IN, vec);
    else if (IN <= 16)
        il::cdf_prologue_small_kernel<16><<<blocks, il::kCdfRowThreads, 0, s>>>(x, q, (int)N, (int)IN, vec);
    else if (IN <= 24)
        il::cdf_prologue_small_kernel<24><<<blocks, il::kCdfRowThreads, 0, s>>>(x, q, (int)N, (int)IN, vec);
    else if (IN <= 32)
        il::cdf_prologue_small_kernel<32><<<blocks, il::kCdfRowThreads, 0, s>>>(x, q, (int)N, (int)IN, vec);
    else
        il::cdf_prologue_kernel<<<blocks, il::kCdfRowThreads, 0, s>>>(x, q, (int)N, (int)IN);
    if ((st = launch_status())) return st;
    return forward_dispatch(xn, IL_F32, table, bias, out, N, IN, OUT, c, sms, s);
}

int il_cdf_backward(const float* gxn, const float* x, const float* gamma, const float* beta, const float* mean,
                    const float* rstd, float* dx, float* dgamma, float* dbeta, int64_t N, int64_t IN, void* stream) {
    if (N < 0 || IN < 1 || IN > 16384 || N > INT32_MAX) return IL_ERR_SHAPE;
    if (N > 0 && (!gxn || !x || !gamma || !beta || !mean || !rstd)) return IL_ERR_NULL;
    int sms = 0;
    int st = check_device(&sms);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if ((st = zero_pair(dgamma, IN, dbeta, IN, s))) return st;
    if (N == 0 || (!dx && !dgamma && !dbeta)) return IL_OK;
    if (IN <= il::kCdfMaxIn) {
        const int vec = (IN % 4 == 0) && ((((uintptr_t)gxn | (uintptr_t)x | (uintptr_t)dx) & 15) == 0);
        // one wave, several tokens per thread: the block reduction runs once per block
        const int64_t want = (N + il::kCdfRowThreads - 1) / il::kCdfRowThreads;
        const unsigned blocks = (unsigned)std::min<int64_t>(want, (int64_t)sms);
        auto run = [&](auto kern) {
            kern<<<blocks, il::kCdfRowThreads, 0, s>>>(gxn, x, gamma, beta, mean, rstd, dx, dgamma, dbeta, (int)N,
                                                       (int)IN, vec);
        };
        if (IN <= 8) run(il::cdf_backward_small_kernel<8>);
        else if (IN <= 16) run(il::cdf_backward_small_kernel<16>);
        else if (IN <= 24) run(il::cdf_backward_small_kernel<24>);
        else run(il::cdf_backward_small_kernel<32>);
        return launch_status();
    }
    const size_t smem = (size_t)(2 * IN) * sizeof(float);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(il::cdf_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return IL_ERR_LAUNCH;
    const unsigned blocks = (unsigned)((N + il::kCdfRowThreads - 1) / il::kCdfRowThreads);
    il::cdf_backward_kernel<<<blocks, il::kCdfRowThreads, smem, s>>>(gxn, x, gamma, beta, mean, rstd, dx, dgamma,
                                                                      dbeta, (int)N, (int)IN);
    return launch_status();
}

int il_layernorm_forward(const float* x, const float* gamma, const float* beta, double eps, float* y, float* mean,
                         float* rstd, int64_t N, int64_t IN, void* stream) {
    if (N < 0 || IN < 1 || IN > il::kCdfMaxIn || N > INT32_MAX) return IL_ERR_SHAPE;
    if (!(eps >= 0.0)) return IL_ERR_VALUE;
    if (N == 0) return IL_OK;
    if (!x || !gamma || !beta || !y || !mean || !rstd) return IL_ERR_NULL;
    int sms = 0;
    int st = check_device(&sms);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    il::CdfArgs q;
    q.gamma = gamma;
    q.beta = beta;
    q.eps = (float)eps;
    q.xn = y;
    q.mean = mean;
    q.rstd = rstd;
    const unsigned blocks = (unsigned)((N + il::kCdfRowThreads - 1) / il::kCdfRowThreads);
    const int vec = (IN % 4 == 0) && ((((uintptr_t)x | (uintptr_t)y) & 15) == 0);
    auto run = [&](auto kern) { kern<<<blocks, il::kCdfRowThreads, 0, s>>>(x, q, (int)N, (int)IN, vec); };
    if (IN <= 8) run(il::cdf_prologue_small_kernel<8, false>);
    else if (IN <= 16) run(il::cdf_prologue_small_kernel<16, false>);
    else if (IN <= 24) run(il::cdf_prologue_small_kernel<24, false>);
    else run(il::cdf_prologue_small_kernel<32, false>);
    return launch_status();
}

int il_layernorm_backward(const float* gy, const float* x, const float* gamma, const float* mean, const float* rstd,
                          float* dx, float* dgamma, float* dbeta, int64_t N, int64_t IN, void* stream) {
    if (N < 0 || IN < 1 || IN > il::kCdfMaxIn || N > INT32_MAX) return IL_ERR_SHAPE;
    if (N > 0 && (!gy || !x || !gamma || !mean || !rstd)) return IL_ERR_NULL;
    int sms = 0;
    int st = check_device(&sms);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if ((st = zero_pair(dgamma, IN, dbeta, IN, s))) return st;
    if (N == 0 || (!dx && !dgamma && !dbeta)) return IL_OK;
    const int vec = (IN % 4 == 0) && ((((uintptr_t)gy | (uintptr_t)x | (uintptr_t)dx) & 15) == 0);
    // one wave, several tokens per thread: the block reduction runs once per block
    const int64_t want = (N + il::kCdfRowThreads - 1) / il::kCdfRowThreads;
    const unsigned blocks = (unsigned)std::min<int64_t>(want, (int64_t)sms);
    auto run = [&](auto kern) {
        kern<<<blocks, il::kCdfRowThreads, 0, s>>>(gy, x, gamma, nullptr, mean, rstd, dx, dgamma, dbeta, (int)N,
                                                   (int)IN, vec);
    };
    if (IN <= 8) run(il::cdf_backward_small_kernel<8, false>);
    else if (IN <= 16) run(il::cdf_backward_small_kernel<16, false>);
    else if (IN <= 24) run(il::cdf_backward_small_kernel<24, false>);
    else run(il::cdf_backward_small_kernel<32, false>);
    return launch_status();
}

int il_attention_forward(const float* q, const float* k, const float* v, float* o, float* lse, int64_t B,
                         int64_t T, int64_t H, int64_t D, double scale, double p, const uint64_t* seed,
                         void* stream) {
    int st = attn_check(B, T, H, D, p, seed, false);
    if (st) return st;
    if (!q || !k || !v || !o || !lse) return IL_ERR_NULL;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const uint32_t thr = attn_threshold(p);
    const float inv_keep = (float)(1.0 / (1.0 - p));
    const int64_t smem = il::attn_fwd_smem((int)T, (int)D);
    const int t = (int)T, h = (int)H;
    const float sc = (float)scale;
    const int S = il::attn_lanes(t, il::kAttnMaxT);
    const int64_t nt = T * S;
#define IL_ATTN_FWD(DD, SS)                                                                                      \
    attn_launch(il::attn_fwd_kernel<DD, SS>, smem, B, nt, H, s, q, k, v, o, lse, t, h, sc, thr, inv_keep, seed)
#define IL_ATTN_FWD_S(DD) (S == 4 ? IL_ATTN_FWD(DD, 4) : S == 2 ? IL_ATTN_FWD(DD, 2) : IL_ATTN_FWD(DD, 1))
    switch (D) {
        case 2: return IL_ATTN_FWD_S(2);
        case 4: return IL_ATTN_FWD_S(4);
        case 8: return IL_ATTN_FWD_S(8);
        default: return IL_ATTN_FWD_S(16);
    }
#undef IL_ATTN_FWD_S
#undef IL_ATTN_FWD
}

int il_attention_backward(const float* q, const float* k, const float* v, const float* o, const float* dout,
                          const float* lse, float* dq, float* dk, float* dv, int64_t B, int64_t T, int64_t H,
                          int64_t D, double scale, double p, const uint64_t* seed, void* stream) {
    int st = attn_check(B, T, H, D, p, seed, true);
    if (st) return st;
    if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv) return IL_ERR_NULL;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const uint32_t thr = attn_threshold(p);
    const float inv_keep = (float)(1.0 / (1.0 - p));
    const int64_t smem = il::attn_bwd_smem((int)T, (int)D);
    const int t = (int)T, h = (int)H;
    const float sc = (float)scale;
    const int S = il::attn_lanes(t, il::attn_max_t((int)D));
    const int64_t nt = T * S;
#define IL_ATTN_BWD(DD, SS)                                                                                    \
    attn_launch(il::attn_bwd_kernel<DD, SS>, smem, B, nt, H, s, q, k, v, o, dout, lse, dq, dk, dv, t, h, sc, thr, \
                inv_keep, seed)
#define IL_ATTN_BWD_S(DD) (S == 4 ? IL_ATTN_BWD(DD, 4) : S == 2 ? IL_ATTN_BWD(DD, 2) : IL_ATTN_BWD(DD, 1))
    switch (D) {
        case 2: return IL_ATTN_BWD_S(2);
        case 4: return IL_ATTN_BWD_S(4);
        case 8: return IL_ATTN_BWD_S(8);
        default: return IL_ATTN_BWD_S(16);
    }
#undef IL_ATTN_BWD_S
#undef IL_ATTN_BWD
}

int il_attention_dropout_mask(uint8_t* keep, int64_t B, int64_t T, int64_t H, double p, const uint64_t* seed,
                              void* stream) {
    int st = attn_check(B, T, H, 4, p, seed, false);
    if (st) return st;
    if (!keep || !seed) return IL_ERR_NULL;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    const int64_t n = B * H * T * T;
    il::attn_mask_kernel<<<grid_for(n, 256, sms), 256, 0, (cudaStream_t)stream>>>(keep, n, (int)T,
                                                                                  attn_threshold(p), seed);
    return launch_status();
}

int64_t il_workspace_bytes(int64_t N, int64_t IN, int64_t OUT, int64_t K, int x_dtype) {
    return il::fast_backward_workspace(N, IN, OUT, K, x_dtype);
}

// Every backward kernel adds into gt and gb; il_backward zeroes them first,
// il_backward_accumulate does not.
static int backward_impl(const float* go, const void* x, int x_dtype, const float* table, void* gx, float* gt,
                         float* gb, int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw, void* workspace,
                         int64_t workspace_bytes, void* stream, bool accumulate) {
    int st = check_common(x, x_dtype, N, IN, K, bw);
    if (st) return st;
    if (OUT < 1) return IL_ERR_SHAPE;
    if (!table) return IL_ERR_NULL;
    if (N > 0 && !go) return IL_ERR_NULL;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const il::BinCfg c = make_cfg(bw, K);
    const int64_t need = il::fast_backward_workspace(N, IN, OUT, K, x_dtype);
    if (need > 0 && (!workspace || workspace_bytes < need)) return IL_ERR_WORKSPACE;
    if (!accumulate && (st = zero_pair(gt, K * IN * OUT, gb, OUT, s))) return st;
    if (N == 0) return IL_OK;
    const KernelChoice path = kernel_choice("AIWN_IL_BACKWARD", "sorted", "gather");
    if (path != kOnlyOther &&
        il::sorted_backward_ok(go, x, x_dtype, table, gx, gt, gb, N, IN, OUT, K, c)) {
        const int rc = il::sorted_backward(go, x, x_dtype, table, gx, gt, gb, N, IN, OUT, c, sms, s);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status();
        }
    }
    if (path != kOnlyPreferred && il::fast_backward_ok(go, x, x_dtype, table, gx, gt, gb, N, IN, OUT, K, c)) {
        int kernels = 0;
        const int rc = il::fast_backward(go, x, x_dtype, table, gx, gt, gb, N, IN, OUT, c, workspace, sms, s,
                                         &kernels);
        if (rc != il::kNotApplicable) {
            if (rc) {
                cudaGetLastError();
                return IL_ERR_LAUNCH;
            }
            return launch_status(kernels);
        }
    }
    if (gx) {
        const unsigned g = grid_for(N * IN, 256, sms);
        if (x_dtype == IL_BF16)
            il::dx_simple_kernel<il::kBF16><<<g, 256, 0, s>>>(go, x, table, gx, N, IN, OUT, c);
        else
            il::dx_simple_kernel<il::kF32><<<g, 256, 0, s>>>(go, x, table, gx, N, IN, OUT, c);
        if ((st = launch_status())) return st;
    }
    if (gt) {
        const unsigned g = grid_for(N * IN * OUT, 256, sms);
        if (x_dtype == IL_BF16)
            il::dtable_simple_kernel<il::kBF16><<<g, 256, 0, s>>>(go, x, gt, N, IN, OUT, c);
        else
            il::dtable_simple_kernel<il::kF32><<<g, 256, 0, s>>>(go, x, gt, N, IN, OUT, c);
        if ((st = launch_status())) return st;
    }
    if (gb) {
        const int64_t rows = 1024;
        dim3 g((unsigned)((OUT + 31) / 32), (unsigned)((N + rows - 1) / rows));
        il::dbias_simple_kernel<<<g, 256, 0, s>>>(go, gb, N, OUT, rows);
        if ((st = launch_status())) return st;
    }
    return IL_OK;
}

int il_backward(const float* go, const void* x, int x_dtype, const float* table, void* gx,
                float* gt, float* gb, int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw,
                void* workspace, int64_t workspace_bytes, void* stream) {
    return backward_impl(go, x, x_dtype, table, gx, gt, gb, N, IN, OUT, K, bw, workspace, workspace_bytes, stream,
                         false);
}

int il_backward_accumulate(const float* go, const void* x, int x_dtype, const float* table, void* gx,
                           float* gt, float* gb, int64_t N, int64_t IN, int64_t OUT, int64_t K, double bw,
                           void* workspace, int64_t workspace_bytes, void* stream) {
    return backward_impl(go, x, x_dtype, table, gx, gt, gb, N, IN, OUT, K, bw, workspace, workspace_bytes, stream,
                         true);
}

int il_bins(const void* x, int x_dtype, int64_t N, int64_t IN, int64_t K, double bw, int32_t* lo,
            int32_t* hi, float* fr, void* stream) {
    int st = check_common(x, x_dtype, N, IN, K, bw);
    if (st) return st;
    if (N == 0) return IL_OK;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    const il::BinCfg c = make_cfg(bw, K);
    const unsigned g = grid_for(N * IN, 256, sms);
    cudaStream_t s = (cudaStream_t)stream;
    if (x_dtype == IL_BF16)
        il::bins_kernel<il::kBF16><<<g, 256, 0, s>>>(x, N * IN, c, lo, hi, fr);
    else
        il::bins_kernel<il::kF32><<<g, 256, 0, s>>>(x, N * IN, c, lo, hi, fr);
    return launch_status();
}

int il_bin_counts(const void* x, int x_dtype, int64_t N, int64_t IN, int64_t K, double bw, uint64_t* counts,
                  void* stream) {
    int st = check_common(x, x_dtype, N, IN, K, bw);
    if (st) return st;
    if (K > 16384) return IL_ERR_SHAPE;  // per-CTA counters live in shared memory
    if (N == 0) return IL_OK;
    if (!counts) return IL_ERR_NULL;
    int sms = 0;
    if ((st = check_device(&sms))) return st;
    const il::BinCfg c = make_cfg(bw, K);
    const unsigned g = grid_for(N * IN, 256, sms);
    cudaStream_t s = (cudaStream_t)stream;
    const size_t smem = (size_t)K * sizeof(unsigned int);
    auto* cnt = reinterpret_cast<unsigned long long*>(counts);
    // K > 12288 counters need more than the default 48 KB of dynamic shared memory
    auto run = [&](auto kern) -> int {
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return IL_ERR_LAUNCH;
        kern<<<g, 256, smem, s>>>(x, N * IN, c, cnt);
        return launch_status();
    };
    return x_dtype == IL_BF16 ? run(il::bin_counts_kernel<il::kBF16>) : run(il::bin_counts_kernel<il::kF32>);
}

int il_adam_step(float* p, const float* g, float* m, float* v, int64_t n, double lr, double beta1,
                 double beta2, double eps, int64_t step, void* stream) {
    if (n < 0 || step < 1) return IL_ERR_SHAPE;
    if (n == 0) return IL_OK;
    if (!p || !g || !m || !v) return IL_ERR_NULL;
    int sms = 0;
    int st = check_device(&sms);
    if (st) return st;
    const double bc1 = 1.0 - pow(beta1, (double)step);
    const double bc2 = 1.0 - pow(beta2, (double)step);
    const unsigned grid = grid_for(n, 256, sms);
    il::adam_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        p, g, m, v, n, (float)beta1, (float)beta2, (float)eps, (float)(lr / bc1), (float)sqrt(bc2));
    return launch_status();
}

int64_t il_allreduce_scratch_bytes(int64_t n, int world) {
    if (n < 0 || world < 1 || world > il::kArMaxRanks) return -1;
    return il::ar_scratch_bytes(n, world);
}

int il_allreduce_sum(float* const* bufs, void* const* scratch, int64_t n, int rank, int world, double scale,
                     double timeout_s, void* stream) {
    if (world < 1 || world > il::kArMaxRanks || rank < 0 || rank >= world || n < 0) return IL_ERR_SHAPE;
    if (!(timeout_s > 0.0) || !(timeout_s <= 3600.0) || !(scale == scale)) return IL_ERR_VALUE;
    if (!bufs || !scratch) return IL_ERR_NULL;
    for (int p = 0; p < world; ++p) {
        if (!bufs[p] || !scratch[p]) return IL_ERR_NULL;
        if ((((uintptr_t)bufs[p]) | ((uintptr_t)scratch[p])) & 255) return IL_ERR_ALIGN;
    }
    if (n == 0) return IL_OK;
    int sms = 0;
    int st = check_device(&sms);
    if (st) return st;
    cudaStream_t s = (cudaStream_t)stream;
    const unsigned long long tns = (unsigned long long)(timeout_s * 1e9);
    if (n <= il::kArLLMaxElems) {
        il::ArLLArgs a;
        memset(&a, 0, sizeof(a));
        a.buf = bufs[rank];
        for (int p = 0; p < world; ++p)
            a.stage[p] = reinterpret_cast<uint2*>(static_cast<char*>(scratch[p]) + il::ar_stage_offset());
        a.ctr = static_cast<uint32_t*>(scratch[rank]) + il::kArCallWord;
        a.n = n;
        a.pairs = il::ar_ll_pairs(n, world);
        a.rank = rank;
        a.world = world;
        a.scale = (float)scale;
        a.timeout_ns = tns;
        // one warp per (32 pairs, rank) at 4 and 8 ranks, one thread per pair
        // otherwise; AIWN_IL_ALLREDUCE=warp|thread picks one (warp: 2, 4, 8 ranks)
        const char* av = getenv("AIWN_IL_ALLREDUCE");
        const bool warp = av && strcmp(av, "warp") == 0   ? il::ll_warp_ok(world)
                          : av && strcmp(av, "thread") == 0 ? false
                                                            : il::ll_warp_default(world);
        if (warp)
            il::launch_allreduce_ll_warp(a, il::ll_warp_blocks(a.pairs, world, sms), s);
        else
            il::launch_allreduce_ll(a, il::ll_blocks(a.pairs, sms), s);
        return launch_status();
    }
    il::ArArgs a;
    memset(&a, 0, sizeof(a));
    for (int p = 0; p < world; ++p) {
        a.bufs[p] = bufs[p];
        a.flags[p] = static_cast<uint32_t*>(scratch[p]);
    }
    const il::ArPlan pl = il::plan_allreduce(n, world, sms);
    a.n = n;
    a.chunk4 = pl.chunk4;
    a.rank = rank;
    a.world = world;
    a.scale = (float)scale;
    a.timeout_ns = tns;
    il::launch_allreduce(a, pl, s);
    return launch_status();
}

int il_allreduce_sum_noalloc(float* const* bufs, int64_t n, int world, double scale, void* const* streams) {
    if (world < 1 || world > kNoAllocMaxRanks || n < 0 || n > kNoAllocMaxElems) return IL_ERR_SHAPE;
    if (!(scale == scale)) return IL_ERR_VALUE;
    if (!bufs || !streams) return IL_ERR_NULL;
    for (int p = 0; p < world; ++p) {
        if (!bufs[p]) return IL_ERR_NULL;
        if ((uintptr_t)bufs[p] & 15) return IL_ERR_ALIGN;
    }
    if (n == 0) return IL_OK;
    int caller = 0, ndev = 0;
    if (cudaGetDevice(&caller) != cudaSuccess || cudaGetDeviceCount(&ndev) != cudaSuccess) {
        cudaGetLastError();
        return IL_ERR_DEVICE;
    }
    if (world > ndev) return IL_ERR_SHAPE;
    int st = noalloc_setup(world);
    // every rank's buffer is final (and the previous call's copies are done) ...
    if (st == IL_OK) st = noalloc_cross_wait(world, streams, false);
    // ... each device sums every buffer into its own scratch ...
    for (int p = 0; p < world && st == IL_OK; ++p) {
        if (cudaSetDevice(p) != cudaSuccess) {
            st = IL_ERR_DEVICE;
            break;
        }
        int sms = 0;
        if ((st = check_device(&sms))) break;
        il::NaArgs a;
        memset(&a, 0, sizeof(a));
        for (int q = 0; q < world; ++q) a.bufs[q] = bufs[q];
        a.scratch = g_noalloc[p].scratch;
        a.n = n;
        a.world = world;
        a.scale = (float)scale;
        il::allreduce_noalloc_sum_kernel<<<grid_for((n + 3) / 4, il::kArThreads, sms), il::kArThreads, 0,
                                           (cudaStream_t)streams[p]>>>(a);
        st = launch_status();
    }
    // ... and once every device has read every buffer, copies its sum in
    if (st == IL_OK) st = noalloc_cross_wait(world, streams, true);
    for (int p = 0; p < world && st == IL_OK; ++p) {
        if (cudaSetDevice(p) != cudaSuccess) {
            st = IL_ERR_DEVICE;
            break;
        }
        int sms = 0;
        if ((st = check_device(&sms))) break;
        il::allreduce_noalloc_copy_kernel<<<grid_for((n + 3) / 4, il::kArThreads, sms), il::kArThreads, 0,
                                            (cudaStream_t)streams[p]>>>(bufs[p], g_noalloc[p].scratch, n);
        st = launch_status();
    }
    cudaGetLastError();
    cudaSetDevice(caller);
    return st;
}

int64_t il_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int il_check_device_status(void* stream) {
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return IL_ERR_LAUNCH;
    unsigned int h = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&h, il::g_il_error, sizeof(h)) != cudaSuccess) return IL_ERR_LAUNCH;
    if (h) cudaMemcpyToSymbol(il::g_il_error, &zero, sizeof(zero));
    return h ? IL_ERR_TIMEOUT : IL_OK;
}

}  // extern "C"
