// il_fast.cuh -- shape-specialised IndexedLinear kernels (placeholder).
#pragma once
#include "il_common.cuh"

namespace il {

inline bool fast_forward_ok(const void*, int, const float*, const float*, const float*, int64_t,
                            int64_t, int64_t, int64_t) {
    return false;
}
inline int fast_forward(const void*, int, const float*, const float*, float*, int64_t, int64_t,
                        int64_t, const BinCfg&, int, cudaStream_t) {
    return 0;
}
inline int64_t fast_backward_workspace(int64_t, int64_t, int64_t, int64_t, int) { return 0; }
inline bool fast_backward_ok(const float*, const void*, int, const float*, const void*,
                             const float*, const float*, int64_t, int64_t, int64_t, int64_t) {
    return false;
}
inline int fast_backward(const float*, const void*, int, const float*, void*, float*, float*,
                         int64_t, int64_t, int64_t, const BinCfg&, void*, int, cudaStream_t) {
    return 0;
}

}  // namespace il
