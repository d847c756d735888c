// Tensor-core GEMV path (placeholder until the mma kernels land): nothing is routed here yet.
#pragma once
#include "kernels.cuh"

namespace xjk {
constexpr int MMA_MAXT = 0;
inline bool mma_supported(const DevMat &) { return false; }
inline void launch_gemv_mma(const GemvJob &, const float *, long long, int, cudaStream_t) {}
}  // namespace xjk
