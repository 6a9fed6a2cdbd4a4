// rowmath.cuh -- per-element arithmetic shared by kernels that must produce
// identical bits on the compress path (many positions per chunk) and the
// decompress path (one position per chunk).
#pragma once
#include <cuda_runtime.h>

namespace boa {

// Causal depthwise conv (k = 4) + SiLU for one channel: window w0..w2 (oldest
// first) plus the current input x.  Sum order bias, oldest tap .. newest, as
// mamba_kernels.cu:158-197 / :370-412; explicit round-to-nearest operations.
__device__ __forceinline__ float conv_tap(float w0, float w1, float w2, float x, float4 k, float bias) {
  float v = bias;
  v = __fadd_rn(v, __fmul_rn(w0, k.x));
  v = __fadd_rn(v, __fmul_rn(w1, k.y));
  v = __fadd_rn(v, __fmul_rn(w2, k.z));
  v = __fadd_rn(v, __fmul_rn(x, k.w));
  return __fdividef(v, __fadd_rn(1.0f, __expf(-v)));  // v * sigmoid(v)
}

}  // namespace boa
