// rnn.cu -- LSTM / GRU gate update, one launch per token position.
//
// Replaces ker_lstm_fused_batch / ker_gru_fused_batch and the per-step
// gather / scatter of LSTMBlockGPU / GRUBlockGPU::forward_chunk
// (rnn_kernels.cu:16-161, :265-324; boa_gpu.hpp:466-501, :567-582).  The
// input projection ih = x W_ih^T + b_ih is one GEMM over all rows of the tile;
// the recurrent projection hh = h W_hh^T + b_hh is a GEMM with one row per
// chunk, run once per position; this kernel then reads row (b, t) of ih in
// place (no gather), updates the state, writes the output row (no scatter)
// and re-splits h into the bf16 hi/lo planes that the next position's
// recurrent GEMM reads through TMA.  Compress and decompress run the same
// kernels per position, so their logits agree bit for bit.
#include "kernels.cuh"
#include "ptx.cuh"

namespace boa {

// repro_sigmoid / repro_tanh (activations.hpp:87-127, GPU branch), with
// CUDA's expf; every product and sum is rounded on its own as in the
// reference build (--fmad=false).
__device__ __forceinline__ float rnn_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float rnn_tanh(float x) {
  if (fabsf(x) > 10.0f) return x > 0.0f ? 1.0f : -1.0f;
  const float e2x = expf(__fmul_rn(2.0f, x));
  return __fdiv_rn(__fadd_rn(e2x, -1.0f), __fadd_rn(e2x, 1.0f));
}

// One thread per (chunk b, four channels).  Gate blocks follow PyTorch's
// order: LSTM [i | f | g | o], GRU [r | z | n], each d wide.
template <bool LSTM>
__global__ void __launch_bounds__(256) rnn_gates_kernel(const float* __restrict__ ih, const float* __restrict__ hh,
                                                         int d, int t, int T, float* __restrict__ hs,
                                                         float* __restrict__ cs, __nv_bfloat16* __restrict__ hl,
                                                         long long hl_plane, float* __restrict__ xo, int B) {
  const int q = d >> 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)B * q) return;
  const int b = (int)(idx / q), j = (int)(idx - (long long)b * q) * 4;
  constexpr int NG = LSTM ? 4 : 3;
  const size_t row = (size_t)b * T + t;
  const float* a = ih + row * NG * d + j;
  const float* r = hh + (size_t)b * NG * d + j;
  float4 ga[NG], gr[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    ga[g] = *reinterpret_cast<const float4*>(a + (size_t)g * d);
    gr[g] = *reinterpret_cast<const float4*>(r + (size_t)g * d);
  }
  const size_t so = (size_t)b * d + j;
  const float4 h4 = *reinterpret_cast<const float4*>(hs + so);
  float hv[4] = {h4.x, h4.y, h4.z, h4.w};
  float cv[4] = {0.f, 0.f, 0.f, 0.f};
  if (LSTM) {
    const float4 c4 = *reinterpret_cast<const float4*>(cs + so);
    cv[0] = c4.x; cv[1] = c4.y; cv[2] = c4.z; cv[3] = c4.w;
  }
  auto el = [](const float4& v, int k) { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; };
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (LSTM) {
      const float iv = rnn_sigmoid(__fadd_rn(el(ga[0], k), el(gr[0], k)));
      const float fv = rnn_sigmoid(__fadd_rn(el(ga[1], k), el(gr[1], k)));
      const float gv = rnn_tanh(__fadd_rn(el(ga[2], k), el(gr[2], k)));
      const float ov = rnn_sigmoid(__fadd_rn(el(ga[3], k), el(gr[3], k)));
      cv[k] = __fadd_rn(__fmul_rn(fv, cv[k]), __fmul_rn(iv, gv));
      hv[k] = __fmul_rn(ov, rnn_tanh(cv[k]));
    } else {
      const float rv = rnn_sigmoid(__fadd_rn(el(ga[0], k), el(gr[0], k)));
      const float zv = rnn_sigmoid(__fadd_rn(el(ga[1], k), el(gr[1], k)));
      const float nv = rnn_tanh(__fadd_rn(el(ga[2], k), __fmul_rn(rv, el(gr[2], k))));
      hv[k] = __fadd_rn(__fmul_rn(__fadd_rn(1.0f, -zv), nv), __fmul_rn(zv, hv[k]));
    }
  }
  const float4 hn = make_float4(hv[0], hv[1], hv[2], hv[3]);
  *reinterpret_cast<float4*>(hs + so) = hn;
  *reinterpret_cast<float4*>(xo + row * d + j) = hn;
  if (LSTM) *reinterpret_cast<float4*>(cs + so) = make_float4(cv[0], cv[1], cv[2], cv[3]);
  __nv_bfloat16 hi[4], lo[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) split_bf16(hv[k], hi[k], lo[k]);
  *reinterpret_cast<uint2*>(hl + so) = *reinterpret_cast<const uint2*>(hi);
  *reinterpret_cast<uint2*>(hl + hl_plane + so) = *reinterpret_cast<const uint2*>(lo);
}

cudaError_t launch_rnn_gates(bool lstm, const float* ih, const float* hh, int d, int t, int T, float* hs, float* cs,
                             __nv_bfloat16* hl, long long hl_plane, float* xo, int B, cudaStream_t st) {
  if (d % 4 != 0 || t < 0 || t >= T || (lstm && !cs)) return cudaErrorInvalidValue;
  const long long n = (long long)B * (d / 4);
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (lstm) rnn_gates_kernel<true><<<grid, 256, 0, st>>>(ih, hh, d, t, T, hs, cs, hl, hl_plane, xo, B);
  else rnn_gates_kernel<false><<<grid, 256, 0, st>>>(ih, hh, d, t, T, hs, cs, hl, hl_plane, xo, B);
  return cudaGetLastError();
}

}  // namespace boa
