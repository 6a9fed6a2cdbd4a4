// gemm.cuh -- declarations for the tcgen05 GEMM and its fused epilogues.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include "coder.cuh"

namespace boa {

// Epilogue selector.  Every GEMM computes ACC[M,N] = A[M,K] * W[N,K]^T in
// fp32 from bf16 hi/lo planes (A = Ah + Al, W = Wh + Wl;
// ACC = Ah*Wh + Ah*Wl + Al*Wh), then one of:
enum EpiMode : int {
  EPI_F32 = 0,         // out_f32 = ACC (+ bias)                      in_proj, x_proj
  EPI_ACT_SPLIT = 1,   // out_hl  = split(act(ACC + bias))            FF1 (GELU), head1 (ReLU)
  EPI_LN_SPLIT = 2,    // out_hl  = split(LN(ACC + bias))             out_proj -> LN2
  EPI_RES_LN = 3,      // x = ACC + bias + x; out_hl = split(LN(x))   FF2 (+ next LN1)
  EPI_LOGITS = 4,      // out_f32 = ACC + bias                        head2, test path
  EPI_HEAD_ENC = 5,    // (low, high) of the next byte per row       head2, compress
  EPI_HEAD_DEC = 6,    // range-decode one byte per row (= chunk)    head2, decompress
};
enum Act : int { ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2, ACT_SILU = 3 };

struct GemmArgs {
  int M, N, K;
  const float* bias;
  float* out_f32;
  int ld_f32;
  __nv_bfloat16* out_hl;  // [2][M][ld_hl] (hi plane, then lo plane)
  int ld_hl;
  long long plane_hl;     // elements between the hi and lo planes
  float* res;             // EPI_RES_LN: residual in, updated x out ([M][N])
  const float* ln_w;      // LN weight/bias; nullptr -> plain split
  const float* ln_b;
  int act;
  // LM-head coder (EPI_HEAD_ENC / EPI_HEAD_DEC)
  float inv_t;
  const uint8_t* tokens;  // compress: input bytes of this batch (chunk b at b*chunk_len)
  uint8_t* out_bytes;     // decompress: output bytes of this batch
  long long n_bytes;      // bytes from the batch's first chunk to the stream end
  int chunk_len;
  int t0, T;              // compress tile: rows are (b, tau), position t0 + tau
  uint2* lf;              // compress: [M] (low, high) per row
  long long stride;       // compress: bytes between lanes' chunks (0 = chunk_len)
  const int* d_t;         // decompress: device step counter
  const long long* lane_base;  // decompress: each lane's chunk offset in out_bytes
  const int* lane_len;         // decompress: each lane's chunk length
  DecState* dstates;      // decompress: one decoder per chunk
  const uint32_t* payload;
  const unsigned long long* offsets;  // word offset of each lane's stream
};

struct PlaneMap;  // opaque TMA descriptor holder (host)

// Launch C = epilogue(A * W^T).  A and W are bf16 hi/lo plane pairs with K
// contiguous.  a_plane / w_plane: elements between hi and lo planes.
// BN (CTA tile width) is 256 unless N is small (x_proj: 48).
cudaError_t gemm_prepare_device();

// The block's feed-forward in one kernel (d_model 64, 128 or 256): with
// a.N = d, x = a.res [M][d] and xn = the LN2 output (hi/lo planes [2][M][d],
// xn_plane elements apart), x += W2 . GELU(W1 . xn + b1) + a.bias and then
// a.out_hl = split(LN(x; a.ln_w, a.ln_b)) (a plain split when a.ln_w is null).
// W1 [2][4d][d], W2 [2][d][4d] (bf16 hi/lo planes).
cudaError_t mlp_launch(const __nv_bfloat16* xn, long long xn_plane, const __nv_bfloat16* w1, long long w1_plane,
                       const __nv_bfloat16* w2, long long w2_plane, const float* b1, const GemmArgs& a,
                       cudaStream_t stream);
cudaError_t mlp_prepare_device();
cudaError_t gemm_launch(int mode, const __nv_bfloat16* A, long long a_plane, int lda_rows,
                        const __nv_bfloat16* W, long long w_plane, const GemmArgs& args,
                        cudaStream_t stream);

}  // namespace boa
