// kernels.cuh -- launchers for the non-GEMM kernels of the compress/decompress
// path (embedding + LayerNorm, causal conv, selective scan, range-coder
// bookkeeping, integer-CDF coder).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include "coder.cuh"

namespace boa {

// Where each row's input token comes from.
struct TokenSrc {
  int mode;               // 0: tokens[row]; 1: compress tile; 2: decompress step
  const uint8_t* bytes;   // mode 0: [M]; mode 1: lane 0's chunk; mode 2: output stream
  long long n_bytes;      // mode 1: bytes from lane 0's chunk to the stream end
  int chunk_len, t0, T;   // mode 1
  const int* d_t;         // mode 2: current step; the token is byte t-1
  long long stride;       // mode 1: bytes between consecutive lanes' chunks (0 = chunk_len;
                          //         S * chunk_len for interleaved warm-start lanes)
  const long long* lane_base;  // mode 2: byte offset of each lane's chunk in `bytes`
  const int* lane_len;         // mode 2: length of each lane's chunk
  // Input position of the first row since the recurrent state was reset:
  // pos0 + (d_pos ? *d_pos : 0).  Only its value mod 3 is used (the conv
  // state is a three-slot ring indexed by position).
  long long pos0;
  const int* d_pos;
};

// x[row] = E[token]; xn = split(LN(x; w, b))   (rows = M, width d)
cudaError_t launch_embed_ln(const TokenSrc& src, const float* emb, int d, float* x, __nv_bfloat16* xn,
                            long long xn_plane, const float* ln_w, const float* ln_b, int M,
                            cudaStream_t st);

// u = silu(causal_conv4(x)) as bf16 hi / lo planes (uhl), x = xz[:, :di]; rows (b, tau) with T rows per
// chunk, row tau being input position p0 + tau (p0 = pos0 + *d_pos).
// conv_state [B][3][di] is a ring holding the three previous inputs: slot
// p % 3 holds the input at position p.
cudaError_t launch_conv(const float* xz, int di, float* conv_state, const float* conv_w, const float* conv_b,
                        __nv_bfloat16* uhl, long long plane, int B, int T, long long pos0,
                        const int* d_pos, cudaStream_t st);

// selective scan with fused dt_proj + softplus + D skip + SiLU(z) gate.
// delta [M][ld_delta] = [dt_in(r) | B(16) | C(16)]; ssm_state [B][16][di];
// negA holds -exp(A_log) * log2(e) per (channel, state).  u comes as the
// conv's bf16 hi / lo planes (used as hi + lo); y * silu(z) leaves as hi / lo
// planes in yhl, a different buffer with the same plane stride.
cudaError_t launch_scan(const float* delta, int ld_delta, int r, const float* dt_w, const float* dt_b,
                        const float* negA, const float* Dv, const float* xz, int di,
                        float* ssm_state, const __nv_bfloat16* uhl, __nv_bfloat16* yhl, long long plane, int B, int T,
                        cudaStream_t st);

cudaError_t scan_prepare_device();
// one bounded mbarrier wait that runs out (failure-detection self-test)
cudaError_t launch_wait_selftest(uint64_t limit_ns, int* ok);

// minGRU recurrence: h = (1-z) h + z g(ht) over T rows per chunk; writes h
// into x_out rows (boa_gpu.hpp:652-693).  zh = [M][2d] (z logits | h~ raw).
cudaError_t launch_mingru(const float* zh, int d, float* h_state, float* x_out, int B, int T, cudaStream_t st);

// LSTM / GRU gate update for position t of a T-position tile: reads
// ih [B*T][G] row b*T+t and hh [B][G] (G = 4d LSTM, 3d GRU), updates h_state
// (and c_state for LSTM) [B][d], writes h to x_out row b*T+t and its bf16
// hi/lo split to hl [2][B][d] (plane elements apart).
cudaError_t launch_rnn_gates(bool lstm, const float* ih, const float* hh, int d, int t, int T, float* h_state,
                             float* c_state, __nv_bfloat16* hl, long long hl_plane, float* x_out, int B,
                             cudaStream_t st);

// x += y (residual), then xn = split(LN(x)) -- minGRU blocks
cudaError_t launch_add_ln(float* x, const float* y, int d, __nv_bfloat16* xn, long long plane,
                          const float* ln_w, const float* ln_b, int M, cudaStream_t st);
// final RMSNorm then split (minGRU head input)
cudaError_t launch_rms_split(const float* x, int d, const float* w, __nv_bfloat16* xn, long long plane, int M,
                             cudaStream_t st);

// compress: encode one tile of (low, high) per lane; lf [B][T]; lane b's
// chunk starts b * stride bytes after lane 0's
cudaError_t launch_encode_tile(const uint2* lf, EncState* es, uint32_t* pitch_buf, int pitch_words, int B,
                               int T, int t0, long long n_bytes, int chunk_len, long long stride, cudaStream_t st);
cudaError_t launch_enc_init(EncState* es, int B, cudaStream_t st);
// failed streams get size failed_size; report = also set the device error word
cudaError_t launch_enc_finish(EncState* es, uint32_t* pitch_buf, int pitch_words, uint32_t* sizes, int B,
                              cudaStream_t st, uint32_t failed_size = 0u, bool report = true);
// exclusive scan of sizes -> offsets (one block), continuing from offsets[0];
// total in offsets[B]
cudaError_t launch_offsets(const uint32_t* sizes, unsigned long long* offsets, int B, cudaStream_t st);
cudaError_t launch_compact(const uint32_t* pitch_buf, int pitch_words, const uint32_t* sizes,
                           const unsigned long long* offsets, uint32_t* payload, int B, cudaStream_t st);
cudaError_t launch_first_bytes(const uint8_t* data, long long n_bytes, int chunk_len, long long stride, uint8_t* first,
                               int B, cudaStream_t st);
// compress, interleaved lanes: lane b's results -> chunk c = iter + b * S
// (sizes, first bytes, and its stream copied into per-chunk slots)
cudaError_t launch_lanes_scatter(const uint32_t* pitch_buf, int pitch_words, const uint32_t* lane_sizes,
                                 const uint8_t* lane_first, uint32_t* slots, uint32_t* sizes, uint8_t* first, int iter,
                                 int S, int B, cudaStream_t st);
// decompress: per-lane view of chunks c = c0 + b * S (stream offset, size,
// first byte, output offset and length)
cudaError_t launch_lanes_gather(const unsigned long long* offsets, const uint32_t* sizes, const uint8_t* first,
                                long long n_bytes, int chunk_len, int c0, int S, int B, unsigned long long* lane_off,
                                uint32_t* lane_size, uint8_t* lane_first, long long* lane_base, int* lane_len,
                                cudaStream_t st);
cudaError_t launch_dec_init(DecState* ds, const uint32_t* payload, const unsigned long long* lane_off,
                            const uint32_t* lane_size, const uint8_t* lane_first, uint8_t* out,
                            const long long* lane_base, const int* lane_len, int B, cudaStream_t st);
cudaError_t launch_set_counter(int* d_t, int value, cudaStream_t st);
// d_t[0] += 1 and d_t[1] += 1 (decode step and input position)
cudaError_t launch_increment(int* d_t, cudaStream_t st);

// integer-CDF coder (configs[1] style): cdf [n_steps][n_streams][257]
cudaError_t launch_rc_encode_cdf(EncState* es, const uint32_t* cdf, const uint8_t* syms, int n_streams,
                                 int n_steps, uint32_t* pitch_buf, int pitch_words, cudaStream_t st,
                                 bool report = true);
cudaError_t launch_rc_decode_init(DecState* ds, const uint32_t* payload, const unsigned long long* offsets,
                                  const uint32_t* sizes, int n_streams, cudaStream_t st);
cudaError_t launch_rc_decode_cdf(DecState* ds, const uint32_t* cdf, const uint32_t* payload,
                                 const unsigned long long* offsets, int n_streams, int n_steps, uint8_t* syms,
                                 cudaStream_t st);
// CDF of logits rows (test hook for the shared CDF code): Q [rows][257]
cudaError_t launch_cdf_rows(const float* logits, int rows, float inv_t, uint32_t* Q, cudaStream_t st);

}  // namespace boa
