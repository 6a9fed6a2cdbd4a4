/*
 * boa_oracle.h -- CPU restatement of BoaConstrictor's compress/decompress path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the B200 product
 * (libboa_b200.so).  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg may load it.  The product never calls it.
 *
 * Every function restates a piece of the reference (AkarshSahlot/boa-constrictor,
 * paths relative to the project root):
 *   model math   portability_solved_cpp/boa_gpu.hpp, mamba_kernels.cu,
 *                inference_kernels.cu, gemm_kernels.cu, rnn_kernels.cu
 *   CDF quantiser portability_solved_cpp/range_coder_kernels.cu:860-925
 *   range coder  portability_solved_cpp/range_coder_kernels.cu:46-60, 279-335,
 *                725-780, 916-968
 * The integer coder is restated exactly (bit-exact).  Model math is fp32 in the
 * reference's operation order but uses the C library's exp/log/tanh in place of
 * CUDA's, so logits agree to a tolerance, not bit for bit.
 */
#ifndef BOA_ORACLE_H
#define BOA_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* backbone codes follow gemm_gpu.hpp:18-33 (mamba=0, lstm=1, gru=2, mingru=3) */
void* orc_load(const char* path, int backbone, int d_model, int n_layers);
void  orc_free(void* model);
const char* orc_last_error(void);

/* Logits for B independent chunks of L tokens each, fresh state per chunk.
 * tokens [B][L] bytes; logits [B][L][256] (head bias included).
 * mode 0 = chunk form (BoaPredictorGPU::forward_chunk, boa_gpu.hpp:1081-1102),
 * mode 1 = step form (BoaPredictorGPU::step_batch, boa_gpu.hpp:1034-1053). */
int orc_logits(void* model, const uint8_t* tokens, int B, int L, int mode, float* logits);

/* Integer CDF of one logits row, range_coder_kernels.cu:860-925.
 * Q has 257 entries; Q[256] = 2^24. */
void orc_cdf_row(const float* logits_row, float inv_temperature, uint32_t* Q);
void orc_cdf_rows(const float* logits, int rows, float inv_temperature, uint32_t* Q);

/* Range coder on explicit integer CDFs (one stream).
 * Q [n][257]; returns the number of 32-bit words written (<= cap) or -1. */
int orc_rc_encode_cdf(const uint32_t* Q, const uint8_t* syms, int n, uint32_t* out, int cap);
int orc_rc_decode_cdf(const uint32_t* Q, int n, const uint32_t* words, int n_words, uint8_t* syms);

/* The Python codec's coder (gpu_range_coder.py): fp32 probability rows are
 * quantised by build_cdf_fast (gpu_range_coder.py:57-79) into K+1 integer
 * CDF entries, then range-coded by encode_kernel / finalize_kernel /
 * decode_step_kernel (:81-215).  probs [n][K], one stream; symbols outside
 * [0, K) are skipped by the encoder, as in the reference.  encode returns the
 * number of words (<= cap) or -1. */
void orc_pyrc_cdf_rows(const float* probs, int rows, int K, uint32_t* cdf);
int orc_pyrc_encode(const float* probs, const int32_t* syms, int n, int K, uint32_t* out, int cap);
int orc_pyrc_decode(const float* probs, int n, int K, const uint32_t* words, int n_words, int32_t* syms);

/* Chunk-parallel codec on host threads.  Chunk i covers
 * data[i*chunk_len, min(n, (i+1)*chunk_len)).  Streams are written at
 * stream_words + i*pitch_words; sizes_words[i] = words used.
 * Returns 0 on success. */
int orc_compress(void* model, const uint8_t* data, size_t n, uint32_t chunk_len,
                 float inv_temperature, int n_threads,
                 uint8_t* first_bytes, uint32_t* stream_words, uint32_t pitch_words,
                 uint32_t* sizes_words);
/* Inverse.  out has room for the whole stream (n bytes); chunk i writes
 * out[i*chunk_len ...] with its chunk length. */
int orc_decompress(void* model, const uint32_t* stream_words, uint32_t pitch_words,
                   const uint32_t* sizes_words, const uint8_t* first_bytes,
                   size_t n, uint32_t chunk_len, float inv_temperature, int n_threads,
                   uint8_t* out);

/* Warm start: W lanes, lane b codes chunks b*S .. b*S+S-1 with carried state. */
int orc_compress_warm(void* model, const uint8_t* data, size_t n, uint32_t chunk_len, uint32_t W,
                      float inv_temperature, int n_threads, uint8_t* first_bytes, uint32_t* stream_words,
                      uint32_t pitch_words, uint32_t* sizes_words);
int orc_decompress_warm(void* model, const uint32_t* stream_words, uint32_t pitch_words,
                        const uint32_t* sizes_words, const uint8_t* first_bytes, size_t n, uint32_t chunk_len,
                        uint32_t W, float inv_temperature, int n_threads, uint8_t* out);

#ifdef __cplusplus
}
#endif
#endif
