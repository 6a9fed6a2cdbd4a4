/*
 * boa_b200.h -- C ABI of the B200-native BoaConstrictor compress/decompress
 * library (libboa_b200.so).
 *
 * The reference (AkarshSahlot/boa-constrictor, portability_solved_cpp/) has no
 * C ABI: its operator surface is C++ free functions on raw device pointers with
 * a global stream and exit(1) on error (gemm_gpu.hpp:68-79, :124-265), driven
 * by BoaPredictorGPU (boa_gpu.hpp:944-1174) and the CLI loops compress_v2 /
 * decompress_v2 (boa.cpp:280-582, :584-817).  Each entry point below names the
 * reference interface it replaces.  Conventions:
 *   - every call returns 0 on success or a negative BOA_E_* code; the message
 *     is available from boa_last_error();
 *   - host pointers are caller-owned; device memory is owned by the handle;
 *   - one handle drives one GPU; distinct handles may be used concurrently
 *     from distinct host threads; a single handle is not re-entrant.
 */
#ifndef BOA_B200_H
#define BOA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BOA_OK 0
#define BOA_E_INVALID (-1)   /* bad argument */
#define BOA_E_CUDA (-2)      /* CUDA runtime error (no GPU, launch failure, ...) */
#define BOA_E_IO (-3)        /* file not readable / writable */
#define BOA_E_FORMAT (-4)    /* weight file or container malformed */
#define BOA_E_DEVICE (-5)    /* device-side check failed (wait timeout, stream overflow) */
#define BOA_E_NOMEM (-6)     /* device allocation failed */

/* Size written by the handle-free encoders (boa_rc_encoder_finish,
 * boa_rc_encode_cdf_noalloc) for a stream whose coding stopped: a coded
 * symbol had an empty interval or one above 2^24, or the stream outgrew its
 * pitch.  Such a stream's words are not a decodable stream. */
#define BOA_STREAM_FAILED 0xFFFFFFFFu

#define BOA_BACKBONE_MAMBA 0 /* gemm_gpu.hpp BackboneType: mamba (mambav1 blocks) */
#define BOA_BACKBONE_LSTM 1   /* LSTMBlockGPU (boa_gpu.hpp:365-502) */
#define BOA_BACKBONE_GRU 2    /* GRUBlockGPU (boa_gpu.hpp:504-600) */
#define BOA_BACKBONE_MINGRU 3 /* MinGRUBlockGPU (boa_gpu.hpp:605-694) */

typedef struct boa_model boa_model;

/* ---- model --------------------------------------------------------------
 * Replaces MambaConfig (gemm_gpu.hpp:38-66), the BoaPredictorGPU constructor
 * and load_weights (boa_gpu.hpp:945-1029).  Reads the .bin layout of
 * convert_boa_weights.py:153-241 ("BOA\0" fp32 or "BOA\1" fp16 header, or a
 * headerless legacy fp32 file); d_model and n_layers are not stored in the
 * file and must be given, as on the reference CLI (boa.cpp:912-919).  The
 * file size must match the dims exactly (BOA_E_FORMAT otherwise).  d_model
 * is one of 64, 80, 128, 160, 256, 512 (the widths of the reference's
 * checkpoints and configs; LSTM / GRU: 64, 128, 256, 512).  An odd dt_rank
 * (ceil(d_model / 16): 5 at 80, 10 at 160) is zero-padded to 8 / 16 on load:
 * the padded terms add exact zeros to the dt projection. */
int boa_model_load(const char* weights_path, int backbone, int d_model, int n_layers, int device,
                   boa_model** out);
/* Every call on a handle runs on the handle's device and leaves the calling
 * thread's current CUDA device as it found it. */
/* Releases the handle and all its device memory (the reference never frees). */
void boa_model_free(boa_model* h);
/* Message of the last failed call on this handle (or of the last failed
 * boa_model_load when h is NULL). */
const char* boa_last_error(const boa_model* h);
/* Replaces gpu_set_temperature (range_coder_kernels.cu:9-12): logits are
 * scaled by 1/T (computed in fp32) before the softmax. */
int boa_set_temperature(boa_model* h, float temperature);
/* Replaces the global g_stream (utility_kernels.cu:5): after this call, work
 * of the handle is ordered after prior work on `cuda_stream` and later work
 * on `cuda_stream` waits for it.  NULL names the legacy default stream (it is
 * an external stream like any other).  Without this call the handle runs on
 * its private stream and callers use boa_sync(). */
int boa_set_stream(boa_model* h, void* cuda_stream);
/* Chunks per batch (--gpu-batch, boa.cpp:310) and tokens per compress tile
 * (--tile, boa.cpp:313-316).  0 = automatic from free device memory
 * (auto_size_params, boa.cpp:109-156). */
int boa_set_batch(boa_model* h, int chunks_per_batch, int tile_tokens);
/* The batch the next compress (compress != 0) or decompress call over
 * n_chunks chunks of chunk_len bytes would run: chunks per batch and positions
 * per compress tile (1 for decompress), as auto_size_params (boa.cpp:109-156)
 * reports them before a run.  Allocates nothing. */
int boa_batch_geometry(boa_model* h, uint32_t n_chunks, uint32_t chunk_len, int compress, int* chunks_per_batch,
                       int* tile_tokens);
/* Allocates now what compress / decompress calls over n_chunks chunks of up
 * to chunk_len bytes will need (work buffers for the batch the call would
 * pick, and the staging of the host-buffer calls), so that those calls
 * allocate nothing: the role of BoaPredictorGPU::allocate_chunk
 * (boa_gpu.hpp:268-300), called before the timed loops.  Buffers only grow;
 * a later call with a larger geometry still allocates. */
int boa_reserve(boa_model* h, uint32_t n_chunks, uint32_t chunk_len);
/* --warm-start (boa.cpp:313-319, :395-435, :608-610): with interleave_batch
 * W > 0 the codec runs W lanes; lane b codes chunks b*S, b*S+1, ... with
 * S = ceil(n_chunks / W), carrying the model state from chunk to chunk (each
 * chunk still has its own range coder and raw first byte).  A container made
 * this way records flags bit0 and W; decode it with the same W.  0 = off. */
int boa_set_warm_start(boa_model* h, uint32_t interleave_batch);
/* Per-chunk stream capacity in 32-bit words used on the device for a chunk
 * length (a tight bound: <= 24.01 bits per byte plus the flush words). */
uint32_t boa_stream_capacity_words(uint32_t chunk_len);

/* ---- host-buffer codec (the body of compress_v2 / decompress_v2) --------
 * Chunk i of the stream covers data[i*chunk_len, min(n, (i+1)*chunk_len)).
 * Compress chunks [first_chunk, first_chunk + n_chunks): writes the raw first
 * byte of each chunk, each chunk's range-coded words concatenated in chunk
 * order into payload (the BOA2 payload, boa.cpp:561-569) and the word count
 * of each chunk into sizes_words.  *payload_words_out = total words.
 * Returns BOA_E_INVALID if payload_cap_words is too small (nothing written). */
int boa_compress_chunks(boa_model* h, const uint8_t* data, size_t n, uint32_t chunk_len, uint32_t first_chunk,
                        uint32_t n_chunks, uint8_t* first_bytes, uint32_t* payload, size_t payload_cap_words,
                        uint32_t* sizes_words, uint64_t* payload_words_out);
/* Inverse: payload holds the n_chunks streams back to back with word counts
 * sizes_words; chunk j (0-based within the call) decodes chunk_lens[j] bytes
 * into out + j*chunk_len.  Replaces the decode loop of boa.cpp:672-774. */
int boa_decompress_chunks(boa_model* h, const uint32_t* payload, const uint32_t* sizes_words,
                          const uint8_t* first_bytes, const uint32_t* chunk_lens, uint32_t chunk_len,
                          uint32_t n_chunks, uint8_t* out);

/* ---- device-buffer codec (inputs already resident in HBM) ---------------
 * Same as above on device pointers, enqueued asynchronously on the handle's
 * stream.  n_bytes counts the bytes from chunk 0 of this call to the end of
 * the stream, so chunk j has min(chunk_len, n_bytes - j*chunk_len) bytes.
 * d_offsets has n_chunks + 1 entries (exclusive prefix of sizes; last =
 * total).  Check boa_sync() before reading results. */
int boa_compress_device(boa_model* h, const uint8_t* d_data, uint64_t n_bytes, uint32_t chunk_len,
                        uint32_t n_chunks, uint8_t* d_first_bytes, uint32_t* d_payload, uint64_t payload_cap_words,
                        uint32_t* d_sizes_words, uint64_t* d_offsets);
int boa_decompress_device(boa_model* h, const uint32_t* d_payload, const uint64_t* d_offsets,
                          const uint32_t* d_sizes_words, const uint8_t* d_first_bytes, uint64_t n_bytes,
                          uint32_t chunk_len, uint32_t n_chunks, uint8_t* d_out);
/* Waits for the handle's work and reports device-side failures
 * (BOA_E_DEVICE).  Kernels record such a failure -- a bounded wait that ran
 * out, a stream longer than its capacity -- in one error word per device,
 * which this call reads and clears: with several handles on one device, a
 * failure is reported to whichever handle synchronises first. */
int boa_sync(boa_model* h);
/* Failure-detection self-test (no counterpart in the reference): one kernel
 * on `device` waits on a barrier that nothing signals, with the bounded wait
 * every kernel of this library uses, cut to limit_us microseconds (1 .. 1e6).
 * The wait gives up, records the timeout in the device's error word and the
 * kernel returns, so the context stays usable.  Returns BOA_E_DEVICE with
 * boa_last_error(NULL) = "device wait timed out" when that happened (the
 * expected outcome; the error word is cleared), BOA_E_INVALID for a bad
 * device or limit, BOA_E_CUDA otherwise. */
int boa_selftest_wait_timeout(int device, uint32_t limit_us);
/* Device memory the handle holds (weights + work buffers + states). */
uint64_t boa_device_bytes(const boa_model* h);

/* ---- instrumentation (the reference's --show-timings, boa.cpp:376-506) ---
 * With profiling on, every kernel launch of the handle is bracketed by CUDA
 * events on the stream it runs on and the decompress step runs without graph
 * capture; boa_profile_read() synchronises and reports, per kernel class,
 * the summed device time and the number of launches since the last read.
 * boa_launch_count() counts every kernel the handle has launched (graph
 * replays included), profiling or not. */
#define BOA_PROF_CLASSES 12
int boa_set_profiling(boa_model* h, int on);
int boa_profile_read(boa_model* h, int kernel_class, double* total_ms, uint64_t* launches);
const char* boa_profile_name(int kernel_class);
uint64_t boa_launch_count(const boa_model* h);

/* ---- model outputs for parity testing ------------------------------------
 * Logits [B][L][256] (head bias included) of B fresh chunks of L tokens.
 * mode 0 runs the compress form (tiles of up to 64 positions per launch
 * with the state carried between them, as compress does and as
 * BoaPredictorGPU::forward_chunk with --tile, boa_gpu.hpp:1081-1102); any L is
 * accepted.  mode 1 runs the
 * decompress form (L single-position steps, as step_batch,
 * boa_gpu.hpp:1034-1053).  Host buffers. */
int boa_model_logits(boa_model* h, const uint8_t* tokens, int B, int L, int mode, float* logits);

/* ---- range coder on explicit integer CDFs --------------------------------
 * CDFs Q[n_steps][n_streams][257] (Q[s] = cumulative frequency of symbols
 * below s, Q[256] = 2^24, strictly increasing), symbols [n_steps][n_streams].
 * The encoder checks the interval of every coded symbol (Q[s] < Q[s+1] <=
 * 2^24) and returns BOA_E_DEVICE for one that is empty or out of range,
 * where the reference would silently write an undecodable stream.
 * Replaces the coder of ker_rc_encode_chunk_parallel_warp / ker_rc_finish /
 * ker_rc_init_decoder / ker_rc_decode_fused_step_warp
 * (range_coder_kernels.cu:46-60, :279-335, :725-780, :916-968) for callers
 * that supply the CDF.  Host buffers; streams are returned back to back like
 * a BOA2 payload. */
int boa_rc_encode_cdf(boa_model* h, const uint32_t* cdf, const uint8_t* syms, int n_streams, int n_steps,
                      uint32_t* payload, size_t payload_cap_words, uint32_t* sizes_words);
int boa_rc_decode_cdf(boa_model* h, const uint32_t* cdf, int n_streams, int n_steps, const uint32_t* payload,
                      const uint32_t* sizes_words, uint8_t* syms);
/* The encoder above without any allocation, for callers that cannot allocate
 * device memory where they encode (a pooled or framework-owned allocator that
 * forbids raw cudaMalloc, a plugin that must keep its memory footprint fixed).
 * No counterpart in the reference.  All pointers are device pointers: the
 * same cdf/syms layout as boa_rc_encode_cdf; stream i is written to
 * d_words + i*pitch_words (pitch_words >= boa_stream_capacity_words(n_steps+1))
 * and its word count to d_sizes[i].  The per-stream coder states live in one
 * static device array of 65536 x 32 bytes (2 MiB), held by every GPU that
 * loads the library until exit; n_streams above 65536 is rejected.  Work is
 * enqueued on `stream` (NULL = legacy default stream), which must belong to
 * the current device (BOA_E_INVALID otherwise), and nothing is synchronised.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress), so make it before any stream capture; the
 * address is kept for the life of the process, so do not call this after a
 * cudaDeviceReset of that device.
 * Every call shares the array and resets the states it uses: calls that
 * overlap on the GPU race.  Argument and launch errors are returned (message
 * in boa_last_error(NULL)).  A stream whose coding stopped on the device (an
 * empty or out-of-range CDF interval, a full pitch) gets d_sizes[i] =
 * BOA_STREAM_FAILED; the other streams are unaffected, and no model handle's
 * error state is touched. */
int boa_rc_encode_cdf_noalloc(const uint32_t* d_cdf, const uint8_t* d_syms, int n_streams, int n_steps,
                              uint32_t* d_words, uint32_t pitch_words, uint32_t* d_sizes, void* stream);
/* ---- the same coder, step-wise on caller-owned device state ---------------
 * Replace gpu_rc_init (range_coder_kernels.cu:46-60), the per-position
 * encode launches (:234-275), gpu_rc_finish_batch (:279-317),
 * gpu_rc_init_decoder (:319-340) and the per-position decode launches
 * (:479-490), on explicit integer CDFs instead of logits.  No handle and no
 * allocation: every pointer is a device pointer the caller owns, states hold
 * boa_rc_state_bytes(decoder) bytes per stream, and each call only enqueues
 * kernels on `stream` (NULL = legacy default stream).  A call codes n_steps
 * positions: cdf [n_steps][n_streams][257] (Q[256] = 2^24), symbols
 * [n_steps][n_streams]; successive calls continue the streams.  Encoder
 * stream i is written to d_words + i*pitch_words; the pitch must hold the
 * whole stream (boa_stream_capacity_words(total steps + 1) is enough).  A
 * stream whose coding stops (empty or out-of-range interval, full pitch) is
 * marked in its state and gets size BOA_STREAM_FAILED from finish.  The
 * decoder reads stream i at d_words + d_offsets[i] (word offsets: i*pitch for
 * the encoder's layout, or a compacted BOA2 payload's offsets) and writes
 * symbols [n_steps][n_streams]. */
size_t boa_rc_state_bytes(int decoder);
int boa_rc_encoder_init(void* d_states, int n_streams, void* stream);
int boa_rc_encode_cdf_steps(void* d_states, const uint32_t* d_cdf, const uint8_t* d_syms, int n_streams, int n_steps,
                            uint32_t* d_words, uint32_t pitch_words, void* stream);
int boa_rc_encoder_finish(void* d_states, uint32_t* d_words, uint32_t pitch_words, uint32_t* d_sizes, int n_streams,
                          void* stream);
int boa_rc_decoder_init(void* d_states, const uint32_t* d_words, const uint64_t* d_offsets, const uint32_t* d_sizes,
                        int n_streams, void* stream);
int boa_rc_decode_cdf_steps(void* d_states, const uint32_t* d_cdf, int n_streams, int n_steps, const uint32_t* d_words,
                            const uint64_t* d_offsets, uint8_t* d_syms, void* stream);
/* The integer CDF the library derives from one or more logits rows
 * ([rows][256] -> [rows][257]); exposes the quantiser of
 * range_coder_kernels.cu:860-925 for testing.  Host buffers. */
int boa_cdf_from_logits(boa_model* h, const float* logits, int rows, float inv_temperature, uint32_t* cdf);

/* ---- BOA2 container (boa.cpp:85-107, :158-277, :538-581) ----------------
 * Serialises a container into buf (cap bytes); *len_out = bytes needed (call
 * with buf = NULL to size).  flags bit0 = warm start; interleave_batch is
 * written as the 4-byte fingerprint field when warm start is set. */
int boa_boa2_build(uint64_t total_size, uint32_t chunk_len, uint32_t n_chunks, uint32_t last_chunk_len,
                   uint32_t flags, uint32_t interleave_batch, const uint8_t* first_bytes,
                   const uint64_t* stream_bytes, const uint8_t* payload, uint8_t* buf, size_t cap,
                   size_t* len_out);
/* Same, with the fingerprint field given verbatim (fp_len <= 255 bytes): the
 * Python BoaFile writer stores blake2s(model class name, digest_size=16)
 * there with flags 0 (boa.py:107-131, :226-240); the C++ writer stores the
 * 4-byte interleave batch under warm start or nothing (boa.cpp:230-237). */
int boa_boa2_build_fp(uint64_t total_size, uint32_t chunk_len, uint32_t n_chunks, uint32_t last_chunk_len,
                      uint32_t flags, const uint8_t* fp, uint32_t fp_len, const uint8_t* first_bytes,
                      const uint64_t* stream_bytes, const uint8_t* payload, uint8_t* buf, size_t cap,
                      size_t* len_out);
typedef struct boa2_info {
  uint64_t total_size;
  uint32_t chunk_len, n_chunks, last_chunk_len, flags, interleave_batch;
  uint32_t index_version; /* 1 or 2 */
  uint64_t payload_offset, payload_bytes;
  uint32_t fp_len;        /* fingerprint field as stored */
  uint8_t fp[255];
} boa2_info;
/* Parses and validates (magic, version, index, CRC-32, ranges).  first_bytes,
 * offsets and lengths (bytes, relative to the payload) may be NULL to query
 * info only; otherwise they need n_chunks entries. */
int boa_boa2_parse(const uint8_t* buf, size_t len, boa2_info* info, uint8_t* first_bytes, uint64_t* offsets,
                   uint64_t* lengths);

/* ---- the Python codec's batch coder (gpu_range_coder.py:57-298) ---------
 * Replaces gpu_range_coder.gpu.queue.RangeCoderBatch, which codec.py's
 * compress_GPU / decompress_GPU (codec.py:11-151) call once per position.
 * Each step takes one fp32 probability row per stream ([n_streams][vocab],
 * device memory), quantises it with build_cdf_fast (cdf[i] = (u32)(P_i *
 * (2^24 - vocab) / P_vocab) + i, P_i the left-to-right fp64 prefix sum) and
 * range-codes one symbol with the same 64-bit-state, 32-bit-word coder as
 * the C++ path.  Streams are bit-for-bit the reference's for equal
 * probabilities.  One handle per stream batch and device; device buffers
 * are the handle's, host buffers the caller's.  d_mask (uint8 or bool, may
 * be NULL) skips streams whose byte is 0; encode also skips symbols outside
 * [0, vocab), as the reference does.  Work goes on `stream` (NULL = legacy
 * default stream) without synchronising, except read / load. */
typedef struct boa_pyrc boa_pyrc;
/* RangeCoderBatch(N, K, pitch) (:217-237); vocab <= 1024, as the reference's
 * 1025-entry CDF array.  Words are zeroed and encoder states reset. */
int boa_pyrc_create(int n_streams, int vocab, int pitch_words, int device, boa_pyrc** out);
void boa_pyrc_free(boa_pyrc* h);
const char* boa_pyrc_last_error(const boa_pyrc* h);
/* encode_step_from_device (:262-269): symbols int32 [n_streams] */
int boa_pyrc_encode_step(boa_pyrc* h, const int32_t* d_symbols, const float* d_probs, const uint8_t* d_mask,
                         void* stream);
/* finalize (:270-274) */
int boa_pyrc_finalize(boa_pyrc* h, void* stream);
/* get_compressed_host / get_sizes_host (:241-245, :275-287): sizes [n_streams]
 * and, when words_host is not NULL, the [n_streams][pitch_words] buffer.
 * BOA_E_DEVICE if a stream outgrew pitch_words (the reference writes past
 * its buffer there). */
int boa_pyrc_read(boa_pyrc* h, uint32_t* words_host, int32_t* sizes_host, void* stream);
/* load_compressed_from_host (:224-240): [n_streams][pitch_words] words and
 * the word count of each stream (<= pitch_words). */
int boa_pyrc_load(boa_pyrc* h, const uint32_t* words_host, const int32_t* sizes_host, void* stream);
/* init_decoder_from_current_bytes (:288-292) */
int boa_pyrc_init_decoder(boa_pyrc* h, void* stream);
/* decode_step_to_device (:293-300): symbols int32 [n_streams] */
int boa_pyrc_decode_step(boa_pyrc* h, const float* d_probs, int32_t* d_out_symbols, const uint8_t* d_mask,
                         void* stream);

#ifdef __cplusplus
}
#endif
#endif /* BOA_B200_H */
