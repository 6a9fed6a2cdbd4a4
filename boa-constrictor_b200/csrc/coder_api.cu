// coder_api.cu -- the integer-CDF range coder as handle-free, step-wise
// device entry points.
//
// The reference drives its coder as separate launches on caller-owned
// device state: gpu_rc_init (range_coder_kernels.cu:46-60), one encode
// launch per position, gpu_rc_finish_batch (:279-317), gpu_rc_init_decoder
// (:319-340) and one decode launch per position.  These entry points keep that
// shape for callers that generate CDFs tile by tile (the configs[1]
// microbenchmark draws every step's distributions on the device): the caller
// owns the coder states (boa_rc_state_bytes each), the CDF tiles and the
// stream buffers; nothing is allocated and no handle is needed.  Failures of
// a stream (an empty CDF interval, a full buffer) are marked on the stream
// itself -- the finish call writes BOA_STREAM_FAILED as its size -- and never
// touch the device error word that model handles read.

namespace {

int coder_args_fail(const char* fn, const char* what) {
  return fail(nullptr, BOA_E_INVALID, std::string(fn) + ": " + what);
}
int coder_launch(const char* fn, cudaError_t e) {
  return e == cudaSuccess ? BOA_OK : fail(nullptr, BOA_E_CUDA, std::string(fn) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

size_t boa_rc_state_bytes(int decoder) { return decoder ? sizeof(boa::DecState) : sizeof(boa::EncState); }

int boa_rc_encoder_init(void* d_states, int n_streams, void* stream) {
  if (!d_states || n_streams <= 0) return coder_args_fail("boa_rc_encoder_init", "null states or no streams");
  return coder_launch("boa_rc_encoder_init",
                      boa::launch_enc_init((boa::EncState*)d_states, n_streams, (cudaStream_t)stream));
}

int boa_rc_encode_cdf_steps(void* d_states, const uint32_t* d_cdf, const uint8_t* d_syms, int n_streams, int n_steps,
                            uint32_t* d_words, uint32_t pitch_words, void* stream) {
  if (!d_states || !d_cdf || !d_syms || !d_words || n_streams <= 0 || n_steps < 0 || pitch_words < 2 ||
      pitch_words > 0x7fffffffu)
    return coder_args_fail("boa_rc_encode_cdf_steps", "null buffer, no streams or bad pitch");
  if (n_steps == 0) return BOA_OK;
  return coder_launch("boa_rc_encode_cdf_steps",
                      boa::launch_rc_encode_cdf((boa::EncState*)d_states, d_cdf, d_syms, n_streams, n_steps, d_words,
                                                (int)pitch_words, (cudaStream_t)stream, false));
}

int boa_rc_encoder_finish(void* d_states, uint32_t* d_words, uint32_t pitch_words, uint32_t* d_sizes, int n_streams,
                          void* stream) {
  if (!d_states || !d_words || !d_sizes || n_streams <= 0 || pitch_words < 2 || pitch_words > 0x7fffffffu)
    return coder_args_fail("boa_rc_encoder_finish", "null buffer, no streams or bad pitch");
  return coder_launch("boa_rc_encoder_finish",
                      boa::launch_enc_finish((boa::EncState*)d_states, d_words, (int)pitch_words, d_sizes, n_streams,
                                             (cudaStream_t)stream, BOA_STREAM_FAILED, false));
}

int boa_rc_decoder_init(void* d_states, const uint32_t* d_words, const uint64_t* d_offsets, const uint32_t* d_sizes,
                        int n_streams, void* stream) {
  if (!d_states || !d_words || !d_offsets || !d_sizes || n_streams <= 0)
    return coder_args_fail("boa_rc_decoder_init", "null buffer or no streams");
  return coder_launch("boa_rc_decoder_init",
                      boa::launch_rc_decode_init((boa::DecState*)d_states, d_words,
                                                 (const unsigned long long*)d_offsets, d_sizes, n_streams,
                                                 (cudaStream_t)stream));
}

int boa_rc_decode_cdf_steps(void* d_states, const uint32_t* d_cdf, int n_streams, int n_steps, const uint32_t* d_words,
                            const uint64_t* d_offsets, uint8_t* d_syms, void* stream) {
  if (!d_states || !d_cdf || !d_words || !d_offsets || !d_syms || n_streams <= 0 || n_steps < 0)
    return coder_args_fail("boa_rc_decode_cdf_steps", "null buffer or no streams");
  if (n_steps == 0) return BOA_OK;
  return coder_launch("boa_rc_decode_cdf_steps",
                      boa::launch_rc_decode_cdf((boa::DecState*)d_states, d_cdf, d_words,
                                                (const unsigned long long*)d_offsets, n_streams, n_steps, d_syms,
                                                (cudaStream_t)stream));
}

}  // extern "C"
