// noalloc.cu -- an integer-CDF range encoder that allocates no memory.
//
// boa_rc_encode_cdf() stages inputs, per-stream coder states and stream
// buffers in memory that the handle allocates.  Some callers cannot allocate
// device memory at the point where they want to encode: code running under a
// custom or pooled allocator that forbids raw cudaMalloc, callers in a
// framework that owns every buffer, or plugins that must not change the
// process's device-memory footprint per call.  For them this file keeps the
// only scratch the encoder needs -- one 32-byte coder state per stream -- in
// a fixed file-scope device array, and the caller passes every input and
// output buffer.
#include <mutex>

namespace boa {

constexpr int kNoAllocMaxStreams = 65536;  // 65536 x 32 B = 2 MiB per GPU, held until exit

// Device scratch shared by every call.  In host code this name is only a
// stand-in for the symbol; the device address comes from
// cudaGetSymbolAddress (see noalloc_scratch below).
static __device__ __align__(256) EncState g_noalloc_states[kNoAllocMaxStreams];

// Device address of g_noalloc_states on the current device, looked up once
// per device (with that device current) and cached for the life of the
// process.  A caller that destroys its primary context (cudaDeviceReset)
// invalidates the cached address, so such a caller must not use this entry
// point afterwards.
static EncState* noalloc_scratch(cudaError_t* err) {
  static std::mutex mu;
  static EncState* addr[64] = {nullptr};
  int dev = 0;
  if ((*err = cudaGetDevice(&dev)) != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) { *err = cudaErrorInvalidDevice; return nullptr; }
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if ((*err = cudaGetSymbolAddress(&p, g_noalloc_states)) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<EncState*>(p);
  }
  *err = cudaSuccess;
  return addr[dev];
}

}  // namespace boa

extern "C" int boa_rc_encode_cdf_noalloc(const uint32_t* d_cdf, const uint8_t* d_syms, int n_streams, int n_steps,
                                         uint32_t* d_words, uint32_t pitch_words, uint32_t* d_sizes, void* stream) {
  if (!d_cdf || !d_syms || !d_words || !d_sizes || n_streams <= 0 || n_steps < 0)
    return fail(nullptr, BOA_E_INVALID, "boa_rc_encode_cdf_noalloc: null buffer or empty size");
  if (n_streams > boa::kNoAllocMaxStreams)
    return fail(nullptr, BOA_E_INVALID,
                "boa_rc_encode_cdf_noalloc: n_streams exceeds the static maximum of " +
                    std::to_string(boa::kNoAllocMaxStreams));
  if (pitch_words < boa_stream_capacity_words((uint32_t)n_steps + 1))
    return fail(nullptr, BOA_E_INVALID,
                "boa_rc_encode_cdf_noalloc: pitch_words below boa_stream_capacity_words(n_steps + 1)");
  cudaError_t e;
  if (stream) {  // the states live on the current device: the stream must belong to it
    int cur = -1, sdev = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cudaStreamGetDevice((cudaStream_t)stream, &sdev) != cudaSuccess ||
        cur != sdev) {
      cudaGetLastError();
      return fail(nullptr, BOA_E_INVALID, "boa_rc_encode_cdf_noalloc: the stream belongs to another device");
    }
  }
  boa::EncState* es = boa::noalloc_scratch(&e);
  if (!es) return fail(nullptr, BOA_E_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  cudaStream_t st = (cudaStream_t)stream;
  // the array keeps the previous call's states: reset every stream used here
  if ((e = boa::launch_enc_init(es, n_streams, st)) != cudaSuccess ||
      (n_steps > 0 &&
       (e = boa::launch_rc_encode_cdf(es, d_cdf, d_syms, n_streams, n_steps, d_words, (int)pitch_words, st,
                                      false)) != cudaSuccess) ||
      (e = boa::launch_enc_finish(es, d_words, (int)pitch_words, d_sizes, n_streams, st, BOA_STREAM_FAILED, false)) !=
          cudaSuccess)
    return fail(nullptr, BOA_E_CUDA, std::string("boa_rc_encode_cdf_noalloc launch: ") + cudaGetErrorString(e));
  return BOA_OK;
}
