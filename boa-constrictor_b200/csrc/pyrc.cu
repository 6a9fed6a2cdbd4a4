// pyrc.cu -- the Python codec's batch range coder, B200 kernels.
//
// Replaces RangeCoderBatch of gpu_range_coder.py (:57-298), the coder that
// codec.py's compress_GPU / decompress_GPU drive once per position with the
// model's softmax rows.  Each step quantises one fp32 probability row per
// stream with build_cdf_fast (:57-79) and range-codes one symbol with the
// 64-bit-state / 32-bit-word coder (:81-215).  Streams it writes are bit-for-bit
// the reference's for the same probabilities, so a .boa file of the Python
// path can be written or read with this coder in place of the reference's.
//
// The reference runs one thread per stream, builds all K+1 CDF entries in a
// 1025-entry local array and reads its row with strided scalar loads.  Here
// one warp handles a stream: the row is read coalesced, the left-to-right fp64
// prefix sums (whose rounding fixes the CDF) run lane to lane through
// shuffles, every lane converts its own entries, and the decoder's symbol
// search is one ballot.  Lane 0 alone updates the coder state.
#include <string>

#include "kernels.cuh"

namespace boa {

struct PyEnc {
  unsigned long long lower, range;
  uint32_t first_inv;
  int inv, w, pad;
};
struct PyDec {
  unsigned long long lower, range, point;
  int r, pad;
};

constexpr unsigned kFull = 0xffffffffu;
constexpr uint32_t kPyTotal = 1u << 24;

// The row quantiser, lane-distributed: lane l owns entries [l*E, l*E + E).
template <int E>
struct PyRow {
  double cum[E];  // P_i, the fp64 sum of probabilities 0..i-1 (left to right)
  double scale;   // (2^24 - K) / P_K
  uint32_t step;  // equal-split increment when P_K is not positive and finite
  bool equal;
  int base, K;

  __device__ __forceinline__ void build(const float* __restrict__ row, int K_, int lane) {
    K = K_;
    base = lane * E;
    float p[E];
    if (E >= 4 && (K & 3) == 0) {
#pragma unroll
      for (int v = 0; v < E / 4; ++v) {
        const int i = base + 4 * v;
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < K) q = __ldg(reinterpret_cast<const float4*>(row + i));
        p[4 * v] = q.x; p[4 * v + 1] = q.y; p[4 * v + 2] = q.z; p[4 * v + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) p[e] = base + e < K ? __ldg(row + base + e) : 0.f;
    }
    // sequential chain: lane l starts from the sum lane l-1 ended with
    double carry = 0.0, c = 0.0;
    for (int src = 0; src < 32; ++src) {
      if (lane == src) {
        c = carry;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          cum[e] = c;
          if (base + e < K) c = __dadd_rn(c, (double)p[e]);
        }
      }
      carry = __shfl_sync(kFull, c, src);
    }
    const double norm = carry;
    const uint32_t free_w = kPyTotal - (uint32_t)K;
    equal = !(norm > 0.0) || !isfinite(norm);
    scale = equal ? 0.0 : __ddiv_rn((double)free_w, norm);
    step = free_w / (uint32_t)K + 1u;
  }
  // cdf of entry base + e (e < E, base + e < K)
  __device__ __forceinline__ uint32_t at(int e) const {
    const uint32_t i = (uint32_t)(base + e);
    return equal ? i * step : __double2uint_rz(__dmul_rn(cum[e], scale)) + i;
  }
  // cdf[i] for any 0 <= i <= K, gathered from its owner lane (all lanes call)
  __device__ __forceinline__ uint32_t get(int i) const {
    uint32_t mine = 0;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (base + e == i) mine = at(e);
    const uint32_t v = __shfl_sync(kFull, mine, (i < K ? i : 0) / E);
    return i >= K ? kPyTotal : v;
  }
};

__device__ __forceinline__ void py_put(uint32_t* out, int pitch, int& w, uint32_t v) {
  if (w < pitch) out[w] = v;
  ++w;  // counted past the pitch: finalize reports the overflow
}

template <int E>
__global__ void __launch_bounds__(128) pyrc_encode_kernel(const int32_t* __restrict__ syms,
                                                          const float* __restrict__ probs, int N, int K,
                                                          uint32_t* __restrict__ words, PyEnc* __restrict__ states,
                                                          int pitch, const uint8_t* __restrict__ mask) {
  const int idx = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (idx >= N) return;
  if (mask && mask[idx] == 0) return;
  const int s = syms[idx];
  if (s < 0 || s >= K) return;
  PyRow<E> row;
  row.build(probs + (size_t)idx * K, K, lane);
  const uint32_t left = row.get(s), right = row.get(s + 1);
  if (lane != 0) return;
  PyEnc st = states[idx];
  uint32_t* out = words + (size_t)idx * pitch;
  const unsigned long long scale = st.range >> 24;
  const unsigned long long old_lower = st.lower;
  st.range = scale * (unsigned long long)(right - left);
  st.lower = st.lower + scale * (unsigned long long)left;
  if (st.inv > 0 && st.lower + st.range > st.lower) {
    const bool carry = st.lower < old_lower;
    py_put(out, pitch, st.w, carry ? st.first_inv + 1u : st.first_inv);
    for (int i = 1; i < st.inv; ++i) py_put(out, pitch, st.w, carry ? 0u : 0xFFFFFFFFu);
    st.inv = 0;
  }
  while (st.range < (1ull << 32)) {
    const uint32_t lw = (uint32_t)(st.lower >> 32);
    st.lower <<= 32;
    st.range <<= 32;
    if (st.inv > 0) {
      if (st.inv < 0x7FFFFFFF) st.inv += 1;
    } else if (st.lower + st.range > st.lower) {
      py_put(out, pitch, st.w, lw);
    } else {
      st.inv = 1;
      st.first_inv = lw;
    }
  }
  states[idx] = st;
}

template <int E>
__global__ void __launch_bounds__(128) pyrc_decode_kernel(const float* __restrict__ probs, int N, int K,
                                                          const uint32_t* __restrict__ words,
                                                          const int32_t* __restrict__ sizes,
                                                          PyDec* __restrict__ states, int pitch,
                                                          int32_t* __restrict__ out_syms,
                                                          const uint8_t* __restrict__ mask) {
  const int idx = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (idx >= N) return;
  if (mask && mask[idx] == 0) return;
  PyRow<E> row;
  row.build(probs + (size_t)idx * K, K, lane);
  PyDec st = states[idx];  // every lane reads the same 32 bytes
  const unsigned long long scale = st.range >> 24;
  unsigned long long q = (st.point - st.lower) / scale;
  if (q >= (1ull << 24)) q = (1ull << 24) - 1ull;
  const uint32_t target = (uint32_t)q;
  // first i >= 1 with cdf[i] > target (cdf[K] = 2^24 always qualifies)
  int first = K;
#pragma unroll
  for (int e = E - 1; e >= 0; --e) {
    const int i = row.base + e;
    if (i >= 1 && i < K && row.at(e) > target) first = i;
  }
  const unsigned hit = __ballot_sync(kFull, first < K);
  const int i = hit ? __shfl_sync(kFull, first, __ffs(hit) - 1) : K;
  int s = i - 1;
  if (s < 0) s = 0;
  if (s >= K) s = K - 1;
  const uint32_t left = row.get(s), right = row.get(s + 1);
  if (lane != 0) return;
  out_syms[idx] = s;
  st.lower = st.lower + scale * (unsigned long long)left;
  st.range = scale * (unsigned long long)(right - left);
  const uint32_t* in = words + (size_t)idx * pitch;
  const int n = sizes[idx];
  while (st.range < (1ull << 32)) {
    st.lower <<= 32;
    st.range <<= 32;
    const uint32_t w = st.r < n ? in[st.r++] : 0u;
    st.point = (st.point << 32) | (unsigned long long)w;
  }
  states[idx] = st;
}

__global__ void pyrc_reset_kernel(PyEnc* st, int32_t* sizes, int N) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  st[i] = PyEnc{0ull, ~0ull, 0u, 0, 0, 0};
  sizes[i] = 0;
}

// finalize_kernel (gpu_range_coder.py:142-168); -1 marks a stream longer than the pitch
__global__ void pyrc_finalize_kernel(PyEnc* states, uint32_t* words, int32_t* sizes, int N, int pitch) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= N) return;
  PyEnc st = states[idx];
  if (st.range == ~0ull) { sizes[idx] = 0; return; }
  uint32_t* out = words + (size_t)idx * pitch;
  const unsigned long long point = st.lower + ((1ull << 32) - 1ull);
  if (st.inv > 0) {
    const bool carry = point < st.lower;
    py_put(out, pitch, st.w, carry ? st.first_inv + 1u : st.first_inv);
    for (int i = 1; i < st.inv; ++i) py_put(out, pitch, st.w, carry ? 0u : 0xFFFFFFFFu);
    st.inv = 0;
  }
  const uint32_t pw = (uint32_t)(point >> 32);
  py_put(out, pitch, st.w, pw);
  if ((uint32_t)((st.lower + st.range) >> 32) == pw) py_put(out, pitch, st.w, 0u);
  states[idx] = st;
  sizes[idx] = st.w <= pitch ? st.w : -1;
}

// init_dec_kernel (gpu_range_coder.py:170-180)
__global__ void pyrc_init_dec_kernel(const uint32_t* words, const int32_t* sizes, PyDec* states, int N, int pitch) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= N) return;
  const uint32_t* in = words + (size_t)idx * pitch;
  PyDec st{0ull, ~0ull, 0ull, 0, 0};
  for (int k = 0; k < 2; ++k) {
    const uint32_t w = st.r < sizes[idx] ? in[st.r++] : 0u;
    st.point = (st.point << 32) | (unsigned long long)w;
  }
  states[idx] = st;
}

template <int E>
static void pyrc_launch_enc(const int32_t* syms, const float* probs, int N, int K, uint32_t* words, PyEnc* st,
                            int pitch, const uint8_t* mask, cudaStream_t s) {
  pyrc_encode_kernel<E><<<(unsigned)((N + 3) / 4), 128, 0, s>>>(syms, probs, N, K, words, st, pitch, mask);
}
template <int E>
static void pyrc_launch_dec(const float* probs, int N, int K, const uint32_t* words, const int32_t* sizes,
                            PyDec* st, int pitch, int32_t* out, const uint8_t* mask, cudaStream_t s) {
  pyrc_decode_kernel<E><<<(unsigned)((N + 3) / 4), 128, 0, s>>>(probs, N, K, words, sizes, st, pitch, out, mask);
}

}  // namespace boa

struct boa_pyrc {
  int device = 0, N = 0, K = 0, pitch = 0;
  void* arena = nullptr;
  boa::PyEnc* enc = nullptr;
  boa::PyDec* dec = nullptr;
  uint32_t* words = nullptr;
  int32_t* sizes = nullptr;
  std::string err;
  ~boa_pyrc() {
    if (arena) { cudaSetDevice(device); cudaFree(arena); }
  }
};

namespace {
int pyrc_fail(boa_pyrc* h, int code, const std::string& msg) {
  if (h) h->err = msg; else g_load_error = msg;
  return code;
}
int pyrc_cuda(boa_pyrc* h, cudaError_t e, const char* where) {
  return pyrc_fail(h, BOA_E_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}
int pyrc_lanes(int K) { return K <= 32 ? 1 : K <= 64 ? 2 : K <= 128 ? 4 : K <= 256 ? 8 : K <= 512 ? 16 : 32; }
}  // namespace

extern "C" {

int boa_pyrc_create(int n_streams, int vocab, int pitch_words, int device, boa_pyrc** out) {
  if (!out) return pyrc_fail(nullptr, BOA_E_INVALID, "out is NULL");
  *out = nullptr;
  if (n_streams <= 0 || vocab <= 0 || vocab > 1024 || pitch_words <= 0)
    return pyrc_fail(nullptr, BOA_E_INVALID, "need n_streams > 0, 1 <= vocab <= 1024 and pitch_words > 0");
  std::unique_ptr<boa_pyrc> h(new boa_pyrc());
  h->device = device; h->N = n_streams; h->K = vocab; h->pitch = pitch_words;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return pyrc_cuda(nullptr, e, "cudaSetDevice");
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t N = (size_t)n_streams;
  const size_t b_enc = al(N * sizeof(boa::PyEnc)), b_dec = al(N * sizeof(boa::PyDec)),
               b_words = al(N * (size_t)pitch_words * 4), b_sizes = al(N * 4);
  if ((e = cudaMalloc(&h->arena, b_enc + b_dec + b_words + b_sizes)) != cudaSuccess) {
    cudaGetLastError();
    return pyrc_fail(nullptr, BOA_E_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  }
  uint8_t* p = (uint8_t*)h->arena;
  h->enc = (boa::PyEnc*)p; p += b_enc;
  h->dec = (boa::PyDec*)p; p += b_dec;
  h->words = (uint32_t*)p; p += b_words;
  h->sizes = (int32_t*)p;
  if ((e = cudaMemset(h->words, 0, N * (size_t)pitch_words * 4)) != cudaSuccess) return pyrc_cuda(nullptr, e, "cudaMemset");
  boa::pyrc_reset_kernel<<<(unsigned)((N + 255) / 256), 256>>>(h->enc, h->sizes, n_streams);
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return pyrc_cuda(nullptr, e, "coder state init");
  *out = h.release();
  return BOA_OK;
}

void boa_pyrc_free(boa_pyrc* h) { delete h; }

const char* boa_pyrc_last_error(const boa_pyrc* h) { return h ? h->err.c_str() : g_load_error.c_str(); }

int boa_pyrc_encode_step(boa_pyrc* h, const int32_t* d_symbols, const float* d_probs, const uint8_t* d_mask,
                         void* stream) {
  if (!h || !d_symbols || !d_probs) return pyrc_fail(h, BOA_E_INVALID, "null argument");
  cudaSetDevice(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  switch (pyrc_lanes(h->K)) {
    case 1: boa::pyrc_launch_enc<1>(d_symbols, d_probs, h->N, h->K, h->words, h->enc, h->pitch, d_mask, s); break;
    case 2: boa::pyrc_launch_enc<2>(d_symbols, d_probs, h->N, h->K, h->words, h->enc, h->pitch, d_mask, s); break;
    case 4: boa::pyrc_launch_enc<4>(d_symbols, d_probs, h->N, h->K, h->words, h->enc, h->pitch, d_mask, s); break;
    case 8: boa::pyrc_launch_enc<8>(d_symbols, d_probs, h->N, h->K, h->words, h->enc, h->pitch, d_mask, s); break;
    case 16: boa::pyrc_launch_enc<16>(d_symbols, d_probs, h->N, h->K, h->words, h->enc, h->pitch, d_mask, s); break;
    default: boa::pyrc_launch_enc<32>(d_symbols, d_probs, h->N, h->K, h->words, h->enc, h->pitch, d_mask, s); break;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "encode step launch");
}

int boa_pyrc_finalize(boa_pyrc* h, void* stream) {
  if (!h) return BOA_E_INVALID;
  cudaSetDevice(h->device);
  boa::pyrc_finalize_kernel<<<(unsigned)((h->N + 127) / 128), 128, 0, (cudaStream_t)stream>>>(h->enc, h->words, h->sizes,
                                                                                              h->N, h->pitch);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "finalize launch");
}

int boa_pyrc_read(boa_pyrc* h, uint32_t* words_host, int32_t* sizes_host, void* stream) {
  if (!h || !sizes_host) return pyrc_fail(h, BOA_E_INVALID, "null argument");
  cudaSetDevice(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(sizes_host, h->sizes, (size_t)h->N * 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && words_host)
    e = cudaMemcpyAsync(words_host, h->words, (size_t)h->N * h->pitch * 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return pyrc_cuda(h, e, "reading streams");
  for (int i = 0; i < h->N; ++i)
    if (sizes_host[i] < 0)
      return pyrc_fail(h, BOA_E_DEVICE, "stream " + std::to_string(i) + " is longer than pitch_words");
  return BOA_OK;
}

int boa_pyrc_load(boa_pyrc* h, const uint32_t* words_host, const int32_t* sizes_host, void* stream) {
  if (!h || !words_host || !sizes_host) return pyrc_fail(h, BOA_E_INVALID, "null argument");
  for (int i = 0; i < h->N; ++i)
    if (sizes_host[i] < 0 || sizes_host[i] > h->pitch)
      return pyrc_fail(h, BOA_E_INVALID, "stream " + std::to_string(i) + " exceeds pitch_words");
  cudaSetDevice(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(h->words, words_host, (size_t)h->N * h->pitch * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(h->sizes, sizes_host, (size_t)h->N * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "loading streams");
}

int boa_pyrc_init_decoder(boa_pyrc* h, void* stream) {
  if (!h) return BOA_E_INVALID;
  cudaSetDevice(h->device);
  boa::pyrc_init_dec_kernel<<<(unsigned)((h->N + 127) / 128), 128, 0, (cudaStream_t)stream>>>(h->words, h->sizes, h->dec,
                                                                                              h->N, h->pitch);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "decoder init launch");
}

int boa_pyrc_decode_step(boa_pyrc* h, const float* d_probs, int32_t* d_out_symbols, const uint8_t* d_mask,
                         void* stream) {
  if (!h || !d_probs || !d_out_symbols) return pyrc_fail(h, BOA_E_INVALID, "null argument");
  cudaSetDevice(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  switch (pyrc_lanes(h->K)) {
    case 1: boa::pyrc_launch_dec<1>(d_probs, h->N, h->K, h->words, h->sizes, h->dec, h->pitch, d_out_symbols, d_mask, s); break;
    case 2: boa::pyrc_launch_dec<2>(d_probs, h->N, h->K, h->words, h->sizes, h->dec, h->pitch, d_out_symbols, d_mask, s); break;
    case 4: boa::pyrc_launch_dec<4>(d_probs, h->N, h->K, h->words, h->sizes, h->dec, h->pitch, d_out_symbols, d_mask, s); break;
    case 8: boa::pyrc_launch_dec<8>(d_probs, h->N, h->K, h->words, h->sizes, h->dec, h->pitch, d_out_symbols, d_mask, s); break;
    case 16: boa::pyrc_launch_dec<16>(d_probs, h->N, h->K, h->words, h->sizes, h->dec, h->pitch, d_out_symbols, d_mask, s); break;
    default: boa::pyrc_launch_dec<32>(d_probs, h->N, h->K, h->words, h->sizes, h->dec, h->pitch, d_out_symbols, d_mask, s); break;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "decode step launch");
}

}  // extern "C"
