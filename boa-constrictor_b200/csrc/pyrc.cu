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
// one lane still owns one stream, but a warp stages the rows of its 32
// streams through shared memory, and each lane runs its own row's fp64 prefix
// sum (whose rounding fixes the CDF).  The encoder needs only P_s, P_s+1 and
// P_K, so it reads the row once and builds no table.  Two staging forms:
//   - K <= 256 with K % 4 == 0 (the codec's K = 256): the warp's 32 rows land
//     in shared memory by one bulk async copy per row; the decoder records P
//     at every 16th entry, binary-searches those marks and scans 16 entries;
//   - any other K (up to 1024): 64-column slabs staged with coalesced loads;
//     the decoder records P at every slab start, picks the slab holding its
//     target and re-reads only that slab.
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

// A warp codes 32 streams, one per lane.  Rows are staged through shared
// memory in slabs of 64 columns (coalesced 128-byte row segments; the tile's
// row stride of 65 words keeps both the staging stores and each lane's reads
// of its own row free of bank conflicts).  Each lane then runs the fp64
// left-to-right sum of its own row -- the order build_cdf_fast rounds in --
// so the chain costs one add per element instead of occupying the warp.
constexpr int kSlab = 64;
constexpr int kPyWarps = 8;
constexpr int kMaxSlabs = 1024 / kSlab + 1;

struct PyTile {
  float t[32 * (kSlab + 1)];
  double bcum[32 * kMaxSlabs];  // decode: P at every slab start, per lane
};

// columns [c0, c0 + 64) of rows row0 .. row0 + 31 (rows >= N read as zero)
__device__ __forceinline__ void py_stage(const float* __restrict__ probs, long long row0, int N, int K, int c0,
                                         float* __restrict__ t, int lane) {
  __syncwarp();
#pragma unroll 16
  for (int r = 0; r < 32; ++r) {
    const long long row = row0 + r;
    float a = 0.f, b = 0.f;
    if (row < N) {
      const float* src = probs + row * K + c0;
      if (c0 + lane < K) a = __ldg(src + lane);
      if (c0 + 32 + lane < K) b = __ldg(src + 32 + lane);
    }
    t[r * (kSlab + 1) + lane] = a;
    t[r * (kSlab + 1) + 32 + lane] = b;
  }
  __syncwarp();
}

__device__ __forceinline__ uint32_t py_cdf(double cum, double scale, uint32_t i) {
  return __double2uint_rz(__dmul_rn(cum, scale)) + i;
}

__device__ __forceinline__ void py_put(uint32_t* out, int pitch, int& w, uint32_t v) {
  if (w < pitch) out[w] = v;
  ++w;  // counted past the pitch: finalize reports the overflow
}

// encode_kernel's state update for the interval [left, right) (gpu_range_coder.py:96-140)
__device__ __forceinline__ void py_encode_update(PyEnc* __restrict__ states, uint32_t* __restrict__ words, int pitch,
                                                 long long idx, uint32_t left, uint32_t right) {
  PyEnc st = states[idx];
  uint32_t* out = words + (size_t)idx * pitch;
  const unsigned long long scl = st.range >> 24;
  const unsigned long long old_lower = st.lower;
  st.range = scl * (unsigned long long)(right - left);
  st.lower = st.lower + scl * (unsigned long long)left;
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

// decode_step_kernel's search (gpu_range_coder.py:196-201): the first i >= 1
// with cdf[i] > target (cdf[K] = 2^24 always qualifies); [left, right) =
// [cdf[i-1], cdf[i]).  `row` holds the K probabilities, bcum the sum P at
// entries 0, stride, 2*stride, ... and `norm` = P_K.  Entries strictly
// increase when no probability is negative, so a binary search over those
// marks finds the last one <= target and the scan starts there; otherwise it
// walks every entry from 1 as the reference does.
__device__ __forceinline__ int py_search(const float* row, const double* bcum, int stride, int K, double norm,
                                         bool neg, uint32_t target, uint32_t& left, uint32_t& right) {
  const uint32_t free_w = kPyTotal - (uint32_t)K;
  if (!(norm > 0.0) || !isfinite(norm)) {
    const uint32_t step = free_w / (uint32_t)K + 1u;
    const int i = (int)min((uint32_t)K, target / step + 1u);
    left = (uint32_t)(i - 1) * step;
    right = i == K ? kPyTotal : (uint32_t)i * step;
    return i;
  }
  const double scale = __ddiv_rn((double)free_w, norm);
  int k = 0;
  if (!neg) {
    int hi = (K + stride - 1) / stride;  // marks k < hi; mark 0 (cdf = 0) always qualifies
    while (hi - k > 1) {
      const int mid = (k + hi) >> 1;
      if (py_cdf(bcum[mid], scale, (uint32_t)(mid * stride)) <= target) k = mid;
      else hi = mid;
    }
  }
  double cc = bcum[k];  // bcum[0] = 0
  uint32_t prev = py_cdf(cc, scale, (uint32_t)(k * stride));
  for (int j = k * stride; j < K; ++j) {
    cc = __dadd_rn(cc, (double)row[j]);
    const int ii = j + 1;
    const uint32_t v = ii == K ? kPyTotal : py_cdf(cc, scale, (uint32_t)ii);
    if (v > target) { left = prev; right = v; return ii; }
    prev = v;
  }
  left = prev;  // not reached: cdf[K] > target
  right = kPyTotal;
  return K;
}

// decode_step_kernel's update and refill (gpu_range_coder.py:202-214)
__device__ __forceinline__ void py_decode_update(PyDec& st, const uint32_t* __restrict__ words,
                                                 const int32_t* __restrict__ sizes, int pitch, long long idx,
                                                 uint32_t left, uint32_t right) {
  const unsigned long long scl = st.range >> 24;
  st.lower = st.lower + scl * (unsigned long long)left;
  st.range = scl * (unsigned long long)(right - left);
  const uint32_t* in = words + (size_t)idx * pitch;
  const int n = sizes[idx];
  while (st.range < (1ull << 32)) {
    st.lower <<= 32;
    st.range <<= 32;
    const uint32_t w = st.r < n ? in[st.r++] : 0u;
    st.point = (st.point << 32) | (unsigned long long)w;
  }
}

__global__ void __launch_bounds__(32 * kPyWarps) pyrc_encode_kernel(const int32_t* __restrict__ syms,
                                                                    const float* __restrict__ probs, int N, int K,
                                                                    uint32_t* __restrict__ words,
                                                                    PyEnc* __restrict__ states, int pitch,
                                                                    const uint8_t* __restrict__ mask) {
  extern __shared__ __align__(16) unsigned char py_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* t = reinterpret_cast<float*>(py_smem) + warp * 32 * (kSlab + 1);
  const long long row0 = ((long long)blockIdx.x * kPyWarps + warp) * 32;
  if (row0 >= N) return;
  const long long idx = row0 + lane;
  int s = -1;
  if (idx < N && (!mask || mask[idx] != 0)) s = syms[idx];
  const bool active = s >= 0 && s < K;
  if (!__any_sync(0xffffffffu, active)) return;
  double c = 0.0, cum_s = 0.0, cum_s1 = 0.0;
  for (int c0 = 0; c0 < K; c0 += kSlab) {
    py_stage(probs, row0, N, K, c0, t, lane);
    const int n = min(kSlab, K - c0);
    const float* mine = t + lane * (kSlab + 1);
    for (int j = 0; j < n; ++j) {
      if (c0 + j == s) cum_s = c;
      c = __dadd_rn(c, (double)mine[j]);
      if (c0 + j == s) cum_s1 = c;
    }
  }
  if (!active) return;
  const uint32_t free_w = kPyTotal - (uint32_t)K;
  uint32_t left, right;
  if (!(c > 0.0) || !isfinite(c)) {
    const uint32_t step = free_w / (uint32_t)K + 1u;
    left = (uint32_t)s * step;
    right = s + 1 == K ? kPyTotal : (uint32_t)(s + 1) * step;
  } else {
    const double scale = __ddiv_rn((double)free_w, c);
    left = py_cdf(cum_s, scale, (uint32_t)s);
    right = s + 1 == K ? kPyTotal : py_cdf(cum_s1, scale, (uint32_t)(s + 1));
  }
  py_encode_update(states, words, pitch, idx, left, right);
}

__global__ void __launch_bounds__(32 * kPyWarps) pyrc_decode_kernel(const float* __restrict__ probs, int N, int K,
                                                                    const uint32_t* __restrict__ words,
                                                                    const int32_t* __restrict__ sizes,
                                                                    PyDec* __restrict__ states, int pitch,
                                                                    int32_t* __restrict__ out_syms,
                                                                    const uint8_t* __restrict__ mask) {
  extern __shared__ __align__(16) unsigned char py_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  PyTile* tile = reinterpret_cast<PyTile*>(py_smem) + warp;
  float* t = tile->t;
  double* bcum = tile->bcum + lane * kMaxSlabs;
  const long long row0 = ((long long)blockIdx.x * kPyWarps + warp) * 32;
  if (row0 >= N) return;
  const long long idx = row0 + lane;
  const bool active = idx < N && (!mask || mask[idx] != 0);
  if (!__any_sync(0xffffffffu, active)) return;
  // pass 1: P_K, with P recorded at every slab start; any negative entry
  // (not a softmax row) sends the search through every entry in order
  double c = 0.0;
  bool neg = false;
  for (int c0 = 0, k = 0; c0 < K; c0 += kSlab, ++k) {
    py_stage(probs, row0, N, K, c0, t, lane);
    bcum[k] = c;
    const int n = min(kSlab, K - c0);
    const float* mine = t + lane * (kSlab + 1);
    for (int j = 0; j < n; ++j) {
      neg |= mine[j] < 0.f;
      c = __dadd_rn(c, (double)mine[j]);
    }
  }
  if (!active) return;
  PyDec st = states[idx];
  const unsigned long long scl = st.range >> 24;
  unsigned long long q = (st.point - st.lower) / scl;
  if (q >= (1ull << 24)) q = (1ull << 24) - 1ull;
  const uint32_t target = (uint32_t)q;
  uint32_t left, right;
  const int i = py_search(probs + idx * K, bcum, kSlab, K, c, neg, target, left, right);
  out_syms[idx] = i - 1;
  py_decode_update(st, words, sizes, pitch, idx, left, right);
  states[idx] = st;
}

// ---- rows of K <= 256 (K % 4 == 0): whole tile by bulk async copy ----------
// The slab loop above keeps only 2 KB per warp in flight and stages serially.
// For the Python codec's K = 256 the warp's 32 rows (32 KB) fit in shared
// memory, so each lane issues one bulk copy for its row onto a single
// mbarrier and the whole tile is in flight at once.  Rows sit 1040 B apart:
// 16-byte aligned for the copies, and the 128-bit reads of 8 consecutive
// lanes (one shared-memory phase) land on distinct bank groups.
constexpr int kBulkStride = 260;
constexpr int kBulkWarps = 2;
constexpr int kBulkMaxK = 256;
constexpr int kBulkMark = 16;  // decode: P recorded every 16 entries

struct PyBulkTile {
  float t[32 * kBulkStride];
  double bcum[32 * (kBulkMaxK / kBulkMark + 1)];  // decode: P at every 16th entry (row padded: no bank conflicts)
  uint64_t bar;
  uint64_t pad;
};

// false when the copies did not land within the wait limit (error word set)
__device__ __forceinline__ bool py_stage_bulk(const float* __restrict__ probs, long long row0, int N, int K,
                                              PyBulkTile* tl, int lane) {
  const int rows = (int)min(32LL, (long long)N - row0);
  if (lane == 0) {
    mbar_init(&tl->bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&tl->bar, (uint32_t)(rows * K * 4));
  }
  __syncwarp();
  if (lane < rows) bulk_load(tl->t + lane * kBulkStride, probs + (row0 + lane) * K, (uint32_t)K * 4u, &tl->bar);
  return mbar_wait(&tl->bar, 0);
}

__global__ void __launch_bounds__(32 * kBulkWarps) pyrc_encode_bulk_kernel(const int32_t* __restrict__ syms,
                                                                           const float* __restrict__ probs, int N,
                                                                           int K, uint32_t* __restrict__ words,
                                                                           PyEnc* __restrict__ states, int pitch,
                                                                           const uint8_t* __restrict__ mask) {
  extern __shared__ __align__(16) unsigned char py_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  PyBulkTile* tl = reinterpret_cast<PyBulkTile*>(py_smem) + warp;
  const long long row0 = ((long long)blockIdx.x * kBulkWarps + warp) * 32;
  if (row0 >= N) return;
  const long long idx = row0 + lane;
  int s = -1;
  if (idx < N && (!mask || mask[idx] != 0)) s = syms[idx];
  const bool active = s >= 0 && s < K;
  if (!__any_sync(0xffffffffu, active)) return;
  if (!py_stage_bulk(probs, row0, N, K, tl, lane)) return;
  if (!active) return;
  const float4* r4 = reinterpret_cast<const float4*>(tl->t + lane * kBulkStride);
  double c = 0.0, cum_s = 0.0, cum_s1 = 0.0;
  const int qs = s >> 2;
  for (int q = 0; q < (K >> 2); ++q) {
    const float4 v = r4[q];
    const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (q == qs && u == (s & 3)) cum_s = c;
      c = __dadd_rn(c, (double)e[u]);
      if (q == qs && u == (s & 3)) cum_s1 = c;
    }
  }
  const uint32_t free_w = kPyTotal - (uint32_t)K;
  uint32_t left, right;
  if (!(c > 0.0) || !isfinite(c)) {
    const uint32_t step = free_w / (uint32_t)K + 1u;
    left = (uint32_t)s * step;
    right = s + 1 == K ? kPyTotal : (uint32_t)(s + 1) * step;
  } else {
    const double scale = __ddiv_rn((double)free_w, c);
    left = py_cdf(cum_s, scale, (uint32_t)s);
    right = s + 1 == K ? kPyTotal : py_cdf(cum_s1, scale, (uint32_t)(s + 1));
  }
  py_encode_update(states, words, pitch, idx, left, right);
}

__global__ void __launch_bounds__(32 * kBulkWarps) pyrc_decode_bulk_kernel(const float* __restrict__ probs, int N,
                                                                           int K, const uint32_t* __restrict__ words,
                                                                           const int32_t* __restrict__ sizes,
                                                                           PyDec* __restrict__ states, int pitch,
                                                                           int32_t* __restrict__ out_syms,
                                                                           const uint8_t* __restrict__ mask) {
  extern __shared__ __align__(16) unsigned char py_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  PyBulkTile* tl = reinterpret_cast<PyBulkTile*>(py_smem) + warp;
  const long long row0 = ((long long)blockIdx.x * kBulkWarps + warp) * 32;
  if (row0 >= N) return;
  const long long idx = row0 + lane;
  const bool active = idx < N && (!mask || mask[idx] != 0);
  if (!__any_sync(0xffffffffu, active)) return;
  if (!py_stage_bulk(probs, row0, N, K, tl, lane)) return;
  if (!active) return;
  const float* row = tl->t + lane * kBulkStride;
  const float4* r4 = reinterpret_cast<const float4*>(row);
  double* bcum = tl->bcum + lane * (kBulkMaxK / kBulkMark + 1);
  double c = 0.0;
  bool neg = false;
  for (int q = 0; q < (K >> 2); ++q) {
    if ((q & (kBulkMark / 4 - 1)) == 0) bcum[q / (kBulkMark / 4)] = c;
    const float4 v = r4[q];
    neg |= v.x < 0.f || v.y < 0.f || v.z < 0.f || v.w < 0.f;
    c = __dadd_rn(c, (double)v.x);
    c = __dadd_rn(c, (double)v.y);
    c = __dadd_rn(c, (double)v.z);
    c = __dadd_rn(c, (double)v.w);
  }
  PyDec st = states[idx];
  const unsigned long long scl = st.range >> 24;
  unsigned long long q = (st.point - st.lower) / scl;
  if (q >= (1ull << 24)) q = (1ull << 24) - 1ull;
  const uint32_t target = (uint32_t)q;
  uint32_t left, right;
  const int i = py_search(row, bcum, kBulkMark, K, c, neg, target, left, right);
  out_syms[idx] = i - 1;
  py_decode_update(st, words, sizes, pitch, idx, left, right);
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

constexpr size_t kPyEncSmem = (size_t)kPyWarps * 32 * (kSlab + 1) * sizeof(float);
constexpr size_t kPyDecSmem = (size_t)kPyWarps * sizeof(PyTile);
constexpr size_t kPyBulkSmem = (size_t)kBulkWarps * sizeof(PyBulkTile);

static cudaError_t pyrc_prepare() {
  static bool done = false;
  if (done) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(pyrc_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPyEncSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(pyrc_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPyDecSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(pyrc_encode_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPyBulkSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(pyrc_decode_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPyBulkSmem);
  if (e == cudaSuccess) done = true;
  return e;
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
    if (arena) { DeviceGuard dev(device); cudaFree(arena); }
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
// the bulk-copy kernels need 16-byte aligned rows: K % 4 == 0 and an aligned base
bool pyrc_bulk_ok(const boa_pyrc* h, const float* probs) {
  return h->K <= boa::kBulkMaxK && (h->K & 3) == 0 && ((uintptr_t)probs & 15) == 0;
}
}  // namespace

extern "C" {

int boa_pyrc_create(int n_streams, int vocab, int pitch_words, int device, boa_pyrc** out) {
  if (!out) return pyrc_fail(nullptr, BOA_E_INVALID, "out is NULL");
  *out = nullptr;
  if (n_streams <= 0 || vocab <= 0 || vocab > 1024 || pitch_words <= 0)
    return pyrc_fail(nullptr, BOA_E_INVALID, "need n_streams > 0, 1 <= vocab <= 1024 and pitch_words > 0");
  std::unique_ptr<boa_pyrc> h(new boa_pyrc());
  h->device = device; h->N = n_streams; h->K = vocab; h->pitch = pitch_words;
  int n_dev = 0;
  cudaError_t e = cudaGetDeviceCount(&n_dev);
  if (e != cudaSuccess) return pyrc_cuda(nullptr, e, "cudaGetDeviceCount");
  if (device < 0 || device >= n_dev) return pyrc_fail(nullptr, BOA_E_CUDA, "no CUDA device " + std::to_string(device));
  DeviceGuard dev(device);
  if ((e = boa::pyrc_prepare()) != cudaSuccess) return pyrc_cuda(nullptr, e, "coder kernel setup");
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
  DeviceGuard dev(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  if (pyrc_bulk_ok(h, d_probs)) {
    const unsigned grid = (unsigned)((h->N + 32 * boa::kBulkWarps - 1) / (32 * boa::kBulkWarps));
    boa::pyrc_encode_bulk_kernel<<<grid, 32 * boa::kBulkWarps, boa::kPyBulkSmem, s>>>(
        d_symbols, d_probs, h->N, h->K, h->words, h->enc, h->pitch, d_mask);
  } else {
    const unsigned grid = (unsigned)((h->N + 32 * boa::kPyWarps - 1) / (32 * boa::kPyWarps));
    boa::pyrc_encode_kernel<<<grid, 32 * boa::kPyWarps, boa::kPyEncSmem, s>>>(d_symbols, d_probs, h->N, h->K,
                                                                             h->words, h->enc, h->pitch, d_mask);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "encode step launch");
}

int boa_pyrc_finalize(boa_pyrc* h, void* stream) {
  if (!h) return BOA_E_INVALID;
  DeviceGuard dev(h->device);
  boa::pyrc_finalize_kernel<<<(unsigned)((h->N + 127) / 128), 128, 0, (cudaStream_t)stream>>>(h->enc, h->words, h->sizes,
                                                                                              h->N, h->pitch);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "finalize launch");
}

int boa_pyrc_read(boa_pyrc* h, uint32_t* words_host, int32_t* sizes_host, void* stream) {
  if (!h || !sizes_host) return pyrc_fail(h, BOA_E_INVALID, "null argument");
  DeviceGuard dev(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(sizes_host, h->sizes, (size_t)h->N * 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && words_host)
    e = cudaMemcpyAsync(words_host, h->words, (size_t)h->N * h->pitch * 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return pyrc_cuda(h, e, "reading streams");
  int code = 0;
  if ((e = cudaMemcpyFromSymbol(&code, boa::g_dev_error, sizeof(int))) != cudaSuccess)
    return pyrc_cuda(h, e, "reading device error word");
  if (code != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(boa::g_dev_error, &zero, sizeof(int));
    return pyrc_fail(h, BOA_E_DEVICE, "a coder kernel's copy wait timed out");
  }
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
  DeviceGuard dev(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(h->words, words_host, (size_t)h->N * h->pitch * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(h->sizes, sizes_host, (size_t)h->N * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "loading streams");
}

int boa_pyrc_init_decoder(boa_pyrc* h, void* stream) {
  if (!h) return BOA_E_INVALID;
  DeviceGuard dev(h->device);
  boa::pyrc_init_dec_kernel<<<(unsigned)((h->N + 127) / 128), 128, 0, (cudaStream_t)stream>>>(h->words, h->sizes, h->dec,
                                                                                              h->N, h->pitch);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "decoder init launch");
}

int boa_pyrc_decode_step(boa_pyrc* h, const float* d_probs, int32_t* d_out_symbols, const uint8_t* d_mask,
                         void* stream) {
  if (!h || !d_probs || !d_out_symbols) return pyrc_fail(h, BOA_E_INVALID, "null argument");
  DeviceGuard dev(h->device);
  cudaStream_t s = (cudaStream_t)stream;
  if (pyrc_bulk_ok(h, d_probs)) {
    const unsigned grid = (unsigned)((h->N + 32 * boa::kBulkWarps - 1) / (32 * boa::kBulkWarps));
    boa::pyrc_decode_bulk_kernel<<<grid, 32 * boa::kBulkWarps, boa::kPyBulkSmem, s>>>(
        d_probs, h->N, h->K, h->words, h->sizes, h->dec, h->pitch, d_out_symbols, d_mask);
  } else {
    const unsigned grid = (unsigned)((h->N + 32 * boa::kPyWarps - 1) / (32 * boa::kPyWarps));
    boa::pyrc_decode_kernel<<<grid, 32 * boa::kPyWarps, boa::kPyDecSmem, s>>>(d_probs, h->N, h->K, h->words,
                                                                             h->sizes, h->dec, h->pitch,
                                                                             d_out_symbols, d_mask);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BOA_OK : pyrc_cuda(h, e, "decode step launch");
}

}  // extern "C"
