// runtime.cpp -- host runtime behind the C ABI: weight loading, device
// arenas, the per-layer launch schedule, and the compress / decompress drivers.
//
// Replaces BoaPredictorGPU / BoaBlockGPU / MambaBlockGPU / MinGRUBlockGPU
// (boa_gpu.hpp:95-1174) and the batch loops of compress_v2 / decompress_v2
// (boa.cpp:390-495, :672-774).
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/boa_b200.h"
#include "gemm.cuh"
#include "kernels.cuh"

using boa::DecState;
using boa::EncState;
using bf16 = __nv_bfloat16;

namespace {

std::string g_load_error;  // boa_model_load failures (no handle yet)

// Makes `device` current for the scope of an API call and restores the
// caller's current device afterwards: no entry point changes it.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != device) cudaSetDevice(device);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
};


struct HL {  // bf16 hi/lo weight planes, [2][N][K]
  bf16* p = nullptr;
  long long plane = 0;
  int N = 0, K = 0;
};

struct LayerW {
  float *ln1w, *ln1b, *ln2w, *ln2b, *ff1_b, *ff2_b;
  HL ff1, ff2;
  // mamba
  HL in, xp, out;
  float *in_b, *conv_w, *conv_b, *dt_w, *dt_b, *negA, *Dv, *out_b;
  // minGRU: [Wz; Wh] stacked into one N = 2d projection
  HL zh;
  float* zh_b;
  // LSTM / GRU: input and recurrent projections, N = G = 4d / 3d
  HL ih, hh;
  float *ih_b, *hh_b;
};

uint16_t f2bf(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

float half2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF, f;
  if (e == 0) {
    if (m == 0) f = sign;
    else { e = 1; while (!(m & 0x400)) { m <<= 1; e--; } m &= 0x3FF; f = sign | ((127 - 15 + e) << 23) | (m << 13); }
  } else if (e == 31) f = sign | 0x7F800000u | (m << 13);
  else f = sign | ((e - 15 + 127) << 23) | (m << 13);
  float r;
  std::memcpy(&r, &f, 4);
  return r;
}

struct FileReader {
  std::vector<uint8_t> buf;
  size_t off = 0;
  bool fp16 = false, ok = true;
  std::vector<float> vec(size_t n) {
    std::vector<float> v(n, 0.f);
    const size_t esz = fp16 ? 2 : 4;
    if (off + n * esz > buf.size()) { ok = false; return v; }
    if (fp16) {
      for (size_t i = 0; i < n; ++i) { uint16_t h; std::memcpy(&h, &buf[off + 2 * i], 2); v[i] = half2f(h); }
    } else {
      std::memcpy(v.data(), &buf[off], n * 4);
    }
    off += n * esz;
    return v;
  }
};

}  // namespace

struct boa_model {
  int device = 0, backbone = 0, d = 0, L = 0, di = 0, r = 0, xpN = 0;
  float inv_t = 1.0f;
  std::string err;
  cudaStream_t own = nullptr, ext = nullptr;
  bool has_ext = false;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  int cfg_batch = 0, cfg_tile = 0;
  uint32_t warm = 0;  // interleave batch of warm-start lanes (0 = off)

  // weights (one arena)
  void* warena = nullptr;
  size_t wbytes = 0;
  float* emb = nullptr;
  std::vector<LayerW> layers;
  float* final_norm = nullptr;
  HL h1, h2;
  float *h1_b = nullptr, *h2_b = nullptr;

  // work buffers (grow-only arena)
  void* work = nullptr;
  size_t work_bytes = 0, rows_cap = 0, chunks_cap = 0, pitch_cap = 0;
  float *x = nullptr, *xz = nullptr, *u = nullptr, *delta = nullptr;
  bf16 *xn = nullptr, *uhl = nullptr;
  float *conv_st = nullptr, *ssm_st = nullptr, *h_st = nullptr;
  float *c_st = nullptr, *hh = nullptr;  // LSTM cell state [L][chunks][d]; recurrent projection [chunks][G]
  bf16* h_hl = nullptr;                    // LSTM / GRU: h split into bf16 hi/lo, [L][2][chunks][d]
  uint2* lf = nullptr;
  EncState* es = nullptr;
  DecState* ds = nullptr;
  uint32_t* pitch_buf = nullptr;
  int* d_t = nullptr;
  // per-lane views (decode) and per-lane results (interleaved compress)
  unsigned long long* lane_off = nullptr;
  uint32_t* lane_size = nullptr;
  uint8_t* lane_first = nullptr;
  long long* lane_base = nullptr;
  int* lane_len = nullptr;
  // per-chunk stream slots for interleaved compress (grow-only)
  uint32_t* slots = nullptr;
  size_t slots_words = 0;
  float* logits = nullptr;
  size_t logits_rows = 0;

  // instrumentation
  bool prof = false;
  struct Pend { int cls; cudaEvent_t a, b; };
  std::vector<Pend> pending;
  std::vector<cudaEvent_t> ev_pool;
  double prof_ms[BOA_PROF_CLASSES] = {0};
  uint64_t prof_n[BOA_PROF_CLASSES] = {0};
  uint64_t launches = 0;

  // host-API staging (grow-only)
  void* io = nullptr;
  size_t io_bytes = 0;

  ~boa_model();
  cudaStream_t stream() const { return own; }
  size_t per_row_bytes() const { return (size_t)40 * d + 4 * (size_t)xpN + 64; }
  bool is_rnn() const { return backbone == BOA_BACKBONE_LSTM || backbone == BOA_BACKBONE_GRU; }
  int gates() const { return (backbone == BOA_BACKBONE_LSTM ? 4 : 3) * d; }
  size_t per_chunk_state_bytes() const {
    if (backbone == BOA_BACKBONE_MAMBA) return (size_t)L * 19 * di * 4;
    if (is_rnn()) return (size_t)L * d * (backbone == BOA_BACKBONE_LSTM ? 12 : 8) + (size_t)gates() * 4;
    return (size_t)L * d * 4;
  }
};

boa_model::~boa_model() {
  DeviceGuard dev(device);
  if (own) cudaStreamSynchronize(own);
  for (auto& p : pending) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
  for (auto e : ev_pool) cudaEventDestroy(e);
  if (warena) cudaFree(warena);
  if (work) cudaFree(work);
  if (slots) cudaFree(slots);
  if (io) cudaFree(io);
  if (logits) cudaFree(logits);
  if (ev_in) cudaEventDestroy(ev_in);
  if (ev_out) cudaEventDestroy(ev_out);
  if (own) cudaStreamDestroy(own);
}

namespace {

int fail(boa_model* m, int code, const std::string& msg) {
  if (m) m->err = msg; else g_load_error = msg;
  return code;
}
int cuda_fail(boa_model* m, cudaError_t e, const char* where) {
  return fail(m, BOA_E_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}
#define BOA_CK(call)                                    \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return cuda_fail(m, e_, #call); \
  } while (0)

// Kernel classes for the instrumentation counters.
enum ProfClass {
  PC_EMBED = 0, PC_IN_PROJ, PC_CONV, PC_X_PROJ, PC_SCAN, PC_OUT_PROJ_LN, PC_FF1, PC_FF2_LN, PC_HEAD1, PC_HEAD2_CODER,
  PC_ENCODE, PC_OTHER
};
// "ffn": the fused feed-forward kernel (d 64, 128, 256), or its first GEMM (other widths)
const char* const kProfNames[BOA_PROF_CLASSES] = {"embed_ln", "in_proj", "conv", "x_proj", "scan", "out_proj_ln",
                                                  "ffn", "ff2_res_ln", "head1", "head2_coder", "encode_tile",
                                                  "other"};

cudaEvent_t pool_event(boa_model* m) {
  if (!m->ev_pool.empty()) { cudaEvent_t e = m->ev_pool.back(); m->ev_pool.pop_back(); return e; }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Brackets one launch: counts it and, when profiling, records events.
struct Launch {
  boa_model* m;
  int cls;
  cudaEvent_t a = nullptr;
  Launch(boa_model* mm, int c) : m(mm), cls(c) {
    m->launches++;
    if (m->prof) { a = pool_event(m); cudaEventRecord(a, m->own); }
  }
  ~Launch() {
    if (a) {
      cudaEvent_t b = pool_event(m);
      cudaEventRecord(b, m->own);
      m->pending.push_back({cls, a, b});
    }
  }
};
#define BOA_LAUNCH(cls, call)    \
  do {                           \
    Launch l_(m, cls);           \
    BOA_CK(call);                \
  } while (0)

// Entry / exit ordering with an external stream (and the handle's device).
struct StreamScope {
  boa_model* m;
  DeviceGuard dev;
  explicit StreamScope(boa_model* mm) : m(mm), dev(mm->device) {
    if (m->has_ext) { cudaEventRecord(m->ev_in, m->ext); cudaStreamWaitEvent(m->own, m->ev_in, 0); }
  }
  ~StreamScope() {
    if (m->has_ext) { cudaEventRecord(m->ev_out, m->own); cudaStreamWaitEvent(m->ext, m->ev_out, 0); }
  }
};

// Ensure work buffers for `rows` activation rows and `chunks` recurrent
// states with per-chunk stream pitch `pitch` words.
int ensure_work(boa_model* m, size_t rows, size_t chunks, size_t pitch) {
  if (rows <= m->rows_cap && chunks <= m->chunks_cap && pitch <= m->pitch_cap) return 0;
  rows = std::max(rows, m->rows_cap);
  chunks = std::max(chunks, m->chunks_cap);
  pitch = std::max(pitch, m->pitch_cap);
  if (m->work) { cudaStreamSynchronize(m->own); cudaFree(m->work); m->work = nullptr; }
  const int d = m->d, di = m->di;
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  size_t off = 0;
  std::vector<std::pair<void**, size_t>> plan = {
      {(void**)&m->x, al(rows * d * 4)},
      {(void**)&m->xn, al(rows * d * 2 * 2)},
      {(void**)&m->xz, al(rows * 4 * d * 4)},
      {(void**)&m->u, al(rows * di * 4)},
      {(void**)&m->uhl, al(rows * di * 2 * 2)},
      {(void**)&m->delta, al(rows * (size_t)m->xpN * 4)},
      {(void**)&m->lf, al(rows * sizeof(uint2))},
      {(void**)&m->es, al(chunks * sizeof(EncState))},
      {(void**)&m->ds, al(chunks * sizeof(DecState))},
      {(void**)&m->pitch_buf, al(chunks * pitch * 4)},
      {(void**)&m->d_t, al(256)},
      {(void**)&m->lane_off, al(chunks * 8)},
      {(void**)&m->lane_size, al(chunks * 4)},
      {(void**)&m->lane_first, al(chunks)},
      {(void**)&m->lane_base, al(chunks * 8)},
      {(void**)&m->lane_len, al(chunks * 4)},
  };
  if (m->backbone == BOA_BACKBONE_MAMBA) {
    plan.push_back({(void**)&m->conv_st, al((size_t)m->L * chunks * 3 * di * 4)});
    plan.push_back({(void**)&m->ssm_st, al((size_t)m->L * chunks * 16 * di * 4)});
  } else {
    plan.push_back({(void**)&m->h_st, al((size_t)m->L * chunks * d * 4)});
    if (m->backbone == BOA_BACKBONE_LSTM) plan.push_back({(void**)&m->c_st, al((size_t)m->L * chunks * d * 4)});
    if (m->is_rnn()) {
      plan.push_back({(void**)&m->h_hl, al((size_t)m->L * 2 * chunks * d * 2)});
      plan.push_back({(void**)&m->hh, al(chunks * (size_t)m->gates() * 4)});
    }
  }
  for (auto& p : plan) off += p.second;
  void* base = nullptr;
  if (cudaMalloc(&base, off) != cudaSuccess) {
    cudaGetLastError();
    m->rows_cap = m->chunks_cap = m->pitch_cap = 0;
    return fail(m, BOA_E_NOMEM, "device allocation of " + std::to_string(off >> 20) + " MiB of work buffers failed");
  }
  m->work = base;
  m->work_bytes = off;
  size_t o = 0;
  for (auto& p : plan) { *p.first = (uint8_t*)base + o; o += p.second; }
  m->rows_cap = rows;
  m->chunks_cap = chunks;
  m->pitch_cap = pitch;
  return 0;
}

void* ensure_io(boa_model* m, size_t bytes) {
  if (bytes <= m->io_bytes) return m->io;
  if (m->io) { cudaStreamSynchronize(m->own); cudaFree(m->io); m->io = nullptr; m->io_bytes = 0; }
  if (cudaMalloc(&m->io, bytes) != cudaSuccess) { cudaGetLastError(); return nullptr; }
  m->io_bytes = bytes;
  return m->io;
}

// Zero the recurrent state of chunks [0, B) in every layer.  Layer l's
// slice starts at l * chunks_cap (the arrays are sized for the largest batch
// seen), so each layer is cleared separately.
int reset_states(boa_model* m, int B) {
  const size_t cap = m->chunks_cap;
  for (int l = 0; l < m->L; ++l) {
    if (m->backbone == BOA_BACKBONE_MAMBA) {
      BOA_CK(cudaMemsetAsync(m->conv_st + (size_t)l * cap * 3 * m->di, 0, (size_t)B * 3 * m->di * 4, m->own));
      BOA_CK(cudaMemsetAsync(m->ssm_st + (size_t)l * cap * 16 * m->di, 0, (size_t)B * 16 * m->di * 4, m->own));
    } else {
      BOA_CK(cudaMemsetAsync(m->h_st + (size_t)l * cap * m->d, 0, (size_t)B * m->d * 4, m->own));
      if (m->c_st) BOA_CK(cudaMemsetAsync(m->c_st + (size_t)l * cap * m->d, 0, (size_t)B * m->d * 4, m->own));
      if (m->h_hl)
        for (int p = 0; p < 2; ++p)
          BOA_CK(cudaMemsetAsync(m->h_hl + ((size_t)l * 2 + p) * cap * m->d, 0, (size_t)B * m->d * 2, m->own));
    }
  }
  return 0;
}

// One forward pass over B chunks x T positions (M = B*T rows).  States are
// laid out per layer for `chunks_cap`-wide batches: layer l's conv state is
// conv_st + l*chunks_cap*3*di.
int forward(boa_model* m, const boa::TokenSrc& src, int B, int T, int head_mode, boa::GemmArgs head) {
  const int M = B * T, d = m->d, di = m->di;
  const long long xn_plane = (long long)m->rows_cap * d, u_plane = (long long)m->rows_cap * di,
                  h_plane = (long long)m->rows_cap * 4 * d;
  cudaStream_t st = m->own;
  bf16* hhl = reinterpret_cast<bf16*>(m->xz);   // FF hidden aliases xz (dead after the scan)
  bf16* headh = reinterpret_cast<bf16*>(m->u);  // head hidden aliases u
  // the scan's y (bf16 hi / lo, plane u_plane) lives in u's fp32 buffer (rows
  // x di x 4 bytes = two bf16 planes): the Mamba conv writes u only as planes
  bf16* ybuf = reinterpret_cast<bf16*>(m->u);
  const long long head_plane = (long long)m->rows_cap * d;
  BOA_LAUNCH(PC_EMBED, boa::launch_embed_ln(src, m->emb, d, m->x, m->xn, xn_plane, m->layers[0].ln1w, m->layers[0].ln1b, M, st));
  for (int l = 0; l < m->L; ++l) {
    const LayerW& w = m->layers[l];
    const bool last = l + 1 == m->L;
    boa::GemmArgs a{};
    a.M = M;
    if (m->backbone == BOA_BACKBONE_MAMBA) {
      float* cst = m->conv_st + (size_t)l * m->chunks_cap * 3 * di;
      float* sst = m->ssm_st + (size_t)l * m->chunks_cap * 16 * di;
      a.N = 2 * di; a.K = d; a.bias = w.in_b; a.out_f32 = m->xz; a.ld_f32 = 2 * di;
      BOA_LAUNCH(PC_IN_PROJ, boa::gemm_launch(boa::EPI_F32, m->xn, xn_plane, 0, w.in.p, w.in.plane, a, st));
      BOA_LAUNCH(PC_CONV, boa::launch_conv(m->xz, di, cst, w.conv_w, w.conv_b, m->uhl, u_plane, B, T, src.pos0,
                                           src.d_pos, st));
      a = boa::GemmArgs{}; a.M = M;
      a.N = m->xpN; a.K = di; a.out_f32 = m->delta; a.ld_f32 = m->xpN;
      BOA_LAUNCH(PC_X_PROJ, boa::gemm_launch(boa::EPI_F32, m->uhl, u_plane, 0, w.xp.p, w.xp.plane, a, st));
      BOA_LAUNCH(PC_SCAN, boa::launch_scan(m->delta, m->xpN, m->r, w.dt_w, w.dt_b, w.negA, w.Dv, m->xz, di, sst, m->uhl, ybuf,
                              u_plane, B, T, st));
      a = boa::GemmArgs{}; a.M = M;
      a.N = d; a.K = di; a.bias = w.out_b; a.out_hl = m->xn; a.ld_hl = d; a.plane_hl = xn_plane;
      a.ln_w = w.ln2w; a.ln_b = w.ln2b;
      BOA_LAUNCH(PC_OUT_PROJ_LN, boa::gemm_launch(boa::EPI_LN_SPLIT, ybuf, u_plane, 0, w.out.p, w.out.plane, a, st));
    } else if (m->is_rnn()) {
      // ih for all M rows, then per position: hh (one row per chunk) and the gate update
      const int G = m->gates();
      const size_t cap = m->chunks_cap;
      float* hst = m->h_st + (size_t)l * cap * d;
      float* cst = m->c_st ? m->c_st + (size_t)l * cap * d : nullptr;
      bf16* hl = m->h_hl + (size_t)l * 2 * cap * d;
      a.N = G; a.K = d; a.bias = w.ih_b; a.out_f32 = m->xz; a.ld_f32 = G;
      BOA_LAUNCH(PC_IN_PROJ, boa::gemm_launch(boa::EPI_F32, m->xn, xn_plane, 0, w.ih.p, w.ih.plane, a, st));
      for (int t = 0; t < T; ++t) {
        boa::GemmArgs r{};
        r.M = B; r.N = G; r.K = d; r.bias = w.hh_b; r.out_f32 = m->hh; r.ld_f32 = G;
        BOA_LAUNCH(PC_X_PROJ, boa::gemm_launch(boa::EPI_F32, hl, (long long)cap * d, 0, w.hh.p, w.hh.plane, r, st));
        BOA_LAUNCH(PC_SCAN, boa::launch_rnn_gates(m->backbone == BOA_BACKBONE_LSTM, m->xz, m->hh, d, t, T, hst, cst,
                                                  hl, (long long)cap * d, m->u, B, st));
      }
      BOA_LAUNCH(PC_OTHER, boa::launch_add_ln(m->x, m->u, d, m->xn, xn_plane, w.ln2w, w.ln2b, M, st));
    } else {
      float* hst = m->h_st + (size_t)l * m->chunks_cap * d;
      a.N = 2 * d; a.K = d; a.bias = w.zh_b; a.out_f32 = m->xz; a.ld_f32 = 2 * d;
      BOA_LAUNCH(PC_IN_PROJ, boa::gemm_launch(boa::EPI_F32, m->xn, xn_plane, 0, w.zh.p, w.zh.plane, a, st));
      BOA_LAUNCH(PC_SCAN, boa::launch_mingru(m->xz, d, hst, m->u, B, T, st));
      BOA_LAUNCH(PC_OTHER, boa::launch_add_ln(m->x, m->u, d, m->xn, xn_plane, w.ln2w, w.ln2b, M, st));
    }
    if (d == 64 || d == 128 || d == 256) {  // fused feed-forward: the hidden activation stays on chip
      a = boa::GemmArgs{}; a.M = M;
      a.N = d; a.bias = w.ff2_b; a.res = m->x; a.out_hl = m->xn; a.ld_hl = d; a.plane_hl = xn_plane;
      if (!last) { a.ln_w = m->layers[l + 1].ln1w; a.ln_b = m->layers[l + 1].ln1b; }
      BOA_LAUNCH(PC_FF1, boa::mlp_launch(m->xn, xn_plane, w.ff1.p, w.ff1.plane, w.ff2.p, w.ff2.plane, w.ff1_b, a, st));
    } else {
      a = boa::GemmArgs{}; a.M = M;
      a.N = 4 * d; a.K = d; a.bias = w.ff1_b; a.out_hl = hhl; a.ld_hl = 4 * d; a.plane_hl = h_plane;
      a.act = boa::ACT_GELU;
      BOA_LAUNCH(PC_FF1, boa::gemm_launch(boa::EPI_ACT_SPLIT, m->xn, xn_plane, 0, w.ff1.p, w.ff1.plane, a, st));
      a = boa::GemmArgs{}; a.M = M;
      a.N = d; a.K = 4 * d; a.bias = w.ff2_b; a.res = m->x; a.out_hl = m->xn; a.ld_hl = d; a.plane_hl = xn_plane;
      if (!last) { a.ln_w = m->layers[l + 1].ln1w; a.ln_b = m->layers[l + 1].ln1b; }
      BOA_LAUNCH(PC_FF2_LN, boa::gemm_launch(boa::EPI_RES_LN, hhl, h_plane, 0, w.ff2.p, w.ff2.plane, a, st));
    }
  }
  if (m->backbone != BOA_BACKBONE_MAMBA)
    BOA_LAUNCH(PC_OTHER, boa::launch_rms_split(m->x, d, m->final_norm, m->xn, xn_plane, M, st));
  boa::GemmArgs a{};
  a.M = M; a.N = d; a.K = d; a.bias = m->h1_b; a.out_hl = headh; a.ld_hl = d; a.plane_hl = head_plane;
  a.act = m->backbone == BOA_BACKBONE_MAMBA ? boa::ACT_RELU : boa::ACT_SILU;
  BOA_LAUNCH(PC_HEAD1, boa::gemm_launch(boa::EPI_ACT_SPLIT, m->xn, xn_plane, 0, m->h1.p, m->h1.plane, a, st));
  head.M = M; head.N = 256; head.K = d; head.bias = m->h2_b; head.inv_t = m->inv_t;
  BOA_LAUNCH(PC_HEAD2_CODER, boa::gemm_launch(head_mode, headh, head_plane, 0, m->h2.p, m->h2.plane, head, st));
  return 0;
}

int read_dev_error(boa_model* m) {
  int code = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&code, boa::g_dev_error, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(m, e, "reading device error word");
  if (code != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(boa::g_dev_error, &zero, sizeof(int));
    return fail(m, BOA_E_DEVICE, code == boa::BOA_ERR_TIMEOUT ? "device wait timed out"
                                 : code == boa::BOA_ERR_STREAM_OVERFLOW ? "range-coded stream exceeded its capacity"
                                 : code == boa::BOA_ERR_BAD_INPUT
                                     ? "a CDF gives a coded symbol an empty interval or one above 2^24"
                                     : "device-side check failed");
  }
  return 0;
}

// Batch sizing: chunks per batch and tokens per compress tile.
void pick_batch(boa_model* m, uint32_t n_chunks, uint32_t chunk_len, bool compress, int& B, int& T) {
  T = compress ? (m->cfg_tile > 0 ? m->cfg_tile : 64) : 1;
  T = std::max(1, std::min<int>(T, (int)std::max<uint32_t>(1, chunk_len - 1)));
  if (m->cfg_batch > 0) {
    B = std::min<int>(m->cfg_batch, (int)n_chunks);
  } else {
    size_t free_b = 0, total = 0;
    cudaMemGetInfo(&free_b, &total);
    free_b += m->work_bytes;
    const size_t budget = (size_t)(free_b * 0.8);
    const size_t pitch = boa_stream_capacity_words(chunk_len);
    const size_t per_chunk = m->per_chunk_state_bytes() + (size_t)T * m->per_row_bytes() + pitch * 4 + 128;
    size_t b = std::max<size_t>(1, budget / per_chunk);
    b = std::min<size_t>(b, 65536);
    B = (int)std::min<size_t>(b, n_chunks);
  }
  B = std::max(1, B);
}

}  // namespace

// Warm-start compress (boa.cpp:313-319, :395-435): W lanes, S = ceil(n/W)
// iterations; in iteration `iter` lane b codes chunk iter + b*S with the model
// state it carried from chunk iter - 1 + b*S (reset only at iter 0); every
// chunk still gets its own range coder and raw first byte.
int compress_interleaved(boa_model* m, const uint8_t* d_data, uint64_t n, uint32_t chunk_len, uint32_t n_chunks,
                         uint8_t* d_first, uint32_t* d_payload, uint32_t* d_sizes, uint64_t* d_offsets) {
  const int W = (int)std::min<uint32_t>(m->warm, n_chunks);
  const int S = (int)((n_chunks + W - 1) / W);
  const uint32_t pitch = boa_stream_capacity_words(chunk_len);
  int T = m->cfg_tile > 0 ? m->cfg_tile : 64;
  T = std::max(1, std::min<int>(T, (int)std::max<uint32_t>(1, chunk_len - 1)));
  if (int rc = ensure_work(m, (size_t)W * T, W, pitch)) return rc;
  const size_t need = (size_t)n_chunks * pitch;
  if (need > m->slots_words) {
    if (m->slots) { cudaStreamSynchronize(m->own); cudaFree(m->slots); m->slots = nullptr; m->slots_words = 0; }
    if (cudaMalloc(&m->slots, need * 4) != cudaSuccess) {
      cudaGetLastError();
      return fail(m, BOA_E_NOMEM, "device allocation of per-chunk stream slots failed");
    }
    m->slots_words = need;
  }
  cudaStream_t st = m->own;
  uint32_t* lane_sizes = reinterpret_cast<uint32_t*>(m->lane_off);  // reuse per-lane scratch
  if (int rc = reset_states(m, W)) return rc;
  for (int iter = 0; iter < S; ++iter) {
    int cur = 0;
    while (cur < W && (uint64_t)cur * S + iter < n_chunks) ++cur;
    if (cur == 0) break;
    const uint8_t* data = d_data + (size_t)iter * chunk_len;
    const long long rem = (long long)(n - (uint64_t)iter * chunk_len);
    const long long stride = (long long)S * chunk_len;
    BOA_LAUNCH(PC_OTHER, boa::launch_enc_init(m->es, cur, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_first_bytes(data, rem, chunk_len, stride, m->lane_first, cur, st));
    // the carried state must have consumed exactly the chunk's bytes (all
    // chunk_len positions, as forward_chunk does), so the last tile is
    // shortened instead of padded
    for (int t0 = 0; t0 < (int)chunk_len; t0 += T) {
      const int Tt = std::min<int>(T, (int)chunk_len - t0);
      // lanes carry their state from chunk to chunk: positions continue at iter * chunk_len
      boa::TokenSrc src{1, data, rem, (int)chunk_len, t0, Tt, nullptr, stride, nullptr, nullptr,
                        (long long)iter * chunk_len + t0, nullptr};
      boa::GemmArgs h{};
      h.tokens = data; h.n_bytes = rem; h.chunk_len = (int)chunk_len; h.stride = stride; h.t0 = t0; h.T = Tt;
      h.lf = m->lf;
      if (int rc = forward(m, src, cur, Tt, boa::EPI_HEAD_ENC, h)) return rc;
      BOA_LAUNCH(PC_ENCODE, boa::launch_encode_tile(m->lf, m->es, m->pitch_buf, (int)pitch, cur, Tt, t0, rem,
                                                    (int)chunk_len, stride, st));
    }
    BOA_LAUNCH(PC_OTHER, boa::launch_enc_finish(m->es, m->pitch_buf, (int)pitch, lane_sizes, cur, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_lanes_scatter(m->pitch_buf, (int)pitch, lane_sizes, m->lane_first, m->slots,
                                                   d_sizes, d_first, iter, S, cur, st));
  }
  for (uint32_t c0 = 0; c0 < n_chunks; c0 += (uint32_t)W) {
    const int Bb = (int)std::min<uint32_t>(W, n_chunks - c0);
    BOA_LAUNCH(PC_OTHER, boa::launch_offsets(d_sizes + c0, (unsigned long long*)d_offsets + c0, Bb, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_compact(m->slots + (size_t)c0 * pitch, (int)pitch, d_sizes + c0,
                                             (unsigned long long*)d_offsets + c0, d_payload, Bb, st));
  }
  return 0;
}

// =============================================================================
extern "C" {

uint32_t boa_stream_capacity_words(uint32_t chunk_len) {
  // <= 24 + log2(256/255) bits per coded byte, plus two init and two flush words
  const uint64_t bits = (uint64_t)chunk_len * 2401 / 100 + 1;
  return (uint32_t)((bits + 31) / 32 + 8);
}

const char* boa_last_error(const boa_model* h) { return h ? h->err.c_str() : g_load_error.c_str(); }

int boa_model_load(const char* path, int backbone, int d, int nl, int device, boa_model** out) {
  if (!out) return fail(nullptr, BOA_E_INVALID, "out is NULL");
  *out = nullptr;
  if (backbone < BOA_BACKBONE_MAMBA || backbone > BOA_BACKBONE_MINGRU)
    return fail(nullptr, BOA_E_INVALID, "backbone must be mamba (0), lstm (1), gru (2) or mingru (3)");
  // widths of the reference's checkpoints (mamba d 64 / 80 / 128, minGRU d 160 / 256) and the configs
  const bool rnn = backbone == BOA_BACKBONE_LSTM || backbone == BOA_BACKBONE_GRU;
  const bool d_ok = d == 64 || d == 128 || d == 256 || d == 512 || (!rnn && (d == 80 || d == 160));
  if (!d_ok || nl <= 0 || nl > 256)
    return fail(nullptr, BOA_E_INVALID,
                "d_model must be 64, 80, 128, 160, 256 or 512 (LSTM / GRU: 64, 128, 256 or 512) and n_layers "
                "in 1..256");
  FileReader R;
  {
    FILE* f = path ? std::fopen(path, "rb") : nullptr;
    if (!f) return fail(nullptr, BOA_E_IO, std::string("cannot open weights: ") + (path ? path : "(null)"));
    std::fseek(f, 0, SEEK_END);
    long sz = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    R.buf.resize(sz > 0 ? (size_t)sz : 0);
    size_t got = sz > 0 ? std::fread(R.buf.data(), 1, (size_t)sz, f) : 0;
    std::fclose(f);
    if (got != R.buf.size()) return fail(nullptr, BOA_E_IO, "short read on weights");
  }
  if (R.buf.size() >= 4 && R.buf[0] == 'B' && R.buf[1] == 'O' && R.buf[2] == 'A') {
    if (R.buf[3] > 1) return fail(nullptr, BOA_E_FORMAT, "unknown BOA weight format byte");
    R.fp16 = R.buf[3] == 1;
    R.off = 4;
  }
  std::unique_ptr<boa_model> m(new boa_model());
  m->device = device; m->backbone = backbone; m->d = d; m->L = nl; m->di = 2 * d;
  // dt_rank = ceil(d / 16) in the file; the scan runs 4, 8, 16 or 32 dt inputs, so an odd rank (d 80: 5,
  // d 160: 10) is zero-padded: x_proj gets zero rows after its dt rows and dt_proj zero columns, which
  // add exact zeros to the dt dot product
  const int r = (d + 15) / 16;
  m->r = r <= 4 ? 4 : r <= 8 ? 8 : r <= 16 ? 16 : 32;
  m->xpN = ((m->r + 32 + 15) / 16) * 16;
  const int di = m->di, rp = m->r;

  // ---- parse in file order into host vectors (boa_gpu.hpp:990-1029)
  struct HostHL { std::vector<uint16_t> v; int N, K; };
  auto make_hl = [](const std::vector<float>& w, int N, int K, int Npad) {
    HostHL h; h.N = Npad; h.K = K; h.v.assign((size_t)2 * Npad * K, 0);
    for (int n = 0; n < N; ++n)
      for (int k = 0; k < K; ++k) {
        const float x = w[(size_t)n * K + k];
        const uint16_t hi = f2bf(x);
        h.v[(size_t)n * K + k] = hi;
        h.v[(size_t)Npad * K + (size_t)n * K + k] = f2bf(x - bf2f(hi));
      }
    return h;
  };
  std::vector<std::vector<float>> f32s;   // fp32 tensors in upload order
  std::vector<HostHL> hls;                 // bf16 pairs in upload order
  std::vector<float> emb = R.vec((size_t)256 * d);
  struct LIdx { int ln1w, ln1b, ln2w, ln2b, ff1_b, ff2_b, in_b, conv_w, conv_b, dt_w, dt_b, negA, Dv, out_b, zh_b;
                int ff1, ff2, in, xp, out, zh, ih, ih_b, hh, hh_b; };
  std::vector<LIdx> li(nl);
  auto addf = [&](std::vector<float> v) { f32s.push_back(std::move(v)); return (int)f32s.size() - 1; };
  auto addh = [&](HostHL h) { hls.push_back(std::move(h)); return (int)hls.size() - 1; };
  for (int l = 0; l < nl; ++l) {
    LIdx& x = li[l];
    x = LIdx{};
    x.ln1w = addf(R.vec(d)); x.ln1b = addf(R.vec(d));
    if (backbone == BOA_BACKBONE_MAMBA) {
      x.in = addh(make_hl(R.vec((size_t)2 * di * d), 2 * di, d, 2 * di));
      x.in_b = addf(R.vec(2 * di));
      x.conv_w = addf(R.vec((size_t)di * 4));
      x.conv_b = addf(R.vec(di));
      {
        // x_proj rows [dt (r) | B (16) | C (16)] -> [dt (r) | 0 (rp - r) | B | C]
        const std::vector<float> xw = R.vec((size_t)(r + 32) * di);
        std::vector<float> xp((size_t)(rp + 32) * di, 0.f);
        std::copy(xw.begin(), xw.begin() + (size_t)r * di, xp.begin());
        std::copy(xw.begin() + (size_t)r * di, xw.end(), xp.begin() + (size_t)rp * di);
        x.xp = addh(make_hl(xp, rp + 32, di, m->xpN));
        // dt_proj [di][r] -> [di][rp]
        const std::vector<float> dw = R.vec((size_t)di * r);
        std::vector<float> dtw((size_t)di * rp, 0.f);
        for (int c = 0; c < di; ++c) std::copy(dw.begin() + (size_t)c * r, dw.begin() + (size_t)(c + 1) * r,
                                               dtw.begin() + (size_t)c * rp);
        x.dt_w = addf(std::move(dtw));
      }
      x.dt_b = addf(R.vec(di));
      std::vector<float> alog = R.vec((size_t)di * 16);
      // stored as A * log2(e) with A = -exp(A_log): the scan evaluates exp(A dt) as 2^(na2 dt)
      for (auto& a : alog) a = -std::exp(a) * 1.44269504088896340736f;
      x.negA = addf(std::move(alog));
      x.Dv = addf(R.vec(di));
      x.out = addh(make_hl(R.vec((size_t)d * di), d, di, d));
      x.out_b = addf(R.vec(d));
    } else if (backbone == BOA_BACKBONE_LSTM || backbone == BOA_BACKBONE_GRU) {
      // w_ih [G][d], b_ih, w_hh [G][d], b_hh (boa_gpu.hpp:413-419, :526-532)
      const int G = (backbone == BOA_BACKBONE_LSTM ? 4 : 3) * d;
      x.ih = addh(make_hl(R.vec((size_t)G * d), G, d, G));
      x.ih_b = addf(R.vec(G));
      x.hh = addh(make_hl(R.vec((size_t)G * d), G, d, G));
      x.hh_b = addf(R.vec(G));
    } else {
      std::vector<float> wz = R.vec((size_t)d * d), bz = R.vec(d), wh = R.vec((size_t)d * d), bh = R.vec(d);
      wz.insert(wz.end(), wh.begin(), wh.end());
      bz.insert(bz.end(), bh.begin(), bh.end());
      x.zh = addh(make_hl(wz, 2 * d, d, 2 * d));
      x.zh_b = addf(std::move(bz));
    }
    x.ln2w = addf(R.vec(d)); x.ln2b = addf(R.vec(d));
    x.ff1 = addh(make_hl(R.vec((size_t)4 * d * d), 4 * d, d, 4 * d));
    x.ff1_b = addf(R.vec(4 * d));
    x.ff2 = addh(make_hl(R.vec((size_t)4 * d * d), d, 4 * d, d));
    x.ff2_b = addf(R.vec(d));
  }
  int fnorm = -1;
  if (backbone != BOA_BACKBONE_MAMBA) fnorm = addf(R.vec(d));
  int h1 = addh(make_hl(R.vec((size_t)d * d), d, d, d));
  int h1b = addf(R.vec(d));
  int h2 = addh(make_hl(R.vec((size_t)256 * d), 256, d, 256));
  int h2b = addf(R.vec(256));
  if (!R.ok || R.off != R.buf.size())
    return fail(nullptr, BOA_E_FORMAT,
                "weight file size does not match d_model=" + std::to_string(d) + " n_layers=" + std::to_string(nl) +
                    " (parsed " + std::to_string(R.off) + " of " + std::to_string(R.buf.size()) + " bytes)");

  // ---- upload into one arena
  int n_dev = 0;
  cudaError_t e = cudaGetDeviceCount(&n_dev);
  if (e != cudaSuccess || device < 0 || device >= n_dev)
    return fail(nullptr, BOA_E_CUDA, std::string("no CUDA device ") + std::to_string(device) +
                                         (e != cudaSuccess ? std::string(": ") + cudaGetErrorString(e) : ""));
  DeviceGuard dev(device);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  size_t total = al(emb.size() * 4);
  for (auto& v : f32s) total += al(v.size() * 4);
  for (auto& h : hls) total += al(h.v.size() * 2);
  if ((e = cudaMalloc(&m->warena, total)) != cudaSuccess) {
    cudaGetLastError();
    return fail(nullptr, BOA_E_NOMEM, std::string("weights cudaMalloc: ") + cudaGetErrorString(e));
  }
  m->wbytes = total;
  uint8_t* p = (uint8_t*)m->warena;
  std::vector<float*> fp(f32s.size());
  std::vector<HL> hp(hls.size());
  auto up = [&](const void* src, size_t bytes) {
    void* dst = p;
    p += al(bytes);
    return cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice) == cudaSuccess ? dst : nullptr;
  };
  bool ok = true;
  m->emb = (float*)up(emb.data(), emb.size() * 4); ok &= m->emb != nullptr;
  for (size_t i = 0; i < f32s.size(); ++i) { fp[i] = (float*)up(f32s[i].data(), f32s[i].size() * 4); ok &= fp[i] != nullptr; }
  for (size_t i = 0; i < hls.size(); ++i) {
    hp[i].p = (bf16*)up(hls[i].v.data(), hls[i].v.size() * 2);
    hp[i].plane = (long long)hls[i].N * hls[i].K;
    hp[i].N = hls[i].N; hp[i].K = hls[i].K;
    ok &= hp[i].p != nullptr;
  }
  if (!ok) return fail(nullptr, BOA_E_CUDA, "weight upload failed");
  m->layers.resize(nl);
  for (int l = 0; l < nl; ++l) {
    const LIdx& x = li[l];
    LayerW& w = m->layers[l];
    w = LayerW{};
    w.ln1w = fp[x.ln1w]; w.ln1b = fp[x.ln1b]; w.ln2w = fp[x.ln2w]; w.ln2b = fp[x.ln2b];
    w.ff1 = hp[x.ff1]; w.ff1_b = fp[x.ff1_b]; w.ff2 = hp[x.ff2]; w.ff2_b = fp[x.ff2_b];
    if (backbone == BOA_BACKBONE_MAMBA) {
      w.in = hp[x.in]; w.in_b = fp[x.in_b]; w.conv_w = fp[x.conv_w]; w.conv_b = fp[x.conv_b];
      w.xp = hp[x.xp]; w.dt_w = fp[x.dt_w]; w.dt_b = fp[x.dt_b]; w.negA = fp[x.negA]; w.Dv = fp[x.Dv];
      w.out = hp[x.out]; w.out_b = fp[x.out_b];
    } else if (backbone == BOA_BACKBONE_LSTM || backbone == BOA_BACKBONE_GRU) {
      w.ih = hp[x.ih]; w.ih_b = fp[x.ih_b]; w.hh = hp[x.hh]; w.hh_b = fp[x.hh_b];
    } else {
      w.zh = hp[x.zh]; w.zh_b = fp[x.zh_b];
    }
  }
  if (fnorm >= 0) m->final_norm = fp[fnorm];
  m->h1 = hp[h1]; m->h1_b = fp[h1b]; m->h2 = hp[h2]; m->h2_b = fp[h2b];
  if ((e = boa::gemm_prepare_device()) != cudaSuccess || (e = boa::scan_prepare_device()) != cudaSuccess ||
      (e = boa::mlp_prepare_device()) != cudaSuccess)
    return fail(nullptr, BOA_E_CUDA, std::string("GEMM kernel setup: ") + cudaGetErrorString(e));
  if ((e = cudaStreamCreateWithFlags(&m->own, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming)) != cudaSuccess)
    return fail(nullptr, BOA_E_CUDA, std::string("stream/event create: ") + cudaGetErrorString(e));
  *out = m.release();
  return BOA_OK;
}

void boa_model_free(boa_model* h) { delete h; }

int boa_set_temperature(boa_model* m, float t) {
  if (!m) return BOA_E_INVALID;
  if (!(t > 0.0f) || !std::isfinite(t)) return fail(m, BOA_E_INVALID, "temperature must be > 0");
  m->inv_t = 1.0f / t;
  return 0;
}

int boa_set_stream(boa_model* m, void* s) {
  if (!m) return BOA_E_INVALID;
  m->ext = (cudaStream_t)s;
  m->has_ext = true;
  return 0;
}

int boa_set_warm_start(boa_model* m, uint32_t interleave_batch) {
  if (!m) return BOA_E_INVALID;
  m->warm = interleave_batch;
  return 0;
}

int boa_set_batch(boa_model* m, int chunks, int tile) {
  if (!m) return BOA_E_INVALID;
  if (chunks < 0 || tile < 0) return fail(m, BOA_E_INVALID, "batch and tile must be >= 0");
  m->cfg_batch = chunks;
  m->cfg_tile = tile;
  return 0;
}

int boa_batch_geometry(boa_model* m, uint32_t n_chunks, uint32_t chunk_len, int compress, int* chunks, int* tile) {
  if (!m) return BOA_E_INVALID;
  if (!chunks || !tile || n_chunks == 0 || chunk_len == 0)
    return fail(m, BOA_E_INVALID, "boa_batch_geometry: null output or empty geometry");
  DeviceGuard dev(m->device);
  int B, T;
  if (m->warm) {
    B = (int)std::min<uint32_t>(m->warm, n_chunks);
    T = compress ? std::max(1, std::min<int>(m->cfg_tile > 0 ? m->cfg_tile : 64, (int)std::max<uint32_t>(1, chunk_len - 1))) : 1;
  } else {
    pick_batch(m, n_chunks, chunk_len, compress != 0, B, T);
  }
  *chunks = B;
  *tile = T;
  return 0;
}

int boa_reserve(boa_model* m, uint32_t n_chunks, uint32_t chunk_len) {
  if (!m) return BOA_E_INVALID;
  if (n_chunks == 0 || chunk_len == 0) return fail(m, BOA_E_INVALID, "boa_reserve: empty geometry");
  DeviceGuard dev(m->device);
  int B, T;
  if (m->warm) {
    B = (int)std::min<uint32_t>(m->warm, n_chunks);
    T = std::max(1, std::min<int>(m->cfg_tile > 0 ? m->cfg_tile : 64, (int)std::max<uint32_t>(1, chunk_len - 1)));
  } else {
    pick_batch(m, n_chunks, chunk_len, true, B, T);
  }
  const uint32_t pitch = boa_stream_capacity_words(chunk_len);
  if (int rc = ensure_work(m, (size_t)B * T, B, pitch)) return rc;  // the compress form; decode needs less
  // staging of the host-buffer calls (boa_compress_chunks / boa_decompress_chunks) for this geometry
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t nb = (size_t)n_chunks * chunk_len, words = (size_t)n_chunks * pitch;
  const size_t io = std::max(al(nb) + al(n_chunks) + al(words * 4) + al((size_t)n_chunks * 4) +
                                 al(((size_t)n_chunks + 1) * 8),
                             al(words * 4 + 4) + al((size_t)n_chunks * 4) + al(((size_t)n_chunks + 1) * 8) +
                                 al(n_chunks) + al(nb));
  if (!ensure_io(m, io)) return fail(m, BOA_E_NOMEM, "boa_reserve: device staging allocation failed");
  return 0;
}

uint64_t boa_device_bytes(const boa_model* m) {
  return m ? (uint64_t)(m->wbytes + m->work_bytes + m->io_bytes) : 0;
}

int boa_selftest_wait_timeout(int device, uint32_t limit_us) {
  int n_dev = 0;
  if (cudaGetDeviceCount(&n_dev) != cudaSuccess || device < 0 || device >= n_dev) {
    cudaGetLastError();
    return fail(nullptr, BOA_E_INVALID, "no such CUDA device");
  }
  if (limit_us == 0 || limit_us > 1000000u) return fail(nullptr, BOA_E_INVALID, "limit_us must be in [1, 1e6]");
  DeviceGuard dev(device);
  int code = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&code, boa::g_dev_error, sizeof(int));
  if (e == cudaSuccess && code != 0) return fail(nullptr, BOA_E_DEVICE, "device error word was already set");
  int* d_ok = nullptr;
  if ((e = cudaMalloc(&d_ok, sizeof(int))) != cudaSuccess) return cuda_fail(nullptr, e, "self-test allocation");
  e = boa::launch_wait_selftest((uint64_t)limit_us * 1000ull, d_ok);
  int ok = -1;
  if (e == cudaSuccess) e = cudaMemcpy(&ok, d_ok, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d_ok);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "self-test launch");
  if (int rc = read_dev_error(nullptr)) return rc;  // expected: the wait ran out
  return fail(nullptr, BOA_E_CUDA, ok ? "self-test barrier completed without an arrival" : "no error recorded");
}

int boa_sync(boa_model* m) {
  if (!m) return BOA_E_INVALID;
  DeviceGuard dev(m->device);
  BOA_CK(cudaStreamSynchronize(m->own));
  if (m->has_ext) BOA_CK(cudaStreamSynchronize(m->ext));
  return read_dev_error(m);
}

int boa_compress_device(boa_model* m, const uint8_t* d_data, uint64_t n, uint32_t chunk_len, uint32_t n_chunks,
                        uint8_t* d_first, uint32_t* d_payload, uint64_t cap_words, uint32_t* d_sizes,
                        uint64_t* d_offsets) {
  if (!m) return BOA_E_INVALID;
  if (chunk_len == 0 || n_chunks == 0 || (uint64_t)(n_chunks - 1) * chunk_len >= n)
    return fail(m, BOA_E_INVALID, "chunk geometry does not match n_bytes");
  const uint32_t pitch = boa_stream_capacity_words(chunk_len);
  if (cap_words < (uint64_t)n_chunks * pitch)
    return fail(m, BOA_E_INVALID, "payload capacity below n_chunks * boa_stream_capacity_words(chunk_len)");
  StreamScope scope(m);
  int B, T;
  pick_batch(m, n_chunks, chunk_len, true, B, T);
  if (int rc = ensure_work(m, (size_t)B * T, B, pitch)) return rc;
  cudaStream_t st = m->own;
  BOA_CK(cudaMemsetAsync(d_offsets, 0, sizeof(uint64_t), st));
  if (m->warm) return compress_interleaved(m, d_data, n, chunk_len, n_chunks, d_first, d_payload, d_sizes, d_offsets);
  for (uint32_t c0 = 0; c0 < n_chunks; c0 += B) {
    const int Bb = (int)std::min<uint32_t>(B, n_chunks - c0);
    const uint8_t* data = d_data + (size_t)c0 * chunk_len;
    const long long rem = (long long)(n - (uint64_t)c0 * chunk_len);
    if (int rc = reset_states(m, Bb)) return rc;
    BOA_LAUNCH(PC_OTHER, boa::launch_enc_init(m->es, Bb, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_first_bytes(data, rem, chunk_len, 0, d_first + c0, Bb, st));
    const int max_len = (int)std::min<long long>(chunk_len, rem);
    for (int t0 = 0; t0 < max_len - 1; t0 += T) {
      boa::TokenSrc src{1, data, rem, (int)chunk_len, t0, T, nullptr, 0, nullptr, nullptr, t0, nullptr};
      boa::GemmArgs h{};
      h.tokens = data; h.n_bytes = rem; h.chunk_len = (int)chunk_len; h.t0 = t0; h.T = T; h.lf = m->lf;
      if (int rc = forward(m, src, Bb, T, boa::EPI_HEAD_ENC, h)) return rc;
      BOA_LAUNCH(PC_ENCODE, boa::launch_encode_tile(m->lf, m->es, m->pitch_buf, (int)pitch, Bb, T, t0, rem,
                                                    (int)chunk_len, 0, st));
    }
    BOA_LAUNCH(PC_OTHER, boa::launch_enc_finish(m->es, m->pitch_buf, (int)pitch, d_sizes + c0, Bb, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_offsets(d_sizes + c0, (unsigned long long*)d_offsets + c0, Bb, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_compact(m->pitch_buf, (int)pitch, d_sizes + c0, (unsigned long long*)d_offsets + c0, d_payload,
                               Bb, st));
  }
  return 0;
}

int boa_decompress_device(boa_model* m, const uint32_t* d_payload, const uint64_t* d_offsets, const uint32_t* d_sizes,
                          const uint8_t* d_first, uint64_t n, uint32_t chunk_len, uint32_t n_chunks, uint8_t* d_out) {
  if (!m) return BOA_E_INVALID;
  if (chunk_len == 0 || n_chunks == 0 || (uint64_t)(n_chunks - 1) * chunk_len >= n)
    return fail(m, BOA_E_INVALID, "chunk geometry does not match n_bytes");
  StreamScope scope(m);
  // lanes: warm start -> W lanes over S interleaved iterations (lane b holds
  // chunk iter + b*S, state carried); otherwise batches of consecutive chunks
  int B, T;
  int S = 1, iters;
  if (m->warm) {
    B = (int)std::min<uint32_t>(m->warm, n_chunks);
    S = (int)((n_chunks + B - 1) / B);
    iters = S;
  } else {
    pick_batch(m, n_chunks, chunk_len, false, B, T);
    iters = (int)((n_chunks + B - 1) / B);
  }
  if (int rc = ensure_work(m, (size_t)B, B, 1)) return rc;
  cudaStream_t st = m->own;
  cudaGraphExec_t exec = nullptr;
  int exec_lanes = -1;
  uint64_t per_step = 0;
  auto done = [&](int rc) {
    if (exec) cudaGraphExecDestroy(exec);
    return rc;
  };
  for (int it = 0; it < iters; ++it) {
    const int c0 = m->warm ? it : it * B;
    int cur;
    if (m->warm) {
      cur = 0;
      while (cur < B && (uint64_t)cur * S + c0 < n_chunks) ++cur;
    } else {
      cur = (int)std::min<uint32_t>(B, n_chunks - (uint32_t)c0);
    }
    if (cur <= 0) break;
    if (!m->warm || it == 0)
      if (int rc = reset_states(m, cur)) return done(rc);
    BOA_LAUNCH(PC_OTHER, boa::launch_lanes_gather((const unsigned long long*)d_offsets, d_sizes, d_first, (long long)n,
                                                  (int)chunk_len, c0, S, cur, m->lane_off, m->lane_size,
                                                  m->lane_first, m->lane_base, m->lane_len, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_dec_init(m->ds, d_payload, m->lane_off, m->lane_size, m->lane_first, d_out,
                                              m->lane_base, m->lane_len, cur, st));
    BOA_LAUNCH(PC_OTHER, boa::launch_set_counter(m->d_t, 1, st));
    // input position of step 1 (d_t[1], advanced with d_t[0]): warm-start lanes
    // continue from the previous chunk, at it * chunk_len
    BOA_LAUNCH(PC_OTHER, boa::launch_set_counter(m->d_t + 1, m->warm ? (int)(((long long)it * chunk_len) % 3) : 0, st));
    const int max_len = (int)std::min<long long>(chunk_len, (long long)n - (long long)c0 * chunk_len);
    if (max_len <= 1 && !m->warm) continue;
    boa::TokenSrc src{2, d_out, (long long)n, (int)chunk_len, 0, 1, m->d_t, 0, m->lane_base, m->lane_len, 0, m->d_t + 1};
    boa::GemmArgs h{};
    h.out_bytes = d_out; h.n_bytes = (long long)n; h.chunk_len = (int)chunk_len; h.d_t = m->d_t; h.dstates = m->ds;
    h.payload = d_payload; h.offsets = m->lane_off; h.lane_base = m->lane_base; h.lane_len = m->lane_len;
    if (m->prof) {  // eager steps so every launch is bracketed by events
      for (int t = 1; t <= (m->warm ? max_len : max_len - 1); ++t) {
        if (int rc = forward(m, src, cur, 1, boa::EPI_HEAD_DEC, h)) return done(rc);
        BOA_LAUNCH(PC_OTHER, boa::launch_increment(m->d_t, st));
      }
      continue;
    }
    if (exec_lanes != cur) {
      // capture one step (model + fused decode + counter); every per-lane
      // quantity is read from device arrays, so the graph serves every
      // iteration with this many lanes (boa.cpp:736-756)
      if (exec) { cudaGraphExecDestroy(exec); exec = nullptr; }
      cudaGraph_t graph = nullptr;
      const uint64_t l0 = m->launches;
      BOA_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      int rc = forward(m, src, cur, 1, boa::EPI_HEAD_DEC, h);
      cudaError_t ei = boa::launch_increment(m->d_t, st);
      cudaError_t ee = cudaStreamEndCapture(st, &graph);
      per_step = m->launches - l0 + 1;
      m->launches = l0;
      if (rc) { if (graph) cudaGraphDestroy(graph); return done(rc); }
      if (ei != cudaSuccess) { if (graph) cudaGraphDestroy(graph); return done(cuda_fail(m, ei, "capture increment")); }
      if (ee != cudaSuccess) return done(cuda_fail(m, ee, "cudaStreamEndCapture"));
      cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) { exec = nullptr; return done(cuda_fail(m, e, "cudaGraphInstantiate")); }
      exec_lanes = cur;
    }
    // warm start: one more step feeds the chunk's last byte into the carried
    // state (the encoder's forward pass consumed it); no byte is decoded then
    const int steps = m->warm ? max_len : max_len - 1;
    for (int t = 1; t <= steps; ++t) {
      cudaError_t e = cudaGraphLaunch(exec, st);
      if (e != cudaSuccess) return done(cuda_fail(m, e, "cudaGraphLaunch"));
      m->launches += per_step;
    }
  }
  return done(0);
}

int boa_compress_chunks(boa_model* m, const uint8_t* data, size_t n, uint32_t chunk_len, uint32_t first_chunk,
                        uint32_t n_chunks, uint8_t* first_bytes, uint32_t* payload, size_t cap_words,
                        uint32_t* sizes, uint64_t* total_out) {
  if (!m) return BOA_E_INVALID;
  if (!data || !first_bytes || !sizes || chunk_len == 0 || n_chunks == 0)
    return fail(m, BOA_E_INVALID, "null buffer or empty range");
  const uint64_t c0 = (uint64_t)first_chunk * chunk_len;
  if (c0 + (uint64_t)(n_chunks - 1) * chunk_len >= n) return fail(m, BOA_E_INVALID, "chunk range beyond the data");
  const uint64_t nb = std::min<uint64_t>(n - c0, (uint64_t)n_chunks * chunk_len);
  const uint32_t pitch = boa_stream_capacity_words(chunk_len);
  const size_t dev_words = (size_t)n_chunks * pitch;
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t need = al(nb) + al(n_chunks) + al(dev_words * 4) + al((size_t)n_chunks * 4) + al(((size_t)n_chunks + 1) * 8);
  {
    StreamScope scope(m);
    uint8_t* io = (uint8_t*)ensure_io(m, need);
    if (!io) return fail(m, BOA_E_NOMEM, "device staging allocation failed");
    uint8_t* d_data = io;
    uint8_t* d_first = d_data + al(nb);
    uint32_t* d_payload = (uint32_t*)(d_first + al(n_chunks));
    uint32_t* d_sizes = (uint32_t*)((uint8_t*)d_payload + al(dev_words * 4));
    uint64_t* d_off = (uint64_t*)((uint8_t*)d_sizes + al((size_t)n_chunks * 4));
    BOA_CK(cudaMemcpyAsync(d_data, data + c0, nb, cudaMemcpyHostToDevice, m->own));
    // compress the range as a stream that ends at the range end
    if (int rc = boa_compress_device(m, d_data, nb, chunk_len, n_chunks, d_first, d_payload, dev_words, d_sizes, d_off))
      return rc;
    uint64_t total = 0;
    BOA_CK(cudaMemcpyAsync(&total, d_off + n_chunks, 8, cudaMemcpyDeviceToHost, m->own));
    BOA_CK(cudaMemcpyAsync(sizes, d_sizes, (size_t)n_chunks * 4, cudaMemcpyDeviceToHost, m->own));
    BOA_CK(cudaMemcpyAsync(first_bytes, d_first, n_chunks, cudaMemcpyDeviceToHost, m->own));
    BOA_CK(cudaStreamSynchronize(m->own));
    if (int rc = read_dev_error(m)) return rc;
    if (total_out) *total_out = total;
    if (!payload || total > cap_words) return fail(m, BOA_E_INVALID, "payload capacity too small");
    BOA_CK(cudaMemcpyAsync(payload, d_payload, total * 4, cudaMemcpyDeviceToHost, m->own));
    BOA_CK(cudaStreamSynchronize(m->own));
  }
  return 0;
}

int boa_decompress_chunks(boa_model* m, const uint32_t* payload, const uint32_t* sizes, const uint8_t* first_bytes,
                          const uint32_t* chunk_lens, uint32_t chunk_len, uint32_t n_chunks, uint8_t* out) {
  if (!m) return BOA_E_INVALID;
  if (!sizes || !first_bytes || !chunk_lens || !out || chunk_len == 0 || n_chunks == 0)
    return fail(m, BOA_E_INVALID, "null buffer or empty range");
  for (uint32_t i = 0; i < n_chunks; ++i)
    if (chunk_lens[i] == 0 || chunk_lens[i] > chunk_len || (i + 1 < n_chunks && chunk_lens[i] != chunk_len))
      return fail(m, BOA_E_INVALID, "chunk lengths must equal chunk_len except the last, which may be shorter");
  uint64_t total = 0;
  for (uint32_t i = 0; i < n_chunks; ++i) total += sizes[i];
  if (total > 0 && !payload) return fail(m, BOA_E_INVALID, "payload is NULL");
  const uint64_t nb = (uint64_t)(n_chunks - 1) * chunk_len + chunk_lens[n_chunks - 1];
  std::vector<uint64_t> off(n_chunks + 1, 0);
  for (uint32_t i = 0; i < n_chunks; ++i) off[i + 1] = off[i] + sizes[i];
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t need = al(total * 4 + 4) + al((size_t)n_chunks * 4) + al((size_t)(n_chunks + 1) * 8) + al(n_chunks) + al(nb);
  StreamScope scope(m);
  uint8_t* io = (uint8_t*)ensure_io(m, need);
  if (!io) return fail(m, BOA_E_NOMEM, "device staging allocation failed");
  uint32_t* d_payload = (uint32_t*)io;
  uint32_t* d_sizes = (uint32_t*)(io + al(total * 4 + 4));
  uint64_t* d_off = (uint64_t*)((uint8_t*)d_sizes + al((size_t)n_chunks * 4));
  uint8_t* d_first = (uint8_t*)d_off + al((size_t)(n_chunks + 1) * 8);
  uint8_t* d_out = d_first + al(n_chunks);
  if (total) BOA_CK(cudaMemcpyAsync(d_payload, payload, total * 4, cudaMemcpyHostToDevice, m->own));
  BOA_CK(cudaMemcpyAsync(d_sizes, sizes, (size_t)n_chunks * 4, cudaMemcpyHostToDevice, m->own));
  BOA_CK(cudaMemcpyAsync(d_off, off.data(), (size_t)(n_chunks + 1) * 8, cudaMemcpyHostToDevice, m->own));
  BOA_CK(cudaMemcpyAsync(d_first, first_bytes, n_chunks, cudaMemcpyHostToDevice, m->own));
  if (int rc = boa_decompress_device(m, d_payload, d_off, d_sizes, d_first, nb, chunk_len, n_chunks, d_out)) return rc;
  BOA_CK(cudaMemcpyAsync(out, d_out, nb, cudaMemcpyDeviceToHost, m->own));
  BOA_CK(cudaStreamSynchronize(m->own));
  return read_dev_error(m);
}

int boa_set_profiling(boa_model* m, int on) {
  if (!m) return BOA_E_INVALID;
  m->prof = on != 0;
  return 0;
}

const char* boa_profile_name(int c) { return (c >= 0 && c < BOA_PROF_CLASSES) ? kProfNames[c] : nullptr; }

uint64_t boa_launch_count(const boa_model* m) { return m ? m->launches : 0; }

int boa_profile_read(boa_model* m, int c, double* total_ms, uint64_t* n) {
  if (!m) return BOA_E_INVALID;
  if (c < 0 || c >= BOA_PROF_CLASSES) return fail(m, BOA_E_INVALID, "kernel class out of range");
  if (!m->pending.empty()) {
    DeviceGuard dev(m->device);
    BOA_CK(cudaStreamSynchronize(m->own));
    for (auto& p : m->pending) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, p.a, p.b);
      m->prof_ms[p.cls] += ms;
      m->prof_n[p.cls] += 1;
      m->ev_pool.push_back(p.a);
      m->ev_pool.push_back(p.b);
    }
    m->pending.clear();
  }
  if (total_ms) *total_ms = m->prof_ms[c];
  if (n) *n = m->prof_n[c];
  m->prof_ms[c] = 0.0;
  m->prof_n[c] = 0;
  return 0;
}

int boa_model_logits(boa_model* m, const uint8_t* tokens, int B, int L, int mode, float* logits) {
  if (!m) return BOA_E_INVALID;
  if (!tokens || !logits || B <= 0 || L <= 0 || (mode != 0 && mode != 1))
    return fail(m, BOA_E_INVALID, "bad logits arguments");
  StreamScope scope(m);
  // compress form: tiles of up to 64 positions with the state carried between
  // them, as compress runs (the scan tile's shared memory bounds a tile)
  const int T = mode == 0 ? std::min(L, 64) : 1;
  if (int rc = ensure_work(m, (size_t)B * T, B, 1)) return rc;
  const size_t tok_b = ((size_t)B * L + 255) & ~size_t(255);
  uint8_t* d_tok = (uint8_t*)ensure_io(m, tok_b + (size_t)B * T * 256 * 4);
  if (!d_tok) return fail(m, BOA_E_NOMEM, "staging allocation failed");
  float* d_lg = (float*)(d_tok + tok_b);
  cudaStream_t st = m->own;
  BOA_CK(cudaMemcpyAsync(d_tok, tokens, (size_t)B * L, cudaMemcpyHostToDevice, st));
  if (int rc = reset_states(m, B)) return rc;
  if (mode == 0) {
    for (int t0 = 0; t0 < L; t0 += T) {
      const int Tt = std::min(T, L - t0);
      boa::TokenSrc src{1, d_tok, (long long)B * L, L, t0, Tt, nullptr, (long long)L, nullptr, nullptr, t0, nullptr};
      boa::GemmArgs h{};
      h.out_f32 = d_lg; h.ld_f32 = 256;
      if (int rc = forward(m, src, B, Tt, boa::EPI_LOGITS, h)) return rc;
      // rows (b, tau) of the tile -> logits[b][t0 + tau]
      BOA_CK(cudaMemcpy2DAsync(logits + (size_t)t0 * 256, (size_t)L * 256 * 4, d_lg, (size_t)Tt * 256 * 4,
                               (size_t)Tt * 256 * 4, (size_t)B, cudaMemcpyDeviceToHost, st));
    }
  } else {
    // step form: token column t of every chunk, one row per chunk
    uint8_t* d_col = (uint8_t*)m->lf;  // B bytes of scratch
    std::vector<uint8_t> col(B);
    std::vector<float> tmp((size_t)B * 256);
    for (int t = 0; t < L; ++t) {
      for (int b = 0; b < B; ++b) col[b] = tokens[(size_t)b * L + t];
      BOA_CK(cudaMemcpyAsync(d_col, col.data(), B, cudaMemcpyHostToDevice, st));
      boa::TokenSrc src{0, d_col, 0, 0, 0, 1, nullptr, 0, nullptr, nullptr, t, nullptr};
      boa::GemmArgs h{};
      h.out_f32 = d_lg; h.ld_f32 = 256;
      if (int rc = forward(m, src, B, 1, boa::EPI_LOGITS, h)) return rc;
      BOA_CK(cudaMemcpyAsync(tmp.data(), d_lg, tmp.size() * 4, cudaMemcpyDeviceToHost, st));
      BOA_CK(cudaStreamSynchronize(st));
      for (int b = 0; b < B; ++b)
        std::memcpy(logits + ((size_t)b * L + t) * 256, &tmp[(size_t)b * 256], 256 * 4);
    }
  }
  BOA_CK(cudaStreamSynchronize(st));
  return read_dev_error(m);
}

int boa_rc_encode_cdf(boa_model* m, const uint32_t* cdf, const uint8_t* syms, int ns, int nt, uint32_t* payload,
                      size_t cap_words, uint32_t* sizes) {
  if (!m) return BOA_E_INVALID;
  if (!cdf || !syms || !sizes || ns <= 0 || nt < 0) return fail(m, BOA_E_INVALID, "bad coder arguments");
  const uint32_t pitch = boa_stream_capacity_words((uint32_t)nt + 1);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t cdf_b = (size_t)nt * ns * 257 * 4, sym_b = (size_t)nt * ns;
  const size_t need = al(cdf_b + 4) + al(sym_b + 1) + al((size_t)ns * pitch * 4) + al((size_t)ns * 4) +
                      al(((size_t)ns + 1) * 8) + al((size_t)ns * sizeof(EncState)) + al((size_t)ns * pitch * 4);
  StreamScope scope(m);
  uint8_t* io = (uint8_t*)ensure_io(m, need);
  if (!io) return fail(m, BOA_E_NOMEM, "staging allocation failed");
  uint32_t* d_cdf = (uint32_t*)io;
  uint8_t* d_sym = io + al(cdf_b + 4);
  uint32_t* d_pitch = (uint32_t*)(d_sym + al(sym_b + 1));
  uint32_t* d_sizes = (uint32_t*)((uint8_t*)d_pitch + al((size_t)ns * pitch * 4));
  unsigned long long* d_off = (unsigned long long*)((uint8_t*)d_sizes + al((size_t)ns * 4));
  EncState* d_es = (EncState*)((uint8_t*)d_off + al(((size_t)ns + 1) * 8));
  uint32_t* d_pay = (uint32_t*)((uint8_t*)d_es + al((size_t)ns * sizeof(EncState)));
  cudaStream_t st = m->own;
  if (nt) {
    BOA_CK(cudaMemcpyAsync(d_cdf, cdf, cdf_b, cudaMemcpyHostToDevice, st));
    BOA_CK(cudaMemcpyAsync(d_sym, syms, sym_b, cudaMemcpyHostToDevice, st));
  }
  BOA_CK(boa::launch_enc_init(d_es, ns, st));
  if (nt) BOA_CK(boa::launch_rc_encode_cdf(d_es, d_cdf, d_sym, ns, nt, d_pitch, (int)pitch, st));
  BOA_CK(boa::launch_enc_finish(d_es, d_pitch, (int)pitch, d_sizes, ns, st));
  BOA_CK(cudaMemsetAsync(d_off, 0, 8, st));
  BOA_CK(boa::launch_offsets(d_sizes, d_off, ns, st));
  BOA_CK(boa::launch_compact(d_pitch, (int)pitch, d_sizes, d_off, d_pay, ns, st));
  uint64_t total = 0;
  BOA_CK(cudaMemcpyAsync(&total, d_off + ns, 8, cudaMemcpyDeviceToHost, st));
  BOA_CK(cudaMemcpyAsync(sizes, d_sizes, (size_t)ns * 4, cudaMemcpyDeviceToHost, st));
  BOA_CK(cudaStreamSynchronize(st));
  if (int rc = read_dev_error(m)) return rc;
  if (total > cap_words || (total && !payload)) return fail(m, BOA_E_INVALID, "payload capacity too small");
  if (total) BOA_CK(cudaMemcpy(payload, d_pay, total * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int boa_rc_decode_cdf(boa_model* m, const uint32_t* cdf, int ns, int nt, const uint32_t* payload,
                      const uint32_t* sizes, uint8_t* syms) {
  if (!m) return BOA_E_INVALID;
  if (!cdf || !sizes || !syms || ns <= 0 || nt < 0) return fail(m, BOA_E_INVALID, "bad coder arguments");
  uint64_t total = 0;
  std::vector<uint64_t> off(ns + 1, 0);
  for (int i = 0; i < ns; ++i) { off[i + 1] = off[i] + sizes[i]; }
  total = off[ns];
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t cdf_b = (size_t)nt * ns * 257 * 4, sym_b = (size_t)nt * ns;
  const size_t need = al(cdf_b + 4) + al(sym_b + 1) + al(total * 4 + 4) + al((size_t)ns * 4) + al(((size_t)ns + 1) * 8) +
                      al((size_t)ns * sizeof(DecState));
  StreamScope scope(m);
  uint8_t* io = (uint8_t*)ensure_io(m, need);
  if (!io) return fail(m, BOA_E_NOMEM, "staging allocation failed");
  uint32_t* d_cdf = (uint32_t*)io;
  uint8_t* d_sym = io + al(cdf_b + 4);
  uint32_t* d_pay = (uint32_t*)(d_sym + al(sym_b + 1));
  uint32_t* d_sizes = (uint32_t*)((uint8_t*)d_pay + al(total * 4 + 4));
  unsigned long long* d_off = (unsigned long long*)((uint8_t*)d_sizes + al((size_t)ns * 4));
  DecState* d_ds = (DecState*)((uint8_t*)d_off + al(((size_t)ns + 1) * 8));
  cudaStream_t st = m->own;
  if (nt) BOA_CK(cudaMemcpyAsync(d_cdf, cdf, cdf_b, cudaMemcpyHostToDevice, st));
  if (total) BOA_CK(cudaMemcpyAsync(d_pay, payload, total * 4, cudaMemcpyHostToDevice, st));
  BOA_CK(cudaMemcpyAsync(d_sizes, sizes, (size_t)ns * 4, cudaMemcpyHostToDevice, st));
  BOA_CK(cudaMemcpyAsync(d_off, off.data(), (size_t)(ns + 1) * 8, cudaMemcpyHostToDevice, st));
  BOA_CK(boa::launch_rc_decode_init(d_ds, d_pay, d_off, d_sizes, ns, st));
  if (nt) BOA_CK(boa::launch_rc_decode_cdf(d_ds, d_cdf, d_pay, d_off, ns, nt, d_sym, st));
  if (nt) BOA_CK(cudaMemcpyAsync(syms, d_sym, sym_b, cudaMemcpyDeviceToHost, st));
  BOA_CK(cudaStreamSynchronize(st));
  return read_dev_error(m);
}

int boa_cdf_from_logits(boa_model* m, const float* logits, int rows, float inv_t, uint32_t* cdf) {
  if (!m) return BOA_E_INVALID;
  if (!logits || !cdf || rows <= 0) return fail(m, BOA_E_INVALID, "bad arguments");
  StreamScope scope(m);
  const size_t lb = (size_t)rows * 256 * 4, qb = (size_t)rows * 257 * 4;
  uint8_t* io = (uint8_t*)ensure_io(m, lb + qb + 256);
  if (!io) return fail(m, BOA_E_NOMEM, "staging allocation failed");
  float* d_l = (float*)io;
  uint32_t* d_q = (uint32_t*)(io + ((lb + 255) & ~size_t(255)));
  BOA_CK(cudaMemcpyAsync(d_l, logits, lb, cudaMemcpyHostToDevice, m->own));
  BOA_CK(boa::launch_cdf_rows(d_l, rows, inv_t, d_q, m->own));
  BOA_CK(cudaMemcpyAsync(cdf, d_q, qb, cudaMemcpyDeviceToHost, m->own));
  BOA_CK(cudaStreamSynchronize(m->own));
  return read_dev_error(m);
}

}  // extern "C"
