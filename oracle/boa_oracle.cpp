// boa_oracle.cpp -- CPU restatement of the BoaConstrictor hot path.
//
// TEST INFRASTRUCTURE ONLY (see boa_oracle.h).  Citations are file:line in the
// reference project (AkarshSahlot/boa-constrictor, portability_solved_cpp/).
//
// Build: oracle/Makefile (g++ -O3 -ffp-contract=off; the reference build uses
// --fmad=false and explicit __fmaf_rn in its GEMM, so contraction stays off and
// the GEMM calls fmaf explicitly).
#include "boa_oracle.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#include <thread>
#include <atomic>
#include <mutex>
#include <algorithm>
#include <functional>

namespace {

thread_local std::string g_err;

enum Backbone { MAMBA = 0, LSTM = 1, GRU = 2, MINGRU = 3 };

// ----------------------------------------------------------------------------
// activations (activations.hpp:59-136 CPU branches; expf in place of repro_exp)
// ----------------------------------------------------------------------------
inline float sigmoidf_(float x) { return 1.0f / (1.0f + std::exp(-x)); }
inline float siluf_(float x) { return x * sigmoidf_(x); }
// repro_tanh: |x|>10 saturates, else (e^{2x}-1)/(e^{2x}+1)  (activations.hpp:88-101)
inline float tanh_ref(float x) {
  float ax = x < 0.f ? -x : x;
  if (ax > 10.0f) return x > 0.f ? 1.0f : -1.0f;
  float e2x = std::exp(2.0f * x);
  return (e2x - 1.0f) / (e2x + 1.0f);
}
// repro_gelu, tanh form (activations.hpp:105-118)
inline float gelu_ref(float x) {
  const float k0 = 0.79788456080286535588f, k1 = 0.044715f;
  float cube = x * x * x;
  float inner = k0 * (x + k1 * cube);
  return 0.5f * x * (1.0f + tanh_ref(inner));
}
// minGRU g(): rnn_kernels.cu:167-169
inline float mingru_g(float x) { return x >= 0.0f ? (x + 0.5f) : (1.0f / (1.0f + std::exp(-x))); }

enum Act { ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2, ACT_SILU = 3 };

// ----------------------------------------------------------------------------
// GEMM: C[m][n] = act(sum_k fma(A[m][k], W[n][k]) + bias[n]) (+ residual)
// Order restated from gemm_kernels.cu:283-310: fmaf over k ascending starting
// at 0, then + bias, then activation, then + residual.  Wt is [K][N].
// ----------------------------------------------------------------------------
void gemm(const float* A, int lda, const float* Wt, const float* bias, float* C, int ldc,
          int M, int K, int N, int act, const float* res = nullptr, int ldr = 0) {
  std::vector<float> acc(N);
  for (int m = 0; m < M; ++m) {
    std::fill(acc.begin(), acc.end(), 0.0f);
    const float* a = A + (size_t)m * lda;
    for (int k = 0; k < K; ++k) {
      const float av = a[k];
      const float* w = Wt + (size_t)k * N;
      for (int n = 0; n < N; ++n) acc[n] = std::fma(av, w[n], acc[n]);
    }
    float* c = C + (size_t)m * ldc;
    for (int n = 0; n < N; ++n) {
      float v = acc[n] + (bias ? bias[n] : 0.0f);
      if (act == ACT_GELU) v = gelu_ref(v);
      else if (act == ACT_RELU) v = std::max(0.0f, v);
      else if (act == ACT_SILU) v = siluf_(v);
      if (res) v += res[(size_t)m * ldr + n];
      c[n] = v;
    }
  }
}

// LayerNorm, var = E[x^2] - mean^2, eps 1e-5 (inference_kernels.cu:229-348)
void layernorm(const float* x, float* y, const float* w, const float* b, int rows, int N) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * N;
    float* yr = y + (size_t)r * N;
    float sum = 0.f, sq = 0.f;
    for (int i = 0; i < N; ++i) { sum += xr[i]; sq += xr[i] * xr[i]; }
    float mean = sum / (float)N;
    float var = sq / (float)N - mean * mean;
    float inv_std = 1.0f / std::sqrt(var + 1e-5f);
    for (int i = 0; i < N; ++i) yr[i] = (xr[i] - mean) * inv_std * w[i] + b[i];
  }
}

// RMSNorm, eps 1e-6, weight only (inference_kernels.cu:63-102)
void rmsnorm(float* x, const float* w, int rows, int N) {
  for (int r = 0; r < rows; ++r) {
    float* xr = x + (size_t)r * N;
    float sq = 0.f;
    for (int i = 0; i < N; ++i) sq += xr[i] * xr[i];
    float inv = 1.0f / std::sqrt(sq / (float)N + 1e-6f);
    for (int i = 0; i < N; ++i) xr[i] = xr[i] * inv * w[i];
  }
}

// transpose [rows][cols] -> [cols][rows]  (boa_gpu.hpp:45-54)
std::vector<float> transpose(const std::vector<float>& w, int rows, int cols) {
  std::vector<float> t(w.size());
  for (int i = 0; i < rows; ++i)
    for (int j = 0; j < cols; ++j) t[(size_t)j * rows + i] = w[(size_t)i * cols + j];
  return t;
}

// ----------------------------------------------------------------------------
// weights (.bin written by convert_boa_weights.py:153-241; read by
// boa_gpu.hpp:990-1029).  "BOA\0" = fp32, "BOA\1" = fp16, else legacy fp32.
// ----------------------------------------------------------------------------
struct Reader {
  const uint8_t* p; size_t n; size_t off = 0; bool fp16 = false; bool ok = true;
  float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF, f;
    if (e == 0) {
      if (m == 0) f = sign;
      else { e = 1; while (!(m & 0x400)) { m <<= 1; e--; } m &= 0x3FF; f = sign | ((127 - 15 + e) << 23) | (m << 13); }
    } else if (e == 31) f = sign | 0x7F800000u | (m << 13);
    else f = sign | ((e - 15 + 127) << 23) | (m << 13);
    float r; std::memcpy(&r, &f, 4); return r;
  }
  std::vector<float> vec(size_t count) {
    std::vector<float> v(count, 0.f);
    size_t esz = fp16 ? 2 : 4;
    if (off + count * esz > n) { ok = false; return v; }
    if (fp16) for (size_t i = 0; i < count; ++i) { uint16_t h; std::memcpy(&h, p + off + 2 * i, 2); v[i] = half_to_float(h); }
    else std::memcpy(v.data(), p + off, count * 4);
    off += count * esz;
    return v;
  }
};

struct MambaW {
  std::vector<float> ln1w, ln1b, in_t, in_b, conv_w, conv_b, xp_t, dt_t, dt_b, negA, D, out_t, out_b;
};
struct GruW { std::vector<float> wz_t, bz, wh_t, bh; };
// LSTM (G = 4d, gates i f g o) and GRU (G = 3d, gates r z n): W_ih / W_hh transposed to [d][G]
struct RnnW { std::vector<float> wih_t, bih, whh_t, bhh; };
struct BlockW {
  MambaW m; GruW g; RnnW rnn;
  std::vector<float> ln1w, ln1b, ln2w, ln2b, ff1_t, ff1_b, ff2_t, ff2_b;
};

struct Model {
  int backbone, d, L, di, dst = 16, dconv = 4, r;
  std::vector<float> emb;
  std::vector<BlockW> blocks;
  std::vector<float> final_norm, h1_t, h1_b, h2_t, h2_b;
};

// ----------------------------------------------------------------------------
// per-chunk recurrent state and a forward over T tokens (chunk form)
// ----------------------------------------------------------------------------
struct State {
  // mamba: conv [L][di][3] (last three inputs, oldest first), ssm [L][di][16]
  std::vector<float> conv, ssm, h, c;  // h: minGRU / LSTM / GRU [L][d]; c: LSTM cell [L][d]
  void init(const Model& M) {
    if (M.backbone == MAMBA) {
      conv.assign((size_t)M.L * M.di * 3, 0.f);
      ssm.assign((size_t)M.L * M.di * M.dst, 0.f);
    } else {
      h.assign((size_t)M.L * M.d, 0.f);
      if (M.backbone == LSTM) c.assign((size_t)M.L * M.d, 0.f);
    }
  }
};

struct Scratch {
  std::vector<float> x, res, xn, xz, u, delta, dt, y, mo, ff, head;
};

// Mamba block backbone over T tokens of ONE chunk, state carried.
// boa_gpu.hpp:298-330 (forward_chunk) with mamba_kernels.cu:370-470 and
// inference_kernels.cu:372-390, mamba_kernels.cu:130-151.
void mamba_forward(const Model& M, const MambaW& W, float* conv_st, float* ssm_st,
                   const float* xin, float* xout, int T, Scratch& s) {
  const int d = M.d, di = M.di, r = M.r, ds = M.dst, sd = r + 2 * ds;
  s.xz.resize((size_t)T * 2 * di); s.u.resize((size_t)T * di); s.delta.resize((size_t)T * sd);
  s.dt.resize((size_t)T * di); s.y.resize((size_t)T * di);
  // 1. in_proj + bias
  gemm(xin, d, W.in_t.data(), W.in_b.data(), s.xz.data(), 2 * di, T, d, 2 * di, ACT_NONE);
  // 2. causal depthwise conv (k=4) + SiLU; window = 3 carried inputs + current.
  //    Sum order: bias, then taps oldest..newest (mamba_kernels.cu:388-403).
  for (int c = 0; c < di; ++c) {
    float* cs = conv_st + (size_t)c * 3;
    const float* w = W.conv_w.data() + (size_t)c * 4;
    for (int t = 0; t < T; ++t) {
      float val = W.conv_b[c];
      for (int k = 0; k < 4; ++k) {
        int te = t - 3 + k;
        float xv = te >= 0 ? s.xz[(size_t)te * 2 * di + c] : cs[3 + te];
        val = val + xv * w[k];
      }
      s.u[(size_t)t * di + c] = val * (1.0f / (1.0f + std::exp(-val)));
    }
    // carry the last three inputs (mamba_kernels.cu:406-411)
    float win[3];
    for (int k = 0; k < 3; ++k) {
      int te = T - 3 + k;
      win[k] = te >= 0 ? s.xz[(size_t)te * 2 * di + c] : cs[3 + te];
    }
    for (int k = 0; k < 3; ++k) cs[k] = win[k];
  }
  // 3. x_proj (no bias) -> [dt_in(r) | B(16) | C(16)]
  gemm(s.u.data(), di, W.xp_t.data(), nullptr, s.delta.data(), sd, T, di, sd, ACT_NONE);
  // 4. dt_proj (no bias) then softplus(x + b)  (inference_kernels.cu:372-390)
  gemm(s.delta.data(), sd, W.dt_t.data(), nullptr, s.dt.data(), di, T, r, di, ACT_NONE);
  for (int t = 0; t < T; ++t)
    for (int c = 0; c < di; ++c) {
      float v = s.dt[(size_t)t * di + c] + W.dt_b[c];
      s.dt[(size_t)t * di + c] = std::log(1.0f + std::exp(v));
    }
  // 5. selective scan (mamba_kernels.cu:414-470) + 6. gate y*silu(z) (:130-151)
  for (int c = 0; c < di; ++c) {
    float* h = ssm_st + (size_t)c * ds;
    const float* nA = W.negA.data() + (size_t)c * ds;
    for (int t = 0; t < T; ++t) {
      float uv = s.u[(size_t)t * di + c], dtv = s.dt[(size_t)t * di + c];
      const float* Bv = s.delta.data() + (size_t)t * sd + r;
      const float* Cv = Bv + ds;
      float yv = 0.f;
      for (int n = 0; n < ds; ++n) {
        float dA = std::exp(nA[n] * dtv);
        float dB = dtv * Bv[n];
        h[n] = dA * h[n] + dB * uv;
        yv = yv + h[n] * Cv[n];
      }
      yv = yv + W.D[c] * uv;
      float z = s.xz[(size_t)t * 2 * di + di + c];
      s.y[(size_t)t * di + c] = yv * (z * (1.0f / (1.0f + std::exp(-z))));
    }
  }
  // 7. out_proj + bias
  gemm(s.y.data(), di, W.out_t.data(), W.out_b.data(), xout, d, T, di, d, ACT_NONE);
}

// minGRU backbone (boa_gpu.hpp:652-693, rnn_kernels.cu:230-263)
void mingru_forward(const Model& M, const GruW& W, float* h, const float* xin, float* xout,
                    int T, Scratch& s) {
  const int d = M.d;
  s.xz.resize((size_t)T * 2 * d);
  float* zl = s.xz.data();
  float* hr = s.xz.data() + (size_t)T * d;
  gemm(xin, d, W.wz_t.data(), W.bz.data(), zl, d, T, d, d, ACT_NONE);
  gemm(xin, d, W.wh_t.data(), W.bh.data(), hr, d, T, d, d, ACT_NONE);
  for (int c = 0; c < d; ++c) {
    float hv = h[c];
    for (int t = 0; t < T; ++t) {
      float z = 1.0f / (1.0f + std::exp(-zl[(size_t)t * d + c]));
      float ht = mingru_g(hr[(size_t)t * d + c]);
      hv = (1.0f - z) * hv + z * ht;
      xout[(size_t)t * d + c] = hv;
    }
    h[c] = hv;
  }
}

// LSTM / GRU backbone over T tokens of one chunk (boa_gpu.hpp:466-501,
// :567-582).  ih = x W_ih^T + b_ih for all T rows at once, then per token
// hh = h W_hh^T + b_hh and the fused gate update of rnn_kernels.cu:16-161
// (GPU_REPRO_MATH branch: repro_sigmoid / repro_tanh, products and sums
// rounded separately).
void rnn_forward(const Model& M, const RnnW& W, float* h, float* c, const float* xin, float* xout,
                 int T, Scratch& s) {
  const int d = M.d, G = (M.backbone == LSTM ? 4 : 3) * d;
  s.xz.resize((size_t)T * G + G);
  float* ih = s.xz.data();
  float* hh = s.xz.data() + (size_t)T * G;
  gemm(xin, d, W.wih_t.data(), W.bih.data(), ih, G, T, d, G, ACT_NONE);
  for (int t = 0; t < T; ++t) {
    gemm(h, d, W.whh_t.data(), W.bhh.data(), hh, G, 1, d, G, ACT_NONE);
    const float* a = ih + (size_t)t * G;
    for (int j = 0; j < d; ++j) {
      if (M.backbone == LSTM) {
        const float iv = sigmoidf_(a[j] + hh[j]);
        const float fv = sigmoidf_(a[d + j] + hh[d + j]);
        const float gv = tanh_ref(a[2 * d + j] + hh[2 * d + j]);
        const float ov = sigmoidf_(a[3 * d + j] + hh[3 * d + j]);
        const float fc = fv * c[j], ig = iv * gv;
        c[j] = fc + ig;
        h[j] = ov * tanh_ref(c[j]);
      } else {
        const float r = sigmoidf_(a[j] + hh[j]);
        const float z = sigmoidf_(a[d + j] + hh[d + j]);
        const float rn = r * hh[2 * d + j];
        const float n = tanh_ref(a[2 * d + j] + rn);
        const float p = (1.0f - z) * n, q = z * h[j];
        h[j] = p + q;
      }
    }
    std::memcpy(xout + (size_t)t * d, h, d * sizeof(float));
  }
}

// Full predictor over T tokens of one chunk (boa_gpu.hpp:1081-1102 / 892-928).
void predictor_forward(const Model& M, State& st, const uint8_t* tok, int T, float* logits, Scratch& s) {
  const int d = M.d;
  s.x.resize((size_t)T * d); s.res.resize((size_t)T * d); s.xn.resize((size_t)T * d);
  s.mo.resize((size_t)T * d); s.ff.resize((size_t)T * 4 * d); s.head.resize((size_t)T * d);
  for (int t = 0; t < T; ++t)  // embedding (utility_kernels.cu:46-72)
    std::memcpy(&s.x[(size_t)t * d], &M.emb[(size_t)tok[t] * d], d * sizeof(float));
  for (int l = 0; l < M.L; ++l) {
    const BlockW& B = M.blocks[l];
    if (M.backbone == MAMBA) {
      // x + FF(LN2(Mamba(LN1(x))))  (boa_gpu.hpp:892-902)
      layernorm(s.x.data(), s.xn.data(), B.ln1w.data(), B.ln1b.data(), T, d);
      mamba_forward(M, B.m, st.conv.data() + (size_t)l * M.di * 3,
                    st.ssm.data() + (size_t)l * M.di * M.dst, s.xn.data(), s.mo.data(), T, s);
      layernorm(s.mo.data(), s.xn.data(), B.ln2w.data(), B.ln2b.data(), T, d);
      gemm(s.xn.data(), d, B.ff1_t.data(), B.ff1_b.data(), s.ff.data(), 4 * d, T, d, 4 * d, ACT_GELU);
      gemm(s.ff.data(), 4 * d, B.ff2_t.data(), B.ff2_b.data(), s.x.data(), d, T, 4 * d, d, ACT_NONE,
           s.x.data(), d);
    } else {
      // x = x + minGRU(LN1 x); x = x + FF(LN2 x)  (boa_gpu.hpp:903-927)
      layernorm(s.x.data(), s.xn.data(), B.ln1w.data(), B.ln1b.data(), T, d);
      if (M.backbone == MINGRU)
        mingru_forward(M, B.g, st.h.data() + (size_t)l * d, s.xn.data(), s.mo.data(), T, s);
      else
        rnn_forward(M, B.rnn, st.h.data() + (size_t)l * d,
                    M.backbone == LSTM ? st.c.data() + (size_t)l * d : nullptr, s.xn.data(), s.mo.data(), T, s);
      for (size_t i = 0; i < (size_t)T * d; ++i) s.x[i] = s.mo[i] + s.x[i];
      layernorm(s.x.data(), s.xn.data(), B.ln2w.data(), B.ln2b.data(), T, d);
      gemm(s.xn.data(), d, B.ff1_t.data(), B.ff1_b.data(), s.ff.data(), 4 * d, T, d, 4 * d, ACT_GELU);
      gemm(s.ff.data(), 4 * d, B.ff2_t.data(), B.ff2_b.data(), s.x.data(), d, T, 4 * d, d, ACT_NONE,
           s.x.data(), d);
    }
  }
  if (M.backbone != MAMBA) rmsnorm(s.x.data(), M.final_norm.data(), T, d);
  int act = M.backbone == MAMBA ? ACT_RELU : ACT_SILU;  // boa_gpu.hpp:1095-1101
  gemm(s.x.data(), d, M.h1_t.data(), M.h1_b.data(), s.head.data(), d, T, d, d, act);
  gemm(s.head.data(), d, M.h2_t.data(), M.h2_b.data(), logits, 256, T, d, 256, ACT_NONE);
}

// ----------------------------------------------------------------------------
// softmax -> integer CDF, restating the warp arithmetic of
// ker_rc_encode_chunk_parallel_warp (range_coder_kernels.cu:860-925) and the
// warp helpers in gemm_gpu_common.cuh:87-123.  Lane l owns symbols 8l..8l+7.
// All double arithmetic follows the same operation order, so for identical
// float exponentials the result is bit-identical; CUDA's __expf is replaced by
// the C library's expf (tolerance only).
// ----------------------------------------------------------------------------
void cdf_row(const float* lg, float inv_t, uint32_t* Q) {
  float mx = -1e30f;
  for (int l = 0; l < 32; ++l) {  // lane max then warpReduceMax (order-free)
    for (int i = 0; i < 8; ++i) mx = std::fmax(mx, lg[l * 8 + i]);
  }
  float e[256];
  double lane_sum[32];
  for (int l = 0; l < 32; ++l) {
    double sd = 0.0;
    for (int i = 0; i < 8; ++i) {
      float v = std::exp((lg[l * 8 + i] - mx) * inv_t);
      e[l * 8 + i] = v;
      sd += (double)v;
    }
    lane_sum[l] = sd;
  }
  // warpReduceSumDouble: shfl_down tree, offsets 16,8,4,2,1; lane 0's result
  double red[32];
  for (int l = 0; l < 32; ++l) red[l] = lane_sum[l];
  for (int off = 16; off > 0; off /= 2) {
    double nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = red[l] + (l + off < 32 ? red[l + off] : red[l]);
    for (int l = 0; l < 32; ++l) red[l] = nv[l];
  }
  const double total = red[0];
  const double inv_sum = 1.0 / total;
  // warpScanSumDouble: Hillis-Steele inclusive scan, offsets 1,2,4,8,16
  double ts[32], sc[32];
  for (int l = 0; l < 32; ++l) { ts[l] = lane_sum[l] * inv_sum; sc[l] = ts[l]; }
  for (int off = 1; off <= 16; off *= 2) {
    double nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = (l >= off) ? sc[l] + sc[l - off] : sc[l];
    for (int l = 0; l < 32; ++l) sc[l] = nv[l];
  }
  double cdf[257];
  for (int l = 0; l < 32; ++l) {
    double run = sc[l] - ts[l];
    for (int i = 0; i < 8; ++i) { cdf[l * 8 + i] = run; run += (double)e[l * 8 + i] * inv_sum; }
  }
  cdf[256] = 1.0;
  // monotone fix-up at lane boundaries, all lanes reading pre-fix-up values
  // (range_coder_kernels.cu:903-913)
  double delta[32];
  for (int l = 0; l < 32; ++l) {
    delta[l] = 0.0;
    if (l > 0) {
      double prev_end = cdf[l * 8 - 1], my_start = cdf[l * 8];
      if (my_start < prev_end) delta[l] = prev_end - my_start;
    }
  }
  for (int l = 1; l < 32; ++l)
    if (delta[l] != 0.0)
      for (int i = 0; i < 8; ++i) cdf[l * 8 + i] += delta[l];
  // quantise: Q_k = (u32)(C_k * (2^24 - 256)) + k; Q_256 = 2^24 (:917-925),
  // with the floor term kept non-decreasing (running maximum).  That equals
  // the reference's Q on every row where its Q is strictly increasing; where
  // the fix-up above leaves C decreasing by an ulp after C reached 1.0, the
  // reference's Q has an empty interval (undecodable) and this repairs it.
  const double scale = (double)((1u << 24) - 256);
  uint32_t rm = 0;
  for (int k = 0; k < 256; ++k) {
    rm = std::max(rm, (uint32_t)(cdf[k] * scale));
    Q[k] = rm + (uint32_t)k;
  }
  Q[256] = 1u << 24;
}

// ----------------------------------------------------------------------------
// integer range coder, 64-bit state, 32-bit words, 24-bit CDF precision.
// Encoder: ker_rc_init (:46-60), update (:927-965), ker_rc_finish (:279-313).
// Decoder: ker_rc_init_decoder (:319-335), step (:725-780).
// ----------------------------------------------------------------------------
struct Enc {
  uint64_t lower = 0, range = ~0ull; int inv = 0; uint32_t first_inv = 0; int w = 0;
};

inline bool enc_symbol(Enc& st, uint32_t left, uint32_t prob, uint32_t* out, int cap) {
  if (prob == 0) prob = 1;
  uint64_t scale = st.range >> 24;
  uint64_t old_lower = st.lower;
  st.range = scale * (uint64_t)prob;
  st.lower = st.lower + scale * (uint64_t)left;
  if (st.inv > 0) {
    uint64_t sum = st.lower + st.range;
    if (sum > st.lower) {
      uint32_t first = (st.lower < old_lower) ? st.first_inv + 1u : st.first_inv;
      uint32_t sub = (st.lower < old_lower) ? 0u : 0xFFFFFFFFu;
      if (st.w + st.inv > cap) return false;
      out[st.w++] = first;
      for (int k = 1; k < st.inv; ++k) out[st.w++] = sub;
      st.inv = 0;
    }
  }
  while (st.range < (1ull << 32)) {
    uint32_t lw = (uint32_t)(st.lower >> 32);
    st.lower <<= 32; st.range <<= 32;
    if (st.inv > 0) st.inv++;
    else {
      uint64_t sum = st.lower + st.range;
      if (sum > st.lower) { if (st.w >= cap) return false; out[st.w++] = lw; }
      else { st.inv = 1; st.first_inv = lw; }
    }
  }
  return true;
}

inline int enc_finish(Enc& st, uint32_t* out, int cap) {
  if (st.range == ~0ull) return 0;  // nothing encoded -> zero words
  uint64_t point = st.lower + ((1ull << 32) - 1ull);
  if (st.inv > 0) {
    uint32_t first = (point < st.lower) ? st.first_inv + 1u : st.first_inv;
    uint32_t sub = (point < st.lower) ? 0u : 0xFFFFFFFFu;
    if (st.w + st.inv > cap) return -1;
    out[st.w++] = first;
    for (int k = 1; k < st.inv; ++k) out[st.w++] = sub;
    st.inv = 0;
  }
  uint32_t pw = (uint32_t)(point >> 32);
  if (st.w + 2 > cap) return -1;
  out[st.w++] = pw;
  uint64_t upper = st.lower + st.range;
  if ((uint32_t)(upper >> 32) == pw) out[st.w++] = 0u;
  return st.w;
}

struct Dec {
  uint64_t lower = 0, range = ~0ull, point = 0; int r = 0;
  const uint32_t* in; int n;
  void init(const uint32_t* words, int n_words) {
    in = words; n = n_words; lower = 0; range = ~0ull; point = 0; r = 0;
    for (int k = 0; k < 2; ++k) { uint32_t w = r < n ? in[r++] : 0u; point = (point << 32) | w; }
  }
  uint32_t target() const {
    uint64_t scale = range >> 24;
    uint64_t q = (point - lower) / scale;
    if (q >= (1ull << 24)) q = (1ull << 24) - 1;
    return (uint32_t)q;
  }
  void update(uint32_t low, uint32_t high) {
    uint64_t scale = range >> 24;
    uint32_t prob = high - low;
    if (prob == 0) prob = 1;
    lower = lower + scale * (uint64_t)low;
    range = scale * (uint64_t)prob;
    while (range < (1ull << 32)) {
      lower <<= 32; range <<= 32;
      uint32_t w = r < n ? in[r++] : 0u;
      point = (point << 32) | w;
    }
  }
};

// decoder symbol search: lowest k with Q_k <= target < Q_{k+1}
// (the warp ballot + __ffs of range_coder_kernels.cu:747-763 finds the lowest)
inline int dec_search(const uint32_t* Q, uint32_t target, uint32_t& lo, uint32_t& hi) {
  for (int k = 0; k < 256; ++k) {
    if (target >= Q[k] && target < Q[k + 1]) { lo = Q[k]; hi = Q[k + 1]; return k; }
  }
  lo = 0; hi = 0; return 0;
}

// ----------------------------------------------------------------------------
// model load
// ----------------------------------------------------------------------------
Model* load_model(const char* path, int backbone, int d, int nl) {
  FILE* f = std::fopen(path, "rb");
  if (!f) { g_err = std::string("cannot open weights: ") + path; return nullptr; }
  std::vector<uint8_t> buf;
  std::fseek(f, 0, SEEK_END); long sz = std::ftell(f); std::fseek(f, 0, SEEK_SET);
  buf.resize(sz > 0 ? sz : 0);
  if (sz > 0 && std::fread(buf.data(), 1, sz, f) != (size_t)sz) { std::fclose(f); g_err = "short read"; return nullptr; }
  std::fclose(f);
  if (backbone < MAMBA || backbone > MINGRU) { g_err = "backbone must be 0 (mamba), 1 (lstm), 2 (gru) or 3 (mingru)"; return nullptr; }
  if (d <= 0 || nl <= 0 || d % 16 != 0) { g_err = "bad model dims"; return nullptr; }
  Reader R{buf.data(), buf.size()};
  if (buf.size() >= 4 && buf[0] == 'B' && buf[1] == 'O' && buf[2] == 'A') { R.fp16 = buf[3] == 1; R.off = 4; }
  Model* M = new Model();
  M->backbone = backbone; M->d = d; M->L = nl; M->di = 2 * d; M->r = (d + 15) / 16;
  const int di = M->di, r = M->r, ds = M->dst;
  M->emb = R.vec((size_t)256 * d);
  M->blocks.resize(nl);
  for (int l = 0; l < nl; ++l) {
    BlockW& B = M->blocks[l];
    B.ln1w = R.vec(d); B.ln1b = R.vec(d);
    if (backbone == MAMBA) {  // boa_gpu.hpp:212-225
      MambaW& W = B.m;
      W.in_t = transpose(R.vec((size_t)2 * di * d), 2 * di, d);
      W.in_b = R.vec(2 * di);
      W.conv_w = R.vec((size_t)di * 4);
      W.conv_b = R.vec(di);
      W.xp_t = transpose(R.vec((size_t)(r + 2 * ds) * di), r + 2 * ds, di);
      W.dt_t = transpose(R.vec((size_t)di * r), di, r);
      W.dt_b = R.vec(di);
      std::vector<float> alog = R.vec((size_t)di * ds);
      W.negA.resize(alog.size());
      for (size_t i = 0; i < alog.size(); ++i) W.negA[i] = -std::exp(alog[i]);
      W.D = R.vec(di);
      W.out_t = transpose(R.vec((size_t)d * di), d, di);
      W.out_b = R.vec(d);
    } else if (backbone == LSTM || backbone == GRU) {  // boa_gpu.hpp:413-419, :526-532
      const int G = (backbone == LSTM ? 4 : 3) * d;
      RnnW& W = B.rnn;
      W.wih_t = transpose(R.vec((size_t)G * d), G, d); W.bih = R.vec(G);
      W.whh_t = transpose(R.vec((size_t)G * d), G, d); W.bhh = R.vec(G);
    } else {  // boa_gpu.hpp:643-648
      GruW& G = B.g;
      G.wz_t = transpose(R.vec((size_t)d * d), d, d); G.bz = R.vec(d);
      G.wh_t = transpose(R.vec((size_t)d * d), d, d); G.bh = R.vec(d);
    }
    B.ln2w = R.vec(d); B.ln2b = R.vec(d);
    B.ff1_t = transpose(R.vec((size_t)4 * d * d), 4 * d, d); B.ff1_b = R.vec(4 * d);
    B.ff2_t = transpose(R.vec((size_t)4 * d * d), d, 4 * d); B.ff2_b = R.vec(d);
  }
  if (backbone != MAMBA) M->final_norm = R.vec(d);
  M->h1_t = transpose(R.vec((size_t)d * d), d, d); M->h1_b = R.vec(d);
  M->h2_t = transpose(R.vec((size_t)256 * d), 256, d); M->h2_b = R.vec(256);
  if (!R.ok || R.off != R.n) {
    g_err = "weight file size does not match the model dims (expected " + std::to_string(R.off) +
            " bytes, file has " + std::to_string(R.n) + ")";
    delete M; return nullptr;
  }
  return M;
}

void parallel_for(int n, int n_threads, const std::function<void(int)>& fn) {
  if (n_threads <= 1 || n <= 1) { for (int i = 0; i < n; ++i) fn(i); return; }
  std::atomic<int> next(0);
  std::vector<std::thread> th;
  int nt = std::min(n_threads, n);
  for (int t = 0; t < nt; ++t)
    th.emplace_back([&]() { for (int i; (i = next.fetch_add(1)) < n;) fn(i); });
  for (auto& x : th) x.join();
}
}  // namespace

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }

void* orc_load(const char* path, int backbone, int d_model, int n_layers) {
  return load_model(path, backbone, d_model, n_layers);
}

void orc_free(void* m) { delete (Model*)m; }

int orc_logits(void* mp, const uint8_t* tokens, int B, int L, int mode, float* logits) {
  const Model& M = *(Model*)mp;
  parallel_for(B, 1, [&](int b) {
    State st; st.init(M); Scratch s;
    const uint8_t* tk = tokens + (size_t)b * L;
    float* lg = logits + (size_t)b * L * 256;
    if (mode == 0) predictor_forward(M, st, tk, L, lg, s);
    else for (int t = 0; t < L; ++t) predictor_forward(M, st, tk + t, 1, lg + (size_t)t * 256, s);
  });
  return 0;
}

void orc_cdf_row(const float* row, float inv_t, uint32_t* Q) { cdf_row(row, inv_t, Q); }

void orc_cdf_rows(const float* lg, int rows, float inv_t, uint32_t* Q) {
  for (int i = 0; i < rows; ++i) cdf_row(lg + (size_t)i * 256, inv_t, Q + (size_t)i * 257);
}

int orc_rc_encode_cdf(const uint32_t* Q, const uint8_t* syms, int n, uint32_t* out, int cap) {
  Enc st;
  for (int i = 0; i < n; ++i) {
    const uint32_t* q = Q + (size_t)i * 257;
    int s = syms[i];
    if (!enc_symbol(st, q[s], q[s + 1] - q[s], out, cap)) return -1;
  }
  return enc_finish(st, out, cap);
}

int orc_rc_decode_cdf(const uint32_t* Q, int n, const uint32_t* words, int n_words, uint8_t* syms) {
  Dec d; d.init(words, n_words);
  for (int i = 0; i < n; ++i) {
    const uint32_t* q = Q + (size_t)i * 257;
    uint32_t lo, hi;
    int s = dec_search(q, d.target(), lo, hi);
    syms[i] = (uint8_t)s;
    d.update(lo, hi);
  }
  return 0;
}

// build_cdf_fast (gpu_range_coder.py:57-79): cdf[i] = (u32)(P_i * scale) + i
// with P_i the left-to-right fp64 sum of the first i probabilities and
// scale = (2^24 - K) / P_K; a non-positive or non-finite P_K gives the equal
// split acc += (2^24 - K) / K + 1.
void orc_pyrc_cdf_rows(const float* probs, int rows, int K, uint32_t* cdf) {
  const uint32_t total = 1u << 24, free_w = total - (uint32_t)K;
  for (int r = 0; r < rows; ++r) {
    const float* p = probs + (size_t)r * K;
    uint32_t* c = cdf + (size_t)r * (K + 1);
    double norm = 0.0;
    for (int i = 0; i < K; ++i) norm += (double)p[i];
    if (!(norm > 0.0) || !std::isfinite(norm)) {
      uint32_t acc = 0;
      for (int i = 0; i < K; ++i) { c[i] = acc; acc += free_w / (uint32_t)K + 1u; }
    } else {
      const double scale = (double)free_w / norm;
      double cum = 0.0;
      for (int i = 0; i < K; ++i) { c[i] = (uint32_t)(cum * scale) + (uint32_t)i; cum += (double)p[i]; }
    }
    c[K] = total;
  }
}

namespace {
// encode_kernel's update (gpu_range_coder.py:81-140): no clamp of prob.
bool pyrc_symbol(Enc& st, uint32_t left, uint32_t prob, uint32_t* out, int cap) {
  const uint64_t scale = st.range >> 24;
  const uint64_t old_lower = st.lower;
  st.range = scale * (uint64_t)prob;
  st.lower = st.lower + scale * (uint64_t)left;
  if (st.inv > 0 && st.lower + st.range > st.lower) {
    const bool carry = st.lower < old_lower;
    if (st.w + st.inv > cap) return false;
    out[st.w++] = carry ? st.first_inv + 1u : st.first_inv;
    for (int k = 1; k < st.inv; ++k) out[st.w++] = carry ? 0u : 0xFFFFFFFFu;
    st.inv = 0;
  }
  while (st.range < (1ull << 32)) {
    const uint32_t lw = (uint32_t)(st.lower >> 32);
    st.lower <<= 32; st.range <<= 32;
    if (st.inv > 0) { if (st.inv < 0x7FFFFFFF) st.inv++; }
    else if (st.lower + st.range > st.lower) { if (st.w >= cap) return false; out[st.w++] = lw; }
    else { st.inv = 1; st.first_inv = lw; }
  }
  return true;
}
}  // namespace

int orc_pyrc_encode(const float* probs, const int32_t* syms, int n, int K, uint32_t* out, int cap) {
  Enc st;
  std::vector<uint32_t> c((size_t)K + 1);
  for (int t = 0; t < n; ++t) {
    const int s = syms[t];
    if (s < 0 || s >= K) continue;
    orc_pyrc_cdf_rows(probs + (size_t)t * K, 1, K, c.data());
    if (!pyrc_symbol(st, c[s], c[s + 1] - c[s], out, cap)) return -1;
  }
  return enc_finish(st, out, cap);  // finalize_kernel (:142-168) is ker_rc_finish's rule
}

int orc_pyrc_decode(const float* probs, int n, int K, const uint32_t* words, int n_words, int32_t* syms) {
  Dec d;
  d.init(words, n_words);
  std::vector<uint32_t> c((size_t)K + 1);
  for (int t = 0; t < n; ++t) {
    orc_pyrc_cdf_rows(probs + (size_t)t * K, 1, K, c.data());
    const uint32_t target = d.target();
    int i = 1;  // decode_step_kernel (:182-215): first i >= 1 with cdf[i] > target
    while (i <= K && !(c[i] > target)) ++i;
    int s = i - 1;
    if (s < 0) s = 0;
    if (s >= K) s = K - 1;
    syms[t] = s;
    const uint64_t scale = d.range >> 24;
    d.lower = d.lower + scale * (uint64_t)c[s];
    d.range = scale * (uint64_t)(c[s + 1] - c[s]);
    while (d.range < (1ull << 32)) {
      d.lower <<= 32; d.range <<= 32;
      const uint32_t w = d.r < d.n ? d.in[d.r++] : 0u;
      d.point = (d.point << 32) | w;
    }
  }
  return 0;
}

int orc_compress(void* mp, const uint8_t* data, size_t n, uint32_t chunk_len, float inv_t,
                 int n_threads, uint8_t* first_bytes, uint32_t* stream_words, uint32_t pitch,
                 uint32_t* sizes) {
  const Model& M = *(Model*)mp;
  if (chunk_len == 0) { g_err = "chunk_len must be > 0"; return -1; }
  const int n_chunks = (int)((n + chunk_len - 1) / chunk_len);
  std::atomic<int> bad(0);
  parallel_for(n_chunks, n_threads, [&](int c) {
    size_t off = (size_t)c * chunk_len;
    int len = (int)std::min<size_t>(chunk_len, n - off);
    const uint8_t* tk = data + off;
    first_bytes[c] = len > 0 ? tk[0] : 0;
    State st; st.init(M); Scratch s; Enc enc;
    uint32_t* out = stream_words + (size_t)c * pitch;
    const int TILE = 256;
    std::vector<float> lg((size_t)TILE * 256);
    uint32_t Q[257];
    // logits at position t predict token t+1 (boa.cpp:441-469 with
    // range_coder_kernels.cu:854-858): positions 0..len-2 are encoded.
    for (int t0 = 0; t0 < len - 1; t0 += TILE) {
      int T = std::min(TILE, len - 1 - t0);
      predictor_forward(M, st, tk + t0, T, lg.data(), s);
      for (int t = 0; t < T; ++t) {
        cdf_row(lg.data() + (size_t)t * 256, inv_t, Q);
        int sym = tk[t0 + t + 1];
        if (!enc_symbol(enc, Q[sym], Q[sym + 1] - Q[sym], out, (int)pitch)) { bad = 1; return; }
      }
    }
    int w = enc_finish(enc, out, (int)pitch);
    if (w < 0) { bad = 1; return; }
    sizes[c] = (uint32_t)w;
  });
  if (bad) { g_err = "stream exceeded pitch"; return -1; }
  return 0;
}

int orc_decompress(void* mp, const uint32_t* stream_words, uint32_t pitch, const uint32_t* sizes,
                   const uint8_t* first_bytes, size_t n, uint32_t chunk_len, float inv_t,
                   int n_threads, uint8_t* out) {
  const Model& M = *(Model*)mp;
  if (chunk_len == 0) { g_err = "chunk_len must be > 0"; return -1; }
  const int n_chunks = (int)((n + chunk_len - 1) / chunk_len);
  parallel_for(n_chunks, n_threads, [&](int c) {
    size_t off = (size_t)c * chunk_len;
    int len = (int)std::min<size_t>(chunk_len, n - off);
    if (len <= 0) return;
    uint8_t* o = out + off;
    o[0] = first_bytes[c];
    State st; st.init(M); Scratch s;
    Dec dec; dec.init(stream_words + (size_t)c * pitch, (int)sizes[c]);
    float lg[256]; uint32_t Q[257];
    for (int t = 1; t < len; ++t) {  // boa.cpp:754-756 with :725-780
      predictor_forward(M, st, o + t - 1, 1, lg, s);
      cdf_row(lg, inv_t, Q);
      uint32_t lo, hi;
      int sym = dec_search(Q, dec.target(), lo, hi);
      o[t] = (uint8_t)sym;
      dec.update(lo, hi);
    }
  });
  return 0;
}

// Warm start (boa.cpp:313-319, :395-435): W lanes; lane b codes chunks
// b*S .. b*S+S-1 (S = ceil(n_chunks / W)) in order, carrying the model state;
// the encoder's forward pass consumes every byte of a chunk (forward_chunk
// over all chunk_size positions), each chunk has its own coder and raw first
// byte.  The decoder feeds a chunk's last byte into the state before moving
// to the lane's next chunk, so it follows the encoder.
int orc_compress_warm(void* mp, const uint8_t* data, size_t n, uint32_t chunk_len, uint32_t W, float inv_t,
                      int n_threads, uint8_t* first_bytes, uint32_t* stream_words, uint32_t pitch, uint32_t* sizes) {
  const Model& M = *(Model*)mp;
  if (chunk_len == 0 || W == 0) { g_err = "chunk_len and W must be > 0"; return -1; }
  const int n_chunks = (int)((n + chunk_len - 1) / chunk_len);
  const int Wl = std::min<int>((int)W, n_chunks), S = (n_chunks + Wl - 1) / Wl;
  std::atomic<int> bad(0);
  parallel_for(Wl, n_threads, [&](int b) {
    State st; st.init(M); Scratch s;
    std::vector<float> lg((size_t)chunk_len * 256);
    uint32_t Q[257];
    for (int i = 0; i < S; ++i) {
      const int c = b * S + i;
      if (c >= n_chunks) break;
      const size_t off = (size_t)c * chunk_len;
      const int len = (int)std::min<size_t>(chunk_len, n - off);
      const uint8_t* tk = data + off;
      first_bytes[c] = tk[0];
      Enc enc;
      uint32_t* out = stream_words + (size_t)c * pitch;
      predictor_forward(M, st, tk, len, lg.data(), s);
      for (int t = 0; t + 1 < len; ++t) {
        cdf_row(lg.data() + (size_t)t * 256, inv_t, Q);
        const int sym = tk[t + 1];
        if (!enc_symbol(enc, Q[sym], Q[sym + 1] - Q[sym], out, (int)pitch)) { bad = 1; return; }
      }
      const int w = enc_finish(enc, out, (int)pitch);
      if (w < 0) { bad = 1; return; }
      sizes[c] = (uint32_t)w;
    }
  });
  if (bad) { g_err = "stream exceeded pitch"; return -1; }
  return 0;
}

int orc_decompress_warm(void* mp, const uint32_t* stream_words, uint32_t pitch, const uint32_t* sizes,
                        const uint8_t* first_bytes, size_t n, uint32_t chunk_len, uint32_t W, float inv_t,
                        int n_threads, uint8_t* out) {
  const Model& M = *(Model*)mp;
  if (chunk_len == 0 || W == 0) { g_err = "chunk_len and W must be > 0"; return -1; }
  const int n_chunks = (int)((n + chunk_len - 1) / chunk_len);
  const int Wl = std::min<int>((int)W, n_chunks), S = (n_chunks + Wl - 1) / Wl;
  parallel_for(Wl, n_threads, [&](int b) {
    State st; st.init(M); Scratch s;
    float lg[256]; uint32_t Q[257];
    for (int i = 0; i < S; ++i) {
      const int c = b * S + i;
      if (c >= n_chunks) break;
      const size_t off = (size_t)c * chunk_len;
      const int len = (int)std::min<size_t>(chunk_len, n - off);
      uint8_t* o = out + off;
      o[0] = first_bytes[c];
      Dec dec; dec.init(stream_words + (size_t)c * pitch, (int)sizes[c]);
      for (int t = 1; t < len; ++t) {
        predictor_forward(M, st, o + t - 1, 1, lg, s);
        cdf_row(lg, inv_t, Q);
        uint32_t lo, hi;
        const int sym = dec_search(Q, dec.target(), lo, hi);
        o[t] = (uint8_t)sym;
        dec.update(lo, hi);
      }
      predictor_forward(M, st, o + len - 1, 1, lg, s);  // the chunk's last byte
    }
  });
  return 0;
}

}  // extern "C"
