// coder.cuh -- softmax -> integer CDF and the 64-bit/32-bit-word range coder,
// as device functions shared by the LM-head epilogue (compress and decompress)
// and the standalone coder kernels.
//
// CDF: the reference builds it with one warp per row, lane l owning symbols
// 8l..8l+7 (range_coder_kernels.cu:860-925, decode twin :661-763).  Here ONE
// thread evaluates the same arithmetic in the same order (lane partial sums,
// shfl_down reduction tree, Hillis-Steele scan, lane-boundary monotone fix-up,
// Q_k = (u32)(C_k * (2^24 - 256)) + k), using explicit round-to-nearest
// intrinsics so no operation is contracted.  Encoder and decoder therefore see
// bit-identical Q_k, and for identical exponentials the values equal the
// reference's.
//
// Coder: restates ker_rc_init (:46-60), the encode update (:927-965),
// ker_rc_finish (:279-313), ker_rc_init_decoder (:319-335) and the decode
// update (:765-780).  Pure integer arithmetic -> bit-exact.
#pragma once
#include <cstdint>
#include "ptx.cuh"

namespace boa {

constexpr uint32_t kCdfTotal = 1u << 24;
constexpr double kCdfScale = (double)((1u << 24) - 256);

struct EncState {  // RCState, gemm_gpu.hpp:115-121
  unsigned long long lower, range;
  int inv;             // inverted_num: pending carry-run length
  uint32_t first_inv;  // first_inv_lower_word
  int w;               // words written
  int bad;             // coding stopped (empty interval or capacity); finish reports the stream as failed
};
struct DecState {  // RCDecState, gemm_gpu.hpp:212-217
  unsigned long long lower, range, point;
  int r;  // words consumed
  int n;  // words available
};

__host__ __device__ __forceinline__ void enc_init(EncState& s) {
  s.lower = 0ull; s.range = ~0ull; s.inv = 0; s.first_inv = 0u; s.w = 0; s.bad = 0;
}

// Encode one symbol with CDF slot [left, left+prob) of 2^24.  Returns false
// (and stops writing) when the stream would exceed `cap` words.
__device__ __forceinline__ bool enc_symbol(EncState& st, uint32_t left, uint32_t prob, uint32_t* out,
                                           int cap) {
  if (prob == 0) prob = 1;
  const unsigned long long scale = st.range >> 24;
  const unsigned long long old_lower = st.lower;
  st.range = scale * (unsigned long long)prob;
  st.lower = st.lower + scale * (unsigned long long)left;
  if (st.inv > 0) {
    const unsigned long long sum = st.lower + st.range;
    if (sum > st.lower) {
      const bool carried = st.lower < old_lower;
      const uint32_t first = carried ? st.first_inv + 1u : st.first_inv;
      const uint32_t sub = carried ? 0u : 0xFFFFFFFFu;
      if (st.w + st.inv > cap) return false;
      out[st.w++] = first;
      for (int k = 1; k < st.inv; ++k) out[st.w++] = sub;
      st.inv = 0;
    }
  }
  while (st.range < (1ull << 32)) {
    const uint32_t lw = (uint32_t)(st.lower >> 32);
    st.lower <<= 32;
    st.range <<= 32;
    if (st.inv > 0) {
      st.inv++;
    } else {
      const unsigned long long sum = st.lower + st.range;
      if (sum > st.lower) {
        if (st.w >= cap) return false;
        out[st.w++] = lw;
      } else {
        st.inv = 1;
        st.first_inv = lw;
      }
    }
  }
  return true;
}

// Flush; returns total words (0 if nothing was encoded) or -1 on overflow.
__device__ __forceinline__ int enc_finish(EncState& st, uint32_t* out, int cap) {
  if (st.range == ~0ull) return 0;
  const unsigned long long point = st.lower + ((1ull << 32) - 1ull);
  if (st.inv > 0) {
    const bool carried = point < st.lower;
    const uint32_t first = carried ? st.first_inv + 1u : st.first_inv;
    const uint32_t sub = carried ? 0u : 0xFFFFFFFFu;
    if (st.w + st.inv > cap) return -1;
    out[st.w++] = first;
    for (int k = 1; k < st.inv; ++k) out[st.w++] = sub;
    st.inv = 0;
  }
  const uint32_t pw = (uint32_t)(point >> 32);
  if (st.w + 2 > cap) return -1;
  out[st.w++] = pw;
  const unsigned long long upper = st.lower + st.range;
  if ((uint32_t)(upper >> 32) == pw) out[st.w++] = 0u;
  return st.w;
}

__device__ __forceinline__ void dec_init(DecState& st, const uint32_t* in, int n) {
  st.lower = 0ull; st.range = ~0ull; st.point = 0ull; st.r = 0; st.n = n;
  for (int k = 0; k < 2; ++k) {
    const uint32_t w = st.r < n ? in[st.r++] : 0u;
    st.point = (st.point << 32) | (unsigned long long)w;
  }
}
// min((point - lower) / scale, 2^24 - 1) with scale = range >> 24, as the
// reference computes it (range_coder_kernels.cu:765-768), without a 64-bit
// integer division: range is normalised to [2^32, 2^64), so scale lies in
// [2^8, 2^40); a single-precision estimate of the quotient (relative error
// a few 2^-24, i.e. off by at most a few units below 2^24) is corrected by
// exact 64-bit multiply-compare steps to the exact floor.
__device__ __forceinline__ uint32_t dec_target(const DecState& st) {
  const unsigned long long scale = st.range >> 24;
  const unsigned long long diff = st.point - st.lower;
  if (diff >= (scale << 24)) return (1u << 24) - 1u;  // quotient >= 2^24: clamped
  float est = __fdividef((float)diff, (float)scale);
  est = fminf(fmaxf(est, 0.0f), 16777215.0f);
  unsigned long long q = (unsigned long long)est;
  unsigned long long prod = q * scale;  // < 2^64: q < 2^24, scale < 2^40
  while (prod > diff) { --q; prod -= scale; }
  while (diff - prod >= scale) { ++q; prod += scale; }
  return (uint32_t)q;
}
__device__ __forceinline__ void dec_update(DecState& st, uint32_t low, uint32_t high, const uint32_t* in) {
  const unsigned long long scale = st.range >> 24;
  uint32_t prob = high - low;
  if (prob == 0) prob = 1;
  st.lower = st.lower + scale * (unsigned long long)low;
  st.range = scale * (unsigned long long)prob;
  while (st.range < (1ull << 32)) {
    st.lower <<= 32;
    st.range <<= 32;
    const uint32_t w = st.r < st.n ? in[st.r++] : 0u;
    st.point = (st.point << 32) | (unsigned long long)w;
  }
}

// ---------------------------------------------------------------------------
// softmax -> CDF for one row held by one thread.
// Src must provide: __device__ void lane(int l, float (&v)[8]) const
// returning the 8 logits (bias already added) of symbols 8l..8l+7, and
// static constexpr bool kCache: when true, cdf_prepare replaces the row's
// values by their exponentials (put(l, e)) once the maximum is known, and
// every later walk over the row reads them instead of evaluating __expf again
// (the same floats, so the same bits).
// ---------------------------------------------------------------------------
struct CdfRow {
  float mx;
  float inv_t;
  double inv_sum;
  double ws[32];  // reference "warp_start" of each lane (pre fix-up CDF at 8l)
};

__device__ __forceinline__ float cdf_exp(float v, float mx, float inv_t) {
  return __expf(__fmul_rn(__fsub_rn(v, mx), inv_t));
}

template <class Src>
__device__ __forceinline__ void cdf_prepare(const Src& src, float inv_t, CdfRow& R) {
  float mx = -1e30f;
#pragma unroll 1
  for (int l = 0; l < 32; ++l) {
    float v[8];
    src.lane(l, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) mx = fmaxf(mx, v[i]);
  }
  R.mx = mx;
  R.inv_t = inv_t;
  double ts[32];
#pragma unroll 1
  for (int l = 0; l < 32; ++l) {
    float v[8];
    src.lane(l, v);
    double sd = 0.0;
    float e[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      e[i] = cdf_exp(v[i], mx, inv_t);
      sd = __dadd_rn(sd, (double)e[i]);
    }
    if constexpr (Src::kCache) src.put(l, e);
    ts[l] = sd;
    R.ws[l] = sd;
  }
  // shfl_down reduction tree; only lanes < off feed lane 0's result
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int l = 0; l < off; ++l) R.ws[l] = __dadd_rn(R.ws[l], R.ws[l + off]);
  const double inv_sum = 1.0 / R.ws[0];
  R.inv_sum = inv_sum;
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    ts[l] = __dmul_rn(ts[l], inv_sum);
    R.ws[l] = ts[l];
  }
  // inclusive Hillis-Steele scan (shfl_up); descending l reads old values
#pragma unroll
  for (int off = 1; off <= 16; off <<= 1)
#pragma unroll
    for (int l = 31; l >= off; --l) R.ws[l] = __dadd_rn(R.ws[l], R.ws[l - off]);
#pragma unroll
  for (int l = 0; l < 32; ++l) R.ws[l] = __dsub_rn(R.ws[l], ts[l]);
}

// pre-fix-up running CDF values of lane l: p[j] = cdf[8l+j], and the lane's
// 8th value p[7] (the "prev_end" its right neighbour compares against).
template <class Src>
__device__ __forceinline__ void cdf_lane(const Src& src, const CdfRow& R, int l, double (&p)[8]) {
  float v[8];
  src.lane(l, v);
  double run = R.ws[l];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    p[i] = run;
    const float e = Src::kCache ? v[i] : cdf_exp(v[i], R.mx, R.inv_t);
    run = __dadd_rn(run, __dmul_rn((double)e, R.inv_sum));
  }
}
__device__ __forceinline__ double cdf_fix(double my_start, double prev_end) {
  return my_start < prev_end ? __dsub_rn(prev_end, my_start) : 0.0;
}
__device__ __forceinline__ double cdf_post(double pre, double delta) {
  return delta != 0.0 ? __dadd_rn(pre, delta) : pre;
}
__device__ __forceinline__ uint32_t cdf_f(double c) { return (uint32_t)__dmul_rn(c, kCdfScale); }

// Q_k = k + max_{j <= k} floor(C_j * (2^24 - 256)).  The reference quantises
// Q_k = k + floor(C_k * (2^24 - 256)) (range_coder_kernels.cu:917-925), which
// is strictly increasing whenever the fixed-up C is non-decreasing.  Its
// lane-boundary fix-up compares each lane's start with the previous lane's
// PRE-fix-up end, so once C has reached 1.0 (a near-certain prediction) a later
// lane can start one ulp lower: Q_k = Q_{k+1}, an empty interval that no
// decoder can resolve (the reference's stream is then undecodable).  The
// running maximum equals the reference's Q on every row where that Q is
// strictly increasing and repairs exactly the rows where it is not.  Within a
// lane C is non-decreasing, so the running maximum only needs each earlier
// lane's last value.

// [low, high) of symbol s (encoder side)
template <class Src>
__device__ __forceinline__ void cdf_symbol(const Src& src, const CdfRow& R, int s, uint32_t& low,
                                           uint32_t& high) {
  const int L = s >> 3, i = s & 7;
  double p[8];
  double dl = 0.0;   // fix-up delta of the lane being read
  uint32_t pm = 0u;  // max of floor(C * scale) over the lanes before L
#pragma unroll 1
  for (int l = 0; l < L; ++l) {
    cdf_lane(src, R, l, p);
    pm = max(pm, cdf_f(cdf_post(p[7], dl)));
    dl = cdf_fix(R.ws[l + 1], p[7]);
  }
  cdf_lane(src, R, L, p);
  low = max(pm, cdf_f(cdf_post(p[i], dl))) + (uint32_t)s;
  if (s == 255) {
    high = kCdfTotal;
  } else if (i < 7) {
    high = max(pm, cdf_f(cdf_post(p[i + 1], dl))) + (uint32_t)(s + 1);
  } else {
    const double d1 = cdf_fix(R.ws[L + 1], p[7]);
    const uint32_t f = max(pm, cdf_f(cdf_post(p[7], dl)));
    high = max(f, cdf_f(cdf_post(R.ws[L + 1], d1))) + (uint32_t)(s + 1);
  }
}

// Decoder search: lowest s with Q_s <= target < Q_{s+1}
// (warp ballot + __ffs in range_coder_kernels.cu:747-763 picks the lowest),
// over the same Q as cdf_symbol.
template <class Src>
__device__ __forceinline__ int cdf_search(const Src& src, const CdfRow& R, uint32_t target, uint32_t& low,
                                          uint32_t& high) {
  double dl = 0.0;   // fix-up delta of the current lane
  uint32_t rm = 0u;  // running max of floor(C * scale) up to the current symbol
  uint32_t q = 0u;   // Q of the current symbol
#pragma unroll 1
  for (int l = 0; l < 32; ++l) {
    double p[8];
    cdf_lane(src, R, l, p);
    double next0 = 1.0, dn = 0.0;
    if (l < 31) {
      dn = cdf_fix(R.ws[l + 1], p[7]);
      next0 = cdf_post(R.ws[l + 1], dn);
    }
    if (l == 0) {
      rm = cdf_f(cdf_post(p[0], dl));
      q = rm;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = 8 * l + j;
      uint32_t qn;
      if (k == 255) {
        qn = kCdfTotal;
      } else {
        rm = max(rm, cdf_f(j < 7 ? cdf_post(p[j + 1], dl) : next0));
        qn = rm + (uint32_t)(k + 1);
      }
      if (target >= q && target < qn) {
        low = q;
        high = qn;
        return k;
      }
      q = qn;
    }
    dl = dn;
  }
  low = 0u;
  high = 0u;
  return 0;
}

}  // namespace boa
