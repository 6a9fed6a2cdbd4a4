// mamba.cu -- non-GEMM kernels of the compress/decompress step.
//
// Row layout: rows are (chunk b, position tau) with T rows per chunk; the
// decompress step is the T = 1 case of the same kernels, so both directions
// run identical arithmetic per row.
#include <algorithm>
#include "kernels.cuh"
#include "rowmath.cuh"

namespace boa {

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int chunk_len_of(long long n_bytes, int chunk_len, int b, long long stride = 0) {
  const long long rem = n_bytes - (long long)b * (stride ? stride : chunk_len);
  return (int)(rem < chunk_len ? (rem > 0 ? rem : 0) : chunk_len);
}

// ---------------------------------------------------------------- embedding + LN
// One warp per row, ceil(D/32) values per lane (the last ones guarded when
// D is not a multiple of 32, as d_model 80).  Restates the embedding gather
// (utility_kernels.cu:46-72) and LN1 (inference_kernels.cu:293-348).
template <int D>
__global__ void embed_ln_kernel(TokenSrc src, const float* __restrict__ emb, float* __restrict__ x,
                                __nv_bfloat16* __restrict__ xn, long long plane, const float* __restrict__ w,
                                const float* __restrict__ bb, int M) {
  constexpr int V = (D + 31) / 32;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  int tok = 0;
  if (src.mode == 0) {
    tok = src.bytes[row];
  } else if (src.mode == 1) {
    const int b = row / src.T, tau = row - b * src.T;
    const int p = src.t0 + tau;
    const long long stride = src.stride ? src.stride : src.chunk_len;
    if (p < chunk_len_of(src.n_bytes, src.chunk_len, b, stride)) tok = src.bytes[(long long)b * stride + p];
  } else {
    const int b = row;
    const int p = *src.d_t - 1;
    if (p >= 0 && p < src.lane_len[b]) tok = src.bytes[src.lane_base[b] + p];
  }
  float v[V];
  float s = 0.f, sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    v[i] = 0.f;
    if (lane + 32 * i < D) {
      v[i] = emb[(size_t)tok * D + lane + 32 * i];
      x[(size_t)row * D + lane + 32 * i] = v[i];
    }
    s += v[i];
    sq += v[i] * v[i];
  }
  s = warp_sum(s);
  sq = warp_sum(sq);
  const float mean = s / (float)D;
  const float var = sq / (float)D - mean * mean;
  const float inv_std = rsqrtf(var + 1e-5f);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c >= D) break;
    const float y = (v[i] - mean) * inv_std * w[c] + bb[c];
    __nv_bfloat16 h, l;
    split_bf16(y, h, l);
    xn[(size_t)row * D + c] = h;
    xn[plane + (size_t)row * D + c] = l;
  }
}

cudaError_t launch_embed_ln(const TokenSrc& src, const float* emb, int d, float* x, __nv_bfloat16* xn,
                            long long plane, const float* w, const float* b, int M, cudaStream_t st) {
  const int rows_per_block = 8;
  dim3 grid((M + rows_per_block - 1) / rows_per_block), block(32 * rows_per_block);
  switch (d) {
    case 64: embed_ln_kernel<64><<<grid, block, 0, st>>>(src, emb, x, xn, plane, w, b, M); break;
    case 80: embed_ln_kernel<80><<<grid, block, 0, st>>>(src, emb, x, xn, plane, w, b, M); break;
    case 128: embed_ln_kernel<128><<<grid, block, 0, st>>>(src, emb, x, xn, plane, w, b, M); break;
    case 160: embed_ln_kernel<160><<<grid, block, 0, st>>>(src, emb, x, xn, plane, w, b, M); break;
    case 256: embed_ln_kernel<256><<<grid, block, 0, st>>>(src, emb, x, xn, plane, w, b, M); break;
    case 512: embed_ln_kernel<512><<<grid, block, 0, st>>>(src, emb, x, xn, plane, w, b, M); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- causal conv
// Causal depthwise conv (k = 4) + SiLU, window = three carried inputs +
// current (mamba_kernels.cu:158-197, :370-412); conv_tap fixes the sum order
// and rounding, so every launch shape computes the same bits.
// Compress tile: one thread per (chunk, 4 channels) walking the T positions,
// with 128-bit loads of x and stores of u and 64-bit stores of each bf16
// plane (d_model is a multiple of 16, so di % 4 == 0).
__global__ void conv4_kernel(const float* __restrict__ xz, int di, float* __restrict__ cst,
                             const float* __restrict__ cw, const float* __restrict__ cb,
                             __nv_bfloat16* __restrict__ uhl, long long plane, int B, int T, int ph) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int q = di / 4;
  if (idx >= (long long)B * q) return;
  const int b = (int)(idx / q), c = (int)(idx - (long long)b * q) * 4;
  float4* s = reinterpret_cast<float4*>(cst + (size_t)b * 3 * di + c);
  // ring: the first row is position p0 (p0 % 3 = ph); slots hold p0-3, p0-2, p0-1
  const int r0 = ph, r1 = ph == 2 ? 0 : ph + 1, r2 = ph == 0 ? 2 : ph - 1;
  float4 w0 = s[r0 * (di / 4)], w1 = s[r1 * (di / 4)], w2 = s[r2 * (di / 4)];
  const float4* k = reinterpret_cast<const float4*>(cw) + c;
  const float4 k0 = k[0], k1 = k[1], k2 = k[2], k3 = k[3];
  const float4 bias = *reinterpret_cast<const float4*>(cb + c);
  constexpr int PB = 8;  // x fetched 8 positions at a time, one batch ahead
  const size_t row0 = (size_t)b * T;
  float4 cx[PB], nx[PB];
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < PB; ++i)
    cx[i] = i < T ? *reinterpret_cast<const float4*>(xz + (row0 + i) * 2 * di + c) : zero;
  for (int t0 = 0; t0 < T; t0 += PB) {
#pragma unroll
    for (int i = 0; i < PB; ++i)
      nx[i] = t0 + PB + i < T ? *reinterpret_cast<const float4*>(xz + (row0 + t0 + PB + i) * 2 * di + c) : zero;
#pragma unroll
    for (int i = 0; i < PB; ++i) {
      if (t0 + i < T) {
        const size_t row = row0 + t0 + i;
        const float4 xt = cx[i];
        float4 o;
        o.x = conv_tap(w0.x, w1.x, w2.x, xt.x, k0, bias.x);
        o.y = conv_tap(w0.y, w1.y, w2.y, xt.y, k1, bias.y);
        o.z = conv_tap(w0.z, w1.z, w2.z, xt.z, k2, bias.z);
        o.w = conv_tap(w0.w, w1.w, w2.w, xt.w, k3, bias.w);
        __nv_bfloat16 h[4], l[4];
        split_bf16(o.x, h[0], l[0]); split_bf16(o.y, h[1], l[1]);
        split_bf16(o.z, h[2], l[2]); split_bf16(o.w, h[3], l[3]);
        *reinterpret_cast<uint2*>(uhl + row * di + c) = *reinterpret_cast<uint2*>(h);
        *reinterpret_cast<uint2*>(uhl + plane + row * di + c) = *reinterpret_cast<uint2*>(l);
        w0 = w1; w1 = w2; w2 = xt;
      }
    }
#pragma unroll
    for (int i = 0; i < PB; ++i) cx[i] = nx[i];
  }
  // after positions p0 .. p0+T-1 the window holds pn-3, pn-2, pn-1 (pn = p0 + T)
  const int pn = (ph + T) % 3;
  const int q0 = pn, q1 = pn == 2 ? 0 : pn + 1, q2 = pn == 0 ? 2 : pn - 1;
  s[q0 * (di / 4)] = w0; s[q1 * (di / 4)] = w1; s[q2 * (di / 4)] = w2;
}

// Decompress step (T = 1): one thread per (chunk, 4 channels), 128-bit
// accesses; the same conv_tap arithmetic as conv4_kernel.
__global__ void conv_step4_kernel(const float* __restrict__ xz, int di, float* __restrict__ cst,
                                  const float* __restrict__ cw, const float* __restrict__ cb,
                                  __nv_bfloat16* __restrict__ uhl, long long plane, int B, int ph0,
                                  const int* __restrict__ d_pos) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int q = di / 4;
  if (idx >= (long long)B * q) return;
  const int b = (int)(idx / q), c = (int)(idx - (long long)b * q) * 4;
  float4* s = reinterpret_cast<float4*>(cst + (size_t)b * 3 * di + c);
  // ring slot p % 3 holds position p; this step is position p, so the slots
  // hold p-3 (oldest, slot ph), p-2 and p-1, and only slot ph is rewritten
  int ph = (ph0 + (d_pos ? *d_pos % 3 : 0)) % 3;
  const int r1 = ph == 2 ? 0 : ph + 1, r2 = ph == 0 ? 2 : ph - 1;
  const float4 s0 = s[ph * (di / 4)], s1 = s[r1 * (di / 4)], s2 = s[r2 * (di / 4)];
  const float4 x = *reinterpret_cast<const float4*>(xz + (size_t)b * 2 * di + c);
  const float4 bias = *reinterpret_cast<const float4*>(cb + c);
  const float4* k = reinterpret_cast<const float4*>(cw) + c;
  float4 o;
  o.x = conv_tap(s0.x, s1.x, s2.x, x.x, k[0], bias.x);
  o.y = conv_tap(s0.y, s1.y, s2.y, x.y, k[1], bias.y);
  o.z = conv_tap(s0.z, s1.z, s2.z, x.z, k[2], bias.z);
  o.w = conv_tap(s0.w, s1.w, s2.w, x.w, k[3], bias.w);
  __nv_bfloat16 h[4], l[4];
  split_bf16(o.x, h[0], l[0]); split_bf16(o.y, h[1], l[1]); split_bf16(o.z, h[2], l[2]); split_bf16(o.w, h[3], l[3]);
  *reinterpret_cast<uint2*>(uhl + (size_t)b * di + c) = *reinterpret_cast<uint2*>(h);
  *reinterpret_cast<uint2*>(uhl + plane + (size_t)b * di + c) = *reinterpret_cast<uint2*>(l);
  s[ph * (di / 4)] = x;
}

cudaError_t launch_conv(const float* xz, int di, float* cst, const float* cw, const float* cb,
                        __nv_bfloat16* uhl, long long plane, int B, int T, long long pos0, const int* d_pos,
                        cudaStream_t st) {
  if (di % 4 != 0 || pos0 < 0) return cudaErrorInvalidValue;
  const int ph0 = (int)(pos0 % 3);
  if (T == 1) {
    const long long n4 = (long long)B * (di / 4);
    conv_step4_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(xz, di, cst, cw, cb, uhl, plane, B, ph0,
                                                                    d_pos);
    return cudaGetLastError();
  }
  if (d_pos) return cudaErrorInvalidValue;  // tiles take their position from the host
  const long long n4 = (long long)B * (di / 4);
  conv4_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(xz, di, cst, cw, cb, uhl, plane, B, T, ph0);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- selective scan
// One (row, channel) update of the selective scan, shared by the tile and the
// step kernels so both compute identical bits:
//   dt = softplus(delta[:R] . Wdt[c] + b)          (dt_proj, inference_kernels.cu:372-390)
//   h_n = exp(A_n dt) h_n + dt B_n u ;  y = sum_n h_n C_n + D u   (mamba_kernels.cu:271-361)
//   out = y * silu(z)                               (mamba_kernels.cu:130-151)
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// na2 holds A * log2(e) (A = -exp(A_log)), so exp(A dt) = 2^(na2 dt).  The
// sixteen states are updated in pairs with packed f32x2 arithmetic; the dt
// dot product and the sum over states keep two partial sums (even / odd
// terms), combined once.  Every caller runs this same sequence.
template <int R>
__device__ __forceinline__ float scan_update(const float4* __restrict__ dl4, const float2 (&wdt2)[R / 2], float bdt,
                                             const float2 (&na2)[8], float2 (&h)[8], float uv, float z, float dsk) {
  // dl4: the row's delta [dt_in(R) | B(16) | C(16)] as aligned float4 (128-bit shared loads)
  float2 acc2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int k4 = 0; k4 < R / 4; ++k4) {
    const float4 q = dl4[k4];
    acc2 = ffma2(make_float2(q.x, q.y), wdt2[2 * k4], acc2);
    acc2 = ffma2(make_float2(q.z, q.w), wdt2[2 * k4 + 1], acc2);
  }
  const float acc = __fadd_rn(acc2.x, acc2.y);
  const float dt = __logf(__fadd_rn(1.0f, __expf(__fadd_rn(acc, bdt))));  // softplus
  const float dtu = __fmul_rn(dt, uv);
  const float2 dt2 = make_float2(dt, dt), dtu2 = make_float2(dtu, dtu);
  float2 y2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int n4 = 0; n4 < 4; ++n4) {
    const float4 b4 = dl4[R / 4 + n4], c4 = dl4[R / 4 + 4 + n4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int p = 2 * n4 + j;
      const float2 bb = j ? make_float2(b4.z, b4.w) : make_float2(b4.x, b4.y);
      const float2 cc = j ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
      const float2 a = fmul2(na2[p], dt2);
      const float2 dA = make_float2(ex2_ftz(a.x), ex2_ftz(a.y));
      h[p] = ffma2(dA, h[p], fmul2(bb, dtu2));
      y2 = ffma2(h[p], cc, y2);
    }
  }
  float y = __fadd_rn(y2.x, y2.y);
  y = __fmaf_rn(uv, dsk, y);
  return __fmul_rn(y, __fdividef(z, __fadd_rn(1.0f, __expf(-z))));  // y * silu(z)
}

// The scan's u input: the conv writes u only as the bf16 hi / lo planes that
// x_proj consumes, and both scan forms use it as hi + lo (about 2^-17
// relative to the fp32 value), with the same rounding everywhere.
__device__ __forceinline__ float u_from_planes(__nv_bfloat16 hi, __nv_bfloat16 lo) {
  return __fadd_rn(__bfloat162float(hi), __bfloat162float(lo));
}

// Selective-scan state layout, shared by both forms: the di channels of a
// chunk are cut into slices of W (a divisor of di), and each (chunk, slice)
// holds its 16 state rows of W floats contiguously, so the decode form moves
// one contiguous block per work item.  W = di keeps the plain [chunk][16][di]
// order.
__host__ __device__ __forceinline__ size_t scan_state_offset(long long b, int c, int di, int W) {
  return (size_t)b * 16 * di + (size_t)(c / W) * 16 * W + (size_t)(c % W);
}
// Slices of at most 256 channels: measured on B200 with 16384 chunks, the
// decode scan takes 189 / 200 / 224 us at W = 256 / 512 / 128 (d_model 256)
// and 387 / 407 us at W = 256 / 512 (d_model 512, 0.93 of the HBM copy rate).
constexpr int kScanSliceMax = 256;
int scan_slice_width(int di) {
  int W = di;
  while (W > kScanSliceMax && W % 2 == 0) W /= 2;
  return W;
}

// Compress form: thread per (chunk, channel), h[16] in registers across the T
// rows of the tile; the chunk's delta rows are staged in shared memory.
// CPT channels per thread (channels c and c + 128): the per-position delta
// row (dt inputs, B, C) is read from shared memory once for all of them, and
// each channel runs the same scan_update sequence as with one channel.
template <int R, int CPT>
__global__ void __launch_bounds__(128, CPT == 1 ? 5 : 3) scan_tile_kernel(
    const float* __restrict__ delta, int ld, const float* __restrict__ dtw, const float* __restrict__ dtb,
    const float* __restrict__ negA, const float* __restrict__ Dv, const float* __restrict__ xz, int di,
    float* __restrict__ hs, const __nv_bfloat16* __restrict__ uhl, __nv_bfloat16* __restrict__ yhl, long long plane,
    int T, int W) {
  extern __shared__ float sdelta[];  // [T][ld]
  const int b = blockIdx.x;  // chunks on x (y stops at 65535)
  const int cbase = blockIdx.y * blockDim.x * CPT + threadIdx.x;
  {
    const float4* src = reinterpret_cast<const float4*>(delta + (size_t)b * T * ld);
    float4* dst = reinterpret_cast<float4*>(sdelta);
    for (int i = threadIdx.x; i < T * ld / 4; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (cbase >= di) return;  // di is a multiple of 128 * CPT whenever CPT > 1
  float2 wdt[CPT][R / 2];
  float2 na[CPT][8], h[CPT][8];
  float* hp[CPT];
  float bdt[CPT], dsk[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = cbase + 128 * j;
#pragma unroll
    for (int k = 0; k < R / 2; ++k) wdt[j][k] = reinterpret_cast<const float2*>(dtw + (size_t)c * R)[k];
    hp[j] = hs + scan_state_offset(b, c, di, W);  // rows n at stride W
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      na[j][p] = reinterpret_cast<const float2*>(negA + (size_t)c * 16)[p];
      h[j][p] = make_float2(hp[j][(size_t)(2 * p) * W], hp[j][(size_t)(2 * p + 1) * W]);
    }
    bdt[j] = dtb[c];
    dsk[j] = Dv[c];
  }
  // u and z are fetched in batches of PB positions, one batch ahead, so each
  // thread keeps several loads in flight instead of waiting once per position.
  constexpr int PB = CPT == 1 ? 4 : 2;
  const size_t row0 = (size_t)b * T;
  // u is prefetched as its raw hi / lo planes and combined only where it is
  // used, so the loads stay in flight across a batch
  __nv_bfloat16 cuh[CPT][PB], cul[CPT][PB], nuh[CPT][PB], nul[CPT][PB];
  float cz[CPT][PB], nz[CPT][PB];
  const __nv_bfloat16 bz = __float2bfloat16_rn(0.f);
#pragma unroll
  for (int j = 0; j < CPT; ++j)
#pragma unroll
    for (int i = 0; i < PB; ++i) {
      const bool ok = i < T;
      const int c = cbase + 128 * j;
      cuh[j][i] = ok ? uhl[(row0 + i) * di + c] : bz;
      cul[j][i] = ok ? uhl[plane + (row0 + i) * di + c] : bz;
      cz[j][i] = ok ? xz[(row0 + i) * 2 * di + di + c] : 0.f;
    }
  for (int t0 = 0; t0 < T; t0 += PB) {
#pragma unroll
    for (int j = 0; j < CPT; ++j)
#pragma unroll
      for (int i = 0; i < PB; ++i) {
        const bool ok = t0 + PB + i < T;
        const int c = cbase + 128 * j;
        nuh[j][i] = ok ? uhl[(row0 + t0 + PB + i) * di + c] : bz;
        nul[j][i] = ok ? uhl[plane + (row0 + t0 + PB + i) * di + c] : bz;
        nz[j][i] = ok ? xz[(row0 + t0 + PB + i) * 2 * di + di + c] : 0.f;
      }
#pragma unroll
    for (int i = 0; i < PB; ++i) {
      const int tau = t0 + i;
      if (tau < T) {
        const size_t row = row0 + tau;
        const float4* dl = reinterpret_cast<const float4*>(sdelta + tau * ld);
        float o[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j)
          o[j] = scan_update<R>(dl, wdt[j], bdt[j], na[j], h[j], u_from_planes(cuh[j][i], cul[j][i]), cz[j][i], dsk[j]);
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
          const int c = cbase + 128 * j;
          __nv_bfloat16 hh, ll;
          split_bf16(o[j], hh, ll);
          yhl[row * di + c] = hh;
          yhl[plane + row * di + c] = ll;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < CPT; ++j)
#pragma unroll
      for (int i = 0; i < PB; ++i) { cuh[j][i] = nuh[j][i]; cul[j][i] = nul[j][i]; cz[j][i] = nz[j][i]; }
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j)
#pragma unroll
    for (int p = 0; p < 8; ++p) { hp[j][(size_t)(2 * p) * W] = h[j][p].x; hp[j][(size_t)(2 * p + 1) * W] = h[j][p].y; }
}

// Decompress form (T = 1): persistent CTAs stream each chunk's 16 x di state
// through shared memory with bulk async copies, so the kernel runs at HBM
// rate instead of being bound by per-thread load latency.  One thread per
// channel; a CTA covers one slice of W channels (16 x W floats of state per
// item, 32 KB at W = 512), several CTAs per SM, and each keeps two items in
// flight ahead of the one it computes.
constexpr int kScanStages = 3;
template <int R>
__global__ void __launch_bounds__(512) scan_step_kernel(const float* __restrict__ delta, int ld,
                                                        const float* __restrict__ dtw, const float* __restrict__ dtb,
                                                        const float* __restrict__ negA, const float* __restrict__ Dv,
                                                        const float* __restrict__ xz,
                                                        int di, float* __restrict__ hs,
                                                        const __nv_bfloat16* __restrict__ uhl,
                                                        __nv_bfloat16* __restrict__ yhl, long long plane, int B) {
  // State layout: see scan_state_offset (one contiguous 16 x W block per item).
  // Work item w = (chunk w / n_sl, channel slice w % n_sl); the block's W
  // threads own channels sl * W + threadIdx.x.  A stage holds one item: its
  // 16 state rows (W floats each; one copy when the slice is the whole row),
  // the u and z slices and the chunk's full delta row.
  extern __shared__ __align__(128) uint8_t sm[];
  const int W = blockDim.x, n_sl = di / W;
  const uint32_t row_bytes = (uint32_t)W * 4, st_bytes = 16u * row_bytes, uz_bytes = row_bytes;
  const uint32_t dl_bytes = ((uint32_t)ld * 4 + 15) & ~15u;
  const uint32_t stage_bytes = st_bytes + 2 * uz_bytes + dl_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kScanStages * stage_bytes);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kScanStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const long long n_items = (long long)B * n_sl;
  auto item = [&](int i) { return (long long)blockIdx.x + (long long)i * gridDim.x; };
  auto state_ptr = [&](long long w) { return hs + (size_t)w * 16 * W; };  // (chunk, slice) blocks in order
  auto issue = [&](int i, int s) {
    const long long w = item(i);
    const long long b = w / n_sl;
    const int c0 = (int)(w % n_sl) * W;
    uint8_t* p = sm + s * stage_bytes;
    mbar_arrive_expect_tx(&full[s], st_bytes + 2 * uz_bytes + (uint32_t)ld * 4);
    bulk_load(p, state_ptr(w), st_bytes, &full[s]);
    // u as its hi and lo planes
    bulk_load(p + st_bytes, uhl + (size_t)b * di + c0, uz_bytes / 2, &full[s]);
    bulk_load(p + st_bytes + uz_bytes / 2, uhl + plane + (size_t)b * di + c0, uz_bytes / 2, &full[s]);
    bulk_load(p + st_bytes + uz_bytes, xz + (size_t)b * 2 * di + di + c0, uz_bytes, &full[s]);
    bulk_load(p + st_bytes + 2 * uz_bytes, delta + (size_t)b * ld, (uint32_t)ld * 4, &full[s]);
  };
  const int n_mine = (int)((n_items - (long long)blockIdx.x + gridDim.x - 1) / gridDim.x);
  // items i + 1 .. i + kScanStages - 1 are in flight while item i is computed;
  // the stage of item i - 1 is refilled once its state store has been read
  if (tid == 0)
    for (int s = 0; s < kScanStages - 1 && s < n_mine; ++s) issue(s, s);
  float2 wdt[R / 2], na[8];
  float bdt = 0.f, dsk = 0.f;
  int c_prev = -1;
  bool alive = true;
  for (int i = 0; i < n_mine; ++i) {
    const int s = i % kScanStages;
    const long long w = item(i);
    const int c = (int)(w % n_sl) * W + tid;
    if (c != c_prev) {  // per-channel parameters (reloaded only when the slice changes)
#pragma unroll
      for (int k = 0; k < R / 2; ++k) wdt[k] = reinterpret_cast<const float2*>(dtw + (size_t)c * R)[k];
#pragma unroll
      for (int p = 0; p < 8; ++p) na[p] = reinterpret_cast<const float2*>(negA + (size_t)c * 16)[p];
      bdt = dtb[c];
      dsk = Dv[c];
      c_prev = c;
    }
    uint8_t* p = sm + s * stage_bytes;
    if (!mbar_wait(&full[s], (i / kScanStages) & 1)) alive = false;
    if (alive) {
      float* hsm = reinterpret_cast<float*>(p);
      const __nv_bfloat16* uhs = reinterpret_cast<const __nv_bfloat16*>(p + st_bytes);  // hi [W] | lo [W]
      const float* zsm = reinterpret_cast<const float*>(p + st_bytes + uz_bytes);
      const float4* dl = reinterpret_cast<const float4*>(p + st_bytes + 2 * uz_bytes);
      float2 h[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) h[q] = make_float2(hsm[(2 * q) * W + tid], hsm[(2 * q + 1) * W + tid]);
      const float o = scan_update<R>(dl, wdt, bdt, na, h, u_from_planes(uhs[tid], uhs[W + tid]), zsm[tid], dsk);
#pragma unroll
      for (int q = 0; q < 8; ++q) { hsm[(2 * q) * W + tid] = h[q].x; hsm[(2 * q + 1) * W + tid] = h[q].y; }
      const long long b = w / n_sl;
      __nv_bfloat16 hh, ll;
      split_bf16(o, hh, ll);
      yhl[(size_t)b * di + c] = hh;
      yhl[plane + (size_t)b * di + c] = ll;
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      if (alive) {
        bulk_store(state_ptr(w), p, st_bytes);
        bulk_commit();
      }
      const int nxt = i + kScanStages - 1;
      if (nxt < n_mine && alive) {
        bulk_wait_read_1();  // item i - 1's store has read its stage
        issue(nxt, nxt % kScanStages);
      }
    }
  }
  if (tid == 0) bulk_wait_all();
}

cudaError_t launch_scan(const float* delta, int ld, int r, const float* dtw, const float* dtb, const float* negA,
                        const float* Dv, const float* xz, int di, float* hs, const __nv_bfloat16* uhl,
                        __nv_bfloat16* yhl,
                        long long plane, int B, int T, cudaStream_t st) {
  if (T == 1 && di <= 1024 && (ld * 4) % 16 == 0) {
    // channel slices of at most 256 (a divisor of di): several small
    // pipelines per SM keep more state bytes in flight than one wide one
    const int W = scan_slice_width(di);
    const size_t stage = (size_t)16 * W * 4 + 2 * (size_t)W * 4 + (((size_t)ld * 4 + 15) & ~size_t(15));
    const size_t sm = kScanStages * stage + kScanStages * 8;
    int dev = 0, n_sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    const int per_sm = (int)std::max<size_t>(1, std::min<size_t>((size_t)(220 * 1024) / sm, 2048 / W));
    const long long items = (long long)B * (di / W);
    const int grid = (int)std::min<long long>(items, (long long)n_sm * per_sm);
    switch (r) {
#define BOA_STEP_CASE(RR)                                                                                          \
  case RR:                                                                                                         \
    scan_step_kernel<RR><<<grid, W, sm, st>>>(delta, ld, dtw, dtb, negA, Dv, xz, di, hs, uhl, yhl, plane, B);        \
    break;
      BOA_STEP_CASE(4)
      BOA_STEP_CASE(8)
      BOA_STEP_CASE(16)
      BOA_STEP_CASE(32)
#undef BOA_STEP_CASE
      default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
  }
  const int W = scan_slice_width(di);
  const int cpt = di % 256 == 0 ? 2 : 1;  // 3.57 against 3.68 ms per 16384 x 64 tile at d_model 256
  dim3 block(128), grid(B, (di + 128 * cpt - 1) / (128 * cpt));
  const size_t sm = (size_t)T * ld * sizeof(float);
  if (sm > 200 * 1024 || (T * ld) % 4) return cudaErrorInvalidValue;
  switch (r) {
#define BOA_SCAN_CASE(RR)                                                                                                \
  case RR:                                                                                                               \
    if (cpt == 2)                                                                                                      \
      scan_tile_kernel<RR, 2><<<grid, block, sm, st>>>(delta, ld, dtw, dtb, negA, Dv, xz, di, hs, uhl, yhl, plane, T, W); \
    else                                                                                                               \
      scan_tile_kernel<RR, 1><<<grid, block, sm, st>>>(delta, ld, dtw, dtb, negA, Dv, xz, di, hs, uhl, yhl, plane, T, W); \
    break;
    BOA_SCAN_CASE(4)
    BOA_SCAN_CASE(8)
    BOA_SCAN_CASE(16)
    BOA_SCAN_CASE(32)
#undef BOA_SCAN_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// attributes for >48 KB dynamic shared memory, set once per device
cudaError_t scan_prepare_device() {
  const int big = 227 * 1024;
  cudaError_t e;
#define BOA_ATTR(RR)                                                                                          \
  if ((e = cudaFuncSetAttribute(scan_step_kernel<RR>, cudaFuncAttributeMaxDynamicSharedMemorySize, big)) != \
      cudaSuccess)                                                                                            \
    return e;                                                                                                 \
  if ((e = cudaFuncSetAttribute(scan_tile_kernel<RR, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big)) != \
      cudaSuccess)                                                                                               \
    return e;                                                                                                    \
  if ((e = cudaFuncSetAttribute(scan_tile_kernel<RR, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big)) != \
      cudaSuccess)                                                                                               \
    return e;
  BOA_ATTR(4)
  BOA_ATTR(8)
  BOA_ATTR(16)
  BOA_ATTR(32)
#undef BOA_ATTR
  return cudaSuccess;
}

// ---------------------------------------------------------------- minGRU
__global__ void mingru_kernel(const float* __restrict__ zh, int d, float* __restrict__ hstate,
                              float* __restrict__ xo, int B, int T) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)B * d) return;
  const int b = (int)(idx / d), c = (int)(idx - (long long)b * d);
  float h = hstate[idx];
  for (int tau = 0; tau < T; ++tau) {
    const size_t row = (size_t)b * T + tau;
    const float z = 1.0f / (1.0f + expf(-zh[row * 2 * d + c]));
    const float hr = zh[row * 2 * d + d + c];
    const float ht = hr >= 0.f ? hr + 0.5f : 1.0f / (1.0f + expf(-hr));
    h = (1.0f - z) * h + z * ht;
    xo[row * d + c] = h;
  }
  hstate[idx] = h;
}
cudaError_t launch_mingru(const float* zh, int d, float* hs, float* xo, int B, int T, cudaStream_t st) {
  const long long n = (long long)B * d;
  mingru_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(zh, d, hs, xo, B, T);
  return cudaGetLastError();
}

template <int D, bool RMS>
__global__ void add_ln_kernel(float* __restrict__ x, const float* __restrict__ y, __nv_bfloat16* __restrict__ xn,
                              long long plane, const float* __restrict__ w, const float* __restrict__ bb, int M) {
  constexpr int V = (D + 31) / 32;  // the last ones guarded when D is not a multiple of 32
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float v[V];
  float s = 0.f, sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    v[i] = 0.f;
    if (lane + 32 * i >= D) continue;
    const size_t o = (size_t)row * D + lane + 32 * i;
    float t = x[o];
    if (y) { t = y[o] + t; x[o] = t; }
    v[i] = t; s += t; sq += t * t;
  }
  s = warp_sum(s);
  sq = warp_sum(sq);
  float mean = 0.f, inv;
  if (RMS) {
    inv = rsqrtf(sq / (float)D + 1e-6f);
  } else {
    mean = s / (float)D;
    inv = rsqrtf(sq / (float)D - mean * mean + 1e-5f);
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = lane + 32 * i;
    if (c >= D) break;
    const float o = RMS ? v[i] * inv * w[c] : (v[i] - mean) * inv * w[c] + bb[c];
    __nv_bfloat16 h, l;
    split_bf16(o, h, l);
    xn[(size_t)row * D + c] = h;
    xn[plane + (size_t)row * D + c] = l;
  }
}
template <bool RMS>
static cudaError_t launch_add_ln_t(float* x, const float* y, int d, __nv_bfloat16* xn, long long plane,
                                   const float* w, const float* b, int M, cudaStream_t st) {
  dim3 grid((M + 7) / 8), block(256);
  switch (d) {
    case 64: add_ln_kernel<64, RMS><<<grid, block, 0, st>>>(x, y, xn, plane, w, b, M); break;
    case 80: add_ln_kernel<80, RMS><<<grid, block, 0, st>>>(x, y, xn, plane, w, b, M); break;
    case 128: add_ln_kernel<128, RMS><<<grid, block, 0, st>>>(x, y, xn, plane, w, b, M); break;
    case 160: add_ln_kernel<160, RMS><<<grid, block, 0, st>>>(x, y, xn, plane, w, b, M); break;
    case 256: add_ln_kernel<256, RMS><<<grid, block, 0, st>>>(x, y, xn, plane, w, b, M); break;
    case 512: add_ln_kernel<512, RMS><<<grid, block, 0, st>>>(x, y, xn, plane, w, b, M); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}
cudaError_t launch_add_ln(float* x, const float* y, int d, __nv_bfloat16* xn, long long plane, const float* w,
                          const float* b, int M, cudaStream_t st) {
  return launch_add_ln_t<false>(x, y, d, xn, plane, w, b, M, st);
}
cudaError_t launch_rms_split(const float* x, int d, const float* w, __nv_bfloat16* xn, long long plane, int M,
                             cudaStream_t st) {
  return launch_add_ln_t<true>(const_cast<float*>(x), nullptr, d, xn, plane, w, nullptr, M, st);
}

// ---------------------------------------------------------------- range coder bookkeeping
__global__ void enc_init_kernel(EncState* es, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) enc_init(es[b]);
}
cudaError_t launch_enc_init(EncState* es, int B, cudaStream_t st) {
  enc_init_kernel<<<(B + 255) / 256, 256, 0, st>>>(es, B);
  return cudaGetLastError();
}

// Thread per chunk: encodes positions t0..t0+T-1 whose next byte exists
// (encode loop of range_coder_kernels.cu:856-966 with the CDF already reduced
// to (low, high) by the head epilogue).
__global__ void encode_tile_kernel(const uint2* __restrict__ lf, EncState* es, uint32_t* pitch_buf, int pitch,
                                   int B, int T, int t0, long long n_bytes, int chunk_len, long long stride) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int len = chunk_len_of(n_bytes, chunk_len, b, stride);
  int n = len - 1 - t0;
  if (n <= 0) return;
  if (n > T) n = T;
  EncState s = es[b];
  if (s.bad) return;
  uint32_t* out = pitch_buf + (size_t)b * pitch;
  const uint2* p = lf + (size_t)b * T;
  for (int i = 0; i < n; ++i) {
    const uint2 v = p[i];
    if (!enc_symbol(s, v.x, v.y - v.x, out, pitch)) { set_dev_error(BOA_ERR_STREAM_OVERFLOW); s.bad = 1; break; }
  }
  es[b] = s;
}
cudaError_t launch_encode_tile(const uint2* lf, EncState* es, uint32_t* pitch_buf, int pitch, int B, int T, int t0,
                               long long n_bytes, int chunk_len, long long stride, cudaStream_t st) {
  encode_tile_kernel<<<(B + 127) / 128, 128, 0, st>>>(lf, es, pitch_buf, pitch, B, T, t0, n_bytes, chunk_len, stride);
  return cudaGetLastError();
}

// Flush every stream.  A stream whose coding stopped (state.bad) or whose
// flush does not fit gets size `failed_size`; `report` also records the
// failure in the device error word (handle-based callers read it there,
// handle-free callers see only the size).
__global__ void enc_finish_kernel(EncState* es, uint32_t* pitch_buf, int pitch, uint32_t* sizes, int B,
                                  uint32_t failed_size, int report) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  EncState s = es[b];
  const int w = s.bad ? -1 : enc_finish(s, pitch_buf + (size_t)b * pitch, pitch);
  if (w < 0 && !s.bad && report) set_dev_error(BOA_ERR_STREAM_OVERFLOW);
  if (w < 0) s.bad = 1;
  sizes[b] = w < 0 ? failed_size : (uint32_t)w;
  es[b] = s;
}
cudaError_t launch_enc_finish(EncState* es, uint32_t* pitch_buf, int pitch, uint32_t* sizes, int B, cudaStream_t st,
                              uint32_t failed_size, bool report) {
  enc_finish_kernel<<<(B + 255) / 256, 256, 0, st>>>(es, pitch_buf, pitch, sizes, B, failed_size, report ? 1 : 0);
  return cudaGetLastError();
}

// single-block exclusive scan; offsets[B] = total
__global__ void offsets_kernel(const uint32_t* sizes, unsigned long long* off, int B) {
  __shared__ unsigned long long part[1024];
  const int t = threadIdx.x, nt = blockDim.x;
  const unsigned long long base = off[0];  // running total of earlier batches
  const int per = (B + nt - 1) / nt;
  const int lo = t * per, hi = min(B, lo + per);
  unsigned long long s = 0;
  for (int i = lo; i < hi; ++i) s += sizes[i];
  part[t] = s;
  __syncthreads();
  if (t == 0) {
    unsigned long long run = base;
    for (int i = 0; i < nt; ++i) { const unsigned long long v = part[i]; part[i] = run; run += v; }
    off[B] = run;
  }
  __syncthreads();
  unsigned long long run = part[t];
  for (int i = lo; i < hi; ++i) { off[i] = run; run += sizes[i]; }
}
cudaError_t launch_offsets(const uint32_t* sizes, unsigned long long* off, int B, cudaStream_t st) {
  offsets_kernel<<<1, 1024, 0, st>>>(sizes, off, B);
  return cudaGetLastError();
}

__global__ void compact_kernel(const uint32_t* __restrict__ pitch_buf, int pitch, const uint32_t* __restrict__ sizes,
                               const unsigned long long* __restrict__ off, uint32_t* __restrict__ payload) {
  const int b = blockIdx.x;
  const uint32_t n = sizes[b];
  const uint32_t* src = pitch_buf + (size_t)b * pitch;
  uint32_t* dst = payload + off[b];
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}
cudaError_t launch_compact(const uint32_t* pitch_buf, int pitch, const uint32_t* sizes,
                           const unsigned long long* off, uint32_t* payload, int B, cudaStream_t st) {
  compact_kernel<<<B, 256, 0, st>>>(pitch_buf, pitch, sizes, off, payload);
  return cudaGetLastError();
}

__global__ void first_bytes_kernel(const uint8_t* data, long long n_bytes, int chunk_len, long long stride,
                                   uint8_t* first, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (!stride) stride = chunk_len;
  first[b] = chunk_len_of(n_bytes, chunk_len, b, stride) > 0 ? data[(long long)b * stride] : 0;
}
cudaError_t launch_first_bytes(const uint8_t* data, long long n_bytes, int chunk_len, long long stride, uint8_t* first,
                               int B, cudaStream_t st) {
  first_bytes_kernel<<<(B + 255) / 256, 256, 0, st>>>(data, n_bytes, chunk_len, stride, first, B);
  return cudaGetLastError();
}

// interleaved (warm-start) lanes: lane b of iteration `iter` coded chunk
// iter + b * S (boa.cpp:395-406, :414); move its results to chunk order
__global__ void lanes_scatter_kernel(const uint32_t* __restrict__ pitch_buf, int pitch,
                                     const uint32_t* __restrict__ lane_sizes, const uint8_t* __restrict__ lane_first,
                                     uint32_t* __restrict__ slots, uint32_t* __restrict__ sizes,
                                     uint8_t* __restrict__ first, int iter, int S) {
  const int b = blockIdx.x;
  const size_t c = (size_t)iter + (size_t)b * S;
  const uint32_t n = lane_sizes[b];
  if (threadIdx.x == 0) { sizes[c] = n; first[c] = lane_first[b]; }
  const uint32_t* src = pitch_buf + (size_t)b * pitch;
  uint32_t* dst = slots + c * pitch;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}
cudaError_t launch_lanes_scatter(const uint32_t* pitch_buf, int pitch, const uint32_t* lane_sizes,
                                 const uint8_t* lane_first, uint32_t* slots, uint32_t* sizes, uint8_t* first, int iter,
                                 int S, int B, cudaStream_t st) {
  lanes_scatter_kernel<<<B, 256, 0, st>>>(pitch_buf, pitch, lane_sizes, lane_first, slots, sizes, first, iter, S);
  return cudaGetLastError();
}

__global__ void lanes_gather_kernel(const unsigned long long* off, const uint32_t* sizes, const uint8_t* first,
                                    long long n_bytes, int chunk_len, int c0, int S, int B,
                                    unsigned long long* lane_off, uint32_t* lane_size, uint8_t* lane_first,
                                    long long* lane_base, int* lane_len) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const long long c = (long long)c0 + (long long)b * S;
  lane_off[b] = off[c];
  lane_size[b] = sizes[c];
  lane_first[b] = first[c];
  lane_base[b] = c * chunk_len;
  const long long rem = n_bytes - c * chunk_len;
  lane_len[b] = (int)(rem < chunk_len ? (rem > 0 ? rem : 0) : chunk_len);
}
cudaError_t launch_lanes_gather(const unsigned long long* off, const uint32_t* sizes, const uint8_t* first,
                                long long n_bytes, int chunk_len, int c0, int S, int B, unsigned long long* lane_off,
                                uint32_t* lane_size, uint8_t* lane_first, long long* lane_base, int* lane_len,
                                cudaStream_t st) {
  lanes_gather_kernel<<<(B + 255) / 256, 256, 0, st>>>(off, sizes, first, n_bytes, chunk_len, c0, S, B, lane_off,
                                                       lane_size, lane_first, lane_base, lane_len);
  return cudaGetLastError();
}

// decoder init (range_coder_kernels.cu:319-335) + raw first byte (:792-826)
__global__ void dec_init_kernel(DecState* ds, const uint32_t* payload, const unsigned long long* off,
                                const uint32_t* sizes, const uint8_t* first, uint8_t* out, const long long* lane_base,
                                const int* lane_len, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  DecState s;
  dec_init(s, payload + off[b], (int)sizes[b]);
  ds[b] = s;
  if (first && lane_len[b] > 0) out[lane_base[b]] = first[b];
}
cudaError_t launch_dec_init(DecState* ds, const uint32_t* payload, const unsigned long long* off, const uint32_t* sizes,
                            const uint8_t* first, uint8_t* out, const long long* lane_base, const int* lane_len, int B,
                            cudaStream_t st) {
  dec_init_kernel<<<(B + 255) / 256, 256, 0, st>>>(ds, payload, off, sizes, first, out, lane_base, lane_len, B);
  return cudaGetLastError();
}
cudaError_t launch_rc_decode_init(DecState* ds, const uint32_t* payload, const unsigned long long* off,
                                  const uint32_t* sizes, int n, cudaStream_t st) {
  dec_init_kernel<<<(n + 255) / 256, 256, 0, st>>>(ds, payload, off, sizes, nullptr, nullptr, nullptr, nullptr, n);
  return cudaGetLastError();
}

// Failure-detection self-test: one thread waits on a shared-memory barrier
// that nothing arrives on.  The bounded wait gives up after limit_ns, records
// BOA_ERR_TIMEOUT in the device error word and the kernel returns normally.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int* ok) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_mbar_init();
  *ok = mbar_wait_for(&bar, 0, limit_ns) ? 1 : 0;
}
cudaError_t launch_wait_selftest(uint64_t limit_ns, int* ok) {
  wait_selftest_kernel<<<1, 1>>>(limit_ns, ok);
  return cudaGetLastError();
}

__global__ void set_counter_kernel(int* d_t, int v) { *d_t = v; }
__global__ void increment_kernel(int* d_t) {
  d_t[0] += 1;
  d_t[1] += 1;
}
cudaError_t launch_set_counter(int* d_t, int v, cudaStream_t st) {
  set_counter_kernel<<<1, 1, 0, st>>>(d_t, v);
  return cudaGetLastError();
}
cudaError_t launch_increment(int* d_t, cudaStream_t st) {
  increment_kernel<<<1, 1, 0, st>>>(d_t);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- integer-CDF coder
// Encoder: thread per stream reads only Q[s] and Q[s+1] of each step.
// A failed stream is marked in its state (and, with `report`, in the device
// error word) and codes nothing more.
__global__ void rc_encode_cdf_kernel(EncState* es, const uint32_t* __restrict__ cdf, const uint8_t* __restrict__ syms,
                                     int n_streams, int n_steps, uint32_t* pitch_buf, int pitch, int report) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_streams) return;
  EncState s = es[i];
  if (s.bad) return;
  uint32_t* out = pitch_buf + (size_t)i * pitch;
  // the loads do not depend on the coder state: fetch 8 steps' (Q[s], Q[s+1])
  // pairs before coding them, so 8 scattered reads per thread are in flight
  constexpr int kAhead = 8;
  for (int t0 = 0; t0 < n_steps && !s.bad; t0 += kAhead) {
    uint32_t lo[kAhead], hi[kAhead];
#pragma unroll
    for (int j = 0; j < kAhead; ++j) {
      if (t0 + j < n_steps) {
        const size_t rowi = (size_t)(t0 + j) * n_streams + i;
        const int sym = __ldcs(syms + rowi);
        const uint32_t* q = cdf + rowi * 257;
        lo[j] = __ldcs(q + sym);
        hi[j] = __ldcs(q + sym + 1);
      }
    }
#pragma unroll
    for (int j = 0; j < kAhead; ++j) {
      if (t0 + j >= n_steps || s.bad) break;
      // a caller-supplied CDF must give the coded symbol a non-empty interval
      // inside [0, 2^24]; anything else would code a stream that cannot decode
      if (hi[j] <= lo[j] || hi[j] > (1u << 24)) { if (report) set_dev_error(BOA_ERR_BAD_INPUT); s.bad = 1; break; }
      if (!enc_symbol(s, lo[j], hi[j] - lo[j], out, pitch)) {
        if (report) set_dev_error(BOA_ERR_STREAM_OVERFLOW);
        s.bad = 1;
        break;
      }
    }
  }
  es[i] = s;
}
cudaError_t launch_rc_encode_cdf(EncState* es, const uint32_t* cdf, const uint8_t* syms, int n_streams, int n_steps,
                                 uint32_t* pitch_buf, int pitch, cudaStream_t st, bool report) {
  rc_encode_cdf_kernel<<<(n_streams + 127) / 128, 128, 0, st>>>(es, cdf, syms, n_streams, n_steps, pitch_buf, pitch,
                                                                report ? 1 : 0);
  return cudaGetLastError();
}

// Decoder: two streams per warp, one per 16-lane half.  Lane l of a half
// holds Q[l + 16k] (k = 0..15), so each of a row's sixteen loads is one
// 64-byte segment per stream, and the next step's row is loaded before the
// current step's search so the two overlap.  Search: the decoded symbol is
// the s with Q[s] <= target < Q[s+1] (range_coder_kernels.cu:743-763).  For a
// non-decreasing CDF the entries <= target are exactly Q[0..s], so every
// lane counts its entries <= target; one warp reduction sums both halves at
// once (half 1's count shifted into the upper 16 bits) and gives s + 1;
// Q[256] = 2^24 exceeds every target.  (The reference's lowest-match rule
// agrees with this on every non-decreasing CDF, which includes every CDF the
// encoder can code.)  A count of 0 (Q[0] > target) decodes symbol 0 with an
// empty interval, as the reference's no-match path does.  The coder state is
// uniform within a half, so the scalar coder arithmetic is shared by two
// streams' worth of lanes instead of one.
__device__ __forceinline__ void dec_row_load(const uint32_t* __restrict__ q, int hl, uint32_t (&v)[16]) {
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = __ldcs(q + hl + 16 * k);
}
__global__ void __launch_bounds__(256) rc_decode_cdf_kernel(DecState* ds, const uint32_t* __restrict__ cdf,
                                                            const uint32_t* __restrict__ payload,
                                                            const unsigned long long* __restrict__ off, int n_streams,
                                                            int n_steps, uint8_t* __restrict__ syms) {
  const int half = (threadIdx.x >> 4) & 1, hl = threadIdx.x & 15;
  const int i = (blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5)) * 2 + half;
  if (i - half >= n_streams) return;        // whole warp past the end
  const bool live = i < n_streams;          // an odd last stream leaves half 1 idle (it still joins the warp ops)
  const int ii = live ? i : i - 1;          // idle half mirrors half 0's reads
  DecState s = ds[ii];
  const uint32_t* in = payload + off[ii];
  uint32_t v[16];
  dec_row_load(cdf + (size_t)ii * 257, hl, v);
  for (int t = 0; t < n_steps; ++t) {
    const size_t rowi = (size_t)t * n_streams + ii;
    uint32_t nv[16];
    if (t + 1 < n_steps) dec_row_load(cdf + (rowi + n_streams) * 257, hl, nv);
    const uint32_t target = dec_target(s);
    unsigned cnt = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) cnt += v[k] <= target ? 1u : 0u;
    const unsigned both = __reduce_add_sync(0xffffffffu, cnt << (16 * half));
    const int c = (int)((both >> (16 * half)) & 0xffffu);
    int sym = 0;
    uint32_t lo = 0, hi = 0;
    const int sk = c > 0 ? c - 1 : 0, k = sk >> 4, kn = (sk + 1) >> 4;
    uint32_t a = v[0], b = v[0];
#pragma unroll
    for (int j = 1; j < 16; ++j) {  // register selects, no local memory
      if (j == k) a = v[j];
      if (j == kn) b = v[j];
    }
    const uint32_t la = __shfl_sync(0xffffffffu, a, half * 16 + (sk & 15));
    const uint32_t lb = __shfl_sync(0xffffffffu, b, half * 16 + ((sk + 1) & 15));
    if (c > 0) {
      sym = sk;
      lo = la;
      hi = sym == 255 ? __ldg(cdf + rowi * 257 + 256) : lb;
    }
    if (hl == 0 && live) syms[rowi] = (uint8_t)sym;
    dec_update(s, lo, hi, in);
    if (t + 1 < n_steps) {
#pragma unroll
      for (int q = 0; q < 16; ++q) v[q] = nv[q];
    }
  }
  if (hl == 0 && live) ds[i] = s;
}
cudaError_t launch_rc_decode_cdf(DecState* ds, const uint32_t* cdf, const uint32_t* payload,
                                 const unsigned long long* off, int n_streams, int n_steps, uint8_t* syms,
                                 cudaStream_t st) {
  const int warps = (n_streams + 1) / 2;
  rc_decode_cdf_kernel<<<(warps + 7) / 8, 256, 0, st>>>(ds, cdf, payload, off, n_streams, n_steps, syms);
  return cudaGetLastError();
}

// test hook: CDF of logits rows with the shared CDF code (one thread per row)
struct GlobalRow {
  const float* p;
  static constexpr bool kCache = false;
  __device__ __forceinline__ void put(int, const float (&)[8]) const {}
  __device__ __forceinline__ void lane(int l, float (&v)[8]) const {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = p[l * 8 + i];
  }
};
__global__ void cdf_rows_kernel(const float* lg, int rows, float inv_t, uint32_t* Q) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  GlobalRow src{lg + (size_t)r * 256};
  CdfRow R;
  cdf_prepare(src, inv_t, R);
  uint32_t* q = Q + (size_t)r * 257;
  for (int s = 0; s < 256; ++s) {
    uint32_t lo, hi;
    cdf_symbol(src, R, s, lo, hi);
    q[s] = lo;
    if (s == 255) q[256] = hi;
  }
}
cudaError_t launch_cdf_rows(const float* lg, int rows, float inv_t, uint32_t* Q, cudaStream_t st) {
  cdf_rows_kernel<<<(rows + 63) / 64, 64, 0, st>>>(lg, rows, inv_t, Q);
  return cudaGetLastError();
}

}  // namespace boa
