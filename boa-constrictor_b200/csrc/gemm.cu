// gemm.cu -- tcgen05 GEMM for sm_100a with fused epilogues.
//
// Replaces the reference's SIMT fp32 GEMM (ker_gemm_register_tiled_64x64_strided,
// gemm_kernels.cu:176-314, launchers :378-426) and the elementwise kernels it
// was followed by (LayerNorm inference_kernels.cu:229-348, the head's softmax
// and CDF in range_coder_kernels.cu:860-925 / :661-763).
//
// CTA tile 128 x BN, K-blocks of 64.  Warp roles (192 threads):
//   warp 0      TMA producer: A hi/lo tiles (128x64) + W hi/lo tiles (BNx64)
//   warp 1      TMEM allocator; lane 0 issues tcgen05.mma (3 per K=16 step:
//               Ah*Wh, Ah*Wl, Al*Wh -> ~fp32 accuracy from bf16 tensor cores)
//   warps 2..5  epilogue: one accumulator row per thread (TMEM lane quarter
//               = warp % 4), fused bias / activation / LayerNorm / residual /
//               LM-head coder.
// No split-K, a fixed K order and one instruction shape: a row's result does
// not depend on M or on where the row sits in the tile, so the compress
// (M = chunks x tokens) and decompress (M = chunks) paths produce bit-identical
// logits and therefore identical CDFs.
#include <cuda.h>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>
#include "gemm.cuh"

namespace boa {

constexpr int kBM = 128, kBK = 64;
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN >= 256 ? 2 : (BN >= 128 ? 3 : 4);
  static constexpr int kABytes = kBM * kBK * 2;  // one plane, 16 KB
  static constexpr int kBBytes = BN * kBK * 2;   // one plane
  static constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;
  static constexpr int kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// GELU (tanh form, activations.hpp:105-118) with tanh(u) = 1 - 2 / (1 + e^{2u})
// from the MUFU exponential: a few instructions instead of an accurate tanhf,
// ~1e-6 relative, deterministic.
__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == ACT_GELU) {
    const float k0 = 0.79788456080286535588f, k1 = 0.044715f;
    const float u = k0 * (v + k1 * v * v * v);
    const float th = 1.0f - __fdividef(2.0f, 1.0f + __expf(2.0f * u));
    return 0.5f * v * (1.0f + th);
  }
  if (act == ACT_RELU) return fmaxf(0.0f, v);
  if (act == ACT_SILU) return v / (1.0f + __expf(-v));
  return v;
}

__device__ __forceinline__ void store_split16(__nv_bfloat16* hi, __nv_bfloat16* lo, const float (&v)[16]) {
  __align__(16) __nv_bfloat16 h[16];
  __align__(16) __nv_bfloat16 l[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) split_bf16(v[j], h[j], l[j]);
  reinterpret_cast<uint4*>(hi)[0] = reinterpret_cast<uint4*>(h)[0];
  reinterpret_cast<uint4*>(hi)[1] = reinterpret_cast<uint4*>(h)[1];
  reinterpret_cast<uint4*>(lo)[0] = reinterpret_cast<uint4*>(l)[0];
  reinterpret_cast<uint4*>(lo)[1] = reinterpret_cast<uint4*>(l)[1];
}
__device__ __forceinline__ void store_f32x16(float* p, const float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 16; j += 4) reinterpret_cast<float4*>(p)[j / 4] = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}

// row source for the CDF code: one logits row staged in shared memory
struct SmemRow {
  float* p;
  static constexpr bool kCache = true;  // the row is this thread's own staging copy
  __device__ __forceinline__ void lane(int l, float (&v)[8]) const {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = p[l * 8 + i];
  }
  __device__ __forceinline__ void put(int l, const float (&e)[8]) const {
#pragma unroll
    for (int i = 0; i < 8; ++i) p[l * 8 + i] = e[i];
  }
};
constexpr int kRowStride = 257;  // floats; odd stride -> conflict-free per-thread rows

template <int BN, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* full = bars;                      // [kStages]
  uint64_t* empty = bars + Cfg::kStages;      // [kStages]
  uint64_t* acc_full = bars + 2 * Cfg::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * Cfg::kStages + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.y * BN;   // row tiles on x: up to 2^31 - 1 of them (y stops at 65535)
  const int m0 = blockIdx.x * kBM;
  const int nkb = (args.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % Cfg::kStages;
        if (kb >= Cfg::kStages) {
          if (!mbar_wait(&empty[s], ((kb / Cfg::kStages) - 1) & 1)) { *abort_flag = 1; break; }
        }
        if (*abort_flag) break;
        uint8_t* st = smem + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
        const int k0 = kb * kBK;
        tma_load_3d(st, &tmA, &full[s], k0, m0, 0);
        tma_load_3d(st + Cfg::kABytes, &tmA, &full[s], k0, m0, 1);
        tma_load_3d(st + 2 * Cfg::kABytes, &tmW, &full[s], k0, n0, 0);
        tma_load_3d(st + 2 * Cfg::kABytes + Cfg::kBBytes, &tmW, &full[s], k0, n0, 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % Cfg::kStages;
        if (!mbar_wait(&full[s], (kb / Cfg::kStages) & 1)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * Cfg::kStageBytes);
        const uint64_t dAh = umma_desc_sw128(st);
        const uint64_t dAl = umma_desc_sw128(st + Cfg::kABytes);
        const uint64_t dWh = umma_desc_sw128(st + 2 * Cfg::kABytes);
        const uint64_t dWl = umma_desc_sw128(st + 2 * Cfg::kABytes + Cfg::kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t adv = (uint64_t)(kk * 32 >> 4);  // 16 bf16 = 32 B along K
          umma_bf16(tmem, dAh + adv, dWh + adv, idesc, (kb | kk) != 0);
          umma_bf16(tmem, dAh + adv, dWl + adv, idesc, 1u);
          umma_bf16(tmem, dAl + adv, dWh + adv, idesc, 1u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r_local = q * 32 + lane;
    const int row = m0 + r_local;
    const bool ok = mbar_wait(acc_full, 0);
    tc_fence_after();
    if (ok && !*abort_flag) {
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
      const bool live = row < args.M;
      if constexpr (MODE == EPI_F32 || MODE == EPI_LOGITS) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(trow + c, v);
          if (args.bias) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += args.bias[n0 + c + j];
          }
          if (live) store_f32x16(args.out_f32 + (size_t)row * args.ld_f32 + n0 + c, v);
        }
      } else if constexpr (MODE == EPI_ACT_SPLIT) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(trow + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = apply_act(v[j] + args.bias[n0 + c + j], args.act);
          if (live) {
            __nv_bfloat16* hi = args.out_hl + (size_t)row * args.ld_hl + n0 + c;
            store_split16(hi, hi + args.plane_hl, v);
          }
        }
      } else if constexpr (MODE == EPI_LN_SPLIT || MODE == EPI_RES_LN) {
        // full row in this tile (BN == N); pass 1: values + moments
        float sum = 0.f, sq = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(trow + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float x = v[j] + args.bias[c + j];
            if constexpr (MODE == EPI_RES_LN) x = x + (live ? args.res[(size_t)row * BN + c + j] : 0.f);
            v[j] = x;
            sum += x;
            sq += x * x;
          }
          if constexpr (MODE == EPI_RES_LN) {
            if (live) store_f32x16(args.res + (size_t)row * BN + c, v);
          }
        }
        const bool norm = args.ln_w != nullptr;
        const float mean = sum / (float)BN;
        const float var = sq / (float)BN - mean * mean;
        const float inv_std = rsqrtf(var + 1e-5f);
        // pass 2: normalise (or plain split of x for the head) and store
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          if constexpr (MODE == EPI_RES_LN) {
            if (live) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                float4 t = reinterpret_cast<const float4*>(args.res + (size_t)row * BN + c)[j / 4];
                v[j] = t.x; v[j + 1] = t.y; v[j + 2] = t.z; v[j + 3] = t.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = 0.f;
            }
          } else {
            tmem_ld16(trow + c, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = v[j] + args.bias[c + j];
          }
          if (norm) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = (v[j] - mean) * inv_std * args.ln_w[c + j] + args.ln_b[c + j];
          }
          if (live) {
            __nv_bfloat16* hi = args.out_hl + (size_t)row * args.ld_hl + c;
            store_split16(hi, hi + args.plane_hl, v);
          }
        }
      } else if constexpr (MODE == EPI_HEAD_ENC || MODE == EPI_HEAD_DEC) {
        // stage the row (logits + bias) in the now idle pipeline smem
        float* srow = reinterpret_cast<float*>(smem) + (size_t)r_local * kRowStride;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(trow + c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) srow[c + j] = v[j] + args.bias[c + j];
        }
        __syncwarp();
        if (live) {
          SmemRow src{srow};
          if constexpr (MODE == EPI_HEAD_ENC) {
            const int b = row / args.T, tau = row - b * args.T;
            const long long base = (long long)b * (args.stride ? args.stride : args.chunk_len);
            const long long rem = args.n_bytes - base;
            const int len = (int)(rem < args.chunk_len ? rem : args.chunk_len);
            const int p = args.t0 + tau;
            uint2 lh = make_uint2(0u, 0u);
            if (p + 1 < len) {
              CdfRow R;
              cdf_prepare(src, args.inv_t, R);
              const int s = args.tokens[base + p + 1];
              cdf_symbol(src, R, s, lh.x, lh.y);
            }
            args.lf[row] = lh;
          } else {
            const int b = row;
            const int t = *args.d_t;
            const long long base = args.lane_base[b];
            const int len = args.lane_len[b];
            if (t < len) {
              DecState st = args.dstates[b];
              const uint32_t* in = args.payload + args.offsets[b];
              const uint32_t target = dec_target(st);
              CdfRow R;
              cdf_prepare(src, args.inv_t, R);
              uint32_t lo, hi;
              const int s = cdf_search(src, R, target, lo, hi);
              args.out_bytes[base + t] = (uint8_t)s;
              dec_update(st, lo, hi, in);
              args.dstates[b] = st;
            }
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// Per-warp 32-row x 16-column staging tile.  The epilogue thread owns one
// accumulator row; global traffic goes through the tile so that every warp
// access covers 8 rows x 64 contiguous bytes with 128-bit operations.  Row
// stride 20 floats keeps 16-byte alignment and conflict-free 128-bit stores.
constexpr int kTileStride = 20;
__device__ __forceinline__ void tile_put_row(float* wb, int lane, const float (&v)[16]) {
  float4* p = reinterpret_cast<float4*>(wb + lane * kTileStride);
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  __syncwarp();
}
__device__ __forceinline__ void tile_get_row(const float* wb, int lane, float (&v)[16]) {
  const float4* p = reinterpret_cast<const float4*>(wb + lane * kTileStride);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 t = p[j];
    v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
  }
  __syncwarp();
}
// lane -> (row r = it*8 + lane/4, columns 4*(lane%4) .. +3)
__device__ __forceinline__ void tile_store_f32(const float* wb, int lane, float* g, size_t ld, int nrows) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2), cc = (lane & 3) * 4;
    if (r < nrows)
      *reinterpret_cast<float4*>(g + (size_t)r * ld + cc) = *reinterpret_cast<const float4*>(wb + r * kTileStride + cc);
  }
  __syncwarp();
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo_col, float hi_col) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo_col, hi_col);  // .x = lo_col (lower address)
  return *reinterpret_cast<uint32_t*>(&t);
}
__device__ __forceinline__ float bf16_lo_half(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi_half(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ void tile_store_split(const float* wb, int lane, __nv_bfloat16* g, long long plane, size_t ld,
                                                 int nrows) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2), cc = (lane & 3) * 4;
    if (r < nrows) {
      const float4 v = *reinterpret_cast<const float4*>(wb + r * kTileStride + cc);
      // hi = bf16(v), lo = bf16(v - hi): the same values as split_bf16
      const uint32_t h01 = pack_bf16x2(v.x, v.y), h23 = pack_bf16x2(v.z, v.w);
      const uint32_t l01 = pack_bf16x2(v.x - bf16_lo_half(h01), v.y - bf16_hi_half(h01));
      const uint32_t l23 = pack_bf16x2(v.z - bf16_lo_half(h23), v.w - bf16_hi_half(h23));
      __nv_bfloat16* gp = g + (size_t)r * ld + cc;
      *reinterpret_cast<uint2*>(gp) = make_uint2(h01, h23);
      *reinterpret_cast<uint2*>(gp + plane) = make_uint2(l01, l23);
    }
  }
  __syncwarp();
}
__device__ __forceinline__ void tile_load_f32(float* wb, int lane, const float* g, size_t ld, int nrows) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2), cc = (lane & 3) * 4;
    *reinterpret_cast<float4*>(wb + r * kTileStride + cc) =
        r < nrows ? *reinterpret_cast<const float4*>(g + (size_t)r * ld + cc) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncwarp();
}
__device__ __forceinline__ void load_bias16(const float* b, float (&o)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 t = reinterpret_cast<const float4*>(b)[j];
    o[4 * j] = t.x; o[4 * j + 1] = t.y; o[4 * j + 2] = t.z; o[4 * j + 3] = t.w;
  }
}

// ------------------------------------------------------------------ persistent
// Persistent form for the row-parallel epilogues (F32, ACT_SPLIT, LN_SPLIT,
// RES_LN): one CTA per SM walks tiles t = blockIdx.x, +gridDim.x, ...; two
// TMEM accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
//   warp 0      TMA producer (continuous across tiles)
//   warp 1      TMEM allocator + MMA issuer
//   warps 2..17 epilogue; warp w reads TMEM lane quarter w % 4 and column
//               quarter (w - 2) / 4.  LayerNorm moments are combined across
//               the four column parts in a fixed order.
constexpr int kEpiWarps = 16;
constexpr int kMaxPersistN = 2048;  // widest N of a persistent GEMM (d_model 512: 4 * 512)
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kPThreads = 64 + kEpiThreads;

// K-block of 32 (64-byte rows, 64-byte swizzle) for wide tiles so four or more
// stages fit and cover TMA latency; 64 (128-byte swizzle) for narrow ones.
// PAIR: a cluster of two CTAs computes a 256-row tile with cta_group::2
// MMAs; each CTA stages its 128 rows of A and half of the tile's W rows.
template <int BN, bool PAIR = false>
struct PCfg {
  static constexpr int kBK = BN >= 128 ? 32 : 64;
  static constexpr int kSwz = kBK * 2;  // swizzle span in bytes (64 or 128)
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = (PAIR ? BN / 2 : BN) * kBK * 2;
  static constexpr int kTileRows = PAIR ? 2 * kBM : kBM;
  static constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;
  static constexpr int kEpiBuf = kEpiWarps * 32 * kTileStride * 4;  // staging tiles
  static constexpr int kRed = kBM * 4 * 2 * 4;
  // bias [N] and ln_w / ln_b [BN].  Narrow tiles (BN < 128) only serve N <= 512
  // (pick_bn: d_model 80's in_proj, N = 320, is the widest), so their staging
  // is small and the room goes to a fourth stage at BN = 48 (x_proj).
  static constexpr int kBiasN = BN < 128 ? 512 : kMaxPersistN;
  static constexpr int kLnN = BN < 128 ? 128 : 512;
  static constexpr int kPrm = (kBiasN + 2 * kLnN) * 4;
  static constexpr int kBudget = 225 * 1024 - 1024 - 256 - kRed - kEpiBuf - kPrm;
  static constexpr int kStages = kBudget / kStageBytes > 8 ? 8 : kBudget / kStageBytes;
  // N > 256 (LayerNorm over d = 512): 256-wide MMAs side by side in one
  // 512-column accumulator, which then cannot be double-buffered.
  static constexpr int kMmaN = BN > 256 ? 256 : BN;
  static constexpr int kNSub = BN / kMmaN;
  static constexpr int kBoxRows = PAIR ? kMmaN / 2 : kMmaN;  // W rows this CTA stages per MMA
  static constexpr int kAccCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : BN <= 256 ? 256 : 512;
  static constexpr int kNumAcc = 2 * kAccCols <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kNumAcc * kAccCols;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256 + kRed + kEpiBuf + kPrm;
  static_assert(kStages >= 2, "pipeline needs at least two stages");
};

template <int BN, int MODE, bool PAIR = false>
__global__ void __launch_bounds__(kPThreads, 1)
gemm_persist_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmO, GemmArgs args) {
  using Cfg = PCfg<BN, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [stages][epilogue staging (1 KB aligned)][barriers][LN partials][params]
  float* ebuf = reinterpret_cast<float*>(smem + Cfg::kStages * Cfg::kStageBytes);  // [kEpiWarps][32][kTileStride]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes + Cfg::kEpiBuf);
  uint64_t* full = bars;
  uint64_t* empty = bars + Cfg::kStages;
  uint64_t* acc_full = bars + 2 * Cfg::kStages;       // [2]
  uint64_t* acc_empty = bars + 2 * Cfg::kStages + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * Cfg::kStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + Cfg::kStages * Cfg::kStageBytes + Cfg::kEpiBuf + 256);  // [128][4][2]
  float* prm = red + kBM * 4 * 2;  // bias [N] | ln_w [BN] | ln_b [BN]
  float* prm_w = prm + Cfg::kBiasN;
  float* prm_b = prm_w + Cfg::kLnN;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles_n = args.N / BN;
  const int n_tiles = n_tiles_n * ((args.M + Cfg::kTileRows - 1) / Cfg::kTileRows);
  const int nkb = (args.K + Cfg::kBK - 1) / Cfg::kBK;
  // tile walk: one per CTA, or one per CTA pair (rank 0 issues the MMAs)
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int t_first = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int t_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int row_off = (int)rank * kBM;  // this CTA's rows within the tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&acc_full[a], 1); mbar_init(&acc_empty[a], (PAIR ? 2 : 1) * kEpiWarps); }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    if (MODE == EPI_F32) prefetch_tmap(&tmO);
  }
  if (warp == 1) {
    if constexpr (PAIR) { tmem_alloc_pair(tmem_slot, Cfg::kTmemCols); tmem_relinquish_pair(); }
    else { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // pair: the MMA issuer signals a barrier in both CTAs; everyone else signals rank 0's
  auto commit_both = [&](uint64_t* bar) {
    if constexpr (PAIR) { umma_commit_pair(cluster_addr(bar, 0)); umma_commit_pair(cluster_addr(bar, 1)); }
    else umma_commit(bar);
  };

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;  // global k-block counter (stage / phase)
      for (int t = t_first; t < n_tiles && !*abort_flag; t += t_step) {
        const int m0 = (t / n_tiles_n) * Cfg::kTileRows + row_off, n0 = (t % n_tiles_n) * BN;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % Cfg::kStages;
          if (g >= Cfg::kStages && !mbar_wait(&empty[s], ((g / Cfg::kStages) - 1) & 1)) { *abort_flag = 1; break; }
          uint8_t* st = smem + s * Cfg::kStageBytes;
          const int k0 = kb * Cfg::kBK;
          if constexpr (PAIR) {
            // both CTAs' bytes land on rank 0's barrier, which rank 0 arms for both
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);
            const uint32_t fb = cluster_addr(&full[s], 0);
            tma_load_3d_pair(st, &tmA, fb, k0, m0, 0);
            tma_load_3d_pair(st + Cfg::kABytes, &tmA, fb, k0, m0, 1);
#pragma unroll
            for (int sub = 0; sub < Cfg::kNSub; ++sub) {
              const int off = sub * Cfg::kBoxRows * Cfg::kBK * 2;
              const int wr = n0 + sub * Cfg::kMmaN + (int)rank * Cfg::kBoxRows;
              tma_load_3d_pair(st + 2 * Cfg::kABytes + off, &tmW, fb, k0, wr, 0);
              tma_load_3d_pair(st + 2 * Cfg::kABytes + Cfg::kBBytes + off, &tmW, fb, k0, wr, 1);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
            tma_load_3d(st, &tmA, &full[s], k0, m0, 0);
            tma_load_3d(st + Cfg::kABytes, &tmA, &full[s], k0, m0, 1);
#pragma unroll
            for (int sub = 0; sub < Cfg::kNSub; ++sub) {
              const int off = sub * Cfg::kBoxRows * Cfg::kBK * 2;
              tma_load_3d(st + 2 * Cfg::kABytes + off, &tmW, &full[s], k0, n0 + sub * Cfg::kBoxRows, 0);
              tma_load_3d(st + 2 * Cfg::kABytes + Cfg::kBBytes + off, &tmW, &full[s], k0, n0 + sub * Cfg::kBoxRows, 1);
            }
          }
        }
      }
      if constexpr (PAIR) {
        // the MMA issuer's last commits to this CTA's empty barriers land
        // before the CTA may exit
        for (int i = g > Cfg::kStages ? g - Cfg::kStages : 0; i < g; ++i)
          if (!mbar_wait(&empty[i % Cfg::kStages], (i / Cfg::kStages) & 1)) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(Cfg::kTileRows, Cfg::kMmaN);
      int g = 0, it = 0;
      for (int t = t_first; t < n_tiles; t += t_step, ++it) {
        const int a = it % Cfg::kNumAcc, use = it / Cfg::kNumAcc;
        const uint32_t acc = tmem + (uint32_t)(a * Cfg::kAccCols);
        if (it >= Cfg::kNumAcc && !mbar_wait(&acc_empty[a], (use - 1) & 1)) { *abort_flag = 1; }
        if (*abort_flag) { commit_both(&acc_full[a]); break; }
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % Cfg::kStages;
          if (!mbar_wait(&full[s], (g / Cfg::kStages) & 1)) { *abort_flag = 1; break; }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * Cfg::kStageBytes);
          const uint64_t dAh = umma_desc_swz<Cfg::kSwz>(st);
          const uint64_t dAl = umma_desc_swz<Cfg::kSwz>(st + Cfg::kABytes);
          const uint64_t dWh = umma_desc_swz<Cfg::kSwz>(st + 2 * Cfg::kABytes);
          const uint64_t dWl = umma_desc_swz<Cfg::kSwz>(st + 2 * Cfg::kABytes + Cfg::kBBytes);
#pragma unroll
          for (int kk = 0; kk < Cfg::kBK / 16; ++kk) {
            const uint64_t adv = (uint64_t)(kk * 32 >> 4);
#pragma unroll
            for (int sub = 0; sub < Cfg::kNSub; ++sub) {
              const uint64_t bo = (uint64_t)((sub * Cfg::kBoxRows * Cfg::kBK * 2) >> 4);
              const uint32_t d = acc + (uint32_t)(sub * Cfg::kMmaN);
              if constexpr (PAIR) {
                umma_bf16_pair(d, dAh + adv, dWh + bo + adv, idesc, (kb | kk) != 0);
                umma_bf16_pair(d, dAh + adv, dWl + bo + adv, idesc, 1u);
                umma_bf16_pair(d, dAl + adv, dWh + bo + adv, idesc, 1u);
              } else {
                umma_bf16(d, dAh + adv, dWh + bo + adv, idesc, (kb | kk) != 0);
                umma_bf16(d, dAh + adv, dWl + bo + adv, idesc, 1u);
                umma_bf16(d, dAl + adv, dWh + bo + adv, idesc, 1u);
              }
            }
          }
          commit_both(&empty[s]);
        }
        commit_both(&acc_full[a]);
        if (*abort_flag) break;
      }
      if constexpr (PAIR) {
        // both CTAs' epilogues have released the last accumulators
        for (int j = it > Cfg::kNumAcc ? it - Cfg::kNumAcc : 0; j < it; ++j)
          if (!mbar_wait(&acc_empty[j % Cfg::kNumAcc], (j / Cfg::kNumAcc) & 1)) break;
      }
    }
  } else {
    // the epilogue's per-column parameters, staged once per CTA: no chunk
    // of any tile waits on a global load for them
    {
      const int et = threadIdx.x - 64;
      for (int i = et; i < args.N; i += kEpiThreads) prm[i] = args.bias ? args.bias[i] : 0.f;
      if (args.ln_w)
        for (int i = et; i < BN; i += kEpiThreads) { prm_w[i] = args.ln_w[i]; prm_b[i] = args.ln_b[i]; }
      named_bar_sync(2, kEpiThreads);
    }
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;  // column quarter 0..3
    const int r_local = q * 32 + lane;
    // column range of this part in whole 16-column chunks
    constexpr int kChunks = BN / 16;
    int it = 0;
    for (int t = t_first; t < n_tiles; t += t_step, ++it) {
      const int a = it % Cfg::kNumAcc, use = it / Cfg::kNumAcc;
      const int m0 = (t / n_tiles_n) * Cfg::kTileRows + row_off, n0 = (t % n_tiles_n) * BN;
      const int c0 = (kChunks * part) / 4 * 16;
      const int c1 = (kChunks * (part + 1)) / 4 * 16;
      // RES_LN: this thread's residual row for the first kPre chunks, loaded
      // while the MMAs still run
      constexpr int kPre = MODE == EPI_RES_LN ? (kChunks / 4 < 2 ? kChunks / 4 : 2) : 0;
      float rpre[kPre > 0 ? kPre : 1][16];
      if constexpr (kPre > 0) {
        const int grow = m0 + r_local;
#pragma unroll
        for (int i = 0; i < kPre; ++i) {
          if (grow < args.M) {
            const float4* src = reinterpret_cast<const float4*>(args.res + (size_t)grow * BN + c0 + 16 * i);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 t4 = src[j];
              rpre[i][4 * j] = t4.x; rpre[i][4 * j + 1] = t4.y; rpre[i][4 * j + 2] = t4.z; rpre[i][4 * j + 3] = t4.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) rpre[i][j] = 0.f;
          }
        }
      }
      // only the barrier outcome decides (uniform across the epilogue warps,
      // which then meet at named barriers)
      const bool ok = mbar_wait(&acc_full[a], use & 1);
      tc_fence_after();
      if (!ok) break;
      const uint32_t trow = tmem + (uint32_t)(a * Cfg::kAccCols) + ((uint32_t)(q * 32) << 16);
      float* wb = ebuf + (warp - 2) * 32 * kTileStride;
      const int wrow0 = m0 + q * 32;
      const int nrows = max(0, min(32, args.M - wrow0));
      if constexpr (MODE == EPI_F32) {
        // Each 32 x 16 chunk leaves through a TMA tensor store: the warp
        // writes it into its staging tile in the 64-byte-swizzled layout of the
        // output map (16-byte unit j of row l at unit j ^ ((l >> 1) & 3), so the
        // 128-bit writes are conflict-free) and lane 0 issues the store.  Rows
        // past M are clipped by the tensor map.
        float4* wrow = reinterpret_cast<float4*>(wb) + lane * 4;
        const int sw = (lane >> 1) & 3;
#pragma unroll 1
        for (int c = c0; c < c1; c += 16) {
          float v[16];
          tmem_ld16(trow + c, v);
          if (args.bias) {
            float bb[16];
            load_bias16(prm + n0 + c, bb);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += bb[j];
          }
          if (lane == 0) bulk_wait_read_all();  // the previous store has read the tile
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j) wrow[j ^ sw] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && nrows > 0) {  // no box wholly past the last row
            tma_store_2d(&tmO, wb, n0 + c, wrow0);
            bulk_commit();
          }
        }
      } else if constexpr (MODE == EPI_ACT_SPLIT) {
#pragma unroll 1
        for (int c = c0; c < c1; c += 16) {
          float v[16];
          tmem_ld16(trow + c, v);
          float bb[16];
          load_bias16(prm + n0 + c, bb);
          if (args.act == ACT_GELU) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = apply_act(v[j] + bb[j], ACT_GELU);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = apply_act(v[j] + bb[j], args.act);
          }
          tile_put_row(wb, lane, v);
          tile_store_split(wb, lane, args.out_hl + (size_t)wrow0 * args.ld_hl + n0 + c, args.plane_hl, args.ld_hl,
                           nrows);
        }
      } else {  // EPI_LN_SPLIT / EPI_RES_LN: BN == N, full row in this tile
        float sum = 0.f, sq = 0.f;
        // pass 1 over one 16-column chunk; r = residual (RES_LN)
        auto pass1 = [&](int c, const float (&r)[16]) {
          float v[16];
          tmem_ld16(trow + c, v);
          float bb[16];
          load_bias16(prm + c, bb);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float x = v[j] + bb[j];
            if constexpr (MODE == EPI_RES_LN) x = x + r[j];
            v[j] = x;
            sum += x;
            sq += x * x;
          }
          if constexpr (MODE == EPI_RES_LN) {
            tile_put_row(wb, lane, v);
            tile_store_f32(wb, lane, args.res + (size_t)wrow0 * BN + c, BN, nrows);
            tmem_st16(trow + c, v);  // keep x in the (consumed) accumulator for pass 2
          }
        };
        int cstart = c0;
        if constexpr (kPre > 0) {
#pragma unroll
          for (int i = 0; i < kPre; ++i) pass1(c0 + 16 * i, rpre[i]);
          cstart = c0 + 16 * kPre;
        }
#pragma unroll 1
        for (int c = cstart; c < c1; c += 16) {
          float r[16];
          if constexpr (MODE == EPI_RES_LN) {
            tile_load_f32(wb, lane, args.res + (size_t)wrow0 * BN + c, BN, nrows);
            tile_get_row(wb, lane, r);
          }
          pass1(c, r);
        }
        if constexpr (MODE == EPI_RES_LN) tmem_st_wait();
        red[(r_local * 4 + part) * 2 + 0] = sum;
        red[(r_local * 4 + part) * 2 + 1] = sq;
        named_bar_sync(1, kEpiThreads);
        // fixed combination order: ((p0 + p1) + p2) + p3
        sum = ((red[(r_local * 4 + 0) * 2] + red[(r_local * 4 + 1) * 2]) + red[(r_local * 4 + 2) * 2]) +
              red[(r_local * 4 + 3) * 2];
        sq = ((red[(r_local * 4 + 0) * 2 + 1] + red[(r_local * 4 + 1) * 2 + 1]) + red[(r_local * 4 + 2) * 2 + 1]) +
             red[(r_local * 4 + 3) * 2 + 1];
        const bool norm = args.ln_w != nullptr;
        const float mean = sum / (float)BN;
        const float var = sq / (float)BN - mean * mean;
        const float inv_std = rsqrtf(var + 1e-5f);
#pragma unroll 1
        for (int c = c0; c < c1; c += 16) {
          float v[16];
          tmem_ld16(trow + c, v);
          if constexpr (MODE == EPI_RES_LN) {
            // v already holds x = acc + bias + residual (written back to TMEM in pass 1)
          } else {
            float bb[16];
            load_bias16(prm + c, bb);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = v[j] + bb[j];
          }
          if (norm) {
            float lw[16], lb[16];
            load_bias16(prm_w + c, lw);
            load_bias16(prm_b + c, lb);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = (v[j] - mean) * inv_std * lw[j] + lb[j];
          }
          tile_put_row(wb, lane, v);
          tile_store_split(wb, lane, args.out_hl + (size_t)wrow0 * args.ld_hl + c, args.plane_hl, args.ld_hl, nrows);
        }
        named_bar_sync(1, kEpiThreads);  // red[] reused by the next tile
      }
      // accumulator a may be overwritten once every epilogue warp has read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(cluster_addr(&acc_empty[a], 0));
        else mbar_arrive(&acc_empty[a]);
      }
    }
  }
  if (MODE == EPI_F32 && warp >= 2 && lane == 0) bulk_wait_all();  // staging tiles stay valid until read
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();  // neither CTA leaves while the other may still signal it
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, Cfg::kTmemCols);
    else tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D map over a [2][rows][K] bf16 plane pair, box = box_k (K) x box_rows x 1,
// swizzle span = box_k * 2 bytes (64 or 128).
static bool make_plane_map(CUtensorMap* map, const void* base, int K, int rows, long long plane, int box_rows,
                           int box_k) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, 2};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)plane * 2};
  cuuint32_t box[3] = {(cuuint32_t)box_k, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, box_k == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D map over an fp32 [rows][ld] output (the first `cols` columns), box 16 x 32,
// 64-byte swizzle: the F32 epilogue's tensor stores
static bool make_out_map_f32(CUtensorMap* map, void* base, int cols, int rows, int ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc || !base || ((uintptr_t)base & 15) || (ld * 4) % 16 || cols % 16) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {16, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int g_num_sms[64] = {0};

// CTA pairs (cta_group::2, 256-row tiles, each CTA staging half of W) for the
// F32 epilogue at compress-tile sizes: in_proj (N = 4d, K = d) runs 8 %
// faster at M = 262144 when each SM streams half the weight bytes.  Decode
// steps (M = one row per chunk) stay on single CTAs, where the pair's start-up
// costs more than it saves.  Both forms issue the same MMA sequence per row
// and give bit-identical outputs, so the choice may depend on M.
static constexpr bool pair_ok(int BN, int MODE) { return (BN == 128 || BN == 256) && MODE == EPI_F32; }
static bool use_pair(int mode, int M) { return mode == EPI_F32 && M >= 65536; }

template <int BN, int MODE>
static cudaError_t launch_pair_t(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to,
                                 const GemmArgs& a, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int tiles = (a.N / BN) * ((a.M + 2 * kBM - 1) / (2 * kBM));
  const int pairs = std::min(tiles, (g_num_sms[dev & 63] > 0 ? g_num_sms[dev & 63] : 148) / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = PCfg<BN, true>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_persist_kernel<BN, MODE, true>, ta, tw, to, a);
}

template <int BN, int MODE>
static cudaError_t launch_t(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const GemmArgs& a,
                            cudaStream_t st) {
  if constexpr (pair_ok(BN, MODE)) {
    if (use_pair(MODE, a.M)) return launch_pair_t<BN, MODE>(ta, tw, to, a, st);
  }
  if constexpr (MODE <= EPI_RES_LN) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int tiles = (a.N / BN) * ((a.M + kBM - 1) / kBM);
    const int grid = std::min(tiles, g_num_sms[dev & 63] > 0 ? g_num_sms[dev & 63] : 148);
    gemm_persist_kernel<BN, MODE><<<grid, kPThreads, PCfg<BN>::kSmem, st>>>(ta, tw, to, a);
  } else {
    using Cfg = GemmCfg<BN>;
    dim3 grid((a.M + kBM - 1) / kBM, a.N / BN);
    gemm_kernel<BN, MODE><<<grid, kThreads, Cfg::kSmem, st>>>(ta, tw, a);
  }
  return cudaGetLastError();
}

template <int BN, int MODE>
static cudaError_t set_attr_t() {
  if constexpr (pair_ok(BN, MODE)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_persist_kernel<BN, MODE, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<BN, true>::kSmem);
    if (e != cudaSuccess) return e;
  }
  if constexpr (MODE <= EPI_RES_LN)
    return cudaFuncSetAttribute(gemm_persist_kernel<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                PCfg<BN>::kSmem);
  else
    return cudaFuncSetAttribute(gemm_kernel<BN, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::kSmem);
}

template <int BN>
static cudaError_t dispatch(int mode, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to,
                            const GemmArgs& a, cudaStream_t st) {
  switch (mode) {
    case EPI_F32: return launch_t<BN, EPI_F32>(ta, tw, to, a, st);
    case EPI_ACT_SPLIT: return launch_t<BN, EPI_ACT_SPLIT>(ta, tw, to, a, st);
    case EPI_LN_SPLIT: return launch_t<BN, EPI_LN_SPLIT>(ta, tw, to, a, st);
    case EPI_RES_LN: return launch_t<BN, EPI_RES_LN>(ta, tw, to, a, st);
    case EPI_LOGITS: return BN == 256 ? launch_t<BN, EPI_LOGITS>(ta, tw, to, a, st) : cudaErrorInvalidValue;
    case EPI_HEAD_ENC: return BN == 256 ? launch_t<BN, EPI_HEAD_ENC>(ta, tw, to, a, st) : cudaErrorInvalidValue;
    case EPI_HEAD_DEC: return BN == 256 ? launch_t<BN, EPI_HEAD_DEC>(ta, tw, to, a, st) : cudaErrorInvalidValue;
  }
  return cudaErrorInvalidValue;
}

template <int BN>
static cudaError_t set_attrs() {
  cudaError_t e;
  if ((e = set_attr_t<BN, EPI_F32>()) != cudaSuccess) return e;
  if ((e = set_attr_t<BN, EPI_ACT_SPLIT>()) != cudaSuccess) return e;
  if ((e = set_attr_t<BN, EPI_LN_SPLIT>()) != cudaSuccess) return e;
  if ((e = set_attr_t<BN, EPI_RES_LN>()) != cudaSuccess) return e;
  if (BN == 256) {
    if ((e = set_attr_t<BN, EPI_LOGITS>()) != cudaSuccess) return e;
    if ((e = set_attr_t<BN, EPI_HEAD_ENC>()) != cudaSuccess) return e;
    if ((e = set_attr_t<BN, EPI_HEAD_DEC>()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Once per device (current device), before any launch or stream capture:
// opt the GEMM kernels into >48 KB dynamic shared memory and resolve the
// tensor-map encoder.
cudaError_t gemm_prepare_device() {
  if (!get_encode_fn()) return cudaErrorNotSupported;
  cudaError_t e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&g_num_sms[dev & 63], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if ((e = set_attrs<48>()) != cudaSuccess) return e;
  if ((e = set_attrs<64>()) != cudaSuccess) return e;
  if ((e = set_attrs<80>()) != cudaSuccess) return e;   // d_model 80: LayerNorm rows, head1
  if ((e = set_attrs<128>()) != cudaSuccess) return e;
  if ((e = set_attrs<160>()) != cudaSuccess) return e;  // d_model 160
  if ((e = set_attrs<256>()) != cudaSuccess) return e;
  if ((e = set_attr_t<512, EPI_LN_SPLIT>()) != cudaSuccess) return e;
  return set_attr_t<512, EPI_RES_LN>();
}

// CTA tile width: a full row for the row-wise epilogues (LayerNorm, coder),
// 256 for wide outputs, else the (padded) width itself.
static int pick_bn(int mode, int N) {
  if ((mode == EPI_LN_SPLIT || mode == EPI_RES_LN) && N == 512) return 512;
  if (mode == EPI_LN_SPLIT || mode == EPI_RES_LN || mode >= EPI_LOGITS) return N;
  if (N % 256 == 0) return 256;
  if (N % 128 == 0 && N > 128) return 128;  // 384 (GRU gates at d=128)
  if (N % 64 == 0 && N > 128) return 64;    // 192 (GRU gates at d=64)
  return N;
}

cudaError_t gemm_launch(int mode, const __nv_bfloat16* A, long long a_plane, int /*unused*/,
                        const __nv_bfloat16* W, long long w_plane, const GemmArgs& args, cudaStream_t stream) {
  if (args.K % 16 != 0 || args.K <= 0 || args.M <= 0) return cudaErrorInvalidValue;
  if (mode <= EPI_RES_LN && args.N > kMaxPersistN) return cudaErrorInvalidValue;  // bias staging size
  if (mode <= EPI_RES_LN && pick_bn(mode, args.N) < 128 && args.N > 512) return cudaErrorInvalidValue;
  const int BN = pick_bn(mode, args.N);
  if (BN != 48 && BN != 64 && BN != 80 && BN != 128 && BN != 160 && BN != 256 && BN != 512)
    return cudaErrorInvalidValue;
  if (mode >= EPI_LOGITS && BN != 256) return cudaErrorInvalidValue;
  // persistent row-parallel modes with BN >= 128 use K-blocks of 32
  const int box_k = (mode <= EPI_RES_LN && BN >= 128) ? 32 : kBK;
  CUtensorMap ta, tw, to;
  std::memset(&to, 0, sizeof(to));
  if (!make_plane_map(&ta, A, args.K, args.M, a_plane, kBM, box_k)) return cudaErrorInvalidValue;
  const bool pair = use_pair(mode, args.M) && (BN == 128 || BN == 256) && mode <= EPI_RES_LN;
  if (!make_plane_map(&tw, W, args.K, args.N, w_plane, pair ? BN / 2 : BN > 256 ? 256 : BN, box_k))
    return cudaErrorInvalidValue;
  if (mode == EPI_F32 && !make_out_map_f32(&to, args.out_f32, args.N, args.M, args.ld_f32)) return cudaErrorInvalidValue;
  switch (BN) {
    case 48: return dispatch<48>(mode, ta, tw, to, args, stream);
    case 64: return dispatch<64>(mode, ta, tw, to, args, stream);
    case 80: return dispatch<80>(mode, ta, tw, to, args, stream);
    case 128: return dispatch<128>(mode, ta, tw, to, args, stream);
    case 160: return dispatch<160>(mode, ta, tw, to, args, stream);
    case 512:
      if (mode == EPI_LN_SPLIT) return launch_t<512, EPI_LN_SPLIT>(ta, tw, to, args, stream);
      if (mode == EPI_RES_LN) return launch_t<512, EPI_RES_LN>(ta, tw, to, args, stream);
      return cudaErrorInvalidValue;
    default: return dispatch<256>(mode, ta, tw, to, args, stream);
  }
}

}  // namespace boa
