// mlp.cu -- the block's feed-forward as one tcgen05 kernel.
//
// Replaces FeedForwardGPU::forward_chunk / step_batch (boa_gpu.hpp:699-766:
// GEMM + bias + GELU, GEMM + bias + residual) and the LayerNorm that follows
// (the next block's LN1, inference_kernels.cu:293-348).  The unfused form
// writes the 4d-wide hidden activation to HBM (as bf16 hi/lo, 8d bytes per
// row) and reads it back; here it never leaves the SM:
//
//   for each 128-wide slice h of the hidden units:
//     acc1[h % 2] (TMEM, 128 cols)  = xn . W1[h]^T               (K = d)
//     hidden      (shared memory)   = split(GELU(acc1 + b1[h]))   (epilogue warps)
//     acc2        (TMEM, d cols)   += hidden . W2[:, h]^T          (K = 128)
//   x += acc2 + b2 ; xn = split(LN(x))                              (epilogue warps)
//
// The MMA warp issues ff1 of slice h+1 before ff2 of slice h, so the GELU of
// slice h overlaps tensor-core work; two ff1 accumulators make that legal.
// Each product is the same sequence of bf16x3 MMAs (hi*hi + hi*lo + lo*hi,
// K ascending) as the two separate GEMMs, and the hidden operand holds the
// same hi/lo values the unfused ff1 epilogue would store.  d <= 256 (TMEM:
// 2 x 128 + d columns).
//
// Warps: 0 TMA producer, 1 TMEM allocator + MMA issuer, 2..17 epilogue
// (TMEM lane quarter warp % 4, column quarter (warp - 2) / 4).
namespace boa {

constexpr int kMlpHC = 128;                    // hidden units per slice
// K-blocks of BK = 32 (64-byte rows, 64-byte swizzle, four 32 KB ring stages)
// or BK = 64 (128-byte rows, 128-byte swizzle, two 64 KB stages): the same
// 128 KB of operands in flight either way, and the same MMA sequence.
constexpr int kMlpRing = 128 * 1024;
constexpr int kMlpHid = 2 * kBM * kMlpHC * 2;  // hidden slice, hi + lo planes: 64 KB
constexpr int kMlpRed = kBM * 4 * 2 * 4;
constexpr int kMlpPrm = (1024 + 3 * 256) * 4;  // b1 [4d] | b2 [d] | ln_w [d] | ln_b [d]
constexpr int kMlpSmem = kMlpRing + kMlpHid + 1024 + 256 + kMlpRed + kMlpPrm;
static_assert(kEpiWarps * 32 * kTileStride * 4 <= kMlpHid, "final epilogue staging lives in the hidden buffer");

template <int D, int BK>
__global__ void __launch_bounds__(kPThreads, 1)
mlp_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW1,
           const __grid_constant__ CUtensorMap tmW2, const float* __restrict__ b1, GemmArgs args) {
  constexpr int NH = 4 * D / kMlpHC;    // hidden slices
  constexpr int kMlpBK = BK;
  constexpr int kMlpStages = BK == 32 ? 4 : 2;
  constexpr int kMlpStage = kMlpRing / kMlpStages;
  constexpr int kSwz = 2 * BK;                   // swizzle span = row bytes
  constexpr int kMlpHidBlock = kBM * BK * 2;     // one K-block of one hidden plane
  constexpr int K1B = D / kMlpBK;       // ff1 K-blocks per slice
  constexpr int K2B = kMlpHC / kMlpBK;  // ff2 K-blocks per slice
  constexpr int kABytes = kBM * kMlpBK * 2;      // A plane of one K-block
  constexpr int kW1Bytes = kMlpHC * kMlpBK * 2;  // W1 plane
  constexpr int kW2Bytes = D * kMlpBK * 2;       // W2 plane
  static_assert(NH % 2 == 0 && D % 64 == 0 && D <= 256, "d_model 64, 128 or 256");
  static_assert(2 * kABytes + 2 * kW1Bytes <= kMlpStage && 2 * kW2Bytes <= kMlpStage, "stage size");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* hid = smem + kMlpRing;  // [plane][K-block][128 rows][2 BK bytes], swizzled like the ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(hid + kMlpHid);
  uint64_t* full = bars;                         // [kMlpStages]
  uint64_t* empty = bars + kMlpStages;           // [kMlpStages]
  uint64_t* acc1_full = bars + 2 * kMlpStages;   // [2]
  uint64_t* acc1_empty = acc1_full + 2;          // [2]
  uint64_t* hid_full = acc1_empty + 2;
  uint64_t* hid_empty = hid_full + 1;
  uint64_t* acc2_full = hid_empty + 1;
  uint64_t* acc2_empty = acc2_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc2_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(hid + kMlpHid + 256);  // [128][4 parts][2]
  float* prm_b1 = red + kBM * 4 * 2;
  float* prm_b2 = prm_b1 + 4 * D;
  float* prm_w = prm_b2 + D;
  float* prm_b = prm_w + D;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (args.M + kBM - 1) / kBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMlpStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&acc1_full[b], 1); mbar_init(&acc1_empty[b], kEpiWarps); }
    mbar_init(hid_full, kEpiWarps);
    mbar_init(hid_empty, 1);
    mbar_init(acc2_full, 1);
    mbar_init(acc2_empty, kEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW1);
    prefetch_tmap(&tmW2);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // acc1[0]: cols 0..127, acc1[1]: 128..255, acc2: 256..256+D

  // The per-tile op order, shared by producer and MMA issuer:
  //   ff1(0), then for h = 1..NH-1: ff1(h), ff2(h-1); then ff2(NH-1).
  // op o -> (is_ff2, slice)
  auto op_of = [](int o, bool& ff2, int& h) {
    if (o == 0) { ff2 = false; h = 0; return; }
    if (o == 2 * NH - 1) { ff2 = true; h = NH - 1; return; }
    ff2 = (o % 2) == 0;
    h = ff2 ? o / 2 - 1 : (o + 1) / 2;
  };

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
        const int m0 = t * kBM;
        for (int o = 0; o < 2 * NH && !*abort_flag; ++o) {
          bool ff2; int h;
          op_of(o, ff2, h);
          const int nkb = ff2 ? K2B : K1B;
          for (int kb = 0; kb < nkb; ++kb, ++g) {
            const int s = g % kMlpStages;
            if (g >= kMlpStages && !mbar_wait(&empty[s], ((g / kMlpStages) - 1) & 1)) { *abort_flag = 1; break; }
            uint8_t* st = smem + s * kMlpStage;
            if (!ff2) {
              mbar_arrive_expect_tx(&full[s], 2 * kABytes + 2 * kW1Bytes);
              const int k0 = kb * kMlpBK;
              tma_load_3d(st, &tmA, &full[s], k0, m0, 0);
              tma_load_3d(st + kABytes, &tmA, &full[s], k0, m0, 1);
              tma_load_3d(st + 2 * kABytes, &tmW1, &full[s], k0, h * kMlpHC, 0);
              tma_load_3d(st + 2 * kABytes + kW1Bytes, &tmW1, &full[s], k0, h * kMlpHC, 1);
            } else {
              mbar_arrive_expect_tx(&full[s], 2 * kW2Bytes);
              const int k0 = h * kMlpHC + kb * kMlpBK;
              tma_load_3d(st, &tmW2, &full[s], k0, 0, 0);
              tma_load_3d(st + kW2Bytes, &tmW2, &full[s], k0, 0, 1);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc1 = umma_idesc_bf16(kBM, kMlpHC);
      constexpr uint32_t idesc2 = umma_idesc_bf16(kBM, D);
      const uint32_t acc2 = tmem + 256;
      int g = 0, it = 0;
      for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
        for (int o = 0; o < 2 * NH; ++o) {
          bool ff2; int h;
          op_of(o, ff2, h);
          const int gh = it * NH + h;  // global slice counter
          if (!ff2) {
            const int b = h & 1, use = gh >> 1;  // NH even: slice parity = buffer
            if (use >= 1 && !mbar_wait(&acc1_empty[b], (use - 1) & 1)) *abort_flag = 1;
          } else {
            if (!mbar_wait(hid_full, gh & 1)) *abort_flag = 1;
            if (h == 0 && it >= 1 && !mbar_wait(acc2_empty, (it - 1) & 1)) *abort_flag = 1;
          }
          if (*abort_flag) break;
          tc_fence_after();
          const int nkb = ff2 ? K2B : K1B;
          for (int kb = 0; kb < nkb; ++kb, ++g) {
            const int s = g % kMlpStages;
            if (!mbar_wait(&full[s], (g / kMlpStages) & 1)) { *abort_flag = 1; break; }
            tc_fence_after();
            const uint32_t st = smem_u32(smem + s * kMlpStage);
            if (!ff2) {
              const uint64_t dAh = umma_desc_swz<kSwz>(st), dAl = umma_desc_swz<kSwz>(st + kABytes);
              const uint64_t dWh = umma_desc_swz<kSwz>(st + 2 * kABytes);
              const uint64_t dWl = umma_desc_swz<kSwz>(st + 2 * kABytes + kW1Bytes);
              const uint32_t d = tmem + (uint32_t)((h & 1) * kMlpHC);
#pragma unroll
              for (int kk = 0; kk < kMlpBK / 16; ++kk) {
                const uint64_t adv = (uint64_t)(kk * 2);  // 32 bytes
                umma_bf16(d, dAh + adv, dWh + adv, idesc1, (kb | kk) != 0);
                umma_bf16(d, dAh + adv, dWl + adv, idesc1, 1u);
                umma_bf16(d, dAl + adv, dWh + adv, idesc1, 1u);
              }
            } else {
              const uint32_t hh = smem_u32(hid + kb * kMlpHidBlock);
              const uint32_t hl = smem_u32(hid + kMlpHid / 2 + kb * kMlpHidBlock);
              const uint64_t dHh = umma_desc_swz<kSwz>(hh), dHl = umma_desc_swz<kSwz>(hl);
              const uint64_t dWh = umma_desc_swz<kSwz>(st), dWl = umma_desc_swz<kSwz>(st + kW2Bytes);
#pragma unroll
              for (int kk = 0; kk < kMlpBK / 16; ++kk) {
                const uint64_t adv = (uint64_t)(kk * 2);
                umma_bf16(acc2, dHh + adv, dWh + adv, idesc2, (h | kb | kk) != 0);
                umma_bf16(acc2, dHh + adv, dWl + adv, idesc2, 1u);
                umma_bf16(acc2, dHl + adv, dWh + adv, idesc2, 1u);
              }
            }
            umma_commit(&empty[s]);
          }
          if (*abort_flag) break;
          if (!ff2) umma_commit(&acc1_full[h & 1]);
          else if (h < NH - 1) umma_commit(hid_empty);
          else umma_commit(acc2_full);
        }
        if (*abort_flag) {
          // release every epilogue wait of this tile so that no warp spins to its limit
          umma_commit(&acc1_full[0]); umma_commit(&acc1_full[1]); umma_commit(acc2_full);
          break;
        }
      }
    }
  } else {
    {
      const int et = threadIdx.x - 64;
      for (int i = et; i < 4 * D; i += kEpiThreads) prm_b1[i] = b1[i];
      for (int i = et; i < D; i += kEpiThreads) {
        prm_b2[i] = args.bias[i];
        prm_w[i] = args.ln_w ? args.ln_w[i] : 0.f;
        prm_b[i] = args.ln_b ? args.ln_b[i] : 0.f;
      }
      named_bar_sync(2, kEpiThreads);
    }
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    const int r_local = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    // 16-byte unit permutation of this row: 64-byte swizzle (4 units per row,
    // pattern repeats every 8 rows) or 128-byte swizzle (8 units per row)
    const int sw = BK == 32 ? (r_local >> 1) & 3 : r_local & 7;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++it) {
      const int m0 = t * kBM;
      const int wrow0 = m0 + q * 32;
      const int nrows = max(0, min(32, args.M - wrow0));
      // ---- hidden slices: GELU(acc1 + b1) -> bf16 hi/lo operand in shared memory
      for (int h = 0; h < NH && ok; ++h) {
        const int gh = it * NH + h, b = h & 1;
        ok = mbar_wait(&acc1_full[b], (gh >> 1) & 1);
        if (ok && h >= 1) ok = mbar_wait(hid_empty, (it * (NH - 1) + h - 1) & 1);
        tc_fence_after();
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int c = part * 32 + 16 * j;  // hidden column within the slice
          float v[16];
          tmem_ld16(tmem + (uint32_t)(b * kMlpHC + c) + lane_off, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = apply_act(v[i] + prm_b1[h * kMlpHC + c + i], ACT_GELU);
          uint32_t hw[8], lw[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            hw[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
            lw[i] = pack_bf16x2(v[2 * i] - bf16_lo_half(hw[i]), v[2 * i + 1] - bf16_hi_half(hw[i]));
          }
          const int kb = c / kMlpBK, u0 = (c % kMlpBK) / 8;  // K-block, first 16-byte unit
          uint8_t* rh = hid + kb * kMlpHidBlock + r_local * (2 * BK);
          uint8_t* rl = rh + kMlpHid / 2;
#pragma unroll
          for (int uu = 0; uu < 2; ++uu) {
            const int unit = (u0 + uu) ^ sw;
            *reinterpret_cast<uint4*>(rh + unit * 16) = make_uint4(hw[4 * uu], hw[4 * uu + 1], hw[4 * uu + 2], hw[4 * uu + 3]);
            *reinterpret_cast<uint4*>(rl + unit * 16) = make_uint4(lw[4 * uu], lw[4 * uu + 1], lw[4 * uu + 2], lw[4 * uu + 3]);
          }
        }
        fence_proxy_async_smem();  // the MMA reads the hidden buffer through the async proxy
        tc_fence_before();
        __syncwarp();
        if (lane == 0) { mbar_arrive(hid_full); mbar_arrive(&acc1_empty[b]); }
      }
      if (!ok) break;
      // ---- x += acc2 + b2 ; xn = split(LN(x)) (as the RES_LN GEMM epilogue)
      constexpr int kChunks = D / 16;
      const int c0 = (kChunks * part) / 4 * 16;
      const int c1 = (kChunks * (part + 1)) / 4 * 16;
      ok = mbar_wait(acc2_full, it & 1);
      tc_fence_after();
      if (!ok) break;
      const uint32_t trow = tmem + 256 + lane_off;
      float* wb = reinterpret_cast<float*>(hid) + (warp - 2) * 32 * kTileStride;  // hidden buffer is free now
      float sum = 0.f, sq = 0.f;
#pragma unroll 1
      for (int c = c0; c < c1; c += 16) {
        float r[16];
        tile_load_f32(wb, lane, args.res + (size_t)wrow0 * D + c, D, nrows);
        tile_get_row(wb, lane, r);
        float v[16];
        tmem_ld16(trow + c, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float x = (v[j] + prm_b2[c + j]) + r[j];
          v[j] = x;
          sum += x;
          sq += x * x;
        }
        tile_put_row(wb, lane, v);
        tile_store_f32(wb, lane, args.res + (size_t)wrow0 * D + c, D, nrows);
        tmem_st16(trow + c, v);
      }
      tmem_st_wait();
      red[(r_local * 4 + part) * 2 + 0] = sum;
      red[(r_local * 4 + part) * 2 + 1] = sq;
      named_bar_sync(1, kEpiThreads);
      sum = ((red[(r_local * 4 + 0) * 2] + red[(r_local * 4 + 1) * 2]) + red[(r_local * 4 + 2) * 2]) +
            red[(r_local * 4 + 3) * 2];
      sq = ((red[(r_local * 4 + 0) * 2 + 1] + red[(r_local * 4 + 1) * 2 + 1]) + red[(r_local * 4 + 2) * 2 + 1]) +
           red[(r_local * 4 + 3) * 2 + 1];
      const bool norm = args.ln_w != nullptr;
      const float mean = sum / (float)D;
      const float var = sq / (float)D - mean * mean;
      const float inv_std = rsqrtf(var + 1e-5f);
#pragma unroll 1
      for (int c = c0; c < c1; c += 16) {
        float v[16];
        tmem_ld16(trow + c, v);
        if (norm) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = (v[j] - mean) * inv_std * prm_w[c + j] + prm_b[c + j];
        }
        tile_put_row(wb, lane, v);
        tile_store_split(wb, lane, args.out_hl + (size_t)wrow0 * args.ld_hl + c, args.plane_hl, args.ld_hl, nrows);
      }
      tc_fence_before();
      named_bar_sync(1, kEpiThreads);  // red[] and the hidden buffer are reused by the next tile
      if (lane == 0) mbar_arrive(acc2_empty);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, int BK>
static cudaError_t mlp_launch_t(const CUtensorMap& ta, const CUtensorMap& t1, const CUtensorMap& t2, const float* b1,
                                const GemmArgs& a, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int tiles = (a.M + kBM - 1) / kBM;
  const int grid = std::min(tiles, g_num_sms[dev & 63] > 0 ? g_num_sms[dev & 63] : 148);
  mlp_kernel<D, BK><<<grid, kPThreads, kMlpSmem, st>>>(ta, t1, t2, b1, a);
  return cudaGetLastError();
}

// K-block width of the fused feed-forward: 64 (two 64 KB stages, 128-byte
// rows).  Against 32 (four 32 KB stages, 64-byte rows) at d_model 256 with
// 16384 chunks, alternating runs: 77.2 against 83.5 us per decode launch and
// 3.71 against 3.86 ms per 64-position compress tile, bit-identical.
constexpr int kMlpBKUsed = 64;

cudaError_t mlp_prepare_device() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(mlp_kernel<64, kMlpBKUsed>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kMlpSmem)) != cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(mlp_kernel<128, kMlpBKUsed>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kMlpSmem)) != cudaSuccess)
    return e;
  return cudaFuncSetAttribute(mlp_kernel<256, kMlpBKUsed>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMlpSmem);
}

cudaError_t mlp_launch(const __nv_bfloat16* xn, long long xn_plane, const __nv_bfloat16* w1, long long w1_plane,
                       const __nv_bfloat16* w2, long long w2_plane, const float* b1, const GemmArgs& a,
                       cudaStream_t stream) {
  const int D = a.N;
  if (a.M <= 0 || !a.res || !a.out_hl || !a.bias || !b1 || (D != 64 && D != 128 && D != 256))
    return cudaErrorInvalidValue;
  CUtensorMap ta, t1, t2;
  if (!make_plane_map(&ta, xn, D, a.M, xn_plane, kBM, kMlpBKUsed)) return cudaErrorInvalidValue;
  if (!make_plane_map(&t1, w1, D, 4 * D, w1_plane, kMlpHC, kMlpBKUsed)) return cudaErrorInvalidValue;
  if (!make_plane_map(&t2, w2, 4 * D, D, w2_plane, D, kMlpBKUsed)) return cudaErrorInvalidValue;
  switch (D) {
    case 64: return mlp_launch_t<64, kMlpBKUsed>(ta, t1, t2, b1, a, stream);
    case 128: return mlp_launch_t<128, kMlpBKUsed>(ta, t1, t2, b1, a, stream);
    default: return mlp_launch_t<256, kMlpBKUsed>(ta, t1, t2, b1, a, stream);
  }
}

}  // namespace boa
