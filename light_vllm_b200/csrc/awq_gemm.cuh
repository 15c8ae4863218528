// AutoAWQ W4A16 linear on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// y[m, n] = sum_k x[m, k] * W[k, n] (+ bias[n]),  W[k, n] = fp16(q - z) * s.
//
// The weight is the UMMA "A" operand (M = 128 output columns per CTA) and the
// activations are "B" (N = BN tokens), so a decode step with a handful of
// tokens still fills the 128-row tensor-core tile ("swap-AB").  Per CTA:
//
//   warp 0        TMEM allocator and the single thread issuing tcgen05.mma
//   warps 1..8    loaders + dequantisers: a cp.async multistage pipeline of
//                 raw stages (int4 tile 64 k x 128 n = 4 KB, the BN x 64
//                 activation tile written in the SWIZZLE_128B K-major operand
//                 layout, fp16 scales and packed zeros of the at most two
//                 groups the tile spans), then int4 -> fp16 W written straight
//                 into the MN-major SWIZZLE_128B A layout; afterwards the
//                 epilogue (TMEM -> registers -> fp16 y).
//
// Every thread issues its own 16-byte cp.async copies, so the load rate is not
// bound by the per-instruction issue cost of bulk tensor copies, which on this
// part limits one issuing warp to roughly one copy per 200 ns.
//
// The dequantisation reproduces the reference's fp16 arithmetic exactly
// (modeling/quantization/awq.py:433-450): a nibble v becomes the fp16 value
// 1024 + v by OR-ing it under the exponent of 1024 (0x6400), the difference of
// two such values is the exact integer q - z, and one fp16 multiply by the
// scale gives the same rounding as the reference's dequantised weight.  With
// the AutoAWQ nibble order (0,2,4,6,1,3,5,7), masks 0x000F000F / 0x00F000F0 of
// the word and of the word shifted by 8 yield the column pairs (0,1), (2,3),
// (4,5), (6,7) as half2 values 1024 + q or 1024 + 16 q; the second form
// produces 16 W (exact scaling; bit-identical for |scale| < 273), which the
// fp32 epilogue multiplies by 1/16.
//
// Small grids split K across CTAs; the partial fp32 tiles go to a workspace
// and the last CTA of a tile (found with a per-tile semaphore) sums them in
// split order, so results are deterministic.
#pragma once

#include "lvb_common.cuh"

namespace lvb {
namespace awq {

constexpr int kTileN = 128;                         // output columns per CTA (UMMA M)
constexpr int kTileK = 64;                          // k per pipeline stage
constexpr int kWordsPerRow = kTileN / 8;            // packed words per k row of a tile
constexpr int kQBytes = kTileK * kWordsPerRow * 4;  // 4096: int4 codes of one stage
constexpr int kScaleBytes = 2 * kTileN * 2;         // 512: fp16 scales of two group rows
constexpr int kZeroBytes = 2 * kWordsPerRow * 4;    // 128: packed zeros of two group rows
constexpr int kABytes = kTileN * kTileK * 2;        // 16384: one dequantised A tile
constexpr int kALbo = 1024;  // byte stride between the two 64-column MN atoms of A
constexpr int kASbo = 2048;  // byte stride between 8-row k groups of A
constexpr int kDequantWarps = 8;
constexpr int kDequantThreads = kDequantWarps * 32;
constexpr int kFirstDequantWarp = 1;
constexpr int kThreads = (kFirstDequantWarp + kDequantWarps) * 32;  // 288

template <int BN>
struct Config {
  static constexpr int kXBytes = BN * kTileK * 2;
  // One raw stage: activation tile (SWIZZLE_128B K-major, first so that it is
  // 1024-byte aligned), int4 codes, scales and zeros of two group rows.
  static constexpr int kQOff = kXBytes;
  static constexpr int kSOff = kQOff + kQBytes;
  static constexpr int kZOff = kSOff + kScaleBytes;
  static constexpr int kStageBytes = ((kZOff + kZeroBytes) + 1023) / 1024 * 1024;
  static constexpr int kOpStages = BN >= 256 ? 2 : BN >= 128 ? 3 : 4;  // dequantised A tiles
  static constexpr int kRawStages = BN >= 256 ? 4 : BN >= 128 ? 6 : BN >= 64 ? 10 : 16;
  // Loads for stage i + kAhead are issued while stage i is dequantised; a raw
  // slot is refilled only after the MMA that read its activation tile is done.
  static constexpr int kAhead = kRawStages - kOpStages;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kAOff = 0;
  static constexpr int kRawOff = kOpStages * kABytes;
  static constexpr int kBarOff = kRawOff + kRawStages * kStageBytes;
  // ready (one per raw slot), a_full, op_empty (one per A slot), acc_full.
  static constexpr int kNumBars = kRawStages + 2 * kOpStages + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 64 + 1024;  // + base alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct Params {
  const uint16_t *x;
  const int32_t *qweight;
  const int32_t *qzeros;
  const uint16_t *scales;
  const uint16_t *bias;  // may be null
  uint16_t *y;
  uint32_t *semaphores;  // per output tile, zero between calls
  float *partials;       // [tiles][splits][BN][128] when splits > 1
  int M, K, N, G;
  int k_tiles;  // ceil(K / 64)
  int splits;
  int n_tiles;
};

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Issue the cp.async copies of one raw stage (k tile `kt`) into `stage` for
// dequantiser thread t (0..255).  Out-of-range rows and columns are zero-filled.
template <int BN>
__device__ __forceinline__ void load_stage(const Params &p, uint32_t stage, int kt, int n0, int m0, int t) {
  using C = Config<BN>;
  const int kb = kt * kTileK;
  const int words = p.N >> 3;
  // int4 codes: 64 rows x 64 bytes, one 16-byte chunk per thread.
  {
    const int r = t >> 2;
    const int w = (t & 3) * 4;
    const bool ok = kb + r < p.K && (n0 >> 3) + w < words;
    const int32_t *src = p.qweight + static_cast<size_t>(ok ? kb + r : 0) * words + (ok ? (n0 >> 3) + w : 0);
    cp_async_16(stage + C::kQOff + r * 64 + w * 4, src, ok ? 16u : 0u);
  }
  // Activation tile: BN rows x 8 chunks of 16 bytes, 128-byte swizzle.
#pragma unroll
  for (int c = t; c < BN * 8; c += kDequantThreads) {
    const int m = c >> 3;
    const int cc = c & 7;
    const bool ok = m0 + m < p.M && kb + cc * 8 < p.K;
    const uint16_t *src = p.x + static_cast<size_t>(ok ? m0 + m : 0) * p.K + (ok ? kb + cc * 8 : 0);
    cp_async_16(stage + m * 128 + ((cc ^ (m & 7)) << 4), src, ok ? 16u : 0u);
  }
  // Scales (2 rows x 16 chunks) and packed zeros (2 rows x 4 chunks) of the
  // group rows g0 and g0 + 1 (a 64-row tile spans at most two groups).
  if (t < 40) {
    const int g0 = kb / p.G;
    const int groups = p.K / p.G;
    if (t < 32) {
      const int gi = t >> 4;
      const int col = (t & 15) * 8;
      const bool ok = g0 + gi < groups && n0 + col < p.N;
      const uint16_t *src = p.scales + static_cast<size_t>(ok ? g0 + gi : 0) * p.N + (ok ? n0 + col : 0);
      cp_async_16(stage + C::kSOff + gi * 256 + (t & 15) * 16, src, ok ? 16u : 0u);
    } else {
      const int c = t - 32;
      const int gi = c >> 2;
      const int w = (c & 3) * 4;
      const bool ok = g0 + gi < groups && (n0 >> 3) + w < words;
      const int32_t *src = p.qzeros + static_cast<size_t>(ok ? g0 + gi : 0) * words + (ok ? (n0 >> 3) + w : 0);
      cp_async_16(stage + C::kZOff + gi * 64 + w * 4, src, ok ? 16u : 0u);
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) awq_gemm_kernel(const Params p) {
  pdl_entry();
  using C = Config<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *a_ring = smem + C::kAOff;
  uint8_t *raw_ring = smem + C::kRawOff;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *ready = bars;  // raw slot landed: all loader threads' cp.async done
  uint64_t *a_full = ready + C::kRawStages;
  uint64_t *op_empty = a_full + C::kOpStages;
  uint64_t *acc_full = op_empty + C::kOpStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 8);
  volatile int *last_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x;
  const int m_tile = blockIdx.y;
  const int split = blockIdx.z;
  const int n0 = n_tile * kTileN;
  const int m0 = m_tile * BN;
  const int kt_begin = static_cast<int>((static_cast<long long>(split) * p.k_tiles) / p.splits);
  const int kt_end = static_cast<int>((static_cast<long long>(split + 1) * p.k_tiles) / p.splits);
  const int nk = kt_end - kt_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kRawStages; ++s) mbar_init(&ready[s], kDequantThreads);
    for (int s = 0; s < C::kOpStages; ++s) {
      mbar_init(&a_full[s], kDequantWarps);
      mbar_init(&op_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    // ---------------- tcgen05.mma issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(kTileN, BN, 0, 0, /*a MN-major*/ 1, 0);
      const uint32_t a_base = smem_u32(a_ring);
      const uint32_t raw_base = smem_u32(raw_ring);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % C::kOpStages;
        const uint32_t ph = (i / C::kOpStages) & 1;
        ok = mbar_wait(&a_full[s], ph, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t x_tile = raw_base + (i % C::kRawStages) * C::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < kTileK / 16; ++kk) {
          const uint64_t adesc =
              umma_smem_desc_sw128(a_base + s * kABytes + kk * 2 * kASbo, kALbo, kASbo);
          const uint64_t bdesc = umma_smem_desc_sw128(x_tile + kk * 32, 16, 1024);
          umma_f16(tmem_d, adesc, bdesc, idesc, (i | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&op_empty[s]);
      }
      umma_commit(acc_full);
      if (!ok) mbar_wait(acc_full, 0, nullptr, kDrainBudgetCycles);
    }
    __syncwarp();
  } else {
    // ---------------- loaders + dequantisers ----------------
    const int t = threadIdx.x - kFirstDequantWarp * 32;
    const int j = t & 15;   // packed word (8 columns) within the tile row
    const int r0 = t >> 4;  // first of the rows r0 + 16 * ii
    const int n_col = n0 + 8 * j;
    const bool col_ok = n_col < p.N;
    const uint32_t raw_base = smem_u32(raw_ring);
    // Byte offsets of this thread's four 16-byte stores in an A tile (rows
    // r0 + 16 * ii, columns 8j..8j+7): MN-major SWIZZLE_128B, 8-row k groups at
    // kASbo, the two 64-column atoms at kALbo, chunk index XOR row-in-group.
    uint32_t a_off[4];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const int r = r0 + 16 * ii;
      const int kr = r & 7;
      a_off[ii] = (r >> 3) * kASbo + (j >> 3) * kALbo + kr * 128 + (((j & 7) ^ kr) << 4);
    }
    // A 64-row tile lies in one group when the group size is a multiple of 64;
    // otherwise (group 32, 96, ...) it can straddle two.
    const bool single_group = (p.G & 63) == 0;
#pragma unroll 1
    for (int i = 0; i < C::kAhead && i < nk; ++i) {
      load_stage<BN>(p, raw_base + (i % C::kRawStages) * C::kStageBytes, kt_begin + i, n0, m0, t);
      cp_async_arrive_noinc(&ready[i % C::kRawStages]);
    }
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int os = i % C::kOpStages;
      const uint32_t oph = (i / C::kOpStages) & 1;
      // A slot free: the MMA of stage i - kOpStages is done, so the raw slot it
      // read (the one stage i + kAhead reuses) is free as well.
      if (!__all_sync(0xffffffffu, mbar_wait(&op_empty[os], oph ^ 1, abort_flag))) { ok = false; break; }
      if (i + C::kAhead < nk) {
        const int sl = (i + C::kAhead) % C::kRawStages;
        load_stage<BN>(p, raw_base + sl * C::kStageBytes, kt_begin + i + C::kAhead, n0, m0, t);
        cp_async_arrive_noinc(&ready[sl]);
      }
      const int rs = i % C::kRawStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&ready[rs], (i / C::kRawStages) & 1, abort_flag))) {
        ok = false;
        break;
      }
      const uint8_t *stage = raw_ring + rs * C::kStageBytes;
      const uint32_t *raw = reinterpret_cast<const uint32_t *>(stage + C::kQOff);
      const uint4 *srow = reinterpret_cast<const uint4 *>(stage + C::kSOff);
      const uint32_t *zrow = reinterpret_cast<const uint32_t *>(stage + C::kZOff);
      uint32_t w[4];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) w[ii] = raw[(r0 + 16 * ii) * kWordsPerRow + j];
      const int k_base = (kt_begin + i) * kTileK;
      // Rows at or beyond `split_row` use the second group row of the stage.
      const int split_row = single_group ? kTileK : (k_base / p.G + 1) * p.G - k_base;
      // Per group row: fp16 scale pairs and the zero points in the two biased
      // forms used below (1024 + z for the low nibble of a byte, 1024 + 16 z
      // for the high nibble).
      uint32_t sc[2][4], zlo[2][2], zhi[2][2];
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const uint4 s4 = srow[gi * (kTileN / 8) + j];
        sc[gi][0] = s4.x; sc[gi][1] = s4.y; sc[gi][2] = s4.z; sc[gi][3] = s4.w;
        const uint32_t zw = zrow[gi * kWordsPerRow + j];
        zlo[gi][0] = (zw & 0x000F000Fu) | 0x64006400u;
        zhi[gi][0] = (zw & 0x00F000F0u) | 0x64006400u;
        zlo[gi][1] = ((zw >> 8) & 0x000F000Fu) | 0x64006400u;
        zhi[gi][1] = ((zw >> 8) & 0x00F000F0u) | 0x64006400u;
      }
      uint8_t *a_tile = a_ring + os * kABytes;
      const bool full_rows = k_base + kTileK <= p.K;
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const int r = r0 + 16 * ii;
        const int gi = r >= split_row ? 1 : 0;
        uint32_t out[4] = {0, 0, 0, 0};
        if (col_ok && (full_rows || k_base + r < p.K)) {
          // Word nibbles (0..7) hold columns (0,2,4,6,1,3,5,7).  Masking the
          // word with 0x000F000F and OR-ing 0x6400 gives the half2 of 1024 + q
          // for columns (0, 1); 0x00F000F0 gives 1024 + 16 q for columns
          // (2, 3); the word shifted by 8 gives columns (4, 5) and (6, 7).
          // Differences of these biased values are the exact integers
          // (q - z) and 16 (q - z); one fp16 multiply by the scale rounds like
          // the reference, and the factor 16 (exact) is removed in the fp32
          // epilogue.
          const uint32_t w8 = w[ii] >> 8;
          const uint32_t q0 = (w[ii] & 0x000F000Fu) | 0x64006400u;
          const uint32_t q1 = (w[ii] & 0x00F000F0u) | 0x64006400u;
          const uint32_t q2 = (w8 & 0x000F000Fu) | 0x64006400u;
          const uint32_t q3 = (w8 & 0x00F000F0u) | 0x64006400u;
          const uint32_t z0 = gi ? zlo[1][0] : zlo[0][0];
          const uint32_t z1 = gi ? zhi[1][0] : zhi[0][0];
          const uint32_t z2 = gi ? zlo[1][1] : zlo[0][1];
          const uint32_t z3 = gi ? zhi[1][1] : zhi[0][1];
          out[0] = h2_bits(__hmul2(__hsub2(bits_h2(q0), bits_h2(z0)), bits_h2(gi ? sc[1][0] : sc[0][0])));
          out[1] = h2_bits(__hmul2(__hsub2(bits_h2(q1), bits_h2(z1)), bits_h2(gi ? sc[1][1] : sc[0][1])));
          out[2] = h2_bits(__hmul2(__hsub2(bits_h2(q2), bits_h2(z2)), bits_h2(gi ? sc[1][2] : sc[0][2])));
          out[3] = h2_bits(__hmul2(__hsub2(bits_h2(q3), bits_h2(z3)), bits_h2(gi ? sc[1][3] : sc[0][3])));
        }
        *reinterpret_cast<uint4 *>(a_tile + a_off[ii]) = make_uint4(out[0], out[1], out[2], out[3]);
      }
      // The A tile (written here) and this thread's activation chunks (written
      // by cp.async, complete after the wait above) are read by the tensor
      // cores through the async proxy.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[os]);
    }
    cp_async_wait_all();

    // ---------------- epilogue ----------------
    if (ok && nk > 0) ok = mbar_wait(acc_full, 0, abort_flag);
    ok = __all_sync(0xffffffffu, ok) && nk > 0;
    tc_fence_after();
    const int quad = warp & 3;
    const int half_idx = (warp - kFirstDequantWarp) >> 2;
    const int n_local = quad * 32 + lane;
    const int n = n0 + n_local;
    const bool n_ok = n < p.N;
    const float bias_n = (p.bias != nullptr && n_ok) ? __half2float(__ushort_as_half(p.bias[n])) : 0.f;
    // Columns 2, 3, 6, 7 of every 8 were accumulated as 16 W (see above).
    const float col_scale = (n & 2) ? 0.0625f : 1.0f;
    constexpr int kCols = BN / 2;
    const int c_begin = half_idx * kCols;
    const uint32_t t_row = tmem_d + (static_cast<uint32_t>(quad * 32) << 16);
    if (p.splits == 1) {
      if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < kCols; c0 += 8) {
          float v[8];
          tmem_ld_32x32b_x8(t_row + c_begin + c0, v);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int m = m0 + c_begin + c0 + c;
            if (m < p.M && n_ok)
              p.y[static_cast<size_t>(m) * p.N + n] =
                  __half_as_ushort(__float2half_rn(fmaf(v[c], col_scale, bias_n)));
          }
        }
      }
    } else if constexpr (BN <= 64) {
      float acc[kCols];
      if (ok) {
#pragma unroll
        for (int c0 = 0; c0 < kCols; c0 += 8) {
          float v[8];
          tmem_ld_32x32b_x8(t_row + c_begin + c0, v);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 8; ++c) acc[c0 + c] = v[c] * col_scale;
        }
      }
      const int tile_id = m_tile * p.n_tiles + n_tile;
      float *part = p.partials + static_cast<size_t>(tile_id) * p.splits * BN * kTileN;
      if (ok) {
#pragma unroll
        for (int c = 0; c < kCols; ++c)
          __stcg(part + (static_cast<size_t>(split) * BN + c_begin + c) * kTileN + n_local, acc[c]);
      }
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kDequantThreads) : "memory");
      if (t == 0) {
        const unsigned int prev = ok ? atomicAdd(p.semaphores + tile_id, 1u) : 0u;
        *last_flag = (ok && prev == static_cast<unsigned int>(p.splits - 1)) ? 1 : 0;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kDequantThreads) : "memory");
      if (*last_flag) {
        __threadfence();
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
          float sum = 0.f;
          for (int s = 0; s < p.splits; ++s) {
            sum += (s == split) ? acc[c]
                                : __ldcg(part + (static_cast<size_t>(s) * BN + c_begin + c) * kTileN + n_local);
          }
          const int m = m0 + c_begin + c;
          if (m < p.M && n_ok)
            p.y[static_cast<size_t>(m) * p.N + n] = __half_as_ushort(__float2half_rn(sum + bias_n));
        }
        if (t == 0) p.semaphores[tile_id] = 0u;
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_d, C::kTmemCols);
  }
}

// Full fp16 weight materialisation: one thread per packed word.
__global__ void awq_dequantize_kernel(const int32_t *__restrict__ qweight,
                                      const int32_t *__restrict__ qzeros,
                                      const uint16_t *__restrict__ scales, uint16_t *__restrict__ w,
                                      int K, int N, int G) {
  const int words_per_row = N >> 3;
  const long long total = static_cast<long long>(K) * words_per_row;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(idx / words_per_row);
    const int j = static_cast<int>(idx % words_per_row);
    const int g = k / G;
    const uint32_t qw = static_cast<uint32_t>(__ldg(qweight + idx));
    const uint32_t zw = static_cast<uint32_t>(__ldg(qzeros + static_cast<size_t>(g) * words_per_row + j));
    const uint4 s4 = __ldg(reinterpret_cast<const uint4 *>(scales + static_cast<size_t>(g) * N + 8 * j));
    const uint32_t sc[4] = {s4.x, s4.y, s4.z, s4.w};
    uint32_t out[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t qh = ((qw >> (4 * q)) & 0x000F000Fu) | 0x64006400u;
      const uint32_t zh = ((zw >> (4 * q)) & 0x000F000Fu) | 0x64006400u;
      out[q] = h2_bits(__hmul2(__hsub2(bits_h2(qh), bits_h2(zh)), bits_h2(sc[q])));
    }
    *reinterpret_cast<uint4 *>(w + static_cast<size_t>(k) * N + 8 * j) =
        make_uint4(out[0], out[1], out[2], out[3]);
  }
}

}  // namespace awq
}  // namespace lvb
