// AutoAWQ W4A16 linear on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// y[m, n] = sum_k x[m, k] * W[k, n] (+ bias[n]),  W[k, n] = fp16(q - z) * s.
//
// The weight is the UMMA "A" operand (M = 128 output columns per CTA) and the
// activations are "B" (N = BN tokens), so a decode step with a handful of
// tokens still fills the 128-row tensor-core tile ("swap-AB").  Per CTA:
//
//   warp 0        TMA producer of the raw int4 tiles (64 k x 128 n = 4 KB)
//   warp 1        TMEM allocator and the single thread issuing tcgen05.mma
//   warp 2        TMA producer of the activation tiles (BN x 64 fp16, SW128)
//   warps 4..11   dequantisers: raw words -> fp16 W tile written straight
//                 into the MN-major SWIZZLE_128B operand layout; afterwards
//                 the epilogue (TMEM -> registers -> fp16 y).
//
// The dequantisation reproduces the reference's fp16 arithmetic exactly
// (modeling/quantization/awq.py:433-450): a nibble v becomes the fp16 value
// 1024 + v by OR-ing it under the exponent of 1024 (0x6400), the difference of
// two such values is the exact integer q - z, and one fp16 multiply by the
// scale gives the same rounding as the reference's dequantised weight.  With
// the AutoAWQ nibble order (0,2,4,6,1,3,5,7), the word shifted right by 4p
// and masked with 0x000F000F yields the column pair (2p, 2p+1) as one half2.
//
// Small grids split K across CTAs; the partial fp32 tiles go to a workspace
// and the last CTA of a tile (found with a per-tile semaphore) sums them in
// split order, so results are deterministic.
#pragma once

#include <cudaTypedefs.h>

#include "lvb_common.cuh"

namespace lvb {
namespace awq {

constexpr int kTileN = 128;                           // output columns per CTA (UMMA M)
constexpr int kTileK = 64;                            // k per pipeline stage
constexpr int kWordsPerRow = kTileN / 8;              // packed words per k row of a tile
constexpr int kRawBytes = kTileK * kWordsPerRow * 4;  // 4096
constexpr int kABytes = kTileN * kTileK * 2;          // 16384
constexpr int kALbo = 1024;  // byte stride between the two 64-column MN atoms
constexpr int kASbo = 2048;  // byte stride between 8-row k groups
constexpr int kDequantWarps = 8;
constexpr int kDequantThreads = kDequantWarps * 32;
constexpr int kFirstDequantWarp = 4;
constexpr int kThreads = (kFirstDequantWarp + kDequantWarps) * 32;  // 384

template <int BN>
struct Config {
  static constexpr int kXBytes = BN * kTileK * 2;
  static constexpr int kOpStages = BN >= 256 ? 3 : 4;
  static constexpr int kRawStages = BN >= 128 ? 8 : 16;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kAOff = 0;
  static constexpr int kXOff = kAOff + kOpStages * kABytes;
  static constexpr int kRawOff = kXOff + kOpStages * kXBytes;
  static constexpr int kBarOff = kRawOff + kRawStages * kRawBytes;
  // raw_full, raw_empty (kRawStages each); x_full, a_full, op_empty
  // (kOpStages each); acc_full.
  static constexpr int kNumBars = 2 * kRawStages + 3 * kOpStages + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 64 + 1024;  // + base alignment slack
};

struct Params {
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

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    awq_gemm_kernel(const __grid_constant__ CUtensorMap qmap,
                    const __grid_constant__ CUtensorMap xmap, const Params p) {
  using C = Config<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *a_ring = smem + C::kAOff;
  uint8_t *x_ring = smem + C::kXOff;
  uint32_t *raw_ring = reinterpret_cast<uint32_t *>(smem + C::kRawOff);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *raw_full = bars;
  uint64_t *raw_empty = raw_full + C::kRawStages;
  uint64_t *x_full = raw_empty + C::kRawStages;
  uint64_t *a_full = x_full + C::kOpStages;
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
    for (int s = 0; s < C::kRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kDequantWarps);
    }
    for (int s = 0; s < C::kOpStages; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&a_full[s], kDequantWarps);
      mbar_init(&op_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&xmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    // ---------------- raw int4 tile producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kRawStages;
        const uint32_t ph = (i / C::kRawStages) & 1;
        if (!mbar_wait(&raw_empty[s], ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&raw_full[s], kRawBytes);
        tma_load_2d(raw_ring + s * (kRawBytes / 4), &qmap, &raw_full[s], n0 / 8,
                    (kt_begin + i) * kTileK);
        issued = i + 1;
      }
      if (*abort_flag) {  // drain copies still in flight before the CTA exits
        for (int i = issued - C::kRawStages < 0 ? 0 : issued - C::kRawStages; i < issued; ++i)
          mbar_wait(&raw_full[i % C::kRawStages], (i / C::kRawStages) & 1, nullptr,
                    kDrainBudgetCycles);
      }
    }
  } else if (warp == 2) {
    // ---------------- activation tile producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kOpStages;
        const uint32_t ph = (i / C::kOpStages) & 1;
        if (!mbar_wait(&op_empty[s], ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&x_full[s], C::kXBytes);
        tma_load_2d(x_ring + s * C::kXBytes, &xmap, &x_full[s], (kt_begin + i) * kTileK, m0);
        issued = i + 1;
      }
      if (*abort_flag) {
        for (int i = issued - C::kOpStages < 0 ? 0 : issued - C::kOpStages; i < issued; ++i)
          mbar_wait(&x_full[i % C::kOpStages], (i / C::kOpStages) & 1, nullptr,
                    kDrainBudgetCycles);
      }
    }
  } else if (warp == 1) {
    // ---------------- tcgen05.mma issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(kTileN, BN, 0, 0, /*a MN-major*/ 1, 0);
      const uint32_t a_base = smem_u32(a_ring);
      const uint32_t x_base = smem_u32(x_ring);
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % C::kOpStages;
        const uint32_t ph = (i / C::kOpStages) & 1;
        ok = mbar_wait(&a_full[s], ph, abort_flag) && mbar_wait(&x_full[s], ph, abort_flag);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTileK / 16; ++kk) {
          const uint64_t adesc =
              umma_smem_desc_sw128(a_base + s * kABytes + kk * 2 * kASbo, kALbo, kASbo);
          const uint64_t bdesc = umma_smem_desc_sw128(x_base + s * C::kXBytes + kk * 32, 16, 1024);
          umma_f16(tmem_d, adesc, bdesc, idesc, (i | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&op_empty[s]);
      }
      umma_commit(acc_full);
      if (!ok) mbar_wait(acc_full, 0, nullptr, kDrainBudgetCycles);
    }
    __syncwarp();
  } else if (warp >= kFirstDequantWarp) {
    // ---------------- dequantisers ----------------
    const int t = threadIdx.x - kFirstDequantWarp * 32;
    const int j = t & 15;   // packed word (8 columns) within the tile row
    const int r0 = t >> 4;  // first of the rows r0 + 16 * ii
    const int n_col = n0 + 8 * j;
    const bool col_ok = n_col < p.N;
    const int words_per_row = p.N >> 3;
    int cached_g = -1;
    uint32_t zq[4] = {0, 0, 0, 0};
    uint32_t sc[4] = {0, 0, 0, 0};
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int rs = i % C::kRawStages;
      const uint32_t rph = (i / C::kRawStages) & 1;
      const int os = i % C::kOpStages;
      const uint32_t oph = (i / C::kOpStages) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[rs], rph, abort_flag))) { ok = false; break; }
      const uint32_t *raw = raw_ring + rs * (kRawBytes / 4);
      uint32_t w[4];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) w[ii] = raw[(r0 + 16 * ii) * kWordsPerRow + j];
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[rs]);
      if (!__all_sync(0xffffffffu, mbar_wait(&op_empty[os], oph ^ 1, abort_flag))) { ok = false; break; }
      uint8_t *a_tile = a_ring + os * kABytes;
      const int k_base = (kt_begin + i) * kTileK;
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const int r = r0 + 16 * ii;
        const int k = k_base + r;
        uint32_t out[4] = {0, 0, 0, 0};
        if (k < p.K && col_ok) {
          const int g = k / p.G;
          if (g != cached_g) {
            cached_g = g;
            const uint32_t zw = static_cast<uint32_t>(
                __ldg(p.qzeros + static_cast<size_t>(g) * words_per_row + (n_col >> 3)));
            const uint4 s4 = __ldg(reinterpret_cast<const uint4 *>(
                p.scales + static_cast<size_t>(g) * p.N + n_col));
            sc[0] = s4.x; sc[1] = s4.y; sc[2] = s4.z; sc[3] = s4.w;
#pragma unroll
            for (int q = 0; q < 4; ++q) zq[q] = ((zw >> (4 * q)) & 0x000F000Fu) | 0x64006400u;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t qh = ((w[ii] >> (4 * q)) & 0x000F000Fu) | 0x64006400u;
            const __half2 d = __hsub2(bits_h2(qh), bits_h2(zq[q]));
            out[q] = h2_bits(__hmul2(d, bits_h2(sc[q])));
          }
        }
        const int kr = r & 7;
        const uint32_t off = (r >> 3) * kASbo + (j >> 3) * kALbo + kr * 128 + (((j & 7) ^ kr) << 4);
        *reinterpret_cast<uint4 *>(a_tile + off) = make_uint4(out[0], out[1], out[2], out[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[os]);
    }

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
              p.y[static_cast<size_t>(m) * p.N + n] = __half_as_ushort(__float2half_rn(v[c] + bias_n));
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
          for (int c = 0; c < 8; ++c) acc[c0 + c] = v[c];
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
  if (warp == 1) {
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
