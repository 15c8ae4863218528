// AutoAWQ W4A16 linear for decode-sized batches (M <= 64) on sm_100a.
//
// y[m, n] = sum_g s[g, n] * sum_{k in g} x[m, k] * (q[k, n] - z[g, n])  (+ bias[n])
//
// Same swap-AB tile as awq_gemm_kernel (128 output columns = UMMA M, BN <= 64
// tokens = UMMA N), but the tensor cores accumulate the exact integers
// (q - z), held exactly in fp16, one quantization group at a time, into
// one of four TMEM buffers; four drain warps apply the fp32 group scale per
// group.  The int4 -> operand conversion is then two integer ops and one fp16
// subtraction per pair of weights (no scale multiply, no rounding), which keeps
// the SM's issue slots far below what streaming the weights at HBM rate needs;
// products and sums are exact in fp32, so the result is closer to the exact
// value than the reference's fp16-rounded dequantised weight.
//
//   warp 0        TMEM allocator, single thread issuing tcgen05.mma: per
//                 k-step into the group's TMEM buffer; commits a buffer when
//                 its group ends and waits for the drain before reusing it
//   warps 1..8    loaders + converters: cp.async multistage pipeline of raw
//                 stages (int4 tile 64 k x 128 n, the activation tile in the
//                 SWIZZLE_128B K-major operand layout, packed zeros of the at
//                 most two groups the tile spans), then (q - z) -> MN-major
//                 SWIZZLE_128B A tile
//   warps 9..12   drain: per group, TMEM -> registers, acc += s * P (fp32);
//                 finally bias, fp16 store or split-K partial + fixup
#pragma once

#include "awq_gemm.cuh"
#include "lvb_common.cuh"

namespace lvb {
namespace awq {

constexpr int kGvWriterWarps = 8;
constexpr int kGvWriters = kGvWriterWarps * 32;
constexpr int kGvFirstWriterWarp = 1;
constexpr int kGvFirstDrainWarp = kGvFirstWriterWarp + kGvWriterWarps;  // 9
constexpr int kGvDrainThreads = 128;
constexpr int kGvThreads = (kGvFirstDrainWarp + 4) * 32;  // 416
constexpr int kGvBuffers = 4;                             // TMEM group buffers
constexpr int kGvScaleRing = 8;                           // groups of scales in flight per drain warp

template <int BN>
struct GvConfig {
  static constexpr int kXBytes = BN * kTileK * 2;
  static constexpr int kQOff = kXBytes;
  static constexpr int kZOff = kQOff + kQBytes;
  static constexpr int kStageBytes = ((kZOff + kZeroBytes) + 1023) / 1024 * 1024;
  static constexpr int kOpStages = 4;
  static constexpr int kRawStages = BN >= 64 ? 10 : 16;
  static constexpr int kAhead = kRawStages - kOpStages;
  static constexpr int kTmemCols = kGvBuffers * BN < 32 ? 32 : kGvBuffers * BN;
  static constexpr int kAOff = 0;
  static constexpr int kRawOff = kOpStages * kABytes;
  static constexpr int kScaleOff = kRawOff + kRawStages * kStageBytes;  // drain scale rings
  static constexpr int kScaleBytes = 4 * kGvScaleRing * 64;
  static constexpr int kBarOff = kScaleOff + kScaleBytes;
  // ready (raw slots), a_full, op_empty (A slots), grp_full, grp_empty.
  static constexpr int kNumBars = kRawStages + 2 * kOpStages + 2 * kGvBuffers;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 64 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int BN>
__device__ __forceinline__ void gv_load_stage(const Params &p, uint32_t stage, int kt, int n0, int m0,
                                              int t) {
  using C = GvConfig<BN>;
  const int kb = kt * kTileK;
  const int words = p.N >> 3;
  {
    const int r = t >> 2;
    const int w = (t & 3) * 4;
    const bool ok = kb + r < p.K && (n0 >> 3) + w < words;
    const int32_t *src = p.qweight + static_cast<size_t>(ok ? kb + r : 0) * words + (ok ? (n0 >> 3) + w : 0);
    cp_async_16(stage + C::kQOff + r * 64 + w * 4, src, ok ? 16u : 0u);
  }
#pragma unroll
  for (int c = t; c < BN * 8; c += kGvWriters) {
    const int m = c >> 3;
    const int cc = c & 7;
    const bool ok = m0 + m < p.M && kb + cc * 8 < p.K;
    const uint16_t *src = p.x + static_cast<size_t>(ok ? m0 + m : 0) * p.K + (ok ? kb + cc * 8 : 0);
    cp_async_16(stage + m * 128 + ((cc ^ (m & 7)) << 4), src, ok ? 16u : 0u);
  }
  if (t < 8) {
    const int g0 = kb / p.G;
    const int gi = t >> 2;
    const int w = (t & 3) * 4;
    const bool ok = g0 + gi < p.K / p.G && (n0 >> 3) + w < words;
    const int32_t *src = p.qzeros + static_cast<size_t>(ok ? g0 + gi : 0) * words + (ok ? (n0 >> 3) + w : 0);
    cp_async_16(stage + C::kZOff + gi * 64 + w * 4, src, ok ? 16u : 0u);
  }
}

template <int BN, bool kSingleGroup>
__global__ void __launch_bounds__(kGvThreads, 1) awq_gemv_kernel(const Params p) {
  using C = GvConfig<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *a_ring = smem + C::kAOff;
  uint8_t *raw_ring = smem + C::kRawOff;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *ready = bars;
  uint64_t *a_full = ready + C::kRawStages;
  uint64_t *op_empty = a_full + C::kOpStages;
  uint64_t *grp_full = op_empty + C::kOpStages;
  uint64_t *grp_empty = grp_full + kGvBuffers;
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
  // Groups this CTA touches: [g_first, g_first + n_groups).
  const int k_lo = kt_begin * kTileK;
  const int k_hi = min(kt_end * kTileK, p.K);
  const int g_first = k_lo / p.G;
  const int n_groups = nk > 0 ? (k_hi - 1) / p.G - g_first + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kRawStages; ++s) mbar_init(&ready[s], kGvWriters);
    for (int s = 0; s < C::kOpStages; ++s) {
      mbar_init(&a_full[s], kGvWriterWarps);
      mbar_init(&op_empty[s], 1);
    }
    for (int b = 0; b < kGvBuffers; ++b) {
      mbar_init(&grp_full[b], 1);
      mbar_init(&grp_empty[b], 4);
    }
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
      int cur = -1;  // local group index being accumulated
      bool first = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % C::kOpStages;
        ok = mbar_wait(&a_full[s], (i / C::kOpStages) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t x_tile = raw_base + (i % C::kRawStages) * C::kStageBytes;
        const int kb = (kt_begin + i) * kTileK;
#pragma unroll
        for (int kk = 0; kk < kTileK / 16; ++kk) {
          const int k = kb + kk * 16;
          if (k >= p.K) break;
          const int gl = k / p.G - g_first;
          if (gl != cur) {
            if (cur >= 0) umma_commit(&grp_full[cur % kGvBuffers]);
            cur = gl;
            ok = mbar_wait(&grp_empty[cur % kGvBuffers], ((cur / kGvBuffers) & 1) ^ 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            first = true;
          }
          const uint64_t adesc =
              umma_smem_desc_sw128(a_base + s * kABytes + kk * 2 * kASbo, kALbo, kASbo);
          const uint64_t bdesc = umma_smem_desc_sw128(x_tile + kk * 32, 16, 1024);
          umma_f16(tmem_d + (cur % kGvBuffers) * BN, adesc, bdesc, idesc, first ? 0u : 1u);
          first = false;
        }
        umma_commit(&op_empty[s]);
      }
      if (cur >= 0) umma_commit(&grp_full[cur % kGvBuffers]);
      if (!ok && cur >= 0) mbar_wait(&grp_full[cur % kGvBuffers], (cur / kGvBuffers) & 1, nullptr, kDrainBudgetCycles);
    }
    __syncwarp();
  } else if (warp < kGvFirstDrainWarp) {
    // ---------------- loaders + converters ----------------
    const int t = threadIdx.x - kGvFirstWriterWarp * 32;
    const int j = t & 15;   // packed word (8 columns) within the tile row
    const int r0 = t >> 4;  // first of the rows r0 + 16 * ii
    const bool col_ok = n0 + 8 * j < p.N;
    const uint32_t raw_base = smem_u32(raw_ring);
    uint32_t a_off[4];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const int r = r0 + 16 * ii;
      const int kr = r & 7;
      a_off[ii] = (r >> 3) * kASbo + (j >> 3) * kALbo + kr * 128 + (((j & 7) ^ kr) << 4);
    }
#pragma unroll 1
    for (int i = 0; i < C::kAhead && i < nk; ++i) {
      gv_load_stage<BN>(p, raw_base + (i % C::kRawStages) * C::kStageBytes, kt_begin + i, n0, m0, t);
      cp_async_arrive_noinc(&ready[i % C::kRawStages]);
    }
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int os = i % C::kOpStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&op_empty[os], ((i / C::kOpStages) & 1) ^ 1, abort_flag))) {
        ok = false;
        break;
      }
      if (i + C::kAhead < nk) {
        const int sl = (i + C::kAhead) % C::kRawStages;
        gv_load_stage<BN>(p, raw_base + sl * C::kStageBytes, kt_begin + i + C::kAhead, n0, m0, t);
        cp_async_arrive_noinc(&ready[sl]);
      }
      const int rs = i % C::kRawStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&ready[rs], (i / C::kRawStages) & 1, abort_flag))) {
        ok = false;
        break;
      }
      const uint8_t *stage = raw_ring + rs * C::kStageBytes;
      const uint32_t *raw = reinterpret_cast<const uint32_t *>(stage + C::kQOff);
      const uint32_t *zrow = reinterpret_cast<const uint32_t *>(stage + C::kZOff);
      uint32_t w[4];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) w[ii] = raw[(r0 + 16 * ii) * kWordsPerRow + j];
      // Zero points as the biased fp16 pairs 1024 + z (low nibble of a byte)
      // and 1024 + 16 z (high nibble), for the group rows of this tile.
      uint32_t zlo[2][2], zhi[2][2];
#pragma unroll
      for (int gi = 0; gi < (kSingleGroup ? 1 : 2); ++gi) {
        const uint32_t zw = zrow[gi * kWordsPerRow + j];
        zlo[gi][0] = (zw & 0x000F000Fu) | 0x64006400u;
        zhi[gi][0] = (zw & 0x00F000F0u) | 0x64006400u;
        zlo[gi][1] = ((zw >> 8) & 0x000F000Fu) | 0x64006400u;
        zhi[gi][1] = ((zw >> 8) & 0x00F000F0u) | 0x64006400u;
      }
      int split_row = kTileK;
      if constexpr (!kSingleGroup) {
        const int k_base = (kt_begin + i) * kTileK;
        split_row = (k_base / p.G + 1) * p.G - k_base;
      }
      uint8_t *a_tile = a_ring + os * kABytes;
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const int gi = kSingleGroup ? 0 : ((r0 + 16 * ii) >= split_row ? 1 : 0);
        // Word nibbles (0..7) hold columns (0,2,4,6,1,3,5,7).  Mask 0x000F000F
        // (OR 0x6400) gives 1024 + q for columns (0, 1), mask 0x00F000F0 gives
        // 1024 + 16 q for columns (2, 3); the word shifted by 8 gives (4, 5)
        // and (6, 7).  Subtracting the biased zero leaves the exact integer
        // q - z (or 16 (q - z)) in fp16; rows past K and columns past N are
        // zero-filled copies and give 0.
        const uint32_t w8 = w[ii] >> 8;
        const uint32_t q0 = (w[ii] & 0x000F000Fu) | 0x64006400u;
        const uint32_t q1 = (w[ii] & 0x00F000F0u) | 0x64006400u;
        const uint32_t q2 = (w8 & 0x000F000Fu) | 0x64006400u;
        const uint32_t q3 = (w8 & 0x00F000F0u) | 0x64006400u;
        uint32_t out[4];
        out[0] = h2_bits(__hsub2(bits_h2(q0), bits_h2(gi ? zlo[1][0] : zlo[0][0])));
        out[1] = h2_bits(__hsub2(bits_h2(q1), bits_h2(gi ? zhi[1][0] : zhi[0][0])));
        out[2] = h2_bits(__hsub2(bits_h2(q2), bits_h2(gi ? zlo[1][1] : zlo[0][1])));
        out[3] = h2_bits(__hsub2(bits_h2(q3), bits_h2(gi ? zhi[1][1] : zhi[0][1])));
        if (!col_ok) out[0] = out[1] = out[2] = out[3] = 0u;
        *reinterpret_cast<uint4 *>(a_tile + a_off[ii]) = make_uint4(out[0], out[1], out[2], out[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[os]);
    }
    (void)ok;
    cp_async_wait_all();
  } else {
    // ---------------- drain: per-group scaling, then the epilogue ----------------
    const int dw = warp - kGvFirstDrainWarp;  // 0..3
    const int quad = warp & 3;                // TMEM lane quadrant this warp may access
    const int n_local = quad * 32 + lane;
    const int n = n0 + n_local;
    const bool n_ok = n < p.N;
    // Columns 2, 3, 6, 7 of every 8 were accumulated as 16 (q - z).
    const float col_factor = (n & 2) ? 0.0625f : 1.0f;
    // Per-warp ring of this warp's 32 scales per group (64 bytes), filled by
    // lanes 0..3 with cp.async kGvScaleRing - 1 groups ahead.
    const uint32_t sring = smem_u32(smem + C::kScaleOff) + dw * kGvScaleRing * 64;
    const uint16_t *sring_ptr = reinterpret_cast<const uint16_t *>(smem + C::kScaleOff + dw * kGvScaleRing * 64);
    auto load_scales = [&](int gl) {
      if (lane < 4) {
        const int col = n0 + quad * 32 + lane * 8;
        const bool ok = gl < n_groups && col < p.N;
        const uint16_t *src = p.scales + static_cast<size_t>(ok ? g_first + gl : 0) * p.N + (ok ? col : 0);
        cp_async_16(sring + (gl % kGvScaleRing) * 64 + lane * 16, src, ok ? 16u : 0u);
      }
      cp_async_commit();
    };
#pragma unroll 1
    for (int gl = 0; gl < kGvScaleRing - 1; ++gl) load_scales(gl);
    float acc[BN];
#pragma unroll
    for (int m = 0; m < BN; ++m) acc[m] = 0.f;
    const uint32_t t_lane = tmem_d + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    for (int gl = 0; gl < n_groups; ++gl) {
      const int b = gl % kGvBuffers;
      load_scales(gl + kGvScaleRing - 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&grp_full[b], (gl / kGvBuffers) & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      asm volatile("cp.async.wait_group %0;" ::"n"(kGvScaleRing - 1) : "memory");
      __syncwarp();
      const float s = __half2float(__ushort_as_half(sring_ptr[(gl % kGvScaleRing) * 32 + lane])) * col_factor;
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 8) {
        float v[8];
        tmem_ld_32x32b_x8(t_lane + b * BN + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c0 + c] = fmaf(s, v[c], acc[c0 + c]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&grp_empty[b]);
    }
    cp_async_wait_all();
    ok = __all_sync(0xffffffffu, ok);
    const float bias_n = (p.bias != nullptr && n_ok) ? __half2float(__ushort_as_half(p.bias[n])) : 0.f;
    if (p.splits == 1) {
      if (ok) {
#pragma unroll
        for (int m = 0; m < BN; ++m)
          if (m0 + m < p.M && n_ok)
            p.y[static_cast<size_t>(m0 + m) * p.N + n] = __half_as_ushort(__float2half_rn(acc[m] + bias_n));
      }
    } else {
      const int tile_id = m_tile * p.n_tiles + n_tile;
      float *part = p.partials + static_cast<size_t>(tile_id) * p.splits * BN * kTileN;
      if (ok) {
#pragma unroll
        for (int m = 0; m < BN; ++m) __stcg(part + (static_cast<size_t>(split) * BN + m) * kTileN + n_local, acc[m]);
      }
      __threadfence();
      asm volatile("bar.sync 2, %0;" ::"n"(kGvDrainThreads) : "memory");
      if (dw == 0 && lane == 0) {
        const unsigned int prev = ok ? atomicAdd(p.semaphores + tile_id, 1u) : 0u;
        *last_flag = (ok && prev == static_cast<unsigned int>(p.splits - 1)) ? 1 : 0;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kGvDrainThreads) : "memory");
      if (*last_flag) {
        __threadfence();
#pragma unroll
        for (int m = 0; m < BN; ++m) {
          float sum = 0.f;
          for (int sp = 0; sp < p.splits; ++sp)
            sum += (sp == split) ? acc[m] : __ldcg(part + (static_cast<size_t>(sp) * BN + m) * kTileN + n_local);
          if (m0 + m < p.M && n_ok)
            p.y[static_cast<size_t>(m0 + m) * p.N + n] = __half_as_ushort(__float2half_rn(sum + bias_n));
        }
        if (dw == 0 && lane == 0) p.semaphores[tile_id] = 0u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_d, C::kTmemCols);
  }
}

}  // namespace awq
}  // namespace lvb
