// W4A16 linear for decode batches of 1..16 rows on warp-level fp16 tensor-core
// MMAs (mma.sync.m16n8k16, fp32 accumulation), straight from the packed codes.
//
// Reference: the decode-sized path of CudaAWQOperation (M <= 255 -> K1
// `gemm_forward_4bit_cuda_m16nXk32`, csrc/awq/gemm_kernels.cu:29-326, 444-501,
// called from modeling/quantization/cuda_awq.py:96-122): y = x @ W (+ bias),
// W[k][n] = (q - z) * s per group of G k.
//
// Here the weight tile is the MMA's A operand (16 output columns x 16 k) and
// the batch is its N (8 token rows per tile, NT tiles), so at 1..16 rows each
// MMA multiplies at most one tile of padding.  The A operand is the
// reference's own dequantised weight,
//
//   W[k][c] = fp16((q - z) * s)   the code OR 0x6400 is the fp16 1024 + q;
//                                 subtracting the half2 (1024 + z) leaves
//                                 q - z exactly, and one fp16 multiply by s
//                                 rounds it as modeling/quantization/
//                                 awq.py:433-450 does,
//   y[t][c] = sum_k W[k][c] x[t][k]   fp16 products, fp32 accumulation in
//                                 the MMA over the whole range (the
//                                 arithmetic of the reference's fp16 matmul,
//                                 awq.py:453-465, up to summation order),
//
// with the fp16 x unchanged (no limbs, no scaling).
//
// Operand order.  Within a 32-k run, packed code word w of a column holds in
// its low nibbles k = 4w + (0, 2, 1, 3) (bytes 0..3) and in its high nibbles
// k = 16 + 4w + (0, 2, 1, 3).  Lane (g, t) of a warp (g = lane / 4,
// t = lane % 4) reads word t of columns g and g + 8 and forms the four A
// registers of one MMA from the low nibbles (k = 4t .. 4t + 3) and four from
// the high nibbles (k = 16 + 4t ..).  An MMA sums over its 16 k in any order,
// so the A halves (k 4t, 4t + 1) and (4t + 2, 4t + 3) stand in the slots of
// the fragment's (2t, 2t + 1) and (2t + 8, 2t + 9) as long as the B operand
// uses the same mapping: its two registers are x[token g][4t .. 4t + 3], one
// 8-byte shared-memory load from the token's row.
//
// CTA: one 128-column packed tile, a range of whole groups (split-K), eight
// consumer warps of 16 columns and one producer warp.  The producer streams
// each stage -- 8 runs of codes (16 KB, contiguous in the packed layout) and
// the matching 256 k of every token row (512 bytes per row, from L2) -- into
// a ring of shared-memory stages with bulk async copies on one mbarrier; the
// codes of the first stages are requested before the kernel that produced x
// has finished (programmatic dependent launch), the x rows after it.  Token
// rows sit 544 bytes apart, so the 8-byte B loads of a warp hit distinct
// banks.  Splits combine through per-split fp32 partials and a semaphore: the
// last CTA of a tile sums them in split order (deterministic), adds the bias
// and writes y.  Every wait is bounded.
#pragma once

#include <cuda_fp16.h>

#include "awq_decode.cuh"
#include "lvb_common.cuh"

namespace lvb {
namespace awqm {

constexpr int kCols = 128;                      // output columns per CTA (one packed tile)
constexpr int kStageRuns = 8;                   // 32-k runs per stage (B200: 8 beat 4 by 4-10 %)
constexpr int kMinStages = 2;                   // ring depth the plan guarantees
constexpr int kMaxStages = 16;                  // the host fills shared memory up to this
constexpr int kCodeBytes = kStageRuns * kCols * 16;   // 16 KB of codes per stage
constexpr int kXRowBytes = kStageRuns * 32 * 2;       // 512 B of one token row per stage
constexpr int kXRow = kXRowBytes + 32;                // row pitch: rows 0..3 on distinct 32-byte bank groups
constexpr int kMaxRows = 16;

// Shared memory: `stages` ring slots of [codes 16 KB][token rows], the
// range's (scale, zero) words [group][128], then the barriers (full[stages],
// empty[stages], sz) and the abort flag.
template <int NT>
struct MmaCfg {
  static constexpr int kRows = 8 * NT;
  static constexpr int kStageBytes = kCodeBytes + kRows * kXRow;
  __host__ __device__ static size_t sz_off(int stages) { return static_cast<size_t>(stages) * kStageBytes; }
  __host__ __device__ static size_t bar_off(int gps, int stages) {
    return sz_off(stages) + static_cast<size_t>(gps) * kCols * 4;
  }
  __host__ __device__ static size_t bytes(int gps, int stages) {
    return bar_off(gps, stages) + (2 * stages + 1) * 8 + 16;
  }
};

struct MmaParams {
  const uint8_t *qpack;    // [n_tiles][k_chunks][128][16 B]
  const uint32_t *szpack;  // [n_tiles][groups][128]: scale bits | zero << 16
  const uint16_t *x;       // [M] rows of x_stride fp16
  int64_t x_stride;
  const uint16_t *bias;    // may be null
  uint16_t *y;             // [M][N]
  uint32_t *semaphores;    // [n_tiles], zero between calls
  float *partials;         // [n_tiles][splits][M][128]
  int M, N;
  int groups, k_chunks, runs_per_group;
  int n_tiles, splits, groups_per_split;
  int stages;              // ring depth, kMinStages..kMaxStages
};

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Consumer warps of CPW columns (16: one A tile; 32: two A tiles sharing
// each B fragment) over the 128 columns of a tile.
template <int CPW>
struct MmaWarps {
  static constexpr int kWarps = kCols / CPW;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kCtaThreads = kThreads + 32;
};

template <int NT, int CPW>
__global__ void __launch_bounds__(MmaWarps<CPW>::kCtaThreads, 3) awq_mma_kernel(const __grid_constant__ MmaParams p) {
  using C = MmaCfg<NT>;
  constexpr int R = C::kRows;
  constexpr int kW = MmaWarps<CPW>::kWarps;
  constexpr int kCT = MmaWarps<CPW>::kThreads;
  constexpr int kCtaT = MmaWarps<CPW>::kCtaThreads;
  constexpr int kTiles = CPW / 16;  // A tiles per warp
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int rpg = p.runs_per_group;
  const int g0 = split * p.groups_per_split;
  const int g1 = min(p.groups, g0 + p.groups_per_split);
  const int run0 = g0 * rpg;
  const int nruns = (g1 - g0) * rpg;
  const int nstages = (nruns + kStageRuns - 1) / kStageRuns;
  const int stages = p.stages;
  const uint32_t *sz_sm = reinterpret_cast<const uint32_t *>(smem + C::sz_off(stages));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::bar_off(p.groups_per_split, stages));
  uint64_t *empty = full + stages;
  uint64_t *sz_bar = empty + stages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sz_bar + 1);
  auto csync = [] { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); };

  // The next kernel of the stream may launch now; it waits for this grid's
  // completion before touching y.
  pdl_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kW);
    }
    mbar_init(sz_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Token rows past M are never copied: they hold zeros (their outputs are
  // never stored, and zeros keep them finite).
  if (p.M < R) {
    const int row_words = kXRow / 16;
    const int per_stage = (R - p.M) * row_words;
    for (int i = tid; i < stages * per_stage; i += kCtaT) {
      const int s = i / per_stage, rem = i - s * per_stage;
      const int row = p.M + rem / row_words, w = rem - (rem / row_words) * row_words;
      *reinterpret_cast<int4 *>(smem + static_cast<size_t>(s) * C::kStageBytes + kCodeBytes + row * kXRow + w * 16) =
          make_int4(0, 0, 0, 0);
    }
  }
  __syncthreads();

  if (warp == kW) {
    // Producer.  Lane 0 sets each stage's byte count and copies its codes;
    // lane t < M copies token row t's slice of the stage.
    const uint8_t *codes = p.qpack + (static_cast<size_t>(tile) * p.k_chunks + run0) * kCols * 16;
    const bool xrow = lane < p.M;
    const uint16_t *xs = p.x + static_cast<size_t>(xrow ? lane : 0) * p.x_stride + static_cast<size_t>(run0) * 32;
    auto stage_runs = [&](int st) { return min(kStageRuns, nruns - st * kStageRuns); };
    auto copy_codes = [&](int st, int slot) {
      const uint32_t runs = static_cast<uint32_t>(stage_runs(st));
      mbar_arrive_expect_tx(&full[slot], runs * kCols * 16 + runs * 64 * static_cast<uint32_t>(p.M));
      awqd::bulk_load(smem + static_cast<size_t>(slot) * C::kStageBytes, codes + static_cast<size_t>(st) * kCodeBytes,
                      runs * kCols * 16, &full[slot]);
    };
    auto copy_x = [&](int st, int slot) {
      if (xrow)
        awqd::bulk_load(smem + static_cast<size_t>(slot) * C::kStageBytes + kCodeBytes + lane * kXRow,
                        xs + static_cast<size_t>(st) * kStageRuns * 32, static_cast<uint32_t>(stage_runs(st)) * 64,
                        &full[slot]);
    };
    if (lane == 0) {
      // The range's (scale, zero) rows are contiguous: one copy.
      const uint32_t sz_bytes = static_cast<uint32_t>(g1 - g0) * kCols * 4;
      mbar_arrive_expect_tx(sz_bar, sz_bytes);
      awqd::bulk_load(smem + C::sz_off(stages), p.szpack + (static_cast<size_t>(tile) * p.groups + g0) * kCols,
                      sz_bytes, sz_bar);
    }
    // The codes do not depend on the previous kernel: the first stages' copies
    // start at once; x does, so its rows follow the wait.
    const int pre = min(nstages, stages);
    if (lane == 0)
      for (int st = 0; st < pre; ++st) copy_codes(st, st);
    pdl_wait();
    __syncwarp();
    for (int st = 0; st < pre; ++st) copy_x(st, st);
    int issued = pre;
    int slot = 0;
    uint32_t phase = 0;  // parity of the empty phase to wait for at `slot`
    for (int st = pre; st < nstages; ++st) {
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&empty[slot], phase, abort_flag);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      if (lane == 0) copy_codes(st, slot);
      __syncwarp();
      copy_x(st, slot);
      issued = st + 1;
      if (++slot == stages) {
        slot = 0;
        phase ^= 1u;
      }
    }
    // Leave only once every copy issued has landed (shared memory must not
    // be written after the CTA ends).
    if (lane == 0) {
      for (int st = max(0, issued - stages); st < issued; ++st)
        mbar_wait(&full[st % stages], (st / stages) & 1, nullptr, kDrainBudgetCycles);
      mbar_wait(sz_bar, 0, nullptr, kDrainBudgetCycles);
    }
    return;
  }

  // y and the partials may still be read by the previous kernel of the stream.
  pdl_wait();
  const int g = lane >> 2, t4 = lane & 3;
  const int c0 = warp * CPW;
  // Two accumulators per (A tile, token tile): k = 0..15 and 16..31 of each
  // run, so consecutive MMAs do not wait on one another; summed at the end.
  float acc[kTiles][NT][4], acc2[kTiles][NT][4];
#pragma unroll
  for (int ct = 0; ct < kTiles; ++ct)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[ct][nt][i] = acc2[ct][nt][i] = 0.f;
  bool ok = mbar_wait(sz_bar, 0, abort_flag);
  // Columns c0 + 16 ct + g and + 8 of the current group: the half2 (1024 + z)
  // subtracted from the codes and the half2 scale.
  uint32_t z_lo[kTiles], z_hi[kTiles], s_lo[kTiles], s_hi[kTiles];
  auto load_group = [&](int gr) {
#pragma unroll
    for (int ct = 0; ct < kTiles; ++ct) {
      const uint32_t w0 = sz_sm[(gr - g0) * kCols + c0 + 16 * ct + g];
      const uint32_t w1 = sz_sm[(gr - g0) * kCols + c0 + 16 * ct + g + 8];
      z_lo[ct] = (0x6400u + (w0 >> 16)) * 0x10001u;
      z_hi[ct] = (0x6400u + (w1 >> 16)) * 0x10001u;
      s_lo[ct] = (w0 & 0xFFFFu) * 0x10001u;
      s_hi[ct] = (w1 & 0xFFFFu) * 0x10001u;
    }
  };
  // W = fp16((q - z) * s) for the two k of each half2 (q - z exact, one
  // rounding: the reference's dequantised weight).
  auto weight = [](uint32_t bits, uint32_t z, uint32_t sc) {
    return hmul2_bits(hsub2_bits((bits & 0x000F000Fu) | 0x64006400u, z), sc);
  };
  int group = g0, run_in_group = 0;
  if (ok) load_group(group);

  int slot = 0;
  uint32_t phase = 0;
  for (int st = 0; st < nstages && ok; ++st) {
    if (!mbar_wait(&full[slot], phase, abort_flag)) {
      ok = false;
      break;
    }
    const uint8_t *sb = smem + static_cast<size_t>(slot) * C::kStageBytes;
    const uint32_t *cw = reinterpret_cast<const uint32_t *>(sb) + (c0 + g) * 4 + t4;
    const uint8_t *xb = sb + kCodeBytes + g * kXRow + t4 * 8;
    const int runs = min(kStageRuns, nruns - st * kStageRuns);
#pragma unroll
    for (int r = 0; r < kStageRuns; ++r) {
      if (r < runs) {
        uint32_t a0[kTiles][4], a1[kTiles][4];
#pragma unroll
        for (int ct = 0; ct < kTiles; ++ct) {
          // Word t4 of columns c0 + 16 ct + g and + 8 (column stride 4 words).
          const uint32_t w0 = cw[r * kCols * 4 + ct * 64], w1 = cw[r * kCols * 4 + ct * 64 + 32];
          a0[ct][0] = weight(w0, z_lo[ct], s_lo[ct]);        // column g,     k 4 t4, 4 t4 + 1
          a0[ct][1] = weight(w1, z_hi[ct], s_hi[ct]);        // column g + 8
          a0[ct][2] = weight(w0 >> 8, z_lo[ct], s_lo[ct]);   // column g,     k 4 t4 + 2, 4 t4 + 3
          a0[ct][3] = weight(w1 >> 8, z_hi[ct], s_hi[ct]);
          a1[ct][0] = weight(w0 >> 4, z_lo[ct], s_lo[ct]);   // k 16 + 4 t4, 16 + 4 t4 + 1
          a1[ct][1] = weight(w1 >> 4, z_hi[ct], s_hi[ct]);
          a1[ct][2] = weight(w0 >> 12, z_lo[ct], s_lo[ct]);  // k 16 + 4 t4 + 2, 16 + 4 t4 + 3
          a1[ct][3] = weight(w1 >> 12, z_hi[ct], s_hi[ct]);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint2 b0 = *reinterpret_cast<const uint2 *>(xb + nt * 8 * kXRow + r * 64);
          const uint2 b1 = *reinterpret_cast<const uint2 *>(xb + nt * 8 * kXRow + r * 64 + 32);
#pragma unroll
          for (int ct = 0; ct < kTiles; ++ct) {
            mma_16816_nv<false>(acc[ct][nt], a0[ct], b0.x, b0.y);
            mma_16816_nv<false>(acc2[ct][nt], a1[ct], b1.x, b1.y);
          }
        }
        if (++run_in_group == rpg) {
          ++group;
          run_in_group = 0;
          if (group < g1) load_group(group);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
  }
#pragma unroll
  for (int ct = 0; ct < kTiles; ++ct)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[ct][nt][i] += acc2[ct][nt][i];
  // A wait that gave up raised the abort flag (and set the error word): the
  // CTA then leaves without output.
  csync();
  if (*abort_flag) return;

  // Fragment element i of (A tile ct, token tile nt): column c0 + 16 ct + g
  // (+ 8 for i >= 2), token 8 nt + 2 t4 (+ 1 for odd i).
  if (p.splits == 1) {
#pragma unroll
    for (int ct = 0; ct < kTiles; ++ct) {
      const int n_lo = tile * kCols + c0 + 16 * ct + g;
      const float b_lo = p.bias ? __half2float(__ushort_as_half(p.bias[n_lo])) : 0.f;
      const float b_hi = p.bias ? __half2float(__ushort_as_half(p.bias[n_lo + 8])) : 0.f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = nt * 8 + 2 * t4 + (i & 1);
          if (t < p.M)
            p.y[static_cast<size_t>(t) * p.N + n_lo + (i >> 1) * 8] =
                __half_as_ushort(__float2half_rn(acc[ct][nt][i] + (i < 2 ? b_lo : b_hi)));
        }
    }
    return;
  }
  float *part = p.partials + (static_cast<size_t>(tile) * p.splits + split) * p.M * kCols;
#pragma unroll
  for (int ct = 0; ct < kTiles; ++ct)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = nt * 8 + 2 * t4 + (i & 1);
        if (t < p.M) part[static_cast<size_t>(t) * kCols + c0 + 16 * ct + g + (i >> 1) * 8] = acc[ct][nt][i];
      }
  __shared__ int last_sm;
  __threadfence();
  csync();
  if (tid == 0) {
    const unsigned prev = atomicAdd(p.semaphores + tile, 1u);
    last_sm = prev == static_cast<unsigned>(p.splits - 1);
  }
  csync();
  if (!last_sm) return;
  __threadfence();
  // Last CTA of the tile: each thread sums up to two 4-column slots of the
  // [M][128] tile over the splits in split order, four splits' loads (of
  // both slots) in flight per round.
  const int slots = p.M * (kCols / 4);
  const float4 *tp = reinterpret_cast<const float4 *>(p.partials + static_cast<size_t>(tile) * p.splits * p.M * kCols);
  constexpr int kBatch = 4;
  for (int s0 = tid; s0 < slots; s0 += 2 * kCT) {
    const int s1 = s0 + kCT;
    const bool two = s1 < slots;
    float4 sum0 = make_float4(0.f, 0.f, 0.f, 0.f), sum1 = sum0;
    for (int sp0 = 0; sp0 < p.splits; sp0 += kBatch) {
      float4 v0[kBatch], v1[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const bool in = sp0 + j < p.splits;
        v0[j] = in ? __ldcg(tp + static_cast<size_t>(sp0 + j) * slots + s0) : make_float4(0.f, 0.f, 0.f, 0.f);
        v1[j] = in && two ? __ldcg(tp + static_cast<size_t>(sp0 + j) * slots + s1) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        if (sp0 + j < p.splits) {
          sum0.x += v0[j].x; sum0.y += v0[j].y; sum0.z += v0[j].z; sum0.w += v0[j].w;
          sum1.x += v1[j].x; sum1.y += v1[j].y; sum1.z += v1[j].z; sum1.w += v1[j].w;
        }
      }
    }
    auto store4 = [&](int sl, const float4 &v) {
      const int t = sl / (kCols / 4), c = tile * kCols + (sl % (kCols / 4)) * 4;
      const float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float b = p.bias ? __half2float(__ushort_as_half(p.bias[c + j])) : 0.f;
        p.y[static_cast<size_t>(t) * p.N + c + j] = __half_as_ushort(__float2half_rn(o[j] + b));
      }
    };
    store4(s0, sum0);
    if (two) store4(s1, sum1);
  }
  if (tid == 0) p.semaphores[tile] = 0u;  // ready for the next call
}

}  // namespace awqm
}  // namespace lvb
