// AutoAWQ W4A16 linear on sm_100a with the dequantised weight written
// straight into tensor memory, over the packed weight layout.
//
// y[m, n] = sum_k x[m, k] * W[k, n] (+ bias[n]),  W[k, n] = fp16(q - z) * s.
//
// The weight is the UMMA "A" operand (M = 128 output columns per CTA) and the
// activations are "B" (N = BN tokens).  A never goes through shared memory:
// every dequantiser thread owns one output column (one TMEM lane), turns 32 of
// its int4 codes into fp16 in registers and stores them with tcgen05.st into
// an A stage in tensor memory; tcgen05.mma then reads A from tensor memory and
// B from shared memory.  Shared memory only carries the streamed int4 codes
// (0.5 byte per weight) and the activation tiles.
//
// Weights are read in the packed layout written once by the pack kernels below
// (column-major int4 runs, 16 bytes = 32 k of one column, 2 KB per 128-column
// x 32-k chunk) so that one contiguous bulk copy fetches a stage and a
// thread's 16 bytes hold exactly the codes its TMEM lane needs.  Within a
// 16-byte run, word w holds k = 4w..4w+3 in nibbles (0, 4, 2, 6) and
// k = 16+4w..16+4w+3 in nibbles (1, 5, 3, 7).  Masking a word with 0x000F000F
// and OR-ing 0x6400 gives the half2 of 1024 + q for (k, k+1); differences with
// the zero point in the same biased form are the exact integers q - z, and one
// fp16 multiply by the scale rounds like the reference's dequantised weight
// (modeling/quantization/awq.py:433-450).  With DUAL, the upper 16 k of a run
// come from the mask 0x00F000F0 as 1024 + 16 q, i.e. 16 (q - z) * s = exactly
// 16 W (|scale| < 273); they accumulate into a second TMEM accumulator (K = 16
// per MMA, so every MMA reads one half only) and the epilogue forms
// D_lo + D_hi / 16 in fp32.  Without DUAL (large N, where the two
// accumulators would not fit next to the A stages) the upper half is shifted
// down first and a single accumulator holds exact W products.
//
// Roles (one CTA per SM):
//   warp 0        bulk copies of the packed codes, one per stage
//   warp 1        activation tile (TMA, 64-byte swizzle, zero fill past m and
//                 k), the stage's (scale, zero) rows and their row table
//   warp 2        TMEM allocator and the single thread issuing tcgen05.mma
//   warps 3..     DG warpgroups of dequantisers; warpgroup w handles the 64-k
//                 blocks w, w + DG, ... of every stage into one of the TMEM A
//                 stages; the first warpgroup also runs the epilogue.
// Grid: (m tiles, column tiles, K splits), m tiles fastest.  Small grids split
// K across CTAs; partial fp32 tiles are summed in split order by the last CTA
// of a tile, so results are deterministic.
#pragma once

#include "lvb_common.cuh"

namespace lvb {
namespace awqd {

constexpr int kTileN = 128;                       // output columns per CTA (UMMA M)
constexpr int kChunkK = 32;                       // k per packed run (16 bytes per column)
constexpr int kChunkBytes = kTileN * 16;          // 2048
constexpr int kBlockK = 64;                       // k per dequantiser work unit
constexpr int kSzRowBytes = kTileN * 4;           // (scale, zero) words of one group
constexpr int kFirstDqWarp = 3;
constexpr int kEpilogueThreads = 128;             // the first dequantiser warpgroup
constexpr int kTmemCols = 512;
constexpr int kSmemBudget = 216 * 1024;

// BN: token rows per CTA (UMMA N).  SB: 64-k blocks per pipeline stage.  DG:
// dequantiser warpgroups (warpgroup w takes blocks w, w + DG, ... of a stage).
// DUAL: the upper 16 k of every 32-k run are dequantised as 16 W and
// accumulate into a second accumulator (one instruction less per code pair);
// otherwise one accumulator and exact W throughout.  TMEM / SMEM_KB: the
// tensor-memory columns and shared-memory bytes one CTA takes (half of each
// lets two CTAs share an SM).
template <int BN, int SB, int DG, bool DUAL, int TMEM = kTmemCols, int SMEM_KB = kSmemBudget / 1024>
struct PackedConfig {
  static constexpr int kTmemAlloc = TMEM;
  static constexpr int kCtasPerSm = TMEM == kTmemCols ? 1 : 2;
  static constexpr int kStageChunks = 2 * SB;
  static constexpr int kQStageBytes = kStageChunks * kChunkBytes;
  static constexpr int kSzStageBytes = kStageChunks * kSzRowBytes;  // at most one group per chunk
  static constexpr int kXChunkBytes = BN * 64;                       // BN rows x 32 k (64-byte swizzle)
  static constexpr int kXBytes = kStageChunks * kXChunkBytes;        // TMA box bytes per stage
  static constexpr int kXOff = 0;
  static constexpr int kQOff = kXBytes;
  static constexpr int kSzOff = kQOff + kQStageBytes;
  static constexpr int kStageBytes = ((kSzOff + kSzStageBytes) + 1023) / 1024 * 1024;
  static constexpr int kStages = SMEM_KB * 1024 / kStageBytes > 8 ? 8 : SMEM_KB * 1024 / kStageBytes;
  // Tensor memory: D_lo [0, BN), D_hi [BN, 2 BN) when DUAL, then the A stages.
  static constexpr int kDHiCol = BN;
  static constexpr int kACol = ((DUAL ? 2 * BN : BN) + 31) / 32 * 32;
  static constexpr int kAStageCols = SB * 32;
  static constexpr int kAStages = (TMEM - kACol) / kAStageCols > 4 ? 4 : (TMEM - kACol) / kAStageCols;
  static constexpr int kBlocksPerGroup = SB / DG;
  static constexpr int kDqWarps = 4 * DG;
  static constexpr int kThreads = (kFirstDqWarp + kDqWarps) * 32;
  static constexpr int kBarOff = kStages * kStageBytes;
  // full, empty (per stage), a_full, a_empty (per A stage), acc_full.
  static constexpr int kNumBars = 2 * kStages + 2 * kAStages + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  // Per stage slot: the (scale, zero) row of each chunk, one byte each,
  // written by the producer so that dequantisers need no division.
  static constexpr int kRowTableOff = kMiscOff + 64;
  static constexpr int kSmemBytes = kRowTableOff + kStages * 8 + 1024;  // + base alignment slack
  static_assert(SB % DG == 0 && kStageChunks <= 8, "stage blocks per warpgroup");
  static_assert(kStages >= 3, "pipeline depth");
  static_assert(kAStages >= 2, "tensor-memory A stages");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(BN % 16 == 0 && BN <= 256, "UMMA N for M = 128");
};

struct DecodeParams {
  const uint8_t *qpack;    // [n_tiles][k_chunks][128][16 B]
  const uint32_t *szpack;  // [n_tiles][groups][128] (scale bits | zero << 16)
  const uint16_t *bias;    // may be null
  uint16_t *y;
  uint32_t *semaphores;    // per output tile, zero between calls
  float *partials;         // [tiles][splits][BN][128] when splits > 1
  int M, K, N, G;
  int groups;
  int k_chunks;            // packed chunks per column tile (K rounded up to 64, / 32)
  int k_blocks;            // k_chunks / 2
  int n_tiles, m_tiles, splits;
};

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The four MMAs of one 64-k block in one asm statement (no instructions
// between them): runs c = 0, 1 of the block, each as its lower 16 k into D_lo
// and its upper 16 k into D_hi (DUAL) or D_lo.  `acc_first` = 0 starts the
// accumulators on the block's first MMAs.
template <bool DUAL>
__device__ __forceinline__ void umma_ts_block(uint32_t d_lo, uint32_t d_hi, uint32_t a, uint64_t b0, uint64_t b1,
                                              uint64_t b2, uint64_t b3, uint32_t idesc, uint32_t acc_first) {
  const uint32_t a1 = a + 8, a2 = a + 16, a3 = a + 24;
  if constexpr (DUAL) {
    asm volatile(
        "{\n\t.reg .pred pf, pt;\n\t"
        "setp.ne.b32 pf, %8, 0;\n\t"
        "setp.eq.b32 pt, %8, %8;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %4, %9, pf;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [%3], %5, %9, pf;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%10], %6, %9, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [%11], %7, %9, pt;\n\t}" ::"r"(d_lo),
        "r"(d_hi), "r"(a), "r"(a1), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(acc_first), "r"(idesc), "r"(a2),
        "r"(a3)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred pf, pt;\n\t"
        "setp.ne.b32 pf, %8, 0;\n\t"
        "setp.eq.b32 pt, %8, %8;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %4, %9, pf;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %5, %9, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%10], %6, %9, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%11], %7, %9, pt;\n\t}" ::"r"(d_lo),
        "r"(d_hi), "r"(a), "r"(a1), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(acc_first), "r"(idesc), "r"(a2),
        "r"(a3)
        : "memory");
  }
}

// K-major SWIZZLE_64B operand: rows of 64 bytes, 8-row groups 512 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_kmajor_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;             // leading byte offset (unused, 16 B)
  d |= static_cast<uint64_t>(512 >> 4) << 32;      // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;             // descriptor version (sm_100)
  d |= static_cast<uint64_t>(4) << 61;             // layout: SWIZZLE_64B
  return d;
}

// 32 lanes x 32 columns of 32-bit words from this thread's registers.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t hsub_hmul(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b)),
                      *reinterpret_cast<__half2 *>(&c));
  return *reinterpret_cast<uint32_t *>(&r);
}

// Dequantise one 16-byte run (32 k of one column) into 16 half2 words in k
// order: out[0..7] = W for k 0..15, out[8..15] = k 16..31, as W (exact) or,
// when DUAL, as 16 W (exact multiple of W for |scale| < 273).
template <bool DUAL>
__device__ __forceinline__ void dequant_run(const uint4 q, uint32_t sz, uint32_t *out) {
  const uint32_t s2 = __byte_perm(sz, 0, 0x1010);  // (scale, scale)
  const uint32_t z = sz >> 16;
  const uint32_t zz = z | (z << 16);
  const uint32_t zlo = zz | 0x64006400u;         // 1024 + z
  const uint32_t zhi = (zz << 4) | 0x64006400u;  // 1024 + 16 z
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w8 = w[i] >> 8;
    out[2 * i] = hsub_hmul((w[i] & 0x000F000Fu) | 0x64006400u, zlo, s2);
    out[2 * i + 1] = hsub_hmul((w8 & 0x000F000Fu) | 0x64006400u, zlo, s2);
    if constexpr (DUAL) {
      out[8 + 2 * i] = hsub_hmul((w[i] & 0x00F000F0u) | 0x64006400u, zhi, s2);
      out[8 + 2 * i + 1] = hsub_hmul((w8 & 0x00F000F0u) | 0x64006400u, zhi, s2);
    } else {
      out[8 + 2 * i] = hsub_hmul(((w[i] >> 4) & 0x000F000Fu) | 0x64006400u, zlo, s2);
      out[8 + 2 * i + 1] = hsub_hmul(((w[i] >> 12) & 0x000F000Fu) | 0x64006400u, zlo, s2);
    }
  }
}

template <int BN, int SB, int DG, bool DUAL, int TMEM = kTmemCols, int SMEM_KB = kSmemBudget / 1024>
__global__ void __launch_bounds__(PackedConfig<BN, SB, DG, DUAL, TMEM, SMEM_KB>::kThreads,
                                  PackedConfig<BN, SB, DG, DUAL, TMEM, SMEM_KB>::kCtasPerSm)
    awq_packed_kernel(const __grid_constant__ CUtensorMap xmap, const DecodeParams p) {
  pdl_entry();
  using C = PackedConfig<BN, SB, DG, DUAL, TMEM, SMEM_KB>;
  constexpr int kAStages = C::kAStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *full = bars;
  uint64_t *empty = full + C::kStages;
  uint64_t *a_full = empty + C::kStages;
  uint64_t *a_empty = a_full + kAStages;
  uint64_t *acc_full = a_empty + kAStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 8);
  volatile int *last_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 16);
  uint32_t *row_table = reinterpret_cast<uint32_t *>(smem + C::kRowTableOff);  // [kStages][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // m tiles vary fastest across the grid, so the CTAs sharing a column tile
  // of weights run together and read it from HBM once.
  const int m_tile = blockIdx.x;
  const int tile = blockIdx.y;
  const int split = blockIdx.z;
  const int tile_id = tile * p.m_tiles + m_tile;
  const int b_begin = static_cast<int>((static_cast<long long>(split) * p.k_blocks) / p.splits);
  const int b_end = static_cast<int>((static_cast<long long>(split + 1) * p.k_blocks) / p.splits);
  const int nblocks = b_end - b_begin;
  const int nstages = (nblocks + SB - 1) / SB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], C::kDqWarps + 1);
    }
    for (int j = 0; j < kAStages; ++j) {
      mbar_init(&a_full[j], C::kDqWarps);
      mbar_init(&a_empty[j], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::kTmemAlloc);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || warp == 1) {
    // ---------------- producers ----------------
    if (lane == 0) {
      bool ok = true;
      int issued = 0;
      for (int ls = 0; ls < nstages; ++ls) {
        const int slot = ls % C::kStages;
        if (ls >= C::kStages && !mbar_wait(&empty[slot], ((ls / C::kStages) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t *stage = smem + slot * C::kStageBytes;
        const int blk0 = b_begin + ls * SB;
        const int nb = min(SB, b_end - blk0);
        const int chunk0 = 2 * blk0;
        if (warp == 0) {
          const uint32_t bytes = static_cast<uint32_t>(2 * nb * kChunkBytes);
          mbar_arrive_expect_tx(&full[slot], bytes);
          bulk_load(stage + C::kQOff,
                    p.qpack + (static_cast<size_t>(tile) * p.k_chunks + chunk0) * kChunkBytes, bytes,
                    &full[slot]);
        } else {
          const int k_first = chunk0 * kChunkK;
          const int k_last = min((chunk0 + 2 * nb) * kChunkK, p.K) - 1;
          const int g_first = min(k_first / p.G, p.groups - 1);
          const int g_last = min(k_last / p.G, p.groups - 1);
          const uint32_t sz_bytes = static_cast<uint32_t>((g_last - g_first + 1) * kSzRowBytes);
          uint32_t rows[2] = {0u, 0u};
          for (int cl = 0; cl < C::kStageChunks; ++cl) {
            const int g = min((chunk0 + cl) * kChunkK / p.G, p.groups - 1) - g_first;
            rows[cl >> 2] |= static_cast<uint32_t>(g) << (8 * (cl & 3));
          }
          // Plain stores, published to the dequantisers by the arrive below.
          row_table[2 * slot] = rows[0];
          row_table[2 * slot + 1] = rows[1];
          mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(C::kXBytes) + sz_bytes);
          tma_load_3d(stage + C::kXOff, &xmap, &full[slot], 0, m_tile * BN, chunk0);
          bulk_load(stage + C::kSzOff,
                    p.szpack + (static_cast<size_t>(tile) * p.groups + g_first) * kTileN, sz_bytes,
                    &full[slot]);
        }
        issued = ls + 1;
      }
      if (!ok) {
        // Let the copies already issued land before the CTA's memory goes away.
        for (int ls = issued > C::kStages ? issued - C::kStages : 0; ls < issued; ++ls)
          mbar_wait(&full[ls % C::kStages], (ls / C::kStages) & 1, nullptr, kDrainBudgetCycles);
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ---------------- tcgen05.mma issuer ----------------
    // Every dequantiser warp arrives once per stage, so one wait covers the
    // stage and its MMAs issue back to back: a tcgen05.mma with N <= 128
    // occupies the tensor pipe for a fixed ~70 cycles, so per-block waits
    // between them would cost more than the MMAs.
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(kTileN, BN, 0, 0, 0, 0);
      bool ok = true;
      for (int ls = 0; ls < nstages && ok; ++ls) {
        const int slot = ls % C::kStages;
        if (!mbar_wait(&full[slot], (ls / C::kStages) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const int nb = min(SB, nblocks - ls * SB);
        const int as = ls % kAStages;
        // Descriptors and addresses of the whole stage are formed before the
        // MMAs: tcgen05.mma holds the issuing thread until the pipe accepts it,
        // so any arithmetic between two MMAs shows up as a gap in the pipe.
        // The start-address field of a descriptor (bits 0..13, address / 16)
        // does not overflow for shared-memory offsets, so descriptors of the
        // stage's tiles differ from the first by (offset / 16).
        const uint64_t bdesc0 = umma_desc_kmajor_sw64(smem_u32(smem + slot * C::kStageBytes + C::kXOff));
        const uint32_t a0 = tmem + C::kACol + as * C::kAStageCols;
        const uint32_t acc0 = ls == 0 ? 0u : 1u;
        // Descriptors of the stage's four B sub-tiles per block: (run c, half h)
        // at (2 b + c) * kXChunkBytes + 32 h.
        uint64_t bd[SB][4];
#pragma unroll
        for (int b = 0; b < SB; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            bd[b][i] = bdesc0 + static_cast<uint64_t>(((2 * b + (i >> 1)) * C::kXChunkBytes + (i & 1) * 32) >> 4);
        if (!mbar_wait(&a_full[as], (ls / kAStages) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int b = 0; b < SB; ++b) {
          if (b < nb)
            umma_ts_block<DUAL>(tmem, tmem + C::kDHiCol, a0 + b * 32, bd[b][0], bd[b][1], bd[b][2], bd[b][3], idesc,
                                b == 0 ? acc0 : 1u);
        }
        umma_commit(&a_empty[as]);
        umma_commit(&empty[slot]);
      }
      umma_commit(acc_full);
      if (!ok) mbar_wait(acc_full, 0, nullptr, kDrainBudgetCycles);
    }
    __syncwarp();
  } else {
    // ---------------- dequantisers ----------------
    const int dw = warp - kFirstDqWarp;
    const int wg = dw >> 2;          // first 64-k block of each stage handled by this warpgroup
    const int quad = warp & 3;       // TMEM lane quadrant this warp may access
    const int col = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    bool ok = true;
    for (int ls = 0; ls < nstages; ++ls) {
      const int slot = ls % C::kStages;
      const int nb = min(SB, nblocks - ls * SB);
      if (!__all_sync(0xffffffffu, mbar_wait(&full[slot], (ls / C::kStages) & 1, abort_flag))) {
        ok = false;
        break;
      }
      const uint8_t *stage = smem + slot * C::kStageBytes;
      const uint32_t rows_lo = row_table[2 * slot];
      const uint32_t rows_hi = row_table[2 * slot + 1];
      uint4 q[C::kBlocksPerGroup][2];
      uint32_t sz[C::kBlocksPerGroup][2];
#pragma unroll
      for (int bi = 0; bi < C::kBlocksPerGroup; ++bi) {
        const int b = wg + bi * DG;
        if (b < nb) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int cl = 2 * b + c;
            q[bi][c] = *reinterpret_cast<const uint4 *>(stage + C::kQOff + cl * kChunkBytes + col * 16);
            const uint32_t g = ((cl < 4 ? rows_lo : rows_hi) >> (8 * (cl & 3))) & 0xFFu;
            sz[bi][c] = *reinterpret_cast<const uint32_t *>(stage + C::kSzOff + g * kSzRowBytes + col * 4);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      uint32_t a[C::kBlocksPerGroup][32];
#pragma unroll
      for (int bi = 0; bi < C::kBlocksPerGroup; ++bi) {
        if (wg + bi * DG < nb) {
          dequant_run<DUAL>(q[bi][0], sz[bi][0], a[bi]);
          dequant_run<DUAL>(q[bi][1], sz[bi][1], a[bi] + 16);
        }
      }
      const int as = ls % kAStages;
      if (ls >= kAStages &&
          !__all_sync(0xffffffffu, mbar_wait(&a_empty[as], ((ls / kAStages) - 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int bi = 0; bi < C::kBlocksPerGroup; ++bi) {
        const int b = wg + bi * DG;
        if (b < nb) tmem_st_32x32b_x32(tmem + lane_base + C::kACol + as * C::kAStageCols + b * 32, a[bi]);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[as]);
    }

    // ---------------- epilogue (first warpgroup) ----------------
    if (wg == 0) {
      if (ok && nblocks > 0) ok = mbar_wait(acc_full, 0, abort_flag);
      ok = __all_sync(0xffffffffu, ok) && nblocks > 0;
      tc_fence_after();
      const int n = tile * kTileN + col;
      const int m0 = m_tile * BN;
      const bool n_ok = n < p.N;
      const float bias_n = (p.bias != nullptr && n_ok) ? __half2float(__ushort_as_half(p.bias[n])) : 0.f;
      float *part = p.partials + static_cast<size_t>(tile_id) * p.splits * BN * kTileN;
      if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 8) {
          float lo[8], hi[8];
          tmem_ld_32x32b_x8(tmem + lane_base + c0, lo);
          if constexpr (DUAL) tmem_ld_32x32b_x8(tmem + lane_base + C::kDHiCol + c0, hi);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float v = DUAL ? fmaf(hi[c], 0.0625f, lo[c]) : lo[c];
            const int m = c0 + c;
            if (p.splits == 1) {
              if (n_ok && m0 + m < p.M)
                p.y[static_cast<size_t>(m0 + m) * p.N + n] = __half_as_ushort(__float2half_rn(v + bias_n));
            } else {
              __stcg(part + (static_cast<size_t>(split) * BN + m) * kTileN + col, v);
            }
          }
        }
      }
      if (p.splits > 1) {
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"n"(kEpilogueThreads) : "memory");
        if (dw == 0 && lane == 0) {
          const unsigned int prev = ok ? atomicAdd(p.semaphores + tile_id, 1u) : 0u;
          *last_flag = (ok && prev == static_cast<unsigned int>(p.splits - 1)) ? 1 : 0;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kEpilogueThreads) : "memory");
        if (*last_flag) {
          __threadfence();
          // Sum the splits in order, 16 rows at a time; the loads of one split
          // are independent of each other.
#pragma unroll 1
          for (int r0 = 0; r0 < BN; r0 += 16) {
            float sum[16];
#pragma unroll
            for (int m = 0; m < 16; ++m) sum[m] = 0.f;
            for (int s = 0; s < p.splits; ++s) {
              float v[16];
#pragma unroll
              for (int m = 0; m < 16; ++m) v[m] = __ldcg(part + (static_cast<size_t>(s) * BN + r0 + m) * kTileN + col);
#pragma unroll
              for (int m = 0; m < 16; ++m) sum[m] += v[m];
            }
            if (n_ok) {
#pragma unroll
              for (int m = 0; m < 16; ++m)
                if (m0 + r0 + m < p.M)
                  p.y[static_cast<size_t>(m0 + r0 + m) * p.N + n] = __half_as_ushort(__float2half_rn(sum[m] + bias_n));
            }
          }
          if (dw == 0 && lane == 0) p.semaphores[tile_id] = 0u;
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemAlloc);
  }
}

// ------------------------------------------------------------------------
// One-time repacking of an AutoAWQ checkpoint into the decode layout.
// ------------------------------------------------------------------------
// AutoAWQ nibble p of a packed word holds column 8j + (0,2,4,6,1,3,5,7)[p];
// the nibble that holds column offset c is kAwqNibbleOf[c].
__device__ __constant__ const int kAwqNibbleOf[8] = {0, 4, 1, 5, 2, 6, 3, 7};

__device__ __forceinline__ uint32_t awq_code(const int32_t *packed, int64_t row, int64_t words, int n) {
  const uint32_t w = static_cast<uint32_t>(packed[row * words + (n >> 3)]);
  return (w >> (4 * kAwqNibbleOf[n & 7])) & 0xFu;
}

// One thread per (column tile, chunk, column): 16 bytes of packed codes.
__global__ void awq_pack_codes_kernel(const int32_t *__restrict__ qweight, uint8_t *__restrict__ qpack, int K,
                                      int N, int k_chunks, int n_tiles) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(n_tiles) * k_chunks * kTileN;
  if (idx >= total) return;
  const int col = static_cast<int>(idx % kTileN);
  const int64_t rest = idx / kTileN;
  const int chunk = static_cast<int>(rest % k_chunks);
  const int tile = static_cast<int>(rest / k_chunks);
  const int n = tile * kTileN + col;
  const int64_t words = N / 8;
  uint32_t out[4] = {0, 0, 0, 0};
  if (n < N) {
    // Nibble slots of word i: k = 4i + (0, 2) at nibbles (0, 2), 4i + (1, 3)
    // at (4, 6); k = 16 + 4i + (0, 2) at (1, 3), 16 + 4i + (1, 3) at (5, 7).
    constexpr int kSlot[4] = {0, 4, 2, 6};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k_lo = chunk * kChunkK + 4 * i + e;
        const int k_hi = k_lo + 16;
        if (k_lo < K) w |= awq_code(qweight, k_lo, words, n) << (4 * kSlot[e]);
        if (k_hi < K) w |= awq_code(qweight, k_hi, words, n) << (4 * (kSlot[e] + 1));
      }
      out[i] = w;
    }
  }
  *reinterpret_cast<uint4 *>(qpack + idx * 16) = make_uint4(out[0], out[1], out[2], out[3]);
}

// One thread per (column tile, group, column): scale bits | zero << 16.
__global__ void awq_pack_groups_kernel(const int32_t *__restrict__ qzeros, const uint16_t *__restrict__ scales,
                                       uint32_t *__restrict__ szpack, int N, int groups, int n_tiles) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(n_tiles) * groups * kTileN;
  if (idx >= total) return;
  const int col = static_cast<int>(idx % kTileN);
  const int64_t rest = idx / kTileN;
  const int g = static_cast<int>(rest % groups);
  const int tile = static_cast<int>(rest / groups);
  const int n = tile * kTileN + col;
  uint32_t v = 0;
  if (n < N) v = static_cast<uint32_t>(scales[static_cast<int64_t>(g) * N + n]) | (awq_code(qzeros, g, N / 8, n) << 16);
  szpack[idx] = v;
}

}  // namespace awqd
}  // namespace lvb
