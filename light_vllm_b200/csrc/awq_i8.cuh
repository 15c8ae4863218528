// AutoAWQ W4A16 linear for decode batches (m <= 16) on the int8 tensor-core
// path: twice the weights per tcgen05.mma of the fp16 path.
//
// y[t, n] = sum_k x[t, k] * (q[k, n] - z[g, n]) * s[g, n]   (g = k / G)
//         = sum_g s[g, n] * (sum_{k in g} q x  -  z[g, n] * sum_{k in g} x).
//
// A tcgen05.mma with M = 128 occupies the tensor pipe for a fixed ~70 cycles
// at small N whatever its kind; with kind::f16 it retires 128 x 16 weights,
// with kind::i8 128 x 32.  So here the weight operand is the raw int4 code q
// as an int8 (exact), written into tensor memory by the dequantisers with two
// logic operations per 8 codes, and the activations enter as four int8
// "limbs": per (token, group) a power-of-two scale a with |x / a| <= 127, and
//     x / a = x0 + x1 / 128 + x2 / 128^2 + x3 / 128^3,
//     x0 = rint(x / a) in [-127, 127], each later limb the rounded residual
//     times 128, in [-64, 64]
// (every residual is exact in fp32).  Relative to the group's largest
// element a, this keeps 29 significant bits: every fp16 value within a
// factor 2^17 of the group's largest is represented exactly, so a group that
// mixes an activation outlier of 10^4 with N(0, 1) values keeps the small
// values' precision (with two limbs they lost it all).  The four limbs are
// four row blocks of the MMA's B operand (N = 4 x 16 = 64), so they cost no
// extra MMA: its time is the same for every N <= 128.  The MMA accumulates,
// exactly in int32, D_l = sum q x_l over one group; the drain warps form
//     v_hi = 128 D0 + D1 - z * sum_k (128 x0 + x1),
//     v_lo = 128 D2 + D3 - z * sum_k (128 x2 + x3)          (exact integers)
// and add s * (a / 128) * (v_hi + v_lo / 128^2) to an fp32 accumulator.  The
// only roundings are the fp32 conversion and accumulation (the limbs are
// exact for the inputs above); the zero point and the scale are applied
// exactly (the reference rounds W to fp16 instead,
// modeling/quantization/awq.py:433-450).
//
// Kernels:
//   awq_act_limbs_kernel  one CTA per group, one warp per token row: the
//                         limbs of x, in the K-major 64-byte-swizzled tile
//                         layout the MMA reads (pre-swizzled, so a stage is
//                         one bulk copy), per (group, token) the scale a / 128
//                         and the integer sums of 128 x0 + x1 and 128 x2 + x3,
//                         and per group whether any token needs limbs 2-3.
//                         Stages whose groups need only limbs 0-1 (ordinary
//                         activations) copy half the limb tile, issue N = 32
//                         MMAs and drain two accumulators per group.
//   awq_i8_kernel<BN>     persistent, one CTA per SM over (128-column tile,
//                         K split) units; launched as a programmatic
//                         dependent of the limb kernel so that its set-up and
//                         code streaming overlap it:
//     warp 0      bulk copies of the packed codes (16 KB per 256-k stage)
//     warp 1      bulk copies of the limb tiles (limbs 0-1, and 2-3 when the
//                 stage needs them: 2 BN rows x 256 k each)
//     warp 2      TMEM allocation and the tcgen05.mma.kind::i8 issuer of
//                 even stages; warp 11 issues the odd stages
//     warps 3..6  code expanders: q nibbles -> int8 A columns in TMEM
//     warps 7..10 drain: per group, int32 D -> fp32 accumulators; epilogue
// Accumulators: a ring of four TMEM slots of one limb pair (N = 32) for two
// groups each; a stage takes one slot (limbs 0-1), or two when it needs limbs
// 2-3, which run as separate N = 32 MMAs over the upper half of each limb
// chunk into the second slot.
// The codes use the packed layout of awq_decode.cuh.  Within a 32-k run, word
// w masked with 0x0F0F0F0F gives the bytes of k = 4w, 4w+2, 4w+1, 4w+3, and
// the word shifted right by 4 those of k = 16+4w, 16+4w+2, 16+4w+1, 16+4w+3;
// the limb tiles store x in the same k order, so A and B agree without any
// byte shuffling.
#pragma once

#include "awq_decode.cuh"
#include "lvb_common.cuh"

namespace lvb {
namespace awqi8 {

using awqd::kChunkBytes;
using awqd::kTileN;

constexpr int kStageBlocks = 4;                       // 64-k blocks per stage
constexpr int kStageChunks = 2 * kStageBlocks;        // 32-k runs per stage
constexpr int kQStageBytes = kStageChunks * kChunkBytes;  // 16 KB of codes
constexpr int kStages = 4;                            // stages in flight (shared memory and TMEM A)
constexpr int kAStageCols = kStageBlocks * 16;        // 16 columns (64 int8) per block
constexpr int kExpandWarp = 3;                        // first code-expander warp
constexpr int kDrainWarp = 7;                         // first drain warp
constexpr int kIssuer2Warp = 11;                      // second MMA issuer (odd stages)
constexpr int kThreads = 12 * 32;
constexpr int kTmemCols = 512;
constexpr int kLimbs = 4;                             // int8 limbs per activation
constexpr int kMaxFlagGroups = 2048;                  // groups whose flags are staged in shared memory

// x / a (exact in fp32: a power-of-two scaling of an fp16 value) into
// kLimbs int8 limbs, x / a = sum_i l[i] / 128^i; each residual is exact.
__device__ __forceinline__ void split_limbs(float r, int (&l)[kLimbs]) {
#pragma unroll
  for (int i = 0; i < kLimbs; ++i) {
    const float li = rintf(r);
    l[i] = static_cast<int>(li);
    r = (r - li) * 128.f;
  }
}

// Whether a (token, group) needs all four limbs.  Two limbs keep 15 bits
// relative to the group's largest element |x|max, an absolute rounding of at
// most |x|max 2^-15 per element.  That is negligible against the group's
// contribution unless the group's typical elements are much smaller than its
// largest -- a massive activation (10^3-10^4 x the rest, as real Qwen2
// checkpoints have in a few channels) beside ordinary values.  The test is
// robust to a few such outliers: when fewer than G / 8 elements exceed
// |x|max / 16, the bulk of the group is small next to |x|max and all four limbs
// are used; otherwise (Gaussian-like groups: ~85 % of elements exceed a
// sixteenth of the maximum) the last two limbs are skipped.
__device__ __forceinline__ int large_count(const float (&v)[4], float amax) {
  const float cut = amax * 0.0625f;
  return (fabsf(v[0]) > cut) + (fabsf(v[1]) > cut) + (fabsf(v[2]) > cut) + (fabsf(v[3]) > cut);
}

__device__ __forceinline__ int needs_four_limbs(int large, int G) { return large * 8 < G ? 1 : 0; }

// Power-of-two exponent e of the limb scale a = 2^e: the smallest a with
// amax / a <= 127 (a = 1 for an all-zero group).
__device__ __forceinline__ int limb_exponent(float amax) {
  int e = 0;
  if (amax > 0.f) frexpf(amax / 127.f, &e);
  return e;
}

// Groups of 128 or 256 k: a 256-k stage holds two groups or one, and the
// MMA issuer, code expanders and drain synchronise once per stage.
template <int BN>
struct I8Config {
  // Accumulator slots: a ring of four, each holding limbs 0-1 (N = 2 BN
  // columns) of up to two groups.  A stage takes one slot, or two when it
  // needs limbs 2-3 (the second slot holds those), so the drain of a stage
  // overlaps the MMAs of the next several.
  static constexpr int kDStages = 4;
  static constexpr int kLimbRows = kLimbs * BN;              // (limb, token) rows of B
  static constexpr int kLimbChunkBytes = kLimbRows * 64;     // the four limbs of one 64-k chunk
  static constexpr int kPairChunkBytes = 2 * BN * 64;        // one limb pair of one 64-k chunk (2 BN rows)
  static constexpr int kPairStageStride = kStageBlocks * kPairChunkBytes;  // limbs 2-3 of a stage in shared memory
  static constexpr int kLimbStageBytes = kStageBlocks * kLimbChunkBytes;
  static constexpr int kQOff = kLimbStageBytes;              // limb tile first (1024-aligned)
  static constexpr int kStageBytes = ((kQOff + kQStageBytes) + 1023) / 1024 * 1024;
  static constexpr int kGroupCols = 2 * BN;                  // int32 accumulator columns per group and limb pair
  static constexpr int kDStageCols = 2 * kGroupCols;         // one slot: up to two groups
  static constexpr int kACol = kDStages * kDStageCols;
  static constexpr int kBarOff = kStages * kStageBytes;
  // full, done, a_full (stages), d_full, d_empty (stage accumulators), fin (per issuer).
  // + flags: the per-group four-limb flags are in shared memory.
  static constexpr int kNumBars = 3 * kStages + 2 * kDStages + 2 + 1;
  static_assert((kDStages & (kDStages - 1)) == 0, "power-of-two accumulator ring");
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  // Per drain warp, two stage slots of per-token scalars (2 groups x BN x 16 bytes).
  static constexpr int kScalOff = (kMiscOff + 64 + 15) / 16 * 16;
  static constexpr int kScalSlotBytes = 2 * BN * 16;
  static constexpr int kScalBytes = 4 * 2 * kScalSlotBytes;
  // Output tile [BN tokens][128 columns] fp16, written to y by one TMA store.
  static constexpr int kYOff = (kScalOff + kScalBytes + 127) / 128 * 128;
  static constexpr int kYBytes = BN * kTileN * 2;
  // Four-limb flag of every group (one byte each), staged once per CTA.
  static constexpr int kFlagOff = kYOff + kYBytes;
  static constexpr int kSmemBytes = kFlagOff + kMaxFlagGroups + 1024;
  static_assert(BN == 16, "int8 path covers 16-row token tiles (N = 4 limbs x 16 rows)");
  static_assert(kACol + kStages * kAStageCols <= kTmemCols, "tensor memory budget");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct I8Params {
  const uint8_t *qpack;      // packed codes [n_tiles][k_chunks][128][16 B]
  const uint32_t *szpack;    // [n_tiles][groups][128] (scale bits | zero << 16)
  const int8_t *limbs;       // [2 limb pairs][K/64][2 BN][64 B], pre-swizzled
  const int4 *scal;          // [groups][BN]: (bits of a / 128, sum of 128 x0 + x1, sum of 128 x2 + x3, four)
  const int *four;           // [groups]: the group's stages use limbs 2 and 3
  const uint16_t *bias;      // may be null
  uint16_t *y;
  uint32_t *semaphores;
  float *partials;           // [n_tiles][splits][BN][128]
  int M, K, N, G;
  int groups, k_chunks, blocks_per_group, bpg_shift;  // blocks per group = 1 << bpg_shift (2 or 4)
  int n_tiles, splits;
};

// Byte offset of k within its 64-k chunk row, in the A column order of the
// code expanders: inside each 4-k quad the order is (0, 2, 1, 3).
__host__ __device__ __forceinline__ int limb_pos(int k64) {
  const int e = k64 & 3;
  return (k64 & ~3) | ((e & 1) << 1) | (e >> 1);
}

// 64-byte swizzle of a K-major tile: 16-byte chunk c of row r lands at
// chunk c ^ ((r >> 1) & 3).
__host__ __device__ __forceinline__ int sw64(int row, int byte) {
  return row * 64 + ((((byte >> 4) ^ ((row >> 1) & 3)) & 3) << 4) + (byte & 15);
}

// One CTA per group, one warp per token row t < BN; rows t >= M are written
// as zeros.  Each lane handles 4 consecutive k (one quad) per pass and stores
// the quad's limbs as one 32-bit word per limb, bytes in the (0, 2, 1, 3)
// order; limb l of token t is row l * BN + t of the tile.  x rows are
// x_stride elements apart.  gated: x holds merged [gate | up] rows of 2K
// values and the activation is fp16(silu(gate) * up), rounded exactly as
// lvb_silu_mul rounds it (the SiLU-mul fused into the down projection).
// four[g] = whether any token of group g needs its last two limbs
// (needs_four_limbs); stages whose groups need none copy and multiply only
// limbs 0 and 1.
template <int BN>
__global__ void __launch_bounds__(32 * BN) awq_act_limbs_kernel(const uint16_t *__restrict__ x, int64_t x_stride,
                                                                int gated, int8_t *__restrict__ limbs,
                                                                int4 *__restrict__ scal, int *__restrict__ four,
                                                                int M, int K, int G) {
  // The AWQ kernel that reads these limbs may start now and overlap this
  // grid; it waits for its completion before touching the outputs.  This
  // grid waits for the kernel that produced x.
  pdl_entry();
  const int g = blockIdx.x;
  const int t = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool row_ok = t < M;
  const uint16_t *xrow = x + static_cast<size_t>(row_ok ? t : 0) * x_stride + static_cast<size_t>(g) * G;
  // Four consecutive activations at k = g * G + i.
  auto load4 = [&](int i) -> uint2 {
    if (!row_ok) return make_uint2(0u, 0u);
    const uint2 gv = *reinterpret_cast<const uint2 *>(xrow + i);
    if (!gated) return gv;
    const uint2 uv = *reinterpret_cast<const uint2 *>(xrow + K + i);
    const float2 g0 = __half22float2(*reinterpret_cast<const __half2 *>(&gv.x));
    const float2 g1 = __half22float2(*reinterpret_cast<const __half2 *>(&gv.y));
    const float2 u0 = __half22float2(*reinterpret_cast<const __half2 *>(&uv.x));
    const float2 u1 = __half22float2(*reinterpret_cast<const __half2 *>(&uv.y));
    const __half2 a0 = __floats2half2_rn(silu_times(g0.x, u0.x), silu_times(g0.y, u0.y));
    const __half2 a1 = __floats2half2_rn(silu_times(g1.x, u1.x), silu_times(g1.y, u1.y));
    return make_uint2(*reinterpret_cast<const uint32_t *>(&a0), *reinterpret_cast<const uint32_t *>(&a1));
  };
  float amax = 0.f;
  for (int i = 4 * lane; i < G; i += 128) {
    const uint2 raw = load4(i);
    const __half2 h0 = *reinterpret_cast<const __half2 *>(&raw.x);
    const __half2 h1 = *reinterpret_cast<const __half2 *>(&raw.y);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(__low2float(h0)), fabsf(__high2float(h0))),
                             fmaxf(fabsf(__low2float(h1)), fabsf(__high2float(h1)))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const int e = limb_exponent(amax);
  const float inv_a = ldexpf(1.f, -e);
  int s01 = 0, s23 = 0, large = 0;
  for (int i = 4 * lane; i < G; i += 128) {
    const uint2 raw = load4(i);
    const __half2 h0 = *reinterpret_cast<const __half2 *>(&raw.x);
    const __half2 h1 = *reinterpret_cast<const __half2 *>(&raw.y);
    const float v[4] = {__low2float(h0), __high2float(h0), __low2float(h1), __high2float(h1)};
    large += large_count(v, amax);
    uint32_t w[kLimbs] = {};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int l[kLimbs];
      split_limbs(v[q] * inv_a, l);
      s01 += l[0] * 128 + l[1];
      s23 += l[2] * 128 + l[3];
      const int pos = ((q & 1) << 1) | (q >> 1);    // byte of k-offset q in the quad
#pragma unroll
      for (int j = 0; j < kLimbs; ++j) w[j] |= (static_cast<uint32_t>(l[j]) & 0xFFu) << (8 * pos);
    }
    const int k = g * G + i;
    // Limb pair q = j / 2 of 64-k chunk c at q * (K / 64) * 2 KB + c * 2 KB;
    // rows (j % 2) * BN + t of the pair's [2 BN][64 B] chunk tile.
    const size_t pair_stride = static_cast<size_t>(K >> 6) * (2 * BN * 64);
    int8_t *tile = limbs + static_cast<size_t>(k >> 6) * (2 * BN * 64);
#pragma unroll
    for (int j = 0; j < kLimbs; ++j)
      *reinterpret_cast<uint32_t *>(tile + (j >> 1) * pair_stride + sw64((j & 1) * BN + t, k & 63)) = w[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s01 += __shfl_xor_sync(0xffffffffu, s01, o);
    s23 += __shfl_xor_sync(0xffffffffu, s23, o);
    large += __shfl_xor_sync(0xffffffffu, large, o);
  }
  const int mine = row_ok ? needs_four_limbs(large, G) : 0;
  if (lane == 0) scal[static_cast<size_t>(g) * BN + t] = make_int4(__float_as_int(ldexpf(1.f, e - 7)), s01, s23, mine);
  const int any = __syncthreads_or(lane == 0 && mine);
  if (threadIdx.x == 0) four[g] = any ? 1 : 0;
}

// y tile store: shared [BN][128] fp16 -> global y at (column n0, row 0);
// rows past m are clipped by the tensor map.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::i8 (s8 x s8 -> s32).
__device__ __forceinline__ void umma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::i8: signed 8-bit A and B, s32 accumulator.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int m, int n) {
  return (2u << 4) |                               // D format: s32
         (1u << 7) |                               // A: signed 8-bit
         (1u << 10) |                              // B: signed 8-bit
         (static_cast<uint32_t>(n >> 3) << 17) |  // N / 8
         (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// One (column tile, K split) work unit of a persistent CTA: its groups,
// blocks and 256-k stages.
struct Unit {
  int tile, split, g_begin, b_begin, nblocks, nstages;
};

__device__ __forceinline__ Unit unit_of(int u, const I8Params &p) {
  // 32-bit arithmetic throughout (a 64-bit division is a long subroutine on
  // the path between units): splits <= 16 and groups < 2^20.
  Unit w;
  const unsigned splits = static_cast<unsigned>(p.splits);
  w.tile = static_cast<int>(static_cast<unsigned>(u) / splits);
  w.split = u - w.tile * p.splits;
  // Splits cover whole groups, so every unit drains complete groups and its
  // stages start on a group boundary.
  w.g_begin = static_cast<int>(static_cast<unsigned>(w.split * p.groups) / splits);
  const int g_end = static_cast<int>(static_cast<unsigned>((w.split + 1) * p.groups) / splits);
  w.b_begin = w.g_begin << p.bpg_shift;
  w.nblocks = (g_end - w.g_begin) << p.bpg_shift;
  w.nstages = (w.nblocks + kStageBlocks - 1) / kStageBlocks;
  return w;
}

// Persistent: CTA c runs units c, c + gridDim.x, ...; every role walks the
// same sequence of stages, numbered gs across units for the rings' slots and
// phases, so the pipeline does not drain between units.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    awq_i8_kernel(const __grid_constant__ CUtensorMap ymap, const I8Params p) {
  using C = I8Config<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *full = bars;                      // codes and limbs of a stage landed
  uint64_t *done = full + kStages;            // the stage's MMAs completed (slot and A stage free)
  uint64_t *a_full = done + kStages;          // the stage's A columns are in tensor memory
  uint64_t *d_full = a_full + kStages;        // a stage accumulator holds finished groups
  uint64_t *d_empty = d_full + C::kDStages;      // the drain has read a stage accumulator
  uint64_t *fin = d_empty + C::kDStages;         // [2]: every MMA of each issuer has completed
  uint64_t *flags_bar = fin + 2;                 // the group flags are in shared memory
  const uint8_t *four_sm = smem + C::kFlagOff;
  // Four-limb flag of group g (shared memory when every group fits there).
  auto four_of = [&](int g) -> bool { return p.groups <= kMaxFlagGroups ? four_sm[g] != 0 : p.four[g] != 0; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 8);
  volatile int *last_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int units = p.n_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&done[s], 1);
      mbar_init(&a_full[s], 4);
    }
    for (int j = 0; j < C::kDStages; ++j) {
      mbar_init(&d_full[j], 1);
      mbar_init(&d_empty[j], 4);
    }
    mbar_init(&fin[0], 1);
    mbar_init(&fin[1], 1);
    mbar_init(flags_bar, 32);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 || warp == 1) {
    // ---------------- producers ----------------
    if (warp == 1) {
      // The activation limbs and group flags come from the preceding prologue
      // launch, which this grid may overlap (programmatic dependent launch):
      // wait for it before the first limb copy; then stage the group flags.
      // The codes do not depend on it.
      asm volatile("griddepcontrol.wait;" ::: "memory");
      if (p.groups <= kMaxFlagGroups) {
        uint8_t *dst = smem + C::kFlagOff;
        for (int g = lane; g < p.groups; g += 32) dst[g] = p.four[g] ? 1 : 0;
      }
      __syncwarp();
      mbar_arrive(flags_bar);
    }
    if (lane == 0) {
      bool ok = true;
      int gs = 0;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = unit_of(u, p);
        for (int ls = 0; ls < w.nstages; ++ls, ++gs) {
          const int slot = gs % kStages;
          if (gs >= kStages && !mbar_wait(&done[slot], ((gs / kStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *stage = smem + slot * C::kStageBytes;
          const int blk0 = w.b_begin + ls * kStageBlocks;
          const int nb = min(kStageBlocks, w.b_begin + w.nblocks - blk0);
          if (warp == 0) {
            const uint32_t bytes = static_cast<uint32_t>(2 * nb * kChunkBytes);
            mbar_arrive_expect_tx(&full[slot], bytes);
            awqd::bulk_load(stage + C::kQOff,
                            p.qpack + (static_cast<size_t>(w.tile) * p.k_chunks + 2 * blk0) * kChunkBytes, bytes,
                            &full[slot]);
          } else {
            // Limb pair 0 (limbs 0-1) of the stage's chunks is one contiguous
            // run of the limb tile, pair 1 another; a two-limb stage copies
            // only the first.
            const int g0 = blk0 >> p.bpg_shift;
            const bool four = four_of(g0) || ((blk0 + nb - 1) >> p.bpg_shift) != g0 && four_of(g0 + 1);
            const uint32_t bytes = static_cast<uint32_t>(nb * C::kPairChunkBytes);
            mbar_arrive_expect_tx(&full[slot], four ? 2 * bytes : bytes);
            const int8_t *src = p.limbs + static_cast<size_t>(blk0) * C::kPairChunkBytes;
            awqd::bulk_load(stage, src, bytes, &full[slot]);
            if (four)
              awqd::bulk_load(stage + C::kPairStageStride, src + static_cast<size_t>(p.k_chunks / 2) * C::kPairChunkBytes,
                              bytes, &full[slot]);
          }
        }
      }
      if (!ok) {
        for (int g = gs > kStages ? gs - kStages : 0; g < gs; ++g)
          mbar_wait(&full[g % kStages], (g / kStages) & 1, nullptr, kDrainBudgetCycles);
      }
    }
    __syncwarp();
  } else if (warp == 2 || warp == kIssuer2Warp) {
    // ---------------- tcgen05.mma issuers ----------------
    // Two threads issue alternate stages (stage parity = issuer), each with
    // one wait set and one commit pair per stage: a stage's waits and
    // bookkeeping overlap the other issuer's MMAs in the tensor pipe.  Stage
    // accumulator ds = parity and A stages s = gs % 4 are private to one
    // issuer, and tcgen05.commit tracks only the issuing thread's MMAs.
    // The limb kernel's flags are read below: wait for it (it precedes this grid).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(kTileN, 2 * BN);  // one limb pair: N = 2 BN
      const int parity = warp == 2 ? 0 : 1;
      bool ok = mbar_wait(flags_bar, 0, abort_flag);
      int gs = 0;
      int sc = 0;  // accumulator slots taken by every stage so far (both issuers count all stages)
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = unit_of(u, p);
        for (int ls = 0; ls < w.nstages; ++ls, ++gs) {
          const int nb = min(kStageBlocks, w.nblocks - ls * kStageBlocks);
          const int blk0 = w.b_begin + ls * kStageBlocks;
          const int g0 = blk0 >> p.bpg_shift;
          const bool four = four_of(g0) || ((blk0 + nb - 1) >> p.bpg_shift) != g0 && four_of(g0 + 1);
          const int slot0 = sc;
          sc += four ? 2 : 1;
          if ((gs & 1) != parity) continue;
          const int s = gs % kStages;
          const int ds0 = slot0 & (C::kDStages - 1), ds1 = (slot0 + 1) & (C::kDStages - 1);
          const uint64_t bdesc0 = awqd::umma_desc_kmajor_sw64(smem_u32(smem + s * C::kStageBytes));
          const uint32_t a0 = tmem + C::kACol + s * kAStageCols;
          if (!mbar_wait(&full[s], (gs / kStages) & 1, abort_flag) ||
              !mbar_wait(&a_full[s], (gs / kStages) & 1, abort_flag) ||
              (slot0 >= C::kDStages && !mbar_wait(&d_empty[ds0], ((slot0 / C::kDStages) - 1) & 1, abort_flag)) ||
              (four && slot0 + 1 >= C::kDStages &&
               !mbar_wait(&d_empty[ds1], (((slot0 + 1) / C::kDStages) - 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int b = 0; b < nb; ++b) {
            const uint32_t dg = (b >> p.bpg_shift) * C::kGroupCols;
            const uint64_t bd = bdesc0 + static_cast<uint64_t>((b * C::kPairChunkBytes) >> 4);
            const uint32_t first = (b & ((1 << p.bpg_shift) - 1)) == 0 ? 0u : 1u;
            umma_i8_ts(tmem + ds0 * C::kDStageCols + dg, a0 + b * 16, bd, idesc, first);
            umma_i8_ts(tmem + ds0 * C::kDStageCols + dg, a0 + b * 16 + 8, bd + 2, idesc, 1u);  // second 32-k run
            if (four) {  // limbs 2-3 into the stage's second slot
              const uint64_t bh = bd + static_cast<uint64_t>(C::kPairStageStride >> 4);
              umma_i8_ts(tmem + ds1 * C::kDStageCols + dg, a0 + b * 16, bh, idesc, first);
              umma_i8_ts(tmem + ds1 * C::kDStageCols + dg, a0 + b * 16 + 8, bh + 2, idesc, 1u);
            }
          }
          umma_commit(&done[s]);
          umma_commit(&d_full[ds0]);
          if (four) umma_commit(&d_full[ds1]);
        }
      }
      // Tensor memory is freed only after every issued MMA has completed.
      umma_commit(&fin[parity]);
      mbar_wait(&fin[parity], 0, nullptr, ok ? kWaitBudgetCycles : kDrainBudgetCycles);
    }
    __syncwarp();
  } else if (warp < kDrainWarp) {
    // ---------------- code expanders ----------------
    // full[s] for stage gs implies done[s] for stage gs - kStages (the
    // producer waited for it before refilling the slot), so A stage s is free.
    const int quad = warp & 3;
    const int col = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    bool ok = true;
    int gs = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const Unit w = unit_of(u, p);
      for (int ls = 0; ls < w.nstages; ++ls, ++gs) {
        const int s = gs % kStages;
        const int nb = min(kStageBlocks, w.nblocks - ls * kStageBlocks);
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (gs / kStages) & 1, abort_flag))) { ok = false; break; }
        const uint8_t *stage = smem + s * C::kStageBytes + C::kQOff;
        uint4 q[kStageChunks];
#pragma unroll
        for (int c = 0; c < kStageChunks; ++c)
          if (c < 2 * nb) q[c] = *reinterpret_cast<const uint4 *>(stage + c * kChunkBytes + col * 16);
        tc_fence_after();
#pragma unroll
        for (int b = 0; b < kStageBlocks; ++b) {
          if (b < nb) {
            uint32_t a[16];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              const uint32_t wd[4] = {q[2 * b + r].x, q[2 * b + r].y, q[2 * b + r].z, q[2 * b + r].w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                a[8 * r + j] = wd[j] & 0x0F0F0F0Fu;
                a[8 * r + 4 + j] = (wd[j] >> 4) & 0x0F0F0F0Fu;
              }
            }
            tmem_st_32x32b_x16(tmem + lane_base + C::kACol + s * kAStageCols + b * 16, a);
          }
        }
        awqd::tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
      }
    }
  } else {
    // ---------------- drain + epilogue ----------------
    const int quad = warp & 3;
    const int col = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const int gps_full = kStageBlocks >> p.bpg_shift;  // groups per full stage (2 or 1)
    // The next stage's (scale, zero) words (registers) and per-token scalars
    // (cp.async into this warp's shared slots) are fetched one stage ahead.
    uint8_t *scal_sm = smem + C::kScalOff + (warp - kDrainWarp) * 2 * C::kScalSlotBytes;
    auto fetch_scal = [&](const Unit &w, int ls, int gs_) {
      const int g0 = w.g_begin + ls * gps_full;
      const int ng = min(kStageBlocks, w.nblocks - ls * kStageBlocks) >> p.bpg_shift;
      if (lane < ng * BN)
        cp_async_16(smem_u32(scal_sm + (gs_ & 1) * C::kScalSlotBytes + lane * 16),
                    reinterpret_cast<const uint8_t *>(p.scal + static_cast<size_t>(g0) * BN) + lane * 16, 16u);
      cp_async_commit();
    };
    // Returned by value, so the loads stay in registers and are waited for
    // only where the words are used.
    auto fetch_sz = [&](const Unit &w, int ls) -> uint2 {
      const int g0 = w.g_begin + ls * gps_full;
      const int ng = min(kStageBlocks, w.nblocks - ls * kStageBlocks) >> p.bpg_shift;
      const uint32_t *szrow = p.szpack + (static_cast<size_t>(w.tile) * p.groups) * kTileN + col;
      return make_uint2(__ldg(szrow + static_cast<size_t>(g0) * kTileN),
                        ng > 1 ? __ldg(szrow + static_cast<size_t>(g0 + 1) * kTileN) : 0u);
    };
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the scalars come from the prologue launch
    bool ok = __all_sync(0xffffffffu, mbar_wait(flags_bar, 0, abort_flag));
    int gs = 0;
    int slots = 0;  // accumulator slots taken by the stages drained so far
    uint2 sz_next = make_uint2(0u, 0u);
    uint2 sz_unit_next = make_uint2(0u, 0u);  // first stage of the next unit, loaded a unit ahead
    int u = blockIdx.x;
    Unit w = unit_of(u, p);
    if (u < units) {
      fetch_scal(w, 0, 0);
      sz_next = fetch_sz(w, 0);
    }
    for (; u < units && ok; u += gridDim.x) {
      w = unit_of(u, p);
      const bool has_next = u + static_cast<int>(gridDim.x) < units;
      const Unit wn = unit_of(has_next ? u + static_cast<int>(gridDim.x) : u, p);
      if (has_next) sz_unit_next = fetch_sz(wn, 0);
      const int n = w.tile * kTileN + col;
      const bool n_ok = n < p.N;
      float acc[BN];
#pragma unroll
      for (int t = 0; t < BN; ++t) acc[t] = 0.f;
      for (int ls = 0; ls < w.nstages; ++ls, ++gs) {
        const uint32_t sz[2] = {sz_next.x, sz_next.y};
        const int ng = min(kStageBlocks, w.nblocks - ls * kStageBlocks) >> p.bpg_shift;
        cp_async_wait_all();
        __syncwarp();
        if (ls + 1 < w.nstages) {
          fetch_scal(w, ls + 1, gs + 1);
          sz_next = fetch_sz(w, ls + 1);
        } else if (has_next) {
          fetch_scal(wn, 0, gs + 1);
          sz_next = sz_unit_next;
        }
        const int4 *sc = reinterpret_cast<const int4 *>(scal_sm + (gs & 1) * C::kScalSlotBytes);  // one per token
        const int sg0 = w.g_begin + ls * gps_full;
        const bool four = four_of(sg0) || (ng > 1 && four_of(sg0 + 1));
        const int ds0 = slots & (C::kDStages - 1), ds1 = (slots + 1) & (C::kDStages - 1);
        if (!__all_sync(0xffffffffu, mbar_wait(&d_full[ds0], (slots / C::kDStages) & 1, abort_flag) &&
                                         (!four || mbar_wait(&d_full[ds1], ((slots + 1) / C::kDStages) & 1,
                                                             abort_flag)))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (j >= ng) break;
          const float s = __half2float(__ushort_as_half(static_cast<uint16_t>(sz[j] & 0xFFFFu)));
          const int z = static_cast<int>(sz[j] >> 16);
          const uint32_t dcol = tmem + lane_base + ds0 * C::kDStageCols + j * C::kGroupCols;
          const uint32_t dcol_hi = tmem + lane_base + ds1 * C::kDStageCols + j * C::kGroupCols;
#pragma unroll
          for (int h = 0; h < BN / 16; ++h) {
            uint32_t d0[16], d1[16];
            tmem_ld_32x32b_x16(dcol + h * 16, d0);
            tmem_ld_32x32b_x16(dcol + BN + h * 16, d1);
            if (four) {  // uniform over the warp
              uint32_t d2[16], d3[16];
              tmem_ld_32x32b_x16(dcol_hi + h * 16, d2);
              tmem_ld_32x32b_x16(dcol_hi + BN + h * 16, d3);
              tmem_wait_ld();
#pragma unroll
              for (int t = 0; t < 16; ++t) {
                const int4 sc4 = sc[j * BN + h * 16 + t];
                const int v_hi = static_cast<int>(d0[t]) * 128 + static_cast<int>(d1[t]) - z * sc4.y;
                const int v_lo = static_cast<int>(d2[t]) * 128 + static_cast<int>(d3[t]) - z * sc4.z;
                const float v = fmaf(static_cast<float>(v_lo), 1.f / 16384.f, static_cast<float>(v_hi));
                acc[h * 16 + t] = fmaf(s * __int_as_float(sc4.x), v, acc[h * 16 + t]);
              }
            } else {
              tmem_wait_ld();
#pragma unroll
              for (int t = 0; t < 16; ++t) {
                const int4 sc4 = sc[j * BN + h * 16 + t];
                const int v_hi = static_cast<int>(d0[t]) * 128 + static_cast<int>(d1[t]) - z * sc4.y;
                acc[h * 16 + t] = fmaf(s * __int_as_float(sc4.x), static_cast<float>(v_hi), acc[h * 16 + t]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&d_empty[ds0]);
          if (four) mbar_arrive(&d_empty[ds1]);
        }
        slots += four ? 2 : 1;
      }
      // ---- epilogue of the unit ----
      ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
      if (!ok) break;
      const float bias_n = (p.bias != nullptr && n_ok) ? __half2float(__ushort_as_half(p.bias[n])) : 0.f;
      if (p.splits == 1) {
        // Stage the tile in shared memory and write it with one TMA store, so
        // the drain does not wait on BN strided global stores.
        uint16_t *ytile = reinterpret_cast<uint16_t *>(smem + C::kYOff);
        if (warp == kDrainWarp && lane == 0) tma_store_wait_read();  // the previous unit's store has read the tile
        asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
        for (int t = 0; t < BN; ++t) ytile[t * kTileN + col] = __half_as_ushort(__float2half_rn(acc[t] + bias_n));
        fence_proxy_async_smem();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (warp == kDrainWarp && lane == 0) tma_store_2d(&ymap, ytile, w.tile * kTileN, 0);
      } else {
        float *part = p.partials + static_cast<size_t>(w.tile) * p.splits * BN * kTileN;
#pragma unroll
        for (int t = 0; t < BN; ++t) __stcg(part + (static_cast<size_t>(w.split) * BN + t) * kTileN + col, acc[t]);
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (warp == kDrainWarp && lane == 0) {
          const unsigned int prev = atomicAdd(p.semaphores + w.tile, 1u);
          *last_flag = prev == static_cast<unsigned int>(p.splits - 1) ? 1 : 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool last = *last_flag != 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");  // every drain thread has read the flag
        if (last) {
          __threadfence();
          float sum[BN];
#pragma unroll
          for (int t = 0; t < BN; ++t) sum[t] = 0.f;
          for (int sp = 0; sp < p.splits; ++sp) {
            float v[BN];
#pragma unroll
            for (int t = 0; t < BN; ++t) v[t] = __ldcg(part + (static_cast<size_t>(sp) * BN + t) * kTileN + col);
#pragma unroll
            for (int t = 0; t < BN; ++t) sum[t] += v[t];
          }
          if (n_ok) {
#pragma unroll
            for (int t = 0; t < BN; ++t)
              if (t < p.M) p.y[static_cast<size_t>(t) * p.N + n] = __half_as_ushort(__float2half_rn(sum[t] + bias_n));
          }
          if (warp == kDrainWarp && lane == 0) p.semaphores[w.tile] = 0u;
        }
      }
    }
    cp_async_wait_all();
    if (warp == kDrainWarp && lane == 0) tma_store_wait_all();
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace awqi8
}  // namespace lvb
