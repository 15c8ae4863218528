// W4A16 GEMV for the smallest decode batches (m <= 4) on sm_100a CUDA cores.
//
// Reference: the decode-sized path of CudaAWQOperation (M <= 255 -> K1
// `gemm_forward_4bit_cuda_m16nXk32`, csrc/awq/gemm_kernels.cu:29-326, 444-501,
// called from modeling/quantization/cuda_awq.py:96-122): y = x @ W (+ bias),
// W[k][n] = (q - z) * s per 128-k group.  At m <= 4 the tensor cores would
// multiply mostly padding, so each output column is reduced on CUDA cores
// with integer dot products, with the limb arithmetic of the int8 path
// (awq_i8.cuh):
//
//   x is split per (token, group) into four int8 limbs,
//   x = a (x0 + x1 / 128 + x2 / 128^2 + x3 / 128^3), a a power of two
//   (exact for every fp16 value within 2^17 of the group's largest); a group
//   where at least G/8 elements exceed a sixteenth of its largest skips x2 and
//   x3 (see awqi8::needs_four_limbs); for each group
//     D_l  = sum q x_l                               (dp4a, exact in int32)
//     v_hi = 128 D0 + D1 - z * sum(128 x0 + x1),  v_lo = 128 D2 + D3 - z * sum(128 x2 + x3)
//     acc += s * (a / 128) * (v_hi + v_lo / 128^2)   (fp32)
//
// Layout: the packed codes of awq_decode.cuh ([n_tile][32-k run][128 columns]
// [16 B]); within a run, word w masked with 0x0F0F0F0F holds k = 4w + (0, 2,
// 1, 3) and shifted right by 4 holds k = 16 + 4w + (0, 2, 1, 3) -- the byte
// order of the limb words, so each (code word, limb word) pair is one dp4a.
//
// One consumer thread per output column (4 warps, one 128-column tile) and
// one producer warp; a CTA covers a range of whole groups (split-K).  The
// producer streams the range's codes -- contiguous in the packed layout --
// into a ring of shared-memory stages with bulk async copies (mbarrier
// complete_tx) from the moment the CTA starts; meanwhile the consumers wait
// for the kernel that produced x (programmatic dependent launch), read the
// range's activations (a few KB, L2-resident; a warp issues the loads of four
// (group, token) pairs before using them) and build their limbs in shared
// memory -- so no separate prologue launch and no global limb buffer exist.
// Groups of up to 256 k.  Consumers then read their
// column's 16 bytes per run from shared memory and the limbs as broadcasts.
// Splits combine through per-split fp32 partials and a semaphore: the last
// CTA of a tile sums them in split order (deterministic), adds the bias and
// writes y.  Every wait is bounded.
#pragma once

#include "awq_i8.cuh"
#include "lvb_common.cuh"

namespace lvb {
namespace awqg {

constexpr int kThreads = 128;      // consumer threads: one output column each
constexpr int kCtaThreads = 160;   // + one producer warp
constexpr int kStageRuns = 8;      // 32-k runs per stage (16 KB of codes)
constexpr int kStages = 2;         // 32 KB ring.  B200, 7B B = 1 decode step: 2.15 ms with five
                                   // 8 KB stages, 2.10 with two 16 KB stages, 2.30 with three
constexpr int kStageBytes = kStageRuns * 128 * 16;
constexpr int kMaxM = 4;
using awqi8::kLimbs;

// QKV epilogue (rope != 0): the output row is a merged QKV projection with
// head size D (64 or 128, so a 128-column tile holds whole heads).  Query
// heads are rotated (Qwen2 half rotation, fp32 from the fp16-rounded outputs,
// one rounding: the arithmetic of rope_kv_write_kernel) and written to y;
// key heads are rotated into the token's paged cache slot and value heads
// copied there (y keeps them unrotated).
struct GemvRope {
  int rope;
  const int32_t *positions;          // [M] RoPE position per token
  const uint16_t *cos, *sin;         // [table_rows][D] fp16
  uint16_t *key_cache, *value_cache;  // [blocks][bs][hkv][D]
  const int32_t *tables;
  int64_t table_stride;
  const int32_t *computed, *qsl, *req;
  int hq, hkv, D, bs, table_rows;
};

struct GemvParams {
  const uint8_t *qpack;    // [n_tiles][k_chunks][128][16 B]
  const uint32_t *szpack;  // [n_tiles][groups][128]: scale bits | zero << 16
  const uint16_t *x;       // [M] rows of x_stride fp16 (gated: merged [gate | up] rows of 2K)
  int64_t x_stride;
  int gated;               // activation = fp16(silu(gate) * up), as lvb_silu_mul rounds it
  const uint16_t *bias;    // may be null
  uint16_t *y;             // [M][N]
  uint32_t *semaphores;    // [n_tiles], zero between calls
  float *partials;         // [n_tiles][splits][M][128]
  int M, K, N, G;
  int groups, k_chunks, runs_per_group;
  int n_tiles, splits, groups_per_split;
  GemvRope r;
};

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

// Final outputs of column n for the MT token rows: y, or the QKV epilogue.
// All 128 consumer threads of the CTA call it together (RoPE exchanges the
// two halves of a head through shared memory).
template <int MT>
__device__ __forceinline__ void gemv_store(const GemvParams &p, int n, const float (&v)[MT]) {
  if (!p.r.rope) {
#pragma unroll
    for (int t = 0; t < MT; ++t)
      if (t < p.M) p.y[static_cast<size_t>(t) * p.N + n] = __half_as_ushort(__float2half_rn(v[t]));
    return;
  }
  __shared__ __half xch[MT][kThreads];
  const int tid = threadIdx.x;
  const GemvRope &r = p.r;
  const int D = r.D, half = D / 2;
  const int head = n / D, i = n - head * D;
  __half h[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    h[t] = __float2half_rn(v[t]);
    xch[t][tid] = h[t];
  }
  consumers_sync();
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    if (t >= p.M) continue;
    const int pos = r.positions[t];
    if (pos < 0 || pos >= r.table_rows) {
      if (tid == 0) record_device_error(LVB_DEVERR_INDEX);
      continue;
    }
    const int q = r.req[t];
    const int lp = r.computed[q] + (t - r.qsl[q]);
    const int64_t slot =
        static_cast<int64_t>(r.tables[static_cast<int64_t>(q) * r.table_stride + lp / r.bs]) * r.bs + lp % r.bs;
    if (head < r.hq + r.hkv) {
      const float self = __half2float(h[t]);
      const float other = __half2float(xch[t][tid ^ half]);
      const float c = __half2float(reinterpret_cast<const __half *>(r.cos)[static_cast<size_t>(pos) * D + i]);
      const float sn = __half2float(reinterpret_cast<const __half *>(r.sin)[static_cast<size_t>(pos) * D + i]);
      // Lower half x1 c1 + (-x2) s1, upper x2 c2 + x1 s2 (the standalone kernels' rope_rotate).
      const __half o = __float2half_rn(rope_rotate(self, c, i < half ? -other : other, sn));
      if (head < r.hq) {
        p.y[static_cast<size_t>(t) * p.N + n] = __half_as_ushort(o);
      } else {
        r.key_cache[(static_cast<size_t>(slot) * r.hkv + (head - r.hq)) * D + i] = __half_as_ushort(o);
        p.y[static_cast<size_t>(t) * p.N + n] = __half_as_ushort(h[t]);
      }
    } else {
      r.value_cache[(static_cast<size_t>(slot) * r.hkv + (head - r.hq - r.hkv)) * D + i] = __half_as_ushort(h[t]);
      p.y[static_cast<size_t>(t) * p.N + n] = __half_as_ushort(h[t]);
    }
  }
}

// Shared memory: code stages, limb words [MT][kLimbs][range_quads] (quad q =
// k offset 4q of the range, bytes in the (0, 2, 1, 3) order), per [group][MT]
// (a / 128, sum of 128 x0 + x1, sum of 128 x2 + x3, 0), the range's (scale,
// zero) words [group][128], then the barriers (full[kStages],
// empty[kStages], sz) and the abort flag.
template <int MT>
struct GemvSmem {
  static constexpr size_t kLimbOff = static_cast<size_t>(kStages) * kStageBytes;
  __host__ __device__ static size_t limb_bytes(int gps, int rpg) {
    return static_cast<size_t>(MT) * kLimbs * gps * rpg * 8 * 4;
  }
  __host__ __device__ static size_t scal_off(int gps, int rpg) { return kLimbOff + limb_bytes(gps, rpg); }
  __host__ __device__ static size_t sz_off(int gps, int rpg) {
    return scal_off(gps, rpg) + static_cast<size_t>(gps) * MT * 16;
  }
  __host__ __device__ static size_t bar_off(int gps, int rpg) { return sz_off(gps, rpg) + static_cast<size_t>(gps) * kThreads * 4; }
  __host__ __device__ static size_t bytes(int gps, int rpg) { return bar_off(gps, rpg) + (2 * kStages + 1) * 8 + 16; }
};

template <int MT>
__global__ void __launch_bounds__(kCtaThreads) awq_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  using S = GemvSmem<MT>;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int rpg = p.runs_per_group;
  const int g0 = split * p.groups_per_split;
  const int g1 = min(p.groups, g0 + p.groups_per_split);
  const int run0 = g0 * rpg, run1 = g1 * rpg;
  const int nruns = run1 - run0;
  const int nstages = (nruns + kStageRuns - 1) / kStageRuns;
  const int range_quads = nruns * 8;
  uint32_t *limb_sm = reinterpret_cast<uint32_t *>(smem + S::kLimbOff);
  int4 *scal_sm = reinterpret_cast<int4 *>(smem + S::scal_off(p.groups_per_split, rpg));
  const uint32_t *sz_sm = reinterpret_cast<const uint32_t *>(smem + S::sz_off(p.groups_per_split, rpg));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::bar_off(p.groups_per_split, rpg));
  uint64_t *empty = full + kStages;
  uint64_t *sz_bar = empty + kStages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(sz_bar + 1);

  // The next kernel of the stream may launch now; it waits for this grid's
  // completion before touching y.
  pdl_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kThreads / 32);
    }
    mbar_init(sz_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kThreads / 32) {
    // Producer: the codes do not depend on the previous kernel, so this starts at once.
    if (lane == 0) {
      // The range's (scale, zero) rows are contiguous: one copy.
      const uint32_t sz_bytes = static_cast<uint32_t>(g1 - g0) * kThreads * 4;
      mbar_arrive_expect_tx(sz_bar, sz_bytes);
      awqd::bulk_load(smem + S::sz_off(p.groups_per_split, rpg),
                      p.szpack + (static_cast<size_t>(tile) * p.groups + g0) * kThreads, sz_bytes, sz_bar);
      const uint8_t *src = p.qpack + (static_cast<size_t>(tile) * p.k_chunks + run0) * 128 * 16;
      int issued = 0;
      for (int st = 0; st < nstages; ++st) {
        const int slot = st % kStages;
        if (st >= kStages && !mbar_wait(&empty[slot], ((st / kStages) - 1) & 1, abort_flag)) break;
        const int runs = min(kStageRuns, nruns - st * kStageRuns);
        const uint32_t bytes = static_cast<uint32_t>(runs) * 128 * 16;
        mbar_arrive_expect_tx(&full[slot], bytes);
        awqd::bulk_load(smem + static_cast<size_t>(slot) * kStageBytes,
                        src + static_cast<size_t>(st) * kStageBytes, bytes, &full[slot]);
        issued = st + 1;
      }
      // Leave only once every copy issued has landed (shared memory must not
      // be written after the CTA ends).
      for (int st = max(0, issued - kStages); st < issued; ++st)
        mbar_wait(&full[st % kStages], (st / kStages) & 1, nullptr);
      mbar_wait(sz_bar, 0, nullptr);
    }
    return;
  }

  // Activations come from the previous kernel of the stream (this grid may
  // have started during its tail): wait for it, then build this range's limbs.
  pdl_wait();
  {
    // Limbs of the range, one warp per (group, token) pair.  A warp takes its
    // pairs kPairBatch at a time and issues every activation load of a batch
    // before using any (one L2 round trip per batch, not two per pair); each
    // lane holds 4 consecutive k per 128 of the group (groups of up to 256).
    constexpr int kPairBatch = 4;
    constexpr int kWarpsC = kThreads / 32;
    const int G = p.G;
    const int ng = g1 - g0;
    const int pairs = ng * MT;
    auto load4 = [&](int gg, int t, int i) -> uint2 {
      if (t >= p.M || i >= G) return make_uint2(0u, 0u);
      const uint16_t *src = p.x + static_cast<size_t>(t) * p.x_stride + static_cast<size_t>(g0 + gg) * G + i;
      const uint2 gv = *reinterpret_cast<const uint2 *>(src);
      if (!p.gated) return gv;
      const uint2 uv = *reinterpret_cast<const uint2 *>(src + p.K);
      const float2 ga = __half22float2(*reinterpret_cast<const __half2 *>(&gv.x));
      const float2 gb = __half22float2(*reinterpret_cast<const __half2 *>(&gv.y));
      const float2 ua = __half22float2(*reinterpret_cast<const __half2 *>(&uv.x));
      const float2 ub = __half22float2(*reinterpret_cast<const __half2 *>(&uv.y));
      const __half2 a0 = __floats2half2_rn(silu_times(ga.x, ua.x), silu_times(ga.y, ua.y));
      const __half2 a1 = __floats2half2_rn(silu_times(gb.x, ub.x), silu_times(gb.y, ub.y));
      return make_uint2(*reinterpret_cast<const uint32_t *>(&a0), *reinterpret_cast<const uint32_t *>(&a1));
    };
    for (int base = warp; base < pairs; base += kWarpsC * kPairBatch) {
      uint2 xv[kPairBatch][2];
#pragma unroll
      for (int b = 0; b < kPairBatch; ++b) {
        const int pr = base + kWarpsC * b;
        const int gg = pr / MT, t = pr - (pr / MT) * MT;
#pragma unroll
        for (int c = 0; c < 2; ++c) xv[b][c] = pr < pairs ? load4(gg, t, 4 * lane + 128 * c) : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int b = 0; b < kPairBatch; ++b) {
        const int pr = base + kWarpsC * b;
        if (pr >= pairs) break;  // uniform over the warp
        const int gg = pr / MT, t = pr - gg * MT;
        float v[2][4];
        float amax = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const __half2 h0 = *reinterpret_cast<const __half2 *>(&xv[b][c].x);
          const __half2 h1 = *reinterpret_cast<const __half2 *>(&xv[b][c].y);
          v[c][0] = __low2float(h0);
          v[c][1] = __high2float(h0);
          v[c][2] = __low2float(h1);
          v[c][3] = __high2float(h1);
          amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c][0]), fabsf(v[c][1])), fmaxf(fabsf(v[c][2]), fabsf(v[c][3]))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int e = awqi8::limb_exponent(amax);
        const float inv_a = ldexpf(1.f, -e);
        int s01 = 0, s23 = 0, large = 0;
        uint32_t *trow = limb_sm + static_cast<size_t>(t) * kLimbs * range_quads;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int i = 4 * lane + 128 * c;
          if (i >= G) break;
          large += awqi8::large_count(v[c], amax);
          uint32_t w[kLimbs] = {};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            int l[kLimbs];
            awqi8::split_limbs(v[c][q] * inv_a, l);
            s01 += l[0] * 128 + l[1];
            s23 += l[2] * 128 + l[3];
            const int pos = ((q & 1) << 1) | (q >> 1);  // byte of k-offset q in the quad
#pragma unroll
            for (int j = 0; j < kLimbs; ++j) w[j] |= (static_cast<uint32_t>(l[j]) & 0xFFu) << (8 * pos);
          }
          const int quad = (gg * G + i) >> 2;
#pragma unroll
          for (int j = 0; j < kLimbs; ++j) trow[static_cast<size_t>(j) * range_quads + quad] = w[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          s01 += __shfl_xor_sync(0xffffffffu, s01, o);
          s23 += __shfl_xor_sync(0xffffffffu, s23, o);
          large += __shfl_xor_sync(0xffffffffu, large, o);
        }
        if (lane == 0)
          scal_sm[pr] = make_int4(__float_as_int(ldexpf(1.f, e - 7)), s01, s23, awqi8::needs_four_limbs(large, G));
      }
    }
  }
  consumers_sync();

  float acc[MT];
  int d[MT][kLimbs];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    acc[t] = 0.f;
#pragma unroll
    for (int j = 0; j < kLimbs; ++j) d[t][j] = 0;
  }
  int group = g0, run_in_group = 0;
  bool ok = mbar_wait(sz_bar, 0, abort_flag);
  // Per token: whether the current group uses four limbs (uniform over the CTA).
  int four[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) four[t] = scal_sm[t].w;

  for (int st = 0; st < nstages && ok; ++st) {
    const int slot = st % kStages;
    if (!mbar_wait(&full[slot], (st / kStages) & 1, abort_flag)) {
      ok = false;
      break;
    }
    const uint4 *stage = reinterpret_cast<const uint4 *>(smem + static_cast<size_t>(slot) * kStageBytes) + tid;
    const int runs = min(kStageRuns, nruns - st * kStageRuns);
#pragma unroll
    for (int r = 0; r < kStageRuns; ++r) {
      if (r < runs) {
        const uint4 c = stage[r * kThreads];
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lo[j] = w[j] & 0x0F0F0F0Fu;
          hi[j] = (w[j] >> 4) & 0x0F0F0F0Fu;
        }
        const int q0 = (st * kStageRuns + r) * 8;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
#pragma unroll
          for (int j = 0; j < kLimbs; ++j) {
            if (j >= 2 && !four[t]) break;  // two-limb group
            const uint4 *l = reinterpret_cast<const uint4 *>(limb_sm + (static_cast<size_t>(t) * kLimbs + j) * range_quads + q0);
            const uint4 a = l[0], b = l[1];
            int acc_l = d[t][j];
            acc_l = __dp4a(static_cast<int>(lo[0]), static_cast<int>(a.x), acc_l);
            acc_l = __dp4a(static_cast<int>(lo[1]), static_cast<int>(a.y), acc_l);
            acc_l = __dp4a(static_cast<int>(lo[2]), static_cast<int>(a.z), acc_l);
            acc_l = __dp4a(static_cast<int>(lo[3]), static_cast<int>(a.w), acc_l);
            acc_l = __dp4a(static_cast<int>(hi[0]), static_cast<int>(b.x), acc_l);
            acc_l = __dp4a(static_cast<int>(hi[1]), static_cast<int>(b.y), acc_l);
            acc_l = __dp4a(static_cast<int>(hi[2]), static_cast<int>(b.z), acc_l);
            acc_l = __dp4a(static_cast<int>(hi[3]), static_cast<int>(b.w), acc_l);
            d[t][j] = acc_l;
          }
        }
        if (++run_in_group == rpg) {
          // Group done: fold the exact integer sums into the fp32 accumulators.
          const uint32_t sz = sz_sm[(group - g0) * kThreads + tid];
          const float s = __half2float(__ushort_as_half(static_cast<unsigned short>(sz & 0xFFFFu)));
          const int z = static_cast<int>(sz >> 16);
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const int4 sc = scal_sm[(group - g0) * MT + t];
            const int v_hi = 128 * d[t][0] + d[t][1] - z * sc.y;
            const int v_lo = four[t] ? 128 * d[t][2] + d[t][3] - z * sc.z : 0;
            const float v = fmaf(static_cast<float>(v_lo), 1.f / 16384.f, static_cast<float>(v_hi));
            acc[t] = fmaf(s * __int_as_float(sc.x), v, acc[t]);
#pragma unroll
            for (int j = 0; j < kLimbs; ++j) d[t][j] = 0;
          }
          ++group;
          run_in_group = 0;
          if (group < g1) {
#pragma unroll
            for (int t = 0; t < MT; ++t) four[t] = scal_sm[(group - g0) * MT + t].w;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  // A wait that gave up raised the abort flag (and set the error word): the
  // CTA then leaves without output.
  consumers_sync();
  if (*abort_flag) return;

  const int n = tile * kThreads + tid;
  if (p.splits == 1) {
    const float b = p.bias ? __half2float(__ushort_as_half(p.bias[n])) : 0.f;
    float v[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) v[t] = acc[t] + b;
    gemv_store<MT>(p, n, v);
    return;
  }
  float *part = p.partials + (static_cast<size_t>(tile) * p.splits + split) * p.M * kThreads;
#pragma unroll
  for (int t = 0; t < MT; ++t)
    if (t < p.M) part[static_cast<size_t>(t) * kThreads + tid] = acc[t];
  __shared__ int last_sm;
  __threadfence();
  consumers_sync();
  if (tid == 0) {
    const unsigned prev = atomicAdd(p.semaphores + tile, 1u);
    last_sm = prev == static_cast<unsigned>(p.splits - 1);
  }
  consumers_sync();
  if (!last_sm) return;
  __threadfence();
  float sum[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) sum[t] = 0.f;
  const float *tp = p.partials + static_cast<size_t>(tile) * p.splits * p.M * kThreads;
  // Eight splits' loads in flight per round, summed in split order.
  constexpr int kBatch = 8;
  for (int sp0 = 0; sp0 < p.splits; sp0 += kBatch) {
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      if (t >= p.M) continue;
      float v[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
        v[b] = sp0 + b < p.splits ? __ldcg(tp + (static_cast<size_t>(sp0 + b) * p.M + t) * kThreads + tid) : 0.f;
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
        if (sp0 + b < p.splits) sum[t] += v[b];
    }
  }
  const float b = p.bias ? __half2float(__ushort_as_half(p.bias[n])) : 0.f;
  float v[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) v[t] = sum[t] + b;
  gemv_store<MT>(p, n, v);
  if (tid == 0) p.semaphores[tile] = 0u;  // ready for the next call
}

}  // namespace awqg
}  // namespace lvb
