// Paged K/V cache write and paged attention for sm_100a.
//
// Cache layout (one layer): K and V are separate [num_blocks, block_size,
// num_kv_heads, head_size] tensors; request r's logical position p lives at
// slot table[r][p / block_size] * block_size + p % block_size.
//
// Three kernels:
//   * paged_kv_write_kernel -- scatters this step's K/V rows to their slots
//     with 16-byte vector copies (one thread per 16 bytes of a row).
//   * paged_attn_general_kernel -- any packed batch: prefill chunks, decode,
//     tree (speculative) visibility, any head size <= 256 that is a multiple
//     of 8, any GQA group.  One CTA per (query token, query head); lanes score
//     32 positions at a time, an fp32 online softmax runs per warp and the four
//     warps merge at the end.
//   * paged_decode_kernel -- decode batches (one linear query per request):
//     one CTA per (request, KV head, context split).  A producer warp streams
//     the split's pages with TMA (K and V boxes of 16 tokens x 64 dims,
//     128-byte swizzle) through an 8-stage shared-memory ring; four consumer
//     warps each take every fourth page and run QK^T and PV for the whole GQA
//     group as 16-row warp MMAs (the group of up to 16 query heads is the MMA's
//     M dimension), with an fp32 online softmax in registers.  P is fed to the
//     PV product as a hi + lo pair of 16-bit values so the probabilities keep
//     fp32-like precision.  The warps merge through shared memory and each
//     split writes its normalised output and log2-sum-exp; paged_merge_kernel
//     combines the splits.
#pragma once

#include "lvb_common.cuh"

namespace lvb {
namespace attn {

// ------------------------------------------------------------------------
// K/V write
// ------------------------------------------------------------------------
struct KVWriteArgs {
  const uint16_t *key;
  int64_t key_stride;
  const uint16_t *value;
  int64_t value_stride;
  uint16_t *key_cache;
  uint16_t *value_cache;
  const int32_t *tables;  // null for explicit slots
  int64_t table_stride;
  const int32_t *computed;
  const int32_t *qsl;
  const int32_t *req;
  const int64_t *slots;  // explicit slots (kv_scatter), else null
  int num_tokens, Hkv, D, bs;
};

__global__ void paged_kv_write_kernel(const KVWriteArgs a) {
  const int t = blockIdx.x;
  int64_t slot;
  if (a.slots != nullptr) {
    slot = a.slots[t];
  } else {
    const int r = a.req[t];
    const int pos = a.computed[r] + (t - a.qsl[r]);
    const int64_t block = a.tables[static_cast<int64_t>(r) * a.table_stride + pos / a.bs];
    slot = block * a.bs + pos % a.bs;
  }
  const int chunks_per_head = a.D >> 3;
  const int chunks = a.Hkv * chunks_per_head;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
    const int h = c / chunks_per_head;
    const int d = (c - h * chunks_per_head) << 3;
    const uint4 kv = *reinterpret_cast<const uint4 *>(a.key + t * a.key_stride + h * a.D + d);
    const uint4 vv = *reinterpret_cast<const uint4 *>(a.value + t * a.value_stride + h * a.D + d);
    const int64_t dst = (slot * a.Hkv + h) * a.D + d;
    *reinterpret_cast<uint4 *>(a.key_cache + dst) = kv;
    *reinterpret_cast<uint4 *>(a.value_cache + dst) = vv;
  }
}

// ------------------------------------------------------------------------
// Attention arguments shared by the kernels
// ------------------------------------------------------------------------
struct AttnArgs {
  const uint16_t *q;
  int64_t q_stride;
  const uint16_t *kc;
  const uint16_t *vc;
  uint16_t *out;
  int64_t o_stride;
  const int32_t *tables;
  int64_t table_stride;
  const int32_t *computed;
  const int32_t *qsl;
  const int32_t *req;
  const uint8_t *vis;        // null = linear layouts
  const int32_t *vis_start;  // per request
  int Hq, Hkv, D, bs;
  float scale_log2;  // softmax scale * log2(e)
  // split-context decode
  float *part_o;    // [num_seqs][Hq][max_splits][D]
  float *part_lse;  // [num_seqs][Hq][max_splits]
  int max_splits;
  int chunk_tokens;  // multiple of 16
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------------
// General kernel
// ------------------------------------------------------------------------
template <bool kBf16, int DPL>
__global__ void __launch_bounds__(128) paged_attn_general_kernel(const AttnArgs a) {
  constexpr int kWarps = 4;
  __shared__ float q_sm[32 * DPL];
  __shared__ float m_sm[kWarps];
  __shared__ float l_sm[kWarps];
  __shared__ float o_sm[kWarps][32 * DPL];

  const int t = blockIdx.x;
  const int h = blockIdx.y;
  const int kvh = h / (a.Hq / a.Hkv);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int D = a.D;

  const int r = a.req[t];
  const int qs = a.qsl[r];
  const int qoff = t - qs;
  const int qlen = a.qsl[r + 1] - qs;
  const int c = a.computed[r];
  const int end = c + (a.vis != nullptr ? qlen : qoff + 1);
  const uint8_t *vis_row = a.vis != nullptr ? a.vis + a.vis_start[r] + static_cast<int64_t>(qoff) * qlen : nullptr;
  const int32_t *table = a.tables + static_cast<int64_t>(r) * a.table_stride;

  for (int d = threadIdx.x; d < 32 * DPL; d += blockDim.x)
    q_sm[d] = d < D ? to_float<kBf16>(a.q[t * a.q_stride + static_cast<int64_t>(h) * D + d]) : 0.f;
  __syncthreads();

  float m_run = -INFINITY;
  float l_run = 0.f;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;

  for (int base = warp * 32; base < end; base += kWarps * 32) {
    const int p = base + lane;
    bool valid = p < end;
    if (valid && p >= c) valid = vis_row != nullptr ? vis_row[p - c] != 0 : (p - c) <= qoff;
    int64_t row = 0;
    float s = -INFINITY;
    if (valid) {
      const int64_t block = table[p / a.bs];
      row = ((block * a.bs + p % a.bs) * a.Hkv + kvh) * D;
      const uint16_t *kp = a.kc + row;
      float dot = 0.f;
      for (int d = 0; d < D; d += 8) {
        const uint4 v = *reinterpret_cast<const uint4 *>(kp + d);
        const uint16_t *e = reinterpret_cast<const uint16_t *>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(to_float<kBf16>(e[i]), q_sm[d + i], dot);
      }
      s = dot * a.scale_log2;
    }
    const float m_new = fmaxf(m_run, warp_max(s));
    if (m_new == -INFINITY) continue;  // nothing visible in this chunk yet
    const float pr = valid ? exp2f(s - m_new) : 0.f;
    const float alpha = exp2f(m_run - m_new);
    l_run = l_run * alpha + warp_sum(pr);
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
    for (int jj = 0; jj < 32; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, pr, jj);
      if (pj == 0.f) continue;
      const int64_t rj = __shfl_sync(0xffffffffu, row, jj);
      const uint16_t *vp = a.vc + rj;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int d = lane * DPL + i;
        if (d < D) acc[i] = fmaf(pj, to_float<kBf16>(vp[d]), acc[i]);
      }
    }
    m_run = m_new;
  }

  if (lane == 0) {
    m_sm[warp] = m_run;
    l_sm[warp] = l_run;
  }
#pragma unroll
  for (int i = 0; i < DPL; ++i) o_sm[warp][lane * DPL + i] = acc[i];
  __syncthreads();
  float m_all = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) m_all = fmaxf(m_all, m_sm[w]);
  float wgt[kWarps];
  float l_all = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    wgt[w] = m_sm[w] == -INFINITY ? 0.f : exp2f(m_sm[w] - m_all);
    l_all += wgt[w] * l_sm[w];
  }
  const float inv = 1.f / l_all;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) o += wgt[w] * o_sm[w][d];
    a.out[t * a.o_stride + static_cast<int64_t>(h) * D + d] = from_float<kBf16>(o * inv);
  }
}

// ------------------------------------------------------------------------
// Split-context decode kernel
// ------------------------------------------------------------------------
constexpr int kDecodeStages = 8;
constexpr int kDecodeConsumerWarps = 4;
constexpr int kDecodeThreads = (kDecodeConsumerWarps + 1) * 32;
constexpr int kPageTokens = 16;
constexpr int kBoxBytes = kPageTokens * 128;  // 16 tokens x 64 dims x 2 B

template <int D>
struct DecodeCfg {
  static constexpr int kBoxes = D / 64;                    // boxes per K (and per V) page
  static constexpr int kStageBytes = 2 * kBoxes * kBoxBytes;
  static constexpr int kRingBytes = kDecodeStages * kStageBytes;
  static constexpr int kMergeBytes = kDecodeConsumerWarps * 16 * D * 4;
  static constexpr int kDataBytes = kRingBytes > kMergeBytes ? kRingBytes : kMergeBytes;
  static constexpr int kBarOff = kDataBytes;
  static constexpr int kStatOff = kBarOff + 2 * kDecodeStages * 8 + 16;
  static constexpr int kSmemBytes = kStatOff + 2 * kDecodeConsumerWarps * 16 * 4 + 1024;
};

template <bool kBf16, int D>
__global__ void __launch_bounds__(kDecodeThreads, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const AttnArgs a) {
  using Cfg = DecodeCfg<D>;
  constexpr int kSteps = D / 16;   // k-steps of QK^T, and dim pairs of PV
  constexpr int kNTiles = D / 8;   // 8-dim output tiles
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOff);
  uint64_t *empty = full + kDecodeStages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kDecodeStages);
  float *m_sm = reinterpret_cast<float *>(smem + Cfg::kStatOff);
  float *l_sm = m_sm + kDecodeConsumerWarps * 16;

  const int seq = blockIdx.z;
  const int kvh = blockIdx.y;
  const int split = blockIdx.x;
  const int ctx = a.computed[seq] + 1;
  const int start = split * a.chunk_tokens;
  if (start >= ctx) return;  // uniform for the whole CTA
  const int end = min(ctx, start + a.chunk_tokens);
  const int p_begin = start / kPageTokens;
  const int npages = (end + kPageTokens - 1) / kPageTokens - p_begin;
  const int group = a.Hq / a.Hkv;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int32_t *table = a.tables + static_cast<int64_t>(seq) * a.table_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecodeStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDecodeConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      int issued = 0;
      for (int i = 0; i < npages; ++i) {
        const int s = i % kDecodeStages;
        const uint32_t ph = (i / kDecodeStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) break;
        const int row = table[p_begin + i] * kPageTokens;
        uint8_t *stage = smem + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
#pragma unroll
        for (int b = 0; b < Cfg::kBoxes; ++b) {
          tma_load_3d(stage + b * kBoxBytes, &kmap, &full[s], b * 64, kvh, row);
          tma_load_3d(stage + (Cfg::kBoxes + b) * kBoxBytes, &vmap, &full[s], b * 64, kvh, row);
        }
        issued = i + 1;
      }
      if (*abort_flag) {
        for (int i = issued - kDecodeStages < 0 ? 0 : issued - kDecodeStages; i < issued; ++i)
          mbar_wait(&full[i % kDecodeStages], (i / kDecodeStages) & 1, nullptr, kDrainBudgetCycles);
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kDecodeThreads) : "memory");
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2;   // MMA row (query head within the group), and +8
  const int cq = lane & 3;   // MMA column pair
  const int t = a.qsl[seq];  // packed token of this request's query
  const uint16_t *qrow = a.q + t * a.q_stride + static_cast<int64_t>(kvh) * group * D;
  uint32_t qa[kSteps][4];
#pragma unroll
  for (int ks = 0; ks < kSteps; ++ks) {
    const int d0 = ks * 16 + 2 * cq;
    qa[ks][0] = g < group ? *reinterpret_cast<const uint32_t *>(qrow + g * D + d0) : 0u;
    qa[ks][1] = g + 8 < group ? *reinterpret_cast<const uint32_t *>(qrow + (g + 8) * D + d0) : 0u;
    qa[ks][2] = g < group ? *reinterpret_cast<const uint32_t *>(qrow + g * D + d0 + 8) : 0u;
    qa[ks][3] = g + 8 < group ? *reinterpret_cast<const uint32_t *>(qrow + (g + 8) * D + d0 + 8) : 0u;
  }
  float o[kNTiles][4];
#pragma unroll
  for (int i = 0; i < kNTiles; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const uint32_t ring = smem_u32(smem);
  // ldmatrix row assignment: matrix mi = lane / 8, row rr = lane % 8.
  const int mi = lane >> 3;
  const int rr = lane & 7;
  bool ok = true;

  for (int i = warp; i < npages; i += kDecodeConsumerWarps) {
    const int s = i % kDecodeStages;
    const uint32_t ph = (i / kDecodeStages) & 1;
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, abort_flag))) { ok = false; break; }
    const uint32_t kbase = ring + s * Cfg::kStageBytes;
    const uint32_t vbase = kbase + Cfg::kBoxes * kBoxBytes;

    // S = Q K^T for the 16 tokens of the page (two 8-token MMA tiles).
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < kSteps; ++ks) {
      const int tok = (mi >> 1) * 8 + rr;
      const int chunk = (ks & 3) * 2 + (mi & 1);
      const uint32_t addr = kbase + (ks >> 2) * kBoxBytes + tok * 128 + ((chunk ^ (tok & 7)) << 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(addr, b0, b1, b2, b3);
      mma_16816<kBf16>(sc[0], qa[ks], b0, b1);
      mma_16816<kBf16>(sc[1], qa[ks], b2, b3);
    }
    // Online softmax (rows g and g + 8; columns = tokens 8 * nt + 2 * cq + {0, 1}).
    const int pos0 = (p_begin + i) * kPageTokens + 2 * cq;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int pos = pos0 + nt * 8 + (e & 1);
        const float v = pos < end ? sc[nt][e] * a.scale_log2 : -INFINITY;
        sc[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
      const float m_new = fmaxf(m_run[hr], mx[hr]);
      alpha[hr] = exp2f(m_run[hr] - m_new);
      m_run[hr] = m_new;
      l_run[hr] *= alpha[hr];
    }
    uint32_t pa_hi[4], pa_lo[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const float p0 = exp2f(sc[nt][2 * hr] - m_run[hr]);
        const float p1 = exp2f(sc[nt][2 * hr + 1] - m_run[hr]);
        l_run[hr] += p0 + p1;
        const uint32_t hi = pack2<kBf16>(p0, p1);
        float h0, h1;
        if constexpr (kBf16) {
          h0 = __uint_as_float(hi << 16);
          h1 = __uint_as_float(hi & 0xFFFF0000u);
        } else {
          const __half2 hh = *reinterpret_cast<const __half2 *>(&hi);
          h0 = __low2float(hh);
          h1 = __high2float(hh);
        }
        pa_hi[nt * 2 + hr] = hi;
        pa_lo[nt * 2 + hr] = pack2<kBf16>(p0 - h0, p1 - h1);
      }
    }
#pragma unroll
    for (int n = 0; n < kNTiles; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // O += P V: A = P (rows = heads, k = the page's 16 tokens).
#pragma unroll
    for (int dp = 0; dp < kSteps; ++dp) {
      const int tok = (mi & 1) * 8 + rr;
      const int chunk = (dp & 3) * 2 + (mi >> 1);
      const uint32_t addr = vbase + (dp >> 2) * kBoxBytes + tok * 128 + ((chunk ^ (tok & 7)) << 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_trans(addr, b0, b1, b2, b3);
      mma_16816<kBf16>(o[2 * dp], pa_hi, b0, b1);
      mma_16816<kBf16>(o[2 * dp], pa_lo, b0, b1);
      mma_16816<kBf16>(o[2 * dp + 1], pa_hi, b2, b3);
      mma_16816<kBf16>(o[2 * dp + 1], pa_lo, b2, b3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // Row sums are spread over the 4 lanes of a row group.
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 1);
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 2);
  }
  // All consumers and the producer meet before the ring is reused.
  asm volatile("bar.sync 1, %0;" ::"n"(kDecodeThreads) : "memory");
  ok = ok && !*abort_flag;

  float *o_sm = reinterpret_cast<float *>(smem);  // [warp][16 rows][D]
  if (cq == 0) {
    m_sm[warp * 16 + g] = m_run[0];
    m_sm[warp * 16 + g + 8] = m_run[1];
    l_sm[warp * 16 + g] = l_run[0];
    l_sm[warp * 16 + g + 8] = l_run[1];
  }
#pragma unroll
  for (int n = 0; n < kNTiles; ++n) {
    const int d = n * 8 + 2 * cq;
    float *row0 = o_sm + (warp * 16 + g) * D;
    float *row1 = o_sm + (warp * 16 + g + 8) * D;
    row0[d] = o[n][0];
    row0[d + 1] = o[n][1];
    row1[d] = o[n][2];
    row1[d + 1] = o[n][3];
  }
  asm volatile("bar.sync 2, %0;" ::"n"(kDecodeConsumerWarps * 32) : "memory");
  if (!ok) return;

  // Merge the four warps; write this split's normalised output and lse.
  const int tid = threadIdx.x;
  for (int idx = tid; idx < group * D; idx += kDecodeConsumerWarps * 32) {
    const int row = idx / D;
    const int d = idx - row * D;
    float m_all = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeConsumerWarps; ++w) m_all = fmaxf(m_all, m_sm[w * 16 + row]);
    float l_all = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeConsumerWarps; ++w) {
      const float mw = m_sm[w * 16 + row];
      const float wt = mw == -INFINITY ? 0.f : exp2f(mw - m_all);
      l_all += wt * l_sm[w * 16 + row];
      acc += wt * o_sm[(w * 16 + row) * D + d];
    }
    const int h = kvh * group + row;
    const int64_t base = (static_cast<int64_t>(seq) * a.Hq + h) * a.max_splits + split;
    a.part_o[base * D + d] = acc / l_all;
    if (d == 0) a.part_lse[base] = m_all + log2f(l_all);
  }
}

// Combine the context splits of each (request, query head).
template <bool kBf16>
__global__ void paged_merge_kernel(const AttnArgs a) {
  const int seq = blockIdx.x;
  const int h = blockIdx.y;
  const int ctx = a.computed[seq] + 1;
  const int nsplit = (ctx + a.chunk_tokens - 1) / a.chunk_tokens;
  const int64_t base = (static_cast<int64_t>(seq) * a.Hq + h) * a.max_splits;
  float m_all = -INFINITY;
  for (int s = 0; s < nsplit; ++s) m_all = fmaxf(m_all, a.part_lse[base + s]);
  float wsum = 0.f;
  for (int s = 0; s < nsplit; ++s) wsum += exp2f(a.part_lse[base + s] - m_all);
  const float inv = 1.f / wsum;
  const int t = a.qsl[seq];
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s)
      acc += exp2f(a.part_lse[base + s] - m_all) * a.part_o[(base + s) * a.D + d];
    a.out[t * a.o_stride + static_cast<int64_t>(h) * a.D + d] = from_float<kBf16>(acc * inv);
  }
}

}  // namespace attn
}  // namespace lvb
