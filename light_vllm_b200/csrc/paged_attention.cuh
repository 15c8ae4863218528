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
//     one CTA per (request, group of up to 4 KV heads, context split).  Warp h
//     owns KV head h of the group for every page of the split: its 32 lanes
//     stream the head's 16-token K and V pages with 16-byte cp.async copies
//     (two rows of 256 contiguous bytes per instruction) into the warp's own
//     shared-memory ring, in the 128-byte-swizzled layout that ldmatrix reads
//     without bank conflicts; completion is tracked per slot by an mbarrier
//     that the copies themselves arrive on.  The warp runs QK^T and PV for its
//     whole GQA group as 16-row warp MMAs (the up-to-16 query heads are the
//     MMA's M dimension), with an fp32 online softmax in registers.  P enters the PV product as a hi + lo pair
//     of 16-bit values so the probabilities keep fp32-like precision.  Each
//     split writes its normalised output and log2-sum-exp; the last split of a
//     request (per-request semaphore) merges them.
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
  // Writes of the step's new positions let the attention launch early (it
  // reads older positions before waiting); explicit slots may be any
  // positions, so then the next launch starts only after this one ends.
  if (a.slots == nullptr) pdl_launch_dependents();
  pdl_wait();
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
  // decode launch order, null = index order: [num_seqs] requests (longest
  // context first), then [num_seqs] their num_computed in that order
  const int32_t *order;
  const uint8_t *vis;        // null = linear layouts
  const int32_t *vis_start;  // per request
  int Hq, Hkv, D, bs;
  float scale_log2;  // softmax scale * log2(e)
  // split-context decode
  float *part_o;    // [num_seqs][Hq][max_splits][D]
  float *part_lse;  // [num_seqs][Hq][max_splits]
  uint32_t *merge_count;  // [num_seqs][Hkv], zero between calls
  int max_splits;
  int chunk_tokens;  // multiple of 16
  int num_seqs;
  int decode_seqs;   // balanced decode schedule: requests (launch order slots 0 .. decode_seqs - 1)
  // split decode kernel: the step's K/V rows ([tokens][Hkv][D], token
  // strides in elements), stored to the newest position's cache slot by the
  // warp that loads that page; null = already in the cache
  const uint16_t *new_k, *new_v;
  int64_t new_k_stride, new_v_stride;
  int heads_per_cta; // balanced decode schedule: KV heads per CTA (merge_count holds pieces per head group)
  // prefill tile kernel: requests order[first_tile_req + blockIdx.y] (the
  // packer lists one-token requests first; the decode kernel serves those), or
  // blockIdx.y itself when order is null
  int first_tile_req;
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

// KV compaction move (tree acceptance): rows of every (slot, head) listed in
// src move to the matching dst slot.  One CTA per (KV head, K or V) stages all
// of its source rows in shared memory before writing any target, so the moves
// may overlap (a target slot that is also a later source).  head_size % 8 == 0.
__global__ void __launch_bounds__(128) kv_move_rows_kernel(uint16_t *__restrict__ key_cache,
                                                           uint16_t *__restrict__ value_cache,
                                                           const int32_t *__restrict__ src,
                                                           const int32_t *__restrict__ dst, int n, int hkv, int d) {
  extern __shared__ __align__(16) uint8_t move_smem[];
  // Moves rows to older positions: no early launch of the next kernel (the
  // decode attention reads older positions before its dependency wait).
  pdl_wait();
  uint4 *rows = reinterpret_cast<uint4 *>(move_smem);
  uint16_t *base = blockIdx.y == 0 ? key_cache : value_cache;
  const int head = blockIdx.x;
  const int vec = d / 8;  // 16-byte vectors per row
  const size_t slot_elems = static_cast<size_t>(hkv) * d;
  for (int i = threadIdx.x; i < n * vec; i += blockDim.x) {
    const int r = i / vec, c = i - r * vec;
    rows[i] = *reinterpret_cast<const uint4 *>(base + static_cast<size_t>(src[r]) * slot_elems + head * d + c * 8);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n * vec; i += blockDim.x) {
    const int r = i / vec, c = i - r * vec;
    *reinterpret_cast<uint4 *>(base + static_cast<size_t>(dst[r]) * slot_elems + head * d + c * 8) = rows[i];
  }
}

// ------------------------------------------------------------------------
// General kernel
// ------------------------------------------------------------------------
template <bool kBf16, int DPL>
__global__ void __launch_bounds__(128) paged_attn_general_kernel(const AttnArgs a) {
  pdl_entry();
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
// Prefill / mixed / tree attention on warp MMAs
// ------------------------------------------------------------------------
// One CTA per (64-row tile, request, KV head).  The rows of a request and KV
// head are its (query token, query head of the GQA group) pairs, token-major:
// row R is token R / G, head R % G.  Four warps take 16 rows each, so one CTA
// covers the whole group for ~64 / G consecutive tokens and every K/V
// position it needs is staged once in shared memory for all of them (the
// reference's grouped Triton kernel shares pages across the group the same
// way, runtime/execution/triton_paged_attention.py:248-391).  K/V stream in
// tiles of 32 positions (two 16-token pages) through a 3-stage cp.async ring,
// 128-byte-swizzled rows that ldmatrix reads without bank conflicts; S = Q K^T
// and O += P V are m16n8k16 warp MMAs with an fp32 online softmax per row.  P
// enters P V in the cache dtype, as a hi + lo pair for bf16 (as in the decode
// kernel).  Visibility: the computed prefix always; inside the query block
// the causal chain, or the request's visibility matrix (tree layouts).
// Positions past a tile's last visible one are not read (zero-filled), so
// never-written cache slots (possibly NaN) never enter P V.
template <int D>
struct PrefillCfg {
  static constexpr int kWarps = 4;
  static constexpr int kRows = 16 * kWarps;
  static constexpr int kTilePos = 32;                     // K/V positions per stage
  static constexpr int kStages = 3;
  static constexpr int kHalfBytes = kTilePos * 128;       // one 64-dim half of a K or V tile
  static constexpr int kKVBytes = (D / 64) * kHalfBytes;  // a K (or V) tile
  static constexpr int kStageBytes = 2 * kKVBytes;        // K then V
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  static constexpr int kChunks = kTilePos * (D / 8);      // 16-byte chunks of a K (or V) tile
};

template <bool kBf16, int D>
__global__ void __launch_bounds__(128) paged_prefill_kernel(const AttnArgs a) {
  pdl_entry();
  using Cfg = PrefillCfg<D>;
  constexpr int kSteps = D / 16;  // k-steps of QK^T, dim pairs of PV
  constexpr int kNTiles = D / 8;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t ring = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int seq = a.order != nullptr ? a.order[a.first_tile_req + blockIdx.y] : static_cast<int>(blockIdx.y);
  const int kvh = blockIdx.z;
  const int G = a.Hq / a.Hkv;
  const int qs = a.qsl[seq];
  const int qlen = a.qsl[seq + 1] - qs;
  const int row0 = blockIdx.x * Cfg::kRows;
  if (row0 >= qlen * G) return;  // uniform for the CTA
  const int c = a.computed[seq];
  const bool tree = a.vis != nullptr;
  const uint8_t *vis = tree ? a.vis + a.vis_start[seq] : nullptr;
  // Last query token of the tile, and the K/V range the tile reads.
  const int last_tok = min(qlen * G, row0 + Cfg::kRows) - 1;
  const int kv_end = c + (tree ? qlen : last_tok / G + 1);
  const int ntiles = (kv_end + Cfg::kTilePos - 1) / Cfg::kTilePos;
  const int32_t *table = a.tables + static_cast<int64_t>(seq) * a.table_stride;
  const int64_t row_elems = static_cast<int64_t>(a.Hkv) * D;
  const int64_t head_off = static_cast<int64_t>(kvh) * D;

  // Stage loader: thread i copies 16-byte chunks i, i + 128, ... of the K and
  // V tiles; positions at or past kv_end are zero-filled.
  auto load_stage = [&](int tile, int slot) {
    const uint32_t kdst = ring + slot * Cfg::kStageBytes;
    const uint32_t vdst = kdst + Cfg::kKVBytes;
#pragma unroll
    for (int u = 0; u < Cfg::kChunks / 128; ++u) {
      const int q = threadIdx.x + 128 * u;
      const int tok = q / (D / 8);
      const int c16 = q - tok * (D / 8);
      const int pos = tile * Cfg::kTilePos + tok;
      const uint32_t off = (c16 >> 3) * Cfg::kHalfBytes + tok * 128 + (((c16 & 7) ^ (tok & 7)) << 4);
      const bool ok = pos < kv_end;
      int64_t src = head_off;
      if (ok) {
        const int64_t block = table[pos >> 4];  // 16-token pages
        src = (block * 16 + (pos & 15)) * row_elems + head_off + c16 * 8;
      }
      cp_async_16(kdst + off, a.kc + src, ok ? 16u : 0u);
      cp_async_16(vdst + off, a.vc + src, ok ? 16u : 0u);
    }
  };
#pragma unroll
  for (int s = 0; s < Cfg::kStages - 1; ++s) {
    if (s < ntiles) load_stage(s, s);
    cp_async_commit();
  }

  // This warp's rows g and g + 8 of the MMA tile.
  const int g = lane >> 2;
  const int cq = lane & 3;
  int tok_r[2], head_r[2];
  bool row_ok[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int R = row0 + warp * 16 + g + 8 * hr;
    row_ok[hr] = R < qlen * G;
    tok_r[hr] = row_ok[hr] ? R / G : 0;
    head_r[hr] = row_ok[hr] ? R - (R / G) * G : 0;
  }
  uint32_t qa[kSteps][4];
  {
    const uint16_t *q0 = a.q + static_cast<int64_t>(qs + tok_r[0]) * a.q_stride +
                         static_cast<int64_t>(kvh * G + head_r[0]) * D;
    const uint16_t *q1 = a.q + static_cast<int64_t>(qs + tok_r[1]) * a.q_stride +
                         static_cast<int64_t>(kvh * G + head_r[1]) * D;
#pragma unroll
    for (int ks = 0; ks < kSteps; ++ks) {
      const int d0 = ks * 16 + 2 * cq;
      qa[ks][0] = row_ok[0] ? *reinterpret_cast<const uint32_t *>(q0 + d0) : 0u;
      qa[ks][1] = row_ok[1] ? *reinterpret_cast<const uint32_t *>(q1 + d0) : 0u;
      qa[ks][2] = row_ok[0] ? *reinterpret_cast<const uint32_t *>(q0 + d0 + 8) : 0u;
      qa[ks][3] = row_ok[1] ? *reinterpret_cast<const uint32_t *>(q1 + d0 + 8) : 0u;
    }
  }
  float o[kNTiles][4];
#pragma unroll
  for (int i = 0; i < kNTiles; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int mi = lane >> 3;
  const int rr = lane & 7;

  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait_group<Cfg::kStages - 2>();
    __syncthreads();  // stage `it` landed for every thread; the slot of it - 1 is free
    if (it + Cfg::kStages - 1 < ntiles) load_stage(it + Cfg::kStages - 1, (it + Cfg::kStages - 1) % Cfg::kStages);
    cp_async_commit();
    const uint32_t kbase = ring + (it % Cfg::kStages) * Cfg::kStageBytes;
    const uint32_t vbase = kbase + Cfg::kKVBytes;

    // S = Q K^T over the stage's 32 positions (four 8-position MMA tiles).
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kSteps; ++ks) {
#pragma unroll
      for (int pp = 0; pp < 2; ++pp) {
        const int tok = pp * 16 + (mi >> 1) * 8 + rr;
        const int chunk = (ks & 3) * 2 + (mi & 1);
        const uint32_t addr = kbase + (ks >> 2) * Cfg::kHalfBytes + tok * 128 + ((chunk ^ (tok & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma_16816<kBf16>(sc[2 * pp], qa[ks], b0, b1);
        mma_16816<kBf16>(sc[2 * pp + 1], qa[ks], b2, b3);
      }
    }
    // Visibility and the online softmax (rows g, g + 8).
    const int pos0 = it * Cfg::kTilePos + 2 * cq;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const int pos = pos0 + nt * 8 + (e & 1);
        bool visible = row_ok[hr] && pos < kv_end;
        if (visible && pos >= c) {
          const int j = pos - c;
          visible = tree ? (j < qlen && vis[static_cast<int64_t>(tok_r[hr]) * qlen + j] != 0) : j <= tok_r[hr];
        }
        const float v = visible ? sc[nt][e] * a.scale_log2 : -INFINITY;
        sc[nt][e] = v;
        mx[hr] = fmaxf(mx[hr], v);
      }
    }
    float alpha[2], m_use[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
      const float m_new = fmaxf(m_run[hr], mx[hr]);
      m_use[hr] = m_new == -INFINITY ? 0.f : m_new;  // a row with nothing visible yet
      alpha[hr] = exp2f(m_run[hr] - m_use[hr]);
      m_run[hr] = m_new;
      l_run[hr] *= alpha[hr];
    }
#pragma unroll
    for (int n = 0; n < kNTiles; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // O += P V, two 16-position k-steps.
#pragma unroll
    for (int kp = 0; kp < 2; ++kp) {
      uint32_t pa_hi[4], pa_lo[4];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int nt = 2 * kp + half;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const float p0 = exp2f(sc[nt][2 * hr] - m_use[hr]);
          const float p1 = exp2f(sc[nt][2 * hr + 1] - m_use[hr]);
          l_run[hr] += p0 + p1;
          const uint32_t hi = pack2<kBf16>(p0, p1);
          pa_hi[half * 2 + hr] = hi;
          if constexpr (kBf16) {
            const float h0 = __uint_as_float(hi << 16);
            const float h1 = __uint_as_float(hi & 0xFFFF0000u);
            pa_lo[half * 2 + hr] = pack2<kBf16>(p0 - h0, p1 - h1);
          }
        }
      }
#pragma unroll
      for (int dp = 0; dp < kSteps; ++dp) {
        const int tok = kp * 16 + (mi & 1) * 8 + rr;
        const int chunk = (dp & 3) * 2 + (mi >> 1);
        const uint32_t addr = vbase + (dp >> 2) * Cfg::kHalfBytes + tok * 128 + ((chunk ^ (tok & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(addr, b0, b1, b2, b3);
        mma_16816<kBf16>(o[2 * dp], pa_hi, b0, b1);
        mma_16816<kBf16>(o[2 * dp + 1], pa_hi, b2, b3);
        if constexpr (kBf16) {
          mma_16816<kBf16>(o[2 * dp], pa_lo, b0, b1);
          mma_16816<kBf16>(o[2 * dp + 1], pa_lo, b2, b3);
        }
      }
    }
  }
  cp_async_wait_all();

#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 1);
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 2);
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    if (!row_ok[hr]) continue;
    const float inv = l_run[hr] > 0.f ? 1.f / l_run[hr] : 0.f;
    uint16_t *dst = a.out + static_cast<int64_t>(qs + tok_r[hr]) * a.o_stride +
                    static_cast<int64_t>(kvh * G + head_r[hr]) * D;
#pragma unroll
    for (int n = 0; n < kNTiles; ++n)
      *reinterpret_cast<uint32_t *>(dst + n * 8 + 2 * cq) = pack2<kBf16>(o[n][2 * hr] * inv, o[n][2 * hr + 1] * inv);
  }
}

// ------------------------------------------------------------------------
// Split-context decode kernel
// ------------------------------------------------------------------------
constexpr int kPageTokens = 16;
constexpr int kBoxBytes = kPageTokens * 128;  // one TMA box: 16 tokens x 64 dims of one head

// HPC = KV heads per CTA, KW = warps per head (KW > 1 only with HPC = 1:
// the warps of a CTA share one head's pages round-robin and merge their
// partial softmax results in shared memory), D = head size.
template <int D, int HPC, int KW = 1>
struct DecodeCfg {
  static_assert(KW == 1 || HPC == 1, "several warps per head only with one head per CTA");
  static constexpr int kBoxes = D / 64;                  // 64-dim halves of a head's row
  static constexpr int kHeadBytes = kBoxes * kBoxBytes;  // one head's 16-token K (or V) page
  static constexpr int kPageBytes = 2 * kHeadBytes;      // K then V
  static constexpr int kWarps = HPC * KW;
  // Page ring per CTA: 96 KB for 2-4 heads or 4 warps on one head; a one-warp
  // CTA keeps 32 KB so that more of them fit on an SM (B = 16, ctx 1024:
  // 21.9 -> 17.1 us on B200).
  static constexpr int kRingBudget = kWarps == 1 ? 32 * 1024 : 96 * 1024;
  static constexpr int kFit = kRingBudget / (kWarps * kPageBytes);
  static constexpr int kStages = kFit < 2 ? 2 : (kFit > 8 ? 8 : kFit);  // per-warp ring depth
  static constexpr int kWarpRing = kStages * kPageBytes;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kBarOff = kWarps * kWarpRing;
  static constexpr int kSmemBytes = kBarOff + kWarps * kStages * 8 + 16 + 1024;
  // Cross-warp merge scratch (KW > 1), reusing the ring: (m, l) per warp and
  // head, then the scaled outputs [KW][up to 16 heads][D] fp32.
  static constexpr int kMergeObufOff = 1024;
  static_assert(KW == 1 || kMergeObufOff + KW * 16 * D * 4 <= kBarOff, "merge scratch (16 heads) fits in the ring");
  static_assert(kWarps * 16 * (D + 4) * 4 <= kBarOff, "output staging (16 heads per warp) fits in the ring");
};

// Decode math of one warp over one (request, KV head): the page's 16 tokens
// on the MMA's M dimension and the GQA group's query heads on N (NT tiles of
// 8 heads), so a group of up to 8 heads fills the N = 8 tile instead of
// padding M = 16 rows:
//   S^T = K Q^T      A = K (16 tokens x 16 dims, ldmatrix), B = Q^T (registers)
//   O^T += V^T P^T   A = V^T (ldmatrix.trans), B = P^T
// P^T leaves the first MMA in the accumulator layout (lane 4 r + c: tokens r
// and r + 8, heads 2 c and 2 c + 1) and enters the second as the B operand
// (tokens 2 c, 2 c + 1, head r): one movmatrix.trans per 8 x 8 block.
// Per 16-token page and 8 heads: kSteps MMAs for S and kSteps (fp16) or
// 2 kSteps (bf16: P as hi + lo) for O.  Each lane holds two heads' running
// max / sum (its partial sum over its tokens; summed over the lanes with the
// same column by finish()) and O^T rows g and g + 8 of every 16-dim m-tile.
template <bool kBf16, int D, int NT>
struct TokMath {
  static constexpr int kSteps = D / 16;  // k-steps of K Q^T; 16-dim m-tiles of V^T P^T
  uint32_t qb[kSteps][NT][2];
  float o[kSteps][NT][4];
  float m_run[NT][2], l_run[NT][2];

  // q_head0: the group's first query head (heads are D apart).
  __device__ __forceinline__ void load_q(const uint16_t *q_head0, int group) {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int h = nt * 8 + g;
      const uint16_t *qr = q_head0 + static_cast<int64_t>(h) * D + 2 * cq;
#pragma unroll
      for (int ks = 0; ks < kSteps; ++ks) {
        qb[ks][nt][0] = h < group ? *reinterpret_cast<const uint32_t *>(qr + ks * 16) : 0u;
        qb[ks][nt][1] = h < group ? *reinterpret_cast<const uint32_t *>(qr + ks * 16 + 8) : 0u;
      }
    }
  }

  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int mt = 0; mt < kSteps; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.f;
    }
  }

  // One page: K and V as two 64-dim boxes each in shared memory (16-byte
  // chunks XOR-swizzled by the token row); pos0 = position of token row 0;
  // positions >= end are masked.  Every page holds at least one position
  // below end, so each head's running max is finite after it.
  __device__ __forceinline__ void page(uint32_t kbase, uint32_t vbase, int pos0, int end, float scale_log2) {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int mi = lane >> 3, rr = lane & 7;
    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kSteps; ++ks) {
      // a0: tokens 0-7 of the k-step's low 8 dims, a1: tokens 8-15, a2 / a3: the high 8 dims.
      const int tok = (mi & 1) * 8 + rr;
      const int chunk = (ks & 3) * 2 + (mi >> 1);
      uint32_t a[4];
      ldsm_x4(kbase + (ks >> 2) * kBoxBytes + tok * 128 + ((chunk ^ (tok & 7)) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_16816_nv<kBf16>(s[nt], a, qb[ks][nt][0], qb[ks][nt][1]);
    }
    const bool ok0 = pos0 + g < end, ok1 = pos0 + g + 8 < end;
    uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float p[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float v0 = ok0 ? s[nt][j] * scale_log2 : -INFINITY;      // token g, head 2 cq + j
        const float v1 = ok1 ? s[nt][2 + j] * scale_log2 : -INFINITY;  // token g + 8
        float mx = fmaxf(v0, v1);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[nt][j], mx);
        const float alpha = exp2f(m_run[nt][j] - m_new);
        m_run[nt][j] = m_new;
        p[j] = exp2f(v0 - m_new);
        p[2 + j] = exp2f(v1 - m_new);
        l_run[nt][j] = l_run[nt][j] * alpha + p[j] + p[2 + j];
#pragma unroll
        for (int mt = 0; mt < kSteps; ++mt) {
          o[mt][nt][j] *= alpha;
          o[mt][nt][2 + j] *= alpha;
        }
      }
      // P enters the MMA in the cache dtype.  bf16 keeps 8 mantissa bits, so
      // its rounding error is carried by a second MMA on the remainder (hi +
      // lo ~ 16 bits); fp16 P (11 bits) is used as is, as the reference's
      // Triton kernel does (tl.dot on fp16 p).
      const uint32_t h0 = pack2<kBf16>(p[0], p[1]);  // tokens 0-7 block, row g
      const uint32_t h1 = pack2<kBf16>(p[2], p[3]);  // tokens 8-15 block
      bh[nt][0] = movmatrix_trans(h0);
      bh[nt][1] = movmatrix_trans(h1);
      if constexpr (kBf16) {
        const uint32_t l0 = pack2<kBf16>(p[0] - __uint_as_float(h0 << 16), p[1] - __uint_as_float(h0 & 0xFFFF0000u));
        const uint32_t l1 = pack2<kBf16>(p[2] - __uint_as_float(h1 << 16), p[3] - __uint_as_float(h1 & 0xFFFF0000u));
        bl[nt][0] = movmatrix_trans(l0);
        bl[nt][1] = movmatrix_trans(l1);
      }
    }
#pragma unroll
    for (int mt = 0; mt < kSteps; ++mt) {
      // a0: dims 0-7 of the m-tile x tokens 0-7 (transposed), a1: dims 8-15,
      // a2 / a3: tokens 8-15.
      const int tok = (mi >> 1) * 8 + rr;
      const int chunk = (mt & 3) * 2 + (mi & 1);
      uint32_t a[4];
      ldsm_x4_trans(vbase + (mt >> 2) * kBoxBytes + tok * 128 + ((chunk ^ (tok & 7)) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_16816_nv<kBf16>(o[mt][nt], a, bh[nt][0], bh[nt][1]);
        if constexpr (kBf16) mma_16816_nv<kBf16>(o[mt][nt], a, bl[nt][0], bl[nt][1]);
      }
    }
  }

  // Sum the lanes' partial softmax denominators (lanes 4 r + c, same c).
  __device__ __forceinline__ void finish() {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float l = l_run[nt][j];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_run[nt][j] = l;
      }
  }

  // Normalised output rows of the group's heads (after finish()): out_head0
  // is head 0's row, heads D apart.
  __device__ __forceinline__ void store(uint16_t *out_head0, int group) const {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int h = nt * 8 + 2 * cq + j;
        if (h >= group) continue;
        const float inv = 1.f / l_run[nt][j];
        uint16_t *dst = out_head0 + static_cast<int64_t>(h) * D + g;
#pragma unroll
        for (int mt = 0; mt < kSteps; ++mt) {
          dst[mt * 16] = from_float<kBf16>(o[mt][nt][j] * inv);
          dst[mt * 16 + 8] = from_float<kBf16>(o[mt][nt][2 + j] * inv);
        }
      }
  }

  // Rows of the staging area used by store_staged: D floats plus 4 of
  // padding, so the lanes' fragment writes (heads 2 c + j, dims g) hit 32
  // distinct banks.
  static constexpr int kStageRow = D + 4;
  static constexpr int kStageBytes = NT * 8 * kStageRow * 4;

  // The normalised output of the group's heads (after finish()) through this
  // warp's `stage` (kStageBytes of shared memory, 16-byte aligned): written
  // as fragments, read back as rows, stored with 16-byte stores -- fp32
  // partial rows at part_o + (head_base + h) * stride * D (kPartial; the
  // log2-sum-exp at part_lse + (head_base + h) * stride), else the output
  // rows in the cache dtype at out_head0 + h * D.
  template <bool kPartial>
  __device__ __forceinline__ void store_staged(float *stage, uint16_t *out_head0, float *part_o, float *part_lse,
                                               int64_t head_base, int64_t stride, int group) const {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int h = nt * 8 + 2 * cq + j;
        const float inv = h < group ? 1.f / l_run[nt][j] : 0.f;
        float *row = stage + h * kStageRow + g;
#pragma unroll
        for (int mt = 0; mt < kSteps; ++mt) {
          row[mt * 16] = o[mt][nt][j] * inv;
          row[mt * 16 + 8] = o[mt][nt][2 + j] * inv;
        }
        if (kPartial && g == 0 && h < group) __stcg(part_lse + (head_base + h) * stride, m_run[nt][j] + log2f(l_run[nt][j]));
      }
    __syncwarp();
    constexpr int kPer = kPartial ? 4 : 8;  // values per 16-byte store
    constexpr int kChunks = D / kPer;
    for (int idx = lane; idx < group * kChunks; idx += 32) {
      const int h = idx / kChunks;
      const int c = idx - h * kChunks;
      const float *src = stage + h * kStageRow + c * kPer;
      if constexpr (kPartial) {
        __stcg(reinterpret_cast<float4 *>(part_o + (head_base + h) * stride * D) + c,
               *reinterpret_cast<const float4 *>(src));
      } else {
        const float4 v0 = *reinterpret_cast<const float4 *>(src);
        const float4 v1 = *reinterpret_cast<const float4 *>(src + 4);
        uint4 w;
        w.x = pack2<kBf16>(v0.x, v0.y);
        w.y = pack2<kBf16>(v0.z, v0.w);
        w.z = pack2<kBf16>(v1.x, v1.y);
        w.w = pack2<kBf16>(v1.z, v1.w);
        *reinterpret_cast<uint4 *>(out_head0 + static_cast<int64_t>(h) * D + c * 8) = w;
      }
    }
  }

  // A split's normalised output and log2-sum-exp: head h's row at
  // part_o + (head_base + h) * stride * D, its lse at part_lse + (head_base +
  // h) * stride (stride = the workspace's splits per head, offset by split).
  __device__ __forceinline__ void store_partial(float *part_o, float *part_lse, int64_t head_base, int64_t stride,
                                                int group) const {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, cq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int h = nt * 8 + 2 * cq + j;
        if (h >= group) continue;
        const float inv = 1.f / l_run[nt][j];
        const int64_t row = (head_base + h) * stride;
        float *dst = part_o + row * D + g;
#pragma unroll
        for (int mt = 0; mt < kSteps; ++mt) {
          __stcg(dst + mt * 16, o[mt][nt][j] * inv);
          __stcg(dst + mt * 16 + 8, o[mt][nt][2 + j] * inv);
        }
        if (g == 0) __stcg(part_lse + row, m_run[nt][j] + log2f(l_run[nt][j]));
      }
  }
};

// Combines the nsplit partial results of `rows` consecutive query heads
// (head0 = request * Hq + first head) into out_row: each split's normalised
// output and log2-sum-exp sit in part_o / part_lse at split index 0 ..
// nsplit - 1.  All kThreads threads of the CTA call it; w_sm holds rows x
// nsplit floats of shared memory.
template <bool kBf16, int D, int kThreads>
__device__ __forceinline__ void merge_partials(const AttnArgs &a, int64_t head0, int rows, int nsplit, float *w_sm,
                                               uint16_t *out_row) {
  const int tid = threadIdx.x;
  // Split weights first (log2-sum-exp -> normalised weights, in shared memory
  // reused from the ring), then the weighted sum with independent loads.
  for (int idx = tid; idx < rows * nsplit; idx += kThreads) {
    const int row = idx / nsplit;
    const int sp = idx - row * nsplit;
    w_sm[idx] = __ldcg(a.part_lse + (head0 + row) * a.max_splits + sp);
  }
  asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory");
  for (int row = tid; row < rows; row += kThreads) {
    float m_all = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) m_all = fmaxf(m_all, w_sm[row * nsplit + sp]);
    float wsum = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float wt = exp2f(w_sm[row * nsplit + sp] - m_all);
      w_sm[row * nsplit + sp] = wt;
      wsum += wt;
    }
    const float inv = 1.f / wsum;
    for (int sp = 0; sp < nsplit; ++sp) w_sm[row * nsplit + sp] *= inv;
  }
  asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory");
  // Weighted sum over the splits.  The partials sit in L2 (written moments
  // ago), so the cost is round trips, not bytes: each thread keeps
  // kMergeOuts float4 outputs x kMergeSplits splits = 16 independent loads in
  // flight per round trip.  Splits are summed in order for every output, so
  // the result does not depend on the thread mapping.
  constexpr int kMergeOuts = 4;
  constexpr int kMergeSplits = 4;
  constexpr int kQuads = D / 4;
  const int total4 = rows * kQuads;
  for (int base = tid; base < total4; base += kThreads * kMergeOuts) {
    float4 acc[kMergeOuts];
    const float4 *src[kMergeOuts];
    const float *wrow[kMergeOuts];
#pragma unroll
    for (int j = 0; j < kMergeOuts; ++j) {
      acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int idx = base + j * kThreads;
      const int row = (idx < total4 ? idx : 0) / kQuads;
      const int q4 = (idx < total4 ? idx : 0) - row * kQuads;
      src[j] = reinterpret_cast<const float4 *>(a.part_o + (head0 + row) * a.max_splits * D) + q4;
      wrow[j] = w_sm + row * nsplit;
    }
    for (int sp0 = 0; sp0 < nsplit; sp0 += kMergeSplits) {
      float4 v[kMergeOuts][kMergeSplits];
#pragma unroll
      for (int j = 0; j < kMergeOuts; ++j)
#pragma unroll
        for (int s = 0; s < kMergeSplits; ++s)
          v[j][s] = (sp0 + s < nsplit && base + j * kThreads < total4) ? __ldcg(src[j] + (sp0 + s) * kQuads)
                                                                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kMergeOuts; ++j)
#pragma unroll
        for (int s = 0; s < kMergeSplits; ++s) {
          const float wt = sp0 + s < nsplit ? wrow[j][sp0 + s] : 0.f;
          acc[j].x = fmaf(wt, v[j][s].x, acc[j].x);
          acc[j].y = fmaf(wt, v[j][s].y, acc[j].y);
          acc[j].z = fmaf(wt, v[j][s].z, acc[j].z);
          acc[j].w = fmaf(wt, v[j][s].w, acc[j].w);
        }
    }
#pragma unroll
    for (int j = 0; j < kMergeOuts; ++j) {
      const int idx = base + j * kThreads;
      if (idx >= total4) continue;
      const int row = idx / kQuads;
      const int q4 = idx - row * kQuads;
      uint32_t *dst = reinterpret_cast<uint32_t *>(out_row + row * D + 4 * q4);
      dst[0] = pack2<kBf16>(acc[j].x, acc[j].y);
      dst[1] = pack2<kBf16>(acc[j].z, acc[j].w);
    }
  }
}

template <bool kBf16, int D, int HPC, int KW = 1, int NT = 1>
__global__ void __launch_bounds__(DecodeCfg<D, HPC, KW>::kThreads, 2)
    paged_decode_kernel(const AttnArgs a) {
  // The previous kernel of the stream may still run: this CTA reads the step
  // metadata and the pages wholly before the request's newest position
  // (written by earlier steps, never by a kernel still running -- this
  // library's K/V writers that let the next launch start early write only
  // the step's new positions) before waiting for it; q, the page holding the
  // newest position and the outputs come after the wait.
  pdl_launch_dependents();
  using Cfg = DecodeCfg<D, HPC, KW>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kSteps = D / 16;  // 16-dim m-tiles of the output
  constexpr int kConsumers = Cfg::kThreads;
  constexpr int kChunksPerLane = Cfg::kHeadBytes / 16 / 32;  // 16-byte copies per lane for K (and V)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t *ready = reinterpret_cast<uint64_t *>(smem + Cfg::kBarOff) + warp * kStages;
  volatile int *abort_flag =
      reinterpret_cast<volatile int *>(reinterpret_cast<uint64_t *>(smem + Cfg::kBarOff) + Cfg::kWarps * kStages);
  volatile int *last_flag = abort_flag + 1;

  // Requests in launch order: the block scheduler starts CTAs in blockIdx
  // order, so putting the longest contexts first leaves the short requests'
  // splits for the end, where they fill the SMs that free up (B200, BASELINE
  // config 2, same data: index order 65.1 us, longest first 62.8, shortest
  // first 66.5).
  // With an order, the request and its context length are two independent
  // loads (the packed order carries the lengths), not a dependent pair.
  const int z = blockIdx.z;
  const int seq = a.order != nullptr ? a.order[z] : z;
  const int ctx = (a.order != nullptr ? a.order[a.num_seqs + z] : a.computed[z]) + 1;
  const int hg = blockIdx.y;  // group of HPC KV heads
  const int split = blockIdx.x;
  const int start = split * a.chunk_tokens;
  if (start >= ctx) return;  // uniform for the whole CTA
  const int end = min(ctx, start + a.chunk_tokens);
  const int p_begin = start / kPageTokens;
  const int npages = (end + kPageTokens - 1) / kPageTokens - p_begin;
  const int group = a.Hq / a.Hkv;
  const int32_t *table = a.tables + static_cast<int64_t>(seq) * a.table_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kWarps * kStages; ++s)
      mbar_init(reinterpret_cast<uint64_t *>(smem + Cfg::kBarOff) + s, 32);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // ---------------- each warp: KV head hg * HPC + warp, every page ----------------
  // (KW > 1: every warp on head hg, pages wsub, wsub + KW, ...)
  const int kvh = KW == 1 ? hg * HPC + warp : hg;
  const int wsub = KW == 1 ? 0 : warp;
  const int my_pages = npages > wsub ? (npages - wsub + KW - 1) / KW : 0;
  const uint32_t ring = smem_u32(smem) + warp * Cfg::kWarpRing;
  const int64_t head_off = static_cast<int64_t>(kvh) * D;
  const int64_t row_elems = static_cast<int64_t>(a.Hkv) * D;  // elements per cache token row
  // Block ids: one per lane, 32 pages at a time, passed around by shuffle.
  int blk_cur = lane < npages ? table[p_begin + lane] : 0;
  int blk_next = 32 + lane < npages ? table[p_begin + 32 + lane] : 0;
  int blk_base = 0;  // page index of blk_cur's lane 0

  // Issue the K and V copies of page `pg` (block id `block`) into `slot`: lane
  // l copies 16-byte chunks l, l + 32, ... of the head's 16 token rows.  Rows
  // at or past the split's end are zero-filled instead of read: their scores
  // are masked, but their V rows still enter P V with weight 0, and a cache
  // slot that was never written may hold NaN bit patterns.
  auto load_page = [&](int pg, int block, int slot) {
    const int valid = end - (p_begin + pg) * kPageTokens;
    const uint32_t kdst = ring + slot * Cfg::kPageBytes;
    const uint32_t vdst = kdst + Cfg::kHeadBytes;
    const int64_t base = static_cast<int64_t>(block) * kPageTokens * row_elems + head_off;
    if (a.new_k != nullptr && valid <= kPageTokens && valid > 0 && end == ctx) {
      // The page holds the request's newest position (ctx - 1): store this
      // step's K/V row of the warp's head into its slot first (this page is
      // only ever loaded after the dependency wait).  Lanes 0 .. D/8 - 1 copy
      // K, the next D/8 lanes V, 16 bytes each.
      const int64_t t = a.qsl[seq];
      const int64_t row = base + static_cast<int64_t>(valid - 1) * row_elems;
      if (lane < D / 8)
        *reinterpret_cast<uint4 *>(const_cast<uint16_t *>(a.kc) + row + lane * 8) =
            *reinterpret_cast<const uint4 *>(a.new_k + t * a.new_k_stride + head_off + lane * 8);
      else if (lane < D / 4)
        *reinterpret_cast<uint4 *>(const_cast<uint16_t *>(a.vc) + row + (lane - D / 8) * 8) =
            *reinterpret_cast<const uint4 *>(a.new_v + t * a.new_v_stride + head_off + (lane - D / 8) * 8);
      __threadfence_block();
      __syncwarp();
    }
#pragma unroll
    for (int u = 0; u < kChunksPerLane; ++u) {
      const int q = lane + 32 * u;                  // chunk of this head's page
      const int tok = q / (D / 8);                   // D / 8 chunks per token row
      const int c16 = q - tok * (D / 8);
      const int half = c16 >> 3;
      const int c = c16 & 7;
      const uint32_t off = half * kBoxBytes + tok * 128 + ((c ^ (tok & 7)) << 4);
      const int64_t src = base + tok * row_elems + c16 * 8;
      const uint32_t bytes = tok < valid ? 16u : 0u;
      cp_async_16(kdst + off, a.kc + (bytes ? src : head_off), bytes);
      cp_async_16(vdst + off, a.vc + (bytes ? src : head_off), bytes);
    }
    cp_async_arrive_noinc(&ready[slot]);
  };
  auto block_of = [&](int pg) {
    // Pages are requested in increasing order; refill the per-lane batch when
    // the request moves past it (the batch after it was prefetched).
    while (pg >= blk_base + 32) {
      blk_cur = blk_next;
      blk_base += 32;
      blk_next = blk_base + 32 + lane < npages ? table[p_begin + blk_base + 32 + lane] : 0;
    }
    return __shfl_sync(0xffffffffu, blk_cur, pg - blk_base);
  };

  bool waited = false;
#pragma unroll 1
  for (int j = 0; j < kStages - 1 && j < my_pages; ++j) {
    const int pg = wsub + j * KW;
    if (!waited && (p_begin + pg + 1) * kPageTokens >= ctx) {
      pdl_wait();
      waited = true;
    }
    load_page(pg, block_of(pg), j % kStages);
  }
  if (!waited) pdl_wait();

  const int g = lane >> 2;  // MMA row group
  const int cq = lane & 3;  // MMA column pair
  const int t = a.qsl[seq];
  TokMath<kBf16, D, NT> mth;
  mth.load_q(a.q + t * a.q_stride + static_cast<int64_t>(kvh) * group * D, group);
  mth.reset();
  bool ok = true;

  for (int i = 0; i < my_pages; ++i) {
    // Keep kStages - 1 pages in flight: the slot refilled here held this
    // warp's previous page, which it finished in the previous iteration.
    if (i + kStages - 1 < my_pages) {
      const int pg_next = wsub + (i + kStages - 1) * KW;
      load_page(pg_next, block_of(pg_next), (i + kStages - 1) % kStages);
    }
    const int pg = wsub + i * KW;
    const int s = i % kStages;
    const uint32_t ph = (i / kStages) & 1;
    if (!__all_sync(0xffffffffu, mbar_wait(&ready[s], ph, abort_flag))) { ok = false; break; }
    const uint32_t kbase = ring + s * Cfg::kPageBytes;
    mth.page(kbase, kbase + Cfg::kHeadBytes, (p_begin + pg) * kPageTokens, end, a.scale_log2);
    __syncwarp();
  }
  cp_async_wait_all();
  mth.finish();
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
  if (!ok || *abort_flag) return;  // a failed wait raised the (CTA-wide) abort flag

  if constexpr (KW > 1) {
    // Merge the warps' partial softmax results: rescale each to the heads'
    // common maximum, sum in shared memory; warp 0 carries the result.
    constexpr int kHeads = NT * 8;
    float *ml = reinterpret_cast<float *>(smem);  // [KW][kHeads][2]: (m, l)
    float *obuf = reinterpret_cast<float *>(smem + Cfg::kMergeObufOff);  // [KW][kHeads][D]
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int h = nt * 8 + 2 * cq + j;
          ml[(warp * kHeads + h) * 2] = mth.m_run[nt][j];
          ml[(warp * kHeads + h) * 2 + 1] = mth.l_run[nt][j];
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int h = nt * 8 + 2 * cq + j;
        float m_all = -INFINITY;
#pragma unroll
        for (int w = 0; w < KW; ++w) m_all = fmaxf(m_all, ml[(w * kHeads + h) * 2]);
        float l_all = 0.f;
#pragma unroll
        for (int w = 0; w < KW; ++w) {
          const float mw = ml[(w * kHeads + h) * 2];
          l_all += mw == -INFINITY ? 0.f : ml[(w * kHeads + h) * 2 + 1] * exp2f(mw - m_all);
        }
        const float sc = mth.m_run[nt][j] == -INFINITY ? 0.f : exp2f(mth.m_run[nt][j] - m_all);
        float *ob = obuf + static_cast<int64_t>(warp * kHeads + h) * D + g;
#pragma unroll
        for (int mt = 0; mt < kSteps; ++mt) {
          ob[mt * 16] = mth.o[mt][nt][j] * sc;
          ob[mt * 16 + 8] = mth.o[mt][nt][2 + j] * sc;
        }
        mth.m_run[nt][j] = m_all;
        mth.l_run[nt][j] = l_all;
      }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
    if (warp == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int h = nt * 8 + 2 * cq + j;
#pragma unroll
          for (int mt = 0; mt < kSteps; ++mt) {
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int w = 0; w < KW; ++w) {
              const float *ob = obuf + static_cast<int64_t>(w * kHeads + h) * D + g;
              s0 += ob[mt * 16];
              s1 += ob[mt * 16 + 8];
            }
            mth.o[mt][nt][j] = s0;
            mth.o[mt][nt][2 + j] = s1;
          }
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");  // scratch free again
  }

  // Each warp writes its own heads: the final output when the request has one
  // split, else this split's normalised output and log2-sum-exp, which
  // decode_merge_kernel (the next launch) combines.  The CTA then ends: a
  // fence, a semaphore and a merge here held the CTA's SM slot, with no page
  // in flight, for about a fifth of the kernel's time on B200 (config 2,
  // pages streamed without the math: 45.2 us without them, 57.3 with).
  const int nsplit = (ctx + a.chunk_tokens - 1) / a.chunk_tokens;
  if (KW == 1 || warp == 0) {
    // Staged through the warp's part of the (now idle) page ring.
    float *stage = reinterpret_cast<float *>(smem + warp * TokMath<kBf16, D, NT>::kStageBytes);
    uint16_t *out_head0 = a.out + t * a.o_stride + static_cast<int64_t>(kvh) * group * D;
    // 16-byte output stores need 16-byte aligned rows (the API asks for 4).
    const bool out16 = ((reinterpret_cast<uintptr_t>(a.out) | static_cast<uintptr_t>(a.o_stride * 2)) & 15u) == 0;
    if (nsplit == 1 && out16)
      mth.template store_staged<false>(stage, out_head0, nullptr, nullptr, 0, 0, group);
    else if (nsplit == 1)
      mth.store(out_head0, group);
    else
      mth.template store_staged<true>(stage, nullptr, a.part_o + static_cast<int64_t>(split) * D, a.part_lse + split,
                                      static_cast<int64_t>(seq) * a.Hq + kvh * group, a.max_splits, group);
  }
}

// Combines the split kernel's partial results: one warp per (query head,
// request in launch order), four heads per CTA (requests with one split were
// written whole).  Lane l holds the log2-sum-exp of splits l, l + 32, ... and
// D / 32 consecutive output values; the weights come from two warp
// reductions and the splits' rows are read eight at a time, summed in split
// order (the result does not depend on the launch shape).  A programmatic
// dependent of the split kernel: it waits for that grid to complete first.
constexpr int kMergeMaxSplits = 256;  // decode_plan's cap
template <bool kBf16, int D, bool kFlat = false>
__global__ void __launch_bounds__(128) decode_merge_kernel(const AttnArgs a) {
  pdl_entry();
  constexpr int kPer = D / 32;  // output values per lane: 4 (D = 128) or 2 (D = 64)
  constexpr int kLse = kMergeMaxSplits / 32;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int z = blockIdx.y;
  if (h >= a.Hq) return;
  const int seq = a.order != nullptr ? a.order[z] : z;
  const int ctx = (a.order != nullptr ? a.order[a.num_seqs + z] : a.computed[z]) + 1;
  // The balanced kernel records each request's piece count (one per KV
  // head group; every group has the same pieces).
  const int nsplit = kFlat ? static_cast<int>(a.merge_count[static_cast<int64_t>(seq) * (a.Hkv / a.heads_per_cta)])
                           : (ctx + a.chunk_tokens - 1) / a.chunk_tokens;
  if (nsplit <= 1) return;
  if (nsplit > a.max_splits || nsplit > kMergeMaxSplits) {
    if (lane == 0) record_device_error(LVB_DEVERR_INDEX);
    return;
  }
  const int64_t row0 = (static_cast<int64_t>(seq) * a.Hq + h) * a.max_splits;
  const float *src = a.part_o + row0 * D + lane * kPer;
  // One round trip for up to kBatch splits: their rows are loaded together
  // with the log2-sum-exps, before the weights are known.
  constexpr int kBatch = 16;
  float v[kBatch][kPer];
  auto load_rows = [&](int s0) {
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int sp = s0 + b;
      if (sp < nsplit) {
        if constexpr (kPer == 4) {
          const float4 t = __ldcg(reinterpret_cast<const float4 *>(src + static_cast<int64_t>(sp) * D));
          v[b][0] = t.x; v[b][1] = t.y; v[b][2] = t.z; v[b][3] = t.w;
        } else {
          const float2 t = __ldcg(reinterpret_cast<const float2 *>(src + static_cast<int64_t>(sp) * D));
          v[b][0] = t.x; v[b][1] = t.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < kPer; ++e) v[b][e] = 0.f;
      }
    }
  };
  float w[kLse];
#pragma unroll
  for (int k = 0; k < kLse; ++k) {
    const int sp = k * 32 + lane;
    w[k] = sp < nsplit ? __ldcg(a.part_lse + row0 + sp) : -INFINITY;
  }
  load_rows(0);
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kLse; ++k) m = fmaxf(m, w[k]);
  m = warp_max(m);
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < kLse; ++k) {
    w[k] = w[k] == -INFINITY ? 0.f : exp2f(w[k] - m);
    sum += w[k];
  }
  const float inv = 1.f / warp_sum(sum);
#pragma unroll
  for (int k = 0; k < kLse; ++k) w[k] *= inv;
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.f;
  // Splits summed in order: s0 = 0, 16, 32, ... (weights by shuffle from
  // lane sp % 32 of register sp / 32).
  for (int s0 = 0; s0 < nsplit; s0 += kBatch) {
    if (s0 > 0) load_rows(s0);
#pragma unroll
    for (int k = 0; k < kLse; ++k) {
      if (k * 32 + 31 < s0 || k * 32 >= s0 + kBatch) continue;
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int sp = s0 + b;
        if (sp / 32 != k) continue;
        const float wt = __shfl_sync(0xffffffffu, w[k], sp & 31);
        if (sp < nsplit) {
#pragma unroll
          for (int e = 0; e < kPer; ++e) acc[e] = fmaf(wt, v[b][e], acc[e]);
        }
      }
    }
  }
  uint16_t *dst = a.out + static_cast<int64_t>(a.qsl[seq]) * a.o_stride + static_cast<int64_t>(h) * D + lane * kPer;
#pragma unroll
  for (int e = 0; e < kPer; e += 2) *reinterpret_cast<uint32_t *>(dst + e) = pack2<kBf16>(acc[e], acc[e + 1]);
}

// ------------------------------------------------------------------------
// Balanced decode schedule
// ------------------------------------------------------------------------
// The split kernel above gives every request the same number of fixed-size
// splits, so a batch of ragged contexts launches many empty CTAs and runs in
// uneven waves.  Here the requests' pages are laid end to end in launch order
// (request z owns flat pages prefix[z] .. prefix[z + 1] - 1) and CTA c takes
// the L flat pages from c L, crossing request boundaries: every CTA but the
// last streams the same number of pages, and the grid is one wave.  A request
// whose pages span several CTAs leaves one partial result per CTA ("piece",
// numbered from the CTA holding its first page); the last piece to finish
// merges them.  One warp per KV head of the CTA's head group.
constexpr int kFlatMinPages = 8;    // fewest pages per CTA: bounds the pieces per request
constexpr int kFlatMaxSeqs = 512;   // requests whose page prefix fits beside the page rings

template <int D, int HPC>
struct FlatCfg {
  using Base = DecodeCfg<D, HPC, 1>;
  // prefix[n + 1], ctx[n], seq[n] (int32) after the barriers and flags
  static constexpr int kTableOff = Base::kBarOff + HPC * Base::kStages * 8 + 16;
  __host__ __device__ static int smem_bytes(int n) { return kTableOff + 12 * (n + 1) + 1024; }
};

// Most pieces a request of max_pages pages can have: a piece holds at least
// one page and every CTA but one holds kFlatMinPages or more.
__host__ __device__ inline int flat_max_pieces(int max_pages) {
  return (max_pages + kFlatMinPages - 1) / kFlatMinPages + 1;
}

template <bool kBf16, int D, int HPC, int NT = 1>
__global__ void __launch_bounds__(HPC * 32, 2) paged_decode_flat_kernel(const AttnArgs a) {
  pdl_entry();
  using Base = DecodeCfg<D, HPC, 1>;
  using Cfg = FlatCfg<D, HPC>;
  constexpr int kStages = Base::kStages;
  constexpr int kThreads = HPC * 32;
  constexpr int kChunksPerLane = Base::kHeadBytes / 16 / 32;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Base::kBarOff);
  uint64_t *ready = bars + warp * kStages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + HPC * kStages);
  volatile int *last_flag = abort_flag + 1;
  const int n = a.decode_seqs;
  int *prefix = reinterpret_cast<int *>(smem + Cfg::kTableOff);  // [n + 1]
  int *ctx_sm = prefix + n + 1;                                   // [n]
  int *seq_sm = ctx_sm + n;                                       // [n]

  for (int z = tid; z < n; z += kThreads) {
    seq_sm[z] = a.order != nullptr ? a.order[z] : z;
    ctx_sm[z] = (a.order != nullptr ? a.order[a.num_seqs + z] : a.computed[z]) + 1;
  }
  if (tid == 0) {
    for (int s = 0; s < HPC * kStages; ++s) mbar_init(bars + s, 32);
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // Exclusive prefix of the page counts: lane l of warp 0 sums a run of
  // requests, one warp scan combines the runs.
  if (warp == 0) {
    const int per = (n + 31) / 32;
    const int z0 = min(n, lane * per);
    const int z1 = min(n, z0 + per);
    int sum = 0;
    for (int z = z0; z < z1; ++z) sum += (ctx_sm[z] + kPageTokens - 1) / kPageTokens;
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
    for (int z = z0; z < z1; ++z) {
      prefix[z] = run;
      run += (ctx_sm[z] + kPageTokens - 1) / kPageTokens;
    }
    if (lane == 31) prefix[n] = incl;
  }
  __syncthreads();
  const int total = prefix[n];
  const int per_cta = max(kFlatMinPages, (total + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x));
  const int g0 = static_cast<int>(blockIdx.x) * per_cta;
  if (g0 >= total) return;  // uniform for the whole CTA
  const int npg = min(total, g0 + per_cta) - g0;
  const int hg = blockIdx.y;
  const int kvh = hg * HPC + warp;
  const int group = a.Hq / a.Hkv;
  const uint32_t ring = smem_u32(smem) + warp * Base::kWarpRing;
  const int64_t head_off = static_cast<int64_t>(kvh) * D;
  const int64_t row_elems = static_cast<int64_t>(a.Hkv) * D;

  // Request slot holding flat page gp (largest z with prefix[z] <= gp; every
  // request has at least one page).
  auto find_req = [&](int gp) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= gp) lo = mid; else hi = mid - 1;
    }
    return lo;
  };
  // Per lane: block id and rows in use of the CTA's page base + lane, for a
  // batch of 32 pages and the batch after it.
  auto fetch = [&](int base, int &blk, int &valid) {
    const int i = base + lane;
    blk = 0;
    valid = 0;
    if (i < npg) {
      const int gp = g0 + i;
      const int z = find_req(gp);
      const int j = gp - prefix[z];
      blk = a.tables[static_cast<int64_t>(seq_sm[z]) * a.table_stride + j];
      valid = ctx_sm[z] - j * kPageTokens;
    }
  };
  int blk_cur, valid_cur, blk_next, valid_next;
  fetch(0, blk_cur, valid_cur);
  fetch(32, blk_next, valid_next);
  int batch_base = 0;

  // Same copy pattern as the split kernel: lane l copies 16-byte chunks l,
  // l + 32, ... of the head's 16 token rows; rows past the request's context
  // are zero-filled (their V rows enter P V with weight 0).
  auto load_page = [&](int i, int slot) {
    while (i >= batch_base + 32) {
      blk_cur = blk_next;
      valid_cur = valid_next;
      batch_base += 32;
      fetch(batch_base + 32, blk_next, valid_next);
    }
    const int block = __shfl_sync(0xffffffffu, blk_cur, i - batch_base);
    const int valid = __shfl_sync(0xffffffffu, valid_cur, i - batch_base);
    const uint32_t kdst = ring + slot * Base::kPageBytes;
    const uint32_t vdst = kdst + Base::kHeadBytes;
    const int64_t base = static_cast<int64_t>(block) * kPageTokens * row_elems + head_off;
#pragma unroll
    for (int u = 0; u < kChunksPerLane; ++u) {
      const int q = lane + 32 * u;
      const int tok = q / (D / 8);
      const int c16 = q - tok * (D / 8);
      const int half = c16 >> 3;
      const int c = c16 & 7;
      const uint32_t off = half * kBoxBytes + tok * 128 + ((c ^ (tok & 7)) << 4);
      const int64_t src = base + tok * row_elems + c16 * 8;
      const uint32_t bytes = tok < valid ? 16u : 0u;
      cp_async_16(kdst + off, a.kc + (bytes ? src : head_off), bytes);
      cp_async_16(vdst + off, a.vc + (bytes ? src : head_off), bytes);
    }
    cp_async_arrive_noinc(&ready[slot]);
  };

#pragma unroll 1
  for (int j = 0; j < kStages - 1 && j < npg; ++j) load_page(j, j);

  TokMath<kBf16, D, NT> mth;
  int z = find_req(g0);
  int seg_first = prefix[z] - g0;  // CTA page index of the request's page 0 (<= 0 for the first segment)
  int seg_end = prefix[z + 1] - g0;
  auto start_segment = [&]() {
    const int seq = seq_sm[z];
    mth.load_q(a.q + static_cast<int64_t>(a.qsl[seq]) * a.q_stride + static_cast<int64_t>(kvh) * group * D, group);
    mth.reset();
  };
  // The segment's output: final rows when the request lies wholly in this
  // CTA, else this CTA's piece (normalised output and log2-sum-exp), which
  // decode_merge_kernel combines.  The CTA holding the request's first page
  // records the request's piece count for it.
  auto finish_segment = [&]() {
    const int seq = seq_sm[z];
    const int first_cta = prefix[z] / per_cta;
    const int pieces = (prefix[z + 1] - 1) / per_cta - first_cta + 1;
    const int piece = static_cast<int>(blockIdx.x) - first_cta;
    mth.finish();
    if (pieces > a.max_splits) {
      if (tid == 0) record_device_error(LVB_DEVERR_INDEX);
      return;
    }
    if (piece == 0 && tid == 0) a.merge_count[seq * (a.Hkv / HPC) + hg] = static_cast<uint32_t>(pieces);
    if (pieces == 1)
      mth.store(a.out + static_cast<int64_t>(a.qsl[seq]) * a.o_stride + static_cast<int64_t>(kvh) * group * D,
                group);
    else
      mth.store_partial(a.part_o + static_cast<int64_t>(piece) * D, a.part_lse + piece,
                        static_cast<int64_t>(seq) * a.Hq + kvh * group, a.max_splits, group);
  };

  start_segment();
  bool ok = true;
  for (int i = 0; i < npg; ++i) {
    if (i + kStages - 1 < npg) load_page(i + kStages - 1, (i + kStages - 1) % kStages);
    if (i == seg_end) {
      finish_segment();
      ++z;
      seg_first = seg_end;
      seg_end = prefix[z + 1] - g0;
      start_segment();
    }
    const int s = i % kStages;
    const uint32_t ph = (i / kStages) & 1;
    if (!__all_sync(0xffffffffu, mbar_wait(&ready[s], ph, abort_flag))) { ok = false; break; }
    const uint32_t kbase = ring + s * Base::kPageBytes;
    mth.page(kbase, kbase + Base::kHeadBytes, (i - seg_first) * kPageTokens, ctx_sm[z], a.scale_log2);
    __syncwarp();
  }
  cp_async_wait_all();
  if (ok) finish_segment();
}

}  // namespace attn
}  // namespace lvb
