// Element-wise steps of a Qwen2 decoder layer that sit between the AWQ
// projections and the attention on sm_100a:
//   * rope_qk: Qwen2 half-rotation RoPE applied in place to the query and key
//     heads of the merged QKV projection output (reference Triton kernel
//     modeling/models/_qwen2_kernels.py:66-133, called from qwen2.py:411):
//       out[i]       = x[i] * cos[p][i]       - x[i + D/2] * sin[p][i]
//       out[i + D/2] = x[i + D/2] * cos[p][i + D/2] + x[i] * sin[p][i + D/2]
//     in fp32 from fp16 x and fp16 cos/sin tables, stored as fp16.
//   * silu_mul: act = silu(gate) * up over the merged gate/up output
//     (reference _qwen2_kernels.py:45-64, 183-202): fp32 arithmetic, one
//     fp16 rounding.
// Both are HBM-bound and tiny next to the projections; rows are read and
// written with 16-byte vectors where the layout allows.
#pragma once

#include "lvb_common.cuh"

namespace lvb {
namespace q2 {

constexpr int kRopeThreads = 256;
constexpr int kSiluThreads = 256;

struct RopeArgs {
  uint16_t *qkv;          // [tokens][row_stride] fp16; query heads at column 0, key heads after them
  int64_t row_stride;     // elements
  const int32_t *positions;
  const uint16_t *cos, *sin;  // [table_rows][D] fp16
  int tokens, hq, hkv, D, table_rows;
};

// kVec: 8 pairs per step with 16-byte loads (D % 16 == 0, 16-byte aligned
// rows and tables); otherwise one pair per step.
template <bool kVec>
__global__ void __launch_bounds__(kRopeThreads) rope_qk_kernel(const __grid_constant__ RopeArgs a) {
  pdl_entry();
  const int t = blockIdx.x;
  const int pos = a.positions[t];
  if (pos < 0 || pos >= a.table_rows) {
    if (threadIdx.x == 0) record_device_error(LVB_DEVERR_INDEX);
    return;
  }
  const int half = a.D / 2;
  const __half *cs = reinterpret_cast<const __half *>(a.cos) + static_cast<size_t>(pos) * a.D;
  const __half *sn = reinterpret_cast<const __half *>(a.sin) + static_cast<size_t>(pos) * a.D;
  __half *row = reinterpret_cast<__half *>(a.qkv) + static_cast<size_t>(t) * a.row_stride;
  if constexpr (kVec) {
    const int per_head = half / 8;
    const int units = (a.hq + a.hkv) * per_head;
    for (int u = threadIdx.x; u < units; u += kRopeThreads) {
      const int head = u / per_head, i = (u - head * per_head) * 8;
      __half *x = row + static_cast<size_t>(head) * a.D;
      const uint4 xa = *reinterpret_cast<const uint4 *>(x + i);
      const uint4 xb = *reinterpret_cast<const uint4 *>(x + i + half);
      const uint4 ca = *reinterpret_cast<const uint4 *>(cs + i);
      const uint4 cb = *reinterpret_cast<const uint4 *>(cs + i + half);
      const uint4 sa = *reinterpret_cast<const uint4 *>(sn + i);
      const uint4 sb = *reinterpret_cast<const uint4 *>(sn + i + half);
      const __half *x1 = reinterpret_cast<const __half *>(&xa), *x2 = reinterpret_cast<const __half *>(&xb);
      const __half *c1 = reinterpret_cast<const __half *>(&ca), *c2 = reinterpret_cast<const __half *>(&cb);
      const __half *s1 = reinterpret_cast<const __half *>(&sa), *s2 = reinterpret_cast<const __half *>(&sb);
      uint4 oa, ob;
      __half *o1 = reinterpret_cast<__half *>(&oa), *o2 = reinterpret_cast<__half *>(&ob);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v1 = __half2float(x1[e]), v2 = __half2float(x2[e]);
        o1[e] = __float2half_rn(rope_rotate(v1, __half2float(c1[e]), -v2, __half2float(s1[e])));
        o2[e] = __float2half_rn(rope_rotate(v2, __half2float(c2[e]), v1, __half2float(s2[e])));
      }
      *reinterpret_cast<uint4 *>(x + i) = oa;
      *reinterpret_cast<uint4 *>(x + i + half) = ob;
    }
  } else {
    const int units = (a.hq + a.hkv) * half;
    for (int u = threadIdx.x; u < units; u += kRopeThreads) {
      const int head = u / half, i = u - head * half;
      __half *x = row + static_cast<size_t>(head) * a.D;
      const float x1 = __half2float(x[i]);
      const float x2 = __half2float(x[i + half]);
      const float o1 = rope_rotate(x1, __half2float(cs[i]), -x2, __half2float(sn[i]));
      const float o2 = rope_rotate(x2, __half2float(cs[i + half]), x1, __half2float(sn[i + half]));
      x[i] = __float2half_rn(o1);
      x[i + half] = __float2half_rn(o2);
    }
  }
}

// RoPE fused with the paged K/V write (the QKV epilogue steps of
// qwen2.py:380-411 and triton_paged_attention.py:31-104): per token, the query
// heads are rotated in place (the attention reads them from the QKV rows), the
// key heads are rotated into the token's cache slot, the value heads copied
// there.  Slot of token t: request r = req[t], position computed[r] + t -
// qsl[r] in r's block table; RoPE position: positions[t].  D % 16 == 0,
// 16-byte aligned rows, tables and cache.
struct RopeKVArgs {
  uint16_t *qkv;
  int64_t row_stride;
  const int32_t *positions;
  const uint16_t *cos, *sin;
  uint16_t *key_cache, *value_cache;  // [blocks][bs][hkv][D]
  const int32_t *tables;
  int64_t table_stride;
  const int32_t *computed, *qsl, *req;
  int tokens, hq, hkv, D, bs, table_rows;
};

__device__ __forceinline__ void rope8(const uint4 xa, const uint4 xb, const uint4 ca, const uint4 cb, const uint4 sa,
                                      const uint4 sb, uint4 &oa, uint4 &ob) {
  const __half *x1 = reinterpret_cast<const __half *>(&xa), *x2 = reinterpret_cast<const __half *>(&xb);
  const __half *c1 = reinterpret_cast<const __half *>(&ca), *c2 = reinterpret_cast<const __half *>(&cb);
  const __half *s1 = reinterpret_cast<const __half *>(&sa), *s2 = reinterpret_cast<const __half *>(&sb);
  __half *o1 = reinterpret_cast<__half *>(&oa), *o2 = reinterpret_cast<__half *>(&ob);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float v1 = __half2float(x1[e]), v2 = __half2float(x2[e]);
    o1[e] = __float2half_rn(rope_rotate(v1, __half2float(c1[e]), -v2, __half2float(s1[e])));
    o2[e] = __float2half_rn(rope_rotate(v2, __half2float(c2[e]), v1, __half2float(s2[e])));
  }
}

__global__ void __launch_bounds__(kRopeThreads) rope_kv_write_kernel(const __grid_constant__ RopeKVArgs a) {
  pdl_entry();
  const int t = blockIdx.x;
  const int pos = a.positions[t];
  if (pos < 0 || pos >= a.table_rows) {
    if (threadIdx.x == 0) record_device_error(LVB_DEVERR_INDEX);
    return;
  }
  const int r = a.req[t];
  const int p = a.computed[r] + (t - a.qsl[r]);
  const int64_t slot = static_cast<int64_t>(a.tables[static_cast<int64_t>(r) * a.table_stride + p / a.bs]) * a.bs + p % a.bs;
  const int half = a.D / 2;
  const int per_head = half / 8;
  const __half *cs = reinterpret_cast<const __half *>(a.cos) + static_cast<size_t>(pos) * a.D;
  const __half *sn = reinterpret_cast<const __half *>(a.sin) + static_cast<size_t>(pos) * a.D;
  __half *row = reinterpret_cast<__half *>(a.qkv) + static_cast<size_t>(t) * a.row_stride;
  __half *kc = reinterpret_cast<__half *>(a.key_cache) + static_cast<size_t>(slot) * a.hkv * a.D;
  __half *vc = reinterpret_cast<__half *>(a.value_cache) + static_cast<size_t>(slot) * a.hkv * a.D;
  const int rope_units = (a.hq + a.hkv) * per_head;
  const int v_units = a.hkv * (a.D / 8);
  for (int u = threadIdx.x; u < rope_units + v_units; u += kRopeThreads) {
    if (u < rope_units) {
      const int head = u / per_head, i = (u - head * per_head) * 8;
      const __half *x = row + static_cast<size_t>(head) * a.D;
      uint4 oa, ob;
      rope8(*reinterpret_cast<const uint4 *>(x + i), *reinterpret_cast<const uint4 *>(x + i + half),
            *reinterpret_cast<const uint4 *>(cs + i), *reinterpret_cast<const uint4 *>(cs + i + half),
            *reinterpret_cast<const uint4 *>(sn + i), *reinterpret_cast<const uint4 *>(sn + i + half), oa, ob);
      __half *dst = head < a.hq ? row + static_cast<size_t>(head) * a.D : kc + static_cast<size_t>(head - a.hq) * a.D;
      *reinterpret_cast<uint4 *>(dst + i) = oa;
      *reinterpret_cast<uint4 *>(dst + i + half) = ob;
    } else {
      const int v = u - rope_units;
      const int h = v / (a.D / 8), d = (v - h * (a.D / 8)) * 8;
      *reinterpret_cast<uint4 *>(vc + static_cast<size_t>(h) * a.D + d) =
          *reinterpret_cast<const uint4 *>(row + static_cast<size_t>(a.hq + a.hkv + h) * a.D + d);
    }
  }
}

struct SiluArgs {
  const uint16_t *gate_up;  // [tokens][in_stride]: gate in columns [0, I), up in [I, 2I)
  int64_t in_stride;
  uint16_t *out;            // [tokens][out_stride], columns [0, I)
  int64_t out_stride;
  int tokens, inter;
};


// I % 8 == 0 and 16-byte aligned rows: one 16-byte vector per thread-step.
__global__ void __launch_bounds__(kSiluThreads) silu_mul_kernel(const __grid_constant__ SiluArgs a) {
  pdl_entry();
  const int vecs = a.inter / 8;
  const size_t total = static_cast<size_t>(a.tokens) * vecs;
  for (size_t i = static_cast<size_t>(blockIdx.x) * kSiluThreads + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * kSiluThreads) {
    const int t = static_cast<int>(i / vecs), c = static_cast<int>(i - static_cast<size_t>(t) * vecs);
    const uint4 gv = *reinterpret_cast<const uint4 *>(a.gate_up + static_cast<size_t>(t) * a.in_stride + c * 8);
    const uint4 uv = *reinterpret_cast<const uint4 *>(a.gate_up + static_cast<size_t>(t) * a.in_stride + a.inter + c * 8);
    const __half2 *g = reinterpret_cast<const __half2 *>(&gv);
    const __half2 *u = reinterpret_cast<const __half2 *>(&uv);
    uint4 ov;
    __half2 *o = reinterpret_cast<__half2 *>(&ov);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 gf = __half22float2(g[e]), uf = __half22float2(u[e]);
      o[e] = __floats2half2_rn(silu_times(gf.x, uf.x), silu_times(gf.y, uf.y));
    }
    *reinterpret_cast<uint4 *>(a.out + static_cast<size_t>(t) * a.out_stride + c * 8) = ov;
  }
}

// ------------------------------------------------------------------------
// Greedy head and embedding
// ------------------------------------------------------------------------
// lm_head_argmax: for each of up to kHeadMaxTokens hidden rows, the greedy
// pick over this rank's vocabulary rows: logit[t][v] = fp16(sum_k h[t][k] W[v][k])
// (fp32 accumulation rounded to fp16, the value F.linear hands to argmax in
// the reference, qwen2.py:665-673, sampling.py:103-112), its maximum and the
// lowest vocabulary index holding it -- without writing the logits.  Each warp
// streams one weight row at a time (16-byte loads, the row read once), the
// hidden rows sit in shared memory as fp32; per token the best (value, index)
// folds into one 64-bit key (orderable value bits, then the complemented
// index so equal values keep the lowest index) by atomicMax, and the last
// CTA to finish turns the keys into indices and values and clears them.
constexpr int kHeadThreads = 256;
constexpr int kHeadMaxTokens = 4;

struct HeadArgs {
  const uint16_t *hidden;  // [tokens][hidden_stride] fp16
  int64_t hidden_stride;
  const uint16_t *weight;  // [vocab][H] fp16 (nn.Linear layout)
  int tokens, H, V;
  int64_t vocab_offset;    // global index of local row 0
  unsigned long long *keys;  // [kHeadMaxTokens], zero between calls
  unsigned int *counter;     // zero between calls
  int64_t *out_index;        // [tokens]
  float *out_value;          // [tokens] or null
};

__device__ __forceinline__ unsigned long long head_key(float v, int row) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(row));
}

__device__ __forceinline__ float head_value(unsigned long long key) {
  uint32_t b = static_cast<uint32_t>(key >> 32);
  b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
  return __uint_as_float(b);
}

template <int TOK>
__global__ void __launch_bounds__(kHeadThreads) lm_head_argmax_kernel(const __grid_constant__ HeadArgs a) {
  extern __shared__ __align__(16) float head_sm[];  // [TOK][H] fp32
  __shared__ unsigned long long best_sm[kHeadThreads / 32][TOK];
  __shared__ int last_sm;
  pdl_entry();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = a.H / 8;
  for (int i = threadIdx.x; i < TOK * chunks; i += kHeadThreads) {
    const int t = i / chunks, c = i - t * chunks;
    const uint4 v = *reinterpret_cast<const uint4 *>(a.hidden + static_cast<size_t>(t) * a.hidden_stride + c * 8);
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
    float4 *dst = reinterpret_cast<float4 *>(head_sm + static_cast<size_t>(t) * a.H + c * 8);
    const float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]), f2 = __half22float2(h[2]),
                 f3 = __half22float2(h[3]);
    dst[0] = make_float4(f0.x, f0.y, f1.x, f1.y);
    dst[1] = make_float4(f2.x, f2.y, f3.x, f3.y);
  }
  __syncthreads();
  unsigned long long best[TOK];
#pragma unroll
  for (int t = 0; t < TOK; ++t) best[t] = 0ull;
  const int warps = gridDim.x * (kHeadThreads / 32);
  for (int row = blockIdx.x * (kHeadThreads / 32) + warp; row < a.V; row += warps) {
    const uint4 *w = reinterpret_cast<const uint4 *>(a.weight + static_cast<size_t>(row) * a.H);
    float acc[TOK];
#pragma unroll
    for (int t = 0; t < TOK; ++t) acc[t] = 0.f;
#pragma unroll 4
    for (int c = lane; c < chunks; c += 32) {
      uint4 wv;
      asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(wv.x), "=r"(wv.y), "=r"(wv.z), "=r"(wv.w)
                   : "l"(w + c));
      const __half2 *wh = reinterpret_cast<const __half2 *>(&wv);
      float wf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(wh[e]);
        wf[2 * e] = f.x;
        wf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int t = 0; t < TOK; ++t) {
        const float4 *hp = reinterpret_cast<const float4 *>(head_sm + static_cast<size_t>(t) * a.H + c * 8);
        const float4 h0 = hp[0], h1 = hp[1];
        acc[t] = fmaf(wf[0], h0.x, acc[t]);
        acc[t] = fmaf(wf[1], h0.y, acc[t]);
        acc[t] = fmaf(wf[2], h0.z, acc[t]);
        acc[t] = fmaf(wf[3], h0.w, acc[t]);
        acc[t] = fmaf(wf[4], h1.x, acc[t]);
        acc[t] = fmaf(wf[5], h1.y, acc[t]);
        acc[t] = fmaf(wf[6], h1.z, acc[t]);
        acc[t] = fmaf(wf[7], h1.w, acc[t]);
      }
    }
#pragma unroll
    for (int t = 0; t < TOK; ++t) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
      const unsigned long long k = head_key(__half2float(__float2half_rn(acc[t])), row);
      best[t] = k > best[t] ? k : best[t];
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < TOK; ++t) best_sm[warp][t] = best[t];
  }
  __syncthreads();
  if (threadIdx.x < TOK && threadIdx.x < a.tokens) {
    unsigned long long k = 0ull;
    for (int w = 0; w < kHeadThreads / 32; ++w) k = best_sm[w][threadIdx.x] > k ? best_sm[w][threadIdx.x] : k;
    atomicMax(a.keys + threadIdx.x, k);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_sm = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last_sm) return;
  __threadfence();
  if (threadIdx.x < a.tokens) {
    const unsigned long long k = atomicExch(a.keys + threadIdx.x, 0ull);
    a.out_index[threadIdx.x] = a.vocab_offset + static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(k));
    if (a.out_value != nullptr) a.out_value[threadIdx.x] = head_value(k);
  }
  if (threadIdx.x == 0) *a.counter = 0u;
}

// Token embedding rows (one CTA per token, 16-byte copies): out[t] =
// table[ids[t] - vocab_start] when vocab_start <= ids[t] < vocab_end, else
// zeros (the masked lookup of a vocab-parallel shard, tensor_parallel.py:
// 296-306; the row sum over ranks is the fused all-reduce that follows).
__global__ void __launch_bounds__(128) embedding_kernel(const int64_t *__restrict__ ids,
                                                        const uint16_t *__restrict__ table, int64_t vocab_start,
                                                        int64_t vocab_end, int H, uint16_t *__restrict__ out,
                                                        int64_t out_stride) {
  pdl_entry();
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  const bool owned = id >= vocab_start && id < vocab_end;
  const uint4 *src = reinterpret_cast<const uint4 *>(table + (owned ? (id - vocab_start) : 0) * H);
  uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<int64_t>(t) * out_stride);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = owned ? src[c] : make_uint4(0u, 0u, 0u, 0u);
}

}  // namespace q2
}  // namespace lvb
