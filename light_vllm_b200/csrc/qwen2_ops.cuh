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
        o1[e] = __float2half_rn(v1 * __half2float(c1[e]) + (-v2) * __half2float(s1[e]));
        o2[e] = __float2half_rn(v2 * __half2float(c2[e]) + v1 * __half2float(s2[e]));
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
      const float o1 = x1 * __half2float(cs[i]) + (-x2) * __half2float(sn[i]);
      const float o2 = x2 * __half2float(cs[i + half]) + x1 * __half2float(sn[i + half]);
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
    o1[e] = __float2half_rn(v1 * __half2float(c1[e]) + (-v2) * __half2float(s1[e]));
    o2[e] = __float2half_rn(v2 * __half2float(c2[e]) + v1 * __half2float(s2[e]));
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

}  // namespace q2
}  // namespace lvb
