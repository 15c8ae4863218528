// Tensor-parallel row-parallel epilogue on sm_100a: one-shot all-reduce of
// the ranks' partial sums over peer memory, fused with the residual add and
// RMSNorm that follow it in a Qwen2 block.
//
// Reference dataflow (modeling/quantization/awq.py:299-304 then
// modeling/models/_qwen2_kernels.py:20-43 via qwen2.py:497-514):
//   h = all_reduce_sum(partial)                 (fp16 tensor)
//   v = fp32(h) + fp32(residual)
//   residual <- fp16(v)
//   out      <- fp16(v * rsqrt(mean(v^2) + eps) * weight)
// Here the sum over ranks is taken in fp32 and rounded to fp16 once (the
// value the reference's all-reduce hands to the norm), then the norm runs in
// fp32 like the reference kernel.
//
// Protocol (world <= 8 ranks, one launch per call, epoch e increasing by one
// per call on every rank):
//   1. every CTA copies its slice of this rank's partial into its own staging
//      buffer e & 1 (peer-readable memory opened through CUDA IPC);
//   2. the last CTA to finish (a per-rank arrival counter) publishes e in
//      flag slot [rank] of every rank's workspace (system-scope release);
//   3. every CTA waits, with a bounded spin, until all flag slots of its own
//      workspace reach e, then reads the ranks' rows with plain peer loads.
// Staging buffers alternate by epoch parity: when a rank writes buffer e & 1
// at call e, every peer has already signalled call e - 1, hence finished call
// e - 2, the last reader of that buffer.  A wait that runs out records
// LVB_DEVERR_TIMEOUT and the CTA leaves its outputs untouched.  The grid is
// at most one CTA per SM, so all its CTAs are resident while they wait.
#pragma once

#include "lvb_common.cuh"

namespace lvb {
namespace ar {

constexpr int kMaxWorld = 8;
constexpr int kThreads = 256;
constexpr int kFlagBytes = 256;     // flags[kMaxWorld] uint32, then the arrival counter at +128
constexpr int kCounterOff = 128;
constexpr int kMaxHidden = 8192;
constexpr int kVec = 8;             // fp16 per 16-byte vector
constexpr int kMaxVecsPerThread = kMaxHidden / (kVec * kThreads);  // 4

struct Args {
  uint8_t *ws[kMaxWorld];   // every rank's workspace base, mapped here (ws[rank] = own)
  int rank, world;
  const uint16_t *partial;  // this rank's partial sums [tokens][hidden]
  uint16_t *residual;       // [tokens][hidden], updated in place
  const uint16_t *weight;   // [hidden]
  uint16_t *out;            // [tokens][hidden]
  int tokens, hidden;
  size_t buf_bytes;         // one staging buffer (max_tokens x hidden fp16)
  float eps;
  uint32_t epoch;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] free from the previous use
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kThreads / 32 ? red[lane] : 0.f;
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return __shfl_sync(0xffffffffu, t, 0);
}

__global__ void __launch_bounds__(kThreads) allreduce_add_rmsnorm_kernel(const __grid_constant__ Args a) {
  __shared__ float red[kThreads / 32];
  __shared__ int ok_sm;
  const int tid = threadIdx.x;
  const size_t buf_off = kFlagBytes + static_cast<size_t>(a.epoch & 1u) * a.buf_bytes;
  uint8_t *own = a.ws[a.rank];
  uint32_t *flags = reinterpret_cast<uint32_t *>(own);
  uint32_t *counter = reinterpret_cast<uint32_t *>(own + kCounterOff);

  // 1. this rank's partial -> own staging buffer
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(a.partial);
    uint4 *dst = reinterpret_cast<uint4 *>(own + buf_off);
    const size_t nvec = static_cast<size_t>(a.tokens) * a.hidden / kVec;
    for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + tid; i < nvec;
         i += static_cast<size_t>(gridDim.x) * kThreads)
      dst[i] = src[i];
  }
  __syncthreads();
  // 2. the last CTA of this rank publishes the epoch to every rank
  if (tid == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(counter, 1u);
    if (prev == gridDim.x - 1) {
      *counter = 0u;  // the next call starts after this grid completes
      __threadfence_system();
      for (int r = 0; r < a.world; ++r) st_release_sys(reinterpret_cast<uint32_t *>(a.ws[r]) + a.rank, a.epoch);
    }
    // 3. wait for every rank's data (bounded)
    int ok = 1;
    const long long start = clock64();
    for (int r = 0; r < a.world && ok; ++r) {
      while (static_cast<int>(ld_acquire_sys(flags + r) - a.epoch) < 0) {
        if (clock64() - start > kWaitBudgetCycles) {
          record_device_error(LVB_DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    ok_sm = ok;
  }
  __syncthreads();
  if (!ok_sm) return;

  // 4. rows: sum over ranks (fp32, rounded to fp16 once), + residual, RMSNorm
  const int nvec_row = a.hidden / kVec;
  for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
    float v[kMaxVecsPerThread][kVec];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxVecsPerThread; ++j) {
      const int c = tid + j * kThreads;
      if (c >= nvec_row) continue;
      const size_t off = (static_cast<size_t>(row) * a.hidden + static_cast<size_t>(c) * kVec) * 2;
      float acc[kVec];
#pragma unroll
      for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
      for (int r = 0; r < a.world; ++r) {
        const uint4 pv = *reinterpret_cast<const uint4 *>(a.ws[r] + buf_off + off);
        const __half2 *h = reinterpret_cast<const __half2 *>(&pv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[2 * e] += __low2float(h[e]);
          acc[2 * e + 1] += __high2float(h[e]);
        }
      }
      const uint4 rv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(a.residual) + off);
      const __half2 *rh = reinterpret_cast<const __half2 *>(&rv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // The reduced hidden state is an fp16 tensor in the reference.
        const float h0 = __half2float(__float2half_rn(acc[2 * e]));
        const float h1 = __half2float(__float2half_rn(acc[2 * e + 1]));
        v[j][2 * e] = h0 + __low2float(rh[e]);
        v[j][2 * e + 1] = h1 + __high2float(rh[e]);
        ss = fmaf(v[j][2 * e], v[j][2 * e], ss);
        ss = fmaf(v[j][2 * e + 1], v[j][2 * e + 1], ss);
      }
    }
    const float total = block_sum(ss, red);
    const float inv = rsqrtf(total / static_cast<float>(a.hidden) + a.eps);
#pragma unroll
    for (int j = 0; j < kMaxVecsPerThread; ++j) {
      const int c = tid + j * kThreads;
      if (c >= nvec_row) continue;
      const size_t off = (static_cast<size_t>(row) * a.hidden + static_cast<size_t>(c) * kVec) * 2;
      const uint4 wv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(a.weight) + c * kVec * 2);
      const __half2 *wh = reinterpret_cast<const __half2 *>(&wv);
      uint4 ro, oo;
      __half2 *rp = reinterpret_cast<__half2 *>(&ro);
      __half2 *op = reinterpret_cast<__half2 *>(&oo);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        rp[e] = __floats2half2_rn(v[j][2 * e], v[j][2 * e + 1]);
        op[e] = __floats2half2_rn(v[j][2 * e] * inv * __low2float(wh[e]), v[j][2 * e + 1] * inv * __high2float(wh[e]));
      }
      *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(a.residual) + off) = ro;
      *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(a.out) + off) = oo;
    }
  }
}

}  // namespace ar
}  // namespace lvb
