// Tensor-parallel row-parallel epilogue on sm_100a: all-reduce of the ranks'
// fp16 partial sums over NVLink peer memory, fused with the residual add and
// RMSNorm that follow it in a Qwen2 block.
//
// Reference dataflow (modeling/quantization/awq.py:299-304 then
// modeling/models/_qwen2_kernels.py:20-43 via qwen2.py:497-514):
//   h = all_reduce_sum(partial)                 (fp16 tensor)
//   v = fp32(h) + fp32(residual)
//   residual <- fp16(v)
//   out      <- fp16(v * rsqrt(mean(v^2) + eps) * weight)
// The sum over ranks is taken in fp32 and rounded to fp16 once (the value the
// reference's all-reduce hands to the norm); the norm runs in fp32 like the
// reference kernel.  With no residual and no weight the kernel is a plain
// all-reduce: out <- h (out may alias partial).
//
// Every rank owns one workspace, mapped by all ranks through CUDA IPC:
//   header  epoch (this rank's call count), arrival counter, rows pushed per
//           sentinel buffer, phase-2 flags flags2[src], per-CTA phase-1
//           flags flags1[cta][src]
//   staging 2 parities x world slots x max_tokens x hidden fp16; slot [src]
//           receives the rows (or flat chunks) rank src pushes here
//   gather  2 parities x max_tokens x hidden fp16 (two-shot only): the
//           reduced rows every owner pushes to every rank
//   sentinel buffers  3 x world slots x max_tokens x hidden fp16, then 3
//           gather slots, filled with the sentinel 0xFFFF when empty
//           (sentinel modes only)
// Call e (read from the device, so the launch can be graph-captured) uses
// parity e & 1.  Data moves by plain 16-byte stores into peer memory; flags
// are system-scope release stores and acquire loads; every wait is bounded
// and records LVB_DEVERR_TIMEOUT when it runs out, after which the workspace
// must be rebuilt.
//
// One-shot (small messages): CTA b pushes its rows (b, b + grid, ...) to
// every peer, raises flags1[b][rank] there, waits for flags1[b][*] at home,
// then reduces those rows from the local staging slots (its own partial is
// read in place) and normalises them.  CTA b only waits for CTA b of the
// other ranks.
// Two-shot (large messages, reduce-scatter + all-gather): the flat element
// range is cut into world owner ranges and each into grid sub-chunks.
// Phase 1: CTA b pushes sub-chunk (c, b) of its partial to owner c.  Phase 2:
// CTA b waits for flags1[b][*], reduces its own sub-chunk and pushes the fp16
// result to every rank's gather buffer; the rank's last CTA to finish raises
// flags2[rank] at every rank.  Phase 3: every CTA waits for flags2[*] and
// normalises its rows from the local gather buffer.  Phase 3 waits on other
// CTAs of its own grid, so the grid never exceeds the CTAs that fit on the
// GPU at once.
//
// Sentinel one-shot (the smallest messages): like one-shot, but without
// flags or fences.  Empty slots hold 0xFFFF in every fp16 lane, a NaN pattern
// the writer never stores (it stores another NaN, 0xFE00, in its place), so
// a reader polls each 16-byte vector until no lane holds the sentinel; the
// data is its own ready flag.  Call e writes buffer e % 3 and clears, at
// home, the rows that call e - 1 received in buffer (e + 2) % 3: every peer
// finished writing it (this rank read all of it) and writes it again only at
// call e + 2, after this call has finished.
//
// Sentinel two-shot (larger messages at world > 2): the flat range is cut
// into world owner ranges and each into grid sub-chunks, as in the two-shot
// mode, but every exchange is a sentinel-marked push.  Phase 1: CTA b pushes
// sub-chunk (c, b) of its partial into owner c's slot [rank].  Phase 2: CTA b
// polls its own sub-chunk from the world - 1 slots, sums, rounds to fp16 and
// pushes the sums into every rank's gather slot.  Phase 3: every CTA polls
// the gather slot for its rows and normalises them.  No flags and no grid
// barrier: each wait is on exactly the data it consumes.  Call e clears, at
// home, what call e - 1 left in buffer (e + 2) % 3 (its own owner range of
// the peer slots and the whole gather slot); header words record the rows and
// the kind of exchange each buffer last received.
//
// Reuse of parity e & 1 at call e + 2 is safe: a rank can start call e + 2
// only after its call e + 1 passed a wait on every peer's call e + 1 pushes,
// and a peer pushes at call e + 1 only after its call e finished.
#pragma once

#include "lvb_common.cuh"

namespace lvb {
namespace ar {

constexpr int kMaxWorld = 8;
constexpr int kThreads = 512;
constexpr int kMaxBlocks = 1024;
constexpr int kMaxHidden = 8192;
constexpr int kVec = 8;  // fp16 per 16-byte vector
constexpr int kMaxVecsPerThread = kMaxHidden / (kVec * kThreads);  // 2
constexpr int kUnroll = 4;                                          // vectors in flight per thread when pushing

// Header layout (bytes).
constexpr int kEpochOff = 0;
constexpr int kCounterOff = 4;
constexpr int kRowsOff = 16;      // uint32 rows received per sentinel buffer [3]
constexpr int kGeometryOff = 32;  // uint32 magic, world, max_tokens, hidden (written at initialisation)
constexpr int kKindOff = 48;      // uint32 kind of data per sentinel buffer [3]: 0 none, 1 one-shot, 2 two-shot
constexpr uint32_t kMagic = 0x4c564152u;
constexpr int kFlags2Off = 64;
constexpr int kFlags1Off = 256;
constexpr size_t kHeaderBytes = 64 * 1024;
static_assert(kFlags1Off + kMaxBlocks * kMaxWorld * 4 <= static_cast<int>(kHeaderBytes), "header too small");

enum Mode : int { kAuto = 0, kOneShot = 1, kTwoShot = 2, kSentinel = 3, kSentinelTwoShot = 4 };
enum Kind : uint32_t { kKindNone = 0, kKindOneShot = 1, kKindTwoShot = 2 };
constexpr uint32_t kSentinelWord = 0xFFFFFFFFu;

struct Args {
  uint8_t *ws[kMaxWorld];   // every rank's workspace base, mapped here (ws[rank] = own)
  int rank, world;
  const uint16_t *partial;  // this rank's partial sums [tokens][hidden]
  uint16_t *residual;       // [tokens][hidden], updated in place; null for a plain all-reduce
  const uint16_t *weight;   // [hidden]; null for a plain all-reduce
  uint16_t *out;            // [tokens][hidden]
  int tokens, hidden;
  size_t slot_bytes;        // one staging slot (max_tokens x hidden fp16)
  float eps;
  int mode;                 // kOneShot, kTwoShot or kSentinel
};

// Staging (2 x world), gather (2), sentinel (3 x world) and sentinel gather (3) slots.
__host__ __device__ constexpr size_t slots_per_workspace(int world) { return 5 * static_cast<size_t>(world) + 5; }
// Slots before the sentinel region (initialised to zero; the rest to 0xFF).
__host__ __device__ constexpr size_t slots_before_sentinel(int world) { return 2 * static_cast<size_t>(world) + 2; }

__host__ __device__ __forceinline__ size_t staging_off(const Args &a, uint32_t parity, int src) {
  return kHeaderBytes + (static_cast<size_t>(parity) * a.world + src) * a.slot_bytes;
}
__host__ __device__ __forceinline__ size_t gather_off(const Args &a, uint32_t parity) {
  return kHeaderBytes + (2 * static_cast<size_t>(a.world) + parity) * a.slot_bytes;
}

__host__ __device__ __forceinline__ size_t sentinel_off(const Args &a, uint32_t buf, int src) {
  return kHeaderBytes + (2 * static_cast<size_t>(a.world) + 2 + static_cast<size_t>(buf) * a.world + src) * a.slot_bytes;
}
__host__ __device__ __forceinline__ size_t sentinel_gather_off(const Args &a, uint32_t buf) {
  return kHeaderBytes + (5 * static_cast<size_t>(a.world) + 2 + buf) * a.slot_bytes;
}

// Owner range [begin, end) of rank c in a flat range of `total` vectors.
__device__ __forceinline__ void owner_range(size_t total, int world, int c, size_t &begin, size_t &end) {
  const size_t per = (total + world - 1) / world;
  begin = min(static_cast<size_t>(c) * per, total);
  end = min(begin + per, total);
}

// Poll a 16-byte vector of peer-pushed data until no lane holds the sentinel.
__device__ __forceinline__ uint4 poll_vec(const void *p, long long start, bool &fail);

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint4 ld_cg(const void *p) { return __ldcg(reinterpret_cast<const uint4 *>(p)); }

__device__ __forceinline__ uint4 ld_volatile(const void *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ bool word_has_sentinel(uint32_t w) {
  return (w & 0xFFFFu) == 0xFFFFu || (w >> 16) == 0xFFFFu;
}
__device__ __forceinline__ bool has_sentinel(uint4 v) {
  return word_has_sentinel(v.x) || word_has_sentinel(v.y) || word_has_sentinel(v.z) || word_has_sentinel(v.w);
}
// Replace the sentinel lane pattern by another NaN (0xFE00).
__device__ __forceinline__ uint32_t sanitize_word(uint32_t w) {
  if ((w & 0xFFFFu) == 0xFFFFu) w = (w & 0xFFFF0000u) | 0xFE00u;
  if ((w >> 16) == 0xFFFFu) w = (w & 0x0000FFFFu) | 0xFE000000u;
  return w;
}
__device__ __forceinline__ uint4 sanitize(uint4 v) {
  return make_uint4(sanitize_word(v.x), sanitize_word(v.y), sanitize_word(v.z), sanitize_word(v.w));
}

__device__ __forceinline__ uint4 poll_vec(const void *p, long long start, bool &fail) {
  uint4 v = ld_volatile(p);
  while (has_sentinel(v) && !fail) {
    if (clock64() - start > kWaitBudgetCycles) {
      record_device_error(LVB_DEVERR_TIMEOUT);
      fail = true;
    }
    v = ld_volatile(p);
  }
  return v;
}

// Thread 0: wait until flags[i * stride] reaches epoch for i < n (bounded).
__device__ __forceinline__ bool wait_flags(const uint32_t *flags, int n, int stride, uint32_t epoch, long long start) {
  for (int i = 0; i < n; ++i) {
    while (static_cast<int>(ld_acquire_sys(flags + i * stride) - epoch) < 0) {
      if (clock64() - start > kWaitBudgetCycles) {
        record_device_error(LVB_DEVERR_TIMEOUT);
        return false;
      }
      __nanosleep(32);
    }
  }
  return true;
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
  for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return __shfl_sync(0xffffffffu, t, 0);
}

__device__ __forceinline__ void add_vec(float (&acc)[kVec], uint4 pv) {
  const __half2 *h = reinterpret_cast<const __half2 *>(&pv);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    acc[2 * e] += __low2float(h[e]);
    acc[2 * e + 1] += __high2float(h[e]);
  }
}

__device__ __forceinline__ uint4 round_vec(const float (&acc)[kVec]) {
  uint4 o;
  __half2 *p = reinterpret_cast<__half2 *>(&o);
#pragma unroll
  for (int e = 0; e < 4; ++e) p[e] = __floats2half2_rn(acc[2 * e], acc[2 * e + 1]);
  return o;
}

// Copy vectors [begin, end) of src (16-byte units) to offset dst_off of every
// listed workspace, kUnroll loads in flight per thread.
__device__ __forceinline__ void push_range(const Args &a, const uint4 *src, size_t begin, size_t end, size_t dst_off,
                                           bool include_self) {
  for (size_t i = begin + threadIdx.x; i < end; i += static_cast<size_t>(kThreads) * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const size_t k = i + static_cast<size_t>(u) * kThreads;
      if (k < end) v[u] = src[k];
    }
    for (int r = 0; r < a.world; ++r) {
      if (r == a.rank && !include_self) continue;
      uint4 *dst = reinterpret_cast<uint4 *>(a.ws[r] + dst_off);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const size_t k = i + static_cast<size_t>(u) * kThreads;
        if (k < end) dst[k] = v[u];
      }
    }
  }
}

// Thread 0 after a CTA-wide barrier: make this CTA's pushes visible, then
// raise flags1[cta][rank] in every peer's workspace.
__device__ __forceinline__ void signal_flags1(const Args &a, uint32_t epoch) {
  __threadfence_system();
  for (int r = 0; r < a.world; ++r) {
    if (r == a.rank) continue;
    st_release_sys(reinterpret_cast<uint32_t *>(a.ws[r] + kFlags1Off) + blockIdx.x * kMaxWorld + a.rank, epoch);
  }
}

// Residual add + RMSNorm (or the plain sum) of one row whose reduced fp16
// vectors are hv[j] for column vectors c = tid + j * kThreads.
__device__ __forceinline__ void finish_row(const Args &a, int row, const uint4 (&hv)[kMaxVecsPerThread], float *red) {
  const int nvec_row = a.hidden / kVec;
  const size_t row_off = static_cast<size_t>(row) * a.hidden * 2;
  if (a.weight == nullptr) {
#pragma unroll
    for (int j = 0; j < kMaxVecsPerThread; ++j) {
      const int c = threadIdx.x + j * kThreads;
      if (c < nvec_row) *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(a.out) + row_off + c * 16) = hv[j];
    }
    return;
  }
  float v[kMaxVecsPerThread][kVec];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVecsPerThread; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c >= nvec_row) continue;
    const uint4 rv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(a.residual) + row_off + c * 16);
    const __half2 *rh = reinterpret_cast<const __half2 *>(&rv);
    const __half2 *hh = reinterpret_cast<const __half2 *>(&hv[j]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[j][2 * e] = __low2float(hh[e]) + __low2float(rh[e]);
      v[j][2 * e + 1] = __high2float(hh[e]) + __high2float(rh[e]);
      ss = fmaf(v[j][2 * e], v[j][2 * e], ss);
      ss = fmaf(v[j][2 * e + 1], v[j][2 * e + 1], ss);
    }
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / static_cast<float>(a.hidden) + a.eps);
#pragma unroll
  for (int j = 0; j < kMaxVecsPerThread; ++j) {
    const int c = threadIdx.x + j * kThreads;
    if (c >= nvec_row) continue;
    const uint4 wv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(a.weight) + c * 16);
    const __half2 *wh = reinterpret_cast<const __half2 *>(&wv);
    uint4 ro, oo;
    __half2 *rp = reinterpret_cast<__half2 *>(&ro);
    __half2 *op = reinterpret_cast<__half2 *>(&oo);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      rp[e] = __floats2half2_rn(v[j][2 * e], v[j][2 * e + 1]);
      op[e] = __floats2half2_rn(v[j][2 * e] * inv * __low2float(wh[e]), v[j][2 * e + 1] * inv * __high2float(wh[e]));
    }
    *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(a.residual) + row_off + c * 16) = ro;
    *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(a.out) + row_off + c * 16) = oo;
  }
}

__global__ void __launch_bounds__(kThreads) allreduce_add_rmsnorm_kernel(const __grid_constant__ Args a) {
  pdl_entry();
  __shared__ float red[kThreads / 32];
  __shared__ int ok_sm;
  __shared__ uint32_t epoch_sm, stale_rows_sm, stale_kind_sm;
  const int tid = threadIdx.x;
  uint8_t *own = a.ws[a.rank];
  uint32_t *counter = reinterpret_cast<uint32_t *>(own + kCounterOff);
  // Every CTA reads the epoch before its thread 0 arrives at the counter; the
  // last arrival advances it for the next call.
  if (tid == 0) {
    // The workspace must have been initialised for this geometry.
    const uint32_t *geo = reinterpret_cast<const uint32_t *>(own + kGeometryOff);
    ok_sm = geo[0] == kMagic && geo[1] == static_cast<uint32_t>(a.world) &&
            static_cast<size_t>(geo[2]) * geo[3] * 2 == a.slot_bytes && geo[3] == static_cast<uint32_t>(a.hidden);
    if (!ok_sm) record_device_error(LVB_DEVERR_INDEX);
    epoch_sm = *reinterpret_cast<volatile uint32_t *>(own + kEpochOff) + 1u;
    stale_rows_sm = reinterpret_cast<const volatile uint32_t *>(own + kRowsOff)[(epoch_sm + 2u) % 3u];
    stale_kind_sm = reinterpret_cast<const volatile uint32_t *>(own + kKindOff)[(epoch_sm + 2u) % 3u];
  }
  __syncthreads();
  if (!ok_sm) return;
  const uint32_t epoch = epoch_sm;
  const uint32_t parity = epoch & 1u;
  const int nvec_row = a.hidden / kVec;
  const uint4 *partial = reinterpret_cast<const uint4 *>(a.partial);
  const long long start = clock64();

  // Sentinel buffers: clear the rows that arrived at the previous call (none
  // unless it ran in sentinel mode).  Every mode does this, so modes mix.
  const uint32_t buf = epoch % 3u, stale = (epoch + 2u) % 3u;
  {
    const int stale_rows = static_cast<int>(stale_rows_sm);
    const uint4 empty = make_uint4(kSentinelWord, kSentinelWord, kSentinelWord, kSentinelWord);
    if (stale_kind_sm == kKindOneShot) {
      for (int row = blockIdx.x; row < stale_rows; row += gridDim.x) {
        const size_t v0 = static_cast<size_t>(row) * nvec_row;
        for (int r = 0; r < a.world; ++r) {
          if (r == a.rank) continue;
          uint4 *dst = reinterpret_cast<uint4 *>(own + sentinel_off(a, stale, r));
          for (int c = tid; c < nvec_row; c += kThreads) dst[v0 + c] = empty;
        }
      }
    } else if (stale_kind_sm == kKindTwoShot) {
      const size_t total = static_cast<size_t>(stale_rows) * nvec_row;
      size_t ob, oe;
      owner_range(total, a.world, a.rank, ob, oe);
      const size_t step = static_cast<size_t>(gridDim.x) * kThreads;
      for (int r = 0; r < a.world; ++r) {
        if (r == a.rank) continue;
        uint4 *dst = reinterpret_cast<uint4 *>(own + sentinel_off(a, stale, r));
        for (size_t i = ob + static_cast<size_t>(blockIdx.x) * kThreads + tid; i < oe; i += step) dst[i] = empty;
      }
      uint4 *gdst = reinterpret_cast<uint4 *>(own + sentinel_gather_off(a, stale));
      for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + tid; i < total; i += step) gdst[i] = empty;
    }
  }
  // The last CTA to arrive records what this call left in the sentinel
  // buffers and advances the epoch.
  auto advance_epoch = [&]() {
    *counter = 0u;
    const bool sentinel = a.mode == kSentinel || a.mode == kSentinelTwoShot;
    reinterpret_cast<volatile uint32_t *>(own + kRowsOff)[buf] = sentinel ? static_cast<uint32_t>(a.tokens) : 0u;
    reinterpret_cast<volatile uint32_t *>(own + kKindOff)[buf] =
        a.mode == kSentinel ? kKindOneShot : a.mode == kSentinelTwoShot ? kKindTwoShot : kKindNone;
    *reinterpret_cast<volatile uint32_t *>(own + kEpochOff) = epoch;
  };

  if (a.mode == kSentinelTwoShot) {
    const size_t total = static_cast<size_t>(a.tokens) * nvec_row;
    // Phase 1: sub-chunk (c, b) of this rank's partial -> owner c's slot [rank].
    for (int c = 0; c < a.world; ++c) {
      if (c == a.rank) continue;
      size_t ob, oe;
      owner_range(total, a.world, c, ob, oe);
      const size_t per_cta = (oe - ob + gridDim.x - 1) / gridDim.x;
      const size_t b0 = min(ob + static_cast<size_t>(blockIdx.x) * per_cta, oe);
      const size_t e0 = min(b0 + per_cta, oe);
      uint4 *dst = reinterpret_cast<uint4 *>(a.ws[c] + sentinel_off(a, buf, a.rank));
      for (size_t i = b0 + tid; i < e0; i += kThreads) dst[i] = sanitize(partial[i]);
    }
    if (tid == 0) {
      const unsigned int prev = atomicAdd(counter, 1u);
      if (prev == gridDim.x - 1) advance_epoch();
    }
    // Phase 2: own sub-chunk: poll the peers' values, sum, push the sums.
    bool fail = false;
    {
      size_t ob, oe;
      owner_range(total, a.world, a.rank, ob, oe);
      const size_t per_cta = (oe - ob + gridDim.x - 1) / gridDim.x;
      const size_t b0 = min(ob + static_cast<size_t>(blockIdx.x) * per_cta, oe);
      const size_t e0 = min(b0 + per_cta, oe);
      const size_t goff = sentinel_gather_off(a, buf);
      for (size_t i = b0 + tid; i < e0; i += kThreads) {
        float acc[kVec];
#pragma unroll
        for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
        for (int r = 0; r < a.world; ++r) {
          const uint4 pv = r == a.rank ? partial[i] : poll_vec(own + sentinel_off(a, buf, r) + i * 16, start, fail);
          add_vec(acc, pv);
        }
        const uint4 hv = sanitize(round_vec(acc));
        for (int r = 0; r < a.world; ++r) reinterpret_cast<uint4 *>(a.ws[r] + goff)[i] = hv;
      }
    }
    // Phase 3: rows b, b + grid, ... from the home gather slot.
    const uint8_t *gather = own + sentinel_gather_off(a, buf);
    for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
      uint4 hv[kMaxVecsPerThread];
#pragma unroll
      for (int j = 0; j < kMaxVecsPerThread; ++j) {
        const int c = tid + j * kThreads;
        if (c < nvec_row) hv[j] = poll_vec(gather + (static_cast<size_t>(row) * nvec_row + c) * 16, start, fail);
      }
      if (__syncthreads_or(fail)) return;
      finish_row(a, row, hv, red);
    }
    return;
  }

  if (a.mode == kSentinel) {
    // ---- sentinel one-shot: rows b, b + grid, ... ----
    for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
      const size_t v0 = static_cast<size_t>(row) * nvec_row;
      const size_t off = sentinel_off(a, buf, a.rank);
      for (int c = tid; c < nvec_row; c += kThreads) {
        const uint4 v = sanitize(partial[v0 + c]);
        for (int r = 0; r < a.world; ++r)
          if (r != a.rank) reinterpret_cast<uint4 *>(a.ws[r] + off)[v0 + c] = v;
      }
    }
    if (tid == 0) {
      const unsigned int prev = atomicAdd(counter, 1u);
      if (prev == gridDim.x - 1) advance_epoch();
    }
    for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
      uint4 hv[kMaxVecsPerThread];
      bool fail = false;
#pragma unroll
      for (int j = 0; j < kMaxVecsPerThread; ++j) {
        const int c = tid + j * kThreads;
        if (c >= nvec_row) continue;
        const size_t vi = static_cast<size_t>(row) * nvec_row + c;
        float acc[kVec];
#pragma unroll
        for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
        for (int r = 0; r < a.world; ++r) {
          uint4 pv;
          if (r == a.rank) {
            pv = partial[vi];
          } else {
            const uint8_t *src = own + sentinel_off(a, buf, r) + vi * 16;
            pv = ld_volatile(src);
            while (has_sentinel(pv) && !fail) {
              if (clock64() - start > kWaitBudgetCycles) {
                record_device_error(LVB_DEVERR_TIMEOUT);
                fail = true;
              }
              pv = ld_volatile(src);
            }
          }
          add_vec(acc, pv);
        }
        hv[j] = round_vec(acc);
      }
      if (__syncthreads_or(fail)) return;
      finish_row(a, row, hv, red);
    }
    return;
  }

  if (a.mode == kOneShot) {
    // ---- one-shot: rows b, b + grid, ... ----
    for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
      const size_t v0 = static_cast<size_t>(row) * nvec_row;
      push_range(a, partial, v0, v0 + nvec_row, staging_off(a, parity, a.rank), false);
    }
    __syncthreads();
    if (tid == 0) {
      signal_flags1(a, epoch);
      const uint32_t *f = reinterpret_cast<const uint32_t *>(own + kFlags1Off) + blockIdx.x * kMaxWorld;
      bool ok = true;
      for (int r = 0; r < a.world && ok; ++r)
        if (r != a.rank) ok = wait_flags(f + r, 1, 1, epoch, start);
      ok_sm = ok;
      __threadfence();
      const unsigned int prev = atomicAdd(counter, 1u);
      if (prev == gridDim.x - 1) advance_epoch();
    }
    __syncthreads();
    if (!ok_sm) return;
    for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
      uint4 hv[kMaxVecsPerThread];
#pragma unroll
      for (int j = 0; j < kMaxVecsPerThread; ++j) {
        const int c = tid + j * kThreads;
        if (c >= nvec_row) continue;
        const size_t vi = static_cast<size_t>(row) * nvec_row + c;
        float acc[kVec];
#pragma unroll
        for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
        for (int r = 0; r < a.world; ++r) {
          const uint4 pv = r == a.rank ? partial[vi] : ld_cg(own + staging_off(a, parity, r) + vi * 16);
          add_vec(acc, pv);
        }
        hv[j] = round_vec(acc);
      }
      finish_row(a, row, hv, red);
    }
    return;
  }

  // ---- two-shot ----
  const size_t total = static_cast<size_t>(a.tokens) * nvec_row;
  const size_t per_owner = (total + a.world - 1) / a.world;
  const size_t per_cta = (per_owner + gridDim.x - 1) / gridDim.x;
  // Phase 1: sub-chunk (c, b) of this rank's partial -> owner c's slot [rank].
  for (int c = 0; c < a.world; ++c) {
    if (c == a.rank) continue;
    const size_t b0 = c * per_owner + blockIdx.x * per_cta;
    const size_t e0 = min(min(b0 + per_cta, (c + 1) * per_owner), total);
    if (b0 >= e0) continue;
    const size_t off = staging_off(a, parity, a.rank);
    const uint4 *src = partial;
    uint4 *dst = reinterpret_cast<uint4 *>(a.ws[c] + off);
    for (size_t i = b0 + tid; i < e0; i += static_cast<size_t>(kThreads) * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const size_t k = i + static_cast<size_t>(u) * kThreads;
        if (k < e0) v[u] = src[k];
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const size_t k = i + static_cast<size_t>(u) * kThreads;
        if (k < e0) dst[k] = v[u];
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    signal_flags1(a, epoch);
    const uint32_t *f = reinterpret_cast<const uint32_t *>(own + kFlags1Off) + blockIdx.x * kMaxWorld;
    bool ok = true;
    for (int r = 0; r < a.world && ok; ++r)
      if (r != a.rank) ok = wait_flags(f + r, 1, 1, epoch, start);
    ok_sm = ok;
  }
  __syncthreads();
  if (!ok_sm) return;
  // Phase 2: reduce the owned sub-chunk, push the fp16 sums to every rank.
  {
    const size_t b0 = a.rank * per_owner + blockIdx.x * per_cta;
    const size_t e0 = min(min(b0 + per_cta, (a.rank + 1) * per_owner), total);
    const size_t goff = gather_off(a, parity);
    for (size_t i = b0 + tid; i < e0; i += static_cast<size_t>(kThreads) * kUnroll) {
      uint4 hv[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const size_t k = i + static_cast<size_t>(u) * kThreads;
        if (k >= e0) continue;
        float acc[kVec];
#pragma unroll
        for (int e = 0; e < kVec; ++e) acc[e] = 0.f;
        for (int r = 0; r < a.world; ++r) {
          const uint4 pv = r == a.rank ? partial[k] : ld_cg(own + staging_off(a, parity, r) + k * 16);
          add_vec(acc, pv);
        }
        hv[u] = round_vec(acc);
      }
      for (int r = 0; r < a.world; ++r) {
        uint4 *dst = reinterpret_cast<uint4 *>(a.ws[r] + goff);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const size_t k = i + static_cast<size_t>(u) * kThreads;
          if (k < e0) dst[k] = hv[u];
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(counter, 1u);
    if (prev == gridDim.x - 1) {
      // Every CTA of this rank has pushed its sums: publish them, then
      // advance the epoch for the next call.
      __threadfence_system();
      for (int r = 0; r < a.world; ++r)
        st_release_sys(reinterpret_cast<uint32_t *>(a.ws[r] + kFlags2Off) + a.rank, epoch);
      advance_epoch();
    }
    ok_sm = wait_flags(reinterpret_cast<const uint32_t *>(own + kFlags2Off), a.world, 1, epoch, start);
  }
  __syncthreads();
  if (!ok_sm) return;
  // Phase 3: rows from the local gather buffer.
  const uint8_t *gather = own + gather_off(a, parity);
  for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
    uint4 hv[kMaxVecsPerThread];
#pragma unroll
    for (int j = 0; j < kMaxVecsPerThread; ++j) {
      const int c = tid + j * kThreads;
      if (c < nvec_row) hv[j] = ld_cg(gather + (static_cast<size_t>(row) * nvec_row + c) * 16);
    }
    finish_row(a, row, hv, red);
  }
}

// One rank: no exchange, no workspace -- residual add + RMSNorm of each row,
// with every input vector loaded before the first reduction.
__global__ void __launch_bounds__(kThreads) add_rmsnorm_kernel(const __grid_constant__ Args a) {
  pdl_entry();
  __shared__ float red[kThreads / 32];
  const int nvec_row = a.hidden / kVec;
  const uint4 *partial = reinterpret_cast<const uint4 *>(a.partial);
  for (int row = blockIdx.x; row < a.tokens; row += gridDim.x) {
    uint4 hv[kMaxVecsPerThread];
#pragma unroll
    for (int j = 0; j < kMaxVecsPerThread; ++j) {
      const int c = threadIdx.x + j * kThreads;
      if (c < nvec_row) hv[j] = partial[static_cast<size_t>(row) * nvec_row + c];
    }
    finish_row(a, row, hv, red);
  }
}

}  // namespace ar
}  // namespace lvb
