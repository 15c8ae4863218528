// C-ABI entry points of the B200 hot-path library (declared in include/lvb200.h).
//
// One translation unit: the kernels live in the .cuh files included below.
// Entry points validate arguments, pick a kernel configuration, encode TMA
// tensor maps on the host (pure host computation, no device traffic) and
// enqueue on the caller's stream.  They never synchronise and never allocate.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/lvb200.h"
#include "awq_gemm.cuh"
#include "awq_gemv.cuh"
#include "awq_mma.cuh"
#include "qwen2_ops.cuh"
#include "awq_decode.cuh"
#include "awq_i8.cuh"
#include "allreduce.cuh"
#include "lvb_common.cuh"
#include "paged_attention.cuh"
#include "step_metadata.cuh"

namespace {

constexpr int kAbiVersion = 8;
constexpr int kMaxDevices = 64;

thread_local char g_last_error[512] = "";

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(LVB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Streaming-multiprocessor count of the current device, queried once per device.
int current_device(int *dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(LVB_ERR_UNSUPPORTED, "device index %d", *dev);
  return LVB_OK;
}

int sm_count(int dev) {
  static int counts[kMaxDevices] = {0};
  if (counts[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    counts[dev] = v;
  }
  return counts[dev];
}

// Opt a kernel into large dynamic shared memory once per (kernel, device).
template <typename Kernel>
int ensure_smem(Kernel kernel, int bytes, int dev, bool *done_flags) {
  if (done_flags[dev]) return LVB_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  done_flags[dev] = true;
  return LVB_OK;
}

// Launch with the programmatic-serialisation attribute: the kernel may start
// while the previous kernel of the stream finishes (each hot-path kernel
// begins with pdl_entry(), which waits for it before any dependent access).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_map(CUtensorMap *map, CUtensorMapDataType type, cuuint32_t rank, const void *base,
               const cuuint64_t *dims, const cuuint64_t *strides_bytes, const cuuint32_t *box,
               CUtensorMapSwizzle swizzle) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return fail(LVB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = encode(map, type, rank, const_cast<void *>(base), dims, strides_bytes, box,
                      elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LVB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return LVB_OK;
}

// ------------------------------------------------------------------------
// AWQ planning
// ------------------------------------------------------------------------
struct AwqPlan {
  int bn, m_tiles, n_tiles, k_tiles, splits;
  size_t sem_bytes, part_bytes;
};

AwqPlan awq_plan(int64_t m, int64_t k, int64_t n, int sms) {
  AwqPlan p{};
  p.bn = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256;
  p.m_tiles = static_cast<int>((m + p.bn - 1) / p.bn);
  p.n_tiles = static_cast<int>((n + lvb::awq::kTileN - 1) / lvb::awq::kTileN);
  p.k_tiles = static_cast<int>((k + lvb::awq::kTileK - 1) / lvb::awq::kTileK);
  const int tiles = p.m_tiles * p.n_tiles;
  p.splits = 1;
  if (p.bn <= 64 && tiles < sms) {
    int s = sms / tiles;
    const int cap = p.k_tiles / 2 > 1 ? p.k_tiles / 2 : 1;
    p.splits = s < cap ? s : cap;
    if (p.splits < 1) p.splits = 1;
  }
  p.sem_bytes = p.splits > 1 ? (static_cast<size_t>(tiles) * 4 + 255) & ~static_cast<size_t>(255) : 0;
  p.part_bytes = p.splits > 1
                     ? static_cast<size_t>(tiles) * p.splits * p.bn * lvb::awq::kTileN * sizeof(float)
                     : 0;
  return p;
}

template <int BN>
int launch_awq(const AwqPlan &plan, const uint16_t *x, const int32_t *qweight,
               const int32_t *qzeros, const uint16_t *scales, const uint16_t *bias, uint16_t *y,
               int64_t m, int64_t k, int64_t n, int64_t g, uint8_t *ws, int dev,
               cudaStream_t stream) {
  using C = lvb::awq::Config<BN>;
  static bool smem_done[kMaxDevices] = {false};
  auto kernel = lvb::awq::awq_gemm_kernel<BN>;
  int rc = ensure_smem(kernel, C::kSmemBytes, dev, smem_done);
  if (rc != LVB_OK) return rc;

  lvb::awq::Params p{};
  p.x = x;
  p.qweight = qweight;
  p.qzeros = qzeros;
  p.scales = scales;
  p.bias = bias;
  p.y = y;
  p.semaphores = reinterpret_cast<uint32_t *>(ws);
  p.partials = plan.splits > 1 ? reinterpret_cast<float *>(ws + plan.sem_bytes) : nullptr;
  p.M = static_cast<int>(m);
  p.K = static_cast<int>(k);
  p.N = static_cast<int>(n);
  p.G = static_cast<int>(g);
  p.k_tiles = plan.k_tiles;
  p.splits = plan.splits;
  p.n_tiles = plan.n_tiles;
  dim3 grid(plan.n_tiles, plan.m_tiles, plan.splits);
  cudaError_t e = launch_pdl(kernel, grid, dim3(lvb::awq::kThreads), C::kSmemBytes, stream, p);
  if (e != cudaSuccess) return cuda_fail(e, "awq_gemm_kernel launch");
  return LVB_OK;
}

// The standard-layout entry points run the fp16-dequantising GEMM for every
// batch size; decode-sized batches are fastest through the packed layout
// (lvb_awq_pack + lvb_awq_linear_packed).
int dispatch_awq(const AwqPlan &plan, const uint16_t *x, const int32_t *qweight, const int32_t *qzeros,
                 const uint16_t *scales, const uint16_t *bias, uint16_t *y, int64_t m, int64_t k, int64_t n,
                 int64_t g, uint8_t *ws, int dev, cudaStream_t s) {
  switch (plan.bn) {
    case 16: return launch_awq<16>(plan, x, qweight, qzeros, scales, bias, y, m, k, n, g, ws, dev, s);
    case 32: return launch_awq<32>(plan, x, qweight, qzeros, scales, bias, y, m, k, n, g, ws, dev, s);
    case 64: return launch_awq<64>(plan, x, qweight, qzeros, scales, bias, y, m, k, n, g, ws, dev, s);
    case 128: return launch_awq<128>(plan, x, qweight, qzeros, scales, bias, y, m, k, n, g, ws, dev, s);
    default: return launch_awq<256>(plan, x, qweight, qzeros, scales, bias, y, m, k, n, g, ws, dev, s);
  }
}

// ------------------------------------------------------------------------
// Packed-layout decode path
// ------------------------------------------------------------------------
struct PackedShape {
  int n_tiles, k_chunks, k_blocks, groups;
  size_t codes_bytes, groups_bytes;
};

PackedShape packed_shape(int64_t k, int64_t n, int64_t g) {
  PackedShape s{};
  s.n_tiles = static_cast<int>((n + lvb::awqd::kTileN - 1) / lvb::awqd::kTileN);
  s.k_blocks = static_cast<int>((k + lvb::awqd::kBlockK - 1) / lvb::awqd::kBlockK);
  s.k_chunks = 2 * s.k_blocks;
  s.groups = static_cast<int>(k / g);
  s.codes_bytes = static_cast<size_t>(s.n_tiles) * s.k_chunks * lvb::awqd::kChunkBytes;
  s.groups_bytes = static_cast<size_t>(s.n_tiles) * s.groups * lvb::awqd::kSzRowBytes;
  return s;
}

struct PackedPlan {
  int bn, m_tiles, splits;
  size_t sem_bytes, part_bytes;
};

// Token tile per batch size: the decode configurations (two accumulators,
// 256-k stages) up to 64 rows, 128 rows with two accumulators, then 256-row
// tiles with one accumulator.
int packed_bn(int64_t m) { return m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256; }

// Two CTAs per SM (half the tensor and shared memory each: 128-k or 64-k
// stages, one dequantiser warpgroup) for the 64- and 128-row token tiles when
// the output tiles alone fill the GPU: measured on B200 they win without
// split-K (m = 64, 3584 x 37888: 46.0 -> 38.5 us; m = 128, 8192 x 29696:
// 136.6 -> 101.8 us) and lose with it (m = 128, 4096 x 8192: 27.6 -> 34.0).
int packed_ctas_per_sm(int bn, const PackedShape &sh, int64_t m, int sms) {
  const int64_t tiles = static_cast<int64_t>(sh.n_tiles) * ((m + bn - 1) / bn);
  return (bn == 64 || bn == 128) && tiles >= sms ? 2 : 1;
}

// Fixed cost of one CTA (TMEM allocation, pipeline fill and drain, partial
// tile write and merge) in 64-k blocks of main-loop work; without it the
// model splits a 4096-deep M = 128 GEMM into 16 CTAs of 4 blocks each and
// runs 4x slower than with 2 splits (ncu: tensor pipe 5 % active).
constexpr long long kPackedCtaOverheadBlocks = 8;

// K splits for grids smaller than the SM count: the split count that
// minimises (waves of CTAs) x (64-k blocks per CTA + the per-CTA overhead),
// fewest splits on ties, among the plans whose split-K workspace fits in
// `max_ws` bytes.
PackedPlan packed_plan(int64_t m, const PackedShape &sh, int sms, size_t max_ws = SIZE_MAX) {
  PackedPlan p{};
  p.bn = packed_bn(m);
  p.m_tiles = static_cast<int>((m + p.bn - 1) / p.bn);
  const long long tiles = static_cast<long long>(sh.n_tiles) * p.m_tiles;
  int best = 1;
  long long best_cost = -1;
  const int max_splits = sh.k_blocks < 16 ? sh.k_blocks : 16;
  const size_t sem = (static_cast<size_t>(tiles) * 4 + 255) & ~static_cast<size_t>(255);
  for (int sp = 1; sp <= max_splits; ++sp) {
    const size_t need = sp > 1 ? sem + static_cast<size_t>(tiles) * sp * p.bn * lvb::awqd::kTileN * sizeof(float) : 0;
    if (need > max_ws) continue;
    const long long ctas = tiles * sp;
    const long long waves = (ctas + sms - 1) / sms;
    const long long cost = waves * ((sh.k_blocks + sp - 1) / sp + kPackedCtaOverheadBlocks);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  p.splits = best;
  p.sem_bytes = p.splits > 1 ? sem : 0;
  p.part_bytes =
      p.splits > 1 ? static_cast<size_t>(tiles) * p.splits * p.bn * lvb::awqd::kTileN * sizeof(float) : 0;
  return p;
}

template <int BN, int SB, int DG, bool DUAL, int TMEM = lvb::awqd::kTmemCols,
          int SMEM_KB = lvb::awqd::kSmemBudget / 1024>
int launch_awq_packed(const PackedPlan &plan, const PackedShape &sh, const uint16_t *x, const uint8_t *codes,
                      const uint32_t *groups, const uint16_t *bias, uint16_t *y, int64_t m, int64_t k,
                      int64_t n, int64_t g, uint8_t *ws, int dev, cudaStream_t stream) {
  using C = lvb::awqd::PackedConfig<BN, SB, DG, DUAL, TMEM, SMEM_KB>;
  static bool smem_done[kMaxDevices] = {false};
  auto kernel = lvb::awqd::awq_packed_kernel<BN, SB, DG, DUAL, TMEM, SMEM_KB>;
  int rc = ensure_smem(kernel, C::kSmemBytes, dev, smem_done);
  if (rc != LVB_OK) return rc;
  // Activations as [k / 32 chunks][m rows][32 k]: one box per stage fetches
  // the stage's 64-byte-swizzled [BN x 32] tiles; rows past m and chunks past
  // k read as zeros.
  CUtensorMap xmap;
  const cuuint64_t dims[3] = {32, static_cast<cuuint64_t>(m), static_cast<cuuint64_t>(k / 32)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(k) * 2, 64};
  const cuuint32_t box[3] = {32, static_cast<cuuint32_t>(BN), static_cast<cuuint32_t>(C::kStageChunks)};
  rc = encode_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc != LVB_OK) return rc;
  lvb::awqd::DecodeParams p{};
  p.qpack = codes;
  p.szpack = groups;
  p.bias = bias;
  p.y = y;
  p.semaphores = reinterpret_cast<uint32_t *>(ws);
  p.partials = plan.splits > 1 ? reinterpret_cast<float *>(ws + plan.sem_bytes) : nullptr;
  p.M = static_cast<int>(m);
  p.K = static_cast<int>(k);
  p.N = static_cast<int>(n);
  p.G = static_cast<int>(g);
  p.groups = sh.groups;
  p.k_chunks = sh.k_chunks;
  p.k_blocks = sh.k_blocks;
  p.n_tiles = sh.n_tiles;
  p.m_tiles = plan.m_tiles;
  p.splits = plan.splits;
  dim3 grid(plan.m_tiles, sh.n_tiles, plan.splits);
  cudaError_t e = launch_pdl(kernel, grid, dim3(C::kThreads), C::kSmemBytes, stream, xmap, p);
  if (e != cudaSuccess) return cuda_fail(e, "awq_packed_kernel launch");
  return LVB_OK;
}

// int8 tensor-core path for decode batches: m <= 16, groups of 128 or 256 k
// (one or two whole groups per 256-k stage).
// The int8 path pays a limb prologue and a persistent-kernel start-up that
// only large weights amortise: measured on B200 at m = 16 it ties the fp16
// packed path at 6-8 MB of packed weights, wins above (34 MB: 20.3 vs 24.2 us;
// 68 MB: 26.9 vs 40.6 us) and loses below (config 1, 2.2 MB: 13.0 vs 8.2 us).
constexpr int64_t kI8MinWeightBytes = int64_t(8) << 20;

// 16-row token tiles only: four activation limbs x 16 rows make the MMA's
// N = 64, and two stage accumulators of two groups fill the tensor memory
// beside the A stages.  Batches of 17..32 rows run the fp16 packed kernel.
bool i8_eligible(int64_t m, int64_t k, int64_t n, int64_t g) {
  return m <= 16 && (g == 128 || g == 256) && k % g == 0 && n % 128 == 0 && k * n / 2 >= kI8MinWeightBytes;
}

struct I8Plan {
  int bn = 0, splits = 1;
  size_t sem_bytes = 0, part_bytes = 0, limb_bytes = 0, scal_bytes = 0, flag_bytes = 0;
  size_t total() const { return sem_bytes + part_bytes + limb_bytes + scal_bytes + flag_bytes; }
};

size_t round256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// bn == 0 when the activation limbs do not fit in `max_ws`.  Splits cover
// whole groups; same cost model as the packed path.
I8Plan i8_plan(int64_t m, int64_t k, const PackedShape &sh, int64_t g, int sms, size_t max_ws = SIZE_MAX) {
  I8Plan p;
  (void)m;
  const int bn = 16;
  p.limb_bytes = round256(static_cast<size_t>(k) * lvb::awqi8::kLimbs * bn);
  p.scal_bytes = round256(static_cast<size_t>(sh.groups) * bn * sizeof(int4));
  p.flag_bytes = round256(static_cast<size_t>(sh.groups) * sizeof(int));
  if (p.limb_bytes + p.scal_bytes + p.flag_bytes > max_ws) return p;
  p.bn = bn;
  const int bpg = static_cast<int>(g / 64);
  const size_t sem = round256(static_cast<size_t>(sh.n_tiles) * 4);
  long long best_cost = -1;
  const int max_splits = sh.groups < 16 ? sh.groups : 16;
  for (int sp = 1; sp <= max_splits; ++sp) {
    const size_t part = sp > 1 ? static_cast<size_t>(sh.n_tiles) * sp * bn * lvb::awqi8::kTileN * sizeof(float) : 0;
    if ((sp > 1 ? sem : 0) + part + p.limb_bytes + p.scal_bytes + p.flag_bytes > max_ws) continue;
    const long long ctas = static_cast<long long>(sh.n_tiles) * sp;
    const long long waves = (ctas + sms - 1) / sms;
    const long long cost = waves * ((sh.groups + sp - 1) / sp) * bpg;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      p.splits = sp;
      p.sem_bytes = sp > 1 ? sem : 0;
      p.part_bytes = part;
    }
  }
  return p;
}

template <int BN>
int launch_awq_i8(const I8Plan &plan, const PackedShape &sh, const uint16_t *x, const uint8_t *codes,
                  const uint32_t *groups, const uint16_t *bias, uint16_t *y, int64_t m, int64_t k, int64_t n,
                  int64_t g, uint8_t *ws, int dev, cudaStream_t stream, int64_t x_stride, int gated) {
  using C = lvb::awqi8::I8Config<BN>;
  static bool smem_done[kMaxDevices] = {false};
  auto kernel = lvb::awqi8::awq_i8_kernel<BN>;
  int rc = ensure_smem(kernel, C::kSmemBytes, dev, smem_done);
  if (rc != LVB_OK) return rc;
  int8_t *limbs = reinterpret_cast<int8_t *>(ws + plan.sem_bytes + plan.part_bytes);
  int4 *scal = reinterpret_cast<int4 *>(ws + plan.sem_bytes + plan.part_bytes + plan.limb_bytes);
  int *four = reinterpret_cast<int *>(ws + plan.sem_bytes + plan.part_bytes + plan.limb_bytes + plan.scal_bytes);
  cudaError_t e = launch_pdl(lvb::awqi8::awq_act_limbs_kernel<BN>, dim3(sh.groups), dim3(32 * BN), 0, stream, x,
                             x_stride, gated, limbs, scal, four, static_cast<int>(m), static_cast<int>(k),
                             static_cast<int>(g));
  if (e != cudaSuccess) return cuda_fail(e, "awq_act_limbs_kernel launch");
  lvb::awqi8::I8Params p{};
  p.qpack = codes;
  p.szpack = groups;
  p.limbs = limbs;
  p.scal = scal;
  p.four = four;
  p.bias = bias;
  p.y = y;
  p.semaphores = reinterpret_cast<uint32_t *>(ws);
  p.partials = plan.splits > 1 ? reinterpret_cast<float *>(ws + plan.sem_bytes) : nullptr;
  p.M = static_cast<int>(m);
  p.K = static_cast<int>(k);
  p.N = static_cast<int>(n);
  p.G = static_cast<int>(g);
  p.groups = sh.groups;
  p.k_chunks = sh.k_chunks;
  p.blocks_per_group = static_cast<int>(g / 64);
  p.bpg_shift = g == 128 ? 1 : 2;
  p.n_tiles = sh.n_tiles;
  p.splits = plan.splits;
  // Persistent grid of at most one CTA per SM, launched as a programmatic
  // dependent of the limb kernel (it waits for the limbs in-kernel).
  const int units = sh.n_tiles * plan.splits;
  const int ctas = units < sm_count(dev) ? units : sm_count(dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(lvb::awqi8::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // y as a [m rows][n] fp16 tensor; a box is one [BN][128] output tile.
  CUtensorMap ymap;
  const cuuint64_t ydims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m)};
  const cuuint64_t ystrides[1] = {static_cast<cuuint64_t>(n) * 2};
  const cuuint32_t ybox[2] = {static_cast<cuuint32_t>(lvb::awqi8::kTileN), static_cast<cuuint32_t>(BN)};
  rc = encode_map(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, y, ydims, ystrides, ybox, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != LVB_OK) return rc;
  e = cudaLaunchKernelEx(&cfg, kernel, ymap, p);
  if (e != cudaSuccess) return cuda_fail(e, "awq_i8_kernel launch");
  return LVB_OK;
}

// ------------------------------------------------------------------------
// GEMV plan (m <= 4, CUDA-core dp4a over the packed layout)
// ------------------------------------------------------------------------
// Measured on B200 (7B gate_up / down / QKV): the GEMV beats the int8
// tensor-core path at one row only (m = 2..4 run it for shapes the int8 path
// does not take).
constexpr int64_t kGemvFastRows = 1;

bool gemv_eligible(int64_t m, int64_t k, int64_t n, int64_t g) {
  return m >= 1 && m <= lvb::awqg::kMaxM && g % 32 == 0 && g <= 256 && k % g == 0 && k % 64 == 0 && n % 128 == 0 &&
         (m <= kGemvFastRows || !(m <= 32 && (g == 128 || g == 256)));
}

struct GemvPlan {
  int mt = 0, splits = 1, gps = 1;
  size_t smem = 0, sem_bytes = 0, part_bytes = 0;
  size_t total() const { return sem_bytes + part_bytes; }
};

constexpr size_t kGemvMaxSmem = 96 * 1024;

// About four 128-thread CTAs per SM, whole groups per split, shared memory
// for the split's limbs within kGemvMaxSmem; mt == 0 when no plan fits in
// `max_ws` (split-K partials and semaphores only: the limbs live in shared
// memory).
GemvPlan gemv_plan(int64_t m, int64_t k, const PackedShape &sh, int64_t g, int sms, size_t max_ws = SIZE_MAX) {
  GemvPlan p;
  (void)k;
  const int mt = m <= 1 ? 1 : m <= 2 ? 2 : 4;
  const int rpg = static_cast<int>(g / 32);
  auto smem_of = [&](int gps) {
    return mt == 1 ? lvb::awqg::GemvSmem<1>::bytes(gps, rpg)
                   : mt == 2 ? lvb::awqg::GemvSmem<2>::bytes(gps, rpg) : lvb::awqg::GemvSmem<4>::bytes(gps, rpg);
  };
  // Four CTAs per SM: best or tied among 2 / 3 / 4 / 6 on every 7B shape
  // (B200); the 16 MB QKV / o shapes sit at an ~8 us latency floor anyway.
  const long long target = 4LL * sms;
  int splits = static_cast<int>((target + sh.n_tiles - 1) / sh.n_tiles);
  if (splits < 1) splits = 1;
  if (splits > sh.groups) splits = sh.groups;
  int gps = (sh.groups + splits - 1) / splits;
  while (smem_of(gps) > kGemvMaxSmem && gps > 1) --gps;
  if (smem_of(gps) > kGemvMaxSmem) return p;
  splits = (sh.groups + gps - 1) / gps;
  // One wave: whole groups per split can round the CTA count past the four
  // resident per SM (7B down, 28 tiles: 7 groups per split gives 22 splits =
  // 616 CTAs, and the 24 of a second wave doubled the launch's time).
  while (static_cast<long long>(sh.n_tiles) * splits > target && gps < sh.groups && smem_of(gps + 1) <= kGemvMaxSmem) {
    ++gps;
    splits = (sh.groups + gps - 1) / gps;
  }
  const size_t sem = round256(static_cast<size_t>(sh.n_tiles) * 4);
  // Fewer splits when the partials do not fit the caller's workspace.
  while (true) {
    const size_t part = splits > 1 ? static_cast<size_t>(sh.n_tiles) * splits * m * lvb::awqg::kThreads * 4 : 0;
    if ((splits > 1 ? sem : 0) + part <= max_ws) {
      p.part_bytes = part;
      p.sem_bytes = splits > 1 ? sem : 0;
      break;
    }
    if (splits == 1) return p;
    const int next_gps = gps + 1;
    if (smem_of(next_gps) > kGemvMaxSmem) return p;
    gps = next_gps;
    splits = (sh.groups + gps - 1) / gps;
  }
  p.mt = mt;
  p.splits = splits;
  p.gps = gps;
  p.smem = smem_of(gps);
  return p;
}

// One launch: the GEMV builds its activation limbs itself and is a
// programmatic dependent of the kernel that produced x (its producer warp
// streams codes before that kernel has finished).
template <int MT>
int launch_awq_gemv(const GemvPlan &plan, const PackedShape &sh, const uint16_t *x, const uint8_t *codes,
                    const uint32_t *groups, const uint16_t *bias, uint16_t *y, int64_t m, int64_t k, int64_t n,
                    int64_t g, uint8_t *ws, int dev, cudaStream_t stream, int64_t x_stride, int gated,
                    const lvb::awqg::GemvRope *rope = nullptr) {
  static bool smem_done[kMaxDevices] = {false};
  auto kernel = lvb::awqg::awq_gemv_kernel<MT>;
  int rc = ensure_smem(kernel, static_cast<int>(kGemvMaxSmem), dev, smem_done);
  if (rc != LVB_OK) return rc;
  lvb::awqg::GemvParams p{};
  p.qpack = codes;
  p.szpack = groups;
  p.x = x;
  p.x_stride = x_stride;
  p.gated = gated;
  p.bias = bias;
  p.y = y;
  p.semaphores = reinterpret_cast<uint32_t *>(ws);
  p.partials = plan.splits > 1 ? reinterpret_cast<float *>(ws + plan.sem_bytes) : nullptr;
  p.M = static_cast<int>(m);
  p.K = static_cast<int>(k);
  p.N = static_cast<int>(n);
  p.G = static_cast<int>(g);
  p.groups = sh.groups;
  p.k_chunks = sh.k_chunks;
  p.runs_per_group = static_cast<int>(g / 32);
  p.n_tiles = sh.n_tiles;
  p.splits = plan.splits;
  p.groups_per_split = plan.gps;
  if (rope != nullptr) p.r = *rope;
  cudaError_t e = launch_pdl(kernel, dim3(static_cast<unsigned>(sh.n_tiles), static_cast<unsigned>(plan.splits)),
                             dim3(lvb::awqg::kCtaThreads), plan.smem, stream, p);
  if (e != cudaSuccess) return cuda_fail(e, "awq_gemv_kernel launch");
  return LVB_OK;
}

// ------------------------------------------------------------------------
// Warp-MMA plan (m <= 16, fp16 mma.sync over the packed layout)
// ------------------------------------------------------------------------
constexpr int64_t kMmaMinRows = 2;
constexpr int kMmaColsPerWarp = 16;  // consumer warps of one 16-column A tile
constexpr size_t kMmaMaxSmem = 72 * 1024;  // with the minimum ring: three CTAs per SM
// Dynamic shared memory one SM offers its CTAs (228 KB less 1 KB reserved and
// 1 KB of static shared memory per CTA, for up to four CTAs).
constexpr size_t kMmaSmPool = 220 * 1024;

// Measured on B200 (m = 2..16, rotating weight copies > L2), against the
// int8 tensor-core path and the fp16 packed kernel: 7B QKV m = 2 11.4 -> 9.1
// us, o 10.7 -> 8.0, down 23.6 -> 18.3 (m = 16: 24.0 -> 21.0), gate_up
// 31.4 -> 27.4 (m = 16: a tie, 31.6), BASELINE config 1 at m = 16 8.3 ->
// 6.4; in the 7B B = 16 decode step, where the int8 path also needs its limb
// launch, 2.84 -> 2.76 ms.  The int8 path remains the fallback when the
// caller's workspace cannot hold this kernel's split-K buffers.
bool mma_eligible(int64_t m, int64_t k, int64_t n, int64_t g, int sms) {
  (void)sms;
  return m >= kMmaMinRows && m <= lvb::awqm::kMaxRows && g % 32 == 0 && k % g == 0 && k % 64 == 0 && n % 128 == 0;
}

struct MmaPlan {
  int nt = 0, splits = 1, gps = 1, stages = lvb::awqm::kMinStages;
  size_t smem = 0, sem_bytes = 0, part_bytes = 0;
  size_t total() const { return sem_bytes + part_bytes; }
};

// About three CTAs per SM in one wave, whole groups per split; then the ring
// takes the shared memory the resident CTAs leave (the kernel is bound by the
// bytes it keeps in flight).  nt == 0 when no plan fits in `max_ws` (split-K
// partials and semaphores).
MmaPlan mma_plan(int64_t m, const PackedShape &sh, int64_t g, int sms, size_t max_ws = SIZE_MAX) {
  MmaPlan p;
  const int nt = m <= 8 ? 1 : 2;
  auto smem_of = [&](int gps, int stages) {
    return nt == 1 ? lvb::awqm::MmaCfg<1>::bytes(gps, stages) : lvb::awqm::MmaCfg<2>::bytes(gps, stages);
  };
  const int min_st = lvb::awqm::kMinStages;
  (void)g;
  const long long target = 3LL * sms;
  int splits = static_cast<int>((target + sh.n_tiles - 1) / sh.n_tiles);
  if (splits < 1) splits = 1;
  if (splits > sh.groups) splits = sh.groups;
  int gps = (sh.groups + splits - 1) / splits;
  while (smem_of(gps, min_st) > kMmaMaxSmem && gps > 1) --gps;
  if (smem_of(gps, min_st) > kMmaMaxSmem) return p;
  splits = (sh.groups + gps - 1) / gps;
  while (static_cast<long long>(sh.n_tiles) * splits > target && gps < sh.groups &&
         smem_of(gps + 1, min_st) <= kMmaMaxSmem) {
    ++gps;
    splits = (sh.groups + gps - 1) / gps;
  }
  const size_t sem = round256(static_cast<size_t>(sh.n_tiles) * 4);
  while (true) {
    const size_t part = splits > 1 ? static_cast<size_t>(sh.n_tiles) * splits * m * lvb::awqm::kCols * 4 : 0;
    if ((splits > 1 ? sem : 0) + part <= max_ws) {
      p.part_bytes = part;
      p.sem_bytes = splits > 1 ? sem : 0;
      break;
    }
    if (splits == 1) return p;
    if (smem_of(gps + 1, min_st) > kMmaMaxSmem) return p;
    ++gps;
    splits = (sh.groups + gps - 1) / gps;
  }
  long long per_sm = (static_cast<long long>(sh.n_tiles) * splits + sms - 1) / sms;
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 4) per_sm = 4;
  const size_t budget = kMmaSmPool / static_cast<size_t>(per_sm);
  int stages = min_st;
  while (stages < lvb::awqm::kMaxStages && smem_of(gps, stages + 1) <= budget) ++stages;
  p.nt = nt;
  p.splits = splits;
  p.gps = gps;
  p.stages = stages;
  p.smem = smem_of(gps, stages);
  return p;
}

template <int NT>
int launch_awq_mma(const MmaPlan &plan, const PackedShape &sh, const uint16_t *x, const uint8_t *codes,
                   const uint32_t *groups, const uint16_t *bias, uint16_t *y, int64_t m, int64_t n, int64_t g,
                   uint8_t *ws, int dev, cudaStream_t stream, int64_t x_stride) {
  static bool smem_done[kMaxDevices] = {false};
  auto kernel = lvb::awqm::awq_mma_kernel<NT, kMmaColsPerWarp>;
  int rc = ensure_smem(kernel, static_cast<int>(kMmaSmPool), dev, smem_done);
  if (rc != LVB_OK) return rc;
  lvb::awqm::MmaParams p{};
  p.qpack = codes;
  p.szpack = groups;
  p.x = x;
  p.x_stride = x_stride;
  p.bias = bias;
  p.y = y;
  p.semaphores = reinterpret_cast<uint32_t *>(ws);
  p.partials = plan.splits > 1 ? reinterpret_cast<float *>(ws + plan.sem_bytes) : nullptr;
  p.M = static_cast<int>(m);
  p.N = static_cast<int>(n);
  p.groups = sh.groups;
  p.k_chunks = sh.k_chunks;
  p.runs_per_group = static_cast<int>(g / 32);
  p.n_tiles = sh.n_tiles;
  p.splits = plan.splits;
  p.groups_per_split = plan.gps;
  p.stages = plan.stages;
  cudaError_t e = launch_pdl(kernel, dim3(static_cast<unsigned>(sh.n_tiles), static_cast<unsigned>(plan.splits)),
                             dim3(lvb::awqm::MmaWarps<kMmaColsPerWarp>::kCtaThreads), plan.smem, stream, p);
  if (e != cudaSuccess) return cuda_fail(e, "awq_mma_kernel launch");
  return LVB_OK;
}

int check_awq_shape(int64_t m, int64_t k, int64_t n, int64_t group_size) {
  if (m < 0 || k <= 0 || n <= 0)
    return fail(LVB_ERR_INVALID, "invalid AWQ shape m=%lld k=%lld n=%lld", (long long)m, (long long)k, (long long)n);
  if (m > INT_MAX || k > INT_MAX || n > INT_MAX) return fail(LVB_ERR_UNSUPPORTED, "AWQ dimension exceeds int32");
  if (group_size <= 0 || group_size % 32 != 0 || k % group_size != 0)
    return fail(LVB_ERR_INVALID, "AWQ group_size %lld must be a positive multiple of 32 dividing k=%lld",
                (long long)group_size, (long long)k);
  if (n % 32 != 0) return fail(LVB_ERR_INVALID, "AWQ output width %lld must be divisible by 32", (long long)n);
  if (k % 8 != 0) return fail(LVB_ERR_INVALID, "AWQ input width %lld must be divisible by 8", (long long)k);
  return LVB_OK;
}

// ------------------------------------------------------------------------
// Attention planning
// ------------------------------------------------------------------------
struct DecodePlan {
  int max_splits, chunk_tokens, heads_per_cta, warps_per_head;
  bool flat;  // balanced schedule (paged_decode_flat_kernel): max_splits bounds the pieces per request
  size_t o_bytes, lse_bytes, count_bytes;
  size_t total() const { return o_bytes + lse_bytes + count_bytes; }
};

// Fewest pages one split covers (shorter splits only add merge traffic):
// measured best on B200 at 8 pages for small batches and 16 from 32 requests
// up (B = 64, ctx 1024: 38.5 -> 34.1 us).
constexpr int64_t kMinSplitPagesSmall = 8;
// Four warps per head (a handful of requests): 4-page splits put more CTAs on
// the context (B200, 7B heads, one request, ctx 1024: 10.3 -> 8.2 us with the
// merge launch; 2-page splits 10.3).
constexpr int64_t kMinSplitPagesTiny = 4;
constexpr int64_t kMinSplitPagesLarge = 16;
// Batches below this many requests run one KV head per CTA.
constexpr int64_t kAttnSmallBatch = 32;
// The balanced schedule (paged_decode_flat_kernel) measured slower than the
// split kernel on the decode batches tried on B200 (config 2: 65.7 vs
// 59.9 us; uniform 2304-token contexts 69.1 vs 69.1), so large batches take
// the split kernel.
constexpr bool kBalancedDecode = false;

DecodePlan decode_plan(int64_t num_seqs, int64_t hq, int64_t hkv, int64_t d, int64_t max_seq_len,
                       int sms) {
  DecodePlan p{};
  const int64_t max_pages = (max_seq_len + lvb::attn::kPageTokens - 1) / lvb::attn::kPageTokens;
  // Small batches: one KV head per CTA, so (request, head) pairs and their
  // merges spread over more SMs.
  const bool small = num_seqs < kAttnSmallBatch;
  const int64_t hpc = small ? 1 : hkv % 4 == 0 ? 4 : hkv % 2 == 0 ? 2 : 1;
  // Very small batches: four warps share each (request, head) split, cutting
  // the serial per-warp page work and widening the split merge (B200, ctx
  // 1024: B = 1 14.0 -> 10.4 us; at B = 16 it loses, 17.1 -> 20.7 us).
  const int64_t kw = small && num_seqs * hkv <= 32 ? 4 : 1;
  const int64_t pairs = num_seqs * (hkv / hpc) > 0 ? num_seqs * (hkv / hpc) : 1;
  const int64_t target = (kw > 1 ? 2LL : 8LL) * sms;  // CTAs: ~8 warps per SM either way
  int64_t splits = (target + pairs - 1) / pairs;
  if (splits < 1) splits = 1;
  if (splits > max_pages) splits = max_pages > 0 ? max_pages : 1;
  if (splits > 256) splits = 256;  // merge weights: (heads per CTA) x splits floats in shared memory
  int64_t chunk_pages = (max_pages + splits - 1) / splits > 0 ? (max_pages + splits - 1) / splits : 1;
  const int64_t min_pages =
      kw > 1 ? kMinSplitPagesTiny : num_seqs < kAttnSmallBatch ? kMinSplitPagesSmall : kMinSplitPagesLarge;
  if (chunk_pages < min_pages) chunk_pages = min_pages;
  splits = (max_pages + chunk_pages - 1) / chunk_pages;
  if (splits < 1) splits = 1;
  p.max_splits = static_cast<int>(splits);
  p.chunk_tokens = static_cast<int>(chunk_pages * lvb::attn::kPageTokens);
  p.heads_per_cta = static_cast<int>(hpc);
  p.warps_per_head = static_cast<int>(kw);
  // Large batches run the balanced schedule when its tables and merge
  // weights fit in shared memory (one CTA's page rings hold the weights).
  p.flat = false;
  if (kBalancedDecode && !small && num_seqs <= lvb::attn::kFlatMaxSeqs && max_pages <= INT_MAX / 2) {
    const int pieces = lvb::attn::flat_max_pieces(static_cast<int>(max_pages));
    const int ring_bytes = hpc == 4   ? (d == 128 ? lvb::attn::DecodeCfg<128, 4>::kBarOff : lvb::attn::DecodeCfg<64, 4>::kBarOff)
                           : hpc == 2 ? (d == 128 ? lvb::attn::DecodeCfg<128, 2>::kBarOff : lvb::attn::DecodeCfg<64, 2>::kBarOff)
                                      : (d == 128 ? lvb::attn::DecodeCfg<128, 1>::kBarOff : lvb::attn::DecodeCfg<64, 1>::kBarOff);
    if (static_cast<int64_t>(hpc) * (hq / hkv) * pieces * 4 <= ring_bytes) {
      p.flat = true;
      splits = pieces;
      p.max_splits = pieces;
    }
  }
  p.o_bytes = (static_cast<size_t>(num_seqs * hq * splits * d) * 4 + 255) & ~static_cast<size_t>(255);
  p.lse_bytes = (static_cast<size_t>(num_seqs * hq * splits) * 4 + 255) & ~static_cast<size_t>(255);
  p.count_bytes = (static_cast<size_t>(num_seqs * hkv) * 4 + 255) & ~static_cast<size_t>(255);
  return p;
}

bool decode_eligible(const uint8_t *vis, int64_t max_query_len, int64_t num_seqs, int64_t num_tokens,
                     int64_t hq, int64_t hkv, int64_t d, int64_t bs) {
  return vis == nullptr && max_query_len == 1 && num_tokens == num_seqs && bs == lvb::attn::kPageTokens &&
         (d == 64 || d == 128) && hq % hkv == 0 && hq / hkv <= 16;
}

bool decode_shape_ok(int64_t hq, int64_t hkv, int64_t d, int64_t bs) {
  return bs == lvb::attn::kPageTokens && (d == 64 || d == 128) && hq % hkv == 0 && hq / hkv <= 16;
}

// Tensor-core tile kernel: head sizes 64 / 128, 16-token blocks, any GQA group.
bool tile_eligible(int64_t hq, int64_t hkv, int64_t d, int64_t bs) {
  return bs == lvb::attn::kPageTokens && (d == 64 || d == 128) && hq % hkv == 0;
}

template <bool kBf16, int D>
int launch_prefill(const lvb::attn::AttnArgs &a, dim3 grid, int dev, cudaStream_t stream) {
  using Cfg = lvb::attn::PrefillCfg<D>;
  static bool smem_done[kMaxDevices] = {false};
  auto kernel = lvb::attn::paged_prefill_kernel<kBf16, D>;
  int rc = ensure_smem(kernel, Cfg::kSmemBytes, dev, smem_done);
  if (rc != LVB_OK) return rc;
  cudaError_t e = launch_pdl(kernel, grid, dim3(128), Cfg::kSmemBytes, stream, a);
  if (e != cudaSuccess) return cuda_fail(e, "paged_prefill_kernel launch");
  return LVB_OK;
}

template <bool kBf16, int D, int HPC, int KW = 1, int NT = 1>
int launch_decode(const lvb::attn::AttnArgs &a, int64_t num_seqs, int64_t num_blocks, int dev,
                  cudaStream_t stream) {
  (void)num_blocks;
  using Cfg = lvb::attn::DecodeCfg<D, HPC, KW>;
  static bool smem_done[kMaxDevices] = {false};
  auto kernel = lvb::attn::paged_decode_kernel<kBf16, D, HPC, KW, NT>;
  int rc = ensure_smem(kernel, Cfg::kSmemBytes, dev, smem_done);
  if (rc != LVB_OK) return rc;
  dim3 grid(a.max_splits, a.Hkv / HPC, static_cast<unsigned>(num_seqs));
  cudaError_t e = launch_pdl(kernel, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, a);
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode_kernel launch");
  if (a.max_splits > 1) {
    e = launch_pdl(lvb::attn::decode_merge_kernel<kBf16, D>, dim3((a.Hq + 3) / 4, static_cast<unsigned>(num_seqs)),
                   dim3(128), 0, stream, a);
    if (e != cudaSuccess) return cuda_fail(e, "decode_merge_kernel launch");
  }
  return LVB_OK;
}

// Balanced schedule: one wave of CTAs (the occupancy calculator's resident
// count per SM x the SM count, over the KV head groups).
template <bool kBf16, int D, int HPC, int NT>
int launch_decode_flat(lvb::attn::AttnArgs a, int64_t num_seqs, int dev, cudaStream_t stream) {
  using Cfg = lvb::attn::FlatCfg<D, HPC>;
  auto kernel = lvb::attn::paged_decode_flat_kernel<kBf16, D, HPC, NT>;
  static bool smem_done[kMaxDevices] = {false};
  static int resident[kMaxDevices] = {0};
  const int max_smem = Cfg::smem_bytes(lvb::attn::kFlatMaxSeqs);
  int rc = ensure_smem(kernel, max_smem, dev, smem_done);
  if (rc != LVB_OK) return rc;
  if (resident[dev] == 0) {
    int nb = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, HPC * 32, max_smem);
    if (e != cudaSuccess) return cuda_fail(e, "paged_decode_flat_kernel occupancy");
    resident[dev] = nb > 0 ? nb : 1;
  }
  a.decode_seqs = static_cast<int>(num_seqs);
  a.heads_per_cta = HPC;
  const int groups = a.Hkv / HPC;
  int ctas = resident[dev] * sm_count(dev) / groups;
  if (ctas < 1) ctas = 1;
  const dim3 grid(static_cast<unsigned>(ctas), static_cast<unsigned>(groups));
  cudaError_t e = launch_pdl(kernel, grid, dim3(HPC * 32), Cfg::smem_bytes(static_cast<int>(num_seqs)), stream, a);
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode_flat_kernel launch");
  e = launch_pdl(lvb::attn::decode_merge_kernel<kBf16, D, true>, dim3((a.Hq + 3) / 4, static_cast<unsigned>(num_seqs)),
                 dim3(128), 0, stream, a);
  if (e != cudaSuccess) return cuda_fail(e, "decode_merge_kernel launch");
  return LVB_OK;
}

// NT = 8-head tiles of the GQA group (groups of up to 8 heads: one).
template <bool kBf16, int D, int NT>
int launch_decode_nt(const lvb::attn::AttnArgs &a, const DecodePlan &plan, int64_t num_seqs, int64_t num_blocks,
                     int dev, cudaStream_t stream) {
  const int heads_per_cta = plan.heads_per_cta, warps_per_head = plan.warps_per_head;
  if (plan.flat) {
    switch (heads_per_cta) {
      case 4: return launch_decode_flat<kBf16, D, 4, NT>(a, num_seqs, dev, stream);
      case 2: return launch_decode_flat<kBf16, D, 2, NT>(a, num_seqs, dev, stream);
      default: return launch_decode_flat<kBf16, D, 1, NT>(a, num_seqs, dev, stream);
    }
  }
  if (warps_per_head == 4) return launch_decode<kBf16, D, 1, 4, NT>(a, num_seqs, num_blocks, dev, stream);
  switch (heads_per_cta) {
    case 4: return launch_decode<kBf16, D, 4, 1, NT>(a, num_seqs, num_blocks, dev, stream);
    case 2: return launch_decode<kBf16, D, 2, 1, NT>(a, num_seqs, num_blocks, dev, stream);
    default: return launch_decode<kBf16, D, 1, 1, NT>(a, num_seqs, num_blocks, dev, stream);
  }
}

template <bool kBf16, int D>
int launch_decode_any(const lvb::attn::AttnArgs &a, const DecodePlan &plan, int64_t num_seqs, int64_t num_blocks,
                      int dev, cudaStream_t stream) {
  return a.Hq / a.Hkv <= 8 ? launch_decode_nt<kBf16, D, 1>(a, plan, num_seqs, num_blocks, dev, stream)
                           : launch_decode_nt<kBf16, D, 2>(a, plan, num_seqs, num_blocks, dev, stream);
}

template <bool kBf16>
int launch_general(const lvb::attn::AttnArgs &a, int64_t num_tokens, cudaStream_t stream) {
  dim3 grid(static_cast<unsigned>(num_tokens), a.Hq);
  const int dpl = (a.D + 31) / 32;
  cudaError_t e;
  if (dpl <= 1)
    e = launch_pdl(lvb::attn::paged_attn_general_kernel<kBf16, 1>, grid, dim3(128), 0, stream, a);
  else if (dpl == 2)
    e = launch_pdl(lvb::attn::paged_attn_general_kernel<kBf16, 2>, grid, dim3(128), 0, stream, a);
  else if (dpl == 3)
    e = launch_pdl(lvb::attn::paged_attn_general_kernel<kBf16, 3>, grid, dim3(128), 0, stream, a);
  else if (dpl == 4)
    e = launch_pdl(lvb::attn::paged_attn_general_kernel<kBf16, 4>, grid, dim3(128), 0, stream, a);
  else
    e = launch_pdl(lvb::attn::paged_attn_general_kernel<kBf16, 8>, grid, dim3(128), 0, stream, a);
  if (e != cudaSuccess) return cuda_fail(e, "paged_attn_general_kernel launch");
  return LVB_OK;
}

// ------------------------------------------------------------------------
// Fixed scratch for lvb_awq_linear_static
// ------------------------------------------------------------------------
// Callers that cannot allocate device memory get the split-K scratch from this
// file-scope array instead.  6 MiB + 4 KiB covers every split-K plan on GPUs
// with up to 192 SMs: at most SMs x 64 x 128 fp32 partials (6 MiB at 192 SMs)
// plus the semaphore block in front of them (one uint32 per output tile,
// rounded to 256 bytes).  It is part of the module image: every device that
// loads the library holds it until the process exits.
constexpr size_t kAwqStaticScratchBytes = (size_t(6) << 20) + 4096;
constexpr size_t kKvMoveMaxSmem = 96 * 1024;  // rows staged by one KV-move CTA
__device__ __align__(256) unsigned char g_awq_static_scratch[kAwqStaticScratchBytes];

// Device address of the array on each device.  In host code the symbol is a
// host-side stand-in, not a device address, so it is looked up once per device
// (with that device current) and only the looked-up pointer reaches a kernel.
// Double-checked: the lock is taken only while a device's address is still
// unknown, so later calls read one atomic.  The cached address belongs to the
// device's primary context; after cudaDeviceReset it is stale.
std::atomic<void *> g_awq_static_scratch_addr[kMaxDevices];
std::mutex g_awq_static_scratch_mu;

int awq_static_scratch(int dev, void **out) {
  void *p = g_awq_static_scratch_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_awq_static_scratch_mu);
    p = g_awq_static_scratch_addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      cudaError_t e = cudaGetSymbolAddress(&p, g_awq_static_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_awq_static_scratch)");
      g_awq_static_scratch_addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return LVB_OK;
}

}  // namespace

extern "C" {

int lvb_abi_version(void) { return kAbiVersion; }

const char *lvb_last_error(void) { return g_last_error; }

int lvb_device_error(uint32_t *error_out) {
  if (error_out == nullptr) return fail(LVB_ERR_INVALID, "error_out is null");
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, lvb::g_device_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  const unsigned int zero = 0;
  e = cudaMemcpyToSymbol(lvb::g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  *error_out = v;
  return LVB_OK;
}

size_t lvb_awq_workspace_bytes(int64_t m, int64_t k, int64_t n, int64_t group_size) {
  if (m <= 0 || k <= 0 || n <= 0) return 0;
  int dev = 0;
  if (current_device(&dev) != LVB_OK) return 0;
  const AwqPlan p = awq_plan(m, k, n, sm_count(dev));
  size_t need = p.sem_bytes + p.part_bytes;
  if (group_size > 0 && group_size % 32 == 0 && k % group_size == 0) {
    const PackedShape sh = packed_shape(k, n, group_size);
    const PackedPlan pp = packed_plan(m, sh, sm_count(dev) * packed_ctas_per_sm(packed_bn(m), sh, m, sm_count(dev)));
    if (pp.sem_bytes + pp.part_bytes > need) need = pp.sem_bytes + pp.part_bytes;
    if (i8_eligible(m, k, n, group_size)) {
      const I8Plan ip = i8_plan(m, k, sh, group_size, sm_count(dev));
      if (ip.total() > need) need = ip.total();
    }
    if (gemv_eligible(m, k, n, group_size)) {
      const GemvPlan gp = gemv_plan(m, k, sh, group_size, sm_count(dev));
      if (gp.total() > need) need = gp.total();
    }
    if (mma_eligible(m, k, n, group_size, sm_count(dev))) {
      // The fused SiLU-mul entry also keeps the m x k activation there.
      const MmaPlan mp = mma_plan(m, sh, group_size, sm_count(dev));
      const size_t with_act = round256(mp.total()) + round256(static_cast<size_t>(m) * k * 2) + 256;
      if (with_act > need) need = with_act;
    }
  }
  return need;
}

int lvb_awq_linear(const uint16_t *x, const int32_t *qweight, const int32_t *qzeros,
                   const uint16_t *scales, const uint16_t *bias, uint16_t *y, int64_t m,
                   int64_t k, int64_t n, int64_t group_size, void *workspace,
                   size_t workspace_bytes, lvb_stream_t stream) {
  if (m < 0 || k <= 0 || n <= 0) return fail(LVB_ERR_INVALID, "invalid AWQ shape m=%lld k=%lld n=%lld",
                                              (long long)m, (long long)k, (long long)n);
  if (m == 0) return LVB_OK;
  if (m > INT_MAX || k > INT_MAX || n > INT_MAX) return fail(LVB_ERR_UNSUPPORTED, "AWQ dimension exceeds int32");
  if (group_size <= 0 || group_size % 32 != 0 || k % group_size != 0)
    return fail(LVB_ERR_INVALID, "AWQ group_size %lld must be a positive multiple of 32 dividing k=%lld",
                (long long)group_size, (long long)k);
  if (n % 32 != 0) return fail(LVB_ERR_INVALID, "AWQ output width %lld must be divisible by 32", (long long)n);
  if (k % 8 != 0) return fail(LVB_ERR_INVALID, "AWQ input width %lld must be divisible by 8", (long long)k);
  if (!x || !qweight || !qzeros || !scales || !y) return fail(LVB_ERR_INVALID, "AWQ null pointer argument");
  if (!aligned16(x) || !aligned16(qweight) || !aligned16(qzeros) || !aligned16(scales) ||
      (workspace && !aligned16(workspace)))
    return fail(LVB_ERR_INVALID, "AWQ x, qweight, scales and workspace must be 16-byte aligned");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const AwqPlan plan = awq_plan(m, k, n, sm_count(dev));
  if ((plan.sem_bytes + plan.part_bytes) > 0 && (workspace == nullptr || workspace_bytes < plan.sem_bytes + plan.part_bytes))
    return fail(LVB_ERR_WORKSPACE, "AWQ workspace of %zu bytes is below the %zu required", workspace_bytes,
                plan.sem_bytes + plan.part_bytes);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return dispatch_awq(plan, x, qweight, qzeros, scales, bias, y, m, k, n, group_size, ws, dev, s);
}

int lvb_awq_dequantize(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales,
                       uint16_t *w, int64_t k, int64_t n, int64_t group_size, lvb_stream_t stream) {
  if (k <= 0 || n <= 0 || n % 8 != 0 || group_size <= 0 || k % group_size != 0)
    return fail(LVB_ERR_INVALID, "invalid AWQ dequantize shape k=%lld n=%lld group=%lld", (long long)k,
                (long long)n, (long long)group_size);
  if (k > INT_MAX || n > INT_MAX) return fail(LVB_ERR_UNSUPPORTED, "AWQ dimension exceeds int32");
  if (!qweight || !qzeros || !scales || !w) return fail(LVB_ERR_INVALID, "AWQ null pointer argument");
  if (!aligned16(scales) || !aligned16(w)) return fail(LVB_ERR_INVALID, "scales and w must be 16-byte aligned");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const long long words = k * (n / 8);
  long long blocks = (words + 255) / 256;
  const long long cap = static_cast<long long>(sm_count(dev)) * 8;
  if (blocks > cap) blocks = cap;
  lvb::awq::awq_dequantize_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                                    reinterpret_cast<cudaStream_t>(stream)>>>(
      qweight, qzeros, scales, w, static_cast<int>(k), static_cast<int>(n), static_cast<int>(group_size));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "awq_dequantize_kernel launch");
  return LVB_OK;
}

int lvb_awq_pack_bytes(int64_t k, int64_t n, int64_t group_size, size_t *codes_bytes, size_t *groups_bytes) {
  int rc = check_awq_shape(0, k, n, group_size);
  if (rc != LVB_OK) return rc;
  if (!codes_bytes || !groups_bytes) return fail(LVB_ERR_INVALID, "AWQ pack null pointer argument");
  const PackedShape sh = packed_shape(k, n, group_size);
  *codes_bytes = sh.codes_bytes;
  *groups_bytes = sh.groups_bytes;
  return LVB_OK;
}

int lvb_awq_pack(const int32_t *qweight, const int32_t *qzeros, const uint16_t *scales, int64_t k, int64_t n,
                 int64_t group_size, void *codes, void *groups, lvb_stream_t stream) {
  int rc = check_awq_shape(0, k, n, group_size);
  if (rc != LVB_OK) return rc;
  if (!qweight || !qzeros || !scales || !codes || !groups) return fail(LVB_ERR_INVALID, "AWQ pack null pointer argument");
  if (!aligned16(codes) || !aligned16(groups)) return fail(LVB_ERR_INVALID, "packed AWQ buffers must be 16-byte aligned");
  int dev = 0;
  rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const PackedShape sh = packed_shape(k, n, group_size);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long code_threads = static_cast<long long>(sh.n_tiles) * sh.k_chunks * lvb::awqd::kTileN;
  lvb::awqd::awq_pack_codes_kernel<<<static_cast<unsigned>((code_threads + 255) / 256), 256, 0, s>>>(
      qweight, static_cast<uint8_t *>(codes), static_cast<int>(k), static_cast<int>(n), sh.k_chunks, sh.n_tiles);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "awq_pack_codes_kernel launch");
  const long long group_threads = static_cast<long long>(sh.n_tiles) * sh.groups * lvb::awqd::kTileN;
  lvb::awqd::awq_pack_groups_kernel<<<static_cast<unsigned>((group_threads + 255) / 256), 256, 0, s>>>(
      qzeros, scales, static_cast<uint32_t *>(groups), static_cast<int>(n), sh.groups, sh.n_tiles);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "awq_pack_groups_kernel launch");
  return LVB_OK;
}

int lvb_awq_linear_packed(const uint16_t *x, const void *codes, const void *groups, const uint16_t *bias,
                          uint16_t *y, int64_t m, int64_t k, int64_t n, int64_t group_size, void *workspace,
                          size_t workspace_bytes, lvb_stream_t stream) {
  int rc = check_awq_shape(m, k, n, group_size);
  if (rc != LVB_OK) return rc;
  if (m == 0) return LVB_OK;
  if (!x || !codes || !groups || !y) return fail(LVB_ERR_INVALID, "AWQ null pointer argument");
  if (!aligned16(x) || !aligned16(codes) || !aligned16(groups) || (workspace && !aligned16(workspace)))
    return fail(LVB_ERR_INVALID, "AWQ x, packed buffers and workspace must be 16-byte aligned");
  int dev = 0;
  rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const PackedShape sh = packed_shape(k, n, group_size);
  const size_t max_ws = workspace != nullptr ? workspace_bytes : 0;
  cudaStream_t stream_ = reinterpret_cast<cudaStream_t>(stream);
  if (mma_eligible(m, k, n, group_size, sm_count(dev))) {
    const MmaPlan mp = mma_plan(m, sh, group_size, sm_count(dev), max_ws);
    const uint8_t *c8 = static_cast<const uint8_t *>(codes);
    const uint32_t *g8 = static_cast<const uint32_t *>(groups);
    uint8_t *w8 = static_cast<uint8_t *>(workspace);
    if (mp.nt == 1) return launch_awq_mma<1>(mp, sh, x, c8, g8, bias, y, m, n, group_size, w8, dev, stream_, k);
    if (mp.nt == 2) return launch_awq_mma<2>(mp, sh, x, c8, g8, bias, y, m, n, group_size, w8, dev, stream_, k);
  }
  if (gemv_eligible(m, k, n, group_size)) {
    const GemvPlan gp = gemv_plan(m, k, sh, group_size, sm_count(dev), max_ws);
    const uint8_t *c8 = static_cast<const uint8_t *>(codes);
    const uint32_t *g8 = static_cast<const uint32_t *>(groups);
    uint8_t *w8 = static_cast<uint8_t *>(workspace);
    if (gp.mt == 1) return launch_awq_gemv<1>(gp, sh, x, c8, g8, bias, y, m, k, n, group_size, w8, dev, stream_, k, 0);
    if (gp.mt == 2) return launch_awq_gemv<2>(gp, sh, x, c8, g8, bias, y, m, k, n, group_size, w8, dev, stream_, k, 0);
    if (gp.mt == 4) return launch_awq_gemv<4>(gp, sh, x, c8, g8, bias, y, m, k, n, group_size, w8, dev, stream_, k, 0);
  }
  if (i8_eligible(m, k, n, group_size) && aligned16(y)) {  // y is written by TMA stores
    const I8Plan ip = i8_plan(m, k, sh, group_size, sm_count(dev), max_ws);
    const uint8_t *c8 = static_cast<const uint8_t *>(codes);
    const uint32_t *g8 = static_cast<const uint32_t *>(groups);
    uint8_t *w8 = static_cast<uint8_t *>(workspace);
    if (ip.bn == 16) return launch_awq_i8<16>(ip, sh, x, c8, g8, bias, y, m, k, n, group_size, w8, dev, stream_, k, 0);
  }
  // The plan never needs more split-K workspace than the caller passed.
  const int per_sm = packed_ctas_per_sm(packed_bn(m), sh, m, sm_count(dev));
  const PackedPlan plan = packed_plan(m, sh, sm_count(dev) * per_sm, max_ws);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint8_t *c = static_cast<const uint8_t *>(codes);
  const uint32_t *g = static_cast<const uint32_t *>(groups);
  switch (plan.bn) {
    case 16: return launch_awq_packed<16, 4, 2, true>(plan, sh, x, c, g, bias, y, m, k, n, group_size, ws, dev, s);
    case 32: return launch_awq_packed<32, 4, 2, true>(plan, sh, x, c, g, bias, y, m, k, n, group_size, ws, dev, s);
    case 64:
      if (per_sm == 2)
        return launch_awq_packed<64, 2, 1, true, 256, 108>(plan, sh, x, c, g, bias, y, m, k, n, group_size, ws, dev, s);
      return launch_awq_packed<64, 4, 2, true>(plan, sh, x, c, g, bias, y, m, k, n, group_size, ws, dev, s);
    case 128:
      if (per_sm == 2)
        return launch_awq_packed<128, 1, 1, false, 256, 108>(plan, sh, x, c, g, bias, y, m, k, n, group_size, ws, dev, s);
      return launch_awq_packed<128, 2, 2, true>(plan, sh, x, c, g, bias, y, m, k, n, group_size, ws, dev, s);
    // 256-row tiles: 128-k stages with two dequantiser warpgroups (each one
    // 64-k block of a stage), three stages in 224 KB of shared memory.
    // Measured on B200 against 64-k stages and one warpgroup (the tensor pipe
    // waited for A stages, 35 % active): m = 2048, 3584 x 37888: 746 -> 664 us
    // (837 TFLOP/s); the 14B prefill shapes at m = 2112: 733 -> 847, 729 ->
    // 872, 649 -> 758 TFLOP/s.
    default:
      return launch_awq_packed<256, 2, 2, false, 512, 224>(plan, sh, x, c, g, bias, y, m, k, n, group_size, ws, dev, s);
  }
}

int lvb_awq_qkv_rope_packed(const uint16_t *x, const void *codes, const void *groups, const uint16_t *bias,
                            uint16_t *y, int64_t m, int64_t k, int64_t n, int64_t group_size, void *workspace,
                            size_t workspace_bytes, const int32_t *positions, const uint16_t *cos_table,
                            const uint16_t *sin_table, int64_t table_rows, uint16_t *key_cache,
                            uint16_t *value_cache, const int32_t *block_tables, int64_t table_stride,
                            const int32_t *num_computed, const int32_t *query_start_loc,
                            const int32_t *request_indices, int64_t num_query_heads, int64_t num_kv_heads,
                            int64_t head_size, int64_t block_size, lvb_stream_t stream) {
  int rc = check_awq_shape(m, k, n, group_size);
  if (rc != LVB_OK) return rc;
  if (m == 0) return LVB_OK;
  if (!x || !codes || !groups || !y || !positions || !cos_table || !sin_table || !key_cache || !value_cache ||
      !block_tables || !num_computed || !query_start_loc || !request_indices)
    return fail(LVB_ERR_INVALID, "QKV epilogue null pointer argument");
  if (!aligned16(x) || !aligned16(codes) || !aligned16(groups) || (workspace && !aligned16(workspace)))
    return fail(LVB_ERR_INVALID, "AWQ x, packed buffers and workspace must be 16-byte aligned");
  if ((head_size != 64 && head_size != 128) || num_query_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 ||
      n != (num_query_heads + 2 * num_kv_heads) * head_size || table_rows <= 0)
    return fail(LVB_ERR_UNSUPPORTED, "QKV epilogue covers head sizes 64 / 128 over merged [q | k | v] rows");
  if (!gemv_eligible(m, k, n, group_size))
    return fail(LVB_ERR_UNSUPPORTED, "QKV epilogue covers the one-row decode GEMV (m = 1)");
  int dev = 0;
  rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const PackedShape sh = packed_shape(k, n, group_size);
  const GemvPlan gp = gemv_plan(m, k, sh, group_size, sm_count(dev), workspace != nullptr ? workspace_bytes : 0);
  if (gp.mt == 0) return fail(LVB_ERR_UNSUPPORTED, "QKV epilogue: the GEMV plan does not fit the workspace");
  lvb::awqg::GemvRope r{};
  r.rope = 1;
  r.positions = positions;
  r.cos = cos_table;
  r.sin = sin_table;
  r.key_cache = key_cache;
  r.value_cache = value_cache;
  r.tables = block_tables;
  r.table_stride = table_stride;
  r.computed = num_computed;
  r.qsl = query_start_loc;
  r.req = request_indices;
  r.hq = static_cast<int>(num_query_heads);
  r.hkv = static_cast<int>(num_kv_heads);
  r.D = static_cast<int>(head_size);
  r.bs = static_cast<int>(block_size);
  r.table_rows = static_cast<int>(table_rows);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const uint8_t *c8 = static_cast<const uint8_t *>(codes);
  const uint32_t *g8 = static_cast<const uint32_t *>(groups);
  uint8_t *w8 = static_cast<uint8_t *>(workspace);
  if (gp.mt == 1) return launch_awq_gemv<1>(gp, sh, x, c8, g8, bias, y, m, k, n, group_size, w8, dev, st, k, 0, &r);
  if (gp.mt == 2) return launch_awq_gemv<2>(gp, sh, x, c8, g8, bias, y, m, k, n, group_size, w8, dev, st, k, 0, &r);
  return launch_awq_gemv<4>(gp, sh, x, c8, g8, bias, y, m, k, n, group_size, w8, dev, st, k, 0, &r);
}

int lvb_awq_silu_linear_packed(const uint16_t *gate_up, int64_t gate_up_stride, const void *codes,
                               const void *groups, const uint16_t *bias, uint16_t *y, int64_t m, int64_t k, int64_t n,
                               int64_t group_size, void *workspace, size_t workspace_bytes, lvb_stream_t stream) {
  int rc = check_awq_shape(m, k, n, group_size);
  if (rc != LVB_OK) return rc;
  if (m == 0) return LVB_OK;
  if (!gate_up || !codes || !groups || !y) return fail(LVB_ERR_INVALID, "AWQ null pointer argument");
  if (gate_up_stride < 2 * k || gate_up_stride % 8 != 0)
    return fail(LVB_ERR_INVALID, "gate/up row stride %lld must cover 2 x %lld values and be a multiple of 8",
                (long long)gate_up_stride, (long long)k);
  if (!aligned16(gate_up) || !aligned16(codes) || !aligned16(groups) || (workspace && !aligned16(workspace)))
    return fail(LVB_ERR_INVALID, "AWQ gate/up, packed buffers and workspace must be 16-byte aligned");
  int dev = 0;
  rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const PackedShape sh = packed_shape(k, n, group_size);
  const size_t max_ws = workspace != nullptr ? workspace_bytes : 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const uint8_t *c8 = static_cast<const uint8_t *>(codes);
  const uint32_t *g8 = static_cast<const uint32_t *>(groups);
  uint8_t *w8 = static_cast<uint8_t *>(workspace);
  if (mma_eligible(m, k, n, group_size, sm_count(dev))) {
    // silu(gate) * up into the workspace behind the split-K buffers, then
    // the warp-MMA projection of it (two launches, programmatic dependents).
    const size_t act = round256(static_cast<size_t>(m) * k * 2);
    const MmaPlan mp = max_ws > act + 256 ? mma_plan(m, sh, group_size, sm_count(dev), max_ws - act - 256) : MmaPlan{};
    if (mp.nt != 0) {
      uint16_t *a16 = reinterpret_cast<uint16_t *>(w8 + round256(mp.total()));
      rc = lvb_silu_mul(gate_up, gate_up_stride, m, k, a16, k, stream);
      if (rc != LVB_OK) return rc;
      if (mp.nt == 1) return launch_awq_mma<1>(mp, sh, a16, c8, g8, bias, y, m, n, group_size, w8, dev, st, k);
      return launch_awq_mma<2>(mp, sh, a16, c8, g8, bias, y, m, n, group_size, w8, dev, st, k);
    }
  }
  if (gemv_eligible(m, k, n, group_size)) {
    const GemvPlan gp = gemv_plan(m, k, sh, group_size, sm_count(dev), max_ws);
    if (gp.mt == 1) return launch_awq_gemv<1>(gp, sh, gate_up, c8, g8, bias, y, m, k, n, group_size, w8, dev, st, gate_up_stride, 1);
    if (gp.mt == 2) return launch_awq_gemv<2>(gp, sh, gate_up, c8, g8, bias, y, m, k, n, group_size, w8, dev, st, gate_up_stride, 1);
    if (gp.mt == 4) return launch_awq_gemv<4>(gp, sh, gate_up, c8, g8, bias, y, m, k, n, group_size, w8, dev, st, gate_up_stride, 1);
  }
  if (i8_eligible(m, k, n, group_size) && aligned16(y)) {
    const I8Plan ip = i8_plan(m, k, sh, group_size, sm_count(dev), max_ws);
    if (ip.bn == 16) return launch_awq_i8<16>(ip, sh, gate_up, c8, g8, bias, y, m, k, n, group_size, w8, dev, st, gate_up_stride, 1);
  }
  return fail(LVB_ERR_UNSUPPORTED, "fused SiLU-mul linear covers decode batches (m <= 16, groups of 128 / 256) only");
}

static int kv_write_common(const lvb::attn::KVWriteArgs &a, int dtype, lvb_stream_t stream) {
  if (dtype != LVB_DTYPE_F16 && dtype != LVB_DTYPE_BF16) return fail(LVB_ERR_INVALID, "unknown dtype %d", dtype);
  if (a.num_tokens < 0 || a.Hkv <= 0 || a.D <= 0 || a.D % 8 != 0)
    return fail(LVB_ERR_INVALID, "invalid K/V shape tokens=%d heads=%d head_size=%d", a.num_tokens, a.Hkv, a.D);
  if (a.num_tokens == 0) return LVB_OK;
  if (a.key_stride % 8 != 0 || a.value_stride % 8 != 0)
    return fail(LVB_ERR_INVALID, "K/V token strides must be multiples of 8 elements");
  if (!aligned16(a.key) || !aligned16(a.value) || !aligned16(a.key_cache) || !aligned16(a.value_cache))
    return fail(LVB_ERR_INVALID, "K/V tensors and caches must be 16-byte aligned");
  const int chunks = a.Hkv * (a.D / 8);
  const int threads = chunks < 256 ? ((chunks + 31) / 32) * 32 : 256;
  cudaError_t e = launch_pdl(lvb::attn::paged_kv_write_kernel, dim3(a.num_tokens), dim3(threads), 0,
                             reinterpret_cast<cudaStream_t>(stream), a);
  if (e != cudaSuccess) return cuda_fail(e, "paged_kv_write_kernel launch");
  return LVB_OK;
}

int lvb_paged_kv_write(const uint16_t *key, int64_t key_token_stride, const uint16_t *value,
                       int64_t value_token_stride, uint16_t *key_cache, uint16_t *value_cache,
                       const int32_t *block_tables, int64_t table_stride,
                       const int32_t *num_computed, const int32_t *query_start_loc,
                       const int32_t *request_indices, int64_t num_tokens, int64_t num_kv_heads,
                       int64_t head_size, int64_t block_size, int dtype, lvb_stream_t stream) {
  if (num_tokens > INT_MAX || block_size <= 0 || block_size > INT_MAX)
    return fail(LVB_ERR_INVALID, "invalid token count or block size");
  if (num_tokens > 0 && (!key || !value || !key_cache || !value_cache || !block_tables || !num_computed ||
                         !query_start_loc || !request_indices))
    return fail(LVB_ERR_INVALID, "paged K/V write null pointer argument");
  lvb::attn::KVWriteArgs a{};
  a.key = key;
  a.key_stride = key_token_stride;
  a.value = value;
  a.value_stride = value_token_stride;
  a.key_cache = key_cache;
  a.value_cache = value_cache;
  a.tables = block_tables;
  a.table_stride = table_stride;
  a.computed = num_computed;
  a.qsl = query_start_loc;
  a.req = request_indices;
  a.slots = nullptr;
  a.num_tokens = static_cast<int>(num_tokens);
  a.Hkv = static_cast<int>(num_kv_heads);
  a.D = static_cast<int>(head_size);
  a.bs = static_cast<int>(block_size);
  return kv_write_common(a, dtype, stream);
}

int lvb_kv_scatter(const uint16_t *key, int64_t key_token_stride, const uint16_t *value,
                   int64_t value_token_stride, uint16_t *key_cache, uint16_t *value_cache,
                   const int64_t *slots, int64_t num_tokens, int64_t num_kv_heads,
                   int64_t head_size, int64_t num_slots, int dtype, lvb_stream_t stream) {
  (void)num_slots;
  if (num_tokens > INT_MAX) return fail(LVB_ERR_INVALID, "token count exceeds int32");
  if (num_tokens > 0 && (!key || !value || !key_cache || !value_cache || !slots))
    return fail(LVB_ERR_INVALID, "K/V scatter null pointer argument");
  lvb::attn::KVWriteArgs a{};
  a.key = key;
  a.key_stride = key_token_stride;
  a.value = value;
  a.value_stride = value_token_stride;
  a.key_cache = key_cache;
  a.value_cache = value_cache;
  a.slots = slots;
  a.num_tokens = static_cast<int>(num_tokens);
  a.Hkv = static_cast<int>(num_kv_heads);
  a.D = static_cast<int>(head_size);
  a.bs = 1;
  return kv_write_common(a, dtype, stream);
}

// Rules of PagedKVCache.compact (runtime/execution/paged_cache.py:257-326),
// in the order that decides which message a caller sees; counts[] =
// {computed, query, reserved, readonly prefix blocks}.  Non-integers reach
// here as -1 (the Python shim maps them), so they fail the rule of the field
// they are in.
int lvb_kv_compact_plan(const int64_t *block_ids, int64_t num_table_blocks, const int64_t *counts,
                        const int64_t *retained, int64_t num_retained, int64_t num_blocks, int64_t block_size,
                        int32_t *src_slots, int32_t *dst_slots, int64_t *moved) {
  if (!counts || !moved || (num_table_blocks > 0 && !block_ids) || (num_retained > 0 && (!retained || !src_slots || !dst_slots)))
    return fail(LVB_ERR_INVALID, "KV compaction null pointer argument");
  if (block_size <= 0 || num_blocks <= 0 || num_table_blocks < 0 || num_retained < 0)
    return fail(LVB_ERR_INVALID, "invalid KV compaction geometry");
  *moved = 0;
  const int64_t computed = counts[0], queries = counts[1], reserved = counts[2], readonly = counts[3];
  if (computed < 0 || queries < 0 || reserved < 0 || readonly < 0)
    return fail(LVB_ERR_INVALID, "paged compact counts must be non-negative integers");
  if (reserved < queries) return fail(LVB_ERR_INVALID, "reserved query tokens must cover every actual query");
  std::vector<int64_t> sorted(retained, retained + num_retained);
  for (int64_t v : sorted)
    if (v < 0) return fail(LVB_ERR_INVALID, "retained query indices must be non-negative integers");
  std::sort(sorted.begin(), sorted.end());
  if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end())
    return fail(LVB_ERR_INVALID, "retained query indices must be unique");
  if (!sorted.empty() && sorted.back() >= queries)
    return fail(LVB_ERR_METADATA, "retained query index exceeds the paged KV tail");
  if (num_table_blocks != (computed + reserved + block_size - 1) / block_size)
    return fail(LVB_ERR_METADATA, "block table does not exactly cover the reserved query slots");
  std::vector<int64_t> ids(block_ids, block_ids + num_table_blocks);
  for (int64_t b : ids)
    if (b < 0 || b >= num_blocks) return fail(LVB_ERR_METADATA, "block table contains an invalid physical block");
  std::sort(ids.begin(), ids.end());
  if (std::adjacent_find(ids.begin(), ids.end()) != ids.end())
    return fail(LVB_ERR_METADATA, "block table aliases a physical block within one request");
  if (readonly * block_size > computed)
    return fail(LVB_ERR_METADATA, "readonly prefix blocks exceed the computed prefix");
  if (num_blocks * block_size > INT_MAX) return fail(LVB_ERR_UNSUPPORTED, "KV slot index exceeds int32");
  auto slot = [&](int64_t pos) { return block_ids[pos / block_size] * block_size + pos % block_size; };
  int64_t changed = 0;
  for (int64_t i = 0; i < num_retained; ++i) {
    src_slots[i] = static_cast<int32_t>(slot(computed + retained[i]));
    dst_slots[i] = static_cast<int32_t>(slot(computed + i));
    changed += src_slots[i] != dst_slots[i];
  }
  *moved = changed;
  return LVB_OK;
}

int lvb_kv_move_rows(uint16_t *key_cache, uint16_t *value_cache, const int32_t *src_slots,
                     const int32_t *dst_slots, int64_t num_rows, int64_t num_kv_heads, int64_t head_size,
                     int64_t num_slots, int dtype, lvb_stream_t stream) {
  (void)num_slots;
  if (dtype != LVB_DTYPE_F16 && dtype != LVB_DTYPE_BF16) return fail(LVB_ERR_INVALID, "unknown dtype %d", dtype);
  if (num_rows < 0 || num_kv_heads <= 0 || head_size <= 0 || head_size % 8 != 0)
    return fail(LVB_ERR_INVALID, "invalid KV move shape (head_size must be a multiple of 8)");
  if (num_rows == 0) return LVB_OK;
  if (!key_cache || !value_cache || !src_slots || !dst_slots) return fail(LVB_ERR_INVALID, "KV move null pointer argument");
  if (!aligned16(key_cache) || !aligned16(value_cache)) return fail(LVB_ERR_INVALID, "KV caches must be 16-byte aligned");
  const size_t smem = static_cast<size_t>(num_rows) * head_size * 2;
  if (smem > kKvMoveMaxSmem)
    return fail(LVB_ERR_UNSUPPORTED, "KV move of %lld rows x %lld values exceeds %zu bytes of shared memory",
                (long long)num_rows, (long long)head_size, kKvMoveMaxSmem);
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  static bool smem_done[kMaxDevices] = {false};
  rc = ensure_smem(lvb::attn::kv_move_rows_kernel, static_cast<int>(kKvMoveMaxSmem), dev, smem_done);
  if (rc != LVB_OK) return rc;
  cudaError_t e = launch_pdl(lvb::attn::kv_move_rows_kernel, dim3(static_cast<unsigned>(num_kv_heads), 2), dim3(128), smem,
                             reinterpret_cast<cudaStream_t>(stream), key_cache, value_cache, src_slots, dst_slots,
                             static_cast<int>(num_rows), static_cast<int>(num_kv_heads), static_cast<int>(head_size));
  if (e != cudaSuccess) return cuda_fail(e, "kv_move_rows_kernel launch");
  return LVB_OK;
}

size_t lvb_paged_attention_workspace_bytes(int64_t num_seqs, int64_t num_q_heads,
                                           int64_t num_kv_heads, int64_t head_size,
                                           int64_t max_seq_len) {
  if (num_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_size <= 0 || max_seq_len <= 0) return 0;
  int dev = 0;
  if (current_device(&dev) != LVB_OK) return 0;
  const DecodePlan p = decode_plan(num_seqs, num_q_heads, num_kv_heads, head_size, max_seq_len, sm_count(dev));
  return p.total();
}

struct StepKV {  // the step's K/V rows for lvb_paged_attention_kv
  const uint16_t *key, *value;
  int64_t key_stride, value_stride;
};

int paged_attention_impl(const StepKV *kv, const uint16_t *query, int64_t query_token_stride,
                         const uint16_t *key_cache, const uint16_t *value_cache, uint16_t *out,
                         int64_t out_token_stride, const int32_t *block_tables, int64_t table_stride,
                         const int32_t *num_computed, const int32_t *query_start_loc,
                         const int32_t *request_indices, const int32_t *request_order, const uint8_t *visibility,
                         const int32_t *visibility_start, int64_t num_seqs, int64_t num_decode_seqs,
                         int64_t num_tokens, int64_t max_query_len, int64_t max_seq_len, int64_t num_q_heads,
                         int64_t num_kv_heads, int64_t head_size, int64_t block_size, int64_t num_blocks,
                         float scale, int dtype, void *workspace, size_t workspace_bytes, lvb_stream_t stream);

int lvb_paged_attention(const uint16_t *query, int64_t query_token_stride,
                        const uint16_t *key_cache, const uint16_t *value_cache, uint16_t *out,
                        int64_t out_token_stride, const int32_t *block_tables,
                        int64_t table_stride, const int32_t *num_computed,
                        const int32_t *query_start_loc, const int32_t *request_indices,
                        const int32_t *request_order,
                        const uint8_t *visibility, const int32_t *visibility_start,
                        int64_t num_seqs, int64_t num_decode_seqs, int64_t num_tokens, int64_t max_query_len,
                        int64_t max_seq_len, int64_t num_q_heads, int64_t num_kv_heads,
                        int64_t head_size, int64_t block_size, int64_t num_blocks, float scale,
                        int dtype, void *workspace, size_t workspace_bytes,
                        lvb_stream_t stream) {
  return paged_attention_impl(nullptr, query, query_token_stride, key_cache, value_cache, out, out_token_stride,
                              block_tables, table_stride, num_computed, query_start_loc, request_indices,
                              request_order, visibility, visibility_start, num_seqs, num_decode_seqs, num_tokens,
                              max_query_len, max_seq_len, num_q_heads, num_kv_heads, head_size, block_size,
                              num_blocks, scale, dtype, workspace, workspace_bytes, stream);
}

int lvb_paged_attention_kv(const uint16_t *key, int64_t key_token_stride, const uint16_t *value,
                           int64_t value_token_stride, const uint16_t *query, int64_t query_token_stride,
                           uint16_t *key_cache, uint16_t *value_cache, uint16_t *out, int64_t out_token_stride,
                           const int32_t *block_tables, int64_t table_stride, const int32_t *num_computed,
                           const int32_t *query_start_loc, const int32_t *request_indices,
                           const int32_t *request_order, const uint8_t *visibility, const int32_t *visibility_start,
                           int64_t num_seqs, int64_t num_decode_seqs, int64_t num_tokens, int64_t max_query_len,
                           int64_t max_seq_len, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                           int64_t block_size, int64_t num_blocks, float scale, int dtype, void *workspace,
                           size_t workspace_bytes, lvb_stream_t stream) {
  const StepKV kv{key, value, key_token_stride, value_token_stride};
  return paged_attention_impl(&kv, query, query_token_stride, key_cache, value_cache, out, out_token_stride,
                              block_tables, table_stride, num_computed, query_start_loc, request_indices,
                              request_order, visibility, visibility_start, num_seqs, num_decode_seqs, num_tokens,
                              max_query_len, max_seq_len, num_q_heads, num_kv_heads, head_size, block_size,
                              num_blocks, scale, dtype, workspace, workspace_bytes, stream);
}

int paged_attention_impl(const StepKV *kv, const uint16_t *query, int64_t query_token_stride,
                         const uint16_t *key_cache, const uint16_t *value_cache, uint16_t *out,
                         int64_t out_token_stride, const int32_t *block_tables, int64_t table_stride,
                         const int32_t *num_computed, const int32_t *query_start_loc,
                         const int32_t *request_indices, const int32_t *request_order, const uint8_t *visibility,
                         const int32_t *visibility_start, int64_t num_seqs, int64_t num_decode_seqs,
                         int64_t num_tokens, int64_t max_query_len, int64_t max_seq_len, int64_t num_q_heads,
                         int64_t num_kv_heads, int64_t head_size, int64_t block_size, int64_t num_blocks,
                         float scale, int dtype, void *workspace, size_t workspace_bytes, lvb_stream_t stream) {
  if (dtype != LVB_DTYPE_F16 && dtype != LVB_DTYPE_BF16) return fail(LVB_ERR_INVALID, "unknown dtype %d", dtype);
  if (num_tokens < 0 || num_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      num_q_heads % num_kv_heads != 0 || block_size <= 0 || num_blocks <= 0)
    return fail(LVB_ERR_INVALID, "invalid paged attention shape");
  if (head_size <= 0 || head_size % 8 != 0 || head_size > 256)
    return fail(LVB_ERR_UNSUPPORTED, "head_size %lld must be a multiple of 8 up to 256", (long long)head_size);
  if (num_tokens == 0) return LVB_OK;
  if (num_tokens > INT_MAX || num_seqs > INT_MAX || max_seq_len > INT_MAX || num_q_heads > 65535)
    return fail(LVB_ERR_UNSUPPORTED, "paged attention size exceeds the launch limits");
  if (!query || !key_cache || !value_cache || !out || !block_tables || !num_computed || !query_start_loc ||
      !request_indices || (visibility != nullptr && visibility_start == nullptr))
    return fail(LVB_ERR_INVALID, "paged attention null pointer argument");
  if (!aligned16(key_cache) || !aligned16(value_cache)) return fail(LVB_ERR_INVALID, "caches must be 16-byte aligned");
  if (query_token_stride % 2 != 0 || (reinterpret_cast<uintptr_t>(query) & 3u) != 0)
    return fail(LVB_ERR_INVALID, "query rows must be 4-byte aligned");
  if (out_token_stride % 2 != 0 || (reinterpret_cast<uintptr_t>(out) & 3u) != 0)
    return fail(LVB_ERR_INVALID, "output rows must be 4-byte aligned");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;

  lvb::attn::AttnArgs a{};
  a.q = query;
  a.q_stride = query_token_stride;
  a.kc = key_cache;
  a.vc = value_cache;
  a.out = out;
  a.o_stride = out_token_stride;
  a.tables = block_tables;
  a.table_stride = table_stride;
  a.computed = num_computed;
  a.qsl = query_start_loc;
  a.req = request_indices;
  a.order = request_order;
  a.num_seqs = static_cast<int>(num_seqs);
  a.vis = visibility;
  a.vis_start = visibility_start;
  a.Hq = static_cast<int>(num_q_heads);
  a.Hkv = static_cast<int>(num_kv_heads);
  a.D = static_cast<int>(head_size);
  a.bs = static_cast<int>(block_size);
  a.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == LVB_DTYPE_BF16;

  const bool all_decode = decode_eligible(visibility, max_query_len, num_seqs, num_tokens, num_q_heads,
                                         num_kv_heads, head_size, block_size);
  const bool tiles = tile_eligible(num_q_heads, num_kv_heads, head_size, block_size);
  if (kv != nullptr && (!kv->key || !kv->value)) return fail(LVB_ERR_INVALID, "paged K/V write null pointer argument");
  if (kv != nullptr) {
    // Decode batches on the split kernel store the step's rows themselves;
    // anything else writes them first with lvb_paged_kv_write.
    const bool rows16 = aligned16(kv->key) && aligned16(kv->value) && kv->key_stride % 8 == 0 &&
                        kv->value_stride % 8 == 0;
    if (all_decode && rows16 && !kBalancedDecode) {
      a.new_k = kv->key;
      a.new_v = kv->value;
      a.new_k_stride = kv->key_stride;
      a.new_v_stride = kv->value_stride;
    } else {
      rc = lvb_paged_kv_write(kv->key, kv->key_stride, kv->value, kv->value_stride, const_cast<uint16_t *>(key_cache),
                              const_cast<uint16_t *>(value_cache), block_tables, table_stride, num_computed,
                              query_start_loc, request_indices, num_tokens, num_kv_heads, head_size, block_size,
                              dtype, stream);
      if (rc != LVB_OK) return rc;
    }
  }
  // One-token requests of a mixed batch: listed first in request_order.
  int64_t n_decode = all_decode ? num_seqs : 0;
  if (!all_decode && tiles && request_order != nullptr && decode_shape_ok(num_q_heads, num_kv_heads, head_size, block_size)) {
    if (num_decode_seqs < 0 || num_decode_seqs > num_seqs)
      return fail(LVB_ERR_INVALID, "num_decode_seqs %lld outside [0, %lld]", (long long)num_decode_seqs,
                  (long long)num_seqs);
    n_decode = num_decode_seqs;
  }
  if (n_decode > 0) {
    const DecodePlan plan = decode_plan(num_seqs, num_q_heads, num_kv_heads, head_size, max_seq_len, sm_count(dev));
    if (workspace == nullptr || workspace_bytes < plan.total() || !aligned16(workspace))
      return fail(LVB_ERR_WORKSPACE, "paged attention workspace of %zu bytes is below the %zu required",
                  workspace_bytes, plan.total());
    a.part_o = static_cast<float *>(workspace);
    a.part_lse = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + plan.o_bytes);
    a.merge_count = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(workspace) + plan.o_bytes + plan.lse_bytes);
    a.max_splits = plan.max_splits;
    a.chunk_tokens = plan.chunk_tokens;
    if (bf16) {
      rc = head_size == 128 ? launch_decode_any<true, 128>(a, plan, n_decode, num_blocks, dev, s)
                            : launch_decode_any<true, 64>(a, plan, n_decode, num_blocks, dev, s);
    } else {
      rc = head_size == 128 ? launch_decode_any<false, 128>(a, plan, n_decode, num_blocks, dev, s)
                            : launch_decode_any<false, 64>(a, plan, n_decode, num_blocks, dev, s);
    }
    if (rc != LVB_OK || all_decode) return rc;
  }
  if (tiles) {
    const int64_t tile_reqs = request_order != nullptr ? num_seqs - n_decode : num_seqs;
    if (tile_reqs == 0) return LVB_OK;
    a.first_tile_req = static_cast<int>(request_order != nullptr ? n_decode : 0);
    const int64_t row_tiles = (max_query_len * (num_q_heads / num_kv_heads) + 63) / 64;
    if (row_tiles > INT_MAX || tile_reqs > 65535) return fail(LVB_ERR_UNSUPPORTED, "prefill tile grid exceeds launch limits");
    const dim3 grid(static_cast<unsigned>(row_tiles), static_cast<unsigned>(tile_reqs), static_cast<unsigned>(num_kv_heads));
    if (bf16) return head_size == 128 ? launch_prefill<true, 128>(a, grid, dev, s) : launch_prefill<true, 64>(a, grid, dev, s);
    return head_size == 128 ? launch_prefill<false, 128>(a, grid, dev, s) : launch_prefill<false, 64>(a, grid, dev, s);
  }
  return bf16 ? launch_general<true>(a, num_tokens, s) : launch_general<false>(a, num_tokens, s);
}

int lvb_awq_linear_static(const uint16_t *x, const int32_t *qweight, const int32_t *qzeros,
                          const uint16_t *scales, const uint16_t *bias, uint16_t *y, int64_t m,
                          int64_t k, int64_t n, int64_t group_size, lvb_stream_t stream) {
  if (m < 0 || k <= 0 || n <= 0) return fail(LVB_ERR_INVALID, "invalid AWQ shape m=%lld k=%lld n=%lld",
                                              (long long)m, (long long)k, (long long)n);
  if (m == 0) return LVB_OK;
  if (m > INT_MAX || k > INT_MAX || n > INT_MAX) return fail(LVB_ERR_UNSUPPORTED, "AWQ dimension exceeds int32");
  if (group_size <= 0 || group_size % 32 != 0 || k % group_size != 0)
    return fail(LVB_ERR_INVALID, "AWQ group_size %lld must be a positive multiple of 32 dividing k=%lld",
                (long long)group_size, (long long)k);
  if (n % 32 != 0) return fail(LVB_ERR_INVALID, "AWQ output width %lld must be divisible by 32", (long long)n);
  if (k % 8 != 0) return fail(LVB_ERR_INVALID, "AWQ input width %lld must be divisible by 8", (long long)k);
  if (!x || !qweight || !qzeros || !scales || !y) return fail(LVB_ERR_INVALID, "AWQ null pointer argument");
  if (!aligned16(x) || !aligned16(qweight) || !aligned16(qzeros) || !aligned16(scales))
    return fail(LVB_ERR_INVALID, "AWQ x, qweight, qzeros and scales must be 16-byte aligned");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const AwqPlan plan = awq_plan(m, k, n, sm_count(dev));
  const size_t need = plan.sem_bytes + plan.part_bytes;
  if (need > kAwqStaticScratchBytes)
    return fail(LVB_ERR_UNSUPPORTED,
                "lvb_awq_linear_static: m=%lld k=%lld n=%lld needs %zu bytes of split-K scratch, above its "
                "fixed %zu-byte buffer; call lvb_awq_linear with a workspace instead",
                (long long)m, (long long)k, (long long)n, need, kAwqStaticScratchBytes);
  void *scratch = nullptr;
  rc = awq_static_scratch(dev, &scratch);
  if (rc != LVB_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (plan.sem_bytes > 0) {
    // The semaphores must start at zero; a completed call leaves them zero, and
    // clearing them here also covers a previous call that was aborted.
    cudaError_t e = cudaMemsetAsync(scratch, 0, plan.sem_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "clearing the static split-K semaphores");
  }
  uint8_t *ws = static_cast<uint8_t *>(scratch);
  return dispatch_awq(plan, x, qweight, qzeros, scales, bias, y, m, k, n, group_size, ws, dev, s);
}

int lvb_pack_step_metadata(const int32_t *block_ids, const int64_t *table_offsets,
                           const int32_t *num_computed, const int32_t *query_lengths,
                           const int32_t *reserved, const int32_t *readonly, int64_t num_seqs,
                           int64_t num_blocks, int64_t block_size, int32_t *out,
                           int64_t out_capacity, int64_t *table_stride_out,
                           int64_t *num_tokens_out) {
  if (num_seqs <= 0 || num_blocks <= 0 || block_size <= 0 || num_blocks > INT_MAX)
    return fail(LVB_ERR_INVALID, "invalid step metadata sizes");
  if (!block_ids || !table_offsets || !num_computed || !query_lengths || !reserved || !readonly || !out ||
      !table_stride_out || !num_tokens_out)
    return fail(LVB_ERR_INVALID, "step metadata null pointer argument");
  int64_t max_blocks = 0, num_tokens = 0;
  for (int64_t r = 0; r < num_seqs; ++r) {
    const int64_t len = table_offsets[r + 1] - table_offsets[r];
    if (len < 0 || query_lengths[r] < 0 || reserved[r] < query_lengths[r] || num_computed[r] < 0 || readonly[r] < 0)
      return fail(LVB_ERR_INVALID, "step metadata row %lld is malformed", (long long)r);
    if (len > max_blocks) max_blocks = len;
    num_tokens += query_lengths[r];
  }
  static thread_local lvb::meta::OwnerTable owners;
  const char *violation = lvb::meta::validate(block_ids, table_offsets, num_computed, reserved, readonly,
                                              num_seqs, num_blocks, block_size, owners);
  if (violation != nullptr) return fail(LVB_ERR_METADATA, "%s", violation);
  const int64_t need = num_seqs * max_blocks + 4 * num_seqs + 1 + num_tokens;
  if (need > out_capacity || num_tokens > INT_MAX)
    return fail(LVB_ERR_WORKSPACE, "step metadata needs %lld int32 slots, buffer has %lld", (long long)need,
                (long long)out_capacity);
  int32_t *tables = out;
  for (int64_t r = 0; r < num_seqs; ++r) {
    const int64_t begin = table_offsets[r];
    const int64_t len = table_offsets[r + 1] - begin;
    int32_t *row = tables + r * max_blocks;
    for (int64_t i = 0; i < len; ++i) row[i] = block_ids[begin + i];
    const int32_t pad = len > 0 ? block_ids[begin] : 0;
    for (int64_t i = len; i < max_blocks; ++i) row[i] = pad;
  }
  int32_t *computed = tables + num_seqs * max_blocks;
  int32_t *qsl = computed + num_seqs;
  int32_t *req = qsl + num_seqs + 1;
  int32_t *order = req + num_tokens;
  int64_t t = 0;
  qsl[0] = 0;
  for (int64_t r = 0; r < num_seqs; ++r) {
    computed[r] = num_computed[r];
    qsl[r + 1] = static_cast<int32_t>(qsl[r] + query_lengths[r]);
    for (int32_t i = 0; i < query_lengths[r]; ++i) req[t++] = static_cast<int32_t>(r);
    order[r] = static_cast<int32_t>(r);
  }
  // Launch order: the one-token (decode) requests first, longest context
  // first, for the split decode kernel; then the others, longest context
  // first, for the prefill tile kernel; ties by index.  Then the listed
  // requests' computed counts.
  std::stable_sort(order, order + num_seqs, [num_computed, query_lengths](int32_t x, int32_t y) {
    const bool dx = query_lengths[x] == 1, dy = query_lengths[y] == 1;
    if (dx != dy) return dx;
    return num_computed[x] + query_lengths[x] > num_computed[y] + query_lengths[y];
  });
  for (int64_t r = 0; r < num_seqs; ++r) order[num_seqs + r] = num_computed[order[r]];
  *table_stride_out = max_blocks;
  *num_tokens_out = num_tokens;
  return LVB_OK;
}

int lvb_event_create(void **event) {
  if (!event) return fail(LVB_ERR_INVALID, "lvb_event_create: null argument");
  cudaEvent_t e = nullptr;
  cudaError_t err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  if (err != cudaSuccess) return cuda_fail(err, "cudaEventCreateWithFlags");
  *event = e;
  return LVB_OK;
}

int lvb_event_destroy(void *event) {
  if (!event) return LVB_OK;
  cudaError_t err = cudaEventDestroy(static_cast<cudaEvent_t>(event));
  return err == cudaSuccess ? LVB_OK : cuda_fail(err, "cudaEventDestroy");
}

int lvb_event_record(void *event, lvb_stream_t stream) {
  if (!event) return fail(LVB_ERR_INVALID, "lvb_event_record: null event");
  cudaError_t err = cudaEventRecord(static_cast<cudaEvent_t>(event), reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LVB_OK : cuda_fail(err, "cudaEventRecord");
}

int lvb_event_wait_host(void *event) {
  if (!event) return LVB_OK;
  cudaEvent_t e = static_cast<cudaEvent_t>(event);
  cudaError_t err = cudaEventQuery(e);
  if (err == cudaErrorNotReady) err = cudaEventSynchronize(e);
  return err == cudaSuccess ? LVB_OK : cuda_fail(err, "waiting for a staging copy");
}

int lvb_stream_wait_event(lvb_stream_t stream, void *event) {
  if (!event) return fail(LVB_ERR_INVALID, "lvb_stream_wait_event: null event");
  cudaError_t err = cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0);
  return err == cudaSuccess ? LVB_OK : cuda_fail(err, "cudaStreamWaitEvent");
}

int lvb_copy_async(void *dst, const void *src, size_t bytes, lvb_stream_t stream) {
  if (bytes == 0) return LVB_OK;
  if (!dst || !src) return fail(LVB_ERR_INVALID, "lvb_copy_async: null pointer");
  cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LVB_OK : cuda_fail(err, "cudaMemcpyAsync");
}

int lvb_stage_step_metadata(const int32_t *block_ids, const int64_t *table_offsets,
                            const int32_t *num_computed, const int32_t *query_lengths,
                            const int32_t *reserved, const int32_t *readonly, int64_t num_seqs,
                            int64_t num_blocks, int64_t block_size, int32_t *pinned_out,
                            int64_t out_capacity, int32_t *device_out, int64_t device_capacity,
                            void *slot_event, lvb_stream_t stream, int64_t *table_stride_out,
                            int64_t *num_tokens_out) {
  if (!device_out || !table_stride_out || !num_tokens_out)
    return fail(LVB_ERR_INVALID, "step metadata staging null pointer argument");
  // The pinned slot may still feed the copy issued the last time it was used.
  int rc = lvb_event_wait_host(slot_event);
  if (rc != LVB_OK) return rc;
  rc = lvb_pack_step_metadata(block_ids, table_offsets, num_computed, query_lengths, reserved, readonly,
                              num_seqs, num_blocks, block_size, pinned_out, out_capacity, table_stride_out,
                              num_tokens_out);
  if (rc != LVB_OK) return rc;
  const int64_t total = num_seqs * *table_stride_out + 4 * num_seqs + 1 + *num_tokens_out;
  if (total > device_capacity)
    return fail(LVB_ERR_WORKSPACE, "step metadata needs %lld int32 slots on the device, buffer has %lld",
                (long long)total, (long long)device_capacity);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemcpyAsync(device_out, pinned_out, static_cast<size_t>(total) * sizeof(int32_t),
                                    cudaMemcpyHostToDevice, s);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync (step metadata)");
  return slot_event ? lvb_event_record(slot_event, stream) : LVB_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------
// Tensor-parallel all-reduce + residual add + RMSNorm over peer memory
// ------------------------------------------------------------------------
int lvb_ipc_alloc(size_t bytes, void **ptr, void *handle_out) {
  if (bytes == 0 || !ptr || !handle_out) return fail(LVB_ERR_INVALID, "lvb_ipc_alloc: invalid argument");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (peer workspace)");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) {
      std::memcpy(handle_out, &h, sizeof(h));
      *ptr = p;
      return LVB_OK;
    }
  }
  cudaFree(p);
  return cuda_fail(e, "preparing a peer workspace");
}

int lvb_ipc_open(const void *handle, void **ptr) {
  if (!handle || !ptr) return fail(LVB_ERR_INVALID, "lvb_ipc_open: invalid argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return LVB_OK;
}

int lvb_ipc_close(void *ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int lvb_ipc_free(void *ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "cudaFree (peer workspace)");
}

size_t lvb_allreduce_workspace_bytes(int world, int64_t max_tokens, int64_t hidden) {
  if (world < 1 || world > lvb::ar::kMaxWorld || max_tokens <= 0 || hidden <= 0) return 0;
  const size_t slot = static_cast<size_t>(max_tokens) * hidden * 2;
  return lvb::ar::kHeaderBytes + lvb::ar::slots_per_workspace(world) * slot;
}

int lvb_allreduce_workspace_init(void *workspace, int world, int64_t max_tokens, int64_t hidden) {
  const size_t total = lvb_allreduce_workspace_bytes(world, max_tokens, hidden);
  if (!workspace || total == 0) return fail(LVB_ERR_INVALID, "lvb_allreduce_workspace_init: invalid argument");
  const size_t slot = static_cast<size_t>(max_tokens) * hidden * 2;
  uint8_t *base = static_cast<uint8_t *>(workspace);
  const size_t sentinel_begin = lvb::ar::kHeaderBytes + lvb::ar::slots_before_sentinel(world) * slot;
  if (max_tokens > INT_MAX || hidden > lvb::ar::kMaxHidden)
    return fail(LVB_ERR_INVALID, "lvb_allreduce_workspace_init: shape too large");
  cudaError_t e = cudaMemset(base, 0, sentinel_begin);
  if (e == cudaSuccess) e = cudaMemset(base + sentinel_begin, 0xFF, total - sentinel_begin);
  const uint32_t geometry[4] = {lvb::ar::kMagic, static_cast<uint32_t>(world), static_cast<uint32_t>(max_tokens),
                                static_cast<uint32_t>(hidden)};
  if (e == cudaSuccess) e = cudaMemcpy(base + lvb::ar::kGeometryOff, geometry, sizeof(geometry), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "initialising an all-reduce workspace");
}

namespace {

// CTAs of the all-reduce kernel that fit on the GPU at once (its two-shot
// phase waits on other CTAs of the same grid).
int allreduce_capacity(int dev) {
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lvb::ar::allreduce_add_rmsnorm_kernel,
                                                    lvb::ar::kThreads, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int cap = sm_count(dev) * per_sm;
  if (cap > lvb::ar::kMaxBlocks) cap = lvb::ar::kMaxBlocks;
  if (dev >= 0 && dev < 64) cached[dev] = cap;
  return cap;
}

// Message bytes up to which the peer-memory kernel beats NCCL's ring
// all-reduce (measured on B200, add + RMSNorm included on our side): world 2
// one-shot up to ~16 MiB (1024 x 8192 fp16 rows); world 4 sentinel two-shot up
// to ~32 MiB (2048 rows, where both reach ~415 GB/s bus bandwidth).
constexpr size_t kPeerMaxBytesWorld2 = size_t(16) << 20;
constexpr size_t kPeerMaxBytes = size_t(32) << 20;
// (world - 1) x message bytes up to which the one-shot push beats the two-shot
// exchange (which moves 2 (world - 1) / world of the message per rank instead
// of world - 1 messages, for one more NVLink round trip); world 4 crossover
// near 64 x 8192 rows.
constexpr size_t kSentinelOneShotMaxPushBytes = size_t(4) << 20;

}  // namespace

size_t lvb_allreduce_peer_max_bytes(int world) {
  if (world <= 1) return SIZE_MAX;
  return world == 2 ? kPeerMaxBytesWorld2 : kPeerMaxBytes;
}

int lvb_allreduce_add_rmsnorm(void *const *workspaces, int rank, int world, const uint16_t *partial,
                              uint16_t *residual, const uint16_t *weight, uint16_t *out, int64_t tokens,
                              int64_t hidden, int64_t max_tokens, float eps, int mode, lvb_stream_t stream) {
  if (world < 1 || world > lvb::ar::kMaxWorld || rank < 0 || rank >= world)
    return fail(LVB_ERR_INVALID, "all-reduce rank %d of world %d (at most %d ranks)", rank, world, lvb::ar::kMaxWorld);
  if (tokens < 0 || tokens > max_tokens || hidden <= 0 || hidden % 8 != 0 || hidden > lvb::ar::kMaxHidden)
    return fail(LVB_ERR_INVALID, "all-reduce shape %lld x %lld (workspace rows %lld; hidden a multiple of 8 up to %d)",
                (long long)tokens, (long long)hidden, (long long)max_tokens, lvb::ar::kMaxHidden);
  if (mode < lvb::ar::kAuto || mode > lvb::ar::kSentinelTwoShot) return fail(LVB_ERR_INVALID, "all-reduce mode %d", mode);
  if (tokens == 0) return LVB_OK;
  if (tokens > INT_MAX / 8) return fail(LVB_ERR_UNSUPPORTED, "token count too large");
  if (!workspaces || !partial || !out) return fail(LVB_ERR_INVALID, "all-reduce null pointer argument");
  if ((residual == nullptr) != (weight == nullptr))
    return fail(LVB_ERR_INVALID, "residual and weight are given together (norm) or both null (plain sum)");
  if (!aligned16(partial) || !aligned16(out) || (residual && (!aligned16(residual) || !aligned16(weight))))
    return fail(LVB_ERR_INVALID, "all-reduce tensors must be 16-byte aligned");
  if (residual && (static_cast<const void *>(residual) == static_cast<const void *>(partial) ||
                   static_cast<const void *>(residual) == static_cast<const void *>(out)))
    return fail(LVB_ERR_INVALID, "residual must not alias partial or out");
  lvb::ar::Args a{};
  if (world == 1) {
    // No exchange: the sum of one partial is the partial itself.
    if (residual == nullptr) {
      if (out == partial) return LVB_OK;
      cudaError_t e = cudaMemcpyAsync(out, partial, static_cast<size_t>(tokens) * hidden * 2, cudaMemcpyDeviceToDevice,
                                      reinterpret_cast<cudaStream_t>(stream));
      return e == cudaSuccess ? LVB_OK : cuda_fail(e, "all-reduce copy (one rank)");
    }
    int dev1 = 0;
    int rc1 = current_device(&dev1);
    if (rc1 != LVB_OK) return rc1;
    a.rank = 0;
    a.world = 1;
    a.partial = partial;
    a.residual = residual;
    a.weight = weight;
    a.out = out;
    a.tokens = static_cast<int>(tokens);
    a.hidden = static_cast<int>(hidden);
    a.eps = eps;
    const int cap1 = 8 * sm_count(dev1);
    const int grid1 = tokens < cap1 ? static_cast<int>(tokens) : cap1;
    cudaError_t e = launch_pdl(lvb::ar::add_rmsnorm_kernel, dim3(grid1), dim3(lvb::ar::kThreads), 0,
                               reinterpret_cast<cudaStream_t>(stream), a);
    return e == cudaSuccess ? LVB_OK : cuda_fail(e, "add_rmsnorm_kernel launch");
  }
  for (int r = 0; r < world; ++r) {
    if (!workspaces[r] || !aligned16(workspaces[r])) return fail(LVB_ERR_INVALID, "peer workspace %d is null or unaligned", r);
    a.ws[r] = static_cast<uint8_t *>(workspaces[r]);
  }
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  a.rank = rank;
  a.world = world;
  a.partial = partial;
  a.residual = residual;
  a.weight = weight;
  a.out = out;
  a.tokens = static_cast<int>(tokens);
  a.hidden = static_cast<int>(hidden);
  a.slot_bytes = static_cast<size_t>(max_tokens) * hidden * 2;
  a.eps = eps;
  const size_t bytes = static_cast<size_t>(tokens) * hidden * 2;
  if (mode == lvb::ar::kAuto)
    mode = (world <= 2 || bytes * (world - 1) <= kSentinelOneShotMaxPushBytes) ? lvb::ar::kSentinel
                                                                               : lvb::ar::kSentinelTwoShot;
  a.mode = mode;
  const int cap = allreduce_capacity(dev);
  int grid;
  if (mode != lvb::ar::kTwoShot && mode != lvb::ar::kSentinelTwoShot) {
    grid = tokens < cap ? static_cast<int>(tokens) : cap;
  } else {
    const int64_t per_owner_vecs = (tokens * hidden / 8 + world - 1) / world;
    int64_t want = (per_owner_vecs + lvb::ar::kThreads - 1) / lvb::ar::kThreads;
    if (want < tokens) want = tokens;
    grid = want < cap ? static_cast<int>(want) : cap;
  }
  cudaError_t e = launch_pdl(lvb::ar::allreduce_add_rmsnorm_kernel, dim3(grid), dim3(lvb::ar::kThreads), 0,
                             reinterpret_cast<cudaStream_t>(stream), a);
  if (e != cudaSuccess) return cuda_fail(e, "allreduce_add_rmsnorm_kernel launch");
  return LVB_OK;
}

/* ------------------------------------------------------------------------ */
/* Qwen2 element-wise layer steps                                            */
/* ------------------------------------------------------------------------ */

int lvb_rope_qk(uint16_t *qkv, int64_t row_stride, int64_t tokens, int64_t num_query_heads, int64_t num_kv_heads,
                int64_t head_size, const int32_t *positions, const uint16_t *cos_table, const uint16_t *sin_table,
                int64_t table_rows, lvb_stream_t stream) {
  if (tokens < 0 || tokens > INT_MAX || num_query_heads <= 0 || num_kv_heads <= 0 || head_size <= 0 ||
      head_size % 2 || head_size > 1024 || table_rows <= 0 || table_rows > INT_MAX)
    return fail(LVB_ERR_INVALID, "rope: invalid shape");
  if (row_stride < (num_query_heads + num_kv_heads) * head_size)
    return fail(LVB_ERR_INVALID, "rope: row stride %lld shorter than the query and key heads", (long long)row_stride);
  if (tokens == 0) return LVB_OK;
  if (!qkv || !positions || !cos_table || !sin_table) return fail(LVB_ERR_INVALID, "rope: null pointer argument");
  lvb::q2::RopeArgs a{};
  a.qkv = qkv;
  a.row_stride = row_stride;
  a.positions = positions;
  a.cos = cos_table;
  a.sin = sin_table;
  a.tokens = static_cast<int>(tokens);
  a.hq = static_cast<int>(num_query_heads);
  a.hkv = static_cast<int>(num_kv_heads);
  a.D = static_cast<int>(head_size);
  a.table_rows = static_cast<int>(table_rows);
  const bool vec = head_size % 16 == 0 && row_stride % 8 == 0 && aligned16(qkv) && aligned16(cos_table) &&
                   aligned16(sin_table);
  cudaError_t e = vec ? launch_pdl(lvb::q2::rope_qk_kernel<true>, dim3(static_cast<unsigned>(tokens)),
                                  dim3(lvb::q2::kRopeThreads), 0, reinterpret_cast<cudaStream_t>(stream), a)
                      : launch_pdl(lvb::q2::rope_qk_kernel<false>, dim3(static_cast<unsigned>(tokens)),
                                   dim3(lvb::q2::kRopeThreads), 0, reinterpret_cast<cudaStream_t>(stream), a);
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "rope_qk_kernel launch");
}

int lvb_rope_kv_write(uint16_t *qkv, int64_t row_stride, int64_t tokens, int64_t num_query_heads,
                      int64_t num_kv_heads, int64_t head_size, const int32_t *positions, const uint16_t *cos_table,
                      const uint16_t *sin_table, int64_t table_rows, uint16_t *key_cache, uint16_t *value_cache,
                      const int32_t *block_tables, int64_t table_stride, const int32_t *num_computed,
                      const int32_t *query_start_loc, const int32_t *request_indices, int64_t block_size,
                      lvb_stream_t stream) {
  if (tokens < 0 || tokens > INT_MAX || num_query_heads <= 0 || num_kv_heads <= 0 || head_size <= 0 ||
      head_size % 16 || head_size > 1024 || table_rows <= 0 || table_rows > INT_MAX || block_size <= 0 ||
      block_size > INT_MAX)
    return fail(LVB_ERR_INVALID, "rope_kv_write: invalid shape (head size a multiple of 16)");
  if (row_stride < (num_query_heads + 2 * num_kv_heads) * head_size || row_stride % 8)
    return fail(LVB_ERR_INVALID, "rope_kv_write: row stride must cover the Q, K and V heads and be a multiple of 8");
  if (tokens == 0) return LVB_OK;
  if (!qkv || !positions || !cos_table || !sin_table || !key_cache || !value_cache || !block_tables ||
      !num_computed || !query_start_loc || !request_indices)
    return fail(LVB_ERR_INVALID, "rope_kv_write: null pointer argument");
  if (!aligned16(qkv) || !aligned16(cos_table) || !aligned16(sin_table) || !aligned16(key_cache) ||
      !aligned16(value_cache))
    return fail(LVB_ERR_INVALID, "rope_kv_write: rows, tables and caches must be 16-byte aligned");
  lvb::q2::RopeKVArgs a{};
  a.qkv = qkv;
  a.row_stride = row_stride;
  a.positions = positions;
  a.cos = cos_table;
  a.sin = sin_table;
  a.key_cache = key_cache;
  a.value_cache = value_cache;
  a.tables = block_tables;
  a.table_stride = table_stride;
  a.computed = num_computed;
  a.qsl = query_start_loc;
  a.req = request_indices;
  a.tokens = static_cast<int>(tokens);
  a.hq = static_cast<int>(num_query_heads);
  a.hkv = static_cast<int>(num_kv_heads);
  a.D = static_cast<int>(head_size);
  a.bs = static_cast<int>(block_size);
  a.table_rows = static_cast<int>(table_rows);
  cudaError_t e = launch_pdl(lvb::q2::rope_kv_write_kernel, dim3(static_cast<unsigned>(tokens)),
                             dim3(lvb::q2::kRopeThreads), 0, reinterpret_cast<cudaStream_t>(stream), a);
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "rope_kv_write_kernel launch");
}

size_t lvb_lm_head_workspace_bytes(void) { return 256; }

int lvb_lm_head_argmax(const uint16_t *hidden, int64_t hidden_stride, int64_t tokens, const uint16_t *weight,
                       int64_t vocab_rows, int64_t hidden_size, int64_t vocab_offset, int64_t *out_index,
                       float *out_value, void *workspace, lvb_stream_t stream) {
  if (tokens < 1 || tokens > lvb::q2::kHeadMaxTokens)
    return fail(LVB_ERR_UNSUPPORTED, "lm_head argmax covers 1..%d tokens, got %lld", lvb::q2::kHeadMaxTokens,
                (long long)tokens);
  if (vocab_rows <= 0 || vocab_rows > INT_MAX || hidden_size <= 0 || hidden_size % 8 || hidden_size > 16384 ||
      hidden_stride < hidden_size || hidden_stride % 8)
    return fail(LVB_ERR_INVALID, "lm_head argmax: invalid shape (hidden size a multiple of 8 up to 16384)");
  if (!hidden || !weight || !out_index || !workspace || !aligned16(hidden) || !aligned16(weight) ||
      !aligned16(workspace))
    return fail(LVB_ERR_INVALID, "lm_head argmax: tensors must be non-null and 16-byte aligned");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  lvb::q2::HeadArgs a{};
  a.hidden = hidden;
  a.hidden_stride = hidden_stride;
  a.weight = weight;
  a.tokens = static_cast<int>(tokens);
  a.H = static_cast<int>(hidden_size);
  a.V = static_cast<int>(vocab_rows);
  a.vocab_offset = vocab_offset;
  a.keys = static_cast<unsigned long long *>(workspace);
  a.counter = reinterpret_cast<unsigned int *>(static_cast<uint8_t *>(workspace) + 8 * lvb::q2::kHeadMaxTokens);
  a.out_index = out_index;
  a.out_value = out_value;
  const int tok = tokens <= 1 ? 1 : tokens <= 2 ? 2 : 4;
  const size_t smem = static_cast<size_t>(tok) * hidden_size * 4;
  // The kernels are opted in once to kHeadMaxSmem of dynamic shared memory
  // (the attribute caps every later launch, so it is set to the largest).
  constexpr size_t kHeadMaxSmem = 200 * 1024;
  if (smem > kHeadMaxSmem)
    return fail(LVB_ERR_UNSUPPORTED, "lm_head argmax: %d rows x %lld hidden values exceed shared memory", tok,
                (long long)hidden_size);
  // Up to four CTAs per SM, as many as the fp32 hidden rows let fit.
  int per_sm = static_cast<int>((200 * 1024) / (smem + 4096));
  if (per_sm > 4) per_sm = 4;
  if (per_sm < 1) per_sm = 1;
  const int64_t rows_per_cta = lvb::q2::kHeadThreads / 32;
  int64_t ctas = static_cast<int64_t>(sm_count(dev)) * per_sm;
  if (ctas > (vocab_rows + rows_per_cta - 1) / rows_per_cta) ctas = (vocab_rows + rows_per_cta - 1) / rows_per_cta;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (tok == 1) {
    static bool done[kMaxDevices] = {false};
    rc = ensure_smem(lvb::q2::lm_head_argmax_kernel<1>, static_cast<int>(kHeadMaxSmem), dev, done);
    if (rc != LVB_OK) return rc;
    e = launch_pdl(lvb::q2::lm_head_argmax_kernel<1>, dim3(static_cast<unsigned>(ctas)), dim3(lvb::q2::kHeadThreads),
                   smem, st, a);
  } else if (tok == 2) {
    static bool done[kMaxDevices] = {false};
    rc = ensure_smem(lvb::q2::lm_head_argmax_kernel<2>, static_cast<int>(kHeadMaxSmem), dev, done);
    if (rc != LVB_OK) return rc;
    e = launch_pdl(lvb::q2::lm_head_argmax_kernel<2>, dim3(static_cast<unsigned>(ctas)), dim3(lvb::q2::kHeadThreads),
                   smem, st, a);
  } else {
    static bool done[kMaxDevices] = {false};
    rc = ensure_smem(lvb::q2::lm_head_argmax_kernel<4>, static_cast<int>(kHeadMaxSmem), dev, done);
    if (rc != LVB_OK) return rc;
    e = launch_pdl(lvb::q2::lm_head_argmax_kernel<4>, dim3(static_cast<unsigned>(ctas)), dim3(lvb::q2::kHeadThreads),
                   smem, st, a);
  }
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "lm_head_argmax_kernel launch");
}

int lvb_embedding(const int64_t *ids, int64_t tokens, const uint16_t *table, int64_t vocab_start, int64_t vocab_end,
                  int64_t hidden_size, uint16_t *out, int64_t out_stride, lvb_stream_t stream) {
  if (tokens < 0 || tokens > INT_MAX || hidden_size <= 0 || hidden_size % 8 || out_stride < hidden_size ||
      out_stride % 8 || vocab_end < vocab_start)
    return fail(LVB_ERR_INVALID, "embedding: invalid shape (hidden size and row stride multiples of 8)");
  if (tokens == 0) return LVB_OK;
  if (!ids || !table || !out || !aligned16(table) || !aligned16(out))
    return fail(LVB_ERR_INVALID, "embedding: tensors must be non-null and 16-byte aligned");
  cudaError_t e = launch_pdl(lvb::q2::embedding_kernel, dim3(static_cast<unsigned>(tokens)), dim3(128), 0,
                             reinterpret_cast<cudaStream_t>(stream), ids, table, vocab_start, vocab_end,
                             static_cast<int>(hidden_size), out, out_stride);
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "embedding_kernel launch");
}

int lvb_silu_mul(const uint16_t *gate_up, int64_t in_stride, int64_t tokens, int64_t intermediate, uint16_t *out,
                 int64_t out_stride, lvb_stream_t stream) {
  if (tokens < 0 || tokens > INT_MAX || intermediate <= 0 || intermediate % 8 || intermediate > INT_MAX / 2)
    return fail(LVB_ERR_INVALID, "silu_mul: intermediate size must be a positive multiple of 8");
  if (in_stride < 2 * intermediate || in_stride % 8 || out_stride < intermediate || out_stride % 8)
    return fail(LVB_ERR_INVALID, "silu_mul: row strides must cover the rows and be multiples of 8");
  if (tokens == 0) return LVB_OK;
  if (!gate_up || !out || !aligned16(gate_up) || !aligned16(out))
    return fail(LVB_ERR_INVALID, "silu_mul: tensors must be non-null and 16-byte aligned");
  lvb::q2::SiluArgs a{};
  a.gate_up = gate_up;
  a.in_stride = in_stride;
  a.out = out;
  a.out_stride = out_stride;
  a.tokens = static_cast<int>(tokens);
  a.inter = static_cast<int>(intermediate);
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != LVB_OK) return rc;
  const int64_t vecs = tokens * (intermediate / 8);
  int64_t blocks = (vecs + lvb::q2::kSiluThreads - 1) / lvb::q2::kSiluThreads;
  const int64_t cap = 8LL * sm_count(dev);
  if (blocks > cap) blocks = cap;
  cudaError_t e = launch_pdl(lvb::q2::silu_mul_kernel, dim3(static_cast<unsigned>(blocks)),
                             dim3(lvb::q2::kSiluThreads), 0, reinterpret_cast<cudaStream_t>(stream), a);
  return e == cudaSuccess ? LVB_OK : cuda_fail(e, "silu_mul_kernel launch");
}
