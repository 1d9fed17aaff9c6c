// C ABI of libwamffn: plans, tensor-map encoding, launch configuration.
// See include/wamffn.h for the contract of every entry point.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "gemm.cuh"
#include "attention.cuh"
#include "pass.cuh"
#include "rowops.cuh"
#include "select.cuh"
#include "wamffn.h"

namespace wamffn {

// Thread 0 waits on a barrier no one arrives on, with a short limit; thread 32
// waits on the same phase with a longer one and must leave through the abort
// flag that thread 0 raises.
__global__ void selftest_wait_timeout_kernel(unsigned int* status, long long limit) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    wait_bounded(smem_addr(&bar), 0u, &abort_flag, status, WAMFFN_DEV_TIMEOUT, limit);
  } else if (threadIdx.x == 32) {
    if (!wait_bounded(smem_addr(&bar), 0u, &abort_flag, nullptr, 0u, 4 * limit) && abort_flag)
      atomicOr(status, kSelftestAbortSeen);
  }
  __syncthreads();
}

}  // namespace wamffn

// Scratch of wamffn_linear_run_static, one copy per device shared by every
// call: a status word in the first 256 bytes, then [splits, rows, n_out] fp32
// split-K partials.
static __device__ __align__(256) unsigned char g_static_scratch[WAMFFN_STATIC_SCRATCH_BYTES];

using namespace wamffn;

namespace {

thread_local std::string g_error;
std::atomic<unsigned long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

#define WAMFFN_CUDA(call)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return fail(WAMFFN_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && (prev == dev || cudaSetDevice(dev) == cudaSuccess))
      ok = true;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool env_flag(const char* name, bool dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return !(v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F');
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor [outer, inner] (inner contiguous, rows `row_bytes` apart),
// box [box_outer, 64] with the 128-byte swizzle.
int encode_operand(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return fail(WAMFFN_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {uint32_t(kBlockK), box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WAMFFN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return WAMFFN_OK;
}

struct DeviceInfo {
  int sm_count = 0;
  bool ready = false;
};
std::mutex g_dev_mu;
DeviceInfo g_dev[64];

// Checks the device is an sm_100 part and raises the kernels' shared-memory limit once.
int prepare_device(int device, int* sm_count) {
  if (device < 0 || device >= 64) return fail(WAMFFN_ERR_INVALID, "bad device %d", device);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceInfo& d = g_dev[device];
  if (!d.ready) {
    int major = 0, minor = 0;
    WAMFFN_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    WAMFFN_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    if (major != 10 || minor != 0)
      return fail(WAMFFN_ERR_UNSUPPORTED, "libwamffn is built for sm_100a; device %d is sm_%d%d",
                  device, major, minor);
    WAMFFN_CUDA(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device));
    DeviceGuard g(device);
    WAMFFN_CUDA(cudaFuncSetAttribute(umma_gemm_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemLimit));
    WAMFFN_CUDA(cudaFuncSetAttribute(umma_gemm_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemLimit));
    WAMFFN_CUDA(cudaFuncSetAttribute(umma_gemm_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemLimit));
    WAMFFN_CUDA(cudaFuncSetAttribute(umma_gemm_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemLimit));
    WAMFFN_CUDA(cudaFuncSetAttribute(masked_attention_kernel<false, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
    WAMFFN_CUDA(cudaFuncSetAttribute(masked_attention_kernel<false, true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
    WAMFFN_CUDA(cudaFuncSetAttribute(masked_attention_kernel<true, false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
    WAMFFN_CUDA(cudaFuncSetAttribute(masked_attention_kernel<true, true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
    cudaFuncAttributes pass_attr{};
    WAMFFN_CUDA(cudaFuncGetAttributes(&pass_attr, stack_pass_kernel));  // its static barriers count too
    WAMFFN_CUDA(cudaFuncSetAttribute(stack_pass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemLimit - int(pass_attr.sharedSizeBytes)));
    d.ready = true;
  }
  *sm_count = d.sm_count;
  return WAMFFN_OK;
}

// ---------------------------------------------------------------- GEMM config
struct GemmConfig {
  int rows = 0, n_out = 0, k_in = 0;
  int group = 1;  // CTAs per UMMA (2 = cta_group::2 pair)
  int groups = 1;      // token groups (grid.z)
  int group_rows = 0;  // rows per token group
  int tok_pad = 0, mma_n0 = 0, mma_n1 = 0, tok_box = 0, n_boxes = 0, b_rows = 0;
  int a_stages = 0, b_stages = 0, splits = 1;
  uint32_t tmem_cols = 0;
  int smem_bytes = 0;
  int sk = 0;  // stream-K CTA groups (pairs with group == 2); 0 = data-parallel grid
};

// Stream-K is opt-in: on B200 it measured slower for the FFN up projection
// (48 vs 36 us at M = 392): with all 148 SMs streaming, each K block's
// operands arrive more slowly (0.72 vs 0.63 us per block), and the helper
// dump and the owner's fix-up move 30 MB of fp32 partials through L2.
bool streamk_enabled() {
  static const bool on = env_flag("WAMFFN_STREAMK", false);
  return on;
}

// Stream-K size for a bias / GELU GEMM whose feature tiles leave SMs idle:
// one range of K blocks per CTA group on every SM, each range within one
// tile's K extent, at most kMaxSkHelpers helper pieces per owner tile.
// 0 when the data-parallel grid already fills the machine.
int streamk_groups(const GemmConfig& c, int sm_count) {
  if (c.splits != 1 || c.groups != 1) return 0;
  const int tiles = c.n_out / (kFeatTile * c.group);
  const int kb = c.k_in / kBlockK;
  const long long units = (long long)tiles * kb;
  for (int g = sm_count / c.group; g > tiles; --g) {
    const long long per = units / g;  // shortest range
    if (per < 1) continue;
    const long long helpers = (kb + per - 1) / per;
    if (helpers <= kMaxSkHelpers && (units + g - 1) / g <= kb) return g;
  }
  return 0;
}

// Bytes of stream-K workspace (helper slots) a plan holds for tok_pad tokens.
size_t streamk_ws_bytes(int sm_count, int tok_pad) { return size_t(sm_count) * tok_pad * kFeatTile * sizeof(float); }

bool pair_enabled() {
  static const bool on = env_flag("WAMFFN_PAIR", true);
  return on;
}

int make_gemm_config(int rows, int n_out, int k_in, int splits, GemmConfig* c, int groups = 1,
                     int smem_budget = kSmemLimit - kSmemReserve - kGemmRowSlack) {
  if (rows < 1 || rows > kMaxTokens * 4)
    return fail(WAMFFN_ERR_UNSUPPORTED, "rows=%d outside [1, %d]", rows, kMaxTokens * 4);
  if (groups < 1 || groups > 4) return fail(WAMFFN_ERR_UNSUPPORTED, "token groups=%d outside [1, 4]", groups);
  const int total_rows = rows;
  rows = (rows + groups - 1) / groups;  // rows per token group
  if (rows > kMaxTokens)
    return fail(WAMFFN_ERR_UNSUPPORTED, "rows per token group=%d above %d", rows, kMaxTokens);
  if ((groups - 1) * rows >= total_rows)
    return fail(WAMFFN_ERR_UNSUPPORTED, "%d rows leave token group %d of %d empty", total_rows, groups - 1, groups);
  if (n_out < kFeatTile || n_out % kFeatTile)
    return fail(WAMFFN_ERR_UNSUPPORTED, "n_out=%d must be a positive multiple of %d", n_out, kFeatTile);
  if (k_in < kBlockK || k_in % kBlockK)
    return fail(WAMFFN_ERR_UNSUPPORTED, "k_in=%d must be a positive multiple of %d", k_in, kBlockK);
  c->rows = total_rows;
  c->groups = groups;
  c->group_rows = rows;
  c->n_out = n_out;
  c->k_in = k_in;
  c->group = (pair_enabled() && (n_out / kFeatTile) % 2 == 0) ? 2 : 1;
  if (c->group == 2) {
    // Pair: each CTA holds half of every UMMA's tokens (multiples of 8 rows).
    if (rows <= 256) {
      c->tok_pad = (rows + 15) / 16 * 16;
      c->mma_n0 = c->tok_pad;
      c->mma_n1 = 0;
      c->n_boxes = 1;
      c->tok_box = c->tok_pad / 2;
    } else {
      // Two UMMAs with N multiples of 16 covering the rows with the least
      // padding (392 -> 208 + 192, 304 -> 160 + 144).  Each CTA stages both
      // halves in boxes of the larger height; the smaller box's extra rows are
      // loaded but not read.
      c->mma_n0 = ((rows + 1) / 2 + 15) / 16 * 16;
      c->mma_n1 = (rows - c->mma_n0 + 15) / 16 * 16;
      c->tok_pad = c->mma_n0 + c->mma_n1;
      c->n_boxes = 2;
      c->tok_box = c->mma_n0 / 2;
    }
    c->b_rows = c->n_boxes * c->tok_box;
  } else {
    c->tok_pad = (rows + 15) / 16 * 16;
    if (c->tok_pad <= 256) {
      c->mma_n0 = c->tok_pad;
      c->mma_n1 = 0;
      c->tok_box = c->tok_pad;
      c->n_boxes = 1;
    } else {
      c->mma_n0 = (c->tok_pad / 16 + 1) / 2 * 16;
      c->mma_n1 = c->tok_pad - c->mma_n0;
      c->tok_box = c->tok_pad / 2;  // multiple of 8: each box starts on a 1024-byte swizzle atom
      c->n_boxes = 2;
    }
    c->b_rows = c->tok_pad;
  }
  uint32_t cols = 32;
  while (cols < uint32_t(c->tok_pad)) cols <<= 1;
  c->tmem_cols = cols;
  // Shared memory: the activation ring (L2 hits, needs depth against the
  // lockstep bursts of all SMs) and the weight ring (HBM stream) share 227 KB.
  const int budget = smem_budget;
  const int b_bytes = c->b_rows * kBlockK * 2;
  c->b_stages = (budget / 2) / b_bytes;
  if (c->b_stages > kMaxBStages) c->b_stages = kMaxBStages;
  if (c->b_stages < 2) c->b_stages = 2;
  c->a_stages = (budget - c->b_stages * b_bytes) / gemm_a_bytes();
  if (c->a_stages > kMaxAStages) c->a_stages = kMaxAStages;
  if (c->a_stages < 2) return fail(WAMFFN_ERR_UNSUPPORTED, "rows=%d leaves fewer than 2 pipeline stages", rows);
  const int k_blocks = k_in / kBlockK;
  if (splits < 1) splits = 1;
  if (splits > k_blocks) splits = k_blocks;
  c->splits = splits;
  c->smem_bytes = c->a_stages * gemm_a_bytes() + c->b_stages * b_bytes + kSmemReserve;
  return WAMFFN_OK;
}

// Split-K heuristic: fill the SMs with (feature tiles x splits) CTAs while
// keeping at least 8 K blocks per split.
int default_splits(int n_out, int k_in, int sm_count) {
  const int tiles = n_out / kFeatTile;
  const int k_blocks = k_in / kBlockK;
  int best = 1;
  for (int s = 1; s <= 16; ++s) {
    if (tiles * s > sm_count) break;
    if (k_blocks / s < 8) break;
    best = s;
  }
  return best;
}

int launch_gemm(const GemmConfig& c, int epi, cudaStream_t stream, const void* weight, bool packed,
                const void* act, const void* bias, void* out, unsigned int* status, bool pdl,
                float* sk_ws = nullptr, unsigned int* sk_flags = nullptr) {
  if (c.sk > 0 && (epi == EPI_PARTIAL_F32 || !sk_ws || !sk_flags))
    return fail(WAMFFN_ERR_INVALID, "stream-K needs a bias or GELU epilogue and its workspace");
  CUtensorMap tm_w, tm_x;
  int rc = packed ? encode_operand(&tm_w, weight, uint64_t(kBlockK), uint64_t(c.n_out) * (c.k_in / kBlockK),
                                   uint64_t(kBlockK) * 2, kFeatTile)
                  : encode_operand(&tm_w, weight, uint64_t(c.k_in), uint64_t(c.n_out), uint64_t(c.k_in) * 2,
                                   kFeatTile);
  if (rc) return rc;
  rc = encode_operand(&tm_x, act, uint64_t(c.k_in), uint64_t(c.rows), uint64_t(c.k_in) * 2,
                      uint32_t(c.tok_box));
  if (rc) return rc;
  GemmParams p{};
  p.tokens = c.rows;
  p.group_rows = c.group_rows;
  p.tok_pad = c.tok_pad;
  p.mma_n0 = c.mma_n0;
  p.mma_n1 = c.mma_n1;
  p.tok_box = c.tok_box;
  p.n_boxes = c.n_boxes;
  p.b_rows = c.b_rows;
  p.k_blocks = c.k_in / kBlockK;
  p.splits = c.splits;
  p.a_stages = c.a_stages;
  p.b_stages = c.b_stages;
  p.n_total = c.n_out;
  p.tmem_cols = c.tmem_cols;
  p.epi = epi;
  p.w_packed = packed ? 1 : 0;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.out = out;
  p.status = status;
  p.sk = c.sk;
  p.sk_tiles = c.n_out / (kFeatTile * c.group);
  p.sk_ws = sk_ws;
  p.sk_flags = sk_flags;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = c.sk > 0 ? dim3(unsigned(c.sk * c.group), 1, 1)
                         : dim3(unsigned(c.n_out / kFeatTile), unsigned(c.splits), unsigned(c.groups));
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = size_t(c.smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = unsigned(c.group);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;  // token groups are independent: clusters of more than 2 CTAs fit fewer SMs
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (c.sk > 0) {
    if (c.group == 2) WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, umma_gemm_kernel<2, true>, tm_w, tm_x, p));
    else WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, umma_gemm_kernel<1, true>, tm_w, tm_x, p));
  } else {
    if (c.group == 2) WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, umma_gemm_kernel<2, false>, tm_w, tm_x, p));
    else WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, umma_gemm_kernel<1, false>, tm_w, tm_x, p));
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

int row_threads(int dim) {
  int t = ((dim / 8) + 31) / 32 * 32;
  if (t < 32) t = 32;
  if (t > kRowThreads) t = kRowThreads;
  return t;
}

int launch_norm(const NormParams& p, int grid, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid), 1, 1);
  cfg.blockDim = dim3(unsigned(row_threads(p.dim)), 1, 1);
  cfg.dynamicSmemBytes = size_t(p.dim) * sizeof(float);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, modnorm_kernel, p));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

int launch_epi(const EpiParams& p, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(p.seq), 1, 1);
  cfg.blockDim = dim3(unsigned(row_threads(p.dim)), 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, rowepi_kernel, p));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

bool pdl_enabled() {
  static const bool on = env_flag("WAMFFN_PDL", true);
  return on;
}

}  // namespace

// ====================================================================== plans
struct wamffn_linear_plan {
  int device = 0;
  int gelu = 0;
  int packed = 0;
  int tuned = 0;
  GemmConfig cfg;
  float* partial = nullptr;      // [splits, rows, n_out] when splits > 1
  __nv_bfloat16* hidden = nullptr;  // [rows, n_out] scratch for wamffn_ffn_run (up plans)
  unsigned int* status = nullptr;
  float* sk_ws = nullptr;           // stream-K helper slots when cfg.sk > 0
  unsigned int* sk_flags = nullptr;
};

struct wamffn_block_plan {
  int device = 0;
  int sm_count = 0;
  int max_rows = 0, max_seq = 0, d = 0, h = 0;
  int tune = 0;
  __nv_bfloat16* gathered = nullptr;  // [max_rows, d]
  __nv_bfloat16* hidden = nullptr;    // [max_rows, h]
  __nv_bfloat16* y = nullptr;         // [max_seq, d] residual scratch when the caller wants no y
  float* partial = nullptr;           // [max_splits, max_rows, d]
  int max_splits = 1;
  int* pos = nullptr;                 // [max_seq]
  unsigned int* status = nullptr;
  unsigned int* pass_bars = nullptr;  // phase counters of the persistent pass kernel
  int pass_ctas = 0;                  // co-resident CTAs of the pass kernel (0: unavailable)
  int split_override[kMaxTokens + 1];  // tuned split-K per row count (0 = heuristic)
  int up_streamk = 1;                 // stream-K up projection when its tiles leave SMs idle
  float* sk_ws = nullptr;             // stream-K helper slots of the up projection
  unsigned int* sk_flags = nullptr;
};

namespace {

int linear_execute(wamffn_linear_plan* plan, cudaStream_t stream, const void* x, const void* weight,
                   const void* bias, void* out) {
  const GemmConfig& c = plan->cfg;
  const bool pdl = pdl_enabled();
  if (c.splits == 1) {
    return launch_gemm(c, plan->gelu ? EPI_GELU_BF16 : EPI_BIAS_BF16, stream, weight, plan->packed, x, bias, out,
                       plan->status, pdl, plan->sk_ws, plan->sk_flags);
  }
  int rc = launch_gemm(c, EPI_PARTIAL_F32, stream, weight, plan->packed, x, nullptr, plan->partial, plan->status,
                       pdl);
  if (rc) return rc;
  EpiParams e{};
  e.partial = plan->partial;
  e.splits = c.splits;
  e.m = c.rows;
  e.dim = c.n_out;
  e.bias = static_cast<const __nv_bfloat16*>(bias);
  e.pos_of_row = nullptr;
  e.seq = c.rows;
  e.output = static_cast<__nv_bfloat16*>(out);
  e.status = plan->status;
  e.pdl = 1;
  return launch_epi(e, stream, pdl);
}

// Times `iters` launches of the plan on scratch operands; returns ms per launch.
// The launches rotate over `copies` weight matrices of w_bytes each (together
// larger than L2), so that every launch streams its weights from HBM, as the
// per-layer weights of a model do.
int time_linear(wamffn_linear_plan* plan, const void* x, const void* w, size_t w_bytes, int copies,
                const void* b, void* out, float* ms) {
  cudaStream_t s;
  WAMFFN_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  cudaEvent_t e0, e1;
  WAMFFN_CUDA(cudaEventCreate(&e0));
  WAMFFN_CUDA(cudaEventCreate(&e1));
  auto weight = [&](int i) { return static_cast<const void*>(static_cast<const char*>(w) + (i % copies) * w_bytes); };
  int rc = WAMFFN_OK;
  for (int i = 0; i < 3 && !rc; ++i) rc = linear_execute(plan, s, x, weight(i), b, out);
  const int iters = 16;
  if (!rc) WAMFFN_CUDA(cudaEventRecord(e0, s));
  for (int i = 0; i < iters && !rc; ++i) rc = linear_execute(plan, s, x, weight(3 + i), b, out);
  if (!rc) {
    WAMFFN_CUDA(cudaEventRecord(e1, s));
    WAMFFN_CUDA(cudaEventSynchronize(e1));
    float t = 0;
    WAMFFN_CUDA(cudaEventElapsedTime(&t, e0, e1));
    *ms = t / iters;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaStreamDestroy(s);
  return rc;
}

}  // namespace

extern "C" {

int wamffn_abi_version(void) { return WAMFFN_ABI_VERSION; }

const char* wamffn_last_error(void) { return g_error.c_str(); }

unsigned long long wamffn_launch_count(void) { return g_launches.load(); }

int wamffn_linear_plan_create(int device, int rows, int n_out, int k_in, int flags, int tune,
                              wamffn_linear_plan** out_plan) {
  if (!out_plan) return fail(WAMFFN_ERR_INVALID, "plan output pointer is null");
  *out_plan = nullptr;
  GemmConfig probe;
  int rc = make_gemm_config(rows, n_out, k_in, 1, &probe);
  if (rc) return rc;
  int sm = 0;
  rc = prepare_device(device, &sm);
  if (rc) return rc;
  DeviceGuard guard(device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", device);
  {
    // Creation allocates and may tune: refuse inside a capture, like the reference.
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    WAMFFN_CUDA(cudaStreamIsCapturing(cudaStreamLegacy, &st));
    if (st != cudaStreamCaptureStatusNone)
      return fail(WAMFFN_ERR_CAPTURE, "GEMM planning must finish before CUDA Graph capture");
  }
  auto* plan = new wamffn_linear_plan();
  plan->device = device;
  plan->gelu = (flags & WAMFFN_LINEAR_GELU) ? 1 : 0;
  plan->packed = (flags & WAMFFN_WEIGHTS_PACKED) ? 1 : 0;
  // GELU is applied in the GEMM epilogue, so a GELU plan never splits K (the
  // split-K reduction applies the bias only).
  rc = make_gemm_config(rows, n_out, k_in, plan->gelu ? 1 : default_splits(n_out, k_in, sm), &plan->cfg);
  if (rc) {
    delete plan;
    return rc;
  }
  // Stream-K for a GELU plan whose tiles leave SMs idle (the split-K reduction
  // of the bias plans fills the machine instead).
  const int sk_candidate = (plan->gelu && streamk_enabled()) ? streamk_groups(plan->cfg, sm) : 0;
  plan->cfg.sk = sk_candidate;
  auto cleanup = [&](int code) {
    wamffn_linear_plan_destroy(plan);
    return code;
  };
  if (cudaMalloc(&plan->status, sizeof(unsigned int)) != cudaSuccess ||
      cudaMemset(plan->status, 0, sizeof(unsigned int)) != cudaSuccess)
    return cleanup(fail(WAMFFN_ERR_CUDA, "status allocation failed"));
  if (plan->gelu && cudaMalloc(&plan->hidden, size_t(rows) * n_out * 2) != cudaSuccess)
    return cleanup(fail(WAMFFN_ERR_CUDA, "hidden scratch allocation failed"));
  if (sk_candidate > 0 &&
      (cudaMalloc(&plan->sk_ws, streamk_ws_bytes(sm, plan->cfg.tok_pad)) != cudaSuccess ||
       cudaMalloc(&plan->sk_flags, size_t(sm) * sizeof(unsigned int)) != cudaSuccess ||
       cudaMemset(plan->sk_flags, 0, size_t(sm) * sizeof(unsigned int)) != cudaSuccess))
    return cleanup(fail(WAMFFN_ERR_CUDA, "stream-K workspace allocation failed"));
  const int tiles = n_out / kFeatTile;
  if (tune) {
    // Candidate layouts -- split-K factor x token groups (grid.z), and for a
    // GELU plan the stream-K grid -- are timed on scratch operands, the way
    // the reference times every candidate algorithm (cpp:121-158).  Split-K
    // moves fp32 partials through L2; token groups re-read each weight tile
    // (from L2 after the first group) but write no partials.
    int max_s = 1;
    for (int s = 2; !plan->gelu && s <= 16 && tiles * s <= 2 * sm && (k_in / kBlockK) / s >= 4; ++s) max_s = s;
    const size_t w_bytes = size_t(n_out) * k_in * 2;
    // Enough weight copies to exceed L2 (at most 16 and 192 MB).
    int copies = int((size_t(160) << 20) / w_bytes) + 1;
    if (copies > 16) copies = 16;
    while (copies > 1 && copies * w_bytes > (size_t(192) << 20)) --copies;
    void *x = nullptr, *w = nullptr, *b = nullptr, *o = nullptr;
    // Short of memory for the copies: time on one (L2-resident) weight copy.
    while (copies > 1 && cudaMalloc(&w, copies * w_bytes) != cudaSuccess) {
      cudaGetLastError();
      w = nullptr;
      copies = 1;
    }
    bool okalloc = cudaMalloc(&x, size_t(rows) * k_in * 2) == cudaSuccess &&
                   (w != nullptr || cudaMalloc(&w, copies * w_bytes) == cudaSuccess) &&
                   cudaMalloc(&b, size_t(n_out) * 2) == cudaSuccess &&
                   cudaMalloc(&o, size_t(rows) * n_out * 2) == cudaSuccess &&
                   (max_s == 1 || cudaMalloc(&plan->partial, size_t(max_s) * rows * n_out * 4) == cudaSuccess);
    if (okalloc) {
      cudaMemset(x, 0x3c, size_t(rows) * k_in * 2);
      cudaMemset(w, 0x3c, copies * w_bytes);
      cudaMemset(b, 0, size_t(n_out) * 2);
      float best = 1e30f;
      int best_s = plan->cfg.splits, best_g = 1, best_sk = 0;
      for (int s = 1; s <= max_s; ++s) {
        for (int g = 1; g <= 4; ++g) {
          if (g > 1 && (tiles * s * g > sm || (rows + g - 1) / g < 16)) break;
          // Candidates: split-K factors x token groups, and for the GELU plan
          // also the stream-K grid.
          const int sks[2] = {0, sk_candidate};
          const int n_sk = (s == 1 && g == 1 && sk_candidate > 0) ? 2 : 1;
          for (int j = 0; j < n_sk; ++j) {
            GemmConfig c;
            if (make_gemm_config(rows, n_out, k_in, s, &c, g)) continue;
            if (c.splits != s) continue;
            c.sk = sks[j];
            plan->cfg = c;
            float ms = 0;
            if (time_linear(plan, x, w, w_bytes, copies, b, o, &ms) == WAMFFN_OK && ms < best) {
              best = ms;
              best_s = s;
              best_g = g;
              best_sk = sks[j];
            }
          }
        }
      }
      make_gemm_config(rows, n_out, k_in, best_s, &plan->cfg, best_g);
      plan->cfg.sk = best_sk;
      plan->tuned = 1;
    }
    cudaFree(x);
    cudaFree(w);
    cudaFree(b);
    cudaFree(o);
    cudaFree(plan->partial);
    plan->partial = nullptr;
    cudaMemset(plan->status, 0, sizeof(unsigned int));
    if (!okalloc) return cleanup(fail(WAMFFN_ERR_CUDA, "tuning scratch allocation failed"));
  }
  if (plan->cfg.splits > 1 &&
      cudaMalloc(&plan->partial, size_t(plan->cfg.splits) * rows * n_out * sizeof(float)) != cudaSuccess)
    return cleanup(fail(WAMFFN_ERR_CUDA, "split-K workspace allocation failed"));
  *out_plan = plan;
  return WAMFFN_OK;
}

int wamffn_linear_plan_destroy(wamffn_linear_plan* plan) {
  if (!plan) return WAMFFN_OK;
  DeviceGuard guard(plan->device);
  cudaFree(plan->partial);
  cudaFree(plan->hidden);
  cudaFree(plan->status);
  cudaFree(plan->sk_ws);
  cudaFree(plan->sk_flags);
  delete plan;
  return WAMFFN_OK;
}

int wamffn_linear_run(wamffn_linear_plan* plan, void* stream, const void* x, const void* weight,
                      const void* bias, void* out) {
  if (!plan) return fail(WAMFFN_ERR_INVALID, "plan is null");
  if (!x || !weight || !bias || !out) return fail(WAMFFN_ERR_INVALID, "null tensor pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(bias) || !aligned16(out))
    return fail(WAMFFN_ERR_INVALID, "tensors must be 16-byte aligned");
  DeviceGuard guard(plan->device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", plan->device);
  return linear_execute(plan, static_cast<cudaStream_t>(stream), x, weight, bias, out);
}

int wamffn_linear_configuration(const wamffn_linear_plan* plan, uint32_t* values, int n) {
  if (!plan || !values) return fail(WAMFFN_ERR_INVALID, "null argument");
  const GemmConfig& c = plan->cfg;
  const uint32_t v[7] = {uint32_t(kFeatTile * c.group), uint32_t(c.tok_pad), uint32_t(c.mma_n1 > 0 ? 2 : 1),
                         uint32_t(c.a_stages * 100 + c.b_stages), uint32_t(c.splits), c.tmem_cols,
                         uint32_t(plan->tuned)};
  for (int i = 0; i < n && i < 7; ++i) values[i] = v[i];
  if (n > 7) values[7] = uint32_t(c.sk);  // stream-K CTA groups (0 = data-parallel grid)
  if (n > 8) values[8] = uint32_t(c.groups);  // token groups (grid.z)
  return WAMFFN_OK;
}

int wamffn_linear_plan_set_layout(wamffn_linear_plan* plan, int splits, int groups) {
  if (!plan) return fail(WAMFFN_ERR_INVALID, "plan is null");
  if (splits < 1 || splits > 16) return fail(WAMFFN_ERR_INVALID, "splits=%d outside [1, 16]", splits);
  if (groups < 1 || groups > 4) return fail(WAMFFN_ERR_INVALID, "groups=%d outside [1, 4]", groups);
  if (plan->gelu && splits != 1)
    return fail(WAMFFN_ERR_INVALID, "a GELU plan never splits K (the split-K reduction applies the bias only)");
  DeviceGuard guard(plan->device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", plan->device);
  {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    WAMFFN_CUDA(cudaStreamIsCapturing(cudaStreamLegacy, &st));
    if (st != cudaStreamCaptureStatusNone)
      return fail(WAMFFN_ERR_CAPTURE, "a plan's layout must be set before CUDA Graph capture");
  }
  GemmConfig c;
  int rc = make_gemm_config(plan->cfg.rows, plan->cfg.n_out, plan->cfg.k_in, splits, &c, groups);
  if (rc) return rc;
  if (c.splits != splits)
    return fail(WAMFFN_ERR_INVALID, "splits=%d exceeds the %d K blocks", splits, plan->cfg.k_in / kBlockK);
  // Launches already enqueued may still read the old workspace.
  WAMFFN_CUDA(cudaDeviceSynchronize());
  if (splits != plan->cfg.splits) {
    cudaFree(plan->partial);
    plan->partial = nullptr;
    if (splits > 1 &&
        cudaMalloc(&plan->partial, size_t(splits) * c.rows * c.n_out * sizeof(float)) != cudaSuccess) {
      make_gemm_config(c.rows, c.n_out, c.k_in, 1, &plan->cfg);  // a plan that still runs
      return fail(WAMFFN_ERR_CUDA, "split-K workspace allocation failed");
    }
  }
  plan->cfg = c;  // data-parallel grid (no stream-K)
  return WAMFFN_OK;
}

int wamffn_linear_status(wamffn_linear_plan* plan, uint32_t* status, int clear) {
  if (!plan || !status) return fail(WAMFFN_ERR_INVALID, "null argument");
  DeviceGuard guard(plan->device);
  WAMFFN_CUDA(cudaDeviceSynchronize());
  WAMFFN_CUDA(cudaMemcpy(status, plan->status, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  if (clear) WAMFFN_CUDA(cudaMemset(plan->status, 0, sizeof(uint32_t)));
  return WAMFFN_OK;
}

}  // extern "C"

namespace {

constexpr size_t kStaticScratchHeader = 256;  // status word, padded to the array's alignment
std::mutex g_static_mu;
void* g_static_base[64] = {};

// Device address of g_static_scratch on `device` (which must be current),
// looked up once per device.
int static_scratch_base(int device, unsigned char** base) {
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_base[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess)
      return fail(WAMFFN_ERR_CUDA, "cudaGetSymbolAddress of the static scratch on device %d: %s", device,
                  cudaGetErrorString(e));
    g_static_base[device] = ptr;
  }
  *base = static_cast<unsigned char*>(g_static_base[device]);
  return WAMFFN_OK;
}

}  // namespace

extern "C" {

int wamffn_linear_run_static(int device, void* stream_, int rows, int n_out, int k_in, int splits, int flags,
                             const void* x, const void* weight, const void* bias, void* out, uint32_t* status) {
  if (flags & ~WAMFFN_WEIGHTS_PACKED)
    return fail(WAMFFN_ERR_INVALID,
                "flags=%d: only WAMFFN_WEIGHTS_PACKED is accepted (the split-K reduction applies the bias only)",
                flags);
  if (splits < 2 || splits > 16) return fail(WAMFFN_ERR_INVALID, "splits=%d outside [2, 16]", splits);
  if (device < 0 || device >= 64) return fail(WAMFFN_ERR_INVALID, "bad device %d", device);
  if (!x || !weight || !bias || !out) return fail(WAMFFN_ERR_INVALID, "null tensor pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(bias) || !aligned16(out))
    return fail(WAMFFN_ERR_INVALID, "tensors must be 16-byte aligned");
  if (status && (reinterpret_cast<uintptr_t>(status) & 3u))
    return fail(WAMFFN_ERR_INVALID, "status must be 4-byte aligned");
  GemmConfig c;
  int rc = make_gemm_config(rows, n_out, k_in, splits, &c);
  if (rc) return rc;
  if (c.splits != splits)
    return fail(WAMFFN_ERR_INVALID, "splits=%d exceeds the %d K blocks of k_in=%d", splits, k_in / kBlockK, k_in);
  const size_t need = kStaticScratchHeader + size_t(splits) * size_t(rows) * size_t(n_out) * sizeof(float);
  if (need > size_t(WAMFFN_STATIC_SCRATCH_BYTES))
    return fail(WAMFFN_ERR_INVALID,
                "splits=%d x rows=%d x n_out=%d fp32 partials need %zu bytes of scratch; the static scratch "
                "holds %zu bytes (WAMFFN_STATIC_SCRATCH_BYTES)",
                splits, rows, n_out, need, size_t(WAMFFN_STATIC_SCRATCH_BYTES));
  int sm = 0;
  rc = prepare_device(device, &sm);
  if (rc) return rc;
  DeviceGuard guard(device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", device);
  unsigned char* base = nullptr;
  rc = static_scratch_base(device, &base);
  if (rc) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  unsigned int* st = reinterpret_cast<unsigned int*>(status);
  if (st == nullptr) {
    st = reinterpret_cast<unsigned int*>(base);
    WAMFFN_CUDA(cudaMemsetAsync(st, 0, sizeof(unsigned int), stream));
  }
  float* partial = reinterpret_cast<float*>(base + kStaticScratchHeader);
  const bool pdl = pdl_enabled();
  // The GEMM overwrites every partial it covers, so the partials need no clearing.
  rc = launch_gemm(c, EPI_PARTIAL_F32, stream, weight, (flags & WAMFFN_WEIGHTS_PACKED) != 0, x, nullptr, partial,
                   st, pdl);
  if (rc) return rc;
  EpiParams e{};
  e.partial = partial;
  e.splits = c.splits;
  e.m = c.rows;
  e.dim = c.n_out;
  e.bias = static_cast<const __nv_bfloat16*>(bias);
  e.pos_of_row = nullptr;
  e.seq = c.rows;
  e.output = static_cast<__nv_bfloat16*>(out);
  e.status = st;
  e.pdl = 1;
  return launch_epi(e, stream, pdl);
}

int wamffn_selftest_wait_timeout(void* stream, uint32_t* status, int64_t limit_cycles) {
  if (!status || (reinterpret_cast<uintptr_t>(status) & 3u))
    return fail(WAMFFN_ERR_INVALID, "status must be a non-null, 4-byte aligned device word");
  if (limit_cycles < 1000 || limit_cycles > 1000000000ll)
    return fail(WAMFFN_ERR_INVALID, "limit_cycles=%lld outside [1e3, 1e9]", (long long)limit_cycles);
  selftest_wait_timeout_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<unsigned int*>(status), static_cast<long long>(limit_cycles));
  WAMFFN_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

int wamffn_ffn_run(wamffn_linear_plan* up, wamffn_linear_plan* down, void* stream, const void* x,
                   const void* w_up, const void* b_up, const void* w_down, const void* b_down,
                   void* out) {
  if (!up || !down) return fail(WAMFFN_ERR_INVALID, "plan is null");
  if (!up->gelu || !up->hidden) return fail(WAMFFN_ERR_INVALID, "the up plan must be a GELU plan");
  if (up->cfg.rows != down->cfg.rows || up->cfg.n_out != down->cfg.k_in ||
      up->cfg.k_in != down->cfg.n_out || up->device != down->device)
    return fail(WAMFFN_ERR_INVALID, "up/down plans do not chain");
  int rc = wamffn_linear_run(up, stream, x, w_up, b_up, up->hidden);
  if (rc) return rc;
  return wamffn_linear_run(down, stream, up->hidden, w_down, b_down, out);
}

int wamffn_modulated_norm(void* stream, const wamffn_norm_args* a) {
  if (!a) return fail(WAMFFN_ERR_INVALID, "args is null");
  if (a->rows < 1 || a->dim < 8 || a->dim % 8 || a->dim > 8 * 1024 * 4)
    return fail(WAMFFN_ERR_INVALID, "rows=%d dim=%d unsupported (dim %% 8 == 0 required)", a->rows, a->dim);
  if (a->mode < 0 || a->mode > 3) return fail(WAMFFN_ERR_INVALID, "mode %d", a->mode);
  if (!a->x || !a->mod || !a->time || !a->y || !a->norm) return fail(WAMFFN_ERR_INVALID, "null tensor pointer");
  if (a->mode > 0 && !a->update) return fail(WAMFFN_ERR_INVALID, "mode %d needs update", a->mode);
  if (a->mode == WAMFFN_FFN_RESIDUAL && !a->previous) return fail(WAMFFN_ERR_INVALID, "mode 3 needs previous");
  if (a->mode == WAMFFN_SELF_RESIDUAL && (!a->weight || !a->bias))
    return fail(WAMFFN_ERR_INVALID, "mode 1 needs weight and bias");
  const void* ptrs[] = {a->x, a->update, a->mod, a->previous, a->time, a->weight, a->bias, a->y, a->norm};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return fail(WAMFFN_ERR_INVALID, "tensors must be 16-byte aligned");
  if (a->x_stride % 8 || a->update_stride % 8 || a->time_stride % 8)
    return fail(WAMFFN_ERR_INVALID, "row strides must be multiples of 8 elements");
  int dev = 0;
  WAMFFN_CUDA(cudaGetDevice(&dev));
  NormParams p{};
  p.x = static_cast<const __nv_bfloat16*>(a->x);
  p.xs = a->x_stride;
  p.update = static_cast<const __nv_bfloat16*>(a->update);
  p.us = a->update_stride;
  p.mod = static_cast<const __nv_bfloat16*>(a->mod);
  p.previous = static_cast<const __nv_bfloat16*>(a->previous);
  p.time = static_cast<const __nv_bfloat16*>(a->time);
  p.ts = a->time_stride;
  p.weight = static_cast<const __nv_bfloat16*>(a->weight);
  p.bias = static_cast<const __nv_bfloat16*>(a->bias);
  p.y = static_cast<__nv_bfloat16*>(a->y);
  p.norm = static_cast<__nv_bfloat16*>(a->norm);
  p.rows = a->rows;
  p.dim = a->dim;
  p.mode = a->mode;
  p.eps = a->eps;
  p.pdl = 1;
  const int nvec = a->dim / 8;
  static const bool reg = env_flag("WAMFFN_NORM_REG", true);
  if (reg && nvec % 32 == 0 && nvec <= kRowThreads) {
    // Register-resident variant (same bits as modnorm_kernel, 4 warps per row).
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(a->rows), 1, 1);
    cfg.blockDim = dim3(kNormRegThreads, 1, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, modnorm_reg_kernel, p));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return WAMFFN_OK;
  }
  return launch_norm(p, a->rows, static_cast<cudaStream_t>(stream), pdl_enabled());
}

int wamffn_block_plan_create(int device, int max_rows, int max_seq, int d_model, int d_hidden,
                             int tune, wamffn_block_plan** out_plan) {
  if (!out_plan) return fail(WAMFFN_ERR_INVALID, "plan output pointer is null");
  *out_plan = nullptr;
  if (max_rows < 1 || max_rows > kMaxTokens || max_seq < 1)
    return fail(WAMFFN_ERR_UNSUPPORTED, "max_rows=%d max_seq=%d unsupported", max_rows, max_seq);
  GemmConfig probe;
  int rc = make_gemm_config(max_rows, d_hidden, d_model, 1, &probe);
  if (rc) return rc;
  rc = make_gemm_config(max_rows, d_model, d_hidden, 1, &probe);
  if (rc) return rc;
  int sm = 0;
  rc = prepare_device(device, &sm);
  if (rc) return rc;
  DeviceGuard guard(device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", device);
  auto* plan = new wamffn_block_plan();
  plan->device = device;
  plan->sm_count = sm;
  plan->max_rows = max_rows;
  plan->max_seq = max_seq;
  plan->d = d_model;
  plan->h = d_hidden;
  plan->tune = tune;
  memset(plan->split_override, 0, sizeof(plan->split_override));
  plan->max_splits = 16;
  auto cleanup = [&](int code) {
    wamffn_block_plan_destroy(plan);
    return code;
  };
  bool ok = cudaMalloc(&plan->gathered, size_t(max_rows) * d_model * 2) == cudaSuccess &&
            cudaMalloc(&plan->hidden, size_t(max_rows) * d_hidden * 2) == cudaSuccess &&
            cudaMalloc(&plan->y, size_t(max_seq) * d_model * 2) == cudaSuccess &&
            cudaMalloc(&plan->partial, size_t(plan->max_splits) * max_rows * d_model * 4) == cudaSuccess &&
            cudaMalloc(&plan->pos, size_t(max_seq) * sizeof(int)) == cudaSuccess &&
            cudaMalloc(&plan->status, sizeof(unsigned int)) == cudaSuccess &&
            cudaMemset(plan->status, 0, sizeof(unsigned int)) == cudaSuccess &&
            cudaMalloc(&plan->pass_bars, (3 * kPassMaxLayers + 1) * sizeof(unsigned int)) == cudaSuccess;
  if (!ok) return cleanup(fail(WAMFFN_ERR_CUDA, "block plan allocation failed"));
  plan->up_streamk = streamk_enabled() ? 1 : 0;
  {
    // Stream-K helper slots for the largest up projection this plan runs.
    GemmConfig c;
    make_gemm_config(max_rows, d_hidden, d_model, 1, &c);
    ok = cudaMalloc(&plan->sk_ws, streamk_ws_bytes(sm, c.tok_pad)) == cudaSuccess &&
         cudaMalloc(&plan->sk_flags, size_t(sm) * sizeof(unsigned int)) == cudaSuccess &&
         cudaMemset(plan->sk_flags, 0, size_t(sm) * sizeof(unsigned int)) == cudaSuccess;
    if (!ok) return cleanup(fail(WAMFFN_ERR_CUDA, "stream-K workspace allocation failed"));
  }
  {
    // The pass kernel's grid barriers need every CTA resident at once: one CTA
    // per SM, in clusters of two.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(sm & ~1), 1, 1);
    cfg.blockDim = dim3(kPassThreads, 1, 1);
    cfg.dynamicSmemBytes = 200 * 1024;  // one CTA per SM, like every real pass launch
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, stack_pass_kernel, &cfg) == cudaSuccess)
      plan->pass_ctas = 2 * clusters < (sm & ~1) ? 2 * clusters : (sm & ~1);
    else
      cudaGetLastError();
  }
  *out_plan = plan;
  return WAMFFN_OK;
}

int wamffn_block_plan_destroy(wamffn_block_plan* plan) {
  if (!plan) return WAMFFN_OK;
  DeviceGuard guard(plan->device);
  cudaFree(plan->gathered);
  cudaFree(plan->hidden);
  cudaFree(plan->y);
  cudaFree(plan->partial);
  cudaFree(plan->pos);
  cudaFree(plan->status);
  cudaFree(plan->pass_bars);
  cudaFree(plan->sk_ws);
  cudaFree(plan->sk_flags);
  delete plan;
  return WAMFFN_OK;
}

namespace {
int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

int block_configs(const wamffn_block_plan* plan, int rows, GemmConfig* up, GemmConfig* down) {
  // The up projection applies GELU in its epilogue: it never splits K; when
  // its feature tiles leave SMs idle it runs as stream-K (on every SM).
  int rc = make_gemm_config(rows, plan->h, plan->d, 1, up);
  if (rc) return rc;
  up->sk = plan->up_streamk ? streamk_groups(*up, plan->sm_count) : 0;
  // Down projection: K = h is long and the output narrow, so the SMs are filled
  // with split-K (optionally x token groups).
  // Token groups (grid.z) halve the partials but made the mainloop HBM-bound
  // (the groups re-stream each weight tile): one group unless overridden.
  static const int groups_env = env_int("WAMFFN_DOWN_GROUPS", 0);
  int groups = groups_env > 0 ? groups_env : 1;
  const int tiles = plan->d / kFeatTile;
  int s = plan->split_override[rows];
  if (s <= 0) {
    s = 1;
    for (int c = 2; c <= 16; ++c) {
      if (tiles * c * groups > plan->sm_count || (plan->h / kBlockK) / c < 8) break;
      s = c;
    }
  }
  if (s > plan->max_splits) s = plan->max_splits;
  return make_gemm_config(rows, plan->d, plan->h, s, down, groups);
}
}  // namespace

int wamffn_block_run(wamffn_block_plan* plan, void* stream_, const wamffn_block_args* a) {
  if (!plan || !a) return fail(WAMFFN_ERR_INVALID, "null argument");
  if (a->rows < 1 || a->rows > plan->max_rows)
    return fail(WAMFFN_ERR_INVALID, "rows=%d outside [1, %d]", a->rows, plan->max_rows);
  if (a->seq < 1 || a->seq > plan->max_seq)
    return fail(WAMFFN_ERR_INVALID, "seq=%d outside [1, %d]", a->seq, plan->max_seq);
  if (!a->indices && a->rows != a->seq)
    return fail(WAMFFN_ERR_INVALID, "without indices rows (%d) must equal seq (%d)", a->rows, a->seq);
  if (a->indices && a->index_bytes != 4 && a->index_bytes != 8)
    return fail(WAMFFN_ERR_INVALID, "index_bytes must be 4 or 8");
  if (a->cache_rows < 0 || a->cache_rows > a->seq)
    return fail(WAMFFN_ERR_INVALID, "cache_rows=%d outside [0, seq]", a->cache_rows);
  if (a->cache_rows > 0 && a->indices && !a->cache_in)
    return fail(WAMFFN_ERR_INVALID, "a gathered block with cache rows needs cache_in");
  if (!a->x || !a->mod || !a->time || !a->w_up || !a->b_up || !a->w_down || !a->b_down)
    return fail(WAMFFN_ERR_INVALID, "null tensor pointer");
  if (a->normalized && a->update)
    return fail(WAMFFN_ERR_INVALID, "a pre-normalised input takes no update (it is already folded in)");
  if (a->time_stride % 8) return fail(WAMFFN_ERR_INVALID, "time_stride must be a multiple of 8");
  const void* ptrs[] = {a->x, a->update, a->normalized, a->mod, a->time, a->w_up, a->b_up, a->w_down,
                        a->b_down, a->cache_in, a->cache_out, a->y, a->output, a->x_out};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return fail(WAMFFN_ERR_INVALID, "tensors must be 16-byte aligned");
  DeviceGuard guard(plan->device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", plan->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const bool pdl = pdl_enabled();
  GemmConfig up, down;
  int rc = block_configs(plan, a->rows, &up, &down);
  if (rc) return rc;

  // With a pre-normalised input the residual is the caller's x itself.
  const __nv_bfloat16* y =
      a->normalized ? static_cast<const __nv_bfloat16*>(a->x)
                    : static_cast<const __nv_bfloat16*>(a->y ? a->y : plan->y);
  // 1. CROSS_RESIDUAL norm (or plain copy) + gather into the activation operand.
  NormParams n{};
  n.gather_only = a->normalized ? 1 : 0;
  n.x = static_cast<const __nv_bfloat16*>(a->normalized ? a->normalized : a->x);
  n.xs = plan->d;
  n.update = static_cast<const __nv_bfloat16*>(a->update);
  n.us = plan->d;
  n.mod = static_cast<const __nv_bfloat16*>(a->mod);
  n.time = static_cast<const __nv_bfloat16*>(a->time);
  n.ts = a->time_stride;
  n.y = a->normalized ? nullptr : const_cast<__nv_bfloat16*>(y);
  n.norm = nullptr;
  n.rows = a->seq;
  n.dim = plan->d;
  n.mode = WAMFFN_CROSS_RESIDUAL;
  n.eps = a->eps;
  n.idx = a->indices;
  n.idx_bytes = a->index_bytes;
  n.m = a->rows;
  n.gathered = plan->gathered;
  n.pos_of_row = plan->pos;
  n.status = plan->status;
  n.pdl = 1;
  rc = launch_norm(n, a->seq > a->rows ? a->seq : a->rows, stream, pdl);
  if (rc) return rc;
  // 2. up projection + bias + GELU -> hidden.
  rc = launch_gemm(up, EPI_GELU_BF16, stream, a->w_up, a->weights_packed != 0, plan->gathered, a->b_up,
                   plan->hidden, plan->status, pdl, plan->sk_ws, plan->sk_flags);
  if (rc) return rc;
  // 3. down projection, split-K fp32 partials.
  rc = launch_gemm(down, EPI_PARTIAL_F32, stream, a->w_down, a->weights_packed != 0, plan->hidden, nullptr,
                   plan->partial, plan->status, pdl);
  if (rc) return rc;
  // 4. reduce + bias, scatter into the cache, gated residual.
  EpiParams e{};
  e.partial = plan->partial;
  e.splits = down.splits;
  e.m = a->rows;
  e.dim = plan->d;
  e.bias = static_cast<const __nv_bfloat16*>(a->b_down);
  e.pos_of_row = plan->pos;
  e.seq = a->seq;
  e.cache_rows = a->cache_rows;
  e.cache_in = static_cast<const __nv_bfloat16*>(a->cache_in);
  e.cache_out = static_cast<__nv_bfloat16*>(a->cache_out);
  e.output = static_cast<__nv_bfloat16*>(a->output);
  e.y = y;
  e.mod = static_cast<const __nv_bfloat16*>(a->mod);
  e.time = static_cast<const __nv_bfloat16*>(a->time);
  e.ts = a->time_stride;
  e.x_out = static_cast<__nv_bfloat16*>(a->x_out);
  e.status = plan->status;
  e.pdl = 1;
  return launch_epi(e, stream, pdl);
}

}  // extern "C"

namespace {

// Split-K of the pass kernel's down projection: the three-kernel stack's
// choice (fill the SMs with tiles x splits, at least 8 K blocks per split),
// capped by the CTA pairs.
int pass_down_splits(const wamffn_block_plan* plan) {
  const int d = plan->d, h = plan->h;
  int splits = 1;
  for (int s = 2; s <= plan->max_splits; ++s) {
    if ((d / kFeatTile) * s > plan->sm_count || (d / 256) * s > plan->pass_ctas / 2 || (h / kBlockK) / s < 8) break;
    splits = s;
  }
  return splits;
}

// The persistent pass kernel (opt-in, WAMFFN_PASS=1) covers the stack when
// every layer's up items fit one per CTA pair (its GELU epilogue borrows the
// idle activation ring) and the geometry is the pair kernel's.  It computes
// the same bits as the three-kernel stack; on B200 it measured about 5 %
// slower per 30-layer pass (its row phase runs on a third of the threads the
// layer-boundary kernel gets), so the three-kernel stack is the default.
bool pass_usable(const wamffn_block_plan* plan, const wamffn_stack_args* a, bool gather) {
  static const bool on = env_flag("WAMFFN_PASS", false);
  if (!on || plan->pass_ctas < 2 || a->layers > kPassMaxLayers) return false;
  if (plan->d > kPassEpiThreads * 8 || plan->d % 256 || plan->h % 256) return false;
  if (!pair_enabled()) return false;
  const int npairs = plan->pass_ctas / 2;
  if (plan->h / 256 > npairs) return false;
  const int row_limit = a->seq > a->rows ? a->seq : a->rows;
  if (row_limit > kPassRowSlots * plan->pass_ctas) return false;
  return true;
}

int pass_class_config(int rows, const wamffn_block_plan* plan, PassClass* c) {
  GemmConfig g;
  int rc = make_gemm_config(rows, plan->h, plan->d, 1, &g);
  if (rc) return rc;
  if (g.group != 2) return fail(WAMFFN_ERR_UNSUPPORTED, "the pass kernel runs 2-SM UMMA pairs only");
  c->rows = rows;
  c->tok_pad = g.tok_pad;
  c->mma_n0 = g.mma_n0;
  c->mma_n1 = g.mma_n1;
  c->tok_box = g.tok_box;
  c->n_boxes = g.n_boxes;
  c->b_rows = g.b_rows;
  return WAMFFN_OK;
}

int launch_pass(wamffn_block_plan* plan, const wamffn_stack_args* a, bool gather, cudaStream_t stream) {
  static PassParams p;  // ~14 KB: kept off the host stack; guarded by the mutex below
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  memset(&p, 0, sizeof(p));
  const int d = plan->d, h = plan->h, L = a->layers;
  p.layers = L;
  p.d = d;
  p.h = h;
  p.seq = a->seq;
  p.first_gathered = gather ? a->first_gathered_layer : L;
  p.w_packed = a->weights_packed != 0;
  int rc = pass_class_config(a->seq, plan, &p.cls[0]);
  if (rc) return rc;
  rc = pass_class_config(gather ? a->rows : a->seq, plan, &p.cls[1]);
  if (rc) return rc;
  p.up_tiles = h / 256;
  p.down_tiles = d / 256;
  const int splits = pass_down_splits(plan);
  p.down_splits = splits;
  // Shared memory: the same ring split as the GEMM kernel; the activation
  // ring also hosts the 24 KB of GELU transpose tiles.
  const int budget = kSmemLimit - kSmemReserve;
  const int b_rows = p.cls[0].b_rows > p.cls[1].b_rows ? p.cls[0].b_rows : p.cls[1].b_rows;
  p.b_stage_bytes = b_rows * kBlockK * 2;
  p.b_stages = (budget / 2) / p.b_stage_bytes;
  if (p.b_stages > kMaxBStages) p.b_stages = kMaxBStages;
  if (p.b_stages < 2) p.b_stages = 2;
  p.b_region_bytes = p.b_stages * p.b_stage_bytes;
  if (p.b_region_bytes < kPassTransposeBytes) p.b_region_bytes = kPassTransposeBytes;
  p.a_stages = (budget - p.b_region_bytes) / gemm_a_bytes();
  if (p.a_stages > kMaxAStages) p.a_stages = kMaxAStages;
  if (p.a_stages < 2) return fail(WAMFFN_ERR_UNSUPPORTED, "pass kernel: fewer than 2 weight stages");
  const size_t smem = 1024 + size_t(p.a_stages) * gemm_a_bytes() + size_t(p.b_region_bytes);
  if (smem + 1024 > size_t(kSmemLimit)) return fail(WAMFFN_ERR_UNSUPPORTED, "pass kernel: %zu bytes of shared memory", smem);
  for (int l = 0; l < L; ++l) {
    const wamffn_layer_weights& w = a->weights[l];
    rc = p.w_packed ? encode_operand(&p.tm_w_up[l], w.w_up, kBlockK, uint64_t(h) * (d / kBlockK), kBlockK * 2, kFeatTile)
                    : encode_operand(&p.tm_w_up[l], w.w_up, d, h, uint64_t(d) * 2, kFeatTile);
    if (rc) return rc;
    rc = p.w_packed ? encode_operand(&p.tm_w_down[l], w.w_down, kBlockK, uint64_t(d) * (h / kBlockK), kBlockK * 2,
                                     kFeatTile)
                    : encode_operand(&p.tm_w_down[l], w.w_down, h, d, uint64_t(h) * 2, kFeatTile);
    if (rc) return rc;
    p.b_up[l] = static_cast<const __nv_bfloat16*>(w.b_up);
    p.b_down[l] = static_cast<const __nv_bfloat16*>(w.b_down);
    p.mod[l] = static_cast<const __nv_bfloat16*>(w.mod);
  }
  for (int c = 0; c < 2; ++c) {
    rc = encode_operand(&p.tm_act[c], plan->gathered, d, p.cls[c].rows, uint64_t(d) * 2, uint32_t(p.cls[c].tok_box));
    if (rc) return rc;
    rc = encode_operand(&p.tm_hid[c], plan->hidden, h, p.cls[c].rows, uint64_t(h) * 2, uint32_t(p.cls[c].tok_box));
    if (rc) return rc;
  }
  p.x = static_cast<const __nv_bfloat16*>(a->x);
  p.time = static_cast<const __nv_bfloat16*>(a->time);
  p.ts = a->time_stride;
  p.y = plan->y;
  p.gathered = plan->gathered;
  p.hidden = plan->hidden;
  p.partial = plan->partial;
  p.idx = gather ? a->indices : nullptr;
  p.idx_bytes = a->index_bytes;
  p.cache_rows = gather ? a->cache_rows : 0;
  p.cache_in = static_cast<const __nv_bfloat16*>(a->cache_in);
  p.cache_out = static_cast<__nv_bfloat16*>(a->cache_out);
  p.x_out = static_cast<__nv_bfloat16*>(a->x_out);
  p.eps = a->eps;
  p.bars = plan->pass_bars;
  p.status = plan->status;
  WAMFFN_CUDA(cudaMemsetAsync(plan->pass_bars, 0, (3 * L + 1) * sizeof(unsigned int), stream));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(plan->pass_ctas), 1, 1);
  cfg.blockDim = dim3(kPassThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, stack_pass_kernel, p));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Shared body of wamffn_stack_run and wamffn_stack_run_tp (allreduce != null).
int stack_run_impl(wamffn_block_plan* plan, void* stream_, const wamffn_stack_args* a, float* reduce_buffer,
                   wamffn_allreduce_fn allreduce, void* user) {
  if (!plan || !a || !a->weights) return fail(WAMFFN_ERR_INVALID, "null argument");
  if (a->layers < 1) return fail(WAMFFN_ERR_INVALID, "layers=%d", a->layers);
  if (a->seq < 1 || a->seq > plan->max_seq || a->seq > plan->max_rows)
    return fail(WAMFFN_ERR_INVALID, "seq=%d outside [1, %d]", a->seq, plan->max_seq < plan->max_rows ? plan->max_seq : plan->max_rows);
  const bool gather = a->indices != nullptr && a->first_gathered_layer < a->layers;
  if (gather && (a->rows < 1 || a->rows > plan->max_rows))
    return fail(WAMFFN_ERR_INVALID, "rows=%d outside [1, %d]", a->rows, plan->max_rows);
  if (gather && a->index_bytes != 4 && a->index_bytes != 8)
    return fail(WAMFFN_ERR_INVALID, "index_bytes must be 4 or 8");
  if (a->first_gathered_layer < 0) return fail(WAMFFN_ERR_INVALID, "first_gathered_layer < 0");
  if (a->cache_rows < 0 || a->cache_rows > a->seq)
    return fail(WAMFFN_ERR_INVALID, "cache_rows=%d outside [0, seq]", a->cache_rows);
  if (gather && a->cache_rows > 0 && !a->cache_in)
    return fail(WAMFFN_ERR_INVALID, "gathered layers with cache rows need cache_in");
  if (!a->x || !a->time || !a->x_out) return fail(WAMFFN_ERR_INVALID, "null tensor pointer");
  if (a->time_stride % 8) return fail(WAMFFN_ERR_INVALID, "time_stride must be a multiple of 8");
  for (int l = 0; l < a->layers; ++l) {
    const wamffn_layer_weights& w = a->weights[l];
    const void* ptrs[] = {w.w_up, w.b_up, w.w_down, w.b_down, w.mod};
    for (const void* q : ptrs)
      if (!q || !aligned16(q)) return fail(WAMFFN_ERR_INVALID, "layer %d: null or unaligned weight", l);
  }
  const void* ptrs[] = {a->x, a->time, a->cache_in, a->cache_out, a->x_out};
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return fail(WAMFFN_ERR_INVALID, "tensors must be 16-byte aligned");
  DeviceGuard guard(plan->device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", plan->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const bool pdl = pdl_enabled();
  const int d = plan->d;
  const size_t layer_cache = size_t(a->cache_rows) * d;
  auto gathered_layer = [&](int l) { return gather && l >= a->first_gathered_layer; };
  auto layer_rows = [&](int l) { return gathered_layer(l) ? a->rows : a->seq; };

  const bool tp = allreduce != nullptr;
  if (tp && (!reduce_buffer || !aligned16(reduce_buffer)))
    return fail(WAMFFN_ERR_INVALID, "the tensor-parallel stack needs a 16-byte aligned reduce buffer");
  if (!tp && pass_usable(plan, a, gather)) return launch_pass(plan, a, gather, stream);

  // Prologue of the first layer: y = x, norm + gather into the activation buffer.
  NormParams n{};
  n.x = static_cast<const __nv_bfloat16*>(a->x);
  n.xs = d;
  n.mod = static_cast<const __nv_bfloat16*>(a->weights[0].mod);
  n.time = static_cast<const __nv_bfloat16*>(a->time);
  n.ts = a->time_stride;
  n.y = plan->y;
  n.rows = a->seq;
  n.dim = d;
  n.mode = WAMFFN_CROSS_RESIDUAL;
  n.eps = a->eps;
  n.idx = gathered_layer(0) ? a->indices : nullptr;
  n.idx_bytes = a->index_bytes;
  n.m = layer_rows(0);
  n.gathered = plan->gathered;
  n.pos_of_row = plan->pos;
  n.status = plan->status;
  n.pdl = 1;
  int rc = launch_norm(n, a->seq > n.m ? a->seq : n.m, stream, pdl);
  if (rc) return rc;
  for (int l = 0; l < a->layers; ++l) {
    const wamffn_layer_weights& w = a->weights[l];
    const int rows = layer_rows(l);
    GemmConfig up, down;
    rc = block_configs(plan, rows, &up, &down);
    if (rc) return rc;
    rc = launch_gemm(up, EPI_GELU_BF16, stream, w.w_up, a->weights_packed != 0, plan->gathered, w.b_up, plan->hidden,
                     plan->status, pdl, plan->sk_ws, plan->sk_flags);
    if (rc) return rc;
    // Unsplit K (concurrent lanes): the GEMM applies the bias and rounds to
    // bf16 itself, the boundary reads half the bytes.  Same values either way.
    const bool direct = !tp && down.splits == 1;
    rc = launch_gemm(down, direct ? EPI_BIAS_BF16 : EPI_PARTIAL_F32, stream, w.w_down, a->weights_packed != 0,
                     plan->hidden, direct ? w.b_down : nullptr, plan->partial, plan->status, pdl);
    if (rc) return rc;
    BoundaryParams b{};
    b.partial = plan->partial;
    b.splits = down.splits;
    b.out_bf16 = direct ? 1 : 0;
    if (tp) {
      // This rank's share of the down projection, summed over its splits,
      // then over the ranks; the boundary reads the one reduced sum.
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(unsigned(rows), 1, 1);
      cfg.blockDim = dim3(unsigned(row_threads(d)), 1, 1);
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, split_sum_kernel, static_cast<const float*>(plan->partial), down.splits,
                                     rows, d, reduce_buffer));
      g_launches.fetch_add(1, std::memory_order_relaxed);
      const int arc = allreduce(user, reduce_buffer, int64_t(rows) * d, stream_);
      if (arc) return fail(arc, "allreduce callback failed at layer %d (status %d)", l, arc);
      b.partial = reduce_buffer;
      b.splits = 1;
    }
    b.m = rows;
    b.dim = d;
    b.seq = a->seq;
    b.bias = static_cast<const __nv_bfloat16*>(w.b_down);
    b.idx = gathered_layer(l) ? a->indices : nullptr;
    b.idx_bytes = a->index_bytes;
    if (gathered_layer(l)) {
      const size_t slot = size_t(l - a->first_gathered_layer) * layer_cache;
      b.cache_rows = a->cache_rows;
      b.cache_in = a->cache_in ? static_cast<const __nv_bfloat16*>(a->cache_in) + slot : nullptr;
      b.cache_out = a->cache_out ? static_cast<__nv_bfloat16*>(a->cache_out) + slot : nullptr;
    }
    b.y = plan->y;
    b.mod = static_cast<const __nv_bfloat16*>(w.mod);
    b.time = static_cast<const __nv_bfloat16*>(a->time);
    b.ts = a->time_stride;
    const bool last = l + 1 == a->layers;
    b.next_mod = last ? nullptr : static_cast<const __nv_bfloat16*>(a->weights[l + 1].mod);
    b.next_idx = (!last && gathered_layer(l + 1)) ? a->indices : nullptr;
    b.next_idx_bytes = a->index_bytes;
    b.next_m = last ? 0 : layer_rows(l + 1);
    b.next_gathered = plan->gathered;
    b.x_final = static_cast<__nv_bfloat16*>(a->x_out);
    b.eps = a->eps;
    b.status = plan->status;
    cudaLaunchConfig_t cfg{};
    const int grid = a->seq > b.next_m ? a->seq : b.next_m;
    cfg.gridDim = dim3(unsigned(grid), 1, 1);
    cfg.blockDim = dim3(unsigned(row_threads(d)), 1, 1);
    cfg.dynamicSmemBytes = size_t(d) * sizeof(float);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (b.out_bf16) WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, boundary_kernel<true>, b));
    else WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, boundary_kernel<false>, b));
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  return WAMFFN_OK;
}

}  // namespace

extern "C" {

int wamffn_stack_run(wamffn_block_plan* plan, void* stream, const wamffn_stack_args* a) {
  return stack_run_impl(plan, stream, a, nullptr, nullptr, nullptr);
}

int wamffn_stack_run_tp(wamffn_block_plan* plan, void* stream, const wamffn_stack_args* a, float* reduce_buffer,
                        wamffn_allreduce_fn allreduce, void* user) {
  if (!allreduce) return fail(WAMFFN_ERR_INVALID, "allreduce callback is null");
  return stack_run_impl(plan, stream, a, reduce_buffer, allreduce, user);
}

int wamffn_block_status(wamffn_block_plan* plan, uint32_t* status, int clear) {
  if (!plan || !status) return fail(WAMFFN_ERR_INVALID, "null argument");
  DeviceGuard guard(plan->device);
  WAMFFN_CUDA(cudaDeviceSynchronize());
  WAMFFN_CUDA(cudaMemcpy(status, plan->status, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  if (clear) WAMFFN_CUDA(cudaMemset(plan->status, 0, sizeof(uint32_t)));
  return WAMFFN_OK;
}

int wamffn_block_plan_set_splits(wamffn_block_plan* plan, int rows, int splits) {
  if (!plan) return fail(WAMFFN_ERR_INVALID, "null plan");
  if (rows < 0 || rows > plan->max_rows)
    return fail(WAMFFN_ERR_INVALID, "rows=%d outside [0, %d]", rows, plan->max_rows);
  if (splits < 0 || splits > plan->max_splits || splits > plan->h / kBlockK)
    return fail(WAMFFN_ERR_INVALID, "splits=%d outside [0, %d]", splits,
                plan->max_splits < plan->h / kBlockK ? plan->max_splits : plan->h / kBlockK);
  if (rows > 0) {
    plan->split_override[rows] = splits;
  } else {
    for (int r = 1; r <= plan->max_rows; ++r) plan->split_override[r] = splits;
  }
  return WAMFFN_OK;
}

int wamffn_block_configuration(const wamffn_block_plan* plan, int rows, uint32_t* values, int n) {
  if (!plan || !values) return fail(WAMFFN_ERR_INVALID, "null argument");
  GemmConfig up, down;
  int rc = block_configs(plan, rows, &up, &down);
  if (rc) return rc;
  const GemmConfig* cs[2] = {&up, &down};
  int k = 0;
  for (const GemmConfig* c : cs) {
    const uint32_t v[7] = {uint32_t(kFeatTile * c->group), uint32_t(c->tok_pad), uint32_t(c->mma_n1 > 0 ? 2 : 1),
                           uint32_t(c->a_stages * 100 + c->b_stages), uint32_t(c->splits), c->tmem_cols, 0u};
    for (int i = 0; i < 7 && k < n; ++i) values[k++] = v[i];
  }
  // Values 14 and 15: stream-K CTA groups of the up and down projections (0 = data-parallel grid).
  for (const GemmConfig* c : cs)
    if (k < n) values[k++] = uint32_t(c->sk);
  return WAMFFN_OK;
}

int wamffn_block_plan_set_streamk(wamffn_block_plan* plan, int enabled) {
  if (!plan) return fail(WAMFFN_ERR_INVALID, "null plan");
  plan->up_streamk = enabled ? 1 : 0;
  return WAMFFN_OK;
}

int wamffn_trace_enable(int device, void* buffer, int records) {
  DeviceGuard guard(device);
  if (!guard.ok) return fail(WAMFFN_ERR_CUDA, "cannot select device %d", device);
  if (buffer && (records < 2 || !aligned16(buffer))) return fail(WAMFFN_ERR_INVALID, "trace buffer too small");
  unsigned long long* ptr = static_cast<unsigned long long*>(buffer);
  unsigned int cap = buffer ? unsigned(records) : 0u;
  WAMFFN_CUDA(cudaMemcpyToSymbol(g_trace, &ptr, sizeof(ptr)));
  WAMFFN_CUDA(cudaMemcpyToSymbol(g_trace_capacity, &cap, sizeof(cap)));
  return WAMFFN_OK;
}

int wamffn_pack_weight(void* stream, const void* src, void* dst, int n_out, int k_in) {
  if (!src || !dst) return fail(WAMFFN_ERR_INVALID, "null tensor pointer");
  if (n_out < kFeatTile || n_out % kFeatTile || k_in < kBlockK || k_in % kBlockK)
    return fail(WAMFFN_ERR_INVALID, "pack needs n_out %% 128 == 0 and k_in %% 64 == 0 (got %d, %d)", n_out, k_in);
  if (!aligned16(src) || !aligned16(dst)) return fail(WAMFFN_ERR_INVALID, "tensors must be 16-byte aligned");
  if (src == dst) return fail(WAMFFN_ERR_INVALID, "pack cannot run in place");
  const long long vectors = (long long)n_out * k_in / 8;
  int blocks = int((vectors + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  pack_weight_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n_out, k_in);
  WAMFFN_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

int wamffn_select_tokens(void* stream, const wamffn_select_args* a) {
  if (!a) return fail(WAMFFN_ERR_INVALID, "args is null");
  if (a->n < 1 || a->n > kSelectThreads) return fail(WAMFFN_ERR_UNSUPPORTED, "n=%d outside [1, %d]", a->n, kSelectThreads);
  if (a->count < 1 || a->count >= a->n) return fail(WAMFFN_ERR_INVALID, "count=%d must be in [1, n)", a->count);
  if (a->seq < a->n) return fail(WAMFFN_ERR_INVALID, "seq=%d < n=%d", a->seq, a->n);
  if (a->dim < 8 || a->dim % 8) return fail(WAMFFN_ERR_INVALID, "dim=%d must be a multiple of 8", a->dim);
  if (!a->now || !a->before || !a->indices) return fail(WAMFFN_ERR_INVALID, "null tensor pointer");
  if (!aligned16(a->now) || !aligned16(a->before) || (a->features_out && !aligned16(a->features_out)) ||
      a->now_stride % 8)
    return fail(WAMFFN_ERR_INVALID, "rows must be 16-byte aligned");
  SelectParams p{};
  p.now = static_cast<const __nv_bfloat16*>(a->now);
  p.now_stride = a->now_stride;
  p.before = static_cast<const __nv_bfloat16*>(a->before);
  p.mandatory = static_cast<const unsigned char*>(a->mandatory);
  p.n = a->n;
  p.dim = a->dim;
  p.count = a->count;
  p.seq = a->seq;
  p.indices = static_cast<long long*>(a->indices);
  p.features_out = static_cast<__nv_bfloat16*>(a->features_out);
  p.pdl = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(kSelectThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, select_tokens_kernel, p));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

int wamffn_rgb_mandatory(void* stream, const void* now, const void* before, int height, int width, int grid_h,
                         int grid_w, void* mandatory) {
  if (!now || !before || !mandatory) return fail(WAMFFN_ERR_INVALID, "null pointer");
  if (height < 1 || width < 1 || grid_h < 1 || grid_w < 1)
    return fail(WAMFFN_ERR_INVALID, "sizes must be positive");
  if (height % grid_h || width % grid_w)
    return fail(WAMFFN_ERR_INVALID, "a %dx%d image does not split into %dx%d patches", height, width, grid_h, grid_w);
  const long long patch_values = (long long)(height / grid_h) * (width / grid_w) * 3;
  if (patch_values * 255 >= (1ll << 24))
    return fail(WAMFFN_ERR_UNSUPPORTED, "patches of %lld values exceed the exact float32 sum range", patch_values);
  if ((long long)grid_h * grid_w > 65535) return fail(WAMFFN_ERR_UNSUPPORTED, "more than 65535 patches");
  RgbParams p{};
  p.now = static_cast<const unsigned char*>(now);
  p.before = static_cast<const unsigned char*>(before);
  p.width = width;
  p.ph = height / grid_h;
  p.pw = width / grid_w;
  p.grid_w = grid_w;
  p.mandatory = static_cast<unsigned char*>(mandatory);
  rgb_mandatory_kernel<<<grid_h * grid_w, kRgbThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  WAMFFN_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

}  // extern "C"

namespace {

// One [batch, rows, heads*128] operand of the attention ops.
struct AttnRows {
  const void* data;
  int64_t row, batch;  // strides in elements
  int rows;
  const char* name;
};

int check_attn_rows(const AttnRows& v, int64_t width) {
  if (!v.data) return fail(WAMFFN_ERR_INVALID, "%s is null", v.name);
  if (!aligned16(v.data)) return fail(WAMFFN_ERR_INVALID, "%s must be 16-byte aligned", v.name);
  // Rows of every batch at one stride (2-D tensor maps over batch x rows).
  if (v.row < width || v.row % 8 || v.batch != v.row * v.rows)
    return fail(WAMFFN_ERR_INVALID,
                "%s strides (%lld, %lld): rows must sit at one stride across batches, >= heads*128, a multiple "
                "of 8 elements",
                v.name, (long long)v.batch, (long long)v.row);
  return WAMFFN_OK;
}

// Tensor map of an operand (no map for an empty one: the kernel never reads it).
int encode_attn_rows(CUtensorMap* map, const AttnRows& v, int64_t width, int batch) {
  if (v.rows == 0) return WAMFFN_OK;
  return encode_operand(map, v.data, uint64_t(width), uint64_t(batch) * v.rows, uint64_t(v.row) * 2, kAttnRows);
}

int check_attn_shape(int head_dim, int key_split, int batch, int heads) {
  if (head_dim != kAttnHeadDim)
    return fail(WAMFFN_ERR_UNSUPPORTED, "head_dim=%d: the kernel runs D = %d", head_dim, kAttnHeadDim);
  if (key_split != 0 && key_split != 1 && key_split != 2 && key_split != 4)
    return fail(WAMFFN_ERR_INVALID, "key_split=%d: 0 (automatic), 1, 2 or 4", key_split);
  if (batch < 1 || heads < 1 || batch > 65535 || heads > 65535)
    return fail(WAMFFN_ERR_INVALID, "batch=%d heads=%d", batch, heads);
  return WAMFFN_OK;
}

// Grid, key split and launch of masked_attention_kernel for segments already
// described in `p` (tiles filled in here).
int launch_attention(void* stream_, const AttnMaps& maps, AttnParams& p, int key_split) {
  int dev = 0, sm = 0;
  WAMFFN_CUDA(cudaGetDevice(&dev));
  int rc = prepare_device(dev, &sm);
  if (rc) return rc;
  int64_t tiles = 0;
  int max_blocks = 0;
  for (int s = 0; s < p.nqseg; ++s) {
    p.qseg[s].tiles = (p.qseg[s].rows + kAttnRows - 1) / kAttnRows;
    tiles += p.qseg[s].tiles;
    int blocks = 0, base = 0;
    for (int t = 0; t < p.nkseg; ++t) {
      const int vis = std::max(0, std::min(p.qseg[s].visible - base, p.krows[t]));
      blocks += (vis + kAttnKeys - 1) / kAttnKeys;
      base += p.krows[t];
    }
    if (p.qseg[s].rows > 0) max_blocks = std::max(max_blocks, blocks);
  }
  if (tiles == 0) return WAMFFN_OK;
  // Key split: the largest of 1, 2, 4 that keeps the grid within one wave
  // (one CTA per SM), or the caller's; halved while it exceeds the key blocks
  // of the longest query tile.
  const int64_t ctas = tiles * p.heads * p.batch;
  int split = 1;
  if (key_split) {
    split = key_split;
  } else {
    for (int s : {2, 4})
      if (ctas * s <= sm) split = s;
  }
  while (split > 1 && split > max_blocks) split >>= 1;
  if (tiles * split > 0x7fffffff) return fail(WAMFFN_ERR_INVALID, "too many query rows");
  p.split = split;
  p.scale_log2 = float((1.0 / sqrt(double(kAttnHeadDim))) * 1.4426950408889634);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(tiles * split), unsigned(p.heads), unsigned(p.batch));
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = kAttnSmem;
  cfg.stream = static_cast<cudaStream_t>(stream_);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: barrier set-up and TMEM allocation overlap
  // the previous kernel; the kernel waits for it before touching global memory.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  auto kernel = p.skip_masked ? (split > 1 ? masked_attention_kernel<true, true> : masked_attention_kernel<true, false>)
                              : (split > 1 ? masked_attention_kernel<false, true> : masked_attention_kernel<false, false>);
  WAMFFN_CUDA(cudaLaunchKernelEx(&cfg, kernel, maps, p));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return WAMFFN_OK;
}

}  // namespace

extern "C" {

int wamffn_masked_attention(void* stream_, const wamffn_attention_args* a) {
  if (!a) return fail(WAMFFN_ERR_INVALID, "args is null");
  int rc = check_attn_shape(a->head_dim, a->key_split, a->batch, a->heads);
  if (rc) return rc;
  if (a->nq < 1 || a->nk < 1) return fail(WAMFFN_ERR_INVALID, "nq=%d nk=%d", a->nq, a->nk);
  if (!a->out || !aligned16(a->out)) return fail(WAMFFN_ERR_INVALID, "out must be a 16-byte aligned pointer");
  const int64_t width = int64_t(a->heads) * kAttnHeadDim;
  const AttnRows views[3] = {{a->q, a->q_row_stride, a->q_batch_stride, a->nq, "q"},
                             {a->k, a->k_row_stride, a->k_batch_stride, a->nk, "k"},
                             {a->v, a->v_row_stride, a->v_batch_stride, a->nk, "v"}};
  for (const auto& v : views)
    if ((rc = check_attn_rows(v, width))) return rc;
  AttnMaps maps{};
  if ((rc = encode_attn_rows(&maps.q[0], views[0], width, a->batch))) return rc;
  if ((rc = encode_attn_rows(&maps.k[0], views[1], width, a->batch))) return rc;
  if ((rc = encode_attn_rows(&maps.v[0], views[2], width, a->batch))) return rc;
  AttnParams p{};
  p.mask = static_cast<const unsigned char*>(a->mask);
  p.mb = a->mask_strides[0];
  p.mh = a->mask_strides[1];
  p.mq = a->mask_strides[2];
  p.mk = a->mask_strides[3];
  // A mask shared by every head and query row lets fully masked key blocks be skipped.
  p.skip_masked = a->mask && p.mh == 0 && p.mq == 0 &&
                  (a->nk + kAttnKeys - 1) / kAttnKeys <= kAttnSkipWords * 32;
  p.qseg[0] = AttnQSeg{static_cast<__nv_bfloat16*>(a->out), int64_t(a->nq) * width, width, a->nq, a->nq, 0, 0, a->nk};
  p.nqseg = 1;
  p.krows[0] = a->nk;
  p.nkseg = 1;
  p.heads = a->heads;
  p.batch = a->batch;
  p.status = static_cast<unsigned int*>(a->status);
  return launch_attention(stream_, maps, p, a->key_split);
}

int wamffn_joint_first_frame_attention(void* stream_, const wamffn_joint_attention_args* a) {
  if (!a) return fail(WAMFFN_ERR_INVALID, "args is null");
  int rc = check_attn_shape(a->head_dim, a->key_split, a->batch, a->heads);
  if (rc) return rc;
  if (a->count < 1 || a->first < 0 || a->first > a->count)
    return fail(WAMFFN_ERR_INVALID, "count=%d first=%d: 0 <= first <= count, count >= 1", a->count, a->first);
  if (!a->out || !aligned16(a->out)) return fail(WAMFFN_ERR_INVALID, "out must be a 16-byte aligned pointer");
  const int64_t width = int64_t(a->heads) * kAttnHeadDim;
  const AttnRows views[3] = {{a->q.data, a->q.row_stride, a->q.batch_stride, a->count, "q"},
                             {a->k.data, a->k.row_stride, a->k.batch_stride, a->count, "k"},
                             {a->v.data, a->v.row_stride, a->v.batch_stride, a->count, "v"}};
  for (const auto& v : views)
    if ((rc = check_attn_rows(v, width))) return rc;
  AttnMaps maps{};
  if ((rc = encode_attn_rows(&maps.q[0], views[0], width, a->batch))) return rc;
  maps.q[1] = maps.q[0];
  if ((rc = encode_attn_rows(&maps.k[0], views[1], width, a->batch))) return rc;
  if ((rc = encode_attn_rows(&maps.v[0], views[2], width, a->batch))) return rc;
  AttnParams p{};
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a->out);
  // Clean first-frame rows see the first frame's keys; every other row sees all.
  p.qseg[0] = AttnQSeg{out, int64_t(a->count) * width, width, a->first, a->count, 0, 0, a->first};
  p.qseg[1] = AttnQSeg{out + int64_t(a->first) * width, int64_t(a->count) * width, width, a->count - a->first,
                       a->count, a->first, 0, a->count};
  p.nqseg = 2;
  p.krows[0] = a->count;
  p.nkseg = 1;
  p.heads = a->heads;
  p.batch = a->batch;
  p.status = static_cast<unsigned int*>(a->status);
  return launch_attention(stream_, maps, p, a->key_split);
}

int wamffn_current_frame_attention(void* stream_, const wamffn_current_frame_args* a) {
  if (!a) return fail(WAMFFN_ERR_INVALID, "args is null");
  int rc = check_attn_shape(a->head_dim, a->key_split, a->batch, a->heads);
  if (rc) return rc;
  if (a->nc < 0 || a->nv < 0 || a->na < 0 || a->nv + a->na < 1 || int64_t(a->nc) + a->nv + a->na > 0x7fffffff)
    return fail(WAMFFN_ERR_INVALID, "nc=%d nv=%d na=%d", a->nc, a->nv, a->na);
  const int64_t width = int64_t(a->heads) * kAttnHeadDim;
  const AttnRows qv{a->qv.data, a->qv.row_stride, a->qv.batch_stride, a->nv, "qv"};
  const AttnRows qa{a->qa.data, a->qa.row_stride, a->qa.batch_stride, a->na, "qa"};
  const AttnRows keys[3] = {{a->ck.data, a->ck.row_stride, a->ck.batch_stride, a->nc, "ck"},
                            {a->kv.data, a->kv.row_stride, a->kv.batch_stride, a->nv, "kv"},
                            {a->ka.data, a->ka.row_stride, a->ka.batch_stride, a->na, "ka"}};
  const AttnRows values[3] = {{a->cv.data, a->cv.row_stride, a->cv.batch_stride, a->nc, "cv"},
                              {a->vv.data, a->vv.row_stride, a->vv.batch_stride, a->nv, "vv"},
                              {a->va.data, a->va.row_stride, a->va.batch_stride, a->na, "va"}};
  const AttnRows all[8] = {qv, qa, keys[0], keys[1], keys[2], values[0], values[1], values[2]};
  for (const auto& v : all)
    if (v.rows > 0 && (rc = check_attn_rows(v, width))) return rc;
  if ((a->nv > 0 && (!a->ov || !aligned16(a->ov))) || (a->na > 0 && (!a->oa || !aligned16(a->oa))))
    return fail(WAMFFN_ERR_INVALID, "ov / oa must be 16-byte aligned pointers");
  AttnMaps maps{};
  if ((rc = encode_attn_rows(&maps.q[0], qv, width, a->batch))) return rc;
  if ((rc = encode_attn_rows(&maps.q[1], qa, width, a->batch))) return rc;
  for (int t = 0; t < 3; ++t) {
    if ((rc = encode_attn_rows(&maps.k[t], keys[t], width, a->batch))) return rc;
    if ((rc = encode_attn_rows(&maps.v[t], values[t], width, a->batch))) return rc;
  }
  AttnParams p{};
  const int total = a->nc + a->nv + a->na;
  p.qseg[0] = AttnQSeg{static_cast<__nv_bfloat16*>(a->ov), int64_t(a->nv) * width, width, a->nv, a->nv, 0, 0, total};
  p.qseg[1] = AttnQSeg{static_cast<__nv_bfloat16*>(a->oa), int64_t(a->na) * width, width, a->na, a->na, 0, 0, total};
  p.nqseg = 2;
  p.krows[0] = a->nc;
  p.krows[1] = a->nv;
  p.krows[2] = a->na;
  p.nkseg = 3;
  p.heads = a->heads;
  p.batch = a->batch;
  p.status = static_cast<unsigned int*>(a->status);
  return launch_attention(stream_, maps, p, a->key_split);
}

}  // extern "C"
