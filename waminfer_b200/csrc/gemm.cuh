// Weight-streaming tcgen05 GEMM for the small-row FFN of the WAMInfer video DiT.
//
// out[t, f] = epilogue( sum_k act[t, k] * weight[f, k] )
//
// The problem is "swap-AB": the weight rows (output features) sit on the UMMA
// M axis (128 per CTA) and the few hundred activation rows (tokens) sit on the
// UMMA N axis, so one CTA holds every token of its 128 features in TMEM
// (<= 512 fp32 columns) and each weight tile is read from HBM exactly once.
// Operands are staged by TMA with the 128-byte swizzle, K-major on both sides
// (torch.nn.Linear's native [out, in] weight layout and row-major activations).
//
// Roles (320 threads):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + UMMA issuer (one elected lane)
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4).., columns split
//               between the two warpgroups
// Grid: (n_total / 128, split_k).  With split_k > 1 each CTA covers a
// contiguous range of K blocks and writes an fp32 partial; a row kernel sums
// the partials in split order (deterministic, no atomics).
#pragma once

#include "ptx.cuh"

namespace wamffn {

enum : int { EPI_GELU_BF16 = 0, EPI_BIAS_BF16 = 1, EPI_PARTIAL_F32 = 2 };

constexpr int kFeatTile = 128;         // UMMA M
constexpr int kBlockK = 64;            // bf16 elements per 128-byte swizzled row
constexpr int kGemmThreads = 320;
constexpr int kMaxTokens = 512;        // TMEM holds 512 fp32 columns
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;     // 227 KB opt-in dynamic shared memory
constexpr int kSmemReserve = 1024 + 256;  // alignment slack + barriers

struct GemmParams {
  int tokens;        // real activation rows
  int tok_pad;       // tokens rounded up to 16
  int mma_n0;        // N of the first UMMA (<= 256, multiple of 16)
  int mma_n1;        // N of the second UMMA (0 when one suffices)
  int tok_box;       // activation rows per TMA box
  int n_boxes;       // TMA boxes per stage for the activation tile
  int k_blocks;      // K / 64
  int splits;        // split-K factor == gridDim.y
  int stages;        // pipeline depth
  int n_total;       // output features (row length of the output)
  uint32_t tmem_cols;
  int epi;
  int pdl;           // 1: wait on the previous grid before reading activations
  const __nv_bfloat16* bias;
  void* out;
  unsigned int* status;
};

__host__ __device__ constexpr int gemm_a_bytes() { return kFeatTile * kBlockK * 2; }
__host__ __device__ inline int gemm_b_bytes(int tok_pad) { return tok_pad * kBlockK * 2; }

__global__ void __launch_bounds__(kGemmThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int a_bytes = gemm_a_bytes();
  const int b_bytes = gemm_b_bytes(p.tok_pad);
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + p.stages * a_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.stages * (a_bytes + b_bytes));
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* tmem_full = bars + 2 * p.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int n0 = blockIdx.x * kFeatTile;
  const int split = blockIdx.y;
  const int kb0 = int((long long)p.k_blocks * split / p.splits);
  const int kb1 = int((long long)p.k_blocks * (split + 1) / p.splits);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    mbar_init(smem_addr(tmem_full), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      const uint64_t pol_w = l2_policy_evict_first();  // weights stream once
      const uint64_t pol_x = l2_policy_evict_last();   // activations are re-read by every CTA
      const uint32_t stage_tx = uint32_t(a_bytes + b_bytes);
      if (p.pdl) pdl_wait_prior();
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % p.stages;
        const uint32_t ph = uint32_t(i / p.stages) & 1u;
        if (!wait_bounded(smem_addr(&empty[s]), ph ^ 1u, abort_flag, p.status, 1u)) break;
        const uint32_t fb = smem_addr(&full[s]);
        mbar_arrive_expect_tx(fb, stage_tx);
        const int kx = (kb0 + i) * kBlockK;
        tma_load_2d(smem_addr(a_base + s * a_bytes), &tm_w, fb, kx, n0, pol_w);
        for (int b = 0; b < p.n_boxes; ++b)
          tma_load_2d(smem_addr(b_base + s * b_bytes + b * p.tok_box * kBlockK * 2), &tm_x, fb, kx,
                      b * p.tok_box, pol_x);
        issued = i + 1;
      }
      if (*abort_flag) {
        // Let the copies already in flight land before the CTA releases its shared memory.
        const int first = issued > p.stages ? issued - p.stages : 0;
        for (int i = first; i < issued; ++i)
          wait_drain(smem_addr(&full[i % p.stages]), uint32_t(i / p.stages) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ UMMA issuer
      const uint32_t idesc0 = umma_idesc_bf16(kFeatTile, p.mma_n0);
      const uint32_t idesc1 = umma_idesc_bf16(kFeatTile, p.mma_n1 > 0 ? p.mma_n1 : 16);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % p.stages;
        const uint32_t ph = uint32_t(i / p.stages) & 1u;
        if (!wait_bounded(smem_addr(&full[s]), ph, abort_flag, p.status, 1u)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_addr(a_base + s * a_bytes);
        const uint32_t b_addr = smem_addr(b_base + s * b_bytes);
        const uint64_t adesc = umma_desc_sw128(a_addr);
        const uint64_t bdesc0 = umma_desc_sw128(b_addr);
        const uint64_t bdesc1 = umma_desc_sw128(b_addr + uint32_t(p.mma_n0) * 128u);
#pragma unroll
        for (int k = 0; k < kBlockK / 16; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          umma_bf16(tmem_base, adesc + 2 * k, bdesc0 + 2 * k, idesc0, acc);
          if (p.mma_n1 > 0)
            umma_bf16(tmem_base + uint32_t(p.mma_n0), adesc + 2 * k, bdesc1 + 2 * k, idesc1, acc);
        }
        umma_commit(smem_addr(&empty[s]));  // frees the stage once these MMAs have read it
      }
      umma_commit(smem_addr(tmem_full));    // accumulator complete (or pipeline aborted)
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;     // which half of the column chunks
    // One lane waits; the verdict is broadcast so the .sync.aligned TMEM loads
    // below are executed by all 32 lanes or by none.
    int ok = 0;
    if (lane == 0) ok = wait_bounded(smem_addr(tmem_full), 0u, abort_flag, p.status, 1u) && !*abort_flag;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    tc_fence_after();
    if (ok) {
      const int f_local = q * 32 + lane;
      const int f = n0 + f_local;
      const int nchunks = (p.tokens + 15) >> 4;
      const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
      if (p.epi == EPI_PARTIAL_F32) {
        float* out = reinterpret_cast<float*>(p.out) + size_t(split) * p.tokens * p.n_total;
        for (int c = half; c < nchunks; c += 2) {
          uint32_t r[16];
          tmem_ld16(lane_addr + uint32_t(c * 16), r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = c * 16 + i;
            if (t < p.tokens) out[size_t(t) * p.n_total + f] = __uint_as_float(r[i]);
          }
        }
      } else {
        // bf16 output through a per-warp shared-memory transpose so that each
        // thread writes 16 contiguous bytes of one token row.
        const float bias = __bfloat162float(p.bias[f]);
        __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(smem) + (warp - 2) * (16 * 32);
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
        const int n_base = n0 + q * 32;
        for (int c = half; c < nchunks; c += 2) {
          uint32_t r[16];
          tmem_ld16(lane_addr + uint32_t(c * 16), r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float v = __uint_as_float(r[i]) + bias;
            if (p.epi == EPI_GELU_BF16) v = gelu_tanh(v);
            tile[i * 32 + lane] = __float2bfloat16_rn(v);
          }
          __syncwarp();
#pragma unroll
          for (int pass = 0; pass < 2; ++pass) {
            const int row = pass * 8 + (lane >> 2);
            const int col = (lane & 3) * 8;
            const int t = c * 16 + row;
            const uint4 v = *reinterpret_cast<const uint4*>(&tile[row * 32 + col]);
            if (t < p.tokens) *reinterpret_cast<uint4*>(&out[size_t(t) * p.n_total + n_base + col]) = v;
          }
          __syncwarp();
        }
      }
    }
  }
  if (threadIdx.x == 0) pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

}  // namespace wamffn
