// Masked multi-head attention of the WAMInfer DiT on tcgen05
// (the reference's op wam_infer::masked_attention_mask_tiles_v4,
// WAMInfer/_triton_attention.py:18-145 and :238-263).
//
//   out[b, q, h] = softmax_k( q[b, q, h] . k[b, k, h] / sqrt(D) , mask[b, h, q, k] ) . v[b, k, h]
//
// with the reference's arithmetic: scores in fp32, scaled by D^-0.5 log2(e)
// and exponentiated with exp2; masked keys (and keys past the sequence) at
// -inf; a running row maximum that is treated as 0 while every key so far is
// masked (an all-masked row outputs zeros, as SDPA does); probabilities
// rounded to bf16 before the value product (the reference's
// probability.to(bf16) dot), the normaliser summed in fp32 from the unrounded
// probabilities, the fp32 accumulator rescaled by exp2(m_old - m_new) at every
// key block, divided by the normaliser at the end, stored as bf16.
//
// One CTA per (128-query tile, head, batch); head dim D = 128.  Key blocks of
// 128 rows stream through a 2-stage TMA ring (K [keys, D] and the transposed
// values V^T [D, keys], both K-major with the 128-byte swizzle, so both
// products use the same operand layout as the FFN GEMMs).  Per key block:
//   warp 5 (one elected lane): S = Q K^T -> TMEM columns [0, 128)   (M = 128 queries, N = 128 keys)
//   warps 0-3 (thread = query row = TMEM lane): read S, mask, row max, exp2,
//              rescale the running O in TMEM, write P (bf16) to shared memory
//   warp 5: O += P V -> TMEM columns [128, 256)                     (M = 128 queries, N = D)
//   warp 4 (one elected lane): TMA loads of Q once and of K / V^T per block.
// Every wait is clock-bounded; a timed-out wait raises WAMFFN_DEV_TIMEOUT.
#pragma once

#include "ptx.cuh"
#include "wamffn.h"

namespace wamffn {

constexpr int kAttnHeadDim = 128;
constexpr int kAttnRows = 128;      // queries per CTA (UMMA M)
constexpr int kAttnKeys = 128;      // keys per block (UMMA N of S, K of P.V)
constexpr int kAttnThreads = 192;   // 4 softmax warps, TMA warp, MMA warp
constexpr int kAttnTile = kAttnRows * 64 * 2;  // one 128-row x 64-element bf16 operand tile (16 KB)
// Shared memory: Q (2 tiles), 2 stages of K (2 tiles) + V^T (2 tiles), P (2 tiles).
constexpr int kAttnSmem = (2 + 2 * 4 + 2) * kAttnTile + 1024 + 256;

struct AttnParams {
  const unsigned char* mask;  // bool, [b, h, q, k] through the strides below, or null
  long long mb, mh, mq, mk;   // mask strides in elements (0 = broadcast)
  __nv_bfloat16* out;         // [batch, nq, heads * D]
  int heads, nq, nk, batch;
  float scale_log2;           // D^-0.5 * log2(e)
  unsigned int* status;
};

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

__global__ void __launch_bounds__(kAttnThreads, 1)
    masked_attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_vt, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;                          // 2 tiles
  uint8_t* kv_s = smem + 2 * kAttnTile;         // stage s: K at +s*4 tiles, V^T at +s*4 tiles + 2 tiles
  uint8_t* p_s = smem + 10 * kAttnTile;         // 2 tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 12 * kAttnTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* o_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kAttnRows, h = blockIdx.y, b = blockIdx.z;
  const int nblocks = (p.nk + kAttnKeys - 1) / kAttnKeys;

  if (threadIdx.x == 0) {
    mbar_init(smem_addr(q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_addr(&kv_full[s]), 1);
      mbar_init(smem_addr(&kv_empty[s]), 1);
    }
    mbar_init(smem_addr(s_full), 1);
    mbar_init(smem_addr(s_free), 4);  // one arrival per softmax warp
    mbar_init(smem_addr(p_full), 4);
    mbar_init(smem_addr(o_done), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_vt);
  }
  if (warp == 5) {
    tmem_alloc(smem_addr(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + kAttnKeys;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA loads
    if (elect_one()) {
      const uint64_t keep = l2_policy_evict_last();  // K / V are re-read by every query tile of the head
      mbar_arrive_expect_tx(smem_addr(q_full), 2 * kAttnTile);
      for (int t = 0; t < 2; ++t)
        tma_load_2d(smem_addr(q_s + t * kAttnTile), &tm_q, smem_addr(q_full), h * kAttnHeadDim + t * 64,
                    b * p.nq + q0, keep);
      int issued = 0;
      for (int j = 0; j < nblocks; ++j) {
        const int s = j & 1;
        if (j >= 2 && !wait_bounded(smem_addr(&kv_empty[s]), uint32_t((j >> 1) - 1) & 1u, abort_flag, p.status,
                                    WAMFFN_DEV_TIMEOUT))
          break;
        issued = j + 1;
        uint8_t* st = kv_s + s * 4 * kAttnTile;
        mbar_arrive_expect_tx(smem_addr(&kv_full[s]), 4 * kAttnTile);
        for (int t = 0; t < 2; ++t) {
          tma_load_2d(smem_addr(st + t * kAttnTile), &tm_k, smem_addr(&kv_full[s]), h * kAttnHeadDim + t * 64,
                      b * p.nk + j * kAttnKeys, keep);
          tma_load_2d(smem_addr(st + (2 + t) * kAttnTile), &tm_vt, smem_addr(&kv_full[s]), j * kAttnKeys + t * 64,
                      (b * p.heads + h) * kAttnHeadDim, keep);
        }
      }
      if (*abort_flag) {
        // Let the copies still in flight land before the CTA gives up its shared memory.
        wait_drain(smem_addr(q_full), 0u);
        for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j)
          wait_drain(smem_addr(&kv_full[j & 1]), uint32_t(j >> 1) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issue
    const uint32_t idesc = umma_idesc_bf16(kAttnRows, kAttnKeys);  // both products are 128 x 128
    int ok = 1;
    if (lane == 0) ok = wait_bounded(smem_addr(q_full), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    for (int j = 0; j < nblocks && ok; ++j) {
      const int s = j & 1;
      if (lane == 0) {
        ok = wait_bounded(smem_addr(&kv_full[s]), uint32_t(j >> 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
        if (ok && j > 0)
          ok = wait_bounded(smem_addr(s_free), uint32_t(j - 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t st = smem_addr(kv_s + s * 4 * kAttnTile);
      if (elect_one()) {
        // S = Q K^T: K = D = 128 in two 64-element tiles, 4 UMMA steps each.
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(tmem_s, umma_desc_sw128(smem_addr(q_s) + t * kAttnTile) + 2 * k,
                      umma_desc_sw128(st + t * kAttnTile) + 2 * k, idesc, (t | k) ? 1u : 0u);
        umma_commit(smem_addr(s_full));
      }
      __syncwarp();
      if (lane == 0) ok = wait_bounded(smem_addr(p_full), uint32_t(j) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        // O += P V: K = 128 keys in two 64-key tiles of P and of V^T.
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(tmem_o, umma_desc_sw128(smem_addr(p_s) + t * kAttnTile) + 2 * k,
                      umma_desc_sw128(st + (2 + t) * kAttnTile) + 2 * k, idesc, (j | t | k) ? 1u : 0u);
        umma_commit(smem_addr(o_done));
        umma_commit(smem_addr(&kv_empty[s]));
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------ softmax warps
    const int r = threadIdx.x;  // query row within the tile == TMEM lane
    const int q = q0 + r;
    const uint32_t lane_base = uint32_t(warp * 32) << 16;
    const unsigned char* mrow =
        p.mask ? p.mask + size_t(b) * p.mb + size_t(h) * p.mh + size_t(q < p.nq ? q : 0) * p.mq : nullptr;
    float m = -INFINITY, l = 0.f;
    int ok = 1;
    for (int j = 0; j < nblocks && ok; ++j) {
      if (lane == 0) ok = wait_bounded(smem_addr(s_full), uint32_t(j) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      float sc[kAttnKeys];
#pragma unroll
      for (int c = 0; c < kAttnKeys / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem_s + lane_base + uint32_t(c * 32), v);
        tmem_wait_ld(v);
#pragma unroll
        for (int i = 0; i < 32; ++i) sc[c * 32 + i] = __uint_as_float(v[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_local(smem_addr(s_free));  // S may be overwritten by the next block
      // Scale, mask, running maximum.
      const int k0 = j * kAttnKeys;
      float bmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < kAttnKeys; ++i) {
        const int key = k0 + i;
        bool valid = key < p.nk;
        if (valid && mrow) valid = mrow[size_t(key) * p.mk] != 0;
        const float v = valid ? sc[i] * p.scale_log2 : -INFINITY;
        sc[i] = v;
        bmax = fmaxf(bmax, v);
      }
      const float m_new = fmaxf(m, bmax);
      const float safe = m_new == -INFINITY ? 0.f : m_new;
      const float corr = ex2_approx(m - safe);
      float bsum = 0.f;
#pragma unroll
      for (int i = 0; i < kAttnKeys; ++i) {
        sc[i] = ex2_approx(sc[i] - safe);
        bsum += sc[i];
      }
      l = l * corr + bsum;
      m = m_new;
      // The previous block's P.V must be complete before O is rescaled and P is overwritten.
      if (j > 0) {
        if (lane == 0)
          ok = wait_bounded(smem_addr(o_done), uint32_t(j - 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kAttnHeadDim / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem_o + lane_base + uint32_t(c * 32), v);
          tmem_wait_ld(v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
          tmem_st32(tmem_o + lane_base + uint32_t(c * 32), v);
        }
        tmem_wait_st();
      }
      // P (bf16) in the 128-byte-swizzled K-major layout of the P.V product.
#pragma unroll
      for (int t = 0; t < 2; ++t) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float* pv = sc + t * 64 + c * 8;
          uint4 u = make_uint4(bf2_pack(pv[0], pv[1]), bf2_pack(pv[2], pv[3]), bf2_pack(pv[4], pv[5]),
                               bf2_pack(pv[6], pv[7]));
          *reinterpret_cast<uint4*>(p_s + t * kAttnTile + sw128_offset(r, c)) = u;
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_local(smem_addr(p_full));
    }
    // Epilogue: O / l for the rows of this tile.
    if (ok) {
      if (lane == 0)
        ok = wait_bounded(smem_addr(o_done), uint32_t(nblocks - 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (ok) {
      tc_fence_after();
      const float denom = l > 0.f ? l : 1.0f;  // all-masked rows: O is 0, the output 0
      __nv_bfloat16* orow = p.out + (size_t(b) * p.nq + q) * size_t(p.heads) * kAttnHeadDim + size_t(h) * kAttnHeadDim;
#pragma unroll 1
      for (int c = 0; c < kAttnHeadDim / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem_o + lane_base + uint32_t(c * 32), v);
        tmem_wait_ld(v);
        if (q < p.nq) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = __fdiv_rn(__uint_as_float(v[i + e]), denom);
            *reinterpret_cast<uint4*>(orow + c * 32 + i) =
                make_uint4(bf2_pack(o[0], o[1]), bf2_pack(o[2], o[3]), bf2_pack(o[4], o[5]), bf2_pack(o[6], o[7]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// V [batch, nk, heads * D] -> V^T [batch * heads * D, nk_pad] (keys contiguous,
// zeros past nk): the K-major operand of the P.V product.
__global__ void transpose_values_kernel(const __nv_bfloat16* __restrict__ v, long long v_row, long long v_batch,
                                        __nv_bfloat16* __restrict__ vt, int heads, int nk, int nk_pad) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int bh = blockIdx.z;
  const int b = bh / heads, h = bh % heads;
  const int k0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int y = ty; y < 32; y += 8) {
    const int key = k0 + y;
    tile[y][tx] = key < nk ? v[size_t(b) * v_batch + size_t(key) * v_row + size_t(h) * kAttnHeadDim + d0 + tx]
                           : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  for (int y = ty; y < 32; y += 8) {
    const int d = d0 + y;
    vt[(size_t(bh) * kAttnHeadDim + d) * nk_pad + k0 + tx] = tile[tx][y];
  }
}

}  // namespace wamffn
