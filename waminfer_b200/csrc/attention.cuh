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
// key block, scaled by the normaliser's reciprocal at the end, stored as bf16.
//
// One CTA per (128-query tile, head, batch); head dim D = 128.  Key blocks of
// 128 rows stream through a 2-stage TMA ring (K and V rows as they lie in
// memory, 128-byte swizzle; K is the K-major operand of Q K^T, V the MN-major
// operand of P V).  Per key block:
//   warp 9 (one elected lane): S = Q K^T -> TMEM columns [0, 128)   (M = 128 queries, N = 128 keys)
//   warps 0-7 (two per TMEM lane quarter: thread = query row x key half):
//              read S, mask, row maximum (exchanged between the halves), exp2,
//              rescale the running O in TMEM, write P (bf16) to shared memory
//   warp 9: O += P V -> TMEM columns [128, 256)                     (M = 128 queries, N = D)
//   warp 8 (one elected lane): TMA loads of Q once and of K / V per block.
// Every wait is a clock-bounded spin (the per-block chain is latency-bound);
// a timed-out wait raises WAMFFN_DEV_TIMEOUT.
#pragma once

#include "gemm.cuh"
#include "ptx.cuh"
#include "wamffn.h"

namespace wamffn {

constexpr int kAttnHeadDim = 128;
constexpr int kAttnRows = 128;      // queries per CTA (UMMA M)
constexpr int kAttnKeys = 128;      // keys per block (UMMA N of S, K of P.V)
constexpr int kAttnSoftmaxWarps = 8;  // two warps per TMEM lane quarter: key / dim halves of each row
constexpr int kAttnThreads = (kAttnSoftmaxWarps + 2) * 32;  // + TMA warp + MMA warp
constexpr int kAttnTile = kAttnRows * 64 * 2;  // one 128-row x 64-element bf16 operand tile (16 KB)
// Shared memory: Q (2 tiles), 2 stages of K (2 tiles) + V (2 tiles), P (2 tiles), row exchange.
constexpr int kAttnSmem = (2 + 2 * 4 + 2) * kAttnTile + 1024 + 256 + 4 * kAttnRows * 4;

// V tiles are consumed as an MN-major operand (dims contiguous, the layout
// TMA writes from V's rows): 64-dim halves 16 KB apart, 8-key groups of the
// 128-byte swizzle 1024 B apart.
constexpr uint32_t kVHalfBytes = kAttnTile;
constexpr uint32_t kVGroupBytes = 1024;

struct AttnParams {
  const unsigned char* mask;  // bool, [b, h, q, k] through the strides below, or null
  long long mb, mh, mq, mk;   // mask strides in elements (0 = broadcast)
  __nv_bfloat16* out;         // [batch, nq, heads * D]
  int heads, nq, nk, batch;
  float scale_log2;           // D^-0.5 * log2(e)
  unsigned int* status;
  uint32_t v_lbo, v_sbo;      // MN-major descriptor offsets of the V operand (bytes)
};

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

// Descriptor of a 128-byte-swizzled MN-major operand.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_byte_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((smem_byte_addr & 0x3FFFFu) >> 4);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    masked_attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;                          // 2 tiles
  uint8_t* kv_s = smem + 2 * kAttnTile;         // stage s: K at +s*4 tiles (2), V at +s*4 tiles + 2 tiles (2)
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
  float* xmax = reinterpret_cast<float*>(smem + 12 * kAttnTile + 256);  // [2 halves][128 rows]
  float* xsum = xmax + 2 * kAttnRows;                                     // [2 halves][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kAttnRows, h = blockIdx.y, b = blockIdx.z;
  const int nblocks = (p.nk + kAttnKeys - 1) / kAttnKeys;
  constexpr int kTmaWarp = kAttnSoftmaxWarps, kMmaWarp = kAttnSoftmaxWarps + 1;

  // Optional phase trace (wamffn_trace_enable): {tag, start, first S ready,
  // last S ready, last P.V done, end, sm, key blocks}, kind 8.
  __shared__ unsigned long long* rec;
  if (threadIdx.x == 0) {
    rec = nullptr;
    if (g_trace != nullptr) {
      const unsigned int slot = atomicAdd(reinterpret_cast<unsigned int*>(g_trace), 1u);
      if (slot + 1 < g_trace_capacity) {
        rec = g_trace + size_t(slot + 1) * kTraceWords;
        rec[0] = (unsigned long long)(blockIdx.x | (blockIdx.y << 16)) | (8ull << 32);
        rec[1] = globaltimer_ns();
        rec[6] = smid();
        rec[7] = (unsigned long long)nblocks;
      }
    }
    mbar_init(smem_addr(q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_addr(&kv_full[s]), 1);
      mbar_init(smem_addr(&kv_empty[s]), 1);
    }
    mbar_init(smem_addr(s_full), 1);
    mbar_init(smem_addr(s_free), kAttnSoftmaxWarps);  // one arrival per softmax warp
    mbar_init(smem_addr(p_full), kAttnSoftmaxWarps);
    mbar_init(smem_addr(o_done), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_addr(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + kAttnKeys;

  if (warp == kTmaWarp) {
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
        if (j >= 2 && !wait_spin(smem_addr(&kv_empty[s]), uint32_t((j >> 1) - 1) & 1u, abort_flag, p.status,
                                    WAMFFN_DEV_TIMEOUT))
          break;
        issued = j + 1;
        uint8_t* st = kv_s + s * 4 * kAttnTile;
        mbar_arrive_expect_tx(smem_addr(&kv_full[s]), 4 * kAttnTile);
        for (int t = 0; t < 2; ++t) {
          // K and V rows of this block, dims [t*64, t*64+64) of the head.
          tma_load_2d(smem_addr(st + t * kAttnTile), &tm_k, smem_addr(&kv_full[s]), h * kAttnHeadDim + t * 64,
                      b * p.nk + j * kAttnKeys, keep);
          tma_load_2d(smem_addr(st + (2 + t) * kAttnTile), &tm_v, smem_addr(&kv_full[s]), h * kAttnHeadDim + t * 64,
                      b * p.nk + j * kAttnKeys, keep);
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
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    const uint32_t idesc_s = umma_idesc_bf16(kAttnRows, kAttnKeys);
    const uint32_t idesc_o = umma_idesc_bf16(kAttnRows, kAttnHeadDim) | (1u << 16);  // B (V) MN-major
    // S of block j + 1 is issued as soon as the softmax has read S of block j,
    // ahead of block j's P.V, so that it is computed while the softmax works.
    auto issue_s = [&](int j) {
      const uint32_t st = smem_addr(kv_s + (j & 1) * 4 * kAttnTile);
      if (elect_one()) {
        // S = Q K^T: K = D = 128 in two 64-element tiles, 4 UMMA steps each.
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(tmem_s, umma_desc_sw128(smem_addr(q_s) + t * kAttnTile) + 2 * k,
                      umma_desc_sw128(st + t * kAttnTile) + 2 * k, idesc_s, (t | k) ? 1u : 0u);
        umma_commit(smem_addr(s_full));
      }
      __syncwarp();
    };
    int ok = 1;
    if (lane == 0)
      ok = wait_spin(smem_addr(q_full), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT) &&
           wait_spin(smem_addr(&kv_full[0]), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; j < nblocks && ok; ++j) {
      if (j + 1 < nblocks) {
        if (lane == 0)
          ok = wait_spin(smem_addr(&kv_full[(j + 1) & 1]), uint32_t((j + 1) >> 1) & 1u, abort_flag, p.status,
                         WAMFFN_DEV_TIMEOUT) &&
               wait_spin(smem_addr(s_free), uint32_t(j) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        issue_s(j + 1);
      }
      if (lane == 0) ok = wait_spin(smem_addr(p_full), uint32_t(j) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t st = smem_addr(kv_s + (j & 1) * 4 * kAttnTile);
      if (elect_one()) {
        // O += P V: K = 128 keys in 8 steps of 16 (P: two K-major 64-key
        // tiles; V: MN-major, 16 keys = two 8-key swizzle groups per step).
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16(tmem_o, umma_desc_sw128(smem_addr(p_s) + (k >> 2) * kAttnTile) + 2 * (k & 3),
                    umma_desc_sw128_mn(st + 2 * kAttnTile + uint32_t(k) * 2 * kVGroupBytes, p.v_lbo, p.v_sbo),
                    idesc_o, (j | k) ? 1u : 0u);
        umma_commit(smem_addr(o_done));
        umma_commit(smem_addr(&kv_empty[j & 1]));
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------ softmax warps
    // Warp w holds TMEM lanes 32 (w % 4).. (query rows) and half = w / 4 of the
    // 128 key columns of S and of the 128 dim columns of O.
    const int r = (warp & 3) * 32 + lane;  // query row within the tile == TMEM lane
    const int half = warp >> 2;
    const int q = q0 + r;
    const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
    const unsigned char* mrow =
        p.mask ? p.mask + size_t(b) * p.mb + size_t(h) * p.mh + size_t(q < p.nq ? q : 0) * p.mq : nullptr;
    const bool mask_vec = mrow && p.mk == 1 && (reinterpret_cast<uintptr_t>(mrow) & 15u) == 0;
    float m = -INFINITY, l = 0.f;  // l: this half's share of the row's normaliser
    int ok = 1;
    // Every softmax warp runs every iteration and reaches every named barrier,
    // also after an abort (the work is then skipped): the two warps sharing a
    // row exchange their maxima through barrier 1.
    for (int j = 0; j < nblocks; ++j) {
      if (lane == 0 && ok)
        ok = wait_spin(smem_addr(s_full), uint32_t(j) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      float sc[64];
      float bmax = -INFINITY;
      const int k0 = j * kAttnKeys + half * 64;
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem_s + lane_base + uint32_t(half * 64 + c * 32), v);
          tmem_wait_ld(v);
#pragma unroll
          for (int i = 0; i < 32; ++i) sc[c * 32 + i] = __uint_as_float(v[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_local(smem_addr(s_free));  // S may be overwritten by the next block
        // Scale, mask, this half's maximum.
        if (!mrow) {
          const int valid_keys = p.nk - k0;  // keys past the sequence are masked
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const float v = i < valid_keys ? sc[i] * p.scale_log2 : -INFINITY;
            sc[i] = v;
            bmax = fmaxf(bmax, v);
          }
        } else if (mask_vec && k0 + 64 <= p.nk) {
#pragma unroll
          for (int v16 = 0; v16 < 4; ++v16) {
            const uint4 mv = *reinterpret_cast<const uint4*>(mrow + k0 + v16 * 16);
            const uint32_t w4[4] = {mv.x, mv.y, mv.z, mv.w};
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const bool keep = ((w4[i >> 2] >> ((i & 3) * 8)) & 0xffu) != 0;
              const float v = keep ? sc[v16 * 16 + i] * p.scale_log2 : -INFINITY;
              sc[v16 * 16 + i] = v;
              bmax = fmaxf(bmax, v);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int key = k0 + i;
            bool valid = key < p.nk;
            if (valid && mrow) valid = mrow[size_t(key) * p.mk] != 0;
            const float v = valid ? sc[i] * p.scale_log2 : -INFINITY;
            sc[i] = v;
            bmax = fmaxf(bmax, v);
          }
        }
      }
      // The row maximum over both halves.
      xmax[half * kAttnRows + r] = bmax;
      named_sync(1, kAttnSoftmaxWarps * 32);
      const float other = xmax[(half ^ 1) * kAttnRows + r];
      named_sync(1, kAttnSoftmaxWarps * 32);  // xmax is rewritten by the next block
      if (!ok) continue;
      if (rec && threadIdx.x == 0) rec[j == 0 ? 2 : 3] = globaltimer_ns();
      const float m_new = fmaxf(m, fmaxf(bmax, other));
      const float safe = m_new == -INFINITY ? 0.f : m_new;
      const float corr = ex2_approx(m - safe);
      float bsum = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        sc[i] = ex2_approx(sc[i] - safe);
        bsum += sc[i];
      }
      l = l * corr + bsum;
      m = m_new;
      // The previous block's P.V must be complete before O is rescaled and P is overwritten.
      if (j > 0) {
        if (lane == 0)
          ok = wait_spin(smem_addr(o_done), uint32_t(j - 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) continue;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem_o + lane_base + uint32_t(half * 64 + c * 32), v);
          tmem_wait_ld(v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
          tmem_st32(tmem_o + lane_base + uint32_t(half * 64 + c * 32), v);
        }
        tmem_wait_st();
      }
      // This half's 64 keys of P (bf16): K-major tile `half` of the P.V product.
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float* pv = sc + c * 8;
        const uint4 u = make_uint4(bf2_pack(pv[0], pv[1]), bf2_pack(pv[2], pv[3]), bf2_pack(pv[4], pv[5]),
                                   bf2_pack(pv[6], pv[7]));
        *reinterpret_cast<uint4*>(p_s + half * kAttnTile + sw128_offset(r, c)) = u;
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_local(smem_addr(p_full));
    }
    // Epilogue: O / l for this half of the row's dims; l summed over both halves.
    xsum[half * kAttnRows + r] = l;
    named_sync(1, kAttnSoftmaxWarps * 32);
    const float lt = half == 0 ? l + xsum[kAttnRows + r] : xsum[r] + l;  // fixed order: key half 0 first
    if (ok) {
      if (lane == 0)
        ok = wait_spin(smem_addr(o_done), uint32_t(nblocks - 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (ok) {
      if (rec && threadIdx.x == 0) rec[4] = globaltimer_ns();
      tc_fence_after();
      const float inv = 1.0f / (lt > 0.f ? lt : 1.0f);  // all-masked rows: O is 0, the output 0
      __nv_bfloat16* orow = p.out + (size_t(b) * p.nq + q) * size_t(p.heads) * kAttnHeadDim + size_t(h) * kAttnHeadDim +
                            half * 64;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem_o + lane_base + uint32_t(half * 64 + c * 32), v);
        tmem_wait_ld(v);
        if (q < p.nq) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = __uint_as_float(v[i + e]) * inv;
            *reinterpret_cast<uint4*>(orow + c * 32 + i) =
                make_uint4(bf2_pack(o[0], o[1]), bf2_pack(o[2], o[3]), bf2_pack(o[4], o[5]), bf2_pack(o[6], o[7]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (rec && threadIdx.x == 0) rec[5] = globaltimer_ns();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace wamffn
