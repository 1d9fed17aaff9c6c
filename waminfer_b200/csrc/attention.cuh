// Multi-head attention of the WAMInfer DiT on tcgen05: the reference's three
// attention ops (WAMInfer/_triton_attention.py) on one kernel.
//
//   masked_attention_mask_tiles_v4   (:18-145, :238-263)  q against k / v, bool mask [b, h, q, k]
//   joint_first_frame_attention_v2   (:267-334)           rows [0, first) see keys [0, first), the rest see all
//   current_frame_attention_v1       (:337-484)           queries (video ++ action) against keys
//                                                         (context ++ video ++ action), never concatenated
//
//   out[b, q, h] = softmax_k( q[b, q, h] . k[b, k, h] / sqrt(D) , masked ) . v[b, k, h]
//
// with the reference's arithmetic: scores in fp32, scaled by D^-0.5 log2(e)
// and exponentiated with exp2; masked keys (and keys past a segment) at -inf;
// a running row maximum that is treated as 0 while every key so far is masked
// (an all-masked row outputs zeros, as SDPA does); probabilities rounded to
// bf16 before the value product (the reference's probability.to(bf16) dot),
// the normaliser summed in fp32 from the unrounded probabilities, the fp32
// accumulator rescaled by exp2(m_old - m_new) at every key block, scaled by
// the normaliser's reciprocal at the end, stored as bf16.
//
// Segments.  The queries are up to two row ranges (each with its own tensor
// map and output rows) and the keys up to three tensors taken as one
// concatenated sequence; a query segment sees a prefix of that sequence.  Key
// blocks of 128 rows never straddle two key tensors: a segment's last block is
// short and its missing keys are masked, which changes only where the blocks
// start, not the function.
//
// One CTA per (128-query tile, head, batch); head dim D = 128.  Key blocks
// stream through a 2-stage TMA ring (K and V rows as they lie in memory,
// 128-byte swizzle; K is the K-major operand of Q K^T, V the MN-major operand
// of P V); a stage's K is refilled as soon as its S is done, its V once its
// P V is done, so that the next blocks' K is resident before it is needed.  Per key block:
//   warp 9 (one elected lane): S = Q K^T -> TMEM columns [0, 128)   (M = 128 queries, N = 128 keys)
//   warps 0-7 (two per TMEM lane quarter: thread = query row x key half):
//              read S, mask, row maximum (exchanged between the halves), exp2,
//              rescale the running O in TMEM, write P (bf16) to shared memory
//   warp 9: O += P V -> TMEM columns [128, 256)                     (M = 128 queries, N = D)
//   warp 8 (one elected lane): TMA loads of Q once and of K / V per block.
// Every wait is a clock-bounded spin (the per-block chain is latency-bound);
// a timed-out wait raises WAMFFN_DEV_TIMEOUT.
//
// Masked-block skip: when the mask is shared by every head and query row (a
// padded text prompt), key blocks in which no key is kept are left out.  Such
// a block adds exactly nothing (probabilities 0, correction 2^0 = 1), so the
// skip changes no bit.
//
// Key split (grids that would leave SMs idle: the 32-query action rows, the
// context attention of 2-3 query tiles per head): a cluster of `split` CTAs
// shares one query tile, each runs the loop above over its share of the key
// blocks, and the partial (maximum, normaliser, unnormalised O) are combined
// through distributed shared memory, each CTA producing 128 / split of the
// output dims.  The split changes where the probabilities' bf16 rounding is
// taken (against the share's running maximum), as the reference's own choice
// of key block size does.
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
constexpr int kAttnMaxQSeg = 2, kAttnMaxKSeg = 3;
constexpr int kAttnSkipWords = 64;  // key-block bitmap of the masked-block skip: up to 2048 blocks
// Shared memory: Q (2 tiles), 2 stages of K (2 tiles) + V (2 tiles), P (2 tiles),
// barriers, row exchange, skip bitmap.
constexpr int kAttnSmem = (2 + 2 * 4 + 2) * kAttnTile + 1024 + 256 + 4 * kAttnRows * 4 + kAttnSkipWords * 4;

// V tiles are consumed as an MN-major operand (dims contiguous, the layout
// TMA writes from V's rows): 64-dim halves 16 KB apart, 8-key groups of the
// 128-byte swizzle 1024 B apart.
constexpr uint32_t kVHalfBytes = kAttnTile;
constexpr uint32_t kVGroupBytes = 1024;

// The tensor maps of one launch (2-D, [batch x rows, width], box 64 x 128).
struct AttnMaps {
  CUtensorMap q[kAttnMaxQSeg];
  CUtensorMap k[kAttnMaxKSeg];
  CUtensorMap v[kAttnMaxKSeg];
};

// A query segment: rows [row0, row0 + rows) of map q[s] in every batch
// (map row = b * map_batch_rows + row0 + i), written to
// out + b * out_batch_stride + i * out_row_stride + h * 128.
struct AttnQSeg {
  __nv_bfloat16* out;
  long long out_batch_stride, out_row_stride;  // elements
  int rows, map_batch_rows, row0;
  int tiles;    // ceil(rows / 128)
  int visible;  // keys seen by the segment: a prefix of the concatenated key segments
};

struct AttnParams {
  const unsigned char* mask;  // bool, [b, h, q, k] through the strides below, or null (one segment each)
  long long mb, mh, mq, mk;   // mask strides in elements (0 = broadcast)
  int skip_masked;            // mh == mq == 0: key blocks without a kept key are skipped (the kSkip kernel)
  AttnQSeg qseg[kAttnMaxQSeg];
  int nqseg;
  int krows[kAttnMaxKSeg];  // rows per batch of key segment t (map row = b * krows[t] + i)
  int nkseg;
  int heads, batch;
  float scale_log2;  // D^-0.5 * log2(e)
  unsigned int* status;
  int split;  // key split: CTAs per cluster sharing one query tile (1, 2 or 4)
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

// Key blocks of one query segment over the concatenated key segments.
struct AttnKeyPlan {
  int blocks[kAttnMaxKSeg];  // 128-key blocks of segment t (of its visible keys)
  int vis[kAttnMaxKSeg];     // visible keys of segment t
  int base[kAttnMaxKSeg];    // index of segment t's first key in the concatenation
  int total;
};

// One key block: segment, first row in the segment, keys valid from that row,
// index of the first key in the concatenated sequence.
struct AttnKeyBlock {
  int seg, row, valid, key;
};

__device__ __forceinline__ AttnKeyBlock attn_block(const AttnKeyPlan& kp, int jj) {
  AttnKeyBlock r;
  int t = 0;
  if (jj >= kp.blocks[0]) {
    jj -= kp.blocks[0];
    t = 1;
    if (jj >= kp.blocks[1]) {
      jj -= kp.blocks[1];
      t = 2;
    }
  }
  const int vis = t == 0 ? kp.vis[0] : t == 1 ? kp.vis[1] : kp.vis[2];
  const int base = t == 0 ? kp.base[0] : t == 1 ? kp.base[1] : kp.base[2];
  r.seg = t;
  r.row = jj * kAttnKeys;
  r.valid = min(kAttnKeys, vis - r.row);
  r.key = base + r.row;
  return r;
}

// Index of the n-th (from 0) set bit of the skip bitmap.
__device__ __forceinline__ int attn_nth_active(const uint32_t* bits, int words, int n) {
  for (int w = 0; w < words; ++w) {
    const uint32_t x = bits[w];
    const int c = __popc(x);
    if (n < c) return w * 32 + int(__fns(x, 0, n + 1));
    n -= c;
  }
  return 0;  // not reached: n < the bitmap's population
}

// kSkip: the masked-block skip is compiled in (p.skip_masked set); kSplit:
// the key-split combine is (p.split > 1).  An instantiation without a feature
// carries none of its code or registers.
template <bool kSkip, bool kSplit>
__global__ void __launch_bounds__(kAttnThreads, 1)
    masked_attention_kernel(const __grid_constant__ AttnMaps maps, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;                          // 2 tiles
  uint8_t* kv_s = smem + 2 * kAttnTile;         // stage s: K at +s*4 tiles (2), V at +s*4 tiles + 2 tiles (2)
  uint8_t* p_s = smem + 10 * kAttnTile;         // 2 tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 12 * kAttnTile);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]  K of a stage landed (S needs only K)
  uint64_t* v_full = bars + 3;    // [2]  V of a stage landed
  uint64_t* k_empty = bars + 5;   // [2]  S of the stage's block is done: its K may be overwritten
  uint64_t* v_empty = bars + 7;   // [2]  P V of the stage's block is done: its V may be overwritten
  uint64_t* s_full = bars + 9;
  uint64_t* s_free = bars + 10;
  uint64_t* p_full = bars + 11;
  uint64_t* o_done = bars + 12;
  uint64_t* xch_full = bars + 13;  // key-split combine: the peers' slots have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xmax = reinterpret_cast<float*>(smem + 12 * kAttnTile + 256);  // [2 halves][128 rows]
  float* xsum = xmax + 2 * kAttnRows;                                     // [2 halves][128 rows]
  uint32_t* skip_bits = reinterpret_cast<uint32_t*>(xsum + 2 * kAttnRows);  // [kAttnSkipWords]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = kSplit ? p.split : 1;
  const int ctile = int(blockIdx.x) / split, rank = int(blockIdx.x) - ctile * split;
  const int h = blockIdx.y, b = blockIdx.z;
  const int seg = (p.nqseg > 1 && ctile >= p.qseg[0].tiles) ? 1 : 0;
  AttnQSeg qs;  // field by field: no dynamically indexed copy of the parameters
  qs.out = seg ? p.qseg[1].out : p.qseg[0].out;
  qs.out_batch_stride = seg ? p.qseg[1].out_batch_stride : p.qseg[0].out_batch_stride;
  qs.out_row_stride = seg ? p.qseg[1].out_row_stride : p.qseg[0].out_row_stride;
  qs.rows = seg ? p.qseg[1].rows : p.qseg[0].rows;
  qs.map_batch_rows = seg ? p.qseg[1].map_batch_rows : p.qseg[0].map_batch_rows;
  qs.row0 = seg ? p.qseg[1].row0 : p.qseg[0].row0;
  qs.visible = seg ? p.qseg[1].visible : p.qseg[0].visible;
  const int q0 = (ctile - (seg ? p.qseg[0].tiles : 0)) * kAttnRows;  // first row of the tile in its segment
  AttnKeyPlan kp;
  {
    int base = 0;
    kp.total = 0;
#pragma unroll
    for (int t = 0; t < kAttnMaxKSeg; ++t) {
      const int rows = t < p.nkseg ? p.krows[t] : 0;
      kp.vis[t] = max(0, min(qs.visible - base, rows));
      kp.blocks[t] = (kp.vis[t] + kAttnKeys - 1) / kAttnKeys;
      kp.base[t] = base;
      base += rows;
      kp.total += kp.blocks[t];
    }
  }
  constexpr int kTmaWarp = kAttnSoftmaxWarps, kMmaWarp = kAttnSoftmaxWarps + 1;
  const int skip_words = (kp.total + 31) / 32;

  const bool tma_lane = threadIdx.x == kTmaWarp * 32;  // sets up the barriers and issues every TMA load
  if (tma_lane) {
    mbar_init(smem_addr(q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_addr(&k_full[s]), 1);
      mbar_init(smem_addr(&v_full[s]), 1);
      mbar_init(smem_addr(&k_empty[s]), 1);
      mbar_init(smem_addr(&v_empty[s]), 1);
    }
    mbar_init(smem_addr(s_full), 1);
    mbar_init(smem_addr(s_free), kAttnSoftmaxWarps);  // one arrival per softmax warp
    mbar_init(smem_addr(p_full), kAttnSoftmaxWarps);
    mbar_init(smem_addr(o_done), 1);
    mbar_init(smem_addr(xch_full), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&maps.q[seg]);
    for (int t = 0; t < p.nkseg; ++t) {
      if (p.krows[t] == 0) continue;  // an empty segment has no map
      prefetch_tensormap(&maps.k[t]);
      prefetch_tensormap(&maps.v[t]);
    }
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_addr(tmem_slot), 256);
    tmem_relinquish();
  }
  // Programmatic dependent launch: the set-up above overlaps the previous
  // kernel on the stream; global memory is touched only after it completed.
  pdl_wait_prior();
  if (threadIdx.x == 0) pdl_launch_dependents();

  // Masked-block skip: the TMA warp builds the bitmap of the key blocks that
  // hold a kept key (lane l tests keys [16 l, 16 l + 16) of each 512-key
  // round; lane 0 writes the words), so that its first lane can issue the
  // first loads at once; the other warps read the bitmap after the
  // block-wide barrier below.
  if (kSkip && warp == kTmaWarp) {
    const int nk = kp.vis[0];  // the skip runs with one key segment
    const unsigned char* mrow = p.mask + size_t(b) * p.mb;
    const bool vec = p.mk == 1 && (reinterpret_cast<uintptr_t>(mrow) & 15u) == 0;
    if (lane == 0)
      for (int w = 0; w < skip_words; ++w) skip_bits[w] = 0u;
    for (int base = 0; base < nk; base += 32 * 16) {
      const int k0 = base + lane * 16;
      bool kept = false;
      if (vec && k0 + 16 <= nk) {
        const uint4 m = *reinterpret_cast<const uint4*>(mrow + k0);
        kept = (m.x | m.y | m.z | m.w) != 0u;
      } else {
        for (int i = 0; i < 16 && k0 + i < nk; ++i) kept |= mrow[size_t(k0 + i) * p.mk] != 0;
      }
      const uint32_t votes = __ballot_sync(0xffffffffu, kept);  // bit l: chunk l of the round
      if (lane == 0)
        for (int i = 0; i < 4; ++i) {  // 128-key block i of the round = chunks 8 i .. 8 i + 7
          const int blk = base / kAttnKeys + i;
          if (((votes >> (8 * i)) & 0xffu) != 0u) skip_bits[blk >> 5] |= 1u << (blk & 31);
        }
    }
    __syncwarp();
  }
  // Active key blocks (known to the TMA warp now, to every thread after the
  // block-wide barrier) and the key block of an active ordinal.
  auto count_active = [&]() {
    int active = kp.total;
    if (kSkip) {
      active = 0;
      for (int w = 0; w < skip_words; ++w) active += __popc(skip_bits[w]);
    }
    return active;
  };
  auto block_of = [&](int o) {
    return attn_block(kp, kSkip ? attn_nth_active(skip_bits, skip_words, o) : o);
  };

  // TMA loads (issued by tma_lane only): Q once, K and V of block j into ring stage j & 1.
  const uint64_t keep = l2_policy_evict_last();  // K / V are re-read by every query tile of the head
  auto issue_q = [&]() {
    mbar_arrive_expect_tx(smem_addr(q_full), 2 * kAttnTile);
    for (int t = 0; t < 2; ++t)
      tma_load_2d(smem_addr(q_s + t * kAttnTile), &maps.q[seg], smem_addr(q_full), h * kAttnHeadDim + t * 64,
                  b * qs.map_batch_rows + qs.row0 + q0, keep);
  };
  // K and V rows of block j, dims [t*64, t*64+64) of the head, into ring
  // stage j & 1 on separate barriers (S needs only K; K is free again once
  // S is done, V only once P V is done).
  auto kv_row = [&](const AttnKeyBlock& kb) {
    return b * (kb.seg == 0 ? p.krows[0] : kb.seg == 1 ? p.krows[1] : p.krows[2]) + kb.row;
  };
  auto issue_k = [&](int j, const AttnKeyBlock& kb) {
    const int s = j & 1;
    uint8_t* st = kv_s + s * 4 * kAttnTile;
    mbar_arrive_expect_tx(smem_addr(&k_full[s]), 2 * kAttnTile);
    for (int t = 0; t < 2; ++t)
      tma_load_2d(smem_addr(st + t * kAttnTile), &maps.k[kb.seg], smem_addr(&k_full[s]), h * kAttnHeadDim + t * 64,
                  kv_row(kb), keep);
  };
  auto issue_v = [&](int j, const AttnKeyBlock& kb) {
    const int s = j & 1;
    uint8_t* st = kv_s + s * 4 * kAttnTile;
    mbar_arrive_expect_tx(smem_addr(&v_full[s]), 2 * kAttnTile);
    for (int t = 0; t < 2; ++t)
      tma_load_2d(smem_addr(st + (2 + t) * kAttnTile), &maps.v[kb.seg], smem_addr(&v_full[s]),
                  h * kAttnHeadDim + t * 64, kv_row(kb), keep);
  };
  // Q and the first two key blocks go out before the block-wide barrier.
  int early = 0;
  if (tma_lane) {
    const int active = count_active();
    const int jb = rank * active / split;
    early = min((rank + 1) * active / split - jb, 2);
    if (early) issue_q();
    for (int j = 0; j < early; ++j) {
      const AttnKeyBlock kb = block_of(jb + j);
      issue_k(j, kb);
      issue_v(j, kb);
    }
  }

  // Optional phase trace (wamffn_trace_enable): {tag, start, first S ready,
  // last S ready (first cluster barrier passed, with a key split), last P.V
  // done, end, sm | key blocks << 32, the peers' slots landed}, kind 8,
  // the CTA's rank in its key-split cluster in tag bits 48-51.
  __shared__ unsigned long long* rec;
  if (threadIdx.x == 0) {
    rec = nullptr;
    if (g_trace != nullptr) {
      const unsigned int slot = atomicAdd(reinterpret_cast<unsigned int*>(g_trace), 1u);
      if (slot + 1 < g_trace_capacity) {
        rec = g_trace + size_t(slot + 1) * kTraceWords;
        rec[0] = (unsigned long long)(blockIdx.x | (blockIdx.y << 16)) | (8ull << 32) | ((unsigned long long)rank << 48);
        rec[1] = globaltimer_ns();
        rec[7] = 0;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // This CTA's share of the active key blocks: ordinals [jb, jb + nblocks).
  const int active = count_active();
  const int jb = rank * active / split;
  const int nblocks = (rank + 1) * active / split - jb;
  if (rec && threadIdx.x == 0) rec[6] = smid() | ((unsigned long long)nblocks << 32);
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + kAttnKeys;

  if (warp == kTmaWarp) {
    // ------------------------------------------------------------ TMA loads
    if (nblocks > 0 && lane == 0) {
      if (!early) issue_q();
      int issued_k = early, issued_v = early;
      for (int j = early; j < nblocks; ++j) {
        const AttnKeyBlock kb = block_of(jb + j);
        const uint32_t parity = uint32_t((j >> 1) - 1) & 1u;  // j >= 2 here
        if (!wait_spin(smem_addr(&k_empty[j & 1]), parity, abort_flag, p.status, WAMFFN_DEV_TIMEOUT)) break;
        issue_k(j, kb);
        issued_k = j + 1;
        if (!wait_spin(smem_addr(&v_empty[j & 1]), parity, abort_flag, p.status, WAMFFN_DEV_TIMEOUT)) break;
        issue_v(j, kb);
        issued_v = j + 1;
      }
      if (*abort_flag) {
        // Let the copies still in flight land before the CTA gives up its shared memory.
        wait_drain(smem_addr(q_full), 0u);
        for (int j = issued_k > 2 ? issued_k - 2 : 0; j < issued_k; ++j)
          wait_drain(smem_addr(&k_full[j & 1]), uint32_t(j >> 1) & 1u);
        for (int j = issued_v > 2 ? issued_v - 2 : 0; j < issued_v; ++j)
          wait_drain(smem_addr(&v_full[j & 1]), uint32_t(j >> 1) & 1u);
      }
    }
    __syncwarp();
    if (split > 1) {  // the softmax warps' two cluster barriers of the key-split combine
      cluster_sync();
      cluster_arrive();
      cluster_wait();
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    const uint32_t idesc_s = umma_idesc_bf16(kAttnRows, kAttnKeys);
    const uint32_t idesc_o = umma_idesc_bf16(kAttnRows, kAttnHeadDim) | (1u << 16);  // B (V) MN-major
    // S of block j + 1 is issued as soon as the softmax has read S of block j
    // and K of block j + 1 has landed, ahead of block j's P.V, so that it is
    // computed while the softmax works.
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
        umma_commit(smem_addr(&k_empty[j & 1]));
      }
      __syncwarp();
    };
    int ok = nblocks > 0;
    if (ok) {
      if (lane == 0)
        ok = wait_spin(smem_addr(q_full), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT) &&
             wait_spin(smem_addr(&k_full[0]), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; j < nblocks && ok; ++j) {
      if (j + 1 < nblocks) {
        if (lane == 0)
          ok = wait_spin(smem_addr(&k_full[(j + 1) & 1]), uint32_t((j + 1) >> 1) & 1u, abort_flag, p.status,
                         WAMFFN_DEV_TIMEOUT) &&
               wait_spin(smem_addr(s_free), uint32_t(j) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        issue_s(j + 1);
      }
      if (lane == 0)
        ok = wait_spin(smem_addr(&v_full[j & 1]), uint32_t(j >> 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT) &&
             wait_spin(smem_addr(p_full), uint32_t(j) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
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
                    umma_desc_sw128_mn(st + 2 * kAttnTile + uint32_t(k) * 2 * kVGroupBytes, kVHalfBytes, kVGroupBytes),
                    idesc_o, (j | k) ? 1u : 0u);
        umma_commit(smem_addr(o_done));
        umma_commit(smem_addr(&v_empty[j & 1]));
      }
      __syncwarp();
    }
    if (split > 1) {
      cluster_sync();
      cluster_arrive();
      cluster_wait();
    }
  } else {
    // ------------------------------------------------------ softmax warps
    // Warp w holds TMEM lanes 32 (w % 4).. (query rows) and half = w / 4 of the
    // 128 key columns of S and of the 128 dim columns of O.
    const int r = (warp & 3) * 32 + lane;  // query row within the tile == TMEM lane
    const int half = warp >> 2;
    const int q = q0 + r;                  // row within the query segment
    const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
    const unsigned char* mrow =
        p.mask ? p.mask + size_t(b) * p.mb + size_t(h) * p.mh + size_t(q < qs.rows ? q : 0) * p.mq : nullptr;
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
      const AttnKeyBlock kb = block_of(jb + j);
      const int k0 = kb.key + half * 64;             // first key of this half in the concatenation
      const int valid_keys = kb.valid - half * 64;   // keys past the segment are masked
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
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const float v = i < valid_keys ? sc[i] * p.scale_log2 : -INFINITY;
            sc[i] = v;
            bmax = fmaxf(bmax, v);
          }
        } else if (mask_vec && valid_keys >= 64) {
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
            bool valid = i < valid_keys;
            if (valid) valid = mrow[size_t(k0 + i) * p.mk] != 0;
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
      if (rec && threadIdx.x == 0 && (j == 0 || split == 1)) rec[j == 0 ? 2 : 3] = globaltimer_ns();
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
    if (ok && nblocks > 0) {
      if (lane == 0)
        ok = wait_spin(smem_addr(o_done), uint32_t(nblocks - 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (ok && rec && threadIdx.x == 0) rec[4] = globaltimer_ns();
    // O of this CTA (zero when it ran no key block: TMEM then holds nothing).
    const bool has_o = nblocks > 0;
    __nv_bfloat16* orow = qs.out + size_t(b) * qs.out_batch_stride + size_t(q < qs.rows ? q : 0) * qs.out_row_stride +
                          size_t(h) * kAttnHeadDim;
    if (split == 1) {
      if (ok) {
        tc_fence_after();
        const float inv = 1.0f / (lt > 0.f ? lt : 1.0f);  // all-masked rows: O is 0, the output 0
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          if (has_o) {
            tmem_ld32(tmem_o + lane_base + uint32_t(half * 64 + c * 32), v);
            tmem_wait_ld(v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0u;
          }
          if (q < qs.rows) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              float o[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] = __uint_as_float(v[i + e]) * inv;
              *reinterpret_cast<uint4*>(orow + half * 64 + c * 32 + i) = make_uint4(
                  bf2_pack(o[0], o[1]), bf2_pack(o[2], o[3]), bf2_pack(o[4], o[5]), bf2_pack(o[6], o[7]));
            }
          }
        }
      }
    } else {
      // Key-split combine over the cluster.  CTA c owns output dims
      // [c W, c W + W), W = 128 / split.  Every CTA stages, for each other
      // CTA, the 32-dim pieces of its unnormalised O rows that CTA owns and the
      // rows' (maximum, normaliser), in the receiver's layout, and sends each
      // staged slot with one bulk copy into the receiver's shared memory.  The
      // owner rescales the split's partial results to their common maximum and
      // sums them in rank order:
      //   O = sum_k O_k 2^(m_k - M),  l = sum_k l_k 2^(m_k - M),  out = O / l.
      // Receive slots sit in stage 0 of the K / V ring, staged slots in stage
      // 1; a CTA's ring is free once its last P.V is done, and peers write
      // into it only after the first cluster barrier.
      // A slot is [128 rows][2] (m, l), then [128 rows][pitch] O; only the
      // tile's rows inside the query segment travel.
      const int W = kAttnHeadDim / split, pitch = W + 4;  // 16-byte row pad: conflict-free 16-byte accesses
      const int live = min(kAttnRows, qs.rows - q0);      // >= 1
      const uint32_t slot_bytes = uint32_t(kAttnRows * 8 + kAttnRows * pitch * 4);
      const uint32_t send_bytes = uint32_t(kAttnRows * 8 + live * pitch * 4);  // a multiple of 16
      uint8_t* recv = kv_s;                   // [split - 1 senders]
      uint8_t* stage = kv_s + 4 * kAttnTile;  // [split - 1 receivers]
      // TMEM loads are warp-wide (.sync.aligned): every lane runs them; only
      // the shared- and global-memory accesses depend on the row.
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col = half * 64 + c * 32;
          const int owner = col / W, off = col - owner * W;
          if (owner == rank) continue;  // warp-uniform
          uint32_t v[32];
          __syncwarp();
          if (has_o) {
            tmem_ld32(tmem_o + lane_base + uint32_t(col), v);
            tmem_wait_ld(v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0u;
          }
          if (r < live) {
            uint8_t* slot = stage + (owner < rank ? owner : owner - 1) * slot_bytes;
            uint4* dst = reinterpret_cast<uint4*>(slot + kAttnRows * 8 + (r * pitch + off) * 4);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            if (off == 0) *reinterpret_cast<float2*>(slot + r * 8) = make_float2(m, lt);
          }
        }
      }
      fence_proxy_async();  // the staged slots are read by the bulk copies
      if (threadIdx.x == 0) mbar_arrive_expect_tx(smem_addr(xch_full), uint32_t(split - 1) * send_bytes);
      named_sync(1, kAttnSoftmaxWarps * 32);
      cluster_sync();  // every CTA of the cluster is done with its ring and expects its slots
      if (rec && threadIdx.x == 0) rec[3] = globaltimer_ns();
      if (threadIdx.x == 0) {
        for (int o = 0; o < split; ++o) {
          if (o == rank) continue;
          const int slot = rank < o ? rank : rank - 1;  // this CTA's slot in CTA o
          bulk_copy_to_cta(map_to_cta(smem_addr(recv + slot * slot_bytes), uint32_t(o)),
                           smem_addr(stage + (o < rank ? o : o - 1) * slot_bytes), send_bytes,
                           map_to_cta(smem_addr(xch_full), uint32_t(o)));
        }
      }
      int got = 1;
      if (lane == 0) got = wait_spin(smem_addr(xch_full), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      got = __shfl_sync(0xffffffffu, got, 0);
      cluster_arrive();  // this CTA's incoming slots have landed
      if (rec && threadIdx.x == 0) rec[7] = globaltimer_ns();
      if (ok && got) {
        auto slot_ml = [&](int k) { return reinterpret_cast<const float*>(recv + k * slot_bytes) + r * 2; };
        const bool row_live = r < live;
        float top = m;
        if (row_live)
          for (int k = 0; k < split - 1; ++k) top = fmaxf(top, slot_ml(k)[0]);
        const float safe = top == -INFINITY ? 0.f : top;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col = half * 64 + c * 32;
          if (col / W != rank) continue;  // warp-uniform
          const int off = col - rank * W;
#pragma unroll
          for (int hc = 0; hc < 2; ++hc) {  // 16 columns at a time: fewer live registers
            const int c16 = col + hc * 16;
            uint32_t v[16];
            __syncwarp();
            if (has_o) {
              tmem_ld16(tmem_o + lane_base + uint32_t(c16), v);
              tmem_wait_ld(v);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = 0u;
            }
            if (row_live) {
              float o[16], lsum = 0.f;
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = 0.f;
              for (int k = 0; k < split; ++k) {  // rank order
                const int slot = k < rank ? k : k - 1;
                const float mk = k == rank ? m : slot_ml(slot)[0];
                const float lk = k == rank ? lt : slot_ml(slot)[1];
                const float f = ex2_approx(mk - safe);
                lsum += lk * f;
                if (k == rank) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) o[i] += __uint_as_float(v[i]) * f;
                } else {
                  const float4* src = reinterpret_cast<const float4*>(recv + slot * slot_bytes + kAttnRows * 8 +
                                                                      (r * pitch + off + hc * 16) * 4);
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    const float4 x = src[i];
                    o[4 * i] += x.x * f;
                    o[4 * i + 1] += x.y * f;
                    o[4 * i + 2] += x.z * f;
                    o[4 * i + 3] += x.w * f;
                  }
                }
              }
              const float inv = 1.0f / (lsum > 0.f ? lsum : 1.0f);
#pragma unroll
              for (int i = 0; i < 16; i += 8)
                *reinterpret_cast<uint4*>(orow + c16 + i) =
                    make_uint4(bf2_pack(o[i] * inv, o[i + 1] * inv), bf2_pack(o[i + 2] * inv, o[i + 3] * inv),
                               bf2_pack(o[i + 4] * inv, o[i + 5] * inv), bf2_pack(o[i + 6] * inv, o[i + 7] * inv));
            }
          }
        }
      }
      cluster_wait();  // every slot of the cluster has landed: no copy still reads a CTA's staging
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
