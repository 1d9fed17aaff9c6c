// Weight-streaming tcgen05 GEMM for the small-row FFN of the WAMInfer video DiT.
//
// out[t, f] = epilogue( sum_k act[t, k] * weight[f, k] )
//
// The problem is "swap-AB": the weight rows (output features) sit on the UMMA
// M axis and the few hundred activation rows (tokens) sit on the UMMA N axis,
// so a CTA holds every token of its 128 features in TMEM (<= 512 fp32
// columns) and each weight tile is read from HBM exactly once.  Operands are
// staged by TMA with the 128-byte swizzle, K-major on both sides
// (torch.nn.Linear's native [out, in] weight layout and row-major activations).
//
// kGroup == 2 (the default for an even number of 128-feature tiles) runs the
// 2-SM UMMA: a cluster of two CTAs computes 256 features; each CTA stages its
// own 128 weight rows and HALF of the activation rows, the leader issues
// tcgen05.mma.cta_group::2 (M = 256) over both CTAs' shared memory, and each
// CTA's TMEM receives its 128 features x all tokens.  Every activation tile
// therefore crosses L2 once per 256 features instead of once per 128, and each
// SM buffers half as many activation bytes per stage.  No load uses cluster
// multicast: each CTA loads its own operands; only the MMA-completion commit
// is multicast to both CTAs' barriers.
//
// The two operands travel through separate shared-memory rings: a ring for
// the 16 KB weight tiles (HBM stream) and a ring for the activation tiles
// (re-read by every CTA pair, L2 hits).  Weights do not depend on the previous
// kernel, so under programmatic dependent launch the weight producer starts
// streaming before the previous kernel has finished; only the activation
// producer waits for it.
//
// Roles (384 threads per CTA):
//   warp 0      weight (A) TMA producer, one lane
//   warp 1      TMEM allocator + UMMA issuer (leader CTA), one lane
//   warp 2      activation (B) TMA producer, one lane
//   warp 3      idle
//   epilogue    all 12 warps once their roles are done: warp w reads TMEM
//               lanes 32*(w%4).. and every third 32-column chunk
// Grid: (n_total / 128, split_k, token groups), clusters of (kGroup, 1,
// token groups): the token groups of one weight tile sit in one cluster, so
// they stream the same weight tiles side by side and share them in L2.  With
// split_k > 1 each CTA covers a contiguous range of K blocks and writes an
// fp32 partial; a row kernel sums the partials in split order
// (deterministic, no atomics).
//
// Stream-K (p.sk > 0, the bias/GELU epilogues): the feature tiles' K blocks
// form one sequence of sk_tiles x k_blocks work units, cut into p.sk equal
// ranges, one per CTA pair (grid.x = sk x kGroup), so every SM does the same
// share of the MMAs even when the tiles do not fill the machine (56 pairs of
// 256 features on 74 SM pairs for the FFN up projection).  A range touches at
// most two tiles: the start of tile b (a helper piece) and the end of tile a
// (the owner piece).  The CTA runs the helper piece first, dumps its fp32
// accumulator to its workspace slot [tokens][128] and raises its flag, then
// runs the owner piece into the freed TMEM; the owner's epilogue waits for
// the helpers of its tile (lower CTA pairs, launched earlier, so the waits
// cannot deadlock) and adds their slots in K order before its own
// accumulator, bias and GELU.  The summation order is fixed, so results are
// deterministic (not bit-equal to the data-parallel grid).
#pragma once

#include "ptx.cuh"
#include "wamffn.h"

namespace wamffn {

enum : int { EPI_GELU_BF16 = 0, EPI_BIAS_BF16 = 1, EPI_PARTIAL_F32 = 2 };

constexpr int kFeatTile = 128;         // feature rows per CTA (UMMA M per CTA)
constexpr int kBlockK = 64;            // bf16 elements per 128-byte swizzled row
constexpr int kGemmThreads = 384;
constexpr int kEpiWarp0 = 4;           // first epilogue warp
constexpr int kMaxTokens = 512;        // TMEM holds 512 fp32 columns
constexpr int kMaxAStages = 16;
constexpr int kMaxBStages = 8;
constexpr int kSmemLimit = 232448;     // 227 KB opt-in dynamic shared memory
constexpr int kSmemReserve = 1024 + 512;  // alignment slack + barriers
// Shared memory the GEMM's rings leave unused so that one row-kernel CTA (a
// 3072-wide fp32 row, 12 KB, plus its own reservation) fits on the SM beside a
// GEMM CTA: concurrent request lanes then run layer-boundary rows on the SMs
// whose GEMM CTA is waiting on its tensor pipe.
constexpr int kGemmRowSlack = 14 * 1024;

struct GemmParams {
  int tokens;        // real activation rows (all token groups)
  int group_rows;    // rows per token group (grid.z); == tokens with one group
  int tok_pad;       // tokens rounded up to the MMA granularity
  int mma_n0;        // N of the first UMMA (<= 256, multiple of 16)
  int mma_n1;        // N of the second UMMA (0 when one suffices)
  int tok_box;       // activation rows per TMA box (per CTA)
  int n_boxes;       // TMA boxes per stage for the activation tile
  int b_rows;        // activation rows per stage held by one CTA
  int k_blocks;      // K / 64
  int splits;        // split-K factor == gridDim.y
  int a_stages;      // weight ring depth
  int b_stages;      // activation ring depth
  int n_total;       // output features (row length of the output)
  uint32_t tmem_cols;
  int epi;
  int w_packed;      // weights in the tile-packed layout (one 16 KB block per tile)
  const __nv_bfloat16* bias;
  void* out;
  unsigned int* status;
  int sk;                   // stream-K CTA pairs (0: data-parallel grid)
  int sk_tiles;             // feature tiles of 128 x kGroup features
  float* sk_ws;             // [sk * kGroup][tok_pad][128] fp32 helper slots
  unsigned int* sk_flags;   // [sk * kGroup]: 1 while a helper slot holds an unread partial
};

constexpr int kMaxSkHelpers = 4;  // helper pieces one owner tile may sum (host-checked)

// The stream-K range of CTA pair `pair`: units [u0, u1) of sk_tiles x k_blocks.
__device__ __forceinline__ long long sk_unit(const GemmParams& p, long long pair) {
  return (long long)p.sk_tiles * p.k_blocks * pair / p.sk;
}

__host__ __device__ constexpr int gemm_a_bytes() { return kFeatTile * kBlockK * 2; }

// Optional phase trace (off unless wamffn_trace_enable registered a buffer):
// record = {tag, start, operands ready, MMAs issued, accumulator ready,
// epilogue done, sm id, k blocks}; globaltimer nanoseconds.
constexpr int kTraceWords = 8;
constexpr unsigned int kTraceBoundary = 7;  // record tag of the layer-boundary kernel
__device__ unsigned long long* g_trace = nullptr;
__device__ unsigned int g_trace_capacity = 0;

__device__ __forceinline__ uint32_t smid() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

// Stream-K helper dump: this warp's TMEM lane quarter (32 features) of the
// accumulator, 32-token chunks grp, grp + ngroups, ..., into a helper slot
// laid out [token][128 features] (slot_q already offset to the thread's
// feature); kept in L2 for the owner that reads it shortly after.
__device__ __forceinline__ void sk_dump(uint32_t lane_addr, float* slot_q, int grp, int ngroups, int tokens) {
  const uint64_t keep = l2_policy_evict_last();
  const int nchunks = (tokens + 31) >> 5;
  for (int c = grp; c < nchunks; c += ngroups) {
    uint32_t r[32];
    tmem_ld32(lane_addr + uint32_t(c * 32), r);
    tmem_wait_ld(r);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int t = c * 32 + i;
      if (t < tokens) st_global_keep(slot_q + size_t(t) * kFeatTile, __uint_as_float(r[i]), keep);
    }
  }
}

template <int kGroup, bool kSK>
__global__ void __launch_bounds__(kGemmThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Clusters are (kGroup, 1, token groups): CTAs 2k and 2k+1 form a UMMA pair.
  const uint32_t rank = kGroup == 2 ? cluster_ctarank() : 0u;
  const uint32_t pair_rank = rank & 1u;
  const uint32_t leader_rank = rank & ~1u;
  const bool leader = pair_rank == 0;
  const uint16_t pair_mask = uint16_t(0x3u << leader_rank);
  // This CTA's token group.
  const int tok_base = blockIdx.z * p.group_rows;
  const int tokens = min(p.group_rows, p.tokens - tok_base);

  const int a_bytes = gemm_a_bytes();
  const int b_bytes = p.b_rows * kBlockK * 2;
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + p.a_stages * a_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_base + p.b_stages * b_bytes);
  uint64_t* full_a = bars;
  uint64_t* empty_a = full_a + p.a_stages;
  uint64_t* full_b = empty_a + p.a_stages;
  uint64_t* empty_b = full_b + p.b_stages;
  // tmem_full[q]: piece q's accumulator is complete (each barrier completes
  // once per launch, so every wait is on parity 0 whenever a warp arrives).
  uint64_t* tmem_full = empty_b + p.b_stages;
  uint64_t* tmem_empty = tmem_full + 2;  // stream-K: the helper piece's accumulator was dumped
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  unsigned int* trace_slot = reinterpret_cast<unsigned int*>(tmem_slot + 2);

  const int split = blockIdx.y;
  // The CTA's pieces in processing order (piece 1 only with stream-K): K
  // blocks [beg, end) of 128-feature tile ftile.  The last piece is the owner
  // piece (epilogue) unless it stops short of its tile's last K block.
  int ft0, beg0, end0, ft1 = 0, beg1 = 0, end1 = 0;
  int npieces = 1;
  int sk_pair = 0, sk_first_helper = 0, sk_helpers = 0;
  if constexpr (!kSK) {
    ft0 = blockIdx.x;
    beg0 = int((long long)p.k_blocks * split / p.splits);
    end0 = int((long long)p.k_blocks * (split + 1) / p.splits);
  } else {
    sk_pair = int(blockIdx.x) / kGroup;
    const int r = int(blockIdx.x) % kGroup;
    const long long u0 = sk_unit(p, sk_pair), u1 = sk_unit(p, sk_pair + 1);
    const int ta = int(u0 / p.k_blocks);
    const int a_beg = int(u0 - (long long)ta * p.k_blocks);
    if (u1 > (long long)(ta + 1) * p.k_blocks) {
      ft0 = (ta + 1) * kGroup + r;  // start of the next tile: helper piece first
      beg0 = 0;
      end0 = int(u1 - (long long)(ta + 1) * p.k_blocks);
      ft1 = ta * kGroup + r;
      beg1 = a_beg;
      end1 = p.k_blocks;
      npieces = 2;
    } else {
      ft0 = ta * kGroup + r;
      beg0 = a_beg;
      end0 = int(u1 - (long long)ta * p.k_blocks);
    }
    const int last_beg = npieces == 2 ? beg1 : beg0, last_end = npieces == 2 ? end1 : end0;
    if (last_end == p.k_blocks && last_beg > 0) {
      // Helpers of the owner tile: the pairs whose ranges hold its K blocks [0, kb_begin).
      const long long first_unit = (long long)ta * p.k_blocks;
      int f = int(first_unit * p.sk / ((long long)p.sk_tiles * p.k_blocks));
      while (f > 0 && sk_unit(p, f) > first_unit) --f;
      while (sk_unit(p, f + 1) <= first_unit) ++f;
      sk_first_helper = f;
      sk_helpers = sk_pair - f;
    }
  }
  const bool owner = !kSK || (npieces == 2 ? end1 : end0) == p.k_blocks;
  const int n0 = (npieces == 2 ? ft1 : ft0) * kFeatTile;  // feature rows of the final piece
  const int nkb = (end0 - beg0) + (end1 - beg1);          // K blocks over all pieces

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.a_stages; ++s) {
      mbar_init(smem_addr(&full_a[s]), 1);
      mbar_init(smem_addr(&empty_a[s]), 1);
    }
    for (int s = 0; s < p.b_stages; ++s) {
      mbar_init(smem_addr(&full_b[s]), 1);
      mbar_init(smem_addr(&empty_b[s]), 1);
    }
    mbar_init(smem_addr(&tmem_full[0]), 1);
    mbar_init(smem_addr(&tmem_full[1]), 1);
    mbar_init(smem_addr(tmem_empty), kGroup);  // one arrival per CTA of the pair (leader's barrier)
    *abort_flag = 0;
    *trace_slot = 0xffffffffu;
    if (g_trace != nullptr) {
      const unsigned int slot = atomicAdd(reinterpret_cast<unsigned int*>(g_trace), 1u);
      if (slot + 1 < g_trace_capacity) {
        *trace_slot = slot + 1;
        unsigned long long* rec = g_trace + size_t(slot + 1) * kTraceWords;
        rec[0] = (unsigned long long)(blockIdx.x | (blockIdx.y << 16)) | ((unsigned long long)p.epi << 32);
        rec[1] = globaltimer_ns();
        rec[6] = smid();
        rec[7] = (unsigned long long)nkb;
      }
    }
    fence_mbar_init();
    prefetch_tensormap(&tm_w);
    prefetch_tensormap(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc_g<kGroup>(smem_addr(tmem_slot), p.tmem_cols);
    tmem_relinquish_g<kGroup>();
  }
  tc_fence_before();
  // Both CTAs' barriers must be initialised before either signals the other.
  if constexpr (kGroup == 2) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 || warp == 2) {
    // -------------------------------------------------------------- producers
    // The whole warp runs the loop (warp-uniform operands); one elected lane
    // issues the barrier arrive and the TMA copies.
    const bool weights = warp == 0;
    const int stages = weights ? p.a_stages : p.b_stages;
    uint64_t* full = weights ? full_a : full_b;
    uint64_t* empty = weights ? empty_a : empty_b;
    uint8_t* ring = weights ? a_base : b_base;
    const int bytes = weights ? a_bytes : b_bytes;
    // Weights stream once (evict first); activations are re-read by every CTA.
    const uint64_t policy = weights ? l2_policy_evict_first() : l2_policy_evict_last();
    // Only the activations depend on the previous kernel in the stream.
    if (!weights) pdl_wait_prior();
    int issued = 0;
    int kb = beg0, ftile = ft0;
    for (int i = 0; i < nkb; ++i, ++kb) {
      if (kSK && kb == end0 && ftile == ft0 && npieces == 2) {
        kb = beg1;
        ftile = ft1;
      }
      const int s = i % stages;
      const uint32_t ph = uint32_t(i / stages) & 1u;
      // One lane polls; the verdict is broadcast so the warp stays converged.
      int ok = 1;
      if (lane == 0) ok = wait_bounded(smem_addr(&empty[s]), ph ^ 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if (elect_one()) {
        const uint32_t local_full = smem_addr(&full[s]);
        // The leader's barrier counts both CTAs' bytes; the peer only adds its copies.
        const uint32_t fb = kGroup == 2 ? map_to_cta(local_full, leader_rank) : local_full;
        if (leader) mbar_arrive_expect_tx(local_full, uint32_t(bytes * kGroup));
        const int kx = kb * kBlockK;
        if (weights) {
          // Packed weights: tile (feature tile, k block) is rows [t*128, t*128+128) of a [*, 64] matrix.
          const int c0 = p.w_packed ? 0 : kx;
          const int c1 = p.w_packed ? (ftile * p.k_blocks + kb) * kFeatTile : ftile * kFeatTile;
          if constexpr (kGroup == 2) tma_load_2d_pair(smem_addr(ring + s * bytes), &tm_w, fb, c0, c1, policy);
          else tma_load_2d(smem_addr(ring + s * bytes), &tm_w, fb, c0, c1, policy);
        } else {
          for (int b = 0; b < p.n_boxes; ++b) {
            const uint32_t dst = smem_addr(ring + s * bytes + b * p.tok_box * kBlockK * 2);
            if constexpr (kGroup == 2) {
              // Box b feeds UMMA b: this CTA holds its rank's half of that UMMA's tokens.
              const int row = b == 0 ? int(pair_rank) * (p.mma_n0 / 2) : p.mma_n0 + int(pair_rank) * (p.mma_n1 / 2);
              tma_load_2d_pair(dst, &tm_x, fb, kx, tok_base + row, policy);
            } else {
              tma_load_2d(dst, &tm_x, fb, kx, tok_base + b * p.tok_box, policy);
            }
          }
        }
      }
      __syncwarp();
      issued = i + 1;
    }
    if (*abort_flag && lane == 0) {
      // Let the copies already in flight land before the CTA releases its
      // shared memory (the peer's copies complete on the leader's barrier,
      // so the peer just waits a bounded moment).
      if (kGroup == 1 || leader) {
        const int first = issued > stages ? issued - stages : 0;
        for (int i = first; i < issued; ++i) wait_drain(smem_addr(&full[i % stages]), uint32_t(i / stages) & 1u);
      } else {
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000ll) {
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- UMMA issuer
    // The whole warp runs the loop; the elected lane issues the MMAs and the
    // commits (a commit tracks the MMAs issued by the same thread).
    if (leader) {
      unsigned long long* rec =
          *trace_slot != 0xffffffffu ? g_trace + size_t(*trace_slot) * kTraceWords : nullptr;
      const int m = kFeatTile * kGroup;
      const uint32_t idesc0 = umma_idesc_bf16(m, p.mma_n0);
      const uint32_t idesc1 = umma_idesc_bf16(m, p.mma_n1 > 0 ? p.mma_n1 : 16);
      // Rows of UMMA 0's activation slice held by this CTA.
      const uint32_t b1_offset = uint32_t(p.mma_n0 / kGroup) * 128u;
      const uint32_t a0 = smem_addr(a_base), b0 = smem_addr(b_base);
      int piece = 0, kb = beg0;
      for (int i = 0; i < nkb; ++i, ++kb) {
        const int sa = i % p.a_stages, sb = i % p.b_stages;
        int ok = 1;
        if (kSK && piece == 0 && kb == end0) {
          // Stream-K: the helper piece is complete.  Release its accumulator to
          // the dump, and start the owner piece once both CTAs have dumped it.
          if (elect_one()) {
            if constexpr (kGroup == 2) umma_commit_pair(smem_addr(&tmem_full[piece]), pair_mask);
            else umma_commit(smem_addr(&tmem_full[piece]));
          }
          __syncwarp();
          piece = 1;
          kb = beg1;
          if (lane == 0)
            ok = wait_bounded(smem_addr(tmem_empty), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
          if (!__shfl_sync(0xffffffffu, ok, 0)) break;
          tc_fence_after();
        }
        const bool first_k = kb == (piece == 0 ? beg0 : beg1);
        if (lane == 0)
          ok = wait_bounded(smem_addr(&full_a[sa]), uint32_t(i / p.a_stages) & 1u, abort_flag, p.status,
                            WAMFFN_DEV_TIMEOUT) &&
               wait_bounded(smem_addr(&full_b[sb]), uint32_t(i / p.b_stages) & 1u, abort_flag, p.status,
                            WAMFFN_DEV_TIMEOUT);
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        tc_fence_after();
        if (i == 0 && rec && lane == 0) rec[2] = globaltimer_ns();
        const uint64_t adesc = umma_desc_sw128(a0 + uint32_t(sa * a_bytes));
        const uint64_t bdesc0 = umma_desc_sw128(b0 + uint32_t(sb * b_bytes));
        const uint64_t bdesc1 = umma_desc_sw128(b0 + uint32_t(sb * b_bytes) + b1_offset);
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k) {
            const uint32_t acc = (!first_k || k > 0) ? 1u : 0u;
            if constexpr (kGroup == 2) {
              umma_bf16_pair(tmem_base, adesc + 2 * k, bdesc0 + 2 * k, idesc0, acc);
              if (p.mma_n1 > 0)
                umma_bf16_pair(tmem_base + uint32_t(p.mma_n0), adesc + 2 * k, bdesc1 + 2 * k, idesc1, acc);
            } else {
              umma_bf16(tmem_base, adesc + 2 * k, bdesc0 + 2 * k, idesc0, acc);
              if (p.mma_n1 > 0)
                umma_bf16(tmem_base + uint32_t(p.mma_n0), adesc + 2 * k, bdesc1 + 2 * k, idesc1, acc);
            }
          }
          // Free both stages (in both CTAs) once these MMAs have read them.
          if constexpr (kGroup == 2) {
            umma_commit_pair(smem_addr(&empty_a[sa]), pair_mask);
            umma_commit_pair(smem_addr(&empty_b[sb]), pair_mask);
          } else {
            umma_commit(smem_addr(&empty_a[sa]));
            umma_commit(smem_addr(&empty_b[sb]));
          }
        }
        __syncwarp();
      }
      // Accumulator complete (or pipeline aborted): release the epilogues.
      if (elect_one()) {
        if constexpr (kGroup == 2) umma_commit_pair(smem_addr(&tmem_full[npieces - 1]), pair_mask);
        else umma_commit(smem_addr(&tmem_full[npieces - 1]));
      }
      __syncwarp();
      if (rec && lane == 0) rec[3] = globaltimer_ns();
    }
    // The next kernel may start its prologue (and its weight stream) now.
    if (lane == 0) pdl_launch_dependents();
  }

  // ------------------------------------------------- stream-K helper dump
  // With two pieces the first is a helper piece: warps 4..11 (two per TMEM
  // lane quarter) dump its accumulator while the roles keep streaming the
  // owner piece's operands, publish the slot, and free TMEM for the owner
  // piece's MMAs (the leader's tmem_empty counts one arrival per CTA).
  float* my_slot = kSK ? p.sk_ws + size_t(sk_pair * kGroup + int(pair_rank)) * p.tok_pad * kFeatTile : nullptr;
  if (kSK && npieces == 2 && warp >= kEpiWarp0) {
    const int q = warp & 3;
    int ok = 0;
    if (lane == 0)
      ok = wait_bounded(smem_addr(&tmem_full[0]), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT) && !*abort_flag;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    tc_fence_after();
    if (ok)
      sk_dump(tmem_base + (uint32_t(q * 32) << 16), my_slot + q * 32 + lane, (warp - kEpiWarp0) >> 2, 2, tokens);
    tc_fence_before();
    named_sync(2, kGemmThreads - kEpiWarp0 * 32);
    if (warp == kEpiWarp0 && lane == 0) {
      if (ok) {
        __threadfence();
        st_release_gpu(&p.sk_flags[sk_pair * kGroup + int(pair_rank)], 1u);
      }
      mbar_arrive_remote(map_to_cta(smem_addr(tmem_empty), leader_rank));
    }
  }

  // ---------------------------------------------------------------- epilogue
  // All 12 warps (producer and issuer warps join once their loops are done):
  // warp w reads TMEM lanes 32*(w%4).. (its 32 features) and takes every third
  // 32-column (token) chunk, starting at chunk w/4.
  {
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int group = warp >> 2;          // 0..2
    // One lane waits; the verdict is broadcast so the .sync.aligned TMEM loads
    // below are executed by all 32 lanes or by none.
    int ok = 0;
    if (lane == 0)
      ok = wait_bounded(smem_addr(&tmem_full[npieces - 1]), 0u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT) &&
           !*abort_flag;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    tc_fence_after();
    unsigned long long* rec =
        (warp == kEpiWarp0 && lane == 0 && *trace_slot != 0xffffffffu) ? g_trace + size_t(*trace_slot) * kTraceWords
                                                                       : nullptr;
    if (rec) rec[4] = globaltimer_ns();
    // Stream-K owner: the helper slots of this tile must be complete.
    const int nh = (kSK && ok && owner) ? sk_helpers : 0;
    if (nh > 0) {
      if (lane == 0) {
        const long long t0 = clock64();
        for (int h = 0; h < nh && ok; ++h) {
          const unsigned int* flag = &p.sk_flags[(sk_first_helper + h) * kGroup + int(pair_rank)];
          while (ld_acquire_gpu(flag) == 0u) {
            if (*abort_flag) { ok = 0; break; }
            if (clock64() - t0 > kWaitLimitCycles) {
              *abort_flag = 1;
              atomicOr(p.status, WAMFFN_DEV_TIMEOUT);
              ok = 0;
              break;
            }
            __nanosleep(64);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (kSK && ok && !owner) {
      // A CTA whose only piece is a helper piece: all 12 warps dump it.
      sk_dump(tmem_base + (uint32_t(q * 32) << 16), my_slot + q * 32 + lane, group, 3, tokens);
    } else if (ok) {
      const int f = n0 + q * 32 + lane;
      const int nchunks = (tokens + 31) >> 5;
      const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
      if (p.epi == EPI_PARTIAL_F32) {
        // Partials are re-read once by the split-K reduction: keep them in L2.
        const uint64_t keep = l2_policy_evict_last();
        float* out = reinterpret_cast<float*>(p.out) + (size_t(split) * p.tokens + tok_base) * p.n_total + f;
        for (int c = group; c < nchunks; c += 3) {
          uint32_t r[32];
          tmem_ld32(lane_addr + uint32_t(c * 32), r);
          tmem_wait_ld(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = c * 32 + i;
            if (t < tokens) st_global_keep(out + size_t(t) * p.n_total, __uint_as_float(r[i]), keep);
          }
        }
      } else {
        // bf16 output through a per-warp shared-memory transpose so that each
        // thread writes 16 contiguous bytes of one token row.  The weight ring
        // is idle once the accumulator is complete, so its first 24 KB hold the
        // transpose tile of every warp.
        const float bias = __bfloat162float(p.bias[f]);
        __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(smem) + warp * (32 * 32);
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
        const int n_base = n0 + q * 32;
        // Helper slots of this thread's feature, in K order.
        const float* hslot = nh > 0 ? p.sk_ws + size_t(sk_first_helper * kGroup + int(pair_rank)) * p.tok_pad * kFeatTile +
                                          q * 32 + lane
                                    : nullptr;
        const size_t hstride = size_t(kGroup) * p.tok_pad * kFeatTile;
        // 16-column chunks: the GELU math keeps 16 values in flight per thread
        // (32 measured slower: the longer dependency chains do not overlap).
        const int nchunks16 = (tokens + 15) >> 4;
        // Software pipeline: the TMEM load of the next chunk is in flight
        // while this chunk's GELU runs.
        uint32_t nxt[16];
        if (group < nchunks16) tmem_ld16(lane_addr + uint32_t(group * 16), nxt);
        for (int c = group; c < nchunks16; c += 3) {
          // Helper partials of this chunk (stream-K owner): summed in K order.
          float hsum[16];
          if (kSK && nh > 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int t = min(c * 16 + i, tokens - 1);
              hsum[i] = __ldcg(hslot + size_t(t) * kFeatTile);
            }
            for (int h = 1; h < nh; ++h) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int t = min(c * 16 + i, tokens - 1);
                hsum[i] += __ldcg(hslot + h * hstride + size_t(t) * kFeatTile);
              }
            }
          }
          tmem_wait_ld(nxt);
          uint32_t r[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) r[i] = nxt[i];
          if (c + 3 < nchunks16) tmem_ld16(lane_addr + uint32_t((c + 3) * 16), nxt);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float acc = __uint_as_float(r[i]);
            if (kSK && nh > 0) acc = hsum[i] + acc;
            float v = acc + bias;
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
            if (t < tokens) *reinterpret_cast<uint4*>(&out[size_t(tok_base + t) * p.n_total + n_base + col]) = v;
          }
          __syncwarp();
        }
      }
    }
    if constexpr (kSK) {
      // Publish a helper-only CTA's slot; an owner clears the flags it consumed
      // (no later reader in this launch; the next launch's helpers set them
      // again only after this launch has completed).
      tc_fence_before();
      named_sync(1, kGemmThreads);
      if (warp == kEpiWarp0 && lane == 0 && ok) {
        if (!owner) {
          __threadfence();
          st_release_gpu(&p.sk_flags[sk_pair * kGroup + int(pair_rank)], 1u);
        }
        for (int h = 0; h < nh; ++h) p.sk_flags[(sk_first_helper + h) * kGroup + int(pair_rank)] = 0u;
      }
    }
  }
  if (warp == kEpiWarp0 && lane == 0 && *trace_slot != 0xffffffffu)
    g_trace[size_t(*trace_slot) * kTraceWords + 5] = globaltimer_ns();
  tc_fence_before();
  // No CTA of a pair may leave while its peer can still signal its barriers.
  if constexpr (kGroup == 2) cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_g<kGroup>(tmem_base, p.tmem_cols);
  }
}

}  // namespace wamffn
