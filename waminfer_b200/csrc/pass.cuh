// Persistent FFN pass: one launch runs every layer of a wamffn_stack_run pass
// (the FFN phases of the 30 WAMInfer video-DiT blocks, WAMInfer/blocks.py:239-271).
//
// The multi-kernel stack launches three kernels per layer (up GEMM, down GEMM,
// layer boundary); every launch boundary costs a drain of the previous grid,
// a refill of the next one's pipeline and a setup.  Here one CTA per SM (pairs
// of CTAs in 2-SM UMMA clusters) stays resident for the whole pass and walks
// the same phases, separated by grid-wide barriers:
//
//   R(l)  row phase: split-K reduction + bias of layer l-1's down projection,
//         history scatter, gated residual, layer l's LayerNorm + adaLN + row
//         gather (for l = 0: the input's norm + gather; for l = L: the final
//         residual only)                                 -> arrive R(l)
//   U(l)  up items: [256 features x all rows] UMMA tiles, K = d, GELU epilogue
//         into the hidden buffer                        -> arrive U(l)
//   D(l)  down items: [256 features x all rows] UMMA tiles over one K slice of
//         h, fp32 partials                              -> arrive D(l)
//
// Weights do not depend on any phase, so the weight producer streams without
// ever waiting on a grid barrier: while a CTA is in its GELU epilogue, a grid
// barrier or a row phase, its weight ring already fills with the next phase's
// tiles.  Only the activation producer waits for R(l) (before the up items)
// and U(l) (before the down items); the row workers wait for D(l-1).
//
// Roles (512 threads):
//   warp 0        weight TMA producer
//   warp 1        TMEM owner (512 columns for the whole pass) + UMMA issuer (leader CTA)
//   warp 2        activation TMA producer
//   warp 3        idle
//   warps 4..15   GEMM epilogues (warp w reads TMEM lanes 32*(w%4).., every third
//                 column chunk) and the row phases (one row at a time, thread t
//                 owning the row's 16-byte vector t, as in the row kernels)
//
// The arithmetic is the multi-kernel stack's, operation for operation: the
// same UMMA sequence per tile, the same split-K slices and reduction order, and
// row reductions that add in the order of the 384-thread row kernels, so a
// pass is bit-identical to the three-kernel stack.
//
// Every wait is bounded: a pipeline wait that runs out, or a grid barrier that
// does not complete, raises the CTA's abort flag and the pass-wide abort word
// and sets WAMFFN_DEV_TIMEOUT; all roles then leave their loops.
#pragma once

#include "gemm.cuh"
#include "rowops.cuh"

namespace wamffn {

constexpr int kPassThreads = 512;
constexpr int kPassMaxLayers = 48;
constexpr int kPassEpiThreads = 384;   // warps 4..15
constexpr int kPassEpiBarrier = 1;     // named barrier of the epilogue warps
constexpr int kPassTransposeBytes = 12 * 32 * 32 * 2;  // per-warp bf16 transpose tiles
constexpr uint32_t kPassTmemCols = 512;
constexpr int kPassRowSlots = 4;       // rows per CTA: max(seq, rows) <= 4 * CTAs; d <= 8 * 384

// GEMM geometry of one row count (the pass has at most two: all rows, gathered rows).
struct PassClass {
  int rows, tok_pad, mma_n0, mma_n1, tok_box, n_boxes, b_rows;
};

struct PassParams {
  CUtensorMap tm_w_up[kPassMaxLayers];
  CUtensorMap tm_w_down[kPassMaxLayers];
  CUtensorMap tm_act[2];  // gathered activations [rows, d], per class
  CUtensorMap tm_hid[2];  // hidden activations [rows, h], per class
  const __nv_bfloat16* b_up[kPassMaxLayers];
  const __nv_bfloat16* b_down[kPassMaxLayers];
  const __nv_bfloat16* mod[kPassMaxLayers];  // block.modulation [6, d]
  PassClass cls[2];
  int layers, d, h, seq;
  int first_gathered;  // layers >= first_gathered run on the gathered rows (class 1)
  int w_packed;
  int up_tiles;        // h / 256
  int down_tiles;      // d / 256
  int down_splits;
  int a_stages, b_stages, b_stage_bytes, b_region_bytes;
  const __nv_bfloat16* x;     // [seq, d] pass input
  const __nv_bfloat16* time;  // per-row time modulation, row stride ts
  long long ts;
  __nv_bfloat16* y;           // [seq, d] residual stream
  __nv_bfloat16* gathered;    // [rows, d] GEMM input of the up projection
  __nv_bfloat16* hidden;      // [rows, h]
  float* partial;             // [down_splits, rows, d]
  const void* idx;            // gather list of the gathered layers (cls[1].rows entries)
  int idx_bytes;
  int cache_rows;
  const __nv_bfloat16* cache_in;  // [layers - first_gathered, cache_rows, d] or null
  __nv_bfloat16* cache_out;
  __nv_bfloat16* x_out;       // [seq, d] pass output
  float eps;
  unsigned int* bars;         // [3 * layers] phase counters, then the abort word; zero at launch
  unsigned int* status;
};

__device__ __forceinline__ int pass_class(const PassParams& p, int l) { return l >= p.first_gathered ? 1 : 0; }

// Optional timeline (wamffn_trace_enable): record 1 + (cta * 3 L + 3 l + phase)
// holds {tag, t1..t5, t6, sm id} for phase R / U / D of layer l, written by
// the roles that own each time stamp (globaltimer ns).
__device__ __forceinline__ unsigned long long* pass_trace(const PassParams& p, int l, int phase) {
  if (g_trace == nullptr) return nullptr;
  const unsigned int slot = 1u + (blockIdx.x * 3u * unsigned(p.layers + 1) + 3u * unsigned(l) + unsigned(phase));
  if (slot >= g_trace_capacity) return nullptr;
  return g_trace + size_t(slot) * kTraceWords;
}

__device__ __forceinline__ void pass_raise_abort(const PassParams& p, volatile int* abort) {
  *abort = 1;
  atomicExch(p.bars + 3 * p.layers, 1u);
}

// Publishes this CTA's writes of a phase (issued by threads that synchronised
// with the caller beforehand) and counts the CTA in the phase's barrier.
__device__ __forceinline__ void pass_arrive(unsigned int* counter) {
  __threadfence();
  fence_proxy_async_global();
  atomicAdd(counter, 1u);
}

// Waits until `counter` reaches `target` (every CTA arrived), or gives up on
// an abort / after kWaitLimitCycles.  Afterwards this thread's later reads, the
// TMA loads it issues included, see every write published by the arrivals.
__device__ __forceinline__ bool pass_wait(const PassParams& p, const unsigned int* counter, unsigned int target,
                                          volatile int* abort) {
  const unsigned int* global_abort = p.bars + 3 * p.layers;
  const long long t0 = clock64();
  while (ld_acquire_gpu(counter) < target) {
    if (*abort || *reinterpret_cast<const volatile unsigned int*>(global_abort)) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      atomicOr(p.status, WAMFFN_DEV_TIMEOUT);
      pass_raise_abort(p, abort);
      return false;
    }
    __nanosleep(32);
  }
  fence_proxy_async_global();
  return true;
}

// Sum over the 12 epilogue warps in the order of block_sum (rowops.cuh): a
// shuffle tree per warp, then the warps in index order; warps beyond the
// row's vectors contribute zeros, as the row kernels' missing warps do.
__device__ __forceinline__ float pass_row_sum(float v, float* red, int nwarps) {
  const int lane = threadIdx.x & 31;
  const int ew = (threadIdx.x >> 5) - 4;  // epilogue warp 0..11
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  named_sync(kPassEpiBarrier, kPassEpiThreads);  // red[] may still be read by a previous reduction
  if (lane == 0) red[ew] = v;
  named_sync(kPassEpiBarrier, kPassEpiThreads);
  float total = 0.f;
  for (int w = 0; w < nwarps; ++w) total += red[w];
  return total;
}

// Gather bookkeeping of one row slot of this CTA, computed once per pass
// (the gather list is an input of the whole pass): the last entry of the list
// naming the row (its GEMM row in a gathered layer), the entries naming it
// (the slots its normalised row is copied to) and whether the list entry at
// index r itself is invalid (that slot is zero-filled).
struct PassRowSlot {
  int j_idx;
  int n_match;
  int bad_slot;
  int matches[kMaxMatches];
};

__device__ void pass_row_setup(const PassParams& p, int r, int et, PassRowSlot* slot) {
  const int m = p.cls[1].rows;
  if (et == 0) {
    slot->j_idx = -1;
    slot->n_match = 0;
    slot->bad_slot = 0;
  }
  named_sync(kPassEpiBarrier, kPassEpiThreads);
  if (p.idx != nullptr) {
    if (et == 0 && r < m) {
      const long long v = load_index(p.idx, p.idx_bytes, r);
      if (v < 0 || v >= p.seq) {
        slot->bad_slot = 1;
        if (v != -1) atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
      }
    }
    if (r < p.seq) {
      for (int j = et; j < m; j += kPassEpiThreads) {
        if (load_index(p.idx, p.idx_bytes, j) == r) {
          atomicMax(&slot->j_idx, j);
          const int k = atomicAdd(&slot->n_match, 1);
          if (k < kMaxMatches) slot->matches[k] = j;
          else atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
        }
      }
    }
  }
  named_sync(kPassEpiBarrier, kPassEpiThreads);
  // A gathered layer neither computes nor caches this row: its FFN output is undefined.
  if (et == 0 && p.idx != nullptr && p.first_gathered < p.layers && r < p.seq && slot->j_idx < 0 &&
      r >= p.cache_rows)
    atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
}

// One row (or gather slot) `r` of phase R(l) by the 384 epilogue threads:
// thread et owns the 16-byte vector et of the row, as in the row kernels, so
// every value and every reduction matches the three-kernel stack bit for bit.
__device__ void pass_row(const PassParams& p, int l, int r, int et, float* red, const PassRowSlot* slot) {
  const int d = p.d;
  const int nvec = d >> 3;
  const bool has_next = l < p.layers;   // a layer follows: norm + gather for it
  const bool has_prev = l > 0;          // a layer precedes: reduce its down projection
  const bool next_gathered = has_next && l >= p.first_gathered;
  const int next_m = has_next ? p.cls[pass_class(p, l)].rows : 0;
  const bool cur_gathered = has_prev && l - 1 >= p.first_gathered;
  const int cur_m = has_prev ? p.cls[pass_class(p, l - 1)].rows : 0;
  const bool active = et < nvec;
  const int e = et * 8;

  // Invalid entries of the next layer's list: the GEMM reads zeros there.
  if (next_gathered && r < next_m && slot->bad_slot && active)
    *reinterpret_cast<uint4*>(p.gathered + size_t(r) * d + e) = make_uint4(0, 0, 0, 0);
  if (r >= p.seq) return;
  const int row = r;
  const int j = !has_prev ? row : (cur_gathered ? slot->j_idx : (row < cur_m ? row : -1));
  const bool cached_row = cur_gathered && row < p.cache_rows;

  float x[8];
  float local = 0.f;
  if (active) {
    if (!has_prev) {
      load8(p.x + size_t(row) * d + e, x);
      store8(p.y + size_t(row) * d + e, x);
    } else {
      // Independent loads: the residual, the gate's modulation and time rows,
      // the bias, then the partials three splits at a time (register budget).
      const int lp = l - 1;
      const size_t slot_off = cur_gathered ? size_t(lp - p.first_gathered) * p.cache_rows * d : 0;
      const uint4 y_pk = *reinterpret_cast<const uint4*>(p.y + size_t(row) * d + e);
      const uint4 g_pk = modulation8_packed(p.mod[lp], p.time, p.ts, row, 5, d, e);
      float o[8];
      if (j >= 0) {
        const uint4 b_pk = *reinterpret_cast<const uint4*>(p.b_down[lp] + e);
        const float* base = p.partial + size_t(j) * d + e;
        const size_t split_stride = size_t(cur_m) * d;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int s0 = 0; s0 < p.down_splits; s0 += 3) {
          float4 part[3][2];
#pragma unroll
          for (int s = 0; s < 3; ++s) {
            if (s0 + s < p.down_splits) {
              const float4* src = reinterpret_cast<const float4*>(base + (s0 + s) * split_stride);
              part[s][0] = src[0];
              part[s][1] = src[1];
            }
          }
#pragma unroll
          for (int s = 0; s < 3; ++s) {
            if (s0 + s < p.down_splits) {
              acc[0] += part[s][0].x; acc[1] += part[s][0].y; acc[2] += part[s][0].z; acc[3] += part[s][0].w;
              acc[4] += part[s][1].x; acc[5] += part[s][1].y; acc[6] += part[s][1].z; acc[7] += part[s][1].w;
            }
          }
        }
        float bb[8];
        unpack8(b_pk, bb);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = bf16_round(acc[i] + bb[i]);
      } else if (cached_row && p.cache_in != nullptr) {
        load8(p.cache_in + slot_off + size_t(row) * d + e, o);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      }
      if (cached_row && p.cache_out != nullptr) store8(p.cache_out + slot_off + size_t(row) * d + e, o);
      float g[8], y[8];
      unpack8(g_pk, g);
      unpack8(y_pk, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = bf16_round(y[i] + bf16_round(g[i] * o[i]));
      store8((has_next ? p.y : p.x_out) + size_t(row) * d + e, x);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) local = __fadd_rn(local, x[i]);
  }
  if (!has_next) return;

  // LayerNorm + adaLN (FFN shift / scale slots 3 and 4 of layer l), gather.
  // The modulation rows are requested before the two reductions.
  uint4 sh_pk = make_uint4(0, 0, 0, 0), sc_pk = make_uint4(0, 0, 0, 0);
  if (active) {
    sh_pk = modulation8_packed(p.mod[l], p.time, p.ts, row, 3, d, e);
    sc_pk = modulation8_packed(p.mod[l], p.time, p.ts, row, 4, d, e);
  }
  const int nwarps = (nvec + 31) >> 5;
  const float mean = pass_row_sum(local, red, nwarps) / float(d);
  local = 0.f;
  if (active) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float c = x[i] - mean;
      local = __fadd_rn(local, __fmul_rn(c, c));  // as the row kernels: no FMA
    }
  }
  const float var = pass_row_sum(local, red, nwarps) / float(d);
  const float rstd = rsqrtf(var + p.eps);
  if (!active) return;
  // Gather slots of the next layer that read this row: its own index
  // (ungathered layer) or the list entries naming it.
  const int nm = next_gathered ? (slot->n_match < kMaxMatches ? slot->n_match : kMaxMatches) : (row < next_m ? 1 : 0);
  float n[8], shift[8], scale[8];
  unpack8(sh_pk, shift);
  unpack8(sc_pk, scale);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float s1 = bf16_round(1.0f + scale[i]);
    n[i] = bf16_round(bf16_round((x[i] - mean) * rstd) * s1) + shift[i];
  }
  for (int k = 0; k < nm; ++k) store8(p.gathered + size_t(next_gathered ? slot->matches[k] : row) * d + e, n);
}

__global__ void __launch_bounds__(kPassThreads, 1) stack_pass_kernel(const __grid_constant__ PassParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t s_bars[2 * kMaxAStages + 2 * kMaxBStages + 2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_verdict;
  __shared__ float s_red[16];
  __shared__ PassRowSlot s_rows[kPassRowSlots];

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t pair_rank = cluster_ctarank() & 1u;  // clusters of two CTAs: a UMMA pair
  const bool leader = pair_rank == 0;
  const uint16_t pair_mask = 0x3;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const unsigned int nctas = gridDim.x;
  volatile int* abort_flag = &s_abort;

  const int a_bytes = gemm_a_bytes();
  uint8_t* a_base = smem;
  uint8_t* b_base = smem + p.a_stages * a_bytes;
  uint64_t* full_a = s_bars;
  uint64_t* empty_a = full_a + p.a_stages;
  uint64_t* full_b = empty_a + p.a_stages;
  uint64_t* empty_b = full_b + p.b_stages;
  uint64_t* tmem_full = empty_b + p.b_stages;
  uint64_t* tmem_empty = tmem_full + 1;  // used in the leader: both CTAs' epilogues arrive

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.a_stages; ++s) {
      mbar_init(smem_addr(&full_a[s]), 1);
      mbar_init(smem_addr(&empty_a[s]), 1);
    }
    for (int s = 0; s < p.b_stages; ++s) {
      mbar_init(smem_addr(&full_b[s]), 1);
      mbar_init(smem_addr(&empty_b[s]), 1);
    }
    mbar_init(smem_addr(tmem_full), 1);
    mbar_init(smem_addr(tmem_empty), 2);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_g<2>(smem_addr(&s_tmem), kPassTmemCols);
    tmem_relinquish_g<2>();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ producers
    const bool weights = warp == 0;
    const int stages = weights ? p.a_stages : p.b_stages;
    uint64_t* full = weights ? full_a : full_b;
    uint64_t* empty = weights ? empty_a : empty_b;
    uint8_t* ring = weights ? a_base : b_base;
    const int slot_bytes = weights ? a_bytes : p.b_stage_bytes;
    const uint64_t policy = weights ? l2_policy_evict_first() : l2_policy_evict_last();
    uint32_t n = 0;  // stages issued so far
    bool ok = true;
    for (int l = 0; l < p.layers && ok; ++l) {
      const PassClass& C = p.cls[pass_class(p, l)];
      for (int kind = 0; kind < 2 && ok; ++kind) {
        const int items = kind == 0 ? p.up_tiles : p.down_tiles * p.down_splits;
        if (pair >= items) continue;
        const CUtensorMap* tm = weights ? (kind == 0 ? &p.tm_w_up[l] : &p.tm_w_down[l])
                                        : (kind == 0 ? &p.tm_act[pass_class(p, l)] : &p.tm_hid[pass_class(p, l)]);
        const int k_blocks = kind == 0 ? p.d / kBlockK : p.h / kBlockK;
        if (!weights) {
          // Activations of this phase exist once every CTA finished R(l) / U(l).
          int go = 1;
          if (lane == 0) {
            go = pass_wait(p, p.bars + 3 * l + kind, nctas, abort_flag);
            if (unsigned long long* rec = pass_trace(p, l, 1 + kind)) rec[6] = globaltimer_ns();
          }
          if (!__shfl_sync(0xffffffffu, go, 0)) {
            ok = false;
            break;
          }
        }
        if (lane == 0) prefetch_tensormap(tm);
        const uint32_t bytes = weights ? uint32_t(a_bytes) : uint32_t(C.b_rows * kBlockK * 2);
        for (int it = pair; it < items && ok; it += npairs) {
          const int tile = kind == 0 ? it : it % p.down_tiles;
          const int split = kind == 0 ? 0 : it / p.down_tiles;
          const int splits = kind == 0 ? 1 : p.down_splits;
          const int kb0 = int((long long)k_blocks * split / splits);
          const int kb1 = int((long long)k_blocks * (split + 1) / splits);
          const int tile128 = 2 * tile + int(pair_rank);
          for (int kb = kb0; kb < kb1; ++kb, ++n) {
            const int s = int(n % uint32_t(stages));
            const uint32_t ph = (n / uint32_t(stages)) & 1u;
            int w_ok = 1;
            if (lane == 0) w_ok = wait_bounded(smem_addr(&empty[s]), ph ^ 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
            if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
              ok = false;
              break;
            }
            if (elect_one()) {
              const uint32_t local_full = smem_addr(&full[s]);
              const uint32_t fb = map_to_cta(local_full, 0);
              if (leader) mbar_arrive_expect_tx(local_full, bytes * 2);
              if (weights) {
                const int c0 = p.w_packed ? 0 : kb * kBlockK;
                const int c1 = p.w_packed ? (tile128 * k_blocks + kb) * kFeatTile : tile128 * kFeatTile;
                tma_load_2d_pair(smem_addr(ring + s * slot_bytes), tm, fb, c0, c1, policy);
              } else {
                for (int b = 0; b < C.n_boxes; ++b) {
                  const uint32_t dst = smem_addr(ring + s * slot_bytes + b * C.tok_box * kBlockK * 2);
                  const int row = b == 0 ? int(pair_rank) * (C.mma_n0 / 2) : C.mma_n0 + int(pair_rank) * (C.mma_n1 / 2);
                  tma_load_2d_pair(dst, tm, fb, kb * kBlockK, row, policy);
                }
              }
            }
            __syncwarp();
          }
        }
      }
    }
    if (!ok) {
      if (lane == 0) pass_raise_abort(p, abort_flag);
      // Let the copies already in flight land before the CTA releases its
      // shared memory (the peer's copies complete on the leader's barrier, so
      // the peer waits a bounded moment instead).
      if (lane == 0) {
        if (leader) {
          const uint32_t first = n > uint32_t(stages) ? n - uint32_t(stages) : 0u;
          for (uint32_t i = first; i < n; ++i)
            wait_drain(smem_addr(&full[i % uint32_t(stages)]), (i / uint32_t(stages)) & 1u);
        } else {
          const long long t0 = clock64();
          while (clock64() - t0 < 2000000ll) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (leader) {
      uint32_t na = 0, nb = 0, item = 0;
      const uint32_t a0 = smem_addr(a_base), b0 = smem_addr(b_base);
      bool ok = true;
      for (int l = 0; l < p.layers && ok; ++l) {
        const PassClass& C = p.cls[pass_class(p, l)];
        const uint32_t idesc0 = umma_idesc_bf16(2 * kFeatTile, C.mma_n0);
        const uint32_t idesc1 = umma_idesc_bf16(2 * kFeatTile, C.mma_n1 > 0 ? C.mma_n1 : 16);
        const uint32_t b1_offset = uint32_t(C.mma_n0 / 2) * 128u;  // UMMA 1's rows in this CTA's slice
        for (int kind = 0; kind < 2 && ok; ++kind) {
          const int items = kind == 0 ? p.up_tiles : p.down_tiles * p.down_splits;
          const int k_blocks = kind == 0 ? p.d / kBlockK : p.h / kBlockK;
          for (int it = pair; it < items && ok; it += npairs, ++item) {
            const int split = kind == 0 ? 0 : it / p.down_tiles;
            const int splits = kind == 0 ? 1 : p.down_splits;
            const int kb0 = int((long long)k_blocks * split / splits);
            const int kb1 = int((long long)k_blocks * (split + 1) / splits);
            // Both CTAs' epilogues must have drained the accumulator of the previous item.
            if (item > 0) {
              int w_ok = 1;
              if (lane == 0)
                w_ok = wait_bounded(smem_addr(tmem_empty), (item - 1) & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT);
              if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            for (int kb = kb0; kb < kb1; ++kb, ++na, ++nb) {
              const int sa = int(na % uint32_t(p.a_stages)), sb = int(nb % uint32_t(p.b_stages));
              int w_ok = 1;
              if (lane == 0)
                w_ok = wait_bounded(smem_addr(&full_a[sa]), (na / uint32_t(p.a_stages)) & 1u, abort_flag, p.status,
                                    WAMFFN_DEV_TIMEOUT) &&
                       wait_bounded(smem_addr(&full_b[sb]), (nb / uint32_t(p.b_stages)) & 1u, abort_flag, p.status,
                                    WAMFFN_DEV_TIMEOUT);
              if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
                ok = false;
                break;
              }
              tc_fence_after();
              if (kb == kb0 && lane == 0)
                if (unsigned long long* rec = pass_trace(p, l, 1 + kind)) rec[2] = globaltimer_ns();
              const uint64_t adesc = umma_desc_sw128(a0 + uint32_t(sa * a_bytes));
              const uint64_t bdesc0 = umma_desc_sw128(b0 + uint32_t(sb * p.b_stage_bytes));
              const uint64_t bdesc1 = umma_desc_sw128(b0 + uint32_t(sb * p.b_stage_bytes) + b1_offset);
              if (elect_one()) {
#pragma unroll
                for (int k = 0; k < kBlockK / 16; ++k) {
                  const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
                  umma_bf16_pair(tmem_base, adesc + 2 * k, bdesc0 + 2 * k, idesc0, acc);
                  if (C.mma_n1 > 0) umma_bf16_pair(tmem_base + uint32_t(C.mma_n0), adesc + 2 * k, bdesc1 + 2 * k, idesc1, acc);
                }
                umma_commit_pair(smem_addr(&empty_a[sa]), pair_mask);
                umma_commit_pair(smem_addr(&empty_b[sb]), pair_mask);
              }
              __syncwarp();
            }
            if (!ok) break;
            if (elect_one()) umma_commit_pair(smem_addr(tmem_full), pair_mask);
            __syncwarp();
            if (lane == 0)
              if (unsigned long long* rec = pass_trace(p, l, 1 + kind)) rec[3] = globaltimer_ns();
          }
        }
      }
      if (!ok && lane == 0) pass_raise_abort(p, abort_flag);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogues + rows
    const int et = threadIdx.x - 128;  // 0..383
    const int ew = warp - 4;           // 0..11
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int group = ew >> 2;         // 0..2: TMEM column-chunk group
    uint32_t item = 0;
    // Rows of this CTA: blockIdx.x + nctas k, k < kPassRowSlots.
    const int row_limit = max(p.seq, p.cls[1].rows);
    for (int k = 0; k < kPassRowSlots; ++k) {
      const int r = blockIdx.x + int(nctas) * k;
      if (r < row_limit) pass_row_setup(p, r, et, &s_rows[k]);
    }
    for (int l = 0; l <= p.layers; ++l) {
      // ---- R(l): needs every CTA's partials of D(l-1).
      unsigned long long* rrec = et == 0 ? pass_trace(p, l, 0) : nullptr;
      if (rrec) {
        rrec[0] = (unsigned long long)blockIdx.x | (unsigned long long)l << 16;
        rrec[1] = globaltimer_ns();
        rrec[7] = smid();
      }
      if (l > 0) {
        if (et == 0) s_verdict = pass_wait(p, p.bars + 3 * (l - 1) + 2, nctas, abort_flag) ? 1 : 0;
        named_sync(kPassEpiBarrier, kPassEpiThreads);
        if (!s_verdict) break;
      }
      if (rrec) rrec[2] = globaltimer_ns();
      {
        const int limit = max(p.seq, l < p.layers ? p.cls[pass_class(p, l)].rows : 0);
        for (int k = 0; k < kPassRowSlots; ++k) {
          const int r = blockIdx.x + int(nctas) * k;
          if (r < limit) pass_row(p, l, r, et, s_red, &s_rows[k]);
        }
      }
      if (l == p.layers) break;
      named_sync(kPassEpiBarrier, kPassEpiThreads);
      if (et == 0) pass_arrive(p.bars + 3 * l);
      if (rrec) rrec[5] = globaltimer_ns();

      // ---- U(l), D(l): drain this pair's accumulators.
      const PassClass& C = p.cls[pass_class(p, l)];
      const int tokens = C.rows;
      bool ok = true;
      for (int kind = 0; kind < 2 && ok; ++kind) {
        const int items = kind == 0 ? p.up_tiles : p.down_tiles * p.down_splits;
        for (int it = pair; it < items; it += npairs, ++item) {
          const int tile128 = 2 * (kind == 0 ? it : it % p.down_tiles) + int(pair_rank);
          const int split = kind == 0 ? 0 : it / p.down_tiles;
          const int n0 = tile128 * kFeatTile;
          unsigned long long* irec = et == 0 ? pass_trace(p, l, 1 + kind) : nullptr;
          if (irec) {
            irec[0] = (unsigned long long)blockIdx.x | (unsigned long long)l << 16 | (unsigned long long)(1 + kind) << 32;
            irec[1] = globaltimer_ns();
            irec[7] = smid();
          }
          if (et == 0)
            s_verdict = wait_bounded(smem_addr(tmem_full), item & 1u, abort_flag, p.status, WAMFFN_DEV_TIMEOUT) &&
                                !*abort_flag
                            ? 1
                            : 0;
          named_sync(kPassEpiBarrier, kPassEpiThreads);
          if (!s_verdict) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (irec) irec[4] = globaltimer_ns();
          const int f = n0 + q * 32 + lane;
          const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
          if (kind == 1) {
            // fp32 partials [split, rows, d]; re-read once by R(l+1): keep them in L2.
            const uint64_t keep = l2_policy_evict_last();
            float* out = p.partial + size_t(split) * tokens * p.d + f;
            const int nchunks = (tokens + 31) >> 5;
            for (int c = group; c < nchunks; c += 3) {
              uint32_t r[32];
              tmem_ld32(lane_addr + uint32_t(c * 32), r);
              tmem_wait_ld(r);
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int t = c * 32 + i;
                if (t < tokens) st_global_keep(out + size_t(t) * p.d, __uint_as_float(r[i]), keep);
              }
            }
          } else {
            // bias + GELU, bf16 through a per-warp transpose tile (in the
            // activation ring, idle until the next grid barrier).
            __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(b_base) + ew * (32 * 32);
            const float bias = __bfloat162float(p.b_up[l][f]);
            const int n_base = n0 + q * 32;
            const int nchunks16 = (tokens + 15) >> 4;
            uint32_t nxt[16];
            if (group < nchunks16) tmem_ld16(lane_addr + uint32_t(group * 16), nxt);
            for (int c = group; c < nchunks16; c += 3) {
              tmem_wait_ld(nxt);
              uint32_t r[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) r[i] = nxt[i];
              if (c + 3 < nchunks16) tmem_ld16(lane_addr + uint32_t((c + 3) * 16), nxt);
#pragma unroll
              for (int i = 0; i < 16; ++i) tile[i * 32 + lane] = __float2bfloat16_rn(gelu_tanh(__uint_as_float(r[i]) + bias));
              __syncwarp();
#pragma unroll
              for (int pass = 0; pass < 2; ++pass) {
                const int row = pass * 8 + (lane >> 2);
                const int col = (lane & 3) * 8;
                const int t = c * 16 + row;
                const uint4 v = *reinterpret_cast<const uint4*>(&tile[row * 32 + col]);
                if (t < tokens) *reinterpret_cast<uint4*>(&p.hidden[size_t(t) * p.h + n_base + col]) = v;
              }
              __syncwarp();
            }
          }
          // Accumulator drained: the leader may start the next item.
          tc_fence_before();
          named_sync(kPassEpiBarrier, kPassEpiThreads);
          if (et == 0) mbar_arrive_remote(map_to_cta(smem_addr(tmem_empty), 0));
          if (irec) irec[5] = globaltimer_ns();
        }
        if (!ok) break;
        if (et == 0) pass_arrive(p.bars + 3 * l + 1 + kind);
      }
      if (!ok) {
        if (et == 0) pass_raise_abort(p, abort_flag);
        break;
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  cluster_sync();  // no CTA of a pair leaves while its peer can still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_g<2>(tmem_base, kPassTmemCols);
  }
}

}  // namespace wamffn
