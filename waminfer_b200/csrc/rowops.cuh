// Row kernels around the two FFN GEMMs.  Both are HBM/L2-bound elementwise
// passes: one CTA per sequence row, 16-byte vector loads/stores.
//
// modnorm_kernel  -- the reference's modulated norm (all four MODEs of
//                    WAMInfer/_triton_inference.py:130-176) with an optional
//                    fused row gather into the GEMM activation buffer
//                    (blocks.py:249-251).
// rowepi_kernel   -- split-K reduction + bias of the down projection, the
//                    cache scatter/concat (blocks.py:259-264) and the gated
//                    residual (_triton_inference.py:158-161, blocks.py:265-268).
#pragma once

#include "ptx.cuh"
#include "wamffn.h"

namespace wamffn {

constexpr int kRowThreads = 384;   // 3072 / 8: one 16-byte vector per thread at d = 3072
constexpr int kMaxMatches = 32;    // gather entries naming one row (duplicates) tracked per CTA

struct NormParams {
  const __nv_bfloat16* x;
  long long xs;
  const __nv_bfloat16* update;
  long long us;
  const __nv_bfloat16* mod;
  const __nv_bfloat16* previous;
  const __nv_bfloat16* time;
  long long ts;
  const __nv_bfloat16* weight;
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;      // [rows, dim] or null
  __nv_bfloat16* norm;   // [rows, dim] or null
  int rows;
  int dim;
  int mode;
  float eps;
  const void* idx;       // gather list or null (identity when gathered != null)
  int idx_bytes;
  int m;                 // gathered rows
  __nv_bfloat16* gathered;  // [m, dim] or null
  int* pos_of_row;       // [rows] or null: last j with idx[j] == row, -1 if none
  unsigned int* status;
  int pdl;
  int gather_only;       // 1: x is already normalised; only gather rows (no y / norm)
};

struct EpiParams {
  const float* partial;  // [splits, m, dim]
  int splits;
  int m;
  int dim;
  const __nv_bfloat16* bias;
  const int* pos_of_row;  // [seq] or null (identity)
  int seq;
  int cache_rows;
  const __nv_bfloat16* cache_in;
  __nv_bfloat16* cache_out;
  __nv_bfloat16* output;
  const __nv_bfloat16* y;
  const __nv_bfloat16* mod;
  const __nv_bfloat16* time;
  long long ts;
  __nv_bfloat16* x_out;
  unsigned int* status;
  int pdl;
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// bf16(mod[slot] + time[row, slot]) for 8 consecutive features (the
// reference's _modulation helper, _triton_inference.py:123-127).
__device__ __forceinline__ void modulation8(const __nv_bfloat16* mod, const __nv_bfloat16* time,
                                            long long ts, int row, int slot, int dim, int e,
                                            float (&out)[8]) {
  float a[8], b[8];
  load8(mod + size_t(slot) * dim + e, a);
  load8(time + size_t(row) * ts + size_t(slot) * dim + e, b);
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = bf16_round(a[i] + b[i]);
}

__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// modulation8 kept packed (the values are bf16 by construction): 4 registers.
__device__ __forceinline__ uint4 modulation8_packed(const __nv_bfloat16* mod, const __nv_bfloat16* time,
                                                    long long ts, int row, int slot, int dim, int e) {
  float v[8];
  modulation8(mod, time, ts, row, slot, dim, e, v);
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return u;
}

// bf16(mod[slot] + time[row, slot]) for 8 consecutive features, packed bf16x2.
__device__ __forceinline__ uint4 modulation8_bf2(const __nv_bfloat16* mod, const __nv_bfloat16* time, long long ts,
                                                 int row, int slot, int dim, int e) {
  return bf2_add4(*reinterpret_cast<const uint4*>(mod + size_t(slot) * dim + e),
                  *reinterpret_cast<const uint4*>(time + size_t(row) * ts + size_t(slot) * dim + e));
}

// adaLN of 8 normalised features, packed: bf16(bf16(n) * bf16(1 + scale)) + shift,
// rounded to bf16 (_triton_inference.py:170-176), with n = (x - mean) * rstd in fp32.
__device__ __forceinline__ uint4 adaln8_bf2(const float* x, float mean, float rstd, uint4 shift, uint4 scale) {
  const uint32_t one2 = 0x3f803f80u;  // bf16x2 {1, 1}
  float n[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) n[i] = (x[i] - mean) * rstd;
  const uint4 nb = make_uint4(bf2_pack(n[0], n[1]), bf2_pack(n[2], n[3]), bf2_pack(n[4], n[5]), bf2_pack(n[6], n[7]));
  const uint4 s1 = make_uint4(bf2_add(one2, scale.x), bf2_add(one2, scale.y), bf2_add(one2, scale.z),
                              bf2_add(one2, scale.w));
  return bf2_add4(bf2_mul4(nb, s1), shift);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = (blockDim.x + 31) >> 5;
  __syncthreads();  // red[] may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < nwarps; ++w) s += red[w];  // fixed order: deterministic
  return s;
}

__device__ __forceinline__ long long load_index(const void* idx, int bytes, int j) {
  return bytes == 8 ? reinterpret_cast<const long long*>(idx)[j]
                    : static_cast<long long>(reinterpret_cast<const int*>(idx)[j]);
}

// Dynamic shared memory: dim floats (the row after the residual update).
__global__ void __launch_bounds__(kRowThreads) modnorm_kernel(const NormParams p) {
  extern __shared__ float xrow[];
  __shared__ float red[32];
  __shared__ int matches[kMaxMatches];
  __shared__ int n_match;
  __shared__ int last_match;
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int nvec = p.dim >> 3;

  if (p.pdl) pdl_wait_prior();
  // Let the next kernel (the GEMM) be scheduled as SMs free up; it still waits
  // for this grid's completion before reading what it writes.
  if (tid == 0) pdl_launch_dependents();

  // Pad / invalid gather entries: the activation row is zero so the GEMM
  // computes on defined data; invalid ones also raise the status bit.
  if (p.gathered != nullptr && p.idx != nullptr && b < p.m) {
    const long long r = load_index(p.idx, p.idx_bytes, b);
    if (r < 0 || r >= p.rows) {
      if (r != -1 && tid == 0) atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
      for (int v = tid; v < nvec; v += blockDim.x)
        *reinterpret_cast<uint4*>(p.gathered + size_t(b) * p.dim + v * 8) = make_uint4(0, 0, 0, 0);
    }
  }
  if (b >= p.rows) return;
  const int row = b;

  // Which gathered slots read this row?
  if (tid == 0) {
    n_match = 0;
    last_match = -1;
  }
  __syncthreads();
  if (p.gathered != nullptr) {
    if (p.idx == nullptr) {
      if (tid == 0 && row < p.m) {
        matches[0] = row;
        n_match = 1;
        last_match = row;
      }
    } else {
      for (int j = tid; j < p.m; j += blockDim.x) {
        if (load_index(p.idx, p.idx_bytes, j) == row) {
          const int slot = atomicAdd(&n_match, 1);
          if (slot < kMaxMatches) matches[slot] = j;
          else atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
          atomicMax(&last_match, j);
        }
      }
    }
  }
  __syncthreads();
  if (p.pos_of_row != nullptr && tid == 0) p.pos_of_row[row] = last_match;

  if (p.gather_only) {
    const int nm = n_match < kMaxMatches ? n_match : kMaxMatches;
    const __nv_bfloat16* src = p.x + size_t(row) * p.xs;
    for (int v = tid; v < nvec; v += blockDim.x) {
      const uint4 val = *reinterpret_cast<const uint4*>(src + v * 8);
      for (int k = 0; k < nm; ++k)
        *reinterpret_cast<uint4*>(p.gathered + size_t(matches[k]) * p.dim + v * 8) = val;
    }
    if (tid == 0) pdl_launch_dependents();
    return;
  }

  // Pass 1: residual update (bf16 rounding after each step) and the row sum.
  const __nv_bfloat16* xr = p.x + size_t(row) * p.xs;
  float local = 0.f;
  for (int v = tid; v < nvec; v += blockDim.x) {
    const int e = v * 8;
    float x[8];
    load8(xr + e, x);
    if (p.mode > 0 && p.update != nullptr) {
      float u[8];
      load8(p.update + size_t(row) * p.us + e, u);
      if (p.mode == WAMFFN_SELF_RESIDUAL || p.mode == WAMFFN_FFN_RESIDUAL) {
        float g[8];
        if (p.mode == WAMFFN_SELF_RESIDUAL) modulation8(p.mod, p.time, p.ts, row, 2, p.dim, e, g);
        else modulation8(p.previous, p.time, p.ts, row, 5, p.dim, e, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) u[i] = bf16_round(g[i] * u[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = bf16_round(x[i] + u[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xrow[e + i] = x[i];
      local = __fadd_rn(local, x[i]);
    }
    if (p.y != nullptr) store8(p.y + size_t(row) * p.dim + e, x);
  }
  const float mean = block_sum(local, red) / float(p.dim);

  // Pass 2: centred second moment.
  local = 0.f;
  for (int v = tid; v < nvec; v += blockDim.x) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float c = xrow[v * 8 + i] - mean;
      local = __fadd_rn(local, __fmul_rn(c, c));  // no FMA: the reference kernel runs without fp fusion
    }
  }
  const float var = block_sum(local, red) / float(p.dim);
  const float rstd = rsqrtf(var + p.eps);

  // Pass 3: normalise, modulate, write norm and the gathered copies.
  const int sh = p.mode == WAMFFN_CROSS_RESIDUAL ? 3 : 0;
  const int sc = p.mode == WAMFFN_CROSS_RESIDUAL ? 4 : 1;
  const int nm = n_match < kMaxMatches ? n_match : kMaxMatches;
  for (int v = tid; v < nvec; v += blockDim.x) {
    const int e = v * 8;
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) n[i] = (xrow[e + i] - mean) * rstd;
    if (p.mode == WAMFFN_SELF_RESIDUAL) {
      float w[8], bb[8];
      load8(p.weight + e, w);
      load8(p.bias + e, bb);
#pragma unroll
      for (int i = 0; i < 8; ++i) n[i] = __fadd_rn(__fmul_rn(n[i], w[i]), bb[i]);
    } else {
      float shift[8], scale[8];
      modulation8(p.mod, p.time, p.ts, row, sh, p.dim, e, shift);
      modulation8(p.mod, p.time, p.ts, row, sc, p.dim, e, scale);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float s1 = bf16_round(1.0f + scale[i]);
        n[i] = bf16_round(bf16_round(n[i]) * s1) + shift[i];
      }
    }
    if (p.norm != nullptr) store8(p.norm + size_t(row) * p.dim + e, n);
    for (int k = 0; k < nm; ++k) store8(p.gathered + size_t(matches[k]) * p.dim + e, n);
  }
  if (tid == 0) pdl_launch_dependents();
}

// The standalone modulated norm (op wam_ffn::modulated_norm) with the row
// held in registers: 4 warps per row, as the reference's Triton kernel runs
// (_triton_inference.py:201-220), every load of the row issued before the
// first reduction.  It computes the same bits as modnorm_kernel: the row
// kernels' reduction order is that of 32-lane groups of consecutive 16-byte
// vectors (a sequential sum of the vector's 8 values, a xor butterfly across
// the group, the group sums added in order), and thread t here holds the
// vectors t, t + 128 and t + 256, i.e. one lane of groups w, w + 4 and w + 8
// (w = t / 32), so each group is reduced by one warp exactly as before.
// For rows of nvec = dim / 8 vectors with nvec % 32 == 0 and nvec <= 384.
constexpr int kNormRegThreads = 128;
constexpr int kNormRegVecs = kRowThreads / kNormRegThreads;  // vectors per thread (3 at dim 3072)

__device__ __forceinline__ void group_sums(float (&v)[kNormRegVecs], float* red, int groups) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kNormRegVecs; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[j] = __fadd_rn(v[j], __shfl_xor_sync(0xffffffffu, v[j], o));
    const int g = warp + j * (kNormRegThreads / 32);
    if (lane == 0 && g < groups) red[g] = v[j];
  }
}

__device__ __forceinline__ float ordered_total(const float* red, int groups) {
  float s = 0.f;
  for (int g = 0; g < groups; ++g) s = __fadd_rn(s, red[g]);
  return s;
}

__global__ void __launch_bounds__(kNormRegThreads) modnorm_reg_kernel(const NormParams p) {
  __shared__ float red[2][kRowThreads / 32];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nvec = p.dim >> 3;
  const int groups = nvec >> 5;
  if (p.pdl) pdl_wait_prior();
  if (tid == 0) pdl_launch_dependents();
  const int mode = p.mode;
  const bool residual = mode > 0 && p.update != nullptr;
  const bool self_res = mode == WAMFFN_SELF_RESIDUAL;
  const int gslot = self_res ? 2 : 5;                       // gate slot of the residual update
  const __nv_bfloat16* gmod = self_res ? p.mod : p.previous;
  const int sh = mode == WAMFFN_CROSS_RESIDUAL ? 3 : 0;
  const int sc = mode == WAMFFN_CROSS_RESIDUAL ? 4 : 1;
  const __nv_bfloat16* trow = p.time + size_t(row) * p.ts;

  // Every load of the row first: x, the update and its gate, the shift and
  // scale (or the affine weight and bias).
  uint4 xv[kNormRegVecs], uv[kNormRegVecs], gm[kNormRegVecs], gt[kNormRegVecs];
  uint4 am[kNormRegVecs], at[kNormRegVecs], bm[kNormRegVecs], bt[kNormRegVecs];
  const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int j = 0; j < kNormRegVecs; ++j) {
    const int v = tid + j * kNormRegThreads;
    const int e = v * 8;
    xv[j] = uv[j] = gm[j] = gt[j] = am[j] = at[j] = bm[j] = bt[j] = zero;
    if (v < nvec) {
      xv[j] = *reinterpret_cast<const uint4*>(p.x + size_t(row) * p.xs + e);
      if (residual) {
        uv[j] = *reinterpret_cast<const uint4*>(p.update + size_t(row) * p.us + e);
        if (self_res || mode == WAMFFN_FFN_RESIDUAL) {
          gm[j] = *reinterpret_cast<const uint4*>(gmod + size_t(gslot) * p.dim + e);
          gt[j] = *reinterpret_cast<const uint4*>(trow + size_t(gslot) * p.dim + e);
        }
      }
      if (self_res) {
        am[j] = *reinterpret_cast<const uint4*>(p.weight + e);
        bm[j] = *reinterpret_cast<const uint4*>(p.bias + e);
      } else {
        am[j] = *reinterpret_cast<const uint4*>(p.mod + size_t(sh) * p.dim + e);
        at[j] = *reinterpret_cast<const uint4*>(trow + size_t(sh) * p.dim + e);
        bm[j] = *reinterpret_cast<const uint4*>(p.mod + size_t(sc) * p.dim + e);
        bt[j] = *reinterpret_cast<const uint4*>(trow + size_t(sc) * p.dim + e);
      }
    }
  }

  // Residual update in packed bf16x2 (each step rounded as the reference
  // rounds it) and the per-vector fp32 sums.
  float x[kNormRegVecs][8], local[kNormRegVecs];
#pragma unroll
  for (int j = 0; j < kNormRegVecs; ++j) {
    if (residual) {
      uint4 u = uv[j];
      if (self_res || mode == WAMFFN_FFN_RESIDUAL) u = bf2_mul4(bf2_add4(gm[j], gt[j]), u);
      xv[j] = bf2_add4(xv[j], u);
    }
    unpack8(xv[j], x[j]);
    local[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) local[j] = __fadd_rn(local[j], x[j][i]);
    const int v = tid + j * kNormRegThreads;
    if (v < nvec && p.y != nullptr) *reinterpret_cast<uint4*>(p.y + size_t(row) * p.dim + v * 8) = xv[j];
  }
  group_sums(local, red[0], groups);
  __syncthreads();
  const float mean = ordered_total(red[0], groups) / float(p.dim);
#pragma unroll
  for (int j = 0; j < kNormRegVecs; ++j) {
    local[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float c = x[j][i] - mean;
      local[j] = __fadd_rn(local[j], __fmul_rn(c, c));
    }
  }
  group_sums(local, red[1], groups);
  __syncthreads();
  const float var = ordered_total(red[1], groups) / float(p.dim);
  const float rstd = rsqrtf(var + p.eps);

  const uint32_t one2 = 0x3f803f80u;  // bf16x2 {1, 1}
#pragma unroll
  for (int j = 0; j < kNormRegVecs; ++j) {
    const int v = tid + j * kNormRegThreads;
    if (v >= nvec) continue;
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) n[i] = (x[j][i] - mean) * rstd;
    uint4 out;
    if (self_res) {
      float a[8], b[8];
      unpack8(am[j], a);
      unpack8(bm[j], b);
#pragma unroll
      for (int i = 0; i < 8; ++i) n[i] = __fadd_rn(__fmul_rn(n[i], a[i]), b[i]);
      out = make_uint4(bf2_pack(n[0], n[1]), bf2_pack(n[2], n[3]), bf2_pack(n[4], n[5]), bf2_pack(n[6], n[7]));
    } else {
      // bf16(bf16(n) * bf16(1 + bf16(mod + time))) + bf16(mod + time), stored as bf16.
      const uint4 shift = bf2_add4(am[j], at[j]);
      const uint4 scale = bf2_add4(bm[j], bt[j]);
      const uint4 s1 = make_uint4(bf2_add(one2, scale.x), bf2_add(one2, scale.y), bf2_add(one2, scale.z),
                                  bf2_add(one2, scale.w));
      const uint4 nb = make_uint4(bf2_pack(n[0], n[1]), bf2_pack(n[2], n[3]), bf2_pack(n[4], n[5]),
                                  bf2_pack(n[6], n[7]));
      out = bf2_add4(bf2_mul4(nb, s1), shift);
    }
    if (p.norm != nullptr) *reinterpret_cast<uint4*>(p.norm + size_t(row) * p.dim + v * 8) = out;
  }
}

constexpr int kEpiSplitsBatch = 3;  // split-K partials loaded per batch of independent loads

// One CTA per sequence row.
__global__ void __launch_bounds__(kRowThreads, 3) rowepi_kernel(const EpiParams p) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nvec = p.dim >> 3;
  if (p.pdl) pdl_wait_prior();
  if (tid == 0) pdl_launch_dependents();
  int j = p.pos_of_row != nullptr ? p.pos_of_row[row] : row;
  if (j >= p.m) j = -1;
  const bool cached_row = row < p.cache_rows;
  if (j < 0 && !cached_row && tid == 0 && p.status) atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
  for (int v = tid; v < nvec; v += blockDim.x) {
    const int e = v * 8;
    float o[8];
    if (j >= 0) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      // Partials in batches of independent loads, summed in split order.
      for (int s0 = 0; s0 < p.splits; s0 += kEpiSplitsBatch) {
        float4 part[kEpiSplitsBatch][2];
#pragma unroll
        for (int s = 0; s < kEpiSplitsBatch; ++s) {
          if (s0 + s < p.splits) {
            const float4* src =
                reinterpret_cast<const float4*>(p.partial + (size_t(s0 + s) * p.m + j) * p.dim + e);
            part[s][0] = src[0];
            part[s][1] = src[1];
          }
        }
#pragma unroll
        for (int s = 0; s < kEpiSplitsBatch; ++s) {
          if (s0 + s < p.splits) {
            acc[0] += part[s][0].x; acc[1] += part[s][0].y; acc[2] += part[s][0].z; acc[3] += part[s][0].w;
            acc[4] += part[s][1].x; acc[5] += part[s][1].y; acc[6] += part[s][1].z; acc[7] += part[s][1].w;
          }
        }
      }
      float bb[8];
      load8(p.bias + e, bb);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = bf16_round(acc[i] + bb[i]);
    } else if (cached_row && p.cache_in != nullptr) {
      load8(p.cache_in + size_t(row) * p.dim + e, o);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = 0.f;
    }
    if (p.output != nullptr) store8(p.output + size_t(row) * p.dim + e, o);
    if (cached_row && p.cache_out != nullptr) store8(p.cache_out + size_t(row) * p.dim + e, o);
    if (p.x_out != nullptr) {
      float g[8], y[8], r[8];
      modulation8(p.mod, p.time, p.ts, row, 5, p.dim, e, g);
      load8(p.y + size_t(row) * p.dim + e, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = y[i] + bf16_round(g[i] * o[i]);
      store8(p.x_out + size_t(row) * p.dim + e, r);
    }
  }
  if (tid == 0) pdl_launch_dependents();
}

// Layer boundary of an FFN stack: the split-K reduction + bias of layer l's
// down projection, the scatter into layer l's history, the gated residual,
// and -- fused on the same row -- layer l+1's LayerNorm / adaLN (FFN shift and
// scale slots) and its row gather.  This is the reference's cross-layer fold
// (the FFN_RESIDUAL norm of WAMInfer/_triton_inference.py:158-176 that
// consumes the deferred FFN output of WAMInfer/blocks.py:269-271) with the
// next layer's FFN prologue in place of its attention prologue.
struct BoundaryParams {
  const float* partial;         // [splits, m, dim] fp32 partials of layer l
  int splits;
  int m;
  int dim;
  int seq;
  const __nv_bfloat16* bias;    // b_down of layer l
  const void* idx;              // gather list of layer l ([m] entries), or null (identity)
  int idx_bytes;
  int cache_rows;
  const __nv_bfloat16* cache_in;
  __nv_bfloat16* cache_out;
  __nv_bfloat16* y;             // [seq, dim] residual of layer l, overwritten by layer l+1's
  const __nv_bfloat16* mod;     // [6, dim] of layer l (gate slot 5)
  const __nv_bfloat16* time;
  long long ts;
  const __nv_bfloat16* next_mod;  // [6, dim] of layer l+1, or null: l is the last layer
  const void* next_idx;         // gather list of layer l+1, or null (identity)
  int next_idx_bytes;
  int next_m;
  __nv_bfloat16* next_gathered; // [next_m, dim]
  __nv_bfloat16* x_final;       // [seq, dim], written after the last layer
  float eps;
  unsigned int* status;
  int out_bf16;                 // 1: `partial` holds bf16 [m, dim] outputs with the bias applied (unsplit K)
};

// Sum of the split-K partials of one rank's down projection, in split order
// ([splits, m, dim] -> [m, dim] fp32), ahead of the cross-rank reduction of
// the tensor-parallel stack.  One CTA per row.
__global__ void __launch_bounds__(kRowThreads) split_sum_kernel(const float* __restrict__ partial, int splits, int m,
                                                              int dim, float* __restrict__ out) {
  pdl_wait_prior();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int row = blockIdx.x;
  for (int v = threadIdx.x; v < (dim >> 2); v += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < splits; ++s) {
      const float4 a = reinterpret_cast<const float4*>(partial + (size_t(s) * m + row) * dim)[v];
      acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
    }
    reinterpret_cast<float4*>(out + size_t(row) * dim)[v] = acc;
  }
}

constexpr int kBoundarySplitsBatch = 2;  // split-K partials loaded per batch of independent loads

// Dynamic shared memory: dim floats.
//
// The gather lists do not depend on the down projection and are read before
// the grid-dependency wait; after it the residual row, the gate, the bias and
// the partials are read in batches of independent loads.  Registers are capped so that three CTAs (three rows)
// stay resident per SM.
// kOutBf16: the down projection ran unsplit and stored bf16(acc + bias) itself
// (p.out_bf16); a separate instantiation keeps the split-K path's registers.
template <bool kOutBf16>
__global__ void __launch_bounds__(kRowThreads, 3) boundary_kernel(const BoundaryParams p) {
  extern __shared__ float xrow[];
  __shared__ float red[32];
  __shared__ int matches[kMaxMatches];
  __shared__ int n_match;
  __shared__ int last_match;   // this layer: last j with idx[j] == row, -1 if none
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int nvec = p.dim >> 3;
  const bool last = p.next_mod == nullptr;

  if (!last && p.next_idx != nullptr && b < p.next_m) {
    const long long r = load_index(p.next_idx, p.next_idx_bytes, b);
    if (r < 0 || r >= p.seq) {
      if (r != -1 && tid == 0) atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
      // The activation buffer is read by the running down projection: zero
      // the slot only after it has finished.
      pdl_wait_prior();
      for (int v = tid; v < nvec; v += blockDim.x)
        *reinterpret_cast<uint4*>(p.next_gathered + size_t(b) * p.dim + v * 8) = make_uint4(0, 0, 0, 0);
    }
  }
  if (b >= p.seq) {
    pdl_wait_prior();
    if (tid == 0) pdl_launch_dependents();
    return;
  }
  const int row = b;
  unsigned long long* rec = nullptr;  // optional timeline record (wamffn_trace_enable)
  if (g_trace != nullptr && tid == 0) {
    const unsigned int slot = atomicAdd(reinterpret_cast<unsigned int*>(g_trace), 1u);
    if (slot + 1 < g_trace_capacity) {
      rec = g_trace + size_t(slot + 1) * kTraceWords;
      rec[0] = (unsigned long long)b | (unsigned long long)kTraceBoundary << 32;
      rec[1] = globaltimer_ns();
      rec[6] = smid();
    }
  }

  // Which entry of this layer's list computed this row, and which entries of
  // the next layer's list read it (both lists are inputs of the whole pass).
  if (tid == 0) {
    n_match = 0;
    last_match = p.idx == nullptr ? (row < p.m ? row : -1) : -1;
  }
  __syncthreads();
  if (p.idx != nullptr) {
    for (int j = tid; j < p.m; j += blockDim.x)
      if (load_index(p.idx, p.idx_bytes, j) == row) atomicMax(&last_match, j);
  }
  if (!last) {
    if (p.next_idx == nullptr) {
      if (tid == 0 && row < p.next_m) {
        matches[0] = row;
        n_match = 1;
      }
    } else {
      for (int j = tid; j < p.next_m; j += blockDim.x) {
        if (load_index(p.next_idx, p.next_idx_bytes, j) == row) {
          const int slot = atomicAdd(&n_match, 1);
          if (slot < kMaxMatches) matches[slot] = j;
          else atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);
        }
      }
    }
  }
  __syncthreads();
  const int j = last_match;
  const bool cached_row = row < p.cache_rows;
  if (j < 0 && !cached_row && tid == 0) atomicOr(p.status, WAMFFN_DEV_BAD_INDEX);

  pdl_wait_prior();
  if (tid == 0) pdl_launch_dependents();
  if (rec) rec[2] = globaltimer_ns();

  // 1. Layer l: reduce, bias, scatter into the history, gated residual.
  float local = 0.f;
  for (int v = tid; v < nvec; v += blockDim.x) {
    const int e = v * 8;
    const uint4 y_packed = *reinterpret_cast<const uint4*>(p.y + size_t(row) * p.dim + e);
    const uint4 g_packed = modulation8_bf2(p.mod, p.time, p.ts, row, 5, p.dim, e);
    uint4 o;  // bf16 FFN output of this row
    if (kOutBf16 && j >= 0) {
      o = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.partial) + size_t(j) * p.dim + e);
    } else if (j >= 0) {
      const float* base = p.partial + size_t(j) * p.dim + e;
      const size_t split_stride = size_t(p.m) * p.dim;
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int s0 = 0; s0 < p.splits; s0 += kBoundarySplitsBatch) {
        float4 part[kBoundarySplitsBatch][2];
#pragma unroll
        for (int s = 0; s < kBoundarySplitsBatch; ++s) {
          if (s0 + s < p.splits) {
            const float4* src = reinterpret_cast<const float4*>(base + (s0 + s) * split_stride);
            part[s][0] = src[0];
            part[s][1] = src[1];
          }
        }
#pragma unroll
        for (int s = 0; s < kBoundarySplitsBatch; ++s) {
          if (s0 + s < p.splits) {
            acc[0] += part[s][0].x; acc[1] += part[s][0].y; acc[2] += part[s][0].z; acc[3] += part[s][0].w;
            acc[4] += part[s][1].x; acc[5] += part[s][1].y; acc[6] += part[s][1].z; acc[7] += part[s][1].w;
          }
        }
      }
      float bb[8];
      load8(p.bias + e, bb);
      o = make_uint4(bf2_pack(acc[0] + bb[0], acc[1] + bb[1]), bf2_pack(acc[2] + bb[2], acc[3] + bb[3]),
                     bf2_pack(acc[4] + bb[4], acc[5] + bb[5]), bf2_pack(acc[6] + bb[6], acc[7] + bb[7]));
    } else if (cached_row && p.cache_in != nullptr) {
      o = *reinterpret_cast<const uint4*>(p.cache_in + size_t(row) * p.dim + e);
    } else {
      o = make_uint4(0, 0, 0, 0);
    }
    if (cached_row && p.cache_out != nullptr) *reinterpret_cast<uint4*>(p.cache_out + size_t(row) * p.dim + e) = o;
    // x = bf16(y + bf16(gate * o)), packed (the same roundings as the fp32 form).
    const uint4 xp = bf2_add4(y_packed, bf2_mul4(g_packed, o));
    float x[8];
    unpack8(xp, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xrow[e + i] = x[i];
      local = __fadd_rn(local, x[i]);
    }
    *reinterpret_cast<uint4*>((last ? p.x_final : p.y) + size_t(row) * p.dim + e) = xp;
  }
  if (rec) rec[3] = rec[4] = globaltimer_ns();
  if (last) {
    if (rec) rec[5] = globaltimer_ns();
    return;
  }

  // 2. Layer l+1: LayerNorm + adaLN (FFN shift/scale slots 3 and 4), gather.
  // The first vector's shift / scale loads overlap the two reductions.
  uint4 pre_shift = make_uint4(0, 0, 0, 0), pre_scale = make_uint4(0, 0, 0, 0);
  if (tid < nvec) {
    pre_shift = modulation8_bf2(p.next_mod, p.time, p.ts, row, 3, p.dim, tid * 8);
    pre_scale = modulation8_bf2(p.next_mod, p.time, p.ts, row, 4, p.dim, tid * 8);
  }
  const float mean = block_sum(local, red) / float(p.dim);
  local = 0.f;
  for (int v = tid; v < nvec; v += blockDim.x) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float c = xrow[v * 8 + i] - mean;
      local = __fadd_rn(local, __fmul_rn(c, c));  // no FMA: the reference kernel runs without fp fusion
    }
  }
  const float var = block_sum(local, red) / float(p.dim);
  const float rstd = rsqrtf(var + p.eps);
  const int nm = n_match < kMaxMatches ? n_match : kMaxMatches;
  for (int v = tid; v < nvec; v += blockDim.x) {
    const int e = v * 8;
    const uint4 shift = v == tid ? pre_shift : modulation8_bf2(p.next_mod, p.time, p.ts, row, 3, p.dim, e);
    const uint4 scale = v == tid ? pre_scale : modulation8_bf2(p.next_mod, p.time, p.ts, row, 4, p.dim, e);
    const uint4 n = adaln8_bf2(xrow + e, mean, rstd, shift, scale);
    for (int k = 0; k < nm; ++k) *reinterpret_cast<uint4*>(p.next_gathered + size_t(matches[k]) * p.dim + e) = n;
  }
  if (rec) rec[5] = globaltimer_ns();
}

// Weight repack: dst[n/128][k/64][128][64] <- src[n][k] (16-byte vectors;
// stores are contiguous, each group of 8 threads reads 128 contiguous bytes).
__global__ void pack_weight_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int n_out, int k_in) {
  const long long kb_count = k_in / 64;
  const long long total = (long long)n_out * k_in / 8;
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const long long c8 = v & 7;
    const long long r = (v >> 3) & 127;
    const long long kb = (v >> 10) % kb_count;
    const long long nt = (v >> 10) / kb_count;
    dst[v] = src[((nt * 128 + r) * k_in + kb * 64) / 8 + c8];
  }
}

}  // namespace wamffn
