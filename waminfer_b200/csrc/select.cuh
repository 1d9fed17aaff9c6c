// Token selection for cross-observation FFN reuse (WAMInfer/approximation.py:55-67).
//
// score[r] = 2 * sum_k |now[r,k] - before[r,k]| / max(sum_k |now[r,k]| + |before[r,k]|, 1e-6)
// in fp32; mandatory rows score +inf.  The `count` best rows by descending
// score (ties: smaller index first, i.e. a stable descending sort) are written
// in ascending order, followed by the future rows n..seq-1.
//
// Summation order (restated element for element by oracle/reuse.py::scores,
// so indices equal the oracle's in every case, near-ties included): each term
// is formed in fp32 as the reference forms it (|now - before| and
// |now| + |before| of bf16 values widened to fp32) and accumulated in fp64.
// Lane l of the row's warp adds the 8-element chunks l, l + 32, l + 64, ...
// in order, element by element; the 32 lane sums are combined by the xor
// butterfly (offsets 16, 8, 4, 2, 1); each total is rounded once to fp32.
// For bf16 activations of magnitude >= 2^-30 (or 0) every term's lowest bit
// is at or above 2^-37 and the fp64 running sum of a 3072-element row stays
// exact, so the fp32 totals are the correctly rounded exact sums: equal to the
// reference's fp32 sums whenever those are exact (whatever torch's reduction
// order), and independent of this kernel's order.
//
// One CTA: n <= 1024 rows of the current frame.  Ranking is an all-pairs count
// (n^2 comparisons), which is exact and order-independent.
#pragma once

#include "ptx.cuh"

namespace wamffn {

constexpr int kSelectThreads = 1024;

struct SelectParams {
  const __nv_bfloat16* now;     // [n, dim] rows with stride now_stride
  long long now_stride;
  const __nv_bfloat16* before;  // [n, dim] contiguous
  const unsigned char* mandatory;  // [n] (bool) or null
  int n;
  int dim;
  int count;
  int seq;
  long long* indices;           // [count + seq - n]
  __nv_bfloat16* features_out;  // [n, dim] copy of `now` or null
  int pdl;
};

__global__ void __launch_bounds__(kSelectThreads) select_tokens_kernel(const SelectParams p) {
  __shared__ float score[kSelectThreads];
  __shared__ int chosen[kSelectThreads];
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nwarps = blockDim.x >> 5;
  if (p.pdl) pdl_wait_prior();

  for (int r = warp; r < p.n; r += nwarps) {
    const __nv_bfloat16* a = p.now + size_t(r) * p.now_stride;
    const __nv_bfloat16* b = p.before + size_t(r) * p.dim;
    double num = 0.0, den = 0.0;
    for (int e = lane * 8; e < p.dim; e += 32 * 8) {
      const uint4 ua = *reinterpret_cast<const uint4*>(a + e);
      const uint4 ub = *reinterpret_cast<const uint4*>(b + e);
      if (p.features_out) *reinterpret_cast<uint4*>(p.features_out + size_t(r) * p.dim + e) = ua;
      const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&ua);
      const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&ub);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 fa = __bfloat1622float2(ha[i]);
        const float2 fb = __bfloat1622float2(hb[i]);
        // fp32 terms exactly as the reference forms them; no contraction into the fp64 adds.
        num = __dadd_rn(num, double(fabsf(__fsub_rn(fa.x, fb.x))));
        num = __dadd_rn(num, double(fabsf(__fsub_rn(fa.y, fb.y))));
        den = __dadd_rn(den, double(__fadd_rn(fabsf(fa.x), fabsf(fb.x))));
        den = __dadd_rn(den, double(__fadd_rn(fabsf(fa.y), fabsf(fb.y))));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      num = __dadd_rn(num, __shfl_xor_sync(0xffffffffu, num, o));
      den = __dadd_rn(den, __shfl_xor_sync(0xffffffffu, den, o));
    }
    if (lane == 0) {
      const float nf = __double2float_rn(num), df = __double2float_rn(den);
      float s = __fdiv_rn(__fmul_rn(2.0f, nf), fmaxf(df, 1e-6f));
      if (p.mandatory && p.mandatory[r]) s = __int_as_float(0x7f800000);  // +inf
      score[r] = s;
    }
  }
  __syncthreads();
  if (tid < p.n) {
    const float s = score[tid];
    int rank = 0;
    for (int j = 0; j < p.n; ++j) {
      const float t = score[j];
      rank += (t > s) || (t == s && j < tid);
    }
    chosen[tid] = rank < p.count;
  }
  __syncthreads();
  if (tid < p.n && chosen[tid]) {
    int pos = 0;
    for (int j = 0; j < tid; ++j) pos += chosen[j];
    p.indices[pos] = tid;
  }
  for (int k = tid; k < p.seq - p.n; k += blockDim.x) p.indices[p.count + k] = p.n + k;
  if (tid == 0) pdl_launch_dependents();
}

// Mandatory rows of TokenReuse.begin (WAMInfer/approximation.py:31-36) for
// uint8 HWC observations: row i (patch (i / grid_w, i % grid_w) of
// ph x pw pixels) is mandatory when the float32 mean of |now - before| over
// its ph x pw x 3 values exceeds 5.  For uint8 inputs every |difference| is an
// integer, so the float32 sum the reference accumulates is exact in any order
// (ph * pw * 3 * 255 < 2^24); the kernel sums integers and divides once, as
// numpy's mean does, which gives the reference's mask bit for bit.
constexpr int kRgbThreads = 256;

struct RgbParams {
  const unsigned char* now;     // [height, width, 3]
  const unsigned char* before;  // [height, width, 3]
  int width;
  int ph, pw;                   // patch height / width in pixels
  int grid_w;
  unsigned char* mandatory;     // [grid_h * grid_w]
};

__global__ void __launch_bounds__(kRgbThreads) rgb_mandatory_kernel(const RgbParams p) {
  __shared__ int partial[kRgbThreads / 32];
  const int patch = blockIdx.x;
  const int py = patch / p.grid_w, px = patch % p.grid_w;
  const int row_bytes = p.pw * 3;
  const int total = p.ph * row_bytes;
  const size_t base = (size_t(py) * p.ph * p.width + size_t(px) * p.pw) * 3;
  int sum = 0;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int r = i / row_bytes, c = i - r * row_bytes;
    const size_t off = base + size_t(r) * p.width * 3 + c;
    sum += abs(int(p.now[off]) - int(p.before[off]));
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < kRgbThreads / 32; ++w) s += partial[w];
    const float mean = __fdiv_rn(float(s), float(total));
    p.mandatory[patch] = mean > 5.0f ? 1 : 0;
  }
}

}  // namespace wamffn
