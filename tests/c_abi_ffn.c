/*
 * A plain C consumer of the library's ABI (no Python, no torch): the FFN of
 * PreparedFFN.forward through wamffn_pack_weight + wamffn_linear_plan_create
 * + wamffn_ffn_run on a small seeded case, checked against a CPU restatement
 * (fp32 sums, bias and tanh-GELU in fp32, bf16 rounding of the hidden and the
 * output, as the prepared path does); then wamffn_masked_attention with a
 * padded-prompt key mask, checked against a CPU softmax with the
 * probabilities rounded to bf16 before the value product.  Built and run by
 * tests/test_gpu_c_abi.py.
 *
 * Exit status 0 when every output is within max(2e-2, one bf16 ulp) of the
 * restatement and mean |error| / mean |reference| is below 5e-3 (the rule of
 * the Python parity tests); 1 otherwise.
 */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "wamffn.h"

enum { ROWS = 40, D = 256, H = 512 };
enum { HEADS = 2, NQ = 40, NK = 70, KEPT = 60, W = HEADS * 128 };

static uint16_t to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest even (finite inputs) */
  return (uint16_t)(u >> 16);
}

static float from_bf16(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static float round_bf16(float f) { return from_bf16(to_bf16(f)); }

static uint32_t rng = 12345u;
static float uniform(void) {
  rng = rng * 1664525u + 1013904223u;
  return ((rng >> 8) + 0.5f) / 16777216.0f;
}
static float gauss(void) { return sqrtf(-2.0f * logf(uniform())) * cosf(6.2831853f * uniform()); }

static float gelu_tanh(float x) { return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x))); }

#define CHECK_CUDA(call)                                                    \
  do {                                                                      \
    cudaError_t e_ = (call);                                                \
    if (e_ != cudaSuccess) {                                                \
      fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));           \
      return 1;                                                             \
    }                                                                       \
  } while (0)
#define CHECK_ABI(call)                                                     \
  do {                                                                      \
    if ((call) != WAMFFN_OK) {                                              \
      fprintf(stderr, "%s: %s\n", #call, wamffn_last_error());              \
      return 1;                                                             \
    }                                                                       \
  } while (0)

int main(void) {
  static uint16_t x[ROWS * D], w_up[H * D], b_up[H], w_down[D * H], b_down[D], out[ROWS * D];
  for (int i = 0; i < ROWS * D; ++i) x[i] = to_bf16(gauss());
  for (int i = 0; i < H * D; ++i) w_up[i] = to_bf16(0.05f * gauss());
  for (int i = 0; i < H; ++i) b_up[i] = to_bf16(0.01f * gauss());
  for (int i = 0; i < D * H; ++i) w_down[i] = to_bf16(0.05f * gauss());
  for (int i = 0; i < D; ++i) b_down[i] = to_bf16(0.01f * gauss());

  if (wamffn_abi_version() != WAMFFN_ABI_VERSION) {
    fprintf(stderr, "unexpected ABI version %d\n", wamffn_abi_version());
    return 1;
  }
  void *dx, *dwu, *dwu_p, *dbu, *dwd, *dwd_p, *dbd, *dout;
  CHECK_CUDA(cudaSetDevice(0));
  CHECK_CUDA(cudaMalloc(&dx, sizeof x));
  CHECK_CUDA(cudaMalloc(&dwu, sizeof w_up));
  CHECK_CUDA(cudaMalloc(&dwu_p, sizeof w_up));
  CHECK_CUDA(cudaMalloc(&dbu, sizeof b_up));
  CHECK_CUDA(cudaMalloc(&dwd, sizeof w_down));
  CHECK_CUDA(cudaMalloc(&dwd_p, sizeof w_down));
  CHECK_CUDA(cudaMalloc(&dbd, sizeof b_down));
  CHECK_CUDA(cudaMalloc(&dout, sizeof out));
  CHECK_CUDA(cudaMemcpy(dx, x, sizeof x, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dwu, w_up, sizeof w_up, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dbu, b_up, sizeof b_up, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dwd, w_down, sizeof w_down, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dbd, b_down, sizeof b_down, cudaMemcpyHostToDevice));

  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreate(&stream));
  wamffn_linear_plan *up = NULL, *down = NULL;
  CHECK_ABI(wamffn_pack_weight(stream, dwu, dwu_p, H, D));
  CHECK_ABI(wamffn_pack_weight(stream, dwd, dwd_p, D, H));
  CHECK_ABI(wamffn_linear_plan_create(0, ROWS, H, D, WAMFFN_LINEAR_GELU | WAMFFN_WEIGHTS_PACKED, 1, &up));
  CHECK_ABI(wamffn_linear_plan_create(0, ROWS, D, H, WAMFFN_WEIGHTS_PACKED, 1, &down));
  CHECK_ABI(wamffn_ffn_run(up, down, stream, dx, dwu_p, dbu, dwd_p, dbd, dout));
  CHECK_CUDA(cudaStreamSynchronize(stream));
  uint32_t status = 0;
  CHECK_ABI(wamffn_linear_status(up, &status, 1));
  if (status) {
    fprintf(stderr, "device status %u\n", status);
    return 1;
  }
  CHECK_CUDA(cudaMemcpy(out, dout, sizeof out, cudaMemcpyDeviceToHost));

  /* Invalid arguments come back as a status with a message, never a crash. */
  wamffn_linear_plan* bad = NULL;
  if (wamffn_linear_plan_create(0, ROWS, 100, D, 0, 0, &bad) == WAMFFN_OK || bad != NULL ||
      strlen(wamffn_last_error()) == 0) {
    fprintf(stderr, "an n_out that is not a multiple of 128 was accepted\n");
    return 1;
  }

  static float hidden[ROWS * H];
  double err_sum = 0.0, ref_sum = 0.0;
  int bad_count = 0;
  for (int r = 0; r < ROWS; ++r) {
    for (int j = 0; j < H; ++j) {
      float acc = 0.0f;
      for (int k = 0; k < D; ++k) acc += from_bf16(x[r * D + k]) * from_bf16(w_up[j * D + k]);
      hidden[r * H + j] = round_bf16(gelu_tanh(acc + from_bf16(b_up[j])));
    }
    for (int j = 0; j < D; ++j) {
      float acc = 0.0f;
      for (int k = 0; k < H; ++k) acc += hidden[r * H + k] * from_bf16(w_down[j * H + k]);
      const float ref = round_bf16(acc + from_bf16(b_down[j]));
      const float got = from_bf16(out[r * D + j]);
      const float ulp = ldexpf(1.0f, (int)floorf(log2f(fabsf(ref) + 1e-30f)) - 7);
      const float tol = fmaxf(2e-2f, ulp);
      if (fabsf(got - ref) > tol) ++bad_count;
      err_sum += fabsf(got - ref);
      ref_sum += fabsf(ref);
    }
  }
  const double rel = err_sum / (ref_sum > 1e-12 ? ref_sum : 1e-12);
  wamffn_linear_plan_destroy(up);
  wamffn_linear_plan_destroy(down);
  printf("c abi ffn: %d of %d outside tolerance, mean relative error %.2e\n", bad_count, ROWS * D, rel);

  /* Masked attention: keys [KEPT, NK) masked for every head and query (a padded prompt). */
  static uint16_t q[NQ * W], k[NK * W], v[NK * W], o[NQ * W];
  static unsigned char mask[NK];
  for (int i = 0; i < NQ * W; ++i) q[i] = to_bf16(gauss());
  for (int i = 0; i < NK * W; ++i) k[i] = to_bf16(gauss());
  for (int i = 0; i < NK * W; ++i) v[i] = to_bf16(gauss());
  for (int i = 0; i < NK; ++i) mask[i] = i < KEPT;
  void *dq, *dk, *dv, *dmask, *dobuf;
  CHECK_CUDA(cudaMalloc(&dq, sizeof q));
  CHECK_CUDA(cudaMalloc(&dk, sizeof k));
  CHECK_CUDA(cudaMalloc(&dv, sizeof v));
  CHECK_CUDA(cudaMalloc(&dmask, sizeof mask));
  CHECK_CUDA(cudaMalloc(&dobuf, sizeof o));
  CHECK_CUDA(cudaMemcpy(dq, q, sizeof q, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dk, k, sizeof k, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dv, v, sizeof v, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dmask, mask, sizeof mask, cudaMemcpyHostToDevice));
  wamffn_attention_args at;
  memset(&at, 0, sizeof at);
  at.q = dq; at.q_row_stride = W; at.q_batch_stride = (int64_t)W * NQ;
  at.k = dk; at.k_row_stride = W; at.k_batch_stride = (int64_t)W * NK;
  at.v = dv; at.v_row_stride = W; at.v_batch_stride = (int64_t)W * NK;
  at.mask = dmask; at.mask_strides[3] = 1; /* [1, 1, 1, NK] broadcast over heads and queries */
  at.out = dobuf; at.batch = 1; at.nq = NQ; at.nk = NK; at.heads = HEADS; at.head_dim = 128;
  CHECK_ABI(wamffn_masked_attention(stream, &at));
  CHECK_CUDA(cudaStreamSynchronize(stream));
  CHECK_CUDA(cudaMemcpy(o, dobuf, sizeof o, cudaMemcpyDeviceToHost));
  int attn_bad = 0;
  double aerr = 0.0, aref = 0.0;
  for (int h = 0; h < HEADS; ++h) {
    for (int i = 0; i < NQ; ++i) {
      float s[NK], top = -INFINITY, norm = 0.0f;
      for (int j = 0; j < KEPT; ++j) {
        float acc = 0.0f;
        for (int d = 0; d < 128; ++d) acc += from_bf16(q[i * W + h * 128 + d]) * from_bf16(k[j * W + h * 128 + d]);
        s[j] = acc * 0.08838834764831845f * 1.4426950408889634f;
        top = fmaxf(top, s[j]);
      }
      for (int j = 0; j < KEPT; ++j) {
        s[j] = exp2f(s[j] - top);
        norm += s[j];
      }
      for (int d = 0; d < 128; ++d) {
        float acc = 0.0f;
        for (int j = 0; j < KEPT; ++j) acc += round_bf16(s[j]) * from_bf16(v[j * W + h * 128 + d]);
        const float ref = acc / norm;
        const float got = from_bf16(o[i * W + h * 128 + d]);
        const float ulp = ldexpf(1.0f, (int)floorf(log2f(fabsf(ref) + 1e-30f)) - 7);
        if (fabsf(got - ref) > fmaxf(2e-2f, ulp)) ++attn_bad;
        aerr += fabsf(got - ref);
        aref += fabsf(ref);
      }
    }
  }
  const double arel = aerr / (aref > 1e-12 ? aref : 1e-12);
  cudaStreamDestroy(stream);
  printf("c abi attention: %d of %d outside tolerance, mean relative error %.2e\n", attn_bad, NQ * W, arel);
  return (bad_count == 0 && rel < 5e-3 && attn_bad == 0 && arel < 5e-3) ? 0 : 1;
}
