/*
 * A plain C consumer of the library's ABI (no Python, no torch): the FFN of
 * PreparedFFN.forward through wamffn_pack_weight + wamffn_linear_plan_create
 * + wamffn_ffn_run on a small seeded case, checked against a CPU restatement
 * (fp32 sums, bias and tanh-GELU in fp32, bf16 rounding of the hidden and the
 * output, as the prepared path does).  Built and run by tests/test_gpu_c_abi.py.
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
  cudaStreamDestroy(stream);
  printf("c abi ffn: %d of %d outside tolerance, mean relative error %.2e\n", bad_count, ROWS * D, rel);
  return (bad_count == 0 && rel < 5e-3) ? 0 : 1;
}
