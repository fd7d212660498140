/* A C host of the library: no Python, no torch.
 *
 * Fills bf16 q/k/v ([batch, heads, tokens, channels], contiguous) from a
 * linear congruential generator with values n/64, |n| <= 128 (exact in bf16),
 * runs fe_evict on its own CUDA stream with a cudaMalloc'd row-statistics
 * workspace, then fe_evict_noalloc on the same inputs, and writes the inputs
 * and both calls' outputs to <prefix>.bin for the Python side to compare:
 *   header int64[8] = {batch, q_heads, kv_heads, tokens, channels, budget, recent, pool}
 *   q, k, v (uint16 bf16 bits), then per call: out (uint16), importance (float),
 *   indices (int64), mask (uint8).
 * Usage: evict_host <prefix> ; exit status 0 on success.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "flash_evict.h"

#define B 2
#define HQ 6
#define HK 2
#define N 1111
#define D 128
#define BUDGET 200
#define RECENT 16
#define POOL 3

static uint64_t lcg_state = 0x9e3779b97f4a7c15ull;

static uint16_t next_bf16(void) {
  lcg_state = lcg_state * 6364136223846793005ull + 1442695040888963407ull;
  const int n = (int)((lcg_state >> 33) % 257u) - 128;
  const float f = (float)n / 64.0f;
  uint32_t bits;
  memcpy(&bits, &f, 4);
  return (uint16_t)(bits >> 16); /* exact: at most 8 significant bits */
}

static int check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

static int check_fe(int rc, const char* what) {
  if (rc != FE_STATUS_OK) {
    fprintf(stderr, "%s: status %d: %s\n", what, rc, fe_last_error());
    return 1;
  }
  return 0;
}

int main(int argc, char** argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: %s <output prefix>\n", argv[0]);
    return 2;
  }
  const size_t nq = (size_t)B * HQ * N * D, nk = (size_t)B * HK * N * D;
  const size_t nimp = (size_t)B * HK * N, nidx = (size_t)B * HK * BUDGET;
  uint16_t* hq = malloc(nq * 2);
  uint16_t* hk = malloc(nk * 2);
  uint16_t* hv = malloc(nk * 2);
  uint16_t* hout = malloc(nq * 2);
  float* himp = malloc(nimp * 4);
  int64_t* hidx = malloc(nidx * 8);
  uint8_t* hmask = malloc(nimp);
  if (!hq || !hk || !hv || !hout || !himp || !hidx || !hmask) return 3;
  for (size_t i = 0; i < nq; ++i) hq[i] = next_bf16();
  for (size_t i = 0; i < nk; ++i) hk[i] = next_bf16();
  for (size_t i = 0; i < nk; ++i) hv[i] = next_bf16();

  void *dq, *dk, *dv, *dout;
  float *dimp, *dstats;
  int64_t* didx;
  uint8_t* dmask;
  cudaStream_t stream;
  if (check_cuda(cudaMalloc(&dq, nq * 2), "cudaMalloc q") || check_cuda(cudaMalloc(&dk, nk * 2), "cudaMalloc k") ||
      check_cuda(cudaMalloc(&dv, nk * 2), "cudaMalloc v") || check_cuda(cudaMalloc(&dout, nq * 2), "cudaMalloc out") ||
      check_cuda(cudaMalloc((void**)&dimp, nimp * 4), "cudaMalloc importance") ||
      check_cuda(cudaMalloc((void**)&dstats, (size_t)B * HQ * N * 2 * 4), "cudaMalloc row stats") ||
      check_cuda(cudaMalloc((void**)&didx, nidx * 8), "cudaMalloc indices") ||
      check_cuda(cudaMalloc((void**)&dmask, nimp), "cudaMalloc mask") ||
      check_cuda(cudaStreamCreate(&stream), "cudaStreamCreate"))
    return 4;
  if (check_cuda(cudaMemcpy(dq, hq, nq * 2, cudaMemcpyHostToDevice), "copy q") ||
      check_cuda(cudaMemcpy(dk, hk, nk * 2, cudaMemcpyHostToDevice), "copy k") ||
      check_cuda(cudaMemcpy(dv, hv, nk * 2, cudaMemcpyHostToDevice), "copy v"))
    return 5;

  const int64_t sq[4] = {(int64_t)HQ * N * D, (int64_t)N * D, D, 1};
  const int64_t sk[4] = {(int64_t)HK * N * D, (int64_t)N * D, D, 1};
  FILE* f;
  char path[4096];
  snprintf(path, sizeof(path), "%s.bin", argv[1]);
  f = fopen(path, "wb");
  if (!f) return 6;
  const int64_t header[8] = {B, HQ, HK, N, D, BUDGET, RECENT, POOL};
  fwrite(header, 8, 8, f);
  fwrite(hq, 2, nq, f);
  fwrite(hk, 2, nk, f);
  fwrite(hv, 2, nk, f);

  for (int call = 0; call < 2; ++call) {
    int rc;
    if (call == 0)
      rc = fe_evict(dq, sq, dk, sk, dv, sk, dout, dimp, didx, dmask, dstats, B, HQ, HK, N, D, FE_DTYPE_BF16, 1,
                    0.08838834764831845f, 0.02f, 0, 1, BUDGET, RECENT, POOL, (void*)stream);
    else
      rc = fe_evict_noalloc(dq, sq, dk, sk, dv, sk, dout, dimp, didx, dmask, B, HQ, HK, N, D, FE_DTYPE_BF16, 1,
                            0.08838834764831845f, 0.02f, 0, 1, BUDGET, RECENT, POOL, (void*)stream);
    if (check_fe(rc, call == 0 ? "fe_evict" : "fe_evict_noalloc")) return 7;
    if (check_cuda(cudaStreamSynchronize(stream), "synchronize")) return 8;
    int status = -1;
    if (check_fe(fe_device_status(0, 0, &status), "fe_device_status") || status != FE_STATUS_OK) return 9;
    if (check_cuda(cudaMemcpy(hout, dout, nq * 2, cudaMemcpyDeviceToHost), "copy out") ||
        check_cuda(cudaMemcpy(himp, dimp, nimp * 4, cudaMemcpyDeviceToHost), "copy importance") ||
        check_cuda(cudaMemcpy(hidx, didx, nidx * 8, cudaMemcpyDeviceToHost), "copy indices") ||
        check_cuda(cudaMemcpy(hmask, dmask, nimp, cudaMemcpyDeviceToHost), "copy mask"))
      return 10;
    fwrite(hout, 2, nq, f);
    fwrite(himp, 4, nimp, f);
    fwrite(hidx, 8, nidx, f);
    fwrite(hmask, 1, nimp, f);
  }
  fclose(f);
  cudaFree(dq);
  cudaFree(dk);
  cudaFree(dv);
  cudaFree(dout);
  cudaFree(dimp);
  cudaFree(dstats);
  cudaFree(didx);
  cudaFree(dmask);
  cudaStreamDestroy(stream);
  printf("ok abi %d\n", fe_abi_version());
  return 0;
}
