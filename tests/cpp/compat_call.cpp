// Calls the library through the reference's own launch-helper signature
// (include/fmha_compat.hpp) exactly as fmha_host.cpp:367-371 does, and
// compares the output bit for bit with a direct fmha_forward_varlen call.
// Exit 0 on success. Built and run by tests/test_compat_gpu.py.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "fmha_compat.hpp"

#define CEIL_DIV(a, b) (a + b - 1) / b

int main() {
  const int batch = 37, hq = 16, hkv = 16, d = 128;
  std::vector<int32_t> sl(batch), cu(batch + 1, 0);
  if (fmha_seqlens_poisson(batch, 16, 42u, 4.0, sl.data()) != FMHA_OK) return 2;
  for (int b = 0; b < batch; ++b) cu[b + 1] = cu[b] + sl[b];
  const long long nq = (long long)batch * hq * d, nkv = (long long)cu[batch] * hkv * d;
  void *Q, *K, *V, *O1, *O2;
  int* dcu;
  cudaMalloc(&Q, nq * 2);
  cudaMalloc(&K, nkv * 2);
  cudaMalloc(&V, nkv * 2);
  cudaMalloc(&O1, nq * 2);
  cudaMalloc(&O2, nq * 2);
  cudaMalloc(&dcu, (batch + 1) * 4);
  cudaMemcpy(dcu, cu.data(), (batch + 1) * 4, cudaMemcpyHostToDevice);
  fmha_fill_normal_bf16(Q, nq, 1, 1, 0, nullptr);
  fmha_fill_normal_bf16(K, nkv, 1, 2, 0, nullptr);
  fmha_fill_normal_bf16(V, nkv, 1, 3, 0, nullptr);
  dim3 gridDim(1, CEIL_DIV(hq, 16), batch);
  dim3 blockDim(256, 1, 1);
  fmha_status_t s1 = launch_fmha_mfma_4x4x4(gridDim, blockDim, 0, Q, K, V, O1, dcu, batch, hq,
                                            hkv, 1, d, d, 1.0f / std::sqrt((float)d));
  fmha_status_t s2 = fmha_forward_varlen(Q, K, V, O2, dcu, batch, hq, hkv, 16, d, 0.0f, nullptr);
  fmha_status_t s3 = launch_fmha_mfma_4x4x4(gridDim, blockDim, 0, Q, K, V, O1, dcu, batch, hq,
                                            hkv, 2, d, d, 1.0f);
  if (cudaDeviceSynchronize() != cudaSuccess) return 3;
  std::vector<uint16_t> a(nq), b(nq);
  cudaMemcpy(a.data(), O1, nq * 2, cudaMemcpyDeviceToHost);
  cudaMemcpy(b.data(), O2, nq * 2, cudaMemcpyDeviceToHost);
  const bool same = std::memcmp(a.data(), b.data(), nq * 2) == 0;
  std::printf("status %d %d %d same %d\n", s1, s2, s3, same);
  return (s1 == FMHA_OK && s2 == FMHA_OK && s3 == FMHA_ERR_UNSUPPORTED && same) ? 0 : 1;
}
