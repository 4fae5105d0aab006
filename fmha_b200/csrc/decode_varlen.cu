// decode_varlen.cu -- decode attention on the reference's packed varlen
// layout: K/V [sum_b S_b, Hkv, D] with cu_seqlens_kv[B+1]
// (fmha_host.cpp:143-157; the reference kernels index it at
// fmha_vectorized_fma_kernel.hpp:113-135), Q/O [B, Hq, 1, D].
//
// Work: batch row b has S_b = cu[b+1] - cu[b] rows per kv head; it is cut into
// 16-row tiles of NU = 16/SMAX_b kv heads each (SMAX_b = next power of two
// >= S_b), so short rows pack several heads into one tile and the score
// reduction/softmax are paid once per 16 rows, as in the dense kernels.
// Persistent warps take batch rows round-robin and walk the row's tiles; for
// each they prefetch every K/V/Q row into registers with 16-byte streaming
// loads, then run the shared tile math for the row's SMAX_b (a warp-uniform
// switch over the five instantiations).
//
// A row length outside [0, max_seqlen_kv] sets the device error word
// (FMHA_ERR_INVALID_ARG, site 5) and that row's output is left unwritten; a
// zero-length row produces zeros (the reference's empty sum).
//
// Compiled once per head_dim: -DFMHA_HEAD_DIM=128 or 256.
#include "decode_common.cuh"

#ifndef FMHA_HEAD_DIM
#error "compile with -DFMHA_HEAD_DIM=128 or 256"
#endif

namespace fmha {

template <int D, int SMAX, int G>
__device__ __forceinline__ void varlen_tile(const VarlenParams& P, int64_t b, int64_t c0, int s_len,
                                            int h0, int nu_valid, float* sc, int lane) {
  using T = Tile16<D, SMAX, G>;
  const int r0 = lane / T::LPR;
  const int cl = lane % T::LPR;
  const int hkv = P.num_heads_kv;
  // Q rows are prefetched with K/V unless that would not fit in registers
  // (many short units x many query heads); then they are loaded per slot.
  constexpr bool kQPre = T::LU * G <= 16;
  uint4 kr[T::NP], vr[T::NP], qr[kQPre ? T::LU : 1][kQPre ? G : 1];
#pragma unroll
  for (int p = 0; p < T::NP; ++p) {
    const int r = r0 * T::NP + p;
    const int u = r / SMAX, s = r % SMAX;
    const bool ok = s < s_len && u < nu_valid;
    const int64_t off = ((c0 + s) * hkv + h0 + u) * D + cl * 8;
    kr[p] = ok ? ldg_stream(P.K + off) : make_uint4(0, 0, 0, 0);
    vr[p] = ok ? ldg_stream(P.V + off) : make_uint4(0, 0, 0, 0);
  }
  const int64_t qrow0 = (b * hkv + h0) * G;  // first query row of the tile
  if constexpr (kQPre) {
#pragma unroll
    for (int us = 0; us < T::LU; ++us) {
      const int u = (r0 * T::NP + us * T::SPL) / SMAX;
#pragma unroll
      for (int g = 0; g < G; ++g)
        qr[us][g] = u < nu_valid ? ldg_stream(P.Q + (qrow0 + u * G + g) * D + cl * 8)
                                 : make_uint4(0, 0, 0, 0);
    }
  }
  auto loadK = [&](int p) { return kr[p]; };
  auto loadV = [&](int p) { return vr[p]; };
  auto loadQ = [&](int us, int u, int g) {
    if constexpr (kQPre) {
      return qr[us][g];
    } else {
      return ldg_stream(P.Q + (qrow0 + u * G + g) * D + cl * 8);
    }
  };
  auto store = [&](int u, const float (&acc)[G][8]) {
    if (u >= nu_valid) return;
    uint16_t* orow = P.O + (qrow0 + u * G) * D + cl * 8;
#pragma unroll
    for (int g = 0; g < G; ++g) stg_stream(orow + g * D, pack8_f16(acc[g]));
  };
  attend_tile16<D, SMAX, G>(loadK, loadV, loadQ, store, s_len, nu_valid, P.scale_log2, sc, lane);
}

template <int D, int G>
__global__ void __launch_bounds__(kLdgThreads) decode_varlen_kernel(const VarlenParams P) {
  constexpr int WPB = kLdgThreads / 32;
  __shared__ float sc_all[WPB][G * 16];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  float* sc = sc_all[warp];
  allow_dependent_launch();
  grid_dependency_wait();  // inputs and outputs may be written by the previous kernel
  // Warps take work items round-robin: item = (batch row, head range of hpi
  // heads, ~4 by default).
  // A long row (one head per tile) is thereby spread over several warps
  // instead of landing on one. The next item's cu_seqlens pair is loaded
  // while this one runs.
  const int hkv = P.num_heads_kv;
  const int qs = P.tiles_per_row;  // head ranges per row
  const int hpi = (hkv + qs - 1) / qs;
  const int64_t items = P.batch * qs;
  const int64_t stride = (int64_t)gridDim.x * WPB;
  int64_t it = (int64_t)blockIdx.x * WPB + warp;
  int c0n = 0, c1n = 0;
  if (it < items) {
    c0n = __ldg(P.cu_seqlens + it / qs);
    c1n = __ldg(P.cu_seqlens + it / qs + 1);
  }
  for (; it < items; it += stride) {
    const int64_t b = it / qs;
    const int q = (int)(it - b * qs);
    const int c0 = c0n;
    const int s_len = c1n - c0;
    if (it + stride < items) {
      c0n = __ldg(P.cu_seqlens + (it + stride) / qs);
      c1n = __ldg(P.cu_seqlens + (it + stride) / qs + 1);
    }
    if (s_len < 0 || s_len > P.max_seqlen) {
      if (lane == 0 && q == 0) report_device_error(P.err, 1u /* FMHA_ERR_INVALID_ARG */, 5u);
      continue;
    }
    const int smax = s_len <= 1 ? 1 : s_len <= 2 ? 2 : s_len <= 4 ? 4 : s_len <= 8 ? 8 : 16;
    const int nu = 16 / smax;
    const int hend = (q + 1) * hpi < hkv ? (q + 1) * hpi : hkv;
    for (int h0 = q * hpi; h0 < hend; h0 += nu) {
      const int nv = hend - h0 < nu ? hend - h0 : nu;
      switch (smax) {
        case 1: varlen_tile<D, 1, G>(P, b, c0, s_len, h0, nv, sc, lane); break;
        case 2: varlen_tile<D, 2, G>(P, b, c0, s_len, h0, nv, sc, lane); break;
        case 4: varlen_tile<D, 4, G>(P, b, c0, s_len, h0, nv, sc, lane); break;
        case 8: varlen_tile<D, 8, G>(P, b, c0, s_len, h0, nv, sc, lane); break;
        default: varlen_tile<D, 16, G>(P, b, c0, s_len, h0, nv, sc, lane); break;
      }
    }
  }
}

#define FMHA_CAT2(a, b) a##b
#define FMHA_CAT(a, b) FMHA_CAT2(a, b)

VarlenFn FMHA_CAT(varlen_kernel_d, FMHA_HEAD_DIM)(int g) {
  constexpr int D = FMHA_HEAD_DIM;
  switch (g) {
    case 1: return decode_varlen_kernel<D, 1>;
    case 2: return decode_varlen_kernel<D, 2>;
    case 4: return decode_varlen_kernel<D, 4>;
    case 8: return decode_varlen_kernel<D, 8>;
    default: return nullptr;
  }
}

}  // namespace fmha
