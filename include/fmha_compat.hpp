// fmha_compat.hpp -- source-level drop-in for the reference's launch helper.
//
// A code base written against HGLiu1998/fmha calls
//   launch_fmha_mfma_4x4x4(grid, block, stream, Q, K, V, O, cu_seqlens_kv,
//                          batch, num_heads_q, num_heads_kv, seqlen_q,
//                          head_dim_q, head_dim_kv, softmax_scale);
// (fmha_mfma_4x4x4_kernel.hpp:370-389, called from fmha_host.cpp:367,382,437)
// on the packed varlen layout: Q/O [B, Hq, 1, D], K/V [sum S_b, Hkv, D] with
// cu_seqlens_kv[B+1] (device int32), bf16 inputs and fp16 output. Including
// this header instead of the reference's kernel headers keeps that call site
// unchanged: the helper forwards to fmha_forward_varlen() of libfmha_b200.
//
// Differences a caller should know:
//  * grid and block are ignored (the library sizes its own persistent grid);
//  * seqlen_q must be 1 and head_dim_q == head_dim_kv in {128, 256}; every
//    row length must lie in 0..16 (the reference's own limit, scores[16]);
//  * Hq != Hkv means grouped-query attention (kv head h / (Hq/Hkv)); the
//    reference indexes K/V with the query head instead;
//  * the softmax weights stay fp32 (the reference's MFMA path rounds them to
//    bf16), so outputs agree with the reference to its own tolerance;
//  * the helper returns the library status (the reference returns void), so
//    existing call sites that ignore it still compile.
#ifndef FMHA_B200_FMHA_COMPAT_HPP
#define FMHA_B200_FMHA_COMPAT_HPP

#include <cuda_runtime.h>

#include "fmha.h"

inline fmha_status_t launch_fmha_mfma_4x4x4(dim3 /*grid*/, dim3 /*block*/, cudaStream_t stream,
                                            const void* Q, const void* K, const void* V, void* O,
                                            const int* cu_seqlens_kv, int batch,
                                            int num_heads_q, int num_heads_kv, int seqlen_q,
                                            int head_dim_q, int head_dim_kv,
                                            float softmax_scale) {
  if (seqlen_q != 1 || head_dim_q != head_dim_kv) return FMHA_ERR_UNSUPPORTED;
  return fmha_forward_varlen(Q, K, V, O, cu_seqlens_kv, batch, num_heads_q, num_heads_kv, 16,
                             head_dim_q, softmax_scale, reinterpret_cast<fmha_stream_t>(stream));
}

#endif  // FMHA_B200_FMHA_COMPAT_HPP
