/*
 * fmha_oracle.h -- CPU restatement of the reference's decode-attention math.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it. Nothing in the fmha_b200 product links or calls it.
 *
 * Parity pin: fmha_oracle_decode_thd() in ref-faithful mode (bf16 P, fp16 O)
 * is checked bit for bit against the reference's own do_validation()
 * (fmha_host.cpp:158-284), compiled from the reference sources by
 * oracle/Makefile into oracle/_ref/, and against the golden fixtures in
 * tests/golden/ that were produced by that build.
 */
#ifndef FMHA_ORACLE_H
#define FMHA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Counter-based seeded input generator shared bit-for-bit with the CUDA
 * harness generator (fmha_fill_normal_bf16): element i of tensor `tensor_id`
 * is a pure function of (seed, tensor_id, offset + i), so any shard or slice
 * regenerates independently of the GPU count. Values approximate N(0,1) by an
 * Irwin-Hall sum of twelve 16-bit uniforms, then round to bf16 (RNE). */
void fmha_oracle_gen_bf16(uint16_t* out, int64_t n, uint64_t seed,
                          uint32_t tensor_id, int64_t offset);

/* Decode attention in the [B,H,S,D] layout of the C ABI.
 *   Q [B,Hq,1,D] bf16, K/V [B,Hkv,S,D] bf16, kv head of query head h is
 *   h / (Hq/Hkv).
 * p_bf16 = 0 ("exact"): fp32 P, output written to O_f32 (may be NULL) and,
 *   fp16-rounded, to O_f16 (may be NULL).
 * p_bf16 = 1 ("ref-faithful"): P rounded to bf16 before P.V, as
 *   fmha_host.cpp:215,225 does.
 * Arithmetic order follows fmha_host.cpp:179-243 (dot in d order, scale
 * after the dot, expf(s - max), sum in s order, divide, P.V in s order).
 * Parallelised over batch with OpenMP when built with -fopenmp. */
void fmha_oracle_decode_bhsd(const uint16_t* Q, const uint16_t* K,
                             const uint16_t* V, int64_t batch, int num_heads_q,
                             int num_heads_kv, int seqlen_kv, int head_dim,
                             int p_bf16, float* O_f32, uint16_t* O_f16);

/* Same math on the reference's packed varlen layout: K/V [sum S_b, Hkv, D]
 * with cu_seqlens_kv[B+1] (fmha_host.cpp:143-157,170-193). */
void fmha_oracle_decode_thd(const uint16_t* Q, const uint16_t* K,
                            const uint16_t* V, const int32_t* cu_seqlens_kv,
                            int64_t batch, int num_heads_q, int num_heads_kv,
                            int head_dim, int p_bf16, float* O_f32,
                            uint16_t* O_f16);

/* Number of OpenMP threads the oracle uses (1 if built without OpenMP). */
int fmha_oracle_threads(void);
void fmha_oracle_set_threads(int n);

/* bf16 / fp16 conversions used by the oracle (RNE). */
float fmha_oracle_bf16_to_f32(uint16_t x);
uint16_t fmha_oracle_f32_to_bf16(float x);
uint16_t fmha_oracle_f32_to_f16(float x);
float fmha_oracle_f16_to_f32(uint16_t x);

#ifdef __cplusplus
}
#endif

#endif /* FMHA_ORACLE_H */
