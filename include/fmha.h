/*
 * fmha.h -- C ABI of the B200 (sm_100a) batched flash-decode attention library
 * (libfmha_b200.so).
 *
 * The hot path is decode attention with one query token per (batch row, head):
 *
 *   O[b,h,:] = softmax(Q[b,h,:] . K[b,kvh,:,:]^T / sqrt(D)) . V[b,kvh,:,:]
 *   kvh = h / (num_heads_q / num_heads_kv)              (grouped-query heads)
 *
 * Q/K/V are bf16, the softmax and both contractions run in fp32 (P is never
 * rounded), O is fp16.
 *
 * Reference interface this replaces: the inline launch helper
 *   launch_fmha_mfma_4x4x4(grid, block, stream, Q, K, V, O, cu_seqlens_kv,
 *                          batch, num_heads_q, num_heads_kv, seqlen_q,
 *                          head_dim_q, head_dim_kv, softmax_scale)
 * (HGLiu1998/fmha fmha_mfma_4x4x4_kernel.hpp:370-389, called from
 * fmha_host.cpp:367,382,437). That helper takes a launch shape and a packed
 * varlen K/V layout; this ABI takes the [B,H,S,D] layout and chooses its own
 * launch shape; fmha_forward_varlen() takes the reference's packed layout.
 *
 * Conventions shared by every entry point:
 *  - pointers are caller-owned device pointers, 16-byte aligned; the library
 *    never frees or keeps them;
 *  - calls are asynchronous on `stream` (0 = legacy default stream) and never
 *    exit, abort or trap: problems come back as an fmha_status_t;
 *  - argument validation happens before any CUDA call, so a rejected call has
 *    no side effects and needs no GPU;
 *  - thread-safe: the only state is a per-device cache of the SM count and of
 *    per-kernel shared-memory attributes, filled under a mutex.
 */
#ifndef FMHA_B200_FMHA_H
#define FMHA_B200_FMHA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t, declared here so this header needs no CUDA. */
typedef struct CUstream_st* fmha_stream_t;

typedef enum {
  FMHA_OK = 0,
  FMHA_ERR_INVALID_ARG = 1,  /* null pointer, non-positive size, Hq % Hkv != 0 */
  FMHA_ERR_UNSUPPORTED = 2,  /* head_dim not 128/256, seqlen_kv not 1..16,
                                Hq/Hkv not 1, 2, 4 or 8 */
  FMHA_ERR_MISALIGNED = 3,   /* a pointer not 16-byte aligned */
  FMHA_ERR_CUDA = 4,         /* a CUDA runtime call or the launch failed */
  FMHA_ERR_DEVICE_TIMEOUT = 5 /* a kernel's bounded wait ran out (read with
                                 fmha_device_error) */
} fmha_status_t;

/* Kernel family selector for fmha_forward_variant(). */
typedef enum {
  FMHA_VARIANT_AUTO = 0, /* per-shape choice measured on B200 */
  FMHA_VARIANT_BULK = 1, /* persistent CTAs, cp.async.bulk + mbarrier ring */
  FMHA_VARIANT_LDG = 2   /* persistent warps, 16-byte vector loads */
} fmha_variant_t;

/*
 * fmha_forward -- decode attention on the [B,H,S,D] layout.
 *   Q [batch, num_heads_q, 1, head_dim]        bf16
 *   K [batch, num_heads_kv, seqlen_kv, head_dim] bf16
 *   V [batch, num_heads_kv, seqlen_kv, head_dim] bf16
 *   O [batch, num_heads_q, 1, head_dim]        fp16 (written)
 * scale = 1/sqrt(head_dim), as the reference host passes
 * (fmha_host.cpp:371). head_dim in {128, 256}; seqlen_kv in 1..16 (rows past
 * seqlen_kv of the 16-row tile are masked with -inf); num_heads_q /
 * num_heads_kv in {1, 2, 4, 8}. batch == 0 is a no-op returning FMHA_OK.
 * Replaces launch_fmha_mfma_4x4x4 (fmha_mfma_4x4x4_kernel.hpp:370-389).
 */
fmha_status_t fmha_forward(const void* Q, const void* K, const void* V,
                           void* O, int batch, int num_heads_q,
                           int num_heads_kv, int seqlen_kv, int head_dim,
                           fmha_stream_t stream);

/* fmha_forward with an explicit kernel family (for benchmarking both).
 * Same reference counterpart as fmha_forward. */
fmha_status_t fmha_forward_variant(const void* Q, const void* K, const void* V,
                                   void* O, int batch, int num_heads_q,
                                   int num_heads_kv, int seqlen_kv,
                                   int head_dim, int variant,
                                   fmha_stream_t stream);

/*
 * fmha_forward_varlen -- decode attention on the reference's packed varlen
 * K/V layout:
 *   Q [batch, num_heads_q, 1, head_dim]                 bf16
 *   K [cu_seqlens_kv[batch], num_heads_kv, head_dim]    bf16 (rows of batch b
 *   V [cu_seqlens_kv[batch], num_heads_kv, head_dim]    are cu[b] .. cu[b+1]-1)
 *   O [batch, num_heads_q, 1, head_dim]                 fp16 (written)
 *   cu_seqlens_kv [batch + 1] int32, device memory, cu[0] = 0, non-decreasing.
 * Each row length cu[b+1]-cu[b] must lie in 0..max_seqlen_kv (max_seqlen_kv
 * in 1..16); a longer row is skipped and reported through fmha_device_error
 * (FMHA_ERR_INVALID_ARG), an empty row yields zeros. softmax_scale == 0 means
 * 1/sqrt(head_dim); a negative, NaN or infinite scale is rejected with
 * FMHA_ERR_INVALID_ARG. Same grouping kvh = h / (Hq/Hkv) as fmha_forward.
 * Replaces launch_fmha_mfma_4x4x4 with its own argument list
 * (fmha_mfma_4x4x4_kernel.hpp:370-389; the layout of fmha_host.cpp:143-157).
 */
fmha_status_t fmha_forward_varlen(const void* Q, const void* K, const void* V,
                                  void* O, const int32_t* cu_seqlens_kv,
                                  int batch, int num_heads_q, int num_heads_kv,
                                  int max_seqlen_kv, int head_dim,
                                  float softmax_scale, fmha_stream_t stream);

/* fmha_forward_varlen with an explicit kernel: FMHA_VARIANT_BULK runs the
 * chunk ring (whole packed rows staged by cp.async.bulk into a shared-memory
 * byte ring), FMHA_VARIANT_LDG the register-prefetch kernel (persistent warps,
 * 16-byte vector loads), FMHA_VARIANT_AUTO the default (the chunk ring, unless
 * the environment variable FMHA_VARLEN_KERNEL=ldg is set when the call is
 * made). Same reference counterpart as fmha_forward_varlen. */
fmha_status_t fmha_forward_varlen_variant(const void* Q, const void* K,
                                          const void* V, void* O,
                                          const int32_t* cu_seqlens_kv,
                                          int batch, int num_heads_q,
                                          int num_heads_kv, int max_seqlen_kv,
                                          int head_dim, float softmax_scale,
                                          int variant, fmha_stream_t stream);

/*
 * fmha_forward_append -- one decode step with a KV cache: writes this step's
 * K/V rows into the cache and attends over the whole prefix, in one kernel.
 *   K_cache, V_cache [batch, num_heads_kv, cache_seqlen, head_dim] bf16; rows
 *     0..seqlen_kv-2 hold the earlier steps (read), row seqlen_kv-1 is
 *     written from K_new / V_new;
 *   K_new, V_new [batch, num_heads_kv, 1, head_dim] bf16 (this step);
 *   Q, O as in fmha_forward.
 * O equals fmha_forward on the first seqlen_kv rows of the updated cache
 * (the new row is taken from K_new/V_new directly, not re-read). seqlen_kv in
 * 1..16, cache_seqlen >= seqlen_kv. No reference counterpart: the reference
 * benchmark has no cache update; this is the producer side of its decode
 * step.
 */
fmha_status_t fmha_forward_append(const void* Q, void* K_cache, void* V_cache,
                                  const void* K_new, const void* V_new, void* O,
                                  int batch, int num_heads_q, int num_heads_kv,
                                  int seqlen_kv, int cache_seqlen, int head_dim,
                                  fmha_stream_t stream);

/*
 * fmha_forward_noalloc -- fmha_forward for callers that cannot allocate
 * device memory (an allocator hook that must not re-enter the allocator, a
 * plug-in whose host owns every device allocation, a fixed memory budget).
 * Same arguments, layouts, scale and status codes as fmha_forward; it always
 * runs the ldg kernel family. Its only scratch, the kernel's work-schedule
 * slot, is a 1152-byte static device array inside the library (held by every
 * GPU that loads it until exit), so no call ever allocates. The first call
 * on a device looks the array's address up and should come before any stream
 * capture. All calls share the array: calls overlapping on the GPU race for
 * it, and the one that finds it taken runs a static schedule (its output is
 * still complete). Limits: at most 4095 CTAs per launch and
 * batch * num_heads_kv <= 2^30, else FMHA_ERR_UNSUPPORTED.
 * No counterpart in the reference (its host allocates everything itself).
 */
fmha_status_t fmha_forward_noalloc(const void* Q, const void* K, const void* V,
                                   void* O, int batch, int num_heads_q,
                                   int num_heads_kv, int seqlen_kv,
                                   int head_dim, fmha_stream_t stream);

/* Human-readable name of a status code (static storage). Reference
 * counterpart: the HIP_CHECK error text (fmha_host.cpp:26-35). */
const char* fmha_status_string(fmha_status_t status);

/* Reads and clears the device-side error word of the current device: 0 when
 * no kernel has reported a problem, else a code whose low byte is the
 * fmha_status_t and whose upper bits say where a bounded wait gave up.
 * Synchronises the current device. No reference counterpart (the reference
 * kernels have no device-side error path). */
fmha_status_t fmha_device_error(int* code);

/*
 * fmha_fill_normal_bf16 -- benchmark/validation harness utility: fills
 * dst[0..n) with the seeded counter-based values
 *   x = bf16( (sum of twelve 16-bit uniforms of splitmix64(seed, tensor_id,
 *             offset + i)) normalised to mean 0, variance 1 )
 * on `stream`. Element i depends only on (seed, tensor_id, offset + i), so a
 * batch shard regenerates the same values whatever the GPU count.
 * Reference counterpart: initialize_random_bfloat16 (fmha_host.cpp:132-141),
 * which draws unseeded U[-1,1] on the host.
 */
fmha_status_t fmha_fill_normal_bf16(void* dst, int64_t n, uint64_t seed,
                                    uint32_t tensor_id, int64_t offset,
                                    fmha_stream_t stream);

/*
 * fmha_seqlens_poisson -- benchmark utility (host memory, no GPU): the
 * reference benchmark's per-row KV lengths, drawn from Poisson(lambda) with a
 * std::mt19937(seed) and redrawn until they lie in [2, max_seqlen_kv].
 * Reference counterpart: FMHAConfig::generate_seqlens_kv
 * (fmha_host.cpp:58-72), which uses seed 42 and lambda 4; with the same C++
 * standard library the sequences are identical.
 */
fmha_status_t fmha_seqlens_poisson(int batch, int max_seqlen_kv, uint32_t seed,
                                   double lambda, int32_t* out);

/* Test hook for the device-side failure path: while `on` is non-zero every
 * fmha_forward / fmha_forward_variant call runs the dense bulk kernel with
 * its producer issuing no copies (the varlen and append entry points ignore
 * the hook) and a 20 ms wait bound, so each consumer's bounded wait runs out,
 * the kernel records FMHA_ERR_DEVICE_TIMEOUT in the device error word and
 * returns without trapping (output is left unwritten). No reference
 * counterpart. */
void fmha_test_inject_stall(int on);

/* Library version string, e.g. "fmha_b200 0.1.0 sm_100a". */
const char* fmha_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FMHA_B200_FMHA_H */
