// decode_bulk.cu -- "bulk" kernel family: persistent CTAs (one per SM) that
// stream contiguous runs of units through a shared-memory ring with 1-D
// cp.async.bulk copies completing on mbarriers, consumed by 8-16 compute
// warps (the launch picks the count per shape).
//
// Per CTA: warp 0 lane 0 is the producer; the other warps consume. The CTA
// owns chunks c = blockIdx.x + k*gridDim.x (k = 0, 1, ...); chunk c covers
// units [c*CU, min((c+1)*CU, units)), i.e. three contiguous byte ranges (K
// slabs, V slabs, Q rows), each moved by one bulk copy into ring stage
// k % NS. A chunk holds CT tiles; consumer warp w takes flat jobs
// f = w, w+ncw, ... (chunk f / CT, tile f % CT), waits for the stage's `full`
// phase, computes the tile from shared memory, arrives on the stage's `empty`
// barrier (count CT) and streams its fp16 output rows straight to global.
//
// Compiled once per head_dim: -DFMHA_HEAD_DIM=128 or 256.
#include "decode_common.cuh"

#ifndef FMHA_HEAD_DIM
#error "compile with -DFMHA_HEAD_DIM=128 or 256"
#endif

namespace fmha {

template <int D, int SMAX, int G>
__global__ void __launch_bounds__(kBulkMaxThreads, 1) decode_bulk_kernel(const Params P) {
  using T = Tile16<D, SMAX, G>;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ncw = (blockDim.x >> 5) - 1;  // consumer warps
  const int NS = P.stages;
  const uint32_t full0 = smem_u32(smem);
  const uint32_t empty0 = full0 + 8u * NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 16 * NS);
  volatile int* issued_ctr = abort_flag + 1;  // chunks whose copies are armed
  const uint32_t ring0 = smem_u32(smem + P.ring_off);

  allow_dependent_launch();
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(full0 + 8u * i, 1);
      mbar_init(empty0 + 8u * i, P.tiles_per_chunk);
    }
    *abort_flag = 0;
    *issued_ctr = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Inputs and outputs may be written by the previous kernel of the stream.
  grid_dependency_wait();
  __syncthreads();

  const int my_chunks =
      P.chunks > (int)blockIdx.x ? (P.chunks - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int s_len = P.s_len;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane != 0) return;
    const uint64_t policy = policy_evict_first();
    int issued = 0;
    const int produce = (P.flags & kFlagStallProducer) ? 0 : my_chunks;
    for (int k = 0; k < produce; ++k) {
      const int st = k % NS;
      if (k >= NS && !mbar_wait(empty0 + 8u * st, ((k / NS) - 1) & 1, abort_flag, P.err,
                                P.wait_timeout_ns, kSiteProducerEmpty))
        break;
      const int64_t chunk = (int64_t)blockIdx.x + (int64_t)k * gridDim.x;
      const int64_t u0 = chunk * P.units_per_chunk;
      const int64_t left = P.units - u0;
      const int nu = left < P.units_per_chunk ? (int)left : P.units_per_chunk;
      const uint32_t kb = (uint32_t)nu * (uint32_t)s_len * (uint32_t)(D * 2);
      const uint32_t qb = (uint32_t)nu * (uint32_t)(G * D * 2);
      const uint32_t bar = full0 + 8u * st;
      const uint32_t dst = ring0 + (uint32_t)st * P.stage_bytes;
      mbar_arrive_expect_tx(bar, 2 * kb + qb);
      bulk_g2s(dst, P.K + u0 * s_len * D, kb, bar, policy);
      bulk_g2s(dst + P.v_off, P.V + u0 * s_len * D, kb, bar, policy);
      bulk_g2s(dst + P.q_off, P.Q + u0 * G * D, qb, bar, policy);
      issued = k + 1;
      __threadfence_block();  // the expect_tx above is visible before the count
      *issued_ctr = issued;
    }
    // Never leave the CTA with copies in flight into its shared memory.
    const int first = issued > NS ? issued - NS : 0;
    for (int k = first; k < issued; ++k)
      mbar_wait(full0 + 8u * (k % NS), (k / NS) & 1, nullptr, P.err, P.wait_timeout_ns,
                kSiteDrain);
    return;
  }

  // ------------------------------------------------------------ consumers
  const int cw = warp - 1;
  float* sc = reinterpret_cast<float*>(smem + P.sc_off) + cw * T::SC;
  const int r0 = lane / T::LPR;
  const int cl = lane % T::LPR;
  const int CT = P.tiles_per_chunk;
  const int jobs = my_chunks * CT;
  for (int f = cw; f < jobs; f += ncw) {
    const int k = f / CT;
    const int j = f - k * CT;
    const int st = k % NS;
    // A parity wait is only meaningful once chunk k's phase is armed: before
    // that the stage may still be in an older phase whose parity differs, and
    // try_wait.parity would report it complete.
    if (!wait_issued(issued_ctr, k, abort_flag, P.err, P.wait_timeout_ns)) break;
    if (!mbar_wait(full0 + 8u * st, (k / NS) & 1, abort_flag, P.err, P.wait_timeout_ns,
                   kSiteConsumerFull))
      break;
    const int64_t chunk = (int64_t)blockIdx.x + (int64_t)k * gridDim.x;
    const int64_t tile_u0 = chunk * P.units_per_chunk + (int64_t)j * T::NU;
    const int64_t left = P.units - tile_u0;
    const int uv = left <= 0 ? 0 : (left < T::NU ? (int)left : T::NU);
    if (uv > 0) {
      const uint32_t sbase = ring0 + (uint32_t)st * P.stage_bytes;
      const uint32_t kbase = sbase + (uint32_t)(j * T::NU * s_len) * (D * 2) + cl * 16;
      const uint32_t vbase = kbase + P.v_off;
      const uint32_t qbase = sbase + P.q_off + (uint32_t)(j * T::NU) * (G * D * 2) + cl * 16;
      auto row_off = [&](int p) -> uint32_t {
        const int r = r0 * T::NP + p;
        return (uint32_t)((r / SMAX) * s_len + (r % SMAX)) * (D * 2);
      };
      auto loadK = [&](int p) { return lds128(kbase + row_off(p)); };
      auto loadV = [&](int p) { return lds128(vbase + row_off(p)); };
      auto loadQ = [&](int, int u, int g) { return lds128(qbase + (uint32_t)(u * G + g) * (D * 2)); };
      auto store = [&](int u, const float (&acc)[G][8]) {
        if (u >= uv) return;
        uint16_t* orow = P.O + (tile_u0 + u) * (G * D) + cl * 8;
#pragma unroll
        for (int g = 0; g < G; ++g) stg_stream(orow + g * D, pack8_f16(acc[g]));
      };
      if constexpr (G >= kMmaMinHeads && SMAX >= 8) {
        // Four or more query heads per unit of 5..16 rows: tensor-core tile,
        // one unit at a time (rows past s_len, including the next unit's, are
        // masked). Measured: G=8 S=16 3.2 -> 6.7-6.9 TB/s (D=256); for G=2 the
        // fp32 CUDA-core tile is faster.
#pragma unroll
        for (int u = 0; u < T::NU; ++u) {
          if (u >= uv) break;
          const int ju = j * T::NU + u;
          const uint32_t k0 = sbase + (uint32_t)(ju * s_len) * (D * 2);
          attend_unit_mma<D, G, SMAX == 8>(k0, k0 + P.v_off, sbase + P.q_off + (uint32_t)ju * (G * D * 2),
                                s_len, P.scale_log2, P.O + (tile_u0 + u) * (G * D), lane);
        }
      } else {
        attend_tile16<D, SMAX, G>(loadK, loadV, loadQ, store, s_len, uv, P.scale_log2, sc, lane);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8u * st);  // stage's shared reads are done
  }
}

#define FMHA_CAT2(a, b) a##b
#define FMHA_CAT(a, b) FMHA_CAT2(a, b)

// Lookup of the instantiation for (SMAX, G) at this translation unit's D.
KernelFn FMHA_CAT(bulk_kernel_d, FMHA_HEAD_DIM)(int smax, int g) {
  constexpr int D = FMHA_HEAD_DIM;
#define FMHA_G(SM)                                      \
  switch (g) {                                          \
    case 1: return decode_bulk_kernel<D, SM, 1>;        \
    case 2: return decode_bulk_kernel<D, SM, 2>;        \
    case 4: return decode_bulk_kernel<D, SM, 4>;        \
    case 8: return decode_bulk_kernel<D, SM, 8>;        \
    default: return nullptr;                            \
  }
  switch (smax) {
    case 1: FMHA_G(1)
    case 2: FMHA_G(2)
    case 4: FMHA_G(4)
    case 8: FMHA_G(8)
    case 16: FMHA_G(16)
    default: return nullptr;
  }
#undef FMHA_G
}

}  // namespace fmha
