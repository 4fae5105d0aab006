// decode_varlen_ring.cu -- the packed-varlen decode kernel built as a
// producer/consumer ring (the register-prefetch form is decode_varlen.cu).
//
// Layout: K/V [sum_b S_b, Hkv, D] with cu_seqlens_kv[B+1]
// (fmha_host.cpp:143-157), Q/O [B, Hq, 1, D]. Batch row b (S_b = cu[b+1] -
// cu[b]) is cut into 16-row tiles of NU = 16/SMAX_b kv heads, SMAX_b the
// next power of two >= S_b.
//
// Per CTA (persistent, one per SM): a contiguous range of batch rows.
//  * Producers (warps 0..P.producers-1, 6 by default) all walk all tiles of the
//    CTA's rows, reading cu_seqlens 31 rows per warp load; producer w gathers
//    tiles k with k % P.producers == w into ring stage k % NS. Lane l
//    copies with 16-byte cp.async exactly the pieces consumer lane l will read
//    (each K/V row is one 512-byte or two 256-byte coalesced warp accesses),
//    then the tile's contiguous query rows; each lane signals completion on
//    the stage's `full` mbarrier with cp.async.mbarrier.arrive.noinc, and
//    lane 0 writes a tile descriptor and adds one ordinary arrive (count 33).
//    NS is a multiple of the producer count, so producer w arms only its own
//    stages and waits on each stage's `empty` phases in order.
//  * Consumers: NS is a multiple of the consumer count and consumer c owns
//    stages c, c+ncw, ...; it takes tiles k = c, c+ncw, ... so it consumes
//    every phase of its stages in order and each parity wait names the next
//    phase. It runs the shared 16-row tile math from shared memory for the
//    tile's SMAX, streams fp16 rows to O and releases the stage on `empty`.
//
// A row length outside [0, max_seqlen_kv] sets the device error word
// (FMHA_ERR_INVALID_ARG, site 5) and the row is skipped; a zero-length row
// yields zeros. Every wait is bounded (globaltimer) and never traps.
//
// Compiled once per head_dim: -DFMHA_HEAD_DIM=128 or 256.
#include "decode_common.cuh"

#ifndef FMHA_HEAD_DIM
#error "compile with -DFMHA_HEAD_DIM=128 or 256"
#endif

namespace fmha {

namespace {

struct TileDesc {
  int64_t b;   // batch row
  int s_len;   // rows per head
  int h0;      // first kv head of the tile
  int nv;      // kv heads in the tile
  int smax;    // power of two >= s_len (1..16)
};
static_assert(sizeof(TileDesc) <= kVarlenDescBytes, "descriptor slot");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "l"(policy)
               : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ int smax_of(int s) {
  return s <= 1 ? 1 : s <= 2 ? 2 : s <= 4 ? 4 : s <= 8 ? 8 : 16;
}

// Producer lane l copies the tile rows consumer lane l reads: row
// r = r0*NP + p is unit r >> lsm, position r & (smax-1). Rows past s_len or
// past nv are not copied (the consumer masks them).
template <int D, int G>
__device__ __forceinline__ void gather_tile(const VarlenParams& P, uint32_t kdst, uint32_t qdst,
                                            int64_t b, int c0, int s_len, int lsm, int h0,
                                            int nv, int lane, uint64_t policy) {
  constexpr int LPR = D / 8, RPP = 32 / LPR, NP = 16 / RPP;
  const int r0 = lane / LPR;
  const int cl = lane % LPR;
  const int hkv = P.num_heads_kv;
  const int smask = (1 << lsm) - 1;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int r = r0 * NP + p;
    const int u = r >> lsm, s = r & smask;
    if (s < s_len && u < nv) {
      const int64_t off = ((int64_t)(c0 + s) * hkv + h0 + u) * D + cl * 8;
      const uint32_t d = kdst + (uint32_t)r * (D * 2) + cl * 16;
      cp_async16(d, P.K + off, policy);
      cp_async16(d + 16 * D * 2, P.V + off, policy);
    }
  }
  const int64_t q0 = (b * hkv + h0) * G * D;
  const int qpieces = nv * G * LPR;
  for (int e = lane; e < qpieces; e += 32)
    cp_async16(qdst + (uint32_t)e * 16, P.Q + q0 + (int64_t)e * 8, policy);
}

template <int D, int SMAX, int G>
__device__ __forceinline__ void consume_tile(const VarlenParams& P, const TileDesc& t,
                                             uint32_t kbase, uint32_t qbase, float* sc,
                                             int lane) {
  using T = Tile16<D, SMAX, G>;
  const int r0 = lane / T::LPR;
  const int cl = lane % T::LPR;
  const uint32_t kl = kbase + cl * 16;
  const uint32_t vl = kl + 16 * D * 2;
  const uint32_t ql = qbase + cl * 16;
  auto loadK = [&](int p) { return lds128(kl + (uint32_t)(r0 * T::NP + p) * (D * 2)); };
  auto loadV = [&](int p) { return lds128(vl + (uint32_t)(r0 * T::NP + p) * (D * 2)); };
  auto loadQ = [&](int, int u, int g) { return lds128(ql + (uint32_t)(u * G + g) * (D * 2)); };
  const int64_t qrow0 = (t.b * P.num_heads_kv + t.h0) * G;
  auto store = [&](int u, const float (&acc)[G][8]) {
    if (u >= t.nv) return;
    uint16_t* orow = P.O + (qrow0 + u * G) * D + cl * 8;
#pragma unroll
    for (int g = 0; g < G; ++g) stg_stream(orow + g * D, pack8_f16(acc[g]));
  };
  attend_tile16<D, SMAX, G>(loadK, loadV, loadQ, store, t.s_len, t.nv, P.scale_log2, sc, lane);
}

}  // namespace

template <int D, int G>
__global__ void __launch_bounds__(kBulkMaxThreads, 1)
    decode_varlen_ring_kernel(const VarlenParams P) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NS = P.stages;
  const uint32_t full0 = smem_u32(smem);
  const uint32_t empty0 = full0 + 8u * NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 16 * NS);
  volatile int* total_ctr = abort_flag + 1;  // tile count once the producers are done, else -1
  unsigned char* ring = smem + P.ring_off;
  const uint32_t ring0 = smem_u32(ring);
  constexpr uint32_t kRow = D * 2;               // bytes per K/V row
  constexpr uint32_t kKOff = kVarlenDescBytes;   // 16 K rows, then 16 V rows
  constexpr uint32_t kQOff = kKOff + 32 * kRow;  // up to 16*G Q rows

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(full0 + 8u * i, 33);  // 32 cp.async completions + the descriptor arrive
      mbar_init(empty0 + 8u * i, 1);
    }
    *abort_flag = 0;
    *total_ctr = -1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const int64_t row_lo = P.batch * blockIdx.x / gridDim.x;
  const int64_t row_hi = P.batch * (blockIdx.x + 1) / gridDim.x;

  if (warp < P.producers) {
    // ----------------------------------------------------------- producers
    const int hkv = P.num_heads_kv;
    const uint64_t policy = policy_evict_first();
    int k = 0;
    bool stop = false;
    for (int64_t base = row_lo; base < row_hi && !stop; base += 31) {
      // Lane l holds cu[base + l]; a window covers 31 rows (32 boundaries).
      const int64_t idx = base + lane;
      const int cu_l = idx <= row_hi ? __ldg(P.cu_seqlens + idx) : 0;
      const int nrows = row_hi - base < 31 ? (int)(row_hi - base) : 31;
      for (int i = 0; i < nrows && !stop; ++i) {
        const int c0 = __shfl_sync(kFullMask, cu_l, i);
        const int s_len = __shfl_sync(kFullMask, cu_l, i + 1) - c0;
        const int64_t b = base + i;
        if (s_len < 0 || s_len > P.max_seqlen) {
          if (lane == 0 && warp == 0) report_device_error(P.err, 1u /* FMHA_ERR_INVALID_ARG */, 5u);
          continue;
        }
        const int smax = smax_of(s_len);
        const int nu = 16 / smax;
        for (int h0 = 0; h0 < hkv; h0 += nu, ++k) {
          if (k % P.producers != warp) continue;
          const int nv = hkv - h0 < nu ? hkv - h0 : nu;
          const int st = k % NS;
          if (k >= NS && !mbar_wait(empty0 + 8u * st, ((k / NS) - 1) & 1, abort_flag, P.err,
                                    P.wait_timeout_ns, kSiteProducerEmpty)) {
            stop = true;
            break;
          }
          const uint32_t sdst = ring0 + (uint32_t)st * P.stage_bytes;
          const uint32_t bar = full0 + 8u * st;
          gather_tile<D, G>(P, sdst + kKOff, sdst + kQOff, b, c0, s_len, 31 - __clz(smax), h0,
                            nv, lane, policy);
          cp_async_arrive_noinc(bar);  // fires when this lane's copies have landed
          if (lane == 0) {
            TileDesc* dsc = reinterpret_cast<TileDesc*>(ring + (size_t)st * P.stage_bytes);
            dsc->b = b;
            dsc->s_len = s_len;
            dsc->h0 = h0;
            dsc->nv = nv;
            dsc->smax = smax;
            mbar_arrive(bar);  // releases the descriptor with the phase
          }
        }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // this lane's copies have landed
    if (lane == 0) {
      if (warp == 0) {
        __threadfence_block();
        *total_ctr = k;  // every producer walks the same tiles
      }
      if (stop) *abort_flag = 1;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - P.producers;
  const int ncw = (blockDim.x >> 5) - P.producers;
  float* sc = reinterpret_cast<float*>(smem + P.sc_off) + cw * (G * 16);
  for (int k = cw;; k += ncw) {
    const int st = k % NS;
    const uint32_t bar = full0 + 8u * st;
    const uint32_t parity = (k / NS) & 1;
    bool have = mbar_try_wait(bar, parity);
    if (!have) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) {
          have = true;
          break;
        }
        const int tot = *total_ctr;
        if ((tot >= 0 && k >= tot) || *abort_flag) break;
        if ((it & 63u) == 0 && globaltimer_ns() - t0 > P.wait_timeout_ns) {
          report_device_error(P.err, 5u /* FMHA_ERR_DEVICE_TIMEOUT */, kSiteConsumerFull);
          *abort_flag = 1;
          break;
        }
      }
    }
    if (!have) break;
    const TileDesc t = *reinterpret_cast<const TileDesc*>(ring + (size_t)st * P.stage_bytes);
    const uint32_t sb = ring0 + (uint32_t)st * P.stage_bytes;
    switch (t.smax) {
      case 1: consume_tile<D, 1, G>(P, t, sb + kKOff, sb + kQOff, sc, lane); break;
      case 2: consume_tile<D, 2, G>(P, t, sb + kKOff, sb + kQOff, sc, lane); break;
      case 4: consume_tile<D, 4, G>(P, t, sb + kKOff, sb + kQOff, sc, lane); break;
      case 8: consume_tile<D, 8, G>(P, t, sb + kKOff, sb + kQOff, sc, lane); break;
      default: consume_tile<D, 16, G>(P, t, sb + kKOff, sb + kQOff, sc, lane); break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8u * st);
  }
}

#define FMHA_CAT2(a, b) a##b
#define FMHA_CAT(a, b) FMHA_CAT2(a, b)

VarlenFn FMHA_CAT(varlen_ring_kernel_d, FMHA_HEAD_DIM)(int g) {
  constexpr int D = FMHA_HEAD_DIM;
  switch (g) {
    case 1: return decode_varlen_ring_kernel<D, 1>;
    case 2: return decode_varlen_ring_kernel<D, 2>;
    case 4: return decode_varlen_ring_kernel<D, 4>;
    case 8: return decode_varlen_ring_kernel<D, 8>;
    default: return nullptr;
  }
}

}  // namespace fmha
