// decode_common.cuh -- shared device code of the sm_100a decode-attention
// kernels: launch parameters, PTX wrappers (mbarrier, cp.async.bulk, streaming
// loads/stores), and the per-warp tile computation both kernel families use.
//
// Work decomposition. A *unit* is one (batch row, kv head) pair: in the
// [B,H,S,D] layout its K slab (S x D bf16), its V slab, its G = Hq/Hkv query
// rows and its G output rows are each contiguous, and consecutive units are
// adjacent, so any run of units is one contiguous byte range per tensor.
// Unit u's K starts at u*S*D, its Q and O at u*G*D. (The reference gives each
// thread block 16 query heads of one batch row and indexes K/V by query head,
// fmha_vectorized_fma_kernel.hpp:113-135; here a warp owns whole kv heads so
// K and V are read once however many query heads share them.)
//
// A *tile* is the work of one warp: ROWS = max(SMAX, RPP) K/V rows, i.e. NU =
// ROWS/SMAX units. Each row is D bf16 = D/8 lanes x 16 bytes, so a warp covers
// RPP = 256/D rows per 16-byte vector access. Lane l owns columns
// (l % LPR)*8 .. +8 of rows p*RPP + l/LPR, p = 0..NP-1; every row a lane
// touches belongs to the same unit.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fmha {

constexpr unsigned kFullMask = 0xffffffffu;
constexpr int kBulkMaxThreads = 544;  // 1 producer warp + up to 16 consumer warps
constexpr int kBulkDefaultWarps = 16;  // consumer warps per CTA
constexpr int kLdgThreads = 256;   // 8 warps
constexpr int kHdrBytes = 1024;    // mbarriers + abort flag of the bulk kernel
constexpr int kMaxStages = 48;
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s
constexpr unsigned long long kStallTimeoutNs = 20000000ull;   // 20 ms (test hook)
// Test hook: the bulk producer issues no copies, so every consumer wait runs
// into its bound and the kernel must report FMHA_ERR_DEVICE_TIMEOUT and exit.
constexpr int kFlagStallProducer = 1;

// Device error word (first error wins). Low byte: fmha_status_t value;
// bits 8..15: the wait site that gave up.
enum : unsigned {
  kSiteProducerEmpty = 1,
  kSiteConsumerFull = 2,
  kSiteDrain = 3,
  kSiteConsumerIssued = 4
};

struct Params {
  const uint16_t* Q;
  const uint16_t* K;
  const uint16_t* V;
  uint16_t* O;
  unsigned int* err;  // device error word (a __device__ variable of the API unit)
  unsigned long long wait_timeout_ns;  // bound on every mbarrier wait
  int flags;                           // kFlag* bits
  int64_t units;     // batch * num_heads_kv
  int s_len;         // seqlen_kv, 1..SMAX
  float scale_log2;  // log2(e) / sqrt(D)
  // bulk family only
  int units_per_chunk;  // CU = tiles_per_chunk * NU
  int tiles_per_chunk;  // CT
  int stages;           // NS
  int chunks;           // ceil(units / CU)
  uint32_t stage_bytes; // bytes per ring stage (128-aligned)
  uint32_t v_off;       // V offset inside a stage (K at 0)
  uint32_t q_off;       // Q offset inside a stage
  uint32_t sc_off;      // per-warp score scratch offset in shared memory
  uint32_t ring_off;    // first stage offset in shared memory
  // fused KV-cache append (ldg family, APPEND instantiations only)
  const uint16_t* K_new;  // [units, D]: this step's K row of every unit
  const uint16_t* V_new;
  int64_t kv_ustride;     // elements between consecutive units' K slabs (cache stride)
  // ldg family: dynamic tail (see sched_join). sched_tag == 0: fully static.
  unsigned long long* sched;  // this launch's schedule word
  uint32_t sched_tag;         // 24-bit launch tag, unique among launches in flight
  int64_t sched_rounds;       // static rounds per warp before the dynamic tail
};

// ------------------------------------------------------------ launch overlap
// Programmatic dependent launch (the host launches with the
// programmatic-stream-serialization attribute): a kernel lets the next
// kernel of its stream start launching right away, so that kernel's CTAs take
// each SM as soon as this one's CTA leaves it instead of after the whole grid
// and a launch gap; the next kernel in turn waits in grid_dependency_wait()
// until this grid has completed and its writes are visible, before it touches
// any memory an earlier kernel may write (inputs and outputs alike). Without
// the attribute both are no-ops.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------ dynamic tail
// A persistent kernel splits its steps into a static part (warp w takes steps
// w, w+W, ... for `sched_rounds` rounds) and a tail that warps claim one step
// at a time, so SMs that stream faster than others take more of the tail and
// all finish together. Each launch uses one schedule slot in device memory
// (a few static slots; the host hands a slot and a tag to each launch):
//   word 0: tag (24 bits, bits 40..63) | users (12 bits, bits 28..39);
//   kSchedLanes claim counters, each on its own 128-byte line: warp w of a
//   CTA claims tail steps R*W + (w % kSchedLanes) + kSchedLanes*c from
//   counter w % kSchedLanes (one counter for every warp would queue ~1200
//   claimers on one address; measured ~4 ns per same-address atomic).
// A slot is all zeros whenever no launch uses it: the last user clears the
// counters and then the word, so no launch ever needs it cleared beforehand.
// Joining and leaving are one atomicAdd each on the word (a CAS loop there,
// with every CTA of the grid arriving at once, cost tens of microseconds):
//  * join: add one user. The old word tells the rest: all zero -> this CTA
//    is the first user and adds its launch's tag; its own tag -> joined; tag
//    0 with users -> the first user is installing, wait (bounded) for its tag;
//    a foreign tag -> leave again and run every step statically (w, w+W, ...).
//  * leave: remove one user. The CTA that removes the last one clears the
//    counters and then the tag (a CAS from "tag, no users" to 0, which fails
//    harmlessly if someone joined meanwhile; that CTA clears it later).
// Coverage: if any CTA joined, each counter runs until its steps pass the
// end, so every tail step is computed; CTAs that did not join compute their
// static share of the tail too (the same values, so writing them twice is
// benign; the same holds for a CTA that joins after the others have cleared
// the slot).
constexpr unsigned long long kSchedUser = 1ull << 28;
constexpr unsigned long long kSchedUserMask = 0xfffull << 28;
constexpr int kSchedLanes = 8;
constexpr int kSchedCtrStride = 16;                       // 64-bit words (128 bytes)
constexpr int kSchedSlotWords = kSchedCtrStride * (kSchedLanes + 1);

__device__ __forceinline__ unsigned long long* sched_counter(unsigned long long* slot, int j) {
  return slot + kSchedCtrStride * (1 + j);
}

__device__ __forceinline__ void sched_leave(unsigned long long* w) {
  const unsigned long long old = atomicAdd(w, 0ull - kSchedUser);
  if ((old & kSchedUserMask) != kSchedUser) return;  // others still use the slot
  for (int j = 0; j < kSchedLanes; ++j) atomicExch(sched_counter(w, j), 0ull);
  __threadfence();
  atomicCAS(w, old - kSchedUser, 0ull);
}

__device__ __forceinline__ bool sched_join(unsigned long long* w, uint32_t tag) {
  if (!w || tag == 0) return false;
  const unsigned long long mine = (unsigned long long)tag << 40;
  unsigned long long old = atomicAdd(w, kSchedUser);
  if (old == 0) {
    atomicAdd(w, mine);  // first user: the tag field was 0
    return true;
  }
  // Tag 0 with users: the first user has not added its tag yet.
  for (int it = 0; (old >> 40) == 0 && it < 100000; ++it) {
    __nanosleep(100);
    old = atomicAdd(w, 0ull);
  }
  if ((old >> 40) == tag) return true;
  sched_leave(w);  // foreign (or still untagged): do not use the slot
  return false;
}

template <int D, int SMAX, int G>
struct TileShape {
  static_assert(D == 128 || D == 256, "head_dim");
  static_assert(SMAX == 1 || SMAX == 2 || SMAX == 4 || SMAX == 8 || SMAX == 16, "SMAX");
  static constexpr int LPR = D / 8;                     // lanes per row
  static constexpr int RPP = 32 / LPR;                  // rows per 16B access
  static constexpr int ROWS = SMAX > RPP ? SMAX : RPP;  // rows per tile
  static constexpr int NU = ROWS / SMAX;                // units per tile
  static constexpr int NP = ROWS / RPP;                 // rows per lane
  static constexpr int LOG_LPR = LPR == 32 ? 5 : 4;
  static constexpr int LOG_NP = NP == 16 ? 4 : NP == 8 ? 3 : NP == 4 ? 2 : NP == 2 ? 1 : 0;
  static constexpr int HOLD_SHIFT = LOG_LPR - LOG_NP;   // see reduce_scatter
  static constexpr int SC = G * ROWS;                   // scores per tile
  static_assert(NP <= LPR, "reduce-scatter needs NP <= LPR");
};

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void report_device_error(unsigned* err, unsigned status,
                                                    unsigned site) {
  if (err) atomicCAS(err, 0u, status | (site << 8));
}

// Bounded wait on an mbarrier phase. Returns false if `abort_flag` was raised
// by another warp or if the wait ran past `timeout_ns` (then the device
// error word is set and the abort flag raised). Never traps.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          volatile int* abort_flag, unsigned* err,
                                          unsigned long long timeout_ns, unsigned site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (abort_flag && *abort_flag) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        report_device_error(err, 5u /* FMHA_ERR_DEVICE_TIMEOUT */, site);
        if (abort_flag) *abort_flag = 1;
        return false;
      }
    }
  }
}

// Bounded wait until the producer has published `*issued > k` (chunk k's
// copies and its `full` phase are armed). Same exit rules as mbar_wait.
__device__ __forceinline__ bool wait_issued(volatile int* issued, int k, volatile int* abort_flag,
                                            unsigned* err, unsigned long long timeout_ns) {
  if (*issued > k) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(64);
    if (*issued > k) return true;
    if ((it & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        report_device_error(err, 5u /* FMHA_ERR_DEVICE_TIMEOUT */, kSiteConsumerIssued);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> shared (no tensor map, no multicast), completing
// `bytes` of transaction count on the mbarrier. dst/src 16-byte aligned, bytes
// a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Streaming 16-byte global load: read-only path, no L1 allocation, 256-byte
// L2 fetch granularity (every byte of a K/V slab is used exactly once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void stg_stream(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ------------------------------------------------------------ arithmetic

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void unpack8(const uint4 w, float (&f)[8]) {
  f[0] = bf_lo(w.x); f[1] = bf_hi(w.x);
  f[2] = bf_lo(w.y); f[3] = bf_hi(w.y);
  f[4] = bf_lo(w.z); f[5] = bf_hi(w.z);
  f[6] = bf_lo(w.w); f[7] = bf_hi(w.w);
}

// acc[c] += p * vf[c] for c = 0..7 with packed fp32 FMAs (sm_100
// fma.rn.f32x2): each lane of the pair is an ordinary round-to-nearest fp32
// FMA, so the result equals the scalar fmaf chain bit for bit, in half the
// instructions.
__device__ __forceinline__ void fma8(float (&acc)[8], float p, const float (&vf)[8]) {
#pragma unroll
  for (int c = 0; c < 8; c += 2) {
    asm("{\n\t.reg .b64 a, b, s;\n\t"
        "mov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\tmov.b64 s, {%4, %4};\n\t"
        "fma.rn.f32x2 a, s, b, a;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "+f"(acc[c]), "+f"(acc[c + 1])
        : "f"(vf[c]), "f"(vf[c + 1]), "f"(p));
  }
}

__device__ __forceinline__ float dot8(const float (&q)[8], const uint4 k) {
  float a = q[0] * bf_lo(k.x);
  a = fmaf(q[1], bf_hi(k.x), a);
  a = fmaf(q[2], bf_lo(k.y), a);
  a = fmaf(q[3], bf_hi(k.y), a);
  a = fmaf(q[4], bf_lo(k.z), a);
  a = fmaf(q[5], bf_hi(k.z), a);
  a = fmaf(q[6], bf_lo(k.w), a);
  a = fmaf(q[7], bf_hi(k.w), a);
  return a;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint4 pack8_f16(const float (&a)[8]) {
  return make_uint4(pack_half2(a[0], a[1]), pack_half2(a[2], a[3]), pack_half2(a[4], a[5]),
                    pack_half2(a[6], a[7]));
}

// Sums N partial values across the LPR lanes of a row group, scattering the
// results: each halving step trades half of the remaining values with the
// partner lane (xor `o`), so N values need N-1 shuffles instead of
// N*log2(LPR). Afterwards lane cl holds the full sum of index
// cl >> HOLD_SHIFT (replicated over the low HOLD_SHIFT lane bits).
template <int N, int O, int M>
__device__ __forceinline__ void reduce_scatter_step(float (&v)[M], int cl) {
  if constexpr (O >= 1) {
    if constexpr (N > 1) {
      constexpr int H = N / 2;
      const bool upper = (cl & O) != 0;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float send = upper ? v[i] : v[i + H];
        const float keep = upper ? v[i + H] : v[i];
        v[i] = keep + __shfl_xor_sync(kFullMask, send, O);
      }
      reduce_scatter_step<H, O / 2>(v, cl);
    } else {
      v[0] += __shfl_xor_sync(kFullMask, v[0], O);
      reduce_scatter_step<1, O / 2>(v, cl);
    }
  }
}

template <int N, int LPR>
__device__ __forceinline__ float reduce_scatter(float (&v)[N], int cl) {
  reduce_scatter_step<N, LPR / 2>(v, cl);
  return v[0];
}

// One warp computes one tile: scores, softmax and P.V for NU units x G query
// heads. `loadK(p)` / `loadV(p)` return this lane's 16 bytes of row
// p*RPP + r0 (only called for valid rows). `q[g]` holds this lane's 8 query
// columns of head g (fp32). `sc` is this warp's G*ROWS float scratch in shared
// memory. On return acc[g][0..7] is this lane's 8 output columns of head g of
// its unit (after the cross-row-group sum when two row groups share a unit).
//
// Math per (unit, head): x_s = (q . k_s) * log2(e)/sqrt(D) for s < s_len
// (-inf beyond, the reference's max_seqlen 16 tile masking); p_s =
// 2^(x_s - max) / sum; o = sum_s p_s v_s. Non-finite inputs behave as in the
// reference (fmha_host.cpp:215-226): a NaN score or a head whose scores are
// all -inf gives NaN weights; only an empty row (s_len == 0) yields zeros.
// P stays fp32 (the reference's vectorized kernel keeps fp32 P, fmha_vectorized_fma_kernel.hpp:256,281-287;
// its host oracle rounds P to bf16, fmha_host.cpp:225, which the fp16-output
// tolerance of this library does not allow).
template <int D, int SMAX, int G, class LoadK, class LoadV>
__device__ __forceinline__ void attend_tile(const float (&q)[G][8], LoadK loadK, LoadV loadV,
                                            int s_len, int units_valid, float scale_log2,
                                            float* sc, int lane, float (&acc)[G][8]) {
  using T = TileShape<D, SMAX, G>;
  const int r0 = lane / T::LPR;
  const int cl = lane % T::LPR;
  auto row_ok = [&](int p) {
    const int r = p * T::RPP + r0;
    return (r % SMAX) < s_len && (r / SMAX) < units_valid;
  };

  __syncwarp();  // previous tile's readers of sc are done

  // 1. scores
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float v[T::NP];
#pragma unroll
    for (int p = 0; p < T::NP; ++p) v[p] = row_ok(p) ? dot8(q[g], loadK(p)) : 0.0f;
    const float s = reduce_scatter<T::NP, T::LPR>(v, cl);
    const int pi = cl >> T::HOLD_SHIFT;
    if ((cl & ((1 << T::HOLD_SHIFT) - 1)) == 0) {
      sc[g * T::ROWS + pi * T::RPP + r0] = row_ok(pi) ? s * scale_log2 : -INFINITY;
    }
  }
  __syncwarp();

  // 2. softmax over segments of SMAX consecutive scores (one unit, one head)
#pragma unroll
  for (int base = 0; base < T::SC; base += 32) {
    const int e = base + lane;
    const float x = e < T::SC ? sc[e] : -INFINITY;
    float m = x;
#pragma unroll
    for (int o = 1; o < SMAX; o <<= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, o));
    const float ex = s_len == 0 ? 0.0f : exp2f(x - m);
    float sum = ex;
#pragma unroll
    for (int o = 1; o < SMAX; o <<= 1) sum += __shfl_xor_sync(kFullMask, sum, o);
    if (e < T::SC) sc[e] = s_len == 0 ? 0.0f : ex / sum;
  }
  __syncwarp();

  // 3. P.V
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[g][c] = 0.0f;
#pragma unroll
  for (int p = 0; p < T::NP; ++p) {
    if (!row_ok(p)) continue;
    float vf[8];
    unpack8(loadV(p), vf);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pr = sc[g * T::ROWS + p * T::RPP + r0];
      fma8(acc[g], pr, vf);
    }
  }
  if constexpr (T::NU == 1 && T::RPP == 2) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[g][c] += __shfl_xor_sync(kFullMask, acc[g][c], 16);
  }
}

// ----------------------------------------------------------------------
// 16-row tiles (bulk family). A tile is always 16 K/V rows = NU = 16/SMAX
// units, whatever seqlen_kv is, so the score reduction, the softmax and their
// warp synchronisations are paid once per 16 rows instead of once per unit.
// Lane l (row group r0 = l / LPR, column block cl = l % LPR) owns rows
// r0*NP + p, p = 0..NP-1 (D=256: all 16 rows; D=128: half of them). Its rows
// fall into LU "slots" of SPL consecutive rows of one unit; only when a unit
// is longer than a lane's rows (D=128, SMAX=16) do the two row groups share a
// unit and sum their P.V partials with one xor-16 shuffle.
template <int D, int SMAX, int G>
struct Tile16 {
  static_assert(D == 128 || D == 256, "head_dim");
  static constexpr int LPR = D / 8;
  static constexpr int RPP = 32 / LPR;
  static constexpr int ROWS = 16;
  static constexpr int NP = ROWS / RPP;                 // rows per lane
  static constexpr int NU = ROWS / SMAX;                // units per tile
  static constexpr int SPL = NP < SMAX ? NP : SMAX;     // rows per slot
  static constexpr int LU = NP / SPL;                   // slots per lane
  static constexpr bool CROSS = SMAX > NP;              // unit spans both row groups
  static constexpr int GB = G < 32 / NP ? G : 32 / NP;  // query heads per score pass
  static constexpr int LOG_LPR = LPR == 32 ? 5 : 4;
  static constexpr int LOG_NP = NP == 16 ? 4 : 3;
  static constexpr int HOLD_SHIFT = LOG_LPR - LOG_NP;
  static constexpr int SC = G * ROWS;
  static_assert(G % GB == 0, "GB");
};

// q . k over 8 bf16 pairs with mixed-precision FMAs (bf16 operands, fp32
// accumulator, sm_100): the bf16 x bf16 product is exact in fp32, so this
// rounds exactly like unpacking both to fp32 and chaining fmaf in the same
// order, without the unpack instructions.
__device__ __forceinline__ float dot8_bf16(const uint4 q, const uint4 k) {
  float a = 0.0f;
  asm("{\n\t.reg .b16 q0, q1, k0, k1;\n\t"
      "mov.b32 {q0, q1}, %1;\n\tmov.b32 {k0, k1}, %5;\n\t"
      "fma.rn.f32.bf16 %0, q0, k0, %0;\n\tfma.rn.f32.bf16 %0, q1, k1, %0;\n\t"
      "mov.b32 {q0, q1}, %2;\n\tmov.b32 {k0, k1}, %6;\n\t"
      "fma.rn.f32.bf16 %0, q0, k0, %0;\n\tfma.rn.f32.bf16 %0, q1, k1, %0;\n\t"
      "mov.b32 {q0, q1}, %3;\n\tmov.b32 {k0, k1}, %7;\n\t"
      "fma.rn.f32.bf16 %0, q0, k0, %0;\n\tfma.rn.f32.bf16 %0, q1, k1, %0;\n\t"
      "mov.b32 {q0, q1}, %4;\n\tmov.b32 {k0, k1}, %8;\n\t"
      "fma.rn.f32.bf16 %0, q0, k0, %0;\n\tfma.rn.f32.bf16 %0, q1, k1, %0;\n\t}"
      : "+f"(a)
      : "r"(q.x), "r"(q.y), "r"(q.z), "r"(q.w), "r"(k.x), "r"(k.y), "r"(k.z), "r"(k.w));
  return a;
}

__device__ __forceinline__ float dot8f(const float (&q)[8], const float (&k)[8]) {
  float a = q[0] * k[0];
#pragma unroll
  for (int c = 1; c < 8; ++c) a = fmaf(q[c], k[c], a);
  return a;
}

// One warp, one 16-row tile. loadK(p)/loadV(p): this lane's 16 bytes of its
// row p (local index 0..NP-1); loadQ(us, u, g): its 16 bytes of query head g
// of tile unit u, the unit of the lane's slot us; store(u, acc): called once per (slot, lane) with the lane's 8
// output columns of every head of unit u -- the caller stores when
// u < units_valid and writer() holds. Same math as attend_tile.
template <int D, int SMAX, int G, class LoadV, class Store>
__device__ __forceinline__ void tile16_softmax_pv(LoadV loadV, Store store, int s_len,
                                                  int units_valid, float* sc, int lane);

template <int D, int SMAX, int G, class LoadK, class LoadV, class LoadQ, class Store>
__device__ __forceinline__ void attend_tile16(LoadK loadK, LoadV loadV, LoadQ loadQ, Store store,
                                              int s_len, int units_valid, float scale_log2,
                                              float* sc, int lane) {
  using T = Tile16<D, SMAX, G>;
  const int r0 = lane / T::LPR;
  const int cl = lane % T::LPR;
  auto row_ok = [&](int p) {
    const int r = r0 * T::NP + p;
    return (r % SMAX) < s_len && (r / SMAX) < units_valid;
  };
  auto slot_unit = [&](int us) { return (r0 * T::NP + us * T::SPL) / SMAX; };

  __syncwarp();
#pragma unroll
  for (int gb = 0; gb < G; gb += T::GB) {
    float v[T::GB][T::NP];
#pragma unroll
    for (int us = 0; us < T::LU; ++us) {
      const int u = slot_unit(us);
      uint4 q[T::GB];
#pragma unroll
      for (int g = 0; g < T::GB; ++g)
        q[g] = u < units_valid ? loadQ(us, u, gb + g) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < T::SPL; ++i) {
        const int p = us * T::SPL + i;
        if (row_ok(p)) {
          const uint4 k = loadK(p);
#pragma unroll
          for (int g = 0; g < T::GB; ++g) v[g][p] = dot8_bf16(q[g], k);
        } else {
#pragma unroll
          for (int g = 0; g < T::GB; ++g) v[g][p] = 0.0f;
        }
      }
    }
#pragma unroll
    for (int g = 0; g < T::GB; ++g) {
      const float s = reduce_scatter<T::NP, T::LPR>(v[g], cl);
      const int pi = cl >> T::HOLD_SHIFT;
      if ((cl & ((1 << T::HOLD_SHIFT) - 1)) == 0)
        sc[(gb + g) * T::ROWS + r0 * T::NP + pi] = row_ok(pi) ? s * scale_log2 : -INFINITY;
    }
  }
  tile16_softmax_pv<D, SMAX, G>(loadV, store, s_len, units_valid, sc, lane);
}

// Softmax over the scores in `sc` (sc[g*16 + r], already scaled by
// log2(e)*scale, -inf for masked rows) and P.V of one 16-row tile on the CUDA
// cores; the second half of attend_tile16, shared with attend_tile16_mq.
template <int D, int SMAX, int G, class LoadV, class Store>
__device__ __forceinline__ void tile16_softmax_pv(LoadV loadV, Store store, int s_len,
                                                  int units_valid, float* sc, int lane) {
  using T = Tile16<D, SMAX, G>;
  const int r0 = lane / T::LPR;
  auto row_ok = [&](int p) {
    const int r = r0 * T::NP + p;
    return (r % SMAX) < s_len && (r / SMAX) < units_valid;
  };
  auto slot_unit = [&](int us) { return (r0 * T::NP + us * T::SPL) / SMAX; };
  __syncwarp();

#pragma unroll
  for (int base = 0; base < T::SC; base += 32) {
    const int e = base + lane;
    const float x = e < T::SC ? sc[e] : -INFINITY;
    float m = x;
#pragma unroll
    for (int o = 1; o < SMAX; o <<= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, o));
    const float ex = s_len == 0 ? 0.0f : exp2f(x - m);
    float sum = ex;
#pragma unroll
    for (int o = 1; o < SMAX; o <<= 1) sum += __shfl_xor_sync(kFullMask, sum, o);
    if (e < T::SC) sc[e] = s_len == 0 ? 0.0f : ex / sum;
  }
  __syncwarp();

#pragma unroll
  for (int us = 0; us < T::LU; ++us) {
    float acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[g][c] = 0.0f;
#pragma unroll
    for (int i = 0; i < T::SPL; ++i) {
      const int p = us * T::SPL + i;
      if (!row_ok(p)) continue;
      float vf[8];
      unpack8(loadV(p), vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pr = sc[g * T::ROWS + r0 * T::NP + p];
        fma8(acc[g], pr, vf);
      }
    }
    if constexpr (T::CROSS) {
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[g][c] += __shfl_xor_sync(kFullMask, acc[g][c], 16);
    }
    if (!T::CROSS || r0 == 0) store(slot_unit(us), acc);
  }
}

__device__ __forceinline__ void mma_16816_rows(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// attend_tile16 with the scores on the tensor cores (mma.sync m16n8k16, bf16
// operands, fp32 accumulation; the products are exact): M = the tile's 16 K
// rows, N = its NU*G query rows (one or two n-tiles), K = D. Lane (g, t)
// loads 16 contiguous bytes of K rows g and g+8 and of query row g (+8) at
// column 32j + 8t; the dot product's order is free, so those 8 columns are
// the lane's k slots of two k-steps in A and B alike. Of C only the entries
// C[r][(unit(r), h)] are kept: each is a separate dot product, so rows and
// query rows of other units (or garbage past the tile) never mix into them.
// krow(r): shared address of tile row r (row base, no column offset);
// qrow(u, h): shared address of query head h of tile unit u. Softmax and P.V
// as in attend_tile16.
template <int D, int SMAX, int G>
struct Tile16Mq {
  static constexpr int NU = 16 / SMAX;
  static constexpr int NQ = NU * G;
  static constexpr int NT = (NQ + 7) / 8;
  static constexpr bool OK = NQ <= 16;  // at most two n-tiles
};

template <int D, int SMAX, int G, class KRow, class QRow, class LoadV, class Store>
__device__ __forceinline__ void attend_tile16_mq(KRow krow, QRow qrow, LoadV loadV, Store store,
                                                 int s_len, int units_valid, float scale_log2,
                                                 float* sc, int lane) {
  using M = Tile16Mq<D, SMAX, G>;
  static_assert(M::OK, "at most 16 query rows per tile");
  const int g = lane >> 2, t = lane & 3;
  const uint4 z = make_uint4(0, 0, 0, 0);
  const int rA = g, rB = g + 8;
  const bool okA = (rA % SMAX) < s_len && (rA / SMAX) < units_valid;
  const bool okB = (rB % SMAX) < s_len && (rB / SMAX) < units_valid;
  const uint32_t col = (uint32_t)t * 16;
  const uint32_t kA = krow(rA) + col, kB = krow(rB) + col;
  uint32_t qa[M::NT];
  bool qok[M::NT];
#pragma unroll
  for (int nt = 0; nt < M::NT; ++nt) {
    const int n = g + 8 * nt;
    qok[nt] = n < M::NQ && n / G < units_valid;
    qa[nt] = qok[nt] ? qrow(n / G, n % G) + col : 0u;
  }
  float c[M::NT][4];
#pragma unroll
  for (int nt = 0; nt < M::NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) c[nt][i] = 0.0f;
  __syncwarp();
#pragma unroll
  for (int j = 0; j < D / 32; ++j) {
    const uint4 a = okA ? lds128(kA + 64 * j) : z;
    const uint4 b = okB ? lds128(kB + 64 * j) : z;
#pragma unroll
    for (int nt = 0; nt < M::NT; ++nt) {
      const uint4 q = qok[nt] ? lds128(qa[nt] + 64 * j) : z;
      mma_16816_rows(c[nt], a.x, b.x, a.y, b.y, q.x, q.y);
      mma_16816_rows(c[nt], a.z, b.z, a.w, b.w, q.z, q.w);
    }
  }
  // c[nt][0..1]: row g, query rows n = 8nt + 2t + {0,1}; c[nt][2..3]: row g+8.
#pragma unroll
  for (int nt = 0; nt < M::NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int n = 8 * nt + 2 * t + (e & 1);
      const int r = e < 2 ? rA : rB;
      if (n < M::NQ && n / G == r / SMAX)
        sc[(n % G) * 16 + r] = (e < 2 ? okA : okB) ? c[nt][e] * scale_log2 : -INFINITY;
    }
  tile16_softmax_pv<D, SMAX, G>(loadV, store, s_len, units_valid, sc, lane);
}

// ----------------------------------------------------------------------
// Tensor-core tile for one unit with several query heads (G = 4 or 8) and up
// to 16 K/V rows, on mma.sync.m16n8k16 (bf16 operands, fp32 accumulation).
// With G heads per kv head the fp32 CUDA-core path spends ~G x 16 x 16 FMAs per
// lane per tile; here the G query rows are the MMA's M rows (rows >= G are
// zero).
//  * S = Q K^T: lane (g = lane/4, t = lane%4) loads 16 contiguous bytes of Q
//    row g and of K rows g and g+8 at column 32j + 8t. The dot product's d
//    order is free, so those 8 columns become this lane's k slots of two
//    k-steps (the same rule in A and B keeps every product paired).
//  * softmax on the accumulators (row g; scores s = 2t, 2t+1, 8+2t, 9+2t),
//    reduced over the 4 lanes of a row; rows >= s_len are -inf.
//  * O = P V: the score accumulators are already in A-fragment order. P is
//    split into bf16 hi + lo (two MMAs) so it keeps ~16 more bits than bf16
//    alone -- P never drops to bf16 precision. V rows s = 2t, 2t+1, 2t+8,
//    2t+9 are loaded 16 bytes at a time at column 8g + 64m and repacked into
//    B fragments; output column n of n-tile (m, i) is then 8n + 64m + i, so
//    each lane ends with 16 contiguous outputs per m of its head.
// Rows past s_len are zeroed in V (garbage there must not meet P = 0).
// Query heads per kv head from which the bulk kernel uses the tensor-core tile
// (for units of 5..16 rows).
#ifndef FMHA_MMA_MIN_HEADS
#define FMHA_MMA_MIN_HEADS 4
#endif
constexpr int kMmaMinHeads = FMHA_MMA_MIN_HEADS;

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t half16(const uint4 v, int i) {  // element i of 8
  const uint32_t w = i < 2 ? v.x : i < 4 ? v.y : i < 6 ? v.z : v.w;
  return (i & 1) ? (w >> 16) : (w & 0xffffu);
}

// HALF: the unit has at most 8 rows (SMAX = 8), so K rows 8-15 -- the next
// unit's, masked anyway -- are neither loaded nor multiplied.
template <int D, int G, bool HALF = false>
__device__ __forceinline__ void attend_unit_mma(uint32_t kbase, uint32_t vbase, uint32_t qbase,
                                                int s_len, float scale_log2, uint16_t* O,
                                                int lane) {
  static_assert(G <= 8, "query heads fill at most 8 of the 16 MMA rows");
  const int g = lane >> 2, t = lane & 3;
  const uint4 z = make_uint4(0, 0, 0, 0);
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < D / 32; ++j) {
    const uint32_t col = (uint32_t)(32 * j + 8 * t) * 2;
    const uint4 qa = g < G ? lds128(qbase + (uint32_t)g * (D * 2) + col) : z;
    const uint4 k0 = lds128(kbase + (uint32_t)g * (D * 2) + col);
    mma_16816(c0, qa.x, qa.y, k0.x, k0.y);
    mma_16816(c0, qa.z, qa.w, k0.z, k0.w);
    if constexpr (!HALF) {
      const uint4 k1 = lds128(kbase + (uint32_t)(g + 8) * (D * 2) + col);
      mma_16816(c1, qa.x, qa.y, k1.x, k1.y);
      mma_16816(c1, qa.z, qa.w, k1.z, k1.w);
    }
  }
  // Scores of row g: s = 2t, 2t+1 (c0), 8+2t, 9+2t (c1).
  float x[4] = {c0[0], c0[1], c1[0], c1[1]};
  const int sidx[4] = {2 * t, 2 * t + 1, 8 + 2 * t, 9 + 2 * t};
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = sidx[i] < s_len ? x[i] * scale_log2 : -INFINITY;
  float m = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
  m = fmaxf(m, __shfl_xor_sync(kFullMask, m, 1));
  m = fmaxf(m, __shfl_xor_sync(kFullMask, m, 2));
  float e[4], sum = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    e[i] = s_len == 0 ? 0.0f : exp2f(x[i] - m);
    sum += e[i];
  }
  sum += __shfl_xor_sync(kFullMask, sum, 1);
  sum += __shfl_xor_sync(kFullMask, sum, 2);
  float p[4], lo[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = s_len == 0 ? 0.0f : e[i] / sum;
  const uint32_t ah0 = pack_bf16x2(p[0], p[1]), ah2 = pack_bf16x2(p[2], p[3]);
  lo[0] = p[0] - __uint_as_float(ah0 << 16);
  lo[1] = p[1] - __uint_as_float(ah0 & 0xffff0000u);
  lo[2] = p[2] - __uint_as_float(ah2 << 16);
  lo[3] = p[3] - __uint_as_float(ah2 & 0xffff0000u);
  const uint32_t al0 = pack_bf16x2(lo[0], lo[1]), al2 = pack_bf16x2(lo[2], lo[3]);

#pragma unroll
  for (int mm = 0; mm < D / 64; ++mm) {
    const uint32_t col = (uint32_t)(8 * g + 64 * mm) * 2;
    const uint4 v0 = 2 * t < s_len ? lds128(vbase + (uint32_t)(2 * t) * (D * 2) + col) : z;
    const uint4 v1 = 2 * t + 1 < s_len ? lds128(vbase + (uint32_t)(2 * t + 1) * (D * 2) + col) : z;
    const uint4 v2 = 2 * t + 8 < s_len ? lds128(vbase + (uint32_t)(2 * t + 8) * (D * 2) + col) : z;
    const uint4 v3 = 2 * t + 9 < s_len ? lds128(vbase + (uint32_t)(2 * t + 9) * (D * 2) + col) : z;
    float o0[8], o1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b0 = half16(v0, i) | (half16(v1, i) << 16);
      const uint32_t b1 = half16(v2, i) | (half16(v3, i) << 16);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      mma_16816(acc, ah0, ah2, b0, b1);
      mma_16816(acc, al0, al2, b0, b1);
      o0[i] = acc[0];  // output column 8*(2t) + 64mm + i
      o1[i] = acc[1];  // output column 8*(2t+1) + 64mm + i
    }
    if (g < G) {
      uint16_t* orow = O + (int64_t)g * D + 16 * t + 64 * mm;
      stg_stream(orow, pack8_f16(o0));
      stg_stream(orow + 8, pack8_f16(o1));
    }
  }
}

// Which lanes store the output, and for which unit of the tile.
template <int D, int SMAX, int G>
struct OutputMap {
  using T = TileShape<D, SMAX, G>;
  __device__ __forceinline__ static int unit(int lane) { return (lane / T::LPR) / SMAX; }
  __device__ __forceinline__ static bool writer(int lane) {
    return !(T::NU == 1 && T::RPP == 2) || (lane / T::LPR) == 0;
  }
};

// Tiles per warp step of the ldg family: enough for 16 K rows and 16 V rows
// per lane in flight, fewer when many query heads share a kv head (their Q
// rows are loaded too).
template <int D, int SMAX, int G>
struct LdgTpi {
  using T = TileShape<D, SMAX, G>;
  static constexpr int by_rows = 16 / T::NP;
  static constexpr int by_q = G >= 8 ? 1 : 8 / G;
  static constexpr int value = by_rows < by_q ? by_rows : by_q;
};

// Kernel entry points (defined in decode_bulk.cu / decode_ldg.cu).
template <int D, int SMAX, int G>
__global__ void decode_bulk_kernel(const Params P);
template <int D, int SMAX, int G, int TPI, bool APPEND>
__global__ void decode_ldg_kernel(const Params P);

using KernelFn = void (*)(const Params);

// Packed varlen layout (K/V [sum S_b, Hkv, D] + cu_seqlens_kv).
struct VarlenParams {
  const uint16_t* Q;
  const uint16_t* K;
  const uint16_t* V;
  uint16_t* O;
  const int32_t* cu_seqlens;  // [batch + 1], device
  unsigned int* err;
  int64_t batch;
  int num_heads_kv;
  int max_seqlen;     // rows longer than this are rejected (device error)
  int tiles_per_row;  // 16-row tiles of a row of length max_seqlen (ldg kernel)
  float scale_log2;   // log2(e) * softmax scale
  // chunk kernel only
  unsigned long long wait_timeout_ns;
  uint32_t stage_bytes;  // ring size in bytes (a multiple of the row size)
  uint32_t sc_off;       // per-consumer-warp score scratch
  uint32_t ring_off;     // first ring byte
  uint32_t chunk_max;    // byte limit of one chunk (<= ring/2)
};
using VarlenFn = void (*)(const VarlenParams);
VarlenFn varlen_kernel_d128(int g);
VarlenFn varlen_kernel_d256(int g);
VarlenFn varlen_chunk_kernel_d128(int g);
VarlenFn varlen_chunk_kernel_d256(int g);
constexpr int kVarlenSlots = 32;           // chunk descriptors in flight per CTA
constexpr uint32_t kVarlenChunkHdr = 8192;  // barriers, counters, descriptors

// Per-head_dim lookups of the instantiation for (SMAX, G); nullptr if absent.
KernelFn bulk_kernel_d128(int smax, int g);
KernelFn bulk_kernel_d256(int smax, int g);
KernelFn ldg_kernel_d128(int smax, int g);
KernelFn ldg_kernel_d256(int smax, int g);
KernelFn ldg_append_kernel_d128(int smax, int g);
KernelFn ldg_append_kernel_d256(int smax, int g);

}  // namespace fmha
