// fmha_api.cu -- the extern "C" boundary of libfmha_b200.so (include/fmha.h):
// argument validation, per-device launch planning and dispatch to the
// head_dim/seqlen/group-specialised kernels, the device error word, and the
// seeded input generator used by the benchmark/validation harness.
//
// Reference interface replaced: launch_fmha_mfma_4x4x4
// (fmha_mfma_4x4x4_kernel.hpp:370-389), which launched with a caller-chosen
// grid, did no validation and silently treated any head_dim != 128 as 256.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <random>
#include <set>
#include <utility>

#include "../../include/fmha.h"
#include "decode_common.cuh"

namespace fmha {

__device__ unsigned int g_fmha_device_error;

// Schedule words of the ldg family's dynamic tail (decode_common.cuh,
// sched_join): one per slot, each 0 whenever no launch is using it. Launches
// take slots round-robin, so launches in flight at the same time normally use
// different words; one that finds its word held by another launch runs
// statically.
constexpr int kSchedSlots = 16;
__device__ __align__(128) unsigned long long g_fmha_sched[kSchedSlots * kSchedSlotWords];

namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int smem_optin = 0;
  unsigned int* err = nullptr;  // device address of g_fmha_device_error
  unsigned long long* sched = nullptr;  // device address of g_fmha_sched
};

std::mutex g_mu;
std::atomic<int> g_test_stall{0};
DeviceInfo g_dev[kMaxDevices];
std::atomic<uint64_t> g_launch_seq[kMaxDevices];
std::set<std::pair<const void*, int>> g_smem_set;      // (kernel, device) with smem attr set
struct OccEntry {
  const void* fn;
  int dev;
  int blocks;
};
OccEntry g_occ[512];
int g_occ_n = 0;

fmha_status_t device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return FMHA_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return FMHA_ERR_CUDA;
    if (cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
        cudaSuccess)
      return FMHA_ERR_CUDA;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fmha_device_error) != cudaSuccess) return FMHA_ERR_CUDA;
    d.err = static_cast<unsigned int*>(p);
    if (cudaGetSymbolAddress(&p, g_fmha_sched) != cudaSuccess) return FMHA_ERR_CUDA;
    d.sched = static_cast<unsigned long long*>(p);
    d.ready = true;
  }
  *out = d;
  return FMHA_OK;
}

// Sets the kernel's dynamic shared-memory limit once per (kernel, device).
fmha_status_t ensure_smem(const void* fn, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(fn, dev);
  if (g_smem_set.count(key)) return FMHA_OK;
  // The limit is set to the device maximum, so one call covers every plan.
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return FMHA_ERR_CUDA;
  g_smem_set.insert(key);
  return FMHA_OK;
}

fmha_status_t blocks_per_sm(const void* fn, int threads, int* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < g_occ_n; ++i)
    if (g_occ[i].fn == fn && g_occ[i].dev == dev) {
      *out = g_occ[i].blocks;
      return FMHA_OK;
    }
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, fn, threads, 0) != cudaSuccess)
    return FMHA_ERR_CUDA;
  if (b < 1) b = 1;
  if (g_occ_n < 512) g_occ[g_occ_n++] = {fn, dev, b};
  *out = b;
  return FMHA_OK;
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

int smax_for(int s) {
  int m = 1;
  while (m < s) m <<= 1;
  return m;
}

int rows_per_access(int d) { return 256 / d; }

// Per-shape default: kernel family and bulk consumer-warp count, from B200
// sweeps (bench.py --sweep, batch 30720; last re-swept after the packed-FMA
// P.V and the ldg kernel's dynamic tail). The ldg family wins where one unit
// already fills a 16-row tile with 512-byte rows (D=256, S=16, one query head
// per kv head), for seqlen 1 with one or two query heads per kv head, and for
// D=256, S<=2 with two; elsewhere the bulk ring wins, with ~10 consumer warps
// for 9-16 row units (leaving ring stages for copies in flight), 16 for
// shorter ones and for D=256 S 5-8. With 4 or 8 query heads per kv head the
// choice flips for D=256 short rows (ldg, except 4 heads at S=1 or S 3-4:
// bulk with 8 warps) and D=128 long rows (16 warps). FMHA_VARIANT (1 bulk,
// 2 ldg) and FMHA_BULK_WARPS override the table.
struct Choice {
  int variant;
  int warps;
};

Choice auto_choice(int d, int smax, int g) {
  static const int forced = env_int("FMHA_VARIANT", 0);
  Choice c{FMHA_VARIANT_BULK, 16};
  if (g >= 4) {
    // 4 or 8 query heads per kv head (S >= 5 runs the bulk kernel's
    // tensor-core tile).
    if (d == 128) c = smax == 1 ? Choice{FMHA_VARIANT_LDG, 0} : Choice{FMHA_VARIANT_BULK, 16};
    else if (smax >= 8) c = {FMHA_VARIANT_BULK, 8};
    else if (g == 4 && (smax == 1 || smax == 4)) c = {FMHA_VARIANT_BULK, 8};
    else c = {FMHA_VARIANT_LDG, 0};
  } else if (d == 256 && smax == 16 && g == 1) c = {FMHA_VARIANT_LDG, 0};
  else if (smax == 1) c = {FMHA_VARIANT_LDG, 0};
  else if (d == 256 && smax == 2 && g == 2) c = {FMHA_VARIANT_LDG, 0};
  else if (d == 256 && smax == 8) c = {FMHA_VARIANT_BULK, 16};
  else if (smax >= 8) c = {FMHA_VARIANT_BULK, 10};
  if (forced == FMHA_VARIANT_BULK || forced == FMHA_VARIANT_LDG) c.variant = forced;
  if (c.warps == 0) c.warps = 10;
  return c;
}

fmha_status_t check_args(const void* Q, const void* K, const void* V, void* O, int batch,
                         int hq, int hkv, int s, int d) {
  if (batch < 0 || hq <= 0 || hkv <= 0 || s <= 0 || d <= 0) return FMHA_ERR_INVALID_ARG;
  if (hq % hkv != 0) return FMHA_ERR_INVALID_ARG;
  if (batch > 0 && (!Q || !K || !V || !O)) return FMHA_ERR_INVALID_ARG;
  if (d != 128 && d != 256) return FMHA_ERR_UNSUPPORTED;
  if (s > 16) return FMHA_ERR_UNSUPPORTED;
  const int g = hq / hkv;
  if (g != 1 && g != 2 && g != 4 && g != 8) return FMHA_ERR_UNSUPPORTED;
  const uintptr_t mis = reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
                        reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(O);
  if (mis & 15u) return FMHA_ERR_MISALIGNED;
  // Offsets are 64-bit throughout; keep the unit count within int32 chunking.
  if ((int64_t)batch * hkv > (int64_t)1 << 30) return FMHA_ERR_UNSUPPORTED;
  return FMHA_OK;
}

// Launches a persistent kernel with programmatic stream serialization, so it
// may begin launching while the previous kernel of the stream finishes (the
// kernel waits in grid_dependency_wait before touching shared data).
// FMHA_NO_PDL=1 launches it the plain way.
template <class Prm>
cudaError_t launch_overlapped(void (*fn)(const Prm), unsigned grid, unsigned block, size_t smem,
                              cudaStream_t stream, const Prm& P) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = env_int("FMHA_NO_PDL", 0) ? 0 : 1;
  return cudaLaunchKernelEx(&cfg, fn, P);
}

// Share of the steps dealt out statically; the rest is the dynamic tail.
constexpr int kStaticPercent = 90;

// Picks a schedule slot and a fresh tag for an eager launch of `ctas` CTAs;
// false (run statically) while the stream is being captured into a CUDA
// graph (a captured launch would replay one tag, and two replays must never
// share a slot's counters), for grids beyond the 12-bit user count, or when
// FMHA_STATIC_SCHEDULE is set.
bool take_slot(const DeviceInfo& dev, int64_t ctas, cudaStream_t stream,
               unsigned long long** slot, uint32_t* tag) {
  if (env_int("FMHA_STATIC_SCHEDULE", 0)) return false;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cap != cudaStreamCaptureStatusNone) return false;
  if (ctas >= 4096) return false;  // 12-bit user count (one user per CTA)
  int dv = 0;
  if (cudaGetDevice(&dv) != cudaSuccess) return false;
  // FMHA_SCHED_SLOTS (1..16) narrows the slot pool; tests use it to make
  // concurrent launches contend for one word.
  int nslots = env_int("FMHA_SCHED_SLOTS", kSchedSlots);
  if (nslots < 1 || nslots > kSchedSlots) nslots = kSchedSlots;
  const uint64_t seq = g_launch_seq[dv].fetch_add(1);
  *slot = dev.sched + (seq % (uint64_t)nslots) * kSchedSlotWords;
  *tag = (uint32_t)(seq % 0xffffffu) + 1u;
  return true;
}

// Fills P's schedule fields for a persistent launch of `ctas` CTAs whose
// `workers` (warps) share `steps` steps: kStaticPercent of the steps static,
// the rest claimed, or all static when take_slot declines.
void plan_schedule(Params& P, const DeviceInfo& dev, int64_t steps, int64_t workers,
                   int64_t ctas, cudaStream_t stream) {
  P.sched = nullptr;
  P.sched_tag = 0;
  P.sched_rounds = 0;
  if (!take_slot(dev, ctas, stream, &P.sched, &P.sched_tag)) return;
  int pct = env_int("FMHA_STATIC_PERCENT", kStaticPercent);  // tuning knob, 0..100
  if (pct < 0 || pct > 100) pct = kStaticPercent;
  P.sched_rounds = steps * pct / 100 / workers;
}

fmha_status_t launch_bulk(Params P, int d, int smax, int g, int warps, const DeviceInfo& dev,
                          cudaStream_t stream) {
  KernelFn fn = d == 128 ? bulk_kernel_d128(smax, g) : bulk_kernel_d256(smax, g);
  if (!fn) return FMHA_ERR_UNSUPPORTED;
  const int rows = 16;  // Tile16: every tile is 16 K/V rows
  const int nu = rows / smax;
  const int s = P.s_len;
  int ncw = env_int("FMHA_BULK_WARPS", warps > 0 ? warps : kBulkDefaultWarps);
  if (ncw < 1) ncw = 1;
  if (ncw > kBulkMaxThreads / 32 - 1) ncw = kBulkMaxThreads / 32 - 1;
  const int64_t tile_bytes = (int64_t)nu * (2LL * s * d * 2 + (int64_t)g * d * 2);
  const int target = env_int("FMHA_STAGE_BYTES", 32768);
  int ct = (int)(target / tile_bytes);
  if (ct < 1) ct = 1;
  const int cu = ct * nu;
  const uint32_t kb = (uint32_t)cu * s * d * 2;
  const uint32_t qb = (uint32_t)cu * g * d * 2;
  const uint32_t stage = (2 * kb + qb + 127u) & ~127u;
  const uint32_t sc_off = kHdrBytes;
  const uint32_t sc_bytes = (uint32_t)ncw * g * rows * 4;
  const uint32_t ring_off = (sc_off + sc_bytes + 1023u) & ~1023u;
  // One CTA per SM by default (the whole shared memory); FMHA_BULK_CTAS_PER_SM
  // splits the SM's 228 KiB (1 KiB reserved per CTA) between several rings.
  const int ctas_per_sm = env_int("FMHA_BULK_CTAS_PER_SM", 1) > 1 ? env_int("FMHA_BULK_CTAS_PER_SM", 1) : 1;
  int budget = dev.smem_optin;
  if (ctas_per_sm > 1 && 233472 / ctas_per_sm - 1024 < budget) budget = 233472 / ctas_per_sm - 1024;
  int ns = (int)((budget - (int64_t)ring_off) / stage);
  const int ns_cap = env_int("FMHA_STAGES", kMaxStages);
  if (ns > ns_cap) ns = ns_cap;
  if (ns > kMaxStages) ns = kMaxStages;
  if (ns < 2) return FMHA_ERR_UNSUPPORTED;
  const uint32_t smem = ring_off + (uint32_t)ns * stage;
  P.units_per_chunk = cu;
  P.tiles_per_chunk = ct;
  P.stages = ns;
  P.chunks = (int)((P.units + cu - 1) / cu);
  P.stage_bytes = stage;
  P.v_off = kb;
  P.q_off = 2 * kb;
  P.sc_off = sc_off;
  P.ring_off = ring_off;
  fmha_status_t st = ensure_smem(reinterpret_cast<const void*>(fn), dev.smem_optin);
  if (st != FMHA_OK) return st;
  int grid = dev.sms * ctas_per_sm;
  if (grid > P.chunks) grid = P.chunks;
  if (launch_overlapped(fn, (unsigned)grid, 32u * (1 + ncw), smem, stream, P) != cudaSuccess) {
    cudaGetLastError();
    return FMHA_ERR_CUDA;
  }
  return FMHA_OK;
}

template <int D>
int ldg_tpi(int smax, int g) {
#define FMHA_T(SM)                                  \
  switch (g) {                                      \
    case 1: return LdgTpi<D, SM, 1>::value;         \
    case 2: return LdgTpi<D, SM, 2>::value;         \
    case 4: return LdgTpi<D, SM, 4>::value;         \
    default: return LdgTpi<D, SM, 8>::value;        \
  }
  switch (smax) {
    case 1: FMHA_T(1)
    case 2: FMHA_T(2)
    case 4: FMHA_T(4)
    case 8: FMHA_T(8)
    default: FMHA_T(16)
  }
#undef FMHA_T
}

fmha_status_t launch_ldg(Params P, int d, int smax, int g, const DeviceInfo& dev,
                         cudaStream_t stream, bool append = false) {
  KernelFn fn = append ? (d == 128 ? ldg_append_kernel_d128(smax, g)
                                   : ldg_append_kernel_d256(smax, g))
                       : (d == 128 ? ldg_kernel_d128(smax, g) : ldg_kernel_d256(smax, g));
  if (!fn) return FMHA_ERR_UNSUPPORTED;
  const int rpp = rows_per_access(d);
  const int rows = smax > rpp ? smax : rpp;
  const int nu = rows / smax;
  const int tpi = d == 128 ? ldg_tpi<128>(smax, g) : ldg_tpi<256>(smax, g);
  const int64_t tiles = (P.units + nu - 1) / nu;
  const int wpb = kLdgThreads / 32;
  int bps = 1;
  fmha_status_t st = blocks_per_sm(reinterpret_cast<const void*>(fn), kLdgThreads, &bps);
  if (st != FMHA_OK) return st;
  const int64_t need = (tiles + (int64_t)wpb * tpi - 1) / ((int64_t)wpb * tpi);
  int64_t grid = (int64_t)dev.sms * bps;
  if (grid > need) grid = need;
  plan_schedule(P, dev, (tiles + tpi - 1) / tpi, grid * wpb, grid, stream);
  if (launch_overlapped(fn, (unsigned)grid, kLdgThreads, 0, stream, P) != cudaSuccess) {
    cudaGetLastError();
    return FMHA_ERR_CUDA;
  }
  return FMHA_OK;
}

// splitmix64 finaliser (Steele, Lea, Flood, OOPSLA 2014).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint16_t gen_one(uint64_t key, uint64_t e) {
  int64_t t = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint64_t h = mix64(key + e * 3u + (uint64_t)j);
    t += (int64_t)(h & 0xffffu) + (int64_t)((h >> 16) & 0xffffu) +
         (int64_t)((h >> 32) & 0xffffu) + (int64_t)(h >> 48);
  }
  const int64_t num = 2 * t + 12 - 12 * 65536;
  const float x = (float)num * (1.0f / 131072.0f);  // exact: |num| < 2^24
  uint32_t u = __float_as_uint(x);
  u += 0x7fffu + ((u >> 16) & 1u);  // bf16 round to nearest even (x is finite)
  return (uint16_t)(u >> 16);
}

__global__ void fill_normal_bf16_kernel(uint16_t* __restrict__ dst, int64_t n, uint64_t key,
                                        int64_t offset) {
  const int64_t groups = (n + 7) / 8;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups;
       gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i0 = gi * 8;
    if (i0 + 8 <= n) {
      uint32_t w[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t lo = gen_one(key, (uint64_t)(offset + i0 + 2 * c));
        const uint32_t hi = gen_one(key, (uint64_t)(offset + i0 + 2 * c + 1));
        w[c] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4*>(dst + i0) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      for (int64_t i = i0; i < n; ++i) dst[i] = gen_one(key, (uint64_t)(offset + i));
    }
  }
}

}  // namespace
}  // namespace fmha

using namespace fmha;

extern "C" {

fmha_status_t fmha_forward_variant(const void* Q, const void* K, const void* V, void* O,
                                   int batch, int num_heads_q, int num_heads_kv, int seqlen_kv,
                                   int head_dim, int variant, fmha_stream_t stream) {
  fmha_status_t st =
      check_args(Q, K, V, O, batch, num_heads_q, num_heads_kv, seqlen_kv, head_dim);
  if (st != FMHA_OK) return st;
  if (variant < FMHA_VARIANT_AUTO || variant > FMHA_VARIANT_LDG) return FMHA_ERR_INVALID_ARG;
  if (batch == 0) return FMHA_OK;
  DeviceInfo dev;
  st = device_info(&dev);
  if (st != FMHA_OK) return st;
  const int g = num_heads_q / num_heads_kv;
  const int smax = smax_for(seqlen_kv);
  Params P;
  std::memset(&P, 0, sizeof(P));
  P.Q = static_cast<const uint16_t*>(Q);
  P.K = static_cast<const uint16_t*>(K);
  P.V = static_cast<const uint16_t*>(V);
  P.O = static_cast<uint16_t*>(O);
  P.err = dev.err;
  P.wait_timeout_ns = kWaitTimeoutNs;
  if (g_test_stall.load()) {
    P.flags |= kFlagStallProducer;
    P.wait_timeout_ns = kStallTimeoutNs;
    variant = FMHA_VARIANT_BULK;
  }
  P.units = (int64_t)batch * num_heads_kv;
  P.s_len = seqlen_kv;
  P.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
  const Choice c = auto_choice(head_dim, smax, g);
  if (variant == FMHA_VARIANT_AUTO) variant = c.variant;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return variant == FMHA_VARIANT_LDG ? launch_ldg(P, head_dim, smax, g, dev, s)
                                     : launch_bulk(P, head_dim, smax, g, c.warps, dev, s);
}

fmha_status_t fmha_forward_varlen_variant(const void* Q, const void* K, const void* V,
                                          void* O, const int32_t* cu_seqlens_kv, int batch,
                                          int num_heads_q, int num_heads_kv, int max_seqlen_kv,
                                          int head_dim, float softmax_scale, int variant,
                                          fmha_stream_t stream) {
  if (variant < FMHA_VARIANT_AUTO || variant > FMHA_VARIANT_LDG) return FMHA_ERR_INVALID_ARG;
  fmha_status_t st =
      check_args(Q, K, V, O, batch, num_heads_q, num_heads_kv, max_seqlen_kv, head_dim);
  if (st != FMHA_OK) return st;
  if (batch > 0 && !cu_seqlens_kv) return FMHA_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(cu_seqlens_kv) & 3u) return FMHA_ERR_MISALIGNED;
  if (!(softmax_scale >= 0.0f) || std::isinf(softmax_scale)) return FMHA_ERR_INVALID_ARG;
  if (batch == 0) return FMHA_OK;
  DeviceInfo dev;
  st = device_info(&dev);
  if (st != FMHA_OK) return st;
  const int g = num_heads_q / num_heads_kv;
  VarlenFn fn = head_dim == 128 ? varlen_kernel_d128(g) : varlen_kernel_d256(g);
  if (!fn) return FMHA_ERR_UNSUPPORTED;
  VarlenParams P;
  std::memset(&P, 0, sizeof(P));
  P.Q = static_cast<const uint16_t*>(Q);
  P.K = static_cast<const uint16_t*>(K);
  P.V = static_cast<const uint16_t*>(V);
  P.O = static_cast<uint16_t*>(O);
  P.cu_seqlens = cu_seqlens_kv;
  P.err = dev.err;
  P.batch = batch;
  P.num_heads_kv = num_heads_kv;
  P.max_seqlen = max_seqlen_kv;
  const int smax = smax_for(max_seqlen_kv);
  const int nu = 16 / smax;
  P.tiles_per_row = (num_heads_kv + nu - 1) / nu;
  const double scale = softmax_scale > 0.0f ? (double)softmax_scale
                                            : 1.0 / std::sqrt((double)head_dim);
  P.scale_log2 = (float)(1.4426950408889634 * scale);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  // AUTO: the chunk ring for both head_dims (on the reference's Poisson(4)
  // table it beats the register-prefetch kernel by 4-27 % at D=256 once its
  // scores run on the tensor cores). FMHA_VARLEN_KERNEL=ldg|chunk, read on
  // every AUTO call, overrides that default.
  if (variant == FMHA_VARIANT_AUTO) {
    const char* kind = std::getenv("FMHA_VARLEN_KERNEL");
    variant = (kind && std::strcmp(kind, "ldg") == 0) ? FMHA_VARIANT_LDG : FMHA_VARIANT_BULK;
  }
  if (variant == FMHA_VARIANT_LDG) {
    int bps = 1;
    st = blocks_per_sm(reinterpret_cast<const void*>(fn), kLdgThreads, &bps);
    if (st != FMHA_OK) return st;
    // Head ranges of ~4 heads per work item (FMHA_VARLEN_SPLIT overrides).
    int qs = num_heads_kv / 4 > 1 ? num_heads_kv / 4 : 1;
    qs = env_int("FMHA_VARLEN_SPLIT", qs);
    if (qs < 1) qs = 1;
    if (qs > num_heads_kv) qs = num_heads_kv;
    P.tiles_per_row = qs;
    int64_t grid = (int64_t)dev.sms * bps;
    const int64_t need = ((int64_t)batch * qs + kLdgThreads / 32 - 1) / (kLdgThreads / 32);
    if (grid > need) grid = need;
    if (launch_overlapped(fn, (unsigned)grid, kLdgThreads, 0, cs, P) != cudaSuccess) {
      cudaGetLastError();
      return FMHA_ERR_CUDA;
    }
    return FMHA_OK;
  }
  // Chunk ring: whole packed rows (or head groups) as chunks of a byte ring.
  VarlenFn cfn = head_dim == 128 ? varlen_chunk_kernel_d128(g) : varlen_chunk_kernel_d256(g);
  if (!cfn) return FMHA_ERR_UNSUPPORTED;
  P.wait_timeout_ns = kWaitTimeoutNs;
  // Consumer warps: 12 at D=256, 16 at D=128 (in-process A/B on the
  // reference's table: 12 beat 16 by 1.5-3 % on every D=256 shape, and lost
  // 5-8 % at D=128).
  int ncw = env_int("FMHA_VARLEN_WARPS", head_dim == 256 ? 12 : 16);
  if (ncw < 1) ncw = 1;
  if (ncw > kBulkMaxThreads / 32 - 1) ncw = kBulkMaxThreads / 32 - 1;
  P.sc_off = kVarlenChunkHdr;
  P.ring_off = (P.sc_off + (uint32_t)ncw * g * 16 * 4 + 1023u) & ~1023u;
  // A multiple of the row size (D*2 bytes, itself a multiple of 128).
  const uint32_t row_b = (uint32_t)head_dim * 2;
  const uint32_t ring = (uint32_t)((dev.smem_optin - (int64_t)P.ring_off) / row_b) * row_b;
  P.stage_bytes = ring;
  uint32_t cmax = (uint32_t)env_int("FMHA_VARLEN_CHUNK", 96 * 1024);
  if (cmax > ring / 2) cmax = ring / 2;
  // One head of the longest row must fit in a chunk.
  const uint32_t one = (uint32_t)(2 * max_seqlen_kv + g) * head_dim * 2;
  if (one > cmax) return FMHA_ERR_UNSUPPORTED;
  P.chunk_max = cmax;
  st = ensure_smem(reinterpret_cast<const void*>(cfn), dev.smem_optin);
  if (st != FMHA_OK) return st;
  const int grid = batch < dev.sms ? batch : dev.sms;
  if (launch_overlapped(cfn, (unsigned)grid, 32u * (1 + ncw), P.ring_off + ring, cs, P) !=
      cudaSuccess) {
    cudaGetLastError();
    return FMHA_ERR_CUDA;
  }
  return FMHA_OK;
}

fmha_status_t fmha_forward_varlen(const void* Q, const void* K, const void* V, void* O,
                                  const int32_t* cu_seqlens_kv, int batch, int num_heads_q,
                                  int num_heads_kv, int max_seqlen_kv, int head_dim,
                                  float softmax_scale, fmha_stream_t stream) {
  return fmha_forward_varlen_variant(Q, K, V, O, cu_seqlens_kv, batch, num_heads_q, num_heads_kv,
                                     max_seqlen_kv, head_dim, softmax_scale, FMHA_VARIANT_AUTO,
                                     stream);
}

fmha_status_t fmha_forward_append(const void* Q, void* K_cache, void* V_cache,
                                  const void* K_new, const void* V_new, void* O, int batch,
                                  int num_heads_q, int num_heads_kv, int seqlen_kv,
                                  int cache_seqlen, int head_dim, fmha_stream_t stream) {
  fmha_status_t st =
      check_args(Q, K_cache, V_cache, O, batch, num_heads_q, num_heads_kv, seqlen_kv, head_dim);
  if (st != FMHA_OK) return st;
  if (batch > 0 && (!K_new || !V_new)) return FMHA_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(K_new) | reinterpret_cast<uintptr_t>(V_new)) & 15u)
    return FMHA_ERR_MISALIGNED;
  if (cache_seqlen < seqlen_kv) return FMHA_ERR_INVALID_ARG;
  if (batch == 0) return FMHA_OK;
  DeviceInfo dev;
  st = device_info(&dev);
  if (st != FMHA_OK) return st;
  Params P;
  std::memset(&P, 0, sizeof(P));
  P.Q = static_cast<const uint16_t*>(Q);
  P.K = static_cast<const uint16_t*>(K_cache);
  P.V = static_cast<const uint16_t*>(V_cache);
  P.O = static_cast<uint16_t*>(O);
  P.K_new = static_cast<const uint16_t*>(K_new);
  P.V_new = static_cast<const uint16_t*>(V_new);
  P.kv_ustride = (int64_t)cache_seqlen * head_dim;
  P.err = dev.err;
  P.wait_timeout_ns = kWaitTimeoutNs;
  P.units = (int64_t)batch * num_heads_kv;
  P.s_len = seqlen_kv;
  P.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
  return launch_ldg(P, head_dim, smax_for(seqlen_kv), num_heads_q / num_heads_kv, dev,
                    reinterpret_cast<cudaStream_t>(stream), true);
}

fmha_status_t fmha_forward(const void* Q, const void* K, const void* V, void* O, int batch,
                           int num_heads_q, int num_heads_kv, int seqlen_kv, int head_dim,
                           fmha_stream_t stream) {
  return fmha_forward_variant(Q, K, V, O, batch, num_heads_q, num_heads_kv, seqlen_kv, head_dim,
                              FMHA_VARIANT_AUTO, stream);
}

const char* fmha_status_string(fmha_status_t status) {
  switch (status) {
    case FMHA_OK: return "FMHA_OK";
    case FMHA_ERR_INVALID_ARG: return "FMHA_ERR_INVALID_ARG: invalid argument";
    case FMHA_ERR_UNSUPPORTED: return "FMHA_ERR_UNSUPPORTED: unsupported shape";
    case FMHA_ERR_MISALIGNED: return "FMHA_ERR_MISALIGNED: pointer not 16-byte aligned";
    case FMHA_ERR_CUDA: return "FMHA_ERR_CUDA: CUDA runtime error";
    case FMHA_ERR_DEVICE_TIMEOUT: return "FMHA_ERR_DEVICE_TIMEOUT: a kernel wait timed out";
    default: return "FMHA_ERR_UNKNOWN";
  }
}

fmha_status_t fmha_device_error(int* code) {
  if (!code) return FMHA_ERR_INVALID_ARG;
  DeviceInfo dev;
  fmha_status_t st = device_info(&dev);
  if (st != FMHA_OK) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return FMHA_ERR_CUDA;
  unsigned int v = 0;
  if (cudaMemcpy(&v, dev.err, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
    return FMHA_ERR_CUDA;
  if (v != 0 && cudaMemset(dev.err, 0, sizeof(v)) != cudaSuccess) return FMHA_ERR_CUDA;
  *code = (int)v;
  return FMHA_OK;
}

fmha_status_t fmha_fill_normal_bf16(void* dst, int64_t n, uint64_t seed, uint32_t tensor_id,
                                    int64_t offset, fmha_stream_t stream) {
  if (n < 0 || offset < 0) return FMHA_ERR_INVALID_ARG;
  if (n == 0) return FMHA_OK;
  if (!dst) return FMHA_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(dst) & 15u) return FMHA_ERR_MISALIGNED;
  DeviceInfo dev;
  fmha_status_t st = device_info(&dev);
  if (st != FMHA_OK) return st;
  const uint64_t key = mix64(seed ^ mix64(((uint64_t)tensor_id << 32) | 0x5bd1e995u));
  const int64_t groups = (n + 7) / 8;
  int64_t grid = (groups + 255) / 256;
  const int64_t cap = (int64_t)dev.sms * 16;
  if (grid > cap) grid = cap;
  fill_normal_bf16_kernel<<<(unsigned)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint16_t*>(dst), n, key, offset);
  return cudaGetLastError() == cudaSuccess ? FMHA_OK : FMHA_ERR_CUDA;
}

void fmha_test_inject_stall(int on) { g_test_stall.store(on ? 1 : 0); }

fmha_status_t fmha_seqlens_poisson(int batch, int max_seqlen_kv, uint32_t seed, double lambda,
                                   int32_t* out) {
  if (batch < 0 || max_seqlen_kv < 2 || !(lambda > 0.0) || (batch > 0 && !out))
    return FMHA_ERR_INVALID_ARG;
  // A lambda far outside [2, max_seqlen_kv] would make the redraw loop run
  // practically forever; the loop is capped and such a lambda is rejected.
  if (!(lambda <= 4.0 * max_seqlen_kv + 64.0)) return FMHA_ERR_INVALID_ARG;
  std::mt19937 gen(seed);
  std::poisson_distribution<int> dist(lambda);
  const long kMaxDraws = 1L << 20;  // per row
  for (int i = 0; i < batch; ++i) {
    int len;
    long draws = 0;
    do {
      if (++draws > kMaxDraws) return FMHA_ERR_INVALID_ARG;
      len = dist(gen);
    } while (len < 2 || len > max_seqlen_kv);
    out[i] = len;
  }
  return FMHA_OK;
}

const char* fmha_version(void) { return "fmha_b200 0.1.0 sm_100a"; }

}  // extern "C"
