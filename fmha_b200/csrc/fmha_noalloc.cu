// fmha_noalloc.cu -- fmha_forward_noalloc: the dense decode-attention call for
// callers that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- an allocator
// or memory-pool hook that must not re-enter the allocator, a driver-level
// plug-in whose host application owns every device allocation, or a caller
// with a fixed memory budget checked up front. Such a caller passes only its
// own inputs and outputs and needs a guarantee that the library takes nothing
// else from the device heap, now or on a later call.
//
// What it runs: the ldg kernel family (decode_ldg.cu) with its dynamic tail.
// The tail's scratch -- one schedule slot: a tag/user word and kSchedLanes
// claim counters, 128 bytes apart -- lives in g_noalloc_scratch below, a
// file-scope static device array of kNoAllocScratchBytes (1152 bytes) that
// every GPU loading the library holds until the process exits. Nothing is
// allocated, on the first call or later.
//
// Set-up: the first call on a device, with that device current, looks up the
// array's device address (cudaGetSymbolAddress; in host code the array's name
// is only a host-side stand-in) and the device's SM count. That first call
// should therefore come before any stream capture. Later calls reuse the
// cached address.
//
// Sharing: every call on a device uses the same array. The slot returns to
// all zeros when its last user leaves, which is what a call needs at its
// start, so no clearing is needed between calls; a call whose kernel finds
// the slot held by another call (calls overlapping on the GPU) does not use
// it and runs its whole schedule statically. Overlapping calls therefore race
// for the scratch; each still computes its own output in full.
//
// Limits: the schedule word counts its users (CTAs) in 12 bits, so a launch
// may use at most kNoAllocMaxCtas CTAs; the kernels index units in 32-bit
// chunks, so batch * num_heads_kv is at most 2^30. Calls beyond either
// return FMHA_ERR_UNSUPPORTED without launching anything (the unit count is
// checked before any CUDA call, the CTA count once the SM count is known).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/fmha.h"
#include "decode_common.cuh"

namespace fmha {
namespace {

constexpr int kNoAllocScratchWords = kSchedSlotWords;  // one schedule slot
constexpr size_t kNoAllocScratchBytes = kNoAllocScratchWords * sizeof(unsigned long long);
static_assert(kNoAllocScratchBytes == 1152, "stated scratch size");
constexpr int kNoAllocMaxCtas = 4095;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocScratchWords];

struct NoAllocDevice {
  bool ready = false;
  int sms = 0;
  unsigned long long* scratch = nullptr;  // device address of g_noalloc_scratch
  uint64_t seq = 0;                       // launches so far (tags)
  const void* occ_fn[64] = {};            // resident CTAs per SM, per kernel
  int occ_bps[64] = {};
  int occ_n = 0;
};

std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];

// Once per device, with it current: the scratch address and the SM count.
fmha_status_t noalloc_setup(int dev, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return FMHA_ERR_CUDA;
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return FMHA_ERR_CUDA;
    d.scratch = static_cast<unsigned long long*>(p);
    d.ready = true;
  }
  *out = &d;
  return FMHA_OK;
}

int smax_of_len(int s) {
  int m = 1;
  while (m < s) m <<= 1;
  return m;
}

template <int D>
int tpi_of(int smax, int g) {
#define FMHA_NA_T(SM)                          \
  switch (g) {                                 \
    case 1: return LdgTpi<D, SM, 1>::value;    \
    case 2: return LdgTpi<D, SM, 2>::value;    \
    case 4: return LdgTpi<D, SM, 4>::value;    \
    default: return LdgTpi<D, SM, 8>::value;   \
  }
  switch (smax) {
    case 1: FMHA_NA_T(1)
    case 2: FMHA_NA_T(2)
    case 4: FMHA_NA_T(4)
    case 8: FMHA_NA_T(8)
    default: FMHA_NA_T(16)
  }
#undef FMHA_NA_T
}

}  // namespace
}  // namespace fmha

using namespace fmha;

extern "C" fmha_status_t fmha_forward_noalloc(const void* Q, const void* K, const void* V,
                                              void* O, int batch, int num_heads_q,
                                              int num_heads_kv, int seqlen_kv, int head_dim,
                                              fmha_stream_t stream) {
  // The same argument rules as fmha_forward, checked before any CUDA call.
  if (batch < 0 || num_heads_q <= 0 || num_heads_kv <= 0 || seqlen_kv <= 0 || head_dim <= 0)
    return FMHA_ERR_INVALID_ARG;
  if (num_heads_q % num_heads_kv != 0) return FMHA_ERR_INVALID_ARG;
  if (batch > 0 && (!Q || !K || !V || !O)) return FMHA_ERR_INVALID_ARG;
  if (head_dim != 128 && head_dim != 256) return FMHA_ERR_UNSUPPORTED;
  if (seqlen_kv > 16) return FMHA_ERR_UNSUPPORTED;
  const int g = num_heads_q / num_heads_kv;
  if (g != 1 && g != 2 && g != 4 && g != 8) return FMHA_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
       reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(O)) & 15u)
    return FMHA_ERR_MISALIGNED;
  if ((int64_t)batch * num_heads_kv > (int64_t)1 << 30) return FMHA_ERR_UNSUPPORTED;
  if (batch == 0) return FMHA_OK;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FMHA_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return FMHA_ERR_CUDA;
  NoAllocDevice* nd = nullptr;
  fmha_status_t st = noalloc_setup(dev, &nd);
  if (st != FMHA_OK) return st;

  const int smax = smax_of_len(seqlen_kv);
  KernelFn fn = head_dim == 128 ? ldg_kernel_d128(smax, g) : ldg_kernel_d256(smax, g);
  if (!fn) return FMHA_ERR_UNSUPPORTED;
  int bps = 0;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    for (int i = 0; i < nd->occ_n; ++i)
      if (nd->occ_fn[i] == reinterpret_cast<const void*>(fn)) bps = nd->occ_bps[i];
  }
  if (bps == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, fn, kLdgThreads, 0) != cudaSuccess)
      return FMHA_ERR_CUDA;
    if (bps < 1) bps = 1;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (nd->occ_n < 64) {
      nd->occ_fn[nd->occ_n] = reinterpret_cast<const void*>(fn);
      nd->occ_bps[nd->occ_n++] = bps;
    }
  }

  Params P;
  std::memset(&P, 0, sizeof(P));
  P.Q = static_cast<const uint16_t*>(Q);
  P.K = static_cast<const uint16_t*>(K);
  P.V = static_cast<const uint16_t*>(V);
  P.O = static_cast<uint16_t*>(O);
  P.err = nullptr;  // the ldg kernels have no waits and report nothing
  P.wait_timeout_ns = kWaitTimeoutNs;
  P.units = (int64_t)batch * num_heads_kv;
  P.s_len = seqlen_kv;
  P.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));

  const int rpa = 256 / head_dim;  // K/V rows per 16-byte warp access
  const int nu = (smax > rpa ? smax : rpa) / smax;
  const int tpi = head_dim == 128 ? tpi_of<128>(smax, g) : tpi_of<256>(smax, g);
  const int wpb = kLdgThreads / 32;
  const int64_t tiles = (P.units + nu - 1) / nu;
  const int64_t steps = (tiles + tpi - 1) / tpi;
  const int64_t need = (steps + wpb - 1) / wpb;
  int64_t grid = (int64_t)nd->sms * bps;
  if (grid > need) grid = need;
  if (grid > kNoAllocMaxCtas) return FMHA_ERR_UNSUPPORTED;

  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(cs, &cap) != cudaSuccess) {
    cudaGetLastError();
    cap = cudaStreamCaptureStatusActive;  // unknown: take the static schedule
  }
  if (cap == cudaStreamCaptureStatusNone) {
    // Dynamic tail on the scratch slot: 90 % of the steps static, a fresh tag.
    uint64_t seq;
    {
      std::lock_guard<std::mutex> lk(g_noalloc_mu);
      seq = nd->seq++;
    }
    P.sched = nd->scratch;
    P.sched_tag = (uint32_t)(seq % 0xffffffu) + 1u;
    P.sched_rounds = steps * 90 / 100 / (grid * wpb);
  }
  fn<<<(unsigned)grid, kLdgThreads, 0, cs>>>(P);
  return cudaGetLastError() == cudaSuccess ? FMHA_OK : FMHA_ERR_CUDA;
}
