// decode_ldg.cu -- "ldg" kernel family: persistent warps that load their
// tiles' K/V rows straight into registers with 16-byte streaming loads
// (ld.global.nc, no L1 allocation, 256-byte L2 fetch), then compute.
//
// Each warp takes TPI consecutive tiles per step (tiles s*TPI .. s*TPI+TPI-1
// of step s) and issues every load of the step before the first arithmetic,
// so each warp keeps TPI*NP*2 16-byte loads per lane in flight. Steps are
// dealt out statically (warp w: w, w+W, ...) for P.sched_rounds rounds; the
// remaining tail is claimed one step at a time from the launch's schedule
// slot (sched_join; warp w claims from counter w % kSchedLanes), each claim
// issued one step ahead so its latency hides behind the current step. This evens out SMs that stream at different rates
// (a static schedule left the slowest SM ~7 % behind the fastest).
// Compiled once per head_dim: -DFMHA_HEAD_DIM=128 or 256.
#include "decode_common.cuh"

#ifndef FMHA_HEAD_DIM
#error "compile with -DFMHA_HEAD_DIM=128 or 256"
#endif

namespace fmha {

// APPEND: the K/V slabs are rows 0..s_len-1 of a cache with P.kv_ustride
// elements per unit; row s_len-1 is this step's new row, read from
// P.K_new/P.V_new ([units, D]) and also written into the cache, in the same
// pass (fused KV-cache append + attend).
template <int D, int SMAX, int G, int TPI, bool APPEND>
__global__ void __launch_bounds__(kLdgThreads) decode_ldg_kernel(const Params P) {
  using T = TileShape<D, SMAX, G>;
  constexpr int WPB = kLdgThreads / 32;
  __shared__ float sc_all[WPB][T::SC];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  float* sc = sc_all[warp];
  const int r0 = lane / T::LPR;
  const int cl = lane % T::LPR;
  const int ul = OutputMap<D, SMAX, G>::unit(lane);
  const int s_len = P.s_len;
  const int64_t tiles = (P.units + T::NU - 1) / T::NU;
  const int64_t steps = (tiles + TPI - 1) / TPI;
  const int64_t gw = (int64_t)blockIdx.x * WPB + warp;
  const int64_t W = (int64_t)gridDim.x * WPB;
  const int64_t R = P.sched_rounds;
  __shared__ int s_joined;
  allow_dependent_launch();
  // The schedule slot is this launch's own; everything else waits for the
  // previous kernel of the stream.
  if (threadIdx.x == 0) s_joined = sched_join(P.sched, P.sched_tag) ? 1 : 0;
  grid_dependency_wait();
  __syncthreads();
  const bool dyn = s_joined != 0;
  // Step of round r: static below R (or always when not joined), else claimed
  // from this warp's counter: tail steps R*W + j + kSchedLanes*c.
  const int j = warp % kSchedLanes;
  unsigned long long* ctr = dyn ? sched_counter(P.sched, j) : nullptr;
  auto tail_step = [&](unsigned long long c) {
    return R * W + j + (int64_t)kSchedLanes * (int64_t)__shfl_sync(kFullMask, c, 0);
  };
  int64_t r = 0;
  int64_t step = gw;
  if (dyn && R == 0) {
    unsigned long long tk = 0;
    if (lane == 0) tk = atomicAdd(ctr, 1ull);
    step = tail_step(tk);
  }

  while (step < steps) {
    const int64_t t0 = step * TPI;
    // Claim the next step now if it comes from the tail; used after this one.
    const bool claim_next = dyn && r + 1 >= R;
    unsigned long long tk = 0;
    if (claim_next && lane == 0) tk = atomicAdd(ctr, 1ull);
    uint4 kr[TPI][T::NP], vr[TPI][T::NP], qr[TPI][G];
    int uv[TPI];
#pragma unroll
    for (int i = 0; i < TPI; ++i) {
      const int64_t tile_u0 = (t0 + i) * T::NU;
      const int64_t left = P.units - tile_u0;
      uv[i] = left <= 0 ? 0 : (left < T::NU ? (int)left : T::NU);
      const int64_t ustride = APPEND ? P.kv_ustride : (int64_t)s_len * D;
      const uint16_t* kb = P.K + tile_u0 * ustride + cl * 8;
      const uint16_t* vb = P.V + tile_u0 * ustride + cl * 8;
#pragma unroll
      for (int p = 0; p < T::NP; ++p) {
        const int r = p * T::RPP + r0;
        const int64_t off = (int64_t)(r / SMAX) * ustride + (int64_t)(r % SMAX) * D;
        const bool ok = (r % SMAX) < s_len && (r / SMAX) < uv[i];
        if (APPEND && ok && (r % SMAX) == s_len - 1) {
          const int64_t noff = (tile_u0 + r / SMAX) * D + cl * 8;
          kr[i][p] = ldg_stream(P.K_new + noff);
          vr[i][p] = ldg_stream(P.V_new + noff);
          stg_stream(const_cast<uint16_t*>(kb + off), kr[i][p]);
          stg_stream(const_cast<uint16_t*>(vb + off), vr[i][p]);
        } else {
          kr[i][p] = ok ? ldg_stream(kb + off) : make_uint4(0, 0, 0, 0);
          vr[i][p] = ok ? ldg_stream(vb + off) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
        qr[i][g] = ul < uv[i] ? ldg_stream(P.Q + (tile_u0 + ul) * (G * D) + g * D + cl * 8)
                              : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < TPI; ++i) {
      if (uv[i] <= 0) continue;  // warp-uniform
      float q[G][8];
#pragma unroll
      for (int g = 0; g < G; ++g) unpack8(qr[i][g], q[g]);
      float acc[G][8];
      auto loadK = [&](int p) { return kr[i][p]; };
      auto loadV = [&](int p) { return vr[i][p]; };
      attend_tile<D, SMAX, G>(q, loadK, loadV, s_len, uv[i], P.scale_log2, sc, lane, acc);
      if (ul < uv[i] && OutputMap<D, SMAX, G>::writer(lane)) {
        uint16_t* orow = P.O + ((t0 + i) * T::NU + ul) * (G * D) + cl * 8;
#pragma unroll
        for (int g = 0; g < G; ++g) stg_stream(orow + g * D, pack8_f16(acc[g]));
      }
    }
    ++r;
    step = claim_next ? tail_step(tk) : gw + r * W;
  }
  __syncthreads();  // every warp of the CTA has made its last claim
  if (dyn && threadIdx.x == 0) sched_leave(P.sched);
}

#define FMHA_CAT2(a, b) a##b
#define FMHA_CAT(a, b) FMHA_CAT2(a, b)

KernelFn FMHA_CAT(ldg_kernel_d, FMHA_HEAD_DIM)(int smax, int g) {
  constexpr int D = FMHA_HEAD_DIM;
#define FMHA_K(SM, GG) decode_ldg_kernel<D, SM, GG, LdgTpi<D, SM, GG>::value, false>
#define FMHA_G(SM)                    \
  switch (g) {                        \
    case 1: return FMHA_K(SM, 1);     \
    case 2: return FMHA_K(SM, 2);     \
    case 4: return FMHA_K(SM, 4);     \
    case 8: return FMHA_K(SM, 8);     \
    default: return nullptr;          \
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
#undef FMHA_K
}

KernelFn FMHA_CAT(ldg_append_kernel_d, FMHA_HEAD_DIM)(int smax, int g) {
  constexpr int D = FMHA_HEAD_DIM;
#define FMHA_K(SM, GG) decode_ldg_kernel<D, SM, GG, LdgTpi<D, SM, GG>::value, true>
#define FMHA_G(SM)                    \
  switch (g) {                        \
    case 1: return FMHA_K(SM, 1);     \
    case 2: return FMHA_K(SM, 2);     \
    case 4: return FMHA_K(SM, 4);     \
    case 8: return FMHA_K(SM, 8);     \
    default: return nullptr;          \
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
#undef FMHA_K
}

}  // namespace fmha
