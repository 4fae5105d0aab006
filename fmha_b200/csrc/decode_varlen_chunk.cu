// decode_varlen_chunk.cu -- packed-varlen decode attention streamed as whole
// batch rows through a shared-memory byte ring (large 1-D bulk copies).
//
// Layout: K/V [sum_b S_b, Hkv, D] with cu_seqlens_kv[B+1]
// (fmha_host.cpp:143-157), Q/O [B, Hq, 1, D].
//
// In the packed layout the K rows of one batch row b, all kv heads, are one
// contiguous block of S_b*Hkv*D elements (so are its V rows, and its Hq query
// rows), and consecutive batch rows are adjacent. A *chunk* is up to
// kChunkRows consecutive whole rows (three contiguous ranges: K, V, Q) that
// fit the chunk limit -- or, for a row too long for the limit on its own, the
// rows of a group of nh consecutive kv heads, whose K rows at one position s
// are one contiguous run of nh*D elements. Packing short rows together keeps
// every chunk large, which is what keeps the bulk copies efficient.
//
// Per CTA (persistent, one per SM): a contiguous range of batch rows holding
// an equal share of the bytes (found by a 16-ary search over cu_seqlens, see
// weight_split), not an equal number of rows.
//  * Producer (warp 0) plans 32 rows at a time: each lane loads its row's
//    cu_seqlens pair and sizes the row, then every lane runs the same greedy
//    packing over the window from shared memory (no shuffle chains), so each
//    lane knows its row's chunk, index, first K/V row and first tile. Per
//    chunk it then allocates the chunk in a circular byte ring whose size is a
//    multiple of one row (D*2 bytes), so a chunk may wrap past the end
//    without any row straddling it (copies that cross are split in two;
//    readers wrap their row offsets), and no space is lost to padding; writes
//    the chunk's descriptor (per-row lengths, offsets and first tiles) into slot
//    c % kSlots, arms the slot's `full` mbarrier with the chunk's byte count
//    and issues the copies: one bulk copy each for K, V and Q of whole rows
//    (lanes 0-2 together), or one K and one V copy per position for a head
//    group.
//    It then publishes the chunk count. Ring space and slots are reclaimed in
//    chunk order by waiting on each slot's `empty` mbarrier, one phase after
//    another (a single producer walks every slot's phases in order).
//  * Consumers (all other warps) take 16-row tiles (NU = 16/SMAX_b kv heads of
//    one chunk) from a shared atomic tile counter, find the tile's chunk among
//    the published ones, wait for its `full` phase (published => armed, so the
//    parity names the right phase), run the shared tile math from shared
//    memory (QK^T on mma.sync when the tile has at most 16 query rows) and
//    stream fp16 rows to O. The last tile of a chunk resets the
//    chunk's tile counter and arrives on its `empty` mbarrier.
//
// A row length outside [0, max_seqlen_kv] sets the device error word
// (FMHA_ERR_INVALID_ARG, site 5) and the row is skipped; a zero-length row
// yields zeros. Every wait is bounded (globaltimer) and never traps; on exit
// the producer waits (bounded) for its own copies still in flight.
//
// Compiled once per head_dim: -DFMHA_HEAD_DIM=128 or 256.
#include "decode_common.cuh"

#ifndef FMHA_HEAD_DIM
#error "compile with -DFMHA_HEAD_DIM=128 or 256"
#endif

namespace fmha {

namespace {

constexpr int kChunkRows = 8;  // whole batch rows per chunk at most

struct alignas(16) ChunkDesc {
  int64_t b0;         // first batch row
  int64_t end_total;  // ring bytes allocated up to the end of this chunk
  uint32_t off;       // chunk start in the ring
  uint32_t kv_bytes;  // bytes of the K part (= of the V part)
  int h0;             // first kv head covered
  int nh;             // kv heads covered (all rows of the chunk)
  int tile_base;      // CTA-local index of the chunk's first tile
  int ntiles;
  int nrows;
  int pad;
  uint16_t krow[kChunkRows];    // first K/V row of row j, relative to the chunk
  uint16_t s_len[kChunkRows];   // rows per head of row j
  uint16_t tstart[kChunkRows];  // tiles of rows < j
};
static_assert(sizeof(ChunkDesc) <= 112, "descriptor size");
constexpr uint32_t kDescStride = 112;
// Producer plan arrays (32 rows + 32 entries of int4) in the header area,
// after the barriers, counters and descriptors.
constexpr uint32_t kPlanOff = 4352;
static_assert(16 * kVarlenSlots + 4 * (4 + kVarlenSlots) + kVarlenSlots * kDescStride + 15 <= kPlanOff &&
                  kPlanOff + 64 * 16 <= kVarlenChunkHdr,
              "header layout");

// What one tile needs: its batch row, length, heads and shared-memory bases.
struct TileRef {
  int64_t b;
  int s_len;
  int h0;         // first kv head of the chunk
  int nh;         // row stride in heads inside the chunk
  uint32_t koff, voff, qoff;  // ring-relative offsets (< R); rows wrap at R
};

__device__ __forceinline__ int smax_of(int s) {
  return s <= 1 ? 1 : s <= 2 ? 2 : s <= 4 ? 4 : s <= 8 ? 8 : 16;
}

template <int D, int SMAX, int G>
__device__ __forceinline__ void chunk_tile(const VarlenParams& P, const TileRef& c, int hl0,
                                           uint32_t ring0, uint32_t R, float* sc, int lane) {
  using T = Tile16<D, SMAX, G>;
  const int r0 = lane / T::LPR;
  const int cl = lane % T::LPR;
  const int nh = c.nh;
  const int nv = nh - hl0 < T::NU ? nh - hl0 : T::NU;
  // Ring addresses wrap at R (a multiple of the row size, so a row never
  // straddles the end).
  auto at = [&](uint32_t off) { return ring0 + (off >= R ? off - R : off) + cl * 16; };
  // Tile row r = (unit u, position s) is chunk row s*nh + hl0 + u.
  auto rowoff = [&](int p) -> uint32_t {
    const int r = r0 * T::NP + p;
    return (uint32_t)((r % SMAX) * nh + hl0 + r / SMAX) * (D * 2);
  };
  auto loadK = [&](int p) { return lds128(at(c.koff + rowoff(p))); };
  auto loadV = [&](int p) { return lds128(at(c.voff + rowoff(p))); };
  auto loadQ = [&](int, int u, int g) {
    return lds128(at(c.qoff + (uint32_t)((hl0 + u) * G + g) * (D * 2)));
  };
  const int64_t qrow0 = (c.b * P.num_heads_kv + c.h0 + hl0) * G;
  auto store = [&](int u, const float (&acc)[G][8]) {
    if (u >= nv) return;
    uint16_t* orow = P.O + (qrow0 + u * G) * D + cl * 8;
#pragma unroll
    for (int g = 0; g < G; ++g) stg_stream(orow + g * D, pack8_f16(acc[g]));
  };
#ifndef FMHA_CHUNK_NO_MQ
  if constexpr (Tile16Mq<D, SMAX, G>::OK) {
    auto base = [&](uint32_t off) { return ring0 + (off >= R ? off - R : off); };
    auto krow = [&](int r) {
      return base(c.koff + (uint32_t)((r % SMAX) * nh + hl0 + r / SMAX) * (D * 2));
    };
    auto qrow = [&](int u, int h) { return base(c.qoff + (uint32_t)((hl0 + u) * G + h) * (D * 2)); };
    attend_tile16_mq<D, SMAX, G>(krow, qrow, loadV, store, c.s_len, nv, P.scale_log2, sc, lane);
    return;
  }
#endif
  attend_tile16<D, SMAX, G>(loadK, loadV, loadQ, store, c.s_len, nv, P.scale_log2, sc, lane);
}

// First batch row b in [0, B] whose start weight W(b) = 2*cu[b] + 2*G*b
// reaches T (the bytes of rows < b, in units of hkv*D*2 bytes: K+V 2*S_b, Q
// and O G each), or B. Lanes 0-15 search one target, lanes 16-31 another;
// 16 probes per half-warp per round (one round of dependent loads), so a
// batch of 30720 rows takes ~5 rounds. Deterministic: the same target gives
// the same row in every CTA. If cu_seqlens is not monotonic (a negative
// length) the ranges built from it may overlap but never leave a gap.
__device__ __forceinline__ int64_t weight_split(const int32_t* cu, int64_t B, int G, int64_t T,
                                                int lane) {
  const int k = (lane & 15) + 1;
  const int sh = lane & 16;
  int64_t lo = -1, hi = B;  // the row is in (lo, hi]
  for (int round = 0; round < 64; ++round) {
    const bool active = hi - lo > 1;
    if (!__any_sync(kFullMask, active)) break;
    const int64_t step = (hi - lo) / 16 > 0 ? (hi - lo) / 16 : 1;
    int64_t p = lo + k * step;
    if (p > hi) p = hi;
    bool ge = true;
    if (active && p < hi) ge = 2 * (int64_t)__ldg(cu + p) + 2 * (int64_t)G * p >= T;
    const unsigned bits = (__ballot_sync(kFullMask, ge) >> sh) & 0xffffu;
    if (active) {
      if (bits == 0) {
        lo += 16 * step;
      } else {
        const int kk = __ffs(bits);
        const int64_t h = lo + kk * step;
        hi = h < hi ? h : hi;
        lo += (kk - 1) * step;
      }
    }
  }
  return hi;
}

}  // namespace

template <int D, int G>
__global__ void __launch_bounds__(kBulkMaxThreads, 1)
    decode_varlen_chunk_kernel(const VarlenParams P) {
  constexpr int M = kVarlenSlots;
  extern __shared__ __align__(1024) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(smem);
  const uint32_t empty0 = full0 + 8u * M;
  volatile int* ctrl = reinterpret_cast<volatile int*>(smem + 16 * M);
  volatile int* abort_flag = ctrl + 0;
  volatile int* published = ctrl + 1;    // chunks whose copies are armed
  volatile int* total_tiles = ctrl + 2;  // tile count once the producer is done, else -1
  int* next_tile = const_cast<int*>(ctrl + 3);
  int* done = const_cast<int*>(ctrl + 4);  // [M] tiles finished per slot
  unsigned char* desc_base = smem + ((16 * M + 4 * (4 + M) + 15) & ~15);
  auto desc_at = [&](int slot) {
    return reinterpret_cast<ChunkDesc*>(desc_base + (size_t)slot * kDescStride);
  };
  unsigned char* ring = smem + P.ring_off;
  const uint32_t ring0 = smem_u32(ring);
  const uint32_t R = P.stage_bytes;  // ring size in bytes (a multiple of the row size D*2)

  allow_dependent_launch();
  if (threadIdx.x == 0) {
    for (int i = 0; i < M; ++i) {
      mbar_init(full0 + 8u * i, 1);
      mbar_init(empty0 + 8u * i, 1);
      done[i] = 0;
    }
    *abort_flag = 0;
    *published = 0;
    *total_tiles = -1;
    *next_tile = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // Inputs and outputs may be written by the previous kernel of the stream.
  grid_dependency_wait();
  __syncthreads();


  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const int hkv = P.num_heads_kv;
    const uint64_t policy = policy_evict_first();
    int64_t tail = 0, head = 0;  // ring bytes ever allocated / ever released
    uint32_t off = 0;            // ring position of `tail` (tail mod R, kept incrementally)
    int c = 0, oldest = 0, tiles = 0;
    bool stop = false;
    // Plan of the current 32-row window: per row {bytes, length, kind,
    // tiles}; per chunk {first row, rows, K/V rows, tiles | kind << 24}.
    int4* win = reinterpret_cast<int4*>(smem + kPlanOff);
    int4* cinfo = win + 32;
    auto heads_per_tile = [](int s_len) {
      const int s = s_len <= 1 ? 1 : s_len <= 2 ? 2 : s_len <= 4 ? 4 : s_len <= 8 ? 8 : 16;
      return 16 / s;
    };

    // Allocates ring space and a slot for a chunk, lets `rows` write the
    // descriptor's per-row entries, writes its header, arms `full`, lets
    // `issue` launch the copies and publishes the chunk.
    auto emit = [&](int64_t b0, int nrows, int h0, int nh, int ntiles, uint32_t kvb, uint32_t qb,
                    auto&& rows, auto&& issue) {
      const uint32_t sz = 2 * kvb + qb;  // whole rows: a multiple of D*2 bytes, <= R/2
      while (oldest <= c - M || tail + sz - head > (int64_t)R) {
        if (!mbar_wait(empty0 + 8u * (oldest % M), (oldest / M) & 1, abort_flag, P.err,
                       P.wait_timeout_ns, kSiteProducerEmpty)) {
          stop = true;
          return;
        }
        head = desc_at(oldest % M)->end_total;
        ++oldest;
      }
      const uint32_t at = off;
      tail += sz;
      off += sz;
      if (off >= R) off -= R;
      const int slot = c % M;
      const uint32_t bar = full0 + 8u * slot;
      ChunkDesc* d = desc_at(slot);
      rows(d);
      if (lane == 0) {
        d->b0 = b0;
        d->end_total = tail;
        d->off = at;
        d->kv_bytes = kvb;
        d->h0 = h0;
        d->nh = nh;
        d->tile_base = tiles;
        d->ntiles = ntiles;
        d->nrows = nrows;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(bar, sz);  // releases the descriptor
      __syncwarp();
      issue(at, bar);
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        *published = c + 1;
      }
      tiles += ntiles;
      ++c;
    };

    // Bulk copy of len bytes to ring offset off (< 2R), split in two where it
    // runs past the end of the ring.
    auto copy_to_ring = [&](uint32_t off, const uint16_t* src, uint32_t len, uint32_t bar) {
      if (off >= R) off -= R;
      const uint32_t first = off + len > R ? R - off : len;
      bulk_g2s(ring0 + off, src, first, bar, policy);
      if (first < len) bulk_g2s(ring0, src + first / 2, len - first, bar, policy);
    };

    // This CTA's rows: an equal share of the bytes (not of the rows; with
    // Poisson lengths equal row counts leave the heaviest CTA ~10 % above
    // the mean at 30720 rows, ~20 % at 3840).
    int64_t row_lo = 0, row_hi = P.batch;
    {
      const int64_t B = P.batch;
      const int64_t wt = 2 * (int64_t)__ldg(P.cu_seqlens + B) + 2 * (int64_t)G * B;
      const int64_t t0 = wt * blockIdx.x / gridDim.x;
      const int64_t t1 = wt * (blockIdx.x + 1) / gridDim.x;
      const int64_t r = weight_split(P.cu_seqlens, B, G, lane < 16 ? t0 : t1, lane);
      const int64_t r0 = __shfl_sync(kFullMask, r, 0), r1 = __shfl_sync(kFullMask, r, 16);
      if (blockIdx.x > 0) row_lo = r0;
      if (blockIdx.x + 1 < gridDim.x) row_hi = r1 > row_lo ? r1 : row_lo;
    }
    for (int64_t base = row_lo; base < row_hi && !stop; base += 32) {
      // One row per lane: length, bytes, tiles and kind (0 whole row, 1 too
      // long for a chunk: head groups, 2 invalid length).
      const int nrow = row_hi - base < 32 ? (int)(row_hi - base) : 32;
      int c0 = 0, c1 = 0;
      if (lane < nrow) {
        c0 = __ldg(P.cu_seqlens + base + lane);
        c1 = __ldg(P.cu_seqlens + base + lane + 1);
      }
      const int s_len = c1 - c0;
      int kind = 0, rt = 0;
      uint64_t rb = 0;
      if (s_len < 0 || s_len > P.max_seqlen) {
        kind = 2;
      } else {
        const int nu = heads_per_tile(s_len);
        rb = (uint64_t)(2 * s_len + G) * (D * 2) * (uint64_t)hkv;
        rt = (hkv + nu - 1) / nu;
        if (rb > P.chunk_max) kind = 1;
      }
      win[lane] = make_int4((int)(rb < 0x7fffffffu ? rb : 0x7fffffffu), s_len, kind, rt);
      __syncwarp();
      // Greedy packing of consecutive whole rows into chunks (at most
      // kChunkRows rows and chunk_max bytes each), run by every lane over the
      // window; rows of kind 1 and 2 are entries of their own. Each lane keeps
      // its row's chunk, index in it, first K/V row and first tile.
      int k = -1, pn = 0, p_rows = 0, p_tiles = 0;
      uint32_t pend = 0;
      int my_k = 0, my_j = 0, my_krow = 0, my_tstart = 0;
      for (int j = 0; j < nrow; ++j) {
        const int4 w = win[j];
        if (w.z != 0) {
          ++k;
          pn = 0;
          if (j == lane) my_k = k;
          continue;
        }
        if (pn == 0 || pn == kChunkRows || pend + (uint32_t)w.x > P.chunk_max) {
          ++k;
          pn = p_rows = p_tiles = 0;
          pend = 0;
        }
        if (j == lane) {
          my_k = k;
          my_j = pn;
          my_krow = p_rows;
          my_tstart = p_tiles;
        }
        ++pn;
        pend += (uint32_t)w.x;
        p_rows += w.y;
        p_tiles += w.w;
      }
      // The last row of each entry records it.
      const int next_k = __shfl_down_sync(kFullMask, my_k, 1);
      if (lane < nrow && (lane == nrow - 1 || next_k != my_k))
        cinfo[my_k] = make_int4(lane - my_j, my_j + 1, my_krow + (kind == 0 ? s_len : 0),
                                (my_tstart + rt) | (kind << 24));
      __syncwarp();

      for (int q = 0; q <= k && !stop; ++q) {
        const int4 ci = cinfo[q];
        const int first = ci.x;
        const int ckind = ci.w >> 24;
        const int64_t b0 = base + first;
        const int cc0 = __shfl_sync(kFullMask, c0, first);
        const int sl0 = __shfl_sync(kFullMask, s_len, first);
        if (ckind == 2) {  // chunks hold consecutive valid rows only
          if (lane == 0) report_device_error(P.err, 1u /* FMHA_ERR_INVALID_ARG */, 5u);
          continue;
        }
        if (ckind == 0) {
          const uint32_t kvb = (uint32_t)ci.z * hkv * (D * 2);
          const uint32_t qb = (uint32_t)(ci.y * hkv * G) * (D * 2);
          const int64_t ksrc = (int64_t)cc0 * hkv * D;
          const int64_t qsrc = b0 * hkv * G * D;
          emit(b0, ci.y, 0, hkv, ci.w & 0xffffff, kvb, qb,
               [&](ChunkDesc* d) {
                 if (lane < nrow && my_k == q) {
                   d->krow[my_j] = (uint16_t)my_krow;
                   d->s_len[my_j] = (uint16_t)s_len;
                   d->tstart[my_j] = (uint16_t)my_tstart;
                 }
               },
               [&](uint32_t dst, uint32_t bar) {
                 // Lanes 0, 1, 2 copy K, V and Q together.
                 if (lane < 3) {
                   const uint16_t* src = lane == 0 ? P.K + ksrc : lane == 1 ? P.V + ksrc : P.Q + qsrc;
                   const uint32_t len = lane < 2 ? kvb : qb;
                   if (len) copy_to_ring(dst + lane * kvb, src, len, bar);
                 }
               });
          continue;
        }
        // Row too long on its own: head groups with one copy per position.
        const int nu = heads_per_tile(sl0);
        const uint32_t per_head = (uint32_t)(2 * sl0 + G) * (D * 2);
        int nh_max = (int)(P.chunk_max / per_head);
        if (nh_max < 1) nh_max = 1;
        if (nh_max > hkv) nh_max = hkv;
        if (nh_max >= nu) nh_max -= nh_max % nu;  // whole tiles per group
        for (int h0 = 0; h0 < hkv && !stop; h0 += nh_max) {
          const int nh = hkv - h0 < nh_max ? hkv - h0 : nh_max;
          const uint32_t kvb = (uint32_t)sl0 * nh * (D * 2);
          const uint32_t qb = (uint32_t)(nh * G) * (D * 2);
          const uint32_t run = (uint32_t)nh * (D * 2);
          const int64_t qsrc = (b0 * hkv + h0) * G * D;
          emit(b0, 1, h0, nh, (nh + nu - 1) / nu, kvb, qb,
               [&](ChunkDesc* d) {
                 if (lane == 0) {
                   d->krow[0] = 0;
                   d->s_len[0] = (uint16_t)sl0;
                   d->tstart[0] = 0;
                 }
               },
               [&](uint32_t dst, uint32_t bar) {
                 if (lane < sl0) {
                   const int64_t ksrc = ((int64_t)(cc0 + lane) * hkv + h0) * D;
                   copy_to_ring(dst + lane * run, P.K + ksrc, run, bar);
                   copy_to_ring(dst + kvb + lane * run, P.V + ksrc, run, bar);
                 }
                 if (lane == 31) copy_to_ring(dst + 2 * kvb, P.Q + qsrc, qb, bar);
               });
        }
      }
      __syncwarp();  // the plan arrays are rewritten by the next window
    }
    if (lane == 0) {
      __threadfence_block();
      if (!stop) *total_tiles = tiles;
      else *abort_flag = 1;
      // Never leave the CTA with copies in flight into its shared memory.
      for (int j = oldest; j < c; ++j)
        mbar_wait(full0 + 8u * (j % M), (j / M) & 1, nullptr, P.err, P.wait_timeout_ns,
                  kSiteDrain);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  float* sc = reinterpret_cast<float*>(smem + P.sc_off) + cw * (G * 16);
  for (;;) {
    int t = 0;
    if (lane == 0) t = atomicAdd(next_tile, 1);
    t = __shfl_sync(kFullMask, t, 0);
    // Wait (bounded) until a published chunk holds tile t, or there is none.
    int c = -1;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      const int pub = *published;
      __threadfence_block();  // descriptors of chunks < pub are visible
      if (pub > 0) {
        const ChunkDesc* last = desc_at((pub - 1) % M);
        if (t < last->tile_base + last->ntiles) {
          c = pub - 1;
          while (desc_at(c % M)->tile_base > t) --c;  // within the last M chunks
          break;
        }
      }
      const int tot = *total_tiles;
      if ((tot >= 0 && t >= tot) || *abort_flag) break;
      if ((it & 15u) == 15u && globaltimer_ns() - t0 > P.wait_timeout_ns) {
        report_device_error(P.err, 5u /* FMHA_ERR_DEVICE_TIMEOUT */, kSiteConsumerIssued);
        *abort_flag = 1;
        break;
      }
    }
    if (c < 0) break;
    const int slot = c % M;
    if (!mbar_wait(full0 + 8u * slot, (c / M) & 1, abort_flag, P.err, P.wait_timeout_ns,
                   kSiteConsumerFull))
      break;
    const ChunkDesc* d = desc_at(slot);
    const int local = t - d->tile_base;
    int j = d->nrows - 1;
    while (j > 0 && d->tstart[j] > local) --j;
    TileRef ref;
    ref.b = d->b0 + j;
    ref.s_len = d->s_len[j];
    ref.h0 = d->h0;
    ref.nh = d->nh;
    ref.koff = d->off + (uint32_t)d->krow[j] * d->nh * (D * 2);
    ref.voff = ref.koff + d->kv_bytes;
    ref.qoff = d->off + 2 * d->kv_bytes + (uint32_t)(j * d->nh * G) * (D * 2);
    const int ntiles = d->ntiles;
    const int smax = smax_of(ref.s_len);
    const int hl0 = (local - d->tstart[j]) * (16 / smax);
    switch (smax) {
      case 1: chunk_tile<D, 1, G>(P, ref, hl0, ring0, R, sc, lane); break;
      case 2: chunk_tile<D, 2, G>(P, ref, hl0, ring0, R, sc, lane); break;
      case 4: chunk_tile<D, 4, G>(P, ref, hl0, ring0, R, sc, lane); break;
      case 8: chunk_tile<D, 8, G>(P, ref, hl0, ring0, R, sc, lane); break;
      default: chunk_tile<D, 16, G>(P, ref, hl0, ring0, R, sc, lane); break;
    }
    __syncwarp();
    if (lane == 0) {
      // The chunk's last tile resets the slot's counter and frees the chunk.
      if (atomicAdd(done + slot, 1) == ntiles - 1) {
        done[slot] = 0;
        __threadfence_block();
        mbar_arrive(empty0 + 8u * slot);
      }
    }
  }
}

#define FMHA_CAT2(a, b) a##b
#define FMHA_CAT(a, b) FMHA_CAT2(a, b)

VarlenFn FMHA_CAT(varlen_chunk_kernel_d, FMHA_HEAD_DIM)(int g) {
  constexpr int D = FMHA_HEAD_DIM;
  switch (g) {
    case 1: return decode_varlen_chunk_kernel<D, 1>;
    case 2: return decode_varlen_chunk_kernel<D, 2>;
    case 4: return decode_varlen_chunk_kernel<D, 4>;
    case 8: return decode_varlen_chunk_kernel<D, 8>;
    default: return nullptr;
  }
}

}  // namespace fmha
