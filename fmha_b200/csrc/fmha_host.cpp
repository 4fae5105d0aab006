// fmha_host.cpp -- benchmark / validation host for libfmha_b200 (C ABI,
// include/fmha.h). B200 counterpart of the reference's host program
// (HGLiu1998/fmha fmha_host.cpp): same config table and argv index
// (fmha_host.cpp:477-533), same warm-up/iteration defaults (5/20,
// fmha_host.cpp:298), same printed metrics (ms/iter, iter/s, TFLOPS, us per
// head, GB/s; fmha_host.cpp:397-432) and the same post-run validation
// (fmha_host.cpp:434-445), with these differences:
//   * K/V use the [B,Hkv,S,D] layout with a fixed seqlen_kv (default 16),
//     inputs come from the library's seeded counter-based generator
//     (fmha_fill_normal_bf16) instead of unseeded U[-1,1];
//   * --gpus N splits the batch into N contiguous shards, one host thread per
//     GPU, started together on a host barrier; the aggregate bandwidth is
//     total bytes / slowest GPU's device time (no collective: shards are
//     independent and outputs stay on their GPUs);
//   * validation recomputes a deterministic sample of batch rows on the CPU
//     (fp32 softmax, the reference's arithmetic order, fmha_host.cpp:179-243)
//     with OpenMP over the host cores, checks max|o-r| <= 2e-3 or <= 1e-2|r|,
//     and reports the CPU time per row as the CPU baseline.
//
// Usage: fmha_host [config_index] [--all] [--gpus N] [--iters N] [--warmups N]
//                  [--seqlen S] [--seed S] [--variant auto|bulk|ldg]
//                  [--validate-rows N] [--json] [--varlen] [--traffic FILE]
//
// --traffic profiles/ncu_traffic.json adds the DRAM bytes ncu measured for the
// config (scaled to its batch) and the bandwidth they give.
// --varlen runs the reference's own benchmark exactly: packed K/V
// [sum S_b, Hkv, D] with cu_seqlens_kv and Poisson(4) lengths in [2, 16]
// from mt19937(42) (fmha_host.cpp:58-82), through fmha_forward_varlen.
#include <cuda_runtime.h>
#include <omp.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "fmha.h"
#include "host_wait.hpp"

namespace {

#define CUDA_CHECK(cmd)                                                                      \
  do {                                                                                       \
    cudaError_t e_ = (cmd);                                                                  \
    if (e_ != cudaSuccess) {                                                                 \
      std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__,    \
                   __LINE__);                                                                \
      std::exit(EXIT_FAILURE);                                                               \
    }                                                                                        \
  } while (0)

#define FMHA_CHECK(cmd)                                                                      \
  do {                                                                                       \
    fmha_status_t s_ = (cmd);                                                                \
    if (s_ != FMHA_OK) {                                                                     \
      std::fprintf(stderr, "fmha error %s at %s:%d\n", fmha_status_string(s_), __FILE__,    \
                   __LINE__);                                                                \
      std::exit(EXIT_FAILURE);                                                               \
    }                                                                                        \
  } while (0)

struct Config {
  int batch, num_heads_q, num_heads_kv, head_dim;
  const char* note;
};

// Index 0..4: the reference's table (fmha_host.cpp:511-517). 5: GQA 32/16.
const Config kConfigs[] = {
    {10, 16, 16, 128, "testing"},
    {30720, 16, 16, 128, "config 0: 16 heads, dim 128"},
    {30720, 16, 16, 256, "config 1: 16 heads, dim 256"},
    {30720, 32, 32, 128, "config 2: 32 heads, dim 128"},
    {30720, 32, 32, 256, "config 3: 32 heads, dim 256"},
    {30720, 32, 16, 256, "GQA: 32 query heads over 16 kv heads, dim 256"},
};
constexpr int kNumConfigs = sizeof(kConfigs) / sizeof(kConfigs[0]);

struct Options {
  int config = -1;
  int gpus = 1;
  int iters = 20;
  int warmups = 5;
  int seqlen = 16;
  uint64_t seed = 0;
  int variant = FMHA_VARIANT_AUTO;
  int validate_rows = 64;
  bool json = false;
  bool varlen = false;  // the reference's packed layout and Poisson(4) seqlens
  std::string traffic;  // measured-traffic table (profiles/ncu_traffic.json), optional
};

// ------------------------------------------------------------ host generator
// Same values as fmha_fill_normal_bf16 (splitmix64 of (seed, tensor, index),
// Irwin-Hall sum of twelve 16-bit uniforms, bf16 RNE).
uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

float f16_to_f32(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 1024), (int)e - 25);
  return s ? -v : v;
}

void gen_bf16(uint16_t* out, int64_t n, uint64_t seed, uint32_t tensor, int64_t offset) {
  const uint64_t key = mix64(seed ^ mix64(((uint64_t)tensor << 32) | 0x5bd1e995u));
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t e = (uint64_t)(offset + i);
    int64_t t = 0;
    for (int j = 0; j < 3; ++j) {
      const uint64_t h = mix64(key + e * 3u + (uint64_t)j);
      t += (int64_t)(h & 0xffffu) + (int64_t)((h >> 16) & 0xffffu) +
           (int64_t)((h >> 32) & 0xffffu) + (int64_t)(h >> 48);
    }
    out[i] = f32_to_bf16((float)(2 * t + 12 - 12 * 65536) * (1.0f / 131072.0f));
  }
}

// ------------------------------------------------------------ CPU check
// One batch row, all heads: fp32 softmax(q.k^T/sqrt(D)) v in the reference's
// operation order (fmha_host.cpp:179-243), P kept in fp32.
// K/V element (head kvh, position j, column c) is at kvh*head_stride +
// j*row_stride + c: [B,H,S,D] has (S*D, D), the packed layout (D, Hkv*D).
void cpu_row(const uint16_t* q, const uint16_t* k, const uint16_t* v, int hq, int hkv, int s,
             int d, int64_t head_stride, int64_t row_stride, float* out) {
  const int g = hq / hkv;
  for (int h = 0; h < hq; ++h) {
    const int kvh = h / g;
    const uint16_t* qh = q + (int64_t)h * d;
    const uint16_t* kh = k + (int64_t)kvh * head_stride;
    const uint16_t* vh = v + (int64_t)kvh * head_stride;
    float sc[16];
    for (int j = 0; j < s; ++j) {
      float acc = 0.f;
      for (int c = 0; c < d; ++c) acc += bf16_to_f32(qh[c]) * bf16_to_f32(kh[(int64_t)j * row_stride + c]);
      sc[j] = acc * (1.0f / std::sqrt((float)d));
    }
    float mx = -INFINITY;
    for (int j = 0; j < s; ++j) mx = std::max(mx, sc[j]);
    float sum = 0.f;
    for (int j = 0; j < s; ++j) sum += std::exp(sc[j] - mx);
    for (int j = 0; j < s; ++j) sc[j] = std::exp(sc[j] - mx) / sum;
    for (int c = 0; c < d; ++c) {
      float acc = 0.f;
      for (int j = 0; j < s; ++j) acc += sc[j] * bf16_to_f32(vh[(int64_t)j * row_stride + c]);
      out[(int64_t)h * d + c] = acc;
    }
  }
}

// ------------------------------------------------------------ per-GPU shard

// Start line for the timed loops. A shard that fails before it gets there
// drops out (drop()), so the others are not left waiting for it.
struct HostBarrier {
  std::mutex mu;
  std::condition_variable cv;
  int count = 0, gen = 0, n = 0;
  void wait() {
    std::unique_lock<std::mutex> lk(mu);
    const int g = gen;
    if (++count >= n) {
      count = 0;
      ++gen;
      cv.notify_all();
    } else {
      cv.wait(lk, [&] { return gen != g; });
    }
  }
  void drop() {
    std::unique_lock<std::mutex> lk(mu);
    --n;
    if (count >= n && count > 0) {
      count = 0;
      ++gen;
      cv.notify_all();
    }
  }
};

struct ShardResult {
  std::string error;  // empty when the shard completed
  double ms_per_iter = 0;
  int64_t rows_checked = 0;
  int64_t bad = 0;
  double max_abs = 0, max_rel = 0;
  double cpu_sec = 0;
  int device_error = 0;
};

// Shard-local error handling: record the failure and leave the shard (the
// other shards keep running and the driver reports every failed shard).
#define SHARD_CUDA(cmd)                                                                      \
  do {                                                                                       \
    cudaError_t e_ = (cmd);                                                                  \
    if (e_ != cudaSuccess) {                                                                 \
      res.error = std::string(#cmd) + ": " + cudaGetErrorString(e_);                         \
      cleanup();                                                                             \
      return;                                                                                \
    }                                                                                        \
  } while (0)
#define SHARD_FMHA(cmd)                                                                      \
  do {                                                                                       \
    fmha_status_t s_ = (cmd);                                                                \
    if (s_ != FMHA_OK) {                                                                     \
      res.error = std::string(#cmd) + ": " + fmha_status_string(s_);                         \
      cleanup();                                                                             \
      return;                                                                                \
    }                                                                                        \
  } while (0)

// Waits for an event by polling with a deadline instead of blocking forever.
// FMHA_HOST_STUCK_SHARD=g (test hook) makes shard g's query report "not
// ready" for ever, with a 2 s deadline, so the timeout path runs without any
// stuck device work.
fmha_host::WaitOutcome wait_event(cudaEvent_t e, double timeout_s, bool stub_stuck,
                                  std::string* why) {
  if (stub_stuck) timeout_s = 2.0;
  return fmha_host::wait_deadline(
      [&] { return stub_stuck ? (int)cudaErrorNotReady : (int)cudaEventQuery(e); },
      (int)cudaSuccess, (int)cudaErrorNotReady,
      [](int c) { return std::string("cudaEventQuery: ") + cudaGetErrorString((cudaError_t)c); },
      timeout_s, why);
}

struct CudaReleaseOps {
  void free_buffer(void* p) { cudaFree(p); }
  void destroy_stream(void* s) { cudaStreamDestroy(static_cast<cudaStream_t>(s)); }
  void destroy_event(void* e) { cudaEventDestroy(static_cast<cudaEvent_t>(e)); }
};

int env_shard(const char* name) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : -1;
}

int injected_failure_shard() { return env_shard("FMHA_HOST_FAIL_SHARD"); }

// cu: global cu_seqlens (varlen mode) or empty.
void run_shard(int gpu, const Config& cfg, const Options& o, int64_t row0, int64_t rows,
               const std::vector<int64_t>& cu, HostBarrier& bar, ShardResult& res) {
  const int hq = cfg.num_heads_q, hkv = cfg.num_heads_kv, d = cfg.head_dim, s = o.seqlen;
  const bool vl = o.varlen;
  const int64_t t0row = vl ? cu[row0] : row0 * s;  // first K/V row (packed) of the shard
  const int64_t nq = rows * hq * d;
  const int64_t nkv = vl ? (cu[row0 + rows] - cu[row0]) * hkv * d : rows * hkv * s * d;
  void *dQ = nullptr, *dK = nullptr, *dV = nullptr, *dO = nullptr, *dCu = nullptr;
  cudaStream_t st = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  bool started = false;    // passed the start line
  bool in_flight = false;  // a wait gave up with this shard's kernels possibly running
  auto cleanup = [&] {
    if (!started) bar.drop();
    fmha_host::ShardHandles h;
    h.buffers[0] = dQ, h.buffers[1] = dK, h.buffers[2] = dV, h.buffers[3] = dO;
    h.buffers[4] = dCu;
    h.stream = st;
    h.events[0] = e0, h.events[1] = e1;
    CudaReleaseOps ops;
    fmha_host::release_shard(h, in_flight, ops);
  };
  if (gpu == injected_failure_shard()) {  // host-side fault injection (no GPU fault)
    res.error = "injected failure (FMHA_HOST_FAIL_SHARD)";
    cleanup();
    return;
  }
  SHARD_CUDA(cudaSetDevice(gpu));
  SHARD_CUDA(cudaMalloc(&dQ, nq * 2));
  SHARD_CUDA(cudaMalloc(&dK, nkv * 2));
  SHARD_CUDA(cudaMalloc(&dV, nkv * 2));
  SHARD_CUDA(cudaMalloc(&dO, nq * 2));
  SHARD_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  fmha_stream_t fs = reinterpret_cast<fmha_stream_t>(st);
  SHARD_FMHA(fmha_fill_normal_bf16(dQ, nq, o.seed, 1, row0 * hq * d, fs));
  SHARD_FMHA(fmha_fill_normal_bf16(dK, nkv, o.seed, 2, t0row * hkv * d, fs));
  SHARD_FMHA(fmha_fill_normal_bf16(dV, nkv, o.seed, 3, t0row * hkv * d, fs));
  SHARD_CUDA(cudaMemsetAsync(dO, 0, nq * 2, st));
  if (vl) {
    std::vector<int32_t> lcu(rows + 1);
    for (int64_t r = 0; r <= rows; ++r) lcu[r] = (int32_t)(cu[row0 + r] - cu[row0]);
    SHARD_CUDA(cudaMalloc(&dCu, (rows + 1) * 4));
    SHARD_CUDA(cudaMemcpy(dCu, lcu.data(), (rows + 1) * 4, cudaMemcpyHostToDevice));
  }
  auto launch = [&] {
    if (vl) {
      SHARD_FMHA(fmha_forward_varlen(dQ, dK, dV, dO, static_cast<const int32_t*>(dCu), (int)rows,
                                     hq, hkv, 16, d, 0.0f, fs));
    } else {
      SHARD_FMHA(fmha_forward_variant(dQ, dK, dV, dO, (int)rows, hq, hkv, s, d, o.variant, fs));
    }
  };
  for (int i = 0; i < o.warmups; ++i) launch();
  SHARD_CUDA(cudaStreamSynchronize(st));
  SHARD_CUDA(cudaEventCreate(&e0));
  SHARD_CUDA(cudaEventCreate(&e1));
  bar.wait();  // every GPU starts its timed loop together
  started = true;
  SHARD_CUDA(cudaEventRecord(e0, st));
  for (int i = 0; i < o.iters; ++i) launch();
  SHARD_CUDA(cudaEventRecord(e1, st));
  const fmha_host::WaitOutcome w =
      wait_event(e1, 120.0, gpu == env_shard("FMHA_HOST_STUCK_SHARD"), &res.error);
  if (w != fmha_host::WaitOutcome::kDone) {
    in_flight = w == fmha_host::WaitOutcome::kTimedOut;
    cleanup();
    return;
  }
  float ms = 0;
  SHARD_CUDA(cudaEventElapsedTime(&ms, e0, e1));
  res.ms_per_iter = ms / o.iters;
  SHARD_FMHA(fmha_device_error(&res.device_error));

  // Validation: a deterministic sample of this shard's rows (all if few).
  std::vector<uint16_t> hO(nq);
  SHARD_CUDA(cudaMemcpy(hO.data(), dO, nq * 2, cudaMemcpyDeviceToHost));
  std::vector<int64_t> pick;
  if (o.validate_rows <= 0 || rows <= o.validate_rows) {
    for (int64_t r = 0; r < rows; ++r) pick.push_back(r);
  } else {
    for (int i = 0; i < o.validate_rows; ++i)
      pick.push_back((int64_t)((mix64((uint64_t)i + 977) % (uint64_t)rows)));
    pick.push_back(0);
    pick.push_back(rows - 1);
  }
  int64_t bad = 0;
  double max_abs = 0, max_rel = 0;
  const auto t0 = std::chrono::steady_clock::now();
#pragma omp parallel for schedule(dynamic) reduction(+ : bad) reduction(max : max_abs, max_rel)
  for (size_t i = 0; i < pick.size(); ++i) {
    const int64_t r = pick[i], gr = row0 + r;
    const int sr = vl ? (int)(cu[gr + 1] - cu[gr]) : s;
    const int64_t kv0 = vl ? cu[gr] * hkv * d : gr * hkv * s * d;  // first element of the row
    std::vector<uint16_t> q(hq * d), k((int64_t)hkv * sr * d), v((int64_t)hkv * sr * d);
    gen_bf16(q.data(), hq * d, o.seed, 1, gr * hq * d);
    gen_bf16(k.data(), (int64_t)hkv * sr * d, o.seed, 2, kv0);
    gen_bf16(v.data(), (int64_t)hkv * sr * d, o.seed, 3, kv0);
    std::vector<float> ref((int64_t)hq * d);
    if (vl) {
      cpu_row(q.data(), k.data(), v.data(), hq, hkv, sr, d, d, (int64_t)hkv * d, ref.data());
    } else {
      cpu_row(q.data(), k.data(), v.data(), hq, hkv, sr, d, (int64_t)sr * d, d, ref.data());
    }
    for (int64_t c = 0; c < (int64_t)hq * d; ++c) {
      const double got = f16_to_f32(hO[r * hq * d + c]);
      const double err = std::fabs(got - ref[c]);
      if (!(err <= 2e-3 || err <= 1e-2 * std::fabs(ref[c]))) ++bad;
      max_abs = std::max(max_abs, err);
      if (std::fabs(ref[c]) >= 0.2) max_rel = std::max(max_rel, err / std::fabs(ref[c]));
    }
  }
  res.cpu_sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  res.rows_checked = (int64_t)pick.size();
  res.bad = bad;
  res.max_abs = max_abs;
  res.max_rel = max_rel;
  cleanup();
}

// DRAM bytes per call of this config from a measured-traffic table: a JSON
// object of config name -> bytes per full-size (batch 30720) launch, as
// bench.py --traffic-from writes it (ncu dram__bytes_read.sum +
// dram__bytes_write.sum). Scaled to `batch` rows; < 0 when absent.
double measured_traffic(const std::string& path, int hq, int hkv, int s, int d, bool varlen,
                        int batch) {
  if (path.empty()) return -1.0;
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return -1.0;
  std::string txt;
  char buf[4096];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) txt.append(buf, n);
  std::fclose(f);
  char key[96];
  if (varlen && hq == hkv)
    std::snprintf(key, sizeof(key), "\"varlen_h%d_d%d\"", hq, d);
  else if (varlen)
    std::snprintf(key, sizeof(key), "\"varlen_gqa_%d_%d_d%d\"", hq, hkv, d);
  else if (hq == hkv)
    std::snprintf(key, sizeof(key), "\"h%d_d%d_s%d\"", hq, d, s);
  else
    std::snprintf(key, sizeof(key), "\"gqa_%d_%d_d%d_s%d\"", hq, hkv, d, s);
  const size_t at = txt.find(key);
  if (at == std::string::npos) return -1.0;
  const size_t colon = txt.find(':', at);
  if (colon == std::string::npos) return -1.0;
  const double full = std::strtod(txt.c_str() + colon + 1, nullptr);
  return full > 0 ? full * batch / 30720.0 : -1.0;
}

bool run_config(int idx, const Options& o) {
  const Config& cfg = kConfigs[idx];
  const int hq = cfg.num_heads_q, hkv = cfg.num_heads_kv, d = cfg.head_dim, s = o.seqlen;
  const int n = std::max(1, std::min(o.gpus, cfg.batch));
  std::vector<ShardResult> res(n);
  std::vector<int64_t> cu;
  int64_t total_rows = (int64_t)cfg.batch * s;  // sum of K/V rows per head
  if (o.varlen) {
    // The reference benchmark's lengths: Poisson(4) in [2, 16], seed 42
    // (fmha_host.cpp:58-72).
    std::vector<int32_t> sl(cfg.batch);
    FMHA_CHECK(fmha_seqlens_poisson(cfg.batch, 16, 42u, 4.0, sl.data()));
    cu.assign(cfg.batch + 1, 0);
    for (int b = 0; b < cfg.batch; ++b) cu[b + 1] = cu[b] + sl[b];
    total_rows = cu[cfg.batch];
  }
  std::vector<std::thread> th;
  HostBarrier bar;
  bar.n = n;
  for (int g = 0; g < n; ++g) {
    const int64_t r0 = (int64_t)cfg.batch * g / n, r1 = (int64_t)cfg.batch * (g + 1) / n;
    th.emplace_back(run_shard, g, std::cref(cfg), std::cref(o), r0, r1 - r0, std::cref(cu),
                    std::ref(bar), std::ref(res[g]));
  }
  for (auto& t : th) t.join();

  double ms = 0, cpu_sec = 0, max_abs = 0, max_rel = 0;
  int64_t bad = 0, checked = 0;
  int dev_err = 0;
  std::string failed;  // "gpu: reason; ..." for every shard that did not complete
  double done_frac = 0.0;  // share of the batch whose shard completed
  for (int g = 0; g < n; ++g) {
    if (res[g].error.empty()) {
      done_frac += (double)((int64_t)cfg.batch * (g + 1) / n - (int64_t)cfg.batch * g / n) / cfg.batch;
      continue;
    }
    failed += (failed.empty() ? "" : "; ") + std::to_string(g) + ": " + res[g].error;
    std::fprintf(stderr, "shard on GPU %d failed: %s\n", g, res[g].error.c_str());
  }
  for (auto& r : res) {
    if (!r.error.empty()) continue;
    ms = std::max(ms, r.ms_per_iter);
    bad += r.bad;
    checked += r.rows_checked;
    cpu_sec += r.cpu_sec;
    max_abs = std::max(max_abs, r.max_abs);
    max_rel = std::max(max_rel, r.max_rel);
    dev_err |= r.device_error;
  }
  const double b = cfg.batch;
  // Byte and flop formulas of fmha_host.cpp:413-414,428-431.
  const double T = (double)total_rows;
  // Bytes and flops of the completed shards (all of them when none failed).
  const double bytes = (2.0 * b * hq * d + 4.0 * T * hkv * d + 2.0 * b * hq * d) * done_frac;
  const double flops = 4.0 * hq * T * d * done_frac;
  const double gbs = ms > 0 ? bytes / (ms * 1e-3) / 1e9 : 0.0;
  const double cpu_ms_per_row = checked ? cpu_sec * 1e3 / checked * n : 0;  // per-thread-set
  const int threads = omp_get_max_threads();
  const bool ok = bad == 0 && dev_err == 0 && failed.empty();
  const bool any = ms > 0;  // at least one shard completed
  const double traffic = measured_traffic(o.traffic, hq, hkv, s, d, o.varlen, cfg.batch);
  const double ncu_gbs = traffic > 0 && ms > 0 ? traffic * done_frac / (ms * 1e-3) / 1e9 : -1.0;
  if (o.json) {
    std::printf(
        "{\"config\": %d, \"note\": \"%s\", \"batch\": %d, \"num_heads_q\": %d, "
        "\"num_heads_kv\": %d, \"seqlen_kv\": %d, \"head_dim\": %d, \"gpus\": %d, "
        "\"us_per_call\": %.3f, \"gbs\": %.1f, \"tflops\": %.3f, \"rows_checked\": %lld, "
        "\"bad\": %lld, \"max_abs_err\": %.3e, \"max_rel_err\": %.3e, \"cpu_ms_per_row\": %.4f, "
        "\"cpu_threads\": %d, \"device_error\": %d, \"varlen\": %s, \"failed_shards\": \"%s\", "
        "\"ncu_dram_bytes\": %.0f, \"ncu_gbs\": %.1f, \"passed\": %s}\n",
        idx, cfg.note, cfg.batch, hq, hkv, o.varlen ? -1 : s, d, n, ms * 1e3, gbs,
        any ? flops / (ms * 1e-3) / 1e12 : 0.0,
        (long long)checked, (long long)bad, max_abs, max_rel, cpu_ms_per_row, threads, dev_err,
        o.varlen ? "true" : "false", failed.c_str(), traffic, ncu_gbs, ok ? "true" : "false");
  } else {
    std::printf("\n=== Configuration %d (%s) ===\n", idx, cfg.note);
    if (o.varlen) {
      std::printf("  Batch %d, heads Q %d, heads KV %d (%s), seqlen_q 1, seqlen_kv Poisson(4) in "
                  "[2,16], avg %.3f, head_dim %d\n",
                  cfg.batch, hq, hkv, hq == hkv ? "MHA" : "GQA", T / b, d);
      std::printf("  Layout Q/O [B,H,1,D], K/V packed [sum S,Hkv,D] + cu_seqlens_kv\n");
    } else {
      std::printf("  Batch %d, heads Q %d, heads KV %d (%s), seqlen_q 1, seqlen_kv %d, head_dim %d\n",
                  cfg.batch, hq, hkv, hq == hkv ? "MHA" : "GQA", s, d);
      std::printf("  Layout Q/O [B,H,1,D], K/V [B,Hkv,S,D]; bf16 in, fp32 softmax, fp16 out\n");
    }
    std::printf("  GPUs %d (batch shards of ~%d rows, no collective)\n", n, cfg.batch / n);
    std::printf("Average time:  %.4f ms per iteration (slowest GPU)\n", ms);
    std::printf("Throughput:    %.1f iter/s\n", 1000.0 / ms);
    std::printf("Performance:   %.3f TFLOPS\n", flops / (ms * 1e-3) / 1e12);
    std::printf("Per-head latency: %.6f us\n", ms * 1e3 / (b * hq));
    std::printf("Memory bandwidth: %.1f GB/s (algorithmic bytes)\n", gbs);
    if (ncu_gbs > 0)
      std::printf("Memory bandwidth: %.1f GB/s (DRAM bytes measured by ncu, %s)\n", ncu_gbs,
                  o.traffic.c_str());
    std::printf("Validation: %lld rows on the CPU (%d OpenMP threads, %.3f ms/row): %s, "
                "max abs err %.3e, max rel err %.3e\n",
                (long long)checked, threads, cpu_ms_per_row, ok ? "passed" : "FAILED", max_abs,
                max_rel);
  }
  return ok;
}

void usage() {
  std::fprintf(stderr,
               "usage: fmha_host [config_index 0..%d] [--all] [--gpus N] [--iters N] "
               "[--warmups N] [--seqlen 1..16] [--seed S] [--variant auto|bulk|ldg] "
               "[--validate-rows N] [--json] [--varlen] [--traffic ncu_traffic.json]\n",
               kNumConfigs - 1);
}

}  // namespace

int main(int argc, char** argv) {
  Options o;
  bool all = false;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&](const char* what) -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "missing value for %s\n", what);
        std::exit(EXIT_FAILURE);
      }
      return argv[++i];
    };
    if (a == "--all") all = true;
    else if (a == "--gpus") o.gpus = std::atoi(next("--gpus"));
    else if (a == "--iters") o.iters = std::atoi(next("--iters"));
    else if (a == "--warmups") o.warmups = std::atoi(next("--warmups"));
    else if (a == "--seqlen") o.seqlen = std::atoi(next("--seqlen"));
    else if (a == "--seed") o.seed = std::strtoull(next("--seed"), nullptr, 10);
    else if (a == "--validate-rows") o.validate_rows = std::atoi(next("--validate-rows"));
    else if (a == "--json") o.json = true;
    else if (a == "--varlen") o.varlen = true;
    else if (a == "--traffic") o.traffic = next("--traffic");
    else if (a == "--variant") {
      std::string v = next("--variant");
      o.variant = v == "bulk" ? FMHA_VARIANT_BULK : v == "ldg" ? FMHA_VARIANT_LDG
                                                                : FMHA_VARIANT_AUTO;
    } else if (a == "-h" || a == "--help") {
      usage();
      return 0;
    } else if (!a.empty() && a[0] != '-') {
      o.config = std::atoi(a.c_str());
      if (o.config < 0 || o.config >= kNumConfigs) {
        std::fprintf(stderr, "Error: config_index must be 0-%d\n", kNumConfigs - 1);
        return EXIT_FAILURE;
      }
    } else {
      usage();
      return EXIT_FAILURE;
    }
  }
  if (o.seqlen < 1 || o.seqlen > 16 || o.iters < 1 || o.warmups < 0 || o.gpus < 1) {
    usage();
    return EXIT_FAILURE;
  }
  int ndev = 0;
  CUDA_CHECK(cudaGetDeviceCount(&ndev));
  if (ndev == 0) {
    std::fprintf(stderr, "Error: no CUDA devices found\n");
    return EXIT_FAILURE;
  }
  if (o.gpus > ndev) {
    std::fprintf(stderr, "Error: --gpus %d but only %d devices\n", o.gpus, ndev);
    return EXIT_FAILURE;
  }
  cudaDeviceProp prop;
  CUDA_CHECK(cudaGetDeviceProperties(&prop, 0));
  if (!o.json) {
    std::printf("Flash decode attention (fmha_b200) - CUDA benchmark\n");
    std::printf("Using: %s (sm_%d%d, %d SMs, %.1f GB), %s\n", prop.name, prop.major, prop.minor,
                prop.multiProcessorCount, prop.totalGlobalMem / 1e9, fmha_version());
  }
  bool ok = true;
  if (o.config >= 0 && !all) {
    ok = run_config(o.config, o);
  } else {
    for (int i = 0; i < kNumConfigs; ++i) ok = run_config(i, o) && ok;
  }
  if (!o.json) std::printf("\n%s\n", ok ? "Benchmark completed successfully!" : "FAILED");
  return ok ? EXIT_SUCCESS : EXIT_FAILURE;
}
