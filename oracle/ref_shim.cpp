/*
 * ref_shim.cpp -- C entry points around the reference's OWN CPU code.
 *
 * TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile into
 * oracle/_ref/libfmha_ref.so by compiling the reference's host file
 * (fmha_host.cpp of HGLiu1998/fmha, included from where it lies, path given by
 * -DFMHA_REF_HOST_CPP) against the stub headers in oracle/ref_stub/. The
 * reference's main() is renamed so it is never linked as an entry point.
 *
 * What is exported:
 *   fmha_ref_do_validation  -- runs the reference's do_validation()
 *                              (fmha_host.cpp:158-284) on caller data, in the
 *                              reference's packed layout, writing its ref_O;
 *                              optionally over several threads, each calling
 *                              do_validation() on a contiguous batch slice.
 *   fmha_ref_generate_seqlens -- FMHAConfig::generate_seqlens_kv()
 *                              (fmha_host.cpp:58-72), Poisson(4) in [2, max].
 * The reference prints diagnostics to stdout in do_validation(); the shim can
 * send fd 1 to /dev/null for the duration so callers keep a clean stdout.
 */
#define main fmha_reference_main_unused
#include FMHA_REF_HOST_CPP
#undef main

#include <fcntl.h>
#include <unistd.h>

#include <cstdint>
#include <cstdio>
#include <thread>
#include <vector>

namespace {

struct StdoutSilencer {
  int saved = -1;
  explicit StdoutSilencer(bool on) {
    if (!on) return;
    std::cout.flush();
    std::fflush(stdout);
    saved = dup(1);
    int devnull = open("/dev/null", O_WRONLY);
    if (devnull >= 0) {
      dup2(devnull, 1);
      close(devnull);
    }
  }
  ~StdoutSilencer() {
    if (saved < 0) return;
    std::cout.flush();
    std::fflush(stdout);
    dup2(saved, 1);
    close(saved);
  }
};

}  // namespace

extern "C" {

/* Q [B,Hq,1,D] bf16; K,V packed [sum S_b, Hkv, D] bf16 with per-row lengths
 * seqlens[B] (each in [1,16]); ref_O [B,Hq,1,D] fp16 is written by the
 * reference; h_O is the output the reference compares against (its own
 * tolerance, fmha_host.cpp:260). Returns 1 when every slice validated. */
int fmha_ref_do_validation(const uint16_t* Q, const uint16_t* K,
                           const uint16_t* V, const int32_t* seqlens,
                           int batch, int num_heads_q, int num_heads_kv,
                           int head_dim, uint16_t* ref_O, const uint16_t* h_O,
                           int threads, int quiet) {
  if (threads < 1) threads = 1;
  if (threads > batch) threads = batch > 0 ? batch : 1;
  std::vector<int64_t> cu(batch + 1, 0);
  for (int b = 0; b < batch; ++b) cu[b + 1] = cu[b] + seqlens[b];
  std::vector<int> ok(threads, 1);
  StdoutSilencer silence(quiet != 0);
  auto run_slice = [&](int t) {
    const int b0 = (int)((int64_t)batch * t / threads);
    const int b1 = (int)((int64_t)batch * (t + 1) / threads);
    if (b1 <= b0) return;
    FMHAConfig cfg(b1 - b0, num_heads_q, num_heads_kv, 1, 16, head_dim, head_dim);
    std::vector<int> sl(seqlens + b0, seqlens + b1);
    std::vector<int> csl = cfg.compute_cu_seqlens_kv(sl);
    const int64_t qoff = (int64_t)b0 * num_heads_q * head_dim;
    const int64_t kvoff = cu[b0] * num_heads_kv * head_dim;
    ok[t] = do_validation(
        cfg, sl, csl,
        reinterpret_cast<bhalf_t*>(const_cast<uint16_t*>(Q + qoff)),
        reinterpret_cast<bhalf_t*>(const_cast<uint16_t*>(K + kvoff)),
        reinterpret_cast<bhalf_t*>(const_cast<uint16_t*>(V + kvoff)),
        reinterpret_cast<half_t*>(ref_O + qoff),
        reinterpret_cast<half_t*>(const_cast<uint16_t*>(h_O + qoff)));
  };
  if (threads == 1) {
    run_slice(0);
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) pool.emplace_back(run_slice, t);
    for (auto& th : pool) th.join();
  }
  int all = 1;
  for (int v : ok) all &= v;
  return all;
}

/* FMHAConfig::generate_seqlens_kv(): mt19937(42), Poisson(4) rejected into
 * [2, max_seqlen_kv]. */
void fmha_ref_generate_seqlens(int batch, int max_seqlen_kv, int32_t* out) {
  FMHAConfig cfg(batch, 1, 1, 1, max_seqlen_kv, 128, 128);
  std::vector<int> s = cfg.generate_seqlens_kv();
  for (int b = 0; b < batch; ++b) out[b] = s[b];
}

int fmha_ref_hardware_threads(void) {
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}

}  // extern "C"
