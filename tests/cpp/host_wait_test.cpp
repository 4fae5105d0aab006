// CPU test of the benchmark host's deadline-bounded wait and release policy
// (fmha_b200/csrc/host_wait.hpp): an event query stub that never completes
// must end in a timeout within the deadline, and a shard whose work may
// still be in flight must release nothing (a real cudaFree would block
// behind the stuck kernels). Built and run by tests/test_host_wait.py.
#include <chrono>
#include <cstdio>
#include <string>

#include "host_wait.hpp"

namespace {
constexpr int kDone = 0, kNotReady = 600, kFault = 700;

struct CountingOps {
  int frees = 0, streams = 0, events = 0;
  void free_buffer(void*) { ++frees; }
  void destroy_stream(void*) { ++streams; }
  void destroy_event(void*) { ++events; }
};

int fails = 0;
void expect(bool ok, const char* what) {
  if (!ok) {
    std::printf("FAIL: %s\n", what);
    ++fails;
  }
}
}  // namespace

int main() {
  using fmha_host::WaitOutcome;
  auto describe = [](int c) { return std::string("code ") + std::to_string(c); };
  std::string why;

  // 1. A query that never completes: the wait gives up after the deadline.
  int polls = 0;
  const auto t0 = std::chrono::steady_clock::now();
  WaitOutcome w = fmha_host::wait_deadline([&] { ++polls; return kNotReady; }, kDone, kNotReady,
                                           describe, 0.2, &why, 100);
  const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  expect(w == WaitOutcome::kTimedOut, "stuck query times out");
  expect(dt >= 0.2 && dt < 5.0, "timeout honours the deadline");
  expect(polls > 1, "the query is polled repeatedly");
  expect(why.find("timed out") != std::string::npos, "timeout is described");

  // 2. A query that completes after a few polls.
  int n = 0;
  w = fmha_host::wait_deadline([&] { return ++n < 5 ? kNotReady : kDone; }, kDone, kNotReady,
                               describe, 5.0, &why, 10);
  expect(w == WaitOutcome::kDone && n == 5, "completion is seen");

  // 3. An error code ends the wait at once and is described.
  w = fmha_host::wait_deadline([&] { return kFault; }, kDone, kNotReady, describe, 5.0, &why);
  expect(w == WaitOutcome::kError && why == "code 700", "errors end the wait");

  // 4. Release policy.
  int dummy[8];
  fmha_host::ShardHandles h;
  for (int i = 0; i < 5; ++i) h.buffers[i] = &dummy[i];
  h.stream = &dummy[5];
  h.events[0] = &dummy[6];
  h.events[1] = &dummy[7];
  CountingOps ops;
  expect(!fmha_host::release_shard(h, /*work_in_flight=*/true, ops), "in-flight: not released");
  expect(ops.frees == 0 && ops.streams == 0 && ops.events == 0, "in-flight: nothing touched");
  expect(fmha_host::release_shard(h, /*work_in_flight=*/false, ops), "idle: released");
  expect(ops.frees == 5 && ops.streams == 1 && ops.events == 2, "idle: everything released");
  expect(fmha_host::release_shard(h, false, ops) && ops.frees == 5, "release is idempotent");

  if (fails == 0) std::printf("host_wait_test: ok\n");
  return fails == 0 ? 0 : 1;
}
