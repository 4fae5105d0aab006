// host_wait.hpp -- deadline-bounded waits for a shard's device work, and the
// release policy that goes with them, for the C++ benchmark host.
//
// CUDA-free on purpose: the query and the release operations are passed in,
// so the policy compiles and is tested on a machine without a GPU
// (tests/cpp/host_wait_test.cpp stubs an event query that never completes).
//
// Why the policy matters: when a wait gives up, the shard's kernels may still
// be running. cudaFree and cudaStreamDestroy synchronise with that work, so a
// "cleanup" at that point would block the shard thread until the stuck
// kernels end, and the timeout would bound nothing. A shard whose work is
// still in flight therefore abandons its device buffers, stream and events
// (they are reclaimed when the process exits) and returns at once.
#ifndef FMHA_B200_HOST_WAIT_HPP
#define FMHA_B200_HOST_WAIT_HPP

#include <chrono>
#include <string>
#include <thread>

namespace fmha_host {

enum class WaitOutcome { kDone, kError, kTimedOut };

// Polls `query()` until it returns `done`, returns something other than
// `not_ready` (an error, described by `describe(code)`), or `timeout_s`
// seconds pass. Sleeps `poll_us` between polls.
template <class Query, class Describe>
WaitOutcome wait_deadline(Query query, int done, int not_ready, Describe describe,
                          double timeout_s, std::string* why, int poll_us = 200) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const int q = query();
    if (q == done) return WaitOutcome::kDone;
    if (q != not_ready) {
      *why = describe(q);
      return WaitOutcome::kError;
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
      *why = "timed out waiting for the shard's kernels (device buffers abandoned, not freed)";
      return WaitOutcome::kTimedOut;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(poll_us));
  }
}

// Device resources of one shard. `Ops` supplies free_buffer(void*),
// destroy_stream(void*) and destroy_event(void*).
struct ShardHandles {
  void* buffers[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  void* stream = nullptr;
  void* events[2] = {nullptr, nullptr};
};

// Releases the shard's resources, unless its kernels may still be running
// (`work_in_flight`): then nothing is touched, so the calling thread never
// blocks behind stuck device work. Returns true when it released them.
template <class Ops>
bool release_shard(ShardHandles& h, bool work_in_flight, Ops& ops) {
  if (work_in_flight) return false;
  for (void*& e : h.events)
    if (e) ops.destroy_event(e), e = nullptr;
  if (h.stream) ops.destroy_stream(h.stream), h.stream = nullptr;
  for (void*& b : h.buffers)
    if (b) ops.free_buffer(b), b = nullptr;
  return true;
}

}  // namespace fmha_host

#endif  // FMHA_B200_HOST_WAIT_HPP
