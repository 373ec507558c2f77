// tp_watchdog.h — host-side failure detection of a tensor-parallel step: wait for the
// step's stream with a deadline, polling the communicator's asynchronous error, and abort
// the communicator when the step fails or the deadline passes, so that no rank blocks
// forever on a peer that died, stalled or skipped a collective. The reference has no
// counterpart (one GPU, fence waits without a limit: src/gpu/engine.rs:312,369).
//
// Plain C++ (no CUDA): the operations are passed in, so the loop is unit-tested on the host
// with fakes (tests/cpp/test_tp_watchdog.cpp) and driven by rrr_tp_wait with the CUDA
// stream query and NCCL's ncclCommGetAsyncError / ncclCommAbort.
#pragma once

namespace rrr {

struct WatchOps {
  void* user;
  int (*stream_state)(void* user);  // 1: the step's work completed, 0: still running, -1: failed
  int (*comm_failed)(void* user);   // nonzero: the communicator reports an asynchronous error
  void (*abort_comm)(void* user);   // aborts the communicator (its pending work ends)
  double (*now_ms)(void* user);     // a monotonic clock
  void (*pause)(void* user);        // a short sleep between polls
};

enum WatchResult : int {
  kWatchDone = 0,         // the step completed
  kWatchStreamError = 1,  // the stream reported an error (the communicator was aborted)
  kWatchCommError = 2,    // the communicator reported an error (and was aborted)
  kWatchTimeout = 3,      // the deadline passed (the communicator was aborted)
};

// Polls until the step completes, fails or `timeout_ms` passes. Completion is checked
// before the deadline, so a step that finished exactly at the deadline counts as done.
inline int tp_watch(const WatchOps& o, double timeout_ms) {
  const double t0 = o.now_ms(o.user);
  for (;;) {
    const int st = o.stream_state(o.user);
    if (st > 0) return kWatchDone;
    if (st < 0) {
      if (o.abort_comm) o.abort_comm(o.user);
      return kWatchStreamError;
    }
    if (o.comm_failed && o.comm_failed(o.user)) {
      if (o.abort_comm) o.abort_comm(o.user);
      return kWatchCommError;
    }
    if (o.now_ms(o.user) - t0 > timeout_ms) {
      if (o.abort_comm) o.abort_comm(o.user);
      return kWatchTimeout;
    }
    o.pause(o.user);
  }
}

}  // namespace rrr
