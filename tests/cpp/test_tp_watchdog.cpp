// Unit test of the tensor-parallel host watchdog (csrc/tp_watchdog.h) with fake operations:
// a step that completes, a stream that fails, a communicator that reports an asynchronous
// error, and a step that never completes (the deadline passes). Each case checks the result
// and whether the communicator was aborted. Prints "ok" and exits 0 when every case passes.
#include <cstdio>

#include "tp_watchdog.h"

namespace {

struct Fake {
  int done_after;    // polls until the stream reports completion (-1: never)
  int fail_after;    // polls until the stream reports an error (-1: never)
  int comm_after;    // polls until the communicator reports an error (-1: never)
  int polls = 0;
  double clock = 0;  // ms, advanced by pause()
  int aborts = 0;
};

int stream_state(void* u) {
  Fake* f = static_cast<Fake*>(u);
  ++f->polls;
  if (f->fail_after >= 0 && f->polls > f->fail_after) return -1;
  if (f->done_after >= 0 && f->polls > f->done_after) return 1;
  return 0;
}
int comm_failed(void* u) {
  Fake* f = static_cast<Fake*>(u);
  return f->comm_after >= 0 && f->polls > f->comm_after;
}
void abort_comm(void* u) { ++static_cast<Fake*>(u)->aborts; }
double now_ms(void* u) { return static_cast<Fake*>(u)->clock; }
void pause(void* u) { static_cast<Fake*>(u)->clock += 1.0; }

int run(Fake& f, double timeout_ms) {
  rrr::WatchOps o{&f, stream_state, comm_failed, abort_comm, now_ms, pause};
  return rrr::tp_watch(o, timeout_ms);
}

}  // namespace

int main() {
  int bad = 0;
  auto check = [&](bool ok, const char* what) {
    if (!ok) {
      std::printf("FAIL %s\n", what);
      ++bad;
    }
  };
  {
    Fake f{5, -1, -1};
    check(run(f, 100) == rrr::kWatchDone && f.aborts == 0, "completes before the deadline");
  }
  {
    Fake f{-1, 3, -1};
    check(run(f, 100) == rrr::kWatchStreamError && f.aborts == 1, "stream error aborts");
  }
  {
    Fake f{-1, -1, 7};
    check(run(f, 100) == rrr::kWatchCommError && f.aborts == 1 && f.clock < 100,
          "communicator error aborts before the deadline");
  }
  {
    Fake f{-1, -1, -1};
    check(run(f, 50) == rrr::kWatchTimeout && f.aborts == 1 && f.clock >= 50 && f.clock <= 52,
          "a step that never completes times out at the deadline");
  }
  {
    Fake f{0, -1, 0};  // completion wins over an error reported at the same poll
    check(run(f, 10) == rrr::kWatchDone && f.aborts == 0, "completion is checked first");
  }
  if (bad) return 1;
  std::printf("ok\n");
  return 0;
}
