// The bounded wait of inferox_b200/csrc/watchdog.h driven by fakes: a stream
// that finishes, a device error, an asynchronous communicator error, and a
// peer that never arrives (the deadline). Prints one line per case; exits
// non-zero on the first wrong outcome. Built and run by tests/test_watchdog.py.
#include <cstdio>

#include "../../inferox_b200/csrc/watchdog.h"

using ifx::WaitEnd;

struct Fake {
  int done_after = -1;      // polls until the work finishes (-1: never)
  int dev_error_at = -1;    // poll at which the device reports an error
  int comm_error_at = -1;   // poll at which the communicator reports one
  int polls = 0, aborts = 0;
  double clock = 0.0;       // fake milliseconds, 1 per pause
};

static WaitEnd run(Fake &f, double timeout_ms) {
  return ifx::bounded_wait(
      [&]() {
        const int p = f.polls++;
        if (f.dev_error_at >= 0 && p >= f.dev_error_at) return -1;
        if (f.done_after >= 0 && p >= f.done_after) return 0;
        return 1;
      },
      [&]() { return f.comm_error_at >= 0 && f.polls > f.comm_error_at; },
      [&]() { ++f.aborts; }, [&]() { return f.clock; }, [&]() { f.clock += 1.0; }, timeout_ms);
}

static int check(const char *name, bool ok) {
  std::printf("%s %s\n", ok ? "ok  " : "FAIL", name);
  return ok ? 0 : 1;
}

int main() {
  int bad = 0;
  {
    Fake f;
    f.done_after = 5;
    bad |= check("finishes: Done, no abort", run(f, 100.0) == WaitEnd::Done && f.aborts == 0 && f.polls == 6);
  }
  {
    Fake f;
    f.done_after = 0;
    bad |= check("already finished: one poll", run(f, 0.0) == WaitEnd::Done && f.polls == 1);
  }
  {
    Fake f;
    f.dev_error_at = 3;
    bad |= check("device error: reported, no abort", run(f, 100.0) == WaitEnd::DeviceError && f.aborts == 0);
  }
  {
    Fake f;
    f.comm_error_at = 4;
    const WaitEnd e = run(f, 100.0);
    bad |= check("communicator error: abort once", e == WaitEnd::CommError && f.aborts == 1 && f.polls == 5);
  }
  {
    Fake f;  // a peer that never reaches the collective
    const WaitEnd e = run(f, 250.0);
    bad |= check("peer never arrives: deadline, abort once",
                 e == WaitEnd::TimedOut && f.aborts == 1 && f.clock > 250.0 && f.clock < 253.0);
  }
  {
    Fake f;  // finishes just before the deadline
    f.done_after = 240;
    bad |= check("finishes before the deadline", run(f, 250.0) == WaitEnd::Done && f.aborts == 0);
  }
  return bad;
}
