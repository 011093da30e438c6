// Bounded host wait for device work that includes collectives.
//
// A tensor-parallel step enqueues NCCL all-reduces between its kernels; if a
// peer rank dies or never reaches the same collective, those kernels wait
// forever and so would a plain cudaStreamSynchronize. bounded_wait() instead
// polls the stream and the communicator's asynchronous error, and on an
// error or when the deadline passes calls `abort` (ncclCommAbort, which ends
// the communicator's outstanding kernels) and reports why. The loop is
// header-only and takes its probes as callables so the host logic is tested
// on CPU with fakes (tests/cpp/watchdog_test.cpp).
#pragma once

namespace ifx {

enum class WaitEnd { Done, DeviceError, CommError, TimedOut };

// query():      0 when the work has finished, 1 while pending, -1 on a device error
// comm_error(): true once the communicator reports an asynchronous error
// abort():      ends the communicator (called at most once, never after Done)
// now_ms():     a monotonic clock in milliseconds
// pause():      yields between polls
template <class Query, class CommErr, class Abort, class Now, class Pause>
WaitEnd bounded_wait(Query query, CommErr comm_error, Abort abort, Now now_ms, Pause pause,
                     double timeout_ms) {
  const double t0 = now_ms();
  for (;;) {
    const int q = query();
    if (q == 0) return WaitEnd::Done;
    if (q < 0) return WaitEnd::DeviceError;
    if (comm_error()) {
      abort();
      return WaitEnd::CommError;
    }
    if (now_ms() - t0 > timeout_ms) {
      abort();
      return WaitEnd::TimedOut;
    }
    pause();
  }
}

}  // namespace ifx
