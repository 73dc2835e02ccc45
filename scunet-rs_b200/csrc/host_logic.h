// Host-only decisions of the library, kept free of CUDA and NCCL types so that a CPU
// test can drive them with fakes (tests/cpu/host_logic_test.cpp):
//
//  * admission: refuse a scratch arena that would not fit in free device memory,
//    BEFORE allocating, and fail open when the free figure cannot be read - the
//    contract of `memguard::check_cuda` (scunet-rs src/memguard.rs:262-285);
//  * the band watchdog: wait for a banded forward whose NCCL halo exchange may never
//    complete (a peer rank that died), polling the stream and the communicator's
//    asynchronous error until a deadline, so the caller gets an error instead of a
//    hang.
#pragma once
#include <cstddef>
#include <cstdio>
#include <string>

namespace scb {

enum class Admit { ok, refuse, unknown_free };

// `query_ok` false: the free-memory query failed. The reference lets the allocation
// decide then (fail open); so does this library.
inline Admit admit_arena(size_t need, bool query_ok, size_t free_bytes) {
  if (!query_ok) return Admit::unknown_free;
  return need > free_bytes ? Admit::refuse : Admit::ok;
}

inline std::string admit_message(int n, int hp, int wp, size_t need, size_t free_bytes) {
  char buf[256];
  snprintf(buf, sizeof buf, "%d x %dx%d needs %.2f GiB of device scratch, %.2f GiB free", n, hp, wp,
           need / 1073741824.0, free_bytes / 1073741824.0);
  return buf;
}

enum class Watch { done, stream_error, peer_error, timeout };

// Poll until the work is done, a poll reports an error, or `timeout_s` passes.
//   query()     -> 0 done, 1 still running, -1 failed (the stream's own error)
//   async_err() -> 0 healthy, non-zero: the communicator saw a failure
//   now()       -> seconds (monotonic)
//   nap()       -> yield between polls
// The deadline is checked after each poll, so a call whose work is already done
// returns `done` even with a zero timeout.
template <class Query, class AsyncErr, class Now, class Nap>
Watch watch_until(Query query, AsyncErr async_err, Now now, Nap nap, double timeout_s) {
  const double t0 = now();
  for (;;) {
    const int q = query();
    if (q == 0) return Watch::done;
    if (q < 0) return Watch::stream_error;
    if (async_err() != 0) return Watch::peer_error;
    if (now() - t0 > timeout_s) return Watch::timeout;
    nap();
  }
}

}  // namespace scb
