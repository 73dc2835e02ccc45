// CPU test of the library's host-only decisions (scunet-rs_b200/csrc/host_logic.h),
// driven with fakes: admission before allocation, failing open when free memory
// cannot be read, and the band watchdog's outcomes (done, stream error, a peer's
// failure, the deadline). Built and run by tests/test_native_cpu.py.
#include <cstdio>
#include <cstdlib>

#include "host_logic.h"

using namespace scb;

static int failures = 0;
#define CHECK(cond)                                                  \
  do {                                                               \
    if (!(cond)) {                                                   \
      std::fprintf(stderr, "FAILED line %d: %s\n", __LINE__, #cond); \
      ++failures;                                                    \
    }                                                                \
  } while (0)

int main() {
  // admission (src/memguard.rs:262-285): refuse before allocating, fail open
  CHECK(admit_arena(10, true, 11) == Admit::ok);
  CHECK(admit_arena(11, true, 11) == Admit::ok);
  CHECK(admit_arena(12, true, 11) == Admit::refuse);
  CHECK(admit_arena(size_t(1) << 40, false, 0) == Admit::unknown_free);  // query failed: let cudaMalloc decide
  const std::string m = admit_message(2, 1088, 1920, size_t(3) << 30, size_t(1) << 30);
  CHECK(m.find("needs 3.00 GiB") != std::string::npos && m.find("1.00 GiB free") != std::string::npos);

  // the watchdog, with a fake clock that advances 1 ms per nap
  double clock = 0;
  auto now = [&]() { return clock; };
  auto nap = [&]() { clock += 0.001; };
  int polls = 0;
  auto healthy = []() { return 0; };

  // done at once, even with a zero timeout
  CHECK(watch_until([]() { return 0; }, healthy, now, nap, 0.0) == Watch::done);
  // done after 50 polls
  polls = 0;
  CHECK(watch_until([&]() { return ++polls >= 50 ? 0 : 1; }, healthy, now, nap, 1.0) == Watch::done);
  CHECK(polls == 50);
  // the stream's own error
  CHECK(watch_until([]() { return -1; }, healthy, now, nap, 1.0) == Watch::stream_error);
  // a peer fails after 10 polls while the stream is still busy
  polls = 0;
  CHECK(watch_until([]() { return 1; }, [&]() { return ++polls >= 10 ? 1 : 0; }, now, nap, 1.0) ==
        Watch::peer_error);
  // nothing ever completes: the deadline (100 ms of fake time) ends the wait
  clock = 0;
  polls = 0;
  CHECK(watch_until([&]() { ++polls; return 1; }, healthy, now, nap, 0.1) == Watch::timeout);
  CHECK(clock >= 0.1 && clock < 0.11 && polls > 90);

  if (failures) return 1;
  std::printf("host logic ok\n");
  return 0;
}
