// Optional per-launch timing: when enabled on the calling thread, every
// kernel launch of this library is bracketed by two CUDA events recorded on
// the launch stream, so a benchmark can read each kernel's device duration
// live (fpb_timing_collect). Disabled by default; costs nothing then.
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "kernels.h"

namespace fpb {

namespace {
struct Rec {
  const char* name;
  cudaEvent_t a;
  cudaEvent_t b;
};
struct TimingState {
  bool enabled = false;
  std::vector<Rec> recs;
  size_t used = 0;
};
thread_local TimingState g_timing;
}  // namespace

int timing_begin(cudaStream_t s) {
  TimingState& t = g_timing;
  if (!t.enabled) return -1;
  if (t.used == t.recs.size()) {
    Rec r{nullptr, nullptr, nullptr};
    if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return -1;
    t.recs.push_back(r);
  }
  const int idx = static_cast<int>(t.used++);
  cudaEventRecord(t.recs[idx].a, s);
  return idx;
}

void timing_end(int idx, cudaStream_t s, const char* name) {
  if (idx < 0) return;
  TimingState& t = g_timing;
  t.recs[idx].name = name;
  cudaEventRecord(t.recs[idx].b, s);
}

}  // namespace fpb

using namespace fpb;

// Enable (1) or disable (0) launch timing on the calling thread; enabling
// clears previously recorded launches.
extern "C" int fpb_timing_enable(int on) {
  g_timing.enabled = on != 0;
  if (on) g_timing.used = 0;
  return kOk;
}

// Synchronise the recorded events and write a JSON object
// {"<kernel>": {"launches": L, "total_ms": T}, ...} into `out`.
// Returns kErrArg when the buffer is too small.
extern "C" int fpb_timing_collect(char* out, size_t cap) {
  if (!out || cap == 0) return kErrArg;
  std::map<std::string, std::pair<long, double>> agg;
  for (size_t i = 0; i < g_timing.used; ++i) {
    Rec& r = g_timing.recs[i];
    if (cudaEventSynchronize(r.b) != cudaSuccess) return kErrCuda;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) return kErrCuda;
    auto& e = agg[r.name ? r.name : "?"];
    e.first += 1;
    e.second += ms;
  }
  std::string js = "{";
  bool first = true;
  for (auto& kv : agg) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "%s\"%s\": {\"launches\": %ld, \"total_ms\": %.6f}",
                  first ? "" : ", ", kv.first.c_str(), kv.second.first, kv.second.second);
    js += buf;
    first = false;
  }
  js += "}";
  if (js.size() + 1 > cap) return kErrArg;
  std::memcpy(out, js.c_str(), js.size() + 1);
  return kOk;
}
