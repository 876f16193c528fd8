// Per-kernel timing of the library's launches (fpa_profile / fpa_profile_report in include/fpa.h).
#include <atomic>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "fpa_internal.h"

namespace fpa {
namespace {

struct Mark {
  const char* name;  // kernel launched after this mark; nullptr closes the call
  cudaEvent_t ev;
};

std::atomic<int> g_on{0};
std::mutex g_mu;
std::vector<Mark> g_marks;
std::vector<cudaEvent_t> g_pool;

}  // namespace

bool prof_on() { return g_on.load(std::memory_order_relaxed) != 0; }

void prof_mark(cudaStream_t s, const char* name) {
  if (!g_on.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lock(g_mu);
  cudaEvent_t ev;
  if (!g_pool.empty()) {
    ev = g_pool.back();
    g_pool.pop_back();
  } else if (cudaEventCreate(&ev) != cudaSuccess) {
    return;
  }
  if (cudaEventRecord(ev, s) != cudaSuccess) {
    g_pool.push_back(ev);
    return;
  }
  g_marks.push_back(Mark{name, ev});
}

}  // namespace fpa

extern "C" FPA_API int fpa_profile(int enable) { return fpa::g_on.exchange(enable ? 1 : 0); }

extern "C" FPA_API int fpa_profile_report(char* buf, size_t len) {
  using namespace fpa;
  std::lock_guard<std::mutex> lock(g_mu);
  std::map<std::string, std::pair<int, double>> acc;
  int rc = 0;
  for (size_t i = 0; i + 1 < g_marks.size(); ++i) {
    if (!g_marks[i].name) continue;
    float ms = 0.f;
    if (cudaEventSynchronize(g_marks[i + 1].ev) != cudaSuccess ||
        cudaEventElapsedTime(&ms, g_marks[i].ev, g_marks[i + 1].ev) != cudaSuccess) {
      rc = -1;
      break;
    }
    auto& a = acc[g_marks[i].name];
    a.first += 1;
    a.second += ms;
  }
  for (auto& m : g_marks) g_pool.push_back(m.ev);
  g_marks.clear();
  if (rc < 0) return rc;
  std::string out;
  char line[256];
  for (auto& kv : acc) {
    snprintf(line, sizeof line, "%s %d %.6f\n", kv.first.c_str(), kv.second.first, kv.second.second);
    out += line;
  }
  if (buf && len) {
    size_t n = out.size() < len - 1 ? out.size() : len - 1;
    out.copy(buf, n);
    buf[n] = 0;
  }
  return int(acc.size());
}
