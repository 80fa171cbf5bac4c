// pf_prof.cu -- see pf_prof.h.
#include <atomic>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "pf_common.cuh"
#include "pf_prof.h"

namespace pf {
namespace prof {

static std::atomic<long long> g_launches{0};
static std::atomic<int> g_enabled{0};

struct Rec {
  const char* name;
  cudaEvent_t a, b;
  double work;
  char unit;
};
static std::mutex g_mu;
static std::vector<Rec> g_recs;
static std::vector<cudaEvent_t> g_pool;
static thread_local int t_open = -1;

static cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}

void on_launch_begin(cudaStream_t st, const char* name, double work, char unit) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!g_enabled.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_mu);
  Rec r{name, take_event(), take_event(), work, unit};
  cudaEventRecord(r.a, st);
  g_recs.push_back(r);
  t_open = (int)g_recs.size() - 1;
}

void on_launch_end(cudaStream_t st) {
  if (t_open < 0) return;
  std::lock_guard<std::mutex> lk(g_mu);
  if (t_open < (int)g_recs.size()) cudaEventRecord(g_recs[t_open].b, st);
  t_open = -1;
}

}  // namespace prof
}  // namespace pf

using namespace pf;

extern "C" PF_API int pf_profile_enable(int on) {
  prof::g_enabled.store(on ? 1 : 0);
  return PF_OK;
}

extern "C" PF_API long long pf_launch_count(void) { return prof::g_launches.load(); }

extern "C" PF_API int pf_profile_report(char* buf, size_t len) {
  using namespace prof;
  std::lock_guard<std::mutex> lk(g_mu);
  struct Agg {
    long long launches = 0;
    double ms = 0.0, work = 0.0;
    char unit = 0;
  };
  std::map<std::string, Agg> agg;
  for (auto& r : g_recs) {
    cudaError_t e = cudaEventSynchronize(r.b);
    if (e != cudaSuccess) return fail(PF_ECUDA, "profile event sync failed: %s", cudaGetErrorString(e));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    auto& v = agg[r.name];
    v.launches += 1;
    v.ms += ms;
    v.work += r.work;
    if (r.unit) v.unit = r.unit;
    g_pool.push_back(r.a);
    g_pool.push_back(r.b);
  }
  g_recs.clear();
  std::string out = "{";
  bool first = true;
  for (auto& kv : agg) {
    char tmp[320];
    const char* unit = kv.second.unit == 'f' ? "flop" : kv.second.unit == 'b' ? "byte" : "";
    snprintf(tmp, sizeof(tmp), "%s\"%s\": [%lld, %.6f, %.6e, \"%s\"]", first ? "" : ", ", kv.first.c_str(),
             kv.second.launches, kv.second.ms, kv.second.work, unit);
    out += tmp;
    first = false;
  }
  out += "}";
  if (buf && len) {
    snprintf(buf, len, "%s", out.c_str());
    if (out.size() + 1 > len) return fail(PF_EINVAL_ARG, "profile report buffer too small (%zu)", out.size() + 1);
  }
  return PF_OK;
}
