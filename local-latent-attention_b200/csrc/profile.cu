#include <mutex>
#include <vector>

#include "llattn.h"
#include "profile.cuh"

namespace llattn {
namespace prof {
namespace {

struct Pending {
  int id, launches;
  cudaEvent_t a, b;
};

std::mutex g_mu;
bool g_enabled = false;
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_pool;
double g_ms[N_IDS];
long long g_launches[N_IDS];

const char* kNames[N_IDS] = {"pool_fwd", "pool_bwd", "latent_fwd", "local_fwd", "gate_fwd",
                             "gate_bwd", "local_bwd", "rout_bwd", "reduce", "latent_bwd",
                             "local_dq", "local_dkv", "decode", "colsum"};

void drain_locked() {
  for (auto& p : g_pending) {
    float ms = 0.f;
    if (cudaEventSynchronize(p.b) == cudaSuccess && cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
      g_ms[p.id] += ms;
      g_launches[p.id] += p.launches;
    }
    g_pool.push_back(p.a);
    g_pool.push_back(p.b);
  }
  g_pending.clear();
}

}  // namespace

const char* name(int id) { return (id >= 0 && id < N_IDS) ? kNames[id] : ""; }

bool enabled() { return g_enabled; }

cudaEvent_t take_event() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

void record(int id, int launches, cudaEvent_t a, cudaEvent_t b) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_pending.push_back({id, launches, a, b});
}

}  // namespace prof
}  // namespace llattn

using namespace llattn::prof;

extern "C" {

int llattn_profile_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_mu);
  drain_locked();
  for (int i = 0; i < N_IDS; ++i) {
    g_ms[i] = 0.0;
    g_launches[i] = 0;
  }
  g_enabled = enable != 0;
  return N_IDS;
}

int llattn_profile_read(double* ms, long long* launches, int n) {
  std::lock_guard<std::mutex> lk(g_mu);
  drain_locked();
  for (int i = 0; i < n && i < N_IDS; ++i) {
    if (ms) ms[i] = g_ms[i];
    if (launches) launches[i] = g_launches[i];
  }
  return N_IDS;
}

const char* llattn_profile_name(int id) { return name(id); }

}  // extern "C"
