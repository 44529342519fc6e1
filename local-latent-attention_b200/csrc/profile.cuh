// Optional per-kernel timing of libllattn launches with CUDA events recorded
// on the launching stream (llattn_profile_enable / llattn_profile_read).
// Host-side state only; when disabled a Scope costs one branch.
#pragma once

#include <cuda_runtime.h>

namespace llattn {
namespace prof {

enum Id {
  POOL_FWD = 0, POOL_BWD, LATENT_FWD, LOCAL_FWD, GATE_FWD, GATE_BWD, LOCAL_BWD, ROUT_BWD, REDUCE, LATENT_BWD,
  LOCAL_DQ, LOCAL_DKV, DECODE, COLSUM,
  N_IDS
};

const char* name(int id);
bool enabled();
void record(int id, int launches, cudaEvent_t a, cudaEvent_t b);
cudaEvent_t take_event();

// Records an event pair around the launches made during its lifetime.
struct Scope {
  int id, launches;
  cudaStream_t s;
  cudaEvent_t a = nullptr;
  Scope(int id_, cudaStream_t s_, int launches_ = 1) : id(id_), launches(launches_), s(s_) {
    if (enabled()) {
      a = take_event();
      if (a) cudaEventRecord(a, s);
    }
  }
  ~Scope() {
    if (a) {
      cudaEvent_t b = take_event();
      if (b) {
        cudaEventRecord(b, s);
        record(id, launches, a, b);
      }
    }
  }
};

}  // namespace prof
}  // namespace llattn
