// Optional per-kernel timing for benchmarks (akt_profile_* in include/akt.h).
//
// While enabled on a thread, every entry point records a CUDA event pair
// around its main kernel, on the stream that kernel is launched on.
// akt_profile_read() waits for the recorded events and returns the summed
// device time and the number of timed launches.  Disabled (the default),
// the hook costs one thread-local branch per call.
#include "profile.cuh"

#include <string>
#include <vector>

namespace akt {

int set_error(int code, const std::string& msg);

namespace {
struct ProfileState {
  bool on = false;
  std::vector<cudaEvent_t> pool;  // start/stop pairs, reused across reads
  size_t used = 0;
  int device = -1;
};
thread_local ProfileState g_prof;

cudaEvent_t take_event() {
  if (g_prof.used == g_prof.pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    g_prof.pool.push_back(e);
  }
  return g_prof.pool[g_prof.used++];
}
}  // namespace

ProfileScope::ProfileScope(cudaStream_t st) : stream_(st), stop_(nullptr) {
  if (!g_prof.on) return;
  cudaEvent_t a = take_event();
  cudaEvent_t b = take_event();
  if (!a || !b) return;
  cudaEventRecord(a, st);
  stop_ = b;
}

ProfileScope::~ProfileScope() {
  if (stop_) cudaEventRecord(static_cast<cudaEvent_t>(stop_), stream_);
}

}  // namespace akt

using namespace akt;

extern "C" {

int akt_profile_enable(int on) {
  g_prof.on = on != 0;
  g_prof.used = 0;
  return AKT_OK;
}

int akt_profile_read(double* total_ms, int64_t* launches) {
  double tot = 0.0;
  int64_t n = 0;
  for (size_t i = 0; i + 1 < g_prof.used; i += 2) {
    cudaError_t e = cudaEventSynchronize(g_prof.pool[i + 1]);
    if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, cudaGetErrorString(e));
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, g_prof.pool[i], g_prof.pool[i + 1]);
    if (e != cudaSuccess) return set_error(AKT_ERR_CUDA, cudaGetErrorString(e));
    tot += ms;
    ++n;
  }
  g_prof.used = 0;
  if (total_ms) *total_ms = tot;
  if (launches) *launches = n;
  return AKT_OK;
}

}  // extern "C"
