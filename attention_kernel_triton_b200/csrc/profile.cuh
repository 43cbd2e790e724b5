// RAII event pair around one kernel launch when akt_profile_enable(1) is set.
#pragma once
#include <cuda_runtime.h>
#include "../../include/akt.h"

namespace akt {
class ProfileScope {
 public:
  explicit ProfileScope(cudaStream_t st);
  ~ProfileScope();
  ProfileScope(const ProfileScope&) = delete;
  ProfileScope& operator=(const ProfileScope&) = delete;

 private:
  cudaStream_t stream_;
  void* stop_;
};
}  // namespace akt
