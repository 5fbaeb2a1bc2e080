#pragma once
#include <cuda_runtime.h>

namespace lf {
namespace rt {
struct ErrorState {
  int code;
  unsigned long long info;
};
ErrorState read_error(cudaStream_t s, bool clear);
void inject_error(int code);
}  // namespace rt
}  // namespace lf
