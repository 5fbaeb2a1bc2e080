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
// Limit of every bounded wait in every kernel, on the current device
// (nanoseconds; default 1e9).
void set_wait_limit_ns(unsigned long long ns);
// Programmatic dependent launch for the kernels of the step (on unless
// LUNAFLUX_PDL=0 or set_pdl(false)).
bool pdl_enabled();
void set_pdl(bool on);
}  // namespace rt
}  // namespace lf
