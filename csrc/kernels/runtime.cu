// Host side of the device error word.  Kernels never trap: they record a code
// in their translation unit's error word and return, so a failed wait or a
// bad index leaves the CUDA context usable and the host decides what to do
// with the step.  This file folds the per-translation-unit words together.
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "common.cuh"
#include "runtime.h"

namespace lf {
namespace rt {

namespace {
struct Hooks {
  ErrReadFn read;
  ErrInjectFn inject;
  WaitLimitFn wait_limit;
};
std::vector<Hooks>& hooks() {
  static std::vector<Hooks> h;
  return h;
}
std::mutex& hooks_mu() {
  static std::mutex m;
  return m;
}
}  // namespace

void register_error_word(ErrReadFn read, ErrInjectFn inject, WaitLimitFn wait_limit) {
  std::lock_guard<std::mutex> g(hooks_mu());
  hooks().push_back({read, inject, wait_limit});
}

void set_wait_limit_ns(unsigned long long ns) {
  std::lock_guard<std::mutex> g(hooks_mu());
  for (auto& h : hooks()) h.wait_limit(ns);
}

ErrorState read_error(cudaStream_t s, bool clear) {
  ErrorState st{0, 0};
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) throw std::runtime_error(std::string("lunaflux: stream sync: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> g(hooks_mu());
  for (auto& h : hooks()) {
    unsigned long long info = 0;
    int code = h.read(clear, &info);
    if (code != 0 && st.code == 0) {
      st.code = code;
      st.info = info;
    }
  }
  return st;
}

}  // namespace rt

void launch_failed(cudaError_t e) {
  throw std::runtime_error(std::string("lunaflux kernel launch: ") + cudaGetErrorString(e));
}

namespace rt {

static int g_pdl = -1;

// On by default (measured +1.2 % on the TP 1 headline); LUNAFLUX_PDL=0 turns it off.
bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* e = getenv("LUNAFLUX_PDL");
    g_pdl = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return g_pdl == 1;
}

void set_pdl(bool on) { g_pdl = on ? 1 : 0; }

void inject_error(int code) {
  std::lock_guard<std::mutex> g(hooks_mu());
  if (!hooks().empty()) hooks().front().inject(code);
}

}  // namespace rt
}  // namespace lf
