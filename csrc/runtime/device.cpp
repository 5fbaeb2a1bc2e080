// Device runtime probe: what this process can run on, with typed reasons.
//
// Reference behaviour: internal/cuda/loader.c (lf_cuda_api_get, :30-167;
// lunaflux_cuda_device_info, :214) resolves the driver and reports typed
// "unavailable" reasons (cuda_abi.h:34-42) instead of failing opaquely.  Here
// the CUDA runtime is linked in, so the probe asks it (and, for the NVLink
// multicast attribute, the driver entry point) and classifies the result:
//
//   ok                  an sm_100 device this build's sm_100a kernels run on
//   no_driver           the CUDA driver is absent or failed to initialise
//   no_device           the driver sees no device
//   unsupported_arch    a device that is not compute capability 10.0
//
// plus, per device pair, whether peer access (NVLink / NVSwitch) is possible,
// and per device whether NVLink multicast (NVLS, used by the fused
// all-reduce) is supported.
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <string>
#include <vector>

namespace lf {
namespace rt {

namespace py = pybind11;

static int multicast_supported(int dev) {
  using GetAttr = CUresult (*)(int*, CUdevice_attribute, CUdevice);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuDeviceGetAttribute", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr) {
    cudaGetLastError();
    return -1;
  }
  int v = 0;
  if (reinterpret_cast<GetAttr>(fn)(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, (CUdevice)dev) != CUDA_SUCCESS)
    return -1;
  return v;
}

py::dict device_report() {
  py::dict r;
  int driver = 0, runtime = 0;
  cudaRuntimeGetVersion(&runtime);
  r["runtime_version"] = runtime;
  if (cudaDriverGetVersion(&driver) != cudaSuccess || driver == 0) {
    cudaGetLastError();
    r["status"] = "no_driver";
    r["driver_version"] = 0;
    r["devices"] = py::list();
    return r;
  }
  r["driver_version"] = driver;
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    r["status"] = e == cudaErrorNoDevice || n == 0 ? "no_device" : "no_driver";
    r["error"] = std::string(cudaGetErrorString(e));
    r["devices"] = py::list();
    return r;
  }
  py::list devs;
  bool all_ok = true;
  for (int i = 0; i < n; ++i) {
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, i);
    py::dict d;
    d["index"] = i;
    d["name"] = std::string(p.name);
    d["cc"] = py::make_tuple(p.major, p.minor);
    d["sms"] = p.multiProcessorCount;
    d["total_bytes"] = (int64_t)p.totalGlobalMem;
    d["l2_bytes"] = p.l2CacheSize;
    d["smem_per_block_optin"] = (int64_t)p.sharedMemPerBlockOptin;
    d["pci_bus_id"] = p.pciBusID;
    d["multicast"] = multicast_supported(i);
    const bool ok = p.major == 10 && p.minor == 0;
    d["status"] = ok ? "ok" : "unsupported_arch";
    all_ok = all_ok && ok;
    py::list peers;
    for (int j = 0; j < n; ++j) {
      int can = 0;
      if (j != i) cudaDeviceCanAccessPeer(&can, i, j);
      peers.append(j == i ? true : can != 0);
    }
    d["peer_access"] = peers;
    devs.append(d);
  }
  r["devices"] = devs;
  r["status"] = all_ok ? "ok" : "unsupported_arch";
  return r;
}

}  // namespace rt
}  // namespace lf
