// NVLink / NVSwitch discovery for h3c_device_info and h3c_nvlink_query: the
// CUDA counterpart of H3Hardware's Machine.detect (Sources/H3Hardware/
// Machine.swift:48-56), which measures the machine at start-up rather than
// assuming it.  Everything here is a read-only NVML query, made through
// dlopen so the library has no link-time NVML dependency; no setting of any
// GPU is changed.
#include <dlfcn.h>

#include <cstdlib>
#include <cstring>

#include "common.cuh"

namespace {

// The NVML entry points used here (signatures as in the public nvml.h).
typedef int (*NvmlInit)(void);
typedef int (*NvmlShutdown)(void);
typedef int (*NvmlHandleByPci)(const char*, void**);
typedef int (*NvmlLinkState)(void*, unsigned int, int*);
typedef int (*NvmlLinkVersion)(void*, unsigned int, unsigned int*);
typedef int (*NvmlRemoteType)(void*, unsigned int, int*);

constexpr int kNvmlSuccess = 0;
constexpr int kNvmlEnabled = 1;
constexpr int kNvmlRemoteGpu = 0x00;
constexpr int kNvmlRemoteSwitch = 0x02;
constexpr unsigned kMaxLinks = 18;  // NVLink 5: 18 links per B200

}  // namespace

extern "C" h3c_status h3c_nvlink_query(const char* pci_bus_id, h3c_nvlink* out) {
  if (!pci_bus_id || !out) return H3C_ERR_INVALID_ARGUMENT;
  std::memset(out, 0, sizeof(*out));
  out->version = -1;
  const char* path = getenv("H3C_NVML_LIB");  // a stand-in NVML for tests
  void* so = dlopen(path ? path : "libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
  if (!so) return H3C_ERR_UNSUPPORTED;
  auto init = (NvmlInit)dlsym(so, "nvmlInit_v2");
  auto shutdown = (NvmlShutdown)dlsym(so, "nvmlShutdown");
  auto by_pci = (NvmlHandleByPci)dlsym(so, "nvmlDeviceGetHandleByPciBusId_v2");
  auto state = (NvmlLinkState)dlsym(so, "nvmlDeviceGetNvLinkState");
  auto version = (NvmlLinkVersion)dlsym(so, "nvmlDeviceGetNvLinkVersion");
  auto remote = (NvmlRemoteType)dlsym(so, "nvmlDeviceGetNvLinkRemoteDeviceType");
  h3c_status st = H3C_ERR_UNSUPPORTED;
  if (init && shutdown && by_pci && state && init() == kNvmlSuccess) {
    void* dev = nullptr;
    if (by_pci(pci_bus_id, &dev) != kNvmlSuccess) {
      st = H3C_ERR_NO_DEVICE;
    } else {
      out->available = 1;
      for (unsigned l = 0; l < kMaxLinks; ++l) {
        int active = 0;
        if (state(dev, l, &active) != kNvmlSuccess || active != kNvmlEnabled) continue;
        out->links_active++;
        unsigned v = 0;
        if (version && out->version < 0 && version(dev, l, &v) == kNvmlSuccess) out->version = (int32_t)v;
        int type = -1;
        if (remote && remote(dev, l, &type) == kNvmlSuccess) {
          if (type == kNvmlRemoteSwitch) out->links_to_switch++;
          else if (type == kNvmlRemoteGpu) out->links_to_gpu++;
        }
      }
      st = H3C_OK;
    }
    shutdown();
  }
  dlclose(so);
  return st;
}
