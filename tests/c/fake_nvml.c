/* A stand-in for libnvidia-ml.so.1 with the few read-only queries the
 * library's NVLink discovery makes, so that the discovery logic can be
 * checked on a machine without a GPU.  It models one HGX B200 at PCI bus id
 * 0000:1B:00.0: links 0-17 active, version 5 (NVML's value for NVLink 5 is
 * reported as is), every link to an NVSwitch except link 17, which reports a
 * GPU peer; any other bus id is unknown. */
#include <string.h>

static int g_init = 0;
int nvmlInit_v2(void) { g_init = 1; return 0; }
int nvmlShutdown(void) { g_init = 0; return 0; }
int nvmlDeviceGetHandleByPciBusId_v2(const char* bus, void** dev) {
  if (!g_init) return 1;
  if (strcmp(bus, "0000:1B:00.0") != 0) return 6; /* NVML_ERROR_NOT_FOUND */
  *dev = (void*)0x1;
  return 0;
}
int nvmlDeviceGetNvLinkState(void* dev, unsigned int link, int* active) {
  (void)dev;
  if (link >= 18) return 2;
  *active = 1;
  return 0;
}
int nvmlDeviceGetNvLinkVersion(void* dev, unsigned int link, unsigned int* v) {
  (void)dev; (void)link;
  *v = 5;
  return 0;
}
int nvmlDeviceGetNvLinkRemoteDeviceType(void* dev, unsigned int link, int* type) {
  (void)dev;
  *type = link == 17 ? 0 : 2;
  return 0;
}
