// Host-side plumbing shared by the entry points: error strings, device properties, launch
// accounting and the programmatic-dependent-launch switch.
#include <cstdlib>
#include <cstring>
#include <string>

#include <cuda_runtime.h>

#include "dm3_internal.h"

namespace dm3 {

namespace {
thread_local std::string g_error;
thread_local int g_launches = 0;
int g_sms[64] = {0};
}  // namespace

void set_error(const std::string& msg) { g_error = msg; }

int sm_count(int device) {
  if (device < 0 || device >= 64) return 148;
  if (g_sms[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    g_sms[device] = v;
  }
  return g_sms[device];
}

void note_launches(int n) { g_launches = n; }

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("DM3_PDL");
    v = (e && std::strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

}  // namespace dm3

extern "C" const char* dm3_last_error(void) { return dm3::g_error.c_str(); }

extern "C" const char* dm3_version(void) { return "0.1.0"; }

extern "C" int dm3_last_launch_count(void) { return dm3::g_launches; }
