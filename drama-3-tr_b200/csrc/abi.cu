// Host-side plumbing shared by the entry points: error strings, device properties, launch
// accounting and the programmatic-dependent-launch switch.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include <cuda.h>
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

bool cluster_path_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("DM3_CLUSTER");
    v = (e && std::strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct MapKey {
  const void* base;
  uint64_t d0, d1, d2, s1, s2;
  uint32_t box_rows;
  bool operator==(const MapKey& o) const {
    return base == o.base && d0 == o.d0 && d1 == o.d1 && d2 == o.d2 && s1 == o.s1 && s2 == o.s2 &&
           box_rows == o.box_rows;
  }
};

constexpr int kMapCache = 256;
struct MapCache {
  std::mutex mu;
  MapKey key[kMapCache];
  CUtensorMap map[kMapCache];
  int used = 0, next = 0;
};
MapCache g_maps;

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(f);
  });
  return fn;
}

}  // namespace

bool tensor_map_3d(CUtensorMap* out, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                   uint64_t stride2, uint32_t box_rows) {
  const MapKey k{base, d0, d1, d2, stride1, stride2, box_rows};
  std::lock_guard<std::mutex> lock(g_maps.mu);
  for (int i = 0; i < g_maps.used; ++i)
    if (g_maps.key[i] == k) {
      *out = g_maps.map[i];
      return true;
    }
  EncodeTiled enc = encoder();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1, stride2};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  CUtensorMap m;
  const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, elem,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r)));
    return false;
  }
  const int slot = g_maps.used < kMapCache ? g_maps.used++ : (g_maps.next++ % kMapCache);
  g_maps.key[slot] = k;
  g_maps.map[slot] = m;
  *out = m;
  return true;
}

}  // namespace dm3

extern "C" const char* dm3_last_error(void) { return dm3::g_error.c_str(); }

extern "C" const char* dm3_version(void) { return "0.1.0"; }

extern "C" int dm3_last_launch_count(void) { return dm3::g_launches; }

extern "C" int dm3_set_wait_limit_ns(uint64_t ns) {
  if (ns == 0) return dm3::set_error("the wait limit must be at least 1 ns"), 1;
  int (*setters[])(uint64_t) = {dm3::wait_limit_gemm, dm3::wait_limit_gemv, dm3::wait_limit_gemv_tc, dm3::wait_limit_moe_decode,
                                dm3::wait_limit_moe_prefill};
  for (auto fn : setters) {
    const int err = fn(ns);
    if (err != 0)
      return dm3::set_error(std::string("setting the wait limit: ") +
                            cudaGetErrorString(static_cast<cudaError_t>(err))), 2;
  }
  return 0;
}
