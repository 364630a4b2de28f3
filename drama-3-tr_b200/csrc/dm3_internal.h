// Limits shared by the host entry points and the kernels, and host-side helpers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda.h>

namespace dm3 {

constexpr int kMaxT = 4;         // activation rows handled by the skinny (decode) kernels
constexpr int kMaxSlots = 33;    // 32 distinct routed experts (4 rows x top-8) + the shared expert
constexpr int kMaxTopK = 8;
constexpr int kMaxRouter = 256;  // router width handled by the in-kernel top-k
constexpr int kMaxH = 2048;      // hidden size handled by the fused MoE kernel
constexpr int kMaxI = 512;       // expert intermediate size handled by the fused MoE kernel
constexpr int kMaxGemvK = 8192;

// Host helpers (abi.cu)
void set_error(const std::string& msg);
int sm_count(int device);
void note_launches(int n);
bool pdl_enabled();
// The decode layer's expert phase as one kernel of thread-block clusters (the default; DM3_CLUSTER=0
// selects the four-kernel chain).
bool cluster_path_enabled();
// Per-file setters of the device wait limit on the current device (cudaError_t as int).
int wait_limit_gemm(uint64_t ns);
int wait_limit_gemv(uint64_t ns);
// Reads and clears the status word of the gemv.cu kernels on the stream (asynchronously).
int gemv_status_async(uint32_t* host_value, CUstream_st* stream);
int wait_limit_gemv_tc(uint64_t ns);
int wait_limit_moe_decode(uint64_t ns);
int wait_limit_moe_prefill(uint64_t ns);
// A 3-D uint8 tensor map over [d2][d1][d0] bytes (row stride stride1, plane stride stride2) whose
// box is 128 bytes x box_rows rows x 1 plane, loaded with the 128-byte swizzle; encodings are cached
// by their arguments. False (with the error set) when the driver rejects them.
bool tensor_map_3d(CUtensorMap* out, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                   uint64_t stride2, uint32_t box_rows);

}  // namespace dm3
