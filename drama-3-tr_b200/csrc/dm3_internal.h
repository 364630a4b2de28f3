// Limits shared by the host entry points and the kernels, and host-side helpers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

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

}  // namespace dm3
