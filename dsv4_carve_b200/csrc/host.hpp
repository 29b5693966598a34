// host.hpp -- host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/exl3_b200.h"

namespace exl3 {

// Thread-local text of the last failing call (exl3_last_error()).
void set_last_error(const char* fmt, ...);

#define EXL3_REQUIRE(cond, code, ...)              \
    do {                                           \
        if (!(cond)) {                             \
            ::exl3::set_last_error(__VA_ARGS__);   \
            return (code);                         \
        }                                          \
    } while (0)

#define EXL3_CUDA(call)                                                              \
    do {                                                                             \
        cudaError_t e_ = (call);                                                     \
        if (e_ != cudaSuccess) {                                                     \
            ::exl3::set_last_error("%s: %s", #call, cudaGetErrorString(e_));         \
            return EXL3_ERR_CUDA;                                                    \
        }                                                                            \
    } while (0)

struct DeviceInfo {
    int sms = 0;
    int max_smem_optin = 0;
};

// Cached per device (guarded by a mutex inside).
int device_info(int device, DeviceInfo* out);

inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace exl3
