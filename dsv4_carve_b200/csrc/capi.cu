// capi.cu -- ABI-wide entry points: version, last error, device cache,
// scratch status word.
#include <cstring>
#include <mutex>
#include <vector>

#include "host.hpp"

namespace exl3 {

static thread_local char g_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int device_info(int device, DeviceInfo* out) {
    static std::mutex mu;
    static std::vector<DeviceInfo> cache;
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0) return EXL3_ERR_ARG;
    if ((int) cache.size() <= device) cache.resize(device + 1);
    DeviceInfo& d = cache[device];
    if (d.sms == 0) {
        EXL3_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device));
        EXL3_CUDA(cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    }
    *out = d;
    return EXL3_OK;
}

}  // namespace exl3

extern "C" int exl3_abi_version(void) { return 2; }

extern "C" const char* exl3_last_error(void) { return exl3::g_last_error; }

extern "C" int exl3_scratch_status(void* scratch, int is_moe, int clear, uint32_t* status, void* stream) {
    (void) is_moe;   // both scratch layouts keep the status word at byte offset 8
    EXL3_REQUIRE(scratch && status, EXL3_ERR_ARG, "exl3_scratch_status: null pointer");
    auto s = static_cast<cudaStream_t>(stream);
    uint32_t* word = reinterpret_cast<uint32_t*>(scratch) + 2;
    EXL3_CUDA(cudaMemcpyAsync(status, word, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    EXL3_CUDA(cudaStreamSynchronize(s));
    if (clear) {
        EXL3_CUDA(cudaMemsetAsync(word, 0, sizeof(uint32_t), s));
        EXL3_CUDA(cudaStreamSynchronize(s));
    }
    return EXL3_OK;
}
