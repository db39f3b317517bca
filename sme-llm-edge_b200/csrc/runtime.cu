// runtime.cu -- error reporting and the per-device status word.
#include <mutex>
#include <string>

#include "common.cuh"

namespace specdec {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int cuda_status(cudaError_t e, const char* what) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    (void)cudaGetLastError();  // clear a non-sticky error so it does not resurface at the next launch check
    return e == cudaErrorMemoryAllocation ? SPECDEC_ENOMEM : SPECDEC_ECUDA;
}

static std::mutex g_status_mu;
static DeviceStatus* g_status[64] = {nullptr};

DeviceStatus* device_status_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (!g_status[dev]) {
        DeviceStatus* p = nullptr;
        if (cudaMalloc(&p, sizeof(DeviceStatus)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(DeviceStatus)) != cudaSuccess) return nullptr;
        g_status[dev] = p;
    }
    return g_status[dev];
}

int check_device_status(cudaStream_t s) {
    DeviceStatus* p = device_status_ptr();
    if (!p) return SPECDEC_OK;
    DeviceStatus h{0, 0};
    SD_CUDA(cudaMemcpyAsync(&h, p, sizeof(h), cudaMemcpyDeviceToHost, s));
    SD_CUDA(cudaStreamSynchronize(s));
    if (h.code) {
        SD_CUDA(cudaMemsetAsync(p, 0, sizeof(DeviceStatus), s));
        set_error("device-side wait gave up at site " + std::to_string(h.where));
        return h.code;
    }
    return SPECDEC_OK;
}

}  // namespace specdec

extern "C" const char* specdec_last_error(void) { return specdec::g_last_error.c_str(); }
extern "C" int specdec_abi_version(void) { return 1; }
