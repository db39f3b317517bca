// runtime.cu -- error reporting and the per-device status word.
#include <mutex>
#include <string>

#include "common.cuh"
#include "ptx.cuh"

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

// One thread waits on phase 0 of an mbarrier that expects one arrival and
// gets none: mbar_wait gives up after its ~2 s limit and the give-up path
// records the timeout, as in every kernel whose producer never delivers.
constexpr int kSelftestWaitSite = 90;
__global__ void wait_timeout_selftest_kernel(DeviceStatus* st) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(s_addr(&bar), 1);
        if (!mbar_wait(s_addr(&bar), 0)) record_timeout(st, kSelftestWaitSite);
    }
}

}  // namespace specdec

extern "C" const char* specdec_last_error(void) { return specdec::g_last_error.c_str(); }
extern "C" int specdec_abi_version(void) { return 1; }

extern "C" int specdec_selftest_wait_timeout(void* stream) {
    using namespace specdec;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DeviceStatus* st = device_status_ptr();
    SD_CHECK(st, SPECDEC_ECUDA, "selftest_wait_timeout: no device status word");
    wait_timeout_selftest_kernel<<<1, 32, 0, s>>>(st);
    SD_LAUNCH_CHECK("wait_timeout_selftest_kernel");
    return check_device_status(s);
}
