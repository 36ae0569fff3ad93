// abi.cu -- library-level entry points and host helpers of the B200 strict-tensor provider.
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "pcu_b200.h"
#include "provider.h"

namespace {

thread_local int g_last_cuda_error = 0;

__global__ void fill_status_kernel(unsigned long long *status, uint64_t count) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (; i < count; i += stride) status[i] = pcu::kStatusOk;
}

__global__ void chain_decide_kernel(pcu::ChainGuard guard) { (void)pcu::chain_admits(guard); }

}  // namespace

namespace pcu {

int chain_decide_only(const ChainGuard &guard, cudaStream_t stream) {
    if (!guard.disp || !guard.decide) return PCU_B200_OK;
    chain_decide_kernel<<<1, 1, 0, stream>>>(guard);
    return pcu_host::launch_status();
}

}  // namespace pcu

namespace pcu_host {

int set_cuda_error(cudaError_t err) {
    g_last_cuda_error = (int)err;
    return PCU_B200_ERROR_CUDA;
}

int launch_status(void) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return set_cuda_error(err);
    return PCU_B200_OK;
}

int sm_count(void) {
    static std::mutex lock;
    static int cached[64] = {0};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
    std::lock_guard<std::mutex> guard(lock);
    if (!cached[device]) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0)
            sms = 148;
        cached[device] = sms;
    }
    return cached[device];
}

}  // namespace pcu_host

extern "C" int pcu_b200_abi_version(void) { return PCU_B200_ABI_VERSION; }

extern "C" const char *pcu_b200_error_string(int code) {
    switch (code) {
    case PCU_B200_OK: return "ok";
    case PCU_B200_ERROR_INVALID_ARGUMENT: return "invalid argument";
    case PCU_B200_ERROR_SIZE_OVERFLOW: return "shape or fault-event domain exceeds the supported range";
    case PCU_B200_ERROR_WORKSPACE: return "workspace missing or too small";
    case PCU_B200_ERROR_CUDA: return "CUDA launch or configuration failure (see pcu_b200_last_cuda_error)";
    case PCU_B200_ERROR_UNSUPPORTED: return "unsupported on this device";
    default: return "unknown error";
    }
}

extern "C" int pcu_b200_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" int pcu_b200_status_reset(uint64_t *status, uint64_t count, void *stream) {
    if (count == 0) return PCU_B200_OK;
    if (!status) return PCU_B200_ERROR_INVALID_ARGUMENT;
    unsigned blocks = (unsigned)((count + 255) / 256 < 1024 ? (count + 255) / 256 : 1024);
    fill_status_kernel<<<blocks, 256, 0, pcu_host::as_stream(stream)>>>(
        reinterpret_cast<unsigned long long *>(status), count);
    return pcu_host::launch_status();
}
