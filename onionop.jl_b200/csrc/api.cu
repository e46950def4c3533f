// Status and device-query plumbing shared by every C-ABI entry point.
// The reference's device query (`shared_memory`, src/NNop.jl:27-30, and
// `_shared_memory`, ext/NNopCUDAExt.jl:6-9) becomes the cached SM-count query
// here; tile shapes are fixed at compile time for sm_100a.
#include "common.cuh"

#include <mutex>

namespace nnop {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(NNOP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    }
    return NNOP_OK;
}

int num_sms() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace nnop

extern "C" {

int nnop_abi_version(void) { return NNOP_B200_ABI_VERSION; }

const char* nnop_last_error(void) { return nnop::g_last_error.c_str(); }

const char* nnop_status_string(int status) {
    switch (status) {
        case NNOP_OK: return "ok";
        case NNOP_ERR_SHAPE: return "invalid or unsupported shape";
        case NNOP_ERR_DTYPE: return "unsupported dtype";
        case NNOP_ERR_ARG: return "invalid argument";
        case NNOP_ERR_WORKSPACE: return "workspace missing or too small";
        case NNOP_ERR_CUDA: return "CUDA error";
        case NNOP_ERR_ALIGN: return "misaligned pointer";
        default: return "unknown status";
    }
}

}  // extern "C"
