// Status codes and error text of the C ABI (include/ssm_b200.h).
#include <string>

#include "common.cuh"

namespace ssm {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return SSM_OK;
    return fail(SSM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int ensure_context(const char* what) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);   // initialises the primary context and makes it current
    if (e == cudaSuccess) return SSM_OK;
    return fail(SSM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace ssm

extern "C" const char* ssm_status_string(int status) {
    switch (status) {
        case SSM_OK: return "ok";
        case SSM_ERR_INVALID: return "invalid argument";
        case SSM_ERR_UNSUPPORTED: return "unsupported dtype or size";
        case SSM_ERR_CUDA: return "CUDA error";
        case SSM_ERR_WORKSPACE: return "workspace too small";
        default: return "unknown status";
    }
}

extern "C" const char* ssm_last_error(void) { return ssm::g_last_error.c_str(); }
