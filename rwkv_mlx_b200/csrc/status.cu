// Error-string plumbing behind rwkv_last_error().
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace rwkv {
static thread_local char g_err[256] = "no error";

int set_cuda_error(cudaError_t e) {
    if (e == cudaSuccess) return RWKV_OK;
    snprintf(g_err, sizeof(g_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
}

int check_launch() { return set_cuda_error(cudaGetLastError()); }

int set_error(int code, const char* msg) {
    snprintf(g_err, sizeof(g_err), "%s", msg);
    return code;
}

void clear_error() { snprintf(g_err, sizeof(g_err), "%s", "no error"); }
}  // namespace rwkv

extern "C" const char* rwkv_last_error(void) { return rwkv::g_err; }
extern "C" int rwkv_abi_version(void) { return 1; }
