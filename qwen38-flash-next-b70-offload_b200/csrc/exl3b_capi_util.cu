// exl3b_capi_util.cu -- thread-local last-error message of the C-ABI.
#include "exl3b_capi_util.h"
#include <string.h>

static thread_local char t_err[512];

int exl3b_fail(int code, const char* msg) {
    snprintf(t_err, sizeof(t_err), "%s", msg ? msg : "error");
    return code;
}

int exl3b_launch_status(const char* where) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return 0;
    snprintf(t_err, sizeof(t_err), "%s: %s", where, cudaGetErrorString(e));
    return EXL3B_ECUDA;
}

extern "C" EXL3B_API const char* exl3b_last_error(void) { return t_err; }

extern "C" EXL3B_API int exl3b_abi_version(void) { return 1; }
