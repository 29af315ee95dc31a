// exl3b_capi_util.h -- error plumbing of the C-ABI entry points (host side).
// Every entry point returns 0 on success or an EXL3B_E* code; exl3b_last_error() returns the message of the
// last failure on the calling thread.  Arguments are validated before any launch, so a rejected call enqueues
// nothing.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#define EXL3B_API __attribute__((visibility("default")))

enum { EXL3B_OK = 0, EXL3B_EINVAL = 1, EXL3B_ECUDA = 2, EXL3B_EUNSUPPORTED = 3 };

int exl3b_fail(int code, const char* msg);
int exl3b_launch_status(const char* where);

#define EXL3B_CHECK(cond, msg)                                  \
    do {                                                        \
        if (!(cond)) return exl3b_fail(EXL3B_EINVAL, (msg));    \
    } while (0)
