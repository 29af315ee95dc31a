// exl3b_noalloc.cu -- exl3b_moe_decode_noalloc: the routed-MoE decode for callers that cannot allocate device memory
// (no cudaMalloc, no caching allocator of their own).  It runs the same kernels as exl3b_moe_decode, with the scratch
// that exl3b_moe_decode takes from the caller placed in a fixed file-scope device array instead.
//
// Limits:
//   * kNoallocScratchBytes = 8 MiB per device: exl3b_moe_decode_workspace(M, topk, H, I) must fit, which covers up to
//     85 tokens at top-10 with H = 2048, I = 768 (about 94 KiB per token there).  Larger calls are rejected with
//     EXL3B_EINVAL before anything is launched.
//   * Set-up: the first call on each device looks the array's device address up (cudaGetSymbolAddress, with that
//     device current) and keeps it; make that first call before any stream capture on the device.
//   * Nothing in the scratch has to start at zero: the first kernel of every call zeroes the counters it uses.
//   * One scratch per device: calls that overlap on one device (different streams or host threads with no ordering
//     between them) race on it.  Order them (one stream, or events).
#include "exl3b_capi_util.h"

#include <cuda_runtime.h>
#include <mutex>

namespace {

constexpr int64_t kNoallocScratchBytes = 8ll << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device.
int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return exl3b_fail(EXL3B_EUNSUPPORTED, "exl3b_moe_decode_noalloc: device index >= 64");
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        if (!ptr) return exl3b_fail(EXL3B_ECUDA, "exl3b_moe_decode_noalloc: null scratch address");
        g_scratch_ptr[dev] = ptr;
    }
    *out = g_scratch_ptr[dev];
    return 0;
}

}  // namespace

extern "C" EXL3B_API int64_t exl3b_moe_decode_workspace(int M, int topk, int H, int I);
extern "C" EXL3B_API int exl3b_moe_decode(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids,
                                          const float* w, int M, int topk, const int64_t* ptrs, const int32_t* kinfo,
                                          int H, int I, int K, int E, void* out, int64_t out_stride, int out_bf16,
                                          void* workspace, int64_t ws_bytes, int flags, void* stream);

extern "C" EXL3B_API int exl3b_moe_decode_noalloc(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids,
                                                  const float* w, int M, int topk, const int64_t* ptrs,
                                                  const int32_t* kinfo, int H, int I, int K, int E, void* out,
                                                  int64_t out_stride, int out_bf16, int flags, void* stream) {
    if (M < 0 || topk < 1) return exl3b_fail(EXL3B_EINVAL, "exl3b_moe_decode_noalloc: bad M / topk");
    // shape errors are reported as such, not as a scratch overflow (the size query returns 0 for them)
    if (H < 128 || I < 128 || H % 128 || I % 128)
        return exl3b_fail(EXL3B_EINVAL, "exl3b_moe_decode_noalloc: H, I must be multiples of 128");
    if (M == 0) return 0;
    const int64_t need = exl3b_moe_decode_workspace(M, topk, H, I);
    if (need <= 0 || need > kNoallocScratchBytes)
        return exl3b_fail(EXL3B_EINVAL,
                          "exl3b_moe_decode_noalloc: M * topk, H, I need more scratch than the fixed 8 MiB; "
                          "call exl3b_moe_decode with a caller workspace");
    void* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    return exl3b_moe_decode(x, x_stride, x_bf16, ids, w, M, topk, ptrs, kinfo, H, I, K, E, out, out_stride, out_bf16,
                            scratch, kNoallocScratchBytes, flags, stream);
}
