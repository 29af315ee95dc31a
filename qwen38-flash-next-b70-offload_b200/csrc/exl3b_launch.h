// exl3b_launch.h -- kernel launch with programmatic dependent launch (PDL).
//
// Kernels of the per-layer chain are launched with cudaLaunchAttributeProgrammaticStreamSerialization, so a
// kernel's blocks may start while the previous kernel on the stream is still running; each kernel executes
// griddepcontrol.wait (pdl_wait) before it reads anything the previous kernels produced, and calls
// griddepcontrol.launch_dependents (pdl_trigger) once the next kernel may be scheduled.  Both instructions are
// no-ops when a kernel was launched without the attribute.  EXL3B_NO_PDL=1 in the environment disables the
// attribute (plain stream order).
#pragma once
#include <cuda_runtime.h>
#include <stdlib.h>

namespace exl3b {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

inline bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("EXL3B_NO_PDL");
        v = (e && e[0] == '1') ? 0 : 1;
    }
    return v == 1;
}

// Profiling hook (exl3b_set_profile_events): records phase event i on stream s when one is set.  Decode: 0 before
// the routing / cache step, 1 before gate-up, 2 before down, 3 after down.  Prefill: 0 before align, 1 before the
// gate-up GEMM, 2 before the down GEMM, 3 after the combine.
void prof_record(int i, cudaStream_t s);

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace exl3b
