// exl3b_router.cu -- router GEMV + softmax top-k (the SGLang TopK the reference plugin consumes at
// plugin/sglang_plugin.tier.py:534-535, 560).
//
// Arithmetic (fixed so that expert ids are bit-exact against the CPU oracle):
//   logit[t,e] = dot(x[t], Wr[e]) + bias[e]; dot = xor-butterfly (offsets 16,8,4,2,1) over 32 chunk partials, chunk
//   c = k in [c*H/32, (c+1)*H/32) accumulated in ascending k with fp32 fma from 0.
//   top-k: largest logits, ties to the lower expert id, descending order.
//   w_i = expf(l_i - l_0) / sum_j expf(l_j - l_0) (softmax renormalised over the selection).
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include "exl3b_launch.h"
#include "exl3b_topk.cuh"

namespace exl3b {

__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int T, int E, int topk,
                                                          int* __restrict__ ids, float* __restrict__ w) {
    __shared__ uint2 cand[8][32];
    pdl_wait();
    pdl_trigger();
    int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    topk_warp(logits, t, E, topk, ids, w, cand[threadIdx.x >> 5]);
}

// One warp per expert, 8 experts per block; blockIdx.y = token chunk of TC tokens.  Lane c owns chunk c:
// its slice of Wr[e] stays in registers across the chunk's tokens.
template <int CL, int TC>
__global__ void __launch_bounds__(256, 2) router_logits_kernel(const __nv_bfloat16* __restrict__ x, long long xs,
                                                            const __nv_bfloat16* __restrict__ wr,
                                                            const float* __restrict__ bias, int T, int H, int E,
                                                            float* __restrict__ logits, int topk, int* __restrict__ ids,
                                                            float* __restrict__ w, int* counter) {
    __shared__ int sh_last;
    __shared__ uint2 cand[8][32];   // fused selection: candidates of each token's warp
    int lane = threadIdx.x & 31;
    int e = blockIdx.x * 8 + (threadIdx.x >> 5);
    constexpr int NV = CL / 8;   // uint4 (8 bf16) per chunk
    uint4 wv[NV];
    // the router weights do not depend on earlier kernels: load them before waiting for x
    const int ec = e < E ? e : E - 1;
    const uint4* wp = reinterpret_cast<const uint4*>(wr + (long long)ec * H + lane * CL);
#pragma unroll
    for (int i = 0; i < NV; ++i) wv[i] = __ldg(wp + i);
    float b = (bias && e < E) ? bias[e] : 0.0f;
    // The fused selection runs on one block, whichever finishes last, once per call: its first instructions and
    // first logit loads on that SM are cold.  Warp 0 of every block runs the same selection code on row 0 of the
    // logits buffer (whatever it holds; nothing is stored: T >= 1 here) while the previous kernel still runs, so
    // the code and the buffer's address translations are warm when the real selection starts (measured: the
    // 48-layer decode step 6% faster).
    if (counter && threadIdx.x < 32) {
        if (!(E % 32 == 0 && E <= 512 && topk <= 32 && topk_warp_thresh(logits, 0, E, topk, ids, w, T < 0, cand[0]))) {
            if (E <= 512) topk_warp_n<16>(logits, 0, E, topk, ids, w, T < 0);
            else topk_warp_n<32>(logits, 0, E, topk, ids, w, T < 0);
        }
    }
    pdl_wait();
    pdl_trigger();
    int t0 = blockIdx.y * TC;
    for (int t = t0; e < E && t < min(T, t0 + TC); ++t) {
        const uint4* xp = reinterpret_cast<const uint4*>(x + (long long)t * xs + lane * CL);
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            uint4 xv = __ldg(xp + i);
            const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
            const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv[i]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float x0 = __uint_as_float(xw[j] << 16), x1 = __uint_as_float(xw[j] & 0xFFFF0000u);
                float w0 = __uint_as_float(ww[j] << 16), w1 = __uint_as_float(ww[j] & 0xFFFF0000u);
                acc = __fmaf_rn(x0, w0, acc);
                acc = __fmaf_rn(x1, w1, acc);
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) __stcg(logits + (long long)t * E + e, bias ? __fadd_rn(acc, b) : acc);
    }
    if (!counter) return;
    // fused selection: the last block to finish runs the top-k of every token (T <= 8, one warp per token)
    // the block barrier orders every warp's logits before thread 0's release; the last block's acquire, then its
    // barrier, make every block's logits visible to all of its threads
    __syncthreads();
    if (threadIdx.x == 0) {
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;\n" : "=r"(old) : "l"(counter) : "memory");
        sh_last = old == (int)(gridDim.x * gridDim.y) - 1;
    }
    __syncthreads();
    if (!sh_last) return;
    int t = threadIdx.x >> 5;
    if (t < T) topk_warp(logits, t, E, topk, ids, w, cand[t]);
    if (threadIdx.x == 0) *counter = 0;
}

// Large-T logits: a CUDA-core GEMM tile (64 tokens x 64 experts per block, 4 x 4 per thread) with the arithmetic
// of router_logits_kernel bit for bit.  There, lane c sums chunk c (k in [c CL, (c + 1) CL)) in ascending k with fp32
// fma from 0, and the xor butterfly (offsets 16, 8, 4, 2, 1) adds the 32 chunk sums as a fixed binary tree whose
// leaves, left to right, are the chunks in 5-bit bit-reversed order (0, 16, 8, 24, 4, ...).  Here each thread
// computes the chunk sums of its outputs in that order and folds each into a 5-level stack like a binary counter
// (a left subtree waits at its level until its right sibling arrives: s = left + right), which forms the same tree.
// Chunks pass through shared memory as fp32, [k][row] (double-buffered, loaded one chunk ahead).
template <int CL>
__global__ void __launch_bounds__(256, 1) router_logits_tiled_kernel(const __nv_bfloat16* __restrict__ x, long long xs,
                                                                     const __nv_bfloat16* __restrict__ wr,
                                                                     const float* __restrict__ bias, int T, int H,
                                                                     int E, float* __restrict__ logits) {
    extern __shared__ __align__(16) float rsm[];
    constexpr int NV = CL / 8;                     // 16-byte vectors per row of a chunk
    constexpr int NLD = (64 * NV + 255) / 256;     // vectors per thread per operand
    float* xsm = rsm;                              // [2][CL][64] tokens
    float* wsm = rsm + 2 * CL * 64;                // [2][CL][64] experts
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int t0 = blockIdx.x * 64, e0 = blockIdx.y * 64;
    uint4 rx[NLD], rw[NLD];
    auto gload = [&](int c) {
#pragma unroll
        for (int q = 0; q < NLD; ++q) {
            const int idx = tid + 256 * q, row = idx & 63, v = idx >> 6;
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            const bool ok = idx < 64 * NV;
            rx[q] = (ok && t0 + row < T) ? __ldg(reinterpret_cast<const uint4*>(x + (long long)(t0 + row) * xs + c * CL + v * 8)) : z;
            rw[q] = (ok && e0 + row < E) ? __ldg(reinterpret_cast<const uint4*>(wr + (long long)(e0 + row) * H + c * CL + v * 8)) : z;
        }
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int q = 0; q < NLD; ++q) {
            const int idx = tid + 256 * q, row = idx & 63, v = idx >> 6;
            if (idx < 64 * NV) {
                const uint32_t xw[4] = {rx[q].x, rx[q].y, rx[q].z, rx[q].w};
                const uint32_t ww[4] = {rw[q].x, rw[q].y, rw[q].z, rw[q].w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int kk = v * 8 + j;
                    const uint32_t xb = (j & 1) ? (xw[j >> 1] & 0xFFFF0000u) : (xw[j >> 1] << 16);
                    const uint32_t wb = (j & 1) ? (ww[j >> 1] & 0xFFFF0000u) : (ww[j >> 1] << 16);
                    xsm[(buf * CL + kk) * 64 + row] = __uint_as_float(xb);
                    wsm[(buf * CL + kk) * 64 + row] = __uint_as_float(wb);
                }
            }
        }
    };
    pdl_wait();
    pdl_trigger();
    float st[5][16];   // left subtrees waiting at each level
#pragma unroll
    for (int l = 0; l < 5; ++l)
#pragma unroll
        for (int q = 0; q < 16; ++q) st[l][q] = 0.0f;
    float sm[16];
    gload(0);
    sstore(0);
    __syncthreads();
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
        if (i + 1 < 32) gload((int)(__brev((unsigned)(i + 1)) >> 27));
        const float* xb = xsm + (i & 1) * CL * 64 + ty * 4;
        const float* wb = wsm + (i & 1) * CL * 64 + tx * 4;
        float pc[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) pc[q] = 0.0f;
#pragma unroll 8
        for (int kk = 0; kk < CL; ++kk) {
            const float4 xv = *reinterpret_cast<const float4*>(xb + kk * 64);
            const float4 wv = *reinterpret_cast<const float4*>(wb + kk * 64);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) pc[a * 4 + b] = __fmaf_rn(xa[a], wa[b], pc[a * 4 + b]);
        }
        bool carry = true;
#pragma unroll
        for (int l = 0; l < 5; ++l) {
            if (carry) {
                if ((i >> l) & 1) {
#pragma unroll
                    for (int q = 0; q < 16; ++q) pc[q] = __fadd_rn(st[l][q], pc[q]);
                } else {
#pragma unroll
                    for (int q = 0; q < 16; ++q) st[l][q] = pc[q];
                    carry = false;
                }
            }
        }
        if (i == 31) {
#pragma unroll
            for (int q = 0; q < 16; ++q) sm[q] = pc[q];
        }
        if (i + 1 < 32) sstore((i + 1) & 1);
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int t = t0 + ty * 4 + a;
        if (t >= T) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int e = e0 + tx * 4 + b;
            if (e < E) __stcg(logits + (long long)t * E + e, bias ? __fadd_rn(sm[a * 4 + b], bias[e]) : sm[a * 4 + b]);
        }
    }
}

// Shared-expert gate (config 5): one warp per token; s = dot(x[t], g) with the router's arithmetic (lane c sums
// chunk c in ascending k with fp32 fma, xor butterfly 16..1), weight = 1 / (1 + expf(-s)).  Writes the extended
// routing [T][topk + 1]: the token's routed picks, then (shared_id, weight).
__global__ void __launch_bounds__(256) shared_gate_kernel(const __nv_bfloat16* __restrict__ x, long long xs,
                                                          const __nv_bfloat16* __restrict__ g, int T, int H,
                                                          const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                          int topk, int shared_id, int32_t* __restrict__ ids_out,
                                                          float* __restrict__ w_out) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    const int cl = H / 32;
    const uint16_t* xr = reinterpret_cast<const uint16_t*>(x) + (long long)t * xs + lane * cl;
    const uint16_t* gr = reinterpret_cast<const uint16_t*>(g) + lane * cl;
    float acc = 0.0f;
    for (int k = 0; k < cl; ++k)
        acc = __fmaf_rn(__uint_as_float((uint32_t)xr[k] << 16), __uint_as_float((uint32_t)gr[k] << 16), acc);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    const int k1 = topk + 1;
    for (int k = lane; k < topk; k += 32) {
        ids_out[(long long)t * k1 + k] = ids[(long long)t * topk + k];
        w_out[(long long)t * k1 + k] = w[(long long)t * topk + k];
    }
    if (lane == 0) {
        ids_out[(long long)t * k1 + topk] = shared_id;
        w_out[(long long)t * k1 + topk] = 1.0f / (1.0f + expf(-acc));
    }
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int exl3b_shared_gate(const void* x_bf16, int64_t x_stride, const void* g_bf16, int T, int H,
                                           const int32_t* ids, const float* w, int topk, int shared_id,
                                           int32_t* ids_out, float* w_out, void* stream) {
    EXL3B_CHECK(x_bf16 && g_bf16 && ids && w && ids_out && w_out, "exl3b_shared_gate: null pointer");
    EXL3B_CHECK(H % 32 == 0 && H > 0 && topk >= 1 && shared_id >= 0, "exl3b_shared_gate: H % 32 == 0, topk >= 1");
    EXL3B_CHECK(x_stride >= H, "exl3b_shared_gate: row stride must be >= H");
    if (T <= 0) return 0;
    cudaError_t e = launch_k(shared_gate_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, (cudaStream_t)stream,
                             (const __nv_bfloat16*)x_bf16, (long long)x_stride, (const __nv_bfloat16*)g_bf16, T, H, ids, w,
                             topk, shared_id, ids_out, w_out);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    return 0;
}

namespace exl3b {
// Logits only (the fused decode entry selects inside its own kernels): the warp-per-expert kernel for T <= 8.
int router_logits_launch(const void* x_bf16, int64_t x_stride, const void* wr_bf16, const float* bias, int T, int H,
                         int E, float* logits, cudaStream_t s) {
    constexpr int TC = 8;
    if (T < 1 || T > TC) return exl3b_fail(EXL3B_EINVAL, "router logits: 1 <= T <= 8");
    dim3 g1((E + 7) / 8, 1);
    const __nv_bfloat16* xp = (const __nv_bfloat16*)x_bf16;
    const __nv_bfloat16* wp = (const __nv_bfloat16*)wr_bf16;
    cudaError_t e = cudaSuccess;
    switch (H / 32) {
#define RL(CLV) case CLV: e = launch_k(router_logits_kernel<CLV, TC>, g1, dim3(256), 0, s, xp, (long long)x_stride, wp, \
                                       bias, T, H, E, logits, 0, (int*)nullptr, (float*)nullptr, (int*)nullptr); break;
        RL(8) RL(16) RL(24) RL(32) RL(40) RL(48) RL(56) RL(64) RL(80) RL(96) RL(128)
#undef RL
        default: return exl3b_fail(EXL3B_EINVAL, "router logits: unsupported H");
    }
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    return 0;
}
}  // namespace exl3b

// Token count from which the tiled logits kernel runs (below it, the warp-per-expert kernel's many small blocks are
// faster).
constexpr int kRouterTiledMinT = 128;

extern "C" EXL3B_API int exl3b_router_topk(const void* x_bf16, int64_t x_stride, const void* wr_bf16, const float* bias,
                                           int T, int H, int E, int topk, int32_t* ids, float* w, float* logits,
                                           int32_t* counter, void* stream) {
    EXL3B_CHECK(x_bf16 && wr_bf16 && ids && w && logits, "exl3b_router_topk: null pointer");
    EXL3B_CHECK(H % 256 == 0 && H <= 4096, "exl3b_router_topk: H must be a multiple of 256, <= 4096");
    EXL3B_CHECK(E >= 1 && E <= 1024, "exl3b_router_topk: 1 <= E <= 1024");
    EXL3B_CHECK(topk >= 1 && topk <= 32 && topk <= E, "exl3b_router_topk: 1 <= topk <= min(32, E)");
    EXL3B_CHECK(x_stride >= H && ((x_stride * 2) % 16) == 0, "exl3b_router_topk: row stride must be >= H, 16-byte multiple");
    EXL3B_CHECK((((uintptr_t)x_bf16) & 15) == 0 && (((uintptr_t)wr_bf16) & 15) == 0, "exl3b_router_topk: 16-byte alignment");
    if (T <= 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    constexpr int TC = 8;
    dim3 g1((E + 7) / 8, (T + TC - 1) / TC);
    const __nv_bfloat16* xp = (const __nv_bfloat16*)x_bf16;
    const __nv_bfloat16* wp = (const __nv_bfloat16*)wr_bf16;
    int* ctr = (counter && T <= TC) ? counter : nullptr;   // fused selection when every token fits one block
    cudaError_t e = cudaSuccess;
    if (T >= kRouterTiledMinT) {
        const dim3 gt((unsigned)((T + 63) / 64), (unsigned)((E + 63) / 64));
        const int CLv = H / 32;
        const size_t smem = (size_t)4 * CLv * 64 * sizeof(float);
        switch (CLv) {
#define RT(CLV) case CLV: { \
            static int attr_dev = -1; int dev = 0; cudaGetDevice(&dev); \
            if (attr_dev != dev) { \
                e = cudaFuncSetAttribute(router_logits_tiled_kernel<CLV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
                if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e)); \
                attr_dev = dev; } \
            e = launch_k(router_logits_tiled_kernel<CLV>, gt, dim3(256), smem, s, xp, x_stride, wp, bias, T, H, E, logits); \
            break; }
            RT(8) RT(16) RT(24) RT(32) RT(40) RT(48) RT(56) RT(64) RT(80) RT(96) RT(128)
#undef RT
            default: return exl3b_fail(EXL3B_EINVAL, "exl3b_router_topk: unsupported H");
        }
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        e = launch_k(router_topk_kernel, dim3((T + 7) / 8), dim3(256), 0, s, (const float*)logits, T, E, topk, ids, w);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        return 0;
    }
    switch (H / 32) {
#define RL(CLV) case CLV: e = launch_k(router_logits_kernel<CLV, TC>, g1, dim3(256), 0, s, xp, x_stride, wp, bias, T, H, E, \
                                       logits, topk, ids, w, ctr); break;
        RL(8) RL(16) RL(24) RL(32) RL(40) RL(48) RL(56) RL(64) RL(80) RL(96) RL(128)
#undef RL
        default: return exl3b_fail(EXL3B_EINVAL, "exl3b_router_topk: unsupported H");
    }
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    if (ctr) return 0;
    e = launch_k(router_topk_kernel, dim3((T + 7) / 8), dim3(256), 0, s, (const float*)logits, T, E, topk, ids, w);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    return 0;
}
