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

namespace exl3b {

// One warp per token: top-k by repeated warp argmax (ties -> lower id), then the renormalised softmax.  MAXJ values
// per lane (E <= 32 MAXJ): instantiated for E <= 512 (16) and E <= 1024 (32).  Not inlined: the router kernel runs
// the same code once early with store = false (see router_logits_kernel).
template <int MAXJ>
__device__ __noinline__ void topk_warp_n(const float* __restrict__ logits, int t, int E, int topk,
                                         int* __restrict__ ids, float* __restrict__ w, bool store) {
    const int lane = threadIdx.x & 31;
    float v[MAXJ];
    const int nj = (E + 31) / 32;
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) {
        int e = lane + 32 * j;
        v[j] = (j < nj && e < E) ? __ldcg(logits + (long long)t * E + e) : -INFINITY;
    }
    unsigned used = 0;   // bit j: expert lane + 32 j already selected
    float sv = 0.0f, s0 = 0.0f, ssum = 0.0f;
    int se = 0;
    for (int k = 0; k < topk; ++k) {
        float bv = -INFINITY;
        int be = 0x7FFFFFFF;
#pragma unroll
        for (int j = 0; j < MAXJ; ++j) {
            int e = lane + 32 * j;
            bool ok = j < nj && e < E && !((used >> j) & 1u);
            if (ok && (v[j] > bv || (v[j] == bv && e < be))) { bv = v[j]; be = e; }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
        }
        if ((be & 31) == lane) used |= 1u << (be >> 5);
        if (k == 0) s0 = bv;
        if (lane == k) { sv = bv; se = be; }   // lane k keeps the k-th selection
    }
    // w_k = expf(l_k - l_0) / sum_j expf(l_j - l_0), the sum in selection order
    float ex = (lane < topk) ? expf(sv - s0) : 0.0f;
    for (int k = 0; k < topk; ++k) ssum += __shfl_sync(0xffffffffu, ex, k);
    if (lane < topk && store) {
        ids[(long long)t * topk + lane] = se;
        w[(long long)t * topk + lane] = ex / ssum;
    }
}

__device__ __forceinline__ void topk_warp(const float* __restrict__ logits, int t, int E, int topk,
                                          int* __restrict__ ids, float* __restrict__ w) {
    if (E <= 512) topk_warp_n<16>(logits, t, E, topk, ids, w, true);
    else topk_warp_n<32>(logits, t, E, topk, ids, w, true);
}

__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int T, int E, int topk,
                                                          int* __restrict__ ids, float* __restrict__ w) {
    pdl_wait();
    pdl_trigger();
    int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    topk_warp(logits, t, E, topk, ids, w);
}

// One warp per expert, 8 experts per block; blockIdx.y = token chunk of TC tokens.  Lane c owns chunk c:
// its slice of Wr[e] stays in registers across the chunk's tokens.
template <int CL, int TC>
__global__ void __launch_bounds__(256) router_logits_kernel(const __nv_bfloat16* __restrict__ x, long long xs,
                                                            const __nv_bfloat16* __restrict__ wr,
                                                            const float* __restrict__ bias, int T, int H, int E,
                                                            float* __restrict__ logits, int topk, int* __restrict__ ids,
                                                            float* __restrict__ w, int* counter) {
    __shared__ int sh_last;
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
        if (E <= 512) topk_warp_n<16>(logits, 0, E, topk, ids, w, T < 0);
        else topk_warp_n<32>(logits, 0, E, topk, ids, w, T < 0);
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
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        int old = atomicAdd(counter, 1);
        sh_last = old == (int)(gridDim.x * gridDim.y) - 1;
    }
    __syncthreads();
    if (!sh_last) return;
    __threadfence();
    int t = threadIdx.x >> 5;
    if (t < T) topk_warp(logits, t, E, topk, ids, w);
    if (threadIdx.x == 0) *counter = 0;
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
