// exl3b_ep.cu -- expert-parallel prefill: the device side of the token dispatch and combine around the
// NCCL all-to-all exchanges.  The reference runs on one GPU; this is the B200 build's extension of its moe_prefill
// (exl3_moe.a8.sycl:792-828) over G GPUs of one node.
//
// Experts are sharded contiguously: rank d owns ids [d E/G, (d+1) E/G).  A rank's tokens are sent once to every
// rank that owns at least one of their picks:
//   plan    : bits[t] = set of destination ranks of token t; per destination an exclusive scan over tokens gives each
//             (t, d) its row in the send buffer (destination-major, ascending t): pos[t][d] (or -1), counts[d],
//             offs[d];
//   fill    : per send row: source token, and the token's topk picks as the destination's local expert ids (-1 for
//             picks owned by other ranks) with their weights;
//   pack    : send_x[row] = x[send_src[row]] (bf16 rows);
//   combine : out[t] = sum over d = 0..G-1 (ascending) of part[pos[t][d]] (fp32 partial sums returned by the
//             destinations), rounded to the output type.
// The exchange EPPrefill runs (one all-to-all each way, equal splits, no host read of the counts) uses:
//   dispatch  : bits, the per-destination ranks of the tokens, and one record per send row in fixed-capacity blocks:
//               destination d's block is rows [d cap, (d + 1) cap), its first counts[d] rows the tokens that pick d
//               (ascending t), each record [x row (H 16-bit values) | topk local ids (int32) | topk weights (fp32) |
//               padding to 16 bytes]; the block's other rows carry ids -1 (no pick) and weights 0, so the
//               destination runs its MoE over all G cap rows and they cost nothing;
//   combine_h : the combine over fp16 partial sums.
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include "exl3b_launch.h"

namespace exl3b {

__global__ void __launch_bounds__(256) ep_bits_kernel(const int32_t* __restrict__ ids, int T, int topk, int E, int G,
                                                      uint32_t* __restrict__ bits) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const int per = E / G;
    uint32_t b = 0;
    for (int k = 0; k < topk; ++k) {
        const int e = ids[(long long)t * topk + k];
        if (e >= 0 && e < E) b |= 1u << (e / per);
        else if (e != -1) set_error(kErrBounds);
    }
    bits[t] = b;
}

// One block of 1024 threads: tokens in chunks of 1024; per destination d, warp ballots give the in-warp ranks and
// thread d scans the 32 warp counts, carrying across chunks.
// cap > 0: destination d's rows start at d cap (fixed-capacity blocks) instead of after the previous destinations'.
__global__ void __launch_bounds__(1024) ep_scan_kernel(const uint32_t* __restrict__ bits, int T, int G,
                                                       long long* __restrict__ counts, long long* __restrict__ offs,
                                                       int* __restrict__ pos, int cap) {
    __shared__ int wcnt[32][32];
    __shared__ int carry[32];
    __shared__ long long soff[33];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const unsigned lt = (1u << lane) - 1u;
    if (tid < 32) carry[tid] = 0;
    __syncthreads();
    for (int c0 = 0; c0 < T; c0 += 1024) {
        const int t = c0 + tid;
        const uint32_t b = t < T ? bits[t] : 0u;
        for (int d = 0; d < G; ++d) {
            const unsigned m = __ballot_sync(0xffffffffu, (b >> d) & 1u);
            if (lane == 0) wcnt[wid][d] = __popc(m);
        }
        __syncthreads();
        if (tid < G) {
            int s = carry[tid];
            for (int w = 0; w < 32; ++w) { const int v = wcnt[w][tid]; wcnt[w][tid] = s; s += v; }
            carry[tid] = s;
        }
        __syncthreads();
        for (int d = 0; d < G; ++d) {
            const unsigned m = __ballot_sync(0xffffffffu, (b >> d) & 1u);
            if (t < T) pos[(long long)t * G + d] = ((b >> d) & 1u) ? wcnt[wid][d] + __popc(m & lt) : -1;
        }
        __syncthreads();
    }
    if (tid == 0) {
        long long o = 0;
        for (int d = 0; d < G; ++d) { counts[d] = carry[d]; offs[d] = o; soff[d] = o; o += carry[d]; }
        offs[G] = o;
        soff[G] = o;
    }
    __syncthreads();
    for (long long i = tid; i < (long long)T * G; i += blockDim.x) {
        const int p = pos[i];
        if (p >= 0) pos[i] = (int)(p + (cap > 0 ? (long long)(i % G) * cap : soff[i % G]));
    }
}

// Thread per (token, destination): the source token of every used send row.
__global__ void __launch_bounds__(256) ep_src_kernel(const int* __restrict__ pos, int T, int G, int* __restrict__ src) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (long long)T * G) return;
    const int r = pos[q];
    if (r >= 0) src[r] = (int)(q / G);
}

// Block per record row of the fixed-capacity send buffer (see the file header).
__global__ void __launch_bounds__(256) ep_record_kernel(const uint4* __restrict__ x, long long xs16, int H,
                                                        const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                        int topk, int E, int G, int cap,
                                                        const long long* __restrict__ counts,
                                                        const int* __restrict__ src, uint8_t* __restrict__ send,
                                                        long long rec) {
    const int r = blockIdx.x;
    const int d = r / cap, j = r - d * cap;
    const bool valid = j < counts[d];
    const int t = valid ? src[r] : -1;
    uint8_t* row = send + (long long)r * rec;
    if (valid) {
        uint4* xo = reinterpret_cast<uint4*>(row);
        for (int c = threadIdx.x; c < H / 8; c += blockDim.x) xo[c] = x[(long long)t * xs16 + c];
    }
    int32_t* io = reinterpret_cast<int32_t*>(row + 2 * (long long)H);
    float* wo = reinterpret_cast<float*>(row + 2 * (long long)H + 4 * topk);
    const int per = E / G;
    for (int k = threadIdx.x; k < topk; k += blockDim.x) {
        int id = -1;
        float wk = 0.0f;
        if (valid) {
            const int e = ids[(long long)t * topk + k];
            if (e >= 0 && e < E && e / per == d) { id = e - d * per; wk = w[(long long)t * topk + k]; }
        }
        io[k] = id;
        wo[k] = wk;
    }
}

// Thread per (token, destination).
__global__ void __launch_bounds__(256) ep_fill_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                      int T, int topk, int E, int G, const int* __restrict__ pos,
                                                      int32_t* __restrict__ send_src, int32_t* __restrict__ send_ids,
                                                      float* __restrict__ send_w) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (long long)T * G) return;
    const int t = (int)(q / G), d = (int)(q % G);
    const int row = pos[q];
    if (row < 0) return;
    const int per = E / G;
    send_src[row] = t;
    for (int k = 0; k < topk; ++k) {
        const int e = ids[(long long)t * topk + k];
        const bool mine = e >= 0 && e < E && e / per == d;
        send_ids[(long long)row * topk + k] = mine ? e - d * per : -1;
        send_w[(long long)row * topk + k] = mine ? w[(long long)t * topk + k] : 0.0f;
    }
}

__global__ void __launch_bounds__(256) ep_pack_kernel(const uint4* __restrict__ x, long long xs16, int n_rows, int h16,
                                                      const int32_t* __restrict__ send_src, uint4* __restrict__ out) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (long long)n_rows * h16) return;
    const int row = (int)(q / h16), c = (int)(q % h16);
    out[q] = x[(long long)send_src[row] * xs16 + c];
}

__global__ void __launch_bounds__(256) ep_combine_kernel(const float* __restrict__ part, const int* __restrict__ pos,
                                                         int T, int G, int H, void* out, long long os, int out_kind) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int h4 = H / 4;
    if (q >= (long long)T * h4) return;
    const int t = (int)(q / h4), c = (int)(q % h4) * 4;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < G; ++d) {
        const int row = pos[(long long)t * G + d];
        if (row < 0) continue;
        const float4 v = *reinterpret_cast<const float4*>(part + (long long)row * H + c);
        s[0] += v.x; s[1] += v.y; s[2] += v.z; s[3] += v.w;
    }
    const long long o = (long long)t * os + c;
    if (out_kind == 2) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o) = make_float4(s[0], s[1], s[2], s[3]);
    } else if (out_kind == 1) {
        __nv_bfloat162 a = __floats2bfloat162_rn(s[0], s[1]), b = __floats2bfloat162_rn(s[2], s[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + o) = u;
    } else {
        __half2 a = __floats2half2_rn(s[0], s[1]), b = __floats2half2_rn(s[2], s[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(out) + o) = u;
    }
}

// As ep_combine_kernel, over fp16 partial sums (summed in fp32).
__global__ void __launch_bounds__(256) ep_combine_h_kernel(const __half* __restrict__ part, const int* __restrict__ pos,
                                                           int T, int G, int H, void* out, long long os, int out_kind) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int h4 = H / 4;
    if (q >= (long long)T * h4) return;
    const int t = (int)(q / h4), c = (int)(q % h4) * 4;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < G; ++d) {
        const int row = pos[(long long)t * G + d];
        if (row < 0) continue;
        const uint2 u = *reinterpret_cast<const uint2*>(part + (long long)row * H + c);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        s[0] += a.x; s[1] += a.y; s[2] += b.x; s[3] += b.y;
    }
    const long long o = (long long)t * os + c;
    if (out_kind == 2) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o) = make_float4(s[0], s[1], s[2], s[3]);
    } else if (out_kind == 1) {
        __nv_bfloat162 a = __floats2bfloat162_rn(s[0], s[1]), b = __floats2bfloat162_rn(s[2], s[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + o) = u;
    } else {
        __half2 a = __floats2half2_rn(s[0], s[1]), b = __floats2half2_rn(s[2], s[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(out) + o) = u;
    }
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int64_t exl3b_ep_record_bytes(int H, int topk) {
    if (H <= 0 || topk <= 0) return 0;
    return ((int64_t)2 * H + (int64_t)8 * topk + 15) / 16 * 16;
}

extern "C" EXL3B_API int exl3b_ep_dispatch(const void* x, int64_t x_stride, const int32_t* ids, const float* w, int T,
                                           int topk, int E, int G, int H, int cap, uint32_t* bits, int64_t* counts,
                                           int32_t* pos, int32_t* src, void* send, void* stream) {
    EXL3B_CHECK(counts && send && (T == 0 || (x && ids && w && bits && pos && src)), "exl3b_ep_dispatch: null pointer");
    EXL3B_CHECK(G >= 1 && G <= 32 && E >= G && E % G == 0 && topk >= 1 && T >= 0 && cap >= T && cap >= 1,
                "exl3b_ep_dispatch: 1 <= G <= 32 ranks dividing the experts evenly, T <= cap");
    EXL3B_CHECK(H % 8 == 0 && x_stride % 8 == 0 && (T == 0 || (((uintptr_t)x) & 15) == 0) && (((uintptr_t)send) & 15) == 0,
                "exl3b_ep_dispatch: 16-byte aligned rows of 16-bit values, H % 8 == 0");
    cudaStream_t s = (cudaStream_t)stream;
    if (T > 0) {
        cudaError_t e = launch_k(ep_bits_kernel, dim3((unsigned)((T + 255) / 256)), dim3(256), 0, s, ids, T, topk, E, G, bits);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    }
    ep_scan_kernel<<<1, 1024, 0, s>>>(bits, T, G, (long long*)counts, (long long*)counts + G, pos, cap);
    if (T > 0) {
        const long long n = (long long)T * G;
        ep_src_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(pos, T, G, src);
    }
    const long long rec = exl3b_ep_record_bytes(H, topk);
    ep_record_kernel<<<(unsigned)((long long)G * cap), 256, 0, s>>>((const uint4*)x, (long long)(x_stride / 8), H, ids, w,
                                                                   topk, E, G, cap, (const long long*)counts, src,
                                                                   (uint8_t*)send, rec);
    return exl3b_launch_status("exl3b_ep_dispatch");
}

extern "C" EXL3B_API int exl3b_ep_combine_h(const void* part, const int32_t* pos, int T, int G, int H, void* out,
                                            int64_t out_stride, int out_kind, void* stream) {
    EXL3B_CHECK(pos && out && (T == 0 || part), "exl3b_ep_combine_h: null pointer");
    EXL3B_CHECK(H % 4 == 0 && out_stride % 4 == 0 && out_kind >= 0 && out_kind <= 2, "exl3b_ep_combine_h: H % 4 == 0");
    if (T <= 0) return 0;
    long long n = (long long)T * (H / 4);
    ep_combine_h_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (const __half*)part, pos, T, G, H, out, (long long)out_stride, out_kind);
    return exl3b_launch_status("exl3b_ep_combine_h");
}

extern "C" EXL3B_API int exl3b_ep_plan(const int32_t* ids, const float* w, int T, int topk, int E, int G,
                                       uint32_t* bits, int64_t* counts, int64_t* offs, int32_t* pos, int32_t* send_src,
                                       int32_t* send_ids, float* send_w, void* stream) {
    EXL3B_CHECK(ids && w && bits && counts && offs && pos && send_src && send_ids && send_w, "exl3b_ep_plan: null pointer");
    EXL3B_CHECK(G >= 1 && G <= 32 && E >= G && E % G == 0 && topk >= 1 && T >= 0,
                "exl3b_ep_plan: 1 <= G <= 32 ranks dividing the experts evenly");
    cudaStream_t s = (cudaStream_t)stream;
    if (T > 0) {
        cudaError_t e = launch_k(ep_bits_kernel, dim3((unsigned)((T + 255) / 256)), dim3(256), 0, s, ids, T, topk, E, G, bits);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    }
    ep_scan_kernel<<<1, 1024, 0, s>>>(bits, T, G, (long long*)counts, (long long*)offs, pos, 0);
    if (T > 0) {
        long long n = (long long)T * G;
        ep_fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ids, w, T, topk, E, G, pos, send_src, send_ids, send_w);
    }
    return exl3b_launch_status("exl3b_ep_plan");
}

extern "C" EXL3B_API int exl3b_ep_pack(const void* x, int64_t x_stride, int H, const int32_t* send_src, int n_rows,
                                       void* send_x, void* stream) {
    EXL3B_CHECK(x && send_src && send_x, "exl3b_ep_pack: null pointer");
    EXL3B_CHECK(H % 8 == 0 && x_stride % 8 == 0 && (((uintptr_t)x) & 15) == 0 && (((uintptr_t)send_x) & 15) == 0,
                "exl3b_ep_pack: 16-byte aligned rows of 16-bit values, H % 8 == 0");
    if (n_rows <= 0) return 0;
    const int h16 = H / 8;
    long long n = (long long)n_rows * h16;
    ep_pack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)x, (long long)(x_stride / 8), n_rows, h16, send_src, (uint4*)send_x);
    return exl3b_launch_status("exl3b_ep_pack");
}

extern "C" EXL3B_API int exl3b_ep_combine(const float* part, const int32_t* pos, int T, int G, int H, void* out,
                                          int64_t out_stride, int out_kind, void* stream) {
    EXL3B_CHECK(pos && out, "exl3b_ep_combine: null pointer");   // part may be NULL when no token was sent
    EXL3B_CHECK(H % 4 == 0 && out_stride % 4 == 0 && out_kind >= 0 && out_kind <= 2, "exl3b_ep_combine: H % 4 == 0");
    if (T <= 0) return 0;
    long long n = (long long)T * (H / 4);
    ep_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(part, pos, T, G, H, out,
                                                                                   (long long)out_stride, out_kind);
    return exl3b_launch_status("exl3b_ep_combine");
}
