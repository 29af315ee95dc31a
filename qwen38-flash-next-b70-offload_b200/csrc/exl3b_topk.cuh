// exl3b_topk.cuh -- the router's top-k selection (one warp per token), shared by the router kernels and the routed
// decode kernels (each file compiles its own copy, within its kernels' register limits).
//   top-k: largest logits, ties to the lower expert id, descending order;
//   w_i = expf(l_i - l_0) / sum_j expf(l_j - l_0) (softmax renormalised over the selection, summed in selection order).
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace exl3b {

// One warp per token: top-k by repeated warp argmax (ties -> lower id), then the renormalised softmax.  MAXJ values
// per lane (E <= 32 MAXJ): instantiated for E <= 512 (16) and E <= 1024 (32).
template <int MAXJ>
static __device__ __forceinline__ void topk_argmax_rounds(const float* __restrict__ logits, int t, int E, int topk,
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

// Order-preserving key of a logit: larger float -> larger unsigned key (-0 counted as +0, as the float compare does).
static __device__ __forceinline__ uint32_t logit_key(float v) {
    const uint32_t b = __float_as_uint(v + 0.0f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Top-k of one token's E logits by one warp in a fixed number of steps (E a multiple of 32, E <= 512, topk <= 32):
// the topk-th largest of the 32 lanes' maxima is a threshold with at least topk logits at or above it; those
// candidates (at most 32, else the function returns false having written nothing) are ranked against each other
// (value descending, ties to the lower id) and the ranks give the selection.  Same ids, order and weights as
// topk_warp_n: the ordering is the same strict total order, and the weights are computed from the same values with
// the same expressions in the same order.  NaN logits return false.  cand: 32 (key, id) pairs of shared memory.
static __device__ __forceinline__ bool topk_threshold(const float* __restrict__ logits, int t, int E, int topk,
                                                      int* __restrict__ ids, float* __restrict__ w, bool store,
                                                      uint2* cand) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int nj = E / 32;
    uint32_t key[16];
    bool nan = false;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float v = j < nj ? __ldcg(logits + (long long)t * E + lane + 32 * j) : 0.0f;
        nan |= v != v;
        key[j] = j < nj ? logit_key(v) : 0u;   // 0: below every real key (-inf maps to 0x007FFFFF)
    }
    if (__any_sync(FULL, nan)) return false;
    uint32_t m = key[0];
#pragma unroll
    for (int j = 1; j < 16; ++j) m = max(m, key[j]);
    // rank of this lane's maximum among the 32 maxima (ties to the lower lane); the lane of rank topk - 1 holds the
    // threshold
    int r = 0;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
        const uint32_t o = __shfl_sync(FULL, m, l);
        r += (o > m || (o == m && l < lane)) ? 1 : 0;
    }
    const unsigned tl = __ballot_sync(FULL, r == topk - 1);
    const uint32_t th = __shfl_sync(FULL, m, __ffs(tl) - 1);
    int c = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) c += key[j] >= th ? 1 : 0;
    int x = c;   // inclusive scan of the candidate counts
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) { const int y = __shfl_up_sync(FULL, x, o); if (lane >= o) x += y; }
    const int n = __shfl_sync(FULL, x, 31);
    if (n > 32) return false;
    int p = x - c;
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (key[j] >= th) cand[p++] = make_uint2(key[j], (uint32_t)(lane + 32 * j));
    __syncwarp();
    const uint2 me = lane < n ? cand[lane] : make_uint2(0u, 0xFFFFFFFFu);
    int rk = 0;
    for (int l = 0; l < n; ++l) {
        const uint2 o = cand[l];   // broadcast read
        rk += (o.x > me.x || (o.x == me.x && o.y < me.y)) ? 1 : 0;
    }
    __syncwarp();
    if (lane < n && rk < topk) cand[rk] = me;   // selections in order (ranks are distinct)
    __syncwarp();
    float sv = 0.0f;
    int se = 0;
    if (lane < topk) {
        const uint2 s = cand[lane];
        const uint32_t b = (s.x & 0x80000000u) ? (s.x & 0x7FFFFFFFu) : ~s.x;
        sv = __uint_as_float(b);
        se = (int)s.y;
    }
    const float s0 = __shfl_sync(FULL, sv, 0);
    float ex = (lane < topk) ? expf(sv - s0) : 0.0f;
    float ssum = 0.0f;
    for (int k = 0; k < topk; ++k) ssum += __shfl_sync(FULL, ex, k);
    if (lane < topk && store) {
        ids[(long long)t * topk + lane] = se;
        w[(long long)t * topk + lane] = ex / ssum;
    }
    __syncwarp();
    return true;
}

// Out-of-line copies (the router kernels run the same code once early, without storing, to warm it).
template <int MAXJ>
static __device__ __noinline__ void topk_warp_n(const float* __restrict__ logits, int t, int E, int topk,
                                                int* __restrict__ ids, float* __restrict__ w, bool store) {
    topk_argmax_rounds<MAXJ>(logits, t, E, topk, ids, w, store);
}
static __device__ __noinline__ bool topk_warp_thresh(const float* __restrict__ logits, int t, int E, int topk,
                                                     int* __restrict__ ids, float* __restrict__ w, bool store,
                                                     uint2* cand) {
    return topk_threshold(logits, t, E, topk, ids, w, store, cand);
}

static __device__ __forceinline__ void topk_warp(const float* __restrict__ logits, int t, int E, int topk,
                                                 int* __restrict__ ids, float* __restrict__ w, uint2* cand = nullptr) {
    if (cand && E % 32 == 0 && E <= 512 && topk <= 32 && topk_warp_thresh(logits, t, E, topk, ids, w, true, cand))
        return;
    if (E <= 512) topk_warp_n<16>(logits, t, E, topk, ids, w, true);
    else topk_warp_n<32>(logits, t, E, topk, ids, w, true);
}

// Inlined into the caller (its register budget): for kernels that select once per block.
static __device__ __forceinline__ void topk_warp_inl(const float* __restrict__ logits, int t, int E, int topk,
                                                     int* __restrict__ ids, float* __restrict__ w, uint2* cand) {
    if (E % 32 == 0 && E <= 512 && topk <= 32 && topk_threshold(logits, t, E, topk, ids, w, true, cand)) return;
    if (E <= 512) topk_argmax_rounds<16>(logits, t, E, topk, ids, w, true);
    else topk_argmax_rounds<32>(logits, t, E, topk, ids, w, true);
}

}  // namespace exl3b
