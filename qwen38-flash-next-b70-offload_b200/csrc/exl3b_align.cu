// exl3b_align.cu -- routing tables: picks bucketed by expert (reference launch_align, exl3_moe.a8.sycl:639-680,
// outputs laid out as make_route :744-757).
//
// The reference places picks with work-group atomics, so the order inside an expert varies run to run.  Here the
// sort is a stable counting sort over any number of picks (ascending pick index inside an expert), in three
// launches: per-block expert histograms, one block that scans them, and a placement pass.
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"

namespace exl3b {

constexpr int kAlignBlock = 1024;

__global__ void __launch_bounds__(kAlignBlock) align_hist_kernel(const int32_t* __restrict__ ids, int P, int E,
                                                                 int* __restrict__ bc) {
    __shared__ int h[1024];
    for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
    __syncthreads();
    int i = blockIdx.x * kAlignBlock + threadIdx.x;
    if (i < P) {
        int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(&h[e], 1);
        else if (e != -1) set_error(kErrBounds);   // -1: no pick (expert-parallel ranks), skipped
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) bc[(size_t)blockIdx.x * E + e] = h[e];
}

struct AlignOut {
    int* act_expert; int* act_start; int* act_cnt; int* act_pstart; int* n_act;
    int* pair_tok; int* pair_of; int* blk_a; int* n_blk; float* pair_w;
    int A, mxb;
};

__global__ void __launch_bounds__(kAlignBlock) align_scan_kernel(int* __restrict__ bc, int nblk, int E, int pad,
                                                                 int* __restrict__ start, AlignOut o) {
    __shared__ int sh_warp[32];
    const int e = threadIdx.x, lane = e & 31, wid = e >> 5;
    int c = 0;
    if (e < E) {
        // per-block offsets inside the expert (exclusive over blocks); the counts are read 16 blocks at a time so
        // that one L2 round trip covers 16 of them
        constexpr int kB = 16;
        for (int b0 = 0; b0 < nblk; b0 += kB) {
            int v[kB];
#pragma unroll
            for (int j = 0; j < kB; ++j) v[j] = b0 + j < nblk ? bc[(size_t)(b0 + j) * E + e] : 0;
#pragma unroll
            for (int j = 0; j < kB; ++j)
                if (b0 + j < nblk) {
                    bc[(size_t)(b0 + j) * E + e] = c;
                    c += v[j];
                }
        }
    }
    int pc = (c + pad - 1) / pad * pad;
    int act = c > 0 ? 1 : 0;
    // three exclusive scans over experts: start (c), active index (act), padded start (pc)
    int vals[3] = {c, act, pc}, pre[3], tot[3];
#pragma unroll
    for (int q = 0; q < 3; ++q) {
        int x = vals[q];
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) { int y = __shfl_up_sync(0xffffffffu, x, s); if (lane >= s) x += y; }
        if (lane == 31) sh_warp[wid] = x;
        __syncthreads();
        if (wid == 0) {
            int t = sh_warp[lane];
#pragma unroll
            for (int s = 1; s < 32; s <<= 1) { int y = __shfl_up_sync(0xffffffffu, t, s); if (lane >= s) t += y; }
            sh_warp[lane] = t;
        }
        __syncthreads();
        pre[q] = (wid ? sh_warp[wid - 1] : 0) + x - vals[q];
        tot[q] = sh_warp[31];
        __syncthreads();
    }
    if (e < E) {
        start[e] = pre[0];
        if (act) {
            int ai = pre[1];
            if (ai < o.A) {
                o.act_expert[ai] = e; o.act_start[ai] = pre[0]; o.act_cnt[ai] = c; o.act_pstart[ai] = pre[2];
            }
            for (int j = 0; j < pc / pad; ++j) {
                int b = pre[2] / pad + j;
                if (b < o.mxb) o.blk_a[b] = ai;
            }
        }
    }
    if (e == 0) { o.n_act[0] = tot[1]; o.n_blk[0] = tot[2] / pad; }
}

__global__ void __launch_bounds__(kAlignBlock) align_place_kernel(const int32_t* __restrict__ ids,
                                                                  const float* __restrict__ w, int P, int topk, int E,
                                                                  const int* __restrict__ bc,
                                                                  const int* __restrict__ start, AlignOut o) {
    __shared__ int run[1024];   // picks of each expert already placed by earlier warps of this block
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int e = threadIdx.x; e < E; e += blockDim.x) run[e] = 0;
    __syncthreads();
    int i = blockIdx.x * kAlignBlock + threadIdx.x;
    int e = (i < P) ? ids[i] : -1;
    bool ok = e >= 0 && e < E;
    unsigned peers = __match_any_sync(0xffffffffu, ok ? e : -1);
    int rank = __popc(peers & ((1u << lane) - 1u));
    int leader_last = 31 - __clz(peers);   // highest lane of the group updates the running count
    if (i < P && !ok) o.pair_of[i] = -1;   // not placed: the combine skips it
    // the pick's global base (expert start + this block's offset) and weight, loaded before the ordered loop
    const int base = ok ? start[e] + bc[(size_t)blockIdx.x * E + e] + rank : 0;
    const float wi = ok ? w[i] : 0.0f;
    for (int s = 0; s < 32; ++s) {
        if (wid == s && ok) {
            int pos = base + run[e];
            o.pair_tok[pos] = i / topk;
            o.pair_w[pos] = wi;
            o.pair_of[i] = pos;
        }
        __syncthreads();
        if (wid == s && ok && lane == leader_last) run[e] += __popc(peers);
        __syncthreads();
    }
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int64_t exl3b_align_scratch(int P, int E) {
    int nblk = (P + kAlignBlock - 1) / kAlignBlock;
    return (int64_t)((size_t)nblk * E + E + 64) * 4;
}

extern "C" EXL3B_API int exl3b_align(const int32_t* ids, const float* w, int P, int topk, int E, int pad, int32_t* ib,
                                     float* pair_w, int A, int mxb, void* scratch, int64_t scratch_bytes, void* stream) {
    EXL3B_CHECK(E >= 1 && E <= 1024 && pad >= 1 && topk >= 1 && P >= 0, "exl3b_align: bad sizes");
    EXL3B_CHECK(A == (P < E ? P : E) && mxb == (P + pad - 1) / pad + A, "exl3b_align: A / mxb do not match P, E, pad");
    EXL3B_CHECK(ids && w && ib && pair_w && scratch, "exl3b_align: null pointer");
    EXL3B_CHECK(scratch_bytes >= exl3b_align_scratch(P, E), "exl3b_align: scratch too small");
    AlignOut o;
    o.act_expert = ib; o.act_start = ib + A; o.act_cnt = ib + 2 * A; o.act_pstart = ib + 3 * A; o.n_act = ib + 4 * A;
    o.pair_tok = ib + 4 * A + 1; o.pair_of = o.pair_tok + P; o.blk_a = o.pair_of + P + 16; o.n_blk = o.blk_a + mxb;
    o.pair_w = pair_w; o.A = A; o.mxb = mxb;
    cudaStream_t s = (cudaStream_t)stream;
    int nblk = (P + kAlignBlock - 1) / kAlignBlock;
    int* bc = (int*)scratch;
    int* start = bc + (size_t)nblk * E;
    if (nblk > 0) align_hist_kernel<<<nblk, kAlignBlock, 0, s>>>(ids, P, E, bc);
    align_scan_kernel<<<1, kAlignBlock, 0, s>>>(bc, nblk, E, pad, start, o);
    if (nblk > 0) align_place_kernel<<<nblk, kAlignBlock, 0, s>>>(ids, w, P, topk, E, bc, start, o);
    return exl3b_launch_status("exl3b_align");
}
