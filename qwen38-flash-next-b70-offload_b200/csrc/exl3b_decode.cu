// exl3b_decode.cu -- routed-MoE decode path (few tokens): the reference's GateUpKernel / DownKernel / CombineKernel
// (exl3_moe.a8.sycl:121-395) re-designed for sm_100a.
//
// Work is grouped by DISTINCT expert (an "entry" = one expert and up to 8 of its picks), so an expert picked by
// several tokens is streamed once.  Each warp owns a unit = (entry, projection, 128-column block, 128-row k block)
// = 8 k-rows x 8 tiles.  Lane l decodes its 8 values of each tile straight into an mma.sync A fragment of W^T
// (exl3b_common.cuh) and one m16n8k16 per tile multiplies it with the 8-token Hadamard-domain activation block
// (fp32 accumulate).  Split-K partials go to a small L2-resident buffer; the last warp to finish a column block
// (atomic arrival counter, no waiting) reduces them in fixed order and runs the epilogue, so results do not depend
// on scheduling:
//   gate/up epilogue (:239-256): g = fp16(FWHT(g) r svh_g), u likewise, a = fp16(SiLU(g) u), a = fp16(a suh_d),
//                                abuf = fp16(FWHT(a) r)
//   down epilogue   (:355-364): y = FWHT(v) (r w) svh_d (fp32)
//   combine         (:387-394): out[m] = sum_k y[m,k] in fixed k order, done by the last column block to finish.
// Picks with weight exactly 0 (tier-masked picks) contribute exactly zero and are skipped (flag bit 0).
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include <algorithm>

namespace exl3b {

constexpr int kTokPerEnt = 8;   // mma n dimension

struct DecodeArgs {
    const void* x; long long xs; int x_bf16;
    const int32_t* ids; const float* w; int M; int topk;
    const int64_t* ptrs; const int32_t* kinfo;
    int H, I, K, E;
    void* out; long long os; int out_bf16;
    int skip_zero;
    // workspace
    int* ent_expert; int* ent_n; int* ent_tok; float* ent_w; int* ent_pick; int* n_ent;
    int* tok_cnt; int* pick_act;
    int* cnt_gu; int* cnt_d; int* cnt_c;
    __half* abuf; float* part_gu; float* part_d; float* y;
    int maxent;
};

__device__ __forceinline__ void expert_k(const DecodeArgs& a, int e, int& kg, int& ku, int& kd) {
    if (a.kinfo) { int v = a.kinfo[e]; kg = v & 15; ku = (v >> 4) & 15; kd = (v >> 8) & 15; }
    else { kg = ku = kd = a.K; }
}

// ------------------------------------------------------------------------------------------------ route prep
// One block: zero the arrival counters, group active picks by expert (ascending id, picks in ascending index),
// count active picks per token and zero the output rows of tokens with none.
__global__ void __launch_bounds__(1024) route_prep_kernel(DecodeArgs a) {
    __shared__ int cnt[1024];
    __shared__ int sh_warp[32];
    const int tid = threadIdx.x, npairs = a.M * a.topk;
    const int nbI = a.I / 128, nbH = a.H / 128;
    for (int i = tid; i < a.maxent * nbI; i += blockDim.x) a.cnt_gu[i] = 0;
    for (int i = tid; i < a.maxent * nbH; i += blockDim.x) a.cnt_d[i] = 0;
    for (int i = tid; i < a.M * nbH; i += blockDim.x) a.cnt_c[i] = 0;
    for (int e = tid; e < a.E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < npairs; i += blockDim.x) {
        int e = a.ids[i];
        bool act = (e >= 0 && e < a.E) && !(a.skip_zero && a.w[i] == 0.0f);
        if ((e < 0 || e >= a.E)) set_error(kErrBounds);
        a.pick_act[i] = act ? 1 : 0;
        if (act) atomicAdd(&cnt[e], 1);
    }
    for (int m = tid; m < a.M; m += blockDim.x) {
        int c = 0;
        for (int k = 0; k < a.topk; ++k) {
            int i = m * a.topk + k;
            int e = a.ids[i];
            c += ((e >= 0 && e < a.E) && !(a.skip_zero && a.w[i] == 0.0f)) ? 1 : 0;
        }
        a.tok_cnt[m] = c;
    }
    __syncthreads();
    // entries per expert (E <= 1024: one expert per thread), exclusive scan
    int e = tid;
    int n = (e < a.E) ? cnt[e] : 0;
    int ne = (n + kTokPerEnt - 1) / kTokPerEnt;
    int lane = tid & 31, wid = tid >> 5;
    int x = ne;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) { int y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
    if (lane == 31) sh_warp[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int s = sh_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) { int y = __shfl_up_sync(0xffffffffu, s, o); if (lane >= o) s += y; }
        sh_warp[lane] = s;
    }
    __syncthreads();
    int base = (wid ? sh_warp[wid - 1] : 0) + x - ne;
    if (tid == 0) a.n_ent[0] = sh_warp[31];
    if (n > 0) {
        int j = 0;
        for (int i = 0; i < npairs && j < n; ++i) {
            if (a.ids[i] != e || !a.pick_act[i]) continue;
            int en = base + j / kTokPerEnt, s = j % kTokPerEnt;
            if (s == 0) { a.ent_expert[en] = e; a.ent_n[en] = min(kTokPerEnt, n - j); }
            a.ent_tok[en * kTokPerEnt + s] = i / a.topk;
            a.ent_w[en * kTokPerEnt + s] = a.w[i];
            a.ent_pick[en * kTokPerEnt + s] = i;
            ++j;
        }
    }
    // tokens without an active pick: zero output row
    for (int m = 0; m < a.M; ++m) {
        if (a.tok_cnt[m] != 0) continue;
        for (int c = tid; c < a.H; c += blockDim.x) {
            if (a.out_bf16 == 2) reinterpret_cast<float*>(a.out)[(long long)m * a.os + c] = 0.0f;
            else if (a.out_bf16) reinterpret_cast<__nv_bfloat16*>(a.out)[(long long)m * a.os + c] = __float2bfloat16(0.0f);
            else reinterpret_cast<__half*>(a.out)[(long long)m * a.os + c] = __float2half(0.0f);
        }
    }
}

// ------------------------------------------------------------------------------------------------ tile strip
// acc[jj] += W^T(tile jj of an 8-tile strip) * B for `rows` consecutive k-rows.  rowp(r) = first word of the strip's
// first PLANAR4 group in k-row r; the strip's second group follows at +4*8K words.  Bfrag(r) gives the 16x8 fp16 B
// fragment (b0, b1) of k-row r.
template <int K, class RowPtr, class BFrag>
__device__ __forceinline__ void strip_mma(float acc[8][4], int rows, RowPtr rowp, BFrag bfrag, const LaneWin<K>& lw) {
    constexpr int W = Geo<K>::W, G = Geo<K>::G;
    uint32_t wa[8], wb[8], wc[8];
    auto load = [&](int r) {
        const uint32_t* p = rowp(r);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            const uint32_t* gp = p + (jj >> 2) * 4 * W + (jj & 3) * G;
            wa[jj] = __ldg(gp + lw.oA);
            wb[jj] = __ldg(gp + lw.oB);
            wc[jj] = LaneWin<K>::kNeedC ? __ldg(gp + lw.oC) : 0u;
        }
    };
    load(0);
    for (int r = 0; r < rows; ++r) {
        uint32_t ca[8], cb[8], cc[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) { ca[jj] = wa[jj]; cb[jj] = wb[jj]; cc[jj] = wc[jj]; }
        if (r + 1 < rows) load(r + 1);
        uint32_t b0, b1;
        bfrag(r, b0, b1);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
            uint32_t f[4];
            decode8<K>(ca[jj], cb[jj], cc[jj], lw.p0, f);
            mma16816(acc[jj], f, b0, b1);
        }
    }
}

// ------------------------------------------------------------------------------------------------ gate|up
template <int K>
__device__ void gu_unit(const DecodeArgs& a, int ent, int proj, int nb, int kb, __half* xs /* [8][128] */) {
    const int lane = threadIdx.x & 31;
    const int e = a.ent_expert[ent], ntok = a.ent_n[ent];
    int kg, ku, kd;
    expert_k(a, e, kg, ku, kd);
    const Geom gm{a.H, a.I, kg, ku, kd};
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(a.ptrs[e]);
    const int nKB = a.H / 128, nbI = a.I / 128;
    // input Hadamard of this 128-block for the entry's tokens (exl3_moe.a8.sycl:179-195)
    const __half* suh = reinterpret_cast<const __half*>(blob + gm.off_suh_g() + (size_t)proj * a.H * 2) + kb * 128;
    float su[4];
    {
        uint2 sv = *reinterpret_cast<const uint2*>(suh + 4 * lane);
        const __half* sh = reinterpret_cast<const __half*>(&sv);
#pragma unroll
        for (int j = 0; j < 4; ++j) su[j] = __half2float(sh[j]);
    }
    for (int t = 0; t < kTokPerEnt; ++t) {
        uint2 o = make_uint2(0u, 0u);
        if (t < ntok) {
            int tok = a.ent_tok[ent * kTokPerEnt + t];
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = rn16(load_act(a.x, a.x_bf16, (size_t)tok * a.xs + kb * 128 + 4 * lane + j) * su[j]);
            fwht128_warp(v, lane);
            __half2 h0 = __floats2half2_rn(v[0] * kRsqrt128, v[1] * kRsqrt128);
            __half2 h1 = __floats2half2_rn(v[2] * kRsqrt128, v[3] * kRsqrt128);
            o.x = *reinterpret_cast<uint32_t*>(&h0);
            o.y = *reinterpret_cast<uint32_t*>(&h1);
        }
        *reinterpret_cast<uint2*>(xs + t * 128 + 4 * lane) = o;
    }
    __syncwarp();
    LaneWin<K> lw;
    lw.init(lane, true);
    const uint32_t* words = reinterpret_cast<const uint32_t*>(blob);
    const size_t rw = gm.gu_row_words();
    const size_t proj_off = proj ? (size_t)(a.I / 16) * 8 * kg : 0;
    const uint32_t* strip0 = words + proj_off + (size_t)(nb * 2) * 4 * Geo<K>::W;
    float acc[8][4];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) acc[jj][0] = acc[jj][1] = acc[jj][2] = acc[jj][3] = 0.0f;
    const int tk = lane >> 2, kq = 2 * (lane & 3);
    strip_mma<K>(acc, 8, [&](int r) { return strip0 + (size_t)(kb * 8 + r) * rw; },
                 [&](int r, uint32_t& b0, uint32_t& b1) {
                     b0 = *reinterpret_cast<const uint32_t*>(xs + tk * 128 + r * 16 + kq);
                     b1 = *reinterpret_cast<const uint32_t*>(xs + tk * 128 + r * 16 + kq + 8);
                 },
                 lw);
    // partials: lane holds (col l/4 [+8], tokens 2(l%4), 2(l%4)+1)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        int t = 2 * (lane & 3) + q;
        if (t < ntok) {
            int pick = a.ent_pick[ent * kTokPerEnt + t];
            float* dst = a.part_gu + ((size_t)(pick * 2 + proj) * nKB + kb) * a.I + nb * 128 + (lane >> 2);
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                dst[jj * 16] = acc[jj][q];
                dst[jj * 16 + 8] = acc[jj][2 + q];
            }
        }
    }
    __syncwarp();
    __threadfence();
    int old = 0;
    if (lane == 0) old = atomicAdd(&a.cnt_gu[ent * nbI + nb], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != 2 * nKB - 1) return;
    __threadfence();
    // epilogue for column block nb of every token of the entry
    const __half* svg = reinterpret_cast<const __half*>(blob + gm.off_svh_g()) + nb * 128 + 4 * lane;
    const __half* svu = reinterpret_cast<const __half*>(blob + gm.off_svh_u()) + nb * 128 + 4 * lane;
    const __half* sud = reinterpret_cast<const __half*>(blob + gm.off_suh_d()) + nb * 128 + 4 * lane;
    for (int t = 0; t < ntok; ++t) {
        int pick = a.ent_pick[ent * kTokPerEnt + t];
        float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
        const float* pg = a.part_gu + (size_t)(pick * 2 + 0) * nKB * a.I + nb * 128 + 4 * lane;
        const float* pu = a.part_gu + (size_t)(pick * 2 + 1) * nKB * a.I + nb * 128 + 4 * lane;
        for (int k = 0; k < nKB; ++k) {
            float4 vg = __ldcg(reinterpret_cast<const float4*>(pg + (size_t)k * a.I));
            float4 vu = __ldcg(reinterpret_cast<const float4*>(pu + (size_t)k * a.I));
            g[0] += vg.x; g[1] += vg.y; g[2] += vg.z; g[3] += vg.w;
            u[0] += vu.x; u[1] += vu.y; u[2] += vu.z; u[3] += vu.w;
        }
        fwht128_warp(g, lane);
        fwht128_warp(u, lane);
        float act[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float gv = rn16(g[j] * kRsqrt128 * __half2float(svg[j]));
            float uv = rn16(u[j] * kRsqrt128 * __half2float(svu[j]));
            float s = gv / (1.0f + expf(-gv)) * uv;
            s = rn16(s);
            act[j] = rn16(s * __half2float(sud[j]));
        }
        fwht128_warp(act, lane);
        __half2 h0 = __floats2half2_rn(act[0] * kRsqrt128, act[1] * kRsqrt128);
        __half2 h1 = __floats2half2_rn(act[2] * kRsqrt128, act[3] * kRsqrt128);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&h0);
        o.y = *reinterpret_cast<uint32_t*>(&h1);
        *reinterpret_cast<uint2*>(a.abuf + (size_t)pick * a.I + nb * 128 + 4 * lane) = o;
    }
    if (lane == 0) a.cnt_gu[ent * nbI + nb] = 0;
}

template <int KFIX>
__global__ void __launch_bounds__(256, 2) gateup_kernel(DecodeArgs a) {
    __shared__ __align__(16) __half xs_all[8][kTokPerEnt * 128];
    __half* xs = xs_all[threadIdx.x >> 5];
    const int nKB = a.H / 128, nbI = a.I / 128;
    const int n_units = a.n_ent[0] * 2 * nbI * nKB;
    const int nw = gridDim.x * 8;
    for (int u = blockIdx.x * 8 + (threadIdx.x >> 5); u < n_units; u += nw) {
        int kb = u % nKB, r = u / nKB;
        int nb = r % nbI; r /= nbI;
        int proj = r & 1, ent = r >> 1;
        if constexpr (KFIX != 0) {
            gu_unit<KFIX>(a, ent, proj, nb, kb, xs);
        } else {
            int kg, ku, kd;
            expert_k(a, a.ent_expert[ent], kg, ku, kd);
            switch (proj ? ku : kg) {
                case 2: gu_unit<2>(a, ent, proj, nb, kb, xs); break;
                case 3: gu_unit<3>(a, ent, proj, nb, kb, xs); break;
                case 4: gu_unit<4>(a, ent, proj, nb, kb, xs); break;
                case 5: gu_unit<5>(a, ent, proj, nb, kb, xs); break;
                default: if ((threadIdx.x & 31) == 0) set_error(kErrGeometry); break;
            }
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------------------------------------ down + combine
template <int K>
__device__ void dn_unit(const DecodeArgs& a, int ent, int nbh, int kbi) {
    const int lane = threadIdx.x & 31;
    const int e = a.ent_expert[ent], ntok = a.ent_n[ent];
    int kg, ku, kd;
    expert_k(a, e, kg, ku, kd);
    const Geom gm{a.H, a.I, kg, ku, kd};
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(a.ptrs[e]);
    const int nKBd = a.I / 128, nbH = a.H / 128;
    LaneWin<K> lw;
    lw.init(lane, true);
    const uint32_t* dw = reinterpret_cast<const uint32_t*>(blob) + gm.gu_words();
    const size_t rw = gm.d_row_words();
    const uint32_t* strip0 = dw + (size_t)(nbh * 2) * 4 * Geo<K>::W;
    const int tk = lane >> 2, kq = 2 * (lane & 3);
    const __half* arow = nullptr;
    if (tk < ntok) arow = a.abuf + (size_t)a.ent_pick[ent * kTokPerEnt + tk] * a.I + kbi * 128 + kq;
    float acc[8][4];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) acc[jj][0] = acc[jj][1] = acc[jj][2] = acc[jj][3] = 0.0f;
    strip_mma<K>(acc, 8, [&](int r) { return strip0 + (size_t)(kbi * 8 + r) * rw; },
                 [&](int r, uint32_t& b0, uint32_t& b1) {
                     if (arow) {
                         b0 = __ldcg(reinterpret_cast<const unsigned int*>(arow + r * 16));
                         b1 = __ldcg(reinterpret_cast<const unsigned int*>(arow + r * 16 + 8));
                     } else {
                         b0 = b1 = 0u;
                     }
                 },
                 lw);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        int t = 2 * (lane & 3) + q;
        if (t < ntok) {
            int pick = a.ent_pick[ent * kTokPerEnt + t];
            float* dst = a.part_d + ((size_t)pick * nKBd + kbi) * a.H + nbh * 128 + (lane >> 2);
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                dst[jj * 16] = acc[jj][q];
                dst[jj * 16 + 8] = acc[jj][2 + q];
            }
        }
    }
    __syncwarp();
    __threadfence();
    int old = 0;
    if (lane == 0) old = atomicAdd(&a.cnt_d[ent * nbH + nbh], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != nKBd - 1) return;
    __threadfence();
    const __half* svd = reinterpret_cast<const __half*>(blob + gm.off_svh_d()) + nbh * 128 + 4 * lane;
    for (int t = 0; t < ntok; ++t) {
        int pick = a.ent_pick[ent * kTokPerEnt + t];
        float wt = a.ent_w[ent * kTokPerEnt + t];
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        const float* pp = a.part_d + (size_t)pick * nKBd * a.H + nbh * 128 + 4 * lane;
        for (int k = 0; k < nKBd; ++k) {
            float4 pv = __ldcg(reinterpret_cast<const float4*>(pp + (size_t)k * a.H));
            v[0] += pv.x; v[1] += pv.y; v[2] += pv.z; v[3] += pv.w;
        }
        fwht128_warp(v, lane);
        float4 yv;
        yv.x = v[0] * (kRsqrt128 * wt) * __half2float(svd[0]);
        yv.y = v[1] * (kRsqrt128 * wt) * __half2float(svd[1]);
        yv.z = v[2] * (kRsqrt128 * wt) * __half2float(svd[2]);
        yv.w = v[3] * (kRsqrt128 * wt) * __half2float(svd[3]);
        __stcg(reinterpret_cast<float4*>(a.y + (size_t)pick * a.H + nbh * 128 + 4 * lane), yv);
        __syncwarp();
        __threadfence();
        int m = pick / a.topk;
        int oc = 0;
        if (lane == 0) oc = atomicAdd(&a.cnt_c[m * nbH + nbh], 1);
        oc = __shfl_sync(0xffffffffu, oc, 0);
        if (oc == a.tok_cnt[m] - 1) {
            __threadfence();
            float s[4] = {0.f, 0.f, 0.f, 0.f};
            for (int k = 0; k < a.topk; ++k) {
                int p = m * a.topk + k;
                if (!a.pick_act[p]) continue;
                float4 q4 = __ldcg(reinterpret_cast<const float4*>(a.y + (size_t)p * a.H + nbh * 128 + 4 * lane));
                s[0] += q4.x; s[1] += q4.y; s[2] += q4.z; s[3] += q4.w;
            }
            long long o = (long long)m * a.os + nbh * 128 + 4 * lane;
            if (a.out_bf16 == 2) {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + o) = make_float4(s[0], s[1], s[2], s[3]);
            } else if (a.out_bf16) {
                __nv_bfloat162 p0 = __floats2bfloat162_rn(s[0], s[1]), p1 = __floats2bfloat162_rn(s[2], s[3]);
                uint2 ov;
                ov.x = *reinterpret_cast<uint32_t*>(&p0);
                ov.y = *reinterpret_cast<uint32_t*>(&p1);
                *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.out) + o) = ov;
            } else {
                __half2 p0 = __floats2half2_rn(s[0], s[1]), p1 = __floats2half2_rn(s[2], s[3]);
                uint2 ov;
                ov.x = *reinterpret_cast<uint32_t*>(&p0);
                ov.y = *reinterpret_cast<uint32_t*>(&p1);
                *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(a.out) + o) = ov;
            }
        }
    }
}

template <int KFIX>
__global__ void __launch_bounds__(256, 2) down_kernel(DecodeArgs a) {
    const int nKBd = a.I / 128, nbH = a.H / 128;
    const int n_units = a.n_ent[0] * nbH * nKBd;
    const int nw = gridDim.x * 8;
    for (int u = blockIdx.x * 8 + (threadIdx.x >> 5); u < n_units; u += nw) {
        int kbi = u % nKBd, r = u / nKBd;
        int nbh = r % nbH, ent = r / nbH;
        if constexpr (KFIX != 0) {
            dn_unit<KFIX>(a, ent, nbh, kbi);
        } else {
            int kg, ku, kd;
            expert_k(a, a.ent_expert[ent], kg, ku, kd);
            switch (kd) {
                case 2: dn_unit<2>(a, ent, nbh, kbi); break;
                case 3: dn_unit<3>(a, ent, nbh, kbi); break;
                case 4: dn_unit<4>(a, ent, nbh, kbi); break;
                case 5: dn_unit<5>(a, ent, nbh, kbi); break;
                default: if ((threadIdx.x & 31) == 0) set_error(kErrGeometry); break;
            }
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------------------------------------ host
struct WsLayout {
    size_t off[16];
    size_t total;
};

static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

// Optional phase events (profiling hook, off by default): recorded before route prep, before gate-up, before down
// and after down on the launch stream.  Process-global; set and cleared by exl3b_set_profile_events.
static cudaEvent_t g_prof_ev[4] = {nullptr, nullptr, nullptr, nullptr};
static inline void prof_record(int i, cudaStream_t s) {
    if (g_prof_ev[i]) cudaEventRecord(g_prof_ev[i], s);
}

static WsLayout ws_layout(int M, int topk, int H, int I) {
    size_t np = (size_t)M * topk, me = np, nbI = I / 128, nbH = H / 128, nKB = H / 128, nKBd = I / 128;
    size_t sizes[15] = {me * 4, me * 4, me * kTokPerEnt * 4, me * kTokPerEnt * 4, me * kTokPerEnt * 4, 16,
                        (size_t)M * 4, np * 4, me * nbI * 4, me * nbH * 4, (size_t)M * nbH * 4,
                        np * I * 2, np * 2 * nKB * I * 4, np * nKBd * H * 4, np * H * 4};
    WsLayout L;
    size_t o = 0;
    for (int i = 0; i < 15; ++i) { L.off[i] = o; o += al256(sizes[i]); }
    L.total = o;
    return L;
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int64_t exl3b_moe_decode_workspace(int M, int topk, int H, int I) {
    if (M <= 0 || topk <= 0 || H <= 0 || I <= 0) return 0;
    return (int64_t)ws_layout(M, topk, H, I).total;
}

extern "C" EXL3B_API int exl3b_moe_decode(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids, const float* w,
                                          int M, int topk, const int64_t* ptrs, const int32_t* kinfo, int H, int I, int K,
                                          int E, void* out, int64_t out_stride, int out_bf16, void* workspace,
                                          int64_t ws_bytes, int flags, void* stream) {
    EXL3B_CHECK(x && ids && w && ptrs && out, "exl3b_moe_decode: null pointer");
    EXL3B_CHECK(H % 128 == 0 && I % 128 == 0 && H >= 128 && I >= 128, "exl3b_moe_decode: H, I must be multiples of 128");
    EXL3B_CHECK(E >= 1 && E <= 1024, "exl3b_moe_decode: 1 <= n_experts <= 1024");
    EXL3B_CHECK(kinfo || (K >= 2 && K <= 5), "exl3b_moe_decode: K must be 2..5 (or pass kinfo)");
    EXL3B_CHECK(topk >= 1 && M >= 0, "exl3b_moe_decode: bad M / topk");
    EXL3B_CHECK(x_stride >= H && out_stride >= H && (x_stride % 4) == 0 && (out_stride % 4) == 0,
                "exl3b_moe_decode: row strides must be >= H and multiples of 4 elements");
    EXL3B_CHECK((((uintptr_t)x) & 7) == 0 && (((uintptr_t)out) & (out_bf16 == 2 ? 15 : 7)) == 0,
                "exl3b_moe_decode: x 8-byte / out 8-byte (fp32: 16-byte) alignment");
    EXL3B_CHECK(out_bf16 >= 0 && out_bf16 <= 2, "exl3b_moe_decode: out dtype code 0 fp16, 1 bf16, 2 fp32");
    if (M == 0) return 0;
    WsLayout L = ws_layout(M, topk, H, I);
    EXL3B_CHECK(workspace && ws_bytes >= (int64_t)L.total, "exl3b_moe_decode: workspace too small");
    EXL3B_CHECK((((uintptr_t)workspace) & 255) == 0, "exl3b_moe_decode: workspace must be 256-byte aligned");
    char* b = (char*)workspace;
    DecodeArgs a{};
    a.x = x; a.xs = x_stride; a.x_bf16 = x_bf16;
    a.ids = ids; a.w = w; a.M = M; a.topk = topk;
    a.ptrs = ptrs; a.kinfo = kinfo;
    a.H = H; a.I = I; a.K = K; a.E = E;
    a.out = out; a.os = out_stride; a.out_bf16 = out_bf16;
    a.skip_zero = (flags & 1) ? 1 : 0;
    a.ent_expert = (int*)(b + L.off[0]); a.ent_n = (int*)(b + L.off[1]); a.ent_tok = (int*)(b + L.off[2]);
    a.ent_w = (float*)(b + L.off[3]); a.ent_pick = (int*)(b + L.off[4]); a.n_ent = (int*)(b + L.off[5]);
    a.tok_cnt = (int*)(b + L.off[6]); a.pick_act = (int*)(b + L.off[7]);
    a.cnt_gu = (int*)(b + L.off[8]); a.cnt_d = (int*)(b + L.off[9]); a.cnt_c = (int*)(b + L.off[10]);
    a.abuf = (__half*)(b + L.off[11]); a.part_gu = (float*)(b + L.off[12]); a.part_d = (float*)(b + L.off[13]);
    a.y = (float*)(b + L.off[14]);
    a.maxent = M * topk;
    cudaStream_t s = (cudaStream_t)stream;
    prof_record(0, s);
    route_prep_kernel<<<1, 1024, 0, s>>>(a);
    int rc = exl3b_launch_status("exl3b_moe_decode(route)");
    if (rc) return rc;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    long long max_gu = (long long)a.maxent * 2 * (I / 128) * (H / 128);
    long long max_dn = (long long)a.maxent * (H / 128) * (I / 128);
    int g1 = (int)std::min<long long>((max_gu + 7) / 8, (long long)nsm * 2);
    int g2 = (int)std::min<long long>((max_dn + 7) / 8, (long long)nsm * 2);
    int kf = kinfo ? 0 : K;
    prof_record(1, s);
    switch (kf) {
        case 0: gateup_kernel<0><<<g1, 256, 0, s>>>(a); break;
        case 2: gateup_kernel<2><<<g1, 256, 0, s>>>(a); break;
        case 3: gateup_kernel<3><<<g1, 256, 0, s>>>(a); break;
        case 4: gateup_kernel<4><<<g1, 256, 0, s>>>(a); break;
        case 5: gateup_kernel<5><<<g1, 256, 0, s>>>(a); break;
    }
    rc = exl3b_launch_status("exl3b_moe_decode(gateup)");
    if (rc) return rc;
    prof_record(2, s);
    switch (kf) {
        case 0: down_kernel<0><<<g2, 256, 0, s>>>(a); break;
        case 2: down_kernel<2><<<g2, 256, 0, s>>>(a); break;
        case 3: down_kernel<3><<<g2, 256, 0, s>>>(a); break;
        case 4: down_kernel<4><<<g2, 256, 0, s>>>(a); break;
        case 5: down_kernel<5><<<g2, 256, 0, s>>>(a); break;
    }
    prof_record(3, s);
    return exl3b_launch_status("exl3b_moe_decode(down)");
}

extern "C" EXL3B_API int exl3b_set_profile_events(void* before_route, void* before_gateup, void* before_down,
                                                  void* after_down) {
    g_prof_ev[0] = (cudaEvent_t)before_route;
    g_prof_ev[1] = (cudaEvent_t)before_gateup;
    g_prof_ev[2] = (cudaEvent_t)before_down;
    g_prof_ev[3] = (cudaEvent_t)after_down;
    return 0;
}
