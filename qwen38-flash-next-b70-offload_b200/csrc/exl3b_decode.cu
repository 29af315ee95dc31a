// exl3b_decode.cu -- routed-MoE decode path (few tokens): the reference's launch_ensure + GateUpKernel + DownKernel +
// CombineKernel (exl3_moe.a8.sycl:121-395, 837-1040, 1229-1314) re-designed for sm_100a.
//
// Three kernels per call, chained with programmatic dependent launch:
//   prep    (1 block): [device cache step: tier mask, LRU stamps, victims, fill plan] + grouping of the active picks
//                      by DISTINCT expert into entries (one expert, up to 8 of its picks), so an expert picked by several
//                      tokens is streamed once;
//   gate-up (grid)   : copies the planned cache fills (host blob -> slot) and runs units (entry, projection, 128-column
//                      block, 128-row k block);
//   down    (grid)   : units (entry, 128-column block of H, 128-row k block of I), the weighted combine, and the cache
//                      commit (ptrs[e] = slot) by the last block to finish.
// Each warp streams its units' 8-tile strips through a private SMEM ring filled by cp.async, decodes each lane's 8
// values of a tile straight into an mma.sync A fragment of W^T (exl3b_common.cuh) and multiplies it with the 8-token
// Hadamard-domain activation block (fp32 accumulate).  Split-K partials go to a small L2-resident buffer; the last
// warp to finish a column block (atomic arrival counter, no waiting) reduces them in fixed order and runs the
// epilogue, so results do not depend on scheduling:
//   gate/up epilogue (:239-256): g = fp16(FWHT(g) r svh_g), u likewise, a = fp16(SiLU(g) u), a = fp16(a suh_d),
//                                abuf = fp16(FWHT(a) r)
//   down epilogue   (:355-364): y = FWHT(v) (r w) svh_d (fp32)
//   combine         (:387-394): out[m] = sum_k y[m,k] in fixed k order, by the last column block to finish.
// Cache fills are read from their host address (ptrs[e] until the commit), like the reference's write-through, while
// the gate-up blocks copy them into their slots.  Picks with weight exactly 0 (tier-masked) contribute exactly zero
// and are skipped (flag bit 0).
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include "exl3b_ensure.cuh"
#include "exl3b_launch.h"
#include <algorithm>

namespace exl3b {

constexpr int kTokPerEnt = 8;   // mma n dimension

struct DecodeArgs {
    const void* x; long long xs; int x_bf16;
    const int32_t* ids; const float* w; int M; int topk;
    int64_t* ptrs; const int32_t* kinfo;
    int H, I, K, E;
    void* out; long long os; int out_bf16;
    int skip_zero;
    // cache fills (cached calls): fill_list [1 + n], fill (slot address per expert of the layer), blob bytes
    const int32_t* fill_list; int64_t* fill; long long blob;
    // workspace
    int* ent_expert; int* ent_n; int* ent_tok; float* ent_w; int* ent_pick; int* n_ent;
    long long* ent_blob; int* ent_k;
    int* tok_cnt; int* pick_act;
    int* cnt_gu; int* cnt_d; int* cnt_c; int* blocks_done;
    __half* abuf; float* part_gu; float* part_d; float* y;
    int maxent;
};

// ------------------------------------------------------------------------------------------------ prep
// Zero the arrival counters, group active picks by expert (ascending id, picks in ascending index), count active
// picks per token and zero the output rows of tokens with none.  All 1024 threads of one block.
__device__ void route_prep_block(const DecodeArgs& a) {
    __shared__ int cnt[1024];
    __shared__ int sh_warp2[32];
    const int tid = threadIdx.x, npairs = a.M * a.topk;
    const int nbI = a.I / 128, nbH = a.H / 128;
    for (int i = tid; i < a.maxent * nbI; i += blockDim.x) a.cnt_gu[i] = 0;
    for (int i = tid; i < a.maxent * nbH; i += blockDim.x) a.cnt_d[i] = 0;
    for (int i = tid; i < a.M * nbH; i += blockDim.x) a.cnt_c[i] = 0;
    if (tid == 0) a.blocks_done[0] = 0;
    for (int e = tid; e < a.E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < npairs; i += blockDim.x) {
        int e = a.ids[i];
        bool ok = e >= 0 && e < a.E;
        bool act = ok && !(a.skip_zero && a.w[i] == 0.0f);
        if (!ok) set_error(kErrBounds);
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
    const int e = tid;
    const int n = (e < a.E) ? cnt[e] : 0;
    const int ne = (n + kTokPerEnt - 1) / kTokPerEnt;
    const int lane = tid & 31, wid = tid >> 5;
    int x = ne;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) { int y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
    if (lane == 31) sh_warp2[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int s = sh_warp2[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) { int y = __shfl_up_sync(0xffffffffu, s, o); if (lane >= o) s += y; }
        sh_warp2[lane] = s;
    }
    __syncthreads();
    const int base = (wid ? sh_warp2[wid - 1] : 0) + x - ne;
    if (tid == 0) a.n_ent[0] = sh_warp2[31];
    if (n > 0) {
        int j = 0;
        for (int i = 0; i < npairs && j < n; ++i) {
            if (a.ids[i] != e || !a.pick_act[i]) continue;
            int en = base + j / kTokPerEnt, s = j % kTokPerEnt;
            if (s == 0) {
                a.ent_expert[en] = e;
                a.ent_n[en] = min(kTokPerEnt, n - j);
                a.ent_blob[en] = (long long)a.ptrs[e];
                a.ent_k[en] = a.kinfo ? a.kinfo[e] : (a.K | (a.K << 4) | (a.K << 8));
                for (int q = 0; q < kTokPerEnt; ++q) { a.ent_tok[en * kTokPerEnt + q] = 0; a.ent_pick[en * kTokPerEnt + q] = 0; }
            }
            a.ent_tok[en * kTokPerEnt + s] = i / a.topk;
            a.ent_w[en * kTokPerEnt + s] = a.w[i];
            a.ent_pick[en * kTokPerEnt + s] = i;
            ++j;
        }
    }
    for (int m = 0; m < a.M; ++m) {
        if (a.tok_cnt[m] != 0) continue;
        for (int c = tid; c < a.H; c += blockDim.x) {
            if (a.out_bf16 == 2) reinterpret_cast<float*>(a.out)[(long long)m * a.os + c] = 0.0f;
            else if (a.out_bf16) reinterpret_cast<__nv_bfloat16*>(a.out)[(long long)m * a.os + c] = __float2bfloat16(0.0f);
            else reinterpret_cast<__half*>(a.out)[(long long)m * a.os + c] = __float2half(0.0f);
        }
    }
}

// Cached calls run the device cache step first (in place on ids / w), then the grouping.
__global__ void __launch_bounds__(1024) prep_kernel(EnsureArgs ea, DecodeArgs da, int cached) {
    pdl_wait();
    pdl_trigger();
    if (cached) {
        ensure_block(ea);
        __syncthreads();
    }
    route_prep_block(da);
}

// ------------------------------------------------------------------------------------------------ streaming core
// Each warp streams its units' 8-tile strips row by row through a private SMEM ring filled with cp.async (16 B,
// L2-only), kStages rows ahead of the decode.  A strip row is 2 PLANAR4 groups; in SMEM each plane of a group is
// padded to 4G + 8 words (D > 1), so the two words a lane reads per tile -- word (tile j, period g, plane i) at
// i*PS + j*G + g -- fall in distinct banks across the warp.  Unit metadata is loaded one unit ahead.
constexpr int kStages = 5;

__device__ __forceinline__ void cp_async16(uint32_t* smem, const void* gmem) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <int K>
struct Ring {
    static constexpr int D = Geo<K>::D, G = Geo<K>::G, W = Geo<K>::W;
    static constexpr int PS = 4 * G + (D > 1 ? 8 : 0);   // plane stride in SMEM (words)
    static constexpr int GS = D * PS;                     // group stride
    static constexpr int ROWW = 2 * GS;                   // one strip row (2 groups)
    static constexpr int CHUNKS = 2 * W;                  // 16-byte chunks of a strip row in global memory
    __device__ static int chunk_dst(int c) {
        int gi = c / W;
        int wg = 4 * (c - gi * W);
        int i = wg / (4 * G);
        return gi * GS + i * PS + (wg - i * 4 * G);
    }
    __device__ static int lane_off(int w) { return (w % D) * PS + w / D; }
};

// Per-lane constants of one K: SMEM offsets of the lane's window words, the window's bit offset, and the SMEM
// destinations of the lane's cp.async chunks of a strip row.
template <int K>
struct LaneK {
    int oA, oB, oC, p0;
    int dst[3];
    __device__ __forceinline__ void init(int lane) {
        using R = Ring<K>;
        int S = ((8 * lane + 1) * K - 16 + 256 * K) % (256 * K);
        int w0 = S >> 5;
        p0 = S & 31;
        oA = R::lane_off(w0);
        oB = R::lane_off((w0 + 1) % (8 * K));
        oC = R::lane_off((w0 + 2) % (8 * K));
#pragma unroll
        for (int q = 0; q < 3; ++q) dst[q] = (lane + 32 * q < R::CHUNKS) ? R::chunk_dst(lane + 32 * q) : 0;
    }
};

constexpr int kRowMaxWords = 2 * 5 * (4 * 8 + 8);   // Ring<5>::ROWW, the largest strip row of K in 2..5
constexpr int kSideWords = 64 + kTokPerEnt * 64;      // gate-up: suh block (128 fp16) + x block of 8 tokens
constexpr int kXsStride = 136;                        // xh row stride (fp16): rows of different tokens hit other banks

template <int KFIX, int PHASE>
struct StreamCfg {
    static constexpr int ROWW = KFIX ? Ring<KFIX>::ROWW : kRowMaxWords;
    static constexpr int STAGE = ROWW;
    static constexpr int WARP_WORDS = kStages * STAGE + (PHASE == 0 ? 2 * kSideWords + kTokPerEnt * kXsStride / 2 : 0);
    static constexpr int SMEM_BYTES = 8 * WARP_WORDS * 4;
};

struct UMeta {
    int valid, ent, f0, f1, f2, K, kv, ntok, tok, pick;   // f0..f2: (proj, nb, kb) gate-up; (nbh, kbi, -) down
    const uint8_t* blob;
};

template <int PHASE>
__device__ __forceinline__ UMeta load_meta(const DecodeArgs& a, int u, int n_units) {
    UMeta m;
    const int lane = threadIdx.x & 31;
    m.valid = u < n_units;
    if (!m.valid) {
        m.ent = 0; m.f0 = m.f1 = m.f2 = 0; m.K = 3; m.kv = 0; m.ntok = 0; m.tok = 0; m.pick = 0; m.blob = nullptr;
        return m;
    }
    if (PHASE == 0) {
        const int nKB = a.H / 128, nbI = a.I / 128;
        m.f2 = u % nKB; int r = u / nKB;
        m.f1 = r % nbI; r /= nbI;
        m.f0 = r & 1; m.ent = r >> 1;
    } else {
        const int nKBd = a.I / 128, nbH = a.H / 128;
        m.f1 = u % nKBd; int r = u / nKBd;
        m.f0 = r % nbH; m.ent = r / nbH; m.f2 = 0;
    }
    m.blob = reinterpret_cast<const uint8_t*>(__ldcg(a.ent_blob + m.ent));
    m.ntok = __ldcg(a.ent_n + m.ent);
    m.kv = __ldcg(a.ent_k + m.ent);
    m.K = PHASE == 0 ? (m.f0 ? (m.kv >> 4) & 15 : m.kv & 15) : (m.kv >> 8) & 15;
    m.tok = lane < kTokPerEnt ? __ldcg(a.ent_tok + m.ent * kTokPerEnt + lane) : 0;
    m.pick = lane < kTokPerEnt ? __ldcg(a.ent_pick + m.ent * kTokPerEnt + lane) : 0;
    return m;
}

// Issue the cp.async copies of stream row r of unit m into `stage` (and, for gate-up row 0, its side slot).
template <int K, int PHASE>
__device__ __forceinline__ void issue_row(const DecodeArgs& a, const UMeta& m, int r, uint32_t* stage, uint32_t* side,
                                          const LaneK<K>& lk) {
    using R = Ring<K>;
    const int lane = threadIdx.x & 31;
    const Geom gm{a.H, a.I, m.kv & 15, (m.kv >> 4) & 15, (m.kv >> 8) & 15};
    const uint32_t* src;
    if (PHASE == 0) {
        const size_t proj_off = m.f0 ? (size_t)(a.I / 16) * 8 * gm.Kg : 0;
        src = reinterpret_cast<const uint32_t*>(m.blob) + (size_t)(m.f2 * 8 + r) * gm.gu_row_words() + proj_off +
              (size_t)(m.f1 * 2) * 4 * R::W;
    } else {
        src = reinterpret_cast<const uint32_t*>(m.blob) + gm.gu_words() + (size_t)(m.f1 * 8 + r) * gm.d_row_words() +
              (size_t)(m.f0 * 2) * 4 * R::W;
    }
#pragma unroll
    for (int q = 0; q < 3; ++q)
        if (lane + 32 * q < R::CHUNKS) cp_async16(stage + lk.dst[q], src + 4 * (lane + 32 * q));
    if (PHASE == 0 && r == 0) {
        if (lane < 16)
            cp_async16(side + lane * 4, m.blob + gm.off_suh_g() + (size_t)m.f0 * a.H * 2 + (size_t)m.f2 * 256 + lane * 16);
#pragma unroll
        for (int c = lane; c < 16 * kTokPerEnt; c += 32) {   // uniform trip count: the shuffle sees every lane
            int t = c >> 4, j = c & 15;
            int tk = __shfl_sync(0xffffffffu, m.tok, t);
            if (t < m.ntok)
                cp_async16(side + 64 + t * 64 + j * 4,
                           reinterpret_cast<const uint8_t*>(a.x) + ((size_t)tk * a.xs + (size_t)m.f2 * 128) * 2 + j * 16);
        }
    }
}

// Decode the 8 tiles of one strip row from `stage` and accumulate acc[jj] += W^T(tile) * B.
template <int K>
__device__ __forceinline__ void consume_row(const uint32_t* stage, uint32_t b0, uint32_t b1, float acc[8][4],
                                            const LaneK<K>& lk) {
    using R = Ring<K>;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
        const uint32_t* gp = stage + (jj >> 2) * R::GS + (jj & 3) * R::G;
        uint32_t wa = gp[lk.oA], wb = gp[lk.oB], wc = LaneWin<K>::kNeedC ? gp[lk.oC] : 0u;
        uint32_t f[4];
        decode8<K>(wa, wb, wc, lk.p0, f);
        mma16816(acc[jj], f, b0, b1);
    }
}

// Gate-up unit prologue: xh = fp16(FWHT(fp16(x * suh)) r) for the unit's 128-block and tokens, from the side slot.
__device__ __forceinline__ void unit_xh(const DecodeArgs& a, const UMeta& m, const uint32_t* side, __half* xs) {
    const int lane = threadIdx.x & 31;
    const __half* suh = reinterpret_cast<const __half*>(side);
    float su[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) su[j] = __half2float(suh[4 * lane + j]);
    for (int t = 0; t < kTokPerEnt; ++t) {
        uint2 o = make_uint2(0u, 0u);
        if (t < m.ntok) {
            const uint16_t* xr = reinterpret_cast<const uint16_t*>(side + 64 + t * 64);
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint16_t bits = xr[4 * lane + j];
                float xv = a.x_bf16 ? __uint_as_float((uint32_t)bits << 16) : __half2float(__ushort_as_half(bits));
                v[j] = rn16(xv * su[j]);
            }
            fwht128_warp(v, lane);
            __half2 h0 = __floats2half2_rn(v[0] * kRsqrt128, v[1] * kRsqrt128);
            __half2 h1 = __floats2half2_rn(v[2] * kRsqrt128, v[3] * kRsqrt128);
            o.x = *reinterpret_cast<uint32_t*>(&h0);
            o.y = *reinterpret_cast<uint32_t*>(&h1);
        }
        *reinterpret_cast<uint2*>(xs + t * kXsStride + 4 * lane) = o;
    }
    __syncwarp();
}

__device__ __forceinline__ void store_out(const DecodeArgs& a, long long o, const float s[4]) {
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

// Unit epilogues: split-K partials, then (last arriver only) the column-block epilogue.
__device__ void gu_epilogue(const DecodeArgs& a, const UMeta& m, float acc[8][4]) {
    const int lane = threadIdx.x & 31;
    const int nKB = a.H / 128, nbI = a.I / 128;
    const int proj = m.f0, nb = m.f1, kb = m.f2;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        int t = 2 * (lane & 3) + q;
        int pick = __shfl_sync(0xffffffffu, m.pick, t);
        if (t < m.ntok) {
            float* dst = a.part_gu + ((size_t)(pick * 2 + proj) * nKB + kb) * a.I + nb * 128 + (lane >> 2);
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                __stcg(dst + jj * 16, acc[jj][q]);
                __stcg(dst + jj * 16 + 8, acc[jj][2 + q]);
            }
        }
    }
    __syncwarp();
    __threadfence();
    int old = 0;
    if (lane == 0) old = atomicAdd(&a.cnt_gu[m.ent * nbI + nb], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != 2 * nKB - 1) return;
    __threadfence();
    const Geom gm{a.H, a.I, m.kv & 15, (m.kv >> 4) & 15, (m.kv >> 8) & 15};
    const __half* svg = reinterpret_cast<const __half*>(m.blob + gm.off_svh_g()) + nb * 128 + 4 * lane;
    const __half* svu = reinterpret_cast<const __half*>(m.blob + gm.off_svh_u()) + nb * 128 + 4 * lane;
    const __half* sud = reinterpret_cast<const __half*>(m.blob + gm.off_suh_d()) + nb * 128 + 4 * lane;
    for (int t = 0; t < m.ntok; ++t) {
        int pick = __shfl_sync(0xffffffffu, m.pick, t);
        float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
        const float* pg = a.part_gu + (size_t)(pick * 2 + 0) * nKB * a.I + nb * 128 + 4 * lane;
        const float* pu = a.part_gu + (size_t)(pick * 2 + 1) * nKB * a.I + nb * 128 + 4 * lane;
#pragma unroll 8
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
            float sl = gv / (1.0f + expf(-gv)) * uv;
            sl = rn16(sl);
            act[j] = rn16(sl * __half2float(sud[j]));
        }
        fwht128_warp(act, lane);
        __half2 h0 = __floats2half2_rn(act[0] * kRsqrt128, act[1] * kRsqrt128);
        __half2 h1 = __floats2half2_rn(act[2] * kRsqrt128, act[3] * kRsqrt128);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&h0);
        o.y = *reinterpret_cast<uint32_t*>(&h1);
        __stcg(reinterpret_cast<uint2*>(a.abuf + (size_t)pick * a.I + nb * 128 + 4 * lane), o);
    }
    if (lane == 0) a.cnt_gu[m.ent * nbI + nb] = 0;
}

__device__ void dn_epilogue(const DecodeArgs& a, const UMeta& m, float acc[8][4]) {
    const int lane = threadIdx.x & 31;
    const int nKBd = a.I / 128, nbH = a.H / 128;
    const int nbh = m.f0, kbi = m.f1;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        int t = 2 * (lane & 3) + q;
        int pick = __shfl_sync(0xffffffffu, m.pick, t);
        if (t < m.ntok) {
            float* dst = a.part_d + ((size_t)pick * nKBd + kbi) * a.H + nbh * 128 + (lane >> 2);
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                __stcg(dst + jj * 16, acc[jj][q]);
                __stcg(dst + jj * 16 + 8, acc[jj][2 + q]);
            }
        }
    }
    __syncwarp();
    __threadfence();
    int old = 0;
    if (lane == 0) old = atomicAdd(&a.cnt_d[m.ent * nbH + nbh], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != nKBd - 1) return;
    __threadfence();
    const Geom gm{a.H, a.I, m.kv & 15, (m.kv >> 4) & 15, (m.kv >> 8) & 15};
    const __half* svd = reinterpret_cast<const __half*>(m.blob + gm.off_svh_d()) + nbh * 128 + 4 * lane;
    for (int t = 0; t < m.ntok; ++t) {
        int pick = __shfl_sync(0xffffffffu, m.pick, t);
        float wt = __ldcg(a.ent_w + m.ent * kTokPerEnt + t);
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        const float* pp = a.part_d + (size_t)pick * nKBd * a.H + nbh * 128 + 4 * lane;
#pragma unroll 6
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
        int mt = pick / a.topk;
        int oc = 0;
        if (lane == 0) oc = atomicAdd(&a.cnt_c[mt * nbH + nbh], 1);
        oc = __shfl_sync(0xffffffffu, oc, 0);
        if (oc == __ldcg(a.tok_cnt + mt) - 1) {
            __threadfence();
            float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
            for (int k = 0; k < a.topk; ++k) {
                int p = mt * a.topk + k;
                if (!__ldcg(a.pick_act + p)) continue;
                float4 q4 = __ldcg(reinterpret_cast<const float4*>(a.y + (size_t)p * a.H + nbh * 128 + 4 * lane));
                s[0] += q4.x; s[1] += q4.y; s[2] += q4.z; s[3] += q4.w;
            }
            store_out(a, (long long)mt * a.os + nbh * 128 + 4 * lane, s);
        }
    }
    if (lane == 0) a.cnt_d[m.ent * nbH + nbh] = 0;
}

template <int K, int PHASE>
__device__ __forceinline__ void issue_k(const DecodeArgs& a, const UMeta& m, int r, uint32_t* stage, uint32_t* side) {
    LaneK<K> lk;
    lk.init(threadIdx.x & 31);
    issue_row<K, PHASE>(a, m, r, stage, side, lk);
}

template <int KFIX, int PHASE>
__device__ __forceinline__ void issue_any(const DecodeArgs& a, const UMeta& m, int r, uint32_t* stage, uint32_t* side,
                                          const LaneK<KFIX ? KFIX : 3>& lkf) {
    if (!m.valid) return;
    if constexpr (KFIX != 0) {
        issue_row<KFIX, PHASE>(a, m, r, stage, side, lkf);
    } else {
        switch (m.K) {
            case 2: issue_k<2, PHASE>(a, m, r, stage, side); break;
            case 3: issue_k<3, PHASE>(a, m, r, stage, side); break;
            case 4: issue_k<4, PHASE>(a, m, r, stage, side); break;
            case 5: issue_k<5, PHASE>(a, m, r, stage, side); break;
            default: break;
        }
    }
}

template <int KFIX>
__device__ __forceinline__ void consume_any(int K, const uint32_t* stage, uint32_t b0, uint32_t b1, float acc[8][4],
                                            const LaneK<KFIX ? KFIX : 3>& lkf) {
    if constexpr (KFIX != 0) {
        consume_row<KFIX>(stage, b0, b1, acc, lkf);
    } else {
        const int lane = threadIdx.x & 31;
        switch (K) {
            case 2: { LaneK<2> l; l.init(lane); consume_row<2>(stage, b0, b1, acc, l); break; }
            case 3: { LaneK<3> l; l.init(lane); consume_row<3>(stage, b0, b1, acc, l); break; }
            case 4: { LaneK<4> l; l.init(lane); consume_row<4>(stage, b0, b1, acc, l); break; }
            case 5: { LaneK<5> l; l.init(lane); consume_row<5>(stage, b0, b1, acc, l); break; }
            default: break;
        }
    }
}

// Cache fills: copy each planned fill's blob (host address ptrs[e], until the commit) into its slot (fill[e]),
// spread over every thread of the grid.
__device__ __forceinline__ void copy_fills(const DecodeArgs& a) {
    if (!a.fill_list) return;
    const int nf = __ldcg(a.fill_list);
    if (nf <= 0) return;
    const long long n16 = a.blob / 16;
    const long long total = (long long)nf * n16;
    for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (long long)gridDim.x * blockDim.x) {
        int i = (int)(q / n16);
        long long off = q - (long long)i * n16;
        int e = __ldcg(a.fill_list + 1 + i);
        const uint4* src = reinterpret_cast<const uint4*>(__ldcg(a.ptrs + e));
        uint4* dst = reinterpret_cast<uint4*>(__ldcg(a.fill + e));
        dst[off] = __ldcg(src + off);
    }
}

// PHASE 0: gate|up units (entry, proj, nb, kb); PHASE 1: down units (entry, nbh, kbi).  Units are interleaved over
// the grid block-major (unit u -> block u % grid), so every SM gets an equal share; each warp runs one continuous row
// stream over its units.
template <int KFIX, int PHASE>
__global__ void __launch_bounds__(256, 2) stream_kernel(DecodeArgs a) {
    using C = StreamCfg<KFIX, PHASE>;
    extern __shared__ __align__(16) uint32_t smem[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    uint32_t* ring = smem + wid * C::WARP_WORDS;
    uint32_t* side = ring + kStages * C::STAGE;                    // gate-up: 2 side slots
    __half* xs = reinterpret_cast<__half*>(side + 2 * kSideWords);  // gate-up: xh [8][kXsStride]
    LaneK<KFIX ? KFIX : 3> lkf;
    lkf.init(lane);
    const int G = gridDim.x;
    auto unit_of = [&](int i) { return (int)blockIdx.x + (wid + 8 * i) * G; };
    // Entries come from the prep kernel (two launches back for the down phase): the down phase loads its first unit
    // and starts streaming weights before waiting for gate-up, whose abuf it needs only for its B operands.
    if (PHASE == 0) pdl_wait();
    const int n_ent = __ldcg(a.n_ent);
    const int n_units = PHASE == 0 ? n_ent * 2 * (a.I / 128) * (a.H / 128) : n_ent * (a.H / 128) * (a.I / 128);
    UMeta mc = load_meta<PHASE>(a, unit_of(0), n_units);
    UMeta mn = load_meta<PHASE>(a, unit_of(1), n_units);
    int ic = 0;
    auto issue = [&](int pos) {
        int i = pos >> 3, r = pos & 7;
        const UMeta& m = (i == ic) ? mc : mn;
        if (i <= ic + 1) issue_any<KFIX, PHASE>(a, m, r, ring + (pos % kStages) * C::STAGE, side + (i & 1) * kSideWords, lkf);
        cp_commit();
    };
    if (mc.valid) {
#pragma unroll
        for (int p = 0; p < kStages - 1; ++p) issue(p);
    }
    if (PHASE == 1) pdl_wait();
    pdl_trigger();
    if (PHASE == 0) copy_fills(a);
    const int tk = lane >> 2, kq = 2 * (lane & 3);
    float acc[8][4];
    uint32_t nb0 = 0, nb1 = 0;   // down: B operand of the next row, loaded one row ahead
    auto load_b = [&](const UMeta& m, int r) {
        int pk = __shfl_sync(0xffffffffu, m.pick, tk);
        if (tk < m.ntok) {
            const __half* ar = a.abuf + (size_t)pk * a.I + m.f1 * 128 + r * 16 + kq;
            nb0 = __ldcg(reinterpret_cast<const unsigned int*>(ar));
            nb1 = __ldcg(reinterpret_cast<const unsigned int*>(ar + 8));
        } else {
            nb0 = nb1 = 0u;
        }
    };
    if (PHASE == 1 && mc.valid) load_b(mc, 0);
    for (int pos = 0; mc.valid; ++pos) {
        const int i = pos >> 3, r = pos & 7;
        if (r == 0 && i > 0) {
            mc = mn;
            ic = i;
            if (!mc.valid) break;
            mn = load_meta<PHASE>(a, unit_of(i + 1), n_units);
        }
        issue(pos + kStages - 1);
        cp_wait<kStages - 1>();
        __syncwarp();
        const uint32_t* stage = ring + (pos % kStages) * C::STAGE;
        if (r == 0) {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) acc[jj][0] = acc[jj][1] = acc[jj][2] = acc[jj][3] = 0.0f;
            if (PHASE == 0) unit_xh(a, mc, side + (i & 1) * kSideWords, xs);
        }
        uint32_t b0, b1;
        if (PHASE == 0) {
            b0 = *reinterpret_cast<const uint32_t*>(xs + tk * kXsStride + r * 16 + kq);
            b1 = *reinterpret_cast<const uint32_t*>(xs + tk * kXsStride + r * 16 + kq + 8);
        } else {
            b0 = nb0;
            b1 = nb1;
            if (r < 7) load_b(mc, r + 1);
            else if (mn.valid) load_b(mn, 0);
        }
        consume_any<KFIX>(mc.K, stage, b0, b1, acc, lkf);
        __syncwarp();
        if (r == 7) {
            if (PHASE == 0) gu_epilogue(a, mc, acc);
            else dn_epilogue(a, mc, acc);
        }
    }
    cp_wait<0>();
    if (PHASE == 1) {
        // the last block to finish commits the cache fills (CombineKernel item 0, exl3_moe.a8.sycl:378-386)
        __syncthreads();
        if (threadIdx.x == 0 && a.fill_list) {
            __threadfence();
            int old = atomicAdd(a.blocks_done, 1);
            if (old == (int)gridDim.x - 1) {
                __threadfence();
                const int nf = __ldcg(a.fill_list);
                for (int q = 0; q < nf; ++q) {
                    int e = __ldcg(a.fill_list + 1 + q);
                    a.ptrs[e] = __ldcg(a.fill + e);
                    a.fill[e] = 0;
                }
                a.blocks_done[0] = 0;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ host
struct WsLayout {
    size_t off[18];
    size_t total;
};

static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

// Optional phase events (profiling hook, off by default): recorded before prep, before gate-up, before down and
// after down on the launch stream.  Process-global; set and cleared by exl3b_set_profile_events.
static cudaEvent_t g_prof_ev[4] = {nullptr, nullptr, nullptr, nullptr};
void prof_record(int i, cudaStream_t s) {
    if (g_prof_ev[i]) cudaEventRecord(g_prof_ev[i], s);
}

static WsLayout ws_layout(int M, int topk, int H, int I) {
    size_t np = (size_t)M * topk, me = np, nbI = I / 128, nbH = H / 128, nKB = H / 128, nKBd = I / 128;
    size_t sizes[18] = {me * 4, me * 4, me * kTokPerEnt * 4, me * kTokPerEnt * 4, me * kTokPerEnt * 4, 16,
                        (size_t)M * 4, np * 4, me * nbI * 4, me * nbH * 4, (size_t)M * nbH * 4,
                        np * I * 2, np * 2 * nKB * I * 4, np * nKBd * H * 4, np * H * 4, me * 8, me * 4, 16};
    WsLayout L;
    size_t o = 0;
    for (int i = 0; i < 18; ++i) { L.off[i] = o; o += al256(sizes[i]); }
    L.total = o;
    return L;
}

template <int KFIX, int PHASE>
static int launch_stream(const DecodeArgs& a, int grid, cudaStream_t s) {
    using C = StreamCfg<KFIX, PHASE>;
    static bool attr_set = false;   // per instantiation; the attribute is per function, set once per process
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(stream_kernel<KFIX, PHASE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM_BYTES);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        attr_set = true;
    }
    cudaError_t e = launch_k(stream_kernel<KFIX, PHASE>, dim3(grid), dim3(256), (size_t)C::SMEM_BYTES, s, a);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    return 0;
}

static int check_args(const void* x, int64_t x_stride, const int32_t* ids, const float* w, int M, int topk,
                      const void* ptrs, const int32_t* kinfo, int H, int I, int K, int E, void* out, int64_t out_stride,
                      int out_bf16) {
    EXL3B_CHECK(x && ids && w && ptrs && out, "exl3b_moe_decode: null pointer");
    EXL3B_CHECK(H % 128 == 0 && I % 128 == 0 && H >= 128 && I >= 128, "exl3b_moe_decode: H, I must be multiples of 128");
    EXL3B_CHECK(E >= 1 && E <= 1024, "exl3b_moe_decode: 1 <= n_experts <= 1024");
    EXL3B_CHECK(kinfo || (K >= 2 && K <= 5), "exl3b_moe_decode: K must be 2..5 (or pass kinfo)");
    EXL3B_CHECK(topk >= 1 && M >= 0, "exl3b_moe_decode: bad M / topk");
    EXL3B_CHECK(x_stride >= H && out_stride >= H && (out_stride % 4) == 0, "exl3b_moe_decode: row strides must be >= H");
    EXL3B_CHECK((((uintptr_t)x) & 15) == 0 && (x_stride % 8) == 0 && (((uintptr_t)out) & (out_bf16 == 2 ? 15 : 7)) == 0,
                "exl3b_moe_decode: x 16-byte aligned with a row stride multiple of 8 elements; out 8-byte (fp32: 16-byte) aligned");
    EXL3B_CHECK(out_bf16 >= 0 && out_bf16 <= 2, "exl3b_moe_decode: out dtype code 0 fp16, 1 bf16, 2 fp32");
    return 0;
}

int victim_copy_launch(const int32_t* vict, const int64_t* host_base, int64_t slot_base, int64_t blob, int E,
                       int64_t hstride, uint8_t* ram_res, int max_victims, cudaStream_t s);

static int run_decode(DecodeArgs& a, const EnsureArgs* ea, void* workspace, int64_t ws_bytes, cudaStream_t s,
                      const int32_t* vict, const int64_t* host_base, int64_t slot_base, int64_t hstride,
                      uint8_t* ram_res, int nvict) {
    const int M = a.M, topk = a.topk, H = a.H, I = a.I;
    WsLayout L = ws_layout(M, topk, H, I);
    EXL3B_CHECK(workspace && ws_bytes >= (int64_t)L.total, "exl3b_moe_decode: workspace too small");
    EXL3B_CHECK((((uintptr_t)workspace) & 255) == 0, "exl3b_moe_decode: workspace must be 256-byte aligned");
    char* b = (char*)workspace;
    a.ent_expert = (int*)(b + L.off[0]); a.ent_n = (int*)(b + L.off[1]); a.ent_tok = (int*)(b + L.off[2]);
    a.ent_w = (float*)(b + L.off[3]); a.ent_pick = (int*)(b + L.off[4]); a.n_ent = (int*)(b + L.off[5]);
    a.tok_cnt = (int*)(b + L.off[6]); a.pick_act = (int*)(b + L.off[7]);
    a.cnt_gu = (int*)(b + L.off[8]); a.cnt_d = (int*)(b + L.off[9]); a.cnt_c = (int*)(b + L.off[10]);
    a.abuf = (__half*)(b + L.off[11]); a.part_gu = (float*)(b + L.off[12]); a.part_d = (float*)(b + L.off[13]);
    a.y = (float*)(b + L.off[14]);
    a.ent_blob = (long long*)(b + L.off[15]); a.ent_k = (int*)(b + L.off[16]); a.blocks_done = (int*)(b + L.off[17]);
    a.maxent = M * topk;
    EnsureArgs none{};
    prof_record(0, s);
    cudaError_t e = launch_k(prep_kernel, dim3(1), dim3(1024), 0, s, ea ? *ea : none, a, ea ? 1 : 0);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    if (vict && nvict > 0) {   // victim write-back must precede the fill copies that overwrite the slots
        int rc = victim_copy_launch(vict, host_base, slot_base, a.blob, a.E, hstride, ram_res, nvict, s);
        if (rc) return rc;
    }
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    // full machine for both phases (2 blocks of 8 warps per SM; 1 for the larger mixed-K ring); units are dealt
    // block-major, so the per-SM share is equal even when there are fewer units than warps
    long long max_gu = (long long)a.maxent * 2 * (I / 128) * (H / 128);
    long long max_dn = (long long)a.maxent * (H / 128) * (I / 128);
    int g1 = (int)std::min<long long>(std::max<long long>(max_gu, 1), (long long)nsm * (a.kinfo ? 1 : 2));
    int g2 = (int)std::min<long long>(std::max<long long>(max_dn, 1), (long long)nsm * 2);
    int kf = a.kinfo ? 0 : a.K;
    int rc = 0;
    prof_record(1, s);
    switch (kf) {
        case 0: rc = launch_stream<0, 0>(a, g1, s); break;
        case 2: rc = launch_stream<2, 0>(a, g1, s); break;
        case 3: rc = launch_stream<3, 0>(a, g1, s); break;
        case 4: rc = launch_stream<4, 0>(a, g1, s); break;
        case 5: rc = launch_stream<5, 0>(a, g1, s); break;
    }
    if (rc) return rc;
    prof_record(2, s);
    switch (kf) {
        case 0: rc = launch_stream<0, 1>(a, g2, s); break;
        case 2: rc = launch_stream<2, 1>(a, g2, s); break;
        case 3: rc = launch_stream<3, 1>(a, g2, s); break;
        case 4: rc = launch_stream<4, 1>(a, g2, s); break;
        case 5: rc = launch_stream<5, 1>(a, g2, s); break;
    }
    if (rc) return rc;
    prof_record(3, s);
    return exl3b_launch_status("exl3b_moe_decode");
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int64_t exl3b_moe_decode_workspace(int M, int topk, int H, int I) {
    if (M <= 0 || topk <= 0 || H <= 0 || I <= 0) return 0;
    return (int64_t)ws_layout(M, topk, H, I).total;
}

static DecodeArgs make_args(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids, const float* w, int M,
                            int topk, int64_t* ptrs, const int32_t* kinfo, int H, int I, int K, int E, void* out,
                            int64_t out_stride, int out_bf16, int flags) {
    DecodeArgs a{};
    a.x = x; a.xs = x_stride; a.x_bf16 = x_bf16;
    a.ids = ids; a.w = w; a.M = M; a.topk = topk;
    a.ptrs = ptrs; a.kinfo = kinfo;
    a.H = H; a.I = I; a.K = K; a.E = E;
    a.out = out; a.os = out_stride; a.out_bf16 = out_bf16;
    a.skip_zero = (flags & 1) ? 1 : 0;
    a.fill_list = nullptr; a.fill = nullptr; a.blob = 0;
    return a;
}

extern "C" EXL3B_API int exl3b_moe_decode(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids, const float* w,
                                          int M, int topk, const int64_t* ptrs, const int32_t* kinfo, int H, int I, int K,
                                          int E, void* out, int64_t out_stride, int out_bf16, void* workspace,
                                          int64_t ws_bytes, int flags, void* stream) {
    int rc = check_args(x, x_stride, ids, w, M, topk, ptrs, kinfo, H, I, K, E, out, out_stride, out_bf16);
    if (rc) return rc;
    if (M == 0) return 0;
    DecodeArgs a = make_args(x, x_stride, x_bf16, ids, w, M, topk, const_cast<int64_t*>(ptrs), kinfo, H, I, K, E, out,
                             out_stride, out_bf16, flags);
    return run_decode(a, nullptr, workspace, ws_bytes, (cudaStream_t)stream, nullptr, nullptr, 0, 0, nullptr, 0);
}

extern "C" EXL3B_API int exl3b_moe_decode_cached(const void* x, int64_t x_stride, int x_bf16, int32_t* ids, float* w, int M,
                                                 int topk, int layer, int64_t* ptrs_all, int32_t* slot_of,
                                                 int32_t* slot_key, int32_t* slot_last, int32_t* tick,
                                                 const int64_t* host_base, int64_t slot_base, int64_t blob, int64_t hstride,
                                                 int64_t* fill_all, int32_t* fill_list, int max_fill, int S,
                                                 const uint8_t* ram_res, int32_t* ring, int ring_cap, const int32_t* safe,
                                                 int32_t* vict, uint8_t* vict_ram_res, int H, int I, int K, int E,
                                                 void* out, int64_t out_stride, int out_bf16, void* workspace,
                                                 int64_t ws_bytes, int flags, void* stream) {
    int rc = check_args(x, x_stride, ids, w, M, topk, ptrs_all, nullptr, H, I, K, E, out, out_stride, out_bf16);
    if (rc) return rc;
    EXL3B_CHECK(layer >= 0 && S > 0 && slot_of && slot_key && slot_last && tick && host_base && fill_all && fill_list,
                "exl3b_moe_decode_cached: cache state missing");
    const int64_t want_blob = (int64_t)Geom{H, I, K, K, K}.blob();
    EXL3B_CHECK(blob == want_blob, "exl3b_moe_decode_cached: blob size does not match H, I, K");
    EXL3B_CHECK(!ram_res || (ring && ring_cap > 0 && safe), "exl3b_moe_decode_cached: tier mask needs ring and safe");
    EXL3B_CHECK(max_fill >= 0, "exl3b_moe_decode_cached: max_fill >= 0");
    if (M == 0) return 0;
    int64_t* ptrs = ptrs_all + (int64_t)layer * E;
    DecodeArgs a = make_args(x, x_stride, x_bf16, ids, w, M, topk, ptrs, nullptr, H, I, K, E, out, out_stride, out_bf16,
                             flags);
    a.fill_list = fill_list;
    a.fill = fill_all + (int64_t)layer * E;
    a.blob = blob;
    int mf = max_fill < E ? max_fill : E;
    EnsureArgs ea{ids, w, M * topk, layer, E, S, ptrs_all, slot_of, slot_key, slot_last, tick, host_base, slot_base, blob,
                  hstride > 0 ? hstride : blob, fill_all, fill_list, mf, 0, nullptr, ram_res, ring, ring_cap, safe, vict};
    int nvict = vict ? std::min(mf, M * topk) : 0;
    return run_decode(a, &ea, workspace, ws_bytes, (cudaStream_t)stream, vict, host_base, slot_base,
                      hstride > 0 ? hstride : blob, vict_ram_res, nvict);
}

extern "C" EXL3B_API int exl3b_set_profile_events(void* before_route, void* before_gateup, void* before_down,
                                                  void* after_down) {
    g_prof_ev[0] = (cudaEvent_t)before_route;
    g_prof_ev[1] = (cudaEvent_t)before_gateup;
    g_prof_ev[2] = (cudaEvent_t)before_down;
    g_prof_ev[3] = (cudaEvent_t)after_down;
    return 0;
}
