// exl3b_prefill.cu -- routed-MoE prefill (many tokens): the reference's moe_prefill (exl3_moe.a8.sycl:792-828;
// GateUpDpasKernel :422-545, DownDpasKernel :548-635, CombineKernel :371-395) re-designed as grouped tcgen05 GEMMs.
//
// Pipeline (all on the caller's stream):
//   align    (exl3b_align.cu): picks sorted by expert, stable;
//   tiles    : 256-row tiles per active expert (a | m-pair << 16);
//   had_in   : xh[p][proj][H] = fp16(FWHT(fp16(x[tok] * suh)) r) per sorted pick p and projection (:462-475);
//   gate-up  : CTA per (tile, 128-column block of I): D_g, D_u [<=256 rows x 128] in TMEM (512 columns);
//              B operands (gate / up W_inner) decoded from the trellis by all 8 warps straight into 128-byte-swizzled
//              shared memory, A operands (xh rows) by cp.async, one thread issues tcgen05.mma (kind::f16, fp32 accumulate),
//              double-buffered against tcgen05.commit mbarriers; epilogue per row from tcgen05.ld: FWHT, svh, SwiGLU,
//              suh_d, FWHT -> abuf[p][I] (fp16, the reference's :531-541);
//   down     : CTA per (tile, 256-column block of H): D [<=256 x 256] in TMEM; epilogue FWHT * r * w * svh_d -> y[p][H]
//              stored fp16 as the reference's prefill does (:626-631, :802);
//   combine  : out[t] = sum_k y[pair_of[t, k]] in fixed k order (fp32), rounded to the output type.
// Weight decode is once per (expert, column block, 256-row tile); rows past an expert's count are computed on
// whatever rows follow in the buffers and never stored.
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include "exl3b_launch.h"
#include "exl3b_tc.cuh"
#include <algorithm>

namespace exl3b {

struct PrefillArgs {
    const void* x; long long xs; int x_bf16;
    int M, topk, P;
    const int64_t* ptrs; const int32_t* kinfo;
    int H, I, K, E;
    void* out; long long os; int out_bf16;
    // align tables
    const int* act_expert; const int* act_start; const int* act_cnt; const int* n_act;
    const int* pair_tok; const float* pair_w; const int* pair_of;
    // prefill buffers
    int* tiles; int* n_tiles;
    __half* xh; __half* abuf; __half* y;
};

__device__ __forceinline__ void expert_kv(const PrefillArgs& p, int e, int& kg, int& ku, int& kd) {
    if (p.kinfo) { int v = p.kinfo[e]; kg = v & 15; ku = (v >> 4) & 15; kd = (v >> 8) & 15; }
    else { kg = ku = kd = p.K; }
}

// ------------------------------------------------------------------------------------------------ tiles
__global__ void __launch_bounds__(1024) tiles_kernel(PrefillArgs p) {
    __shared__ int sh_warp[32];
    pdl_wait();
    pdl_trigger();
    const int a = threadIdx.x, lane = a & 31, wid = a >> 5;
    const int na = *p.n_act;
    int nt = (a < na) ? (p.act_cnt[a] + 255) / 256 : 0;
    int x = nt;
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
    int base = (wid ? sh_warp[wid - 1] : 0) + x - nt;
    for (int j = 0; j < nt; ++j) p.tiles[base + j] = a | (j << 16);
    if (a == 0) *p.n_tiles = sh_warp[31];
}

// ------------------------------------------------------------------------------------------------ had_in
// One thread per (sorted pick p, projection, 128-block kb): the 128 values stay in registers for the FWHT.
__device__ __forceinline__ void fwht128_regs(float v[128]) {
#pragma unroll
    for (int h = 1; h < 128; h <<= 1)
#pragma unroll
        for (int i = 0; i < 128; i += 2 * h)
#pragma unroll
            for (int j = i; j < i + h; ++j) {
                float a = v[j], b = v[j + h];
                v[j] = a + b;
                v[j + h] = a - b;
            }
}

__global__ void __launch_bounds__(128) had_in_kernel(PrefillArgs p) {
    pdl_wait();
    pdl_trigger();
    const int nkb = p.H / 128;
    const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (long long)p.P * 2 * nkb) return;
    const int kb = (int)(gid % nkb);
    const int proj = (int)((gid / nkb) & 1);
    const int pr = (int)(gid / (2 * nkb));
    // active expert of pick pr: last a with act_start[a] <= pr
    const int na = *p.n_act;
    int lo = 0, hi = na - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (p.act_start[mid] <= pr) lo = mid; else hi = mid - 1;
    }
    const int e = p.act_expert[lo];
    int kg, ku, kd;
    expert_kv(p, e, kg, ku, kd);
    const Geom gm{p.H, p.I, kg, ku, kd};
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(p.ptrs[e]);
    const uint4* sp = reinterpret_cast<const uint4*>(blob + gm.off_suh_g() + (size_t)proj * p.H * 2 + (size_t)kb * 256);
    const int tok = p.pair_tok[pr];
    const uint4* xp = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.x) + ((size_t)tok * p.xs + (size_t)kb * 128) * 2);
    float v[128];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        uint4 xv = __ldg(xp + q), sv = __ldg(sp + q);
        const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
        const uint32_t* sw = reinterpret_cast<const uint32_t*>(&sv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float x0, x1;
            if (p.x_bf16) { x0 = __uint_as_float(xw[j] << 16); x1 = __uint_as_float(xw[j] & 0xFFFF0000u); }
            else { __half2 h = *reinterpret_cast<const __half2*>(&xw[j]); x0 = __low2float(h); x1 = __high2float(h); }
            __half2 s = *reinterpret_cast<const __half2*>(&sw[j]);
            v[q * 8 + 2 * j] = rn16(x0 * __low2float(s));
            v[q * 8 + 2 * j + 1] = rn16(x1 * __high2float(s));
        }
    }
    fwht128_regs(v);
    uint4* op = reinterpret_cast<uint4*>(p.xh + ((size_t)pr * 2 + proj) * p.H + (size_t)kb * 128);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 h = __floats2half2_rn(v[q * 8 + 2 * j] * kRsqrt128, v[q * 8 + 2 * j + 1] * kRsqrt128);
            ow[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        op[q] = o;
    }
}

// ------------------------------------------------------------------------------------------------ grouped GEMM
// Shared memory per stage: PHASE 0 (gate-up): A[proj][mt] 4 x 16 KB (128 rows x 64 fp16, SW128), B[proj] 2 x 16 KB
// (128 columns x 64 fp16); PHASE 1 (down): A[mt] 2 x 16 KB, B 32 KB (256 columns x 64 fp16).
template <int PHASE>
struct GemmCfg {
    static constexpr int A_BYTES = PHASE == 0 ? 4 * 16384 : 2 * 16384;
    static constexpr int B_BYTES = 32768;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int SMEM = 1024 + 2 * STAGE + 1024;   // alignment slack + 2 stages + barriers / vectors
};

// Per-warp B-operand work of one K-chunk (64 k = 4 tile rows x this warp's 2 column tiles): the trellis words of the
// chunk are prefetched into registers one chunk ahead, then decoded into the 128-byte-swizzled B tile.
struct BWork {
    const uint32_t* wbase;   // first word of this warp's projection region
    size_t row_words;        // words per tile row
    int ctg, ctl;            // first column tile (within the projection / within the CTA's B tile)
    uint32_t wa[8], wb[8], wc[8];
};

template <int K>
__device__ __forceinline__ void bwork_load(BWork& bw, int c) {
    constexpr int W = Geo<K>::W, G = Geo<K>::G;
    LaneWin<K> lw;
    lw.init(threadIdx.x & 31, true);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            int ct = bw.ctg + j;
            const uint32_t* gp = bw.wbase + (size_t)(c * 4 + rr) * bw.row_words + (size_t)(ct >> 2) * 4 * W + (ct & 3) * G;
            bw.wa[rr * 2 + j] = __ldg(gp + lw.oA);
            bw.wb[rr * 2 + j] = __ldg(gp + lw.oB);
            bw.wc[rr * 2 + j] = LaneWin<K>::kNeedC ? __ldg(gp + lw.oC) : 0u;
        }
}

template <int K>
__device__ __forceinline__ void bwork_decode(BWork& bw, int c, int nchunks, uint8_t* sBp) {
    const int lane = threadIdx.x & 31;
    LaneWin<K> lw;
    lw.init(lane, true);
    uint32_t ca[8], cb[8], cc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { ca[i] = bw.wa[i]; cb[i] = bw.wb[i]; cc[i] = bw.wc[i]; }
    if (c + 1 < nchunks) bwork_load<K>(bw, c + 1);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            uint32_t f[4];
            decode8<K>(ca[rr * 2 + j], cb[rr * 2 + j], cc[rr * 2 + j], lw.p0, f);
            const int n0 = (bw.ctl + j) * 16 + (lane >> 2);
            const int k0 = rr * 16 + 2 * (lane & 3);
            *reinterpret_cast<uint32_t*>(sBp + sw128_off(n0, k0)) = f[0];
            *reinterpret_cast<uint32_t*>(sBp + sw128_off(n0, k0 + 8)) = f[2];
            *reinterpret_cast<uint32_t*>(sBp + sw128_off(n0 + 8, k0)) = f[1];
            *reinterpret_cast<uint32_t*>(sBp + sw128_off(n0 + 8, k0 + 8)) = f[3];
        }
}

__device__ __forceinline__ void bwork_load_any(int K, BWork& bw, int c) {
    switch (K) {
        case 2: bwork_load<2>(bw, c); break;
        case 3: bwork_load<3>(bw, c); break;
        case 4: bwork_load<4>(bw, c); break;
        case 5: bwork_load<5>(bw, c); break;
        default: break;
    }
}
__device__ __forceinline__ void bwork_decode_any(int K, BWork& bw, int c, int nchunks, uint8_t* sBp) {
    switch (K) {
        case 2: bwork_decode<2>(bw, c, nchunks, sBp); break;
        case 3: bwork_decode<3>(bw, c, nchunks, sBp); break;
        case 4: bwork_decode<4>(bw, c, nchunks, sBp); break;
        case 5: bwork_decode<5>(bw, c, nchunks, sBp); break;
        default: break;
    }
}

// K loop of one CTA: A by cp.async, B by decode, one thread issues the chunk's MMAs and commits them to the stage's
// mbarrier; a stage is rewritten only after the commit of the MMAs that read it (two chunks earlier).
template <int PHASE>
__device__ __forceinline__ void gemm_mainloop(const PrefillArgs& p, uint8_t* sbase, uint64_t* mbar, uint32_t tbase,
                                              int e, int row0, int rows, int nb, const Geom& gm, int Kw) {
    using C = GemmCfg<PHASE>;
    const int tid = threadIdx.x, wid = tid >> 5;
    const int KD = PHASE == 0 ? p.H : p.I;
    const int nchunks = KD / 64;
    const int nmt = rows > 128 ? 2 : 1;
    const uint32_t* words = reinterpret_cast<const uint32_t*>(p.ptrs[e]);
    const int pj = PHASE == 0 ? (wid >> 2) : 0;
    BWork bw;
    bw.ctl = PHASE == 0 ? (wid & 3) * 2 : wid * 2;
    bw.ctg = PHASE == 0 ? nb * 8 + bw.ctl : nb * 16 + bw.ctl;
    bw.row_words = PHASE == 0 ? gm.gu_row_words() : gm.d_row_words();
    bw.wbase = words + (PHASE == 0 ? (pj ? (size_t)(gm.I / 16) * 8 * gm.Kg : 0) : gm.gu_words());
    bwork_load_any(Kw, bw, 0);
    uint32_t parity[2] = {0u, 0u};
    const uint32_t idesc = idesc_f16(128, PHASE == 0 ? 128 : 256);
    for (int c = 0; c < nchunks; ++c) {
        const int s = c & 1;
        uint8_t* sA = sbase + s * C::STAGE;
        uint8_t* sB = sA + C::A_BYTES;
        if (c >= 2) {
            mbar_wait(&mbar[s], parity[s]);
            parity[s] ^= 1u;
        }
        if (PHASE == 0) {
            for (int q = tid; q < 2 * 2 * 128 * 8; q += 256) {
                int ch = q & 7, r = (q >> 3) & 127, mt = (q >> 10) & 1, pjq = q >> 11;
                if (mt >= nmt) continue;
                const __half* src = p.xh + ((size_t)(row0 + mt * 128 + r) * 2 + pjq) * p.H + (size_t)c * 64 + ch * 8;
                uint32_t dst = smem_u32(sA + (pjq * 2 + mt) * 16384 + sw128_off(r, ch * 8));
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
            }
        } else {
            for (int q = tid; q < 2 * 128 * 8; q += 256) {
                int ch = q & 7, r = (q >> 3) & 127, mt = q >> 10;
                if (mt >= nmt) continue;
                const __half* src = p.abuf + (size_t)(row0 + mt * 128 + r) * p.I + (size_t)c * 64 + ch * 8;
                uint32_t dst = smem_u32(sA + mt * 16384 + sw128_off(r, ch * 8));
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        bwork_decode_any(Kw, bw, c, nchunks, sB + (PHASE == 0 ? pj * 16384 : 0));
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t aA = smem_u32(sA), aB = smem_u32(sB);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint32_t acc = (c > 0 || ks > 0) ? 1u : 0u;
                if (PHASE == 0) {
#pragma unroll
                    for (int q = 0; q < 2; ++q)
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt) {
                            if (mt >= nmt) continue;
                            uint64_t da = smem_desc_k128(aA + (q * 2 + mt) * 16384 + ks * 32);
                            uint64_t db = smem_desc_k128(aB + q * 16384 + ks * 32);
                            umma_f16(tbase + (uint32_t)((mt * 2 + q) * 128), da, db, idesc, acc);
                        }
                } else {
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        if (mt >= nmt) continue;
                        uint64_t da = smem_desc_k128(aA + mt * 16384 + ks * 32);
                        uint64_t db = smem_desc_k128(aB + ks * 32);
                        umma_f16(tbase + (uint32_t)(mt * 256), da, db, idesc, acc);
                    }
                }
            }
            umma_commit(&mbar[s]);
        }
    }
    const int sl = (nchunks - 1) & 1;
    mbar_wait(&mbar[sl], parity[sl]);
    tc_fence_after();
}

// Epilogue helpers: the thread owns TMEM lane (row) 32*(wid%4) + lane of M-tile mt = wid / 4.
__device__ __forceinline__ void tmem_row128(uint32_t taddr, float v[128]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) tmem_ld32(taddr + q * 32, v + q * 32);
}

template <int PHASE>
__global__ void __launch_bounds__(256, 1) prefill_gemm_kernel(PrefillArgs p) {
    using C = GemmCfg<PHASE>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* tail = sbase + 2 * C::STAGE;
    uint64_t* mbar = reinterpret_cast<uint64_t*>(tail);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tail + 16);
    __half* vec = reinterpret_cast<__half*>(tail + 64);   // epilogue vectors (3 x 128 or 256 fp16)
    const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
    pdl_wait();
    pdl_trigger();
    const int NB = PHASE == 0 ? p.I / 128 : p.H / 256;
    const int n_tiles = *p.n_tiles;
    const int b = blockIdx.x;
    if (b >= n_tiles * NB) return;
    const int tv = p.tiles[b / NB], nb = b % NB;
    const int a = tv & 0xFFFF, mp = tv >> 16;
    const int e = p.act_expert[a], cnt = p.act_cnt[a];
    const int row0 = p.act_start[a] + mp * 256;
    const int rows = min(256, cnt - mp * 256);
    int kg, ku, kd;
    expert_kv(p, e, kg, ku, kd);
    const Geom gm{p.H, p.I, kg, ku, kd};
    const int Kw = PHASE == 0 ? (wid >> 2 ? ku : kg) : kd;   // this warp's tensor K (gate / up / down)
    if (wid == 0) tmem_alloc(tslot, 512);
    if (tid == 32) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    // epilogue vectors into shared memory
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(p.ptrs[e]);
    if (PHASE == 0) {
        for (int j = tid; j < 3 * 128; j += 256) {
            int which = j >> 7, col = nb * 128 + (j & 127);
            const __half* src = reinterpret_cast<const __half*>(blob + (which == 0 ? gm.off_svh_g() : which == 1 ? gm.off_svh_u()
                                                                                                     : gm.off_suh_d()));
            vec[j] = src[col];
        }
    } else {
        for (int j = tid; j < 256; j += 256) vec[j] = reinterpret_cast<const __half*>(blob + gm.off_svh_d())[nb * 256 + j];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    // mixed-K experts: every warp decodes with its own tensor's K (gate/up halves can differ)
    if (Kw < 2 || Kw > 5) { if (lane == 0) set_error(kErrGeometry); }
    gemm_mainloop<PHASE>(p, sbase, mbar, tbase, e, row0, rows, nb, gm, Kw);
    // ---- epilogue
    const int mt = wid >> 2;
    const int rloc = 32 * (wid & 3) + lane;
    const bool valid = mt * 128 + rloc < rows;
    const uint32_t tl = tbase + ((uint32_t)(32 * (wid & 3)) << 16);
    float v[128];
    if (PHASE == 0) {
        const int pr = row0 + mt * 128 + rloc;
        uint32_t gh[64];
        tmem_row128(tl + (uint32_t)((mt * 2 + 0) * 128), v);
        fwht128_regs(v);
#pragma unroll
        for (int j = 0; j < 128; j += 2) {
            float g0 = rn16(v[j] * kRsqrt128 * __half2float(vec[j]));
            float g1 = rn16(v[j + 1] * kRsqrt128 * __half2float(vec[j + 1]));
            __half2 h = __floats2half2_rn(g0, g1);
            gh[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
        }
        tmem_row128(tl + (uint32_t)((mt * 2 + 1) * 128), v);
        fwht128_regs(v);
#pragma unroll
        for (int j = 0; j < 128; ++j) {
            float u = rn16(v[j] * kRsqrt128 * __half2float(vec[128 + j]));
            __half2 h2 = *reinterpret_cast<__half2*>(&gh[j >> 1]);
            float g = (j & 1) ? __high2float(h2) : __low2float(h2);
            float sl = g / (1.0f + expf(-g)) * u;
            sl = rn16(sl);
            v[j] = rn16(sl * __half2float(vec[256 + j]));
        }
        fwht128_regs(v);
        if (valid) {
            uint4* op = reinterpret_cast<uint4*>(p.abuf + (size_t)pr * p.I + (size_t)nb * 128);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                uint4 o;
                uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __half2 h = __floats2half2_rn(v[q * 8 + 2 * j] * kRsqrt128, v[q * 8 + 2 * j + 1] * kRsqrt128);
                    ow[j] = *reinterpret_cast<uint32_t*>(&h);
                }
                op[q] = o;
            }
        }
    } else {
        const int pr = row0 + mt * 128 + rloc;
        const float wt = valid ? p.pair_w[pr] : 0.0f;
#pragma unroll 1
        for (int hb = 0; hb < 2; ++hb) {
            tmem_row128(tl + (uint32_t)(mt * 256 + hb * 128), v);
            fwht128_regs(v);
            if (valid) {
                uint4* op = reinterpret_cast<uint4*>(p.y + (size_t)pr * p.H + (size_t)nb * 256 + hb * 128);
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    uint4 o;
                    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        int c0 = hb * 128 + q * 8 + 2 * j;
                        float y0 = v[q * 8 + 2 * j] * (kRsqrt128 * wt) * __half2float(vec[c0]);
                        float y1 = v[q * 8 + 2 * j + 1] * (kRsqrt128 * wt) * __half2float(vec[c0 + 1]);
                        __half2 h = __floats2half2_rn(y0, y1);
                        ow[j] = *reinterpret_cast<uint32_t*>(&h);
                    }
                    op[q] = o;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (wid == 0) tmem_dealloc(tbase, 512);
}

// ------------------------------------------------------------------------------------------------ combine
__global__ void __launch_bounds__(256) prefill_combine_kernel(PrefillArgs p) {
    pdl_wait();
    pdl_trigger();
    const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int nc = p.H / 8;
    if (gid >= (long long)p.M * nc) return;
    const int t = (int)(gid / nc), c8 = (int)(gid % nc) * 8;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < p.topk; ++k) {
        int pr = p.pair_of[t * p.topk + k];
        uint4 q = *reinterpret_cast<const uint4*>(p.y + (size_t)pr * p.H + c8);
        const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
        for (int j = 0; j < 4; ++j) { s[2 * j] += __low2float(h[j]); s[2 * j + 1] += __high2float(h[j]); }
    }
    const long long o = (long long)t * p.os + c8;
    if (p.out_bf16 == 2) {
        float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + o);
        d[0] = make_float4(s[0], s[1], s[2], s[3]);
        d[1] = make_float4(s[4], s[5], s[6], s[7]);
    } else {
        uint4 q;
        uint32_t* qw = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (p.out_bf16) { __nv_bfloat162 b = __floats2bfloat162_rn(s[2 * j], s[2 * j + 1]); qw[j] = *reinterpret_cast<uint32_t*>(&b); }
            else { __half2 b = __floats2half2_rn(s[2 * j], s[2 * j + 1]); qw[j] = *reinterpret_cast<uint32_t*>(&b); }
        }
        if (p.out_bf16) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + o) = q;
        else *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.out) + o) = q;
    }
}

// ------------------------------------------------------------------------------------------------ host
struct PfLayout {
    size_t ib, fb, scr, tiles, ntiles, xh, abuf, y, total;
    int A, mxb;
};

static size_t al1k(size_t v) { return (v + 1023) & ~(size_t)1023; }

}  // namespace exl3b
extern "C" int64_t exl3b_align_scratch(int P, int E);
namespace exl3b {

static PfLayout pf_layout(int M, int topk, int H, int I, int E) {
    PfLayout L;
    const size_t P = (size_t)M * topk;
    L.A = (int)std::min<size_t>(P, (size_t)E);
    const int pad = 256;
    L.mxb = (int)((P + pad - 1) / pad) + L.A;
    size_t o = 0;
    L.ib = o; o += al1k((4 * (size_t)L.A + 1 + 2 * P + 16 + L.mxb + 1) * 4);
    L.fb = o; o += al1k(std::max<size_t>(P, 1) * 4);
    L.scr = o; o += al1k((size_t)exl3b_align_scratch((int)P, E));
    L.tiles = o; o += al1k(((P + 255) / 256 + L.A + 1) * 4);
    L.ntiles = o; o += 1024;
    L.xh = o; o += al1k((P + 256) * 2 * (size_t)H * 2);
    L.abuf = o; o += al1k((P + 256) * (size_t)I * 2);
    L.y = o; o += al1k(P * (size_t)H * 2);
    L.total = o;
    return L;
}

template <int PHASE>
static int launch_gemm(const PrefillArgs& p, int grid, cudaStream_t s) {
    using C = GemmCfg<PHASE>;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(prefill_gemm_kernel<PHASE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        attr = true;
    }
    cudaError_t e = launch_k(prefill_gemm_kernel<PHASE>, dim3(grid), dim3(256), (size_t)C::SMEM, s, p);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    return 0;
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int exl3b_align(const int32_t* ids, const float* w, int P, int topk, int E, int pad, int32_t* ib,
                                     float* pair_w, int A, int mxb, void* scratch, int64_t scratch_bytes, void* stream);

extern "C" EXL3B_API int64_t exl3b_moe_prefill_workspace(int M, int topk, int H, int I, int E) {
    if (M <= 0 || topk <= 0) return 0;
    return (int64_t)pf_layout(M, topk, H, I, E).total;
}

extern "C" EXL3B_API int exl3b_moe_prefill(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids, const float* w,
                                           int M, int topk, const int64_t* ptrs, const int32_t* kinfo, int H, int I, int K,
                                           int E, void* out, int64_t out_stride, int out_bf16, void* workspace,
                                           int64_t ws_bytes, int flags, void* stream) {
    (void)flags;
    EXL3B_CHECK(x && ids && w && ptrs && out, "exl3b_moe_prefill: null pointer");
    EXL3B_CHECK(H % 256 == 0 && I % 128 == 0 && H >= 256 && I >= 128, "exl3b_moe_prefill: H % 256 == 0, I % 128 == 0");
    EXL3B_CHECK(E >= 1 && E <= 1024, "exl3b_moe_prefill: 1 <= n_experts <= 1024");
    EXL3B_CHECK(kinfo || (K >= 2 && K <= 5), "exl3b_moe_prefill: K must be 2..5 (or pass kinfo)");
    EXL3B_CHECK(topk >= 1 && M >= 0, "exl3b_moe_prefill: bad M / topk");
    EXL3B_CHECK((((uintptr_t)x) & 15) == 0 && (x_stride % 8) == 0 && x_stride >= H, "exl3b_moe_prefill: x alignment / stride");
    EXL3B_CHECK((((uintptr_t)out) & 15) == 0 && (out_stride % 8) == 0 && out_stride >= H, "exl3b_moe_prefill: out alignment / stride");
    EXL3B_CHECK(out_bf16 >= 0 && out_bf16 <= 2, "exl3b_moe_prefill: out dtype code 0 fp16, 1 bf16, 2 fp32");
    if (M == 0) return 0;
    PfLayout L = pf_layout(M, topk, H, I, E);
    EXL3B_CHECK(workspace && ws_bytes >= (int64_t)L.total, "exl3b_moe_prefill: workspace too small");
    EXL3B_CHECK((((uintptr_t)workspace) & 1023) == 0, "exl3b_moe_prefill: workspace must be 1024-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    char* b = (char*)workspace;
    const int P = M * topk;
    int32_t* ib = (int32_t*)(b + L.ib);
    int rc = exl3b_align(ids, w, P, topk, E, 256, ib, (float*)(b + L.fb), L.A, L.mxb, b + L.scr,
                         exl3b_align_scratch(P, E), stream);
    if (rc) return rc;
    PrefillArgs p{};
    p.x = x; p.xs = x_stride; p.x_bf16 = x_bf16;
    p.M = M; p.topk = topk; p.P = P;
    p.ptrs = ptrs; p.kinfo = kinfo;
    p.H = H; p.I = I; p.K = K; p.E = E;
    p.out = out; p.os = out_stride; p.out_bf16 = out_bf16;
    const int A = L.A;
    p.act_expert = ib; p.act_start = ib + A; p.act_cnt = ib + 2 * A; p.n_act = ib + 4 * A;
    p.pair_tok = ib + 4 * A + 1; p.pair_of = p.pair_tok + P; p.pair_w = (const float*)(b + L.fb);
    p.tiles = (int*)(b + L.tiles); p.n_tiles = (int*)(b + L.ntiles);
    p.xh = (__half*)(b + L.xh); p.abuf = (__half*)(b + L.abuf); p.y = (__half*)(b + L.y);
    cudaError_t e = launch_k(tiles_kernel, dim3(1), dim3(1024), 0, s, p);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    long long nh = (long long)P * 2 * (H / 128);
    e = launch_k(had_in_kernel, dim3((unsigned)((nh + 127) / 128)), dim3(128), 0, s, p);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    const int max_tiles = (P + 255) / 256 + A;
    rc = launch_gemm<0>(p, max_tiles * (I / 128), s);
    if (rc) return rc;
    rc = launch_gemm<1>(p, max_tiles * (H / 256), s);
    if (rc) return rc;
    long long nc = (long long)M * (H / 8);
    e = launch_k(prefill_combine_kernel, dim3((unsigned)((nc + 255) / 256)), dim3(256), 0, s, p);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    return exl3b_launch_status("exl3b_moe_prefill");
}
