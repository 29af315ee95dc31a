// exl3b_prefill.cu -- routed-MoE prefill (many tokens): the reference's moe_prefill (exl3_moe.a8.sycl:792-828;
// GateUpDpasKernel :422-545, DownDpasKernel :548-635, CombineKernel :371-395) re-designed as grouped tcgen05 GEMMs.
//
// Pipeline (all on the caller's stream):
//   align    (exl3b_align.cu): picks sorted by expert, stable;
//   tiles    : 256-row tiles per active expert (a | m-pair << 16);
//   had_in   : xh[proj][p][H] = fp16(FWHT(fp16(x[tok] * suh)) r) per sorted pick p and projection (:462-475), one warp
//              per pick;
//   gate-up  : CTA per (tile, 128-column block of I), warp-specialised:
//                warp 9 (one lane) streams the A operand (xh rows, 64-k chunks) with TMA into 128-byte-swizzled
//                shared memory; warps 0-7 decode the B operands (gate / up W_inner, 16x16 trellis tiles) in registers
//                and store them with stmatrix into the same swizzled layout; warp 8 (one lane) issues tcgen05.mma
//                (kind::f16, fp32 accumulate) into TMEM: D_g, D_u [<= 256 rows x 128] (512 columns).  Stages are
//                handed over with mbarriers (TMA bytes, decoder arrivals, tcgen05.commit);
//              epilogue per row from tcgen05.ld: FWHT, svh, SwiGLU, suh_d, FWHT -> abuf[p][I] (fp16, :531-541);
//   down     : same structure, CTA per (tile, 256-column block of H): D [<= 256 x 256]; epilogue FWHT * r * w * svh_d
//              -> y[p][H] stored fp16 as the reference's prefill does (:626-631, :802);
//   combine  : out[t] = sum_k y[pair_of[t, k]] in fixed k order (fp32), rounded to the output type.
// Weights are decoded once per (expert, column block, 256-row tile); rows past an expert's count are computed on
// whatever rows follow in the buffers and never stored.  Every wait is bounded (exl3b_tc.cuh mbar_wait).
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include "exl3b_launch.h"
#include "exl3b_tc.cuh"
#include <cuda.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>

namespace exl3b {

struct PrefillArgs {
    const void* x; long long xs; int x_bf16;
    int M, topk, P, Prow;
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
// One warp per sorted pick, 32 blocks of 8 warps per 256-row tile (the tile gives the expert); 8 128-blocks per warp
// step: lane l holds 32 consecutive values (quarter l%4) of block l/4.  FWHT strides 1..16 run inside the lane,
// strides 32 and 64 pair lanes l^1 and l^2 (the reference's butterfly order, stage by stage).  Per warp step the
// lane's x chunk and both projections' suh chunks are loaded in one round and both products rounded to fp16 before
// the two FWHTs: x is read once for the two projections and a pick takes two load round trips instead of four.
// One in-lane butterfly stage of stride HS >= 2 over the lane's 32 values, on float2 pairs.
template <int HS>
__device__ __forceinline__ void had_stage2(float v[32]) {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int j = (t / (HS / 2)) * (2 * HS) + (t % (HS / 2)) * 2;
        const float2 a = make_float2(v[j], v[j + 1]), b = make_float2(v[j + HS], v[j + HS + 1]);
        const float2 sm = f2_add(a, b), df = f2_sub(a, b);
        v[j] = sm.x; v[j + 1] = sm.y;
        v[j + HS] = df.x; v[j + HS + 1] = df.y;
    }
}

__global__ void __launch_bounds__(256, 3) had_in_kernel(PrefillArgs p) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x >> 5;
    if (tile >= *p.n_tiles) return;
    const int tv = p.tiles[tile];
    const int a = tv & 0xFFFF, r = (tv >> 16) * 256 + (blockIdx.x & 31) * 8 + (threadIdx.x >> 5);
    if (r >= p.act_cnt[a]) return;
    const int pr = p.act_start[a] + r;
    const int e = p.act_expert[a];
    int kg, ku, kd;
    expert_kv(p, e, kg, ku, kd);
    const Geom gm{p.H, p.I, kg, ku, kd};
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(p.ptrs[e]);
    const int tok = p.pair_tok[pr];
    const uint16_t* xr = reinterpret_cast<const uint16_t*>(p.x) + (size_t)tok * p.xs;
    const int nblk = p.H / 128, g = lane >> 2, sub = lane & 3;
    const uint16_t* suh = reinterpret_cast<const uint16_t*>(blob + gm.off_suh_g());   // gate; up at + H
#pragma unroll 1
    for (int kb0 = 0; kb0 < nblk; kb0 += 8) {
        const int kb = kb0 + g;
        const bool act = kb < nblk;
        const int i0 = kb * 128 + sub * 32;
        // the lane's 32 inputs of both projections, y = fp16(x suh): x and both suh chunks are loaded in one round,
        // x once for the two projections
        uint4 xv[4], sv[2][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            xv[q] = act ? *reinterpret_cast<const uint4*>(xr + i0 + q * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int pj = 0; pj < 2; ++pj)
                sv[pj][q] = act ? __ldg(reinterpret_cast<const uint4*>(suh + (size_t)pj * p.H + i0 + q * 8))
                                : make_uint4(0, 0, 0, 0);
        }
        uint32_t yw[2][16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t xw[4] = {xv[q].x, xv[q].y, xv[q].z, xv[q].w};
#pragma unroll
            for (int pj = 0; pj < 2; ++pj) {
                const uint32_t sw[4] = {sv[pj][q].x, sv[pj][q].y, sv[pj][q].z, sv[pj][q].w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    float x0, x1;
                    if (p.x_bf16) { x0 = __uint_as_float(xw[h] << 16); x1 = __uint_as_float(xw[h] & 0xFFFF0000u); }
                    else { x0 = __half2float(__ushort_as_half((unsigned short)(xw[h] & 0xFFFFu))); x1 = __half2float(__ushort_as_half((unsigned short)(xw[h] >> 16))); }
                    const float s0 = __half2float(__ushort_as_half((unsigned short)(sw[h] & 0xFFFFu)));
                    const float s1 = __half2float(__ushort_as_half((unsigned short)(sw[h] >> 16)));
                    __half2 hv = __floats2half2_rn(x0 * s0, x1 * s1);
                    yw[pj][q * 4 + h] = *reinterpret_cast<uint32_t*>(&hv);
                }
            }
        }
#pragma unroll
        for (int proj = 0; proj < 2; ++proj) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&yw[proj][j]));
                v[2 * j] = f.x;
                v[2 * j + 1] = f.y;
            }
            // stride 1 inside a float2 (scalar); strides 2..16 on float2 pairs (j, j + 1), (j + hs, j + hs + 1)
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const float a = v[j], b = v[j + 1];
                v[j] = a + b;
                v[j + 1] = a - b;
            }
            had_stage2<2>(v);
            had_stage2<4>(v);
            had_stage2<8>(v);
            had_stage2<16>(v);
            // strides 32, 64: the lower lane gets o + v, the upper o - v = fma(v, -1, o)
#pragma unroll
            for (int m = 1; m <= 2; m <<= 1) {
                const float sg = (lane & m) ? -1.0f : 1.0f;
                const float2 sg2 = make_float2(sg, sg);
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float2 o = make_float2(__shfl_xor_sync(0xffffffffu, v[j], m),
                                                 __shfl_xor_sync(0xffffffffu, v[j + 1], m));
                    const float2 r = f2_fma(make_float2(v[j], v[j + 1]), sg2, o);
                    v[j] = r.x; v[j + 1] = r.y;
                }
            }
            if (act) {
                __half* dst = p.xh + ((size_t)proj * p.Prow + pr) * p.H;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t ow[4];
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        __half2 h = __floats2half2_rn(v[q * 8 + 2 * jj] * kRsqrt128, v[q * 8 + 2 * jj + 1] * kRsqrt128);
                        ow[jj] = *reinterpret_cast<uint32_t*>(&h);
                    }
                    *reinterpret_cast<uint4*>(dst + i0 + q * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ grouped GEMM
// Shared memory per stage: PHASE 0 (gate-up): A[proj][mt] 4 x 16 KB (128 rows x 64 fp16, SW128), B[proj] 2 x 16 KB
// (128 columns x 64 fp16); PHASE 1 (down): A[mt] 2 x 16 KB, B 32 KB (256 columns x 64 fp16).  After the stages: the
// mbarriers, the TMEM base slot and the epilogue vectors.
// Then each decoder warp's ring of trellis words (kWordRing bytes): the words of its 2 column tiles for the next
// chunks, filled by cp.async several chunks ahead of the decode.
constexpr int kWordRing = 4096;   // per decoder warp: 4 chunks at K <= 4, 3 at K = 5

template <int PHASE>
struct GemmCfg {
    static constexpr int NST = PHASE == 0 ? 2 : 3;
    static constexpr int A_BYTES = PHASE == 0 ? 4 * 16384 : 2 * 16384;
    static constexpr int B_BYTES = 32768;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int SMEM = 1024 + NST * STAGE + 1024 + 8 * kWordRing;
    static constexpr int THREADS = 320;   // warps 0-7 decode + epilogue, warp 8 MMA + TMEM, warp 9 TMA
};
static_assert(GemmCfg<0>::SMEM <= 227 * 1024 && GemmCfg<1>::SMEM <= 227 * 1024, "prefill GEMM shared memory");

static __device__ __forceinline__ void pf_cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
static __device__ __forceinline__ void pf_cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
static __device__ __forceinline__ void pf_cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

struct DecCtx {
    const uint32_t* wbase;   // first word of this warp's projection region (row 0)
    size_t row_words;        // words per tile row
    int ctg;                 // first global column tile of the warp's 2 tiles
    uint32_t sboff;          // byte offset of the warp's first tile inside a stage's B region
};

// Decoder warp: 2 column tiles x 4 tile rows (64 k) per chunk.  The pair (even ctg, ctg + 1) lies in one PLANAR4
// group, so per tile row its words are D contiguous plane segments of 2 G words (moe_offload.py:68-73 layout); the
// warp copies them with cp.async into its word ring NW - 1 chunks ahead, [chunk][tile row][plane][tile][period], and
// each lane reads its window words from there.
template <int K, int PHASE>
__device__ __forceinline__ void decode_loop(const DecCtx& d, uint8_t* sbase, uint8_t* wring, uint64_t* full_b,
                                            uint64_t* empty, int nchunks) {
    using C = GemmCfg<PHASE>;
    constexpr int W = Geo<K>::W, G = Geo<K>::G, D = Geo<K>::D;
    constexpr int SEGW = 2 * G, ROWW = D * SEGW, CHW = 4 * ROWW;   // words: plane segment, tile row, chunk
    constexpr int NW = (kWordRing / 4) / CHW >= 4 ? 4 : 3;
    static_assert(NW * CHW * 4 <= kWordRing && NW >= 3, "decoder word ring");
    const int lane = threadIdx.x & 31;
    // the lane's window words (plain word w of tile 0: plane w % D, period w / D) in the ring's layout
    int oA, oB, oC, p0;
    {
        constexpr int NB = 256 * K;
        const int S = (((8 * lane + 1) * K - 16) % NB + NB) % NB;
        const int w0 = S >> 5;
        p0 = S & 31;
        const int wA = w0, wB = (w0 + 1) % (8 * K), wC = (w0 + 2) % (8 * K);
        oA = (wA % D) * SEGW + wA / D;
        oB = (wB % D) * SEGW + wB / D;
        oC = (wC % D) * SEGW + wC / D;
    }
    const int nl = (lane & 7) + 8 * ((lane >> 3) & 1), kc = (lane >> 4) & 1;
    uint32_t soff[4];
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) soff[rr] = (uint32_t)nl * 128u + ((uint32_t)((2 * rr + kc) ^ (lane & 7)) << 4);
    const uint32_t* gp = d.wbase + (size_t)(d.ctg >> 2) * 4 * W + (d.ctg & 3) * G;   // plane 0 of the pair, row 0
    const uint32_t wr0 = smem_u32(wring);
    const uint32_t* wr = reinterpret_cast<const uint32_t*>(wring);
    auto issue = [&](int c) {
        if (c < nchunks) {
            const uint32_t dst0 = wr0 + (uint32_t)((c % NW) * CHW) * 4u;
#pragma unroll
            for (int q0 = 0; q0 < CHW / 4; q0 += 32) {
                const int q = q0 + lane;   // 16-byte piece: tile row, plane, 4-word piece of the segment
                if (q < CHW / 4) {
                    const int rr = q / (ROWW / 4), rem = q % (ROWW / 4), i = rem / (SEGW / 4), k4 = rem % (SEGW / 4);
                    pf_cp_async16(dst0 + (uint32_t)(rr * ROWW + i * SEGW + 4 * k4) * 4u,
                                  gp + (size_t)(c * 4 + rr) * d.row_words + i * 4 * G + 4 * k4);
                }
            }
        }
        pf_cp_commit();
    };
#pragma unroll
    for (int c = 0; c < NW - 1; ++c) issue(c);
    const uint32_t s0 = smem_u32(sbase) + C::A_BYTES + d.sboff;
#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
        const int s = c % C::NST;
        issue(c + NW - 1);
        pf_cp_wait<NW - 1>();
        __syncwarp();
        const uint32_t* cw = wr + (c % NW) * CHW;
        if (c >= C::NST) mbar_wait(&empty[s], (uint32_t)((c / C::NST) - 1) & 1u);
        const uint32_t sb = s0 + (uint32_t)s * C::STAGE;
#pragma unroll
        for (int rr = 0; rr < 4; ++rr)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t* tw = cw + rr * ROWW + j * G;
                uint32_t f[4];
                decode8<K>(tw[oA], tw[oB], LaneWin<K>::kNeedC ? tw[oC] : 0u, p0, f);
                stmatrix_x4(sb + (uint32_t)j * 2048u + soff[rr], f[0], f[1], f[2], f[3]);
            }
        fence_async_smem();
        mbar_arrive(&full_b[s]);
        __syncwarp();   // every lane has read the ring slot before the next chunk's copies overwrite it
    }
    pf_cp_wait<0>();
}

template <int PHASE>
__device__ __forceinline__ void decode_loop_any(int K, const DecCtx& d, uint8_t* sbase, uint8_t* wring, uint64_t* full_b,
                                                uint64_t* empty, int nchunks) {
    switch (K) {
        case 2: decode_loop<2, PHASE>(d, sbase, wring, full_b, empty, nchunks); break;
        case 3: decode_loop<3, PHASE>(d, sbase, wring, full_b, empty, nchunks); break;
        case 4: decode_loop<4, PHASE>(d, sbase, wring, full_b, empty, nchunks); break;
        case 5: decode_loop<5, PHASE>(d, sbase, wring, full_b, empty, nchunks); break;
        default:
            // unsupported K (already flagged kErrGeometry): no decode, but the stage hand-over still runs so that
            // no other role of the CTA waits on these warps
            for (int c = 0; c < nchunks; ++c) {
                const int s = c % GemmCfg<PHASE>::NST;
                if (c >= GemmCfg<PHASE>::NST) mbar_wait(&empty[s], (uint32_t)((c / GemmCfg<PHASE>::NST) - 1) & 1u);
                mbar_arrive(&full_b[s]);
            }
            break;
    }
}

// Epilogue helper: the thread owns TMEM lane (row) 32*(wid%4) + lane of M-tile mt = wid / 4.
__device__ __forceinline__ void tmem_row128(uint32_t taddr, float v[128]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) tmem_ld32(taddr + q * 32, v + q * 32);
}

// One butterfly stage of stride HS >= 2 over a row of 128 registers: the pairs (j, j + 1) and (j + HS, j + HS + 1)
// as float2s (32 packed additions and 32 packed subtractions).
template <int HS>
__device__ __forceinline__ void fwht128_stage2(float v[128]) {
#pragma unroll
    for (int t = 0; t < 32; ++t) {
        const int j = (t / (HS / 2)) * (2 * HS) + (t % (HS / 2)) * 2;
        const float2 a = make_float2(v[j], v[j + 1]), b = make_float2(v[j + HS], v[j + HS + 1]);
        const float2 sm = f2_add(a, b), df = f2_sub(a, b);
        v[j] = sm.x; v[j + 1] = sm.y;
        v[j + HS] = df.x; v[j + HS + 1] = df.y;
    }
}

// FWHT-128 of one row in registers, strides 1, 2, ..., 64 in that order (a + b / a - b per butterfly).  Stride 1
// pairs the two halves of a float2 and runs scalar; strides 2..64 run on float2 pairs with the same roundings.
__device__ __forceinline__ void fwht128_regs(float v[128]) {
#pragma unroll
    for (int j = 0; j < 128; j += 2) {
        const float a = v[j], b = v[j + 1];
        v[j] = a + b;
        v[j + 1] = a - b;
    }
    fwht128_stage2<2>(v);
    fwht128_stage2<4>(v);
    fwht128_stage2<8>(v);
    fwht128_stage2<16>(v);
    fwht128_stage2<32>(v);
    fwht128_stage2<64>(v);
}

template <int PHASE>
// One CTA per SM (TMEM 512 columns, ~194 KB shared memory).  10 warps put 3 warps on two of the four SM
// sub-partitions, whose register files hold 16,384 registers each: at most 168 registers per thread.
__global__ void __launch_bounds__(320, 1) prefill_gemm_kernel(PrefillArgs p, const __grid_constant__ CUtensorMap tmA) {
    using C = GemmCfg<PHASE>;
    constexpr int NST = C::NST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* tail = sbase + NST * C::STAGE;
    uint64_t* full_a = reinterpret_cast<uint64_t*>(tail);
    uint64_t* full_b = full_a + NST;
    uint64_t* empty = full_b + NST;
    uint64_t* done = empty + NST;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tail + 128);
    __half* vec = reinterpret_cast<__half*>(tail + 256);   // epilogue vectors (3 x 128 or 256 fp16)
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
    const int nmt = rows > 128 ? 2 : 1;
    int kg, ku, kd;
    expert_kv(p, e, kg, ku, kd);
    const Geom gm{p.H, p.I, kg, ku, kd};
    const int KD = PHASE == 0 ? p.H : p.I;
    const int nchunks = KD / 64;
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(p.ptrs[e]);
    if (wid == 8) tmem_alloc(tslot, 512);
    if (tid == 9 * 32) {
        // full_a: one arrival (expect_tx) + TMA bytes; full_b: 256 decoder arrivals; empty / done: tcgen05.commit
        for (int i = 0; i < 3 * NST + 1; ++i) mbar_init(&full_a[i], (i >= NST && i < 2 * NST) ? 256u : 1u);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        prefetch_tmap(&tmA);
    }
    if (tid < 256) {
        if (PHASE == 0) {
            for (int j = tid; j < 3 * 128; j += 256) {
                int which = j >> 7, col = nb * 128 + (j & 127);
                const __half* src = reinterpret_cast<const __half*>(
                    blob + (which == 0 ? gm.off_svh_g() : which == 1 ? gm.off_svh_u() : gm.off_suh_d()));
                vec[j] = src[col];
            }
        } else {
            vec[tid] = reinterpret_cast<const __half*>(blob + gm.off_svh_d())[nb * 256 + tid];
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (wid < 8) {
        // ---- B decoders
        const int Kw = PHASE == 0 ? (wid >> 2 ? ku : kg) : kd;
        if (Kw < 2 || Kw > 5) { if (lane == 0) set_error(kErrGeometry); }
        const uint32_t* words = reinterpret_cast<const uint32_t*>(blob);
        DecCtx d;
        if (PHASE == 0) {
            const int pj = wid >> 2, ctl = (wid & 3) * 2;
            d.wbase = words + (pj ? (size_t)(gm.I / 16) * 8 * gm.Kg : 0);
            d.row_words = gm.gu_row_words();
            d.ctg = nb * 8 + ctl;
            d.sboff = (uint32_t)pj * 16384u + (uint32_t)ctl * 2048u;
        } else {
            const int ctl = wid * 2;
            d.wbase = words + gm.gu_words();
            d.row_words = gm.d_row_words();
            d.ctg = nb * 16 + ctl;
            d.sboff = (uint32_t)ctl * 2048u;
        }
        decode_loop_any<PHASE>(Kw, d, sbase, tail + 1024 + wid * kWordRing, full_b, empty, nchunks);
    } else if (tid == 8 * 32) {
        // ---- MMA issuer
        const uint32_t idesc = idesc_f16(128, PHASE == 0 ? 128 : 256);
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
            const int s = c % NST;
            const uint32_t ph = (uint32_t)(c / NST) & 1u;
            mbar_wait(&full_a[s], ph);
            mbar_wait(&full_b[s], ph);
            tc_fence_after();
            const uint32_t aA = smem_u32(sbase + s * C::STAGE), aB = aA + C::A_BYTES;
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
            umma_commit(&empty[s]);
        }
        umma_commit(done);
    } else if (tid == 9 * 32) {
        // ---- A producer (TMA)
        const uint32_t bytes = (uint32_t)(PHASE == 0 ? 2 : 1) * (uint32_t)nmt * 16384u;
        // the stages hold NST chunks; the boxes of the next kPfAhead chunks beyond them are prefetched into L2, so that
        // a stage's load, issued when the MMA frees it, reads L2 rather than DRAM (one chunk ahead measured best: 3 and
        // 6 were 0.2% and 1.6% slower per layer)
        constexpr int kPfAhead = 1;
        auto prefetch = [&](int c) {
            if (c >= nchunks) return;
            if (PHASE == 0) {
                for (int q = 0; q < 2; ++q)
                    for (int mt = 0; mt < nmt; ++mt) tma_prefetch_2d(&tmA, c * 64, q * p.Prow + row0 + mt * 128);
            } else {
                for (int mt = 0; mt < nmt; ++mt) tma_prefetch_2d(&tmA, c * 64, row0 + mt * 128);
            }
        };
        for (int c = NST; c < NST + kPfAhead; ++c) prefetch(c);
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
            const int s = c % NST;
            prefetch(c + NST + kPfAhead);
            if (c >= NST) mbar_wait(&empty[s], (uint32_t)((c / NST) - 1) & 1u);
            uint8_t* sA = sbase + s * C::STAGE;
            mbar_arrive_expect_tx(&full_a[s], bytes);
            if (PHASE == 0) {
                for (int q = 0; q < 2; ++q)
                    for (int mt = 0; mt < nmt; ++mt)
                        tma_load_2d(sA + (q * 2 + mt) * 16384, &tmA, c * 64, q * p.Prow + row0 + mt * 128, &full_a[s]);
            } else {
                for (int mt = 0; mt < nmt; ++mt)
                    tma_load_2d(sA + mt * 16384, &tmA, c * 64, row0 + mt * 128, &full_a[s]);
            }
        }
        // every load issued has landed before the CTA can exit (bounded)
        for (int c = max(0, nchunks - NST); c < nchunks; ++c) mbar_wait(&full_a[c % NST], (uint32_t)(c / NST) & 1u);
    }

    // ---- epilogue (warps 0-7); a warp whose 32 rows are all past the tile's row count has nothing to store
    if (wid < 8 && (wid >> 2) * 128 + 32 * (wid & 3) < rows) {
        mbar_wait(done, 0);
        tc_fence_after();
        const int mt = wid >> 2;
        const int rloc = 32 * (wid & 3) + lane;
        const bool valid = mt * 128 + rloc < rows;
        const uint32_t tl = tbase + ((uint32_t)(32 * (wid & 3)) << 16);
        const int pr = row0 + mt * 128 + rloc;
        float v[128];
        if (PHASE == 0) {
            // the stages are free after `done`: per row, g (fp16) at stg, u (fp16) at stu, 16-byte chunks swizzled.
            // Three passes share one FWHT: gate (TMEM) -> g, up (TMEM) -> u then SwiGLU, a (stg) -> abuf.
            uint8_t* stg = sbase + tid * 256;
            uint8_t* stu = sbase + 65536 + tid * 256;
#pragma unroll 1
            for (int pass = 0; pass < 3; ++pass) {
                if (pass < 2) {
                    tmem_row128(tl + (uint32_t)((mt * 2 + pass) * 128), v);
                } else {
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        const uint4 aq = *reinterpret_cast<const uint4*>(stg + ((q ^ (tid & 15)) << 4));
                        const uint32_t aw[4] = {aq.x, aq.y, aq.z, aq.w};
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj)
                            v[q * 8 + jj] = __half2float(__ushort_as_half((unsigned short)(aw[jj >> 1] >> (16 * (jj & 1)))));
                    }
                }
                fwht128_regs(v);
                if (pass < 2) {
                    const __half* sv = vec + pass * 128;
                    uint8_t* st = pass ? stu : stg;
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        uint4 o;
                        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            const int j = q * 8 + 2 * jj;
                            const float2 t = f2_mul(f2_mul(make_float2(v[j], v[j + 1]), make_float2(kRsqrt128, kRsqrt128)),
                                                    __half22float2(*reinterpret_cast<const __half2*>(sv + j)));
                            __half2 h = __float22half2_rn(t);
                            ow[jj] = *reinterpret_cast<uint32_t*>(&h);
                        }
                        *reinterpret_cast<uint4*>(st + ((q ^ (tid & 15)) << 4)) = o;
                    }
                } else if (valid) {
                    uint4* op = reinterpret_cast<uint4*>(p.abuf + (size_t)pr * p.I + (size_t)nb * 128);
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        uint4 o;
                        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            __half2 h = __float22half2_rn(f2_mul(make_float2(v[q * 8 + 2 * jj], v[q * 8 + 2 * jj + 1]),
                                                                 make_float2(kRsqrt128, kRsqrt128)));
                            ow[jj] = *reinterpret_cast<uint32_t*>(&h);
                        }
                        op[q] = o;
                    }
                }
                if (pass == 1) {
                    // SwiGLU and suh_d, 8 values at a time: a = fp16(fp16(silu(g) u) suh_d), written over g
#pragma unroll 2
                    for (int q = 0; q < 16; ++q) {
                        const uint32_t off = (uint32_t)((q ^ (tid & 15)) << 4);
                        const uint4 gq = *reinterpret_cast<const uint4*>(stg + off);
                        const uint4 uq = *reinterpret_cast<const uint4*>(stu + off);
                        const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w}, uw[4] = {uq.x, uq.y, uq.z, uq.w};
                        uint32_t ow[4];
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            const __half2 g2 = *reinterpret_cast<const __half2*>(&gw[jj]);
                            const __half2 u2 = *reinterpret_cast<const __half2*>(&uw[jj]);
                            const int j = q * 8 + 2 * jj;
                            float g0 = __low2float(g2), g1 = __high2float(g2);
                            // SiLU with the hardware exp2 / reciprocal approximations (~2 ulp of fp32, far below the
                            // fp16 rounding that follows)
                            float a0 = rn16(__fdividef(g0, 1.0f + __expf(-g0)) * __low2float(u2));
                            float a1 = rn16(__fdividef(g1, 1.0f + __expf(-g1)) * __high2float(u2));
                            __half2 h = __floats2half2_rn(a0 * __half2float(vec[256 + j]), a1 * __half2float(vec[256 + j + 1]));
                            ow[jj] = *reinterpret_cast<uint32_t*>(&h);
                        }
                        *reinterpret_cast<uint4*>(stg + off) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
                    }
                }
            }
        } else {
            const float wt = valid ? p.pair_w[pr] : 0.0f;
            const float2 rw2 = make_float2(kRsqrt128 * wt, kRsqrt128 * wt);
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
                        for (int jj = 0; jj < 4; ++jj) {
                            const int c0 = hb * 128 + q * 8 + 2 * jj;
                            const float2 t = f2_mul(f2_mul(make_float2(v[q * 8 + 2 * jj], v[q * 8 + 2 * jj + 1]), rw2),
                                                    __half22float2(*reinterpret_cast<const __half2*>(vec + c0)));
                            __half2 h = __float22half2_rn(t);
                            ow[jj] = *reinterpret_cast<uint32_t*>(&h);
                        }
                        op[q] = o;
                    }
                }
            }
        }
    }
    __syncwarp();   // warps 8, 9: lanes 1-31 wait here for the lane that ran the MMA / TMA loop
    tc_fence_before();
    __syncthreads();
    if (wid == 8) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
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
        const int pr = p.pair_of[t * p.topk + k];
        if (pr < 0) continue;   // no pick (id -1)
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
    int A, mxb, Prow;
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
    L.Prow = (int)(P + 256);   // xh / abuf rows: the last tile reads up to 255 rows past the final pick
    size_t o = 0;
    L.ib = o; o += al1k((4 * (size_t)L.A + 1 + 2 * P + 16 + L.mxb + 1) * 4);
    L.fb = o; o += al1k(std::max<size_t>(P, 1) * 4);
    L.scr = o; o += al1k((size_t)exl3b_align_scratch((int)P, E));
    L.tiles = o; o += al1k(((P + 255) / 256 + L.A + 1) * 4);
    L.ntiles = o; o += 1024;
    L.xh = o; o += al1k((size_t)L.Prow * 2 * (size_t)H * 2);
    L.abuf = o; o += al1k((size_t)L.Prow * (size_t)I * 2);
    L.y = o; o += al1k(P * (size_t)H * 2);
    L.total = o;
    return L;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 2-D fp16 row-major [rows][inner] map with 64 x 128 boxes in the 128-byte swizzle (one K-major UMMA operand tile).
static int make_tmap(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
    if (!enc) return exl3b_fail(EXL3B_ECUDA, "exl3b_moe_prefill: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return exl3b_fail(EXL3B_ECUDA, "exl3b_moe_prefill: cuTensorMapEncodeTiled failed");
    return 0;
}

template <int PHASE>
static int launch_gemm(const PrefillArgs& p, const CUtensorMap& tm, int grid, cudaStream_t s) {
    using C = GemmCfg<PHASE>;
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(prefill_gemm_kernel<PHASE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        attr_dev = dev;
    }
    cudaError_t e = launch_k(prefill_gemm_kernel<PHASE>, dim3(grid), dim3(C::THREADS), (size_t)C::SMEM, s, p, tm);
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
    EXL3B_CHECK((long long)M * topk + 256 < (1ll << 30), "exl3b_moe_prefill: too many picks");
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
    prof_record(0, s);
    int rc = exl3b_align(ids, w, P, topk, E, 256, ib, (float*)(b + L.fb), L.A, L.mxb, b + L.scr,
                         exl3b_align_scratch(P, E), stream);
    if (rc) return rc;
    PrefillArgs p{};
    p.x = x; p.xs = x_stride; p.x_bf16 = x_bf16;
    p.M = M; p.topk = topk; p.P = P; p.Prow = L.Prow;
    p.ptrs = ptrs; p.kinfo = kinfo;
    p.H = H; p.I = I; p.K = K; p.E = E;
    p.out = out; p.os = out_stride; p.out_bf16 = out_bf16;
    const int A = L.A;
    p.act_expert = ib; p.act_start = ib + A; p.act_cnt = ib + 2 * A; p.n_act = ib + 4 * A;
    p.pair_tok = ib + 4 * A + 1; p.pair_of = p.pair_tok + P; p.pair_w = (const float*)(b + L.fb);
    p.tiles = (int*)(b + L.tiles); p.n_tiles = (int*)(b + L.ntiles);
    p.xh = (__half*)(b + L.xh); p.abuf = (__half*)(b + L.abuf); p.y = (__half*)(b + L.y);
    CUtensorMap tm_xh, tm_ab;
    rc = make_tmap(&tm_xh, p.xh, (uint64_t)H, (uint64_t)2 * L.Prow);
    if (rc) return rc;
    rc = make_tmap(&tm_ab, p.abuf, (uint64_t)I, (uint64_t)L.Prow);
    if (rc) return rc;
    cudaError_t e = launch_k(tiles_kernel, dim3(1), dim3(1024), 0, s, p);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    const int max_tiles = (P + 255) / 256 + A;
    e = launch_k(had_in_kernel, dim3((unsigned)max_tiles * 32u), dim3(256), 0, s, p);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    prof_record(1, s);
    rc = launch_gemm<0>(p, tm_xh, max_tiles * (I / 128), s);
    if (rc) return rc;
    prof_record(2, s);
    rc = launch_gemm<1>(p, tm_ab, max_tiles * (H / 256), s);
    if (rc) return rc;
    long long nc = (long long)M * (H / 8);
    e = launch_k(prefill_combine_kernel, dim3((unsigned)((nc + 255) / 256)), dim3(256), 0, s, p);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    prof_record(3, s);
    return exl3b_launch_status("exl3b_moe_prefill");
}
