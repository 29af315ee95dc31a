// exl3b_decode.cu -- routed-MoE decode path (few tokens): the reference's launch_ensure + GateUpKernel + DownKernel +
// CombineKernel (exl3_moe.a8.sycl:121-395, 837-1040, 1229-1314) re-designed for sm_100a.
//
// Three kernels per call (after the router), chained with programmatic dependent launch:
//   prep    (1 block): [device cache step: tier mask, LRU stamps, victims, fill plan] + grouping of the active picks
//                      by DISTINCT expert into entries (one expert, up to 8 of its picks), so an expert picked by several
//                      tokens is streamed once;
//   gate-up (clusters of 4 CTAs per (entry, 128-column block of I)): each CTA streams split-K units (projection,
//                      128-row k block) of one projection; the CTAs' sums meet in rank 0's shared memory (DSMEM), which
//                      runs the epilogue; then the CTAs copy the planned cache fills (host blob -> slot);
//   down    (one CTA per (entry, 128-column block of H)): the item's strip rows split evenly over the 8 warps, a
//                      shared-memory reduction, the epilogue and the weighted combine, and the cache commit
//                      (ptrs[e] = slot) by the last block to arrive.
// Small batches (<= 32 picks) skip the wait for prep: gate-up and down group the picks themselves (group_small) and the
// tier mask's rewrite of ids / w is written by the last down block.
// Each warp streams its units' 8-tile strips through a private SMEM ring filled by cp.async, decodes each lane's 8
// values of a tile straight into an mma.sync A fragment of W^T (exl3b_common.cuh) and multiplies it with the 8-token
// Hadamard-domain activation block (fp32 accumulate).  Every reduction runs in a fixed order (warp order, cluster
// rank order, pick order), so results do not depend on scheduling:
//   gate/up epilogue (:239-256): g = fp16(FWHT(g) r svh_g), u likewise, a = fp16(SiLU(g) u), a = fp16(a suh_d),
//                                abuf = fp16(FWHT(a) r)
//   down epilogue   (:355-364): y = FWHT(v) (r w) svh_d (fp32)
//   combine         (:387-394): out[m] = sum_k y[m,k] in fixed k order, by the last of the token's picks to finish.
// Cache fills are read from their host address (ptrs[e] until the commit), like the reference's write-through, while
// the gate-up blocks copy them into their slots.  Picks with weight exactly 0 (tier-masked) contribute exactly zero
// and are skipped (flag bit 0).
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"
#include "exl3b_ensure.cuh"
#include "exl3b_launch.h"
#include "exl3b_topk.cuh"
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
    int* cnt_c; int* blocks_done;
    __half* abuf; float* y;
    int maxent;
    // small batches (M <= kTokPerEnt, M topk <= kSmallPicks): the gate-up and down kernels group the picks themselves
    // from ids / w and the layer's tier state (t_*: null without a cache or tier); the tier mask's in-place rewrite
    // of ids / w is then done by the last down block
    int small;
    const int32_t* t_slot_of; const uint8_t* t_ram_res; const int32_t* t_safe;
    // routed small batches (exl3b_moe_decode_cached_routed): the router's logits [M][E]; prep, gate-up and down select
    // each token's top-k from them themselves (prep also writes ids / w for the caller)
    const float* logits; int routed;
};


constexpr int kSmallPicks = 32;   // small-batch mode: up to 32 picks (3 tokens at top-10)
static_assert(kSmallPicks <= kDeferMaskMax, "the cache step defers the tier-mask rewrite of every small batch");

// Grouping of a small batch in shared memory (the entry tables of route_prep_block, plus per-pick flags).
struct SmallTab {
    long long blob[kSmallPicks];
    int kv[kSmallPicks];
    float w[kSmallPicks][kTokPerEnt];
    unsigned char ntok[kSmallPicks];
    unsigned char tok[kSmallPicks][kTokPerEnt];
    unsigned char pick[kSmallPicks][kTokPerEnt];
    unsigned char act[kSmallPicks];      // pick active (weight != 0 when skipping zero weights)
    unsigned char masked[kSmallPicks];   // tier-masked: becomes (safe, 0)
    unsigned char tok_cnt[kTokPerEnt];
    int n, safe;
    int rid[kSmallPicks];     // routed: the picks selected in this block
    float rw[kSmallPicks];
};

// Routed small batches: warps 0 .. M - 1 select their token's picks into tb.rid / tb.rw (cand: 32 uint2 of scratch
// shared memory per warp, 8 bytes apart by warp); the caller synchronises the block before group_small reads them.
__device__ __forceinline__ void routed_select(const DecodeArgs& a, SmallTab& tb, uint2* cand_warp) {
    const int wid = threadIdx.x >> 5;
    if (wid < a.M) topk_warp_inl(a.logits, wid, a.E, a.topk, tb.rid, tb.rw, cand_warp);   // row wid of rid / rw
}

// ------------------------------------------------------------------------------------------------ prep
// Zero the arrival counters, group active picks by expert (ascending id, picks in ascending index), count active
// picks per token and zero the output rows of tokens with none.  All 1024 threads of one block; the picks pass
// through shared memory in chunks of kPrepChunk (one expert per thread scans each chunk for its picks).
constexpr int kPrepChunk = 2048;

__device__ __forceinline__ void route_prep_block(const DecodeArgs& a) {
    __shared__ int cnt[1024];
    __shared__ int sh_warp2[32];
    __shared__ int s_ids[kPrepChunk];
    __shared__ float s_w[kPrepChunk];
    const int tid = threadIdx.x, npairs = a.M * a.topk;
    const int nbH = a.H / 128;
    for (int i = tid; i < a.M * nbH; i += blockDim.x) a.cnt_c[i] = 0;
    if (tid == 0) a.blocks_done[0] = 0;
    for (int e = tid; e < a.E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    // pass 1: activity flags, per-expert counts, per-token counts (tokens never straddle a chunk)
    const int chunk = (kPrepChunk / a.topk) * a.topk;
    for (int c0 = 0; c0 < npairs; c0 += chunk) {
        const int c1 = min(npairs, c0 + chunk);
        for (int i = c0 + tid; i < c1; i += blockDim.x) {
            int e = a.ids[i];
            bool ok = e >= 0 && e < a.E;
            bool act = ok && !(a.skip_zero && a.w[i] == 0.0f);
            if (!ok && e != -1) set_error(kErrBounds);   // -1: no pick (expert-parallel ranks)
            a.pick_act[i] = act ? 1 : 0;
            s_ids[i - c0] = act ? e : -1;
            if (act) atomicAdd(&cnt[e], 1);
        }
        __syncthreads();
        for (int m = c0 / a.topk + tid; m < c1 / a.topk; m += blockDim.x) {
            int c = 0;
            for (int k = 0; k < a.topk; ++k) c += s_ids[m * a.topk + k - c0] >= 0 ? 1 : 0;
            a.tok_cnt[m] = c;
            if (c == 0) {   // no active pick: the token's output row is zero
                for (int col = 0; col < a.H; ++col) {
                    if (a.out_bf16 == 2) reinterpret_cast<float*>(a.out)[(long long)m * a.os + col] = 0.0f;
                    else if (a.out_bf16) reinterpret_cast<__nv_bfloat16*>(a.out)[(long long)m * a.os + col] = __float2bfloat16(0.0f);
                    else reinterpret_cast<__half*>(a.out)[(long long)m * a.os + col] = __float2half(0.0f);
                }
            }
        }
        __syncthreads();
    }
    // entry bases: exclusive scan of ceil(count / kTokPerEnt) over experts
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
    // pass 2: every expert thread collects its picks in ascending index
    int j = 0;
    for (int c0 = 0; c0 < npairs; c0 += chunk) {
        const int c1 = min(npairs, c0 + chunk);
        __syncthreads();
        for (int i = c0 + tid; i < c1; i += blockDim.x) {
            s_ids[i - c0] = a.pick_act[i] ? a.ids[i] : -1;
            s_w[i - c0] = a.w[i];
        }
        __syncthreads();
        if (n > 0 && j < n) {
            for (int i = c0; i < c1 && j < n; ++i) {
                if (s_ids[i - c0] != e) continue;
                int en = base + j / kTokPerEnt, sl = j % kTokPerEnt;
                if (sl == 0) {
                    a.ent_expert[en] = e;
                    a.ent_n[en] = min(kTokPerEnt, n - j);
                    a.ent_blob[en] = (long long)a.ptrs[e];
                    a.ent_k[en] = a.kinfo ? a.kinfo[e] : (a.K | (a.K << 4) | (a.K << 8));
                    for (int q = 0; q < kTokPerEnt; ++q) { a.ent_tok[en * kTokPerEnt + q] = 0; a.ent_pick[en * kTokPerEnt + q] = 0; }
                }
                a.ent_tok[en * kTokPerEnt + sl] = i / a.topk;
                a.ent_w[en * kTokPerEnt + sl] = s_w[i - c0];
                a.ent_pick[en * kTokPerEnt + sl] = i;
                ++j;
            }
        }
    }
}

// Small batches (M <= kTokPerEnt tokens, at most 128 picks) in one warp, without block barriers: the same results as
// ensure_block + route_prep_block when every pick is a hit or tier-masked (no cache miss, ids in range).  Returns
// false, having written nothing, when that does not hold; the caller then runs the block path.
__device__ __forceinline__ bool prep_fast_warp(const EnsureArgs& ea, const DecodeArgs& a, int cached) {
    constexpr int J = 4;   // picks per lane: i = lane + 32 j
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int np = a.M * a.topk, E = a.E;
    const unsigned lt = (1u << lane) - 1u;
    const int kpack = a.K | (a.K << 4) | (a.K << 8);
    int id[J];
    float wv[J];
    bool val[J], none[J] = {false, false, false, false};
    bool bad = false;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int i = lane + 32 * j;
        val[j] = i < np;
        id[j] = val[j] ? a.ids[i] : 0;
        wv[j] = val[j] ? a.w[i] : 0.0f;
        if (val[j] && id[j] == -1 && !cached) { val[j] = false; none[j] = true; }   // no pick
        bad |= val[j] && (id[j] < 0 || id[j] >= E);
    }
    if (__any_sync(FULL, bad)) return false;
    const bool tier = cached && ea.ram_res != nullptr;
    const int L = cached ? ea.layer : 0;
    const int safe = tier ? ea.safe[L] : 0;
    const int ring0 = tier ? ea.ring[0] : 0;
    const int tick0 = cached ? ea.tick[0] : 0;
    const int so_safe = tier ? ea.slot_of[L * E + safe] : -1;
    int so[J], kv[J];
    long long pt[J];
    bool masked[J];
    bool miss = false;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        so[j] = -1; kv[j] = kpack; pt[j] = 0; masked[j] = false;
        if (val[j]) {
            const int key = L * E + id[j];
            so[j] = cached ? ea.slot_of[key] : 0;
            const bool in_ram = tier ? ea.ram_res[key] != 0 : true;
            pt[j] = (long long)a.ptrs[id[j]];
            if (a.kinfo) kv[j] = a.kinfo[id[j]];
            masked[j] = tier && so[j] < 0 && !in_ram;
            miss |= cached && !masked[j] && so[j] < 0;
            miss |= masked[j] && so_safe < 0;   // the safe expert itself would be a miss
        }
    }
    if (__any_sync(FULL, miss)) return false;
    if (cached) {
        const long long pt_safe = tier ? (long long)a.ptrs[safe] : 0;
        const int kv_safe = (tier && a.kinfo) ? a.kinfo[safe] : kpack;
        // 1. tier mask in ascending pick index: ring log, pick -> (safe, 0).  Of a call's masked picks only the last
        // ring_cap land in the ring (sequentially, earlier ones would be overwritten within the call): each slot is
        // written once, so parallel writes give the sequential result.
        int nmask = 0;
#pragma unroll
        for (int j = 0; j < J; ++j) nmask += __popc(__ballot_sync(FULL, masked[j]));
        int base = ring0;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const unsigned bm = __ballot_sync(FULL, masked[j]);
            if (masked[j]) {
                const int i = lane + 32 * j;
                const int c = base - ring0 + __popc(bm & lt);   // rank among the call's masked picks
                if (c >= nmask - ea.ring_cap) ea.ring[1 + ((base + __popc(bm & lt)) % ea.ring_cap)] = L * E + id[j];
                if (!ea.defer_mask) {   // deferred: the last down block rewrites ids / w
                    ea.ids[i] = safe;
                    ea.w[i] = 0.0f;
                }
                id[j] = safe; wv[j] = 0.0f; so[j] = so_safe; pt[j] = pt_safe; kv[j] = kv_safe;
            }
            base += __popc(bm);
        }
        // 2.-4. tick; every used slot stamped with it unless pinned (T exceeds every unpinned stamp: a max)
        const int T = tick0 + 1;
#pragma unroll
        for (int j = 0; j < J; ++j)
            if (val[j] && so[j] >= 0) atomicMax(&ea.slot_last[so[j]], T);
        if (lane == 0) {
            if (tier) ea.ring[0] = base;
            ea.tick[0] = T;
            ea.fill_list[0] = 0;
            if (ea.vict) ea.vict[0] = 0;
        }
    }
    // grouping: one entry per distinct active expert (M <= kTokPerEnt: an expert has at most M picks), ascending id,
    // its picks in ascending index
    bool act[J];
    int sl[J], cnt[J], en[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        act[j] = val[j] && !(a.skip_zero && wv[j] == 0.0f);
        sl[j] = 0; cnt[j] = 0; en[j] = 0;
    }
#pragma unroll
    for (int qj = 0; qj < J; ++qj) {
        if (qj * 32 >= np) break;
        for (int ql = 0; ql < 32 && qj * 32 + ql < np; ++ql) {
            const int eq = __shfl_sync(FULL, id[qj], ql);
            const int aq = __shfl_sync(FULL, (int)act[qj], ql);
#pragma unroll
            for (int j = 0; j < J; ++j)
                if (act[j] && aq && eq == id[j]) {
                    ++cnt[j];
                    if (qj * 32 + ql < lane + 32 * j) ++sl[j];
                }
        }
    }
    int ndist = 0;
#pragma unroll
    for (int qj = 0; qj < J; ++qj) {
        if (qj * 32 >= np) break;
        const bool first_q = act[qj] && sl[qj] == 0;
        ndist += __popc(__ballot_sync(FULL, first_q));
        for (int ql = 0; ql < 32 && qj * 32 + ql < np; ++ql) {
            const int eq = __shfl_sync(FULL, id[qj], ql);
            const int fq = __shfl_sync(FULL, (int)first_q, ql);
#pragma unroll
            for (int j = 0; j < J; ++j)
                if (fq && eq < id[j]) ++en[j];
        }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int i = lane + 32 * j;
        if (val[j] || none[j]) a.pick_act[i] = act[j] ? 1 : 0;
        if (!act[j]) continue;
        const int e8 = en[j] * kTokPerEnt;
        if (sl[j] == 0) {
            a.ent_expert[en[j]] = id[j];
            a.ent_n[en[j]] = cnt[j];
            a.ent_blob[en[j]] = pt[j];
            a.ent_k[en[j]] = kv[j];
            for (int q = cnt[j]; q < kTokPerEnt; ++q) { a.ent_tok[e8 + q] = 0; a.ent_pick[e8 + q] = 0; }
        }
        a.ent_tok[e8 + sl[j]] = i / a.topk;
        a.ent_w[e8 + sl[j]] = wv[j];
        a.ent_pick[e8 + sl[j]] = i;
    }
    if (lane == 0) a.n_ent[0] = ndist;
    for (int m = 0; m < a.M; ++m) {
        int c = 0;
#pragma unroll
        for (int j = 0; j < J; ++j) c += (act[j] && (lane + 32 * j) / a.topk == m) ? 1 : 0;
        c = __reduce_add_sync(FULL, (unsigned)c);
        if (lane == 0) a.tok_cnt[m] = c;
        if (c == 0) {   // no active pick: the token's output row is zero
            for (int col = lane; col < a.H; col += 32) {
                if (a.out_bf16 == 2) reinterpret_cast<float*>(a.out)[(long long)m * a.os + col] = 0.0f;
                else if (a.out_bf16) reinterpret_cast<__nv_bfloat16*>(a.out)[(long long)m * a.os + col] = __float2bfloat16(0.0f);
                else reinterpret_cast<__half*>(a.out)[(long long)m * a.os + col] = __float2half(0.0f);
            }
        }
    }
    return true;
}

// One warp groups a small batch into tb (the caller synchronises the block afterwards): the same picks per expert
// (in ascending pick index, at most kTokPerEnt per entry) and token counts as prep's grouping after the tier mask,
// computed from the call's ids / w (read from L2: they were written by kernels before this one) and the read-only
// tier state.  Entries are numbered in the order of their experts' first picks (prep numbers them by expert id; no
// result depends on the order).  Concurrent cache-state writes by the prep kernel do not change the result: a miss
// keeps reading its host copy until the commit, and the mask of a picked key does not depend on slot assignment.
__device__ __forceinline__ void group_small(const DecodeArgs& a, SmallTab& tb) {
    static_assert(kSmallPicks == 32, "one pick per lane");
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int np = a.M * a.topk, E = a.E;
    const int kpack = a.K | (a.K << 4) | (a.K << 8);
    const bool tier = a.t_ram_res != nullptr && a.t_slot_of != nullptr && a.t_safe != nullptr;
    // two dependent rounds of L2 loads: (ids, w, safe), then every table entry the pick may need (its own and the
    // safe expert's), selected afterwards
    const int safe = tier ? __ldcg(a.t_safe) : 0;
    int id = lane < np ? (a.routed ? tb.rid[lane] : __ldcg(a.ids + lane)) : -1;
    float wv = lane < np ? (a.routed ? tb.rw[lane] : __ldcg(a.w + lane)) : 0.0f;
    const bool safe_ok = tier && safe >= 0 && safe < E;
    const long long p_safe = safe_ok ? (long long)__ldcg(a.ptrs + safe) : 0;
    const int k_safe = (safe_ok && a.kinfo) ? __ldcg(a.kinfo + safe) : kpack;
    const bool inr = id >= 0 && id < E;
    const int so = (inr && tier) ? __ldcg(a.t_slot_of + id) : 0;
    const int rr = (inr && tier) ? (int)__ldcg(a.t_ram_res + id) : 1;
    long long pt = inr ? (long long)__ldcg(a.ptrs + id) : 0;
    int kv = (inr && a.kinfo) ? __ldcg(a.kinfo + id) : kpack;
    const bool msk = inr && tier && so < 0 && rr == 0;
    if (msk) { id = safe; wv = 0.0f; pt = p_safe; kv = k_safe; }
    const bool act = inr && !(msk && !safe_ok) && !(a.skip_zero && wv == 0.0f);
    // lanes of the same expert; rank among them; entries of up to kTokPerEnt picks in order of first pick
    const unsigned lt = (1u << lane) - 1u;
    const unsigned grp = __match_any_sync(FULL, act ? id : -2 - lane);
    const int sl = __popc(grp & lt), cnt = __popc(grp);
    const int lead = __ffs(grp) - 1;
    const bool first = act && sl == 0;
    const int nent = first ? (cnt + kTokPerEnt - 1) / kTokPerEnt : 0;   // entries of the lead lane's expert
    int base;   // entries before the expert's first one
    if (__any_sync(FULL, nent > 1)) {
        int x = nent;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) { const int y = __shfl_up_sync(FULL, x, o); if (lane >= o) x += y; }
        base = __shfl_sync(FULL, x - nent, lead);
    } else {
        base = __popc(__ballot_sync(FULL, first) & ((1u << lead) - 1u));
    }
    const int ndist = __reduce_add_sync(FULL, (unsigned)nent);
    if (lane < kSmallPicks) { tb.act[lane] = act ? 1 : 0; tb.masked[lane] = msk ? 1 : 0; }
    if (act) {
        const int en = base + sl / kTokPerEnt, q = sl % kTokPerEnt;
        const int nt = min(kTokPerEnt, cnt - (sl / kTokPerEnt) * kTokPerEnt);
        if (q == 0) {
            tb.blob[en] = pt;
            tb.kv[en] = kv;
            tb.ntok[en] = (unsigned char)nt;
            for (int r = nt; r < kTokPerEnt; ++r) { tb.tok[en][r] = 0; tb.pick[en][r] = 0; tb.w[en][r] = 0.0f; }
        }
        tb.tok[en][q] = (unsigned char)(lane / a.topk);
        tb.pick[en][q] = (unsigned char)lane;
        tb.w[en][q] = wv;
    }
    for (int m = 0; m < a.M; ++m) {
        const int c = __popc(__ballot_sync(FULL, act && lane / a.topk == m));
        if (lane == 0) tb.tok_cnt[m] = (unsigned char)c;
    }
    if (lane == 0) { tb.n = ndist; tb.safe = safe; }
}

// Cached calls run the device cache step first (in place on ids / w), then the grouping.  Small batches try the
// one-warp path first (the other warps zero the arrival counters meanwhile).
__global__ void __launch_bounds__(1024, 1) prep_kernel(EnsureArgs ea, DecodeArgs da, int cached) {   // 64 registers: no spills
    __shared__ int sh_fast;
    __shared__ uint2 sh_cand[kTokPerEnt][32];
    pdl_wait();
    pdl_trigger();
    if (da.routed) {   // the call's picks (the router op's outputs), selected here from the logits
        const int wid = threadIdx.x >> 5;
        if (wid < da.M)
            topk_warp_inl(da.logits, wid, da.E, da.topk, const_cast<int32_t*>(da.ids), const_cast<float*>(da.w),
                          sh_cand[wid]);   // row wid of ids / w
        __syncthreads();
    }
    if (da.M <= kTokPerEnt && da.M * da.topk <= 128 && !(cached && ea.prefetch)) {
        if (threadIdx.x < 32) {
            const bool ok = prep_fast_warp(ea, da, cached);
            if (threadIdx.x == 0) sh_fast = ok ? 1 : 0;
        } else {
            const int nbH = da.H / 128;
            for (int i = threadIdx.x - 32; i < da.M * nbH; i += blockDim.x - 32) da.cnt_c[i] = 0;
            if (threadIdx.x == 32) da.blocks_done[0] = 0;
        }
        __syncthreads();
        if (sh_fast) return;
    }
    if (cached) {
        ensure_block(ea);
        __syncthreads();
    }
    route_prep_block(da);
}

// ------------------------------------------------------------------------------------------------ streaming core
// Each warp streams its units' 8-tile strips row by row through a private SMEM ring filled with cp.async (16 B,
// L2-only), NST - 1 rows ahead of the decode.  A strip row is 2 PLANAR4 groups; in SMEM each plane of a group is
// padded to 4G + 8 words (D > 1), so the two words a lane reads per tile -- word (tile j, period g, plane i) at
// i*PS + j*G + g -- fall in distinct banks across the warp.  Unit metadata is loaded one unit ahead.
constexpr int kStages = 4;   // ring rows of gate-up (and of down for K = 5); divides the 8 rows of a unit

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
static_assert(kTokPerEnt * kXsStride * 2 <= kTokPerEnt * 128 * 4, "down B operand fits the warp's accumulator area");

template <int KFIX, int PHASE>
struct StreamCfg {
    static constexpr int ROWW = KFIX ? Ring<KFIX>::ROWW : kRowMaxWords;
    static constexpr int STAGE = ROWW;
    // down with rows of <= 1 KB keeps a whole unit in flight: its CTAs issue 7 of the 8 rows before they wait for
    // the gate-up kernel, so that only the decode is left once abuf is ready
    static constexpr int NST = (PHASE == 1 && ROWW <= 256) ? 8 : kStages;
    static constexpr int WARP_WORDS = NST * STAGE + (PHASE == 0 ? 2 * kSideWords + kTokPerEnt * kXsStride / 2 : 0);
    static constexpr int SMEM_BYTES = 8 * WARP_WORDS * 4;
};

struct UMeta {
    int valid, ent, f0, f1, f2, K, kv, ntok, tok, pick;   // f0..f2: (proj, nb, kb) gate-up; (nbh, first row, -) down
    int nr;                // strip rows of the unit: 8 (gate-up), 1..8 (down)
    const uint8_t* blob;
    const uint32_t* src;   // first word of the unit's strip (row 0)
    int rs;                // words between strip rows
};

template <int PHASE>
__device__ __forceinline__ UMeta load_meta(const DecodeArgs& a, int u, int n_units, const SmallTab* tb) {
    UMeta m;
    const int lane = threadIdx.x & 31;
    m.valid = u < n_units;
    if (!m.valid) {
        m.ent = 0; m.f0 = m.f1 = m.f2 = 0; m.K = 3; m.kv = 0; m.ntok = 0; m.tok = 0; m.pick = 0; m.blob = nullptr;
        m.src = nullptr; m.rs = 0; m.nr = 0;
        return m;
    }
    if (PHASE == 0) {
        const int nKB = a.H / 128, nbI = a.I / 128;
        m.f2 = u % nKB; int r = u / nKB;
        m.f1 = r % nbI; r /= nbI;
        m.f0 = r & 1; m.ent = r >> 1;
        m.nr = 8;
    } else {
        // down unit u = ((ent nbH + nbh) 8 + w) nch + c: chunk c (<= 8 rows) of warp w's rows [w R, (w + 1) R) of the
        // item's I/16 strip rows, R = I/128
        const int R = a.I / 128, nch = (R + 7) / 8, nbH = a.H / 128;
        const int c = u % nch; int r = u / nch;
        const int w = r % 8; r /= 8;
        m.f1 = w * R + 8 * c;
        m.nr = min(8, R - 8 * c);
        m.f0 = r % nbH; m.ent = r / nbH; m.f2 = 0;
    }
    if (tb) {
        m.blob = reinterpret_cast<const uint8_t*>(tb->blob[m.ent]);
        m.ntok = tb->ntok[m.ent];
        m.kv = tb->kv[m.ent];
        m.tok = lane < kTokPerEnt ? tb->tok[m.ent][lane] : 0;
        m.pick = lane < kTokPerEnt ? tb->pick[m.ent][lane] : 0;
    } else {
        m.blob = reinterpret_cast<const uint8_t*>(__ldcg(a.ent_blob + m.ent));
        m.ntok = __ldcg(a.ent_n + m.ent);
        m.kv = __ldcg(a.ent_k + m.ent);
        m.tok = lane < kTokPerEnt ? __ldcg(a.ent_tok + m.ent * kTokPerEnt + lane) : 0;
        m.pick = lane < kTokPerEnt ? __ldcg(a.ent_pick + m.ent * kTokPerEnt + lane) : 0;
    }
    m.K = PHASE == 0 ? (m.f0 ? (m.kv >> 4) & 15 : m.kv & 15) : (m.kv >> 8) & 15;
    const Geom gm{a.H, a.I, m.kv & 15, (m.kv >> 4) & 15, (m.kv >> 8) & 15};
    const uint32_t* words = reinterpret_cast<const uint32_t*>(m.blob);
    if (PHASE == 0) {
        m.rs = (int)gm.gu_row_words();
        m.src = words + (size_t)(m.f2 * 8) * m.rs + (m.f0 ? (size_t)(a.I / 16) * 8 * gm.Kg : 0) + (size_t)(m.f1 * 2) * 4 * 8 * m.K;
    } else {
        m.rs = (int)gm.d_row_words();
        m.src = words + gm.gu_words() + (size_t)m.f1 * m.rs + (size_t)(m.f0 * 2) * 4 * 8 * m.K;
    }
    return m;
}

// Issue the cp.async copies of stream row r of unit m into `stage` (and, for gate-up row 0, its side slot: the
// unit's suh block and the x blocks of its tokens).
template <int K, int PHASE>
__device__ __forceinline__ void issue_row(const DecodeArgs& a, const UMeta& m, int r, uint32_t* stage, uint32_t* side,
                                          const LaneK<K>& lk) {
    using R = Ring<K>;
    const int lane = threadIdx.x & 31;
    const uint32_t* src = m.src + (size_t)r * m.rs;
#pragma unroll
    for (int q = 0; q < 3; ++q)
        if (lane + 32 * q < R::CHUNKS) cp_async16(stage + lk.dst[q], src + 4 * (lane + 32 * q));
    if (PHASE == 0 && r == 0) {
        const Geom gm{a.H, a.I, m.kv & 15, (m.kv >> 4) & 15, (m.kv >> 8) & 15};
        if (lane < 16)
            cp_async16(side + lane * 4, m.blob + gm.off_suh_g() + (size_t)m.f0 * a.H * 2 + (size_t)m.f2 * 256 + lane * 16);
        for (int c0 = 0; c0 < 16 * m.ntok; c0 += 32) {   // uniform trip count: the shuffle sees every lane
            const int c = c0 + lane, t = (c >> 4) & 7, j = c & 15;
            const int tk = __shfl_sync(0xffffffffu, m.tok, t);
            if (c < 16 * m.ntok)
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
    for (int t = 0; t < m.ntok; ++t) {   // columns of padding tokens are never read back
        uint2 o = make_uint2(0u, 0u);
        {
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

// Item epilogues (one warp per token t of the entry; lane holds columns 4 lane .. 4 lane + 3 of the 128-block).
// Gate-up (:239-256): g = fp16(FWHT(g) r svh_g), u likewise, a = fp16(SiLU(g) u), a = fp16(a suh_d),
// abuf = fp16(FWHT(a) r).
// The lane's scale vectors (svh_g, svh_u, suh_d: 4 fp16 each at columns 4 lane..) and the token's pick index, loaded
// before the item's decode so that the epilogue waits on no global load.
// Non-coherent 8-byte load issued where it stands (volatile: not sunk to its first use), so that the scale vectors
// of an item's epilogue are in flight during the item's decode.
__device__ __forceinline__ uint2 ldg_early(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

struct GuEpi {
    uint2 svg, svu, sud;
    int pick;
};
__device__ __forceinline__ GuEpi gu_epi_load(const DecodeArgs& a, int ent, int nb, int t, const SmallTab* tb) {
    const int lane = threadIdx.x & 31;
    const int kv = tb ? tb->kv[ent] : __ldcg(a.ent_k + ent);
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(tb ? tb->blob[ent] : __ldcg(a.ent_blob + ent));
    const Geom gm{a.H, a.I, kv & 15, (kv >> 4) & 15, (kv >> 8) & 15};
    const size_t col = (size_t)(nb * 128 + 4 * lane) * 2;
    GuEpi q;
    q.svg = ldg_early(blob + gm.off_svh_g() + col);
    q.svu = ldg_early(blob + gm.off_svh_u() + col);
    q.sud = ldg_early(blob + gm.off_suh_d() + col);
    q.pick = tb ? tb->pick[ent][t] : __ldcg(a.ent_pick + ent * kTokPerEnt + t);
    return q;
}

__device__ __forceinline__ void gu_token_epilogue(const DecodeArgs& a, const GuEpi& q, int nb, const float g_in[4],
                                                  const float u_in[4]) {
    const int lane = threadIdx.x & 31;
    const __half* svg = reinterpret_cast<const __half*>(&q.svg);
    const __half* svu = reinterpret_cast<const __half*>(&q.svu);
    const __half* sud = reinterpret_cast<const __half*>(&q.sud);
    const int pick = q.pick;
    float g[4] = {g_in[0], g_in[1], g_in[2], g_in[3]}, u[4] = {u_in[0], u_in[1], u_in[2], u_in[3]};
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

// Down (:355-364): y = FWHT(v) (r w) svh_d (fp32); then the combine (:387-394) of the token's 128-block by the last
// of its active picks to finish: out[m] = sum_k y[m,k] in fixed k order.
__device__ __forceinline__ uint2 dn_epi_load(const DecodeArgs& a, int ent, int nbh, const SmallTab* tb) {
    const int lane = threadIdx.x & 31;
    const int kv = tb ? tb->kv[ent] : __ldcg(a.ent_k + ent);
    const uint8_t* blob = reinterpret_cast<const uint8_t*>(tb ? tb->blob[ent] : __ldcg(a.ent_blob + ent));
    const Geom gm{a.H, a.I, kv & 15, (kv >> 4) & 15, (kv >> 8) & 15};
    return ldg_early(blob + gm.off_svh_d() + (size_t)(nbh * 128 + 4 * lane) * 2);
}

__device__ __forceinline__ void dn_token_epilogue(const DecodeArgs& a, int ent, int nbh, int t, const float v_in[4],
                                                  const SmallTab* tb, const uint2 v_svd) {
    const int lane = threadIdx.x & 31;
    const int nbH = a.H / 128;
    const __half* svd = reinterpret_cast<const __half*>(&v_svd);
    const int pick = tb ? tb->pick[ent][t] : __ldcg(a.ent_pick + ent * kTokPerEnt + t);
    const float wt = tb ? tb->w[ent][t] : __ldcg(a.ent_w + ent * kTokPerEnt + t);
    float v[4] = {v_in[0], v_in[1], v_in[2], v_in[3]};
    fwht128_warp(v, lane);
    float4 yv;
    yv.x = v[0] * (kRsqrt128 * wt) * __half2float(svd[0]);
    yv.y = v[1] * (kRsqrt128 * wt) * __half2float(svd[1]);
    yv.z = v[2] * (kRsqrt128 * wt) * __half2float(svd[2]);
    yv.w = v[3] * (kRsqrt128 * wt) * __half2float(svd[3]);
    __stcg(reinterpret_cast<float4*>(a.y + (size_t)pick * a.H + nbh * 128 + 4 * lane), yv);
    // the warp barrier orders every lane's y store before lane 0's release; for the last arrival, lane 0's acquire
    // and the warp barrier after it make the other picks' rows visible to every lane
    __syncwarp();
    const int mt = pick / a.topk;
    int oc = 0;
    if (lane == 0)
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;\n" : "=r"(oc) : "l"(&a.cnt_c[mt * nbH + nbh]) : "memory");
    oc = __shfl_sync(0xffffffffu, oc, 0);
    __syncwarp();
    const int tcnt = tb ? (int)tb->tok_cnt[mt] : __ldcg(a.tok_cnt + mt);
    if (oc == tcnt - 1) {
        // up to 12 picks' rows and flags loaded at once (one round trip), then summed in pick order; rows of
        // inactive picks (in bounds, never written this call) are loaded and skipped
        constexpr int kComb = 12;
        float sm[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k0 = 0; k0 < a.topk; k0 += kComb) {
            float4 q4[kComb];
            int on[kComb];
#pragma unroll
            for (int j = 0; j < kComb; ++j) {
                const int k = k0 + j, pp = mt * a.topk + k;
                on[j] = k < a.topk ? (tb ? (int)tb->act[pp] : __ldcg(a.pick_act + pp)) : 0;
                q4[j] = k < a.topk ? __ldcg(reinterpret_cast<const float4*>(a.y + (size_t)pp * a.H + nbh * 128 + 4 * lane))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < kComb; ++j)
                if (on[j]) { sm[0] += q4[j].x; sm[1] += q4[j].y; sm[2] += q4[j].z; sm[3] += q4[j].w; }
        }
        store_out(a, (long long)mt * a.os + nbh * 128 + 4 * lane, sm);
    }
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

// Stream a warp's units (unit ids u0, u0 + ustep, ... : nu of them, all of one item) row by row through the warp's
// SMEM ring (C::NST - 1 rows in flight) and accumulate W^T B over all of them
// into acc.  PHASE 1 waits for the previous kernel (wait_pdl) after the ring prologue is issued, before its first
// read of abuf.
template <int KFIX, int PHASE>
__device__ __forceinline__ void run_units(const DecodeArgs& a, int u0, int ustep, int nu, uint32_t* ring, uint32_t* side,
                                          __half* xs, float acc[8][4], const LaneK<KFIX ? KFIX : 3>& lkf, bool wait_pdl,
                                          const SmallTab* tb) {
    using C = StreamCfg<KFIX, PHASE>;
    constexpr int NST = C::NST;
    static_assert(8 % NST == 0, "ring slots must repeat every unit");
    const int lane = threadIdx.x & 31;
    auto meta = [&](int i) { return load_meta<PHASE>(a, u0 + i * ustep, i < nu ? 0x7FFFFFFF : 0, tb); };
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) acc[jj][0] = acc[jj][1] = acc[jj][2] = acc[jj][3] = 0.0f;
    UMeta mc = meta(0);
    if (mc.valid) {
#pragma unroll
        for (int r = 0; r < NST - 1; ++r) {
            if (PHASE == 0 || r < mc.nr) issue_any<KFIX, PHASE>(a, mc, r, ring + r * C::STAGE, side, lkf);
            cp_commit();
        }
    }
    if (PHASE == 1 && wait_pdl) {
        pdl_wait();
        pdl_trigger();
    }
    const int tk = lane >> 2, kq = 2 * (lane & 3);
    for (int i = 0; i < nu; ++i) {
        const UMeta mn = meta(i + 1);
        uint32_t* sd = side + (i & 1) * kSideWords;
        uint32_t* sdn = side + ((i + 1) & 1) * kSideWords;
        if (PHASE == 1) {
            // down: the unit's B operand (the unit's 16 nr k-values of each token's abuf row, written by the gate-up
            // kernel) into xs, one L2 round trip per unit instead of one per row (plain loads: the ring's copy groups
            // stay in flight)
            for (int c0 = 0; c0 < 16 * mc.ntok; c0 += 32) {   // uniform trip count: the shuffle sees every lane
                const int c = c0 + lane, t = (c >> 4) & 7, j = c & 15;
                const int pk = __shfl_sync(0xffffffffu, mc.pick, t);
                if (c < 16 * mc.ntok && j < 2 * mc.nr)
                    *reinterpret_cast<uint4*>(xs + t * kXsStride + j * 8) =
                        __ldcg(reinterpret_cast<const uint4*>(a.abuf + (size_t)pk * a.I + mc.f1 * 16 + j * 8));
            }
            __syncwarp();
        }
#pragma unroll 2   // two rows per iteration: the loop body stays in the instruction cache (a fully unrolled unit is
                   // straight-line code fetched once per SM, measured 10% slower)
        for (int r = 0; r < 8; ++r) {
            constexpr int L = NST - 1;
            const int rr = r + L;   // row issued now: of this unit, or (rr >= 8) of the next one
            // a unit of fewer than 8 rows is its warp's last: nothing follows it
            if (rr < 8) { if (PHASE == 0 || rr < mc.nr) issue_any<KFIX, PHASE>(a, mc, rr, ring + (rr % NST) * C::STAGE, sd, lkf); }
            else if (mn.valid && (PHASE == 0 || rr - 8 < mn.nr)) issue_any<KFIX, PHASE>(a, mn, rr - 8, ring + (rr % NST) * C::STAGE, sdn, lkf);
            cp_commit();
            cp_wait<NST - 1>();
            __syncwarp();
            const uint32_t* stage = ring + (r % NST) * C::STAGE;
            if (PHASE == 0 && r == 0) unit_xh(a, mc, sd, xs);
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xs + tk * kXsStride + r * 16 + kq);
            const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xs + tk * kXsStride + r * 16 + kq + 8);
            if (PHASE == 0 || r < mc.nr) consume_any<KFIX>(mc.K, stage, b0, b1, acc, lkf);
            __syncwarp();
        }
        mc = mn;
    }
    cp_wait<0>();
    __syncwarp();
}

// acc (mma accumulator layout: acc[jj][q] = column jj*16 + lane/4 (+8 for q >= 2), token 2(lane%4) + (q & 1)) ->
// red[token][column] (128 columns x kTokPerEnt tokens).
__device__ __forceinline__ void acc_to_smem(const float acc[8][4], float* red) {
    const int lane = threadIdx.x & 31;
    const int c0 = lane >> 2, t0 = 2 * (lane & 3);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
        red[(t0 + 0) * 128 + jj * 16 + c0] = acc[jj][0];
        red[(t0 + 1) * 128 + jj * 16 + c0] = acc[jj][1];
        red[(t0 + 0) * 128 + jj * 16 + c0 + 8] = acc[jj][2];
        red[(t0 + 1) * 128 + jj * 16 + c0 + 8] = acc[jj][3];
    }
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
// Cluster-wide barrier (release / acquire): every CTA of the cluster reaches it the same number of times.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// Store to the shared memory of CTA `rank` of this cluster at the address this CTA uses for `p`.
__device__ __forceinline__ void st_dsmem(float* p, uint32_t rank, float v) {
    uint32_t la = (uint32_t)__cvta_generic_to_shared(p), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

// Gate-up: a cluster of cs CTAs (4, or 2 when H/128 is odd) per item (entry, 128-column block of I).  The item's
// 2 H/128 units (proj, 128-row k-block) are split evenly: CTA rank r takes units of projection r / (cs/2), k-blocks
// (r % (cs/2)) * upc + w + 8 j for its warp w.  Each CTA sums its warps' accumulators in shared memory (fixed
// order); CTAs r > 0 store the sums of the item's tokens into rank 0's gather slot r - 1 (DSMEM), rank 0 keeps its
// own in place.  After one cluster barrier rank 0 adds the sums of each projection in rank order and runs the
// epilogue, one warp per token.  Items are dealt to clusters round-robin; no global partials, no atomics.
// Dynamic shared memory: 8 warp areas, the gather slots ((cs - 1) x min(M, 8) tokens x 128 fp32), the small-batch
// table.
__host__ __device__ constexpr int gu_gather_tokens(int M) { return M < 1 ? 1 : (M < kTokPerEnt ? M : kTokPerEnt); }
__host__ __device__ constexpr int gu_gather_floats(int cs, int M) { return (cs - 1) * gu_gather_tokens(M) * 128; }

template <int KFIX>
__global__ void __launch_bounds__(256, 2) gu_cluster_kernel(DecodeArgs a) {
    using C = StreamCfg<KFIX, 0>;
    extern __shared__ __align__(16) uint32_t smem[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    uint32_t* ring = smem + wid * C::WARP_WORDS;
    uint32_t* side = ring + C::NST * C::STAGE;
    __half* xs = reinterpret_cast<__half*>(side + 2 * kSideWords);
    const int mt = gu_gather_tokens(a.M);   // tokens per gather slot
    float* gather = reinterpret_cast<float*>(smem + 8 * C::WARP_WORDS);   // rank 0: slots [rank - 1][token][128]
    SmallTab* tab = reinterpret_cast<SmallTab*>(gather + gu_gather_floats((int)cluster_nctarank(), a.M));
    LaneK<KFIX ? KFIX : 3> lkf;
    lkf.init(lane);
    const int cs = (int)cluster_nctarank(), rank = (int)cluster_ctarank();
    const int cid = (int)blockIdx.x / cs, ncl = (int)gridDim.x / cs;
    // every CTA of the cluster has started before the first DSMEM store: arrive now, wait before that store
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
    bool cl_wait = true;
    const SmallTab* tb = nullptr;
    int n_ent;
    if (a.small) {
        // grouping in this CTA: no wait for the prep kernel until the cache fills (below)
        pdl_trigger();
        if (a.routed) {
            routed_select(a, *tab, reinterpret_cast<uint2*>(ring));   // the rings are free until the stream starts
            __syncthreads();
        }
        if (wid == 0) group_small(a, *tab);
        __syncthreads();
        tb = tab;
        n_ent = tab->n;
    } else {
        pdl_wait();
        pdl_trigger();
        n_ent = __ldcg(a.n_ent);
    }
    const int nKB = a.H / 128, nbI = a.I / 128;
    const int n_items = n_ent * nbI;
    const int half = cs / 2, upc = nKB / half;     // units per CTA, all of one projection
    const int proj = rank / half, kb0 = (rank % half) * upc;
    for (int item = cid; item < n_items; item += ncl) {
        const int ent = item / nbI, nb = item % nbI;
        const int nu = upc > wid ? (upc - wid + 7) / 8 : 0;
        const int u0 = ((ent * 2 + proj) * nbI + nb) * nKB + kb0 + wid;
        GuEpi epi{};
        const int ntok_e = tb ? (int)tb->ntok[ent] : __ldcg(a.ent_n + ent);
        if (rank == 0 && wid < ntok_e) epi = gu_epi_load(a, ent, nb, wid, tb);
        float acc[8][4];
        run_units<KFIX, 0>(a, u0, 8, nu, ring, side, xs, acc, lkf, false, tb);
        float* red = reinterpret_cast<float*>(ring);   // the warp's ring, side and xs are free now
        const int nwu = upc < 8 ? upc : 8;             // warps with units
        if (wid < nwu) acc_to_smem(acc, red);
        if (cl_wait) {
            asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
            cl_wait = false;
        }
        __syncthreads();
        // the gather slots hold mt tokens: an entry holds up to kTokPerEnt picks, more than mt only when a token
        // picks one expert several times; such entries go through the slots in chunks of mt tokens
        for (int t0 = 0; t0 < ntok_e; t0 += mt) {
            const int nt = min(mt, ntok_e - t0);
            for (int q = t0 * 128 + threadIdx.x; q < (t0 + nt) * 128; q += 256) {
                float sm = 0.0f;
                for (int w = 0; w < nwu; ++w) sm += reinterpret_cast<const float*>(smem + w * C::WARP_WORDS)[q];
                if (rank == 0) reinterpret_cast<float*>(smem)[q] = sm;   // in place: this thread alone reads index q
                else st_dsmem(gather + (rank - 1) * (mt * 128) + (q - t0 * 128), 0, sm);
            }
            cluster_sync_all();   // release / acquire: the gather slots are visible to rank 0; this CTA's reads of
                                  // the warps' sums are done before the next item reuses the rings
            if (rank == 0 && wid >= t0 && wid < t0 + nt) {
                float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
                for (int r = 0; r < cs; ++r) {
                    const float* src = r == 0 ? reinterpret_cast<const float*>(smem) + wid * 128
                                              : gather + (r - 1) * (mt * 128) + (wid - t0) * 128;
                    const float4 s4 = *reinterpret_cast<const float4*>(src + 4 * lane);
                    float* d = r < half ? g : u;
                    d[0] += s4.x; d[1] += s4.y; d[2] += s4.z; d[3] += s4.w;
                }
                gu_token_epilogue(a, epi, nb, g, u);
            }
            // rank 0 has read the gather slots before the cluster's next chunk or item overwrites them
            if (t0 + mt < ntok_e || item + ncl < n_items) cluster_sync_all();
        }
    }
    if (cl_wait) asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
    // cache fills are read by no kernel of this call (picks of a filled expert read its host copy until the commit
    // at the end of the down phase): copied after the items, off the decode's critical path (small batches wait for
    // the cache step here, whose fill list they need)
    if (a.small) pdl_wait();
    copy_fills(a);
}

// Down: one CTA per item (entry, 128-column block of H); the item's I/16 strip rows are split evenly over the 8
// warps (I/128 consecutive rows each).  The first item's weight rows are issued before the wait for the gate-up
// kernel (only abuf depends on it).
template <int KFIX>
__global__ void __launch_bounds__(256, 2) dn_item_kernel(DecodeArgs a) {
    using C = StreamCfg<KFIX, 1>;
    extern __shared__ __align__(16) uint32_t smem[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    uint32_t* ring = smem + wid * C::WARP_WORDS;
    float* red_all = reinterpret_cast<float*>(smem + 8 * C::WARP_WORDS);   // warps' accumulators [warp][token][128]
    float* red = red_all + wid * kTokPerEnt * 128;
    SmallTab* tab = reinterpret_cast<SmallTab*>(red_all + 8 * kTokPerEnt * 128);
    LaneK<KFIX ? KFIX : 3> lkf;
    lkf.init(lane);
    const SmallTab* tb = nullptr;
    int n_ent;
    if (a.small) {   // own grouping, as the gate-up kernel
        if (a.routed) {
            routed_select(a, *tab, reinterpret_cast<uint2*>(ring));
            __syncthreads();
        }
        if (wid == 0) group_small(a, *tab);
        __syncthreads();
        tb = tab;
        n_ent = tab->n;
    } else {
        n_ent = __ldcg(a.n_ent);   // prep finished before the gate-up kernel could let this one start
    }
    const int nKBd = a.I / 128, nbH = a.H / 128;
    const int n_items = n_ent * nbH;
    // The last block commits the cache fills (CombineKernel item 0, exl3_moe.a8.sycl:378-386); for small batches it
    // also writes the tier mask into ids / w and zeroes the rows of tokens without an active pick.  A block arrives
    // once it is past the wait for the gate-up kernel (the fills are copied, every other kernel of the call is done
    // with ids / w and the table) and past its own grouping, i.e. after its first item's stream; the arrival's
    // round trip then overlaps the item's epilogue.
    __shared__ int sh_last_blk;
    const bool need_last = a.fill_list || a.small;
    auto arrive = [&]() {
        if (threadIdx.x == 0) {
            int last = 0;
            if (need_last) {
                __threadfence();
                last = atomicAdd(a.blocks_done, 1) == (int)gridDim.x - 1;
            }
            sh_last_blk = last;
        }
    };
    bool first = true;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int ent = item / nbH, nbh = item % nbH;
        const int nch = (nKBd + 7) / 8;   // the warp's I/128 strip rows, in units of up to 8
        const int u0 = ((ent * nbH + nbh) * 8 + wid) * nch;
        const int ntok = tb ? (int)tb->ntok[ent] : __ldcg(a.ent_n + ent);
        uint2 svd = make_uint2(0u, 0u);
        if (wid < ntok) svd = dn_epi_load(a, ent, nbh, tb);
        float acc[8][4];
        // the warp's accumulator area holds the B operand during the stream (kTokPerEnt x kXsStride fp16 fit)
        run_units<KFIX, 1>(a, u0, 1, nch, ring, nullptr, reinterpret_cast<__half*>(red), acc, lkf, first, tb);
        if (first) arrive();
        first = false;
        const int nwu = 8;   // every warp has I/128 >= 1 rows
        acc_to_smem(acc, red);
        __syncthreads();
        if (wid < ntok) {   // the token's warp sums the warps' accumulators in warp order
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            for (int w = 0; w < nwu; ++w) {
                const float4 s4 = *reinterpret_cast<const float4*>(red_all + (w * kTokPerEnt + wid) * 128 + 4 * lane);
                v[0] += s4.x; v[1] += s4.y; v[2] += s4.z; v[3] += s4.w;
            }
            dn_token_epilogue(a, ent, nbh, wid, v, tb, svd);
        }
        __syncthreads();
    }
    if (first) {   // no item: still order this block after the gate-up kernel
        pdl_wait();
        pdl_trigger();
        arrive();
    }
    __syncthreads();
    if (!sh_last_blk) return;
    __threadfence();
    if (threadIdx.x == 0) {
        if (a.fill_list) {
            const int nf = __ldcg(a.fill_list);
            for (int q = 0; q < nf; ++q) {
                int e = __ldcg(a.fill_list + 1 + q);
                a.ptrs[e] = __ldcg(a.fill + e);
                a.fill[e] = 0;
            }
        }
        a.blocks_done[0] = 0;
    }
    if (a.small) {
        const int np = a.M * a.topk;
        for (int i = threadIdx.x; i < np; i += blockDim.x)
            if (tab->masked[i]) {
                const_cast<int32_t*>(a.ids)[i] = tab->safe;
                const_cast<float*>(a.w)[i] = 0.0f;
            }
        for (int m = 0; m < a.M; ++m) {
            if (tab->tok_cnt[m] != 0) continue;
            for (int c = threadIdx.x; c < a.H; c += blockDim.x) {
                if (a.out_bf16 == 2) reinterpret_cast<float*>(a.out)[(long long)m * a.os + c] = 0.0f;
                else if (a.out_bf16) reinterpret_cast<__nv_bfloat16*>(a.out)[(long long)m * a.os + c] = __float2bfloat16(0.0f);
                else reinterpret_cast<__half*>(a.out)[(long long)m * a.os + c] = __float2half(0.0f);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ host
// Decode workspace: the entry tables (prep's grouping), per-token / per-pick flags and counters, the activation
// rows between the kernels (abuf: fp16 [pick][I]) and the weighted pick outputs (y: fp32 [pick][H]), 256-byte
// aligned pieces.
enum WsPart { kWsEntExpert, kWsEntN, kWsEntTok, kWsEntW, kWsEntPick, kWsNEnt, kWsTokCnt, kWsPickAct, kWsCntC, kWsAbuf,
              kWsY, kWsEntBlob, kWsEntK, kWsBlocksDone, kWsParts };
struct WsLayout {
    size_t off[kWsParts];
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
    const size_t np = (size_t)M * topk, me = np, nbH = H / 128;
    size_t sizes[kWsParts];
    sizes[kWsEntExpert] = me * 4;
    sizes[kWsEntN] = me * 4;
    sizes[kWsEntTok] = me * kTokPerEnt * 4;
    sizes[kWsEntW] = me * kTokPerEnt * 4;
    sizes[kWsEntPick] = me * kTokPerEnt * 4;
    sizes[kWsNEnt] = 16;
    sizes[kWsTokCnt] = (size_t)M * 4;
    sizes[kWsPickAct] = np * 4;
    sizes[kWsCntC] = (size_t)M * nbH * 4;
    sizes[kWsAbuf] = np * I * 2;
    sizes[kWsY] = np * H * 4;
    sizes[kWsEntBlob] = me * 8;
    sizes[kWsEntK] = me * 4;
    sizes[kWsBlocksDone] = 16;
    WsLayout L;
    size_t o = 0;
    for (int i = 0; i < kWsParts; ++i) { L.off[i] = o; o += al256(sizes[i]); }
    L.total = o;
    return L;
}

template <int KFIX>
static int launch_gu(const DecodeArgs& a, int nclusters, int cs, cudaStream_t s) {
    using C = StreamCfg<KFIX, 0>;
    constexpr int smem_max = C::SMEM_BYTES + gu_gather_floats(4, kTokPerEnt) * 4 + (int)sizeof(SmallTab);
    const int smem = C::SMEM_BYTES + gu_gather_floats(cs, a.M) * 4 + (int)sizeof(SmallTab);
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(gu_cluster_kernel<KFIX>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        attr_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nclusters * cs);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cs;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gu_cluster_kernel<KFIX>, a);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    return 0;
}

template <int KFIX>
static int launch_dn(const DecodeArgs& a, int grid, cudaStream_t s) {
    using C = StreamCfg<KFIX, 1>;
    constexpr int smem = C::SMEM_BYTES + 8 * kTokPerEnt * 128 * 4 + (int)sizeof(SmallTab);
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(dn_item_kernel<KFIX>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
        attr_dev = dev;
    }
    cudaError_t e = launch_k(dn_item_kernel<KFIX>, dim3(grid), dim3(256), (size_t)smem, s, a);
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
bool vring_active();
int vring_launch(const int32_t* vict, int64_t slot_base, int64_t blob, int max_victims, cudaStream_t s);

static int run_decode(DecodeArgs& a, const EnsureArgs* ea, void* workspace, int64_t ws_bytes, cudaStream_t s,
                      const int32_t* vict, const int64_t* host_base, int64_t slot_base, int64_t hstride,
                      uint8_t* ram_res, int nvict) {
    const int M = a.M, topk = a.topk, H = a.H, I = a.I;
    WsLayout L = ws_layout(M, topk, H, I);
    EXL3B_CHECK(workspace && ws_bytes >= (int64_t)L.total, "exl3b_moe_decode: workspace too small");
    EXL3B_CHECK((((uintptr_t)workspace) & 255) == 0, "exl3b_moe_decode: workspace must be 256-byte aligned");
    char* b = (char*)workspace;
    a.ent_expert = (int*)(b + L.off[kWsEntExpert]); a.ent_n = (int*)(b + L.off[kWsEntN]);
    a.ent_tok = (int*)(b + L.off[kWsEntTok]); a.ent_w = (float*)(b + L.off[kWsEntW]);
    a.ent_pick = (int*)(b + L.off[kWsEntPick]); a.n_ent = (int*)(b + L.off[kWsNEnt]);
    a.tok_cnt = (int*)(b + L.off[kWsTokCnt]); a.pick_act = (int*)(b + L.off[kWsPickAct]);
    a.cnt_c = (int*)(b + L.off[kWsCntC]); a.abuf = (__half*)(b + L.off[kWsAbuf]); a.y = (float*)(b + L.off[kWsY]);
    a.ent_blob = (long long*)(b + L.off[kWsEntBlob]); a.ent_k = (int*)(b + L.off[kWsEntK]);
    a.blocks_done = (int*)(b + L.off[kWsBlocksDone]);
    a.maxent = M * topk;
    a.small = (M <= kTokPerEnt && M * topk <= kSmallPicks && !(ea && ea->prefetch)) ? 1 : 0;
    EXL3B_CHECK(!a.routed || a.small, "exl3b_moe_decode_cached_routed: in-kernel selection is for small batches only");
    EnsureArgs none{};
    prof_record(0, s);
    cudaError_t e = launch_k(prep_kernel, dim3(1), dim3(1024), 0, s, ea ? *ea : none, a, ea ? 1 : 0);
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    if (vict && nvict > 0) {   // victim write-back must precede the fill copies that overwrite the slots
        int rc = vring_active() ? vring_launch(vict, slot_base, a.blob, nvict, s)
                                : victim_copy_launch(vict, host_base, slot_base, a.blob, a.E, hstride, ram_res, nvict, s);
        if (rc) return rc;
    }
    // gate-up: clusters of 4 CTAs (2 when H/128 is odd), one per (entry, 128-column block) up to a cap; down: one
    // CTA per (entry, 128-column block of H) up to a cap; both loop over further items
    const int nKB = H / 128;
    const int cs = (nKB % 2 == 0) ? 4 : 2;
    const long long gu_items = (long long)a.maxent * (I / 128);
    const long long dn_items = (long long)a.maxent * (H / 128);
    const int ncl = (int)std::min<long long>(std::max<long long>(gu_items, 1), 4096 / cs);
    const int g2 = (int)std::min<long long>(std::max<long long>(dn_items, 1), 4096);
    int kf = a.kinfo ? 0 : a.K;
    int rc = 0;
    prof_record(1, s);
    switch (kf) {
        case 0: rc = launch_gu<0>(a, ncl, cs, s); break;
        case 2: rc = launch_gu<2>(a, ncl, cs, s); break;
        case 3: rc = launch_gu<3>(a, ncl, cs, s); break;
        case 4: rc = launch_gu<4>(a, ncl, cs, s); break;
        case 5: rc = launch_gu<5>(a, ncl, cs, s); break;
    }
    if (rc) return rc;
    prof_record(2, s);
    switch (kf) {
        case 0: rc = launch_dn<0>(a, g2, s); break;
        case 2: rc = launch_dn<2>(a, g2, s); break;
        case 3: rc = launch_dn<3>(a, g2, s); break;
        case 4: rc = launch_dn<4>(a, g2, s); break;
        case 5: rc = launch_dn<5>(a, g2, s); break;
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

namespace exl3b {
int router_logits_launch(const void* x_bf16, int64_t x_stride, const void* wr_bf16, const float* bias, int T, int H,
                         int E, float* logits, cudaStream_t s);
}

// Cached decode; with logits set (routed entry, small batches) the kernels select the picks from them.
static int decode_cached_impl(const void* x, int64_t x_stride, int x_bf16, int32_t* ids, float* w, int M, int topk,
                              int layer, int64_t* ptrs_all, int32_t* slot_of, int32_t* slot_key, int32_t* slot_last,
                              int32_t* tick, const int64_t* host_base, int64_t slot_base, int64_t blob, int64_t hstride,
                              int64_t* fill_all, int32_t* fill_list, int max_fill, int S, const uint8_t* ram_res,
                              int32_t* ring, int ring_cap, const int32_t* safe, int32_t* vict, uint8_t* vict_ram_res,
                              int H, int I, int K, int E, void* out, int64_t out_stride, int out_bf16, void* workspace,
                              int64_t ws_bytes, int flags, void* stream, const float* logits) {
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
    a.logits = logits;
    a.routed = logits ? 1 : 0;
    int mf = max_fill < E ? max_fill : E;
    EnsureArgs ea{ids, w, M * topk, layer, E, S, ptrs_all, slot_of, slot_key, slot_last, tick, host_base, slot_base, blob,
                  hstride > 0 ? hstride : blob, fill_all, fill_list, mf, 0, nullptr, ram_res, ring, ring_cap, safe, vict};
    // small batches: the decode kernels group the picks themselves and the tier mask is written back at the end
    a.t_slot_of = slot_of + (int64_t)layer * E;
    a.t_ram_res = ram_res ? ram_res + (int64_t)layer * E : nullptr;
    a.t_safe = safe ? safe + layer : nullptr;
    ea.defer_mask = (M <= kTokPerEnt && M * topk <= kSmallPicks) ? 1 : 0;
    int nvict = vict ? std::min(mf, M * topk) : 0;
    return run_decode(a, &ea, workspace, ws_bytes, (cudaStream_t)stream, vict, host_base, slot_base,
                      hstride > 0 ? hstride : blob, vict_ram_res, nvict);
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
    return decode_cached_impl(x, x_stride, x_bf16, ids, w, M, topk, layer, ptrs_all, slot_of, slot_key, slot_last, tick,
                              host_base, slot_base, blob, hstride, fill_all, fill_list, max_fill, S, ram_res, ring,
                              ring_cap, safe, vict, vict_ram_res, H, I, K, E, out, out_stride, out_bf16, workspace,
                              ws_bytes, flags, stream, nullptr);
}

extern "C" int exl3b_router_topk(const void* x_bf16, int64_t x_stride, const void* wr_bf16, const float* bias, int T,
                                 int H, int E, int topk, int32_t* ids, float* w, float* logits, int32_t* counter,
                                 void* stream);

extern "C" EXL3B_API int exl3b_moe_decode_cached_routed(const void* x_bf16, int64_t x_stride, const void* wr_bf16,
                                                        const float* bias, float* logits, int32_t* ids, float* w, int M,
                                                        int topk, int layer, int64_t* ptrs_all, int32_t* slot_of,
                                                        int32_t* slot_key, int32_t* slot_last, int32_t* tick,
                                                        const int64_t* host_base, int64_t slot_base, int64_t blob,
                                                        int64_t hstride, int64_t* fill_all, int32_t* fill_list,
                                                        int max_fill, int S, const uint8_t* ram_res, int32_t* ring,
                                                        int ring_cap, const int32_t* safe, int32_t* vict,
                                                        uint8_t* vict_ram_res, int H, int I, int K, int E, void* out,
                                                        int64_t out_stride, int out_bf16, void* workspace,
                                                        int64_t ws_bytes, int flags, int32_t* counter, void* stream) {
    EXL3B_CHECK(x_bf16 && wr_bf16 && logits && ids && w, "exl3b_moe_decode_cached_routed: null pointer");
    EXL3B_CHECK(topk >= 1 && topk <= 32 && topk <= E, "exl3b_moe_decode_cached_routed: 1 <= topk <= min(32, E)");
    if (M == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (M <= kTokPerEnt && M * topk <= kSmallPicks) {
        // small batch: logits only, the decode kernels select (prep writes ids / w)
        EXL3B_CHECK(H % 256 == 0 && H <= 4096 && x_stride >= H && ((x_stride * 2) % 16) == 0 &&
                        (((uintptr_t)x_bf16) & 15) == 0 && (((uintptr_t)wr_bf16) & 15) == 0,
                    "exl3b_moe_decode_cached_routed: router operand shape / alignment");
        int rc = router_logits_launch(x_bf16, x_stride, wr_bf16, bias, M, H, E, logits, s);
        if (rc) return rc;
        return decode_cached_impl(x_bf16, x_stride, 1, ids, w, M, topk, layer, ptrs_all, slot_of, slot_key, slot_last,
                                  tick, host_base, slot_base, blob, hstride, fill_all, fill_list, max_fill, S, ram_res,
                                  ring, ring_cap, safe, vict, vict_ram_res, H, I, K, E, out, out_stride, out_bf16,
                                  workspace, ws_bytes, flags, stream, logits);
    }
    // larger batches: the router op, then the cached decode
    int rc = exl3b_router_topk(x_bf16, x_stride, wr_bf16, bias, M, H, E, topk, ids, w, logits, counter, stream);
    if (rc) return rc;
    return decode_cached_impl(x_bf16, x_stride, 1, ids, w, M, topk, layer, ptrs_all, slot_of, slot_key, slot_last, tick,
                              host_base, slot_base, blob, hstride, fill_all, fill_list, max_fill, S, ram_res, ring,
                              ring_cap, safe, vict, vict_ram_res, H, I, K, E, out, out_stride, out_bf16, workspace,
                              ws_bytes, flags, stream, nullptr);
}

extern "C" EXL3B_API int exl3b_set_profile_events(void* before_route, void* before_gateup, void* before_down,
                                                  void* after_down) {
    g_prof_ev[0] = (cudaEvent_t)before_route;
    g_prof_ev[1] = (cudaEvent_t)before_gateup;
    g_prof_ev[2] = (cudaEvent_t)before_down;
    g_prof_ev[3] = (cudaEvent_t)after_down;
    return 0;
}
