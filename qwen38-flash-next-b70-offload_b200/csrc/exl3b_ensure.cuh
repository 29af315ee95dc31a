// exl3b_ensure.cuh -- the device expert cache step as a block-level device function (1024 threads), shared by the
// standalone ensure kernel and the fused decode prologue.  Reference: launch_ensure (exl3_moe.a8.sycl:837-1040).
//
// Deterministic rule in place of the reference's atomic orders:
//   mask:    picks in ascending index log ring[1 + (ring[0]++ % cap)] = key and become (safe[layer], 0);
//   misses:  ascending expert id, the first min(max_fill, E) of them get slots;
//   victims: the nm smallest (u = slot_last + 1, slot index) among slots with slot_last < T (exact LRU);
//   pairing: i-th miss <-> i-th selected slot in ascending slot index.
#pragma once
#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kEnsureThreads = 1024;
constexpr int kDeferMaskMax = 64;   // most picks of a call whose tier-mask rewrite may be deferred

// Block-wide exclusive scan of one int per thread (1024 threads); returns the prefix, *total gets the sum.
__device__ __forceinline__ int block_scan(int v, int* total, int* sh_warp /* [32] */) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh_warp[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int s = sh_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        sh_warp[lane] = s;   // inclusive per-warp totals
    }
    __syncthreads();
    int base = wid ? sh_warp[wid - 1] : 0;
    *total = sh_warp[31];
    __syncthreads();
    return base + x - v;
}

// LRU order key of slot s at tick T: 0 for an empty slot (slot_last -1), else its last use + 1.  A slot used at this
// tick (slot_last >= T: a hit of this call, or pinned at 0x7FFFFFFF) is not eligible and has no key.
__device__ __forceinline__ bool lru_key(int last, int T, uint32_t& key) {
    if (last >= T) return false;
    key = (uint32_t)(last + 1);
    return true;
}

struct EnsureArgs {
    int32_t* ids; float* w; int npairs; int layer; int E; int S;
    int64_t* ptrs_all; int32_t* slot_of; int32_t* slot_key; int32_t* slot_last; int32_t* tick;
    const int64_t* host_base; int64_t slot_base; int64_t blob; int64_t hstride;
    int64_t* fill_all; int32_t* fill_list; int max_fill; int prefetch; int32_t* pf_slot;
    const uint8_t* ram_res; int32_t* ring; int ring_cap; const int32_t* safe; int32_t* vict;
    int defer_mask = 0;   // 1 (npairs <= kDeferMaskMax): the masked picks' in-place (safe, 0) rewrite of ids / w is left to the caller's last
                          // kernel (npairs <= 32); the step itself uses the masked ids
};

__device__ __forceinline__ void ensure_block(const EnsureArgs& a) {
    __shared__ int sh_warp[32];
    __shared__ int sh_T, sh_nm, sh_want, sh_bin, sh_base_ring;
    __shared__ unsigned char need[1024];
    __shared__ int miss[1024];
    __shared__ int vslot[1024];
    __shared__ int hist[256];
    __shared__ unsigned char s_msk[kDeferMaskMax];   // defer_mask: picks masked by step 1
    const int tid = threadIdx.x;
    const int E = a.E, S = a.S, L = a.layer;
    int total;

    // 1. tier mask, picks in ascending index
    if (a.defer_mask)
        for (int i = tid; i < kDeferMaskMax; i += kEnsureThreads) s_msk[i] = 0;
    if (a.ram_res && !a.prefetch) {
        // the call's masked-pick count first: only the last ring_cap of them land in the ring (sequentially, earlier
        // ones would be overwritten within the call), so every slot is written once and parallel writes give the
        // sequential result
        int nmask = 0;
        for (int c0 = 0; c0 < a.npairs; c0 += kEnsureThreads) {
            int i = c0 + tid, flag = 0;
            if (i < a.npairs) {
                const int key = L * E + a.ids[i];
                flag = (a.slot_of[key] < 0 && !a.ram_res[key]) ? 1 : 0;
            }
            block_scan(flag, &total, sh_warp);
            nmask += total;
        }
        if (tid == 0) sh_base_ring = a.ring[0];
        __syncthreads();
        const int ring0 = sh_base_ring;
        for (int c0 = 0; c0 < a.npairs; c0 += kEnsureThreads) {
            int i = c0 + tid;
            int flag = 0, key = 0;
            if (i < a.npairs) {
                key = L * E + a.ids[i];
                flag = (a.slot_of[key] < 0 && !a.ram_res[key]) ? 1 : 0;
            }
            int pre = block_scan(flag, &total, sh_warp);
            if (flag) {
                int c = sh_base_ring + pre;
                if (c - ring0 >= nmask - a.ring_cap) a.ring[1 + (c % a.ring_cap)] = key;
                if (a.defer_mask) {
                    s_msk[i] = 1;
                } else {
                    a.ids[i] = a.safe[L];
                    a.w[i] = 0.0f;
                }
            }
            __syncthreads();
            if (tid == 0) sh_base_ring += total;
            __syncthreads();
        }
        if (tid == 0) a.ring[0] = sh_base_ring;
    }
    // 2. tick
    if (tid == 0) sh_T = a.prefetch ? a.tick[0] : (a.tick[0] = a.tick[0] + 1);
    for (int e = tid; e < E; e += kEnsureThreads) need[e] = 0;
    __syncthreads();
    for (int i = tid; i < a.npairs; i += kEnsureThreads) {
        int e = (a.defer_mask && s_msk[i]) ? a.safe[L] : a.ids[i];
        if (e >= 0 && e < E) need[e] = 1;
        else set_error(kErrBounds);
    }
    __syncthreads();
    const int T = sh_T;
    // 3./4. hits are stamped, misses listed in ascending expert id (E <= 1024: one expert per thread)
    int is_miss = 0;
    if (tid < E && need[tid]) {
        int s = a.slot_of[L * E + tid];
        if (s >= 0) {
            if (a.slot_last[s] != 0x7FFFFFFF) a.slot_last[s] = T;
        } else {
            is_miss = 1;
        }
    }
    int mrank = block_scan(is_miss, &total, sh_warp);
    if (is_miss) miss[mrank] = tid;
    int mf = a.max_fill < E ? a.max_fill : E;
    int nm = S > 0 ? (total < mf ? total : mf) : 0;
    __syncthreads();   // slot_last stamps visible to the whole block
    if (nm == 0) {     // every pick a hit (or masked): no slot scan
        if (tid == 0) { a.fill_list[0] = 0; if (a.vict) a.vict[0] = 0; }
        return;
    }
    // 5. eligible slots (contiguous chunk per thread, ascending slot index overall)
    const int C = (S + kEnsureThreads - 1) / kEnsureThreads;
    const int s0 = tid * C, s1 = min(S, s0 + C);
    int elig = 0, empty = 0;
    for (int s = s0; s < s1; ++s) {
        uint32_t k;
        if (lru_key(a.slot_last[s], T, k)) { ++elig; empty += (k == 0); }
    }
    block_scan(elig, &total, sh_warp);
    int n_elig = total;
    block_scan(empty, &total, sh_warp);
    int n_empty = total;
    if (nm > n_elig) nm = n_elig;
    if (nm == 0) {
        if (tid == 0) { a.fill_list[0] = 0; if (a.vict) a.vict[0] = 0; }
        return;
    }
    // 6. tau = nm-th smallest u (radix select, 4 x 8 bits); want = how many slots with u == tau to take
    uint32_t prefix = 0;
    int want = nm;
    if (n_empty >= nm) {
        prefix = 0;   // enough empty slots (u = 0)
    } else {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = tid; b < 256; b += kEnsureThreads) hist[b] = 0;
            __syncthreads();
            // histogram of byte `shift` over the eligible keys whose higher bytes equal the prefix found so far
            const uint64_t high = (uint64_t)prefix >> (shift + 8);
            for (int s = s0; s < s1; ++s) {
                uint32_t k;
                if (lru_key(a.slot_last[s], T, k) && ((uint64_t)k >> (shift + 8)) == high)
                    atomicAdd(&hist[(k >> shift) & 255], 1);
            }
            __syncthreads();
            if (tid < 32) {
                // serial-in-lane scan over 8 bins each, then a warp scan of the lane sums
                int loc[8], sum = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) { loc[j] = hist[tid * 8 + j]; sum += loc[j]; }
                int x = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    int y = __shfl_up_sync(0xffffffffu, x, o);
                    if (tid >= o) x += y;
                }
                int cum = x - sum;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (cum < want && want <= cum + loc[j]) { sh_bin = tid * 8 + j; sh_want = want - cum; }
                    cum += loc[j];
                }
            }
            __syncthreads();
            prefix |= (uint32_t)sh_bin << shift;
            want = sh_want;
            __syncthreads();
        }
    }
    // 7. selection: every eligible u < tau plus the first `want` (ascending slot index) with u == tau
    int n_eq = 0;
    for (int s = s0; s < s1; ++s) {
        uint32_t k;
        n_eq += lru_key(a.slot_last[s], T, k) && k == prefix;
    }
    const int eq_before = block_scan(n_eq, &total, sh_warp);
    // this thread's chunk in slot order: calls take(s) for every selected slot (the keys equal to tau are numbered
    // across the block from eq_before, and the first `want` of them are selected)
    auto for_each_selected = [&](auto&& take) {
        int eq = eq_before;
        for (int s = s0; s < s1; ++s) {
            uint32_t k;
            if (!lru_key(a.slot_last[s], T, k) || k > prefix) continue;
            if (k == prefix && eq++ >= want) continue;
            take(s);
        }
    };
    int nsel = 0;
    for_each_selected([&](int) { ++nsel; });
    int r = block_scan(nsel, &total, sh_warp);
    for_each_selected([&](int s) { if (r < 1024) vslot[r] = s; ++r; });
    if (tid == 0) sh_nm = total < nm ? total : nm;
    __syncthreads();
    nm = sh_nm;
    // 8. assignment (distinct slots, distinct experts)
    for (int mi = tid; mi < nm; mi += kEnsureThreads) {
        int s = vslot[mi], e = miss[mi];
        int old = a.slot_key[s];
        if (a.vict) {
            a.vict[1 + 2 * mi] = (old >= 0 && a.ram_res && a.ram_res[old]) ? -1 : old;
            a.vict[2 + 2 * mi] = s;
        }
        if (old >= 0) {
            a.slot_of[old] = -1;
            a.ptrs_all[old] = a.host_base[old / E] + (int64_t)(old % E) * a.hstride;
        }
        int key = L * E + e;
        a.slot_key[s] = key;
        a.slot_of[key] = s;
        a.slot_last[s] = T;
        if (a.prefetch) a.pf_slot[mi] = s;
        else a.fill_all[key] = a.slot_base + (int64_t)s * a.blob;
        a.fill_list[1 + mi] = e;
    }
    if (tid == 0) { a.fill_list[0] = nm; if (a.vict) a.vict[0] = nm; }
}


}  // namespace exl3b
