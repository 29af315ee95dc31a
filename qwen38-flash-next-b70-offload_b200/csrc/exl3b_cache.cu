// exl3b_cache.cu -- device-managed LRU expert cache (reference: launch_ensure, exl3_moe.a8.sycl:837-1040;
// VictimCopyKernel :1168-1189; PrefetchCopyKernel :1146-1165; the commit of CombineKernel :378-386).
//
// One block of 1024 threads, graph-safe, no host involvement.  The reference's slot assignment depends on the
// order of work-group atomics; this build fixes every order so the resulting cache state is reproducible:
//   mask:    picks in ascending index log ring[1 + (ring[0]++ % cap)] = key and become (safe[layer], 0);
//   misses:  ascending expert id, the first min(max_fill, E) of them get slots;
//   victims: the nm smallest (u = slot_last + 1, slot index) among slots with slot_last < T (exact LRU);
//   pairing: i-th miss <-> i-th selected slot in ascending slot index.
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"

namespace exl3b {

constexpr int kEnsureThreads = 1024;

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

struct EnsureArgs {
    int32_t* ids; float* w; int npairs; int layer; int E; int S;
    int64_t* ptrs_all; int32_t* slot_of; int32_t* slot_key; int32_t* slot_last; int32_t* tick;
    const int64_t* host_base; int64_t slot_base; int64_t blob; int64_t hstride;
    int64_t* fill_all; int32_t* fill_list; int max_fill; int prefetch; int32_t* pf_slot;
    const uint8_t* ram_res; int32_t* ring; int ring_cap; const int32_t* safe; int32_t* vict;
};

__global__ void __launch_bounds__(kEnsureThreads) ensure_kernel(EnsureArgs a) {
    __shared__ int sh_warp[32];
    __shared__ int sh_T, sh_nm, sh_want, sh_bin, sh_base_ring;
    __shared__ unsigned char need[1024];
    __shared__ int miss[1024];
    __shared__ int vslot[1024];
    __shared__ int hist[256];
    const int tid = threadIdx.x;
    const int E = a.E, S = a.S, L = a.layer;
    int total;

    // 1. tier mask, picks in ascending index
    if (a.ram_res && !a.prefetch) {
        if (tid == 0) sh_base_ring = a.ring[0];
        __syncthreads();
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
                a.ring[1 + (c % a.ring_cap)] = key;
                a.ids[i] = a.safe[L];
                a.w[i] = 0.0f;
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
        int e = a.ids[i];
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
    // 5. eligible slots (contiguous chunk per thread, ascending slot index overall)
    const int C = (S + kEnsureThreads - 1) / kEnsureThreads;
    const int s0 = tid * C, s1 = min(S, s0 + C);
    int elig = 0, empty = 0;
    for (int s = s0; s < s1; ++s) {
        int la = a.slot_last[s];
        if (la < T) { ++elig; empty += (la == -1); }
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
            uint32_t hmask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
            for (int s = s0; s < s1; ++s) {
                int la = a.slot_last[s];
                if (la >= T) continue;
                uint32_t u = (uint32_t)(la + 1);
                if ((u & hmask) != (prefix & hmask)) continue;
                atomicAdd(&hist[(u >> shift) & 255], 1);
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
        int la = a.slot_last[s];
        if (la < T && (uint32_t)(la + 1) == prefix) ++n_eq;
    }
    int eq_before = block_scan(n_eq, &total, sh_warp);
    int nsel = 0;
    {
        int eq = eq_before;
        for (int s = s0; s < s1; ++s) {
            int la = a.slot_last[s];
            if (la >= T) continue;
            uint32_t u = (uint32_t)(la + 1);
            if (u < prefix) ++nsel;
            else if (u == prefix) { if (eq < want) ++nsel; ++eq; }
        }
    }
    int sel_before = block_scan(nsel, &total, sh_warp);
    {
        int eq = eq_before, r = sel_before;
        for (int s = s0; s < s1; ++s) {
            int la = a.slot_last[s];
            if (la >= T) continue;
            uint32_t u = (uint32_t)(la + 1);
            bool take = false;
            if (u < prefix) take = true;
            else if (u == prefix) { take = eq < want; ++eq; }
            if (take) { if (r < 1024) vslot[r] = s; ++r; }
        }
    }
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

// Copy planned fills host blob -> device slot, 16 B per thread per step; block = (fill i, 64 KiB chunk).
// src = ptrs[e] (the host address: ensure never repoints the new owner), dst = fill[e] (or the prefetch slot).
__global__ void __launch_bounds__(256) fill_copy_kernel(const int32_t* __restrict__ fill_list,
                                                        const int64_t* __restrict__ ptrs, const int64_t* __restrict__ fill,
                                                        const int32_t* __restrict__ pf_slot, int64_t slot_base,
                                                        int64_t blob, int chunks) {
    int i = blockIdx.x / chunks, c = blockIdx.x % chunks;
    if (i >= fill_list[0]) return;
    int e = fill_list[1 + i];
    const uint4* src = reinterpret_cast<const uint4*>(ptrs[e]);
    uint4* dst = reinterpret_cast<uint4*>(pf_slot ? slot_base + (int64_t)pf_slot[i] * blob : fill[e]);
    int64_t n16 = blob / 16;
    int64_t b0 = (int64_t)c * 4096, b1 = min(n16, b0 + 4096);
    for (int64_t q = b0 + threadIdx.x; q < b1; q += blockDim.x) dst[q] = src[q];
}

// Victim write-back (exl3_moe.a8.sycl:1168-1189): slot -> its RAM-tier address; the victim is flagged resident.
__global__ void __launch_bounds__(256) victim_copy_kernel(const int32_t* __restrict__ vict,
                                                          const int64_t* __restrict__ host_base, int64_t slot_base,
                                                          int64_t blob, int E, int chunks, int64_t hstride,
                                                          uint8_t* ram_res) {
    int i = blockIdx.x / chunks, c = blockIdx.x % chunks;
    if (i >= vict[0]) return;
    int old = vict[1 + 2 * i], s = vict[2 + 2 * i];
    if (old < 0) return;
    if (ram_res && c == 0 && threadIdx.x == 0) ram_res[old] = 1;
    const uint4* src = reinterpret_cast<const uint4*>(slot_base + (int64_t)s * blob);
    uint4* dst = reinterpret_cast<uint4*>(host_base[old / E] + (int64_t)(old % E) * hstride);
    int64_t n16 = blob / 16;
    int64_t b0 = (int64_t)c * 4096, b1 = min(n16, b0 + 4096);
    for (int64_t q = b0 + threadIdx.x; q < b1; q += blockDim.x) dst[q] = src[q];
}

// Commit of the planned fills: ptrs[e] = fill[e], fill[e] = 0 (prefetch mode: ptrs[e] = slot address).
__global__ void commit_kernel(const int32_t* __restrict__ fill_list, int64_t* ptrs, int64_t* fill,
                              const int32_t* __restrict__ pf_slot, int64_t slot_base, int64_t blob) {
    int n = fill_list[0];
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        int e = fill_list[1 + i];
        if (pf_slot) ptrs[e] = slot_base + (int64_t)pf_slot[i] * blob;
        else { ptrs[e] = fill[e]; fill[e] = 0; }
    }
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int exl3b_ensure(int32_t* ids, float* w, int npairs, int layer, int E, int S, int64_t* ptrs_all,
                                      int32_t* slot_of, int32_t* slot_key, int32_t* slot_last, int32_t* tick,
                                      const int64_t* host_base, int64_t slot_base, int64_t blob, int64_t hstride,
                                      int64_t* fill_all, int32_t* fill_list, int max_fill, int prefetch,
                                      int32_t* pf_slot, const uint8_t* ram_res, int32_t* ring, int ring_cap,
                                      const int32_t* safe, int32_t* vict, void* stream) {
    EXL3B_CHECK(E >= 1 && E <= 1024, "exl3b_ensure: 1 <= n_experts <= 1024");
    EXL3B_CHECK(npairs >= 0 && layer >= 0 && S >= 0, "exl3b_ensure: bad sizes");
    EXL3B_CHECK(ids && ptrs_all && slot_of && tick && host_base && fill_list, "exl3b_ensure: null pointer");
    EXL3B_CHECK(S == 0 || (slot_key && slot_last), "exl3b_ensure: slot tables missing");
    EXL3B_CHECK(prefetch ? pf_slot != nullptr : fill_all != nullptr, "exl3b_ensure: fill_all / pf_slot missing");
    EXL3B_CHECK(!ram_res || prefetch || (w && ring && ring_cap > 0 && safe), "exl3b_ensure: tier mask needs w, ring, safe");
    EXL3B_CHECK(max_fill >= 0, "exl3b_ensure: max_fill >= 0");
    EnsureArgs a{ids, w, npairs, layer, E, S, ptrs_all, slot_of, slot_key, slot_last, tick, host_base, slot_base, blob,
                 hstride > 0 ? hstride : blob, fill_all, fill_list, max_fill, prefetch, pf_slot, ram_res, ring, ring_cap,
                 safe, vict};
    ensure_kernel<<<1, kEnsureThreads, 0, (cudaStream_t)stream>>>(a);
    return exl3b_launch_status("exl3b_ensure");
}

extern "C" EXL3B_API int exl3b_fill_copy(const int32_t* fill_list, const int64_t* ptrs, const int64_t* fill,
                                         const int32_t* pf_slot, int64_t slot_base, int64_t blob, int max_fills,
                                         void* stream) {
    EXL3B_CHECK(fill_list && ptrs && (fill || pf_slot), "exl3b_fill_copy: null pointer");
    EXL3B_CHECK(blob % 16 == 0, "exl3b_fill_copy: blob size must be a multiple of 16");
    if (max_fills <= 0) return 0;
    int chunks = (int)((blob / 16 + 4095) / 4096);
    fill_copy_kernel<<<max_fills * chunks, 256, 0, (cudaStream_t)stream>>>(fill_list, ptrs, fill, pf_slot, slot_base,
                                                                             blob, chunks);
    return exl3b_launch_status("exl3b_fill_copy");
}

extern "C" EXL3B_API int exl3b_victim_copy(const int32_t* vict, const int64_t* host_base, int64_t slot_base, int64_t blob,
                                           int E, int64_t hstride, uint8_t* ram_res, int max_victims, void* stream) {
    EXL3B_CHECK(vict && host_base, "exl3b_victim_copy: null pointer");
    EXL3B_CHECK(blob % 16 == 0 && (hstride <= 0 || hstride % 16 == 0), "exl3b_victim_copy: 16-byte multiples");
    if (max_victims <= 0) return 0;
    int chunks = (int)((blob / 16 + 4095) / 4096);
    victim_copy_kernel<<<max_victims * chunks, 256, 0, (cudaStream_t)stream>>>(vict, host_base, slot_base, blob, E, chunks,
                                                                                 hstride > 0 ? hstride : blob, ram_res);
    return exl3b_launch_status("exl3b_victim_copy");
}

extern "C" EXL3B_API int exl3b_commit(const int32_t* fill_list, int64_t* ptrs, int64_t* fill, const int32_t* pf_slot,
                                      int64_t slot_base, int64_t blob, void* stream) {
    EXL3B_CHECK(fill_list && ptrs && (fill || pf_slot), "exl3b_commit: null pointer");
    commit_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(fill_list, ptrs, fill, pf_slot, slot_base, blob);
    return exl3b_launch_status("exl3b_commit");
}
