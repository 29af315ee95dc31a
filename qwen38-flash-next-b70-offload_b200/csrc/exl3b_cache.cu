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
#include "exl3b_ensure.cuh"

namespace exl3b {

__global__ void __launch_bounds__(kEnsureThreads) ensure_kernel(EnsureArgs a) { ensure_block(a); }

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

int victim_copy_launch(const int32_t* vict, const int64_t* host_base, int64_t slot_base, int64_t blob, int E,
                       int64_t hstride, uint8_t* ram_res, int max_victims, cudaStream_t s) {
    int chunks = (int)((blob / 16 + 4095) / 4096);
    victim_copy_kernel<<<max_victims * chunks, 256, 0, s>>>(vict, host_base, slot_base, blob, E, chunks,
                                                            hstride > 0 ? hstride : blob, ram_res);
    return exl3b_launch_status("victim copy");
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
