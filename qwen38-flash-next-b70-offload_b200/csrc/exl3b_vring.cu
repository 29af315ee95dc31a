// exl3b_vring.cu -- victim ring: the RAM-tier write-back of evicted VRAM experts through a ring of VRAM slots
// (reference: the a9 variant of launch_ensure / VictimCopyKernel, experimental/n111-victim-ring/a9.patch).
//
// Without a ring, a victim whose RAM copy the tier dropped is copied from its VRAM slot to its host row by the SMs,
// over PCIe / C2C, inside the decode step, and the kernel sets ram_res.  With a ring (exl3b_set_victim_ring), the
// same victim is copied device to device into a free ring slot instead and ram_res is not set: the host loop drains
// the ring to RAM on a copy stream, flags the key only once that copy completed, and then frees the ring slot.  The
// device never writes a host row, so the host alone decides when a row is valid.
//
// meta (int32 [4 + 2K], device): [0] next search position, [1] claim sequence (monotonic), [2] victims dropped because
// the ring was full, [3] K, then key[K] (-1 = free, else the key waiting to be drained) and seq[K] (claim number).
// sel (int32, >= max victims per call, device): ring slot of each victim entry of the current call, -1 = no copy.
// buf: K ring slots of blob bytes (device).
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"

namespace exl3b {

struct VringCfg {
    int32_t* meta = nullptr;
    int32_t* sel = nullptr;
    int64_t base = 0;
    int64_t bytes = 0;
    int K = 0;
};

static VringCfg g_vring;   // process-wide, read at launch (set between calls, like the other cache settings)

bool vring_active() { return g_vring.meta != nullptr; }

// Claims in victim-list order, each scanning from the next search position for a free slot (serial: the victims of a
// call and K are small).  A slot becomes free only when the host writes key = -1 after draining it.  Compiled for
// the device (one thread of vring_claim_kernel) and for the host (exl3b_vring_claim_host, which tests call).
__host__ __device__ inline void vring_claim(const int32_t* vict, int32_t* meta, int32_t* sel, int K) {
    int32_t* key = meta + 4;
    int32_t* seq = meta + 4 + K;
    int p = meta[0];
    if (p < 0 || p >= K) {
#ifdef __CUDA_ARCH__
        set_error(kErrBounds);
#endif
        p = 0;
    }
    const int n = vict[0];
    for (int i = 0; i < n; ++i) {
        const int old = vict[1 + 2 * i];
        int r = -1;
        if (old >= 0) {
            for (int j = 0; j < K && r < 0; ++j) {
                const int q = (p + j) % K;
                if (key[q] < 0) r = q;
            }
            if (r >= 0) {
                key[r] = old;
                seq[r] = ++meta[1];
                p = (r + 1) % K;
            } else {
                meta[2] += 1;
            }
        }
        sel[i] = r;
    }
    meta[0] = p;
}

__global__ void vring_claim_kernel(const int32_t* __restrict__ vict, int32_t* meta, int32_t* sel, int K) {
    if (threadIdx.x == 0) vring_claim(vict, meta, sel, K);
}

// Victim slot -> its ring slot, 16 B per thread per step; block = (victim entry, 64 KiB chunk).
__global__ void __launch_bounds__(256) vring_copy_kernel(const int32_t* __restrict__ vict,
                                                         const int32_t* __restrict__ sel, int64_t slot_base,
                                                         int64_t ring_base, int64_t blob, int chunks, int K) {
    const int i = blockIdx.x / chunks, c = blockIdx.x % chunks;
    if (i >= vict[0]) return;
    const int r = sel[i];
    if (r < 0) return;
    if (r >= K) { if (threadIdx.x == 0 && c == 0) set_error(kErrBounds); return; }
    const uint4* src = reinterpret_cast<const uint4*>(slot_base + (int64_t)vict[2 + 2 * i] * blob);
    uint4* dst = reinterpret_cast<uint4*>(ring_base + (int64_t)r * blob);
    const int64_t n16 = blob / 16;
    const int64_t b0 = (int64_t)c * 4096, b1 = min(n16, b0 + 4096);
    for (int64_t q = b0 + threadIdx.x; q < b1; q += blockDim.x) dst[q] = src[q];
}

int vring_launch(const int32_t* vict, int64_t slot_base, int64_t blob, int max_victims, cudaStream_t s) {
    const VringCfg c = g_vring;
    if ((int64_t)c.K * blob > c.bytes)
        return exl3b_fail(EXL3B_EINVAL, "victim ring: the ring buffer holds fewer than K blobs of this layer's size");
    vring_claim_kernel<<<1, 32, 0, s>>>(vict, c.meta, c.sel, c.K);
    const int chunks = (int)((blob / 16 + 4095) / 4096);
    vring_copy_kernel<<<max_victims * chunks, 256, 0, s>>>(vict, c.sel, slot_base, c.base, blob, chunks, c.K);
    return exl3b_launch_status("victim ring");
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int exl3b_set_victim_ring(int32_t* meta, int32_t* sel, void* buf, int64_t buf_bytes, int K) {
    if (!meta) {
        g_vring = VringCfg{};
        return 0;
    }
    EXL3B_CHECK(sel && buf && K > 0 && buf_bytes > 0, "exl3b_set_victim_ring: meta, sel, buf, buf_bytes and K > 0");
    EXL3B_CHECK((((uintptr_t)buf) & 15) == 0, "exl3b_set_victim_ring: buf must be 16-byte aligned");
    g_vring = VringCfg{meta, sel, (int64_t)(uintptr_t)buf, buf_bytes, K};
    return 0;
}

// Test hook, not part of the drop-in surface: the device's claim rule run on host memory.
extern "C" EXL3B_API void exl3b_vring_claim_host(const int32_t* vict, int32_t* meta, int32_t* sel, int K) {
    vring_claim(vict, meta, sel, K);
}
