// exl3b_dequant.cu -- standalone trellis dequantisation (W_inner fp16), bit-exact with the reference codec.
//
// Contract of the reference's reconstruct (exl3_esimd.h:869-936, exl3_ops.sycl:539-555): a tile matrix
// [k/16][n/16][8K words] -> fp16 W_inner [k][n] (Hadamard domain, no scales).  This build reads either the
// checkpoint (plain tile-major) word order or the blob's PLANAR4 order (moe_offload.py:68-73).
#include "exl3b_common.cuh"
#include "exl3b_capi_util.h"

namespace exl3b {

__device__ int g_status = 0;

// One warp per tile; lane l decodes values t = 8l..8l+7 and stores them at their (row, col).
template <int K>
__global__ void __launch_bounds__(256) dequant_kernel(const uint32_t* __restrict__ words, int rows16, long long row_stride,
                                                      int tile0, int ntiles, int planar, __half* __restrict__ w,
                                                      long long ldw) {
    int lane = threadIdx.x & 31;
    long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (gw >= (long long)rows16 * ntiles) return;
    int r = (int)(gw / ntiles), c = (int)(gw % ntiles);
    LaneWin<K> lw;
    lw.init(lane, planar != 0);
    const uint32_t* row = words + (long long)r * row_stride;
    int tc = tile0 + c;
    const uint32_t* tb;
    int add;
    if (planar) { tb = row + (long long)(tc >> 2) * 4 * Geo<K>::W; add = (tc & 3) * Geo<K>::G; }
    else { tb = row + (long long)tc * Geo<K>::W; add = 0; }
    uint32_t a = tb[lw.oA + add], b = tb[lw.oB + add];
    uint32_t cc = LaneWin<K>::kNeedC ? tb[lw.oC + add] : 0u;
    uint32_t f[4];
    decode8<K>(a, b, cc, lw.p0, f);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int rr, cl;
            frag_pos(lane, q, h, rr, cl);
            unsigned short bits = (unsigned short)(h ? (f[q] >> 16) : (f[q] & 0xFFFFu));
            w[((long long)r * 16 + rr) * ldw + (long long)c * 16 + cl] = __ushort_as_half(bits);
        }
    }
}

}  // namespace exl3b

using namespace exl3b;

extern "C" EXL3B_API int exl3b_dequant(const void* words, int rows16, int64_t row_stride_words, int tile0, int ntiles,
                                       int K, int planar, void* w_fp16, int64_t ldw, void* stream) {
    EXL3B_CHECK(words && w_fp16, "exl3b_dequant: null pointer");
    EXL3B_CHECK(rows16 >= 0 && ntiles >= 0 && tile0 >= 0 && ldw >= (int64_t)ntiles * 16, "exl3b_dequant: bad shape");
    EXL3B_CHECK(!planar || (tile0 % 4) == 0, "exl3b_dequant: PLANAR4 rows need tile0 % 4 == 0");
    EXL3B_CHECK(((uintptr_t)words & 3) == 0, "exl3b_dequant: words must be 4-byte aligned");
    long long n = (long long)rows16 * ntiles;
    if (n == 0) return 0;
    int threads = 256;
    long long blocks = (n + 7) / 8;
    cudaStream_t s = (cudaStream_t)stream;
    const uint32_t* wp = (const uint32_t*)words;
    __half* o = (__half*)w_fp16;
    switch (K) {
        case 2: dequant_kernel<2><<<(unsigned)blocks, threads, 0, s>>>(wp, rows16, row_stride_words, tile0, ntiles, planar, o, ldw); break;
        case 3: dequant_kernel<3><<<(unsigned)blocks, threads, 0, s>>>(wp, rows16, row_stride_words, tile0, ntiles, planar, o, ldw); break;
        case 4: dequant_kernel<4><<<(unsigned)blocks, threads, 0, s>>>(wp, rows16, row_stride_words, tile0, ntiles, planar, o, ldw); break;
        case 5: dequant_kernel<5><<<(unsigned)blocks, threads, 0, s>>>(wp, rows16, row_stride_words, tile0, ntiles, planar, o, ldw); break;
        default: return exl3b_fail(EXL3B_EINVAL, "exl3b_dequant: K must be 2..5");
    }
    return exl3b_launch_status("exl3b_dequant");
}

extern "C" EXL3B_API int exl3b_blob_dequant(const void* blob, int H, int I, int Kg, int Ku, int Kd, int proj, void* w_fp16,
                                            void* stream) {
    EXL3B_CHECK(proj >= 0 && proj <= 2, "exl3b_blob_dequant: proj must be 0 (gate), 1 (up) or 2 (down)");
    EXL3B_CHECK(H % 128 == 0 && I % 128 == 0, "exl3b_blob_dequant: H and I must be multiples of 128");
    Geom g{H, I, Kg, Ku, Kd};
    const uint32_t* tr = (const uint32_t*)blob;
    if (proj < 2) {
        const uint32_t* base = tr + (proj == 1 ? (size_t)(I / 16) * 8 * Kg : 0);
        return exl3b_dequant(base, H / 16, (int64_t)g.gu_row_words(), 0, I / 16, proj == 1 ? Ku : Kg, 1, w_fp16, I, stream);
    }
    return exl3b_dequant(tr + g.gu_words(), I / 16, (int64_t)g.d_row_words(), 0, H / 16, Kd, 1, w_fp16, H, stream);
}

extern "C" EXL3B_API int64_t exl3b_blob_bytes(int H, int I, int Kg, int Ku, int Kd) {
    return (int64_t)Geom{H, I, Kg, Ku, Kd}.blob();
}

extern "C" EXL3B_API int exl3b_device_status(int* host_status, int clear, void* stream) {
    EXL3B_CHECK(host_status, "exl3b_device_status: null pointer");
    cudaStream_t s = (cudaStream_t)stream;
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && clear) {
        int z = 0;
        e = cudaMemcpyToSymbolAsync(g_status, &z, sizeof(int), 0, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    if (e != cudaSuccess) return exl3b_fail(EXL3B_ECUDA, cudaGetErrorString(e));
    *host_status = v;
    return 0;
}
