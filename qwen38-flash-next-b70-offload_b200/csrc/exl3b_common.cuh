// exl3b_common.cuh -- shared device code for the B200 EXL3 MoE kernels (sm_100a).
//
// EXL3 trellis tile (exl3_esimd.h:4-9 in the reference): a 16x16 block of weights stored as 8K uint32 words, one
// circular MSB-first bit stream of 256*K bits.  Value t (0..255) is the 16-bit window that ends at bit (t+1)*K and
// sits at row (input dim) 8*((t>>1)&1) + 2*((t>>3)&3) + (t&1), column (output dim) (t>>5) + 8*((t>>2)&1).
// The mul1 codebook maps a state st to fp16( (1024 + bytesum(st * 0x83DCD12D)) * c1 + c2 ) with one rounding
// (exl3_esimd.h:45-67).
//
// B200 mapping: lane l of a warp decodes the 8 consecutive values t = 8l .. 8l+7 of a tile.  With that split the
// tile position map above is exactly the mma.sync m16n8k16 operand layout for the TRANSPOSED tile W^T (16 output
// columns x 16 inputs): value i of lane l is (n = l/4 + 8*bit2(i), k = 2*(l%4) + bit0(i) + 8*bit1(i)), i.e. A
// fragment registers R0 = {v0,v1}, R1 = {v4,v5}, R2 = {v2,v3}, R3 = {v6,v7}.  The decoded tile never leaves
// registers: one m16n8k16 per tile computes 16 output columns for up to 8 tokens.
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace exl3b {

// ------------------------------------------------------------------------------------------------ status word
// Device-side error bits (bounds / bounded waits).  Kernels OR bits in; the host reads and clears the word with
// exl3b_device_status().  Never __trap(): a kernel that detects an error records it and returns.
enum : int {
    kErrBounds = 1,     // an index outside the buffer it addresses was skipped
    kErrWait = 2,       // a bounded wait gave up
    kErrGeometry = 4,   // a shape the kernel cannot handle reached it
};
extern __device__ int g_status;
__device__ __forceinline__ void set_error(int bit) { atomicOr(&g_status, bit); }

// ------------------------------------------------------------------------------------------------ geometry
// Blob layout (exl3_moe.a8.sycl:42-54), generalised to one K per tensor: gate|up rows of I/16 gate tiles (8*Kg
// words) then I/16 up tiles (8*Ku words), PLANAR4 per row; down rows of H/16 tiles (8*Kd words); then fp16 vectors
// suh_g[H] suh_u[H] svh_g[I] svh_u[I] suh_d[I] svh_d[H].
struct Geom {
    int H, I, Kg, Ku, Kd;
    __host__ __device__ size_t gu_row_words() const { return (size_t)(I / 16) * 8 * (Kg + Ku); }
    __host__ __device__ size_t gu_words() const { return (size_t)(H / 16) * gu_row_words(); }
    __host__ __device__ size_t d_row_words() const { return (size_t)(H / 16) * 8 * Kd; }
    __host__ __device__ size_t d_words() const { return (size_t)(I / 16) * d_row_words(); }
    __host__ __device__ size_t off_vec() const { return (gu_words() + d_words()) * 4; }
    __host__ __device__ size_t off_suh_g() const { return off_vec(); }
    __host__ __device__ size_t off_suh_u() const { return off_vec() + (size_t)H * 2; }
    __host__ __device__ size_t off_svh_g() const { return off_vec() + (size_t)H * 4; }
    __host__ __device__ size_t off_svh_u() const { return off_vec() + (size_t)H * 4 + (size_t)I * 2; }
    __host__ __device__ size_t off_suh_d() const { return off_vec() + (size_t)H * 4 + (size_t)I * 4; }
    __host__ __device__ size_t off_svh_d() const { return off_vec() + (size_t)H * 4 + (size_t)I * 6; }
    __host__ __device__ size_t blob() const { return off_vec() + (size_t)(3 * H + 3 * I) * 2; }
};

// Per-expert K triple packed as Kg | Ku << 4 | Kd << 8 (mixed-bitrate stores); uniform stores pass K.
__host__ __device__ __forceinline__ int kinfo_pack(int kg, int ku, int kd) { return kg | (ku << 4) | (kd << 8); }

constexpr float kRsqrt128 = 0.08838834764831845f;

// ------------------------------------------------------------------------------------------------ codec
// Gcd-period geometry (exl3_esimd.h:28-35): D words hold V values; G = periods per tile.
template <int K> struct Geo {
    static constexpr int gcd(int a, int b) { return b == 0 ? a : gcd(b, a % b); }
    static constexpr int g = gcd(K, 32);
    static constexpr int D = K / g;
    static constexpr int G = 256 / (32 / g);
    static constexpr int W = 8 * K;
};

// Offset (in words) of plain word w of tile j inside its PLANAR4 group of 4 tiles (moe_offload.py:68-73):
// word (tile j, period g = w / D, plane i = w % D) is stored at i*4G + j*G + g.
template <int K>
__host__ __device__ __forceinline__ int planar_base(int w) {
    return (w % Geo<K>::D) * 4 * Geo<K>::G + w / Geo<K>::D;
}

// Per-lane constants of the decode: the word offsets (relative to the tile's group start, tile 0) of the up to 3
// words that hold the lane's bit window, and the bit offset p0 of the window start inside the first word.
template <int K>
struct LaneWin {
    int oA, oB, oC;   // group-relative offsets for tile 0; add j*G for tile j (planar) or j*8K (plain)
    int p0;
    __device__ __forceinline__ void init(int lane, bool planar) {
        constexpr int NB = 256 * K;
        int S = (8 * lane + 1) * K - 16;
        S = ((S % NB) + NB) % NB;
        int w0 = S >> 5;
        p0 = S & 31;
        int wA = w0, wB = (w0 + 1) % (8 * K), wC = (w0 + 2) % (8 * K);
        if (planar) { oA = planar_base<K>(wA); oB = planar_base<K>(wB); oC = planar_base<K>(wC); }
        else { oA = wA; oB = wB; oC = wC; }
    }
    static constexpr bool kNeedC = (K >= 5);   // window of 7K+16 bits fits two aligned words unless K >= 5
};

// mul1 for two states -> packed fp16x2 {lo = st0, hi = st1}: x = st * 0x83DCD12D; dp4a gives 0x6400 + bytesum, whose
// low 16 bits are the fp16 bit pattern of 1024 + bytesum (exact); one fp16x2 fma applies c1, c2 with one rounding.
__device__ __forceinline__ uint32_t mul1_pair(uint32_t st0, uint32_t st1) {
    uint32_t x0 = st0 * 0x83DCD12Du, x1 = st1 * 0x83DCD12Du;
    uint32_t h0 = __dp4a(x0, 0x01010101u, 0x6400u);   // unsigned byte dot product: 0x6400 + sum of the 4 bytes
    uint32_t h1 = __dp4a(x1, 0x01010101u, 0x6400u);
    // {lo = h0, hi = h1}: both are < 2^16, so a byte permute packs them (ALU pipe, off the multiply-add pipe that
    // the multiplies and dp4a use)
    uint32_t hp = __byte_perm(h0, h1, 0x5410);
    __half2 h = *reinterpret_cast<__half2*>(&hp);
    const __half2 c1 = __halves2half2(__ushort_as_half((unsigned short)0x1eee), __ushort_as_half((unsigned short)0x1eee));
    const __half2 c2 = __halves2half2(__ushort_as_half((unsigned short)0xc931), __ushort_as_half((unsigned short)0xc931));
    __half2 r = __hfma2(h, c1, c2);
    return *reinterpret_cast<uint32_t*>(&r);
}

// State of value i (0..7) from the lane's aligned 64-bit window V = vh:vl (bit 0 of the window = MSB of vh).
template <int K, int i>
__device__ __forceinline__ uint32_t win_state(uint32_t vh, uint32_t vl) {
    constexpr int sh = 48 - i * K;
    if constexpr (sh >= 32) {
        if constexpr (sh == 48) return vh >> 16;
        else return (vh >> (sh - 32)) & 0xFFFFu;
    } else {
        return __funnelshift_r(vl, vh, sh) & 0xFFFFu;
    }
}

// Decode the lane's 8 values of one tile into the 4 A-fragment registers of W^T (see file header).
// a, b, c: the words at offsets oA, oB, oC of the lane window (c unused for K < 5).
template <int K>
__device__ __forceinline__ void decode8(uint32_t a, uint32_t b, uint32_t c, int p0, uint32_t r[4]) {
    uint32_t vh = __funnelshift_l(b, a, p0);
    uint32_t vl = LaneWin<K>::kNeedC ? __funnelshift_l(c, b, p0) : (b << p0);
    r[0] = mul1_pair(win_state<K, 0>(vh, vl), win_state<K, 1>(vh, vl));
    r[2] = mul1_pair(win_state<K, 2>(vh, vl), win_state<K, 3>(vh, vl));
    r[1] = mul1_pair(win_state<K, 4>(vh, vl), win_state<K, 5>(vh, vl));
    r[3] = mul1_pair(win_state<K, 6>(vh, vl), win_state<K, 7>(vh, vl));
}

// (row, col) inside the tile of fp16 half h (0/1) of A-fragment register q (0..3) of lane l (inverse of the map).
__device__ __forceinline__ void frag_pos(int lane, int q, int h, int& row, int& col) {
    // R0 = {v0,v1}, R1 = {v4,v5}, R2 = {v2,v3}, R3 = {v6,v7}; v_i at (k = 2(l%4)+bit0 + 8 bit1, n = l/4 + 8 bit2)
    int i = (q == 0 ? 0 : q == 1 ? 4 : q == 2 ? 2 : 6) + h;
    row = 2 * (lane & 3) + (i & 1) + 8 * ((i >> 1) & 1);
    col = (lane >> 2) + 8 * ((i >> 2) & 1);
}

// ------------------------------------------------------------------------------------------------ MMA
// D[16 x 8] += A[16 x 16] * B[16 x 8], fp16 inputs, fp32 accumulate (m16n8k16, row.col).
__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------------------------------------ packed fp32
// sm_100 issues two fp32 adds, multiplies or FMAs of a float2 as one instruction; each component rounds exactly as
// the scalar operation does.  a - b is formed as fma(b, -1, a): b * -1 is exact, so the single rounding is that of
// a - b.
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    float2 r;
    asm("{\n .reg .b64 pa, pb, pd;\n mov.b64 pa, {%2, %3};\n mov.b64 pb, {%4, %5};\n"
        " add.rn.f32x2 pd, pa, pb;\n mov.b64 {%0, %1}, pd;\n}\n"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
    float2 r;
    asm("{\n .reg .b64 pa, pb, pd;\n mov.b64 pa, {%2, %3};\n mov.b64 pb, {%4, %5};\n"
        " mul.rn.f32x2 pd, pa, pb;\n mov.b64 {%0, %1}, pd;\n}\n"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
    float2 r;
    asm("{\n .reg .b64 pa, pb, pc, pd;\n mov.b64 pa, {%2, %3};\n mov.b64 pb, {%4, %5};\n mov.b64 pc, {%6, %7};\n"
        " fma.rn.f32x2 pd, pa, pb, pc;\n mov.b64 {%0, %1}, pd;\n}\n"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return r;
}
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) { return f2_fma(b, make_float2(-1.0f, -1.0f), a); }

// ------------------------------------------------------------------------------------------------ FWHT
// In-warp FWHT-128 of one row held as 4 consecutive values per lane (v[j] = element 4*lane + j), Sylvester order,
// unnormalised, fp32 butterflies with strides 1, 2, 4, ..., 64 (exl3_esimd.h:210-221): strides 1 and 2 are inside
// the lane, strides 4..64 pair lanes lane ^ (stride/4).  Each butterfly computes a+b / a-b exactly as the reference;
// stride 2 and the cross-lane strides run on float2 pairs (v0, v1), (v2, v3).
__device__ __forceinline__ void fwht128_warp(float v[4], int lane) {
    float a, b;
    a = v[0]; b = v[1]; v[0] = a + b; v[1] = a - b;
    a = v[2]; b = v[3]; v[2] = a + b; v[3] = a - b;
    float2 p = make_float2(v[0], v[1]), q = make_float2(v[2], v[3]);
    {
        const float2 s = f2_add(p, q), d = f2_sub(p, q);
        p = s; q = d;
    }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        // lower element (lane without bit m) holds a, upper holds b: lower gets a + b = o + v, upper gets a - b =
        // o - v, i.e. fma(v, sign, o) with sign = -1 on the upper lane (v * -1 is exact)
        const float sg = (lane & m) ? -1.0f : 1.0f;
        const float2 sg2 = make_float2(sg, sg);
        const float2 op = make_float2(__shfl_xor_sync(0xffffffffu, p.x, m), __shfl_xor_sync(0xffffffffu, p.y, m));
        const float2 oq = make_float2(__shfl_xor_sync(0xffffffffu, q.x, m), __shfl_xor_sync(0xffffffffu, q.y, m));
        p = f2_fma(p, sg2, op);
        q = f2_fma(q, sg2, oq);
    }
    v[0] = p.x; v[1] = p.y; v[2] = q.x; v[3] = q.y;
}

__device__ __forceinline__ float rn16(float f) { return __half2float(__float2half_rn(f)); }

__device__ __forceinline__ float load_act(const void* x, bool bf16, size_t i) {
    return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i])
                : __half2float(reinterpret_cast<const __half*>(x)[i]);
}

}  // namespace exl3b
