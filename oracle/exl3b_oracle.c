/*
 * exl3b_oracle.c -- CPU restatement of the reference EXL3 routed-expert MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA kernels in
 * qwen38-flash-next-b70-offload_b200/csrc.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it.  The product path never calls it.
 *
 * Parity status: partially pinned.  The reference (SYCL/ESIMD for an Intel GPU) cannot be built or
 * run here and commits no golden vectors for this path.  What pins this restatement:
 *   - the two independent statements of the mul1 codebook inside the reference
 *     (kernels/moe-a8/exl3_esimd.h:40-68 vector form, kernels/moe-a8/exl3_moe.a8.sycl:1365-1377
 *     scalar form) agree with ora_mul1() on all 65,536 states (tests/test_oracle_codec.py);
 *   - the codebook range bound kQ8WMax = 3.453125 (experimental/n111-victim-ring/csrc/exl3_ops.sycl:522-525);
 *   - the blob sizes the reference asserts: 1,862,400 B at (H, I, K) = (2560, 640, 3)
 *     (kernels/moe-a8/exl3_moe.a8.sycl:7, experimental/n111-victim-ring/n111_test.py:21-23);
 *   - the cached-path == uncached-path identity (experimental/n111-victim-ring/n111_test.py:207-211);
 *   - the blob bytes of the reference's own packer (plugin/exl3xpu/moe_offload.py:68-89, pure torch, run
 *     on the CPU by tests/golden/make_ref_pack.py into tests/golden/ref_pack.npz): this restatement reads
 *     those blobs back to the checkpoint words it was given (tests/test_oracle_codec.py).
 * Layer outputs (floating point) are therefore compared within the north-star tolerance.
 *
 * Every function cites the reference file:line it restates.  Arithmetic is kept in the same
 * precision and rounding points as the reference: fp32 FWHT butterflies, fp16 roundings of
 * xh / g / u / act / abuf, fp32 epilogues.  Dot products (the GEMV/GEMM sums) are accumulated in
 * double here (the reference accumulates fp16 tile-row partials in fp32 for decode and fp32 in XMX
 * for prefill; neither order is reproducible on a CPU, so the oracle uses the most accurate sum).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------------------------------
 * IEEE conversions (round to nearest even).  fp16 and bf16 are passed as uint16_t bit patterns.
 */
EXPORT float ora_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t b;
    if (e == 0) {
        if (m == 0) {
            b = s;
        } else { /* subnormal: value = m * 2^-24 */
            float f = (float)m * 5.9604644775390625e-08f;
            memcpy(&b, &f, 4);
            b |= s;
        }
    } else if (e == 31) {
        b = s | 0x7F800000u | (m << 13);
    } else {
        b = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* Round a double to the nearest fp16 (ties to even), with subnormals and overflow to inf. */
EXPORT uint16_t ora_f64_to_f16(double v) {
    uint16_t sign = 0;
    if (isnan(v)) return 0x7E00;
    if (signbit(v)) { sign = 0x8000; v = -v; }
    if (v == 0.0) return sign;
    if (v >= 65520.0) return sign | 0x7C00; /* >= max + half ulp rounds to inf */
    int ex;
    (void)frexp(v, &ex);          /* v = f * 2^ex, f in [0.5, 1) */
    int e = ex - 1;               /* v in [2^e, 2^(e+1)) */
    if (e < -14) e = -14;         /* subnormal range shares the 2^-24 quantum */
    double q = ldexp(1.0, e - 10); /* value of one ulp */
    double n = v / q;             /* exact: division by a power of two */
    double fl = floor(n), fr = n - fl;
    uint64_t mant = (uint64_t)fl;
    if (fr > 0.5 || (fr == 0.5 && (mant & 1))) mant++;
    /* re-encode mant * 2^(e-10) */
    if (mant == 0) return sign;
    if (e == -14 && mant < 1024) return sign | (uint16_t)mant; /* subnormal */
    if (mant >= 2048) { mant >>= 1; e++; }
    if (e > 15) return sign | 0x7C00;
    return sign | (uint16_t)((e + 15) << 10) | (uint16_t)(mant - 1024);
}

EXPORT uint16_t ora_f32_to_f16(float f) { return ora_f64_to_f16((double)f); }

/* fp32 value rounded through fp16 (the reference's convert<float>(convert<fp16>(v))). */
static inline float rn16(float f) { return ora_f16_to_f32(ora_f32_to_f16(f)); }

EXPORT float ora_bf16_to_f32(uint16_t h) {
    uint32_t b = (uint32_t)h << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

EXPORT uint16_t ora_f32_to_bf16(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x40);
    uint32_t lsb = (b >> 16) & 1;
    b += 0x7FFFu + lsb;
    return (uint16_t)(b >> 16);
}

/* ------------------------------------------------------------------------------------------------
 * Trellis codec.
 *
 * mul1 codebook: kernels/moe-a8/exl3_esimd.h:45-68 (decode_cb_h<CB=2>): x = st * 0x83DCD12D (mod 2^32),
 * h = 1024 + sum of the four bytes of x (exact in fp16: the dp4a with accumulator 0x6400 yields the
 * fp16 bit pattern of 1024 + byte sum), w = fp16(h * 0.00676727294921875 - 10.3828125) with ONE
 * rounding (fp16 fma).  The scalar restatement at kernels/moe-a8/exl3_moe.a8.sycl:1365-1377 computes
 * the same value in fp32 (exact: h*c1 has at most 22 significant bits) and rounds once to fp16.
 */
EXPORT uint16_t ora_mul1(uint32_t st) {
    uint32_t x = (st & 0xFFFFu) * 0x83DCD12Du;
    uint32_t bs = (x & 255u) + ((x >> 8) & 255u) + ((x >> 16) & 255u) + (x >> 24);
    double h = 1024.0 + (double)bs;
    return ora_f64_to_f16(h * 0.00676727294921875 + (-10.3828125));
}

/* Position of value t (0..255) inside its 16x16 tile: kernels/moe-a8/exl3_esimd.h:4-9. */
EXPORT int ora_tile_row(int t) { return 8 * ((t >> 1) & 1) + 2 * ((t >> 3) & 3) + (t & 1); }
EXPORT int ora_tile_col(int t) { return (t >> 5) + 8 * ((t >> 2) & 1); }

/*
 * 16-bit state of value t in a tile whose 8K words are given in plain (tile-major) order.
 * The tile is one circular MSB-first bit stream of 256*K bits; value t is the 16-bit window that
 * ends at bit (t+1)*K (exl3_esimd.h:4-6 and the word/shift form of tile_states, :120-149; the
 * circular previous word of period 0 is the tile's last word, load_words :155-169).
 */
EXPORT uint32_t ora_tile_state(const uint32_t* tw, int K, int t) {
    int nbits = 256 * K, end = (t + 1) * K;
    int b0 = ((end - 16) % nbits + nbits) % nbits;   /* first bit of the window (circular) */
    /* gather the 16 bits MSB-first: bits b0 .. b0+15 (mod nbits) */
    uint32_t st = 0;
    int w = b0 >> 5, o = b0 & 31;
    if (o <= 16 && b0 + 16 <= nbits) {
        st = (tw[w] >> (16 - o)) & 0xFFFFu;                 /* window inside one word */
    } else {
        for (int b = 0; b < 16; ++b) {
            int bb = (b0 + b) % nbits;
            st = (st << 1) | ((tw[bb >> 5] >> (31 - (bb & 31))) & 1u);
        }
    }
    return st;
}

/* gcd-period geometry of Geo<K> (exl3_esimd.h:28-35): D words hold V whole values, G periods per tile. */
static int gcd_i(int a, int b) { return b == 0 ? a : gcd_i(b, a % b); }
EXPORT int ora_geo_D(int K) { return K / gcd_i(K, 32); }
EXPORT int ora_geo_G(int K) { return 256 / (32 / gcd_i(K, 32)); }

/*
 * PLANAR4 word order (moe_offload.py:68-73, exl3_moe.a8.sycl:8-11): within a k-row, tiles are grouped
 * by 4 along n; word (tile j, period g, plane i) -- plain word index D*g + i of tile j -- is stored at
 * group offset i*(4*G) + j*G + g.  With D = 1 (even K) this is the plain order.
 * Returns the group-relative offset of plain word w of tile j.
 */
EXPORT int ora_planar_offset(int K, int j, int w) {
    int D = ora_geo_D(K), G = ora_geo_G(K);
    int g = w / D, i = w % D;
    return i * (4 * G) + j * G + g;
}

/* Gather one tile's words (plain order) from a PLANAR4 row: row points at the row start, tile c. */
static void load_tile_planar(const uint32_t* row, int K, int c, uint32_t* tw) {
    int W = 8 * K;
    const uint32_t* grp = row + (size_t)(c / 4) * 4 * W;
    for (int w = 0; w < W; ++w) tw[w] = grp[ora_planar_offset(K, c % 4, w)];
}

/* Decode one tile (plain word order) to fp16 bits laid out [16 rows][16 cols]. */
EXPORT void ora_decode_tile(const uint32_t* tw, int K, uint16_t* out) {
    for (int t = 0; t < 256; ++t)
        out[ora_tile_row(t) * 16 + ora_tile_col(t)] = ora_mul1(ora_tile_state(tw, K, t));
}

/*
 * Dequantise a tile matrix to W_inner fp16 [rows16*16][ntiles*16] (ld = ldw):
 * words: row r starts at words + r*row_stride (words), tiles tile0 .. tile0+ntiles-1 of that row.
 * planar: 1 = PLANAR4 rows (blob layout; tile0 must be a multiple of 4), 0 = plain tile-major rows
 * (checkpoint layout).  This is the dequant contract of ReconstructKernel (exl3_esimd.h:869-936).
 */
EXPORT void ora_dequant(const uint32_t* words, int rows16, size_t row_stride, int tile0, int ntiles, int K,
                        int planar, uint16_t* w, size_t ldw) {
    uint32_t tw[8 * 16];
    uint16_t tile[256];
    int W = 8 * K;
    for (int r = 0; r < rows16; ++r) {
        const uint32_t* row = words + (size_t)r * row_stride;
        for (int c = 0; c < ntiles; ++c) {
            if (planar) load_tile_planar(row, K, tile0 + c, tw);
            else memcpy(tw, row + (size_t)(tile0 + c) * W, (size_t)W * 4);
            ora_decode_tile(tw, K, tile);
            for (int i = 0; i < 16; ++i)
                for (int j = 0; j < 16; ++j) w[((size_t)r * 16 + i) * ldw + (size_t)c * 16 + j] = tile[i * 16 + j];
        }
    }
}

/* ------------------------------------------------------------------------------------------------
 * Blob geometry (exl3_moe.a8.sycl:42-54, moe_offload.py:8-13), generalised to a K per tensor:
 *   gate|up trellis: H/16 rows, each row = I/16 gate tiles (8*Kg words) then I/16 up tiles (8*Ku words),
 *                    PLANAR4 per row;
 *   down trellis:    I/16 rows of H/16 tiles (8*Kd words), PLANAR4 per row;
 *   fp16 vectors:    suh_g[H] suh_u[H] svh_g[I] svh_u[I] suh_d[I] svh_d[H].
 * With Kg = Ku = Kd = K this is exactly the reference layout.
 */
typedef struct { int H, I, Kg, Ku, Kd; } OraGeom;

static size_t gu_words(const OraGeom* g) { return (size_t)(g->H / 16) * (g->I / 16) * 8 * (g->Kg + g->Ku); }
static size_t d_words(const OraGeom* g) { return (size_t)(g->I / 16) * (g->H / 16) * 8 * g->Kd; }
static size_t off_vec(const OraGeom* g) { return (gu_words(g) + d_words(g)) * 4; }

EXPORT int64_t ora_blob_bytes(int H, int I, int Kg, int Ku, int Kd) {
    OraGeom g = {H, I, Kg, Ku, Kd};
    return (int64_t)(off_vec(&g) + (size_t)(3 * H + 3 * I) * 2);
}

/* proj 0 = gate, 1 = up -> W_inner [H][I]; proj 2 = down -> W_inner [I][H]. */
EXPORT void ora_blob_dequant(const uint8_t* blob, int H, int I, int Kg, int Ku, int Kd, int proj, uint16_t* w) {
    OraGeom g = {H, I, Kg, Ku, Kd};
    const uint32_t* tr = (const uint32_t*)blob;
    if (proj == 0 || proj == 1) {
        size_t rs = (size_t)(I / 16) * 8 * (Kg + Ku);
        const uint32_t* base = tr + (proj == 1 ? (size_t)(I / 16) * 8 * Kg : 0);
        ora_dequant(base, H / 16, rs, 0, I / 16, proj == 1 ? Ku : Kg, 1, w, (size_t)I);
    } else {
        ora_dequant(tr + gu_words(&g), I / 16, (size_t)(H / 16) * 8 * Kd, 0, H / 16, Kd, 1, w, (size_t)H);
    }
}

/* ------------------------------------------------------------------------------------------------
 * FWHT-128, Sylvester order, unnormalised, butterfly strides 1, 2, ..., 64 in fp32
 * (exl3_esimd.h:210-221); the caller multiplies by kRsqrt128 (exl3_esimd.h:223).
 */
static const float kRsqrt128 = 0.08838834764831845f;

EXPORT void ora_fwht128(float* v) {
    for (int h = 1; h < 128; h <<= 1)
        for (int i = 0; i < 128; i += 2 * h)
            for (int j = i; j < i + h; ++j) {
                float a = v[j], b = v[j + h];
                v[j] = a + b;
                v[j + h] = a - b;
            }
}

/*
 * Input transform of one 128-block (exl3_moe.a8.sycl:179-195, GateUpKernel; same in GateUpDpasKernel
 * :462-475): xh = fp16( FWHT( fp16(x * suh) ) * r ).  x is bf16 (as in the benchmarks) or fp16.
 */
static void had_in_block(const uint16_t* x, int x_is_bf16, const uint16_t* suh, uint16_t* xh) {
    float v[128];
    for (int i = 0; i < 128; ++i) {
        float xv = x_is_bf16 ? ora_bf16_to_f32(x[i]) : ora_f16_to_f32(x[i]);
        v[i] = rn16(xv * ora_f16_to_f32(suh[i]));
    }
    ora_fwht128(v);
    for (int i = 0; i < 128; ++i) xh[i] = ora_f32_to_f16(v[i] * kRsqrt128);
}

EXPORT void ora_had_in(const uint16_t* x, int x_is_bf16, const uint16_t* suh, int n, uint16_t* xh) {
    for (int b = 0; b < n / 128; ++b) had_in_block(x + b * 128, x_is_bf16, suh + b * 128, xh + b * 128);
}

static const uint16_t* vec_ptr(const uint8_t* blob, const OraGeom* g, int which) {
    /* which: 0 suh_g, 1 suh_u, 2 svh_g, 3 svh_u, 4 suh_d, 5 svh_d (exl3_moe.a8.sycl:47-52) */
    size_t o = off_vec(g);
    size_t H = (size_t)g->H, I = (size_t)g->I;
    size_t offs[6] = {0, H, 2 * H, 2 * H + I, 2 * H + 2 * I, 2 * H + 3 * I};
    return (const uint16_t*)(blob + o + offs[which] * 2);
}

/*
 * One (token, pick) of the routed MoE, decode semantics:
 *   gate/up: exl3_moe.a8.sycl:121-258 (GateUpKernel), epilogue :239-256;
 *   down:    exl3_moe.a8.sycl:264-366 (DownKernel), epilogue :355-364.
 * wg, wu: W_inner gate/up [H][I] (fp16 bits); wd: W_inner down [I][H].  Returns y[H] fp32 and the
 * down-input abuf[I] fp16 bits (Hadamard domain).
 */
static void expert_forward(const uint16_t* x, int x_is_bf16, const uint8_t* blob, const OraGeom* g,
                           const uint16_t* wg, const uint16_t* wu, const uint16_t* wd, float wpick,
                           uint16_t* abuf, float* y) {
    int H = g->H, I = g->I;
    uint16_t* xg = (uint16_t*)malloc((size_t)H * 2);
    uint16_t* xu = (uint16_t*)malloc((size_t)H * 2);
    float* gg = (float*)malloc((size_t)I * 4);
    float* uu = (float*)malloc((size_t)I * 4);
    float* vv = (float*)malloc((size_t)H * 4);
    ora_had_in(x, x_is_bf16, vec_ptr(blob, g, 0), H, xg);
    ora_had_in(x, x_is_bf16, vec_ptr(blob, g, 1), H, xu);
    float* xgf = (float*)malloc((size_t)H * 4);
    float* xuf = (float*)malloc((size_t)H * 4);
    for (int k = 0; k < H; ++k) { xgf[k] = ora_f16_to_f32(xg[k]); xuf[k] = ora_f16_to_f32(xu[k]); }
    /* decoded weights: fp16 -> fp32 table lookup is exact */
    for (int n = 0; n < I; ++n) {
        double sg = 0.0, su = 0.0;
        for (int k = 0; k < H; ++k) {
            sg += (double)xgf[k] * (double)ora_f16_to_f32(wg[(size_t)k * I + n]);
            su += (double)xuf[k] * (double)ora_f16_to_f32(wu[(size_t)k * I + n]);
        }
        gg[n] = (float)sg;
        uu[n] = (float)su;
    }
    const uint16_t* svg = vec_ptr(blob, g, 2);
    const uint16_t* svu = vec_ptr(blob, g, 3);
    const uint16_t* sud = vec_ptr(blob, g, 4);
    const uint16_t* svd = vec_ptr(blob, g, 5);
    for (int nb = 0; nb < I / 128; ++nb) {
        float* gb = gg + nb * 128;
        float* ub = uu + nb * 128;
        float act[128];
        ora_fwht128(gb);
        ora_fwht128(ub);
        for (int i = 0; i < 128; ++i) {
            float gv = rn16(gb[i] * kRsqrt128 * ora_f16_to_f32(svg[nb * 128 + i]));
            float uv = rn16(ub[i] * kRsqrt128 * ora_f16_to_f32(svu[nb * 128 + i]));
            float a = gv / (1.0f + expf(-gv)) * uv; /* SiLU(g) * u, :248 */
            a = rn16(a);
            act[i] = rn16(a * ora_f16_to_f32(sud[nb * 128 + i]));
        }
        ora_fwht128(act);
        for (int i = 0; i < 128; ++i) abuf[nb * 128 + i] = ora_f32_to_f16(act[i] * kRsqrt128);
    }
    float* af = (float*)malloc((size_t)I * 4);
    for (int k = 0; k < I; ++k) af[k] = ora_f16_to_f32(abuf[k]);
    for (int n = 0; n < H; ++n) {
        double s = 0.0;
        for (int k = 0; k < I; ++k) s += (double)af[k] * (double)ora_f16_to_f32(wd[(size_t)k * H + n]);
        vv[n] = (float)s;
    }
    for (int nb = 0; nb < H / 128; ++nb) {
        float* vb = vv + nb * 128;
        ora_fwht128(vb);
        for (int i = 0; i < 128; ++i) y[nb * 128 + i] = vb[i] * (kRsqrt128 * wpick) * ora_f16_to_f32(svd[nb * 128 + i]);
    }
    free(xg); free(xu); free(gg); free(uu); free(vv); free(xgf); free(xuf); free(af);
}

/*
 * Full routed-MoE layer (moe_forward semantics, exl3_moe.a8.sycl:1263-1314): for every token m and pick
 * k, y = expert(ids[m,k]) weighted by w[m,k]; out[m] = sum_k y in fixed k order (CombineKernel
 * :371-395) rounded to bf16 (out_bf16 = 1) or fp16.  blobs[e] points at expert e's blob; kinfo
 * (optional, may be NULL) gives per-expert (Kg, Ku, Kd) packed as Kg | Ku << 4 | Kd << 8, else K.
 * Picks with weight exactly 0 still run (the reference computes them); y_out (optional) receives
 * every pick's fp32 y in [M*topk][H] pick order and abuf_out (optional) the fp16 down inputs.
 */
EXPORT void ora_moe_layer(const uint16_t* x, int x_is_bf16, const int32_t* ids, const float* w, int M, int topk,
                          const uint8_t* const* blobs, const int32_t* kinfo, int H, int I, int K, int out_bf16,
                          void* out_v, float* y_out, uint16_t* abuf_out) {
    /* out_bf16: 0 fp16 bits, 1 bf16 bits, 2 fp32 (the layer output before its final rounding) */
    uint16_t* out = (uint16_t*)out_v;
    float* out_f = (float*)out_v;
    float* y = (float*)malloc((size_t)H * 4);
    float* acc = (float*)malloc((size_t)H * 4);
    uint16_t* abuf = (uint16_t*)malloc((size_t)I * 2);
    uint16_t* wg = (uint16_t*)malloc((size_t)H * I * 2);
    uint16_t* wu = (uint16_t*)malloc((size_t)H * I * 2);
    uint16_t* wd = (uint16_t*)malloc((size_t)H * I * 2);
    for (int m = 0; m < M; ++m) {
        for (int i = 0; i < H; ++i) acc[i] = 0.0f;
        for (int k = 0; k < topk; ++k) {
            int e = ids[m * topk + k];
            OraGeom g = {H, I, K, K, K};
            if (kinfo) { g.Kg = kinfo[e] & 15; g.Ku = (kinfo[e] >> 4) & 15; g.Kd = (kinfo[e] >> 8) & 15; }
            const uint8_t* blob = blobs[e];
            ora_blob_dequant(blob, H, I, g.Kg, g.Ku, g.Kd, 0, wg);
            ora_blob_dequant(blob, H, I, g.Kg, g.Ku, g.Kd, 1, wu);
            ora_blob_dequant(blob, H, I, g.Kg, g.Ku, g.Kd, 2, wd);
            expert_forward(x + (size_t)m * H, x_is_bf16, blob, &g, wg, wu, wd, w[m * topk + k], abuf, y);
            if (y_out) memcpy(y_out + ((size_t)m * topk + k) * H, y, (size_t)H * 4);
            if (abuf_out) memcpy(abuf_out + ((size_t)m * topk + k) * I, abuf, (size_t)I * 2);
            for (int i = 0; i < H; ++i) acc[i] += y[i];
        }
        for (int i = 0; i < H; ++i) {
            if (out_bf16 == 2) out_f[(size_t)m * H + i] = acc[i];
            else out[(size_t)m * H + i] = out_bf16 ? ora_f32_to_bf16(acc[i]) : ora_f32_to_f16(acc[i]);
        }
    }
    free(y); free(acc); free(abuf); free(wg); free(wu); free(wd);
}

/*
 * All picks of ONE expert (n picks: token rows x + tok[i] * x_stride, weights w[i]) -> y [n][H] fp32, with exactly
 * expert_forward's arithmetic per pick: the weights are dequantised once and the GEMV sums run in the same ascending
 * k order per output (k outer, outputs inner).  y_half = 1 rounds y to fp16 (the prefill's stored y, :626-631).
 * Threads may call this concurrently for different experts.
 */
EXPORT void ora_expert_picks(const uint16_t* x, int64_t x_stride, int x_is_bf16, const int32_t* tok, const float* w,
                             int n, const uint8_t* blob, int Kg, int Ku, int Kd, int H, int I, int y_half, float* y) {
    OraGeom g = {H, I, Kg, Kg, Kd};
    g.Ku = Ku;
    uint16_t* wh = (uint16_t*)malloc((size_t)H * I * 2);
    float* wg = (float*)malloc((size_t)H * I * 4);
    float* wu = (float*)malloc((size_t)H * I * 4);
    float* wd = (float*)malloc((size_t)H * I * 4);
    ora_blob_dequant(blob, H, I, Kg, Ku, Kd, 0, wh);
    for (size_t q = 0; q < (size_t)H * I; ++q) wg[q] = ora_f16_to_f32(wh[q]);
    ora_blob_dequant(blob, H, I, Kg, Ku, Kd, 1, wh);
    for (size_t q = 0; q < (size_t)H * I; ++q) wu[q] = ora_f16_to_f32(wh[q]);
    ora_blob_dequant(blob, H, I, Kg, Ku, Kd, 2, wh);
    for (size_t q = 0; q < (size_t)H * I; ++q) wd[q] = ora_f16_to_f32(wh[q]);
    uint16_t* xg = (uint16_t*)malloc((size_t)H * 2);
    uint16_t* xu = (uint16_t*)malloc((size_t)H * 2);
    uint16_t* abuf = (uint16_t*)malloc((size_t)I * 2);
    double* sg = (double*)malloc((size_t)I * 8);
    double* su = (double*)malloc((size_t)I * 8);
    double* sd = (double*)malloc((size_t)H * 8);
    float* gg = (float*)malloc((size_t)I * 4);
    float* uu = (float*)malloc((size_t)I * 4);
    float* vv = (float*)malloc((size_t)H * 4);
    const uint16_t* svg = vec_ptr(blob, &g, 2);
    const uint16_t* svu = vec_ptr(blob, &g, 3);
    const uint16_t* sud = vec_ptr(blob, &g, 4);
    const uint16_t* svd = vec_ptr(blob, &g, 5);
    for (int p = 0; p < n; ++p) {
        const uint16_t* xr = x + (size_t)tok[p] * x_stride;
        ora_had_in(xr, x_is_bf16, vec_ptr(blob, &g, 0), H, xg);
        ora_had_in(xr, x_is_bf16, vec_ptr(blob, &g, 1), H, xu);
        for (int c = 0; c < I; ++c) { sg[c] = 0.0; su[c] = 0.0; }
        for (int k = 0; k < H; ++k) {
            const double a = (double)ora_f16_to_f32(xg[k]), b = (double)ora_f16_to_f32(xu[k]);
            const float* rg = wg + (size_t)k * I;
            const float* ru = wu + (size_t)k * I;
            for (int c = 0; c < I; ++c) { sg[c] += a * (double)rg[c]; su[c] += b * (double)ru[c]; }
        }
        for (int c = 0; c < I; ++c) { gg[c] = (float)sg[c]; uu[c] = (float)su[c]; }
        for (int nb = 0; nb < I / 128; ++nb) {
            float* gb = gg + nb * 128;
            float* ub = uu + nb * 128;
            float act[128];
            ora_fwht128(gb);
            ora_fwht128(ub);
            for (int i = 0; i < 128; ++i) {
                float gv = rn16(gb[i] * kRsqrt128 * ora_f16_to_f32(svg[nb * 128 + i]));
                float uv = rn16(ub[i] * kRsqrt128 * ora_f16_to_f32(svu[nb * 128 + i]));
                float a = gv / (1.0f + expf(-gv)) * uv;
                a = rn16(a);
                act[i] = rn16(a * ora_f16_to_f32(sud[nb * 128 + i]));
            }
            ora_fwht128(act);
            for (int i = 0; i < 128; ++i) abuf[nb * 128 + i] = ora_f32_to_f16(act[i] * kRsqrt128);
        }
        for (int c = 0; c < H; ++c) sd[c] = 0.0;
        for (int k = 0; k < I; ++k) {
            const double a = (double)ora_f16_to_f32(abuf[k]);
            const float* rd = wd + (size_t)k * H;
            for (int c = 0; c < H; ++c) sd[c] += a * (double)rd[c];
        }
        for (int c = 0; c < H; ++c) vv[c] = (float)sd[c];
        float* yp = y + (size_t)p * H;
        for (int nb = 0; nb < H / 128; ++nb) {
            float* vb = vv + nb * 128;
            ora_fwht128(vb);
            for (int i = 0; i < 128; ++i) {
                float v = vb[i] * (kRsqrt128 * w[p]) * ora_f16_to_f32(svd[nb * 128 + i]);
                yp[nb * 128 + i] = y_half ? ora_f16_to_f32(ora_f32_to_f16(v)) : v;
            }
        }
    }
    free(wh); free(wg); free(wu); free(wd); free(xg); free(xu); free(abuf);
    free(sg); free(su); free(sd); free(gg); free(uu); free(vv);
}

/*
 * Dense EXL3 GLU (the config-5 shared expert): same math as one routed pick with weight 1, through
 * the dense linear contract (experimental/n111-victim-ring/csrc/exl3_ops.sycl:651-757: input Hadamard,
 * W_inner GEMM, output Hadamard * svh; the GLU glue SiLU(gate)*up happens between linears in the
 * model).  The shared expert is stored as one blob of the routed layout, so this reuses expert_forward.
 * y is fp32 [H], un-gated; the caller applies sigmoid(x . g_s) (the model's shared-expert gate).
 */
EXPORT void ora_dense_glu(const uint16_t* x, int x_is_bf16, const uint8_t* blob, int H, int I, int Kg, int Ku,
                          int Kd, float* y) {
    OraGeom g = {H, I, Kg, Ku, Kd};
    uint16_t* wg = (uint16_t*)malloc((size_t)H * I * 2);
    uint16_t* wu = (uint16_t*)malloc((size_t)H * I * 2);
    uint16_t* wd = (uint16_t*)malloc((size_t)H * I * 2);
    uint16_t* abuf = (uint16_t*)malloc((size_t)I * 2);
    ora_blob_dequant(blob, H, I, Kg, Ku, Kd, 0, wg);
    ora_blob_dequant(blob, H, I, Kg, Ku, Kd, 1, wu);
    ora_blob_dequant(blob, H, I, Kg, Ku, Kd, 2, wd);
    expert_forward(x, x_is_bf16, blob, &g, wg, wu, wd, 1.0f, abuf, y);
    free(wg); free(wu); free(wd); free(abuf);
}

/*
 * Shared-expert gate (config 5; the model's shared_expert_gate, a bf16 Linear(H -> 1) followed by a sigmoid):
 * s = dot(x, g) with the router's arithmetic (ora_router_dot), weight = 1 / (1 + expf(-s)).  The shared expert
 * then enters the combine as one more pick per token, after the routed picks.
 */
EXPORT float ora_router_dot(const uint16_t* x, const uint16_t* wr, int H);
EXPORT float ora_shared_gate(const uint16_t* x, const uint16_t* g, int H) {
    const float s = ora_router_dot(x, g, H);
    return 1.0f / (1.0f + expf(-s));
}

/* ------------------------------------------------------------------------------------------------
 * Router (SGLang TopK semantics consumed at plugin/sglang_plugin.tier.py:534-535, 560; SGLang itself
 * is not vendored, so this build defines the arithmetic exactly and the CUDA kernel follows it):
 *   logit[t,e] = dot(x[t,:], Wr[e,:]) + bias[e], where dot is the sum of 32 chunk partials:
 *     partial c (c = 0..31) covers k in [c*H/32, (c+1)*H/32), accumulated in ascending k with
 *     fp32 fma starting from 0; the 32 partials are combined by the xor butterfly
 *     v[l] = v[l] + v[l ^ o] for o = 16, 8, 4, 2, 1 (the value of lane 0 is the result).
 *   top-k: largest logits, ties to the lower expert id, output in descending order.
 *   weights: softmax over the selected logits (equal to the renormalised full softmax):
 *     w_i = expf(l_i - l_0) / sum_j expf(l_j - l_0), sum in selection order.
 */
EXPORT float ora_router_dot(const uint16_t* x, const uint16_t* wr, int H) {
    float v[32];
    int cl = H / 32;
    for (int c = 0; c < 32; ++c) {
        float a = 0.0f;
        for (int k = c * cl; k < (c + 1) * cl; ++k) a = fmaf(ora_bf16_to_f32(x[k]), ora_bf16_to_f32(wr[k]), a);
        v[c] = a;
    }
    for (int o = 16; o >= 1; o >>= 1) {
        float nv[32];
        for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
        memcpy(v, nv, sizeof(v));
    }
    return v[0];
}

EXPORT void ora_router(const uint16_t* x, const uint16_t* wr, const float* bias, int T, int H, int E, int topk,
                       int32_t* ids, float* w, float* logits_out) {
    float* lg = (float*)malloc((size_t)E * 4);
    unsigned char* used = (unsigned char*)malloc((size_t)E);
    for (int t = 0; t < T; ++t) {
        for (int e = 0; e < E; ++e) {
            float d = ora_router_dot(x + (size_t)t * H, wr + (size_t)e * H, H);
            lg[e] = bias ? d + bias[e] : d;
            if (logits_out) logits_out[(size_t)t * E + e] = lg[e];
            used[e] = 0;
        }
        float sel[64];
        for (int k = 0; k < topk; ++k) {
            int best = -1;
            for (int e = 0; e < E; ++e) {
                if (used[e]) continue;
                if (best < 0 || lg[e] > lg[best]) best = e; /* strict: ties keep the lower id */
            }
            used[best] = 1;
            ids[(size_t)t * topk + k] = best;
            sel[k] = lg[best];
        }
        float s = 0.0f, ex[64];
        for (int k = 0; k < topk; ++k) { ex[k] = expf(sel[k] - sel[0]); s += ex[k]; }
        for (int k = 0; k < topk; ++k) w[(size_t)t * topk + k] = ex[k] / s;
    }
    free(lg); free(used);
}

/* ------------------------------------------------------------------------------------------------
 * Align (launch_align, exl3_moe.a8.sycl:639-680): histogram of picks per expert, exclusive scans,
 * active-expert list in ascending id, pairs bucketed by expert.  The reference's intra-expert order
 * depends on atomics (:674-676); this build fixes it to ascending pick index (a stable counting sort).
 * Outputs as in make_route (:744-757): act_expert/start/cnt/pstart[n_act], pair_tok/pair_w/pair_of
 * [npairs], blk_a [n_blk] (row-block -> active index, rows padded to `pad`).
 */
EXPORT void ora_align(const int32_t* ids, const float* w, int npairs, int topk, int E, int pad, int32_t* act_expert,
                      int32_t* act_start, int32_t* act_cnt, int32_t* act_pstart, int32_t* n_act, int32_t* pair_tok,
                      float* pair_w, int32_t* pair_of, int32_t* blk_a, int32_t* n_blk) {
    int* cnt = (int*)calloc((size_t)E, sizeof(int));
    int* start = (int*)calloc((size_t)E, sizeof(int));
    int* fill = (int*)calloc((size_t)E, sizeof(int));
    /* id -1 is "no pick" (an expert-parallel rank's picks owned by other ranks): not placed, pair_of = -1 */
    for (int i = 0; i < npairs; ++i) if (ids[i] >= 0) cnt[ids[i]]++;
    int st = 0, pst = 0, na = 0;
    for (int e = 0; e < E; ++e) {
        start[e] = st;
        int pc = (cnt[e] + pad - 1) / pad * pad;
        if (cnt[e] > 0) {
            act_expert[na] = e; act_start[na] = st; act_cnt[na] = cnt[e]; act_pstart[na] = pst;
            if (blk_a) for (int j = 0; j < pc / pad; ++j) blk_a[pst / pad + j] = na;
            na++;
        }
        st += cnt[e];
        pst += pc;
    }
    *n_act = na;
    if (n_blk) *n_blk = pst / pad;
    for (int i = 0; i < npairs; ++i) {
        int e = ids[i];
        if (e < 0) { pair_of[i] = -1; continue; }
        int pos = start[e] + fill[e]++;
        pair_tok[pos] = i / topk;
        pair_w[pos] = w[i];
        pair_of[i] = pos;
    }
    free(cnt); free(start); free(fill);
}

/* ------------------------------------------------------------------------------------------------
 * Device expert cache step (launch_ensure, exl3_moe.a8.sycl:837-1040) with this build's deterministic
 * rule in place of the reference's atomic orders:
 *   1. tier mask (:902-914), picks in ascending index: a pick whose key = layer*E + id has
 *      slot_of[key] < 0 and ram_res[key] == 0 is logged to ring[1 + (ring[0]++ % cap)] and replaced
 *      by (safe[layer], weight 0) in place.
 *   2. T = ++tick (prefetch mode: T = tick).
 *   3. hits (:919-921): slot_last[s] = T unless the slot is pinned (INT_MAX).
 *   4. misses in ascending expert id; at most min(max_fill, E) of them (the first ones) get slots.
 *   5. victims (:927-1000): among slots with slot_last < T, the nm smallest keys (u, s) with
 *      u = slot_last + 1 (empty = 0) -- exact LRU, ties to the lower slot index.
 *   6. pairing: the i-th miss takes the i-th selected slot in ascending slot index; assignment as
 *      :1002-1019 (old owner repointed to host_base[old/E] + (old%E)*hstride, fill_all[key] =
 *      slot_base + s*blob, fill_list = [n, e...]; prefetch mode writes pf_slot instead of fill_all).
 *   vict (optional, may be NULL): [n, (old_key or -1 when its RAM copy is resident, slot) x n].
 * Returns the number of fills.
 */
EXPORT int ora_ensure(int32_t* ids, float* w, int npairs, int layer, int E, int S, int64_t* ptrs_all,
                      int32_t* slot_of, int32_t* slot_key, int32_t* slot_last, int32_t* tick,
                      const int64_t* host_base, int64_t slot_base, int64_t blob, int64_t hstride, int64_t* fill_all,
                      int32_t* fill_list, int max_fill, int prefetch, int32_t* pf_slot, const uint8_t* ram_res,
                      int32_t* ring, int ring_cap, const int32_t* safe, int32_t* vict) {
    if (ram_res && !prefetch) {
        for (int i = 0; i < npairs; ++i) {
            int key = layer * E + ids[i];
            if (slot_of[key] < 0 && !ram_res[key]) {
                int c = ring[0]++;
                ring[1 + c % ring_cap] = key;
                ids[i] = safe[layer];
                w[i] = 0.0f;
            }
        }
    }
    int T = prefetch ? tick[0] : ++tick[0];
    unsigned char* need = (unsigned char*)calloc((size_t)E, 1);
    int* miss = (int*)malloc((size_t)E * sizeof(int));
    for (int i = 0; i < npairs; ++i) need[ids[i]] = 1;
    int nmiss = 0;
    for (int e = 0; e < E; ++e) {
        if (!need[e]) continue;
        int s = slot_of[layer * E + e];
        if (s >= 0) {
            if (slot_last[s] != 0x7FFFFFFF) slot_last[s] = T;
        } else {
            miss[nmiss++] = e;
        }
    }
    int mf = max_fill < E ? max_fill : E;
    int nm = S > 0 ? (nmiss < mf ? nmiss : mf) : 0;
    int elig = 0;
    for (int s = 0; s < S; ++s) elig += slot_last[s] < T;
    if (nm > elig) nm = elig;
    if (nm == 0) {
        fill_list[0] = 0;
        if (vict) vict[0] = 0;
        free(need); free(miss);
        return 0;
    }
    /* select the nm smallest (u, s) among eligible slots */
    unsigned char* sel = (unsigned char*)calloc((size_t)S, 1);
    for (int k = 0; k < nm; ++k) {
        int best = -1;
        uint32_t bu = 0;
        for (int s = 0; s < S; ++s) {
            if (sel[s] || slot_last[s] >= T) continue;
            uint32_t u = (uint32_t)(slot_last[s] + 1);
            if (best < 0 || u < bu) { best = s; bu = u; }
        }
        sel[best] = 1;
    }
    int mi = 0;
    for (int s = 0; s < S && mi < nm; ++s) {
        if (!sel[s]) continue;
        int e = miss[mi];
        int old = slot_key[s];
        if (vict) {
            vict[1 + 2 * mi] = (old >= 0 && ram_res && ram_res[old]) ? -1 : old;
            vict[2 + 2 * mi] = s;
        }
        if (old >= 0) {
            slot_of[old] = -1;
            ptrs_all[old] = host_base[old / E] + (int64_t)(old % E) * hstride;
        }
        int key = layer * E + e;
        slot_key[s] = key;
        slot_of[key] = s;
        slot_last[s] = T;
        if (prefetch) pf_slot[mi] = s;
        else fill_all[key] = slot_base + (int64_t)s * blob;
        fill_list[1 + mi] = e;
        mi++;
    }
    fill_list[0] = nm;
    if (vict) vict[0] = nm;
    free(need); free(miss); free(sel);
    return nm;
}

/* Cache commit at the end of a cached call (CombineKernel item 0, exl3_moe.a8.sycl:378-386). */
EXPORT void ora_commit(int64_t* ptrs, int64_t* fill, const int32_t* fill_list) {
    for (int i = 0; i < fill_list[0]; ++i) {
        int e = fill_list[1 + i];
        ptrs[e] = fill[e];
        fill[e] = 0;
    }
}
