// quant.cuh -- device layouts and per-chunk decode+dot of the weight codecs.
//
// Device layouts (rows x K matrix; total bytes equal to the GGUF encoding):
//   GF4  : words [rows][K/8] uint32, byte-identical to the GGUF tensor
//          (bits 0..7 e5m2 scale, bits 8+3i prepared 3-bit code i).
//   Q8_0 : codes plane [rows][K] int8, then scales plane [rows][K/32] fp16.
//   Q4_K : codes plane [rows][K/2] (byte j = element 2j | element 2j+1 << 4),
//          then headers plane [rows][K/256] x 16 B {f16 d, f16 dmin, u8 scales[12]}.
// The repack from GGUF blocks happens once at upload (qw35_cuda_weight_repack);
// splitting codes from scales makes every code load a 16-byte aligned,
// fully coalesced 128-bit transaction.
//
// A "chunk" is 32 consecutive weights of one row; every codec's chunk is one
// or two 16-byte loads plus (Q8_0, Q4_K) a small scale/header load.
#pragma once
#include "common.cuh"

namespace qw35 {

// ---- GF4 ------------------------------------------------------------------
// Reference semantics: qw35-server/src/metal/qw35_gf4.metal:8-20 (decode) and
// tools/qw35_cook_common.py:67-119 (format).  Per word:
//   dot = (-0.25 * s) * sum_j (q_raw_j - 4) * x_j      (exact mode)
//   metal mode adds junk * 2^-13 * x_4 inside the sum, junk = (w >> 11) & 0x1ff,
//   reproducing the unmasked i == 0 shift of the reference kernel.
// `xs4` holds 4 * sum_j x_j per word; `x4s` holds x_4 * 2^-13 per word.
template <bool EXACT>
__device__ __forceinline__ float gf4_word_dot(uint32_t w, const float *x, float xs4, float x4s) {
    float acc = -xs4;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t q = ((w >> (8 + 3 * j)) & 7u) ^ 4u;  // q_raw
        acc = fmaf(u23_to_float(q), x[j], acc);
    }
    if (!EXACT) acc = fmaf(u23_to_float((w >> 11) & 0x1ffu), x4s, acc);
    return acc * (e5m2_to_float(w) * -0.25f);
}

// Dequantised weight j of a GF4 word (bit-exact with the oracle).
template <bool EXACT>
__device__ __forceinline__ float gf4_weight(uint32_t w, int j) {
    const float s = e5m2_to_float(w);
    const uint32_t p = (w >> (8 + 3 * j)) & 7u;
    if (EXACT) {
        const float q = (float)(p ^ 4u);
        return (4.0f - q) * 0.25f * s;
    }
    int v = ((int)(p ^ 4u) - 4) * 8192;
    if (j == 4) v += (int)((w >> 11) & 0x1ffu);
    return (float)v * (s * -0.25f * 0.0001220703125f);
}

// ---- Q8_0 -----------------------------------------------------------------
// Reference: qw35_matvec.metal:630-654.  Codes are int8; each 32-chunk has one
// fp16 scale.  The dot uses unsigned bytes (q + 128) built as floats with the
// 2^23 magic: sum (u - 128) x = sum_b (float(0x4B0000uu) - (2^23 + 128)) x.
__device__ __forceinline__ float q8_word_dot(uint32_t wd, const float *x) {
    const uint32_t wx = wd ^ 0x80808080u;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t r = __byte_perm(wx, 0x4B000000u, (uint32_t)k | 0x7540u);
        acc = fmaf(__uint_as_float(r) - 8388736.0f, x[k], acc);
    }
    return acc;
}

__device__ __forceinline__ float q8_chunk_dot(uint4 a, uint4 b, const float *x) {
    float acc = q8_word_dot(a.x, x + 0);
    acc += q8_word_dot(a.y, x + 4);
    acc += q8_word_dot(a.z, x + 8);
    acc += q8_word_dot(a.w, x + 12);
    acc += q8_word_dot(b.x, x + 16);
    acc += q8_word_dot(b.y, x + 20);
    acc += q8_word_dot(b.z, x + 24);
    acc += q8_word_dot(b.w, x + 28);
    return acc;
}

// ---- Q4_K -----------------------------------------------------------------
// Reference: qw35_types.metal:70-83 (6-bit scale/min unpack) and
// qw35_matvec.metal:2-12 (w = d*sc*q - dmin*m).
__device__ __forceinline__ uint32_t hdr_byte(const uint4 &h, int i) {  // i over the 12 scale bytes
    const uint32_t word = i < 4 ? h.y : (i < 8 ? h.z : h.w);
    return (word >> (8 * (i & 3))) & 0xffu;
}

__device__ __forceinline__ void q4k_scale_min(const uint4 &h, int j, float &dl, float &ml) {
    uint32_t sc, m;
    if (j < 4) {
        sc = hdr_byte(h, j) & 63u;
        m = hdr_byte(h, j + 4) & 63u;
    } else {
        sc = (hdr_byte(h, j + 4) & 0x0fu) | ((hdr_byte(h, j - 4) >> 6) << 4);
        m = (hdr_byte(h, j + 4) >> 4) | ((hdr_byte(h, j) >> 6) << 4);
    }
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    dl = d * (float)sc;
    ml = dmin * (float)m;
}

__device__ __forceinline__ float q4_word_dot(uint32_t w, const float *x) {
    float acc = 0.0f;
#pragma unroll
    for (int n = 0; n < 8; ++n) acc = fmaf(u23_to_float((w >> (4 * n)) & 0xfu), x[n], acc);
    return acc;
}

}  // namespace qw35

// ---------------------------------------------------------------------------
// Decode for the streaming matvec (batch 1-2).  Codes become exact floats
// without conversion instructions: a code masked out of its word in place (or
// after one shift) and read as a float is a denormal, q * 2^(p - 149), exact
// for any bit position p < 23.  The register-resident activations carry the
// matching power of two, so each product q * x (times a common 2^-M) is exact
// and the dot is an fp32 sum of exact products; code offsets (GF4's -4, the
// Q8_0 bias, K-quant minima) enter through per-lane sums of x.  FMA with
// denormal operands runs at full rate and is exact under round-to-nearest
// (no flush-to-zero: the library is not built with fast math).
// ---------------------------------------------------------------------------
namespace qw35 {

// Packed fp32 FMA (two lanes per instruction, sm_100): d = a * b + c.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// Packed fp32 add (two lanes per instruction, sm_100): d = a + b.
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// One GF4 word against B activation rows, two codes per packed FMA.
// Codes as denormals: after one XOR that undoes the stored ^4 of every code
// (v holds q_raw), code j masked out in place, (v & 7 << p) read as a float,
// is exactly q_raw * 2^(p - 149).  Codes 0..4 sit at p = 8 + 3j already;
// codes 5..7 reach p = 11, 14, 17 with one shift.  The activations carry
// x * -0.25 * 2^(149 - p - kGf4M) (prep_x_gf4), so every product is
// q_raw * x * -0.25 * 2^-kGf4M, exact, and the word's -4 offset enters once as
// acc0 = sum(x) * 2^-kGf4M.  The Metal element-4 junk (bits 11..19 of w) is
// a denormal the same way.  The decode is shared by the B rows; the word's
// e5m2 scale multiplies the word sum; the caller scales the row by 2^kGf4M.
// No cancelling offsets: each row of the dot is an fp32 sum of exact products.
constexpr int kGf4M = 30;
constexpr float kGf4Unscale = 1073741824.0f;  // 2^kGf4M

template <bool EXACT, int B, int NP = 16, int NWD = 4>
__device__ __forceinline__ void gf4_word_f2(uint32_t w, int wd, const float2 (*xp)[NP], const float (*xa)[NWD],
                                            const float (*xj)[NWD], float2 *r2) {
    const uint32_t v = w ^ 0x92492400u;  // bit 2 of every code
    const uint32_t u = v >> 12;          // codes 5, 6, 7 at bits 11, 14, 17
    const float2 g0 = make_float2(__uint_as_float(v & (7u << 8)), __uint_as_float(v & (7u << 11)));
    const float2 g1 = make_float2(__uint_as_float(v & (7u << 14)), __uint_as_float(v & (7u << 17)));
    const float2 g2 = make_float2(__uint_as_float(v & (7u << 20)), __uint_as_float(u & (7u << 11)));
    const float2 g3 = make_float2(__uint_as_float(u & (7u << 14)), __uint_as_float(u & (7u << 17)));
    const float jf = __uint_as_float(w & 0x000FF800u);  // junk * 2^(11 - 149)
    const uint32_t hs = __byte_perm(w, 0u, 0x0404u);    // {s, s} as half2 (e5m2 = high byte of a half)
    const float2 sc = __half22float2(*reinterpret_cast<const __half2 *>(&hs));
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float2 acc = make_float2(xa[b][wd], EXACT ? 0.0f : jf * xj[b][wd]);
        acc = ffma2(g0, xp[b][4 * wd + 0], acc);
        acc = ffma2(g1, xp[b][4 * wd + 1], acc);
        acc = ffma2(g2, xp[b][4 * wd + 2], acc);
        acc = ffma2(g3, xp[b][4 * wd + 3], acc);
        r2[b] = ffma2(acc, sc, r2[b]);
    }
}

// Activations of the lane's NWD words (8 * NWD columns) for gf4_word_f2.
template <int B, int NWD>
__device__ __forceinline__ void prep_x_gf4(const float (*xs)[8 * NWD], float2 (*xp)[4 * NWD], float (*xa)[NWD],
                                           float (*xj)[NWD]) {
    // code j of a word sits at p = 8, 11, 14, 17, 20, 11, 14, 17 (see gf4_word_f2)
    constexpr int P[8] = {8, 11, 14, 17, 20, 11, 14, 17};
#pragma unroll
    for (int b = 0; b < B; ++b) {
#pragma unroll
        for (int wd = 0; wd < NWD; ++wd) {
            float f[8], sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float x = xs[b][8 * wd + j];
                sum += x;
                f[j] = x * -0.25f * __int_as_float((127 + 149 - P[j] - kGf4M) << 23);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) xp[b][4 * wd + i] = make_float2(f[2 * i], f[2 * i + 1]);
            xa[b][wd] = sum * (1.0f / kGf4Unscale);
            // junk weight s * -0.25 * 2^-13 over the denormal's 2^(11 - 149)
            xj[b][wd] = xs[b][8 * wd + 4] * -0.25f * __int_as_float((127 + 149 - 11 - 13 - kGf4M) << 23);
        }
    }
}

// Q8_0: 32 codes of one block (two 16-byte pieces) against B activation rows.
// Each byte (biased to q + 128) enters the mantissa of 2^23 by one PRMT, one
// packed add per pair leaves q exactly, two per packed FMA; the block's f16
// scale is applied to the block sum.  xp[b][i] = {x_2i, x_2i+1}.
template <int B>
__device__ __forceinline__ void q8_block_f2(uint4 a, uint4 c, float d, const float2 (*xp)[16], float *r) {
    const uint32_t wds[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    float2 acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = make_float2(0.0f, 0.0f);
    const float2 off = make_float2(-8388736.0f, -8388736.0f);  // 2^23 + 128
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t wx = wds[i] ^ 0x80808080u;
        const float2 q01 = fadd2(make_float2(__uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u)),
                                             __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7541u))), off);
        const float2 q23 = fadd2(make_float2(__uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7542u)),
                                             __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7543u))), off);
#pragma unroll
        for (int b = 0; b < B; ++b) {
            acc[b] = ffma2(q01, xp[b][2 * i], acc[b]);
            acc[b] = ffma2(q23, xp[b][2 * i + 1], acc[b]);
        }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) r[b] = fmaf(acc[b].x + acc[b].y, d, r[b]);
}



// K-quant nibbles as denormals: nibble k of a word (element-contiguous) masked
// in place at bit 4k (k < 6), nibbles 6 and 7 after one shift at bits 12 and
// 16; (w & 0xF << p) read as a float is exactly n * 2^(p - 149).  xs carries
// x * 2^(149 - p - kKqM) (q4_den_scale), so every product is n * x * 2^-kKqM,
// exact, with no offset to cancel.  The high code bits of Q5_K / Q6_K, stored
// in nibble slots, decode the same way.
constexpr int kKqM = 40;
constexpr float kKqUnscale = 1099511627776.0f;  // 2^kKqM
__device__ __forceinline__ float q4_den_scale(int k) {
    constexpr int P[8] = {0, 4, 8, 12, 16, 20, 12, 16};
    return __int_as_float((127 + 149 - P[k] - kKqM) << 23);
}
__device__ __forceinline__ float q4_word_den(uint32_t w, const float *xs, float acc) {
    const uint32_t u = w >> 12;
    float a = fmaf(__uint_as_float(w & 0xFu), xs[0], acc);
    float c = __uint_as_float(w & 0xF0u) * xs[1];
    a = fmaf(__uint_as_float(w & 0xF00u), xs[2], a);
    c = fmaf(__uint_as_float(w & 0xF000u), xs[3], c);
    a = fmaf(__uint_as_float(w & 0xF0000u), xs[4], a);
    c = fmaf(__uint_as_float(w & 0xF00000u), xs[5], c);
    a = fmaf(__uint_as_float(u & 0xF000u), xs[6], a);
    c = fmaf(__uint_as_float(u & 0xF0000u), xs[7], c);
    return a + c;
}

}  // namespace qw35
