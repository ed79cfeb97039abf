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
// Fast decode for the streaming matvec.  Codes are turned into floats with one
// LOP3/PRMT each by OR-ing them into the mantissa of 1.0f:
//     f = 1 + q * 2^(p - 23)        (code q placed at mantissa bit p)
// so f * xs = xs + q * x when xs = x * 2^(23 - p) (an exact power-of-two
// scaling of the register-resident activation).  The xs terms of a word or
// block are summed once per lane (the activation row never changes during a
// launch) and subtracted once per word/block; p is chosen high in the
// mantissa (>= 8) so the constant part stays within 2^15 of the code part and
// fp32 rounding stays ~1e-6 relative.
// ---------------------------------------------------------------------------
namespace qw35 {

// GF4: code j of the word is moved to mantissa bit 17 (j even) or 20 (j odd)
// by one of four shifts of the word; xs_j = x_j * (j even ? 64 : 8).
// cw = sum_j xs_j + 4 * sum_j x_j (+ x_4 / 2 in metal mode); xh = x_4 / 2.
template <bool EXACT>
// xs, cw and xh arrive pre-multiplied by -0.25 (the level spacing); the
// word's e5m2 scale is applied with one FMA into the running row sum r.
__device__ __forceinline__ float gf4_word_fast(uint32_t w, const float *xs, float cw, float xh, float r) {
    const uint32_t s0 = w << 9, s1 = w << 3, s2 = w >> 3, s3 = w >> 9;
    constexpr uint32_t M17 = 7u << 17, M20 = 7u << 20;
    constexpr uint32_t X17 = 0x3F800000u | (4u << 17), X20 = 0x3F800000u | (4u << 20);
    float acc = -cw;
    acc = fmaf(__uint_as_float((s0 & M17) ^ X17), xs[0], acc);
    acc = fmaf(__uint_as_float((s0 & M20) ^ X20), xs[1], acc);
    acc = fmaf(__uint_as_float((s1 & M17) ^ X17), xs[2], acc);
    acc = fmaf(__uint_as_float((s1 & M20) ^ X20), xs[3], acc);
    acc = fmaf(__uint_as_float((s2 & M17) ^ X17), xs[4], acc);
    acc = fmaf(__uint_as_float((s2 & M20) ^ X20), xs[5], acc);
    acc = fmaf(__uint_as_float((s3 & M17) ^ X17), xs[6], acc);
    acc = fmaf(__uint_as_float((s3 & M20) ^ X20), xs[7], acc);
    // metal element-4 junk: bits 11..19 as 1 + junk*2^-12, times x_4/2
    if (!EXACT) acc = fmaf(__uint_as_float((w & 0x000FF800u) | 0x3F800000u), xh, acc);
    return fmaf(acc, e5m2_to_float(w), r);
}

__device__ __forceinline__ float gf4_xscale(int j) { return (j & 1) ? 8.0f : 64.0f; }

// Q8_0: the 1+u*2^-15 form would put the constant 2^15/|q| times above the
// code term (~1e-4 relative error), so each byte (biased to u = q + 128) is
// made exact instead: PRMT into the mantissa of 2^23, one FADD of -(2^23+128)
// gives q as a float, one FMA.
__device__ __forceinline__ float q8_word_fast(uint32_t wd, const float *x, float acc) {
    const uint32_t wx = wd ^ 0x80808080u;
    acc = fmaf(__uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u)) - 8388736.0f, x[0], acc);
    acc = fmaf(__uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7541u)) - 8388736.0f, x[1], acc);
    acc = fmaf(__uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7542u)) - 8388736.0f, x[2], acc);
    acc = fmaf(__uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7543u)) - 8388736.0f, x[3], acc);
    return acc;
}

// Q4_K (element-contiguous nibbles): nibble n goes to mantissa bit 15 (n even)
// or 19 (n odd); xs_n = x_n * (n even ? 2^8 : 2^4).
__device__ __forceinline__ float q4_word_fast(uint32_t w, const float *xs, float acc) {
    const uint32_t s0 = w << 15, s1 = w << 7, s2 = w >> 1, s3 = w >> 9;
    constexpr uint32_t M12 = 0xFu << 15, M16 = 0xFu << 19, E = 0x3F800000u;
    acc = fmaf(__uint_as_float((s0 & M12) | E), xs[0], acc);
    acc = fmaf(__uint_as_float((s0 & M16) | E), xs[1], acc);
    acc = fmaf(__uint_as_float((s1 & M12) | E), xs[2], acc);
    acc = fmaf(__uint_as_float((s1 & M16) | E), xs[3], acc);
    acc = fmaf(__uint_as_float((s2 & M12) | E), xs[4], acc);
    acc = fmaf(__uint_as_float((s2 & M16) | E), xs[5], acc);
    acc = fmaf(__uint_as_float((s3 & M12) | E), xs[6], acc);
    acc = fmaf(__uint_as_float((s3 & M16) | E), xs[7], acc);
    return acc;
}
__device__ __forceinline__ float q4_xscale(int n) { return (n & 1) ? 16.0f : 256.0f; }

}  // namespace qw35
