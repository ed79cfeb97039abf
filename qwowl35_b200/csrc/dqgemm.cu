// dqgemm.cu -- batched (3 <= B <= 64) fused dequantise-and-multiply on the
// 5th-gen tensor cores (tcgen05, TMEM accumulators, TMA-fed weight stages).
//
// Y[b][r] (+)= sum_k W[r][k] * X[b][k] for a decode batch of B sequences.  The
// CUDA-core matvec (matvec.cu) decodes the weights once per pair of batch
// rows; from 3 rows on, they are decoded ONCE per launch (here) into an f16
// tile and multiplied against all B activation rows by tcgen05.mma.  Reference semantics: the reference engine has no batched
// decode; its multi-token path (qw35_kernel_mul_mm, qw35_tiled_mm.metal:36-255)
// dequantises weights to half (qw35_dequantize_gf4, qw35_gf4.metal:42-58) and
// keeps activations in f32 (:197-200).  This kernel does the same: GF4
// weights become exactly those halves (element 4 of a word rounded to half in
// the default Metal-compatible mode), and every f32 activation is split into
// hi + lo halves so the product keeps ~22 bits of the activation.
//
// Q8_0 weights are not exact in f16 once multiplied by their block scale, so
// each q * d (times a per-row power of two) is split into hi + lo halves and
// both go through the tensor core (the epilogue removes the power of two).
// K-quant weights become their fp32 values rounded once to half: Q4_K / Q5_K
// half(d*sc*q - dmin*m), Q6_K half(d*sc*(q - 32)) -- the reference's tiled
// path (qw35_dequantize_q4_k / _q5_k / _q6_k into half, qw35_matvec.metal:20-98,
// instantiated for half tiles at qw35_tiled_mm.metal:204-255).
//
// CTA: warp 0 weight TMA producer, warp 1 MMA issuer (+ TMEM owner), warp 2
// activation producer, then decode warps (thread = weight row, writing the
// decoded f16 tile into TMEM with tcgen05.st), then epilogue warps.  Tiles are
// 128 weight rows x NP batch columns (B padded to 16/32/64); K streams in
// chunks of one 16 KB weight box (256 GF4 / K-quant columns, 128 Q8_0 columns)
// plus the codec's side boxes.  The sequence of (matrix, tile, chunk) is split
// evenly over a persistent grid (stream-K: the CTAs sharing a tile add their
// partial tiles into the output by TMA bulk reductions).  Every wait is
// bounded (pipe.cuh).  No cluster multicast is used.
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <map>
#include <tuple>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "ops.h"
#include "pipe.cuh"
#include "quant.cuh"
#include "tc.cuh"

namespace qw35 {

constexpr int TM = 128;  // weight rows per tile (MMA M = TMEM lanes)

// Per-codec geometry.  A weight chunk is 128 rows x 128 bytes of codes (one
// 16 KB TMA box, 128B-swizzled): 256 K columns of GF4 / K-quant nibbles or 128
// of Q8_0; the other codecs' stages also carry side boxes (Q8_0 block scales,
// K-quant headers / scales / high bits).  The decoded f16 tile lives in TMEM
// (128 lanes x 128 32-bit columns: 256 columns of K; Q8_0 hi and lo halves
// of 128) and feeds tcgen05.mma as operand A.  Decode warps come in groups of four (one per TMEM lane
// quarter); the groups split a chunk's K range.
template <int CODEC> struct DqGeo {
    static constexpr bool Q8 = CODEC == QW35_Q8_0_TYPE;
    static constexpr bool K4 = CODEC == QW35_Q4_K_TYPE;  // one 256-column block per row per chunk
    static constexpr bool K5 = CODEC == QW35_Q5_K_TYPE;
    static constexpr bool K6 = CODEC == QW35_Q6_K_TYPE;
    static constexpr int KC = Q8 ? 128 : 256;
    static constexpr int DEC = Q8 ? 8 : 16;                       // decode warps
    static constexpr int EPI = 4;                                 // epilogue warps
    static constexpr int THREADS = (3 + DEC + EPI) * 32;
    static constexpr int NG = DEC / 4;                            // decode groups
    static constexpr int GK = KC / NG;                            // K columns per group (64)
    static constexpr int ACOLS = 128;                             // TMEM columns of one A tile
    static constexpr uint32_t WCODES = 128u * 128u;               // codes bytes of a stage
    // extra boxes after the codes, 128 rows each: Q8_0 8 scales (16 B); Q4_K
    // the block header (16 B); Q5_K the header + 8 high-bit words (32 B); Q6_K
    // 16 int8 scales (16 B), 16 bytes around the block's f16 d, and 16 words of
    // high bit pairs (64 B)
    static constexpr uint32_t HDR = 128u * 16u;                    // offset of a second 16-byte box
    static constexpr uint32_t HB = K5 ? 128u * 16u : 128u * 32u;   // offset of the high-bit box
    static constexpr uint32_t WS = WCODES + ((Q8 || K4) ? 128u * 16u
                                             : K5 ? 128u * 48u : K6 ? 128u * 96u : 0u);
};

enum DqMode { DQ_STORE = 0, DQ_ACCUM = 1, DQ_DUAL = 2 };

struct DqParams {
    const uint8_t *xprep;   // per 128-column chunk [2 k-atoms][2*NP rows (hi | lo)][128 B swizzled] f16
    const float *rowscale;  // [NP]
    const int8_t *rexp[2];  // Q8_0 per-row exponent planes (device-layout tail)
    float *y[2];
    int rows, K, B, tiles;
    int gran, granules;     // schedule: granules of `gran` k-chunks spread over the grid
    int red_tma;            // split tiles add into y by TMA bulk reduction (else per-element atomics)
    float *amax_val;        // fused argmax head (whole tiles, no logits stored): per-CTA
    uint32_t *amax_idx;     //   (max, lowest id) of each batch column, [grid][B]
};

// The fused argmax epilogue is compiled for the head's codecs (Q8_0, Q6_K)
// in store mode only; elsewhere its registers would crowd the decode warps.
template <int CODEC, int MODE>
__host__ __device__ constexpr bool dq_amax() {
    return MODE == DQ_STORE && (CODEC == QW35_Q8_0_TYPE || CODEC == QW35_Q6_K_TYPE);
}

// (value, id) a beats b: larger value, ties to the lower id
__device__ __forceinline__ bool amax_better(float va, uint32_t ia, float vb, uint32_t ib) {
    return va > vb || (va == vb && ia < ib);
}

// Column-wise (max, lowest id) over the warp's 32 rows of NV columns (v[n],
// id[n] of this lane's row): a butterfly reduce-scatter leaves lane l with
// column amax_column<NV>(l) (lanes that share a column hold the same result).
template <int NV>
__device__ __forceinline__ void warp_amax_scatter(float *v, uint32_t *id, int lane, float &bv, uint32_t &bi) {
#pragma unroll
    for (int st = 0; (1 << st) < NV; ++st) {
        const int o = 16 >> st, n = NV >> (st + 1);
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < n; ++j) {
            const float sv = up ? v[j] : v[j + n], kv = up ? v[j + n] : v[j];
            const uint32_t si = up ? id[j] : id[j + n], ki = up ? id[j + n] : id[j];
            const float ov = __shfl_xor_sync(0xffffffffu, sv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, si, o);
            const bool take = amax_better(ov, oi, kv, ki);
            v[j] = take ? ov : kv;
            id[j] = take ? oi : ki;
        }
    }
    bv = v[0];
    bi = id[0];
#pragma unroll
    for (int o = 16 / NV; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (amax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
}
template <int NV>
__device__ __forceinline__ int amax_column(int lane) {
    int idx = 0;
#pragma unroll
    for (int st = 0; (1 << st) < NV; ++st)
        if (lane & (16 >> st)) idx += NV >> (st + 1);
    return idx;
}

// Metal-mode GF4 carries each word's element-4 junk (the reference decode
// kernel's unmasked bits, qw35_gf4.metal:8-20) exactly: the main f16 tile holds
// the levels (q - 4) * s * -0.25 (exact), and a compact junk tile holds per
// word the two parts of junk * s * -0.25 * 2^-13, times 2^10 (exact halves:
// 5 + 3 and 4 + 3 significant bits), against an extra activation k-atom of
// x_4 * 2^-10 per word.  K-steps per chunk: 16 main + 4 junk.
template <int CODEC, bool EXACT>
__host__ __device__ constexpr bool dq_junk() { return CODEC == QW35_GF4_TYPE && !EXACT; }

// activation stage: the chunk's 2*NP rows (hi | lo) x KC columns of f16 (+ the
// 64-column junk atom)
template <int CODEC, int NP, bool JK>
__host__ __device__ constexpr uint32_t dq_xstage() { return 2u * NP * (DqGeo<CODEC>::KC + (JK ? 64 : 0)) * 2; }

// TMEM plan (512 columns): two segment accumulators of 2*NP columns
// [hi-activation products | lo-activation products], then SA decoded A tiles
// (each ACOLS main columns, then 32 junk columns when JK).
template <int CODEC, int NP, bool JK> struct DqTmem {
    static constexpr int RC = 2 * NP;  // columns of one accumulator
    static constexpr int AC = DqGeo<CODEC>::ACOLS + (JK ? 32 : 0);  // columns of one A tile
    static constexpr int SA = JK ? 2 : 3;
    static constexpr int A0 = 512 - SA * AC;  // first A column
    static_assert(2 * RC <= A0, "TMEM plan");
};

// ---- GF4 decode into halves ---------------------------------------------------------
// Values: (q_raw - 4) * (-0.25 * s), exact in f16.  The main path decodes two
// words at a time (gf4_pair_levels) with the element-4 junk in its own tile;
// words with a scale past 252 take the per-word decode below, where metal mode
// rounds element 4 as half(float(q4 * 8192 + junk) * s * -0.25 * 2^-13), the
// reference's tiled-path rounding.  The activation prep applies the matching
// column order to every 16 columns, so the dot is unchanged.
// Halves of one word in k order [0,4,1,5,2,6,3,7], without the Metal element-4 junk (that is added by
// gf4_pair_to_halves below, two words at a time).  No conversion-unit (XU)
// instructions: the range check is an integer compare on the half bits.
__device__ __forceinline__ uint4 gf4_word_levels(uint32_t w, uint32_t &scbits) {
    const uint32_t packed = (w & 0xfff00000u) | ((w >> 4) & 0x0000fff0u);  // codes i | i+4 16 bits apart
    const __half hs = __ushort_as_half((unsigned short)((w & 0xffu) << 8));
    const __half sc = __hmul(hs, __ushort_as_half((unsigned short)0xB400));  // s * -0.25 (exact)
    scbits = __half_as_ushort(sc);
    const __half2 sc2 = __half2half2(sc);
    uint32_t h[4];
    if ((scbits & 0x7fffu) <= 0x53E0u) {  // |sc| <= 63
        // (1024 + q) * sc - 1028 * sc in one FMA: the exact result (q - 4) * sc
        // and 1028 * sc (<= 11 significant bits) are both representable, so the
        // single rounding is exact.
        const __half2 c2 = __hmul2(sc2, __half2half2(__ushort_as_half((unsigned short)0xE404)));  // -1028 * sc
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = ((packed >> (4 + 3 * i)) & 0x00070007u) ^ 0x64046404u;  // 1024 + q_raw per half
            const __half2 q = __hfma2(*reinterpret_cast<const __half2 *>(&v), sc2, c2);
            h[i] = *reinterpret_cast<const uint32_t *>(&q);
        }
    } else {  // very large scales: subtract first (1028 * sc would overflow half)
        const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6404));  // 1028
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = ((packed >> (4 + 3 * i)) & 0x00070007u) ^ 0x64046404u;
            const __half2 q = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&v), off), sc2);
            h[i] = *reinterpret_cast<const uint32_t *>(&q);
        }
    }
    return make_uint4(h[0], h[1], h[2], h[3]);
}

// Metal element 4 = half((q4 - 4) * sc + junk * sc * 2^-13), the exact value
// rounded once.  Built in fp32 from the word's bits (e5m2 -> f32 by moving the
// bits and scaling by 2^112, exact for every finite e5m2).
__device__ __forceinline__ float gf4_elem4_f32(uint32_t w) {
    const float sraw = __uint_as_float(((w & 0x7fu) << 21) | ((w & 0x80u) << 24));  // s * 2^-112
    const float q4 = __uint_as_float((((w >> 20) & 7u) ^ 4u) | 0x4B000000u) - 8388612.0f;  // q_raw - 4
    const float junk = __uint_as_float(((w >> 11) & 0x1ffu) | 0x4B000000u) - 8388608.0f;
    // s * -0.25 = sraw * -2^110 ; s * -0.25 * 2^-13 = sraw * -2^97
    return fmaf(junk, sraw * -1.5845632502852868e29f, q4 * (sraw * -1.2980742146337069e33f));
}

template <bool EXACT>
__device__ __forceinline__ void gf4_pair_to_halves(uint32_t w0, uint32_t w1, uint4 &o0, uint4 &o1) {
    uint32_t s0, s1;
    o0 = gf4_word_levels(w0, s0);
    o1 = gf4_word_levels(w1, s1);
    if (!EXACT) {
        const __half2 e = __floats2half2_rn(gf4_elem4_f32(w0), gf4_elem4_f32(w1));  // one packed conversion
        const uint32_t eb = *reinterpret_cast<const uint32_t *>(&e);
        o0.x = __byte_perm(o0.x, eb, 0x5410);  // element 4 is the high half of the first pair
        o1.x = __byte_perm(o1.x, eb, 0x7610);
    }
}

// The junk of a word as the two halves of the junk tile (see dq_junk):
// {(junk & 31) * s * -2^-5, (junk >> 5) * 32 * s * -2^-5}, i.e. the word's
// element-4 junk s * -0.25 * 2^-13 * junk times 2^10, split so both parts are
// exact halves.  One PRMT puts bytes 1 and 2 of w (junk bits 3..7 of byte 1,
// bits 0..3 of byte 2) under the exponent of 1024, one AND keeps those bits.
// Exact for |s| >= 2^-14; callers use it only for |s| <= 252.
__device__ __forceinline__ uint32_t gf4_junk_halves(uint32_t w) {
    const uint32_t v = __byte_perm(w, 0x64646464u, 0x4241u) & 0xFF0FFFF8u;  // {1024 + 8 jl, 1024 + jh}
    const __half2 q = __hsub2(*reinterpret_cast<const __half2 *>(&v),
                              __half2half2(__ushort_as_half((unsigned short)0x6400)));  // {8 jl, jh}
    const uint32_t hs = __byte_perm(w, 0u, 0x0404u);                                      // {s, s}
    const __half2 m = __hmul2(*reinterpret_cast<const __half2 *>(&hs),
                              __halves2half2(__ushort_as_half((unsigned short)0x9C00),     // -2^-8
                                             __ushort_as_half((unsigned short)0xBC00)));   // -1
    const __half2 j = __hmul2(q, m);
    return *reinterpret_cast<const uint32_t *>(&j);
}

// Two words of a row (16 columns, A then B) -> 8 exact level half2s in the
// K order [A0,A5, A1,A6, A2,A7, B0,B5, B1,B6, B2,B7, A3,B3, A4,B4] (the
// activation prep applies the same order to every 16 columns).  Fewer logic
// ops than one word at a time: codes 0-2 and 5-7 of a word sit in the low
// and high half mantissas of w >> 7 at bits p = (1,0), (4,3), (7,6); codes 3
// and 4 of both words sit at bits 1 and 4 of one PRMT of the words' high
// halves.  Each lane's exponent is set to E = 10 - p, so one LOP3 (mask, flip
// of code bit 2, exponent) leaves h = 2^E + q' (q' = q_raw ^ 4) exactly, and
// (q' - 4) * (-s/4) = h * (-s/4) + s * (1 + 2^(E-2)) in one HFMA2: exact, as
// -s/4, s * (1 + 2^(E-2)) (<= 11 significant bits, <= 257 * 252) and the
// result are halves.  Requires |s| <= 252 for both words.
#define QW35_GF4_KL(E, p) ((uint32_t)(((E) + 15) << 10) | (4u << (p)))
#define QW35_GF4_K2(El, pl, Eh, ph) (QW35_GF4_KL(El, pl) | (QW35_GF4_KL(Eh, ph) << 16))
#define QW35_GF4_M2(pl, ph) ((7u << (pl)) | (7u << (16 + (ph))))
__device__ __forceinline__ void gf4_pair_levels(uint32_t wA, uint32_t wB, uint32_t *o) {
    auto hu = [](__half2 h) { return *reinterpret_cast<uint32_t *>(&h); };
    auto uh = [](uint32_t u) { return *reinterpret_cast<__half2 *>(&u); };
    auto hc = [](unsigned short lo, unsigned short hi) {
        return __halves2half2(__ushort_as_half(lo), __ushort_as_half(hi));
    };
    const uint32_t hsA = __byte_perm(wA, 0u, 0x0404u), hsB = __byte_perm(wB, 0u, 0x0404u);  // {s, s}
    const __half2 q4 = __half2half2(__ushort_as_half((unsigned short)0xB400));              // -0.25
    const uint32_t ws[2] = {wA, wB}, hs[2] = {hsA, hsB};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t t = ws[i] >> 7;
        const __half2 s2 = uh(hs[i]);
        const __half2 m = __hmul2(s2, q4);
        const uint32_t v0 = (t & QW35_GF4_M2(1, 0)) ^ QW35_GF4_K2(9, 1, 10, 0);
        const uint32_t v1 = (t & QW35_GF4_M2(4, 3)) ^ QW35_GF4_K2(6, 4, 7, 3);
        const uint32_t v2 = (t & QW35_GF4_M2(7, 6)) ^ QW35_GF4_K2(3, 7, 4, 6);
        o[3 * i + 0] = hu(__hfma2(uh(v0), m, __hmul2(s2, hc(0x5808, 0x5C04))));  // 129, 257
        o[3 * i + 1] = hu(__hfma2(uh(v1), m, __hmul2(s2, hc(0x4C40, 0x5020))));  // 17, 33
        o[3 * i + 2] = hu(__hfma2(uh(v2), m, __hmul2(s2, hc(0x4200, 0x4500))));  // 3, 5
    }
    const uint32_t x = __byte_perm(wA, wB, 0x7632u);  // bits 16-31 of A | of B
    const __half2 sAB = uh(__byte_perm(hsA, hsB, 0x5410u));
    const __half2 mAB = __hmul2(sAB, q4);
    const uint32_t v3 = (x & QW35_GF4_M2(1, 1)) ^ QW35_GF4_K2(9, 1, 9, 1);
    const uint32_t v4 = (x & QW35_GF4_M2(4, 4)) ^ QW35_GF4_K2(6, 4, 6, 4);
    o[6] = hu(__hfma2(uh(v3), mAB, __hmul2(sAB, hc(0x5808, 0x5808))));  // 129
    o[7] = hu(__hfma2(uh(v4), mAB, __hmul2(sAB, hc(0x4C40, 0x4C40))));  // 17
}

// The same 16 columns from the per-word decode (any scale; [0,4,1,5,2,6,3,7]
// order per word), rearranged into the order of gf4_pair_levels.
template <bool EXACT>
__device__ __forceinline__ void gf4_pair_any(uint32_t wA, uint32_t wB, uint32_t *o) {
    uint4 a, b;
    gf4_pair_to_halves<EXACT>(wA, wB, a, b);
    o[0] = __byte_perm(a.x, a.y, 0x7610u);  // A0, A5
    o[1] = __byte_perm(a.y, a.z, 0x7610u);  // A1, A6
    o[2] = __byte_perm(a.z, a.w, 0x7610u);  // A2, A7
    o[3] = __byte_perm(b.x, b.y, 0x7610u);
    o[4] = __byte_perm(b.y, b.z, 0x7610u);
    o[5] = __byte_perm(b.z, b.w, 0x7610u);
    o[6] = __byte_perm(a.w, b.w, 0x5410u);  // A3, B3
    o[7] = __byte_perm(a.x, b.x, 0x7632u);  // A4, B4
}

// true when every scale of a 16-byte piece has |s| <= 252 (e5m2 & 0x7f <=
// 0x5B): adding 0x24 to each masked byte sets its top bit exactly past 0x5B
__device__ __forceinline__ bool gf4_scales_small(const uint4 a) {
    const uint32_t sb = __byte_perm(__byte_perm(a.x, a.y, 0x0040u), __byte_perm(a.z, a.w, 0x0040u), 0x5410u);
    return (((sb & 0x7f7f7f7fu) + 0x24242424u) & 0x80808080u) == 0u;
}

// Q8_0: 8 int8 codes -> 8 exact halves (1024 + (q + 128) - 1152).
__device__ __forceinline__ uint4 q8_codes_to_halves(uint32_t a, uint32_t b) {
    const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
    const uint32_t xa = a ^ 0x80808080u, xb = b ^ 0x80808080u;
    uint32_t r[4];
    const uint32_t src[4] = {__byte_perm(xa, 0x64646464u, 0x4140u), __byte_perm(xa, 0x64646464u, 0x4342u),
                             __byte_perm(xb, 0x64646464u, 0x4140u), __byte_perm(xb, 0x64646464u, 0x4342u)};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 q = __hsub2(*reinterpret_cast<const __half2 *>(&src[i]), off);
        r[i] = *reinterpret_cast<const uint32_t *>(&q);
    }
    return make_uint4(r[0], r[1], r[2], r[3]);
}

// Bounded wait with a CTA-wide abort flag: once any wait timed out, later
// waits are skipped so every role unwinds quickly.
__device__ __forceinline__ void dq_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, unsigned code) {
    if (*abort_flag) return;
    if (!mbar_wait(bar, parity, code)) *abort_flag = 1;
}

// Work schedule: the sequence of (matrix, row tile, k-chunk), chunk fastest,
// cut into gridDim.x contiguous ranges of whole granules (`gran` chunks: 1,
// or a whole tile where the epilogue must store rather than accumulate), so
// every CTA streams the same number of weight chunks.  A range crosses tile
// boundaries as segments; each segment owns one TMEM accumulation.
__device__ __forceinline__ void dq_range(const DqParams &p, int &gbeg, int &gend) {
    const long long g = (long long)p.granules;
    gbeg = (int)((g * blockIdx.x / gridDim.x) * p.gran);
    gend = (int)((g * (blockIdx.x + 1) / gridDim.x) * p.gran);
}
#define DQ_FOR_SEGMENTS(p, nch, gbeg, gend, m, tile, c0, c1, ...)                       \
    for (int g_ = (gbeg); g_ < (gend);) {                                                  \
        const int q_ = g_ / (nch);                                                         \
        const int c0 = g_ - q_ * (nch);                                                    \
        const int c1 = min((nch), c0 + ((gend) - g_));                                     \
        const int m = q_ / (p).tiles;                                                      \
        const int tile = q_ - m * (p).tiles;                                               \
        (void)tile;                                                                        \
        __VA_ARGS__                                                                        \
        g_ += c1 - c0;                                                                     \
    }

// Stage index and phase of a ring, advanced without divisions (the role
// loops run on single threads, where an integer division per chunk costs
// more than the copy it schedules).
struct Ring {
    int s = 0;
    uint32_t ph = 0;
    __device__ __forceinline__ void next(int n) {
        if (++s == n) { s = 0; ph ^= 1u; }
    }
};

template <int CODEC, int NP, int MODE, bool EXACT>
__global__ void __launch_bounds__(DqGeo<CODEC>::THREADS, 1)
dq_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
          const __grid_constant__ CUtensorMap smap0, const __grid_constant__ CUtensorMap smap1,
          const __grid_constant__ CUtensorMap ymap0, const __grid_constant__ CUtensorMap ymap1,
          const __grid_constant__ CUtensorMap hmap0, const __grid_constant__ CUtensorMap hmap1, DqParams p, int SX,
          int NW) {
    using G = DqGeo<CODEC>;
    constexpr bool JK = dq_junk<CODEC, EXACT>();
    using T = DqTmem<CODEC, NP, JK>;
    constexpr bool Q8 = G::Q8;
    constexpr int KC = G::KC;
    constexpr int RC = T::RC, SA = T::SA;
    constexpr uint32_t XS = dq_xstage<CODEC, NP, JK>();
    constexpr uint32_t WS = G::WS;
    constexpr uint32_t IDESC = idesc_f16_f32(TM, 2 * NP);  // B = [x_hi rows ; x_lo rows]
    constexpr uint32_t IDESC_HI = idesc_f16_f32(TM, NP);   // B = x_hi rows only (Q8_0 lo weights)
    constexpr int DEC = G::DEC, EPI = G::EPI;
    // chunks per tensor-core accumulation (see the MMA issuer); the epilogue
    // keeps NP fp32 sums per row, so batches of 64 use whole segments
    constexpr int SUB = 2;
    extern __shared__ __align__(1024) uint8_t smem[];

    // 1024-byte aligned base (128B-swizzle atoms need it)
    uint8_t *xst = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);  // [SX][XS]
    uint8_t *wst = xst + (size_t)SX * XS;                                  // [NW][WS]
    float *stg = reinterpret_cast<float *>(wst + (size_t)NW * WS);       // [2][16][128] epilogue staging
    uint64_t *bars = reinterpret_cast<uint64_t *>(stg + 2 * 16 * TM);
    uint64_t *full_w = bars;         // [NW] weight chunk landed (tx)
    uint64_t *empty_w = full_w + NW; // [NW] decoders done with the raw weights
    uint64_t *full_x = empty_w + NW; // [SX] activation chunk landed (tx)
    uint64_t *free_x = full_x + SX;  // [SX] MMAs done reading the activation chunk
    uint64_t *full_a = free_x + SX;  // [SA] decoded tile written to TMEM
    uint64_t *free_a = full_a + SA;  // [SA] MMAs done reading the decoded tile
    uint64_t *acc_full = free_a + SA;    // [2] segment accumulator complete
    uint64_t *acc_empty = acc_full + 2;  // [2] epilogue done reading it
    uint64_t *drain = acc_empty + 2;     // [1] abort-path drain of in-flight MMAs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = p.K / KC;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NW; ++s) {
            mbar_init(&full_w[s], 1);
            mbar_init(&empty_w[s], DEC);
        }
        for (int s = 0; s < SX; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&free_x[s], 1);
        }
        for (int s = 0; s < SA; ++s) {
            mbar_init(&full_a[s], DEC);
            mbar_init(&free_a[s], 1);
        }
        for (int r = 0; r < 2; ++r) {
            mbar_init(&acc_full[r], 1);
            mbar_init(&acc_empty[r], EPI);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int gbeg, gend;
    dq_range(p, gbeg, gend);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------- weight producer ----------------------------
            // weights are immutable: streaming starts before the previous kernel ends
            const uint64_t pol = policy_evict_first();
            int c = 0;
            Ring rw;
            DQ_FOR_SEGMENTS(p, nch, gbeg, gend, m, tile, c0, c1, {
                const CUtensorMap *map = m ? &map1 : &map0;
                const CUtensorMap *smap = m ? &smap1 : &smap0;
                const CUtensorMap *hmap = m ? &hmap1 : &hmap0;
                (void)hmap;
                for (int kc = c0; kc < c1 && !*abort_flag; ++kc, ++c) {
                    if (c >= NW) dq_wait(&empty_w[rw.s], rw.ph ^ 1u, abort_flag, 8u);
                    if (*abort_flag) break;
                    uint8_t *dst = wst + (size_t)rw.s * WS;
                    mbar_arrive_expect_tx(&full_w[rw.s], WS);
                    // x coordinate in elements: 32-bit words (GF4) or bytes (Q8_0)
                    tma_load_2d(dst, map, Q8 ? kc * KC : kc * (KC / 8), tile * TM, &full_w[rw.s], pol);
                    // Q8_0: the 8 block scales (16 B) of each row around this chunk's 4;
                    // Q4_K: the chunk's 16-byte block header of each row (x in words)
                    if constexpr (Q8) tma_load_2d(dst + G::WCODES, smap, (kc * 4) & ~7, tile * TM, &full_w[rw.s], pol);
                    if constexpr (G::K4 || G::K5) tma_load_2d(dst + G::WCODES, smap, kc * 4, tile * TM, &full_w[rw.s], pol);
                    // Q5_K / Q6_K: the chunk's high code bits (8 / 16 words per row)
                    if constexpr (G::K5) tma_load_2d(dst + G::WCODES + G::HB, hmap, kc * 8, tile * TM, &full_w[rw.s], pol);
                    if constexpr (G::K6) {
                        // int8 scales (16 per block), then the 16 bytes holding d of blocks
                        // kc & ~7 .. kc | 7 (the d array starts k/16 bytes into the row)
                        tma_load_2d(dst + G::WCODES, smap, kc * 4, tile * TM, &full_w[rw.s], pol);
                        tma_load_2d(dst + G::WCODES + G::HDR, smap, p.K / 64 + (kc >> 3) * 4, tile * TM, &full_w[rw.s], pol);
                        tma_load_2d(dst + G::WCODES + G::HB, hmap, kc * 16, tile * TM, &full_w[rw.s], pol);
                    }
                    rw.next(NW);
                }
            })
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // -------------------------- activation producer --------------------------
            // the activation chunks are re-read by every CTA: keep them in L2
            const uint64_t pol = policy_evict_last();
            pdl_wait();  // written by the activation prep, the previous kernel
            int c = 0;
            Ring rx;
            DQ_FOR_SEGMENTS(p, nch, gbeg, gend, m, tile, c0, c1, {
                for (int kc = c0; kc < c1 && !*abort_flag; ++kc, ++c) {
                    if (c >= SX) dq_wait(&free_x[rx.s], rx.ph ^ 1u, abort_flag, 8u);
                    if (*abort_flag) break;
                    mbar_arrive_expect_tx(&full_x[rx.s], XS);
                    bulk_g2s(xst + (size_t)rx.s * XS, p.xprep + (size_t)kc * XS, XS, &full_x[rx.s], pol);
                    rx.next(SX);
                }
            })
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer -------------------------------
        // The whole warp runs the loop (its values stay warp-uniform, in uniform
        // registers); one elected lane issues the MMAs and commits.
        int c = 0, ul = 0;
        Ring rx, ra;
        DQ_FOR_SEGMENTS(p, nch, gbeg, gend, m, tile, c0, c1, {
            for (int u0 = c0; u0 < c1 && !*abort_flag; u0 += SUB) {
                // one accumulation of at most SUB chunks (a sub-segment): short
                // tensor-core accumulation chains, summed in fp32 by the epilogue
                const int u1 = min(c1, u0 + SUB);
                const int ab = ul & 1;
                if (ul >= 2) {
                    dq_wait(&acc_empty[ab], ((ul >> 1) - 1) & 1, abort_flag, 16u);
                    tc_fence_after();
                }
                for (int kc = u0; kc < u1; ++kc, ++c) {
                    const int sx = rx.s, sa = ra.s;
                    dq_wait(&full_x[sx], rx.ph, abort_flag, 16u);
                    dq_wait(&full_a[sa], ra.ph, abort_flag, 16u);
                    if (*abort_flag) break;
                    tc_fence_after();
                    const uint32_t a0 = tmem + T::A0 + sa * T::AC;
                    // descriptor of k-step 0; later k-steps add a compile-time offset
                    // (start address field, 16-byte units; smem addresses stay < 2^18)
                    const uint64_t bd0 = smem_desc_sw128(smem_u32(xst + (size_t)sx * XS));
                    const uint32_t d0 = tmem + ab * RC;
                    if (elect_one()) {
                        tc_mma_f16_ts(d0, a0, bd0, IDESC, kc > u0 ? 1u : 0u);
                        if constexpr (Q8) tc_mma_f16_ts_acc(d0, a0 + 64, bd0, IDESC_HI);
#pragma unroll
                        for (int j = 1; j < KC / 16; ++j) {
                            // B: [k-atom of 64][2*NP rows][128 B swizzled]; k-step j = 16 columns
                            const uint64_t bd = bd0 + (uint64_t)((((j >> 2) * (2 * NP * 128)) + (j & 3) * 32) >> 4);
                            // A: 16 f16 of K = 8 TMEM columns (Q8_0: hi tile, lo tile 64 columns on)
                            tc_mma_f16_ts_acc(d0, a0 + j * 8, bd, IDESC);
                            if constexpr (Q8) tc_mma_f16_ts_acc(d0, a0 + 64 + j * 8, bd, IDESC_HI);
                        }
                        if constexpr (JK) {
                            // junk tile (TMEM columns ACOLS..ACOLS+31) x the junk atom (the fifth)
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const uint64_t bd = bd0 + (uint64_t)((4 * (2 * NP * 128) + j * 32) >> 4);
                                tc_mma_f16_ts_acc(d0, a0 + G::ACOLS + j * 8, bd, IDESC);
                            }
                        }
                        tc_commit(&free_a[sa]);
                        tc_commit(&free_x[sx]);
                        if (kc + 1 == u1) tc_commit(&acc_full[ab]);
                    }
                    __syncwarp();
                    rx.next(SX);
                    ra.next(SA);
                }
                ++ul;
            }
        })
    } else if (warp < 3 + DEC) {
        // -------------------------------- decoders --------------------------------
        // thread = one weight row (its TMEM lane); group g of four warps decodes
        // K columns [g*GK, g*GK + GK) of the chunk.  The codes of a stage are
        // 128B-swizzled: 16-byte piece q of row r sits at q ^ (r % 8), so the
        // eight rows of a quarter-warp hit distinct banks.
        const int dw = warp - 3;
        const int grp = dw >> 2;
        const int quarter = warp & 3;  // TMEM lane quarter this warp may access
        const int r = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        int c = 0;
        Ring rw, ra;
        DQ_FOR_SEGMENTS(p, nch, gbeg, gend, m, tile, c0, c1, {
            float e2 = 1.0f;  // Q8_0: 2^e of this row (exact f32 power of two)
            if constexpr (Q8) {
                const int row = tile * TM + r;
                const int e = row < p.rows ? (int)p.rexp[m][row] : 0;
                e2 = __int_as_float((e + 127) << 23);
            }
            for (int kc = c0; kc < c1 && !*abort_flag; ++kc, ++c) {
                const int sw = rw.s, sa = ra.s;
                dq_wait(&full_w[sw], rw.ph, abort_flag, 32u);
                if (c >= SA) dq_wait(&free_a[sa], ra.ph ^ 1u, abort_flag, 32u);
                if (*abort_flag) break;
                tc_fence_after();
                const uint8_t *row = wst + (size_t)sw * WS + r * 128;
                const uint32_t tcol = tmem + lane_addr + T::A0 + sa * T::AC + grp * 32;
                if constexpr (G::K4 || G::K5 || G::K6) {
                    // K-quants: 64 columns = pieces 2g, 2g+1 of the row (32 weights each).
                    // Low nibbles plus, for Q5_K / Q6_K, the high bits (stored in nibble
                    // slots) are merged into bytes with one bit-select each (even
                    // elements: slot bits moved up by 4; odd: in place), then each byte
                    // enters the mantissa of 2^23 by one PRMT.  Value = the reference's
                    // fp32 dl*q - ml (Q4_K, Q5_K: dl*q is exact, one rounding) or
                    // d*sc*(q - 32) (Q6_K, exact), rounded once to half.
                    const uint8_t *aux = wst + (size_t)sw * WS + G::WCODES;
                    uint32_t o[32];
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const int pc = 2 * grp + i;  // piece = 32 elements of the block
                        const uint4 w4 = *reinterpret_cast<const uint4 *>(row + ((pc ^ (r & 7)) << 4));
                        const uint32_t ws4[4] = {w4.x, w4.y, w4.z, w4.w};
                        float mul[4], sub4[4];  // per word: value = mul * (byte float) - sub
                        uint32_t hp[4];          // per word: high parts in nibble slots (bits 0-1 of a slot)
                        if constexpr (G::K4 || G::K5) {
                            float dl, ml;
                            q4k_scale_min(*reinterpret_cast<const uint4 *>(aux + r * 16), pc, dl, ml);
                            const uint32_t hb = G::K5 ? *reinterpret_cast<const uint32_t *>(aux + G::HB + r * 32 + pc * 4) : 0u;
#pragma unroll
                            for (int wd = 0; wd < 4; ++wd) {
                                mul[wd] = dl;
                                sub4[wd] = ml;
                                hp[wd] = (hb >> wd) & 0x11111111u;
                            }
                        } else {
                            const uint32_t sc2 = *reinterpret_cast<const unsigned short *>(aux + r * 16 + pc * 2);
                            const float d = __half2float(__ushort_as_half(
                                *reinterpret_cast<const unsigned short *>(aux + G::HDR + r * 16 + (kc & 7) * 2)));
                            const uint2 hb = *reinterpret_cast<const uint2 *>(aux + G::HB + r * 64 + pc * 8);
                            const float d0 = d * (float)(int8_t)(sc2 & 0xffu), d1 = d * (float)(int8_t)(sc2 >> 8);
                            mul[0] = d0; mul[1] = d0; mul[2] = d1; mul[3] = d1;
                            hp[0] = hb.x & 0x33333333u; hp[1] = (hb.x >> 2) & 0x33333333u;
                            hp[2] = hb.y & 0x33333333u; hp[3] = (hb.y >> 2) & 0x33333333u;
                            sub4[0] = sub4[1] = sub4[2] = sub4[3] = 0.0f;
                        }
                        // byte-float offset: 2^23 (+ 32 for Q6_K's code bias)
                        constexpr float kOff = G::K6 ? 8388640.0f : 8388608.0f;
#pragma unroll
                        for (int wd = 0; wd < 4; ++wd) {
                            const uint32_t wv = ws4[wd];
                            // bytes of ce: elements 0,2,4,6; of co: elements 1,3,5,7
                            const uint32_t ce = (wv & 0x0F0F0F0Fu) | ((hp[wd] << 4) & 0xF0F0F0F0u);
                            const uint32_t co = ((wv >> 4) & 0x0F0F0F0Fu) | (hp[wd] & 0xF0F0F0F0u);
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const float qe = __uint_as_float(__byte_perm(ce, 0x4B000000u, 0x7540u | t)) - kOff;
                                const float qo = __uint_as_float(__byte_perm(co, 0x4B000000u, 0x7540u | t)) - kOff;
                                const float ve = G::K6 ? mul[wd] * qe : fmaf(mul[wd], qe, -sub4[wd]);
                                const float vo = G::K6 ? mul[wd] * qo : fmaf(mul[wd], qo, -sub4[wd]);
                                const __half2 hv = __floats2half2_rn(ve, vo);
                                o[16 * i + 4 * wd + t] = *reinterpret_cast<const uint32_t *>(&hv);
                            }
                        }
                    }
                    tmem_st32(tcol, o);
                } else if constexpr (!Q8) {
                    // 64 columns = 8 words = pieces 2g, 2g+1 of the row
                    const uint4 wa = *reinterpret_cast<const uint4 *>(row + (((2 * grp) ^ (r & 7)) << 4));
                    const uint4 wb = *reinterpret_cast<const uint4 *>(row + (((2 * grp + 1) ^ (r & 7)) << 4));
                    // word pairs (16 columns each) in the gf4_pair_levels order; a
                    // 16-byte piece holding a scale past 252 (rare) takes the per-word
                    // decode (Metal mode: element 4 rounded with its junk, the tiled-path
                    // semantics, junk halves zero)
                    uint32_t o[32];
                    const uint32_t wd[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                    const bool small[2] = {gf4_scales_small(wa), gf4_scales_small(wb)};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (small[i >> 1]) gf4_pair_levels(wd[2 * i], wd[2 * i + 1], o + 8 * i);
                        else gf4_pair_any<EXACT>(wd[2 * i], wd[2 * i + 1], o + 8 * i);
                    }
                    if constexpr (JK) {
                        uint32_t jk[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) jk[i] = small[i >> 2] ? gf4_junk_halves(wd[i]) : 0u;
                        // junk tile columns ACOLS + 8 * grp .. (word 8 * grp + i at column i)
                        tmem_st8(tmem + lane_addr + T::A0 + sa * T::AC + G::ACOLS + grp * 8, jk);
                    }
                    tmem_st32(tcol, o);
                } else {
                    // 64 codes = pieces 4g .. 4g+3 of the row, blocks 2g and 2g+1 of the
                    // chunk.  Each weight q * d * 2^e becomes hi = half(q * ds) and
                    // lo = q * ds - hi (exact: the residual has <= 8 significant bits),
                    // with ds = half(d * 2^e) (exact unless d is ~2^-21 of the row max).
                    const uint32_t d2 = *reinterpret_cast<const uint32_t *>(
                        wst + (size_t)sw * WS + G::WCODES + r * 16 + (((kc & 1) * 4 + 2 * grp) << 1));
                    const __half2 dh = *reinterpret_cast<const __half2 *>(&d2);
                    const __half2 ds = __floats2half2_rn(__low2float(dh) * e2, __high2float(dh) * e2);
                    uint32_t hi[32], lo[32];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint4 w4 = *reinterpret_cast<const uint4 *>(row + (((4 * grp + i) ^ (r & 7)) << 4));
                        const __half2 s2 = __half2half2(i < 2 ? __low2half(ds) : __high2half(ds));
                        const uint4 q0 = q8_codes_to_halves(w4.x, w4.y), q1 = q8_codes_to_halves(w4.z, w4.w);
                        const uint32_t qs[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                        for (int t = 0; t < 8; ++t) {
                            const __half2 q = *reinterpret_cast<const __half2 *>(&qs[t]);
                            const __half2 h = __hmul2(q, s2);
                            const __half2 l = __hfma2(q, s2, __hneg2(h));
                            hi[8 * i + t] = *reinterpret_cast<const uint32_t *>(&h);
                            lo[8 * i + t] = *reinterpret_cast<const uint32_t *>(&l);
                        }
                    }
                    tmem_st32(tcol, hi);
                    tmem_st32(tcol + 64, lo);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&empty_w[sw]);
                    mbar_arrive(&full_a[sa]);
                }
                rw.next(NW);
                ra.next(SA);
            }
        })
    } else {
        // -------------------------------- epilogue --------------------------------
        // one warp per TMEM lane quarter: row quarter*32 + lane, all NP columns
        pdl_wait();  // rowscale / residual y come from earlier kernels
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        const int ew = warp - 3 - DEC;
        // batch-row scales, lane n holding column n (and 32 + n): broadcast by shuffles
        const float rs0 = lane < p.B ? p.rowscale[lane] : 0.0f;
        const float rs1 = (NP > 32 && 32 + lane < p.B) ? p.rowscale[32 + lane] : 0.0f;
        int ul = 0, sg = 0;
        float amax_v = -INFINITY;  // fused argmax: best of column amax_column<NP>(lane) so far
        uint32_t amax_i = 0xffffffffu;
        DQ_FOR_SEGMENTS(p, nch, gbeg, gend, m, tile, c0, c1, {
            if (!*abort_flag) {
                const int row = tile * TM + row_in_tile;
                float es = 1.0f;  // Q8_0: 2^-e of the row
                if constexpr (Q8) {
                    const int e = row < p.rows ? (int)p.rexp[m][row] : 0;
                    es = __int_as_float((127 - e) << 23);
                }
                float *y = p.y[MODE == DQ_DUAL ? m : 0];
                // Split tiles (stream-K: several CTAs per tile, and accumulate mode)
                // add into y: by TMA bulk reduction of 16-column boxes staged in
                // shared memory (the adds run in L2), else by per-element atomics.
                // Whole-tile schedules (gran == nch) store.
                const bool split = MODE == DQ_ACCUM || p.gran < nch;
                const CUtensorMap *ymap = (MODE == DQ_DUAL && m) ? &ymap1 : &ymap0;
                // 16 columns of the row's result (hi + lo products), scaled and written
                auto emit16 = [&](int n0, const float *sum) {
                    float v[16];
#pragma unroll
                    for (int n = 0; n < 16; ++n) {
                        const float rs = __shfl_sync(0xffffffffu, n0 + n < 32 ? rs0 : rs1, (n0 + n) & 31);
                        v[n] = sum[n] * es * rs;
                    }
                    if (split && p.red_tma) {
                        float *buf = stg + (sg & 1) * (16 * TM);
                        // the reduction issued two boxes ago must have read this buffer
                        if (ew == 0 && lane == 0) bulk_wait_read<1>();
                        named_sync(1, EPI * 32);
#pragma unroll
                        for (int n = 0; n < 16; ++n) buf[n * TM + row_in_tile] = v[n];  // [column][row]
                        fence_async_smem();
                        named_sync(1, EPI * 32);
                        if (ew == 0 && lane == 0 && !*abort_flag) {
                            // rows >= p.rows and columns >= B fall outside the map: not written
                            tma_reduce_add_2d(ymap, tile * TM, n0, buf);
                            bulk_commit();
                        }
                        ++sg;
                    } else if (row < p.rows && !*abort_flag) {
#pragma unroll
                        for (int n = 0; n < 16; ++n) {
                            if (n0 + n < p.B) {
                                float *dst = y + (size_t)(n0 + n) * p.rows + row;
                                if (split) atomicAdd(dst, v[n]);
                                else *dst = v[n];
                            }
                        }
                    }
                };
                if constexpr (NP <= 32) {
                    // the segment's sub-segment accumulators, summed in fp32
                    float acc[NP];
#pragma unroll
                    for (int n = 0; n < NP; ++n) acc[n] = 0.0f;
                    for (int u0 = c0; u0 < c1 && !*abort_flag; u0 += SUB) {
                        const int ab = ul & 1;
                        dq_wait(&acc_full[ab], (ul >> 1) & 1, abort_flag, 64u);
                        tc_fence_after();
#pragma unroll
                        for (int n0 = 0; n0 < NP; n0 += 16) {
                            uint32_t th[16], tl[16];
                            tmem_ld16_async(tmem + lane_addr + ab * RC + n0, th);
                            tmem_ld16_async(tmem + lane_addr + ab * RC + NP + n0, tl);
                            tmem_ld_wait();
#pragma unroll
                            for (int n = 0; n < 16; ++n)
                                acc[n0 + n] += __uint_as_float(th[n]) + __uint_as_float(tl[n]);
                        }
                        // accumulator read out: the MMA may reuse it
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[ab]);
                        ++ul;
                    }
                    if (dq_amax<CODEC, MODE>() && p.amax_val != nullptr) {
                        // whole tile: this row's logits of every batch column, reduced over
                        // the warp's rows into the running (max, lowest id) per column
                        uint32_t ids[NP];
#pragma unroll
                        for (int n = 0; n < NP; ++n) {
                            const float rs = __shfl_sync(0xffffffffu, n < 32 ? rs0 : rs1, n & 31);
                            acc[n] = row < p.rows ? acc[n] * es * rs : -INFINITY;
                            ids[n] = row < p.rows ? (uint32_t)row : 0xffffffffu;
                        }
                        float tv;
                        uint32_t ti;
                        warp_amax_scatter<NP>(acc, ids, lane, tv, ti);
                        if (amax_better(tv, ti, amax_v, amax_i)) { amax_v = tv; amax_i = ti; }
                    } else {
#pragma unroll
                        for (int n0 = 0; n0 < NP; n0 += 16) emit16(n0, acc + n0);
                    }
                } else {
                    // one accumulation per segment, streamed out 16 columns at a time
                    const int ab = ul & 1;
                    dq_wait(&acc_full[ab], (ul >> 1) & 1, abort_flag, 64u);
                    tc_fence_after();
#pragma unroll
                    for (int n0 = 0; n0 < NP; n0 += 16) {
                        uint32_t th[16], tl[16];
                        tmem_ld16_async(tmem + lane_addr + ab * RC + n0, th);
                        tmem_ld16_async(tmem + lane_addr + ab * RC + NP + n0, tl);
                        tmem_ld_wait();
                        if (n0 + 16 >= NP) {  // accumulator read out: the MMA may reuse it
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&acc_empty[ab]);
                        }
                        float sum[16];
#pragma unroll
                        for (int n = 0; n < 16; ++n) sum[n] = __uint_as_float(th[n]) + __uint_as_float(tl[n]);
                        emit16(n0, sum);
                    }
                    ++ul;
                }
            }
        })
        if (ew == 0 && lane == 0) bulk_wait_all();  // our reductions are complete before exit
        if constexpr (NP <= 32 && dq_amax<CODEC, MODE>()) {
            if (p.amax_val != nullptr) {
                // the epilogue warps' column bests, combined in warp order (the staging
                // buffer is free: whole-tile schedules store nothing through it)
                float *sv = stg;
                uint32_t *si = reinterpret_cast<uint32_t *>(stg + 128);
                sv[ew * 32 + lane] = amax_v;
                si[ew * 32 + lane] = amax_i;
                named_sync(1, EPI * 32);
                if (ew == 0) {
                    float bv = sv[lane];
                    uint32_t bi = si[lane];
                    for (int w = 1; w < EPI; ++w)
                        if (amax_better(sv[w * 32 + lane], si[w * 32 + lane], bv, bi)) {
                            bv = sv[w * 32 + lane];
                            bi = si[w * 32 + lane];
                        }
                    const int col = amax_column<NP>(lane);
                    if (col < p.B) {  // lanes sharing a column write the same pair
                        p.amax_val[(size_t)blockIdx.x * p.B + col] = bv;
                        p.amax_idx[(size_t)blockIdx.x * p.B + col] = bi;
                    }
                }
            }
        }
    }

    // No programmatic launch trigger in this kernel: the next one (normally the
    // next matvec's activation prep) launches when this grid exits.  Launched
    // earlier, its CTAs wait beside ours and take issue slots from the decode
    // warps (a trigger from any thread counts for the whole CTA, and the idle
    // lanes of the role warps would reach it at once).
    // ---- teardown: nothing of ours may be in flight when TMEM is released ----
    if (warp == 1 && *abort_flag) {
        // the MMA issuer (the elected lane, as in the issue loop) drains its own
        // tensor-core work (bounded) before TMEM goes
        __syncwarp();
        if (elect_one()) {
            tc_commit(drain);
            mbar_wait(drain, 0, 128u);
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// activation prep: RMS norm (optional), per-row power-of-two scale, f32 ->
// hi + lo halves in the MMA's K-major swizzled layout (one CTA per padded
// batch row); zeroes the outputs that split tiles add into.
// ---------------------------------------------------------------------------
template <typename XT>
__device__ __forceinline__ void load8(const XT *p, float *v) {
    if constexpr (sizeof(XT) == 4) {
        const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
            v[2 * i] = __low2float(h);
            v[2 * i + 1] = __high2float(h);
        }
    }
}

// One CTA (128 threads) per padded batch row n; each thread handles groups of
// 8 consecutive columns (one 16-byte piece of the swizzled tile for hi and one
// for lo).  Pass 1 reduces sum(x^2) (RMS norm) and max|x * w| together; pass 2
// writes.  128 threads keep the CTA small enough to share an SM with a
// running matvec CTA.
template <typename XT>
__global__ void __launch_bounds__(128) dq_prep_kernel(const XT *x, const float *norm_w, float eps, int K, int B, int NP,
                                                      int gf4_perm, int junk, __half *xh, float *rowscale, float *zero0,
                                                      float *zero1, int zero_rows) {
    __shared__ float red_s[4], red_m[4];
    pdl_trigger();  // the matvec may start streaming its weights now
    pdl_wait();     // x (and the outputs zeroed below) belong to earlier kernels
    const int n = blockIdx.x;
    const int G = K >> 3;
    const XT *xr = x + (size_t)(n < B ? n : 0) * K;
    float inv = 1.0f, e2 = 1.0f;
    if (n < B) {
        float ss = 0.0f, mx = 0.0f;
        for (int g = threadIdx.x; g < G; g += 128) {
            float v[8];
            load8(xr + g * 8, v);
            if (norm_w) {
                const float4 w0 = *reinterpret_cast<const float4 *>(norm_w + g * 8);
                const float4 w1 = *reinterpret_cast<const float4 *>(norm_w + g * 8 + 4);
                const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    ss = fmaf(v[i], v[i], ss);
                    mx = fmaxf(mx, fabsf(v[i] * w[i]));
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[i]));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, o);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        if ((threadIdx.x & 31) == 0) {
            red_s[threadIdx.x >> 5] = ss;
            red_m[threadIdx.x >> 5] = mx;
        }
        __syncthreads();
        ss = (red_s[0] + red_s[1]) + (red_s[2] + red_s[3]);
        mx = fmaxf(fmaxf(red_m[0], red_m[1]), fmaxf(red_m[2], red_m[3]));
        if (norm_w) {
            inv = rsqrtf(ss / (float)K + eps);
            mx *= inv;
        }
        int ex = 0;
        if (mx > 0.0f && isfinite(mx)) {
            frexpf(mx, &ex);
            ex -= 15;  // max |v| * 2^-ex in [2^14, 2^15) (2x margin for rounding of the max)
        }
        e2 = ldexpf(1.0f, ex);
        if (threadIdx.x == 0) rowscale[n] = e2;
    } else if (threadIdx.x == 0) {
        rowscale[n] = 1.0f;
    }
    const float rs = 1.0f / e2;  // exact power of two
    // GF4 tiles hold each 16 columns (two words A, B) in the order
    // [A0,A5,A1,A6,A2,A7,B0,B5,B1,B6,B2,B7,A3,B3,A4,B4] (gf4_pair_levels)
    constexpr int kPerm16[16] = {0, 5, 1, 6, 2, 7, 8, 13, 9, 14, 10, 15, 3, 11, 4, 12};
    for (int g = threadIdx.x; g < (G >> 1); g += 128) {
        float v[16];
        if (n < B) {
            load8(xr + g * 16, v);
            load8(xr + g * 16 + 8, v + 8);
            if (norm_w) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float4 w0 = *reinterpret_cast<const float4 *>(norm_w + g * 16 + 8 * h);
                    const float4 w1 = *reinterpret_cast<const float4 *>(norm_w + g * 16 + 8 * h + 4);
                    const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[8 * h + i] = (v[8 * h + i] * inv * w[i]) * rs;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = v[i] * rs;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a = gf4_perm ? v[kPerm16[2 * i]] : v[2 * i], b = gf4_perm ? v[kPerm16[2 * i + 1]] : v[2 * i + 1];
            const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
            const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
            hw[i] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
            lw[i] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
        }
        // k-atoms of 64 columns [2*NP rows: hi rows, then lo rows][128 B swizzled],
        // per 256 columns the four atoms of the chunk, then (junk) the junk atom
        const int k = g * 16;
        const size_t atom = (size_t)(k >> 8) * (junk ? 5 : 4) + ((k & 255) >> 6);
        uint8_t *base = reinterpret_cast<uint8_t *>(xh) + atom * (2 * NP) * 128;
        const uint32_t c = (uint32_t)((k & 63) >> 3);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            *reinterpret_cast<uint4 *>(base + sw128_off((uint32_t)n, c + h)) =
                make_uint4(hw[4 * h], hw[4 * h + 1], hw[4 * h + 2], hw[4 * h + 3]);
            *reinterpret_cast<uint4 *>(base + sw128_off((uint32_t)(NP + n), c + h)) =
                make_uint4(lw[4 * h], lw[4 * h + 1], lw[4 * h + 2], lw[4 * h + 3]);
        }
        if (junk) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                // word w of the chunk: junk-atom columns 2w, 2w+1 both hold x_4 * 2^-10 (hi | lo rows)
                const float a = v[8 * h + 4] * 0.0009765625f;
                const __half ha = __float2half_rn(a), la = __float2half_rn(a - __half2float(ha));
                const uint32_t w = (uint32_t)(((k + 8 * h) & 255) >> 3);
                uint8_t *jb = reinterpret_cast<uint8_t *>(xh) + ((size_t)(k >> 8) * 5 + 4) * (2 * NP) * 128 + (w & 3) * 4;
                *reinterpret_cast<uint32_t *>(jb + sw128_off((uint32_t)n, w >> 2)) = (uint32_t)__half_as_ushort(ha) * 0x10001u;
                *reinterpret_cast<uint32_t *>(jb + sw128_off((uint32_t)(NP + n), w >> 2)) = (uint32_t)__half_as_ushort(la) * 0x10001u;
            }
        }
    }
    if (n < B && (zero0 || zero1)) {
        __syncthreads();  // every read of x row n is done (y may alias x)
        for (int z = 0; z < 2; ++z) {
            float *zp = z ? zero1 : zero0;
            if (!zp) continue;
            float *row = zp + (size_t)n * zero_rows;
            // 16-byte stores over the aligned middle of the row, scalars at its ends
            const int head = (int)(((16u - ((uintptr_t)row & 15u)) & 15u) >> 2);
            const int h = head < zero_rows ? head : zero_rows;
            if (threadIdx.x < h) row[threadIdx.x] = 0.0f;
            const int nv = (zero_rows - h) >> 2;
            float4 *v = reinterpret_cast<float4 *>(row + h);
            for (int i = threadIdx.x; i < nv; i += 128) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = h + 4 * nv + threadIdx.x; r < zero_rows; r += 128) row[r] = 0.0f;
        }
    }
}

// h = silu(gate) * up over [B][rows]
__global__ void dq_swiglu_kernel(const float *g, const float *u, float *h, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        h[i] = silu_f(g[i]) * u[i];
}

cudaError_t swiglu_run(const float *gate, const float *up, float *h, size_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    dq_swiglu_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, st>>>(gate, up, h, n);
    return cudaGetLastError();
}

// final (max, lowest id) over per-CTA partials (matvec.cu)
__global__ void argmax_reduce_kernel(const float *pv, const uint32_t *pi, int n, int B, uint32_t *out_tok,
                                     float *out_val);

// lowest-id argmax of each logits row (one CTA of 1024 threads per row)
__global__ void __launch_bounds__(1024) dq_argmax_rows_kernel(const float *logits, int V, uint32_t *tok, float *val) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    const float *l = logits + (size_t)blockIdx.x * V;
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (int i = threadIdx.x; i < V; i += 1024) {
        const float v = l[i];
        if (v > bv) { bv = v; bi = (uint32_t)i; }  // ascending i per thread: keeps the lowest id
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        bv = sv[threadIdx.x];
        bi = si[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (threadIdx.x == 0) {
            tok[blockIdx.x] = bi;
            if (val) val[blockIdx.x] = bv;
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Tensor map over the codes plane of a device-layout weight (cached: weights are immutable).
bool weight_map(uint32_t type_id, const void *w, uint32_t rows, uint32_t k, CUtensorMap *out) {
    static std::mutex mu;
    static std::map<std::tuple<const void *, uint32_t, uint32_t, uint32_t>, CUtensorMap> cache;
    std::lock_guard<std::mutex> g(mu);
    auto key = std::make_tuple(w, type_id, rows, k);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    CUtensorMap m;
    cuuint64_t dims[2], strides[1];
    cuuint32_t box[2], estr[2] = {1, 1};
    CUtensorMapDataType dt;
    // 128 rows x 128 bytes per box, 128B-swizzled (16-byte piece q of row r at q ^ (r % 8))
    if (type_id != QW35_Q8_0_TYPE) {  // k/2 bytes of nibbles per row (Q5_K / Q6_K: then the high bits)
        dt = CU_TENSOR_MAP_DATA_TYPE_UINT32;
        dims[0] = k / 8; dims[1] = rows;
        strides[0] = type_id == QW35_Q5_K_TYPE ? (cuuint64_t)k / 2 + k / 8
                   : type_id == QW35_Q6_K_TYPE ? (cuuint64_t)k / 2 + k / 4 : (cuuint64_t)k / 2;
        box[0] = 32; box[1] = TM;
    } else {
        dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
        dims[0] = k; dims[1] = rows; strides[0] = k;
        box[0] = 128; box[1] = TM;
    }
    if (fn(&m, dt, 2, const_cast<void *>(w), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return false;
    cache[key] = m;
    *out = m;
    return true;
}

// Tensor map over the Q8_0 scales plane ([rows][K/32] f16): boxes of 8 scales
// (16 bytes, two chunks) x 128 rows.
bool scale_map(const void *w, uint32_t rows, uint32_t k, CUtensorMap *out) {
    static std::mutex mu;
    static std::map<std::tuple<const void *, uint32_t, uint32_t>, CUtensorMap> cache;
    std::lock_guard<std::mutex> g(mu);
    auto key = std::make_tuple(w, rows, k);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    CUtensorMap m;
    cuuint64_t dims[2] = {k / 32, rows}, strides[1] = {(cuuint64_t)(k / 32) * 2};
    cuuint32_t box[2] = {8, TM}, estr[2] = {1, 1};
    void *base = static_cast<uint8_t *>(const_cast<void *>(w)) + (size_t)rows * k;
    if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return false;
    cache[key] = m;
    *out = m;
    return true;
}

// Unswizzled uint32 tensor map over a [rows][dim0 words] region at `base`
// with a row pitch of `pitch` bytes, boxes of box0 words x 128 rows (cached:
// weights are immutable).  Serves the K-quant side planes: Q4_K / Q5_K block
// headers, Q6_K scales and d, Q5_K / Q6_K high bits.
bool plain_map(const void *base, uint64_t dim0, uint32_t rows, uint64_t pitch, uint32_t box0, CUtensorMap *out) {
    static std::mutex mu;
    static std::map<std::tuple<const void *, uint64_t, uint32_t, uint64_t, uint32_t>, CUtensorMap> cache;
    std::lock_guard<std::mutex> g(mu);
    auto key = std::make_tuple(base, dim0, rows, pitch, box0);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    CUtensorMap m;
    cuuint64_t dims[2] = {dim0, rows}, strides[1] = {pitch};
    cuuint32_t box[2] = {box0, TM}, estr[2] = {1, 1};
    if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    cache[key] = m;
    *out = m;
    return true;
}

// Side-plane maps of a K-quant weight: s = headers (Q4_K / Q5_K, one 16-byte
// box per block) or the Q6_K scales row (16-byte boxes); h = high bits (Q5_K
// 8 words, Q6_K 16 words per block).
bool kquant_maps(uint32_t type_id, const void *w, uint32_t rows, uint32_t k, CUtensorMap *s, CUtensorMap *h) {
    const uint8_t *b = static_cast<const uint8_t *>(w);
    if (type_id == QW35_Q4_K_TYPE) return plain_map(b + (size_t)rows * (k / 2), k / 64, rows, k / 16, 4, s);
    if (type_id == QW35_Q5_K_TYPE) {
        const uint64_t cr = k / 2 + k / 8;
        return plain_map(b + (size_t)rows * cr, k / 64, rows, k / 16, 4, s) &&
               plain_map(b + k / 2, k / 32, rows, cr, 8, h);
    }
    if (type_id == QW35_Q6_K_TYPE) {
        const uint64_t cr = k / 2 + k / 4, sr = q6k_scale_row(k);
        return plain_map(b + (size_t)rows * cr, sr / 4, rows, sr, 4, s) && plain_map(b + k / 2, k / 16, rows, cr, 16, h);
    }
    return false;
}

// Tensor map over an output y [B][rows] f32 (x = row, y = batch column): boxes
// of 128 rows x 16 columns for the epilogue's bulk reductions.
bool out_map(const void *y, uint32_t rows, uint32_t B, CUtensorMap *out) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {rows, B}, strides[1] = {(cuuint64_t)rows * 4};
    cuuint32_t box[2] = {TM, 16}, estr[2] = {1, 1};
    return fn(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(y), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int dq_np(int B) { return B <= 16 ? 16 : 32; }

}  // namespace

bool dq_supported(const MatvecArgs &a) {
    // TMA needs 16-byte aligned weights; the activation prep reads x and the
    // norm weight 16 bytes at a time
    auto a16 = [](const void *p) { return ((uintptr_t)p & 15u) == 0; };
    // K % 256: GF4 / K-quant chunks are 256 columns; Q8_0 scale boxes span two 128-column chunks
    return a.batch >= kDqMinBatch && a.batch <= 64 &&
           (a.type_id == QW35_GF4_TYPE || a.type_id == QW35_Q8_0_TYPE || a.type_id == QW35_Q4_K_TYPE ||
            a.type_id == QW35_Q5_K_TYPE || a.type_id == QW35_Q6_K_TYPE) &&
           a.k % 256 == 0 &&
           a16(a.w0) && a16(a.w1) && a16(a.x) && a16(a.norm_w) && encode_fn() != nullptr &&
           !getenv("QW35_NO_TCGEN05");
}

// Scratch layout of one batched matvec: activation tiles (hi | lo rows), row
// scales, gate|up or logits outputs (modes 2 / 3).
struct DqScratch {
    size_t x, rowscale, ext, total;
};
static DqScratch dq_scratch_layout(int B, uint32_t k, uint32_t rows_out, size_t ext_bytes) {
    const int NP = dq_np(B);
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    DqScratch l{};
    l.x = 0;
    l.rowscale = up((size_t)2 * NP * k * 2 * 5 / 4);  // (GF4 metal mode: + a junk atom per 256 columns)
    l.ext = l.rowscale + 256;
    l.total = up(l.ext + ext_bytes);
    return l;
}

size_t dq_scratch_bytes(int B, uint32_t k, uint32_t rows_out) {
    return dq_scratch_layout(B, k, rows_out, (size_t)2 * B * rows_out * 4).total;
}

struct DqMaps {
    CUtensorMap m0, m1, s0, s1, y0, y1, h0, h1;  // codes, side planes, outputs, high bits (per matrix)
};

template <int CODEC, int NP, int MODE, bool EXACT>
static cudaError_t dq_launch(const DqMaps &M, DqParams p, cudaStream_t st) {
    auto kern = dq_kernel<CODEC, NP, MODE, EXACT>;
    // SX activation stages (two when they are 64 KB), then as many weight stages as fit
    // stages <= 176 KB (+ 16 KB epilogue staging), so a 128-thread activation
    // prep CTA fits beside it on the SM
    constexpr uint32_t budget = 176u * 1024u;
    constexpr bool JK = dq_junk<CODEC, EXACT>();
    constexpr uint32_t xs = dq_xstage<CODEC, NP, JK>(), ws = DqGeo<CODEC>::WS;
    int SX = xs >= 65536u ? 2 : 3;
    // (at least two weight stages: Q6_K's 28 KB stages then pass the budget)
    int NW = std::max(2, std::min(4, (int)((budget - SX * xs) / ws)));
    using T = DqTmem<CODEC, NP, JK>;
    const size_t smem = 1024 + (size_t)SX * xs + (size_t)NW * ws + 2 * 16 * TM * 4 +
                        (2 * NW + 2 * SX + 2 * T::SA + 4 + 1) * 8 + 16;
    {
        cudaError_t e = qw35h::smem_optin((const void *)kern, 227 * 1024);
        if (e != cudaSuccess) return e;
    }
    const int grid = std::min(p.granules, qw35h::sm_count());
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DqGeo<CODEC>::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = getenv("QW35_NO_PDL") ? 0 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, M.m0, M.m1, M.s0, M.s1, M.y0, M.y1, M.h0, M.h1, p, SX, NW);
    return e;
}

template <int CODEC, int NP>
static cudaError_t dq_dispatch_mode(int mode, bool exact, const DqMaps &M, const DqParams &p, cudaStream_t st) {
    if constexpr (CODEC == QW35_GF4_TYPE) {
        if (!exact) {
            if (mode == DQ_STORE) return dq_launch<CODEC, NP, DQ_STORE, false>(M, p, st);
            if (mode == DQ_ACCUM) return dq_launch<CODEC, NP, DQ_ACCUM, false>(M, p, st);
            return dq_launch<CODEC, NP, DQ_DUAL, false>(M, p, st);
        }
    }
    if (mode == DQ_STORE) return dq_launch<CODEC, NP, DQ_STORE, true>(M, p, st);
    if (mode == DQ_ACCUM) return dq_launch<CODEC, NP, DQ_ACCUM, true>(M, p, st);
    return dq_launch<CODEC, NP, DQ_DUAL, true>(M, p, st);
}

template <int CODEC>
static cudaError_t dq_dispatch_np(int NP, int mode, bool exact, const DqMaps &M, const DqParams &p, cudaStream_t st) {
    if (NP == 16) return dq_dispatch_mode<CODEC, 16>(mode, exact, M, p, st);
    return dq_dispatch_mode<CODEC, 32>(mode, exact, M, p, st);
}

static cudaError_t dq_enqueue(const MatvecArgs &a, int mode, uint32_t *tok, float *val, const DqScratch &lay,
                              void *scr, DqMaps &M, cudaStream_t st);

// mode: 0 store, 1 accumulate, 2 swiglu pair, 3 logits for the argmax head
cudaError_t dq_run(const MatvecArgs &a, int mode, uint32_t *tok, float *val, cudaStream_t st) {
    if (a.batch > 32) {
        // two launches of at most 32 rows: the epilogue sums each row's short
        // tensor-core accumulations in registers, 32 batch columns at most
        MatvecArgs h = a;
        h.batch = 32;
        cudaError_t e = dq_run(h, mode, tok, val, st);
        if (e != cudaSuccess) return e;
        const size_t xes = a.x_dtype == QW35_F16_TYPE ? 2 : 4;
        h = a;
        h.batch = a.batch - 32;
        h.x = static_cast<const uint8_t *>(a.x) + (size_t)32 * a.k * xes;
        if (a.y) h.y = a.y + (size_t)32 * a.rows;
        return dq_run(h, mode, tok ? tok + 32 : nullptr, val ? val + 32 : nullptr, st);
    }
    const int B = a.batch, rows = (int)a.rows;
    const bool dual = mode == 2;
    DqMaps M;
    CUtensorMap &m0 = M.m0, &m1 = M.m1;
    if (!weight_map(a.type_id, a.w0, a.rows, a.k, &m0)) return cudaErrorInvalidValue;
    if (dual && !weight_map(a.type_id, a.w1, a.rows, a.k, &m1)) return cudaErrorInvalidValue;
    if (!dual) m1 = m0;
    // side planes: Q8_0 scales, K-quant headers / scales and high bits (unused maps stay copies)
    M.s0 = M.h0 = m0;
    M.s1 = M.h1 = m1;
    if (a.type_id == QW35_Q8_0_TYPE) {
        if (!scale_map(a.w0, a.rows, a.k, &M.s0)) return cudaErrorInvalidValue;
        if (dual && !scale_map(a.w1, a.rows, a.k, &M.s1)) return cudaErrorInvalidValue;
    } else if (a.type_id != QW35_GF4_TYPE) {
        if (!kquant_maps(a.type_id, a.w0, a.rows, a.k, &M.s0, &M.h0)) return cudaErrorInvalidValue;
        if (dual && !kquant_maps(a.type_id, a.w1, a.rows, a.k, &M.s1, &M.h1)) return cudaErrorInvalidValue;
    }
    if (!dual) {
        M.s1 = M.s0;
        M.h1 = M.h0;
    }
    // mode 3 without a logits buffer (Q8_0 / Q6_K heads): the argmax is fused
    // into the epilogue and only per-CTA partials ([grid][B] value + id) go
    // through the scratch
    const bool amax_fused = mode == 3 && !a.y && (a.type_id == QW35_Q8_0_TYPE || a.type_id == QW35_Q6_K_TYPE);
    const size_t extra = (mode == 2) ? (size_t)2 * B * rows * 4
                         : amax_fused ? (size_t)qw35h::sm_count() * B * 8
                         : (mode == 3 && !a.y) ? (size_t)B * rows * 4 : 0;
    const DqScratch lay = dq_scratch_layout(B, a.k, a.rows, extra);
    // the caller's scratch (a runtime owns one for its lifetime), else a
    // stream-ordered allocation returned after this call's kernels
    void *scr = a.scratch;
    cudaError_t e = cudaSuccess;
    if (scr) {
        if (a.scratch_bytes < lay.total) return cudaErrorInvalidValue;
    } else {
        e = cudaMallocAsync(&scr, lay.total, st);
        if (e != cudaSuccess) return e;
        e = dq_enqueue(a, mode, tok, val, lay, scr, M, st);
        cudaError_t f = cudaFreeAsync(scr, st);
        return e != cudaSuccess ? e : f;
    }
    return dq_enqueue(a, mode, tok, val, lay, scr, M, st);
}

static cudaError_t dq_enqueue(const MatvecArgs &a, int mode, uint32_t *tok, float *val, const DqScratch &lay,
                              void *scr, DqMaps &M, cudaStream_t st) {
    const int B = a.batch, NP = dq_np(B);
    const int K = (int)a.k, rows = (int)a.rows;
    const bool dual = mode == 2;
    CUtensorMap &m0 = M.m0;
    cudaError_t e = cudaSuccess;
    uint8_t *base = static_cast<uint8_t *>(scr);
    __half *xh = reinterpret_cast<__half *>(base + lay.x);
    float *rowscale = reinterpret_cast<float *>(base + lay.rowscale);
    float *ext = reinterpret_cast<float *>(base + lay.ext);

    const int tiles = (rows + TM - 1) / TM;
    const int nch = K / (a.type_id == QW35_Q8_0_TYPE ? DqGeo<QW35_Q8_0_TYPE>::KC : DqGeo<QW35_GF4_TYPE>::KC);
    // logits (mode 3) are stored, never accumulated: whole tiles per CTA
    const int gran = mode == 3 ? nch : 1;
    DqParams p{};
    p.xprep = base;
    p.rowscale = rowscale;
    p.rows = rows;
    p.K = K;
    p.B = B;
    p.tiles = tiles;
    p.gran = gran;
    p.granules = tiles * (dual ? 2 : 1) * (nch / gran);
    float *y0, *y1 = nullptr;
    int dmode;
    if (mode == 2) { y0 = ext; y1 = ext + (size_t)B * rows; dmode = DQ_DUAL; }
    else if (mode == 3) { y0 = a.y ? a.y : ext; dmode = DQ_STORE; }
    else { y0 = a.y; dmode = mode == 1 ? DQ_ACCUM : DQ_STORE; }
    const bool fused_amax = mode == 3 && !a.y && (a.type_id == QW35_Q8_0_TYPE || a.type_id == QW35_Q6_K_TYPE);
    const int grid = std::min(p.granules, qw35h::sm_count());  // as dq_launch
    if (fused_amax) {
        p.amax_val = ext;
        p.amax_idx = reinterpret_cast<uint32_t *>(ext + (size_t)grid * B);
    }
    p.y[0] = y0;
    p.y[1] = y1;
    if (a.type_id == QW35_Q8_0_TYPE) {
        // row exponent plane: after the codes (rows * K) and scales (rows * K / 16) planes
        const size_t off = (size_t)rows * (K / 32) * 34;
        p.rexp[0] = reinterpret_cast<const int8_t *>(static_cast<const uint8_t *>(a.w0) + off);
        p.rexp[1] = dual ? reinterpret_cast<const int8_t *>(static_cast<const uint8_t *>(a.w1) + off) : p.rexp[0];
    }
    // outputs that split tiles add into start at zero
    const bool zero = dmode != DQ_ACCUM && gran < nch;
    // TMA bulk reductions need 16-byte aligned outputs with 16-byte row strides
    CUtensorMap &y0m = M.y0, &y1m = M.y1;
    y0m = y1m = m0;
    p.red_tma = (rows % 4 == 0) && ((uintptr_t)y0 & 15u) == 0 && (!dual || ((uintptr_t)y1 & 15u) == 0) &&
                out_map(y0, rows, B, &y0m) && (!dual || out_map(y1, rows, B, &y1m));
    if (!dual) y1m = y0m;
    const bool gperm = a.type_id == QW35_GF4_TYPE;
    const int junk = (a.type_id == QW35_GF4_TYPE && !(a.flags & QW35_MV_GF4_EXACT)) ? 1 : 0;
    {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(NP);
        cfg.blockDim = dim3(128);
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = getenv("QW35_NO_PDL") ? 0 : 1;
        if (a.x_dtype == QW35_F16_TYPE)
            e = cudaLaunchKernelEx(&cfg, dq_prep_kernel<__half>, static_cast<const __half *>(a.x), a.norm_w, a.eps, K,
                                   B, NP, (int)gperm, junk, xh, rowscale, zero ? y0 : nullptr, zero ? y1 : nullptr, rows);
        else
            e = cudaLaunchKernelEx(&cfg, dq_prep_kernel<float>, static_cast<const float *>(a.x), a.norm_w, a.eps, K, B,
                                   NP, (int)gperm, junk, xh, rowscale, zero ? y0 : nullptr, zero ? y1 : nullptr, rows);
        if (e != cudaSuccess) return e;
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const bool exact = (a.flags & QW35_MV_GF4_EXACT) != 0;
    switch (a.type_id) {
        case QW35_GF4_TYPE: e = dq_dispatch_np<QW35_GF4_TYPE>(NP, dmode, exact, M, p, st); break;
        case QW35_Q8_0_TYPE: e = dq_dispatch_np<QW35_Q8_0_TYPE>(NP, dmode, true, M, p, st); break;
        case QW35_Q4_K_TYPE: e = dq_dispatch_np<QW35_Q4_K_TYPE>(NP, dmode, true, M, p, st); break;
        case QW35_Q5_K_TYPE: e = dq_dispatch_np<QW35_Q5_K_TYPE>(NP, dmode, true, M, p, st); break;
        case QW35_Q6_K_TYPE: e = dq_dispatch_np<QW35_Q6_K_TYPE>(NP, dmode, true, M, p, st); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    if (mode == 2) {
        const size_t n = (size_t)B * rows;
        dq_swiglu_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, st>>>(y0, y1, a.y, n);
        e = cudaGetLastError();
    } else if (mode == 3 && fused_amax) {
        argmax_reduce_kernel<<<B, 256, 0, st>>>(p.amax_val, p.amax_idx, grid, B, tok, val);
        e = cudaGetLastError();
    } else if (mode == 3) {
        dq_argmax_rows_kernel<<<B, 1024, 0, st>>>(y0, rows, tok, val);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace qw35
