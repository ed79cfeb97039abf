// dqgemm.cu -- batched (B >= 16) fused dequantise-and-multiply on the 5th-gen
// tensor cores (tcgen05, TMEM accumulators, TMA-fed weight stages).
//
// Y[b][r] (+)= sum_k W[r][k] * X[b][k] for a decode batch of B sequences.  At
// B >= 16 the weight stream is shared by B tokens, so the CUDA-core matvec
// (matvec.cu) becomes FMA-bound; here each weight is decoded ONCE per launch
// into an f16 tile and multiplied against all B activation rows by
// tcgen05.mma.  Reference semantics: the reference engine has no batched
// decode; its multi-token path (qw35_kernel_mul_mm, qw35_tiled_mm.metal:36-255)
// dequantises weights to half (qw35_dequantize_gf4, qw35_gf4.metal:42-58) and
// keeps activations in f32 (:197-200).  This kernel does the same: GF4
// weights become exactly those halves (element 4 of a word rounded to half in
// the default Metal-compatible mode), and every f32 activation is split into
// hi + lo halves so the product keeps ~22 bits of the activation.
//
// Q8_0 weights are not exact in f16 once multiplied by their block scale, so
// the int8 codes (exact) go through the tensor core per 32-column block into a
// rotating set of TMEM accumulators and the epilogue warps apply the f16 block
// scale in fp32 (acc += d * block_sum): bit-for-bit the reference's
// per-block arithmetic up to summation order.
//
// CTA: warp 0 TMA producer, warp 1 MMA issuer (+ TMEM owner), then decode
// warps, then epilogue warps (counts per codec in DqWarps).  Tiles are 128 weight rows x NP batch columns (B padded to a
// multiple of 16); K streams in 128-column chunks through S shared-memory
// stages; work units (matrix, row tile, K split) are spread over a persistent
// grid.  Every wait is bounded (pipe.cuh).  No cluster multicast is used.
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
#include "tc.cuh"

namespace qw35 {

constexpr int TM = 128;     // weight rows per tile (MMA M)
constexpr int KC = 128;     // K columns per stage
constexpr int NKB = KC / 8; // 16 k-blocks of 8 per stage
// warp roles per codec: GF4 decode is the bottleneck (16 decode warps, the
// once-per-unit epilogue needs 4); Q8_0 decodes cheaply but scales every
// 32-column block in the epilogue (8 + 8).
template <int CODEC> struct DqWarps {
    static constexpr int DEC = CODEC == QW35_GF4_TYPE ? 16 : 8;
    static constexpr int EPI = CODEC == QW35_GF4_TYPE ? 4 : 8;
    static constexpr int THREADS = (2 + DEC + EPI) * 32;
};

enum DqMode { DQ_STORE = 0, DQ_ACCUM = 1, DQ_DUAL = 2 };

struct DqParams {
    const uint8_t *xprep;   // per 128-column chunk [2 k-atoms][2*NP rows (hi | lo)][128 B swizzled] f16
    const float *rowscale;  // [NP]
    const uint8_t *sc[2];   // Q8_0 scales planes [rows][K/32] f16
    float *y[2];
    int rows, K, B, ksplit, tiles, units;
    uint32_t wbytes;        // bytes of one weight stage (TMA box)
    unsigned long long *trace;  // debug: per-chunk event stamps of CTA 0 (QW35_DQ_TRACE), or null
};
// trace layout: [chunk][6] = producer issue, decoder sees full, decoder done,
// mma sees full_a, mma committed, (unused)
#define DQ_TRACE(c, slot) \
    do { if (p.trace && blockIdx.x == 0 && (c) < 256) p.trace[(c) * 6 + (slot)] = globaltimer(); } while (0)

struct DqSmem {  // offsets into dynamic shared memory
    uint32_t w, x, a, bar, tmem, abort_;
    int S;
};

template <int CODEC, int NP>
__host__ __device__ constexpr uint32_t dq_wstage() {
    return CODEC == QW35_GF4_TYPE ? TM * KC / 2 : TM * KC;
}
template <int NP>
__host__ __device__ constexpr uint32_t dq_xstage() { return 2u * NP * KC * 2; }  // hi + lo
__host__ __device__ constexpr uint32_t dq_astage() { return TM * KC * 2; }

// TMEM columns for the accumulators.
// GF4: 2 unit buffers x 4 independent accumulators (hi/lo x even/odd k-step),
// so consecutive MMAs never wait on each other's accumulator.  Q8_0: rotating
// per-block regions (consecutive blocks already use different regions).
constexpr int GF4_NACC = 1;
template <int CODEC, int NP>
__host__ __device__ constexpr int dq_regions() {
    return CODEC == QW35_GF4_TYPE ? 2 : (512 / (2 * NP) < 8 ? 512 / (2 * NP) : 8);
}
// one accumulator = 2*NP columns: [hi-activation products | lo-activation products]
template <int CODEC, int NP>
__host__ __device__ constexpr int dq_region_cols() { return CODEC == QW35_GF4_TYPE ? GF4_NACC * 2 * NP : 2 * NP; }
template <int CODEC, int NP>
__host__ __device__ constexpr uint32_t dq_tmem_cols() {
    constexpr int cols = dq_regions<CODEC, NP>() * dq_region_cols<CODEC, NP>();
    return cols <= 32 ? 32u : cols <= 64 ? 64u : cols <= 128 ? 128u : cols <= 256 ? 256u : 512u;
}

// ---- decode of one 16-byte chunk of a weight row into 8 halves --------------------
// GF4: one word -> 8 halves in k order [0,4,1,5,2,6,3,7] (the activation prep
// applies the same permutation inside every 8-column group, so the dot is
// unchanged).  Values: (q_raw - 4) * (-0.25 * s), exact in f16; in metal mode
// element 4 is half(float(q4 * 8192 + junk) * s * -0.25 * 2^-13), the
// reference's tiled-path rounding.
// Halves of one word, without the Metal element-4 junk (that is added by
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

template <int CODEC, int NP, int MODE, bool EXACT>
__global__ void __launch_bounds__(DqWarps<CODEC>::THREADS, 1)
dq_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1, DqParams p, int S) {
    constexpr int R = dq_regions<CODEC, NP>();
    constexpr uint32_t TCOLS = dq_tmem_cols<CODEC, NP>();
    constexpr uint32_t XS = dq_xstage<NP>();
    constexpr uint32_t AS = dq_astage();
    constexpr uint32_t IDESC = idesc_f16_f32(TM, 2 * NP);  // B = [x_hi rows ; x_lo rows]
    constexpr int RC = dq_region_cols<CODEC, NP>();
    constexpr bool BLOCKED = CODEC != QW35_GF4_TYPE;
    constexpr int DQ_DEC_WARPS = DqWarps<CODEC>::DEC;
    constexpr int DQ_EPI_WARPS = DqWarps<CODEC>::EPI;
    extern __shared__ __align__(1024) uint8_t smem[];

    const uint32_t WS = p.wbytes;
    // 1024-byte aligned base (128B-swizzle atoms need it)
    uint8_t *wst = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);  // [S][WS]
    uint8_t *xst = wst + (size_t)S * WS;            // [S][XS]
    uint8_t *ast = xst + (size_t)S * XS;            // [S][AS]
    uint64_t *bars = reinterpret_cast<uint64_t *>(ast + (size_t)S * AS);
    uint64_t *full = bars;                          // [S] producer tx
    uint64_t *empty_w = full + S;                   // [S] decoders done with raw weights
    uint64_t *full_a = empty_w + S;                 // [S] decoded tile ready
    uint64_t *mma_done = full_a + S;                // [S] MMA done with A and X
    uint64_t *acc_full = mma_done + S;              // [R]
    uint64_t *acc_empty = acc_full + R;             // [R]
    uint64_t *drain = acc_empty + R;                // [1] abort-path drain of in-flight MMAs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = p.K / KC;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty_w[s], DQ_DEC_WARPS);
            mbar_init(&full_a[s], DQ_DEC_WARPS);
            mbar_init(&mma_done[s], 1);
        }
        for (int r = 0; r < R; ++r) {
            mbar_init(&acc_full[r], 1);
            mbar_init(&acc_empty[r], DQ_EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_trigger();

    // unit u -> (matrix, tile, split)
    auto unit_of = [&](int u, int &m, int &tile, int &c0, int &c1) {
        const int per_m = p.tiles * p.ksplit;
        m = u / per_m;
        const int rem = u - m * per_m;
        tile = rem / p.ksplit;
        const int s = rem - tile * p.ksplit;
        c0 = (s * nch) / p.ksplit;
        c1 = ((s + 1) * nch) / p.ksplit;
    };

    if (warp == 0) {
        // ------------------------------- producer -------------------------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            pdl_wait();  // the activation prep of this matvec was written by the previous kernel
            int c = 0;
            for (int u = blockIdx.x; u < p.units; u += gridDim.x) {
                int m, tile, c0, c1;
                unit_of(u, m, tile, c0, c1);
                for (int kc = c0; kc < c1; ++kc, ++c) {
                    const int s = c % S, ph = c / S;
                    if (c >= S) {
                        dq_wait(&empty_w[s], (ph - 1) & 1, abort_flag, 8u);
                        dq_wait(&mma_done[s], (ph - 1) & 1, abort_flag, 8u);
                    }
                    if (*abort_flag) break;
                    DQ_TRACE(c, 0);
                    mbar_arrive_expect_tx(&full[s], WS + XS);
                    const int xk = CODEC == QW35_GF4_TYPE ? kc * (KC / 8) : kc * KC;  // element coordinate
                    tma_load_2d(wst + (size_t)s * WS, m ? &map1 : &map0, xk, tile * TM, &full[s], pol);
                    bulk_g2s(xst + (size_t)s * XS, p.xprep + (size_t)kc * XS, XS, &full[s], pol);
                }
                if (*abort_flag) break;
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer -------------------------------
        if (lane == 0) {
            int c = 0, blk = 0, ul = 0;
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x, ++ul) {
                int m, tile, c0, c1;
                unit_of(u, m, tile, c0, c1);
                const int ab = ul & 1;
                if (!BLOCKED && ul >= 2) {
                    dq_wait(&acc_empty[ab], ((ul >> 1) - 1) & 1, abort_flag, 16u);
                    tc_fence_after();
                }
                for (int kc = c0; kc < c1; ++kc, ++c) {
                    const int s = c % S, ph = c / S;
                    dq_wait(&full_a[s], ph & 1, abort_flag, 16u);
                    if (*abort_flag) break;
                    DQ_TRACE(c, 3);
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(ast + (size_t)s * AS);
                    const uint32_t x0 = smem_u32(xst + (size_t)s * XS);
#pragma unroll
                    for (int j = 0; j < KC / 16; ++j) {
                        // operands: [k-atom of 64][rows][128 B swizzled]; k-step j = 16 columns
                        const uint32_t ka = j >> 2, kofs = (j & 3) * 32;
                        const uint64_t ad = smem_desc_sw128(a0 + ka * (TM * 128) + kofs);
                        const uint64_t bd = smem_desc_sw128(x0 + ka * (2 * NP * 128) + kofs);
                        if constexpr (!BLOCKED) {
                            const uint32_t d = tmem + ab * RC;
                            tc_mma_f16(d, ad, bd, IDESC, (kc > c0 || j > 0) ? 1u : 0u);
                        } else {
                            const int r = blk % R;
                            if ((j & 1) == 0 && blk >= R) {
                                dq_wait(&acc_empty[r], ((blk / R) - 1) & 1, abort_flag, 16u);
                                tc_fence_after();
                            }
                            const uint32_t d = tmem + r * RC;
                            tc_mma_f16(d, ad, bd, IDESC, (j & 1) ? 1u : 0u);
                            if (j & 1) {
                                tc_commit(&acc_full[r]);
                                ++blk;
                            }
                        }
                    }
                    tc_commit(&mma_done[s]);
                    DQ_TRACE(c, 4);
                }
                if constexpr (!BLOCKED) tc_commit(&acc_full[ab]);
            }
        }
    } else if (warp < 2 + DQ_DEC_WARPS) {
        // -------------------------------- decoders --------------------------------
        // items (row, 16-byte piece of the row): consecutive threads take
        // consecutive pieces, so every quarter-warp reads 128 contiguous bytes
        constexpr int QPR = CODEC == QW35_GF4_TYPE ? 4 : 8;   // 16-byte pieces per row
        constexpr int NT = DQ_DEC_WARPS * 32;
        const int t = threadIdx.x - 64;
        int c = 0;
        for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
            int m, tile, c0, c1;
            unit_of(u, m, tile, c0, c1);
            for (int kc = c0; kc < c1; ++kc, ++c) {
                const int s = c % S, ph = c / S;
                dq_wait(&full[s], ph & 1, abort_flag, 32u);
                if (t == 0) DQ_TRACE(c, 1);
                if (c >= S) dq_wait(&mma_done[s], (ph - 1) & 1, abort_flag, 32u);
                if (*abort_flag) break;
                uint8_t *a = ast + (size_t)s * AS;
                const uint8_t *wst_s = wst + (size_t)s * WS;
#pragma unroll
                for (int it = t; it < TM * QPR; it += NT) {
                    // 16-item groups, each 8-lane phase conflict-free both on the
                    // staged-weight read (bank group of row*WS/TM + q*16) and on the
                    // swizzled store (chunk ^ row%8): GF4 covers rows 4g..4g+3 with
                    // row bit 1 = q bit 1 ^ phase; Q8_0 rows 2g..2g+1 with row bit 0 =
                    // q bit 2 ^ phase.
                    const int l = it & 15, ph8 = (l >> 3) & 1;
                    int r, q;
                    if constexpr (CODEC == QW35_GF4_TYPE) {
                        q = l & 3;
                        r = (it >> 4) * 4 + ((l >> 2) & 1) + 2 * ((q >> 1) ^ ph8);
                    } else {
                        q = l & 7;
                        r = (it >> 4) * 2 + ((q >> 2) ^ ph8);
                    }
                    const uint4 w4 = *reinterpret_cast<const uint4 *>(wst_s + (size_t)r * (WS / TM) + q * 16);
                    // k-block kb (8 columns) -> atom kb / 8, chunk kb % 8 of row r
                    auto aslot = [&](int kb) -> uint4 * {
                        return reinterpret_cast<uint4 *>(a + (size_t)(kb >> 3) * (TM * 128) + sw128_off(r, kb & 7));
                    };
                    if constexpr (CODEC == QW35_GF4_TYPE) {
                        uint4 o0, o1, o2, o3;
                        gf4_pair_to_halves<EXACT>(w4.x, w4.y, o0, o1);
                        gf4_pair_to_halves<EXACT>(w4.z, w4.w, o2, o3);
                        *aslot(4 * q + 0) = o0;
                        *aslot(4 * q + 1) = o1;
                        *aslot(4 * q + 2) = o2;
                        *aslot(4 * q + 3) = o3;
                    } else {
                        *aslot(2 * q) = q8_codes_to_halves(w4.x, w4.y);
                        *aslot(2 * q + 1) = q8_codes_to_halves(w4.z, w4.w);
                    }
                }
                fence_async_smem();  // generic-proxy writes -> visible to the tensor core
                __syncwarp();
                if (t == 0) DQ_TRACE(c, 2);
                if (lane == 0) {
                    mbar_arrive(&empty_w[s]);
                    mbar_arrive(&full_a[s]);
                }
            }
        }
    } else {
        // -------------------------------- epilogue --------------------------------
        // EPI/4 warps per TMEM lane quarter, each owning NP/(EPI/4) columns
        pdl_wait();  // rowscale / residual y come from earlier kernels
        constexpr int NH = NP / (DQ_EPI_WARPS / 4);
        const int ew = warp - 2 - DQ_DEC_WARPS;
        const int quarter = warp & 3;            // TMEM lane quarter this warp may access
        const int n0 = (ew >> 2) * NH;
        const int row_in_tile = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        int blk = 0, ul = 0;
        for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x, ++ul) {
            int m, tile, c0, c1;
            unit_of(u, m, tile, c0, c1);
            const int row = tile * TM + row_in_tile;
            float acc[NH];
#pragma unroll
            for (int n = 0; n < NH; ++n) acc[n] = 0.0f;
            if constexpr (!BLOCKED) {
                const int ab = ul & 1;
                dq_wait(&acc_full[ab], (ul >> 1) & 1, abort_flag, 64u);
                tc_fence_after();
#pragma unroll
                for (int part = 0; part < 2; ++part) {  // hi and lo activation products
                    float tv[NH];
                    tmem_ld_cols<NH>(tmem + lane_addr + ab * RC + part * NP + n0, tv);
#pragma unroll
                    for (int n = 0; n < NH; ++n) acc[n] += tv[n];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[ab]);
            } else {
                const uint16_t *scl = reinterpret_cast<const uint16_t *>(p.sc[m]) + (size_t)row * (p.K / 32);
                for (int kc = c0; kc < c1; ++kc) {
                    uint2 dpk = make_uint2(0, 0);
                    if (row < p.rows) dpk = *reinterpret_cast<const uint2 *>(scl + kc * 4);
                    const uint32_t dw[2] = {dpk.x, dpk.y};
#pragma unroll
                    for (int b4 = 0; b4 < 4; ++b4, ++blk) {
                        const int rg = blk % R;
                        dq_wait(&acc_full[rg], (blk / R) & 1, abort_flag, 64u);
                        tc_fence_after();
                        float tv[NH], tl[NH];
                        tmem_ld_cols<NH>(tmem + lane_addr + rg * RC + n0, tv);
                        tmem_ld_cols<NH>(tmem + lane_addr + rg * RC + NP + n0, tl);
#pragma unroll
                        for (int n = 0; n < NH; ++n) tv[n] += tl[n];
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[rg]);
                        const float d =
                            __half2float(__ushort_as_half((unsigned short)((dw[b4 >> 1] >> (16 * (b4 & 1))) & 0xffffu)));
#pragma unroll
                        for (int n = 0; n < NH; ++n) acc[n] = fmaf(d, tv[n], acc[n]);
                    }
                }
            }
            if (row < p.rows && !*abort_flag) {
                float *y = p.y[MODE == DQ_DUAL ? m : 0];
                const bool atomic = MODE == DQ_ACCUM || p.ksplit > 1;
#pragma unroll
                for (int n = 0; n < NH; ++n) {
                    if (n0 + n < p.B) {
                        const float v = acc[n] * p.rowscale[n0 + n];
                        float *dst = y + (size_t)(n0 + n) * p.rows + row;
                        if (atomic) atomicAdd(dst, v);
                        else *dst = v;
                    }
                }
            }
        }
    }

    // ---- teardown: nothing of ours may be in flight when TMEM is released ----
    if (threadIdx.x == 32 && *abort_flag) {
        // the MMA issuer drains its own tensor-core work (bounded) before TMEM goes
        tc_commit(drain);
        mbar_wait(drain, 0, 128u);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TCOLS);
}

// ---------------------------------------------------------------------------
// activation prep: RMS norm (optional), per-row power-of-two scale, f32 ->
// hi + lo halves in the MMA's K-major core-matrix layout (one CTA per padded
// batch row); zeroes the outputs that split-K accumulates into.
// ---------------------------------------------------------------------------
template <typename XT>
__global__ void __launch_bounds__(256) dq_prep_kernel(const XT *x, const float *norm_w, float eps, int K, int B, int NP,
                                                      int gf4_perm, __half *xh, __half *xl, float *rowscale,
                                                      float *zero0, float *zero1, int zero_rows) {
    __shared__ float red[32];
    const int n = blockIdx.x;
    const XT *xr = x + (size_t)(n < B ? n : 0) * K;
    float inv = 1.0f, e2 = 1.0f;
    if (n < B) {
        float ss = 0.0f;
        if (norm_w) {
            for (int k = threadIdx.x; k < K; k += 256) {
                const float v = to_f32(xr[k]);
                ss = fmaf(v, v, ss);
            }
            ss = block_sum(ss, red);
            inv = rsqrtf(ss / (float)K + eps);
        }
        float mx = 0.0f;
        for (int k = threadIdx.x; k < K; k += 256) {
            const float v = norm_w ? to_f32(xr[k]) * inv * norm_w[k] : to_f32(xr[k]);
            mx = fmaxf(mx, fabsf(v));
        }
        mx = warp_max(mx);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
        __syncthreads();
        mx = 0.0f;
        for (int i = 0; i < 8; ++i) mx = fmaxf(mx, red[i]);
        int ex = 0;
        if (mx > 0.0f && isfinite(mx)) {
            frexpf(mx, &ex);
            ex -= 15;  // max |v| * 2^-ex in [2^14, 2^15)
        }
        e2 = ldexpf(1.0f, ex);
        if (threadIdx.x == 0) rowscale[n] = e2;
        if (zero0)
            for (int r = threadIdx.x; r < zero_rows; r += 256) zero0[(size_t)n * zero_rows + r] = 0.0f;
        if (zero1)
            for (int r = threadIdx.x; r < zero_rows; r += 256) zero1[(size_t)n * zero_rows + r] = 0.0f;
    } else if (threadIdx.x == 0) {
        rowscale[n] = 1.0f;
    }
    const float rs = 1.0f / e2;  // exact power of two
    for (int k = threadIdx.x; k < K; k += 256) {
        float v = 0.0f;
        if (n < B) v = (norm_w ? to_f32(xr[k]) * inv * norm_w[k] : to_f32(xr[k])) * rs;
        const __half hi = __float2half_rn(v);
        const __half lo = __float2half_rn(v - __half2float(hi));
        // per 128-column chunk: [k-atom of 64][2*NP rows: hi rows, then lo rows][128 B swizzled]
        const int i = k & 7, kl = k & 127;
        const int slot = gf4_perm ? (i < 4 ? 2 * i : 2 * (i - 4) + 1) : i;
        const size_t base = (size_t)(k >> 7) * (2 * NP) * 128 + (size_t)(kl >> 6) * (2 * NP) * 64 + slot;
        const uint32_t c = (uint32_t)((kl & 63) >> 3);
        xh[base + sw128_off((uint32_t)n, c) / 2] = hi;
        xh[base + sw128_off((uint32_t)(NP + n), c) / 2] = lo;
    }
}

// h = silu(gate) * up over [B][rows]
__global__ void dq_swiglu_kernel(const float *g, const float *u, float *h, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        h[i] = silu_f(g[i]) * u[i];
}

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
    if (type_id == QW35_GF4_TYPE) {
        dt = CU_TENSOR_MAP_DATA_TYPE_UINT32;
        dims[0] = k / 8; dims[1] = rows; strides[0] = (cuuint64_t)k / 2;
        box[0] = KC / 8; box[1] = TM;
    } else {
        dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
        dims[0] = k; dims[1] = rows; strides[0] = k;
        box[0] = KC; box[1] = TM;
    }
    if (fn(&m, dt, 2, const_cast<void *>(w), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return false;
    cache[key] = m;
    *out = m;
    return true;
}

// Per-device scratch for the activation prep and the two-pass epilogues.
// Grows only outside stream capture (the runtime reserves it up front).
struct Scratch {
    void *ptr = nullptr;
    size_t bytes = 0;
};
std::mutex g_scratch_mu;
Scratch g_scratch[64];

cudaError_t scratch_get(size_t bytes, void **out, cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_scratch_mu);
    Scratch &s = g_scratch[dev];
    if (s.bytes < bytes) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (st) cudaStreamIsCapturing(st, &cs);
        if (cs != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return e;
        if (s.ptr) cudaFree(s.ptr);
        s.ptr = nullptr;
        s.bytes = 0;
        e = cudaMalloc(&s.ptr, bytes);
        if (e != cudaSuccess) return e;
        s.bytes = bytes;
    }
    *out = s.ptr;
    return cudaSuccess;
}

int dq_np(int B) { return B <= 16 ? 16 : (B <= 32 ? 32 : 64); }

}  // namespace

bool dq_supported(const MatvecArgs &a) {
    return a.batch >= 16 && a.batch <= 64 && (a.type_id == QW35_GF4_TYPE || a.type_id == QW35_Q8_0_TYPE) &&
           a.k % KC == 0 && encode_fn() != nullptr && !getenv("QW35_NO_TCGEN05");
}

size_t dq_scratch_bytes(int B, uint32_t k, uint32_t rows_out) {
    const int NP = dq_np(B);
    return (size_t)2 * NP * k * 2 + 256 + (size_t)2 * B * rows_out * 4 + 256;
}

cudaError_t dq_reserve(int max_batch, uint32_t max_k, uint32_t max_rows_out) {
    void *p = nullptr;
    return scratch_get(dq_scratch_bytes(max_batch, max_k, max_rows_out), &p, nullptr);
}

template <int CODEC, int NP, int MODE, bool EXACT>
static cudaError_t dq_launch(const CUtensorMap &m0, const CUtensorMap &m1, DqParams p, cudaStream_t st) {
    auto kern = dq_kernel<CODEC, NP, MODE, EXACT>;
    constexpr uint32_t stage = dq_wstage<CODEC, NP>() + dq_xstage<NP>() + dq_astage();
    const int S = (int)std::min<uint32_t>(4u, (198u * 1024u) / stage);
    const size_t smem = 1024 + (size_t)S * stage + (4 * S + 2 * dq_regions<CODEC, NP>() + 1) * 8 + 16;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    p.wbytes = dq_wstage<CODEC, NP>();
    static unsigned long long *trace = nullptr;
    if (getenv("QW35_DQ_TRACE")) {
        if (!trace) cudaMalloc(&trace, 256 * 6 * 8);
        cudaMemsetAsync(trace, 0, 256 * 6 * 8, st);
        p.trace = trace;
    }
    const int grid = std::min(p.units, qw35h::sm_count());
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DqWarps<CODEC>::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = getenv("QW35_NO_PDL") ? 0 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, m0, m1, p, S);
    if (p.trace) {
        unsigned long long h[256 * 6];
        cudaMemcpy(h, trace, sizeof(h), cudaMemcpyDeviceToHost);
        const unsigned long long t0 = h[0];
        fprintf(stderr, "dq trace units=%d grid=%d S=%d ksplit=%d (ns from first issue)\n", p.units, grid, S, p.ksplit);
        for (int c = 0; c < 256 && h[c * 6]; ++c)
            fprintf(stderr, "c%3d issue %7lld full %7lld dec %7lld mma %7lld done %7lld\n", c, (long long)(h[c * 6] - t0),
                    (long long)(h[c * 6 + 1] - t0), (long long)(h[c * 6 + 2] - t0), (long long)(h[c * 6 + 3] - t0),
                    (long long)(h[c * 6 + 4] - t0));
    }
    return e;
}

template <int CODEC, int NP>
static cudaError_t dq_dispatch_mode(int mode, bool exact, const CUtensorMap &m0, const CUtensorMap &m1,
                                    const DqParams &p, cudaStream_t st) {
    if (CODEC == QW35_GF4_TYPE && !exact) {
        if (mode == DQ_STORE) return dq_launch<CODEC, NP, DQ_STORE, false>(m0, m1, p, st);
        if (mode == DQ_ACCUM) return dq_launch<CODEC, NP, DQ_ACCUM, false>(m0, m1, p, st);
        return dq_launch<CODEC, NP, DQ_DUAL, false>(m0, m1, p, st);
    }
    if (mode == DQ_STORE) return dq_launch<CODEC, NP, DQ_STORE, true>(m0, m1, p, st);
    if (mode == DQ_ACCUM) return dq_launch<CODEC, NP, DQ_ACCUM, true>(m0, m1, p, st);
    return dq_launch<CODEC, NP, DQ_DUAL, true>(m0, m1, p, st);
}

// mode: 0 store, 1 accumulate, 2 swiglu pair, 3 logits for the argmax head
cudaError_t dq_run(const MatvecArgs &a, int mode, uint32_t *tok, float *val, cudaStream_t st) {
    const int B = a.batch, NP = dq_np(B);
    const int K = (int)a.k, rows = (int)a.rows;
    const bool dual = mode == 2;
    CUtensorMap m0, m1;
    if (!weight_map(a.type_id, a.w0, a.rows, a.k, &m0)) return cudaErrorInvalidValue;
    if (dual && !weight_map(a.type_id, a.w1, a.rows, a.k, &m1)) return cudaErrorInvalidValue;
    if (!dual) m1 = m0;
    // scratch: [xh | xl] halves, rowscale, then (swiglu) gate|up or (head) logits
    const size_t xbytes = (size_t)NP * K * 2;
    const size_t extra = (mode == 2) ? (size_t)2 * B * rows * 4 : (mode == 3 && !a.y) ? (size_t)B * rows * 4 : 0;
    void *scr = nullptr;
    cudaError_t e = scratch_get(2 * xbytes + 256 + extra + 256, &scr, st);
    if (e != cudaSuccess) return e;
    uint8_t *base = static_cast<uint8_t *>(scr);
    __half *xh = reinterpret_cast<__half *>(base);
    __half *xl = reinterpret_cast<__half *>(base + xbytes);
    float *rowscale = reinterpret_cast<float *>(base + 2 * xbytes);
    float *ext = reinterpret_cast<float *>(base + 2 * xbytes + 256);

    const int tiles = (rows + TM - 1) / TM;
    const int nch = K / KC;
    const int sms = qw35h::sm_count();
    const int per_m_tiles = tiles * (dual ? 2 : 1);
    int ksplit = (3 * sms + per_m_tiles - 1) / per_m_tiles;
    ksplit = std::max(1, std::min(ksplit, nch / 4 > 0 ? nch / 4 : 1));
    if (mode == 3) ksplit = 1;  // logits: plain stores, no atomics

    DqParams p{};
    p.xprep = base;
    p.rowscale = rowscale;
    p.rows = rows;
    p.K = K;
    p.B = B;
    p.ksplit = ksplit;
    p.tiles = tiles;
    p.units = tiles * ksplit * (dual ? 2 : 1);
    float *y0, *y1 = nullptr;
    int dmode;
    if (mode == 2) { y0 = ext; y1 = ext + (size_t)B * rows; dmode = DQ_DUAL; }
    else if (mode == 3) { y0 = a.y ? a.y : ext; dmode = DQ_STORE; }
    else { y0 = a.y; dmode = mode == 1 ? DQ_ACCUM : DQ_STORE; }
    p.y[0] = y0;
    p.y[1] = y1;
    if (a.type_id == QW35_Q8_0_TYPE) {
        p.sc[0] = static_cast<const uint8_t *>(a.w0) + (size_t)rows * K;
        p.sc[1] = dual ? static_cast<const uint8_t *>(a.w1) + (size_t)rows * K : p.sc[0];
    }
    // prep (+ zeroing of split-K outputs)
    const bool zero = dmode != DQ_ACCUM && ksplit > 1;
    const bool gperm = a.type_id == QW35_GF4_TYPE;
    if (a.x_dtype == QW35_F16_TYPE)
        dq_prep_kernel<__half><<<NP, 256, 0, st>>>(static_cast<const __half *>(a.x), a.norm_w, a.eps, K, B, NP, gperm,
                                                  xh, xl, rowscale, zero ? y0 : nullptr, zero ? y1 : nullptr, rows);
    else
        dq_prep_kernel<float><<<NP, 256, 0, st>>>(static_cast<const float *>(a.x), a.norm_w, a.eps, K, B, NP, gperm,
                                                 xh, xl, rowscale, zero ? y0 : nullptr, zero ? y1 : nullptr, rows);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const bool exact = (a.flags & QW35_MV_GF4_EXACT) != 0;
    if (a.type_id == QW35_GF4_TYPE) {
        if (NP == 16) e = dq_dispatch_mode<QW35_GF4_TYPE, 16>(dmode, exact, m0, m1, p, st);
        else if (NP == 32) e = dq_dispatch_mode<QW35_GF4_TYPE, 32>(dmode, exact, m0, m1, p, st);
        else e = dq_dispatch_mode<QW35_GF4_TYPE, 64>(dmode, exact, m0, m1, p, st);
    } else {
        if (NP == 16) e = dq_dispatch_mode<QW35_Q8_0_TYPE, 16>(dmode, true, m0, m1, p, st);
        else if (NP == 32) e = dq_dispatch_mode<QW35_Q8_0_TYPE, 32>(dmode, true, m0, m1, p, st);
        else e = dq_dispatch_mode<QW35_Q8_0_TYPE, 64>(dmode, true, m0, m1, p, st);
    }
    if (e != cudaSuccess) return e;
    if (mode == 2) {
        const size_t n = (size_t)B * rows;
        dq_swiglu_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, st>>>(y0, y1, a.y, n);
        e = cudaGetLastError();
    } else if (mode == 3) {
        dq_argmax_rows_kernel<<<B, 1024, 0, st>>>(y0, rows, tok, val);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace qw35
