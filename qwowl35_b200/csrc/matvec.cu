// matvec.cu -- fused dequantise-and-multiply for GF4 / Q8_0 / Q4_K / Q5_K / Q6_K on sm_100a.
//
// Replaces the reference's decode matvec family:
//   qw35_decode_matmul_gf4_2row[_residual]_f32   qw35_gf4.metal:99-136, :209-246
//   qw35_ffn_gate_up_swiglu_gf4_f32              qw35_gf4.metal:62-96
//   qw35_output_gf4_argmax_partials_16row_f32    qw35_gf4.metal:140-206
//   qw35_decode_matmul_q8_0[_residual]_f32       qw35_matvec.metal:630-683
//   qw35_decode_matmul_q4_k_2row[_residual]_f32  qw35_matvec.metal:171-353
//   qw35_decode_matmul_q5_k_2row_f32             qw35_matvec.metal:355-456
//   qw35_decode_matmul_q6_k_llama[_residual]_f32 qw35_matvec.metal:458-628
//   qw35_output_q6_k_argmax_partials_16row_f32   qw35_output.metal:2-139
//   qw35_output_argmax_reduce_partials_f32       qw35_output.metal:141-182
//   qw35_rms_norm_weight_f32 (fused as a prologue) qw35_core.metal:14-48
//
// B200 design.  A persistent CTA owns a contiguous range of rows.  One
// producer warp streams the packed weights of G-row groups into a ring of
// shared-memory stages with bulk copies (the TMA engine, untiled, L2
// evict-first) completing on mbarriers; it starts before the previous kernel
// has finished (programmatic dependent launch), because weights do not
// depend on it.  KW x RS consumer warps then wait for the activation row
// (griddepcontrol.wait), keep it in registers for the whole launch (lane l of
// warp kw owns the 32 columns of chunk kw*32+l), and decode every code with
// one logic op + one FMA (quant.cuh "fast decode").  Per-row partials reduce
// with warp shuffles, then across the KW warps through shared memory.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "ops.h"
#include "pipe.cuh"
#include "quant.cuh"

namespace qw35 {

enum MvMode { MV_STORE = 0, MV_ACCUM = 1, MV_SWIGLU = 2, MV_ARGMAX = 3 };

constexpr int kStages = 4;

struct MvParams {
    const uint8_t *w0;
    const uint8_t *w1;   // up matrix for MV_SWIGLU
    const void *x;       // [B][K], f32 or f16
    const float *norm_w; // fused RMS norm weight [K] or nullptr
    float eps;
    float *y;            // [B][rows] (MV_ARGMAX: optional logits)
    float *part_val;     // MV_ARGMAX partials [grid][B]
    uint32_t *part_idx;
    int rows, K, rows_per_cta, kw, rs, G;
    uint32_t code_row, scale_row;  // bytes per row in the codes / scales planes
    uint32_t stage_bytes;          // per matrix
};

template <int CODEC> struct Codec;
template <> struct Codec<QW35_GF4_TYPE> { static constexpr int NC = 8; };   // per-lane constants per b
template <> struct Codec<QW35_Q8_0_TYPE> { static constexpr int NC = 1; };
template <> struct Codec<QW35_Q4_K_TYPE> { static constexpr int NC = 2; };
template <> struct Codec<QW35_Q5_K_TYPE> { static constexpr int NC = 2; };
template <> struct Codec<QW35_Q6_K_TYPE> { static constexpr int NC = 2; };  // one per 16-weight sub-block

template <typename XT>
__device__ __forceinline__ void load_x32(float *dst, const XT *src) {
    if constexpr (sizeof(XT) == 4) {
        const float4 *p = reinterpret_cast<const float4 *>(src);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = p[i];
            dst[4 * i] = v.x; dst[4 * i + 1] = v.y; dst[4 * i + 2] = v.z; dst[4 * i + 3] = v.w;
        }
    } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(src);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = p[i];
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&u[k]));
                dst[8 * i + 2 * k] = f.x;
                dst[8 * i + 2 * k + 1] = f.y;
            }
        }
    }
}

// K-quants: turn the lane's 32 activations into the scaled form + constants
// (GF4 and Q8_0 prepare theirs in prep_x_gf4 / as pairs).
template <int CODEC, bool EXACT>
__device__ __forceinline__ void prep_x(float *xs, float *cst) {
    if constexpr (CODEC == QW35_Q6_K_TYPE) {
        // per 16-weight sub-block: the code offset of -32 subtracts 32 * sum(x)
        // (scaled like the products, see q4_word_den)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float s = 0.0f;
#pragma unroll
            for (int i = 16 * h; i < 16 * h + 16; ++i) {
                s += xs[i];
                xs[i] *= q4_den_scale(i & 7);
            }
            cst[h] = 32.0f * s * (1.0f / kKqUnscale);
        }
    } else {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            s += xs[i];
            xs[i] *= q4_den_scale(i & 7);
        }
        cst[0] = 0.0f;
        cst[1] = s * (1.0f / kKqUnscale);  // the dmin * m term
    }
}

// K-quants: dot of the lane's chunk of one row (weights in shared memory) with x.
template <int CODEC, bool EXACT>
__device__ __forceinline__ float chunk_fast(const uint8_t *codes, const uint8_t *scales, int c, const float *xs,
                                            const float *cst, int K) {
    if constexpr (CODEC == QW35_Q5_K_TYPE) {
        // chunk c is sub-block c & 7 of block c >> 3; the high bits of word w
        // sit at bit w of each nibble slot of one uint32
        const uint4 w = *reinterpret_cast<const uint4 *>(codes + c * 16);
        const uint32_t hb = *reinterpret_cast<const uint32_t *>(codes + K / 2 + c * 4);
        const uint4 h = *reinterpret_cast<const uint4 *>(scales + (c >> 3) * 16);
        float dl, ml;
        q4k_scale_min(h, c & 7, dl, ml);
        constexpr uint32_t M1 = 0x11111111u;
        float acc = q4_word_den(w.x, xs + 0, 0.0f), hacc = q4_word_den(hb & M1, xs + 0, 0.0f);
        acc = q4_word_den(w.y, xs + 8, acc);
        hacc = q4_word_den((hb >> 1) & M1, xs + 8, hacc);
        acc = q4_word_den(w.z, xs + 16, acc);
        hacc = q4_word_den((hb >> 2) & M1, xs + 16, hacc);
        acc = q4_word_den(w.w, xs + 24, acc);
        hacc = q4_word_den((hb >> 3) & M1, xs + 24, hacc);
        return (dl * fmaf(16.0f, hacc, acc) - ml * cst[1]) * kKqUnscale;
    } else if constexpr (CODEC == QW35_Q6_K_TYPE) {
        // chunk c = sub-blocks 2c, 2c+1; high pairs of 16 weights per uint32
        const uint4 w = *reinterpret_cast<const uint4 *>(codes + c * 16);
        const uint2 hb = *reinterpret_cast<const uint2 *>(codes + K / 2 + c * 8);
        const uint32_t sc2 = *reinterpret_cast<const unsigned short *>(scales + c * 2);
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(scales + K / 16 + (c >> 3) * 2)));
        constexpr uint32_t M2 = 0x33333333u;
        float a0 = q4_word_den(w.x, xs + 0, -cst[0]), a1 = q4_word_den(w.z, xs + 16, -cst[1]);
        float h0 = q4_word_den(hb.x & M2, xs + 0, 0.0f), h1 = q4_word_den(hb.y & M2, xs + 16, 0.0f);
        a0 = q4_word_den(w.y, xs + 8, a0);
        a1 = q4_word_den(w.w, xs + 24, a1);
        h0 = q4_word_den((hb.x >> 2) & M2, xs + 8, h0);
        h1 = q4_word_den((hb.y >> 2) & M2, xs + 24, h1);
        const float s0 = (float)(int8_t)(sc2 & 0xffu), s1 = (float)(int8_t)(sc2 >> 8);
        return d * fmaf(s0, fmaf(16.0f, h0, a0), s1 * fmaf(16.0f, h1, a1)) * kKqUnscale;
    } else {
        const uint4 w = *reinterpret_cast<const uint4 *>(codes + c * 16);
        const uint4 h = *reinterpret_cast<const uint4 *>(scales + (c >> 3) * 16);
        float dl, ml;
        q4k_scale_min(h, c & 7, dl, ml);
        const float a = q4_word_den(w.y, xs + 8, q4_word_den(w.x, xs + 0, 0.0f));
        const float c = q4_word_den(w.w, xs + 24, q4_word_den(w.z, xs + 16, 0.0f));
        return (dl * (a + c) - ml * cst[1]) * kKqUnscale;
    }
}

// Sum each of NV per-lane values over the warp with a butterfly reduce-scatter:
// the first log2(NV) exchange steps halve the values a lane keeps (one shuffle
// per kept pair instead of one per value and step), the rest are plain
// butterfly steps.  Returns the total of value mv_scatter_index<NV>(lane).
template <int NV>
__device__ __forceinline__ float warp_reduce_scatter(float *v, int lane) {
#pragma unroll
    for (int st = 0; (1 << st) < NV; ++st) {
        const int o = 16 >> st, n = NV >> (st + 1);
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < n; ++j) {
            const float send = up ? v[j] : v[j + n];
            const float keep = up ? v[j + n] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float t = v[0];
#pragma unroll
    for (int o = 16 / NV; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

template <int NV>
__device__ __forceinline__ int mv_scatter_index(int lane) {
    int idx = 0;
#pragma unroll
    for (int st = 0; (1 << st) < NV; ++st)
        if (lane & (16 >> st)) idx += NV >> (st + 1);
    return idx;
}

// GF4 / Q8_0 rows per consumer warp per stage (the stage holds G = rows * RS rows)
template <int CODEC, int MODE> constexpr int rows_per_warp() {
    return CODEC == QW35_GF4_TYPE ? (MODE == 2 ? 2 : 4) : (MODE == 2 ? 1 : 2);
}
// Consumer warps per CTA (at most; Q8_0 takes 8 where it can, see mv_geometry)
template <int B> constexpr int mv_max_warps() { return 12; }
// 32-column chunks each consumer lane owns (its activations stay in registers):
// two for batch-1 GF4, which halves the per-row reduction work per weight
template <int CODEC, int B> constexpr int mv_lane_chunks() { return 1; }

// Shared-memory carve-up (dynamic): [NM][kStages][stage_bytes] weights |
// [row of the CTA][B][NM][KW] partials | 64 floats scratch | 2*kStages
// mbarriers | abort.  Each consumer warp writes its own partial slot of every
// row it handles (no stage-wide barrier); the rows are summed in a fixed order
// and written once, after the last stage.
template <int CODEC, int B, int MODE, bool EXACT, typename XT>
__global__ void __launch_bounds__((mv_max_warps<B>() + 1) * 32, 1) mv_kernel(MvParams p) {
    constexpr int NM = MODE == MV_SWIGLU ? 2 : 1;
    constexpr int NC = Codec<CODEC>::NC;
    extern __shared__ __align__(128) uint8_t smem[];

    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int KW = p.kw, RS = p.rs, G = p.G;
    const int ncw = KW * RS;  // consumer warps
    const int ncons = ncw * 32;
    const uint32_t SB = p.stage_bytes;
    uint8_t *wbuf = smem;
    float *part = reinterpret_cast<float *>(smem + (size_t)NM * kStages * SB);
    // contiguous, balanced split of the row groups over the grid
    const int groups_total = (p.rows + G - 1) / G;
    const int max_rows = (groups_total + gridDim.x - 1) / gridDim.x * G;
    float *red = part + (size_t)max_rows * B * NM * KW;
    uint64_t *full = reinterpret_cast<uint64_t *>(red + 64);
    uint64_t *empty = full + kStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kStages);

    const int g0 = (int)(((long long)blockIdx.x * groups_total) / gridDim.x);
    const int g1 = (int)(((long long)(blockIdx.x + 1) * groups_total) / gridDim.x);
    const int r0 = g0 * G;
    const int r1 = min(p.rows, g1 * G);
    const int ngroups = g1 - g0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ncw);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    pdl_trigger();

    if (wid == ncw) {
        // ------------------------------ producer ---------------------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            const uint8_t *mats[2] = {p.w0, p.w1};
            const size_t codes_plane = (size_t)p.rows * p.code_row;
            int issued = 0;
            for (int g = 0; g < ngroups; ++g) {
                const int s = g % kStages;
                if (g >= kStages && !*abort_flag) {
                    if (!mbar_wait(&empty[s], ((g / kStages) - 1) & 1, 1u)) *abort_flag = 1;
                }
                if (*abort_flag) break;
                const int row0 = r0 + g * G;
                const int nr = min(G, r1 - row0);
                const uint32_t cb = nr * p.code_row, sbytes = nr * p.scale_row;
                mbar_arrive_expect_tx(&full[s], NM * (cb + sbytes));
#pragma unroll
                for (int m = 0; m < NM; ++m) {
                    uint8_t *dst = wbuf + ((size_t)m * kStages + s) * SB;
                    bulk_g2s(dst, mats[m] + (size_t)row0 * p.code_row, cb, &full[s], pol);
                    if (sbytes)
                        bulk_g2s(dst + (size_t)G * p.code_row, mats[m] + codes_plane + (size_t)row0 * p.scale_row,
                                 sbytes, &full[s], pol);
                }
                issued = g + 1;
            }
            if (*abort_flag) {  // never leave with copies in flight
                for (int g = max(0, issued - kStages); g < issued; ++g)
                    mbar_wait(&full[g % kStages], (g / kStages) & 1, 4u);
            }
        }
        return;
    }

    // -------------------------------- consumers ------------------------------
    constexpr int LC = mv_lane_chunks<CODEC, B>();
    const int kw = wid % KW, rs = wid / KW;
    const int nchunk = p.K / (32 * LC);
    const int c = kw * 32 + lane;  // the lane's columns: [c * 32 * LC, (c + 1) * 32 * LC)
    const bool active = c < nchunk;
    pdl_wait();  // the activation row is written by the previous kernel

    float xs[B][32 * LC];
    float cst[B][NC];
    const XT *xg = reinterpret_cast<const XT *>(p.x);
#pragma unroll
    for (int b = 0; b < B; ++b) {
#pragma unroll
        for (int q = 0; q < LC; ++q) {
            if (active) {
                load_x32<XT>(xs[b] + 32 * q, xg + (size_t)b * p.K + ((size_t)c * LC + q) * 32);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) xs[b][32 * q + i] = 0.0f;
            }
        }
    }
    if (p.norm_w != nullptr) {
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < 32 * LC; ++i) ss = fmaf(xs[b][i], xs[b][i], ss);
            ss = warp_sum(ss);
            if (lane == 0 && rs == 0) red[kw] = ss;
            named_sync(1, ncons);
            float tot = 0.0f;
            for (int i = 0; i < KW; ++i) tot += red[i];
            named_sync(1, ncons);
            const float inv = rsqrtf(tot / (float)p.K + p.eps);
            if (active) {
                const float4 *nw = reinterpret_cast<const float4 *>(p.norm_w + (size_t)c * 32 * LC);
#pragma unroll
                for (int i = 0; i < 8 * LC; ++i) {
                    const float4 w4 = __ldg(nw + i);
                    xs[b][4 * i] = xs[b][4 * i] * inv * w4.x;
                    xs[b][4 * i + 1] = xs[b][4 * i + 1] * inv * w4.y;
                    xs[b][4 * i + 2] = xs[b][4 * i + 2] * inv * w4.z;
                    xs[b][4 * i + 3] = xs[b][4 * i + 3] * inv * w4.w;
                }
            }
        }
    }
    // GF4: activations as scaled pairs for the packed exact-level decode
    float2 xp[B][16 * LC];
    float xa[B][4 * LC], xj[B][4 * LC];
    if constexpr (CODEC == QW35_GF4_TYPE) {
        prep_x_gf4<B, 4 * LC>(xs, xp, xa, xj);
    } else if constexpr (CODEC == QW35_Q8_0_TYPE) {
#pragma unroll
        for (int b = 0; b < B; ++b)
#pragma unroll
            for (int i = 0; i < 16; ++i) xp[b][i] = make_float2(xs[b][2 * i], xs[b][2 * i + 1]);
    } else {
#pragma unroll
        for (int b = 0; b < B; ++b) prep_x<CODEC, EXACT>(xs[b], cst[b]);
    }


    for (int g = 0; g < ngroups; ++g) {
        const int s = g % kStages;
        if (!*abort_flag) {
            if (!mbar_wait(&full[s], (g / kStages) & 1, 2u)) *abort_flag = 1;
        }
        const int nr = min(G, r1 - (r0 + g * G));
        float *pg = part + (size_t)g * G * B * NM * KW;  // this stage's rows
        if constexpr (CODEC == QW35_GF4_TYPE || CODEC == QW35_Q8_0_TYPE) {
            // this warp's rows of the stage: rs + j * RS, all in flight at once;
            // rows past nr run on stale stage bytes and are never stored
            constexpr int NRW = rows_per_warp<CODEC, MODE>();
            constexpr int NV = NRW * NM * B;
            float v[NV];
            const int cc = active ? c : 0;
#pragma unroll
            for (int j = 0; j < NRW; ++j) {
                const int i = rs + j * RS;
#pragma unroll
                for (int m = 0; m < NM; ++m) {
                    const uint8_t *st = wbuf + ((size_t)m * kStages + s) * SB;
                    if constexpr (CODEC == QW35_GF4_TYPE) {
                        float2 r2[B];
#pragma unroll
                        for (int b = 0; b < B; ++b) r2[b] = make_float2(0.0f, 0.0f);
#pragma unroll
                        for (int q = 0; q < LC; ++q) {
                            const uint4 wv = *reinterpret_cast<const uint4 *>(st + (size_t)i * p.code_row + (cc * LC + q) * 16);
                            gf4_word_f2<EXACT, B, 16 * LC, 4 * LC>(wv.x, 4 * q + 0, xp, xa, xj, r2);
                            gf4_word_f2<EXACT, B, 16 * LC, 4 * LC>(wv.y, 4 * q + 1, xp, xa, xj, r2);
                            gf4_word_f2<EXACT, B, 16 * LC, 4 * LC>(wv.z, 4 * q + 2, xp, xa, xj, r2);
                            gf4_word_f2<EXACT, B, 16 * LC, 4 * LC>(wv.w, 4 * q + 3, xp, xa, xj, r2);
                        }
#pragma unroll
                        for (int b = 0; b < B; ++b) v[(j * NM + m) * B + b] = active ? (r2[b].x + r2[b].y) * kGf4Unscale : 0.0f;
                    } else {
                        const uint8_t *codes = st + (size_t)i * p.code_row + cc * 32;
                        const uint4 a0 = *reinterpret_cast<const uint4 *>(codes);
                        const uint4 a1 = *reinterpret_cast<const uint4 *>(codes + 16);
                        const unsigned short sb = *reinterpret_cast<const unsigned short *>(
                            st + (size_t)G * p.code_row + (size_t)i * p.scale_row + cc * 2);
                        float r[B];
#pragma unroll
                        for (int b = 0; b < B; ++b) r[b] = 0.0f;
                        q8_block_f2<B>(a0, a1, __half2float(__ushort_as_half(sb)), xp, r);
#pragma unroll
                        for (int b = 0; b < B; ++b) v[(j * NM + m) * B + b] = active ? r[b] : 0.0f;
                    }
                }
            }
            const float tot = warp_reduce_scatter<NV>(v, lane);
            if ((lane & (32 / NV - 1)) == 0) {
                const int idx = mv_scatter_index<NV>(lane);
                const int b = idx % B, m = (idx / B) % NM, j = idx / (B * NM);
                pg[(((rs + j * RS) * B + b) * NM + m) * KW + kw] = tot;
            }
        } else
        for (int i = rs; i < G; i += RS) {
            float acc[NM][B];
#pragma unroll
            for (int m = 0; m < NM; ++m) {
                const uint8_t *st = wbuf + ((size_t)m * kStages + s) * SB;
                const uint8_t *codes = st + (size_t)i * p.code_row;
                const uint8_t *scales = st + (size_t)G * p.code_row + (size_t)i * p.scale_row;
#pragma unroll
                for (int b = 0; b < B; ++b)
                    acc[m][b] = (active && i < nr) ? chunk_fast<CODEC, EXACT>(codes, scales, c, xs[b], cst[b], p.K) : 0.0f;
            }
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float v = warp_sum(acc[m][b]);
                    if (lane == 0) pg[((i * B + b) * NM + m) * KW + kw] = v;
                }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage
    }

    // ---- the CTA's rows: partials summed in a fixed order, written once ----
    named_sync(1, ncons);
    const int nrows = r1 - r0;
    float best_v[B];
    uint32_t best_i[B];
#pragma unroll
    for (int b = 0; b < B; ++b) { best_v[b] = -INFINITY; best_i[b] = 0xffffffffu; }
    for (int t = threadIdx.x; t < nrows * B; t += ncons) {
        const int b = t / nrows, rr = t - b * nrows;  // consecutive threads: consecutive rows
        const float *pp = part + ((size_t)rr * B + b) * NM * KW;
        float s0 = 0.0f;
        for (int k = 0; k < KW; ++k) s0 += pp[k];
        float *yo = p.y + (size_t)b * p.rows + r0 + rr;
        if constexpr (MODE == MV_STORE) {
            *yo = s0;
        } else if constexpr (MODE == MV_ACCUM) {
            *yo += s0;
        } else if constexpr (MODE == MV_SWIGLU) {
            float s1 = 0.0f;
            for (int k = 0; k < KW; ++k) s1 += pp[KW + k];
            *yo = silu_f(s0) * s1;
        } else {
            if (p.y != nullptr) *yo = s0;
            // a thread's rows ascend within each batch row: keeps the lowest id on ties
#pragma unroll
            for (int bb = 0; bb < B; ++bb)
                if (bb == b && s0 > best_v[bb]) { best_v[bb] = s0; best_i[bb] = (uint32_t)(r0 + rr); }
        }
    }

    if constexpr (MODE == MV_ARGMAX) {
        // per batch row: (max, lowest id) over the warp by shuffles, then over the
        // consumer warps through shared memory (ncw * B <= 32 slots)
        float *bv = red;
        uint32_t *bi = reinterpret_cast<uint32_t *>(red + 32);
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float v = best_v[b];
            uint32_t id = best_i[b];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, id, o);
                if (ov > v || (ov == v && oi < id)) { v = ov; id = oi; }
            }
            if (lane == 0) { bv[wid * B + b] = v; bi[wid * B + b] = id; }
        }
        named_sync(1, ncons);
        if ((int)threadIdx.x < B) {
            float v = -INFINITY;
            uint32_t id = 0xffffffffu;
            for (int w = 0; w < ncw; ++w) {
                const float tv = bv[w * B + threadIdx.x];
                const uint32_t ti = bi[w * B + threadIdx.x];
                if (tv > v || (tv == v && ti < id)) { v = tv; id = ti; }
            }
            p.part_val[(size_t)blockIdx.x * B + threadIdx.x] = v;
            p.part_idx[(size_t)blockIdx.x * B + threadIdx.x] = id;
        }
    }
}

// Final argmax over per-CTA partials; ties resolve to the smallest id
// (qw35_output.metal:141-182).  One CTA of 256 threads per batch row.
__global__ void argmax_reduce_kernel(const float *pv, const uint32_t *pi, int n, int B, uint32_t *out_tok,
                                     float *out_val) {
    __shared__ float sv[256];
    __shared__ uint32_t si[256];
    const int b = blockIdx.x;
    float v = -INFINITY;
    uint32_t id = 0xffffffffu;
    for (int i = threadIdx.x; i < n; i += 256) {
        const float tv = pv[(size_t)i * B + b];
        const uint32_t ti = pi[(size_t)i * B + b];
        if (tv > v || (tv == v && ti < id)) { v = tv; id = ti; }
    }
    sv[threadIdx.x] = v;
    si[threadIdx.x] = id;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if ((int)threadIdx.x < s) {
            const float rv = sv[threadIdx.x + s];
            const uint32_t ri = si[threadIdx.x + s];
            if (rv > sv[threadIdx.x] || (rv == sv[threadIdx.x] && ri < si[threadIdx.x])) {
                sv[threadIdx.x] = rv;
                si[threadIdx.x] = ri;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        out_tok[b] = si[0];
        if (out_val) out_val[b] = sv[0];
    }
}

// ---------------------------------------------------------------------------
// host-side launch
// ---------------------------------------------------------------------------
struct MvGeom {
    int kw, rs, G, threads, ctas, rows_per_cta;
    uint32_t code_row, scale_row, stage_bytes;
    size_t smem;
};

static void codec_rows(uint32_t type_id, int K, uint32_t &code_row, uint32_t &scale_row) {
    if (type_id == QW35_GF4_TYPE) { code_row = K / 2; scale_row = 0; }
    else if (type_id == QW35_Q8_0_TYPE) { code_row = K; scale_row = K / 16; }
    else if (type_id == QW35_Q5_K_TYPE) { code_row = K / 2 + K / 8; scale_row = K / 16; }
    else if (type_id == QW35_Q6_K_TYPE) { code_row = K / 2 + K / 4; scale_row = q6k_scale_row(K); }
    else { code_row = K / 2; scale_row = K / 16; }
}

template <int CODEC, int B, int MODE>
static MvGeom mv_geometry(int rows, int K, const void *kern) {
    constexpr int NM = MODE == MV_SWIGLU ? 2 : 1;
    MvGeom g;
    const int nchunk = K / (32 * mv_lane_chunks<CODEC, B>());
    g.kw = (nchunk + 31) / 32;
    codec_rows(CODEC, K, g.code_row, g.scale_row);
    const uint32_t rb = g.code_row + g.scale_row;
    if (CODEC == QW35_GF4_TYPE || CODEC == QW35_Q8_0_TYPE) {
        // up to mv_max_warps consumer warps, each with rows_per_warp rows of a stage
        // in flight; Q8_0 (80 registers) takes 8 where its K allows, so two CTAs
        // share an SM (measured: 12352 x 4096 11.8 -> 10.9 us, head 174 -> 159 us)
        const int CW = (CODEC == QW35_Q8_0_TYPE && g.kw <= 8) ? 8 : mv_max_warps<B>();
        g.rs = g.kw >= CW ? 1 : CW / g.kw;
        g.G = rows_per_warp<CODEC, MODE>() * g.rs;
    } else {
        g.rs = g.kw >= 8 ? 1 : 8 / g.kw;
        g.G = (int)(20 * 1024 / rb);
    }
    g.threads = (g.kw * g.rs + 1) * 32;
    if (CODEC != QW35_GF4_TYPE && CODEC != QW35_Q8_0_TYPE) g.G = g.G < 1 ? 1 : (g.G > 16 ? 16 : g.G);
    g.stage_bytes = ((uint32_t)g.G * rb + 127u) & ~127u;
    // stages + 64 floats + mbarriers, then the CTA's row partials, which depend
    // on the grid (rows per CTA): sized for the grid the occupancy allows
    const size_t base = (size_t)NM * kStages * g.stage_bytes + 64 * 4 + 2 * kStages * 8 + 16;
    const int groups = (rows + g.G - 1) / g.G;
    auto part_bytes = [&](int ctas) {
        return (size_t)((groups + ctas - 1) / ctas) * g.G * B * NM * g.kw * 4;
    };
    int occ = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, g.threads, base);
    if (occ < 1) occ = 1;
    g.ctas = std::min(groups, qw35h::sm_count() * occ);
    g.smem = base + part_bytes(g.ctas);
    int occ2 = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ2, kern, g.threads, g.smem);
    if (occ2 < 1) occ2 = 1;
    if (occ2 < occ) {
        g.ctas = std::min(groups, qw35h::sm_count() * occ2);
        g.smem = base + part_bytes(g.ctas);
    }
    g.rows_per_cta = 0;  // the kernel splits the groups evenly over the grid
    return g;
}

template <int CODEC, int B, int MODE, bool EXACT, typename XT>
static cudaError_t mv_launch(MvParams p, cudaStream_t st, int *ctas_out) {
    auto kern = mv_kernel<CODEC, B, MODE, EXACT, XT>;
    {
        cudaError_t e = qw35h::smem_optin((const void *)kern, 200 * 1024);
        if (e != cudaSuccess) return e;
    }
    MvGeom g = mv_geometry<CODEC, B, MODE>(p.rows, p.K, (const void *)kern);
    if (g.kw > 12 || g.smem > 200 * 1024) return cudaErrorInvalidValue;
    if (MODE == MV_ARGMAX && (p.part_val == nullptr || g.kw * g.rs * B > 32)) return cudaErrorInvalidValue;
    p.kw = g.kw;
    p.rs = g.rs;
    p.G = g.G;
    p.rows_per_cta = g.rows_per_cta;
    p.code_row = g.code_row;
    p.scale_row = g.scale_row;
    p.stage_bytes = g.stage_bytes;
    if (ctas_out) *ctas_out = g.ctas;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(g.ctas);
    cfg.blockDim = dim3(g.threads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    static const bool no_pdl = getenv("QW35_NO_PDL") != nullptr;
    cfg.attrs = attr;
    cfg.numAttrs = no_pdl ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int CODEC, int MODE, bool EXACT, typename XT>
static cudaError_t mv_dispatch_b(MvParams p, int B, cudaStream_t st, int *ctas) {
    switch (B) {
        case 1: return mv_launch<CODEC, 1, MODE, EXACT, XT>(p, st, ctas);
        case 2: return mv_launch<CODEC, 2, MODE, EXACT, XT>(p, st, ctas);
        default: return cudaErrorInvalidValue;
    }
}

template <int MODE, bool EXACT, typename XT>
static cudaError_t mv_dispatch_codec(uint32_t type_id, MvParams p, int B, cudaStream_t st, int *ctas) {
    switch (type_id) {
        case QW35_GF4_TYPE: return mv_dispatch_b<QW35_GF4_TYPE, MODE, EXACT, XT>(p, B, st, ctas);
        case QW35_Q8_0_TYPE: return mv_dispatch_b<QW35_Q8_0_TYPE, MODE, true, XT>(p, B, st, ctas);
        case QW35_Q4_K_TYPE: return mv_dispatch_b<QW35_Q4_K_TYPE, MODE, true, XT>(p, B, st, ctas);
        case QW35_Q5_K_TYPE: return mv_dispatch_b<QW35_Q5_K_TYPE, MODE, true, XT>(p, B, st, ctas);
        case QW35_Q6_K_TYPE: return mv_dispatch_b<QW35_Q6_K_TYPE, MODE, true, XT>(p, B, st, ctas);
        default: return cudaErrorInvalidValue;
    }
}

template <int MODE>
static cudaError_t mv_dispatch(const MatvecArgs &a, MvParams p, int B, cudaStream_t st, int *ctas) {
    const bool exact = (a.flags & QW35_MV_GF4_EXACT) != 0;
    if (a.x_dtype == QW35_F16_TYPE) {
        return exact ? mv_dispatch_codec<MODE, true, __half>(a.type_id, p, B, st, ctas)
                     : mv_dispatch_codec<MODE, false, __half>(a.type_id, p, B, st, ctas);
    }
    return exact ? mv_dispatch_codec<MODE, true, float>(a.type_id, p, B, st, ctas)
                 : mv_dispatch_codec<MODE, false, float>(a.type_id, p, B, st, ctas);
}

static MvParams base_params(const MatvecArgs &a, int b0) {
    const size_t xes = a.x_dtype == QW35_F16_TYPE ? 2 : 4;
    MvParams p{};
    p.w0 = static_cast<const uint8_t *>(a.w0);
    p.w1 = static_cast<const uint8_t *>(a.w1);
    p.x = static_cast<const uint8_t *>(a.x) + (size_t)b0 * a.k * xes;
    p.norm_w = a.norm_w;
    p.eps = a.eps;
    p.y = a.y ? a.y + (size_t)b0 * a.rows : nullptr;
    p.rows = (int)a.rows;
    p.K = (int)a.k;
    return p;
}

// Batch rows beyond the register-resident tile of two are processed in tiles
// of two; each tile re-reads the weights (from L2 when they fit).
cudaError_t matvec_run(const MatvecArgs &a, cudaStream_t st) {
    if (dq_supported(a)) return dq_run(a, a.mode, nullptr, nullptr, st);  // tensor-core path, B >= kDqMinBatch
    for (int b0 = 0; b0 < a.batch; b0 += 2) {
        const int nb = a.batch - b0 < 2 ? a.batch - b0 : 2;
        MvParams p = base_params(a, b0);
        cudaError_t e;
        switch (a.mode) {
            case MV_STORE: e = mv_dispatch<MV_STORE>(a, p, nb, st, nullptr); break;
            case MV_ACCUM: e = mv_dispatch<MV_ACCUM>(a, p, nb, st, nullptr); break;
            case MV_SWIGLU: e = mv_dispatch<MV_SWIGLU>(a, p, nb, st, nullptr); break;
            default: return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

size_t argmax_workspace_bytes(uint32_t rows, uint32_t batch) {
    (void)rows;
    (void)batch;
    const size_t n = (size_t)qw35h::sm_count() * 8;  // >= any persistent grid of the head
    return 2 * n * 2 * sizeof(float) + 256;          // two halves of [n][2]: values | indices
}

cudaError_t argmax_head_run(const MatvecArgs &a, uint32_t *tok, float *val, void *ws, size_t ws_bytes,
                            cudaStream_t st) {
    if (ws_bytes < argmax_workspace_bytes(a.rows, a.batch)) return cudaErrorInvalidValue;
    if (dq_supported(a)) return dq_run(a, 3, tok, val, st);  // tensor-core path, B >= kDqMinBatch
    const size_t half_ws = ws_bytes / 2;
    for (int b0 = 0; b0 < a.batch; b0 += 2) {
        const int nb = a.batch - b0 < 2 ? a.batch - b0 : 2;
        MvParams p = base_params(a, b0);
        p.part_val = static_cast<float *>(ws);
        p.part_idx = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(ws) + half_ws);
        int ctas = 0;
        cudaError_t e = mv_dispatch<MV_ARGMAX>(a, p, nb, st, &ctas);
        if (e != cudaSuccess) return e;
        if ((size_t)ctas * nb * 4 > half_ws) return cudaErrorInvalidValue;
        argmax_reduce_kernel<<<nb, 256, 0, st>>>(p.part_val, p.part_idx, ctas, nb, tok + b0, val ? val + b0 : nullptr);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

unsigned int device_error_read_and_clear() {
    unsigned int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(v));
    if (v) cudaMemcpyToSymbol(g_dev_error, &z, sizeof(z));
    return v;
}

}  // namespace qw35
