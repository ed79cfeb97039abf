// matvec.cu -- fused dequantise-and-multiply for GF4 / Q8_0 / Q4_K on sm_100a.
//
// Replaces the reference's decode matvec family:
//   qw35_decode_matmul_gf4_2row[_residual]_f32   qw35_gf4.metal:99-136, :209-246
//   qw35_ffn_gate_up_swiglu_gf4_f32              qw35_gf4.metal:62-96
//   qw35_output_gf4_argmax_partials_16row_f32    qw35_gf4.metal:140-206
//   qw35_decode_matmul_q8_0[_residual]_f32       qw35_matvec.metal:630-683
//   qw35_decode_matmul_q4_k_2row[_residual]_f32  qw35_matvec.metal:171-353
//   qw35_output_argmax_reduce_partials_f32       qw35_output.metal:141-182
//   qw35_rms_norm_weight_f32 (fused as a prologue) qw35_core.metal:14-48
//
// Design (B200): the activation row stays in REGISTERS for the whole launch.
// A CTA is KW x RS warps: KW warps span K (lane l of warp kw owns the 32
// consecutive columns of chunk kw*32+l), RS independent row streams walk the
// CTA's contiguous row range in groups of G rows.  Every weight byte is
// loaded exactly once with a 128-bit non-allocating load; x is read once per
// CTA (not once per row), so the only steady-state traffic is the weight
// stream.  Per-row partials reduce with warp shuffles, then across the KW
// warps through shared memory.  The grid is persistent (<= resident CTAs),
// rows are split evenly across CTAs.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "quant.cuh"
#include "ops.h"

namespace qw35 {

enum MvMode { MV_STORE = 0, MV_ACCUM = 1, MV_SWIGLU = 2, MV_ARGMAX = 3 };

struct MvParams {
    const uint8_t *w0;
    const uint8_t *w1;   // up matrix for MV_SWIGLU
    const void *x;       // [B][K], f32 or f16
    const float *norm_w; // fused RMS norm weight [K] or nullptr
    float eps;
    float *y;            // [B][rows] (MV_ARGMAX: optional logits)
    float *part_val;     // MV_ARGMAX partials [grid][B]
    uint32_t *part_idx;
    int rows, K, rows_per_cta, kw;
};

template <int CODEC> struct CodecTraits;
template <> struct CodecTraits<QW35_GF4_TYPE> { static constexpr int G = 8; };
template <> struct CodecTraits<QW35_Q8_0_TYPE> { static constexpr int G = 4; };
template <> struct CodecTraits<QW35_Q4_K_TYPE> { static constexpr int G = 8; };

template <int CODEC>
struct ChunkLoad {
    uint4 a, b;      // codes (b only for Q8_0)
    uint32_t s;      // Q8_0 fp16 scale bits
    uint4 h;         // Q4_K header
};

template <int CODEC>
__device__ __forceinline__ void load_chunk(ChunkLoad<CODEC> &L, const uint8_t *w, int rows, int K, int row, int c) {
    if constexpr (CODEC == QW35_GF4_TYPE) {
        L.a = ldg_stream(w + (size_t)row * (K / 2) + (size_t)c * 16);
    } else if constexpr (CODEC == QW35_Q8_0_TYPE) {
        const uint8_t *codes = w + (size_t)row * K + (size_t)c * 32;
        L.a = ldg_stream(codes);
        L.b = ldg_stream(codes + 16);
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(w + (size_t)rows * K);
        L.s = __ldg(sc + (size_t)row * (K / 32) + c);
    } else {
        L.a = ldg_stream(w + (size_t)row * (K / 2) + (size_t)c * 16);
        const uint8_t *hdr = w + (size_t)rows * (K / 2) + ((size_t)row * (K / 256) + (c >> 3)) * 16;
        L.h = __ldg(reinterpret_cast<const uint4 *>(hdr));
    }
}

template <int CODEC, bool EXACT>
__device__ __forceinline__ float chunk_dot(const ChunkLoad<CODEC> &L, const float *x, const float *aux, int c) {
    if constexpr (CODEC == QW35_GF4_TYPE) {
        // aux[0..3] = 4*sum(x) per word, aux[4..7] = x_4 * 2^-13 per word
        float r = gf4_word_dot<EXACT>(L.a.x, x + 0, aux[0], aux[4]);
        r += gf4_word_dot<EXACT>(L.a.y, x + 8, aux[1], aux[5]);
        r += gf4_word_dot<EXACT>(L.a.z, x + 16, aux[2], aux[6]);
        r += gf4_word_dot<EXACT>(L.a.w, x + 24, aux[3], aux[7]);
        return r;
    } else if constexpr (CODEC == QW35_Q8_0_TYPE) {
        const float d = __half2float(__ushort_as_half((unsigned short)L.s));
        return q8_chunk_dot(L.a, L.b, x) * d;
    } else {
        float dl, ml;
        q4k_scale_min(L.h, c & 7, dl, ml);
        float acc = q4_word_dot(L.a.x, x + 0);
        acc += q4_word_dot(L.a.y, x + 8);
        acc += q4_word_dot(L.a.z, x + 16);
        acc += q4_word_dot(L.a.w, x + 24);
        return dl * acc - ml * aux[0];  // aux[0] = sum of the chunk's x
    }
}

template <typename XT>
__device__ __forceinline__ void load_x32(float *dst, const XT *src) {
    if constexpr (sizeof(XT) == 4) {
        const float4 *p = reinterpret_cast<const float4 *>(src);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = __ldg(p + i);
            dst[4 * i] = v.x; dst[4 * i + 1] = v.y; dst[4 * i + 2] = v.z; dst[4 * i + 3] = v.w;
        }
    } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(src);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = __ldg(p + i);
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

constexpr int kMaxKW = 16;

template <int CODEC, int B, int MODE, bool EXACT, typename XT>
__global__ void __launch_bounds__(384) mv_kernel(MvParams p) {
    constexpr int G = CodecTraits<CODEC>::G;
    constexpr int NM = MODE == MV_SWIGLU ? 2 : 1;
    constexpr int NAUX = CODEC == QW35_GF4_TYPE ? 8 : 1;
    extern __shared__ float smem[];  // [2 buf][RS][G][B][NM][KW] partials + 32 scratch

    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int KW = p.kw;
    const int RS = (blockDim.x >> 5) / KW;
    const int kw = wid % KW;
    const int stream = wid / KW;
    const int nchunk = p.K >> 5;
    const int c = kw * 32 + lane;
    const bool active = c < nchunk;
    float *red = smem + 2 * RS * G * B * NM * KW;  // 32 + B floats of scratch

    // ---- x (+ fused RMS norm) into registers -------------------------------
    float xr[B][32];
    float aux[B][NAUX];
    const XT *xg = reinterpret_cast<const XT *>(p.x);
#pragma unroll
    for (int b = 0; b < B; ++b) {
        if (active) {
            load_x32<XT>(xr[b], xg + (size_t)b * p.K + (size_t)c * 32);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) xr[b][i] = 0.0f;
        }
    }
    if (p.norm_w != nullptr) {
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) ss = fmaf(xr[b][i], xr[b][i], ss);
            ss = warp_sum(ss);
            if (lane == 0 && stream == 0) red[kw] = ss;
            __syncthreads();
            float tot = 0.0f;
            for (int i = 0; i < KW; ++i) tot += red[i];
            __syncthreads();
            const float inv = rsqrtf(tot / (float)p.K + p.eps);
            if (active) {
                const float4 *nw = reinterpret_cast<const float4 *>(p.norm_w + (size_t)c * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 w4 = __ldg(nw + i);
                    xr[b][4 * i] = xr[b][4 * i] * inv * w4.x;
                    xr[b][4 * i + 1] = xr[b][4 * i + 1] * inv * w4.y;
                    xr[b][4 * i + 2] = xr[b][4 * i + 2] * inv * w4.z;
                    xr[b][4 * i + 3] = xr[b][4 * i + 3] * inv * w4.w;
                }
            }
        }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
        if constexpr (CODEC == QW35_GF4_TYPE) {
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j) s += xr[b][8 * wd + j];
                aux[b][wd] = 4.0f * s;
                aux[b][4 + wd] = xr[b][8 * wd + 4] * 0.0001220703125f;
            }
        } else {
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) s += xr[b][i];
            aux[b][0] = s;
        }
    }

    // ---- stream the CTA's rows -------------------------------------------
    const int r0 = blockIdx.x * p.rows_per_cta;
    const int r1 = min(p.rows, r0 + p.rows_per_cta);
    const int iters = (p.rows_per_cta + RS * G - 1) / (RS * G);
    float best_v[B];
    uint32_t best_i[B];
#pragma unroll
    for (int b = 0; b < B; ++b) { best_v[b] = -INFINITY; best_i[b] = 0xffffffffu; }
    const int fin_slots = RS * G * B;  // finaliser threads, one per (stream, g, b)
    const int ft = threadIdx.x;
    const int f_s = ft / (G * B), f_g = (ft / B) % G, f_b = ft % B;

    for (int it = 0; it < iters; ++it) {
        const int base = r0 + (it * RS + stream) * G;
        float acc[NM][G][B];
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            ChunkLoad<CODEC> L[G];
#pragma unroll
            for (int g = 0; g < G; ++g)
                if (active && base + g < r1) load_chunk<CODEC>(L[g], m ? p.w1 : p.w0, p.rows, p.K, base + g, c);
#pragma unroll
            for (int g = 0; g < G; ++g) {
#pragma unroll
                for (int b = 0; b < B; ++b)
                    acc[m][g][b] = (active && base + g < r1) ? chunk_dot<CODEC, EXACT>(L[g], xr[b], aux[b], c) : 0.0f;
            }
        }
        float *part = smem + (it & 1) * RS * G * B * NM * KW;
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float v = warp_sum(acc[m][g][b]);
                    if (lane == 0) part[(((stream * G + g) * B + b) * NM + m) * KW + kw] = v;
                }
        __syncthreads();
        if (ft < fin_slots) {
            const int row = r0 + (it * RS + f_s) * G + f_g;
            if (row < r1) {
                const float *pp = part + ((f_s * G + f_g) * B + f_b) * NM * KW;
                float s0 = 0.0f;
                for (int i = 0; i < KW; ++i) s0 += pp[i];
                float *yo = p.y + (size_t)f_b * p.rows + row;
                if constexpr (MODE == MV_STORE) {
                    *yo = s0;
                } else if constexpr (MODE == MV_ACCUM) {
                    *yo += s0;
                } else if constexpr (MODE == MV_SWIGLU) {
                    float s1 = 0.0f;
                    for (int i = 0; i < KW; ++i) s1 += pp[KW + i];
                    *yo = silu_f(s0) * s1;
                } else {
                    if (p.y != nullptr) *yo = s0;
                    // rows arrive in increasing order per thread: strict > keeps the lowest id
                    if (s0 > best_v[0]) { best_v[0] = s0; best_i[0] = (uint32_t)row; }
                }
            }
        }
        // the double-buffered partials make one barrier per group sufficient
    }

    if constexpr (MODE == MV_ARGMAX) {
        // reduce (best_v, best_i) of the finaliser threads per batch row b
        __syncthreads();
        float *bv = smem;
        uint32_t *bi = reinterpret_cast<uint32_t *>(smem + fin_slots);
        if (ft < fin_slots) { bv[ft] = best_v[0]; bi[ft] = best_i[0]; }
        __syncthreads();
        if (ft < B) {
            float v = -INFINITY;
            uint32_t id = 0xffffffffu;
            for (int t = ft; t < fin_slots; t += B) {
                const float tv = bv[t];
                const uint32_t ti = bi[t];
                if (tv > v || (tv == v && ti < id)) { v = tv; id = ti; }
            }
            p.part_val[(size_t)blockIdx.x * B + ft] = v;
            p.part_idx[(size_t)blockIdx.x * B + ft] = id;
        }
    }
}

// Final argmax over per-CTA partials; ties resolve to the smallest id
// (qw35_output.metal:141-182).  One CTA of 256 threads per batch row.
__global__ void argmax_reduce_kernel(const float *pv, const uint32_t *pi, int n, int B,
                                     uint32_t *out_tok, float *out_val) {
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
    int kw, rs, threads, ctas, rows_per_cta;
    size_t smem;
};

template <int CODEC, int B, int MODE>
static MvGeom mv_geometry(int rows, int K, const void *kern) {
    constexpr int G = CodecTraits<CODEC>::G;
    constexpr int NM = MODE == MV_SWIGLU ? 2 : 1;
    MvGeom g;
    const int nchunk = K / 32;
    g.kw = (nchunk + 31) / 32;
    g.rs = g.kw >= 8 ? 1 : 8 / g.kw;
    g.threads = g.kw * g.rs * 32;
    const size_t part = (size_t)2 * g.rs * G * B * NM * g.kw;
    const size_t fin = (size_t)2 * g.rs * G * B;
    g.smem = (part > fin ? part : fin) * sizeof(float) + 64 * sizeof(float);
    int occ = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, g.threads, g.smem);
    if (occ < 1) occ = 1;
    const int max_ctas = qw35h::sm_count() * occ;
    const int unit = g.rs * G;
    const int units = (rows + unit - 1) / unit;
    int ctas = units < max_ctas ? units : max_ctas;
    const int units_per_cta = (units + ctas - 1) / ctas;
    g.rows_per_cta = units_per_cta * unit;
    g.ctas = (rows + g.rows_per_cta - 1) / g.rows_per_cta;
    return g;
}

template <int CODEC, int B, int MODE, bool EXACT, typename XT>
static cudaError_t mv_launch(MvParams p, cudaStream_t st, int *ctas_out) {
    auto kern = mv_kernel<CODEC, B, MODE, EXACT, XT>;
    MvGeom g = mv_geometry<CODEC, B, MODE>(p.rows, p.K, (const void *)kern);
    if (g.kw > kMaxKW) return cudaErrorInvalidValue;
    if (g.smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
    p.kw = g.kw;
    p.rows_per_cta = g.rows_per_cta;
    if (ctas_out) *ctas_out = g.ctas;
    if (MODE == MV_ARGMAX && p.part_val == nullptr) return cudaErrorInvalidValue;
    kern<<<g.ctas, g.threads, g.smem, st>>>(p);
    return cudaGetLastError();
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

// Batch rows beyond the register-resident tile are processed in tiles of
// two; each tile re-reads the weights (from L2 when they fit).
cudaError_t matvec_run(const MatvecArgs &a, cudaStream_t st) {
    const size_t xes = a.x_dtype == QW35_F16_TYPE ? 2 : 4;
    for (int b0 = 0; b0 < a.batch; b0 += 2) {
        const int nb = a.batch - b0 < 2 ? a.batch - b0 : 2;
        MvParams p{};
        p.w0 = static_cast<const uint8_t *>(a.w0);
        p.w1 = static_cast<const uint8_t *>(a.w1);
        p.x = static_cast<const uint8_t *>(a.x) + (size_t)b0 * a.k * xes;
        p.norm_w = a.norm_w;
        p.eps = a.eps;
        p.y = a.y ? a.y + (size_t)b0 * a.rows : nullptr;
        p.rows = (int)a.rows;
        p.K = (int)a.k;
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
    const size_t n = (size_t)qw35h::sm_count() * 16;  // >= any persistent grid
    return n * 2 * ((batch + 1) / 2 * 2) * sizeof(float) * 2 + 256;
}

cudaError_t argmax_head_run(const MatvecArgs &a, uint32_t *tok, float *val, void *ws, size_t ws_bytes,
                            cudaStream_t st) {
    if (ws_bytes < argmax_workspace_bytes(a.rows, a.batch)) return cudaErrorInvalidValue;
    const size_t xes = a.x_dtype == QW35_F16_TYPE ? 2 : 4;
    const size_t half_ws = ws_bytes / 2;
    for (int b0 = 0; b0 < a.batch; b0 += 2) {
        const int nb = a.batch - b0 < 2 ? a.batch - b0 : 2;
        MvParams p{};
        p.w0 = static_cast<const uint8_t *>(a.w0);
        p.x = static_cast<const uint8_t *>(a.x) + (size_t)b0 * a.k * xes;
        p.norm_w = a.norm_w;
        p.eps = a.eps;
        p.y = a.y ? a.y + (size_t)b0 * a.rows : nullptr;
        p.part_val = static_cast<float *>(ws);
        p.part_idx = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(ws) + half_ws);
        p.rows = (int)a.rows;
        p.K = (int)a.k;
        int ctas = 0;
        cudaError_t e = mv_dispatch<MV_ARGMAX>(a, p, nb, st, &ctas);
        if (e != cudaSuccess) return e;
        argmax_reduce_kernel<<<nb, 256, 0, st>>>(p.part_val, p.part_idx, ctas, nb, tok + b0,
                                                 val ? val + b0 : nullptr);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace qw35
