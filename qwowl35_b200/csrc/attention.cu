// attention.cu -- gated GQA decode attention over the chunk-table KV cache.
//
// Reference:
//   qw35_attn_decode_preprocess_f32        qw35_attention.metal:29-112
//   q8_0 KV twins (quantize / decode)      qw35_attention.metal:425-793
//   qw35_attention_gqa_flash_decode_f32    qw35_attention.metal:211-292
//   ..._split_f32 (8-way split-K + merge)  qw35_attention.metal:302-414
//   dispatch / split threshold             Qw35MetalRuntime+Attention.m:80-111
//
// KV layout: each sequence owns a table of 256-position chunks; chunk c of
// sequence i lives at chunk_ptrs[i * max_chunks + c] (any device address, no
// contiguity between chunks).  Inside a chunk, one attention layer's K plane
// (at k_off) and V plane (at v_off) are [4 kv heads][256 pos][256 dim] f16, so
// one (kv head, chunk) tile is a single contiguous 128 KiB run.
//
// Decode (B200 design): split-K over fixed 1024-position splits of the
// attended range; one CTA per (split, kv head, sequence) serves all 4 query
// heads of the GQA group from ONE read of K and V (the reference re-reads the
// cache once per query head).  Each warp walks 256 positions, 8 at a time:
// 128-bit loads of K/V rows, fp32 dots for the 4 heads, a 31-shuffle
// transpose-reduction, online softmax per head.  A second kernel merges the
// splits and applies the sigmoid output gate.
#include <mutex>

#include "common.cuh"
#include "ops.h"

namespace qw35 {

constexpr int AH = 16;      // query heads
constexpr int AKV = 4;      // kv heads
constexpr int AHD = 256;    // head dim
constexpr int AGRP = AH / AKV;
constexpr int ACHUNK = 256; // positions per chunk
constexpr int ASPLIT = 256;  // positions per split (4 warps x 64): ~2 waves of CTAs at batch 32, ctx 4096
constexpr int QFULL = AH * AHD * 2;  // q | gate per head
constexpr int ASTG = 3;     // cp.async stages per warp in the split kernel (8 positions each)
constexpr size_t ASMEM = (size_t)4 * ASTG * 2 * 8 * 32 * 16;  // 48 KiB of K/V staging per CTA
// q8_0 planes: per warp a ring of raw q8_0 rows plus one dequantised f16 stage
constexpr size_t ARAWQ8 = (size_t)ASTG * 2 * 8 * kKvQ8Row;             // 13,056 B
constexpr size_t AQ8D = 16 * 8 * 4;                                     // block scales [16 rows][8 blocks] f32
constexpr size_t ASMEM_Q8 = (size_t)4 * (ARAWQ8 + 2 * 8 * 32 * 16 + AQ8D);  // 87,040 B

// One q8_0 block of 32 values held 8 per lane by 4 consecutive lanes (lane % 4
// = the lane's quarter): qw35_q8_0_quantize_block (qw35_attention.metal:429-440).
// d = amax / 127 in fp32, codes round(x * (1 / d)) (half away from zero)
// clamped to +-127 with the fp32 d, the block stores half(d).  `blk` points at
// the block's 34 bytes {f16 d; int8 qs[32]}; every lane of the warp calls this.
__device__ __forceinline__ void q8_block_store(const float *x, uint8_t *blk, int lane) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float y = __fmul_rn(x[i], id);  // a plain product, as the reference (no contraction)
        int q = (int)roundf(y);
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        packed[i >> 2] |= ((uint32_t)q & 0xffu) << (8 * (i & 3));
    }
    // the block starts 2 bytes before the codes; codes of quarter j at 2 + 8 j:
    // even addresses, so 16-bit stores
    unsigned short *qd = reinterpret_cast<unsigned short *>(blk + 2 + 8 * (lane & 3));
    qd[0] = (unsigned short)(packed[0] & 0xffffu);
    qd[1] = (unsigned short)(packed[0] >> 16);
    qd[2] = (unsigned short)(packed[1] & 0xffffu);
    qd[3] = (unsigned short)(packed[1] >> 16);
    if ((lane & 3) == 0) *reinterpret_cast<unsigned short *>(blk) = __half_as_ushort(__float2half_rn(d));
}

// ---- preprocess: RMS norm + NeoX RoPE + f16 (or q8_0) KV write ----------------
// One warp per head row (16 q heads + 4 kv heads = 20 warps): every row's
// load -> norm -> RoPE -> store chain runs at once.
constexpr int APRE_THREADS = (AH + AKV) * 32;
__global__ void __launch_bounds__(APRE_THREADS) attn_pre_kernel(AttnPreArgs p) {
    const int seq = blockIdx.x;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int pos = p.pos[seq];
    const float *src = p.qkv + (size_t)seq * p.qkv_stride;
    const int d0 = lane * 8;
    for (int task = wid; task < AH + AKV; task += APRE_THREADS / 32) {
        const bool isq = task < AH;
        const int h = isq ? task : task - AH;
        const float *x = isq ? src + h * 2 * AHD : src + QFULL + h * AHD;
        const float *nw = isq ? p.q_norm_w : p.k_norm_w;
        float v[8];
        float ss = 0.0f;
        if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {  // a row stride of 4k floats: 16-byte loads
            const float4 a = *reinterpret_cast<const float4 *>(x + d0), b = *reinterpret_cast<const float4 *>(x + d0 + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = x[d0 + i];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / (float)AHD + p.eps);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * nw[d0 + i];
        // RoPE over dims [0, 64): lanes 0..3 hold dims 0..31, lanes 4..7 hold 32..63
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float partner = __shfl_xor_sync(0xffffffffu, v[i], 4);
            if (lane < 8) {
                const int pair = (d0 + i) & 31;
                const float theta = (float)pos * p.rope_freq[pair];
                float sn, cs;
                sincosf(theta, &sn, &cs);
                o[i] = lane < 4 ? (v[i] * cs - partner * sn) : (partner * sn + v[i] * cs);
            } else {
                o[i] = v[i];
            }
        }
        if (isq) {
            float *qo = p.q_out + ((size_t)seq * AH + h) * AHD + d0;
            float *go = p.gate_out + ((size_t)seq * AH + h) * AHD + d0;
#pragma unroll
            for (int i = 0; i < 8; ++i) { qo[i] = o[i]; go[i] = x[AHD + d0 + i]; }
        } else if (p.kv_q8) {
            // q8_0 rows: lanes 4b..4b+3 hold block b (dims 32b..32b+31) of the head row
            const size_t trow = p.slots ? (size_t)p.slots[seq] : (size_t)seq;
            const uint64_t base = p.chunk_ptrs[trow * p.max_chunks + pos / ACHUNK];
            const size_t row = ((size_t)h * ACHUNK + (pos % ACHUNK)) * kKvQ8Row + 34 * (lane >> 2);
            const float *vs = src + QFULL + AKV * AHD + h * AHD + d0;
            float vv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) vv[i] = vs[i];
            q8_block_store(o, reinterpret_cast<uint8_t *>(base + p.k_off + row), lane);
            q8_block_store(vv, reinterpret_cast<uint8_t *>(base + p.v_off + row), lane);
        } else {
            const size_t trow = p.slots ? (size_t)p.slots[seq] : (size_t)seq;
            const uint64_t base = p.chunk_ptrs[trow * p.max_chunks + pos / ACHUNK];
            const size_t row = ((size_t)h * ACHUNK + (pos % ACHUNK)) * AHD + d0;
            __half *kp = reinterpret_cast<__half *>(base + p.k_off) + row;
            __half *vp = reinterpret_cast<__half *>(base + p.v_off) + row;
            const float *vs = src + QFULL + AKV * AHD + h * AHD + d0;
            __align__(16) __half kh[8], vh[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) { kh[i] = __float2half_rn(o[i]); vh[i] = __float2half_rn(vs[i]); }
            *reinterpret_cast<uint4 *>(kp) = *reinterpret_cast<const uint4 *>(kh);
            *reinterpret_cast<uint4 *>(vp) = *reinterpret_cast<const uint4 *>(vh);
        }
    }
}

// ---- split-K decode -----------------------------------------------------------
// 16-byte global -> shared copy (L2 only); zero-filled when !valid.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void h8_to_f(const uint4 &u, float *f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&w[k]));
        f[2 * k] = t.x;
        f[2 * k + 1] = t.y;
    }
}

struct SplitPart {  // per (seq, head, split): m, l then acc[256] in a separate array
    float m, l;
};

__device__ __forceinline__ void attended_range(int L, int window, int sink, int &total, int &sk, int &rstart) {
    sk = max(0, min(sink, L));
    if (window <= 0 || sk + window >= L) {
        sk = 0; rstart = 0; total = L;
    } else {
        rstart = L - window; total = sk + window;
    }
}

// m16n8k16 f16 x f16 -> f32 (legacy warp MMA; this kernel is bound by HBM, the
// tensor cores only retire its arithmetic)
__device__ __forceinline__ void mma16816(float *d, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t *r, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t *r, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// a = hi + lo in f16 (hi rounded, lo the rounded remainder): ~22 bits of a
__device__ __forceinline__ void split_h2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = pack_h2(a - hf.x, b - hf.y);
}

// One CTA per (split of ASPLIT positions, kv head, sequence); 4 warps take
// ASPLIT/4 consecutive positions each, 8 per step.  Scores S^T = K Q^T and
// the output O^T += V^T P^T run on mma.sync (M = 16: the step's 8 positions
// fill rows 0-7 and repeat in rows 8-15, whose results are dropped; N = 8:
// the group's 4 query heads, zero-padded).  q and p enter as f16 hi + lo
// pairs (two MMAs each), so both products keep ~22 bits; K and V are the
// cache's f16.  Lane (g = lane/4, t = lane%4) holds the scores of position
// g for heads 2t, 2t+1 and O^T rows (dims) 16 j + g, + 8 for the same heads;
// lanes with t >= 2 carry the padding.
// Q8: the planes hold q8_0 rows (272 B per head-row); each warp stages the raw
// rows with cp.async and, per step, turns the codes into the same swizzled f16
// tile (the int8 codes, exact in half) and the block scales d into a small
// f32 table.  The scale goes in after the MMA, in fp32, as the reference
// computes d * q (qw35_attention.metal:665-682): scores accumulate per 32-dim
// block (two k-steps) and add d_K * block sum; for the values, each 32-dim
// block b multiplies P by d_V[position][b] before it is split into the f16
// hi / lo operand.
template <bool Q8>
__global__ void __launch_bounds__(128) attn_split_kernel(AttnArgs p, int nsplit_max) {
    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int L = p.seq_len[seq];
    int total, sk, rstart;
    attended_range(L, p.window, p.sink, total, sk, rstart);
    const int nsplit = (total + ASPLIT - 1) / ASPLIT;
    if (split >= nsplit) return;

    __shared__ float wm[4][AGRP], wl[4][AGRP];
    __shared__ __align__(16) float wacc[4][AGRP][AHD];

    // B fragments of Q^T (k = dims, n = head g): k-step j needs dims
    // 16j + 2t, +1 (b0) and 16j + 8 + 2t, +1 (b1); pre-scaled by sm_scale.
    uint32_t qh[16][2], ql[16][2];
    {
        const bool real = g < AGRP;
        const float *qr = p.q + ((size_t)seq * AH + kvh * AGRP + (real ? g : 0)) * AHD;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
                const float2 v = *reinterpret_cast<const float2 *>(qr + 16 * j + 8 * hb + 2 * t4);
                const float a = real ? v.x * p.scale : 0.0f, b = real ? v.y * p.scale : 0.0f;
                split_h2(a, b, qh[j][hb], ql[j][hb]);
            }
        }
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float ma = -INFINITY, mb = -INFINITY, la = 0.0f, lb = 0.0f;  // heads 2t, 2t+1

    const int i0 = split * ASPLIT + wid * (ASPLIT / 4);
    const int i1 = min(i0 + ASPLIT / 4, total);
    const uint64_t *ctab = p.chunk_ptrs + (p.slots ? (size_t)p.slots[seq] : (size_t)seq) * p.max_chunks;
    const size_t head_off = (size_t)kvh * ACHUNK * AHD;

    // Per-warp ring of ASTG stages; a stage holds K then V of 8 positions, each
    // row's 16-byte piece c stored at c ^ (row % 8) so ldmatrix reads hit eight
    // distinct bank groups (cp.async, zero-filled past i1).
    extern __shared__ __align__(16) uint4 ring[];  // [4 warps][ASTG][2][8 rows][32 pieces]
    // (Q8: [4 warps] x {raw [ASTG][2][8 rows][272 B], f16 tile [2][8 rows][32 pieces]})
    uint4 *wring = Q8 ? ring + (size_t)wid * ((ARAWQ8 + 2 * 8 * 32 * 16 + AQ8D) / 16) : ring + (size_t)wid * ASTG * 2 * 8 * 32;
    uint8_t *wraw = reinterpret_cast<uint8_t *>(wring);
    uint4 *wtile = wring + ARAWQ8 / 16;
    float *wdsc = reinterpret_cast<float *>(wtile + 2 * 8 * 32);  // [16 rows: K 0-7, V 8-15][8 blocks]
    auto issue = [&](int ib, int stage) {
        if constexpr (Q8) {
            // 2 x 8 rows of 17 16-byte pieces; pieces past i1 are zero-filled
            uint8_t *dst = wraw + (size_t)stage * 2 * 8 * kKvQ8Row;
            for (int q = lane; q < 2 * 8 * 17; q += 32) {
                const int kv = q >= 8 * 17 ? 1 : 0;
                const int rem = q - kv * 8 * 17;
                const int r = rem / 17, pc = rem - r * 17;
                const int idx = ib + r;
                const bool ok = idx < i1;
                const int pos = ok ? (idx < sk ? idx : rstart + (idx - sk)) : 0;
                const uint64_t base = ctab[ok ? pos / ACHUNK : 0];
                const size_t off = ((size_t)kvh * ACHUNK + (size_t)(pos % ACHUNK)) * kKvQ8Row + (size_t)pc * 16;
                cp_async16(dst + (kv * 8 + r) * kKvQ8Row + pc * 16,
                           reinterpret_cast<const void *>(base + (kv ? p.v_off : p.k_off) + off), ok);
            }
            return;
        }
        uint4 *dst = wring + (size_t)stage * 2 * 8 * 32;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int idx = ib + r;
            const bool ok = idx < i1;
            const int pos = ok ? (idx < sk ? idx : rstart + (idx - sk)) : 0;
            const uint64_t base = ctab[ok ? pos / ACHUNK : 0];
            const size_t off = (head_off + (size_t)(pos % ACHUNK) * AHD + lane * 8) * sizeof(__half);
            const int pc = lane ^ r;
            cp_async16(dst + r * 32 + pc, reinterpret_cast<const void *>(base + p.k_off + off), ok);
            cp_async16(dst + (8 + r) * 32 + pc, reinterpret_cast<const void *>(base + p.v_off + off), ok);
        }
    };
#pragma unroll
    for (int s0 = 0; s0 < ASTG - 1; ++s0) {
        if (i0 + 8 * s0 < i1) issue(i0 + 8 * s0, s0);
        cp_async_commit();
    }
    const int lr = lane & 7;  // ldmatrix row (position) this lane addresses
    int stage = 0;
    for (int ib = i0; ib < i1; ib += 8) {
        {   // next block into the stage consumed last iteration
            const int nb = ib + 8 * (ASTG - 1);
            int ns = stage + ASTG - 1;
            if (ns >= ASTG) ns -= ASTG;
            if (nb < i1) issue(nb, ns);
            cp_async_commit();
        }
        cp_async_wait<ASTG - 1>();  // this block's group has landed
        __syncwarp();
        const uint4 *ks = wring + (size_t)stage * 2 * 8 * 32;
        if constexpr (Q8) {
            // raw rows -> f16 code tile: lane = 16-byte piece (dims 8 lane .. +7) =
            // quarter lane % 4 of block lane / 4; q + 1152 - 1152 in half is exact;
            // the block's d goes to the f32 table
            const uint8_t *rs = wraw + (size_t)stage * 2 * 8 * kKvQ8Row + 34 * (lane >> 2);
            const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
#pragma unroll
            for (int kr = 0; kr < 16; ++kr) {  // K rows 0-7, then V rows 0-7
                const uint8_t *blk = rs + kr * kKvQ8Row;
                if ((lane & 3) == 0)
                    wdsc[kr * 8 + (lane >> 2)] =
                        __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(blk)));
                const unsigned short *qd = reinterpret_cast<const unsigned short *>(blk + 2 + 8 * (lane & 3));
                uint32_t hw[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t two = (uint32_t)qd[u] ^ 0x8080u;  // biased codes q + 128
                    const uint32_t v = __byte_perm(two, 0x64646464u, 0x4140u);  // halves 1024 + (q + 128)
                    const __half2 h = __hsub2(*reinterpret_cast<const __half2 *>(&v), off);
                    hw[u] = *reinterpret_cast<const uint32_t *>(&h);
                }
                const int r = kr & 7;
                wtile[(kr >> 3) * 8 * 32 + r * 32 + (lane ^ r)] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            }
            __syncwarp();
            ks = wtile;
        }
        const uint4 *vs = ks + 8 * 32;

        // S^T (16 x 8) = K (16 x 256) Q^T (256 x 8): A rows = positions (rows 8-15 repeat 0-7)
        // four independent accumulators (q hi / lo x even / odd k-step) keep four
        // MMA chains in flight instead of one 32-long dependent chain
        float sc[4];
        if constexpr (Q8) {
            // per 32-dim block: codes x q over two k-steps, then + d_K[row g][block] * sum
            sc[0] = sc[1] = sc[2] = sc[3] = 0.0f;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                float ah[4] = {}, al[4] = {};
#pragma unroll
                for (int j = 2 * b; j < 2 * b + 2; ++j) {
                    uint32_t a[4];
                    const int c = 2 * j + ((lane >> 4) & 1);
                    ldsm_x4(a, ks + lr * 32 + (c ^ lr));
                    mma16816(ah, a, qh[j][0], qh[j][1]);
                    mma16816(al, a, ql[j][0], ql[j][1]);
                }
                const float d = wdsc[g * 8 + b];
#pragma unroll
                for (int i = 0; i < 4; ++i) sc[i] = fmaf(d, ah[i] + al[i], sc[i]);
            }
        } else {
            float acc4[4][4] = {};
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                uint32_t a[4];
                const int c = 2 * j + ((lane >> 4) & 1);  // matrices 2, 3: dims + 8
                ldsm_x4(a, ks + lr * 32 + (c ^ lr));
                mma16816(acc4[j & 1], a, qh[j][0], qh[j][1]);
                mma16816(acc4[2 + (j & 1)], a, ql[j][0], ql[j][1]);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) sc[i] = (acc4[0][i] + acc4[1][i]) + (acc4[2][i] + acc4[3][i]);
        }
        // online softmax of heads 2t, 2t+1 over this step's 8 positions (lane rows g)
        const bool valid = ib + g < i1;
        const float sa = valid ? sc[0] : -INFINITY, sb = valid ? sc[1] : -INFINITY;
        float bma = sa, bmb = sb;
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            bma = fmaxf(bma, __shfl_xor_sync(0xffffffffu, bma, off));
            bmb = fmaxf(bmb, __shfl_xor_sync(0xffffffffu, bmb, off));
        }
        const float na = fmaxf(ma, bma), nb2 = fmaxf(mb, bmb);
        const float pa = sa == -INFINITY ? 0.0f : expf(sa - na);
        const float pb = sb == -INFINITY ? 0.0f : expf(sb - nb2);
        float ra = pa, rb = pb;
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            ra += __shfl_xor_sync(0xffffffffu, ra, off);
            rb += __shfl_xor_sync(0xffffffffu, rb, off);
        }
        const float alpha_a = ma == -INFINITY ? 0.0f : expf(ma - na);
        const float alpha_b = mb == -INFINITY ? 0.0f : expf(mb - nb2);
        la = la * alpha_a + ra;
        lb = lb * alpha_b + rb;
        if (__any_sync(0xffffffffu, na != ma || nb2 != mb)) {  // a running max moved: rescale O
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                o[j][0] *= alpha_a; o[j][1] *= alpha_b; o[j][2] *= alpha_a; o[j][3] *= alpha_b;
            }
        }
        ma = na;
        mb = nb2;
        // B fragment of P^T (k = positions 2t, 2t+1; n = head g): from lanes
        // (2t, g/2) and (2t+1, g/2), their head-pair slot g%2; heads >= 4 are zero
        const int src0 = (2 * t4) * 4 + (g >> 1), src1 = src0 + 4;
        const float x0a = __shfl_sync(0xffffffffu, pa, src0), x0b = __shfl_sync(0xffffffffu, pb, src0);
        const float x1a = __shfl_sync(0xffffffffu, pa, src1), x1b = __shfl_sync(0xffffffffu, pb, src1);
        const float p0 = g < AGRP ? ((g & 1) ? x0b : x0a) : 0.0f;
        const float p1 = g < AGRP ? ((g & 1) ? x1b : x1a) : 0.0f;
        // O^T (256 x 8) += V^T (256 x 16) P^T (16 x 8): positions 8-15 have p = 0
        if constexpr (Q8) {
            // dims block b = j / 2: P rows (positions 2t, 2t+1) times d_V[position][b],
            // times 2^8 so small products keep their bits in the f16 hi / lo halves
            // (the partials are scaled back below)
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                uint32_t ph, pl;
                split_h2(p0 * (wdsc[(8 + 2 * t4) * 8 + b] * 256.0f), p1 * (wdsc[(9 + 2 * t4) * 8 + b] * 256.0f), ph,
                         pl);
#pragma unroll
                for (int j = 2 * b; j < 2 * b + 2; ++j) {
                    uint32_t a[4];
                    const int c = 2 * j + ((lane >> 3) & 1);
                    ldsm_x4_t(a, vs + lr * 32 + (c ^ lr));
                    mma16816(o[j], a, ph, 0u);
                    mma16816(o[j], a, pl, 0u);
                }
            }
        } else {
            uint32_t ph, pl;
            split_h2(p0, p1, ph, pl);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                uint32_t a[4];
                const int c = 2 * j + ((lane >> 3) & 1);  // matrices 1, 3: dims + 8
                ldsm_x4_t(a, vs + lr * 32 + (c ^ lr));
                mma16816(o[j], a, ph, 0u);
                mma16816(o[j], a, pl, 0u);
            }
        }
        __syncwarp();  // the stage may be refilled by the next iteration's issue
        if (++stage == ASTG) stage = 0;
    }

    // merge the 4 warps, write the split partial
    if (g == 0 && t4 < 2) {
        wm[wid][2 * t4] = ma; wm[wid][2 * t4 + 1] = mb;
        wl[wid][2 * t4] = la; wl[wid][2 * t4 + 1] = lb;
    }
    if (t4 < 2) {
        constexpr float osc = Q8 ? 1.0f / 256.0f : 1.0f;  // Q8: undo the 2^8 of the value operand
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            wacc[wid][2 * t4][16 * j + g] = o[j][0] * osc;
            wacc[wid][2 * t4 + 1][16 * j + g] = o[j][1] * osc;
            wacc[wid][2 * t4][16 * j + g + 8] = o[j][2] * osc;
            wacc[wid][2 * t4 + 1][16 * j + g + 8] = o[j][3] * osc;
        }
    }
    __syncthreads();
    const size_t nsm = (size_t)nsplit_max;
    SplitPart *parts = static_cast<SplitPart *>(p.ws);
    float *pacc = reinterpret_cast<float *>(static_cast<uint8_t *>(p.ws) +
                                            (size_t)p.n_seq * AH * nsm * sizeof(SplitPart));
    for (int e = threadIdx.x; e < AGRP * AHD; e += 128) {
        const int hh = e / AHD, d = e % AHD;
        float ms = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) ms = fmaxf(ms, wm[w][hh]);
        float ls = 0.0f, as = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float f = wm[w][hh] == -INFINITY ? 0.0f : expf(wm[w][hh] - ms);
            ls += f * wl[w][hh];
            as += f * wacc[w][hh][d];
        }
        const size_t slot = ((size_t)seq * AH + kvh * AGRP + hh) * nsm + split;
        pacc[slot * AHD + d] = as;
        if (d == 0) { parts[slot].m = ms; parts[slot].l = ls; }
    }
}

__global__ void __launch_bounds__(256) attn_combine_kernel(AttnArgs p, int nsplit_max) {
    const int h = blockIdx.x, seq = blockIdx.y, d = threadIdx.x;
    const int L = p.seq_len[seq];
    int total, sk, rstart;
    attended_range(L, p.window, p.sink, total, sk, rstart);
    const int nsplit = (total + ASPLIT - 1) / ASPLIT;
    const size_t nsm = (size_t)nsplit_max;
    const SplitPart *parts = static_cast<const SplitPart *>(p.ws);
    const float *pacc = reinterpret_cast<const float *>(static_cast<const uint8_t *>(p.ws) +
                                                        (size_t)p.n_seq * AH * nsm * sizeof(SplitPart));
    const size_t base = ((size_t)seq * AH + h) * nsm;
    float ms = -INFINITY;
    for (int s = 0; s < nsplit; ++s) ms = fmaxf(ms, parts[base + s].m);
    float ls = 0.0f, as = 0.0f;
    for (int s = 0; s < nsplit; ++s) {
        const float mm = parts[base + s].m;
        const float f = mm == -INFINITY ? 0.0f : expf(mm - ms);
        ls += f * parts[base + s].l;
        as += f * pacc[(base + s) * AHD + d];
    }
    float o = ls > 0.0f ? as / ls : 0.0f;
    if (p.gate) o *= sigmoid_f(p.gate[((size_t)seq * AH + h) * AHD + d]);
    p.out[(size_t)seq * p.out_stride + h * AHD + d] = o;
}

size_t attn_workspace_bytes(int n_seq, int max_len) {
    const size_t ns = (size_t)((max_len + ASPLIT - 1) / ASPLIT);
    return (size_t)n_seq * AH * ns * (sizeof(SplitPart) + AHD * sizeof(float));
}

cudaError_t attn_preprocess_run(const AttnPreArgs &a, cudaStream_t st) {
    if (a.n_seq <= 0) return cudaSuccess;
    attn_pre_kernel<<<a.n_seq, APRE_THREADS, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t attn_decode_run(const AttnArgs &a, cudaStream_t st) {
    if (a.n_seq <= 0) return cudaSuccess;
    if (a.max_len <= 0 || a.n_seq > 65535) return cudaErrorInvalidValue;
    if (a.ws_bytes < attn_workspace_bytes(a.n_seq, a.max_len)) return cudaErrorInvalidValue;
    const int ns = (a.max_len + ASPLIT - 1) / ASPLIT;
    dim3 g1(ns, AKV, a.n_seq);
    cudaError_t e0;
    if (a.kv_q8) {
        e0 = qw35h::smem_optin((const void *)attn_split_kernel<true>, (int)ASMEM_Q8);
        if (e0 != cudaSuccess) return e0;
        attn_split_kernel<true><<<g1, 128, ASMEM_Q8, st>>>(a, ns);
    } else {
        e0 = qw35h::smem_optin((const void *)attn_split_kernel<false>, (int)ASMEM);
        if (e0 != cudaSuccess) return e0;
        attn_split_kernel<false><<<g1, 128, ASMEM, st>>>(a, ns);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    dim3 g2(AH, a.n_seq);
    attn_combine_kernel<<<g2, 256, 0, st>>>(a, ns);
    return cudaGetLastError();
}

}  // namespace qw35

// ---------------------------------------------------------------------------
// Allocation-free variant of the split-K decode.
//
// Some callers cannot allocate device memory at the point where they decode:
// an engine whose GPU memory is owned by another allocator and not reachable
// across the FFI, a host with a fixed memory budget that reserves everything
// up front, or a latency-critical loop that must not pay cudaMalloc's implicit
// device synchronisation.  For them the split partials live in one static
// device array of kNoAllocScratchBytes, held by every GPU that loads this
// library until the process exits.  The array's host-side symbol is not a
// device address, so its device address is looked up once per device with
// cudaGetSymbolAddress (on the first call for that device, with that device
// current) and handed to the unchanged kernels.  Every call shares the array:
// calls that overlap on the GPU (different streams, no ordering) race on it.
// Nothing in it has to start at zero: the split kernel writes every partial
// the combine kernel reads, in the same call.
// ---------------------------------------------------------------------------
namespace qw35 {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB
static __device__ __align__(256) uint8_t g_attn_scratch[kNoAllocScratchBytes];

static cudaError_t noalloc_scratch(void **ptr) {
    static std::mutex mu;
    static void *addr[64] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    if (addr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
    }
    *ptr = addr[dev];
    return cudaSuccess;
}

size_t attn_noalloc_limit() { return kNoAllocScratchBytes; }

cudaError_t attn_decode_noalloc_run(AttnArgs a, cudaStream_t st) {
    void *scratch = nullptr;
    cudaError_t e = noalloc_scratch(&scratch);
    if (e != cudaSuccess) return e;
    a.ws = scratch;
    a.ws_bytes = kNoAllocScratchBytes;
    return attn_decode_run(a, st);
}

}  // namespace qw35
