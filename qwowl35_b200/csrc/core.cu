// core.cu -- weight repack / dequant, embedding gather, RMS norm.
//
// Reference: qw35_get_row_q4_k_f32 / qw35_get_row_q8_0_f32
// (qw35_matvec.metal:100-149), qw35_rms_norm_weight_f32 (qw35_core.metal:14-48).
#include <mutex>
#include <set>
#include <tuple>

#include "common.cuh"
#include "ops.h"
#include "quant.cuh"

namespace qw35h {
int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (cached[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 1;
    }
    return cached[dev];
}

// The dynamic shared-memory opt-in is a per-device property of a kernel: it is
// recorded per (device, kernel) under a lock, so a process that launches on
// several devices, from several host threads, sets it once on each.
cudaError_t smem_optin(const void *func, int bytes) {
    static std::mutex mu;
    static std::set<std::tuple<int, const void *, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> g(mu);
    const auto key = std::make_tuple(dev, func, bytes);
    if (done.count(key)) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert(key);
    return e;
}
}  // namespace qw35h

namespace qw35 {

// ---- GGUF -> device layout ------------------------------------------------------
// Q8_0: one thread per 34-byte block: 32 codes to the codes plane, d to the scales plane.
__global__ void repack_q8_0_kernel(const uint8_t *src, uint8_t *dst, size_t nblk, size_t rows, uint32_t k) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const uint8_t *s = src + b * 34;
    uint8_t *codes = dst + b * 32;
    uint16_t *scales = reinterpret_cast<uint16_t *>(dst + rows * k);
    uint32_t tmp[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        tmp[i] = (uint32_t)s[2 + 4 * i] | ((uint32_t)s[3 + 4 * i] << 8) | ((uint32_t)s[4 + 4 * i] << 16) |
                 ((uint32_t)s[5 + 4 * i] << 24);
    reinterpret_cast<uint4 *>(codes)[0] = make_uint4(tmp[0], tmp[1], tmp[2], tmp[3]);
    reinterpret_cast<uint4 *>(codes)[1] = make_uint4(tmp[4], tmp[5], tmp[6], tmp[7]);
    scales[b] = (uint16_t)s[0] | ((uint16_t)s[1] << 8);
}

// Q8_0 row exponents (device-layout tail plane, one int8 per row): e with
// 128 * max|d| * 2^e < 2^15, i.e. e = 7 - floor(log2(max|d|)) (0 for an
// all-zero or non-finite row).  The tensor-core matvec splits q * d * 2^e
// into exact f16 hi + lo halves and removes 2^e in its epilogue.
__global__ void q8_0_row_exp_kernel(uint8_t *dst, uint32_t rows, uint32_t k) {
    const uint32_t r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint16_t *scales = reinterpret_cast<const uint16_t *>(dst + (size_t)rows * k) + (size_t)r * (k / 32);
    uint32_t mx = 0;  // max of |d| bits (monotone for finite halves)
    for (uint32_t b = threadIdx.x & 31; b < k / 32; b += 32) {
        const uint32_t a = scales[b] & 0x7fffu;
        mx = a > mx ? a : mx;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint32_t v = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = v > mx ? v : mx;
    }
    if ((threadIdx.x & 31) == 0) {
        int e = 0;
        if (mx != 0 && mx < 0x7c00u) {
            const int ex = (int)(mx >> 10);  // biased exponent, 0 for subnormals
            int m = ex - 15;                 // floor(log2) of a normal half
            if (ex == 0) m = 31 - __clz(mx & 0x3ffu) - 24;  // subnormal: mantissa * 2^-24
            e = 7 - m;
        }
        int8_t *ep = reinterpret_cast<int8_t *>(dst + (size_t)rows * (k / 32) * 34);
        ep[r] = (int8_t)e;
    }
}

// Q4_K: one thread per 144-byte block.  GGUF qs byte 32g+l holds element 64g+l
// (low nibble) and 64g+32+l (high); the device codes plane holds elements in
// order, two per byte.  The 16-byte header (d, dmin, scales) is kept verbatim.
__global__ void repack_q4_k_kernel(const uint8_t *src, uint8_t *dst, size_t nblk, size_t rows, uint32_t k) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const uint8_t *s = src + b * 144;
    uint8_t *codes = dst + b * 128;
    uint8_t *hdr = dst + rows * (k / 2) + b * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) hdr[i] = s[i];
    const uint8_t *qs = s + 16;
    for (int j = 0; j < 128; ++j) {
        const int e0 = 2 * j, e1 = 2 * j + 1;
        auto nib = [&](int e) -> uint32_t {
            const int g = e / 64, r = e % 64;
            const uint8_t byte = qs[32 * g + (r % 32)];
            return r < 32 ? (byte & 0xf) : (byte >> 4);
        };
        codes[j] = (uint8_t)(nib(e0) | (nib(e1) << 4));
    }
}

// GGUF code of element e of a Q5_K block (qw35_matvec.metal:41-64): nibble of
// qs[32(j/2) + l] (low for even sub-block j) plus 16 * bit j of qh[l].
__device__ __forceinline__ uint32_t q5k_code(const uint8_t *s, int e) {
    const int j = e >> 5, l = e & 31;
    const uint8_t byte = s[48 + 32 * (j >> 1) + l];
    const uint32_t lo = (j & 1) ? (byte >> 4) : (byte & 0xfu);
    return lo | (((uint32_t)(s[16 + l] >> j) & 1u) << 4);
}

// GGUF code of element e of a Q6_K block (qw35_matvec.metal:66-98): element
// 128h + 32m + l takes a nibble of ql[64h + 32(m&1) + l] (high for m >= 2) and
// bits 2m..2m+1 of qh[32h + l].
__device__ __forceinline__ uint32_t q6k_code(const uint8_t *s, int e) {
    const int h = e >> 7, m = (e >> 5) & 3, l = e & 31;
    const uint8_t byte = s[64 * h + 32 * (m & 1) + l];
    const uint32_t lo = m < 2 ? (byte & 0xfu) : (byte >> 4);
    return lo | ((((uint32_t)s[128 + 32 * h + l] >> (2 * m)) & 3u) << 4);
}

// Q5_K / Q6_K: one thread per 256-weight block, into the layout described in
// common.cuh (element-ordered nibbles, high parts in nibble slots).
template <int TYPE>
__global__ void repack_k56_kernel(const uint8_t *src, uint8_t *dst, size_t nblk, size_t rows, uint32_t k) {
    const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const uint32_t nbr = k / 256;
    const size_t r = b / nbr;
    const uint32_t bi = (uint32_t)(b % nbr);
    constexpr uint32_t kBlk = TYPE == QW35_Q5_K_TYPE ? 176 : 210;
    const uint8_t *s = src + b * kBlk;
    const size_t code_row = TYPE == QW35_Q5_K_TYPE ? (size_t)k / 2 + k / 8 : (size_t)k / 2 + k / 4;
    uint8_t *row = dst + r * code_row;
    uint32_t code[256];
#pragma unroll 4
    for (int e = 0; e < 256; ++e) code[e] = TYPE == QW35_Q5_K_TYPE ? q5k_code(s, e) : q6k_code(s, e);
    for (int j = 0; j < 128; ++j) row[bi * 128 + j] = (uint8_t)((code[2 * j] & 15u) | ((code[2 * j + 1] & 15u) << 4));
    uint32_t *hw = reinterpret_cast<uint32_t *>(row + k / 2);
    if (TYPE == QW35_Q5_K_TYPE) {
        for (int j = 0; j < 8; ++j) {  // sub-block j: bit 4n + w <- element 32j + 8w + n
            uint32_t v = 0;
            for (int w = 0; w < 4; ++w)
                for (int n = 0; n < 8; ++n) v |= (code[32 * j + 8 * w + n] >> 4) << (4 * n + w);
            hw[bi * 8 + j] = v;
        }
        uint8_t *hdr = dst + rows * code_row + b * 16;
        for (int i = 0; i < 16; ++i) hdr[i] = s[i];
    } else {
        for (int t = 0; t < 16; ++t) {  // 16 weights: bits 4n.. <- element n, 4n+2.. <- element 8+n
            uint32_t v = 0;
            for (int n = 0; n < 8; ++n) v |= ((code[16 * t + n] >> 4) << (4 * n)) | ((code[16 * t + 8 + n] >> 4) << (4 * n + 2));
            hw[bi * 16 + t] = v;
        }
        uint8_t *sr = dst + rows * code_row + r * q6k_scale_row(k);
        for (int i = 0; i < 16; ++i) sr[bi * 16 + i] = s[192 + i];
        sr[k / 16 + 2 * bi] = s[208];
        sr[k / 16 + 2 * bi + 1] = s[209];
        if (bi == 0)
            for (uint32_t i = k / 16 + k / 128; i < q6k_scale_row(k); ++i) sr[i] = 0;
    }
}

cudaError_t weight_repack(uint32_t type_id, const void *src, void *dst, uint32_t rows, uint32_t k, cudaStream_t st) {
    const uint8_t *s = static_cast<const uint8_t *>(src);
    uint8_t *d = static_cast<uint8_t *>(dst);
    if (type_id == QW35_GF4_TYPE || type_id == QW35_F32_TYPE) {
        const size_t bytes = type_id == QW35_GF4_TYPE ? (size_t)rows * k / 2 : (size_t)rows * k * 4;
        return cudaMemcpyAsync(d, s, bytes, cudaMemcpyDeviceToDevice, st);
    }
    if (type_id == QW35_Q8_0_TYPE) {
        const size_t nb = (size_t)rows * (k / 32);
        repack_q8_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, st>>>(s, d, nb, rows, k);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        q8_0_row_exp_kernel<<<(rows + 7) / 8, 256, 0, st>>>(d, rows, k);
        return cudaGetLastError();
    }
    if (type_id == QW35_Q4_K_TYPE) {
        const size_t nb = (size_t)rows * (k / 256);
        repack_q4_k_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, st>>>(s, d, nb, rows, k);
        return cudaGetLastError();
    }
    if (type_id == QW35_Q5_K_TYPE || type_id == QW35_Q6_K_TYPE) {
        const size_t nb = (size_t)rows * (k / 256);
        const unsigned grid = (unsigned)((nb + 63) / 64);
        if (type_id == QW35_Q5_K_TYPE) repack_k56_kernel<QW35_Q5_K_TYPE><<<grid, 64, 0, st>>>(s, d, nb, rows, k);
        else repack_k56_kernel<QW35_Q6_K_TYPE><<<grid, 64, 0, st>>>(s, d, nb, rows, k);
        return cudaGetLastError();
    }
    return cudaErrorInvalidValue;
}

// ---- dequantise one element (device layout) ---------------------------------------
template <bool EXACT>
__device__ __forceinline__ float dequant_at(uint32_t type_id, const uint8_t *w, size_t rows, uint32_t k, size_t r,
                                            uint32_t c) {
    if (type_id == QW35_GF4_TYPE) {
        const uint32_t word = reinterpret_cast<const uint32_t *>(w)[r * (k / 8) + c / 8];
        return gf4_weight<EXACT>(word, (int)(c & 7));
    }
    if (type_id == QW35_Q8_0_TYPE) {
        const int8_t q = reinterpret_cast<const int8_t *>(w)[r * k + c];
        const uint16_t dbits = reinterpret_cast<const uint16_t *>(w + rows * k)[r * (k / 32) + c / 32];
        return (float)q * __half2float(__ushort_as_half(dbits));
    }
    if (type_id == QW35_Q4_K_TYPE) {
        const uint8_t byte = w[r * (k / 2) + c / 2];
        const uint32_t q = (c & 1) ? (byte >> 4) : (byte & 0xf);
        const uint4 h = *reinterpret_cast<const uint4 *>(w + rows * (k / 2) + (r * (k / 256) + c / 256) * 16);
        float dl, ml;
        q4k_scale_min(h, (int)((c % 256) / 32), dl, ml);
        return dl * (float)q - ml;
    }
    if (type_id == QW35_Q5_K_TYPE) {
        const uint8_t *row = w + r * ((size_t)k / 2 + k / 8);
        const uint8_t byte = row[c / 2];
        const uint32_t lo = (c & 1) ? (byte >> 4) : (byte & 0xf);
        const uint32_t hw = reinterpret_cast<const uint32_t *>(row + k / 2)[c / 32];
        const uint32_t e = c & 31;
        const uint32_t q = lo | (((hw >> (4 * (e & 7) + (e >> 3))) & 1u) << 4);
        const uint4 h = *reinterpret_cast<const uint4 *>(w + rows * ((size_t)k / 2 + k / 8) + (r * (k / 256) + c / 256) * 16);
        float dl, ml;
        q4k_scale_min(h, (int)((c % 256) / 32), dl, ml);
        return dl * (float)q - ml;  // d*sc*q is exact: one rounding, as gguf-py
    }
    if (type_id == QW35_Q6_K_TYPE) {
        const size_t code_row = (size_t)k / 2 + k / 4;
        const uint8_t *row = w + r * code_row;
        const uint8_t byte = row[c / 2];
        const uint32_t lo = (c & 1) ? (byte >> 4) : (byte & 0xf);
        const uint32_t hw = reinterpret_cast<const uint32_t *>(row + k / 2)[c / 16];
        const uint32_t e = c & 15;
        const uint32_t q = lo | (((hw >> (4 * (e & 7) + 2 * (e >> 3))) & 3u) << 4);
        const uint8_t *sr = w + rows * code_row + r * q6k_scale_row(k);
        const float sc = (float)reinterpret_cast<const int8_t *>(sr)[c / 16];
        const float d = __half2float(__ushort_as_half(reinterpret_cast<const unsigned short *>(sr + k / 16)[c / 256]));
        return (d * sc) * (float)((int)q - 32);  // both products exact in fp32
    }
    return reinterpret_cast<const float *>(w)[r * k + c];
}

template <bool EXACT>
__global__ void dequant_kernel(uint32_t type_id, const uint8_t *w, float *out, size_t rows, uint32_t k) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * k) return;
    out[i] = dequant_at<EXACT>(type_id, w, rows, k, i / k, (uint32_t)(i % k));
}

cudaError_t weight_dequant(uint32_t type_id, const void *w, float *out, uint32_t rows, uint32_t k, uint32_t flags,
                           cudaStream_t st) {
    const size_t n = (size_t)rows * k;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (flags & QW35_MV_GF4_EXACT)
        dequant_kernel<true><<<blocks, 256, 0, st>>>(type_id, static_cast<const uint8_t *>(w), out, rows, k);
    else
        dequant_kernel<false><<<blocks, 256, 0, st>>>(type_id, static_cast<const uint8_t *>(w), out, rows, k);
    return cudaGetLastError();
}

// ---- embedding row gather (qw35_matvec.metal:100-149) -------------------------------
__global__ void embed_kernel(uint32_t type_id, const uint8_t *w, const uint32_t *tokens, size_t vocab, uint32_t k,
                             float *out) {
    const int i = blockIdx.y;
    const uint32_t tok = tokens[i];
    for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < k; c += gridDim.x * blockDim.x)
        out[(size_t)i * k + c] = dequant_at<true>(type_id, w, vocab, k, tok, c);
}

cudaError_t embed_rows(uint32_t type_id, const void *w, size_t vocab, const uint32_t *tokens, int n,
                             uint32_t k, float *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    dim3 grid((k + 255) / 256, n);
    embed_kernel<<<grid, 256, 0, st>>>(type_id, static_cast<const uint8_t *>(w), tokens, vocab, k, out);
    return cudaGetLastError();
}

// ---- RMS norm (qw35_core.metal:14-48), one CTA per row ------------------------------
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *x, const float *w, float *out, int k, float eps) {
    __shared__ float red[32];
    const float *xr = x + (size_t)blockIdx.x * k;
    float s = 0.0f;
    for (int i = threadIdx.x; i < k; i += 256) s = fmaf(xr[i], xr[i], s);
    s = block_sum(s, red);
    const float inv = rsqrtf(s / (float)k + eps);
    for (int i = threadIdx.x; i < k; i += 256) out[(size_t)blockIdx.x * k + i] = xr[i] * inv * w[i];
}

cudaError_t rms_norm_run(const float *x, const float *w, float *out, int n, int k, float eps, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    rms_norm_kernel<<<n, 256, 0, st>>>(x, w, out, k, eps);
    return cudaGetLastError();
}

}  // namespace qw35
