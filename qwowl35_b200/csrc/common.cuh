// common.cuh -- shared device helpers for the qw35 B200 decode path (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define QW35_GF4_TYPE 100u
#define QW35_Q8_0_TYPE 8u
#define QW35_Q4_K_TYPE 12u
#define QW35_Q5_K_TYPE 13u
#define QW35_Q6_K_TYPE 14u
#define QW35_F32_TYPE 0u
#define QW35_F16_TYPE 1u

namespace qw35 {

constexpr int kWarp = 32;

// Device layout of the K-quants with a fifth/sixth code bit, per row of k
// weights (k % 256 == 0):
//   Q5_K codes plane row: k/2 bytes of element-ordered nibbles, then k/8 bytes
//        of high bits, one uint32 per 32-weight sub-block j: bit 4n + w holds
//        the high bit of element 8w + n of the sub-block (w = 0..3, n = 0..7).
//        Header plane row: the 16-byte {d, dmin, scales[12]} of each block.
//   Q6_K codes plane row: k/2 bytes of element-ordered low nibbles, then k/4
//        bytes of high bit pairs, one uint32 per 16 weights: bits 4n..4n+1 hold
//        element n's pair, bits 4n+2..4n+3 element 8+n's.
//        Scales plane row (q6k_scale_row bytes): k/16 int8 sub-block scales,
//        then the k/256 f16 block scales d, zero-padded to 16 bytes.
// The two-bits-per-nibble-slot placement lets the matvec decode a high part
// with the same shift-and-mask steps as a nibble.
__host__ __device__ constexpr uint32_t q6k_scale_row(uint32_t k) { return (k / 16 + k / 128 + 15u) & ~15u; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `red` needs 32 floats.
__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    return warp_sum(t);
}

// SiLU / sigmoid / softplus with the reference's formulas (qw35_types.metal:40-68).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

// e5m2 byte -> float through fp16 (byte << 8), exact.
__device__ __forceinline__ float e5m2_to_float(uint32_t byte) {
    return __half2float(__ushort_as_half((unsigned short)((byte & 0xffu) << 8)));
}

// Exact float of a small unsigned integer u < 2^23 via the 2^23 magic.
__device__ __forceinline__ float u23_to_float(uint32_t u) {
    return __uint_as_float(0x4B000000u | u) - 8388608.0f;
}

// Read-only 128-bit global load that bypasses L1 allocation (weights are
// streamed exactly once per launch).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

}  // namespace qw35

// Host-side helpers shared by the launch wrappers.
namespace qw35h {
int sm_count();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (current device, kernel)
cudaError_t smem_optin(const void *func, int bytes);
}
