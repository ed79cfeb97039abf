// deltanet.cu -- Gated DeltaNet decode step on sm_100a.
//
// Reference: qw35_ssm_conv_recurrent_gate_norm_step128_par_f32,
// qw35-server/src/metal/qw35_ssm.metal:260-451 (launch: Qw35MetalRuntime+SSM.m:30-54).
//
// Per layer and sequence: 32 value heads x 128 state rows x 128 columns of
// fp32 state (2 MiB), read once and written once.  The reference runs one
// 256-thread threadgroup per qk group (16 per sequence).  Here a thread-block
// CLUSTER of 8 CTAs owns one qk group g: CTA rank r handles value head
// g + 16*(r/4) and state rows [32*(r%4), 32*(r%4)+32).  That gives 128 CTAs
// per sequence (one per SM at batch 1) and keeps every state byte on a
// single coalesced 512-byte row walk.  Cross-CTA pieces use the cluster:
//   * the q/k conv window is read by all 8 CTAs, so rank 0 retires the
//     conv-state shift only after a cluster barrier;
//   * the per-head RMS of y spans the 4 CTAs of a head and is exchanged
//     through distributed shared memory.
#include <cooperative_groups.h>

#include "common.cuh"
#include "ops.h"

namespace cg = cooperative_groups;

namespace qw35 {

constexpr int DS = 128;         // state size (head dim)
constexpr int NQK = 16;         // qk groups
constexpr int NV = 32;          // value heads
constexpr int CONV_CH = 8192;   // q(2048) | k(2048) | v(4096)
constexpr int ZOFF = CONV_CH;   // z follows qkv in the fused projection
constexpr int BOFF = ZOFF + 4096;
constexpr int AOFF = BOFF + NV;
constexpr int ROWS = 32;        // state rows per CTA

// Delta-rule update of this CTA's 32 rows.  4 warps x 8 rows; each lane owns
// 4 consecutive state columns (one float4) of every row.
// This thread's 4 state columns of its warp's 8 rows (streamed: read once).
__device__ __forceinline__ void load_rows(const float *S, float4 *sv) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        sv[i] = __ldcs(reinterpret_cast<const float4 *>(S + (size_t)(wid * 8 + i) * DS) + lane);
}

__device__ __forceinline__ void delta_rows(float *S, const float4 *sv, const float4 kc, const float4 qc,
                                           const float *vrow, float gate, float beta, float kq, float scale,
                                           float *ysm) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float kd[8], qd[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        kd[i] = sv[i].x * kc.x + sv[i].y * kc.y + sv[i].z * kc.z + sv[i].w * kc.w;
        qd[i] = sv[i].x * qc.x + sv[i].y * qc.y + sv[i].z * qc.z + sv[i].w * qc.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            kd[i] += __shfl_xor_sync(0xffffffffu, kd[i], o);
            qd[i] += __shfl_xor_sync(0xffffffffu, qd[i], o);
        }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = wid * 8 + i;
        const float delta = (vrow[r] - gate * kd[i]) * beta;
        float4 n;
        n.x = sv[i].x * gate + kc.x * delta;
        n.y = sv[i].y * gate + kc.y * delta;
        n.z = sv[i].z * gate + kc.z * delta;
        n.w = sv[i].w * gate + kc.w * delta;
        __stcs(reinterpret_cast<float4 *>(S + (size_t)r * DS) + lane, n);  // written once, not re-read soon
        if (lane == 0) ysm[r] = (gate * qd[i] + delta * kq) * scale;
    }
}

__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(128)
deltanet_step_kernel(DeltaNetArgs p) {
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();  // == blockIdx.x
    const int g = blockIdx.y;
    const int seq = blockIdx.z;
    const int h = g + NQK * (rank >> 2);
    const int rb = rank & 3;
    const int tid = threadIdx.x;
    const long long slot = p.slots ? (long long)p.slots[seq] : (long long)seq;

    __shared__ __align__(16) float qn_s[DS];
    __shared__ __align__(16) float kn_s[DS];
    __shared__ float v_s[ROWS];
    __shared__ float y_s[ROWS];
    __shared__ float red[32];
    __shared__ float ssq;

    const float *proj = p.proj + (size_t)seq * p.proj_stride;
    float *cs = p.conv_state + slot * p.conv_stride;
    float *S = p.ssm_state + slot * p.ssm_stride + ((size_t)h * DS + rb * ROWS) * DS;

    // the state rows are the bulk of the traffic: their loads go out first and
    // land while the conv / norm prologue runs
    float4 sv[8];
    load_rows(S, sv);

    // (1) conv + SiLU of this group's q and k channels (every CTA of the cluster)
    const int qc = g * DS + tid, kc = NQK * DS + g * DS + tid;
    const float q0 = cs[qc * 3 + 0], q1 = cs[qc * 3 + 1], q2 = cs[qc * 3 + 2], qx = proj[qc];
    const float k0 = cs[kc * 3 + 0], k1 = cs[kc * 3 + 1], k2 = cs[kc * 3 + 2], kx = proj[kc];
    const float4 wq = reinterpret_cast<const float4 *>(p.conv_w)[qc];
    const float4 wk = reinterpret_cast<const float4 *>(p.conv_w)[kc];
    const float q = silu_f(q0 * wq.x + q1 * wq.y + q2 * wq.z + qx * wq.w);
    const float k = silu_f(k0 * wk.x + k1 * wk.y + k2 * wk.z + kx * wk.w);

    // value channels owned by this CTA (exclusive: shift their window right away)
    if (tid < ROWS) {
        const int vc = 2 * NQK * DS + h * DS + rb * ROWS + tid;
        const float v0 = cs[vc * 3 + 0], v1 = cs[vc * 3 + 1], v2 = cs[vc * 3 + 2], vx = proj[vc];
        const float4 wv = reinterpret_cast<const float4 *>(p.conv_w)[vc];
        v_s[tid] = silu_f(v0 * wv.x + v1 * wv.y + v2 * wv.z + vx * wv.w);
        cs[vc * 3 + 0] = v1;
        cs[vc * 3 + 1] = v2;
        cs[vc * 3 + 2] = vx;
    }

    // (2) L2 norms with max(norm, eps) and the normalised k.q dot
    const float q_ss = block_sum(q * q, red);
    const float k_ss = block_sum(k * k, red);
    const float qn = q * (1.0f / fmaxf(sqrtf(q_ss), p.eps));
    const float kn = k * (1.0f / fmaxf(sqrtf(k_ss), p.eps));
    const float kq = block_sum(qn * kn, red);
    qn_s[tid] = qn;
    kn_s[tid] = kn;

    // every CTA has read the old q/k window: rank 0 retires the shift
    cluster.sync();
    if (rank == 0) {
        cs[qc * 3 + 0] = q1; cs[qc * 3 + 1] = q2; cs[qc * 3 + 2] = qx;
        cs[kc * 3 + 0] = k1; cs[kc * 3 + 1] = k2; cs[kc * 3 + 2] = kx;
    }

    // (3) gates and the delta-rule state update
    const float beta = sigmoid_f(proj[BOFF + h]);
    const float gate = expf(softplus_f(proj[AOFF + h] + p.dt[h]) * p.a[h]);
    const int lane = tid & 31;
    const float4 kc4 = reinterpret_cast<const float4 *>(kn_s)[lane];
    const float4 qc4 = reinterpret_cast<const float4 *>(qn_s)[lane];
    delta_rows(S, sv, kc4, qc4, v_s, gate, beta, kq, 0.08838834764831845f, y_s);
    __syncthreads();

    // (4) per-head RMS of y across the 4 CTAs of this head (DSMEM)
    float y2 = tid < ROWS ? y_s[tid] * y_s[tid] : 0.0f;
    y2 = block_sum(y2, red);
    if (tid == 0) ssq = y2;
    cluster.sync();
    float tot = 0.0f;
    const int first = rank & 4;
#pragma unroll
    for (int r = 0; r < 4; ++r) tot += *cluster.map_shared_rank(&ssq, first + r);
    const float inv = rsqrtf(tot / (float)DS + p.eps);
    if (tid < ROWS) {
        const int d = rb * ROWS + tid;
        const float z = proj[ZOFF + h * DS + d];
        p.out[(size_t)seq * p.out_stride + h * DS + d] = y_s[tid] * inv * p.norm_w[d] * silu_f(z);
    }
    cluster.sync();  // peers may still read ssq
}

// Recurrent core only (config 3 of the benchmark): prepared q/k/v, beta, g.
__global__ void __launch_bounds__(128) deltanet_core_kernel(DeltaCoreArgs p) {
    const int rb = blockIdx.x & 3;
    const int h = blockIdx.x >> 2;
    const int seq = blockIdx.y;
    const int tid = threadIdx.x;
    const int g = h % NQK;
    float *S = p.state + (((size_t)seq * NV + h) * DS + rb * ROWS) * DS;
    float4 sv[8];
    load_rows(S, sv);  // issued first: lands while q/k/v are staged
    __shared__ __align__(16) float qn_s[DS];
    __shared__ __align__(16) float kn_s[DS];
    __shared__ float v_s[ROWS];
    __shared__ float y_s[ROWS];
    __shared__ float red[32];
    const float qv = __half2float(p.q[((size_t)seq * NQK + g) * DS + tid]);
    const float kv = __half2float(p.k[((size_t)seq * NQK + g) * DS + tid]);
    qn_s[tid] = qv;
    kn_s[tid] = kv;
    if (tid < ROWS) v_s[tid] = __half2float(p.v[((size_t)seq * NV + h) * DS + rb * ROWS + tid]);
    const float kq = block_sum(qv * kv, red);
    const float beta = p.beta[(size_t)seq * NV + h];
    const float gate = expf(p.g[(size_t)seq * NV + h]);
    const int lane = tid & 31;
    const float4 kc4 = reinterpret_cast<const float4 *>(kn_s)[lane];
    const float4 qc4 = reinterpret_cast<const float4 *>(qn_s)[lane];
    delta_rows(S, sv, kc4, qc4, v_s, gate, beta, kq, p.scale, y_s);
    __syncthreads();
    if (tid < ROWS) p.y[((size_t)seq * NV + h) * DS + rb * ROWS + tid] = y_s[tid];
}

cudaError_t deltanet_step_run(const DeltaNetArgs &a, cudaStream_t st) {
    if (a.n_seq <= 0) return cudaSuccess;
    if (a.n_seq > 65535) return cudaErrorInvalidValue;
    dim3 grid(8, NQK, a.n_seq);
    deltanet_step_kernel<<<grid, 128, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t deltanet_core_run(const DeltaCoreArgs &a, cudaStream_t st) {
    if (a.n_seq <= 0) return cudaSuccess;
    if (a.n_seq > 65535) return cudaErrorInvalidValue;
    dim3 grid(NV * 4, a.n_seq);
    deltanet_core_kernel<<<grid, 128, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace qw35
