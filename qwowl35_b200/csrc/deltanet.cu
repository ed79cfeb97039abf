// deltanet.cu -- Gated DeltaNet decode step on sm_100a.
//
// Reference: qw35_ssm_conv_recurrent_gate_norm_step128_par_f32,
// qw35-server/src/metal/qw35_ssm.metal:260-451 (launch: Qw35MetalRuntime+SSM.m:30-54).
//
// Per layer and sequence: 32 value heads x 128 state rows x 128 columns of
// fp32 state (2 MiB), read once and written once.  The reference runs one
// 256-thread threadgroup per qk group (16 per sequence).  Here one 512-thread
// CTA owns one value head (all 128 state rows, so the per-head RMS of y stays
// in the CTA), and the two heads g and g + 16 that share qk group g form a
// thread-block cluster of 2: both read the group's q/k conv window, so rank 0
// retires the conv-state shift only after a cluster barrier.  Every state
// byte is on a coalesced 512-byte row walk, issued at kernel entry.
#include <cooperative_groups.h>
#include <cstdlib>

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

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(512)
deltanet_step_kernel(DeltaNetArgs p) {
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();  // == blockIdx.x: value head g or g + 16
    const int g = blockIdx.y;
    const int seq = blockIdx.z;
    const int h = g + NQK * rank;
    const int tid = threadIdx.x;
    const long long slot = p.slots ? (long long)p.slots[seq] : (long long)seq;

    __shared__ __align__(16) float qn_s[DS];
    __shared__ __align__(16) float kn_s[DS];
    __shared__ float v_s[DS];
    __shared__ float y_s[DS];
    __shared__ float red[32];

    const float *proj = p.proj + (size_t)seq * p.proj_stride;
    float *cs = p.conv_state + slot * p.conv_stride;
    float *S = p.ssm_state + slot * p.ssm_stride + (size_t)h * DS * DS;

    // the head's 128 state rows are the bulk of the traffic: their loads go
    // out first (16 warps x 8 rows) and land while the prologue runs
    float4 sv[8];
    load_rows(S, sv);

    // (1) conv + SiLU: threads 0..127 the group's q channels, 128..255 its k
    // channels (both read by the two CTAs of the cluster), 256..383 this
    // head's value channels (exclusive: their window shifts right away)
    float q = 0.0f, k = 0.0f, qwin[3] = {0.f, 0.f, 0.f}, qx = 0.0f;
    int ch = -1;
    if (tid < 2 * DS) {
        ch = tid < DS ? g * DS + tid : NQK * DS + g * DS + (tid - DS);
        qwin[0] = cs[ch * 3 + 0]; qwin[1] = cs[ch * 3 + 1]; qwin[2] = cs[ch * 3 + 2];
        qx = proj[ch];
        const float4 w = reinterpret_cast<const float4 *>(p.conv_w)[ch];
        const float o = silu_f(qwin[0] * w.x + qwin[1] * w.y + qwin[2] * w.z + qx * w.w);
        if (tid < DS) q = o;
        else k = o;
    } else if (tid < 3 * DS) {
        const int d = tid - 2 * DS;
        const int vc = 2 * NQK * DS + h * DS + d;
        const float v0 = cs[vc * 3 + 0], v1 = cs[vc * 3 + 1], v2 = cs[vc * 3 + 2], vx = proj[vc];
        const float4 wv = reinterpret_cast<const float4 *>(p.conv_w)[vc];
        v_s[d] = silu_f(v0 * wv.x + v1 * wv.y + v2 * wv.z + vx * wv.w);
        cs[vc * 3 + 0] = v1;
        cs[vc * 3 + 1] = v2;
        cs[vc * 3 + 2] = vx;
    }

    // (2) L2 norms with max(norm, eps) and the normalised k.q dot
    const float q_ss = block_sum(q * q, red);
    const float k_ss = block_sum(k * k, red);
    if (tid < DS) qn_s[tid] = q * (1.0f / fmaxf(sqrtf(q_ss), p.eps));
    else if (tid < 2 * DS) kn_s[tid - DS] = k * (1.0f / fmaxf(sqrtf(k_ss), p.eps));
    __syncthreads();
    const float kq = block_sum(tid < DS ? qn_s[tid] * kn_s[tid] : 0.0f, red);

    // both heads of the group have read the old q/k window: rank 0 retires the shift
    cluster.sync();
    if (rank == 0 && ch >= 0) {
        cs[ch * 3 + 0] = qwin[1];
        cs[ch * 3 + 1] = qwin[2];
        cs[ch * 3 + 2] = qx;
    }

    // (3) gates and the delta-rule state update (16 warps x 8 rows)
    const float beta = sigmoid_f(proj[BOFF + h]);
    const float gate = expf(softplus_f(proj[AOFF + h] + p.dt[h]) * p.a[h]);
    const int lane = tid & 31;
    const float4 kc4 = reinterpret_cast<const float4 *>(kn_s)[lane];
    const float4 qc4 = reinterpret_cast<const float4 *>(qn_s)[lane];
    delta_rows(S, sv, kc4, qc4, v_s, gate, beta, kq, 0.08838834764831845f, y_s);
    __syncthreads();

    // (4) per-head RMS of y (all 128 rows are in this CTA), gated output
    const float y2 = block_sum(tid < DS ? y_s[tid] * y_s[tid] : 0.0f, red);
    const float inv = rsqrtf(y2 / (float)DS + p.eps);
    if (tid < DS) {
        const float z = proj[ZOFF + h * DS + tid];
        p.out[(size_t)seq * p.out_stride + h * DS + tid] = y_s[tid] * inv * p.norm_w[tid] * silu_f(z);
    }
}

// ---- small batches: a value head split over four CTAs ---------------------------
// With few sequences the one-CTA-per-head layout leaves most SMs idle (32 CTAs
// for one sequence).  Here a cluster of 8 CTAs covers the two heads of a qk
// group x four quarters of their 128 state rows (128 threads, 32 rows each):
// every CTA recomputes the group's q / k conv and norms (256 channels), the
// quarter's v rows and their window shift are its own, rank 0 retires the q / k
// window shift after a cluster barrier, and the per-head RMS of y is summed
// over the four quarters through distributed shared memory in a fixed order.
__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(128)
deltanet_step_quarter_kernel(DeltaNetArgs p) {
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();  // head half (rank / 4), row quarter (rank % 4)
    const int g = blockIdx.y;
    const int seq = blockIdx.z;
    const int h = g + NQK * (rank >> 2);
    const int qr = rank & 3;
    const int tid = threadIdx.x;
    const long long slot = p.slots ? (long long)p.slots[seq] : (long long)seq;

    __shared__ __align__(16) float qn_s[DS];
    __shared__ __align__(16) float kn_s[DS];
    __shared__ float v_s[ROWS];
    __shared__ float y_s[ROWS];
    __shared__ float red[32];
    __shared__ float ysq;

    const float *proj = p.proj + (size_t)seq * p.proj_stride;
    float *cs = p.conv_state + slot * p.conv_stride;
    float *S = p.ssm_state + slot * p.ssm_stride + (size_t)h * DS * DS + (size_t)qr * ROWS * DS;

    float4 sv[8];
    load_rows(S, sv);  // 4 warps x 8 rows of this quarter

    // (1) conv + SiLU: thread d computes q and k channel d of the group; threads
    // 0..31 the quarter's value channels (their window shifts right away)
    const int qc = g * DS + tid, kc = NQK * DS + g * DS + tid;
    const float qw0 = cs[qc * 3 + 0], qw1 = cs[qc * 3 + 1], qw2 = cs[qc * 3 + 2], qx = proj[qc];
    const float kw0 = cs[kc * 3 + 0], kw1 = cs[kc * 3 + 1], kw2 = cs[kc * 3 + 2], kx = proj[kc];
    const float4 wq = reinterpret_cast<const float4 *>(p.conv_w)[qc];
    const float4 wk = reinterpret_cast<const float4 *>(p.conv_w)[kc];
    const float q = silu_f(qw0 * wq.x + qw1 * wq.y + qw2 * wq.z + qx * wq.w);
    const float k = silu_f(kw0 * wk.x + kw1 * wk.y + kw2 * wk.z + kx * wk.w);
    if (tid < ROWS) {
        const int vc = 2 * NQK * DS + h * DS + qr * ROWS + tid;
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
    qn_s[tid] = q * (1.0f / fmaxf(sqrtf(q_ss), p.eps));
    kn_s[tid] = k * (1.0f / fmaxf(sqrtf(k_ss), p.eps));
    __syncthreads();
    const float kq = block_sum(qn_s[tid] * kn_s[tid], red);

    // every CTA of the cluster has read the old q/k window: rank 0 retires the shift
    cluster.sync();
    if (rank == 0) {
        cs[qc * 3 + 0] = qw1; cs[qc * 3 + 1] = qw2; cs[qc * 3 + 2] = qx;
        cs[kc * 3 + 0] = kw1; cs[kc * 3 + 1] = kw2; cs[kc * 3 + 2] = kx;
    }

    // (3) gates and the delta-rule update of the quarter's 32 rows
    const float beta = sigmoid_f(proj[BOFF + h]);
    const float gate = expf(softplus_f(proj[AOFF + h] + p.dt[h]) * p.a[h]);
    const int lane = tid & 31;
    const float4 kc4 = reinterpret_cast<const float4 *>(kn_s)[lane];
    const float4 qc4 = reinterpret_cast<const float4 *>(qn_s)[lane];
    delta_rows(S, sv, kc4, qc4, v_s, gate, beta, kq, 0.08838834764831845f, y_s);
    __syncthreads();

    // (4) the head's RMS of y: the four quarters' sums of squares, in rank order
    const float y2 = block_sum(tid < ROWS ? y_s[tid] * y_s[tid] : 0.0f, red);
    if (tid == 0) ysq = y2;
    cluster.sync();
    float tot = 0.0f;
    const int r0 = rank & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) tot += *cluster.map_shared_rank(&ysq, r0 + i);
    const float inv = rsqrtf(tot / (float)DS + p.eps);
    if (tid < ROWS) {
        const int d = qr * ROWS + tid;
        const float z = proj[ZOFF + h * DS + d];
        p.out[(size_t)seq * p.out_stride + h * DS + d] = y_s[tid] * inv * p.norm_w[d] * silu_f(z);
    }
    cluster.sync();  // the other CTAs' reads of ysq are done before this CTA exits
}

// ---- a run of T tokens of one sequence (prefill) ------------------------------
// The step kernel's CTA / cluster layout, looping over the run's tokens with
// the head's 128 x 128 state in registers (read once, written once per run)
// and the conv windows in registers (q/k windows written back by rank 0 after
// a cluster barrier, v windows by their own CTA).  Per token t it reads
// projection row t and writes output row t; the reference's batched prefill
// recurrence (qw35_ssm_recurrent_step128_batch_rows_f32, qw35_ssm.metal:453-535)
// likewise walks the rows in order with the state on chip.
__device__ __forceinline__ void delta_rows_reg(float4 *sv, const float4 kc, const float4 qc, const float *vrow,
                                               float gate, float beta, float kq, float scale, float *ysm) {
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
        sv[i].x = sv[i].x * gate + kc.x * delta;
        sv[i].y = sv[i].y * gate + kc.y * delta;
        sv[i].z = sv[i].z * gate + kc.z * delta;
        sv[i].w = sv[i].w * gate + kc.w * delta;
        if (lane == 0) ysm[r] = (gate * qd[i] + delta * kq) * scale;
    }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(512)
deltanet_run_kernel(DeltaNetArgs p, int T) {
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int g = blockIdx.y;
    const int h = g + NQK * rank;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const long long slot = p.slots ? (long long)p.slots[0] : 0;

    __shared__ __align__(16) float qn_s[DS];
    __shared__ __align__(16) float kn_s[DS];
    __shared__ float v_s[DS];
    __shared__ float y_s[DS];
    __shared__ float red[32];

    float *cs = p.conv_state + slot * p.conv_stride;
    float *S = p.ssm_state + slot * p.ssm_stride + (size_t)h * DS * DS;
    float4 sv[8];
    load_rows(S, sv);

    // conv windows: threads 0..255 the group's q / k channels, 256..383 this head's v channels
    int ch = -1;
    float win[3] = {0.f, 0.f, 0.f};
    float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < 2 * DS) ch = tid < DS ? g * DS + tid : NQK * DS + g * DS + (tid - DS);
    else if (tid < 3 * DS) ch = 2 * NQK * DS + h * DS + (tid - 2 * DS);
    if (ch >= 0) {
        win[0] = cs[ch * 3 + 0]; win[1] = cs[ch * 3 + 1]; win[2] = cs[ch * 3 + 2];
        cw = reinterpret_cast<const float4 *>(p.conv_w)[ch];
    }
    for (int t = 0; t < T; ++t) {
        const float *proj = p.proj + (size_t)t * p.proj_stride;
        float q = 0.0f, k = 0.0f;
        if (ch >= 0) {
            const float x = proj[ch];
            const float o = silu_f(win[0] * cw.x + win[1] * cw.y + win[2] * cw.z + x * cw.w);
            win[0] = win[1]; win[1] = win[2]; win[2] = x;
            if (tid < DS) q = o;
            else if (tid < 2 * DS) k = o;
            else v_s[tid - 2 * DS] = o;
        }
        const float q_ss = block_sum(q * q, red);
        const float k_ss = block_sum(k * k, red);
        if (tid < DS) qn_s[tid] = q * (1.0f / fmaxf(sqrtf(q_ss), p.eps));
        else if (tid < 2 * DS) kn_s[tid - DS] = k * (1.0f / fmaxf(sqrtf(k_ss), p.eps));
        __syncthreads();
        const float kq = block_sum(tid < DS ? qn_s[tid] * kn_s[tid] : 0.0f, red);
        const float beta = sigmoid_f(proj[BOFF + h]);
        const float gate = expf(softplus_f(proj[AOFF + h] + p.dt[h]) * p.a[h]);
        const float4 kc4 = reinterpret_cast<const float4 *>(kn_s)[lane];
        const float4 qc4 = reinterpret_cast<const float4 *>(qn_s)[lane];
        delta_rows_reg(sv, kc4, qc4, v_s, gate, beta, kq, 0.08838834764831845f, y_s);
        __syncthreads();
        const float y2 = block_sum(tid < DS ? y_s[tid] * y_s[tid] : 0.0f, red);
        const float inv = rsqrtf(y2 / (float)DS + p.eps);
        if (tid < DS) {
            const float z = proj[ZOFF + h * DS + tid];
            p.out[(size_t)t * p.out_stride + h * DS + tid] = y_s[tid] * inv * p.norm_w[tid] * silu_f(z);
        }
    }
    // state rows, written once
#pragma unroll
    for (int i = 0; i < 8; ++i) __stcs(reinterpret_cast<float4 *>(S + (size_t)(wid * 8 + i) * DS) + lane, sv[i]);
    // v windows are this head's own; the q / k windows are shared by the pair:
    // rank 0 writes them once both CTAs have read the old ones (at entry)
    if (tid >= 2 * DS && ch >= 0) {
        cs[ch * 3 + 0] = win[0]; cs[ch * 3 + 1] = win[1]; cs[ch * 3 + 2] = win[2];
    }
    cluster.sync();
    if (rank == 0 && tid < 2 * DS) {
        cs[ch * 3 + 0] = win[0]; cs[ch * 3 + 1] = win[1]; cs[ch * 3 + 2] = win[2];
    }
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
    if (a.n_seq <= 4) {
        // few sequences: four CTAs per head fill the SMs (cluster of 8 per qk group)
        deltanet_step_quarter_kernel<<<dim3(8, NQK, a.n_seq), 128, 0, st>>>(a);
        return cudaGetLastError();
    }
    dim3 grid(2, NQK, a.n_seq);
    deltanet_step_kernel<<<grid, 512, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t deltanet_run_tokens(const DeltaNetArgs &a, int T, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    dim3 grid(2, NQK, 1);
    deltanet_run_kernel<<<grid, 512, 0, st>>>(a, T);
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
