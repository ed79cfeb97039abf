// ops.h -- internal C++ interface between the launch wrappers, the runtime
// and the extern "C" boundary.  No torch types anywhere.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/qw35_cuda.h"

namespace qw35 {

struct MatvecArgs {
    uint32_t type_id = 0;
    const void *w0 = nullptr;      // device layout (see quant.cuh)
    const void *w1 = nullptr;      // second matrix (gate/up pair)
    const void *x = nullptr;       // [batch][k]
    uint32_t x_dtype = 0;          // QW35_F32_TYPE / QW35_F16_TYPE
    const float *norm_w = nullptr; // fused RMS-norm prologue weight, or null
    float eps = 1e-6f;
    float *y = nullptr;            // [batch][rows]
    uint32_t rows = 0, k = 0;
    int batch = 1;
    int mode = 0;                  // 0 store, 1 accumulate, 2 swiglu pair
    uint32_t flags = 0;
    // tensor-core path scratch (activation tiles, row scales, two-pass
    // outputs), owned by the caller: dq_scratch_bytes(batch, k, rows) bytes.
    // Null: the call takes a stream-ordered allocation of its own.
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
};

cudaError_t matvec_run(const MatvecArgs &a, cudaStream_t st);
// h = silu(gate) * up, elementwise over n floats (h may alias gate)
cudaError_t swiglu_run(const float *gate, const float *up, float *h, size_t n, cudaStream_t st);
size_t argmax_workspace_bytes(uint32_t rows, uint32_t batch);
cudaError_t argmax_head_run(const MatvecArgs &a, uint32_t *tok, float *val, void *ws, size_t ws_bytes,
                            cudaStream_t st);

// tcgen05 batched path (dqgemm.cu): kDqMinBatch <= B <= 64, every codec, k % 256 == 0,
// 16-byte aligned weights, activations and norm weight.
constexpr int kDqMinBatch = 3;  // from 3 rows the CUDA-core path needs 2+ weight passes
bool dq_supported(const MatvecArgs &a);
cudaError_t dq_run(const MatvecArgs &a, int mode, uint32_t *tok, float *val, cudaStream_t st);
size_t dq_scratch_bytes(int B, uint32_t k, uint32_t rows_out);

cudaError_t weight_repack(uint32_t type_id, const void *src, void *dst, uint32_t rows, uint32_t k,
                          cudaStream_t st);
cudaError_t weight_dequant(uint32_t type_id, const void *w, float *out, uint32_t rows, uint32_t k,
                           uint32_t flags, cudaStream_t st);
cudaError_t embed_rows(uint32_t type_id, const void *w, size_t vocab, const uint32_t *tokens, int n,
                       uint32_t k, float *out, cudaStream_t st);

// ---- Gated DeltaNet -------------------------------------------------------
struct DeltaNetArgs {
    int n_seq = 0;
    const float *proj = nullptr;   // [n_seq][proj_stride]: qkv(8192) | z(4096) | beta(32) | alpha(32)
    int proj_stride = 0;
    const float *conv_w = nullptr; // [8192][4]
    const float *dt = nullptr;     // [32]
    const float *a = nullptr;      // [32]
    const float *norm_w = nullptr; // [128]
    float *conv_state = nullptr;   // base; seq i at + slot[i] * conv_stride floats
    float *ssm_state = nullptr;    // base; seq i at + slot[i] * ssm_stride floats
    const int32_t *slots = nullptr;// [n_seq] state slot per sequence (device); null = identity
    long long conv_stride = 0, ssm_stride = 0;
    float *out = nullptr;          // [n_seq][4096]
    int out_stride = 4096;
    float eps = 1e-6f;
};
cudaError_t deltanet_step_run(const DeltaNetArgs &a, cudaStream_t st);
// T consecutive tokens of ONE sequence (slot a.slots[0]): projection row t at
// a.proj + t * proj_stride, output row t at a.out + t * out_stride
cudaError_t deltanet_run_tokens(const DeltaNetArgs &a, int T, cudaStream_t st);

struct DeltaCoreArgs {
    int n_seq = 0;
    const __half *q = nullptr, *k = nullptr, *v = nullptr;  // [n][16][128], [n][16][128], [n][32][128]
    const float *beta = nullptr, *g = nullptr;              // [n][32]
    float *state = nullptr;                                 // [n][32][128][128]
    float *y = nullptr;                                     // [n][32][128]
    float scale = 0.08838834764831845f;
};
cudaError_t deltanet_core_run(const DeltaCoreArgs &a, cudaStream_t st);

// ---- attention --------------------------------------------------------------
struct AttnPreArgs {
    int n_seq = 0;
    const float *qkv = nullptr;    // [n][stride]: q_full(16*512) | k(1024) | v(1024)
    int qkv_stride = 0;
    const float *q_norm_w = nullptr, *k_norm_w = nullptr;  // [256]
    const float *rope_freq = nullptr;                      // [32]
    const int32_t *pos = nullptr;                          // [n]
    const uint64_t *chunk_ptrs = nullptr;                  // [rows][max_chunks] chunk base addresses
    const int32_t *slots = nullptr;                        // chunk-table row per sequence (null = i)
    int max_chunks = 0;
    long long k_off = 0, v_off = 0;                        // byte offsets of this layer's K / V planes
    float *q_out = nullptr;        // [n][16][256]
    float *gate_out = nullptr;     // [n][16][256]
    float eps = 1e-6f;
    int kv_q8 = 0;                 // 1: the planes hold q8_0 rows (kKvQ8Row bytes per head-row)
};
cudaError_t attn_preprocess_run(const AttnPreArgs &a, cudaStream_t st);

// q8_0 KV rows: 8 blocks {f16 d; int8 qs[32]} per 256-dim head row
// (qw35_attention.metal:425-445); a plane is [4 kv heads][256 pos][272 B].
constexpr int kKvQ8Row = 8 * 34;

struct AttnArgs {
    int n_seq = 0;
    const float *q = nullptr;      // [n][16][256]
    const float *gate = nullptr;   // [n][16][256] or null
    const int32_t *seq_len = nullptr;  // [n] tokens in cache (pos + 1)
    const uint64_t *chunk_ptrs = nullptr;
    const int32_t *slots = nullptr;
    int max_chunks = 0;
    long long k_off = 0, v_off = 0;
    int window = 0, sink = 0;
    int max_len = 0;               // upper bound of seq_len (sizes the split grid)
    float scale = 0.0625f;
    float *out = nullptr;          // [n][16][256]
    int out_stride = 4096;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    int kv_q8 = 0;                 // 1: q8_0 planes (see kKvQ8Row)
};
size_t attn_workspace_bytes(int n_seq, int max_len);
cudaError_t attn_decode_run(const AttnArgs &a, cudaStream_t st);
size_t attn_noalloc_limit();
cudaError_t attn_decode_noalloc_run(AttnArgs a, cudaStream_t st);  // ws taken from a static device array

unsigned int device_error_read_and_clear();

cudaError_t rms_norm_run(const float *x, const float *w, float *out, int n, int k, float eps, cudaStream_t st);

}  // namespace qw35
