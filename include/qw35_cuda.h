// qw35_cuda.h -- B200 extensions of the decode C ABI: per-op kernel entry
// points and the batched (multi-sequence) runtime.
//
// The reference engine decodes one sequence per runtime and exposes no
// per-op entry points (qw35-server/src/metal/bridge/Qw35FFI.h:18-118).  The
// functions below are additions: the single-sequence qw35_metal_* surface in
// qw35_ffi.h maps onto sequence slot 0 of the same runtime.  Conventions are
// the reference's: return 1 (or a size) on success, 0 on failure with a
// NUL-terminated message in err[err_len]; device pointers are plain
// addresses on the current CUDA device; `stream` is a cudaStream_t (NULL =
// legacy default stream).  Per-op calls are asynchronous on that stream;
// a per-op matvec that needs tensor-core scratch takes it from the stream's
// memory pool (cudaMallocAsync / cudaFreeAsync on `stream`), so it never
// synchronises the device and never shares scratch with another call.
#ifndef QW35_CUDA_H
#define QW35_CUDA_H

#include <stddef.h>
#include <stdint.h>

#include "qw35_ffi.h"

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

// GGUF tensor type ids handled by the kernels (loader/tensors.rs:123-172).
#define QW35_TYPE_F32 0u
#define QW35_TYPE_F16 1u
#define QW35_TYPE_Q8_0 8u
#define QW35_TYPE_Q4_K 12u
#define QW35_TYPE_Q5_K 13u
#define QW35_TYPE_Q6_K 14u
#define QW35_TYPE_GF4 100u

// Matvec flags.  Default GF4 decode is bit-exact with the reference decode
// kernel qw35_gf4_dot8_vec_f32 (qw35_gf4.metal:8-20), including its element-4
// quirk; QW35_MV_GF4_EXACT selects the cooker's exact reconstruction
// (4 - q) * 0.25 * s (tools/qw35_cook_common.py:67-80).
#define QW35_MV_GF4_EXACT 1u

// KV cache granularity: positions per chunk.
#define QW35_KV_CHUNK 256u

// Library / device ------------------------------------------------------------
int qw35_cuda_device_count(void);
int qw35_cuda_set_device(int device, char *err, uintptr_t err_len);
const char *qw35_cuda_build_info(void);
// Bounded device-side waits record a nonzero code here instead of hanging;
// returns the code seen since the last call (0 = none) and clears it.
uint32_t qw35_cuda_device_error(void);

// Weights ---------------------------------------------------------------------
// Bytes of a rows x k matrix of `type_id` in GGUF block layout.
uint64_t qw35_cuda_weight_bytes(uint32_t type_id, uint32_t rows, uint32_t k);
// Bytes of the same matrix in device layout: as GGUF, except Q8_0, which adds a
// plane of one exponent byte per row (16-byte padded) for the tensor-core path.
uint64_t qw35_cuda_device_bytes(uint32_t type_id, uint32_t rows, uint32_t k);
// GGUF block layout (device memory) -> device layout (quant.cuh); dst holds
// qw35_cuda_device_bytes.  src != dst.
int qw35_cuda_weight_repack(uint32_t type_id, const void *src, void *dst, uint32_t rows, uint32_t k,
                            void *stream, char *err, uintptr_t err_len);
// Device-layout weights -> float32 [rows][k] (bit-exact dequantisation).
int qw35_cuda_dequant(uint32_t type_id, const void *w, float *out, uint32_t rows, uint32_t k, uint32_t flags,
                      void *stream, char *err, uintptr_t err_len);

// Matvec family (qw35_gf4.metal:62-246, qw35_matvec.metal:171-683) -------------
// y[b][r] (+)= sum_k W[r][k] x[b][k]; x is f32 (x_dtype 0) or f16 (x_dtype 1),
// fp32 accumulation.  k % 256 == 0.
int qw35_cuda_matvec(uint32_t type_id, const void *w, const void *x, uint32_t x_dtype, float *y, uint32_t rows,
                     uint32_t k, uint32_t batch, int accumulate, uint32_t flags, void *stream, char *err,
                     uintptr_t err_len);
// h[b][r] = silu(Wg[r].x[b]) * (Wu[r].x[b])   (qw35_gf4.metal:62-96)
int qw35_cuda_gate_up_swiglu(uint32_t type_id, const void *w_gate, const void *w_up, const void *x,
                             uint32_t x_dtype, float *h, uint32_t rows, uint32_t k, uint32_t batch,
                             uint32_t flags, void *stream, char *err, uintptr_t err_len);
// Fused head matvec + argmax (qw35_gf4.metal:140-206 + qw35_output.metal:141-182):
// token[b] = lowest id of the largest logit; logits optionally stored [batch][rows].
uint64_t qw35_cuda_argmax_workspace_bytes(uint32_t rows, uint32_t batch);
int qw35_cuda_argmax_head(uint32_t type_id, const void *w, const float *x, float *logits, uint32_t rows, uint32_t k,
                          uint32_t batch, uint32_t *token, float *logit, void *workspace, uint64_t workspace_bytes,
                          uint32_t flags, void *stream, char *err, uintptr_t err_len);

// Gated DeltaNet (qw35_ssm.metal:260-451) ------------------------------------
// Fused decode step for one layer over n_seq sequences.  proj[i] holds
// qkv(8192) | z(4096) | beta(32) | alpha(32) at stride proj_stride floats.
// conv_state: per slot [8192][3] f32 at stride conv_stride floats; ssm_state:
// per slot [32][128 v][128 k] f32 at stride ssm_stride floats; slots[i] (device
// int32, or NULL for i) picks the state slot of sequence i.  out [n][4096].
int qw35_cuda_deltanet_step(uint32_t n_seq, const float *proj, uint32_t proj_stride, const float *conv_w,
                            const float *dt, const float *a, const float *norm_w, float *conv_state,
                            uint64_t conv_stride, float *ssm_state, uint64_t ssm_stride, const int32_t *slots,
                            float *out, float eps, void *stream, char *err, uintptr_t err_len);
// Recurrent core only: q, k [n][16][128] f16 (L2-normalised),
// v [n][32][128] f16, beta [n][32] (post-sigmoid), g [n][32] log-decay;
// state [n][32][128][128] f32 updated in place; y [n][32][128] f32.
int qw35_cuda_deltanet_core(uint32_t n_seq, const uint16_t *q, const uint16_t *k, const uint16_t *v,
                            const float *beta, const float *g, float *state, float *y, void *stream, char *err,
                            uintptr_t err_len);

// GQA decode attention over the chunk table (qw35_attention.metal:29-414) ---
// chunk_ptrs [n][max_chunks]: device address of the chunk holding positions
// [256c, 256c+256) of sequence i.  Within a chunk this layer's K plane starts
// at byte k_off and V at v_off; each plane is [4 kv heads][256 pos][256 dim] f16.
int qw35_cuda_attn_preprocess(uint32_t n_seq, const float *qkv, uint32_t qkv_stride, const float *q_norm_w,
                              const float *k_norm_w, const float *rope_freq, const int32_t *pos,
                              const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off, uint64_t v_off,
                              float *q_out, float *gate_out, float eps, void *stream, char *err,
                              uintptr_t err_len);
uint64_t qw35_cuda_gqa_workspace_bytes(uint32_t n_seq, uint32_t max_len);
int qw35_cuda_gqa_decode(uint32_t n_seq, const float *q, const float *gate, const int32_t *seq_len,
                         uint32_t max_len, const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off,
                         uint64_t v_off, int32_t window, int32_t sink, float *out, void *workspace,
                         uint64_t workspace_bytes, void *stream, char *err, uintptr_t err_len);

// q8_0 KV twins (qw35_attn_decode_preprocess_q8_0_f32 and
// qw35_attention_gqa_flash_decode[_split]_q8_0_f32, qw35_attention.metal:425-793):
// same arguments, planes of [4 kv heads][256 pos][8 blocks {f16 d; int8 qs[32]}]
// (272 bytes per head-row).  The preprocess quantises each 32-value block of
// K (after norm + RoPE) and V as the reference does: d = amax / 127, codes
// round(x / d) clamped to +-127, d stored as f16.
int qw35_cuda_attn_preprocess_q8_0(uint32_t n_seq, const float *qkv, uint32_t qkv_stride, const float *q_norm_w,
                                   const float *k_norm_w, const float *rope_freq, const int32_t *pos,
                                   const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off, uint64_t v_off,
                                   float *q_out, float *gate_out, float eps, void *stream, char *err,
                                   uintptr_t err_len);
int qw35_cuda_gqa_decode_q8_0(uint32_t n_seq, const float *q, const float *gate, const int32_t *seq_len,
                              uint32_t max_len, const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off,
                              uint64_t v_off, int32_t window, int32_t sink, float *out, void *workspace,
                              uint64_t workspace_bytes, void *stream, char *err, uintptr_t err_len);

// Allocation-free twin of qw35_cuda_gqa_decode (no counterpart in the
// reference).  For callers that cannot allocate device memory where they
// decode (their GPU memory belongs to another allocator, or a cudaMalloc and
// its implicit synchronisation is not allowed there): the split partials use
// a static 16 MiB device array inside the library instead of a caller
// workspace, so this call allocates nothing.  Arguments and results are those
// of qw35_cuda_gqa_decode without the workspace.  Fails (0 + message) when
// qw35_cuda_gqa_workspace_bytes(n_seq, max_len) exceeds
// qw35_cuda_gqa_noalloc_max_bytes().  The first call on a device looks up the
// array's device address (make it before any stream capture); all calls share
// the array, so calls that may run concurrently on the GPU must not overlap.
// The looked-up address is kept for the life of the process: after a
// cudaDeviceReset of a device this entry point must not be called on it.
uint64_t qw35_cuda_gqa_noalloc_max_bytes(void);
int qw35_cuda_gqa_decode_noalloc(uint32_t n_seq, const float *q, const float *gate, const int32_t *seq_len,
                                 uint32_t max_len, const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off,
                                 uint64_t v_off, int32_t window, int32_t sink, float *out, void *stream, char *err,
                                 uintptr_t err_len);

// Batched runtime (extension of Qw35FFI.h) -----------------------------------
// Sequences live in slots; slot 0 is the one the qw35_metal_* calls use.
// Same arguments as qw35_metal_runtime_create plus the number of sequence
// slots (qw35_metal_runtime_create uses 1, or $QW35_MAX_SEQS when set).
void *qw35_cuda_runtime_create(const void *model_map, uint64_t model_size, const qw35_metal_tensor_desc *tensors,
                               uintptr_t tensor_count, const qw35_metal_hparams *hparams, uint32_t ctx_size,
                               uint32_t vocab_size, uint32_t prefill_chunk, uint32_t kv_cache_type,
                               uint32_t max_seqs, char *err, uintptr_t err_len);
int qw35_cuda_runtime_seq_alloc(void *runtime, uint32_t *seq_id, char *err, uintptr_t err_len);
int qw35_cuda_runtime_seq_free(void *runtime, uint32_t seq_id, char *err, uintptr_t err_len);
int qw35_cuda_runtime_seq_reset(void *runtime, uint32_t seq_id, char *err, uintptr_t err_len);
uint32_t qw35_cuda_runtime_max_seqs(void *runtime);
// Copy sequence src (recurrent state and KV chunks) into allocated sequence
// dst; both then continue from the same prefix.  Waits for the device.
int qw35_cuda_runtime_seq_fork(void *runtime, uint32_t src, uint32_t dst, char *err, uintptr_t err_len);
// Benchmark helper (no counterpart in the reference): gives sequence seq_id a
// KV cache of `positions` rows in every attention layer, filled with
// deterministic pseudo-random values from `seed` (f16 planes: uniform in
// [-2, 2); q8_0 planes: d = 2/127, codes uniform in [-127, 127]), so a long
// context can be decoded without prefilling it.  The recurrent state is left
// as it is.  Waits for the device.
int qw35_cuda_runtime_seq_fill_synthetic(void *runtime, uint32_t seq_id, uint32_t positions, uint64_t seed,
                                         char *err, uintptr_t err_len);
// One decode step for n sequences (token ids and positions are host arrays).
int qw35_cuda_runtime_eval_batch(void *runtime, uint32_t n, const uint32_t *seq_ids, const uint32_t *tokens,
                                 const uint32_t *pos, int logits_mode, char *err, uintptr_t err_len);
// Waits, then reads the greedy tokens / logits of the last eval_batch.
int qw35_cuda_runtime_argmax_batch(void *runtime, uint32_t n, uint32_t *tokens, float *logits, char *err,
                                   uintptr_t err_len);
int qw35_cuda_runtime_copy_logits_batch(void *runtime, uint32_t n, float *dst, uintptr_t len, char *err,
                                        uintptr_t err_len);
// Per-slot recurrent state blob [conv f32 | ssm f32] (same size as state_size).
int qw35_cuda_runtime_seq_state_export(void *runtime, uint32_t seq_id, uint8_t *buf, uint64_t len, char *err,
                                       uintptr_t err_len);
int qw35_cuda_runtime_seq_state_import(void *runtime, uint32_t seq_id, const uint8_t *buf, uint64_t len,
                                       char *err, uintptr_t err_len);
// The CUDA stream every step of this runtime is enqueued on (cudaStream_t),
// for callers that order their own work or timing events against it.
void *qw35_cuda_runtime_stream(void *runtime);
// Kernels in the last step's launch (the captured graph's kernel nodes).
uint32_t qw35_cuda_runtime_last_step_kernels(void *runtime);
// Device bytes held by the runtime's KV chunk pool and by the shared weights.
uint64_t qw35_cuda_runtime_kv_bytes(void *runtime);
uint64_t qw35_cuda_runtime_weight_bytes(void *runtime);
// Device address (and, in *bytes, the size) of the scratch this runtime's
// tensor-core matvecs use.  Each runtime owns its scratch from create to
// destroy; its captured step graphs hold this address, which never changes.
// 0 when no batch of the runtime reaches the tensor-core path.
uint64_t qw35_cuda_runtime_scratch(void *runtime, uint64_t *bytes);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif  // QW35_CUDA_H
