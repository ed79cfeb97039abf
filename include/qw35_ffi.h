// qw35_ffi.h -- drop-in C ABI of the decode runtime, implemented for CUDA.
//
// The exported symbols, signatures and structs are the ones the reference
// engine's Rust wrapper binds (qw35-server/src/metal/bridge.rs:77-164), as
// declared by qw35-server/src/metal/bridge/Qw35FFI.h:18-118 and
// Qw35MetalTypes.h:9-66.  They keep their qw35_metal_* names so the Rust
// crate links against libqw35cuda.so unchanged; the implementation behind
// them is the B200 runtime (runtime.cu).  Structs are ABI-identical
// (field order and types) because Rust marshals them by layout.
//
// Conventions (Qw35FFI.h:3-4, Qw35FFI.m:15-18): every function reports
// failure by returning 0/NULL and writing a NUL-terminated message into the
// caller's err[err_len]; eval_* calls are asynchronous and GPU errors surface
// at the next waiting call (argmax, copy_logits, sync, reset, state_*).
#ifndef QW35_FFI_H
#define QW35_FFI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

// Qw35MetalTypes.h:9-16
typedef struct {
    uint64_t bytes;
    uint64_t mapped_bytes;
    uint64_t touches;
    uint64_t checksum;
    double elapsed_ms;
    uint32_t view_count;
} qw35_metal_warm_report;

// Qw35MetalTypes.h:18-27.  dims[0] is the innermost (K) extent, dims[1] rows.
typedef struct {
    const uint8_t *name;
    uintptr_t name_len;
    uint64_t dims[4];
    uint32_t n_dims;
    uint32_t type_id;
    uint64_t abs_offset;
    uint64_t bytes;
    uint64_t elements;
} qw35_metal_tensor_desc;

// Qw35MetalTypes.h:29-59 (append-only).
typedef struct {
    uint32_t transformer_layers;
    uint32_t embedding_length;
    uint32_t feed_forward_length;
    uint32_t attention_heads;
    uint32_t attention_kv_heads;
    uint32_t attention_key_length;
    uint32_t attention_value_length;
    uint32_t rope_dimension_count;
    int32_t rope_sections[4];
    float rope_freq_base;
    float rms_epsilon;
    uint32_t ssm_conv_kernel;
    uint32_t ssm_state_size;
    uint32_t ssm_group_count;
    uint32_t ssm_time_step_rank;
    uint32_t ssm_inner_size;
    uint32_t full_attention_interval;
    int32_t attn_window;
    int32_t attn_sink;
    uint32_t attn_gate;
    uint32_t n_cls_out;
} qw35_metal_hparams;

// Qw35MetalTypes.h:62-66
typedef enum {
    QW35_LOGITS_NONE = 0,
    QW35_LOGITS_ARGMAX = 1,
    QW35_LOGITS_FULL = 2,
} qw35_logits_mode;

// Qw35FFI.h:19 -- 1 if a CUDA device is visible.
int qw35_metal_has_device(void);

// Qw35FFI.h:22-33 -- touch the model mapping (page warm-up).  The metallib
// arguments are accepted and ignored (there is no shader library on CUDA).
int qw35_metal_warm_model_views(const void *model_map, uint64_t model_size, uint64_t map_offset,
                                uint64_t map_size, uint64_t max_tensor_bytes, const uint8_t *metallib,
                                uintptr_t metallib_len, uint64_t stride, qw35_metal_warm_report *report,
                                char *err, uintptr_t err_len);

// Qw35FFI.h:37-50 -- upload the mapped model to HBM (shared across runtimes
// created over the same mapping) and allocate one decode slot.
void *qw35_metal_runtime_create(const void *model_map, uint64_t model_size,
                                const qw35_metal_tensor_desc *tensors, uintptr_t tensor_count,
                                const qw35_metal_hparams *hparams, uint32_t ctx_size, uint32_t vocab_size,
                                uint32_t prefill_chunk, uint32_t kv_cache_type, const uint8_t *metallib,
                                uintptr_t metallib_len, char *err, uintptr_t err_len);

// Qw35FFI.h:52 -- NULL-safe.
void qw35_metal_runtime_destroy(void *runtime);

// Qw35FFI.h:55 -- drain, zero recurrent state, return KV chunks beyond the first.
int qw35_metal_runtime_reset(void *runtime, char *err, uintptr_t err_len);

// Qw35FFI.h:59-69 -- recurrent state blob: [conv_state f32 | ssm_state f32].
uint64_t qw35_metal_runtime_state_size(void *runtime);
int qw35_metal_runtime_state_export(void *runtime, uint8_t *buf, uint64_t len, char *err, uintptr_t err_len);
int qw35_metal_runtime_state_import(void *runtime, const uint8_t *buf, uint64_t len, char *err,
                                    uintptr_t err_len);

// Qw35FFI.h:72
int qw35_metal_runtime_sync(void *runtime, char *err, uintptr_t err_len);

// Qw35FFI.h:78-79 -- raise-only context ceiling.
int qw35_metal_runtime_set_ctx(void *runtime, uint32_t new_ctx, char *err, uintptr_t err_len);

// Qw35FFI.h:85 -- negative values clamp to 0.
void qw35_metal_runtime_set_attn_sink(void *runtime, int32_t sink);

// Qw35FFI.h:89-95 -- one token, asynchronous.
int qw35_metal_runtime_eval_token(void *runtime, uint32_t token, uint32_t pos, int logits_mode, char *err,
                                  uintptr_t err_len);

// Qw35FFI.h:97-104 -- a run of tokens (len <= prefill_chunk); head on the last.
int qw35_metal_runtime_eval_tokens(void *runtime, const uint32_t *tokens, uintptr_t len, uint32_t pos0,
                                   int logits_mode, char *err, uintptr_t err_len);

// Qw35FFI.h:106-111
int qw35_metal_runtime_argmax(void *runtime, uint32_t *token, float *logit, char *err, uintptr_t err_len);

// Qw35FFI.h:113-118 -- len >= vocab.
int qw35_metal_runtime_copy_logits(void *runtime, float *dst, uintptr_t len, char *err, uintptr_t err_len);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif  // QW35_FFI_H
