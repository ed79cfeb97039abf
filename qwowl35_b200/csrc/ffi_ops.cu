// ffi_ops.cu -- extern "C" per-op entry points (include/qw35_cuda.h).
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "ops.h"

namespace {

void set_err(char *err, uintptr_t len, const char *fmt, const char *detail) {
    if (!err || len == 0) return;
    snprintf(err, (size_t)len, fmt, detail ? detail : "");
}

int cuda_ok(cudaError_t e, const char *what, char *err, uintptr_t len) {
    if (e == cudaSuccess) return 1;
    if (err && len) snprintf(err, (size_t)len, "%s: %s", what, cudaGetErrorString(e));
    return 0;
}

bool type_ok(uint32_t t) {
    return t == QW35_GF4_TYPE || t == QW35_Q8_0_TYPE || t == QW35_Q4_K_TYPE || t == QW35_Q5_K_TYPE ||
           t == QW35_Q6_K_TYPE;
}

int check_shape(uint32_t type_id, uint32_t rows, uint32_t k, uint32_t batch, char *err, uintptr_t len) {
    if (!type_ok(type_id)) {
        set_err(err, len, "unsupported weight type%s", "");
        return 0;
    }
    if (rows == 0 || k == 0 || k % 256 != 0 || k > 12288) {
        set_err(err, len, "invalid matvec shape (k must be a positive multiple of 256, at most 12288)%s", "");
        return 0;
    }
    if (batch == 0 || batch > 64) {
        set_err(err, len, "batch must be in [1, 64]%s", "");
        return 0;
    }
    return 1;
}

}  // namespace

extern "C" {

int qw35_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int qw35_cuda_set_device(int device, char *err, uintptr_t err_len) {
    return cuda_ok(cudaSetDevice(device), "cudaSetDevice", err, err_len);
}

uint32_t qw35_cuda_device_error(void) { return qw35::device_error_read_and_clear(); }

const char *qw35_cuda_build_info(void) { return "qw35cuda sm_100a (" __DATE__ ")"; }

uint64_t qw35_cuda_weight_bytes(uint32_t type_id, uint32_t rows, uint32_t k) {
    switch (type_id) {
        case QW35_GF4_TYPE: return (uint64_t)rows * (k / 8) * 4;
        case QW35_Q8_0_TYPE: return (uint64_t)rows * (k / 32) * 34;
        case QW35_Q4_K_TYPE: return (uint64_t)rows * (k / 256) * 144;
        case QW35_Q5_K_TYPE: return (uint64_t)rows * (k / 256) * 176;
        case QW35_Q6_K_TYPE: return (uint64_t)rows * (k / 256) * 210;
        case QW35_F32_TYPE: return (uint64_t)rows * k * 4;
        default: return 0;
    }
}

uint64_t qw35_cuda_device_bytes(uint32_t type_id, uint32_t rows, uint32_t k) {
    const uint64_t raw = qw35_cuda_weight_bytes(type_id, rows, k);
    // Q8_0 carries one exponent byte per row after its scales plane (16-byte padded)
    if (type_id == QW35_Q8_0_TYPE && raw) return raw + (((uint64_t)rows + 15) & ~(uint64_t)15);
    // Q6_K rows of scales (k/16 int8 + k/128 bytes of f16 d) are padded to 16 bytes
    if (type_id == QW35_Q6_K_TYPE && raw) return (uint64_t)rows * (3 * (k / 4) + qw35::q6k_scale_row(k));
    return raw;
}

int qw35_cuda_weight_repack(uint32_t type_id, const void *src, void *dst, uint32_t rows, uint32_t k, void *stream,
                            char *err, uintptr_t err_len) {
    if (!check_shape(type_id, rows, k, 1, err, err_len)) return 0;
    if (!src || !dst || src == dst) {
        set_err(err, err_len, "repack needs distinct non-null src and dst%s", "");
        return 0;
    }
    return cuda_ok(qw35::weight_repack(type_id, src, dst, rows, k, (cudaStream_t)stream), "repack", err, err_len);
}

int qw35_cuda_dequant(uint32_t type_id, const void *w, float *out, uint32_t rows, uint32_t k, uint32_t flags,
                      void *stream, char *err, uintptr_t err_len) {
    if (!check_shape(type_id, rows, k, 1, err, err_len)) return 0;
    if (!w || !out) {
        set_err(err, err_len, "null pointer%s", "");
        return 0;
    }
    return cuda_ok(qw35::weight_dequant(type_id, w, out, rows, k, flags, (cudaStream_t)stream), "dequant", err,
                   err_len);
}

int qw35_cuda_matvec(uint32_t type_id, const void *w, const void *x, uint32_t x_dtype, float *y, uint32_t rows,
                     uint32_t k, uint32_t batch, int accumulate, uint32_t flags, void *stream, char *err,
                     uintptr_t err_len) {
    if (!check_shape(type_id, rows, k, batch, err, err_len)) return 0;
    if (!w || !x || !y || x_dtype > 1) {
        set_err(err, err_len, "invalid matvec arguments%s", "");
        return 0;
    }
    qw35::MatvecArgs a;
    a.type_id = type_id; a.w0 = w; a.x = x; a.x_dtype = x_dtype; a.y = y;
    a.rows = rows; a.k = k; a.batch = (int)batch; a.mode = accumulate ? 1 : 0; a.flags = flags;
    return cuda_ok(qw35::matvec_run(a, (cudaStream_t)stream), "matvec", err, err_len);
}

int qw35_cuda_gate_up_swiglu(uint32_t type_id, const void *w_gate, const void *w_up, const void *x,
                             uint32_t x_dtype, float *h, uint32_t rows, uint32_t k, uint32_t batch, uint32_t flags,
                             void *stream, char *err, uintptr_t err_len) {
    if (!check_shape(type_id, rows, k, batch, err, err_len)) return 0;
    if (!w_gate || !w_up || !x || !h || x_dtype > 1) {
        set_err(err, err_len, "invalid gate/up arguments%s", "");
        return 0;
    }
    qw35::MatvecArgs a;
    a.type_id = type_id; a.w0 = w_gate; a.w1 = w_up; a.x = x; a.x_dtype = x_dtype; a.y = h;
    a.rows = rows; a.k = k; a.batch = (int)batch; a.mode = 2; a.flags = flags;
    return cuda_ok(qw35::matvec_run(a, (cudaStream_t)stream), "gate_up_swiglu", err, err_len);
}

uint64_t qw35_cuda_argmax_workspace_bytes(uint32_t rows, uint32_t batch) {
    return qw35::argmax_workspace_bytes(rows, batch);
}

int qw35_cuda_argmax_head(uint32_t type_id, const void *w, const float *x, float *logits, uint32_t rows, uint32_t k,
                          uint32_t batch, uint32_t *token, float *logit, void *workspace, uint64_t workspace_bytes,
                          uint32_t flags, void *stream, char *err, uintptr_t err_len) {
    if (!check_shape(type_id, rows, k, batch, err, err_len)) return 0;
    if (!w || !x || !token || !workspace) {
        set_err(err, err_len, "invalid argmax arguments%s", "");
        return 0;
    }
    if (workspace_bytes < qw35::argmax_workspace_bytes(rows, batch)) {
        set_err(err, err_len, "argmax workspace too small%s", "");
        return 0;
    }
    qw35::MatvecArgs a;
    a.type_id = type_id; a.w0 = w; a.x = x; a.x_dtype = 0; a.y = logits;
    a.rows = rows; a.k = k; a.batch = (int)batch; a.mode = 3; a.flags = flags;
    return cuda_ok(qw35::argmax_head_run(a, token, logit, workspace, workspace_bytes, (cudaStream_t)stream),
                   "argmax_head", err, err_len);
}

int qw35_cuda_deltanet_step(uint32_t n_seq, const float *proj, uint32_t proj_stride, const float *conv_w,
                            const float *dt, const float *a_log, const float *norm_w, float *conv_state,
                            uint64_t conv_stride, float *ssm_state, uint64_t ssm_stride, const int32_t *slots,
                            float *out, float eps, void *stream, char *err, uintptr_t err_len) {
    if (n_seq == 0) return 1;
    if (!proj || !conv_w || !dt || !a_log || !norm_w || !conv_state || !ssm_state || !out || proj_stride < 12352 ||
        n_seq > 65535) {
        set_err(err, err_len, "invalid deltanet arguments%s", "");
        return 0;
    }
    qw35::DeltaNetArgs a;
    a.n_seq = (int)n_seq; a.proj = proj; a.proj_stride = (int)proj_stride; a.conv_w = conv_w; a.dt = dt;
    a.a = a_log; a.norm_w = norm_w; a.conv_state = conv_state; a.conv_stride = (long long)conv_stride;
    a.ssm_state = ssm_state; a.ssm_stride = (long long)ssm_stride; a.slots = slots; a.out = out; a.eps = eps;
    return cuda_ok(qw35::deltanet_step_run(a, (cudaStream_t)stream), "deltanet_step", err, err_len);
}

int qw35_cuda_deltanet_core(uint32_t n_seq, const uint16_t *q, const uint16_t *k, const uint16_t *v,
                            const float *beta, const float *g, float *state, float *y, void *stream, char *err,
                            uintptr_t err_len) {
    if (n_seq == 0) return 1;
    if (!q || !k || !v || !beta || !g || !state || !y || n_seq > 65535) {
        set_err(err, err_len, "invalid deltanet core arguments%s", "");
        return 0;
    }
    qw35::DeltaCoreArgs a;
    a.n_seq = (int)n_seq;
    a.q = reinterpret_cast<const __half *>(q);
    a.k = reinterpret_cast<const __half *>(k);
    a.v = reinterpret_cast<const __half *>(v);
    a.beta = beta; a.g = g; a.state = state; a.y = y;
    return cuda_ok(qw35::deltanet_core_run(a, (cudaStream_t)stream), "deltanet_core", err, err_len);
}

static int attn_pre_impl(int kv_q8, uint32_t n_seq, const float *qkv, uint32_t qkv_stride, const float *q_norm_w,
                              const float *k_norm_w, const float *rope_freq, const int32_t *pos,
                              const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off, uint64_t v_off,
                              float *q_out, float *gate_out, float eps, void *stream, char *err,
                              uintptr_t err_len) {
    if (n_seq == 0) return 1;
    if (!qkv || !q_norm_w || !k_norm_w || !rope_freq || !pos || !chunk_ptrs || !q_out || !gate_out ||
        qkv_stride < 10240 || max_chunks == 0 || (k_off % 16) || (v_off % 16)) {
        set_err(err, err_len, "invalid attention preprocess arguments%s", "");
        return 0;
    }
    qw35::AttnPreArgs a;
    a.n_seq = (int)n_seq; a.qkv = qkv; a.qkv_stride = (int)qkv_stride; a.q_norm_w = q_norm_w;
    a.k_norm_w = k_norm_w; a.rope_freq = rope_freq; a.pos = pos; a.chunk_ptrs = chunk_ptrs;
    a.max_chunks = (int)max_chunks; a.k_off = (long long)k_off; a.v_off = (long long)v_off;
    a.q_out = q_out; a.gate_out = gate_out; a.eps = eps; a.kv_q8 = kv_q8;
    return cuda_ok(qw35::attn_preprocess_run(a, (cudaStream_t)stream), "attn_preprocess", err, err_len);
}

int qw35_cuda_attn_preprocess(uint32_t n_seq, const float *qkv, uint32_t qkv_stride, const float *q_norm_w,
                              const float *k_norm_w, const float *rope_freq, const int32_t *pos,
                              const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off, uint64_t v_off,
                              float *q_out, float *gate_out, float eps, void *stream, char *err,
                              uintptr_t err_len) {
    return attn_pre_impl(0, n_seq, qkv, qkv_stride, q_norm_w, k_norm_w, rope_freq, pos, chunk_ptrs, max_chunks, k_off,
                         v_off, q_out, gate_out, eps, stream, err, err_len);
}

int qw35_cuda_attn_preprocess_q8_0(uint32_t n_seq, const float *qkv, uint32_t qkv_stride, const float *q_norm_w,
                                   const float *k_norm_w, const float *rope_freq, const int32_t *pos,
                                   const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off, uint64_t v_off,
                                   float *q_out, float *gate_out, float eps, void *stream, char *err,
                                   uintptr_t err_len) {
    return attn_pre_impl(1, n_seq, qkv, qkv_stride, q_norm_w, k_norm_w, rope_freq, pos, chunk_ptrs, max_chunks, k_off,
                         v_off, q_out, gate_out, eps, stream, err, err_len);
}

uint64_t qw35_cuda_gqa_workspace_bytes(uint32_t n_seq, uint32_t max_len) {
    return qw35::attn_workspace_bytes((int)n_seq, (int)max_len);
}

static int gqa_decode_impl(int kv_q8, uint32_t n_seq, const float *q, const float *gate, const int32_t *seq_len,
                         uint32_t max_len, const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off,
                         uint64_t v_off, int32_t window, int32_t sink, float *out, void *workspace,
                         uint64_t workspace_bytes, void *stream, char *err, uintptr_t err_len) {
    if (n_seq == 0) return 1;
    if (!q || !seq_len || !chunk_ptrs || !out || !workspace || max_len == 0 || max_chunks == 0 ||
        (uint64_t)max_chunks * QW35_KV_CHUNK < max_len || n_seq > 65535 || (k_off % 16) || (v_off % 16)) {
        set_err(err, err_len, "invalid attention arguments%s", "");
        return 0;
    }
    if (workspace_bytes < qw35::attn_workspace_bytes((int)n_seq, (int)max_len)) {
        set_err(err, err_len, "attention workspace too small%s", "");
        return 0;
    }
    qw35::AttnArgs a;
    a.n_seq = (int)n_seq; a.q = q; a.gate = gate; a.seq_len = seq_len; a.chunk_ptrs = chunk_ptrs;
    a.max_chunks = (int)max_chunks; a.k_off = (long long)k_off; a.v_off = (long long)v_off;
    a.window = window; a.sink = sink < 0 ? 0 : sink; a.max_len = (int)max_len; a.out = out;
    a.ws = workspace; a.ws_bytes = workspace_bytes; a.kv_q8 = kv_q8;
    return cuda_ok(qw35::attn_decode_run(a, (cudaStream_t)stream), "gqa_decode", err, err_len);
}

int qw35_cuda_gqa_decode(uint32_t n_seq, const float *q, const float *gate, const int32_t *seq_len,
                         uint32_t max_len, const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off,
                         uint64_t v_off, int32_t window, int32_t sink, float *out, void *workspace,
                         uint64_t workspace_bytes, void *stream, char *err, uintptr_t err_len) {
    return gqa_decode_impl(0, n_seq, q, gate, seq_len, max_len, chunk_ptrs, max_chunks, k_off, v_off, window, sink, out,
                           workspace, workspace_bytes, stream, err, err_len);
}

int qw35_cuda_gqa_decode_q8_0(uint32_t n_seq, const float *q, const float *gate, const int32_t *seq_len,
                              uint32_t max_len, const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off,
                              uint64_t v_off, int32_t window, int32_t sink, float *out, void *workspace,
                              uint64_t workspace_bytes, void *stream, char *err, uintptr_t err_len) {
    return gqa_decode_impl(1, n_seq, q, gate, seq_len, max_len, chunk_ptrs, max_chunks, k_off, v_off, window, sink, out,
                           workspace, workspace_bytes, stream, err, err_len);
}

uint64_t qw35_cuda_gqa_noalloc_max_bytes(void) { return qw35::attn_noalloc_limit(); }

int qw35_cuda_gqa_decode_noalloc(uint32_t n_seq, const float *q, const float *gate, const int32_t *seq_len,
                                 uint32_t max_len, const uint64_t *chunk_ptrs, uint32_t max_chunks, uint64_t k_off,
                                 uint64_t v_off, int32_t window, int32_t sink, float *out, void *stream, char *err,
                                 uintptr_t err_len) {
    if (n_seq == 0) return 1;
    if (!q || !seq_len || !chunk_ptrs || !out || max_len == 0 || max_chunks == 0 ||
        (uint64_t)max_chunks * QW35_KV_CHUNK < max_len || n_seq > 65535 || (k_off % 16) || (v_off % 16)) {
        set_err(err, err_len, "invalid attention arguments%s", "");
        return 0;
    }
    const size_t need = qw35::attn_workspace_bytes((int)n_seq, (int)max_len);
    if (need > qw35::attn_noalloc_limit()) {
        if (err && err_len)
            snprintf(err, (size_t)err_len,
                     "allocation-free attention needs %zu bytes of split partials for n_seq=%u, max_len=%u; "
                     "the static scratch holds %zu (use qw35_cuda_gqa_decode with a workspace)",
                     need, n_seq, max_len, qw35::attn_noalloc_limit());
        return 0;
    }
    qw35::AttnArgs a;
    a.n_seq = (int)n_seq; a.q = q; a.gate = gate; a.seq_len = seq_len; a.chunk_ptrs = chunk_ptrs;
    a.max_chunks = (int)max_chunks; a.k_off = (long long)k_off; a.v_off = (long long)v_off;
    a.window = window; a.sink = sink < 0 ? 0 : sink; a.max_len = (int)max_len; a.out = out;
    return cuda_ok(qw35::attn_decode_noalloc_run(a, (cudaStream_t)stream), "gqa_decode_noalloc", err, err_len);
}

}  // extern "C"
