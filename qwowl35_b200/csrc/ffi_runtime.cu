// ffi_runtime.cu -- extern "C" runtime surface: the reference's qw35_metal_*
// functions (qw35-server/src/metal/bridge/Qw35FFI.m:201-431 is the code they
// replace) and the batched qw35_cuda_runtime_* extensions.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>

#include "runtime.h"

using qw35::Runtime;

namespace {

std::mutex g_mu;
std::set<void *> g_live;  // live handles: a stale or foreign pointer is rejected, not dereferenced

void set_err(char *err, uintptr_t len, const char *msg) {
    if (!err || len == 0) return;
    snprintf(err, (size_t)len, "%s", msg ? msg : "unknown CUDA runtime error");
}

Runtime *lookup(void *h) {
    std::lock_guard<std::mutex> g(g_mu);
    return g_live.count(h) ? static_cast<Runtime *>(h) : nullptr;
}

struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = 0;
        cudaGetDevice(&cur);
        if (cur != prev) cudaSetDevice(prev);
    }
};

// Run `fn` on a live runtime, mapping exceptions to the err buffer.
template <typename F>
int guarded(void *h, char *err, uintptr_t len, F &&fn) {
    Runtime *rt = lookup(h);
    if (!rt) {
        set_err(err, len, "invalid qw35 runtime handle");
        return 0;
    }
    DeviceGuard dg(rt->device);
    try {
        fn(rt);
        return 1;
    } catch (const std::exception &e) {
        set_err(err, len, e.what());
        return 0;
    }
}

void *create(const void *map, uint64_t size, const qw35_metal_tensor_desc *tensors, uintptr_t count,
             const qw35_metal_hparams *hp, uint32_t ctx, uint32_t vocab, uint32_t prefill_chunk, uint32_t kv_type,
             uint32_t max_seqs, char *err, uintptr_t len) {
    if (!map || !size || !tensors || !count || !hp) {
        set_err(err, len, "invalid runtime creation inputs");
        return nullptr;
    }
    // kv_cache_type (bridge.rs:31-42): 0 = f16, 1 = q8_0
    if (kv_type > 1) {
        set_err(err, len, "invalid kv_cache_type (0 = f16, 1 = q8_0)");
        return nullptr;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        set_err(err, len, "no CUDA device is available");
        return nullptr;
    }
    try {
        auto ms = qw35::shared_model(map, size, tensors, count, *hp, vocab);
        Runtime *rt = qw35::create_runtime(ms, *hp, ctx, vocab, prefill_chunk, max_seqs, kv_type);
        std::lock_guard<std::mutex> g(g_mu);
        g_live.insert(rt);
        return rt;
    } catch (const std::exception &e) {
        set_err(err, len, e.what());
        return nullptr;
    }
}

}  // namespace

extern "C" {

int qw35_metal_has_device(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n > 0;
}

int qw35_metal_warm_model_views(const void *model_map, uint64_t model_size, uint64_t map_offset, uint64_t map_size,
                                uint64_t max_tensor_bytes, const uint8_t *metallib, uintptr_t metallib_len,
                                uint64_t stride, qw35_metal_warm_report *report, char *err, uintptr_t err_len) {
    (void)metallib;
    (void)metallib_len;
    (void)max_tensor_bytes;
    if (report) memset(report, 0, sizeof(*report));
    if (!model_map || model_size == 0) {
        set_err(err, err_len, "invalid warmup inputs");
        return 0;
    }
    if (map_offset > model_size || map_size > model_size - map_offset) {
        set_err(err, err_len, "warmup range lies outside the model mapping");
        return 0;
    }
    const auto t0 = std::chrono::steady_clock::now();
    const uint64_t step = stride ? stride : 4096;
    const volatile uint8_t *p = static_cast<const uint8_t *>(model_map) + map_offset;
    uint64_t sum = 0, touches = 0;
    for (uint64_t off = 0; off < map_size; off += step, ++touches) sum += p[off];
    if (report) {
        report->bytes = map_size;
        report->mapped_bytes = map_size;
        report->touches = touches;
        report->checksum = sum;
        report->elapsed_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        report->view_count = 1;
    }
    return 1;
}

void *qw35_metal_runtime_create(const void *model_map, uint64_t model_size, const qw35_metal_tensor_desc *tensors,
                                uintptr_t tensor_count, const qw35_metal_hparams *hparams, uint32_t ctx_size,
                                uint32_t vocab_size, uint32_t prefill_chunk, uint32_t kv_cache_type,
                                const uint8_t *metallib, uintptr_t metallib_len, char *err, uintptr_t err_len) {
    (void)metallib;
    (void)metallib_len;
    uint32_t max_seqs = 1;
    if (const char *e = getenv("QW35_MAX_SEQS")) {
        const long v = strtol(e, nullptr, 10);
        if (v >= 1 && v <= 1024) max_seqs = (uint32_t)v;
    }
    return create(model_map, model_size, tensors, tensor_count, hparams, ctx_size, vocab_size, prefill_chunk,
                  kv_cache_type, max_seqs, err, err_len);
}

void *qw35_cuda_runtime_create(const void *model_map, uint64_t model_size, const qw35_metal_tensor_desc *tensors,
                               uintptr_t tensor_count, const qw35_metal_hparams *hparams, uint32_t ctx_size,
                               uint32_t vocab_size, uint32_t prefill_chunk, uint32_t kv_cache_type,
                               uint32_t max_seqs, char *err, uintptr_t err_len) {
    return create(model_map, model_size, tensors, tensor_count, hparams, ctx_size, vocab_size, prefill_chunk,
                  kv_cache_type, max_seqs, err, err_len);
}

void qw35_metal_runtime_destroy(void *runtime) {
    if (!runtime) return;
    Runtime *rt = nullptr;
    {
        std::lock_guard<std::mutex> g(g_mu);
        if (!g_live.erase(runtime)) return;
        rt = static_cast<Runtime *>(runtime);
    }
    delete rt;
}

int qw35_metal_runtime_reset(void *runtime, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [](Runtime *rt) { qw35::rt_reset_slot(rt, 0); });
}

uint64_t qw35_metal_runtime_state_size(void *runtime) {
    Runtime *rt = lookup(runtime);
    return rt ? qw35::rt_state_size(rt) : 0;
}

int qw35_metal_runtime_state_export(void *runtime, uint8_t *buf, uint64_t len, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) { qw35::rt_state_export(rt, 0, buf, len); });
}

int qw35_metal_runtime_state_import(void *runtime, const uint8_t *buf, uint64_t len, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) { qw35::rt_state_import(rt, 0, buf, len); });
}

int qw35_metal_runtime_sync(void *runtime, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [](Runtime *rt) { qw35::rt_wait(rt); });
}

int qw35_metal_runtime_set_ctx(void *runtime, uint32_t new_ctx, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) { qw35::rt_set_ctx(rt, new_ctx); });
}

void qw35_metal_runtime_set_attn_sink(void *runtime, int32_t sink) {
    Runtime *rt = lookup(runtime);
    if (!rt) return;
    const int s = sink < 0 ? 0 : sink;
    if (s != rt->attn_sink) {
        rt->attn_sink = s;  // baked into captured graphs: drop them
        DeviceGuard dg(rt->device);
        cudaStreamSynchronize(rt->stream);
        for (auto &kv : rt->graphs) cudaGraphExecDestroy(kv.second);
        rt->graphs.clear();
    }
}

int qw35_metal_runtime_eval_token(void *runtime, uint32_t token, uint32_t pos, int logits_mode, char *err,
                                  uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        const uint32_t seq = 0;
        qw35::rt_enqueue_step(rt, 1, &seq, &token, &pos, logits_mode);
    });
}

int qw35_metal_runtime_eval_tokens(void *runtime, const uint32_t *tokens, uintptr_t len, uint32_t pos0,
                                   int logits_mode, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (!tokens || len == 0) qw35::fail("empty token run");
        if (len > rt->prefill_chunk) qw35::fail("token run longer than the prefill chunk");
        if ((uint64_t)pos0 + len > rt->ctx) qw35::fail("requested position exceeds allocated context");
        const uint32_t seq = 0;
        if (rt->batched_prefill && len > 1) {
            // one pass per run of up to rt->rows tokens: weights are
            // read once per run instead of once per token; the head only on the last
            for (uintptr_t i = 0; i < len; i += rt->rows) {
                const uint32_t m = (uint32_t)std::min<uintptr_t>(rt->rows, len - i);
                qw35::rt_enqueue_prefill(rt, seq, tokens + i, m, pos0 + (uint32_t)i,
                                         i + m == len ? logits_mode : QW35_LOGITS_NONE);
            }
            return;
        }
        // otherwise a run is evaluated as consecutive decode steps, the head only on the last
        for (uintptr_t i = 0; i < len; ++i) {
            const uint32_t pos = pos0 + (uint32_t)i;
            const int mode = i + 1 == len ? logits_mode : QW35_LOGITS_NONE;
            qw35::rt_enqueue_step(rt, 1, &seq, &tokens[i], &pos, mode);
        }
    });
}

int qw35_metal_runtime_argmax(void *runtime, uint32_t *token, float *logit, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (!token || !logit) qw35::fail("invalid argmax output pointers");
        qw35::rt_wait(rt);
        if (rt->last_mode != QW35_LOGITS_ARGMAX) qw35::fail("the last eval did not run the argmax head");
        *token = rt->h_argmax_tok[0];
        *logit = rt->h_argmax_val[0];
    });
}

int qw35_metal_runtime_copy_logits(void *runtime, float *dst, uintptr_t len, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (!dst || len < rt->vocab) qw35::fail("invalid logits readback buffer");
        qw35::rt_wait(rt);
        qw35::ck(cudaMemcpy(dst, rt->logits, (size_t)rt->vocab * 4, cudaMemcpyDeviceToHost), "logits readback");
    });
}

// ---- batched extensions --------------------------------------------------------
int qw35_cuda_runtime_seq_alloc(void *runtime, uint32_t *seq_id, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (!seq_id) qw35::fail("null seq_id");
        for (uint32_t s = 0; s < rt->max_seqs; ++s)
            if (!rt->slot_used[s]) {
                rt->slot_used[s] = true;
                qw35::rt_reset_slot(rt, s);
                *seq_id = s;
                return;
            }
        qw35::fail("all %u sequence slots are in use", rt->max_seqs);
    });
}

int qw35_cuda_runtime_seq_free(void *runtime, uint32_t seq_id, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (seq_id == 0 || seq_id >= rt->max_seqs || !rt->slot_used[seq_id])
            qw35::fail("sequence %u is not an allocated slot (slot 0 is permanent)", seq_id);
        qw35::rt_wait(rt);
        qw35::rt_reset_slot(rt, seq_id);
        qw35::rt_release_kv(rt, seq_id, 0);
        rt->slot_used[seq_id] = false;
    });
}

int qw35_cuda_runtime_seq_reset(void *runtime, uint32_t seq_id, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (seq_id >= rt->max_seqs || !rt->slot_used[seq_id]) qw35::fail("sequence %u is not allocated", seq_id);
        qw35::rt_reset_slot(rt, seq_id);
    });
}

int qw35_cuda_runtime_seq_fork(void *runtime, uint32_t src, uint32_t dst, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (src >= rt->max_seqs || !rt->slot_used[src] || dst >= rt->max_seqs || !rt->slot_used[dst])
            qw35::fail("fork needs two allocated sequences");
        qw35::rt_fork(rt, src, dst);
    });
}

int qw35_cuda_runtime_seq_fill_synthetic(void *runtime, uint32_t seq_id, uint32_t positions, uint64_t seed,
                                         char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (seq_id >= rt->max_seqs || !rt->slot_used[seq_id]) qw35::fail("sequence %u is not allocated", seq_id);
        if (positions > rt->ctx) qw35::fail("%u positions exceed the context of %u", positions, rt->ctx);
        qw35::rt_fill_synthetic(rt, seq_id, positions, seed);
    });
}

uint32_t qw35_cuda_runtime_max_seqs(void *runtime) {
    Runtime *rt = lookup(runtime);
    return rt ? rt->max_seqs : 0;
}

int qw35_cuda_runtime_eval_batch(void *runtime, uint32_t n, const uint32_t *seq_ids, const uint32_t *tokens,
                                 const uint32_t *pos, int logits_mode, char *err, uintptr_t err_len) {
    return guarded(runtime, err, err_len,
                   [&](Runtime *rt) { qw35::rt_enqueue_step(rt, n, seq_ids, tokens, pos, logits_mode); });
}

int qw35_cuda_runtime_argmax_batch(void *runtime, uint32_t n, uint32_t *tokens, float *logits, char *err,
                                   uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (!tokens) qw35::fail("null token output");
        qw35::rt_wait(rt);
        if (rt->last_mode != QW35_LOGITS_ARGMAX || n > (uint32_t)rt->last_n)
            qw35::fail("the last eval did not produce %u argmax results", n);
        memcpy(tokens, rt->h_argmax_tok, 4ull * n);
        if (logits) memcpy(logits, rt->h_argmax_val, 4ull * n);
    });
}

int qw35_cuda_runtime_copy_logits_batch(void *runtime, uint32_t n, float *dst, uintptr_t len, char *err,
                                        uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (!dst || len < (uintptr_t)n * rt->vocab) qw35::fail("invalid logits readback buffer");
        if (rt->last_mode != QW35_LOGITS_FULL || n > (uint32_t)rt->last_n)
            qw35::fail("the last eval did not produce %u logits rows", n);
        qw35::rt_wait(rt);
        qw35::ck(cudaMemcpy(dst, rt->logits, (size_t)n * rt->vocab * 4, cudaMemcpyDeviceToHost), "logits readback");
    });
}

int qw35_cuda_runtime_seq_state_export(void *runtime, uint32_t seq_id, uint8_t *buf, uint64_t len, char *err,
                                       uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (seq_id >= rt->max_seqs || !rt->slot_used[seq_id]) qw35::fail("sequence %u is not allocated", seq_id);
        qw35::rt_state_export(rt, seq_id, buf, len);
    });
}

int qw35_cuda_runtime_seq_state_import(void *runtime, uint32_t seq_id, const uint8_t *buf, uint64_t len, char *err,
                                       uintptr_t err_len) {
    return guarded(runtime, err, err_len, [&](Runtime *rt) {
        if (seq_id >= rt->max_seqs || !rt->slot_used[seq_id]) qw35::fail("sequence %u is not allocated", seq_id);
        qw35::rt_state_import(rt, seq_id, buf, len);
    });
}

void *qw35_cuda_runtime_stream(void *runtime) {
    Runtime *rt = lookup(runtime);
    return rt ? (void *)rt->stream : nullptr;
}

uint32_t qw35_cuda_runtime_last_step_kernels(void *runtime) {
    Runtime *rt = lookup(runtime);
    return rt ? rt->last_kernels : 0;
}

uint64_t qw35_cuda_runtime_kv_bytes(void *runtime) {
    Runtime *rt = lookup(runtime);
    return rt ? rt->kv_bytes : 0;
}

uint64_t qw35_cuda_runtime_weight_bytes(void *runtime) {
    Runtime *rt = lookup(runtime);
    return rt ? rt->model->bytes : 0;
}

uint64_t qw35_cuda_runtime_scratch(void *runtime, uint64_t *bytes) {
    Runtime *rt = lookup(runtime);
    if (bytes) *bytes = rt ? rt->dq_scratch_bytes : 0;
    return rt ? reinterpret_cast<uint64_t>(rt->dq_scratch) : 0;
}

}  // extern "C"
