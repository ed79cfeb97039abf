// runtime.h -- the B200 decode runtime behind the qw35_metal_* C ABI.
//
// Mirrors the reference runtime's responsibilities
// (qw35-server/src/metal/bridge/Qw35MetalRuntime.m): shared weights per
// model mapping (:42-80), recurrent state buffers (:374-460), the
// append-only KV cache (:496-538, :713-735), per-token decode orchestration
// (:807-880, :1170-1221) and the output head (Qw35MetalRuntime+Output.m).
// The B200 design differs where the hardware does: weights are uploaded once
// to HBM in a coalescing-friendly layout, every step is one CUDA graph
// replay, sequences of a ragged batch share each weight read, and the KV
// cache is a pool of 256-position chunks addressed through a chunk table.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <map>
#include <stdexcept>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/qw35_cuda.h"
#include "ops.h"

namespace qw35 {

struct DevTensor {
    uint32_t type_id = 0;
    uint32_t rows = 0, k = 0;   // rows = dims[1] (or 1), k = dims[0]
    void *ptr = nullptr;        // device layout
    uint64_t bytes = 0;
};

struct ProjPart {  // one matvec of a (possibly concatenated) projection
    DevTensor w;
    uint32_t out_off = 0;       // float offset in the projection output row
};

struct LayerW {
    bool attn = false;
    const float *attn_norm = nullptr, *post_norm = nullptr;
    std::vector<ProjPart> proj;     // delta: qkv|z|beta|alpha ; attn: q|k|v (one part per run of one type)
    uint32_t proj_rows = 0;
    DevTensor out;                  // ssm_out / attn_output
    DevTensor gate, up, down;
    // delta
    const float *conv_w = nullptr, *dt = nullptr, *a = nullptr, *ssm_norm = nullptr;
    // attention
    const float *q_norm = nullptr, *k_norm = nullptr;
    int slot = 0;                   // delta slot or attention slot
};

// Weights uploaded once per (device, model mapping); shared by every runtime
// created over the same mapping (reference: Qw35MetalRuntime.m:42-80).
struct ModelStore {
    int device = 0;
    qw35_metal_hparams hp{};
    uint32_t vocab = 0;
    std::vector<LayerW> layers;
    DevTensor tok_embd, output;
    const float *output_norm = nullptr;
    std::vector<void *> allocations;
    uint64_t bytes = 0;
    int n_delta = 0, n_attn = 0;
    bool mixed = false;  // some projection has parts of different types, or gate/up types differ
    ~ModelStore();
};

struct StepKey {
    int n, mode, maxlen;
    int prefill = 0;  // 1: the n rows are consecutive positions of one sequence
    bool operator<(const StepKey &o) const {
        if (n != o.n) return n < o.n;
        if (mode != o.mode) return mode < o.mode;
        if (maxlen != o.maxlen) return maxlen < o.maxlen;
        return prefill < o.prefill;
    }
};

struct Runtime {
    int device = 0;
    std::shared_ptr<ModelStore> model;
    qw35_metal_hparams hp{};
    uint32_t ctx = 0, vocab = 0, prefill_chunk = 1;
    uint32_t max_seqs = 1;
    uint32_t rows = 1;             // rows of the step buffers: max_seqs, or a longer prefill run
    bool batched_prefill = false;  // eval_tokens runs a token run as one batched pass (default; QW35_PREFILL=0 off)
    bool prefill_dn_run = false;   // ... with one DeltaNet launch per layer for the whole run (default; QW35_PREFILL=1 off)
    int attn_window = 0, attn_sink = 0;
    cudaStream_t stream = nullptr;
    std::string deferred_error;

    // recurrent state [slot][n_delta][...]
    float *conv_state = nullptr, *ssm_state = nullptr;
    size_t conv_per_layer = 0, ssm_per_layer = 0;  // floats
    std::vector<bool> slot_used;

    // KV chunk pool
    size_t chunk_bytes = 0, plane_bytes = 0;
    int kv_q8 = 0;                               // kv_cache_type 1: q8_0 planes
    uint32_t max_chunks = 0;                     // per sequence (ctx ceiling / 256)
    uint32_t table_chunks = 0;                   // columns of the device chunk table
    std::vector<void *> arenas;
    std::vector<uint64_t> free_chunks;
    std::vector<std::vector<uint64_t>> seq_chunks;
    uint64_t *d_chunk_table = nullptr;           // [max_seqs][table_chunks]
    std::vector<uint64_t> h_chunk_table;
    uint64_t kv_bytes = 0;

    // step buffers
    struct StepIn { int32_t slot, pos, len; uint32_t token; };
    StepIn *h_in = nullptr;                       // pinned
    int32_t *d_slot = nullptr, *d_pos = nullptr, *d_len = nullptr;
    uint32_t *d_tok = nullptr;
    int32_t *d_in = nullptr;                      // packed [4][max_seqs]
    int32_t *h_pack = nullptr;                    // pinned packed inputs
    cudaEvent_t in_done = nullptr;
    float *act = nullptr, *proj = nullptr, *core = nullptr, *hbuf = nullptr, *qbuf = nullptr, *gbuf = nullptr;
    float *logits = nullptr;
    float *mixed_tmp = nullptr;  // [max_seqs][max(proj_stride, ffn)], only for mixed-type models
    uint32_t *d_argmax_tok = nullptr;
    float *d_argmax_val = nullptr;
    uint32_t *h_argmax_tok = nullptr;
    float *h_argmax_val = nullptr;
    void *argmax_ws = nullptr;
    size_t argmax_ws_bytes = 0;
    void *attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    void *dq_scratch = nullptr;     // tensor-core matvec scratch, owned for the runtime's lifetime
    size_t dq_scratch_bytes = 0;    // (its graphs hold this address; it never moves)
    float *rope_freq = nullptr;
    uint32_t proj_stride = 0;

    std::map<StepKey, cudaGraphExec_t> graphs;
    std::map<StepKey, uint32_t> graph_kernels;
    uint32_t last_kernels = 0;
    int last_n = 0, last_mode = 0;
    bool use_graphs = true;

    ~Runtime();
};

struct RtError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void ck(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        char buf[256];
        snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
        throw RtError(buf);
    }
}

[[noreturn]] inline void fail(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    throw RtError(buf);
}

std::shared_ptr<ModelStore> load_model(const void *map, uint64_t map_size, const qw35_metal_tensor_desc *descs,
                                       uintptr_t n, const qw35_metal_hparams &hp, uint32_t vocab);
std::shared_ptr<ModelStore> shared_model(const void *map, uint64_t map_size, const qw35_metal_tensor_desc *descs,
                                         uintptr_t n, const qw35_metal_hparams &hp, uint32_t vocab);
Runtime *create_runtime(std::shared_ptr<ModelStore> ms, const qw35_metal_hparams &hp, uint32_t ctx, uint32_t vocab,
                        uint32_t prefill_chunk, uint32_t max_seqs, uint32_t kv_type = 0);
void rt_enqueue_step(Runtime *rt, uint32_t n, const uint32_t *seq_ids, const uint32_t *tokens,
                     const uint32_t *pos, int mode);
// tokens[0..len) of one sequence at positions pos0.. as one pass (len <= rt->rows);
// the head runs on the last token only
void rt_enqueue_prefill(Runtime *rt, uint32_t seq, const uint32_t *tokens, uint32_t len, uint32_t pos0, int mode);
void rt_wait(Runtime *rt);
void rt_release_kv(Runtime *rt, uint32_t slot, size_t keep);
void rt_ensure_kv(Runtime *rt, uint32_t slot, uint64_t positions);
void rt_reset_slot(Runtime *rt, uint32_t slot);
void rt_set_ctx(Runtime *rt, uint32_t ctx);
void rt_fork(Runtime *rt, uint32_t src, uint32_t dst);
// KV rows [0, positions) of every attention layer of `slot` filled with
// deterministic pseudo-random values (benchmark contexts without a prefill)
void rt_fill_synthetic(Runtime *rt, uint32_t slot, uint32_t positions, uint64_t seed);
uint64_t rt_state_size(const Runtime *rt);
void rt_state_export(Runtime *rt, uint32_t slot, uint8_t *buf, uint64_t len);
void rt_state_import(Runtime *rt, uint32_t slot, const uint8_t *buf, uint64_t len);

}  // namespace qw35
