// runtime_step.cu -- runtime creation, KV chunk pool, decode-step encoding
// and CUDA-graph replay.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "runtime.h"

namespace qw35 {

constexpr uint32_t kChunk = QW35_KV_CHUNK;
constexpr uint32_t kMaxCtx = 64u * 4096u;   // addressable ceiling, as the reference (Qw35MetalRuntime.m:168-178)
constexpr uint32_t kArenaChunks = 16;
constexpr uint32_t kDeltaProj = 8192 + 4096 + 32 + 32;
constexpr uint32_t kAttnProj = 16 * 512 + 1024 + 1024;

// ---------------------------------------------------------------------------
// shared weights per (device, mapping)
// ---------------------------------------------------------------------------
std::shared_ptr<ModelStore> shared_model(const void *map, uint64_t map_size, const qw35_metal_tensor_desc *descs,
                                         uintptr_t n, const qw35_metal_hparams &hp, uint32_t vocab) {
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, std::weak_ptr<ModelStore>> cache;
    int dev = 0;
    ck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> g(mu);
    auto key = std::make_pair(dev, map);
    auto it = cache.find(key);
    if (it != cache.end()) {
        if (auto sp = it->second.lock()) {
            if (sp->vocab != vocab || memcmp(&sp->hp, &hp, offsetof(qw35_metal_hparams, attn_window)) != 0)
                fail("a runtime over this model mapping already exists with different hyper-parameters");
            return sp;
        }
    }
    auto sp = load_model(map, map_size, descs, n, hp, vocab);
    cache[key] = sp;
    return sp;
}

// ---------------------------------------------------------------------------
// lifetime
// ---------------------------------------------------------------------------
Runtime::~Runtime() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    for (auto &kv : graphs) cudaGraphExecDestroy(kv.second);
    void *dev_ptrs[] = {conv_state, ssm_state, d_chunk_table, d_in, act, proj, core, hbuf, qbuf, gbuf,
                        logits, d_argmax_tok, d_argmax_val, argmax_ws, attn_ws, rope_freq, mixed_tmp,
                        dq_scratch};
    for (void *p : dev_ptrs)
        if (p) cudaFree(p);
    for (void *p : arenas) cudaFree(p);
    if (h_pack) cudaFreeHost(h_pack);
    if (h_argmax_tok) cudaFreeHost(h_argmax_tok);
    if (h_argmax_val) cudaFreeHost(h_argmax_val);
    if (in_done) cudaEventDestroy(in_done);
    if (stream) cudaStreamDestroy(stream);
    model.reset();
    cudaSetDevice(prev);
}

template <typename T>
static T *dmalloc(size_t count) {
    void *p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 256)), "cudaMalloc(runtime)");
    return static_cast<T *>(p);
}

Runtime *create_runtime(std::shared_ptr<ModelStore> ms, const qw35_metal_hparams &hp, uint32_t ctx, uint32_t vocab,
                        uint32_t prefill_chunk, uint32_t max_seqs, uint32_t kv_type) {
    if (ctx == 0) fail("ctx must be positive");
    if (ctx > kMaxCtx) fail("--ctx %u exceeds the maximum %u tokens the KV cache can address", ctx, kMaxCtx);
    if (max_seqs == 0 || max_seqs > 1024) fail("max_seqs must be in [1, 1024]");
    std::unique_ptr<Runtime> rt(new Runtime());
    rt->device = ms->device;
    rt->model = ms;
    // this runtime's own hyper-parameters: the weights may be shared with runtimes
    // created with another attention window / sink (the rest must match, see
    // shared_model)
    rt->hp = hp;
    rt->ctx = ctx;
    rt->vocab = vocab;
    rt->prefill_chunk = prefill_chunk ? prefill_chunk : 1;
    rt->max_seqs = max_seqs;
    rt->attn_window = hp.attn_window;
    rt->attn_sink = hp.attn_sink < 0 ? 0 : hp.attn_sink;
    rt->use_graphs = getenv("QW35_NO_GRAPH") == nullptr;
    ck(cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    ck(cudaEventCreateWithFlags(&rt->in_done, cudaEventDisableTiming), "cudaEventCreate");

    const uint32_t S = max_seqs, H = 4096, F = ms->hp.feed_forward_length;
    rt->conv_per_layer = 8192ull * 3;
    rt->ssm_per_layer = 32ull * 128 * 128;
    const size_t nd = (size_t)std::max(ms->n_delta, 1);
    rt->conv_state = dmalloc<float>(S * nd * rt->conv_per_layer);
    rt->ssm_state = dmalloc<float>(S * nd * rt->ssm_per_layer);
    ck(cudaMemset(rt->conv_state, 0, S * nd * rt->conv_per_layer * 4), "memset");
    ck(cudaMemset(rt->ssm_state, 0, S * nd * rt->ssm_per_layer * 4), "memset");
    rt->slot_used.assign(S, false);
    rt->slot_used[0] = true;  // slot 0 backs the single-sequence qw35_metal_* surface

    // one attention layer's K (or V) plane of a chunk: [4 kv heads][256 pos][256 dims]
    // f16, or q8_0 rows of kKvQ8Row bytes (reference bridge.rs:31-42, kv_cache_type)
    rt->kv_q8 = kv_type == 1 ? 1 : 0;
    rt->plane_bytes = rt->kv_q8 ? 4ull * kChunk * kKvQ8Row : 4ull * kChunk * 256 * 2;
    rt->chunk_bytes = (size_t)ms->n_attn * 2 * rt->plane_bytes;
    rt->table_chunks = kMaxCtx / kChunk;
    rt->seq_chunks.assign(S, {});
    rt->h_chunk_table.assign((size_t)S * rt->table_chunks, 0);
    rt->d_chunk_table = dmalloc<uint64_t>((size_t)S * rt->table_chunks);
    ck(cudaMemset(rt->d_chunk_table, 0, (size_t)S * rt->table_chunks * 8), "memset");

    // step buffers hold max_seqs rows, or a batched prefill run (<= 64 tokens) when longer
    // eval_tokens runs a token run as one batched pass, its DeltaNet recurrence
    // as one run kernel per layer; QW35_PREFILL=1 keeps the batched pass with
    // per-token DeltaNet steps, QW35_PREFILL=0 runs consecutive decode steps
    {
        const char *pf = getenv("QW35_PREFILL");
        rt->batched_prefill = !(pf && strcmp(pf, "0") == 0);
        rt->prefill_dn_run = rt->batched_prefill && !(pf && strcmp(pf, "1") == 0);
    }
    const uint32_t R = rt->batched_prefill ? std::max<uint32_t>(S, std::min<uint32_t>(rt->prefill_chunk, 64)) : S;
    rt->rows = R;
    rt->d_in = dmalloc<int32_t>(4ull * R);
    rt->d_slot = rt->d_in;
    rt->d_pos = rt->d_in + R;
    rt->d_len = rt->d_in + 2 * R;
    rt->d_tok = reinterpret_cast<uint32_t *>(rt->d_in + 3 * R);
    ck(cudaMallocHost(reinterpret_cast<void **>(&rt->h_pack), 16ull * R), "cudaMallocHost");
    ck(cudaMallocHost(reinterpret_cast<void **>(&rt->h_argmax_tok), 4ull * S), "cudaMallocHost");
    ck(cudaMallocHost(reinterpret_cast<void **>(&rt->h_argmax_val), 4ull * S), "cudaMallocHost");

    rt->proj_stride = std::max(kDeltaProj, kAttnProj);
    rt->act = dmalloc<float>((size_t)R * H);
    rt->proj = dmalloc<float>((size_t)R * rt->proj_stride);
    rt->core = dmalloc<float>((size_t)R * H);
    rt->hbuf = dmalloc<float>((size_t)R * F);
    rt->qbuf = dmalloc<float>((size_t)R * H);
    rt->gbuf = dmalloc<float>((size_t)R * H);
    rt->logits = dmalloc<float>((size_t)S * vocab);
    if (rt->model->mixed) rt->mixed_tmp = dmalloc<float>((size_t)R * std::max<uint32_t>(rt->proj_stride, F));
    rt->d_argmax_tok = dmalloc<uint32_t>(S);
    rt->d_argmax_val = dmalloc<float>(S);
    rt->argmax_ws_bytes = argmax_workspace_bytes(vocab, S);
    rt->argmax_ws = dmalloc<uint8_t>(rt->argmax_ws_bytes);
    rt->attn_ws_bytes = attn_workspace_bytes((int)R, (int)kMaxCtx);
    rt->attn_ws = dmalloc<uint8_t>(rt->attn_ws_bytes);

    // scratch of the batched tensor-core matvec, owned by this runtime: its
    // graphs capture the address, so it is sized here for the largest matvec
    // a step can run and freed only with the runtime (a prefill run of R rows
    // runs the head on its last row only)
    {
        const uint32_t kmax = std::max<uint32_t>(H, F);
        size_t need = 0;
        if (R >= (uint32_t)kDqMinBatch) need = std::max(need, dq_scratch_bytes((int)std::min<uint32_t>(R, 64), kmax, std::max(F, rt->proj_stride)));
        if (S >= (uint32_t)kDqMinBatch)
            need = std::max(need, dq_scratch_bytes((int)std::min<uint32_t>(S, 64), kmax, std::max({vocab, F, rt->proj_stride})));
        if (need) {
            rt->dq_scratch = dmalloc<uint8_t>(need);
            rt->dq_scratch_bytes = need;
        }
    }

    // RoPE ladder freq[i] = base^(-2i/n_rot) in fp32 (Qw35MetalRuntime.m:772-795)
    float freq[32];
    for (uint32_t i = 0; i < 32; ++i) freq[i] = powf(ms->hp.rope_freq_base, -((float)(i * 2u)) / 64.0f);
    rt->rope_freq = dmalloc<float>(32);
    ck(cudaMemcpy(rt->rope_freq, freq, sizeof(freq), cudaMemcpyHostToDevice), "upload rope");

    // slot 0 starts with one chunk, as the reference starts with one slab
    if (ms->n_attn > 0) {
        rt_ensure_kv(rt.get(), 0, 1);
    }
    ck(cudaDeviceSynchronize(), "runtime init");
    return rt.release();
}

// ---------------------------------------------------------------------------
// KV chunk pool: append-only per sequence, no copies, no moves
// (reference: ensureKvCapacityForPositions, Qw35MetalRuntime.m:496-538)
// ---------------------------------------------------------------------------
void rt_ensure_kv(Runtime *rt, uint32_t slot, uint64_t positions) {
    if (rt->model->n_attn == 0) return;
    const uint64_t need = (positions + kChunk - 1) / kChunk;
    auto &chunks = rt->seq_chunks[slot];
    while (chunks.size() < need) {
        if (rt->free_chunks.empty()) {
            void *arena = nullptr;
            ck(cudaMalloc(&arena, rt->chunk_bytes * kArenaChunks), "failed to grow the KV cache");
            rt->arenas.push_back(arena);
            rt->kv_bytes += rt->chunk_bytes * kArenaChunks;
            for (uint32_t i = kArenaChunks; i-- > 0;)
                rt->free_chunks.push_back(reinterpret_cast<uint64_t>(arena) + i * rt->chunk_bytes);
        }
        const uint64_t c = rt->free_chunks.back();
        rt->free_chunks.pop_back();
        const size_t idx = (size_t)slot * rt->table_chunks + chunks.size();
        chunks.push_back(c);
        rt->h_chunk_table[idx] = c;
        // pageable source: the copy is staged before the call returns, ordered on the stream
        ck(cudaMemcpyAsync(rt->d_chunk_table + idx, &rt->h_chunk_table[idx], 8, cudaMemcpyHostToDevice, rt->stream),
           "chunk table update");
    }
}

void rt_release_kv(Runtime *rt, uint32_t slot, size_t keep) {
    auto &chunks = rt->seq_chunks[slot];
    while (chunks.size() > keep) {
        rt->free_chunks.push_back(chunks.back());
        rt->h_chunk_table[(size_t)slot * rt->table_chunks + chunks.size() - 1] = 0;
        chunks.pop_back();
    }
}

void rt_wait(Runtime *rt) {
    cudaError_t e = cudaStreamSynchronize(rt->stream);
    if (e != cudaSuccess) fail("CUDA decode step failed: %s", cudaGetErrorString(e));
    if (const unsigned code = device_error_read_and_clear())
        fail("a device pipeline wait timed out (code %u); results of the last step are invalid", code);
}

void rt_reset_slot(Runtime *rt, uint32_t slot) {
    rt_wait(rt);
    const size_t nd = (size_t)std::max(rt->model->n_delta, 1);
    ck(cudaMemsetAsync(rt->conv_state + slot * nd * rt->conv_per_layer, 0, nd * rt->conv_per_layer * 4, rt->stream),
       "reset");
    ck(cudaMemsetAsync(rt->ssm_state + slot * nd * rt->ssm_per_layer, 0, nd * rt->ssm_per_layer * 4, rt->stream),
       "reset");
    rt_release_kv(rt, slot, rt->model->n_attn > 0 ? 1 : 0);
    if (rt->model->n_attn > 0 && rt->seq_chunks[slot].empty()) rt_ensure_kv(rt, slot, 1);
    rt_wait(rt);
}

// Copy sequence `src` (recurrent state and every KV chunk it holds) into `dst`,
// so both continue from the same prefix (session fork / shared prompt).
void rt_fork(Runtime *rt, uint32_t src, uint32_t dst) {
    if (src == dst) fail("fork source and destination are the same sequence");
    rt_wait(rt);
    const size_t nd = (size_t)std::max(rt->model->n_delta, 1);
    ck(cudaMemcpyAsync(rt->conv_state + dst * nd * rt->conv_per_layer, rt->conv_state + src * nd * rt->conv_per_layer,
                       nd * rt->conv_per_layer * 4, cudaMemcpyDeviceToDevice, rt->stream), "fork state");
    ck(cudaMemcpyAsync(rt->ssm_state + dst * nd * rt->ssm_per_layer, rt->ssm_state + src * nd * rt->ssm_per_layer,
                       nd * rt->ssm_per_layer * 4, cudaMemcpyDeviceToDevice, rt->stream), "fork state");
    const size_t n = rt->seq_chunks[src].size();
    rt_release_kv(rt, dst, 0);
    rt_ensure_kv(rt, dst, (uint64_t)n * QW35_KV_CHUNK);
    for (size_t c = 0; c < n; ++c)
        ck(cudaMemcpyAsync(reinterpret_cast<void *>(rt->seq_chunks[dst][c]),
                           reinterpret_cast<const void *>(rt->seq_chunks[src][c]), rt->chunk_bytes,
                           cudaMemcpyDeviceToDevice, rt->stream), "fork kv");
    rt_wait(rt);
}

// Pseudo-random KV contents: f16 planes get values uniform in [-2, 2) from a
// hash of (seed, chunk, element); q8_0 planes get blocks {d = 2/127 as f16,
// codes uniform in [-127, 127]}.  One CTA per (chunk, slice of the chunk).
__device__ __forceinline__ uint32_t fill_hash(uint64_t a) {
    a ^= a >> 33;
    a *= 0xff51afd7ed558ccdull;
    a ^= a >> 33;
    a *= 0xc4ceb9fe1a85ec53ull;
    a ^= a >> 33;
    return (uint32_t)a;
}

__global__ void kv_fill_kernel(const uint64_t *chunks, size_t chunk_bytes, int kv_q8, uint64_t seed) {
    uint8_t *base = reinterpret_cast<uint8_t *>(chunks[blockIdx.y]);
    const uint64_t key = seed * 0x9E3779B97F4A7C15ull + blockIdx.y;
    if (!kv_q8) {
        const size_t n = chunk_bytes / 4;  // half2 words
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
            const uint32_t h = fill_hash(key * 0x100000001B3ull + i);
            const float a = (float)(h & 0xffffu) * (4.0f / 65536.0f) - 2.0f;
            const float b = (float)(h >> 16) * (4.0f / 65536.0f) - 2.0f;
            reinterpret_cast<__half2 *>(base)[i] = __floats2half2_rn(a, b);
        }
    } else {
        const size_t n = chunk_bytes / 34;  // q8_0 blocks {f16 d; int8 qs[32]}
        const __half d = __float2half_rn(2.0f / 127.0f);
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
            uint8_t *blk = base + i * 34;
            *reinterpret_cast<__half *>(blk) = d;
            for (int j = 0; j < 32; j += 4) {
                const uint32_t h = fill_hash(key * 0x100000001B3ull + i * 8 + (j >> 2));
#pragma unroll
                for (int t = 0; t < 4; ++t) blk[2 + j + t] = (uint8_t)(int8_t)((int)((h >> (8 * t)) % 255u) - 127);
            }
        }
    }
}

void rt_fill_synthetic(Runtime *rt, uint32_t slot, uint32_t positions, uint64_t seed) {
    if (rt->model->n_attn == 0 || positions == 0) return;
    rt_ensure_kv(rt, slot, positions);
    const uint32_t nch = (positions + kChunk - 1) / kChunk;
    kv_fill_kernel<<<dim3(64, nch), 256, 0, rt->stream>>>(rt->d_chunk_table + (size_t)slot * rt->table_chunks,
                                                          rt->chunk_bytes, rt->kv_q8, seed);
    ck(cudaGetLastError(), "kv fill");
    rt_wait(rt);
}

void rt_set_ctx(Runtime *rt, uint32_t ctx) {
    if (ctx <= rt->ctx) return;
    if (ctx > kMaxCtx) fail("ctx %u exceeds the maximum %u tokens the KV cache can address", ctx, kMaxCtx);
    rt->ctx = ctx;
}

uint64_t rt_state_size(const Runtime *rt) {
    const size_t nd = (size_t)std::max(rt->model->n_delta, 1);
    return (uint64_t)nd * (rt->conv_per_layer + rt->ssm_per_layer) * 4;
}

void rt_state_export(Runtime *rt, uint32_t slot, uint8_t *buf, uint64_t len) {
    rt_wait(rt);
    if (!buf || len != rt_state_size(rt)) fail("state export buffer size mismatch");
    const size_t nd = (size_t)std::max(rt->model->n_delta, 1);
    const size_t cb = nd * rt->conv_per_layer * 4;
    ck(cudaMemcpy(buf, rt->conv_state + slot * nd * rt->conv_per_layer, cb, cudaMemcpyDeviceToHost), "export");
    ck(cudaMemcpy(buf + cb, rt->ssm_state + slot * nd * rt->ssm_per_layer, nd * rt->ssm_per_layer * 4,
                  cudaMemcpyDeviceToHost), "export");
}

void rt_state_import(Runtime *rt, uint32_t slot, const uint8_t *buf, uint64_t len) {
    rt_wait(rt);
    if (!buf || len != rt_state_size(rt)) fail("state import buffer size mismatch");
    const size_t nd = (size_t)std::max(rt->model->n_delta, 1);
    const size_t cb = nd * rt->conv_per_layer * 4;
    ck(cudaMemcpy(rt->conv_state + slot * nd * rt->conv_per_layer, buf, cb, cudaMemcpyHostToDevice), "import");
    ck(cudaMemcpy(rt->ssm_state + slot * nd * rt->ssm_per_layer, buf + cb, nd * rt->ssm_per_layer * 4,
                  cudaMemcpyHostToDevice), "import");
}

}  // namespace qw35
