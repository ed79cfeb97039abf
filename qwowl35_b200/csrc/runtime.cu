// runtime.cu -- model upload, slots, KV chunk pool and decode orchestration.
// (Extern "C" wrappers live in ffi_runtime.cu.)
#include <algorithm>
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

#include "common.cuh"
#include "runtime.h"

namespace qw35 {

// ---------------------------------------------------------------------------
// model upload
// ---------------------------------------------------------------------------
ModelStore::~ModelStore() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    for (void *p : allocations) cudaFree(p);
    cudaSetDevice(prev);
}

namespace {

struct HostTensor {
    const qw35_metal_tensor_desc *d = nullptr;
    const uint8_t *data = nullptr;
};

struct Loader {
    const uint8_t *map;
    uint64_t map_size;
    std::map<std::string, HostTensor> byname;
    ModelStore &ms;
    void *staging = nullptr;
    size_t staging_bytes = 0;

    Loader(const void *m, uint64_t size, const qw35_metal_tensor_desc *descs, uintptr_t n, ModelStore &s)
        : map(static_cast<const uint8_t *>(m)), map_size(size), ms(s) {
        for (uintptr_t i = 0; i < n; ++i) {
            const auto &d = descs[i];
            if (!d.name) fail("tensor %zu has no name", (size_t)i);
            if (d.abs_offset > map_size || d.bytes > map_size - d.abs_offset)
                fail("tensor %.*s lies outside the model mapping", (int)d.name_len, (const char *)d.name);
            byname[std::string((const char *)d.name, d.name_len)] = HostTensor{&d, map + d.abs_offset};
        }
    }
    ~Loader() {
        if (staging) cudaFree(staging);
    }

    const HostTensor &get(const std::string &name) {
        auto it = byname.find(name);
        if (it == byname.end()) fail("missing tensor %s", name.c_str());
        return it->second;
    }

    void *dalloc(size_t bytes) {
        void *p = nullptr;
        ck(cudaMalloc(&p, bytes < 256 ? 256 : bytes), "cudaMalloc(weights)");
        ms.allocations.push_back(p);
        ms.bytes += bytes;
        return p;
    }
    void *stage(size_t bytes) {
        if (bytes > staging_bytes) {
            if (staging) cudaFree(staging);
            staging = nullptr;
            ck(cudaMalloc(&staging, bytes), "cudaMalloc(staging)");
            staging_bytes = bytes;
        }
        return staging;
    }

    static uint64_t tbytes(uint32_t type, uint64_t rows, uint64_t k) {
        return qw35_cuda_weight_bytes(type, (uint32_t)rows, (uint32_t)k);
    }

    // f32 vector/matrix of exactly `elems` elements
    const float *f32(const std::string &name, uint64_t elems) {
        const HostTensor &t = get(name);
        if (t.d->type_id != QW35_F32_TYPE) fail("%s must be f32 (type %u)", name.c_str(), t.d->type_id);
        if (t.d->elements != elems || t.d->bytes != elems * 4)
            fail("%s has %llu elements, expected %llu", name.c_str(), (unsigned long long)t.d->elements,
                 (unsigned long long)elems);
        void *p = dalloc(elems * 4);
        ck(cudaMemcpy(p, t.data, elems * 4, cudaMemcpyHostToDevice), "upload");
        return static_cast<const float *>(p);
    }

    // quantised matrices concatenated by rows (same type and K), repacked
    DevTensor matrix_cat(const std::vector<std::string> &names, uint64_t k_expect) {
        uint32_t type = 0;
        uint64_t rows = 0, k = 0;
        for (size_t i = 0; i < names.size(); ++i) {
            const HostTensor &t = get(names[i]);
            const uint64_t tk = t.d->dims[0], tr = t.d->n_dims >= 2 ? t.d->dims[1] : 1;
            if (i == 0) { type = t.d->type_id; k = tk; }
            if (t.d->type_id != type || tk != k) fail("%s: mixed type/K in a fused projection", names[i].c_str());
            if (t.d->type_id != QW35_GF4_TYPE && t.d->type_id != QW35_Q8_0_TYPE && t.d->type_id != QW35_Q4_K_TYPE &&
                t.d->type_id != QW35_Q5_K_TYPE && t.d->type_id != QW35_Q6_K_TYPE)
                fail("%s: unsupported weight type %u", names[i].c_str(), t.d->type_id);
            if (t.d->bytes != tbytes(type, tr, tk)) fail("%s: byte size does not match its type", names[i].c_str());
            rows += tr;
        }
        if (k != k_expect || k % 256) fail("%s: K=%llu, expected %llu", names[0].c_str(), (unsigned long long)k,
                                           (unsigned long long)k_expect);
        const uint64_t bytes = tbytes(type, rows, k);
        uint8_t *st = static_cast<uint8_t *>(stage(bytes));
        uint64_t off = 0;
        for (const auto &n : names) {  // GGUF row concatenation == byte concatenation
            const HostTensor &t = get(n);
            ck(cudaMemcpy(st + off, t.data, t.d->bytes, cudaMemcpyHostToDevice), "upload");
            off += t.d->bytes;
        }
        DevTensor dt;
        dt.type_id = type; dt.rows = (uint32_t)rows; dt.k = (uint32_t)k;
        dt.bytes = qw35_cuda_device_bytes(type, dt.rows, dt.k);
        dt.ptr = dalloc(dt.bytes);
        ck(weight_repack(type, st, dt.ptr, dt.rows, dt.k, 0), "repack");
        ck(cudaDeviceSynchronize(), "repack sync");
        return dt;
    }
    // A fused projection as runs of consecutive same-type tensors, each run
    // concatenated into one matrix (the reference's GGUFs mix types inside
    // a projection group, e.g. a Q6_K attn_v beside Q4_K attn_q / attn_k).
    std::vector<ProjPart> matrix_parts(const std::vector<std::string> &names, uint64_t k_expect) {
        std::vector<ProjPart> parts;
        uint32_t off = 0;
        for (size_t i = 0; i < names.size();) {
            size_t j = i + 1;
            while (j < names.size() && get(names[j]).d->type_id == get(names[i]).d->type_id) ++j;
            ProjPart pp;
            pp.w = matrix_cat(std::vector<std::string>(names.begin() + i, names.begin() + j), k_expect);
            pp.out_off = off;
            off += pp.w.rows;
            parts.push_back(pp);
            i = j;
        }
        return parts;
    }
    DevTensor matrix(const std::string &name, uint64_t k, uint64_t rows_expect) {
        DevTensor t = matrix_cat({name}, k);
        if (rows_expect && t.rows != rows_expect)
            fail("%s has %u rows, expected %llu", name.c_str(), t.rows, (unsigned long long)rows_expect);
        return t;
    }
};

void check_hparams(const qw35_metal_hparams &h) {
    if (h.embedding_length != 4096 || h.attention_heads != 16 || h.attention_kv_heads != 4 ||
        h.attention_key_length != 256 || h.attention_value_length != 256 || h.rope_dimension_count != 64 ||
        h.ssm_conv_kernel != 4 || h.ssm_state_size != 128 || h.ssm_group_count != 16 ||
        h.ssm_time_step_rank != 32 || h.ssm_inner_size != 4096)
        fail("unsupported hyper-parameters: the CUDA kernels are specialised for the Qwen3.5-9B geometry "
             "(emb 4096, 16/4 heads of 256, rope 64, ssm 4/128/16/32/4096)");
    if (h.attn_gate != 1) fail("ungated attention (attn_gate=0) is not supported by the CUDA runtime");
    if (h.n_cls_out != 0) fail("classification heads (n_cls_out) are not supported by the CUDA runtime");
    if (h.transformer_layers == 0 || h.transformer_layers > 256) fail("invalid layer count");
    if (h.feed_forward_length == 0 || h.feed_forward_length % 256) fail("feed_forward_length must be a multiple of 256");
}

}  // namespace

std::shared_ptr<ModelStore> load_model(const void *map, uint64_t map_size, const qw35_metal_tensor_desc *descs,
                                       uintptr_t n, const qw35_metal_hparams &hp, uint32_t vocab) {
    check_hparams(hp);
    auto ms = std::make_shared<ModelStore>();
    ck(cudaGetDevice(&ms->device), "cudaGetDevice");
    ms->hp = hp;
    ms->vocab = vocab;
    Loader L(map, map_size, descs, n, *ms);
    const uint64_t H = hp.embedding_length, F = hp.feed_forward_length;
    const uint32_t interval = hp.full_attention_interval ? hp.full_attention_interval : 4;

    ms->tok_embd = L.matrix("token_embd.weight", H, vocab);
    if (ms->tok_embd.type_id == QW35_GF4_TYPE) fail("token_embd.weight must be a block (q8_0 / q4_k / q5_k / q6_k) type");
    ms->output = L.matrix("output.weight", H, vocab);
    ms->output_norm = L.f32("output_norm.weight", H);

    for (uint32_t il = 0; il < hp.transformer_layers; ++il) {
        const std::string p = "blk." + std::to_string(il) + ".";
        LayerW lw;
        lw.attn = ((il + 1) % interval) == 0;
        lw.attn_norm = L.f32(p + "attn_norm.weight", H);
        lw.post_norm = L.f32(p + "post_attention_norm.weight", H);
        if (lw.attn) {
            lw.slot = ms->n_attn++;
            lw.proj = L.matrix_parts({p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"}, H);
            lw.proj_rows = lw.proj.back().out_off + lw.proj.back().w.rows;
            if (lw.proj_rows != 16 * 512 + 1024 + 1024)
                fail("%sattn_q/k/v have %u rows, expected 10240", p.c_str(), lw.proj_rows);
            lw.q_norm = L.f32(p + "attn_q_norm.weight", 256);
            lw.k_norm = L.f32(p + "attn_k_norm.weight", 256);
            lw.out = L.matrix(p + "attn_output.weight", 4096, H);
        } else {
            lw.slot = ms->n_delta++;
            lw.proj = L.matrix_parts({p + "attn_qkv.weight", p + "attn_gate.weight", p + "ssm_beta.weight",
                                      p + "ssm_alpha.weight"}, H);
            lw.proj_rows = lw.proj.back().out_off + lw.proj.back().w.rows;
            if (lw.proj_rows != 8192 + 4096 + 32 + 32)
                fail("%sdelta projections have %u rows, expected 12352", p.c_str(), lw.proj_rows);
            lw.conv_w = L.f32(p + "ssm_conv1d.weight", 8192ull * 4);
            lw.dt = L.f32(p + "ssm_dt.bias", 32);
            lw.a = L.f32(p + "ssm_a", 32);
            lw.ssm_norm = L.f32(p + "ssm_norm.weight", 128);
            lw.out = L.matrix(p + "ssm_out.weight", 4096, H);
        }
        lw.gate = L.matrix(p + "ffn_gate.weight", H, F);
        lw.up = L.matrix(p + "ffn_up.weight", H, F);
        lw.down = L.matrix(p + "ffn_down.weight", F, H);
        if (lw.proj.size() > 1 || lw.gate.type_id != lw.up.type_id) ms->mixed = true;
        ms->layers.push_back(lw);
    }
    return ms;
}

}  // namespace qw35
