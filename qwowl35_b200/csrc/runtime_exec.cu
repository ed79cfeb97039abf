// runtime_exec.cu -- one decode step for a ragged batch, as kernels on the
// runtime stream, captured once per (batch size, head mode, length bucket)
// into a CUDA graph and replayed.
//
// Kernel order per step (reference: encodeDecodeLayers, Qw35MetalRuntime.m:1170-1221):
//   embed -> per layer { [norm+proj] -> mixer -> [out proj +residual] ->
//                        [norm+gate/up+SwiGLU] -> [down +residual] } -> [norm+head]
// RMS norms are fused into the prologue of the following matvec, residual
// adds into the epilogue of the preceding one, so the residual stream `act`
// is touched only by fused kernels (the reference fuses the same pairs,
// Qw35MetalRuntime.m:8-12).
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "runtime.h"

namespace qw35 {

void rt_ensure_kv(Runtime *rt, uint32_t slot, uint64_t positions);

static void mv(Runtime *rt, const DevTensor &w, const void *x, const float *norm_w, float *y, int n, int mode,
               const DevTensor *w_up = nullptr) {
    MatvecArgs a;
    a.type_id = w.type_id;
    a.w0 = w.ptr;
    a.w1 = w_up ? w_up->ptr : nullptr;
    a.x = x;
    a.x_dtype = 0;
    a.norm_w = norm_w;
    a.eps = rt->hp.rms_epsilon;
    a.y = y;
    a.rows = w.rows;
    a.k = w.k;
    a.batch = n;
    a.mode = mode;
    a.scratch = rt->dq_scratch;
    a.scratch_bytes = rt->dq_scratch_bytes;
    ck(matvec_run(a, rt->stream), "matvec");
}

// A projection of several parts (runs of one weight type): each part's
// matvec writes [n][part rows] into scratch, and one strided 2-D copy places
// it at its offset in the [n][proj_rows] projection output.
static void proj_mv(Runtime *rt, const LayerW &lw, int n) {
    if (lw.proj.size() == 1) {
        mv(rt, lw.proj[0].w, rt->act, lw.attn_norm, rt->proj, n, 0);
        return;
    }
    for (const ProjPart &pp : lw.proj) {
        mv(rt, pp.w, rt->act, lw.attn_norm, rt->mixed_tmp, n, 0);
        ck(cudaMemcpy2DAsync(rt->proj + pp.out_off, (size_t)lw.proj_rows * 4, rt->mixed_tmp, (size_t)pp.w.rows * 4,
                             (size_t)pp.w.rows * 4, (size_t)n, cudaMemcpyDeviceToDevice, rt->stream),
           "projection part copy");
    }
}

// gate/up + SwiGLU: one fused launch when both have one type, else two
// matvecs and an elementwise SwiGLU.
static void ffn_gate_up(Runtime *rt, const LayerW &lw, int n) {
    if (lw.gate.type_id == lw.up.type_id) {
        mv(rt, lw.gate, rt->act, lw.post_norm, rt->hbuf, n, 2, &lw.up);
        return;
    }
    mv(rt, lw.gate, rt->act, lw.post_norm, rt->hbuf, n, 0);
    mv(rt, lw.up, rt->act, lw.post_norm, rt->mixed_tmp, n, 0);
    ck(swiglu_run(rt->hbuf, rt->mixed_tmp, rt->hbuf, (size_t)n * lw.gate.rows, rt->stream), "swiglu");
}

// prefill: the n rows are positions pos0 .. pos0 + n - 1 of ONE sequence.
// Matvecs, attention preprocess and attention then run over all n rows at
// once (row t attends to positions <= pos0 + t, whose K/V the preprocess has
// just written); the DeltaNet recurrence runs row by row (n launches of one
// sequence, in order), and the head only on the last row.
static void encode_step(Runtime *rt, int n, int mode, int maxlen, bool prefill = false) {
    ModelStore &ms = *rt->model;
    cudaStream_t st = rt->stream;
    const float eps = rt->hp.rms_epsilon;
    ck(embed_rows(ms.tok_embd.type_id, ms.tok_embd.ptr, ms.tok_embd.rows, rt->d_tok, n, 4096, rt->act, st), "embed");
    const size_t nd = (size_t)std::max(ms.n_delta, 1);
    for (const LayerW &lw : ms.layers) {
        proj_mv(rt, lw, n);
        if (!lw.attn) {
            DeltaNetArgs d;
            d.n_seq = n;
            d.proj = rt->proj;
            d.proj_stride = (int)lw.proj_rows;
            d.conv_w = lw.conv_w;
            d.dt = lw.dt;
            d.a = lw.a;
            d.norm_w = lw.ssm_norm;
            d.conv_state = rt->conv_state + (size_t)lw.slot * rt->conv_per_layer;
            d.ssm_state = rt->ssm_state + (size_t)lw.slot * rt->ssm_per_layer;
            d.conv_stride = (long long)(nd * rt->conv_per_layer);
            d.ssm_stride = (long long)(nd * rt->ssm_per_layer);
            d.slots = rt->d_slot;
            d.out = rt->core;
            d.out_stride = 4096;
            d.eps = eps;
            if (!prefill) {
                ck(deltanet_step_run(d, st), "deltanet");
            } else if (rt->prefill_dn_run) {
                ck(deltanet_run_tokens(d, n, st), "deltanet run");  // rows in order, state on chip
            } else {
                for (int t = 0; t < n; ++t) {  // the recurrence is sequential over the run
                    DeltaNetArgs dt = d;
                    dt.n_seq = 1;
                    dt.proj = rt->proj + (size_t)t * lw.proj_rows;
                    dt.slots = rt->d_slot + t;
                    dt.out = rt->core + (size_t)t * 4096;
                    ck(deltanet_step_run(dt, st), "deltanet");
                }
            }
        } else {
            const long long k_off = (long long)lw.slot * 2 * (long long)rt->plane_bytes;
            AttnPreArgs pa;
            pa.n_seq = n;
            pa.qkv = rt->proj;
            pa.qkv_stride = (int)lw.proj_rows;
            pa.q_norm_w = lw.q_norm;
            pa.k_norm_w = lw.k_norm;
            pa.rope_freq = rt->rope_freq;
            pa.pos = rt->d_pos;
            pa.chunk_ptrs = rt->d_chunk_table;
            pa.slots = rt->d_slot;
            pa.max_chunks = (int)rt->table_chunks;
            pa.k_off = k_off;
            pa.v_off = k_off + (long long)rt->plane_bytes;
            pa.q_out = rt->qbuf;
            pa.gate_out = rt->gbuf;
            pa.eps = eps;
            pa.kv_q8 = rt->kv_q8;
            ck(attn_preprocess_run(pa, st), "attn preprocess");
            AttnArgs aa;
            aa.n_seq = n;
            aa.q = rt->qbuf;
            aa.gate = rt->gbuf;
            aa.seq_len = rt->d_len;
            aa.chunk_ptrs = rt->d_chunk_table;
            aa.slots = rt->d_slot;
            aa.max_chunks = (int)rt->table_chunks;
            aa.k_off = pa.k_off;
            aa.v_off = pa.v_off;
            aa.window = rt->attn_window;
            aa.sink = rt->attn_sink;
            aa.max_len = maxlen;
            aa.out = rt->core;
            aa.out_stride = 4096;
            aa.ws = rt->attn_ws;
            aa.ws_bytes = rt->attn_ws_bytes;
            aa.kv_q8 = rt->kv_q8;
            ck(attn_decode_run(aa, st), "attention");
        }
        mv(rt, lw.out, rt->core, nullptr, rt->act, n, 1);
        ffn_gate_up(rt, lw, n);
        mv(rt, lw.down, rt->hbuf, nullptr, rt->act, n, 1);
    }
    // head: every row, or the last row of a prefill run
    const float *hx = prefill ? rt->act + (size_t)(n - 1) * 4096 : rt->act;
    const int hn = prefill ? 1 : n;
    if (mode == QW35_LOGITS_ARGMAX) {
        MatvecArgs a;
        a.type_id = ms.output.type_id;
        a.w0 = ms.output.ptr;
        a.x = hx;
        a.norm_w = ms.output_norm;
        a.eps = eps;
        a.rows = ms.output.rows;
        a.k = ms.output.k;
        a.batch = hn;
        a.scratch = rt->dq_scratch;
        a.scratch_bytes = rt->dq_scratch_bytes;
        ck(argmax_head_run(a, rt->d_argmax_tok, rt->d_argmax_val, rt->argmax_ws, rt->argmax_ws_bytes, st),
           "argmax head");
    } else if (mode == QW35_LOGITS_FULL) {
        mv(rt, ms.output, hx, ms.output_norm, rt->logits, hn, 0);
    }
}

static int len_bucket(uint32_t maxpos_plus1, uint32_t cap) {
    uint32_t b = 1024;
    while (b < maxpos_plus1) b <<= 1;
    return (int)std::min(b, cap);
}

// inputs -> pinned staging (reused once the previous step's copy finished) -> device
template <typename SlotOf>
static void stage_inputs(Runtime *rt, uint32_t n, SlotOf slot_of, const uint32_t *tokens, const uint32_t *pos) {
    ck(cudaEventSynchronize(rt->in_done), "input staging");
    const uint32_t R = rt->rows;
    for (uint32_t i = 0; i < n; ++i) {
        rt->h_pack[i] = (int32_t)slot_of(i);
        rt->h_pack[R + i] = (int32_t)pos[i];
        rt->h_pack[2 * R + i] = (int32_t)pos[i] + 1;
        rt->h_pack[3 * R + i] = (int32_t)tokens[i];
    }
    ck(cudaMemcpyAsync(rt->d_in, rt->h_pack, 16ull * R, cudaMemcpyHostToDevice, rt->stream), "input copy");
    ck(cudaEventRecord(rt->in_done, rt->stream), "event");
}

// Encode (or replay the CUDA graph of) one step and queue the argmax readback.
static void run_step(Runtime *rt, uint32_t n, int mode, int maxlen, bool prefill) {
    if (!rt->use_graphs) {
        encode_step(rt, (int)n, mode, maxlen, prefill);
    } else {
        StepKey key{(int)n, mode, maxlen, prefill ? 1 : 0};
        auto it = rt->graphs.find(key);
        if (it == rt->graphs.end()) {
            cudaGraph_t g = nullptr;
            ck(cudaStreamBeginCapture(rt->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
            try {
                encode_step(rt, (int)n, mode, maxlen, prefill);
            } catch (...) {
                cudaStreamEndCapture(rt->stream, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            ck(cudaStreamEndCapture(rt->stream, &g), "end capture");
            size_t nn = 0;
            ck(cudaGraphGetNodes(g, nullptr, &nn), "graph nodes");
            std::vector<cudaGraphNode_t> nodes(nn);
            uint32_t nk = 0;
            if (nn) ck(cudaGraphGetNodes(g, nodes.data(), &nn), "graph nodes");
            for (auto nd : nodes) {
                cudaGraphNodeType ty;
                if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++nk;
            }
            rt->graph_kernels[key] = nk;
            cudaGraphExec_t ge = nullptr;
            cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
            cudaGraphDestroy(g);
            ck(e, "graph instantiate");
            it = rt->graphs.emplace(key, ge).first;
        }
        ck(cudaGraphLaunch(it->second, rt->stream), "graph launch");
        rt->last_kernels = rt->graph_kernels[key];
    }
    const uint32_t nout = prefill ? 1 : n;  // rows the head ran on
    if (mode == QW35_LOGITS_ARGMAX) {
        ck(cudaMemcpyAsync(rt->h_argmax_tok, rt->d_argmax_tok, 4ull * nout, cudaMemcpyDeviceToHost, rt->stream), "d2h");
        ck(cudaMemcpyAsync(rt->h_argmax_val, rt->d_argmax_val, 4ull * nout, cudaMemcpyDeviceToHost, rt->stream), "d2h");
    }
    rt->last_n = (int)nout;
    rt->last_mode = mode;
}

void rt_enqueue_step(Runtime *rt, uint32_t n, const uint32_t *seq_ids, const uint32_t *tokens, const uint32_t *pos,
                     int mode) {
    if (n == 0 || n > rt->max_seqs) fail("batch size %u outside [1, %u]", n, rt->max_seqs);
    if (mode < 0 || mode > 2) fail("invalid logits mode %d", mode);
    if (!tokens || !pos) fail("null token/position array");
    uint32_t maxp = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t s = seq_ids ? seq_ids[i] : i;
        if (s >= rt->max_seqs || !rt->slot_used[s]) fail("sequence %u is not allocated", s);
        for (uint32_t j = 0; j < i; ++j)
            if ((seq_ids ? seq_ids[j] : j) == s) fail("sequence %u appears twice in one batch", s);
        if (pos[i] >= rt->ctx) fail("requested position exceeds allocated context");
        if (tokens[i] >= rt->vocab) fail("token id is outside the Qw35 vocabulary");
        maxp = std::max(maxp, pos[i] + 1);
    }
    for (uint32_t i = 0; i < n; ++i) rt_ensure_kv(rt, seq_ids ? seq_ids[i] : i, (uint64_t)pos[i] + 1);

    stage_inputs(rt, n, [&](uint32_t i) { return seq_ids ? seq_ids[i] : i; }, tokens, pos);
    run_step(rt, n, mode, len_bucket(maxp, rt->table_chunks * QW35_KV_CHUNK), false);
}

void rt_enqueue_prefill(Runtime *rt, uint32_t seq, const uint32_t *tokens, uint32_t len, uint32_t pos0, int mode) {
    if (len == 0 || len > rt->rows) fail("prefill run of %u tokens outside [1, %u]", len, rt->rows);
    if (mode < 0 || mode > 2) fail("invalid logits mode %d", mode);
    if (!tokens) fail("null token array");
    if (seq >= rt->max_seqs || !rt->slot_used[seq]) fail("sequence %u is not allocated", seq);
    if ((uint64_t)pos0 + len > rt->ctx) fail("requested position exceeds allocated context");
    for (uint32_t i = 0; i < len; ++i)
        if (tokens[i] >= rt->vocab) fail("token id is outside the Qw35 vocabulary");
    rt_ensure_kv(rt, seq, (uint64_t)pos0 + len);
    std::vector<uint32_t> pos(len);
    for (uint32_t i = 0; i < len; ++i) pos[i] = pos0 + i;
    stage_inputs(rt, len, [&](uint32_t) { return seq; }, tokens, pos.data());
    run_step(rt, len, mode, len_bucket(pos0 + len, rt->table_chunks * QW35_KV_CHUNK), true);
}

}  // namespace qw35
