// model_internal.h -- the RbtModel context shared by model.cu (one-token forward)
// and model_prefill.cu (the batched prompt); not part of the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "../../include/rbt_moe.h"

namespace rbt {

struct Step {
    int token, pos;
};

// Row buffers of the batched prompt, for `cap` tokens.
struct PrefillBufs {
    int cap = 0;
    int32_t* tokens = nullptr;  // [cap]
    float* x = nullptr;         // [cap, dim] residual rows
    float* qkv = nullptr;       // [cap, nq + 2 nkv]
    float* ao = nullptr;        // [cap, nq] attention output
    float* xf = nullptr;        // [cap, max(dim, nq)] f32 GEMM input rows (f32 models)
    void* hi = nullptr;         // [cap, max(dim, nq)] bf16 GEMM input rows, x = hi + lo (bf16 models)
    void* lo = nullptr;
    int32_t* routing = nullptr; // [cap, n_layers, top_k]
    int logit_rows = 0;
    float* logits = nullptr;    // [logit_rows, vocab]
    size_t att_bytes = 0;       // tensor-core attention scratch (bf16 models): scores, P, q|k|v splits
    void* att = nullptr;
};

}  // namespace rbt

struct RbtModel;
namespace rbt {
void prefill_free(RbtModel* m);  // model_prefill.cu: the batched prompt's buffers
cudaError_t launch_attn_decode_rows(const RbtModel* m, int layer, const Step* steps, const float* qkv, int n,
                                    float* ao, float* part, unsigned* done, cudaStream_t s);
// The MoE block of layer l on T rows of x (device) on stream s: on this GPU, or
// through the expert-parallel group once the model's MoE context is connected.
int model_moe_block(RbtModel* m, int l, float* x, int T, int32_t* routing, int routing_stride, cudaStream_t s);
// The MoE context's rows for a call of T rows (the expert-parallel group's
// every-rank total when connected), for rbt_moe_reserve.
int model_moe_rows(RbtModel* m, int T);
// 0 if T rows fit one call of the model's MoE context, else fails with the message
int model_moe_fits(RbtModel* m, int T);
void model_drop_graphs(RbtModel* m);
}  // namespace rbt

struct RbtModel {
    RbtModelConfig cfg{};
    int ctx = 0, device = 0, sm_count = 0;
    RbtMoe* moe = nullptr;
    cudaStream_t stream = nullptr;
    size_t esz = 0;
    // weights
    void* tok_emb = nullptr;
    void* lm_head = nullptr;
    float* final_norm = nullptr;
    struct Layer {
        float* attn_norm = nullptr;
        float* q_norm = nullptr;
        float* k_norm = nullptr;
        void* wqkv = nullptr;  // [wq; wk; wv] rows, contiguous
        void* wo = nullptr;
        bool loaded = false;
    };
    std::vector<Layer> layers;
    bool globals = false;
    // state
    float *x = nullptr, *qkv = nullptr, *part = nullptr, *ao = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    int n_seq = 1;  // KV caches: n_seq sequences, [n_seq][n_layers][n_kv_heads][ctx][head_dim] (sequence 0 first)
    int32_t* routing = nullptr;
    unsigned* done = nullptr;
    unsigned* status = nullptr;  // attention's error word (a bounded wait that ran out)
    rbt::Step* step = nullptr;
    // pinned host staging
    rbt::Step* h_step = nullptr;
    float* h_logits = nullptr;
    int32_t* h_routing = nullptr;
    unsigned* h_status = nullptr;
    // batched prompt (model_prefill.cu): row buffers, grown on demand
    rbt::PrefillBufs pf;
    float* proj_part = nullptr;  // split-K partial sums of the small-batch projections
    size_t proj_part_bytes = 0;
    // batched decode (rbt_model_decode_batch), one token per sequence, for dcap rows
    int dcap = 0;
    rbt::Step* steps = nullptr;    // [dcap] (token, position) of each row
    float* dpart = nullptr;        // [dcap][n_heads][n_splits][head_dim + 2] attention split partials
    unsigned* ddone = nullptr;     // [dcap][n_heads] finished splits, zero between calls
    int32_t* dnext = nullptr;      // [dcap] greedy ids
    rbt::Step* h_steps = nullptr;  // [dcap] pinned staging of the steps
    // graphs: [0] without lm_head, [1] with
    cudaGraphExec_t graph[2] = {nullptr, nullptr};
    unsigned long long graph_gen = 0;  // the MoE workspace generation the graphs were captured with
    int n_splits = 0;
};
