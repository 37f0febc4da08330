/*
 * rbt_moe.h -- C ABI of librbt_moe.so, the sm_100a (B200) implementation of the
 * RABBIT2 engine's MoE feed-forward.
 *
 * The reference engine (rabbit2/src/rabbit2.c) has no library boundary: the MoE
 * block is inline code in forward() (rabbit2.c:511-542) on top of the static
 * matvec() (:357-390) and get_expert() (:261-300).  These entry points are the
 * calls a maintainer puts in place of that block (rabbit2_b200/engine/
 * rbt_engine_hook.h holds the engine-side calls, patch_engine.py beside it the
 * edits).  All pointers are plain C pointers; no CUDA or torch types appear.
 *
 * Conventions, mirroring the reference's own functions:
 *   - every int-returning call returns 1 on success and 0 on error, like
 *     forward()/load_model() (rabbit2.c:199,455); the message goes to stderr
 *     and to rbt_moe_last_error();
 *   - one host thread drives a context (the reference is single-threaded);
 *   - matrices are row-major [out, in] in the model dtype (0 = f32, 1 = bf16),
 *     vectors are f32, and an expert is the .rbt2 blob w1[H,D] | w3[H,D] |
 *     w2[D,H], expert_stride bytes apart (rabbit2.c:166-193).
 */
#ifndef RBT_MOE_H
#define RBT_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RBT_MOE_DT_F32 0
#define RBT_MOE_DT_BF16 1
#define RBT_MOE_MAX_TOPK 64     /* MAX_TOPK, rabbit2.c:59 */
#define RBT_MOE_MAX_EXPERTS 256

/* The MoE part of the model config (Config, rabbit2.c:63-68) plus the expert
 * stride the loader computes (Model.expert_stride, rabbit2.c:173). */
typedef struct RbtMoeConfig {
    int32_t dim;            /* D */
    int32_t n_experts;      /* E */
    int32_t top_k;          /* K */
    int32_t expert_hidden;  /* H */
    int32_t n_layers;
    int32_t dtype;          /* RBT_MOE_DT_F32 or RBT_MOE_DT_BF16 */
    int32_t norm_topk;      /* 1: renormalise the chosen weights to sum to 1 */
    float rms_eps;
    uint64_t expert_stride; /* bytes between expert blobs */
} RbtMoeConfig;

typedef struct RbtMoe RbtMoe; /* opaque context: one per (model, GPU) */

/* Create a context on CUDA device `device`.  Replaces the expert cache set-up
 * (expert_cache_init, rabbit2.c:236-253): experts live in HBM instead. */
int rbt_moe_create(RbtMoe **out, const RbtMoeConfig *cfg, int device);
void rbt_moe_destroy(RbtMoe *m);

/* Upload one layer's MoE weights from host memory (e.g. the mmap'd .rbt2):
 * ffn_norm [D] f32 (may be NULL if only rbt_moe_ffn is used), router [E,D],
 * experts = the layer's first expert blob (E blobs, expert_stride apart).
 * Replaces get_expert() (rabbit2.c:261-300): one copy, then resident in HBM. */
int rbt_moe_load_layer(RbtMoe *m, int layer, const float *ffn_norm, const void *router, const void *experts);

/* Same as rbt_moe_load_layer, but binds DEVICE pointers the caller owns and
 * keeps alive (no copy). */
int rbt_moe_bind_layer(RbtMoe *m, int layer, const float *d_ffn_norm, const void *d_router, const void *d_experts);

/* Optional additive router-logit bias [E] f32 (host pointer), applied before the
 * softmax; NULL removes it.  Not in the reference (its router has no bias): it
 * only builds skewed-routing workloads.  Without it results equal the reference. */
int rbt_moe_set_router_bias(RbtMoe *m, int layer, const float *bias);

/* The MoE block of forward(), rabbit2.c:512-542, for n_tokens rows at once:
 *   x[t] += MoE(rmsnorm(x[t], ffn_norm))        x: [n_tokens, D] f32, in place
 * routing_out (may be NULL) receives the chosen experts in selection order,
 * row t at routing_out + t*routing_stride (the engine passes
 * routing + layer*top_k with stride n_layers*top_k).  Host pointers; returns
 * after the results are in host memory. */
int rbt_moe_block(RbtMoe *m, int layer, float *x, int n_tokens, int32_t *routing_out, int routing_stride);

/* The MoE feed-forward without the norm and residual, rabbit2.c:513-541:
 *   moe_out[t] = sum_k w_k * W2_k (silu(W1_k xb[t]) * (W3_k xb[t]))
 * xb, moe_out: [n_tokens, D] f32 host pointers. */
int rbt_moe_ffn(RbtMoe *m, int layer, const float *xb, int n_tokens, float *moe_out, int32_t *routing_out,
                int routing_stride);

/* Device-pointer forms of the two calls above, enqueued on `stream` (a
 * cudaStream_t, passed through as is: NULL is the CUDA default stream) without
 * synchronising; they allocate nothing once rbt_moe_reserve covered n_tokens,
 * so they can be captured into a CUDA graph.  x/xb/out/routing_out must be
 * device pointers; xb may equal moe_out. */
int rbt_moe_block_device(RbtMoe *m, int layer, float *d_x, int n_tokens, int32_t *d_routing_out,
                         int routing_stride, void *stream);
int rbt_moe_ffn_device(RbtMoe *m, int layer, const float *d_xb, int n_tokens, float *d_moe_out,
                       int32_t *d_routing_out, int routing_stride, void *stream);

/* ---- Expert parallelism across the GPUs of one node (no counterpart in the
 * reference, which runs one CPU process; the per-GPU arithmetic is that of
 * rabbit2.c:512-542).  GPU g of N owns experts [g*E/N, (g+1)*E/N) and the whole
 * router.  Each GPU routes its own tokens (bit-exact, as rbt_moe_block), stores
 * every token's row once into each GPU that owns one of its top-k experts (plain
 * stores to peer memory over NVLink: a token whose experts are all local never
 * leaves its GPU), runs its experts on the rows it received, stores each row's
 * partial output back into the sender's memory, and adds the partials that come
 * back in ascending GPU order.  Completion is signalled with flags holding a
 * per-call epoch, so the layer needs no host synchronisation and can be captured
 * in a CUDA graph.  Every GPU of the group must make the same sequence of calls
 * (SPMD); each passes its own n_tokens <= max_tokens.
 * Failure detection: every wait for another GPU is bounded (rbt_moe_ep_set_timeout,
 * default 2 s); one that runs out leaves the layer's output invalid and a status
 * code (0x701 rows never arrived, 0x702 partial rows never came back, 0x703 a peer
 * reported a failure of its own) that rbt_moe_status returns.  After a failure the
 * group's epochs disagree: destroy every context of the group (the counterpart of
 * aborting a communicator). */

/* Make this context rank `rank` of an expert-parallel group of n_ranks GPUs
 * (n_ranks <= 8, dividing n_experts), for calls of up to max_tokens tokens per GPU.
 * Narrows the context to its expert slice as rbt_moe_set_expert_range does, and
 * allocates its receive/return block (2 * n_ranks * max_tokens rows of dim floats
 * plus ids, weights and flags).  Call before any layer is loaded or bound. */
int rbt_moe_ep_init(RbtMoe *m, int rank, int n_ranks, int max_tokens);

/* One GPU per process: the 64-byte IPC handle of this context's block
 * (cudaIpcMemHandle_t), to be gathered by the caller from every rank in rank order
 * (n_ranks * 64 bytes) and passed to rbt_moe_ep_connect on every rank. */
int rbt_moe_ep_handle(RbtMoe *m, void *handle_out);
int rbt_moe_ep_connect(RbtMoe *m, const void *handles);

/* Every GPU in this process (ms[g] is rank g; one host thread drives them all):
 * enables peer access between their devices and connects them directly. */
int rbt_moe_ep_connect_local(RbtMoe *const *ms, int n);

/* Wait limit for the flags of other GPUs, in ns (>= 1000). */
int rbt_moe_ep_set_timeout(RbtMoe *m, uint64_t timeout_ns);

/* The expert-parallel MoE block of forward(), rabbit2.c:512-542, on this GPU's
 * n_tokens rows: d_x += MoE(rmsnorm(d_x)) in place; d_routing_out (may be NULL)
 * receives the global expert ids.  Device pointers, enqueued on `stream` without
 * synchronising; allocates nothing once rbt_moe_reserve covered n_ranks *
 * max_tokens rows. */
int rbt_moe_ep_block_device(RbtMoe *m, int layer, float *d_x, int n_tokens, int32_t *d_routing_out,
                            int routing_stride, void *stream);

/* The same for a group connected by rbt_moe_ep_connect_local, with host buffers:
 * GPU 0 (ms[0]) takes the n_tokens rows of x (in place) and returns the routing
 * rows as rbt_moe_block does; every GPU runs its experts.  Returns after the
 * results are in host memory; 0 with a message if any GPU failed. */
int rbt_moe_ep_block(RbtMoe *const *ms, int n, int layer, float *x, int n_tokens, int32_t *routing_out,
                     int routing_stride);

/* Bound, in ns, of the one-token kernel's waits on its other CTAs (the published
 * router logits, the grid barrier); 0 restores the default of 2 s.  A wait that
 * runs out ends the call with a status code (0x601 logits, 0x602 barrier): the
 * host-pointer calls return 0 with the message, the device calls leave the code
 * for rbt_moe_status, and both clear the kernel's words for the next call.  Waits
 * on the CTA's own copies keep their own bound (copies of valid memory end). */
int rbt_moe_set_timeout(RbtMoe *m, uint64_t timeout_ns);

/* The status word of the context's kernels (0: none failed), cleared after reading
 * (with the one-token kernel's words); synchronises the device.  Device-pointer
 * calls report their kernels' failures (a bounded wait that ran out) only here. */
int rbt_moe_status(RbtMoe *m, unsigned *status_out);

/* The router of the layer alone, for n_tokens rows: block != 0 gives d_xb =
 * rmsnorm(d_x) (rabbit2.c:512), block == 0 copies d_x into d_xb; then d_idx
 * [n_tokens, top_k] receives the expert ids in selection order and d_wt the combine
 * weights (rabbit2.c:513-531), bit-exact as in rbt_moe_block.  Device pointers. */
int rbt_moe_route_device(RbtMoe *m, int layer, const float *d_x, int n_tokens, int block, float *d_xb,
                         int32_t *d_idx, float *d_wt, void *stream);

/* Reserve the context's device workspace for up to n_tokens rows per call, so
 * that later calls of that size allocate nothing (e.g. before stream capture). */
int rbt_moe_reserve(RbtMoe *m, int n_tokens);

/* Per-expert routed-token counts of the most recent call, [n_experts] int32
 * (host pointer), in the key=value spirit of the engine's cache counters. */
int rbt_moe_expert_histogram(RbtMoe *m, int32_t *counts_out);

/* Force the path for later calls: 0 automatic (default), 1 CUDA-core GEMV
 * (weight streaming through shared memory when the shapes allow it), 2 the
 * tcgen05 grouped GEMM (bf16, D and H multiples of 128), 3 the plain CUDA-core
 * GEMV with a separate combine (any dtype and shape), 4 the single-kernel
 * batch-1 decode (bf16, one token, D <= 2048; automatic for one token). */
int rbt_moe_set_path(RbtMoe *m, int path);

/* Launch accounting and per-stage device timing.  Stages: 0 rmsnorm, 1 router +
 * top-k + permute, 2 gate/up + SwiGLU, 3 down, 4 combine, 5 operand gather
 * (GEMM path), 6 the fused one-token decode kernel, 7 the expert-parallel plan,
 * dispatch, receive, return and combine.  With timing on, every call records a CUDA event at each stage
 * boundary on its stream (as graph nodes when the stream is being captured)
 * and nothing waits; stage_ms sums the intervals recorded since the last reset,
 * read from the events' latest timestamps (so after a graph replay it holds
 * that replay's times).  Event gaps include host launch latency unless the
 * calls run from a CUDA graph.  The reference's only timing is wall clock on
 * stderr (rabbit2.c:742-744). */
#define RBT_MOE_STAGES 8
typedef struct RbtMoeProfile {
    int64_t calls;                           /* MoE calls since the last reset */
    int64_t launches;                        /* kernels this context launched since the reset */
    double stage_ms[RBT_MOE_STAGES];         /* summed device time per stage (timing on) */
    int64_t stage_launches[RBT_MOE_STAGES];  /* kernels per stage */
} RbtMoeProfile;

/* timing: 1 on, 0 off, -1 unchanged; reset: zero the counters after reading;
 * out may be NULL. */
int rbt_moe_profile(RbtMoe *m, int timing, int reset, RbtMoeProfile *out);

/* Router logits of the most recent block/ffn/route call, [n_tokens, n_experts]
 * f32 (host pointer; n_tokens <= that call's): the engine's s->router right
 * after the matvec of rabbit2.c:513 (plus the optional bias), before the
 * softmax.  Synchronises the device. */
int rbt_moe_router_logits(RbtMoe *m, float *logits_out, int n_tokens);

/* ---- Self-checks of the routing arithmetic (no counterpart in the reference:
 * they expose, on their own, the two pieces the router reproduces bit for bit).
 *   rbt_expf_device: d_out[i] = expf(x_i), x_i the float with bit pattern
 *     first_bits + i, evaluated as this process's libm expf evaluates it (the
 *     softmax's exp, rabbit2.c:403; rbt_host_expf_variant() says which of the
 *     two x86-64 glibc builds of it the host resolved: 1 FMA, 0 without).
 *   rbt_seq_sumsq_device: d_out[r] = the sequential f32 sum of d_x[r, i]^2 over
 *     i = 0 .. n-1, rmsnorm's sum (rabbit2.c:394), for rows of n <= 16384 floats.
 * Device pointers, enqueued on `stream` without synchronising. */
int rbt_expf_device(uint32_t first_bits, int64_t n, float *d_out, void *stream);
int rbt_seq_sumsq_device(const float *d_x, int rows, int n, float *d_out, void *stream);
int rbt_host_expf_variant(void);

/* The one-token MoE block for callers that cannot allocate GPU memory.  No
 * counterpart in the reference (its engine has no GPU and no allocator
 * constraints); it exists for code that runs inside a framework which already
 * owns the device memory (a caching allocator, or a server that reserves most
 * of HBM up front), and for latency-critical decode loops that cannot take
 * cudaMalloc's implicit synchronisation.  It needs no context and calls no
 * cudaMalloc, cudaFree or allocating library routine: its scratch is a fixed
 * RBT_MOE_NOALLOC_SCRATCH_BYTES array in the library's own device memory,
 * present on every GPU that loads the library until the process exits.
 *
 * Runs on the calling thread's current CUDA device, enqueued on `stream`
 * (NULL = default stream), without synchronising.  All pointers are device
 * pointers: the layer's weights exactly as for rbt_moe_bind_layer,
 * d_router_bias may be NULL, and d_routing_out ([top_k] int32) may be NULL.
 * d_ffn_norm != NULL gives the block form, d_out = d_x + MoE(rmsnorm(d_x))
 * (d_out may equal d_x); d_ffn_norm == NULL gives d_out = MoE(d_x).
 * Limits: bf16 weights, dim <= 2048 and a multiple of 16, expert_hidden a
 * multiple of 8, n_experts <= 256, top_k <= 64, 16-byte aligned
 * d_x/d_router/d_experts/d_ffn_norm, and scratch of (SM count x dim) floats plus the
 * routing buffers within RBT_MOE_NOALLOC_SCRATCH_BYTES (1.5 MiB: a 148-SM
 * B200 at dim 2048 needs 1.16 MiB); other models are rejected with an error.  The first call on a device looks
 * up the array's device address; make that first call before any stream
 * capture.  Calls share the array: two calls whose kernels overlap on the GPU
 * (unordered streams) race. */
#define RBT_MOE_NOALLOC_SCRATCH_BYTES 1572864
int rbt_moe_decode_noalloc(const RbtMoeConfig *cfg, const float *d_ffn_norm, const void *d_router,
                           const float *d_router_bias, const void *d_experts, const float *d_x, float *d_out,
                           int32_t *d_routing_out, void *stream);

/* Error status of the most recent rbt_moe_decode_noalloc kernel on the calling
 * thread's current device.  rbt_moe_decode_noalloc returns 1 as soon as its
 * kernel is enqueued, so it cannot report what goes wrong inside the kernel;
 * this call copies the kernel's status word from the fixed array on `stream`,
 * synchronises that stream and stores it in *status_out: 0 when the kernel
 * completed normally, otherwise its error code -- 0x603 when no valid routing
 * could be formed (NaN or Inf in d_x), 0x600-0x6ff when a bounded wait between
 * CTAs ran out.  After a non-zero status d_out and d_routing_out hold no
 * result.  Allocates nothing. */
int rbt_moe_decode_noalloc_status(void *stream, unsigned *status_out);

/* ---- The whole forward() on the GPU (rabbit2.c:455-550) ----
 * The engine's forward(Model*, State*, token, pos, routing_out) computes one
 * token: embedding row, then per layer RMSNorm, Q/K/V projections, whole-
 * projection QK-norm, RoPE, causal attention over the KV cache, the output
 * projection and residual, then the MoE block; then the final norm and lm_head.
 * An RbtModel holds every weight and the KV cache in HBM and runs that token as
 * one CUDA graph; the MoE blocks are rbt_moe_block's kernels. */

/* The engine's Config (rabbit2.c:63-68, the on-disk header fields in order) plus
 * Model.expert_stride (rabbit2.c:173). */
typedef struct RbtModelConfig {
    int32_t vocab, dim, n_layers, n_heads, n_kv_heads, head_dim;
    int32_t n_experts, top_k, expert_hidden, max_seq;
    int32_t dtype, qk_norm, norm_topk;
    float rope_theta, rms_eps;
    uint64_t expert_stride;
} RbtModelConfig;

typedef struct RbtModel RbtModel; /* opaque: weights, KV cache and graphs on one GPU */

/* Create a model on CUDA device `device` with a KV cache of `ctx` positions
 * (1..max_seq); the State of rabbit2.c:101-106 lives on the GPU. */
int rbt_model_create(RbtModel **out, const RbtModelConfig *cfg, int ctx, int device);
void rbt_model_destroy(RbtModel *m);

/* Upload weights from host memory (the mmap'd .rbt2; Model/LayerOff offsets of
 * rabbit2.c:70-100): tok_emb [vocab,dim], final_norm [dim] f32, lm_head
 * [vocab,dim]; per layer attn_norm [dim], wq [n_heads*head_dim, dim], wk and wv
 * [n_kv_heads*head_dim, dim], wo [dim, n_heads*head_dim], q_norm/k_norm (f32,
 * NULL when qk_norm is 0), ffn_norm [dim], router [n_experts, dim] and the
 * layer's first expert blob.  Every layer and the globals must be loaded before
 * rbt_model_forward. */
int rbt_model_load_globals(RbtModel *m, const void *tok_emb, const float *final_norm, const void *lm_head);
int rbt_model_load_layer(RbtModel *m, int layer, const float *attn_norm, const void *wq, const void *wk,
                         const void *wv, const void *wo, const float *q_norm, const float *k_norm,
                         const float *ffn_norm, const void *router, const void *experts);

/* forward(): the token at position pos (0 <= pos < ctx; positions are filled in
 * order, as the engine does).  logits [vocab] (host, or NULL to skip lm_head)
 * and routing_out [n_layers*top_k] (host, or NULL) receive the engine's
 * s->logits and routing rows. */
int rbt_model_forward(RbtModel *m, int token, int pos, float *logits, int32_t *routing_out);

/* The prompt loop of the engine's main() (rabbit2.c:703-714) in one call:
 * forward() for tokens[0..n_tokens) at positions pos0 .. pos0 + n_tokens, run
 * layer by layer over all of them (the projections as GEMMs, the MoE blocks on
 * the tensor-core path).  logits [logit_rows, vocab] (host) receive the logits of
 * the LAST logit_rows tokens (0: none; 1: what the sampler reads; n_tokens: every
 * row, as --dump writes them); routing_out [n_tokens, n_layers, top_k] (host) or
 * NULL.  The KV cache is the one rbt_model_forward uses: decoding continues at
 * pos0 + n_tokens.  Needs head_dim 64 or 128. */
int rbt_model_prefill(RbtModel *m, const int32_t *tokens, int n_tokens, int pos0, float *logits, int logit_rows,
                      int32_t *routing_out);

/* ---- several sequences (serving): the reference decodes one sequence per
 * process (rabbit2.c:716-738); these calls keep n_seq sequences' KV caches on the
 * GPU and decode one token of each in one call.
 *
 * rbt_model_set_sequences: KV caches for n_seq >= 1 sequences (the model starts
 * with 1), every cache zeroed.  Sequence 0 is the one rbt_model_forward and
 * rbt_model_prefill use.
 *
 * rbt_model_prefill_seq: rbt_model_prefill into the cache of sequence seq.
 *
 * rbt_model_decode_batch: forward() for n rows (1 <= n <= n_seq), row i the token
 * tokens[i] of sequence i at position pos[i] (its cache holds positions
 * 0..pos[i]-1, filled by earlier calls).  The projections run as GEMMs over the n
 * rows and the MoE block over all n rows at once; each row's attention reads
 * only its own sequence's cache.  Outputs (host, each may be NULL): logits
 * [n, vocab]; next [n], each row's greedy id as the engine's argmax
 * (rabbit2.c:552-556: the first maximum); routing_out [n, n_layers, top_k].  Row
 * i's results equal rbt_model_forward's for that token within the GEMMs'
 * summation order (f32 models) or operand split (bf16 models).
 *
 * rbt_model_set_router_bias: rbt_moe_set_router_bias on the model's MoE layers
 * (a popularity skew for load-imbalance workloads; not in the reference).
 *
 * rbt_model_moe: the model's MoE context, for rbt_moe_ep_init / _handle /
 * _connect / _connect_local / _set_timeout / rbt_moe_status.  Once it is
 * connected to an expert-parallel group (rbt_moe_ep_init before the layers are
 * loaded, each layer's `experts` pointing at this rank's first expert), every
 * MoE block of rbt_model_forward, _prefill* and _decode_batch runs through the
 * group, and every rank of the group must make the same sequence of calls (the
 * row counts may differ, up to max_tokens). */
int rbt_model_set_sequences(RbtModel *m, int n_seq);
int rbt_model_prefill_seq(RbtModel *m, int seq, const int32_t *tokens, int n_tokens, int pos0, float *logits,
                          int logit_rows, int32_t *routing_out);
int rbt_model_decode_batch(RbtModel *m, const int32_t *tokens, const int32_t *pos, int n, float *logits,
                           int32_t *next, int32_t *routing_out);
int rbt_model_set_router_bias(RbtModel *m, int layer, const float *bias);
RbtMoe *rbt_model_moe(RbtModel *m);

/* Last error message of the calling thread ("" if none). */
const char *rbt_moe_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* RBT_MOE_H */
