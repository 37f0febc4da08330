/*
 * rbt_engine_hook.h -- the glue a RABBIT2 engine build includes to run its MoE
 * blocks on the GPU through librbt_moe.so (include/rbt_moe.h).
 *
 * Included by rabbit2.c right before forward() (it uses the engine's Model,
 * State, LayerOff, VEC, MAT and its rmsnorm / matvec, all defined above
 * forward(), and rbt_engine_attention_block: forward()'s own attention half,
 * which patch_engine.py copies into a function of its own).  Call sites:
 *   main(), argument loop:  --device cpu|cuda   sets rbt_engine_device
 *                           --prefill batch|token   sets rbt_engine_prefill_mode
 *                           --offload moe|all       sets rbt_engine_offload
 *                           --routing-trace FILE    sets rbt_engine_trace_path
 *                           --ep N                  sets rbt_engine_ep_arg
 *   main(), after load_model():  rbt_engine_init(&m)
 *   forward(), first statement (rabbit2.c:455):
 *       { int g = rbt_engine_forward(m, s, token, pos, routing_out);
 *         if (g < 0) return 0; if (g) return 1; }
 *   forward(), first line of the MoE block (rabbit2.c:511):
 *       { int g = rbt_engine_moe(m, l, s->x, routing_out + (size_t)l * c->top_k);
 *         if (g < 0) return 0; if (g) continue; }
 *   main(), before the prompt loop (rabbit2.c:703-704):
 *       const int pre = rbt_engine_prefill(&m, &s, tokens, nt, routing, fl, fr);
 *       (on -1: close the dump files, return 1), and the loop starts at
 *       i = pre ? nt : 0.
 *   main(), after each forward() of the prompt loop and of the --gen loop:
 *       rbt_engine_record(&m, routing)
 *   main(), after the timing line (rabbit2.c:742-744): rbt_engine_report(&m)
 * Every run (cpu or cuda) counts the experts each layer routed its tokens to and
 * reports them at exit as stderr lines in the engine's key=value style
 * (rabbit2.c:745-751):  expert histogram: layer=<l> tokens=<n> counts=<c0>,<c1>,...
 * --routing-trace FILE writes every processed token's routing row, int32
 * [n_layers][top_k] per token in processing order -- the layout of --dump's
 * routing file (rabbit2.c:711-712), which tools/benchmark_cache.py replays.
 * With --device cpu (the default) nothing changes: the engine's own CPU block runs.
 * With --device cuda every layer's router and expert blobs are copied once from
 * the mapped file into HBM, and each MoE block is one rbt_moe_block() call that
 * returns x updated in place and the layer's routing row, as the CPU block does.
 * With --device cuda --offload all every weight is copied, and each forward() is
 * one rbt_model_forward() call (attention and lm_head on the GPU as well).
 * With --device cuda --ep N (N > 1; the MoE offload) the experts are split over GPUs
 * 0..N-1 of this process: GPU g holds experts [g*E/N, (g+1)*E/N) of every layer,
 * and each MoE block is one rbt_moe_ep_block() call: GPU 0 routes the tokens, every
 * GPU runs its experts on the rows routed to it (rows and partial results move
 * over NVLink peer memory), and GPU 0 adds the partials in GPU order.
 */
#ifndef RBT_ENGINE_HOOK_H
#define RBT_ENGINE_HOOK_H

#include "rbt_moe.h"

static const char *rbt_engine_device = NULL;
static const char *rbt_engine_prefill_mode = NULL;  /* --prefill batch|token */
static const char *rbt_engine_offload = NULL;       /* --offload moe|all */
static const char *rbt_engine_trace_path = NULL;   /* --routing-trace FILE */
static const char *rbt_engine_ep_arg = NULL;        /* --ep N */
static int rbt_engine_ep = 1;                       /* GPUs the experts are split over */
static RbtMoe *rbt_engine_ep_ctx[8];
static RbtMoe *rbt_engine_ctx = NULL;
static RbtModel *rbt_engine_model = NULL;           /* --offload all: the whole forward() */
static FILE *rbt_engine_trace = NULL;
static long long *rbt_engine_hist = NULL;           /* [n_layers][n_experts] routed tokens */
static long long rbt_engine_tokens = 0;

/* One processed token's routing rows [n_layers][top_k]: the histogram, and the trace. */
static void rbt_engine_record(const Model *m, const int32_t *routing) {
    const Config *c = &m->c;
    if (rbt_engine_hist) {
        for (int l = 0; l < c->n_layers; l++)
            for (int k = 0; k < c->top_k; k++) {
                const int e = routing[(size_t)l * c->top_k + k];
                if (e >= 0 && e < c->n_experts) rbt_engine_hist[(size_t)l * c->n_experts + e]++;
            }
        rbt_engine_tokens++;
    }
    if (rbt_engine_trace)
        fwrite(routing, sizeof(int32_t), (size_t)c->n_layers * c->top_k, rbt_engine_trace);
}

/* At exit: the per-layer expert histogram on stderr; the trace file closed. */
static void rbt_engine_report(const Model *m) {
    const Config *c = &m->c;
    if (rbt_engine_hist && rbt_engine_tokens > 0) {
        for (int l = 0; l < c->n_layers; l++) {
            fprintf(stderr, "expert histogram: layer=%d tokens=%lld counts=", l, rbt_engine_tokens);
            for (int e = 0; e < c->n_experts; e++)
                fprintf(stderr, "%s%lld", e ? "," : "", rbt_engine_hist[(size_t)l * c->n_experts + e]);
            fprintf(stderr, "\n");
        }
    }
    if (rbt_engine_trace) {
        fclose(rbt_engine_trace);
        rbt_engine_trace = NULL;
    }
    free(rbt_engine_hist);
    rbt_engine_hist = NULL;
}

static int rbt_engine_init(Model *m) {
    if (rbt_engine_prefill_mode && strcmp(rbt_engine_prefill_mode, "batch") != 0 &&
        strcmp(rbt_engine_prefill_mode, "token") != 0) {
        fprintf(stderr, "--prefill must be batch or token\n");
        return 0;
    }
    if (rbt_engine_offload && strcmp(rbt_engine_offload, "moe") != 0 && strcmp(rbt_engine_offload, "all") != 0) {
        fprintf(stderr, "--offload must be moe or all\n");
        return 0;
    }
    rbt_engine_hist = (long long *)calloc((size_t)m->c.n_layers * m->c.n_experts, sizeof(long long));
    if (rbt_engine_trace_path && !(rbt_engine_trace = fopen(rbt_engine_trace_path, "wb"))) {
        fprintf(stderr, "cannot open the routing trace %s\n", rbt_engine_trace_path);
        return 0;
    }
    if (!rbt_engine_device || !strcmp(rbt_engine_device, "cpu")) return 1;
    if (strcmp(rbt_engine_device, "cuda") != 0) {
        fprintf(stderr, "--device must be cpu or cuda\n");
        return 0;
    }
    const Config *c = &m->c;
    if (rbt_engine_ep_arg) {
        rbt_engine_ep = atoi(rbt_engine_ep_arg);
        if (rbt_engine_ep < 1 || rbt_engine_ep > 8 || c->n_experts % rbt_engine_ep != 0) {
            fprintf(stderr, "--ep must be 1..8 and divide n_experts (%d)\n", c->n_experts);
            return 0;
        }
        if (rbt_engine_ep > 1 && rbt_engine_offload && !strcmp(rbt_engine_offload, "all")) {
            fprintf(stderr, "--ep splits the MoE offload's experts; it does not combine with --offload all\n");
            return 0;
        }
    }
    if (rbt_engine_offload && !strcmp(rbt_engine_offload, "all")) {
        /* every weight and a KV cache of max_seq positions in HBM (the engine
           picks its --ctx later; it never exceeds max_seq) */
        RbtModelConfig mc;
        mc.vocab = c->vocab;
        mc.dim = c->dim;
        mc.n_layers = c->n_layers;
        mc.n_heads = c->n_heads;
        mc.n_kv_heads = c->n_kv_heads;
        mc.head_dim = c->head_dim;
        mc.n_experts = c->n_experts;
        mc.top_k = c->top_k;
        mc.expert_hidden = c->expert_hidden;
        mc.max_seq = c->max_seq;
        mc.dtype = c->dtype;
        mc.qk_norm = c->qk_norm;
        mc.norm_topk = c->norm_topk;
        mc.rope_theta = c->rope_theta;
        mc.rms_eps = c->rms_eps;
        mc.expert_stride = (uint64_t)m->expert_stride;
        if (!rbt_model_create(&rbt_engine_model, &mc, c->max_seq, 0)) return 0;
        if (!rbt_model_load_globals(rbt_engine_model, MAT(m, m->tok_emb), VEC(m, m->final_norm), MAT(m, m->lm_head)))
            return 0;
        for (int l = 0; l < c->n_layers; l++) {
            const LayerOff *ly = &m->layers[l];
            if (!rbt_model_load_layer(rbt_engine_model, l, VEC(m, ly->attn_norm), MAT(m, ly->wq), MAT(m, ly->wk),
                                      MAT(m, ly->wv), MAT(m, ly->wo), c->qk_norm ? VEC(m, ly->q_norm) : NULL,
                                      c->qk_norm ? VEC(m, ly->k_norm) : NULL, VEC(m, ly->ffn_norm),
                                      MAT(m, ly->router), m->map.base + ly->experts))
                return 0;
        }
        fprintf(stderr, "forward device: cuda (librbt_moe, whole model resident)\n");
        return 1;
    }
    RbtMoeConfig cfg;
    cfg.dim = c->dim;
    cfg.n_experts = c->n_experts;
    cfg.top_k = c->top_k;
    cfg.expert_hidden = c->expert_hidden;
    cfg.n_layers = c->n_layers;
    cfg.dtype = c->dtype;
    cfg.norm_topk = c->norm_topk;
    cfg.rms_eps = c->rms_eps;
    cfg.expert_stride = (uint64_t)m->expert_stride;
    if (rbt_engine_ep > 1) {
        /* one context per GPU, each holding its slice of every layer's experts; the
           prompt can reach max_seq tokens in one batched call */
        const int epr = c->n_experts / rbt_engine_ep;
        for (int g = 0; g < rbt_engine_ep; g++) {
            if (!rbt_moe_create(&rbt_engine_ep_ctx[g], &cfg, g) ||
                !rbt_moe_ep_init(rbt_engine_ep_ctx[g], g, rbt_engine_ep, c->max_seq))
                return 0;
            for (int l = 0; l < c->n_layers; l++) {
                const LayerOff *ly = &m->layers[l];
                if (!rbt_moe_load_layer(rbt_engine_ep_ctx[g], l, VEC(m, ly->ffn_norm), MAT(m, ly->router),
                                        m->map.base + ly->experts + (size_t)g * epr * m->expert_stride))
                    return 0;
            }
        }
        if (!rbt_moe_ep_connect_local(rbt_engine_ep_ctx, rbt_engine_ep)) return 0;
        rbt_engine_ctx = rbt_engine_ep_ctx[0];
        fprintf(stderr, "moe device: cuda (librbt_moe, experts split over %d GPUs, %d layers resident)\n",
                rbt_engine_ep, c->n_layers);
        return 1;
    }
    if (!rbt_moe_create(&rbt_engine_ctx, &cfg, 0)) return 0;
    for (int l = 0; l < c->n_layers; l++) {
        const LayerOff *ly = &m->layers[l];
        if (!rbt_moe_load_layer(rbt_engine_ctx, l, VEC(m, ly->ffn_norm), MAT(m, ly->router),
                                m->map.base + ly->experts))
            return 0;
    }
    fprintf(stderr, "moe device: cuda (librbt_moe, %d layers resident)\n", c->n_layers);
    return 1;
}

/* --offload all: forward() for one token on the GPU, s->logits and the routing
 * rows filled as the engine's own forward() fills them.  1: done; 0: not
 * enabled (run the engine's forward); -1: error. */
static int rbt_engine_forward(Model *m, State *s, int token, int pos, int32_t *routing_out) {
    (void)m;
    if (!rbt_engine_model) return 0;
    return rbt_model_forward(rbt_engine_model, token, pos, s->logits, routing_out) ? 1 : -1;
}

/* 1: the GPU ran the block; 0: not enabled (run the CPU block); -1: error. */
static int rbt_engine_moe(Model *m, int layer, float *x, int32_t *routing_row) {
    if (!rbt_engine_ctx) return 0;
    if (rbt_engine_ep > 1)
        return rbt_moe_ep_block(rbt_engine_ep_ctx, rbt_engine_ep, layer, x, 1, routing_row, m->c.top_k) ? 1 : -1;
    return rbt_moe_block(rbt_engine_ctx, layer, x, 1, routing_row, m->c.top_k) ? 1 : -1;
}

/* ---- the prompt as one batch per layer ----
 * The engine's prompt loop runs forward() token by token, so each MoE block sees
 * one token.  With --device cuda the prompt instead runs layer by layer: every
 * prompt token's attention half of layer l (on the CPU, as the engine computes it),
 * then ONE rbt_moe_block call for all of them, which the library runs on the
 * tensor cores.  Attention of token t at layer l reads the KV cache of positions
 * <= t of layer l only, which tokens 0..t have written by then, so the order
 * changes no value.  With --offload all the whole prompt is one
 * rbt_model_prefill call instead.  --prefill token keeps the engine's per-token
 * loop. */

/* Layer l's attention half for the token at position pos; x [dim] is updated in
 * place.  This is forward()'s own code for it (rbt_engine_attention_block, on
 * s->x), so the results are the same bits as the engine's per-token loop. */
static void rbt_engine_attention(Model *m, State *s, int l, float *x, int pos) {
    const size_t bytes = (size_t)m->c.dim * sizeof(float);
    memcpy(s->x, x, bytes);
    rbt_engine_attention_block(m, s, l, pos);
    memcpy(x, s->x, bytes);
}

/* --offload all: the whole prompt in one rbt_model_prefill call (every layer on
 * the GPU over all prompt rows); the outputs as rbt_engine_prefill below
 * describes them. */
static int rbt_engine_prefill_model(Model *m, State *s, const int *tokens, int nt, int32_t *routing, FILE *fl,
                                    FILE *fr) {
    const Config *c = &m->c;
    const size_t row = (size_t)c->n_layers * c->top_k;
    const int rows = fl ? nt : 1;  /* logits of every token for --dump, else of the last */
    float *lg = (float *)malloc((size_t)rows * c->vocab * sizeof(float));
    int32_t *R = (int32_t *)malloc((size_t)nt * row * sizeof(int32_t));
    int32_t *tok = (int32_t *)malloc((size_t)nt * sizeof(int32_t));
    int ok = lg && R && tok;
    if (!ok) fprintf(stderr, "out of memory for the batched prompt (try --prefill token)\n");
    for (int t = 0; ok && t < nt; t++) tok[t] = tokens[t];
    if (ok) ok = rbt_model_prefill(rbt_engine_model, tok, nt, 0, lg, rows, R);
    for (int t = 0; ok && fl && t < nt; t++)
        if (fwrite(lg + (size_t)t * c->vocab, sizeof(float), (size_t)c->vocab, fl) != (size_t)c->vocab ||
            fwrite(R + (size_t)t * row, sizeof(int32_t), row, fr) != row) {
            fprintf(stderr, "cannot write the dump files\n");
            ok = 0;
        }
    if (ok) {
        memcpy(s->logits, lg + (size_t)(rows - 1) * c->vocab, (size_t)c->vocab * sizeof(float));
        memcpy(routing, R + (size_t)(nt - 1) * row, row * sizeof(int32_t));
        for (int t = 0; t < nt; t++) rbt_engine_record(m, R + (size_t)t * row);
    }
    free(lg);
    free(R);
    free(tok);
    return ok ? 1 : -1;
}

/* The prompt tokens[0..nt) at positions 0..nt: 1 when it ran here (the last
 * token's logits in s->logits and its routing rows in `routing`, as the engine's
 * loop leaves them; with --dump every token's logits and routing rows written to
 * fl / fr in the engine's format), 0 when not enabled (the engine's loop runs),
 * -1 on an error (message on stderr). */
static int rbt_engine_prefill(Model *m, State *s, const int *tokens, int nt, int32_t *routing, FILE *fl,
                              FILE *fr) {
    if (nt < 2 || (rbt_engine_prefill_mode && !strcmp(rbt_engine_prefill_mode, "token"))) return 0;
    if (rbt_engine_model) return rbt_engine_prefill_model(m, s, tokens, nt, routing, fl, fr);
    if (!rbt_engine_ctx) return 0;
    const Config *c = &m->c;
    const int D = c->dim;
    const size_t row = (size_t)c->n_layers * c->top_k;  /* routing ints per token */
    float *X = (float *)malloc((size_t)nt * D * sizeof(float));
    int32_t *R = (int32_t *)malloc((size_t)nt * row * sizeof(int32_t));
    if (!X || !R) {
        free(X);
        free(R);
        fprintf(stderr, "out of memory for the batched prompt (try --prefill token)\n");
        return -1;
    }
    for (int t = 0; t < nt; t++) {  /* embedding rows, converted as forward() does */
        float *x = X + (size_t)t * D;
        if (c->dtype == DT_F32) {
            memcpy(x, (const float *)MAT(m, m->tok_emb) + (size_t)tokens[t] * D, (size_t)D * sizeof(float));
        } else {
            const uint16_t *e = (const uint16_t *)MAT(m, m->tok_emb) + (size_t)tokens[t] * D;
            for (int i = 0; i < D; i++) x[i] = bf16f(e[i]);
        }
    }
    int ok = 1;
    for (int l = 0; ok && l < c->n_layers; l++) {
        for (int t = 0; t < nt; t++) rbt_engine_attention(m, s, l, X + (size_t)t * D, t);
        ok = rbt_engine_ep > 1
                 ? rbt_moe_ep_block(rbt_engine_ep_ctx, rbt_engine_ep, l, X, nt, R + (size_t)l * c->top_k, (int)row)
                 : rbt_moe_block(rbt_engine_ctx, l, X, nt, R + (size_t)l * c->top_k, (int)row);
    }
    /* final norm and lm_head: every token for --dump, else the last one only */
    for (int t = fl ? 0 : nt - 1; ok && t < nt; t++) {
        rmsnorm(s->xb, X + (size_t)t * D, VEC(m, m->final_norm), D, c->rms_eps);
        matvec(s->logits, MAT(m, m->lm_head), c->dtype, s->xb, c->vocab, D);
        if (fl && (fwrite(s->logits, sizeof(float), (size_t)c->vocab, fl) != (size_t)c->vocab ||
                   fwrite(R + (size_t)t * row, sizeof(int32_t), row, fr) != row)) {
            fprintf(stderr, "cannot write the dump files\n");
            ok = 0;
        }
    }
    if (ok) {
        memcpy(routing, R + (size_t)(nt - 1) * row, row * sizeof(int32_t));
        for (int t = 0; t < nt; t++) rbt_engine_record(m, R + (size_t)t * row);
    }
    free(X);
    free(R);
    return ok ? 1 : -1;
}

#endif /* RBT_ENGINE_HOOK_H */
