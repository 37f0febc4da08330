/*
 * rbt_engine_hook.h -- the glue a RABBIT2 engine build includes to run its MoE
 * blocks on the GPU through librbt_moe.so (include/rbt_moe.h).
 *
 * Included by rabbit2.c right before forward() (it uses the engine's Model,
 * LayerOff, VEC and MAT from rabbit2.c:63-103,230-231).  Three call sites:
 *   main(), argument loop:  --device cpu|cuda   sets rbt_engine_device
 *   main(), after load_model():  rbt_engine_init(&m)
 *   forward(), first line of the MoE block (rabbit2.c:511):
 *       { int g = rbt_engine_moe(m, l, s->x, routing_out + (size_t)l * c->top_k);
 *         if (g < 0) return 0; if (g) continue; }
 * With --device cpu (the default) nothing changes: the engine's own CPU block runs.
 * With --device cuda every layer's router and expert blobs are copied once from
 * the mapped file into HBM, and each MoE block is one rbt_moe_block() call that
 * returns x updated in place and the layer's routing row, as the CPU block does.
 */
#ifndef RBT_ENGINE_HOOK_H
#define RBT_ENGINE_HOOK_H

#include "rbt_moe.h"

static const char *rbt_engine_device = NULL;
static RbtMoe *rbt_engine_ctx = NULL;

static int rbt_engine_init(Model *m) {
    if (!rbt_engine_device || !strcmp(rbt_engine_device, "cpu")) return 1;
    if (strcmp(rbt_engine_device, "cuda") != 0) {
        fprintf(stderr, "--device must be cpu or cuda\n");
        return 0;
    }
    const Config *c = &m->c;
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

/* 1: the GPU ran the block; 0: not enabled (run the CPU block); -1: error. */
static int rbt_engine_moe(Model *m, int layer, float *x, int32_t *routing_row) {
    if (!rbt_engine_ctx) return 0;
    return rbt_moe_block(rbt_engine_ctx, layer, x, 1, routing_row, m->c.top_k) ? 1 : -1;
}

#endif /* RBT_ENGINE_HOOK_H */
