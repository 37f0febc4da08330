/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference engine's own source (rabbit2/src/rabbit2.c, included
 * from where it lies; its main() is renamed by -Dmain=rbt_ref_main) and exposes
 * its static kernels matvec/softmax/silu/rmsnorm through the MoE control flow of
 * rabbit2.c:512-541, so that the CPU restatement in moe_oracle.c can be checked
 * bit-for-bit against the reference's compiled arithmetic, and so that bench.py
 * can time the reference's own CPU MoE layer ("kind": "reference").
 *
 * Built by oracle/Makefile into oracle/_ref/ only.  The router bias is the same
 * workload extension as in moe_oracle.c (NULL = reference behaviour).
 */
#include RABBIT2_SRC

#include <pthread.h>

#include "moe_oracle.h"

/* Select the reference's matvec kernel: 0 scalar (its default and parity
 * oracle), 1 AVX2 (rabbit2.c:312-321).  Returns the kernel actually selected. */
int ref_set_kernel(int avx2) {
    use_avx2 = avx2 && cpu_has_avx2();
    return use_avx2;
}

typedef struct {
    const OrcMoeLayer *L;
    const float *x;
    float *out;
    int32_t *routing;
    int routing_stride;
    int block;
    int t0, t1, ok;
} RefJob;

static void *ref_worker(void *arg) {
    RefJob *j = (RefJob *)arg;
    const OrcMoeLayer *L = j->L;
    const int D = L->D, H = L->H, E = L->E, K = L->K;
    float *router = (float *)malloc(sizeof(float) * (size_t)E);
    float *h1 = (float *)malloc(sizeof(float) * (size_t)H);
    float *h3 = (float *)malloc(sizeof(float) * (size_t)H);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)D);
    float *xb = (float *)malloc(sizeof(float) * (size_t)D);
    unsigned char *used = (unsigned char *)malloc((size_t)E);
    j->ok = router && h1 && h3 && tmp && xb && used;
    const size_t esz = L->dtype == DT_BF16 ? 2 : 4;
    const size_t mat_bytes = (size_t)H * D * esz;
    for (int t = j->t0; j->ok && t < j->t1; t++) {
        const float *xt = j->x + (size_t)t * D;
        float *moe = j->out + (size_t)t * D;
        if (j->block) rmsnorm(xb, xt, L->ffn_norm, D, L->rms_eps);
        else memcpy(xb, xt, sizeof(float) * (size_t)D);
        /* rabbit2.c:513-528 */
        matvec(router, L->router, L->dtype, xb, E, D);
        if (L->router_bias)
            for (int e = 0; e < E; e++) router[e] += L->router_bias[e];
        softmax(router, E);
        int idx[MAX_TOPK];
        float wt[MAX_TOPK], wsum = 0.0f;
        memset(used, 0, (size_t)E);
        for (int k = 0; k < K; k++) {
            int best = -1;
            for (int e = 0; e < E; e++)
                if (!used[e] && (best < 0 || router[e] > router[best])) best = e;
            used[best] = 1;
            idx[k] = best;
            wt[k] = router[best];
            wsum += wt[k];
            if (j->routing) j->routing[(size_t)t * j->routing_stride + k] = best;
        }
        /* rabbit2.c:530-541 (get_expert reduced to its mmap branch, :262-264) */
        memset(moe, 0, (size_t)D * sizeof(float));
        for (int k = 0; k < K; k++) {
            const unsigned char *eb = (const unsigned char *)L->experts + (size_t)idx[k] * L->expert_stride;
            matvec(h1, eb, L->dtype, xb, H, D);
            matvec(h3, eb + mat_bytes, L->dtype, xb, H, D);
            for (int i = 0; i < H; i++) h1[i] = silu(h1[i]) * h3[i];
            matvec(tmp, eb + 2 * mat_bytes, L->dtype, h1, D, H);
            const float wk = L->norm_topk ? wt[k] / wsum : wt[k];
            for (int i = 0; i < D; i++) moe[i] += wk * tmp[i];
        }
        if (j->block)
            for (int i = 0; i < D; i++) moe[i] = xt[i] + moe[i]; /* rabbit2.c:542 */
    }
    free(router); free(h1); free(h3); free(tmp); free(xb); free(used);
    return NULL;
}

static int ref_run(const OrcMoeLayer *L, const float *x, int T, float *out, int32_t *routing, int routing_stride,
                   int block, int nthreads) {
    if (!L || !x || !out || T < 0 || L->K < 1 || L->K > MAX_TOPK || L->K > L->E) return 0;
    if (block && !L->ffn_norm) return 0;
    if (routing_stride <= 0) routing_stride = L->K;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > T) nthreads = T > 0 ? T : 1;
    RefJob *jobs = (RefJob *)calloc((size_t)nthreads, sizeof(RefJob));
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    int *started = (int *)calloc((size_t)nthreads, sizeof(int));
    if (!jobs || !th || !started) { free(jobs); free(th); free(started); return 0; }
    for (int i = 0; i < nthreads; i++)
        jobs[i] = (RefJob){L, x, out, routing, routing_stride, block,
                           (int)((long)T * i / nthreads), (int)((long)T * (i + 1) / nthreads), 0};
    int ok = 1;
    for (int i = 1; i < nthreads; i++) started[i] = pthread_create(&th[i], NULL, ref_worker, &jobs[i]) == 0;
    ref_worker(&jobs[0]);
    for (int i = 1; i < nthreads; i++) {
        if (started[i]) pthread_join(th[i], NULL);
        else ref_worker(&jobs[i]);
    }
    for (int i = 0; i < nthreads; i++) ok &= jobs[i].ok;
    free(jobs); free(th); free(started);
    return ok;
}

int ref_moe_ffn(const OrcMoeLayer *L, const float *xb, int T, float *moe_out, int32_t *routing, int routing_stride,
                int nthreads) {
    return ref_run(L, xb, T, moe_out, routing, routing_stride, 0, nthreads);
}

int ref_moe_block(const OrcMoeLayer *L, const float *x, int T, float *x_out, int32_t *routing, int routing_stride,
                  int nthreads) {
    return ref_run(L, x, T, x_out, routing, routing_stride, 1, nthreads);
}

/* The engine's greedy decode loop (rabbit2.c:703-738 at temperature 0: forward() for
 * every prompt token, then argmax and forward() per generated token) on a model whose
 * .rbt2 bytes are held in memory at `image` (size bytes), in place of the engine's
 * mmap of the file (map_file, rabbit2.c:129-157).  The header checks of load_model
 * (rabbit2.c:199-228) are restated; layout(), state_init(), forward() and argmax()
 * are the reference's own.  Times the two phases with the engine's clock (now_sec)
 * as its stderr line does (rabbit2.c:742-744).  ids_out [n_gen]. */
int ref_decode_image(const unsigned char *image, size_t size, int avx2, const int32_t *prompt, int n_prompt,
                     int n_gen, int32_t *ids_out, double *sec_prompt, double *sec_gen) {
    Model m;
    memset(&m, 0, sizeof m);
    m.map.base = (unsigned char *)image;
    m.map.size = size;
    if (size < HEADER_BYTES || memcmp(image, "RBT2", 4) != 0) return 0;
    uint32_t version;
    memcpy(&version, image + 4, 4);
    if (version != 2) return 0;
    memcpy(&m.c, image + 8, sizeof(Config));
    const Config *c = &m.c;
    if (c->vocab <= 0 || c->dim <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 ||
        c->top_k <= 0 || c->top_k > c->n_experts || c->top_k > MAX_TOPK || n_prompt < 1 || n_gen < 1)
        return 0;
    m.esz = (c->dtype == DT_BF16) ? 2 : 4;
    m.layers = (LayerOff *)calloc((size_t)c->n_layers, sizeof(LayerOff));
    if (!m.layers) return 0;
    layout(&m);
    if (layout_end(&m) > size) { free(m.layers); return 0; }
    use_avx2 = avx2 && cpu_has_avx2();
    State s;
    memset(&s, 0, sizeof s);
    state_init(&s, c, n_prompt + n_gen);
    int32_t *routing = (int32_t *)calloc((size_t)c->n_layers * c->top_k, sizeof(int32_t));
    int ok = state_ok(&s) && routing;
    double t0 = now_sec();
    for (int i = 0; ok && i < n_prompt; i++) ok = forward(&m, &s, prompt[i], i, routing);
    double t1 = now_sec();
    for (int g = 0, pos = n_prompt; ok && g < n_gen; g++) {
        const int next = argmax(s.logits, c->vocab);
        ids_out[g] = next;
        if (g + 1 < n_gen) ok = forward(&m, &s, next, pos++, routing);
    }
    double t2 = now_sec();
    *sec_prompt = t1 - t0;
    *sec_gen = t2 - t1;
    free(routing);
    free(s.x); free(s.xb); free(s.q); free(s.k); free(s.v); free(s.att); free(s.attn_out); free(s.router);
    free(s.h1); free(s.h3); free(s.tmp); free(s.moe); free(s.logits); free(s.kcache); free(s.vcache); free(s.used);
    free(m.layers);
    return ok;
}
