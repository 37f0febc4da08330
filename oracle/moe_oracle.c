/*
 * moe_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C restatement of the RABBIT2 engine's MoE feed-forward, the path that
 * librbt_moe.so replaces on the GPU.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load this library.  Every function cites the
 * reference source it restates (rabbit2/src/rabbit2.c in Stanley03-arch/RABBITM2).
 *
 * Arithmetic policy (what makes routing bit-exact against the reference):
 *   - build with -ffp-contract=off: the reference is compiled by gcc -O2 for
 *     baseline x86-64, which has no FMA, so every product is rounded before it is
 *     added (rabbit2.c:325 states the same no-FMA policy for its AVX2 kernel);
 *   - the scalar matvec keeps four interleaved fp32 partial sums and combines
 *     them as (s0+s1)+(s2+s3) (rabbit2.c:364-373, :378-387);
 *   - softmax uses libm expf and a sequential sum (rabbit2.c:399-405).
 *
 * One extension the reference does not have: an optional additive router bias
 * b[e], applied to the router logits before the softmax.  It exists only to
 * build the skewed (Zipf) routing workloads; NULL means "no bias", which is the
 * reference behaviour exactly.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "moe_oracle.h"

static inline float orc_bf16(uint16_t h) {
    /* bf16 -> f32 widening by a 16-bit shift (rabbit2.c:304-309). */
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* out[r] = dot(W[r,:], x), W [rows, cols] row-major f32 or bf16.
 * Scalar order of rabbit2.c:357-390: four partial sums over i = 0,1,2,3 mod 4,
 * the tail (cols % 4) folded into s0, result (s0+s1)+(s2+s3). */
void orc_matvec(float *out, const void *W, int dtype, const float *x, int rows, int cols) {
    for (int r = 0; r < rows; r++) {
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        int i = 0;
        if (dtype == ORC_DT_F32) {
            const float *w = (const float *)W + (size_t)r * cols;
            for (; i + 3 < cols; i += 4) {
                s0 += w[i] * x[i];
                s1 += w[i + 1] * x[i + 1];
                s2 += w[i + 2] * x[i + 2];
                s3 += w[i + 3] * x[i + 3];
            }
            for (; i < cols; i++) s0 += w[i] * x[i];
        } else {
            const uint16_t *w = (const uint16_t *)W + (size_t)r * cols;
            for (; i + 3 < cols; i += 4) {
                s0 += orc_bf16(w[i]) * x[i];
                s1 += orc_bf16(w[i + 1]) * x[i + 1];
                s2 += orc_bf16(w[i + 2]) * x[i + 2];
                s3 += orc_bf16(w[i + 3]) * x[i + 3];
            }
            for (; i < cols; i++) s0 += orc_bf16(w[i]) * x[i];
        }
        out[r] = (s0 + s1) + (s2 + s3);
    }
}

/* RMSNorm of rabbit2.c:392-397: sequential sum of squares, 1/sqrtf, then (x*inv)*w. */
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

/* In-place softmax of rabbit2.c:399-405: max-subtract, expf, sequential sum, divide. */
void orc_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* silu of rabbit2.c:407. */
static float orc_silu(float v) { return v / (1.0f + expf(-v)); }

/* Router + softmax + greedy top-k for one token (rabbit2.c:513-528).
 * probs: scratch [E].  idx/wt: [K] in selection order (descending prob, lowest
 * index first among equal probs: strict '>' at rabbit2.c:522).  Returns wsum. */
static float orc_route_one(const OrcMoeLayer *L, const float *xb, float *probs, unsigned char *used,
                           int32_t *idx, float *wt) {
    orc_matvec(probs, L->router, L->dtype, xb, L->E, L->D);
    if (L->router_bias)
        for (int e = 0; e < L->E; e++) probs[e] += L->router_bias[e];
    orc_softmax(probs, L->E);
    memset(used, 0, (size_t)L->E);
    float wsum = 0.0f;
    for (int k = 0; k < L->K; k++) {
        int best = -1;
        for (int e = 0; e < L->E; e++)
            if (!used[e] && (best < 0 || probs[e] > probs[best])) best = e;
        used[best] = 1;
        idx[k] = best;
        wt[k] = probs[best];
        wsum += wt[k];
    }
    return wsum;
}

/* One token of the MoE FFN: rabbit2.c:513-541 (moe[] starts at zero, experts
 * are applied in selection order, moe += wk * (W2 . (silu(W1 x) * (W3 x)))). */
static void orc_ffn_one(const OrcMoeLayer *L, const float *xb, float *moe, int32_t *route_out, float *wt_out,
                        float *scratch, unsigned char *used) {
    const int D = L->D, H = L->H, K = L->K;
    float *probs = scratch;             /* [E] */
    float *h1 = probs + L->E;           /* [H] */
    float *h3 = h1 + H;                 /* [H] */
    float *tmp = h3 + H;                /* [D] */
    int32_t idx[ORC_MAX_TOPK];
    float wt[ORC_MAX_TOPK];
    const float wsum = orc_route_one(L, xb, probs, used, idx, wt);
    const size_t esz = L->dtype == ORC_DT_BF16 ? 2 : 4;
    const size_t mat_bytes = (size_t)H * D * esz;
    memset(moe, 0, (size_t)D * sizeof(float));
    for (int k = 0; k < K; k++) {
        const unsigned char *eb = (const unsigned char *)L->experts + (size_t)idx[k] * L->expert_stride;
        orc_matvec(h1, eb, L->dtype, xb, H, D);                 /* w1 (gate) */
        orc_matvec(h3, eb + mat_bytes, L->dtype, xb, H, D);     /* w3 (up)   */
        for (int i = 0; i < H; i++) h1[i] = orc_silu(h1[i]) * h3[i];
        orc_matvec(tmp, eb + 2 * mat_bytes, L->dtype, h1, D, H); /* w2 (down) */
        const float wk = L->norm_topk ? wt[k] / wsum : wt[k];
        for (int i = 0; i < D; i++) moe[i] += wk * tmp[i];
        if (route_out) route_out[k] = idx[k];
        if (wt_out) wt_out[k] = wk;
    }
}

typedef struct {
    const OrcMoeLayer *L;
    const float *x;       /* [T, D] */
    float *out;           /* [T, D] */
    int32_t *routing;     /* [T, routing_stride] or NULL */
    int routing_stride;
    float *weights;       /* [T, K] or NULL */
    int block;            /* 1: x is the residual stream, out = x + moe(rmsnorm(x)) */
    int t0, t1;
    int ok;
} OrcJob;

static void *orc_worker(void *arg) {
    OrcJob *j = (OrcJob *)arg;
    const OrcMoeLayer *L = j->L;
    const int D = L->D;
    float *scratch = (float *)malloc(sizeof(float) * ((size_t)L->E + 2 * (size_t)L->H + 2 * (size_t)D));
    unsigned char *used = (unsigned char *)malloc((size_t)L->E);
    if (!scratch || !used) {
        free(scratch);
        free(used);
        j->ok = 0;
        return NULL;
    }
    float *xb = scratch + L->E + 2 * (size_t)L->H + D; /* [D] */
    for (int t = j->t0; t < j->t1; t++) {
        const float *xt = j->x + (size_t)t * D;
        float *ot = j->out + (size_t)t * D;
        int32_t *rt = j->routing ? j->routing + (size_t)t * j->routing_stride : NULL;
        float *wt = j->weights ? j->weights + (size_t)t * L->K : NULL;
        if (j->block) {
            /* rabbit2.c:512 then :542 (x += moe). */
            orc_rmsnorm(xb, xt, L->ffn_norm, D, L->rms_eps);
            orc_ffn_one(L, xb, ot, rt, wt, scratch, used);
            for (int i = 0; i < D; i++) ot[i] = xt[i] + ot[i];
        } else {
            orc_ffn_one(L, xt, ot, rt, wt, scratch, used);
        }
    }
    free(scratch);
    free(used);
    j->ok = 1;
    return NULL;
}

static int orc_run(const OrcMoeLayer *L, const float *x, int T, float *out, int32_t *routing, int routing_stride,
                   float *weights, int block, int nthreads) {
    if (!L || !x || !out || T < 0 || L->K < 1 || L->K > ORC_MAX_TOPK || L->K > L->E) return 0;
    if (block && !L->ffn_norm) return 0;
    if (routing_stride <= 0) routing_stride = L->K;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > T) nthreads = T > 0 ? T : 1;
    OrcJob *jobs = (OrcJob *)calloc((size_t)nthreads, sizeof(OrcJob));
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    if (!jobs || !th) {
        free(jobs);
        free(th);
        return 0;
    }
    for (int i = 0; i < nthreads; i++) {
        jobs[i] = (OrcJob){L, x, out, routing, routing_stride, weights, block,
                           (int)((long)T * i / nthreads), (int)((long)T * (i + 1) / nthreads), 0};
    }
    int ok = 1;
    if (nthreads == 1) {
        orc_worker(&jobs[0]);
        ok = jobs[0].ok;
    } else {
        for (int i = 0; i < nthreads; i++)
            if (pthread_create(&th[i], NULL, orc_worker, &jobs[i]) != 0) { jobs[i].ok = -1; }
        for (int i = 0; i < nthreads; i++) {
            if (jobs[i].ok == -1) { orc_worker(&jobs[i]); }
            else pthread_join(th[i], NULL);
            ok &= jobs[i].ok == 1;
        }
    }
    free(jobs);
    free(th);
    return ok;
}

int orc_moe_ffn(const OrcMoeLayer *L, const float *xb, int T, float *moe_out, int32_t *routing, int routing_stride,
                float *weights, int nthreads) {
    return orc_run(L, xb, T, moe_out, routing, routing_stride, weights, 0, nthreads);
}

int orc_moe_block(const OrcMoeLayer *L, const float *x, int T, float *x_out, int32_t *routing, int routing_stride,
                  int nthreads) {
    return orc_run(L, x, T, x_out, routing, routing_stride, NULL, 1, nthreads);
}

int orc_router_topk(const OrcMoeLayer *L, const float *xb, int T, int32_t *idx, float *wt, float *probs_out) {
    float *probs = (float *)malloc(sizeof(float) * (size_t)L->E);
    unsigned char *used = (unsigned char *)malloc((size_t)L->E);
    if (!probs || !used) {
        free(probs);
        free(used);
        return 0;
    }
    for (int t = 0; t < T; t++) {
        float w[ORC_MAX_TOPK];
        const float wsum = orc_route_one(L, xb + (size_t)t * L->D, probs, used, idx + (size_t)t * L->K, w);
        for (int k = 0; k < L->K; k++) wt[(size_t)t * L->K + k] = L->norm_topk ? w[k] / wsum : w[k];
        if (probs_out) memcpy(probs_out + (size_t)t * L->E, probs, sizeof(float) * (size_t)L->E);
    }
    free(probs);
    free(used);
    return 1;
}

/* Counting-sort permutation of the routed slots, the grouping the GPU kernels
 * build (the reference has none: it walks the k experts of one token in order). */
int orc_permute(const int32_t *idx, int T, int K, int E, int32_t *counts, int32_t *offsets, int32_t *perm) {
    memset(counts, 0, sizeof(int32_t) * (size_t)E);
    for (long s = 0; s < (long)T * K; s++) {
        if (idx[s] < 0 || idx[s] >= E) return 0;
        counts[idx[s]]++;
    }
    offsets[0] = 0;
    for (int e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    int32_t *fill = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
    if (!fill) return 0;
    memcpy(fill, offsets, sizeof(int32_t) * (size_t)E);
    for (long s = 0; s < (long)T * K; s++) perm[fill[idx[s]]++] = (int32_t)s;
    free(fill);
    return 1;
}

/* Router logits for T tokens, [T, E]: the matvec of rabbit2.c:513 (plus the
 * optional bias), before the softmax. */
int orc_router_logits(const OrcMoeLayer *L, const float *xb, int T, float *logits) {
    for (int t = 0; t < T; t++) {
        float *lg = logits + (size_t)t * L->E;
        orc_matvec(lg, L->router, L->dtype, xb + (size_t)t * L->D, L->E, L->D);
        if (L->router_bias)
            for (int e = 0; e < L->E; e++) lg[e] += L->router_bias[e];
    }
    return 1;
}

/* out[r] = the sequential sum of x[r, i]^2, i = 0..n-1 (rmsnorm's ss, rabbit2.c:394). */
void orc_seq_sumsq(const float *x, int rows, int n, float *out) {
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (size_t)r * n;
        float ss = 0.0f;
        for (int i = 0; i < n; i++) ss += xr[i] * xr[i];
        out[r] = ss;
    }
}

/* Compare got[i] with libm expf(x_i), x_i the float with bit pattern first_bits + i
 * (the host's expf, the one rabbit2.c:403 calls).  Returns the number of
 * bit-level mismatches; *first_bad gets the first mismatching i (or -1). */
typedef struct {
    uint32_t first_bits;
    int64_t i0, i1;
    const float *got;
    int64_t bad, first;
} OrcExpfJob;

static void *orc_expf_worker(void *p) {
    OrcExpfJob *j = (OrcExpfJob *)p;
    j->bad = 0;
    j->first = -1;
    for (int64_t i = j->i0; i < j->i1; i++) {
        const uint32_t u = j->first_bits + (uint32_t)i;
        float x, y;
        memcpy(&x, &u, 4);
        y = expf(x);
        if (memcmp(&y, &j->got[i], 4) != 0) {
            if (j->first < 0) j->first = i;
            j->bad++;
        }
    }
    return NULL;
}

int64_t orc_expf_mismatch(uint32_t first_bits, int64_t n, const float *got, int nthreads, int64_t *first_bad) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    OrcExpfJob jobs[256];
    pthread_t th[256];
    for (int k = 0; k < nthreads; k++) {
        jobs[k].first_bits = first_bits;
        jobs[k].i0 = n * k / nthreads;
        jobs[k].i1 = n * (k + 1) / nthreads;
        jobs[k].got = got;
        pthread_create(&th[k], NULL, orc_expf_worker, &jobs[k]);
    }
    int64_t bad = 0, first = -1;
    for (int k = 0; k < nthreads; k++) {
        pthread_join(th[k], NULL);
        bad += jobs[k].bad;
        if (first < 0 && jobs[k].first >= 0) first = jobs[k].first;
    }
    if (first_bad) *first_bad = first;
    return bad;
}
