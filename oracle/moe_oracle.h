/* moe_oracle.h -- TEST INFRASTRUCTURE ONLY: the CPU checker for librbt_moe.so.
 * Restates the MoE feed-forward of rabbit2/src/rabbit2.c:511-542. */
#ifndef RBT_MOE_ORACLE_H
#define RBT_MOE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#define ORC_DT_F32 0
#define ORC_DT_BF16 1
#define ORC_MAX_TOPK 64 /* rabbit2.c:59 */

typedef struct {
    int D, H, E, K;          /* Config.dim, expert_hidden, n_experts, top_k */
    int dtype;               /* Config.dtype: 0 f32, 1 bf16 (rabbit2.c:60-61) */
    int norm_topk;           /* Config.norm_topk */
    float rms_eps;           /* Config.rms_eps */
    const float *ffn_norm;   /* [D] f32, only for the block form */
    const void *router;      /* [E, D] dtype */
    const float *router_bias;/* [E] or NULL (workload extension, see moe_oracle.c) */
    const void *experts;     /* E blobs w1[H,D] | w3[H,D] | w2[D,H], expert_stride bytes apart */
    size_t expert_stride;
} OrcMoeLayer;

void orc_matvec(float *out, const void *W, int dtype, const float *x, int rows, int cols);
void orc_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
void orc_softmax(float *x, int n);
int orc_moe_ffn(const OrcMoeLayer *L, const float *xb, int T, float *moe_out, int32_t *routing, int routing_stride,
                float *weights, int nthreads);
int orc_moe_block(const OrcMoeLayer *L, const float *x, int T, float *x_out, int32_t *routing, int routing_stride,
                  int nthreads);
int orc_router_topk(const OrcMoeLayer *L, const float *xb, int T, int32_t *idx, float *wt, float *probs_out);
int orc_permute(const int32_t *idx, int T, int K, int E, int32_t *counts, int32_t *offsets, int32_t *perm);
int orc_router_logits(const OrcMoeLayer *L, const float *xb, int T, float *logits);
void orc_seq_sumsq(const float *x, int rows, int n, float *out);
int64_t orc_expf_mismatch(uint32_t first_bits, int64_t n, const float *got, int nthreads, int64_t *first_bad);
#endif
