// model_prefill.cu -- the engine's forward() for a whole prompt at once
// (rbt_model_prefill): positions pos0 .. pos0 + T of one sequence, layer by layer,
// with every per-token matrix-vector product of forward() (rabbit2.c:455-550)
// turned into a GEMM over the T rows:
//
//   embed_rows             X[t] = tok_emb[tokens[t]]                        (:461-467)
//   per layer l:
//     norm_split           rmsnorm(X) rows, as bf16 hi + lo (or f32 rows)   (:473)
//     GEMM                 QKV = rows . [wq;wk;wv]^T                        (:474-476)
//     qk_rope_kv           whole-projection QK-norm, RoPE at pos0 + t,      (:477-486)
//                          k and v into the KV cache
//     attn_prefill         causal attention over cache positions <= pos0+t  (:487-506)
//     split + GEMM         X += AO . wo^T                                   (:507-508)
//     rbt_moe_block_device X += MoE(rmsnorm(X)), all T rows (tensor cores)  (:511-542)
//   norm_split + GEMM      logits of the last rows = rmsnorm(X) . lm_head^T (:545-546)
//
// The projections are dense GEMMs on the tensor cores (gemm_tc.cu: launch_tc_dense)
// and the attention a fused tcgen05 kernel (attn_tc.cu).  bf16 weights are exact
// in bf16; the f32 activation rows are split into bf16 hi = rn(x) and lo =
// rn(x - hi) (16 significant bits), and each product is two MMAs (hi and lo) with
// f32 accumulation into the same output -- the precision scheme of the MoE
// tensor-core path.  f32 models take CUDA-core forms of both.  The KV cache is
// the one the one-token forward uses, so decode continues from pos0 + T.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "../../include/rbt_moe.h"
#include "common.cuh"
#include "kernels.h"
#include "model_internal.h"

namespace rbt {
void set_last_error(const char* msg);
int moe_status_ok(RbtMoe* m);
}  // namespace rbt

namespace {

using namespace rbt;

int fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    fprintf(stderr, "rbt_model: %s\n", buf);
    set_last_error(buf);
    return 0;
}

#define CU(call)                                                                                  \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) return fail("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                           __FILE__, __LINE__);                                   \
    } while (0)

constexpr int kRowThreads = 256;
constexpr int kRowVec4 = 2;   // float4s per thread of a row: dim, n_heads*head_dim <= 2048
constexpr int kQB = 32;       // query rows per attention CTA
constexpr int kKT = 64;       // key positions per tile
constexpr int kAttnPThreads = 256;

// ---------------------------------------------------------------- row kernels
template <typename WT>
__global__ void embed_rows_kernel(const WT* emb, int D, const int32_t* tokens, float* x) {
    const int t = blockIdx.x;
    const size_t row = (size_t)tokens[t] * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) x[(size_t)t * D + i] = WeightTraits<WT>::load1(emb + row + i);
}

// the batched decode's rows: X[i] = tok_emb[steps[i].token]
template <typename WT>
__global__ void embed_steps_kernel(const WT* emb, int D, const Step* steps, float* x) {
    const int t = blockIdx.x;
    const size_t row = (size_t)steps[t].token * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) x[(size_t)t * D + i] = WeightTraits<WT>::load1(emb + row + i);
}

// Greedy id of each logits row as the engine's argmax (rabbit2.c:552-556): best
// starts at 0 and moves to i only when v[i] > v[best], so the first of equal
// maxima wins, NaNs never win, and a NaN at index 0 keeps 0.  Each thread scans
// its indices in ascending order; the block then reduces (value, index) pairs,
// the larger value first, the lower index among equals.
constexpr int kArgmaxThreads = 512;
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const float* logits, int vocab, int32_t* out) {
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    const float* v = logits + (size_t)blockIdx.x * vocab;
    float bv = -INFINITY;
    int bi = -1;  // no candidate yet (every value seen so far was NaN)
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float x = __ldg(v + i);
        if (x > bv || (bi < 0 && x == bv)) {
            bv = x;
            bi = i;
        }
    }
    auto better = [](float av, int ai, float cv, int ci) {  // is (cv, ci) ahead of (av, ai)?
        if (ci < 0) return false;
        if (ai < 0) return true;
        return cv > av || (cv == av && ci < ai);
    };
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL_MASK, bv, o);
        const int oi = __shfl_xor_sync(FULL_MASK, bi, o);
        if (better(bv, bi, ov, oi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; w++)
            if (better(bv, bi, sv[w], si[w])) {
                bv = sv[w];
                bi = si[w];
            }
        out[blockIdx.x] = (bi < 0 || isnan(__ldg(v))) ? 0 : bi;
    }
}

// Row t of x (n floats, row stride ld_in): rmsnorm with weights w (or none), then
// either f32 rows (xf) or bf16 hi/lo rows (hi, lo), row stride ld_out.
// The sum of squares is in a fixed order; (x * inv) * w as rmsnorm() rounds it.
__global__ void __launch_bounds__(kRowThreads) norm_split_kernel(const float* x, int ld_in, int n, const float* w,
                                                                 float eps, int ld_out, float* xf, uint16_t* hi,
                                                                 uint16_t* lo) {
    __shared__ float red[kRowThreads / 32];
    const int t = blockIdx.x, tid = threadIdx.x, n4 = n / 4;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * ld_in);
    float4 v[kRowVec4];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < kRowVec4; k++) {
        const int i4 = tid + k * kRowThreads;
        if (i4 < n4) {
            v[k] = xr[i4];
            ss = fmaf(v[k].x, v[k].x, ss);
            ss = fmaf(v[k].y, v[k].y, ss);
            ss = fmaf(v[k].z, v[k].z, ss);
            ss = fmaf(v[k].w, v[k].w, ss);
        }
    }
    float inv = 1.0f;
    if (w) {
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int i = 0; i < kRowThreads / 32; i++) tot += red[i];
        inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, (float)n), eps));
    }
#pragma unroll
    for (int k = 0; k < kRowVec4; k++) {
        const int i4 = tid + k * kRowThreads;
        if (i4 >= n4) continue;
        float e[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        if (w) {
            const float4 wv = reinterpret_cast<const float4*>(w)[i4];
            const float ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int q = 0; q < 4; q++) e[q] = __fmul_rn(__fmul_rn(e[q], inv), ww[q]);
        }
        const size_t o = (size_t)t * ld_out + 4 * (size_t)i4;
        if (xf) {
            *reinterpret_cast<float4*>(xf + o) = make_float4(e[0], e[1], e[2], e[3]);
        } else {  // four bf16 hi and four lo as one 8-byte store each
            uint32_t hw[2], lw[2];
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const __nv_bfloat16 h0 = __float2bfloat16_rn(e[2 * q]), h1 = __float2bfloat16_rn(e[2 * q + 1]);
                const __nv_bfloat16 l0 = __float2bfloat16_rn(e[2 * q] - __bfloat162float(h0));
                const __nv_bfloat16 l1 = __float2bfloat16_rn(e[2 * q + 1] - __bfloat162float(h1));
                hw[q] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
                lw[q] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
            }
            *reinterpret_cast<uint2*>(hi + o) = make_uint2(hw[0], hw[1]);
            *reinterpret_cast<uint2*>(lo + o) = make_uint2(lw[0], lw[1]);
        }
    }
}

// Row t of q|k|v: QK-norm over the whole q and k projections (rabbit2.c:477-480),
// RoPE at position pos0 + t (:481-482, the engine's angle table), q written back
// in place, k and v stored in the head-major KV cache (:484-486).
__global__ void __launch_bounds__(kRowThreads) qk_rope_kv_kernel(float* qkv, int nq, int nkv, int hd,
                                                                 const float* q_norm, const float* k_norm, float eps,
                                                                 const float* rope_cos, const float* rope_sin,
                                                                 int pos0, float* kc, float* vc, int ctx) {
    __shared__ float red[kRowThreads / 32], red2[kRowThreads / 32];
    const int t = blockIdx.x, tid = threadIdx.x, pos = pos0 + t, half = hd / 2;
    float* row = qkv + (size_t)t * (nq + 2 * nkv);
    float inv_q = 1.0f, inv_k = 1.0f;
    if (q_norm) {
        float sq = 0.0f, sk = 0.0f;
        for (int i = tid; i < nq; i += kRowThreads) sq = fmaf(row[i], row[i], sq);
        for (int i = tid; i < nkv; i += kRowThreads) sk = fmaf(row[nq + i], row[nq + i], sk);
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        if ((tid & 31) == 0) {
            red[tid >> 5] = sq;
            red2[tid >> 5] = sk;
        }
        __syncthreads();
        float tq = 0.0f, tk = 0.0f;
        for (int i = 0; i < kRowThreads / 32; i++) {
            tq += red[i];
            tk += red2[i];
        }
        inv_q = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tq, (float)nq), eps));
        inv_k = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tk, (float)nkv), eps));
    }
    const float* cs = rope_cos + (size_t)pos * half;
    const float* sn = rope_sin + (size_t)pos * half;
    // (i, i + half) pairs of every head, two adjacent i per thread (8-byte accesses;
    // head_dim is a multiple of 4)
    const int hh = half / 2, nqp = nq / 4, nkp = nkv / 4;
    for (int j = tid; j < nqp + nkp; j += kRowThreads) {
        const bool is_q = j < nqp;
        const int jj = is_q ? j : j - nqp, h = jj / hh, i = (jj % hh) * 2;
        float* p = row + (is_q ? 0 : nq) + (size_t)h * hd;
        const float2 a2 = *reinterpret_cast<const float2*>(p + i), b2 = *reinterpret_cast<const float2*>(p + i + half);
        const float2 c2 = *reinterpret_cast<const float2*>(cs + i), s2 = *reinterpret_cast<const float2*>(sn + i);
        float a[2] = {a2.x, a2.y}, b[2] = {b2.x, b2.y};
        const float cc[2] = {c2.x, c2.y}, ss[2] = {s2.x, s2.y};
        const float* w = is_q ? q_norm : k_norm;
        float ra[2], rb[2];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            if (w) {
                const float inv = is_q ? inv_q : inv_k;
                a[u] = __fmul_rn(__fmul_rn(a[u], inv), w[(size_t)h * hd + i + u]);
                b[u] = __fmul_rn(__fmul_rn(b[u], inv), w[(size_t)h * hd + i + u + half]);
            }
            ra[u] = __fsub_rn(__fmul_rn(a[u], cc[u]), __fmul_rn(b[u], ss[u]));
            rb[u] = __fadd_rn(__fmul_rn(b[u], cc[u]), __fmul_rn(a[u], ss[u]));
        }
        float* dst = is_q ? p : kc + ((size_t)h * ctx + pos) * hd;
        *reinterpret_cast<float2*>(dst + i) = make_float2(ra[0], ra[1]);
        *reinterpret_cast<float2*>(dst + i + half) = make_float2(rb[0], rb[1]);
    }
    for (int j = tid; j < nkv / 4; j += kRowThreads) {  // v rows into the cache, 16 bytes at a time
        const int h = (4 * j) / hd, i = (4 * j) % hd;
        *reinterpret_cast<float4*>(vc + ((size_t)h * ctx + pos) * hd + i) =
            *reinterpret_cast<const float4*>(row + nq + nkv + 4 * j);
    }
}

// ---------------------------------------------------------------- causal attention
// CTA (head h, block of kQB query rows): the rows' attention over cache positions
// 0 .. pos0 + t (rabbit2.c:487-506) with an online softmax over tiles of kKT
// positions in shared memory: scores = q . k * scale, running max and sum, and
// the exp-weighted V sum, divided by the sum at the end.  Thread (r = tid / 8,
// g = tid % 8) owns score columns g + 8 j and output dims 4 (g + 8 k) .. + 4 of
// query row r.
template <int HD>
__global__ void __launch_bounds__(kAttnPThreads) attn_prefill_kernel(const float* qkv, int nq, int nkv, int n_heads,
                                                                     int n_kv_heads, const float* kc, const float* vc,
                                                                     int ctx, int pos0, int T, float scale,
                                                                     float* ao) {
    constexpr int LD = HD + 4;  // padded rows: the 8 column groups of a warp hit different banks
    constexpr int DV = HD / 32;  // float4s of output per thread
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                    // [kQB][LD]
    float* Ks = Qs + kQB * LD;         // [kKT][LD]
    float* Vs = Ks + kKT * LD;         // [kKT][LD]
    float* Ps = Vs + kKT * LD;         // [kQB][kKT]
    const int h = blockIdx.x, tb = blockIdx.y, tid = threadIdx.x;
    const int r = tid >> 3, g = tid & 7;
    const int t0 = tb * kQB, nrow = min(kQB, T - t0);
    const int kvh = h / (n_heads / n_kv_heads);
    const int row_stride = nq + 2 * nkv;
    for (int e = tid; e < kQB * (HD / 4); e += kAttnPThreads) {
        const int rr = e / (HD / 4), c4 = e % (HD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rr < nrow) v = reinterpret_cast<const float4*>(qkv + (size_t)(t0 + rr) * row_stride + (size_t)h * HD)[c4];
        *reinterpret_cast<float4*>(Qs + rr * LD + 4 * c4) = v;
    }
    const int my_t = t0 + r, my_pos = pos0 + my_t;  // this thread's query row and its position
    const int last = pos0 + t0 + nrow - 1;            // the block's last position
    float m_run = -INFINITY, l_run = 0.0f;
    float4 o[DV];
#pragma unroll
    for (int k = 0; k < DV; k++) o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* kb = kc + (size_t)kvh * ctx * HD;
    const float* vb = vc + (size_t)kvh * ctx * HD;
    for (int p0 = 0; p0 <= last; p0 += kKT) {
        __syncthreads();  // the previous tile is consumed (and Qs written, on the first pass)
        const int np = min(kKT, last + 1 - p0);
        for (int e = tid; e < kKT * (HD / 4); e += kAttnPThreads) {
            const int rr = e / (HD / 4), c4 = e % (HD / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (rr < np) {
                kv = reinterpret_cast<const float4*>(kb + (size_t)(p0 + rr) * HD)[c4];
                vv = reinterpret_cast<const float4*>(vb + (size_t)(p0 + rr) * HD)[c4];
            }
            *reinterpret_cast<float4*>(Ks + rr * LD + 4 * c4) = kv;
            *reinterpret_cast<float4*>(Vs + rr * LD + 4 * c4) = vv;
        }
        __syncthreads();
        // q . k for the thread's 8 columns: 16-byte loads, 8 independent accumulators
        float s[kKT / 8];
#pragma unroll
        for (int j = 0; j < kKT / 8; j++) s[j] = 0.0f;
#pragma unroll 4
        for (int i4 = 0; i4 < HD / 4; i4++) {
            const float4 q4 = *reinterpret_cast<const float4*>(Qs + r * LD + 4 * i4);
#pragma unroll
            for (int j = 0; j < kKT / 8; j++) {
                const float4 k4 = *reinterpret_cast<const float4*>(Ks + (g + 8 * j) * LD + 4 * i4);
                s[j] = fmaf(q4.x, k4.x, s[j]);
                s[j] = fmaf(q4.y, k4.y, s[j]);
                s[j] = fmaf(q4.z, k4.z, s[j]);
                s[j] = fmaf(q4.w, k4.w, s[j]);
            }
        }
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < kKT / 8; j++) {
            const int c = g + 8 * j, p = p0 + c;
            s[j] = (c < np && p <= my_pos && r < nrow) ? s[j] * scale : -INFINITY;
            tmax = fmaxf(tmax, s[j]);
        }
        // the row's 8 threads are adjacent lanes
        tmax = fmaxf(tmax, __shfl_xor_sync(FULL_MASK, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(FULL_MASK, tmax, 2));
        tmax = fmaxf(tmax, __shfl_xor_sync(FULL_MASK, tmax, 4));
        const float m_new = fmaxf(m_run, tmax);
        const float alpha = m_new == -INFINITY ? 1.0f : expf(m_run - m_new);
        float psum = 0.0f;
#pragma unroll
        for (int j = 0; j < kKT / 8; j++) {
            const float pv = s[j] == -INFINITY ? 0.0f : expf(s[j] - m_new);
            Ps[r * kKT + g + 8 * j] = pv;
            psum += pv;
        }
        psum += __shfl_xor_sync(FULL_MASK, psum, 1);
        psum += __shfl_xor_sync(FULL_MASK, psum, 2);
        psum += __shfl_xor_sync(FULL_MASK, psum, 4);
        l_run = l_run * alpha + psum;
        m_run = m_new;
        __syncwarp();
#pragma unroll
        for (int k = 0; k < DV; k++) {
            o[k].x *= alpha;
            o[k].y *= alpha;
            o[k].z *= alpha;
            o[k].w *= alpha;
        }
        for (int c = 0; c < np; c++) {
            const float pv = Ps[r * kKT + c];
#pragma unroll
            for (int k = 0; k < DV; k++) {
                const float4 vv = *reinterpret_cast<const float4*>(Vs + c * LD + 4 * (g + 8 * k));
                o[k].x = fmaf(pv, vv.x, o[k].x);
                o[k].y = fmaf(pv, vv.y, o[k].y);
                o[k].z = fmaf(pv, vv.z, o[k].z);
                o[k].w = fmaf(pv, vv.w, o[k].w);
            }
        }
    }
    if (r < nrow) {
        float* out = ao + (size_t)my_t * nq + (size_t)h * HD;
#pragma unroll
        for (int k = 0; k < DV; k++)
            *reinterpret_cast<float4*>(out + 4 * (g + 8 * k)) =
                make_float4(o[k].x / l_run, o[k].y / l_run, o[k].z / l_run, o[k].w / l_run);
    }
}

size_t attn_prefill_smem(int hd) { return (size_t)((kQB + 2 * kKT) * (hd + 4) + kQB * kKT) * sizeof(float); }

cudaError_t launch_attn_prefill(int hd, dim3 grid, cudaStream_t s, const float* qkv, int nq, int nkv, int n_heads,
                                int n_kv_heads, const float* kc, const float* vc, int ctx, int pos0, int T,
                                float scale, float* ao) {
    const size_t smem = attn_prefill_smem(hd);
    switch (hd) {
#define RBT_ATTN_CASE(HDV)                                                                                      \
    case HDV: {                                                                                                 \
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel<HDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                             (int)smem);                                                        \
        if (e != cudaSuccess) return e;                                                                         \
        attn_prefill_kernel<HDV><<<grid, kAttnPThreads, smem, s>>>(qkv, nq, nkv, n_heads, n_kv_heads, kc, vc,   \
                                                                   ctx, pos0, T, scale, ao);                    \
        return cudaGetLastError();                                                                              \
    }
        RBT_ATTN_CASE(64)
        RBT_ATTN_CASE(128)
#undef RBT_ATTN_CASE
        default:
            return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------- GEMMs
// out[T, N] (row pitch ldc) (+)= rows[T, K] . W[N, K]^T on the CUDA cores: f32
// weights, and bf16 shapes the tensor-core tiles do not cover (N % 128, K % 64).
// The rows are the f32 rows (f32 models) or hi + lo (bf16 models, the values the
// tensor-core form multiplies).  Each output is one f32 FMA chain in ascending k.
constexpr int kPjTile = 64;   // outputs per CTA along N and along T
constexpr int kPjK = 16;      // K elements per shared-memory stage
template <typename WT>
__global__ void __launch_bounds__(256) proj_rows_kernel(const WT* __restrict__ W, int N, int K,
                                                        const float* __restrict__ xf, const uint16_t* __restrict__ xhi,
                                                        const uint16_t* __restrict__ xlo, int ld_in, int T,
                                                        float* out, int ldc, int accumulate) {
    __shared__ float ws[kPjK][kPjTile + 1];
    __shared__ float xs[kPjK][kPjTile + 1];
    const int n0 = blockIdx.x * kPjTile, t0 = blockIdx.y * kPjTile;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // outputs n0 + tx + 16 i, t0 + ty + 16 j
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += kPjK) {
        for (int i = threadIdx.x; i < kPjK * kPjTile; i += 256) {
            const int r = i / kPjK, kk = i - r * kPjK, k = k0 + kk;
            const int n = n0 + r, t = t0 + r;
            ws[kk][r] = (n < N && k < K) ? WeightTraits<WT>::load1(W + (size_t)n * K + k) : 0.0f;
            float v = 0.0f;
            if (t < T && k < K) {
                const size_t o = (size_t)t * ld_in + k;
                v = xf ? xf[o] : __uint_as_float((uint32_t)xhi[o] << 16) + __uint_as_float((uint32_t)xlo[o] << 16);
            }
            xs[kk][r] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kPjK; kk++) {
            float wv[4], xv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) wv[i] = ws[kk][tx + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; j++) xv[j] = xs[kk][ty + 16 * j];
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int i = 0; i < 4; i++) acc[j][i] = fmaf(xv[j], wv[i], acc[j][i]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int t = t0 + ty + 16 * j;
        if (t >= T) continue;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int n = n0 + tx + 16 * i;
            if (n >= N) continue;
            float* o = out + (size_t)t * ldc + n;
            *o = accumulate ? *o + acc[j][i] : acc[j][i];
        }
    }
}

// out[T, N] (row pitch ldc) (+)= rows[T, K] . W[N, K]^T.  bf16 models: the
// tensor-core GEMM over the hi and lo rows (two MMAs per K step into one f32
// accumulator); f32 models and untiled shapes: the CUDA-core kernel above.
int proj(RbtModel* m, const void* W, int N, int K, int T, int ld_in, float* out, int ldc, bool accumulate) {
    if (T <= 0) return 1;
    cudaStream_t s = m->stream;
    if (m->cfg.dtype == RBT_MOE_DT_BF16) {
        const size_t need = tc_dense_part_bytes(N, K, T, m->sm_count);
        if (need > m->proj_part_bytes) {  // split-K scratch, grown on demand
            cudaFree(m->proj_part);
            m->proj_part = nullptr;
            m->proj_part_bytes = 0;
            CU(cudaMalloc((void**)&m->proj_part, need));
            m->proj_part_bytes = need;
        }
        const cudaError_t e = launch_tc_dense(W, N, K, m->pf.hi, m->pf.lo, ld_in, T, out, ldc, accumulate, m->status,
                                              m->proj_part, m->proj_part_bytes, m->sm_count, s);
        if (e == cudaSuccess) return 1;
        if (e != cudaErrorNotSupported) return fail("tensor-core projection: %s", cudaGetErrorString(e));
    }
    const dim3 grid((N + kPjTile - 1) / kPjTile, (T + kPjTile - 1) / kPjTile);
    if (m->cfg.dtype == RBT_MOE_DT_BF16)
        proj_rows_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(W), N, K, nullptr,
                                                         static_cast<const uint16_t*>(m->pf.hi),
                                                         static_cast<const uint16_t*>(m->pf.lo), ld_in, T, out, ldc,
                                                         accumulate);
    else
        proj_rows_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(W), N, K, m->pf.xf, nullptr, nullptr,
                                                      ld_in, T, out, ldc, accumulate);
    CU(cudaGetLastError());
    return 1;
}

// Attention of T query rows (q in the qkv rows, after RoPE) over cache positions
// [0, pos0 + T) into ao [T, nq], bf16 models: the tensor-core kernel of attn_tc.cu
// (S = Q K^T and O = P V as bf16 hi/lo MMAs, an exact two-pass softmax).
int attn_tensor(RbtModel* m, int T, int pos0, const float* kc, const float* vc) {
    const RbtModelConfig& c = m->cfg;
    const int nq = c.n_heads * c.head_dim, nqkv = nq + 2 * c.n_kv_heads * c.head_dim;
    CU(launch_attn_tc(m->pf.qkv, nqkv, c.n_heads, c.n_kv_heads, c.head_dim, kc, vc, m->ctx, pos0, T, m->pf.att,
                      m->pf.att_bytes, m->pf.ao, m->status, m->stream));
    return 1;
}

size_t attn_tensor_bytes(const RbtModelConfig& c, int T, int nk) {
    return attn_tc_scratch_bytes(T, c.n_heads * c.head_dim, c.n_kv_heads, c.head_dim, nk);
}

// the GEMM input rows: rmsnorm(src rows) with w, or src rows as they are (w == nullptr)
int split_rows(RbtModel* m, const float* src, int ld_src, int n, int rows, const float* w, int ld_out) {
    const bool bf = m->cfg.dtype == RBT_MOE_DT_BF16;
    norm_split_kernel<<<rows, kRowThreads, 0, m->stream>>>(src, ld_src, n, w, m->cfg.rms_eps, ld_out,
                                                          bf ? nullptr : m->pf.xf,
                                                          bf ? static_cast<uint16_t*>(m->pf.hi) : nullptr,
                                                          bf ? static_cast<uint16_t*>(m->pf.lo) : nullptr);
    CU(cudaGetLastError());
    return 1;
}

int nq_of(const RbtModelConfig& c) { return c.n_heads * c.head_dim; }
int nkv_of(const RbtModelConfig& c) { return c.n_kv_heads * c.head_dim; }

int reserve(RbtModel* m, int T, int pos0, int logit_rows) {
    const RbtModelConfig& c = m->cfg;
    PrefillBufs& b = m->pf;
    if (T > b.cap) {
        void* old[] = {b.tokens, b.x, b.qkv, b.ao, b.xf, b.hi, b.lo, b.routing};
        for (void* p : old) cudaFree(p);
        // capacity 0 until every buffer exists: a failed allocation leaves nothing to reuse
        b = PrefillBufs{0,       nullptr,  nullptr,     nullptr,     nullptr, nullptr, nullptr,
                        nullptr, nullptr,  b.logit_rows, b.logits, b.att_bytes, b.att};
        const size_t wide = (size_t)(c.dim > nq_of(c) ? c.dim : nq_of(c));
        const size_t rows = (size_t)T;
        CU(cudaMalloc((void**)&b.tokens, rows * 4));
        CU(cudaMalloc((void**)&b.x, rows * c.dim * 4));
        CU(cudaMalloc((void**)&b.qkv, rows * (nq_of(c) + 2 * nkv_of(c)) * 4));
        CU(cudaMalloc((void**)&b.ao, rows * nq_of(c) * 4));
        if (c.dtype == RBT_MOE_DT_BF16) {
            CU(cudaMalloc(&b.hi, rows * wide * 2));
            CU(cudaMalloc(&b.lo, rows * wide * 2));
        } else {
            CU(cudaMalloc((void**)&b.xf, rows * wide * 4));
        }
        CU(cudaMalloc((void**)&b.routing, rows * c.n_layers * c.top_k * 4));
        b.cap = T;
    }
    if (c.dtype == RBT_MOE_DT_BF16) {
        const size_t need = attn_tensor_bytes(c, T, pos0 + T);
        if (need > b.att_bytes) {
            cudaFree(b.att);
            b.att = nullptr;
            b.att_bytes = 0;
            CU(cudaMalloc(&b.att, need));
            b.att_bytes = need;
        }
    }
    if (logit_rows > b.logit_rows) {
        cudaFree(b.logits);
        b.logits = nullptr;
        b.logit_rows = 0;
        CU(cudaMalloc((void**)&b.logits, (size_t)logit_rows * c.vocab * 4));
        b.logit_rows = logit_rows;
    }
    if (!rbt_moe_reserve(m->moe, model_moe_rows(m, T))) return 0;
    return 1;
}

// The batched decode's per-row buffers for n rows: steps, attention partials and
// split counters (zero between calls), greedy ids, pinned staging of the steps.
int reserve_decode(RbtModel* m, int n) {
    if (n <= m->dcap) return 1;
    const RbtModelConfig& c = m->cfg;
    cudaFree(m->steps);
    cudaFree(m->dpart);
    cudaFree(m->ddone);
    cudaFree(m->dnext);
    cudaFreeHost(m->h_steps);
    m->steps = nullptr;
    m->dpart = nullptr;
    m->ddone = nullptr;
    m->dnext = nullptr;
    m->h_steps = nullptr;
    m->dcap = 0;
    CU(cudaMalloc((void**)&m->steps, (size_t)n * sizeof(Step)));
    CU(cudaMalloc((void**)&m->dpart, (size_t)n * c.n_heads * m->n_splits * (c.head_dim + 2) * 4));
    CU(cudaMalloc((void**)&m->ddone, (size_t)n * c.n_heads * 4));
    CU(cudaMalloc((void**)&m->dnext, (size_t)n * 4));
    CU(cudaMallocHost((void**)&m->h_steps, (size_t)n * sizeof(Step)));
    CU(cudaMemset(m->ddone, 0, (size_t)n * c.n_heads * 4));
    m->dcap = n;
    return 1;
}

template <typename WT>
int run_prefill(RbtModel* m, int seq, int T, int pos0, int logit_rows) {
    const RbtModelConfig& c = m->cfg;
    const int D = c.dim, nq = nq_of(c), nkv = nkv_of(c), nqkv = nq + 2 * nkv, L = c.n_layers, K = c.top_k;
    const int wide = D > nq ? D : nq;
    cudaStream_t s = m->stream;
    PrefillBufs& b = m->pf;
    embed_rows_kernel<WT><<<T, 256, 0, s>>>(static_cast<const WT*>(m->tok_emb), D, b.tokens, b.x);
    CU(cudaGetLastError());
    const dim3 agrid(c.n_heads, (T + kQB - 1) / kQB);
    for (int l = 0; l < L; l++) {
        const RbtModel::Layer& Ly = m->layers[l];
        if (!split_rows(m, b.x, D, D, T, Ly.attn_norm, wide)) return 0;
        if (!proj(m, Ly.wqkv, nqkv, D, T, wide, b.qkv, nqkv, false)) return 0;
        float* kc = m->kc + ((size_t)seq * L + l) * m->ctx * nkv;
        float* vc = m->vc + ((size_t)seq * L + l) * m->ctx * nkv;
        qk_rope_kv_kernel<<<T, kRowThreads, 0, s>>>(b.qkv, nq, nkv, c.head_dim, c.qk_norm ? Ly.q_norm : nullptr,
                                                   c.qk_norm ? Ly.k_norm : nullptr, c.rms_eps, m->rope_cos,
                                                   m->rope_sin, pos0, kc, vc, m->ctx);
        CU(cudaGetLastError());
        if (c.dtype == RBT_MOE_DT_BF16) {
            if (!attn_tensor(m, T, pos0, kc, vc)) return 0;
        } else {
            CU(launch_attn_prefill(c.head_dim, agrid, s, b.qkv, nq, nkv, c.n_heads, c.n_kv_heads, kc, vc, m->ctx, pos0,
                                   T, 1.0f / sqrtf((float)c.head_dim), b.ao));
        }
        if (!split_rows(m, b.ao, nq, nq, T, nullptr, wide)) return 0;
        if (!proj(m, Ly.wo, D, nq, T, wide, b.x, D, true)) return 0;
        if (!model_moe_block(m, l, b.x, T, b.routing + (size_t)l * K, L * K, s)) return 0;
    }
    if (logit_rows > 0) {
        const float* last = b.x + (size_t)(T - logit_rows) * D;
        if (!split_rows(m, last, D, D, logit_rows, m->final_norm, wide)) return 0;
        if (!proj(m, m->lm_head, c.vocab, D, logit_rows, wide, b.logits, c.vocab, false)) return 0;
    }
    return 1;
}

// One decode step of n sequences (rbt_model_decode_batch): row i is the token of
// sequence i at its own position.  forward() for every row at once: the
// projections as GEMMs over the n rows (as in the prompt), the attention of each
// row over its own sequence's cache (the one-token kernel, one grid slice per row),
// the MoE block over the n rows, and the logits rows.
template <typename WT>
int run_decode(RbtModel* m, int n, bool want_logits) {
    const RbtModelConfig& c = m->cfg;
    const int D = c.dim, nq = nq_of(c), nkv = nkv_of(c), nqkv = nq + 2 * nkv, L = c.n_layers, K = c.top_k;
    const int wide = D > nq ? D : nq;
    cudaStream_t s = m->stream;
    PrefillBufs& b = m->pf;
    embed_steps_kernel<WT><<<n, 256, 0, s>>>(static_cast<const WT*>(m->tok_emb), D, m->steps, b.x);
    CU(cudaGetLastError());
    for (int l = 0; l < L; l++) {
        const RbtModel::Layer& Ly = m->layers[l];
        if (!split_rows(m, b.x, D, D, n, Ly.attn_norm, wide)) return 0;
        if (!proj(m, Ly.wqkv, nqkv, D, n, wide, b.qkv, nqkv, false)) return 0;
        CU(launch_attn_decode_rows(m, l, m->steps, b.qkv, n, b.ao, m->dpart, m->ddone, s));
        if (!split_rows(m, b.ao, nq, nq, n, nullptr, wide)) return 0;
        if (!proj(m, Ly.wo, D, nq, n, wide, b.x, D, true)) return 0;
        if (!model_moe_block(m, l, b.x, n, b.routing + (size_t)l * K, L * K, s)) return 0;
    }
    if (want_logits) {
        if (!split_rows(m, b.x, D, D, n, m->final_norm, wide)) return 0;
        if (!proj(m, m->lm_head, c.vocab, D, n, wide, b.logits, c.vocab, false)) return 0;
        argmax_rows_kernel<<<n, kArgmaxThreads, 0, s>>>(b.logits, c.vocab, m->dnext);
        CU(cudaGetLastError());
    }
    return 1;
}

// the checks every whole-prompt or batched call makes before it runs
int check_ready(RbtModel* m) {
    const RbtModelConfig& c = m->cfg;
    if (!m->globals) return fail("globals not loaded (rbt_model_load_globals)");
    for (int l = 0; l < c.n_layers; l++)
        if (!m->layers[l].loaded) return fail("layer %d not loaded (rbt_model_load_layer)", l);
    return 1;
}

}  // namespace

namespace rbt {
void prefill_free(RbtModel* m) {
    PrefillBufs& b = m->pf;
    void* bufs[] = {b.tokens, b.x, b.qkv, b.ao, b.xf, b.hi, b.lo, b.routing, b.logits, b.att};
    for (void* p : bufs) cudaFree(p);
    b = PrefillBufs{};
    cudaFree(m->proj_part);
    m->proj_part = nullptr;
    m->proj_part_bytes = 0;
}
}  // namespace rbt

extern "C" int rbt_model_prefill(RbtModel* m, const int32_t* tokens, int n_tokens, int pos0, float* logits,
                                 int logit_rows, int32_t* routing_out) {
    return rbt_model_prefill_seq(m, 0, tokens, n_tokens, pos0, logits, logit_rows, routing_out);
}

extern "C" int rbt_model_prefill_seq(RbtModel* m, int seq, const int32_t* tokens, int n_tokens, int pos0,
                                     float* logits, int logit_rows, int32_t* routing_out) {
    if (!m) return fail("null model");
    if (seq < 0 || seq >= m->n_seq) return fail("sequence %d outside the %d KV caches", seq, m->n_seq);
    const RbtModelConfig& c = m->cfg;
    if (n_tokens <= 0 || !tokens) return fail("no tokens");
    if (pos0 < 0 || pos0 + n_tokens > m->ctx)
        return fail("positions %d..%d outside the KV cache of %d", pos0, pos0 + n_tokens - 1, m->ctx);
    if (logit_rows < 0 || logit_rows > n_tokens || (logit_rows > 0 && !logits))
        return fail("logit_rows %d must be in [0, n_tokens] with a logits buffer", logit_rows);
    if (c.head_dim != 64 && c.head_dim != 128) return fail("batched prompt needs head_dim 64 or 128");
    for (int t = 0; t < n_tokens; t++)
        if (tokens[t] < 0 || tokens[t] >= c.vocab) return fail("token %d out of range", tokens[t]);
    if (!check_ready(m) || !model_moe_fits(m, n_tokens)) return 0;
    CU(cudaSetDevice(m->device));
    if (!reserve(m, n_tokens, pos0, logit_rows)) return 0;
    CU(cudaMemcpyAsync(m->pf.tokens, tokens, (size_t)n_tokens * 4, cudaMemcpyHostToDevice, m->stream));
    const int ok = c.dtype == RBT_MOE_DT_BF16 ? run_prefill<uint16_t>(m, seq, n_tokens, pos0, logit_rows)
                                              : run_prefill<float>(m, seq, n_tokens, pos0, logit_rows);
    if (!ok) {
        cudaStreamSynchronize(m->stream);
        return 0;
    }
    if (logit_rows > 0)
        CU(cudaMemcpyAsync(logits, m->pf.logits, (size_t)logit_rows * c.vocab * 4, cudaMemcpyDeviceToHost, m->stream));
    if (routing_out)
        CU(cudaMemcpyAsync(routing_out, m->pf.routing, (size_t)n_tokens * c.n_layers * c.top_k * 4,
                           cudaMemcpyDeviceToHost, m->stream));
    CU(cudaMemcpyAsync(m->h_status, m->status, sizeof(unsigned), cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    if (*m->h_status) {
        const unsigned st = *m->h_status;
        *m->h_status = 0;
        CU(cudaMemset(m->status, 0, sizeof(unsigned)));
        return fail("a bounded wait in the projection or attention kernels ran out (code 0x%x)", st);
    }
    return moe_status_ok(m->moe);
}

extern "C" int rbt_model_decode_batch(RbtModel* m, const int32_t* tokens, const int32_t* pos, int n, float* logits,
                                      int32_t* next, int32_t* routing_out) {
    if (!m) return fail("null model");
    const RbtModelConfig& c = m->cfg;
    if (n < 1 || n > m->n_seq) return fail("n %d outside [1, %d] (the sequences of rbt_model_set_sequences)", n,
                                           m->n_seq);
    if (!tokens || !pos) return fail("null tokens or positions");
    for (int i = 0; i < n; i++) {
        if (tokens[i] < 0 || tokens[i] >= c.vocab) return fail("row %d: token %d out of range", i, tokens[i]);
        if (pos[i] < 0 || pos[i] >= m->ctx)
            return fail("row %d: position %d outside the KV cache of %d", i, pos[i], m->ctx);
    }
    if (!check_ready(m) || !model_moe_fits(m, n)) return 0;
    CU(cudaSetDevice(m->device));
    const bool want = logits || next;
    if (!reserve(m, n, 0, want ? n : 0) || !reserve_decode(m, n)) return 0;
    for (int i = 0; i < n; i++) {
        m->h_steps[i].token = tokens[i];
        m->h_steps[i].pos = pos[i];
    }
    cudaStream_t s = m->stream;
    CU(cudaMemcpyAsync(m->steps, m->h_steps, (size_t)n * sizeof(Step), cudaMemcpyHostToDevice, s));
    const int ok = c.dtype == RBT_MOE_DT_BF16 ? run_decode<uint16_t>(m, n, want) : run_decode<float>(m, n, want);
    if (!ok) {
        cudaStreamSynchronize(s);
        return 0;
    }
    if (logits) CU(cudaMemcpyAsync(logits, m->pf.logits, (size_t)n * c.vocab * 4, cudaMemcpyDeviceToHost, s));
    if (next) CU(cudaMemcpyAsync(next, m->dnext, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    if (routing_out)
        CU(cudaMemcpyAsync(routing_out, m->pf.routing, (size_t)n * c.n_layers * c.top_k * 4, cudaMemcpyDeviceToHost,
                           s));
    CU(cudaMemcpyAsync(m->h_status, m->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
    CU(cudaStreamSynchronize(s));
    if (*m->h_status) {
        const unsigned st = *m->h_status;
        *m->h_status = 0;
        CU(cudaMemset(m->status, 0, sizeof(unsigned)));
        return fail("a bounded wait in the projection or attention kernels ran out (code 0x%x)", st);
    }
    return moe_status_ok(m->moe);
}
