// model.cu -- the rest of the engine's forward() on the GPU (rabbit2.c:455-550):
// embedding, attention half of every layer, final norm and lm_head.  The MoE
// blocks are rbt_moe_block_device (moe_api.cu) on the same stream.
//
// One token (decode, batch 1) per call, as forward() does.  Everything the engine
// keeps in State (rabbit2.c:101-106) lives in HBM: the residual x, q|k|v, the KV
// cache (f32, as the engine keeps it, but head-major: [n_layers][n_kv_heads][ctx]
// [head_dim], so one head's run of positions is contiguous), the logits.  The
// token and position are read from device memory, so the whole token -- 2 + 4 L
// kernels -- is one CUDA graph, replayed per token:
//
//   embed                       x = tok_emb[token]                       (:461-467)
//   per layer l:
//     norm_gemv                 q|k|v = [wq;wk;wv] . rmsnorm(x)          (:473-476)
//     attn_decode (heads x splits)
//                               whole-projection QK-norm, RoPE at pos,    (:477-483)
//                               k, v into the cache, scores, softmax, the (:485-506)
//                               weighted V sum of one split of positions;
//                               the last split of a head to finish merges
//                               the splits (max / sum rescaling)
//     out_proj                  x += wo . attn_out                       (:507-508)
//     rbt_moe_block_device      x += MoE(rmsnorm(x))                     (:511-542)
//   norm_gemv                   logits = lm_head . rmsnorm(x)            (:545-546)
//
// The GEMVs stream each weight row once with 16-byte loads (HBM-bound: at the
// OLMoE shape 24 MB q|k|v + 8 MB wo per layer and 206 MB of lm_head per token).
// Arithmetic is fp32; sums are in a fixed order, so results are deterministic,
// and differ from the engine's sequential sums by reassociation only.  RoPE
// uses a table of the engine's own angles (fp64 pow/cos/sin, rounded to f32,
// computed on the host by the same formula as rope(), rabbit2.c:410-421).
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <new>
#include <vector>

#include "../../include/rbt_moe.h"
#include "common.cuh"
#include "kernels.h"
#include "model_internal.h"
#include "tc_ptx.cuh"

namespace rbt {
void set_last_error(const char* msg);
int moe_status_ok(RbtMoe* m);
unsigned long long moe_workspace_generation(RbtMoe* m);
unsigned* moe_status_word(RbtMoe* m);
int moe_ep_rows(RbtMoe* m);
int moe_ep_cap(RbtMoe* m);
}  // namespace rbt

namespace {

using namespace rbt;
using namespace rbt::tc;
using rbt::Step;

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

constexpr int kGemvThreads = 256;
constexpr int kGemvCtasPerSm = 4;
constexpr int kGemvUnroll = 8;   // 16-byte weight loads in flight per lane
constexpr int kMaxVec4 = 2;      // float4s of an input vector per GEMV thread: dim, n_heads*head_dim <= 2048
constexpr int kAttnThreads = 128;
constexpr int kSplit = 64;       // positions per attention split
constexpr int kMaxHeadDim = 256;
constexpr int kAttnVec4 = 16;    // float4s of q|k per attention thread: nq + nkv <= 8192
constexpr int kMaxSplits = 128;  // ctx <= kMaxSplits x kSplit
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ void record_error(unsigned* status, unsigned code) { atomicCAS(status, 0u, code); }

// ---------------------------------------------------------------- embedding
template <typename WT>
__global__ void embed_kernel(const WT* emb, int D, const Step* step, float* x) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t row = (size_t)step->token * D;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < D; i += gridDim.x * blockDim.x)
        x[i] = WeightTraits<WT>::load1(emb + row + i);
}

// ---------------------------------------------------------------- GEMV rows
// Warp-per-row GEMV: row r = W[r, :] . xs (xs: `cols` floats in shared memory),
// rows r = global warp, + total warps, ...  A row is read in chunks of
// 32 lanes x kGemvUnroll 16-byte loads, all in flight before the products.
template <typename WT>
__device__ __forceinline__ void load_chunk(const WT* W, int cols, int r, int v0, uint4 (&q)[kGemvUnroll]) {
    const int lane = threadIdx.x & 31, nvec = cols / WeightTraits<WT>::kVec;
    const uint4* wr = reinterpret_cast<const uint4*>(W + (size_t)r * cols);
#pragma unroll
    for (int u = 0; u < kGemvUnroll; u++) {
        const int v = v0 + lane + 32 * u;
        q[u] = v < nvec ? ld_stream16(wr + v) : make_uint4(0, 0, 0, 0);
    }
}

template <typename WT>
__device__ __forceinline__ float dot_chunk(const float* xs, int cols, int v0, const uint4 (&q)[kGemvUnroll],
                                           float acc) {
    constexpr int kV = WeightTraits<WT>::kVec;
    const int lane = threadIdx.x & 31, nvec = cols / kV;
#pragma unroll
    for (int u = 0; u < kGemvUnroll; u++) {
        const int v = v0 + lane + 32 * u;
        if (v < nvec) {
            float f[kV];
            WeightTraits<WT>::unpack(q[u], f);
            const float* xv = xs + (size_t)v * kV;
#pragma unroll
            for (int e = 0; e < kV; e++) acc = fmaf(f[e], xv[e], acc);
        }
    }
    return acc;
}

// The rows of this warp; the first chunk of its first row is already in q
// (loaded before the kernel waited for its inputs).  epi(r, dot) stores a row.
template <typename WT, typename Epi>
__device__ __forceinline__ void gemv_rows(const float* xs, int cols, const WT* W, int rows, uint4 (&q)[kGemvUnroll],
                                          Epi epi) {
    const int lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int nvec = cols / WeightTraits<WT>::kVec;
    const int r0 = blockIdx.x * nwarps + (threadIdx.x >> 5);
    for (int r = r0; r < rows; r += gridDim.x * nwarps) {
        float acc = 0.0f;
        for (int v0 = 0; v0 < nvec; v0 += 32 * kGemvUnroll) {
            if (r != r0 || v0 != 0) load_chunk<WT>(W, cols, r, v0, q);
            acc = dot_chunk<WT>(xs, cols, v0, q, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) epi(r, acc);
    }
}

template <typename WT>
__device__ __forceinline__ void prefetch_first_chunk(const WT* W, int cols, int rows, uint4 (&q)[kGemvUnroll]) {
    const int r0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r0 < rows) load_chunk<WT>(W, cols, r0, 0, q);
}

// out[r] = W[r, :] . rmsnorm(x, nw) for r < rows.  Every CTA normalises x itself
// with the same fixed-order sum, so all hold the same bits (rmsnorm, rabbit2.c:392-397).
// The weights are static: the first chunk of every warp's first row is loaded
// before griddepcontrol.wait, overlapping the previous kernel's tail.
template <typename WT>
__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm) norm_gemv_kernel(const float* x, const float* nw, float eps,
                                                                 int D, const WT* W, int rows, float* out) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float red[kGemvThreads / 32];
    uint4 q[kGemvUnroll];
    prefetch_first_chunk<WT>(W, D, rows, q);
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // x and the norm weights: every 16-byte load in flight at once (D <= kMaxVec4 x 4 x threads)
    float4 xv[kMaxVec4], wv[kMaxVec4];
    float ss = 0.0f;
    const int n4 = D / 4;
#pragma unroll
    for (int k = 0; k < kMaxVec4; k++) {
        const int i4 = threadIdx.x + k * kGemvThreads;
        if (i4 < n4) {
            xv[k] = __ldcg(reinterpret_cast<const float4*>(x) + i4);
            wv[k] = __ldg(reinterpret_cast<const float4*>(nw) + i4);
        }
    }
#pragma unroll
    for (int k = 0; k < kMaxVec4; k++)
        if (threadIdx.x + k * kGemvThreads < n4) {
            ss = fmaf(xv[k].x, xv[k].x, ss);
            ss = fmaf(xv[k].y, xv[k].y, ss);
            ss = fmaf(xv[k].z, xv[k].z, ss);
            ss = fmaf(xv[k].w, xv[k].w, ss);
        }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += red[w];
    const float inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, (float)D), eps));
#pragma unroll
    for (int k = 0; k < kMaxVec4; k++) {
        const int i4 = threadIdx.x + k * kGemvThreads;
        if (i4 < n4)
            reinterpret_cast<float4*>(xs)[i4] =
                make_float4(__fmul_rn(__fmul_rn(xv[k].x, inv), wv[k].x), __fmul_rn(__fmul_rn(xv[k].y, inv), wv[k].y),
                            __fmul_rn(__fmul_rn(xv[k].z, inv), wv[k].z), __fmul_rn(__fmul_rn(xv[k].w, inv), wv[k].w));
    }
    __syncthreads();
    gemv_rows<WT>(xs, D, W, rows, q, [&](int r, float v) { out[r] = v; });
}

// x[r] += wo[r, :] . attn_out  (rabbit2.c:507-508).  It does not let the next
// kernel (the cooperative MoE kernel) start early.
template <typename WT>
__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm) out_proj_kernel(const float* ao, int nq, const WT* wo, int D,
                                                                float* x) {
    extern __shared__ __align__(16) float xs[];
    uint4 q[kGemvUnroll];
    prefetch_first_chunk<WT>(wo, nq, D, q);
    pdl_wait();
    float4 av[kMaxVec4];
#pragma unroll
    for (int k = 0; k < kMaxVec4; k++) {
        const int i4 = threadIdx.x + k * kGemvThreads;
        if (i4 < nq / 4) av[k] = __ldcg(reinterpret_cast<const float4*>(ao) + i4);
    }
#pragma unroll
    for (int k = 0; k < kMaxVec4; k++) {
        const int i4 = threadIdx.x + k * kGemvThreads;
        if (i4 < nq / 4) reinterpret_cast<float4*>(xs)[i4] = av[k];
    }
    __syncthreads();
    gemv_rows<WT>(xs, nq, wo, D, q, [&](int r, float v) { x[r] = __fadd_rn(x[r], v); });
}

// ---------------------------------------------------------------- attention
struct AttnArgs {
    const float* qkv;       // [nq + 2 nkv]: q | k | v of this token
    const float* q_norm;    // [nq] or nullptr (no QK-norm)
    const float* k_norm;    // [nkv]
    float eps, scale;
    const float* rope_cos;  // [ctx][head_dim / 2]
    const float* rope_sin;
    float* kc;              // this layer's cache, head-major [n_kv_heads][ctx][head_dim]
    float* vc;
    const Step* step;
    float* part;            // [n_heads][n_splits][head_dim + 2]: max, sum, weighted V
    float* ao;              // [nq] attention output
    unsigned* done;         // [n_heads] finished splits, zero between calls
    unsigned* status;       // error word
    int n_heads, n_kv_heads, hd, ctx, n_splits;
    // batched decode (gridDim.z rows, one token of its own sequence each): row z reads
    // step[z], qkv + z*qkv_stride, its sequence's cache at kc/vc + z*kv_stride, and
    // writes part/done/ao + z*(part_stride, n_heads, ao_stride).  0 for one token.
    long qkv_stride, kv_stride, part_stride, ao_stride;
};

// CTA (head h, split s) covers positions [s kSplit, min((s+1) kSplit, pos+1)).
// The cached positions of the split (all below pos) are one contiguous run per
// kv head: two bulk copies bring K and V into shared memory, issued before the
// kernel waits for this token's q|k|v (the cache was written by earlier tokens).
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs args) {
    extern __shared__ __align__(128) float kv_s[];  // K [kSplit][hd] | V [kSplit][hd]
    __shared__ __align__(16) float qh[kMaxHeadDim], kn[kMaxHeadDim], vn[kMaxHeadDim];
    __shared__ float sc[kSplit];
    __shared__ float red[kAttnThreads / 32], red2[kAttnThreads / 32];
    __shared__ float s_m[kMaxSplits], s_w[kMaxSplits];
    __shared__ unsigned s_last;
    __shared__ uint64_t bar;
    // this row's views (batched decode; row 0 is the arguments themselves)
    const long z = blockIdx.z;
    AttnArgs a = args;
    a.step = args.step + z;
    a.qkv = args.qkv + z * args.qkv_stride;
    a.kc = args.kc + z * args.kv_stride;
    a.vc = args.vc + z * args.kv_stride;
    a.part = args.part + z * args.part_stride;
    a.ao = args.ao + z * args.ao_stride;
    a.done = args.done + z * args.n_heads;
    const int h = blockIdx.x, s = blockIdx.y, hd = a.hd;
    const int pos = a.step->pos;  // written by the graph's first copy, before every kernel of the token
    const int t0 = s * kSplit;
    if (t0 > pos) return;  // a split past the current position: no work, not counted
    const int t1 = min(t0 + kSplit, pos + 1);
    const int nc = min(t1, pos) - t0;  // cached positions (position pos is this token's)
    const int group = a.n_heads / a.n_kv_heads, kvh = h / group;
    float* Ks = kv_s;
    float* Vs = kv_s + (size_t)kSplit * hd;
    const size_t run = ((size_t)kvh * a.ctx + t0) * hd;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        if (nc > 0) {
            mbar_arrive_expect_tx(&bar, 2u * nc * hd * 4);
            bulk_load(Ks, a.kc + run, (uint32_t)nc * hd * 4, &bar);
            bulk_load(Vs, a.vc + run, (uint32_t)nc * hd * 4, &bar);
        }
    }
    const int nq = a.n_heads * hd, nkv = a.n_kv_heads * hd;
    const int half = hd / 2, i = threadIdx.x;  // thread i < half owns the pair (i, i + half)
    const bool has_new = pos < t1;  // this split holds position pos: k and v of this token
    // static inputs before the wait: the RoPE row of pos and the QK-norm weights
    float cs = 0.0f, sn = 0.0f, wqa = 1.0f, wqb = 1.0f, wka = 1.0f, wkb = 1.0f;
    if (i < half) {
        cs = a.rope_cos[(size_t)pos * half + i];
        sn = a.rope_sin[(size_t)pos * half + i];
        if (a.q_norm) {
            wqa = a.q_norm[(size_t)h * hd + i];
            wqb = a.q_norm[(size_t)h * hd + i + half];
            wka = a.k_norm[(size_t)kvh * hd + i];
            wkb = a.k_norm[(size_t)kvh * hd + i + half];
        }
    }
    pdl_wait();
    pdl_launch_dependents();
    // this token's inputs in one round of loads: the head's q pair, the k pair and
    // v of its kv head, and for the QK-norm all of q|k (16-byte loads)
    float qa = 0.0f, qb = 0.0f, ka = 0.0f, kb = 0.0f, va = 0.0f, vb = 0.0f;
    if (i < half) {
        qa = __ldcg(a.qkv + (size_t)h * hd + i);
        qb = __ldcg(a.qkv + (size_t)h * hd + i + half);
        if (has_new) {
            ka = __ldcg(a.qkv + nq + (size_t)kvh * hd + i);
            kb = __ldcg(a.qkv + nq + (size_t)kvh * hd + i + half);
        }
    }
    if (has_new) {
        const float* v = a.qkv + nq + nkv + (size_t)kvh * hd;
        if (i < hd) va = __ldcg(v + i);
        if (i + kAttnThreads < hd) vb = __ldcg(v + i + kAttnThreads);
    }
    // QK-norm factors of the whole q and k projections (rabbit2.c:477-480), both
    // sums reduced together
    float inv_q = 1.0f, inv_k = 1.0f;
    if (a.q_norm) {
        const int nq4 = nq / 4, n4 = (nq + nkv) / 4;
        float4 v[kAttnVec4];
#pragma unroll
        for (int k = 0; k < kAttnVec4; k++) {
            const int i4 = threadIdx.x + k * kAttnThreads;
            if (i4 < n4) v[k] = __ldcg(reinterpret_cast<const float4*>(a.qkv) + i4);
        }
        float sq = 0.0f, sk = 0.0f;
#pragma unroll
        for (int k = 0; k < kAttnVec4; k++) {
            const int i4 = threadIdx.x + k * kAttnThreads;
            if (i4 < n4) {
                float t = fmaf(v[k].x, v[k].x, 0.0f);
                t = fmaf(v[k].y, v[k].y, t);
                t = fmaf(v[k].z, v[k].z, t);
                t = fmaf(v[k].w, v[k].w, t);
                if (i4 < nq4) sq += t;
                else sk += t;
            }
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        if (lane == 0) {
            red[warp] = sq;
            red2[warp] = sk;
        }
        __syncthreads();
        float tq = 0.0f, tk = 0.0f;
        for (int w = 0; w < kAttnThreads / 32; w++) {
            tq += red[w];
            tk += red2[w];
        }
        inv_q = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tq, (float)nq), a.eps));
        inv_k = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tk, (float)nkv), a.eps));
    }
    // QK-norm (x * inv * w, rmsnorm of rabbit2.c:392-397), then RoPE:
    // p[i] = a cs - b sn, p[i + half] = b cs + a sn (rabbit2.c:418-419)
    if (i < half) {
        if (a.q_norm) {
            qa = __fmul_rn(__fmul_rn(qa, inv_q), wqa);
            qb = __fmul_rn(__fmul_rn(qb, inv_q), wqb);
            ka = __fmul_rn(__fmul_rn(ka, inv_k), wka);
            kb = __fmul_rn(__fmul_rn(kb, inv_k), wkb);
        }
        qh[i] = __fsub_rn(__fmul_rn(qa, cs), __fmul_rn(qb, sn));
        qh[i + half] = __fadd_rn(__fmul_rn(qb, cs), __fmul_rn(qa, sn));
        if (has_new) {
            kn[i] = __fsub_rn(__fmul_rn(ka, cs), __fmul_rn(kb, sn));
            kn[i + half] = __fadd_rn(__fmul_rn(kb, cs), __fmul_rn(ka, sn));
        }
    }
    if (has_new) {
        if (i < hd) vn[i] = va;
        if (i + kAttnThreads < hd) vn[i + kAttnThreads] = vb;
    }
    __syncthreads();  // (also publishes the mbarrier's initialisation)
    if (has_new && h % group == 0) {  // one head of the group stores them (rabbit2.c:484-486)
        const size_t at = ((size_t)kvh * a.ctx + pos) * hd;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            a.kc[at + i] = kn[i];
            a.vc[at + i] = vn[i];
        }
    }
    if (nc > 0) {
        const bool got = mbar_wait_bounded(&bar, 0, kWaitNs);
        if (!__syncthreads_and(got)) {
            // the copies are of valid memory and end; wait for them (bounded) before leaving
            if (threadIdx.x == 0) {
                record_error(a.status, 0x701);
                (void)mbar_wait_bounded(&bar, 0, kWaitNs);
            }
            __syncthreads();
            return;
        }
    }
    // scores (rabbit2.c:488-495): warp w takes positions t0 + w, t0 + w + 4, ...
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int t = t0 + warp; t < t1; t += nwarps) {
        const float* kt = t == pos ? kn : Ks + (size_t)(t - t0) * hd;
        float d = 0.0f;
        for (int i = lane; i < hd; i += 32) d = fmaf(qh[i], kt[i], d);
        d = warp_sum(d);
        if (lane == 0) sc[t - t0] = d * a.scale;
    }
    __syncthreads();
    // this split's max, exp sum and exp-weighted V (softmax, rabbit2.c:399-405,496-505)
    const int n = t1 - t0;
    float mx = -INFINITY;
    for (int j = 0; j < n; j++) mx = fmaxf(mx, sc[j]);
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) sc[j] = expf(sc[j] - mx);
    __syncthreads();
    float l = 0.0f;
    for (int j = 0; j < n; j++) l += sc[j];
    float* pp = a.part + ((size_t)h * a.n_splits + s) * (hd + 2);
    const bool only = pos < kSplit;  // one split: it is the whole softmax, no merge
    for (int c = threadIdx.x; c < hd; c += blockDim.x) {
        float o = 0.0f;
        for (int j = 0; j < nc; j++) o = fmaf(sc[j], Vs[(size_t)j * hd + c], o);
        if (has_new) o = fmaf(sc[n - 1], vn[c], o);
        if (only)
            a.ao[(size_t)h * hd + c] = o / l;
        else
            pp[2 + c] = o;
    }
    if (only) return;
    if (threadIdx.x == 0) {
        pp[0] = mx;
        pp[1] = l;
    }
    // the last split of head h to finish merges all of them (every writer fences
    // its partial before the count is taken)
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned n_act = (unsigned)(pos / kSplit + 1);
        const unsigned prev = atomicAdd(a.done + h, 1u);
        s_last = prev + 1 == n_act;
        if (s_last) a.done[h] = 0;  // every split of this call has arrived: reset for the next
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int n_act = pos / kSplit + 1;
    const float* ph = a.part + (size_t)h * a.n_splits * (hd + 2);
    // every split's max and sum into shared memory (one load each, all in flight)
    for (int j = threadIdx.x; j < n_act; j += blockDim.x) {
        s_m[j] = __ldcg(ph + (size_t)j * (hd + 2));
        s_w[j] = __ldcg(ph + (size_t)j * (hd + 2) + 1);
    }
    __syncthreads();
    float M = -INFINITY;
    for (int j = 0; j < n_act; j++) M = fmaxf(M, s_m[j]);
    float L = 0.0f;
    for (int j = 0; j < n_act; j++) L += s_w[j] * expf(s_m[j] - M);
    __syncthreads();
    for (int j = threadIdx.x; j < n_act; j += blockDim.x) s_w[j] = expf(s_m[j] - M);  // split weights
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float o = 0.0f;
#pragma unroll 8
        for (int j = 0; j < n_act; j++) o = fmaf(__ldcg(ph + (size_t)j * (hd + 2) + 2 + i), s_w[j], o);
        a.ao[(size_t)h * hd + i] = o / L;
    }
}

size_t attn_smem_bytes(int hd) { return (size_t)2 * kSplit * hd * sizeof(float); }

// ---------------------------------------------------------------- batched decode attention
// CTA (head h, split s, row z) of the batched decode (rbt_model_decode_batch): row z's
// attention over positions [s kRSplit, min((s+1) kRSplit, pos+1)) of its own sequence's
// cache, with an online softmax over chunks of kRChunk positions.  The chunks' K and
// V runs stream through a kRStages-slot ring of bulk copies, so the copies of later
// chunks are in flight while a chunk is computed (a 64-position CTA of the one-token
// kernel copies, then computes).  Splits merge as in the one-token kernel (the last
// split of a head rescales the others' partials).  Same inputs and outputs as
// attn_decode_kernel; head_dim a multiple of 32, at most 256.
constexpr int kRChunk = 32;
constexpr int kRStages = 2;
constexpr int kRSplit = 1024;
constexpr int kRThreads = 128;
static_assert(kRChunk == 32, "a chunk's positions map onto the lanes of a warp");
constexpr int kRMaxQ = kMaxHeadDim / 32;           // q values per lane
constexpr int kRMaxV = kMaxHeadDim / kRThreads;    // output dims per thread

size_t attn_rows_smem_bytes(int hd) { return (size_t)kRStages * 2 * kRChunk * hd * sizeof(float); }

__global__ void __launch_bounds__(kRThreads) attn_rows_kernel(const AttnArgs args) {
    extern __shared__ __align__(128) float ring[];  // [stage][K | V][kRChunk][hd]
    __shared__ __align__(16) float qh[kMaxHeadDim], kn[kMaxHeadDim], vn[kMaxHeadDim];
    __shared__ float sc[kRChunk];
    __shared__ float red[kRThreads / 32], red2[kRThreads / 32];
    __shared__ float s_m[kMaxSplits], s_w[kMaxSplits];
    __shared__ unsigned s_last;
    __shared__ uint64_t full[kRStages];
    const long z = blockIdx.z;
    AttnArgs a = args;
    a.step = args.step + z;
    a.qkv = args.qkv + z * args.qkv_stride;
    a.kc = args.kc + z * args.kv_stride;
    a.vc = args.vc + z * args.kv_stride;
    a.part = args.part + z * args.part_stride;
    a.ao = args.ao + z * args.ao_stride;
    a.done = args.done + z * args.n_heads;
    const int h = blockIdx.x, s = blockIdx.y, hd = a.hd, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int pos = a.step->pos;
    const int t0 = s * kRSplit;
    if (t0 > pos) return;
    const int t1 = min(t0 + kRSplit, pos + 1);
    const int nchunks = (t1 - t0 + kRChunk - 1) / kRChunk;
    const int group = a.n_heads / a.n_kv_heads, kvh = h / group;
    const size_t stage_floats = (size_t)2 * kRChunk * hd;
    const float* kbase = a.kc + ((size_t)kvh * a.ctx) * hd;
    const float* vbase = a.vc + ((size_t)kvh * a.ctx) * hd;
    // chunk c covers positions [t0 + c kRChunk, ...); its cached part (< pos) is copied
    auto issue = [&](int c) {
        const int c0 = t0 + c * kRChunk, c1 = min(c0 + kRChunk, t1), nc = min(c1, pos) - c0;
        uint64_t* bar = &full[c % kRStages];
        float* st = ring + (size_t)(c % kRStages) * stage_floats;
        if (nc > 0) {
            mbar_arrive_expect_tx(bar, 2u * nc * hd * 4);
            bulk_load(st, kbase + (size_t)c0 * hd, (uint32_t)nc * hd * 4, bar);
            bulk_load(st + (size_t)kRChunk * hd, vbase + (size_t)c0 * hd, (uint32_t)nc * hd * 4, bar);
        } else {
            mbar_arrive(bar);  // nothing cached in this chunk (it holds only position pos)
        }
    };
    if (tid == 0) {
        for (int b = 0; b < kRStages; b++) mbar_init(&full[b], 1);
        fence_mbar_init();
        for (int c = 0; c < nchunks && c < kRStages; c++) issue(c);
    }
    const int nq = a.n_heads * hd, nkv = a.n_kv_heads * hd, half = hd / 2;
    const bool has_new = pos < t1;  // this split holds position pos: k and v of this token
    float cs = 0.0f, sn = 0.0f, wqa = 1.0f, wqb = 1.0f, wka = 1.0f, wkb = 1.0f;
    if (tid < half) {
        cs = a.rope_cos[(size_t)pos * half + tid];
        sn = a.rope_sin[(size_t)pos * half + tid];
        if (a.q_norm) {
            wqa = a.q_norm[(size_t)h * hd + tid];
            wqb = a.q_norm[(size_t)h * hd + tid + half];
            wka = a.k_norm[(size_t)kvh * hd + tid];
            wkb = a.k_norm[(size_t)kvh * hd + tid + half];
        }
    }
    float qa = 0.0f, qb = 0.0f, ka = 0.0f, kb = 0.0f, va = 0.0f, vb = 0.0f;
    if (tid < half) {
        qa = __ldcg(a.qkv + (size_t)h * hd + tid);
        qb = __ldcg(a.qkv + (size_t)h * hd + tid + half);
        if (has_new) {
            ka = __ldcg(a.qkv + nq + (size_t)kvh * hd + tid);
            kb = __ldcg(a.qkv + nq + (size_t)kvh * hd + tid + half);
        }
    }
    if (has_new) {
        const float* v = a.qkv + nq + nkv + (size_t)kvh * hd;
        if (tid < hd) va = __ldcg(v + tid);
        if (tid + kRThreads < hd) vb = __ldcg(v + tid + kRThreads);
    }
    // QK-norm over the whole q and k projections (rabbit2.c:477-480)
    float inv_q = 1.0f, inv_k = 1.0f;
    if (a.q_norm) {
        const int nq4 = nq / 4, n4 = (nq + nkv) / 4;
        float sq = 0.0f, sk = 0.0f;
        for (int i4 = tid; i4 < n4; i4 += kRThreads) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(a.qkv) + i4);
            float t = fmaf(v.x, v.x, 0.0f);
            t = fmaf(v.y, v.y, t);
            t = fmaf(v.z, v.z, t);
            t = fmaf(v.w, v.w, t);
            if (i4 < nq4) sq += t;
            else sk += t;
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        if (lane == 0) {
            red[warp] = sq;
            red2[warp] = sk;
        }
        __syncthreads();
        float tq = 0.0f, tk = 0.0f;
        for (int w = 0; w < kRThreads / 32; w++) {
            tq += red[w];
            tk += red2[w];
        }
        inv_q = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tq, (float)nq), a.eps));
        inv_k = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tk, (float)nkv), a.eps));
    }
    // RoPE (rabbit2.c:418-419): p[i] = a cs - b sn, p[i + half] = b cs + a sn
    if (tid < half) {
        if (a.q_norm) {
            qa = __fmul_rn(__fmul_rn(qa, inv_q), wqa);
            qb = __fmul_rn(__fmul_rn(qb, inv_q), wqb);
            ka = __fmul_rn(__fmul_rn(ka, inv_k), wka);
            kb = __fmul_rn(__fmul_rn(kb, inv_k), wkb);
        }
        qh[tid] = __fsub_rn(__fmul_rn(qa, cs), __fmul_rn(qb, sn));
        qh[tid + half] = __fadd_rn(__fmul_rn(qb, cs), __fmul_rn(qa, sn));
        if (has_new) {
            kn[tid] = __fsub_rn(__fmul_rn(ka, cs), __fmul_rn(kb, sn));
            kn[tid + half] = __fadd_rn(__fmul_rn(kb, cs), __fmul_rn(ka, sn));
        }
    }
    if (has_new) {
        if (tid < hd) vn[tid] = va;
        if (tid + kRThreads < hd) vn[tid + kRThreads] = vb;
    }
    __syncthreads();  // (also publishes the mbarriers' initialisation)
    if (has_new && h % group == 0) {  // one head of the group stores them (rabbit2.c:484-486)
        const size_t at = ((size_t)kvh * a.ctx + pos) * hd;
        for (int i = tid; i < hd; i += kRThreads) {
            a.kc[at + i] = kn[i];
            a.vc[at + i] = vn[i];
        }
    }
    const int nqv = hd / 32;  // q values per lane: q[lane + 32 u]
    float qr[kRMaxQ];
#pragma unroll
    for (int u = 0; u < kRMaxQ; u++) qr[u] = u < nqv ? qh[lane + 32 * u] : 0.0f;
    float m_run = -INFINITY, l_run = 0.0f, o[kRMaxV];
#pragma unroll
    for (int v = 0; v < kRMaxV; v++) o[v] = 0.0f;
    for (int c = 0; c < nchunks; c++) {
        const int c0 = t0 + c * kRChunk, nv = min(c0 + kRChunk, t1) - c0;
        float* Ks = ring + (size_t)(c % kRStages) * stage_floats;
        float* Vs = Ks + (size_t)kRChunk * hd;
        const bool got = mbar_wait_bounded(&full[c % kRStages], (uint32_t)(c / kRStages) & 1u, kWaitNs);
        if (!__syncthreads_and(got)) {
            // the copies are of valid memory and end: wait (bounded) for those in flight
            if (tid == 0) {
                record_error(a.status, 0x701);
                for (int d = c; d < nchunks && d < c + kRStages; d++)
                    (void)mbar_wait_bounded(&full[d % kRStages], (uint32_t)(d / kRStages) & 1u, kWaitNs);
            }
            __syncthreads();
            return;
        }
        if (has_new && pos < c0 + nv) {  // this token's k and v take the row of position pos
            const int jp = pos - c0;
            for (int i = tid; i < hd; i += kRThreads) {
                Ks[(size_t)jp * hd + i] = kn[i];
                Vs[(size_t)jp * hd + i] = vn[i];
            }
            __syncthreads();
        }
        // scores (rabbit2.c:488-495): warp w takes positions 8w .. 8w+7 of the chunk
        {
            float d[kRChunk / (kRThreads / 32)];
#pragma unroll
            for (int i = 0; i < kRChunk / (kRThreads / 32); i++) {
                const int j = warp * (kRChunk / (kRThreads / 32)) + i;
                float acc = 0.0f;
                if (j < nv) {
                    const float* kr = Ks + (size_t)j * hd + lane;
#pragma unroll
                    for (int u = 0; u < kRMaxQ; u++)
                        if (u < nqv) acc = fmaf(qr[u], kr[32 * u], acc);
                }
                d[i] = acc;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int i = 0; i < kRChunk / (kRThreads / 32); i++) d[i] += __shfl_xor_sync(FULL_MASK, d[i], off);
            if (lane < kRChunk / (kRThreads / 32)) {
                float mine = d[0];
#pragma unroll
                for (int i = 1; i < kRChunk / (kRThreads / 32); i++)
                    if (lane == i) mine = d[i];
                const int j = warp * (kRChunk / (kRThreads / 32)) + lane;
                if (j < nv) sc[j] = mine * a.scale;
            }
        }
        __syncthreads();
        // online softmax (rabbit2.c:399-405, 496-505), every warp for itself: lane j holds
        // position j's score, the max and the exp sum by shuffles, the weights stay in lanes
        const float sj = lane < nv ? sc[lane] : -INFINITY;
        float cm = sj;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(FULL_MASK, cm, off));
        const float m_new = fmaxf(m_run, cm);
        const float alpha = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
        const float pl = lane < nv ? expf(sj - m_new) : 0.0f;
        l_run = l_run * alpha + warp_sum(pl);
#pragma unroll
        for (int v = 0; v < kRMaxV; v++) {
            const int col = tid + kRThreads * v;
            float acc = o[v] * alpha;
            for (int j = 0; j < nv; j++) {
                const float pjv = __shfl_sync(FULL_MASK, pl, j);
                if (col < hd) acc = fmaf(pjv, Vs[(size_t)j * hd + col], acc);
            }
            o[v] = acc;
        }
        m_run = m_new;
        __syncthreads();  // stage c % kRStages is free again
        if (tid == 0 && c + kRStages < nchunks) issue(c + kRStages);
    }
    if (pos < kRSplit) {  // one split: it is the whole softmax, no merge
#pragma unroll
        for (int v = 0; v < kRMaxV; v++) {
            const int col = tid + kRThreads * v;
            if (col < hd) a.ao[(size_t)h * hd + col] = o[v] / l_run;
        }
        return;
    }
    float* pp = a.part + ((size_t)h * a.n_splits + s) * (hd + 2);
#pragma unroll
    for (int v = 0; v < kRMaxV; v++) {
        const int col = tid + kRThreads * v;
        if (col < hd) pp[2 + col] = o[v];
    }
    if (tid == 0) {
        pp[0] = m_run;
        pp[1] = l_run;
    }
    // the last split of head h to finish merges all of them
    __threadfence();
    __syncthreads();
    const int n_act = pos / kRSplit + 1;
    if (tid == 0) {
        const unsigned prev = atomicAdd(a.done + h, 1u);
        s_last = prev + 1 == (unsigned)n_act;
        if (s_last) a.done[h] = 0;  // every split of this call has arrived: reset for the next
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* ph = a.part + (size_t)h * a.n_splits * (hd + 2);
    for (int j = tid; j < n_act; j += kRThreads) {
        s_m[j] = __ldcg(ph + (size_t)j * (hd + 2));
        s_w[j] = __ldcg(ph + (size_t)j * (hd + 2) + 1);
    }
    __syncthreads();
    float M = -INFINITY;
    for (int j = 0; j < n_act; j++) M = fmaxf(M, s_m[j]);
    float L = 0.0f;
    for (int j = 0; j < n_act; j++) L += s_w[j] * expf(s_m[j] - M);
    __syncthreads();
    for (int j = tid; j < n_act; j += kRThreads) s_w[j] = expf(s_m[j] - M);  // split weights
    __syncthreads();
    for (int i = tid; i < hd; i += kRThreads) {
        float acc = 0.0f;
        for (int j = 0; j < n_act; j++) acc = fmaf(__ldcg(ph + (size_t)j * (hd + 2) + 2 + i), s_w[j], acc);
        a.ao[(size_t)h * hd + i] = acc / L;
    }
}

}  // namespace

namespace rbt {
// Batched decode attention (model_prefill.cu): rows 0..n-1, each one token of its own
// sequence, q|k|v rows of nqkv floats, caches kv_stride floats apart per sequence.
cudaError_t launch_attn_decode_rows(const RbtModel* m, int layer, const Step* steps, const float* qkv, int n,
                                    float* ao, float* part, unsigned* done, cudaStream_t s) {
    const RbtModelConfig& c = m->cfg;
    const int nq = c.n_heads * c.head_dim, nkv = c.n_kv_heads * c.head_dim;
    AttnArgs a{};
    a.qkv = qkv;
    a.q_norm = c.qk_norm ? m->layers[layer].q_norm : nullptr;
    a.k_norm = c.qk_norm ? m->layers[layer].k_norm : nullptr;
    a.eps = c.rms_eps;
    a.scale = 1.0f / sqrtf((float)c.head_dim);
    a.rope_cos = m->rope_cos;
    a.rope_sin = m->rope_sin;
    a.kc = m->kc + (size_t)layer * m->ctx * nkv;
    a.vc = m->vc + (size_t)layer * m->ctx * nkv;
    a.step = steps;
    a.part = part;
    a.ao = ao;
    a.done = done;
    a.status = m->status;
    a.ctx = m->ctx;
    a.n_heads = c.n_heads;
    a.n_kv_heads = c.n_kv_heads;
    a.hd = c.head_dim;
    a.n_splits = m->n_splits;
    a.qkv_stride = nq + 2 * nkv;
    a.kv_stride = (long)c.n_layers * m->ctx * nkv;
    a.part_stride = (long)c.n_heads * m->n_splits * (c.head_dim + 2);
    a.ao_stride = nq;
    if (c.head_dim % 32 == 0) {  // the pipelined kernel: a few CTAs of kRSplit positions per row and head
        const int splits = (m->ctx + kRSplit - 1) / kRSplit;
        attn_rows_kernel<<<dim3(c.n_heads, splits, n), kRThreads, attn_rows_smem_bytes(c.head_dim), s>>>(a);
        return cudaGetLastError();
    }
    attn_decode_kernel<<<dim3(c.n_heads, m->n_splits, n), kAttnThreads, attn_smem_bytes(c.head_dim), s>>>(a);
    return cudaGetLastError();
}
}  // namespace rbt

namespace {

// ---------------------------------------------------------------- launches
// Launch with programmatic stream serialization: each kernel calls
// griddepcontrol.wait before it reads what the previous one wrote.
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

}  // namespace


namespace {

int nq_of(const RbtModelConfig& c) { return c.n_heads * c.head_dim; }
int nkv_of(const RbtModelConfig& c) { return c.n_kv_heads * c.head_dim; }

template <typename T>
int dalloc(T** p, size_t bytes) {
    CU(cudaMalloc((void**)p, bytes));
    return 1;
}

int upload(void** dst, const void* src, size_t bytes) {
    if (!*dst) CU(cudaMalloc(dst, bytes));
    CU(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice));
    return 1;
}

template <typename WT>
int enqueue_token(RbtModel* m, bool with_logits) {
    const RbtModelConfig& c = m->cfg;
    const int D = c.dim, nq = nq_of(c), nkv = nkv_of(c), rows_qkv = nq + 2 * nkv;
    cudaStream_t s = m->stream;
    CU(cudaMemcpyAsync(m->step, m->h_step, sizeof(Step), cudaMemcpyHostToDevice, s));
    CU(launch_pdl(embed_kernel<WT>, dim3((D + 255) / 256), dim3(256), 0, s, (const WT*)m->tok_emb, D,
                  (const Step*)m->step, m->x));
    const int gemv_grid = m->sm_count * kGemvCtasPerSm;
    for (int l = 0; l < c.n_layers; l++) {
        const RbtModel::Layer& L = m->layers[l];
        CU(launch_pdl(norm_gemv_kernel<WT>, dim3(gemv_grid), dim3(kGemvThreads), (size_t)D * 4, s,
                      (const float*)m->x, (const float*)L.attn_norm, c.rms_eps, D, (const WT*)L.wqkv, rows_qkv,
                      m->qkv));
        AttnArgs a{};
        a.qkv = m->qkv;
        a.q_norm = c.qk_norm ? L.q_norm : nullptr;
        a.k_norm = c.qk_norm ? L.k_norm : nullptr;
        a.eps = c.rms_eps;
        a.scale = 1.0f / sqrtf((float)c.head_dim);
        a.rope_cos = m->rope_cos;
        a.rope_sin = m->rope_sin;
        a.kc = m->kc + (size_t)l * m->ctx * nkv;
        a.vc = m->vc + (size_t)l * m->ctx * nkv;
        a.step = m->step;
        a.part = m->part;
        a.ao = m->ao;
        a.done = m->done;
        a.status = m->status;
        a.ctx = m->ctx;
        a.n_heads = c.n_heads;
        a.n_kv_heads = c.n_kv_heads;
        a.hd = c.head_dim;
        a.n_splits = m->n_splits;
        CU(launch_pdl(attn_decode_kernel, dim3(c.n_heads, m->n_splits), dim3(kAttnThreads),
                      attn_smem_bytes(c.head_dim), s, a));
        CU(launch_pdl(out_proj_kernel<WT>, dim3(gemv_grid), dim3(kGemvThreads), (size_t)nq * 4, s, (const float*)m->ao,
                      nq, (const WT*)L.wo, D, m->x));
        if (!rbt::model_moe_block(m, l, m->x, 1, m->routing + (size_t)l * c.top_k, c.top_k, s)) return 0;
    }
    CU(cudaMemcpyAsync(m->h_routing, m->routing, sizeof(int32_t) * c.n_layers * c.top_k, cudaMemcpyDeviceToHost, s));
    CU(cudaMemcpyAsync(m->h_status, m->status, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
    if (unsigned* ms = moe_status_word(m->moe))  // the MoE kernels' status comes back with the token
        CU(cudaMemcpyAsync(m->h_status + 1, ms, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
    if (with_logits) {
        CU(launch_pdl(norm_gemv_kernel<WT>, dim3(gemv_grid), dim3(kGemvThreads), (size_t)D * 4, s,
                      (const float*)m->x, (const float*)m->final_norm, c.rms_eps, D, (const WT*)m->lm_head, c.vocab,
                      m->logits));
        CU(cudaMemcpyAsync(m->h_logits, m->logits, sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, s));
    }
    return 1;
}

int build_graph(RbtModel* m, bool with_logits) {
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    const int ok = m->cfg.dtype == RBT_MOE_DT_BF16 ? enqueue_token<uint16_t>(m, with_logits)
                                                   : enqueue_token<float>(m, with_logits);
    const cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (!ok) {
        if (g) cudaGraphDestroy(g);
        return 0;
    }
    if (e != cudaSuccess) return fail("stream capture of the token failed: %s", cudaGetErrorString(e));
    const cudaError_t ei = cudaGraphInstantiate(&m->graph[with_logits], g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) return fail("graph instantiation failed: %s", cudaGetErrorString(ei));
    return 1;
}

// device state, pinned staging and the RoPE table of a new model
int init_state(RbtModel* m) {
    const RbtModelConfig& c = m->cfg;
    const int ctx = m->ctx;
    cudaDeviceProp prop;
    CU(cudaGetDeviceProperties(&prop, m->device));
    m->sm_count = prop.multiProcessorCount;
    CU(cudaSetDevice(m->device));
    CU(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    const int nq = nq_of(c), nkv = nkv_of(c), half = c.head_dim / 2;
    const size_t kv = (size_t)c.n_layers * ctx * nkv * sizeof(float);
    if (!dalloc(&m->x, (size_t)c.dim * 4) || !dalloc(&m->qkv, (size_t)(nq + 2 * nkv) * 4) ||
        !dalloc(&m->part, (size_t)c.n_heads * m->n_splits * (c.head_dim + 2) * 4) || !dalloc(&m->ao, (size_t)nq * 4) ||
        !dalloc(&m->logits, (size_t)c.vocab * 4) || !dalloc(&m->kc, kv) || !dalloc(&m->vc, kv) ||
        !dalloc(&m->rope_cos, (size_t)ctx * half * 4) || !dalloc(&m->rope_sin, (size_t)ctx * half * 4) ||
        !dalloc(&m->routing, (size_t)c.n_layers * c.top_k * 4) || !dalloc(&m->done, (size_t)c.n_heads * 4) ||
        !dalloc(&m->step, sizeof(Step)) || !dalloc(&m->status, sizeof(unsigned)))
        return 0;
    CU(cudaMemset(m->status, 0, sizeof(unsigned)));
    CU(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)attn_smem_bytes(c.head_dim)));
    if (c.head_dim % 32 == 0)
        CU(cudaFuncSetAttribute(attn_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_rows_smem_bytes(c.head_dim)));
    CU(cudaMemset(m->kc, 0, kv));
    CU(cudaMemset(m->vc, 0, kv));
    CU(cudaMemset(m->done, 0, (size_t)c.n_heads * 4));
    CU(cudaMallocHost((void**)&m->h_step, sizeof(Step)));
    CU(cudaMallocHost((void**)&m->h_logits, (size_t)c.vocab * 4));
    CU(cudaMallocHost((void**)&m->h_routing, (size_t)c.n_layers * c.top_k * 4));
    CU(cudaMallocHost((void**)&m->h_status, 2 * sizeof(unsigned)));  // attention's, the MoE kernels'
    m->h_status[0] = m->h_status[1] = 0;
    // the engine's RoPE angles (rope(), rabbit2.c:410-421): fp64 pow/cos/sin rounded to f32
    std::vector<float> cs((size_t)ctx * half), sn((size_t)ctx * half);
    for (int p = 0; p < ctx; p++)
        for (int i = 0; i < half; i++) {
            const double freq = pow((double)c.rope_theta, -2.0 * i / c.head_dim);
            const double ang = p * freq;
            cs[(size_t)p * half + i] = (float)cos(ang);
            sn[(size_t)p * half + i] = (float)sin(ang);
        }
    CU(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    return rbt_moe_reserve(m->moe, 1);
}

}  // namespace

namespace rbt {
int model_moe_block(RbtModel* m, int l, float* x, int T, int32_t* routing, int routing_stride, cudaStream_t s) {
    if (moe_ep_rows(m->moe)) return rbt_moe_ep_block_device(m->moe, l, x, T, routing, routing_stride, (void*)s);
    return rbt_moe_block_device(m->moe, l, x, T, routing, routing_stride, (void*)s);
}

int model_moe_rows(RbtModel* m, int T) {
    const int ep = moe_ep_rows(m->moe);
    return ep > T ? ep : T;
}

int model_moe_fits(RbtModel* m, int T) {
    const int cap = moe_ep_cap(m->moe);
    if (cap && T > cap) return fail("%d rows above the expert-parallel group's max_tokens %d", T, cap);
    return 1;
}

// The graphs hold device addresses (the KV caches, the MoE workspace, the router
// bias): changing any of them drops the graphs, which are captured again.
void model_drop_graphs(RbtModel* m) {
    for (cudaGraphExec_t& g : m->graph)
        if (g) {
            cudaGraphExecDestroy(g);
            g = nullptr;
        }
}
}  // namespace rbt

extern "C" {

int rbt_model_set_sequences(RbtModel* m, int n_seq) {
    if (!m) return fail("null model");
    if (n_seq < 1) return fail("n_seq must be >= 1 (got %d)", n_seq);
    CU(cudaSetDevice(m->device));
    CU(cudaStreamSynchronize(m->stream));
    const RbtModelConfig& c = m->cfg;
    const size_t kv = (size_t)n_seq * c.n_layers * m->ctx * nkv_of(c) * sizeof(float);
    model_drop_graphs(m);
    cudaFree(m->kc);
    cudaFree(m->vc);
    m->kc = m->vc = nullptr;
    m->n_seq = 0;
    if (!dalloc(&m->kc, kv) || !dalloc(&m->vc, kv)) {
        cudaFree(m->kc);
        m->kc = nullptr;
        return 0;
    }
    CU(cudaMemset(m->kc, 0, kv));
    CU(cudaMemset(m->vc, 0, kv));
    m->n_seq = n_seq;
    return 1;
}

int rbt_model_set_router_bias(RbtModel* m, int layer, const float* bias) {
    if (!m) return fail("null model");
    CU(cudaSetDevice(m->device));
    CU(cudaStreamSynchronize(m->stream));
    model_drop_graphs(m);
    return rbt_moe_set_router_bias(m->moe, layer, bias);
}

RbtMoe* rbt_model_moe(RbtModel* m) { return m ? m->moe : nullptr; }

int rbt_model_create(RbtModel** out, const RbtModelConfig* cfg, int ctx, int device) {
    if (!out || !cfg) return fail("null argument");
    *out = nullptr;
    const RbtModelConfig& c = *cfg;
    if (c.vocab <= 0 || c.dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0)
        return fail("invalid config: dims must be positive");
    if (c.dtype != RBT_MOE_DT_F32 && c.dtype != RBT_MOE_DT_BF16) return fail("dtype must be 0 (f32) or 1 (bf16)");
    if (c.n_heads % c.n_kv_heads) return fail("n_heads %d is not a multiple of n_kv_heads %d", c.n_heads, c.n_kv_heads);
    if (c.head_dim % 4 || c.head_dim > kMaxHeadDim)  // 16-byte runs of the KV cache for the bulk copies
        return fail("head_dim %d must be a multiple of 4 and <= %d", c.head_dim, kMaxHeadDim);
    const int vec = c.dtype == RBT_MOE_DT_BF16 ? 8 : 4;  // elements per 16-byte load
    if (c.dim % vec || nq_of(c) % vec) return fail("dim and n_heads*head_dim must be multiples of %d", vec);
    if (ctx <= 0 || ctx > c.max_seq) return fail("ctx %d out of range [1, max_seq %d]", ctx, c.max_seq);
    if (ctx > kMaxSplits * kSplit) return fail("ctx %d above the supported %d", ctx, kMaxSplits * kSplit);
    if (c.dim > kMaxVec4 * 4 * kGemvThreads || nq_of(c) > kMaxVec4 * 4 * kGemvThreads ||
        nq_of(c) + nkv_of(c) > kAttnVec4 * 4 * kAttnThreads)
        return fail("dim and n_heads*head_dim must be <= %d", kMaxVec4 * 4 * kGemvThreads);
    RbtMoeConfig mc;
    mc.dim = c.dim;
    mc.n_experts = c.n_experts;
    mc.top_k = c.top_k;
    mc.expert_hidden = c.expert_hidden;
    mc.n_layers = c.n_layers;
    mc.dtype = c.dtype;
    mc.norm_topk = c.norm_topk;
    mc.rms_eps = c.rms_eps;
    mc.expert_stride = c.expert_stride;
    RbtMoe* moe = nullptr;
    if (!rbt_moe_create(&moe, &mc, device)) return 0;  // validates the MoE part and the device
    RbtModel* m = new (std::nothrow) RbtModel();
    if (!m) {
        rbt_moe_destroy(moe);
        return fail("out of host memory");
    }
    m->cfg = c;
    m->ctx = ctx;
    m->device = device;
    m->moe = moe;
    m->esz = c.dtype == RBT_MOE_DT_BF16 ? 2 : 4;
    m->layers.resize(c.n_layers);
    m->n_splits = (ctx + kSplit - 1) / kSplit;
    if (!init_state(m)) {
        rbt_model_destroy(m);
        return 0;
    }
    *out = m;
    return 1;
}

void rbt_model_destroy(RbtModel* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    for (cudaGraphExec_t& g : m->graph)
        if (g) cudaGraphExecDestroy(g);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (RbtModel::Layer& L : m->layers) {
        cudaFree(L.attn_norm);
        cudaFree(L.q_norm);
        cudaFree(L.k_norm);
        cudaFree(L.wqkv);
        cudaFree(L.wo);
    }
    cudaFree(m->tok_emb);
    cudaFree(m->lm_head);
    cudaFree(m->final_norm);
    void* bufs[] = {m->x, m->qkv, m->part, m->ao, m->logits, m->kc, m->vc, m->rope_cos, m->rope_sin, m->routing,
                    m->done, m->step, m->status, m->steps, m->dpart, m->ddone, m->dnext};
    for (void* p : bufs) cudaFree(p);
    cudaFreeHost(m->h_step);
    cudaFreeHost(m->h_logits);
    cudaFreeHost(m->h_routing);
    cudaFreeHost(m->h_status);
    cudaFreeHost(m->h_steps);
    rbt::prefill_free(m);
    if (m->stream) cudaStreamDestroy(m->stream);
    rbt_moe_destroy(m->moe);
    delete m;
}

int rbt_model_load_globals(RbtModel* m, const void* tok_emb, const float* final_norm, const void* lm_head) {
    if (!m) return fail("null model");
    if (!tok_emb || !final_norm || !lm_head) return fail("null weight pointer");
    CU(cudaSetDevice(m->device));
    const RbtModelConfig& c = m->cfg;
    const size_t mat = (size_t)c.vocab * c.dim * m->esz;
    if (!upload(&m->tok_emb, tok_emb, mat) || !upload((void**)&m->final_norm, final_norm, (size_t)c.dim * 4) ||
        !upload(&m->lm_head, lm_head, mat))
        return 0;
    m->globals = true;
    return 1;
}

int rbt_model_load_layer(RbtModel* m, int layer, const float* attn_norm, const void* wq, const void* wk,
                         const void* wv, const void* wo, const float* q_norm, const float* k_norm,
                         const float* ffn_norm, const void* router, const void* experts) {
    if (!m) return fail("null model");
    const RbtModelConfig& c = m->cfg;
    if (layer < 0 || layer >= c.n_layers) return fail("layer %d out of range [0, %d)", layer, c.n_layers);
    if (!attn_norm || !wq || !wk || !wv || !wo || !ffn_norm || !router || !experts)
        return fail("null weight pointer");
    if (c.qk_norm && (!q_norm || !k_norm)) return fail("qk_norm is set but q_norm/k_norm is null");
    CU(cudaSetDevice(m->device));
    RbtModel::Layer& L = m->layers[layer];
    const int D = c.dim, nq = nq_of(c), nkv = nkv_of(c);
    const size_t qb = (size_t)nq * D * m->esz, kb = (size_t)nkv * D * m->esz;
    if (!L.wqkv) CU(cudaMalloc(&L.wqkv, qb + 2 * kb));
    uint8_t* w = static_cast<uint8_t*>(L.wqkv);
    CU(cudaMemcpy(w, wq, qb, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(w + qb, wk, kb, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(w + qb + kb, wv, kb, cudaMemcpyHostToDevice));
    if (!upload(&L.wo, wo, (size_t)D * nq * m->esz) || !upload((void**)&L.attn_norm, attn_norm, (size_t)D * 4))
        return 0;
    if (c.qk_norm &&
        (!upload((void**)&L.q_norm, q_norm, (size_t)nq * 4) || !upload((void**)&L.k_norm, k_norm, (size_t)nkv * 4)))
        return 0;
    if (!rbt_moe_load_layer(m->moe, layer, ffn_norm, router, experts)) return 0;
    L.loaded = true;
    return 1;
}

int rbt_model_forward(RbtModel* m, int token, int pos, float* logits, int32_t* routing_out) {
    if (!m) return fail("null model");
    const RbtModelConfig& c = m->cfg;
    if (token < 0 || token >= c.vocab) return fail("token %d out of range", token);
    if (pos < 0 || pos >= m->ctx) return fail("position %d outside the KV cache of %d", pos, m->ctx);
    if (!m->globals) return fail("globals not loaded (rbt_model_load_globals)");
    for (int l = 0; l < c.n_layers; l++)
        if (!m->layers[l].loaded) return fail("layer %d not loaded (rbt_model_load_layer)", l);
    CU(cudaSetDevice(m->device));
    // the graphs hold the MoE workspace's addresses: a larger call since they were
    // captured (rbt_model_prefill) reallocated it, so capture them again
    const unsigned long long gen = moe_workspace_generation(m->moe);
    if (gen != m->graph_gen) {
        model_drop_graphs(m);
        m->graph_gen = gen;
    }
    const int with = logits != nullptr;
    if (!m->graph[with] && !build_graph(m, with)) return 0;
    m->h_step->token = token;
    m->h_step->pos = pos;
    CU(cudaGraphLaunch(m->graph[with], m->stream));
    CU(cudaStreamSynchronize(m->stream));
    if (*m->h_status) {
        const unsigned st = *m->h_status;
        CU(cudaMemset(m->status, 0, sizeof(unsigned)));
        return fail("attention: a bounded wait for the KV tiles ran out (code 0x%x)", st);
    }
    if (m->h_status[1] && !moe_status_ok(m->moe)) return 0;  // (reports and clears it)
    if (logits) memcpy(logits, m->h_logits, sizeof(float) * c.vocab);
    if (routing_out) memcpy(routing_out, m->h_routing, sizeof(int32_t) * c.n_layers * c.top_k);
    return 1;
}

}  // extern "C"
