// router.cu -- K1: router logits, softmax and greedy top-k, plus the permutation
// of routed (token, k) slots by expert.  Replaces rabbit2.c:513-528.
//
// Bit-exactness with the reference's scalar CPU path:
//  * logits: each (token, expert) dot product is four sequential fp32 chains
//    over i = 0,1,2,3 (mod 4), tail folded into chain 0, combined as
//    (s0+s1)+(s2+s3) (rabbit2.c:378-387).  Every product and sum is an explicit
//    __fmul_rn / __fadd_rn: the reference has no FMA, so no contraction here.
//  * softmax: the max, then exp(l - max) rounded to f32, a sequential sum in
//    expert order, then an IEEE division (rabbit2.c:399-405).  exp is taken in
//    double and rounded once, i.e. correctly rounded; glibc's expf equals that
//    except on ~8e-5 of inputs, where the two differ by one ulp.
//  * top-k: K rounds of "largest unused probability, lowest index on ties"
//    (strict '>' scan, rabbit2.c:519-528).
//
// Work split: a CTA computes the logits of a token tile x 8 experts.  The last
// CTA to finish a token tile (atomic counter) runs softmax/top-k for its tokens;
// the last token tile to finish builds the expert permutation.  Counters are
// returned to zero by the CTA that consumed them, so no memset between calls.
#include "common.cuh"
#include "kernels.h"

namespace rbt {
namespace {

constexpr int kThreads = 256;
constexpr int kExpertsPerCta = 8;
constexpr int kSmallTokens = 8;          // token tile of the thread-per-chain kernel
constexpr int kSmallChunk = 2048;        // columns staged per pass (small kernel)
constexpr int kSmallStride = kSmallChunk + 4;  // == 4 (mod 32): conflict-free chain reads
constexpr int kLargeChunk = 128;
constexpr int kLargeStride = kLargeChunk + 4;

template <typename WT>
__device__ __forceinline__ float load_w(const WT* p);
template <>
__device__ __forceinline__ float load_w<uint16_t>(const uint16_t* p) { return bf16_bits_to_f32(*p); }
template <>
__device__ __forceinline__ float load_w<float>(const float* p) { return *p; }

// Stage rows [r0, r0+rows) x columns [c0, c0+cols) of a row-major [*, D] matrix
// into shared memory as f32 (row stride `ss` floats, a multiple of 4).  Rows at
// or past `nrows` are left unwritten: the results that would read them are
// never stored.  16-byte vector loads when the rows allow them.
template <typename T>
__device__ __forceinline__ void stage_rows(float* dst, int ss, const T* src, int D, int r0, int rows, int nrows,
                                           int c0, int cols) {
    constexpr int V = 16 / sizeof(T);
    const int valid = max(0, min(rows, nrows - r0));
    const bool vec = (D % V == 0) && (c0 % V == 0) && (cols % V == 0) &&
                     ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
    if (vec) {
        const int vpr = cols / V;
        for (int i = threadIdx.x; i < valid * vpr; i += blockDim.x) {
            const int r = i / vpr, cv = i - r * vpr;
            const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)(r0 + r) * D + c0 + cv * V);
            float f[V];
            WeightTraits<T>::unpack(v, f);
            float* d = dst + r * ss + cv * V;
#pragma unroll
            for (int q = 0; q < V; q += 4) *reinterpret_cast<float4*>(d + q) = make_float4(f[q], f[q + 1], f[q + 2], f[q + 3]);
        }
    } else {
        for (int i = threadIdx.x; i < valid * cols; i += blockDim.x) {
            const int r = i / cols, c = i - r * cols;
            dst[r * ss + c] = load_w<T>(src + (size_t)(r0 + r) * D + c0 + c);
        }
    }
}

// Softmax + top-k of one token tile, one warp per token (rabbit2.c:514-528).
__device__ void finish_tokens(const RouterArgs& a, int t0, int tcount) {
    __shared__ float s_ex[kThreads / 32][kMaxExperts];
    __shared__ int32_t s_idx[kThreads / 32][kMaxTopK];
    __shared__ float s_w[kThreads / 32][kMaxTopK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = a.E, K = a.K;
    constexpr int NJ = kMaxExperts / 32;
    for (int tl = warp; tl < tcount; tl += kThreads / 32) {
        const int t = t0 + tl;
        float l[NJ];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            l[j] = (e < E) ? __ldcg(a.logits + (size_t)t * E + e) : -INFINITY;
            mx = fmaxf(mx, l[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, o));
        float p[NJ];
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            p[j] = (float)exp((double)__fsub_rn(l[j], mx));
            if (e < E) s_ex[warp][e] = p[j];
        }
        __syncwarp();
        float sum = 0.0f;
        if (lane == 0)
            for (int e = 0; e < E; e++) sum = __fadd_rn(sum, s_ex[warp][e]);
        sum = __shfl_sync(FULL_MASK, sum, 0);
#pragma unroll
        for (int j = 0; j < NJ; j++) p[j] = __fdiv_rn(p[j], sum);
        unsigned used = 0;
        for (int k = 0; k < K; k++) {
            float bp = -INFINITY;
            int be = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < NJ; j++) {
                const int e = lane + 32 * j;
                if (e < E && !((used >> j) & 1u) && (p[j] > bp || be == 0x7fffffff)) {
                    bp = p[j];
                    be = e;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float op = __shfl_xor_sync(FULL_MASK, bp, o);
                const int oe = __shfl_xor_sync(FULL_MASK, be, o);
                if (oe != 0x7fffffff && (be == 0x7fffffff || op > bp || (op == bp && oe < be))) {
                    bp = op;
                    be = oe;
                }
            }
            if ((be & 31) == lane) used |= 1u << (be >> 5);
            if (lane == 0) {
                s_idx[warp][k] = be;
                s_w[warp][k] = bp;
            }
        }
        __syncwarp();
        float wsum = 0.0f;
        for (int k = 0; k < K; k++) wsum = __fadd_rn(wsum, s_w[warp][k]);  // every lane, same order
        for (int k = lane; k < K; k += 32) {
            const float w = a.norm_topk ? __fdiv_rn(s_w[warp][k], wsum) : s_w[warp][k];
            a.idx[(size_t)t * K + k] = s_idx[warp][k];
            a.wt[(size_t)t * K + k] = w;
            if (a.routing_out) a.routing_out[(size_t)t * a.routing_stride + k] = s_idx[warp][k];
        }
        __syncwarp();
    }
}

// Stable counting sort of all T*K slots by expert (one CTA).
__device__ void build_permutation(const RouterArgs& a) {
    __shared__ int32_t s_cnt[kMaxExperts];
    __shared__ int32_t s_base[kMaxExperts];
    __shared__ int32_t s_wcnt[kThreads / 32][kMaxExperts];
    const int E = a.E, S = a.T * a.K;
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int e = tid; e < E; e += kThreads) s_cnt[e] = 0;
    for (int i = tid; i < (kThreads / 32) * kMaxExperts; i += kThreads) (&s_wcnt[0][0])[i] = 0;
    __syncthreads();
    for (int s = tid; s < S; s += kThreads) atomicAdd(&s_cnt[__ldcg(a.idx + s)], 1);
    __syncthreads();
    if (tid == 0) {
        int run = 0, na = 0;
        for (int e = 0; e < E; e++) {
            a.offsets[e] = run;
            s_base[e] = run;
            a.counts[e] = s_cnt[e];
            if (s_cnt[e] > 0) a.active[na++] = e;
            run += s_cnt[e];
        }
        a.offsets[E] = run;
        *a.n_active = na;
    }
    __syncthreads();
    for (int c0 = 0; c0 < S; c0 += kThreads) {
        const int s = c0 + tid;
        const int e = (s < S) ? __ldcg(a.idx + s) : -1;
        const unsigned peers = __match_any_sync(FULL_MASK, e);
        const int rank = __popc(peers & lanemask_lt());
        if (e >= 0 && rank == 0) s_wcnt[warp][e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int pre = 0;
            for (int w = 0; w < warp; w++) pre += s_wcnt[w][e];
            const int pos = s_base[e] + pre + rank;
            a.perm[pos] = s;
            a.slot_pos[s] = pos;
        }
        __syncthreads();
        for (int ee = tid; ee < E; ee += kThreads) {
            int tot = 0;
            for (int w = 0; w < kThreads / 32; w++) {
                tot += s_wcnt[w][ee];
                s_wcnt[w][ee] = 0;
            }
            s_base[ee] += tot;
        }
        __syncthreads();
    }
}

// After this CTA's logits are written: the last CTA of the token tile runs
// softmax/top-k; the last finished tile builds the permutation.
__device__ void tile_epilogue(const RouterArgs& a, int t0, int tcount) {
    __shared__ unsigned s_ticket;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(a.tile_counter + blockIdx.x, 1u);
    __syncthreads();
    if (s_ticket != gridDim.y - 1) return;
    __threadfence();
    finish_tokens(a, t0, tcount);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        a.tile_counter[blockIdx.x] = 0;
        s_ticket = atomicAdd(a.done_counter, 1u);
    }
    __syncthreads();
    if (s_ticket != gridDim.x - 1) return;
    __threadfence();
    build_permutation(a);
    if (threadIdx.x == 0) *a.done_counter = 0;
}

// Small T: one thread per (token, expert, chain): warp = token, lanes = 8
// experts x 4 chains.  Each chain is a sequential run of D/4 multiply-adds.
template <typename WT>
__global__ void __launch_bounds__(kThreads) router_small_kernel(RouterArgs a) {
    extern __shared__ float smem[];
    float* ws = smem;                                   // [8][kSmallStride]
    float* xs = smem + kExpertsPerCta * kSmallStride;   // [8][kSmallStride]
    const int lane = threadIdx.x & 31;
    const int c = lane & 3, el = lane >> 2, tl = threadIdx.x >> 5;
    const int t0 = blockIdx.x * kSmallTokens, e0 = blockIdx.y * kExpertsPerCta;
    const int tcount = min(kSmallTokens, a.T - t0);
    const int D = a.D, D4 = D & ~3;
    const WT* W = static_cast<const WT*>(a.router);
    float s = 0.0f;
    for (int c0 = 0; c0 < D; c0 += kSmallChunk) {
        const int cols = min(kSmallChunk, D - c0);
        __syncthreads();
        stage_rows<WT>(ws, kSmallStride, W, D, e0, kExpertsPerCta, a.E, c0, cols);
        stage_rows<float>(xs, kSmallStride, a.xb, D, t0, kSmallTokens, a.T, c0, cols);
        __syncthreads();
        const float* wr = ws + el * kSmallStride;
        const float* xr = xs + tl * kSmallStride;
        const int main_end = min(cols, D4 - c0);  // columns of this chunk in the 4-chain part
        // eight chain steps per pass: the loads run ahead, the adds keep their order
        int i = c;
        for (; i + 28 < main_end; i += 32) {
            float w[8], x[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                w[u] = wr[i + 4 * u];
                x[u] = xr[i + 4 * u];
            }
#pragma unroll
            for (int u = 0; u < 8; u++) s = __fadd_rn(s, __fmul_rn(w[u], x[u]));
        }
        for (; i < main_end; i += 4) s = __fadd_rn(s, __fmul_rn(wr[i], xr[i]));
        if (c == 0)
            for (int i = max(main_end, 0); i < cols; i++) s = __fadd_rn(s, __fmul_rn(wr[i], xr[i]));
    }
    // (s0 + s1) + (s2 + s3) across the four chain lanes
    const float s1 = __shfl_down_sync(FULL_MASK, s, 1);
    const float a01 = __fadd_rn(s, s1);  // lanes c=0: s0+s1, c=2: s2+s3
    const float a23 = __shfl_down_sync(FULL_MASK, a01, 2);
    const int e = e0 + el, t = t0 + tl;
    if (c == 0 && e < a.E && tl < tcount) {
        float logit = __fadd_rn(a01, a23);
        if (a.bias) logit = __fadd_rn(logit, a.bias[e]);
        a.logits[(size_t)t * a.E + e] = logit;
    }
    tile_epilogue(a, t0, tcount);
}

// Larger T: one thread per (expert, token group) holding all four chains for
// J tokens; tokens of a tile are tg + 32*j.
template <typename WT, int J>
__global__ void __launch_bounds__(kThreads) router_large_kernel(RouterArgs a) {
    extern __shared__ float smem[];
    float* ws = smem;                                   // [8][kLargeStride]
    float* xs = smem + kExpertsPerCta * kLargeStride;   // [32*J][kLargeStride]
    constexpr int TT = 32 * J;
    const int el = threadIdx.x & 7, tg = threadIdx.x >> 3;
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * kExpertsPerCta;
    const int tcount = min(TT, a.T - t0);
    const int D = a.D, D4 = D & ~3;
    const WT* W = static_cast<const WT*>(a.router);
    float acc[J][4];
#pragma unroll
    for (int j = 0; j < J; j++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc[j][q] = 0.0f;
    for (int c0 = 0; c0 < D; c0 += kLargeChunk) {
        const int cols = min(kLargeChunk, D - c0);
        __syncthreads();
        stage_rows<WT>(ws, kLargeStride, W, D, e0, kExpertsPerCta, a.E, c0, cols);
        stage_rows<float>(xs, kLargeStride, a.xb, D, t0, TT, a.T, c0, cols);
        __syncthreads();
        const float* wr = ws + el * kLargeStride;
        const int main_end = max(0, min(cols, D4 - c0));
        for (int i = 0; i < main_end; i += 4) {
            const float4 w = *reinterpret_cast<const float4*>(wr + i);
#pragma unroll
            for (int j = 0; j < J; j++) {
                const float4 x = *reinterpret_cast<const float4*>(xs + (tg + 32 * j) * kLargeStride + i);
                acc[j][0] = __fadd_rn(acc[j][0], __fmul_rn(w.x, x.x));
                acc[j][1] = __fadd_rn(acc[j][1], __fmul_rn(w.y, x.y));
                acc[j][2] = __fadd_rn(acc[j][2], __fmul_rn(w.z, x.z));
                acc[j][3] = __fadd_rn(acc[j][3], __fmul_rn(w.w, x.w));
            }
        }
        for (int i = main_end; i < cols; i++)
#pragma unroll
            for (int j = 0; j < J; j++)
                acc[j][0] = __fadd_rn(acc[j][0], __fmul_rn(wr[i], xs[(tg + 32 * j) * kLargeStride + i]));
    }
    const int e = e0 + el;
#pragma unroll
    for (int j = 0; j < J; j++) {
        const int tl = tg + 32 * j;
        if (e < a.E && tl < tcount) {
            float logit = __fadd_rn(__fadd_rn(acc[j][0], acc[j][1]), __fadd_rn(acc[j][2], acc[j][3]));
            if (a.bias) logit = __fadd_rn(logit, a.bias[e]);
            a.logits[(size_t)(t0 + tl) * a.E + e] = logit;
        }
    }
    tile_epilogue(a, t0, tcount);
}

template <typename KernelT>
cudaError_t launch_with_smem(KernelT kernel, dim3 grid, size_t smem, const RouterArgs& a, cudaStream_t s) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    kernel<<<grid, kThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <typename WT>
cudaError_t launch_typed(const RouterArgs& a, cudaStream_t s) {
    const int egroups = (a.E + kExpertsPerCta - 1) / kExpertsPerCta;
    if (a.T <= kSmallTokens) {
        const size_t smem = 2ull * kExpertsPerCta * kSmallStride * sizeof(float);
        return launch_with_smem(router_small_kernel<WT>, dim3(1, egroups), smem, a, s);
    }
    auto grid_for = [&](int tt) { return dim3((a.T + tt - 1) / tt, egroups); };
    if (a.T >= 2048) {
        const size_t smem = (size_t)(kExpertsPerCta + 128) * kLargeStride * sizeof(float);
        return launch_with_smem(router_large_kernel<WT, 4>, grid_for(128), smem, a, s);
    }
    if (a.T >= 512) {
        const size_t smem = (size_t)(kExpertsPerCta + 64) * kLargeStride * sizeof(float);
        return launch_with_smem(router_large_kernel<WT, 2>, grid_for(64), smem, a, s);
    }
    const size_t smem = (size_t)(kExpertsPerCta + 32) * kLargeStride * sizeof(float);
    return launch_with_smem(router_large_kernel<WT, 1>, grid_for(32), smem, a, s);
}

}  // namespace

// Token tiles the router grid uses for T tokens (sizes the tile counters).
int router_token_tiles(int T) {
    if (T <= kSmallTokens) return 1;
    const int tt = T >= 2048 ? 128 : (T >= 512 ? 64 : 32);
    return (T + tt - 1) / tt;
}

cudaError_t launch_router(const RouterArgs& a, cudaStream_t s) {
    if (a.T <= 0) return cudaSuccess;
    return a.dtype == 1 ? launch_typed<uint16_t>(a, s) : launch_typed<float>(a, s);
}

}  // namespace rbt
