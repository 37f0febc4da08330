// router.cu -- K1: router logits, softmax and greedy top-k, plus the permutation
// of routed (token, k) slots by expert.  Replaces rabbit2.c:513-528.
//
// Bit-exactness with the reference's scalar CPU path:
//  * logits: each (token, expert) dot product is four sequential fp32 chains
//    over i = 0,1,2,3 (mod 4), tail folded into chain 0, combined as
//    (s0+s1)+(s2+s3) (rabbit2.c:378-387).  Every product and sum is an explicit
//    __fmul_rn / __fadd_rn: the reference has no FMA, so no contraction here.
//  * softmax: the max, then expf(l - max), a sequential sum in expert order,
//    then an IEEE division (rabbit2.c:399-405).  expf is the host libm's own
//    method, bit for bit (expf_ref, exact_math.cuh).
//  * the block form's rmsnorm (rabbit2.c:392-397): the sum of squares is the
//    reference's sequential f32 sum, reproduced exactly (block_seq_sum).
//  * top-k: K rounds of "largest unused probability, lowest index on ties"
//    (strict '>' scan, rabbit2.c:519-528).
//
// Work split: a CTA computes the logits of a token tile x 8 experts.  The last
// CTA to finish a token tile (atomic counter) runs softmax/top-k for its tokens;
// the last token tile to finish builds the expert permutation.  Counters are
// returned to zero by the CTA that consumed them, so no memset between calls.
#include <stdlib.h>

#include <math.h>
#include <stdio.h>

#include "common.cuh"
#include "exact_math.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rbt {

int host_expf_fma() {
    static int variant = -1;
    if (variant < 0) {
        // expf(-0x1.f8cbb2p+5) is one of the two floats on which the contracted
        // and the separately rounded evaluations differ
        volatile float x = -0x1.f8cbb2p+5f;
        const float y = expf(x);
        if (y == 0x1.f45326p-92f) {
            variant = 1;
        } else if (y == 0x1.f45324p-92f) {
            variant = 0;
        } else {
            fprintf(stderr, "rbt_moe: this libm's expf(%a) = %a is not the table method's; routing can differ "
                            "from the host engine where two probabilities are within an ulp\n", (double)x, (double)y);
            variant = 1;
        }
    }
    return variant;
}

namespace {

using namespace tc;

#ifdef RBT_ROUTER_TIMELINE
// Optional phase timestamps (%globaltimer) of every CTA of the last launch, read
// back with rbt_router_timeline_read(); built only with -DRBT_ROUTER_TIMELINE.
__device__ unsigned long long g_rtl[4096][16];
#define RTL(i)                                                                                \
    do {                                                                                      \
        if (threadIdx.x == 0) {                                                               \
            const unsigned cta_ = blockIdx.y * gridDim.x + blockIdx.x;                        \
            unsigned long long t_;                                                            \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                            \
            if (cta_ < 4096) g_rtl[cta_][i] = t_;                                             \
        }                                                                                     \
    } while (0)
#else
#define RTL(i) \
    do {       \
    } while (0)
#endif

constexpr int kThreads = 256;
constexpr int kExpertsPerCta = 8;
constexpr int kSmallTokens = 8;          // token tile of the thread-per-chain kernel
constexpr int kMidTokens = 256;          // the thread-per-chain kernel up to this many tokens
constexpr int kSmallChunk = 1024;        // columns staged per pass (small kernel): 66 KB, 3 CTAs per SM
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
// never stored.  Each thread issues up to 8 independent 16-byte loads before
// converting and storing, so a chunk costs one memory latency, not eight.
template <typename T>
__device__ __forceinline__ void stage_rows(float* dst, int ss, const T* src, int D, int r0, int rows, int nrows,
                                           int c0, int cols) {
    constexpr int V = 16 / sizeof(T);
    constexpr int B = 8;
    const int valid = max(0, min(rows, nrows - r0));
    const bool vec = (D % V == 0) && (c0 % V == 0) && (cols % V == 0) &&
                     ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
    if (vec) {
        const int vpr = cols / V, n = valid * vpr;
        for (int base = threadIdx.x; base < n; base += blockDim.x * B) {
            uint4 v[B];
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int i = base + b * blockDim.x;
                if (i < n) {
                    const int r = i / vpr, cv = i - r * vpr;
                    v[b] = *reinterpret_cast<const uint4*>(src + (size_t)(r0 + r) * D + c0 + cv * V);
                }
            }
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int i = base + b * blockDim.x;
                if (i < n) {
                    const int r = i / vpr, cv = i - r * vpr;
                    float f[V];
                    WeightTraits<T>::unpack(v[b], f);
                    float* d = dst + r * ss + cv * V;
#pragma unroll
                    for (int q = 0; q < V; q += 4)
                        *reinterpret_cast<float4*>(d + q) = make_float4(f[q], f[q + 1], f[q + 2], f[q + 3]);
                }
            }
        }
    } else {
        for (int i = threadIdx.x; i < valid * cols; i += blockDim.x) {
            const int r = i / cols, c = i - r * cols;
            dst[r * ss + c] = load_w<T>(src + (size_t)(r0 + r) * D + c0 + c);
        }
    }
}

// Exclusive prefix sum over the 256 threads of a CTA (all threads call it).
__device__ __forceinline__ int block_exclusive_scan(int v, int* total) {
    __shared__ int s_warp[kThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(FULL_MASK, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    int base = 0, all = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; w++) {
        base += (w < warp) ? s_warp[w] : 0;
        all += s_warp[w];
    }
    __syncthreads();
    if (total) *total = all;
    return base + incl - v;
}

// Softmax + top-k of one token, by one warp (rabbit2.c:514-528).  `lrow` holds
// the E logits (shared or global memory; kGlobal reads bypass L1 because other
// CTAs wrote them).  Writes idx/wt/routing_out of token t and leaves the chosen
// experts in s_idx[0..K).
template <int NJ, bool kGlobal>
__device__ void topk_token(const RouterArgs& a, const float* lrow, int t, float* s_ex, int32_t* s_idx, float* s_w) {
    const int lane = threadIdx.x & 31;
    const int E = a.E, K = a.K;
    float l[NJ];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int e = lane + 32 * j;
        l[j] = (e < E) ? (kGlobal ? __ldcg(lrow + e) : lrow[e]) : -INFINITY;
        mx = fmaxf(mx, l[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, o));
    float p[NJ];
    const uint64_t tab = expf_tab_lane();
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int e = lane + 32 * j;
        const float v = expf_ref_warp(e < E ? __fsub_rn(l[j], mx) : 0.0f, a.expf_fma, tab);
        p[j] = (e < E) ? v : 0.0f;
        if (e < E) s_ex[e] = p[j];
    }
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0)
        for (int e = 0; e < E; e++) sum = __fadd_rn(sum, s_ex[e]);
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
            s_idx[k] = be;
            s_w[k] = bp;
        }
    }
    __syncwarp();
    float wsum = 0.0f;
    for (int k = 0; k < K; k++) wsum = __fadd_rn(wsum, s_w[k]);  // every lane, same order
    for (int k = lane; k < K; k += 32) {
        const float w = a.norm_topk ? __fdiv_rn(s_w[k], wsum) : s_w[k];
        a.idx[(size_t)t * K + k] = s_idx[k];
        a.wt[(size_t)t * K + k] = w;
        if (a.routing_out) a.routing_out[(size_t)t * a.routing_stride + k] = s_idx[k];
    }
    __syncwarp();
}

// Softmax + top-k of a token tile whose logits other CTAs wrote, one warp per token.
__device__ void finish_tokens(const RouterArgs& a, int t0, int tcount) {
    __shared__ float s_ex[kThreads / 32][kMaxExperts];
    __shared__ int32_t s_idx[kThreads / 32][kMaxTopK];
    __shared__ float s_w[kThreads / 32][kMaxTopK];
    const int warp = threadIdx.x >> 5;
    for (int tl = warp; tl < tcount; tl += kThreads / 32)
        topk_token<kMaxExperts / 32, true>(a, a.logits + (size_t)(t0 + tl) * a.E, t0 + tl, s_ex[warp], s_idx[warp],
                                           s_w[warp]);
}

// Given this thread's expert count (thread e, e < E), write counts, offsets,
// the active-expert list and n_active; optionally keep the offsets in s_off.
__device__ void publish_offsets(const RouterArgs& a, int cnt, int* s_off) {
    const int e = threadIdx.x;
    int total = 0;
    const int off = block_exclusive_scan(cnt, &total);
    int n_act = 0;
    const int apos = block_exclusive_scan(cnt > 0 ? 1 : 0, &n_act);
    if (e < a.E) {
        a.offsets[e] = off;
        a.counts[e] = cnt;
        if (cnt > 0) a.active[apos] = e;
        if (s_off) s_off[e] = off;
    }
    if (e == 0) {
        a.offsets[a.E] = total;
        *a.n_active = n_act;
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
    publish_offsets(a, tid < E ? s_cnt[tid] : 0, s_base);
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

__device__ void rank_tile_slots(const RouterArgs& a, const int32_t* s_eidx, int nslots, int slot0, int tile);
__device__ void finish_tiles(const RouterArgs& a, int ntiles);

// After this CTA's logits are written: the last CTA of the token tile runs
// softmax/top-k for its tokens.  With one token tile the same CTA then builds
// the permutation; with several (a.tile_tokens set), each tile ranks its slots
// per expert, the last tile turns the tile counts into offsets and tile bases,
// and scatter_kernel places the slots.
__device__ void tile_epilogue(const RouterArgs& a, int t0, int tcount) {
    __shared__ unsigned s_ticket;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(a.tile_counter + blockIdx.x, 1u);
    __syncthreads();
    RTL(3);
    if (s_ticket != gridDim.y - 1) return;
    __threadfence();
    finish_tokens(a, t0, tcount);
    RTL(4);
    if (a.tile_tokens > 0 && gridDim.x > 1) {
        __shared__ int32_t s_eidx[kSmallTokens * kMaxTopK];
        __syncthreads();
        for (int i = threadIdx.x; i < tcount * a.K; i += kThreads) s_eidx[i] = a.idx[(size_t)t0 * a.K + i];
        __syncthreads();
        rank_tile_slots(a, s_eidx, tcount * a.K, t0 * a.K, blockIdx.x);
        RTL(5);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            a.tile_counter[blockIdx.x] = 0;
            s_ticket = atomicAdd(a.done_counter, 1u);
        }
        __syncthreads();
        RTL(6);
        if (s_ticket != gridDim.x - 1) return;
        __threadfence();
        finish_tiles(a, gridDim.x);
        RTL(7);
        return;
    }
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
    RTL(0);
    for (int c0 = 0; c0 < D; c0 += kSmallChunk) {
        const int cols = min(kSmallChunk, D - c0);
        __syncthreads();
        stage_rows<WT>(ws, kSmallStride, W, D, e0, kExpertsPerCta, a.E, c0, cols);
        stage_rows<float>(xs, kSmallStride, a.xb, D, t0, kSmallTokens, a.T, c0, cols);
        __syncthreads();
        if (c0 == 0) RTL(1);
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
    RTL(2);
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

// ---------------------------------------------------------------------------
// Wide router (E <= 64, D % 4 == 0, T > 8): one CTA holds every expert for a
// tile of 16 tokens, so softmax/top-k need no other CTA.  Thread (e, g) keeps
// the four chains of expert e for tokens g, g+4, g+8, g+12 (scalar __fmul_rn /
// __fadd_rn: packed f32x2 chains measured 1-4 ulp away from the reference's
// logits on most tokens, so they are not used).  Router-weight and activation
// chunks of 128 columns are double-buffered in shared memory with cp.async.
// Each tile then ranks its routed slots per expert (stable) and publishes its
// per-expert counts; the last tile turns the counts into expert offsets and
// per-tile bases, and scatter_kernel places every slot.
constexpr int kWideTokens = 16;
constexpr int kWideChunk = 128;
constexpr int kWideExperts = 64;
constexpr int kWideXStride = kWideChunk + 4;  // floats: 528-byte rows (16-byte aligned)


__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename WT>
struct WideCfg {
    // router rows in shared memory: 128 elements + a skew that staggers rows by
    // two banks (bf16) / four banks (f32) so a warp's 32 experts read conflict-free
    static constexpr int kWStride = kWideChunk + (sizeof(WT) == 2 ? 4 : 4);
    static constexpr int kWBytes = kWideExperts * kWStride * (int)sizeof(WT);
    static constexpr int kXBytes = kWideTokens * kWideXStride * 4;
    static constexpr int kStageBytes = kWBytes + kXBytes;
    static constexpr int kSmem = 2 * kStageBytes;
};

// Stable per-tile ranking of routed slots by expert; writes slot_rank[] and the
// tile's per-expert counts.  s_eidx: the tile's chosen experts, slot order.
__device__ void rank_tile_slots(const RouterArgs& a, const int32_t* s_eidx, int nslots, int slot0, int tile) {
    __shared__ int32_t s_cnt[kMaxExperts];
    __shared__ int32_t s_wcnt[kThreads / 32][kMaxExperts];
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int e = tid; e < a.E; e += kThreads) s_cnt[e] = 0;
    for (int i = tid; i < (kThreads / 32) * kMaxExperts; i += kThreads) (&s_wcnt[0][0])[i] = 0;
    __syncthreads();
    for (int c0 = 0; c0 < nslots; c0 += kThreads) {
        const int sl = c0 + tid;
        const int e = (sl < nslots) ? s_eidx[sl] : -1;
        const unsigned peers = __match_any_sync(FULL_MASK, e);
        const int rank = __popc(peers & lanemask_lt());
        if (e >= 0 && rank == 0) s_wcnt[warp][e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int pre = s_cnt[e];
            for (int w = 0; w < warp; w++) pre += s_wcnt[w][e];
            a.slot_rank[slot0 + sl] = pre + rank;
        }
        __syncthreads();
        for (int ee = tid; ee < a.E; ee += kThreads) {
            int tot = 0;
            for (int w = 0; w < kThreads / 32; w++) {
                tot += s_wcnt[w][ee];
                s_wcnt[w][ee] = 0;
            }
            s_cnt[ee] += tot;
        }
        __syncthreads();
    }
    for (int e = tid; e < a.E; e += kThreads) a.tile_cnt[(size_t)tile * a.E + e] = s_cnt[e];
}

// Run by the last token tile: per-expert totals (counts, offsets, active list)
// and every tile's first position per expert.
__device__ void finish_tiles(const RouterArgs& a, int ntiles) {
    const int tid = threadIdx.x, E = a.E;
    // thread (pe, part) owns the contiguous tile range [part*n/P, (part+1)*n/P) of
    // expert pe (P = 256 / E parts, 1 to 4); the per-tile counts are read 32 loads
    // at a time, since L2 latency (not bandwidth) is the cost of this single-CTA step
    constexpr int kMaxParts = 4;
    constexpr int kFinLd = 32;
    __shared__ int s_part[kMaxParts][kMaxExperts];
    __shared__ int s_off[kMaxExperts];
    const int P = max(1, min(kMaxParts, kThreads / E));
    const int pe = tid % E, part = tid / E;
    const bool mine = part < P;
    const int tb0 = (int)((long)part * ntiles / P), tb1 = (int)((long)(part + 1) * ntiles / P);
    int psum = 0;
    if (mine)
        for (int t = tb0; t < tb1; t += kFinLd) {
            int c[kFinLd];
#pragma unroll
            for (int k = 0; k < kFinLd; k++) c[k] = t + k < tb1 ? __ldcg(a.tile_cnt + (size_t)(t + k) * E + pe) : 0;
#pragma unroll
            for (int k = 0; k < kFinLd; k++) psum += c[k];
        }
    if (mine) s_part[part][pe] = psum;
    __syncthreads();
    int tot = 0;
    if (tid < E)
        for (int p = 0; p < P; p++) tot += s_part[p][tid];
    publish_offsets(a, tot, s_off);
    __syncthreads();
    if (mine) {
        int run = s_off[pe];
        for (int p = 0; p < part; p++) run += s_part[p][pe];
        for (int t = tb0; t < tb1; t += kFinLd) {
            int c[kFinLd];
#pragma unroll
            for (int k = 0; k < kFinLd; k++) c[k] = t + k < tb1 ? __ldcg(a.tile_cnt + (size_t)(t + k) * E + pe) : 0;
#pragma unroll
            for (int k = 0; k < kFinLd; k++)
                if (t + k < tb1) {
                    a.tile_base[(size_t)(t + k) * E + pe] = run;
                    run += c[k];
                }
        }
    }
    if (tid == 0) *a.done_counter = 0;
}

template <typename WT>
__global__ void __launch_bounds__(kThreads) router_wide_kernel(RouterArgs a) {
    using C = WideCfg<WT>;
    extern __shared__ __align__(16) uint8_t wsmem[];
    __shared__ float s_logit[kWideTokens][kWideExperts];
    __shared__ float s_ex[kThreads / 32][kWideExperts];
    __shared__ float s_w[kThreads / 32][kMaxTopK];
    __shared__ int32_t s_eidx[kWideTokens * kMaxTopK];
    const int tid = threadIdx.x;
    const int e = tid & 63, g = tid >> 6;
    const int t0 = blockIdx.x * kWideTokens;
    const int tcount = min(kWideTokens, a.T - t0);
    const int D = a.D, E = a.E;
    const WT* W = static_cast<const WT*>(a.router);
    const int nch = (D + kWideChunk - 1) / kWideChunk;

    auto issue = [&](int ch, int buf) {
        uint8_t* st = wsmem + buf * C::kStageBytes;
        WT* ws = reinterpret_cast<WT*>(st);
        float* xs = reinterpret_cast<float*>(st + C::kWBytes);
        const int c0 = ch * kWideChunk, cols = min(kWideChunk, D - c0);
        if (sizeof(WT) == 2) {  // 4 bf16 = 8 bytes per copy
            const int per_row = cols / 4;
            for (int i = tid; i < E * per_row; i += kThreads) {
                const int r = i / per_row, q = i - r * per_row;
                cp_async8(ws + r * C::kWStride + q * 4, W + (size_t)r * D + c0 + q * 4);
            }
        } else {  // 4 f32 = 16 bytes per copy
            const int per_row = cols / 4;
            for (int i = tid; i < E * per_row; i += kThreads) {
                const int r = i / per_row, q = i - r * per_row;
                cp_async16(ws + r * C::kWStride + q * 4, W + (size_t)r * D + c0 + q * 4);
            }
        }
        const int per_row = cols / 4;
        for (int i = tid; i < tcount * per_row; i += kThreads) {
            const int r = i / per_row, q = i - r * per_row;
            cp_async16(xs + r * kWideXStride + q * 4, a.xb + (size_t)(t0 + r) * D + c0 + q * 4);
        }
        cp_async_commit();
    };

    // the four chains of 4 tokens, separately rounded products and sums (__fmul_rn /
    // __fadd_rn are never contracted into an FMA)
    float c0[4], c1[4], c2[4], c3[4];
#pragma unroll
    for (int j = 0; j < 4; j++) c0[j] = c1[j] = c2[j] = c3[j] = 0.0f;
    issue(0, 0);
    for (int ch = 0; ch < nch; ch++) {
        if (ch + 1 < nch) {
            issue(ch + 1, (ch + 1) & 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint8_t* st = wsmem + (ch & 1) * C::kStageBytes;
        const WT* wr = reinterpret_cast<const WT*>(st) + e * C::kWStride;
        const float* xs = reinterpret_cast<const float*>(st + C::kWBytes);
        const int cols = min(kWideChunk, D - ch * kWideChunk);
        if (e < E) {
#pragma unroll 4
            for (int i = 0; i < cols; i += 4) {
                float w0, w1, w2, w3;
                if (sizeof(WT) == 2) {
                    const uint2 q = *reinterpret_cast<const uint2*>(wr + i);
                    w0 = __uint_as_float(q.x << 16);
                    w1 = __uint_as_float(q.x & 0xffff0000u);
                    w2 = __uint_as_float(q.y << 16);
                    w3 = __uint_as_float(q.y & 0xffff0000u);
                } else {
                    const float4 q = *reinterpret_cast<const float4*>(wr + i);
                    w0 = q.x; w1 = q.y; w2 = q.z; w3 = q.w;
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float4 x = *reinterpret_cast<const float4*>(xs + (g + 4 * j) * kWideXStride + i);
                    c0[j] = __fadd_rn(c0[j], __fmul_rn(w0, x.x));
                    c1[j] = __fadd_rn(c1[j], __fmul_rn(w1, x.y));
                    c2[j] = __fadd_rn(c2[j], __fmul_rn(w2, x.z));
                    c3[j] = __fadd_rn(c3[j], __fmul_rn(w3, x.w));
                }
            }
        }
        __syncthreads();
    }
    if (e < E) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int tl = g + 4 * j;
            float logit = __fadd_rn(__fadd_rn(c0[j], c1[j]), __fadd_rn(c2[j], c3[j]));
            if (a.bias) logit = __fadd_rn(logit, a.bias[e]);
            s_logit[tl][e] = logit;
            if (t0 + tl < a.T) a.logits[(size_t)(t0 + tl) * E + e] = logit;
        }
    }
    __syncthreads();
    const int warp = tid >> 5;
    for (int tl = warp; tl < tcount; tl += kThreads / 32)
        topk_token<2, false>(a, s_logit[tl], t0 + tl, s_ex[warp], s_eidx + tl * a.K, s_w[warp]);
    __syncthreads();
    rank_tile_slots(a, s_eidx, tcount * a.K, t0 * a.K, blockIdx.x);

    // the last tile to finish turns per-tile counts into offsets and tile bases
    __shared__ unsigned s_ticket;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_ticket = atomicAdd(a.done_counter, 1u);
    __syncthreads();
    if (s_ticket != gridDim.x - 1) return;
    __threadfence();
    finish_tiles(a, gridDim.x);
}

// Places every routed slot of a tile: position = tile base of its expert + its
// stable rank within the tile.
__global__ void __launch_bounds__(kThreads) scatter_kernel(RouterArgs a) {
    RTL(14);
    const int t0 = blockIdx.x * a.tile_tokens;
    const int nslots = min(a.tile_tokens, a.T - t0) * a.K;
    for (int sl = threadIdx.x; sl < nslots; sl += kThreads) {
        const int s = t0 * a.K + sl;
        const int e = a.idx[s];
        if (e < 0 || e >= a.E) {  // a slot computed on another GPU (expert parallelism)
            a.slot_pos[s] = -1;
            continue;
        }
        const int pos = a.tile_base[(size_t)blockIdx.x * a.E + e] + a.slot_rank[s];
        a.perm[pos] = s;
        a.slot_pos[s] = pos;
    }
    RTL(15);
}

// The permutation of routing that comes from outside (expert parallelism): a.idx
// holds expert ids of this GPU's range, or -1 for slots other GPUs compute.  Tiles
// of 16 tokens rank their slots per expert; the last tile computes offsets and
// tile bases; scatter_kernel places the slots (and marks the others -1).
__global__ void __launch_bounds__(kThreads) route_given_kernel(RouterArgs a) {
    __shared__ int32_t s_eidx[kWideTokens * kMaxTopK];
    const int t0 = blockIdx.x * kWideTokens;
    const int nslots = min(kWideTokens, a.T - t0) * a.K;
    for (int i = threadIdx.x; i < nslots; i += kThreads) {
        const int e = a.idx[(size_t)t0 * a.K + i];
        s_eidx[i] = (e >= 0 && e < a.E) ? e : -1;
    }
    __syncthreads();
    rank_tile_slots(a, s_eidx, nslots, t0 * a.K, blockIdx.x);
    __shared__ unsigned s_ticket;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_ticket = atomicAdd(a.done_counter, 1u);
    __syncthreads();
    if (s_ticket != gridDim.x - 1) return;
    __threadfence();
    finish_tiles(a, gridDim.x);
}

// ---------------------------------------------------------------------------
// Token router (bf16, E <= 64, D % 256 == 0, 2 <= T <= 256): one
// CTA per token holds all E x 4 chains, so softmax and top-k need no other CTA,
// and the last CTA builds the whole permutation.  Thread 4e + c runs chain c of
// expert e.  The router is read from a chain-major copy made when the layer is
// bound (router_to_chain_major): group g of 8 consecutive chain elements of
// every (e, c) is one 16-byte piece, and all 4E pieces of a group are adjacent,
//   cm[((g * E + e) * 4 + c) * 8 + u] = W[e][c + 4 (8 g + u)],
// so a warp reads 512 contiguous bytes per group and a chunk of kTokGroups
// groups is one contiguous bulk copy.  Chunks stream through a 3-slot ring.
constexpr int kTokMaxE = 64;
constexpr int kTokGroups = 8;           // 16-byte groups per chunk: 64 chain elements
constexpr int kTokBufs = 3;
constexpr int kTokMaxTokens = 256;
constexpr uint64_t kTokWaitNs = 2000000000ull;

__host__ __device__ inline size_t tok_chunk_bytes(int E) { return (size_t)kTokGroups * E * 4 * 16; }
__host__ __device__ inline size_t tok_smem_bytes(int D, int E) {
    const size_t x = (size_t)4 * (D / 4 + 4) * sizeof(float);
    const size_t ring = kTokBufs * tok_chunk_bytes(E);
    // the last CTA's permutation tables: masks, slot k per (token, expert), part counts, offsets
    const size_t stage = (size_t)kTokMaxTokens * sizeof(uint64_t) + (size_t)kTokMaxTokens * kTokMaxE +
                         (size_t)(kThreads + kTokMaxE) * sizeof(int);
    return (ring > stage ? ring : stage) + x;
}

__global__ void router_cm_kernel(const uint16_t* w, int E, int D, uint16_t* cm) {
    const size_t n = (size_t)E * D;
    for (size_t o = (size_t)blockIdx.x * blockDim.x + threadIdx.x; o < n; o += (size_t)gridDim.x * blockDim.x) {
        const int u = (int)(o & 7), c = (int)((o >> 3) & 3);
        const size_t ge = o >> 5;  // g * E + e
        const int e = (int)(ge % E), g = (int)(ge / E);
        cm[o] = w[(size_t)e * D + c + 4 * (8 * g + u)];
    }
}

__global__ void __launch_bounds__(kThreads) router_tok_kernel(RouterArgs a) {
    extern __shared__ __align__(128) uint8_t tsm[];
    __shared__ uint64_t full[kTokBufs];
    __shared__ float s_logit[kTokMaxE];
    __shared__ __align__(16) float s_prob[kTokMaxE];
    __shared__ float s_red[kThreads / 32];
    __shared__ int s_cnt[kThreads / 32];
    __shared__ int32_t s_idx[kMaxTopK];
    __shared__ float s_p[kMaxTopK];
    __shared__ unsigned long long s_seen;
    __shared__ unsigned s_ticket;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t = blockIdx.x, D = a.D, E = a.E, K = a.K, T = a.T;
    const int q4 = D / 4, nq = D / (32 * kTokGroups), xs = q4 + 4;
    const size_t cbytes = tok_chunk_bytes(E), celems = cbytes / 2;
    uint16_t* ring = reinterpret_cast<uint16_t*>(tsm);
    float* xcm = reinterpret_cast<float*>(tsm + (tok_smem_bytes(D, E) - (size_t)4 * xs * sizeof(float)));
    const uint16_t* cm = a.router_cm;
    int n_issued = 0;  // copies issued (thread 0)
    RTL(0);
    if (tid == 0) {
        s_seen = 0ull;
        for (int b = 0; b < kTokBufs; b++) mbar_init(&full[b], 1);
        fence_mbar_init();
        for (int q = 0; q < nq && q < kTokBufs; q++) {
            mbar_arrive_expect_tx(&full[q], (uint32_t)cbytes);
            bulk_load(ring + (size_t)q * celems, cm + (size_t)q * celems, (uint32_t)cbytes, &full[q]);
            n_issued++;
        }
    }
    // the block form's rmsnorm of this token (rabbit2.c:512): the sum of squares
    // is the reference's sequential f32 sum (block_seq_sum; the squares are staged
    // in the xcm area, which then receives xb); xb is also written for the kernels
    // that follow
    float inv = 1.0f;
    if (a.norm_w) {
        __shared__ SeqSumSmem s_seq;
        const float4* xr4 = reinterpret_cast<const float4*>(a.x_raw + (size_t)t * D);
        for (int i4 = tid; i4 < q4; i4 += kThreads) {
            const float4 v = xr4[i4];
            reinterpret_cast<float4*>(xcm)[i4] =
                make_float4(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y), __fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w));
        }
        __syncthreads();
        const float ss = block_seq_sum<kThreads>(xcm, D, s_seq);
        inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), a.eps));
    }
    // this token's xb, chain-major: xcm[c][j] = xb[t][c + 4 j] (rows 4 banks apart)
    for (int i4 = tid; i4 < q4; i4 += kThreads) {
        float4 v;
        if (a.norm_w) {
            const float4 x = reinterpret_cast<const float4*>(a.x_raw + (size_t)t * D)[i4];
            const float4 w = reinterpret_cast<const float4*>(a.norm_w)[i4];
            v = make_float4(__fmul_rn(__fmul_rn(x.x, inv), w.x), __fmul_rn(__fmul_rn(x.y, inv), w.y),
                            __fmul_rn(__fmul_rn(x.z, inv), w.z), __fmul_rn(__fmul_rn(x.w, inv), w.w));
            reinterpret_cast<float4*>(const_cast<float*>(a.xb) + (size_t)t * D)[i4] = v;
        } else {
            v = reinterpret_cast<const float4*>(a.xb + (size_t)t * D)[i4];
        }
        xcm[i4] = v.x;
        xcm[xs + i4] = v.y;
        xcm[2 * xs + i4] = v.z;
        xcm[3 * xs + i4] = v.w;
    }
    for (int k = tid; k < K; k += kThreads) a.slot_pos[(size_t)t * K + k] = -1;  // until placed
    __syncthreads();  // x staged, barriers initialised
    RTL(1);
    const int e = tid >> 2, c = tid & 3;
    const bool chain = e < E;
    float s = 0.0f;
    bool ok = true;
    for (int q = 0; q < nq; q++) {
        const int b = q % kTokBufs;
        ok = ok && mbar_wait_bounded(&full[b], (uint32_t)(q / kTokBufs) & 1u, kTokWaitNs);
        if (ok && chain) {
            const uint4* wq = reinterpret_cast<const uint4*>(ring + (size_t)b * celems) + tid;
            const float* xq = xcm + c * xs + q * (8 * kTokGroups);
#pragma unroll
            for (int g = 0; g < kTokGroups; g++) {
                const uint4 w = wq[g * 4 * E];
                const float4 x0 = *reinterpret_cast<const float4*>(xq + 8 * g);
                const float4 x1 = *reinterpret_cast<const float4*>(xq + 8 * g + 4);
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.x << 16), x0.x));
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.x & 0xffff0000u), x0.y));
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.y << 16), x0.z));
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.y & 0xffff0000u), x0.w));
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.z << 16), x1.x));
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.z & 0xffff0000u), x1.y));
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.w << 16), x1.z));
                s = __fadd_rn(s, __fmul_rn(__uint_as_float(w.w & 0xffff0000u), x1.w));
            }
        }
        __syncthreads();  // slot b is free again
        if (tid == 0 && ok && q + kTokBufs < nq) {
            mbar_arrive_expect_tx(&full[b], (uint32_t)cbytes);
            bulk_load(ring + (size_t)b * celems, cm + (size_t)(q + kTokBufs) * celems, (uint32_t)cbytes, &full[b]);
            n_issued++;
        }
    }
    if (tid == 0 && !ok) {
        // a wait ran out: wait (bounded) for the copies still in flight (the latest
        // phase of each slot) before this CTA's shared memory can be given up
        for (int q = n_issued - kTokBufs < 0 ? 0 : n_issued - kTokBufs; q < n_issued; q++)
            (void)mbar_wait_bounded(&full[q % kTokBufs], (uint32_t)(q / kTokBufs) & 1u, kTokWaitNs);
    }
    RTL(2);
    // (s0 + s1) + (s2 + s3) across the four chain lanes of an expert
    const float s1 = __shfl_down_sync(FULL_MASK, s, 1);
    const float a01 = __fadd_rn(s, s1);
    const float a23 = __shfl_down_sync(FULL_MASK, a01, 2);
    if (chain && c == 0) {
        float logit = __fadd_rn(a01, a23);
        if (a.bias) logit = __fadd_rn(logit, a.bias[e]);
        s_logit[e] = logit;
    }
    if (!ok && tid == 0 && a.status) atomicCAS(a.status, 0u, 0x640u);
    __syncthreads();
    // softmax (rabbit2.c:399-405): thread e < E owns expert e
    const float lg = tid < E ? s_logit[tid] : -INFINITY;
    float mx = lg;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
    for (int w = 1; w < (E + 31) / 32; w++) mx = fmaxf(mx, s_red[w]);
    // the host libm's expf (rabbit2.c:403), by whole warps
    float pe = 0.0f;
    if (warp < (E + 31) / 32) {
        const float v = expf_ref_warp(tid < E ? __fsub_rn(lg, mx) : 0.0f, a.expf_fma, expf_tab_lane());
        if (tid < E) pe = v;
    }
    if (tid < E) s_prob[tid] = pe;
    __syncthreads();
    if (tid == 0) {  // the sequential sum in expert order (rabbit2.c:403)
        float sum = 0.0f;
        int f = 0;
        for (; f + 4 <= E; f += 4) {
            const float4 v = *reinterpret_cast<const float4*>(s_prob + f);
            sum = __fadd_rn(sum, v.x);
            sum = __fadd_rn(sum, v.y);
            sum = __fadd_rn(sum, v.z);
            sum = __fadd_rn(sum, v.w);
        }
        for (; f < E; f++) sum = __fadd_rn(sum, s_prob[f]);
        s_red[0] = sum;
    }
    __syncthreads();
    if (tid < E) {
        s_prob[tid] = __fdiv_rn(pe, s_red[0]);
        a.logits[(size_t)t * E + tid] = lg;
    }
    __syncthreads();
    RTL(3);
    // top-k by rank (rabbit2.c:519-528): expert e is chosen in round r when exactly r
    // experts beat it (higher probability, or equal and lower index); 4 threads per
    // expert, each counting a quarter of the rivals
    {
        const int re = tid >> 2, part = tid & 3;
        int r = 0;
        float pr = 0.0f;
        if (re < E) {
            pr = s_prob[re];
            const int f0 = part * E / 4, f1 = (part + 1) * E / 4;
            for (int f = f0; f < f1; f++) {
                const float pf = s_prob[f];
                r += (pf > pr) || (pf == pr && f < re);
            }
        }
        r += __shfl_xor_sync(FULL_MASK, r, 1);
        r += __shfl_xor_sync(FULL_MASK, r, 2);
        const bool chosen = re < E && part == 0 && r < K;
        if (chosen) atomicOr(&s_seen, 1ull << r);
        const unsigned m = __ballot_sync(FULL_MASK, chosen);
        if (lane == 0) s_cnt[warp] = __popc(m);
        __syncthreads();
        int n_chosen = 0;
        for (int w = 0; w < kThreads / 32; w++) n_chosen += s_cnt[w];
        // A consistent ranking gives ranks 0..K-1 to exactly K experts.  A NaN
        // probability breaks the order (every comparison with it is false); the token
        // then takes experts 0..K-1 (its output is NaN, as the reference's would be).
        const bool valid = n_chosen == K && s_seen == (K == 64 ? ~0ull : (1ull << K) - 1);
        if (valid && chosen) {
            s_idx[r] = re;
            s_p[r] = pr;
        }
        if (!valid)
            for (int k = tid; k < K; k += kThreads) {
                s_idx[k] = k;
                s_p[k] = s_prob[k];
            }
    }
    __syncthreads();
    if (warp == 0) {
        float wsum = 0.0f;
        if (a.norm_topk)  // the sequential sum in selection order (rabbit2.c:529-531)
            for (int k = 0; k < K; k++) wsum = __fadd_rn(wsum, s_p[k]);
        unsigned long long mask = 0ull;
        for (int k = lane; k < K; k += 32) {
            const int ek = s_idx[k];
            a.idx[(size_t)t * K + k] = ek;
            a.wt[(size_t)t * K + k] = a.norm_topk ? __fdiv_rn(s_p[k], wsum) : s_p[k];
            if (a.routing_out) a.routing_out[(size_t)t * a.routing_stride + k] = ek;
            mask |= 1ull << ek;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mask |= __shfl_xor_sync(FULL_MASK, mask, o);
        if (lane == 0) reinterpret_cast<unsigned long long*>(a.tile_cnt)[t] = mask;
    }
    // the last CTA to finish builds the permutation of all T*K slots
    __threadfence();
    __syncthreads();
    if (tid == 0) s_ticket = atomicAdd(a.done_counter, 1u);
    __syncthreads();
    RTL(4);
    if (s_ticket != (unsigned)T - 1) return;
    __threadfence();
    // (the ring is free now) every token's mask and each (token, expert)'s slot k
    unsigned long long* smask = reinterpret_cast<unsigned long long*>(tsm);               // [T]
    uint8_t* kpos = tsm + (size_t)kTokMaxTokens * sizeof(unsigned long long);             // [T][E]
    int* s_part = reinterpret_cast<int*>(kpos + (size_t)kTokMaxTokens * kTokMaxE);        // [P][E]
    int* s_off = s_part + kThreads;                                                       // [E]
    for (int i = tid; i < T; i += kThreads) smask[i] = __ldcg(reinterpret_cast<const unsigned long long*>(a.tile_cnt) + i);
    // (loads of 8 slots in flight at a time: one L2 round trip per 8, not per slot)
    for (int sl0 = 0; sl0 < T * K; sl0 += 8 * kThreads) {
        int ek[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int sl = sl0 + u * kThreads + tid;
            ek[u] = sl < T * K ? __ldcg(a.idx + sl) : -1;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int sl = sl0 + u * kThreads + tid;
            if (ek[u] >= 0 && ek[u] < E) kpos[(sl / K) * E + ek[u]] = (uint8_t)(sl % K);
        }
    }
    __syncthreads();
    // thread (xe, part): the tokens of its contiguous part routed to expert xe
    const int P = kThreads / E, xe = tid % E, part = tid / E;
    const bool mine = part < P;
    const int u0 = (int)((long)T * part / P), u1 = (int)((long)T * (part + 1) / P);
    int pc = 0;
    if (mine)
        for (int i = u0; i < u1; i++) pc += (int)((smask[i] >> xe) & 1ull);
    if (mine) s_part[part * E + xe] = pc;
    __syncthreads();
    int cnt = 0;
    if (tid < E)
        for (int p = 0; p < P; p++) cnt += s_part[p * E + tid];
    int total = 0;
    const int off = block_exclusive_scan(cnt, &total);
    int n_act = 0;
    const int apos = block_exclusive_scan(cnt > 0 ? 1 : 0, &n_act);
    if (tid < E) {
        a.counts[tid] = cnt;
        a.offsets[tid] = off;
        if (cnt > 0) a.active[apos] = tid;
        s_off[tid] = off;
    }
    if (tid == 0) {
        a.offsets[E] = total;
        *a.n_active = n_act;
        *a.done_counter = 0;
    }
    __syncthreads();
    // the expert's slots in token order (stable, as the reference's per-token loop)
    if (mine) {
        int pos = s_off[xe];
        for (int p = 0; p < part; p++) pos += s_part[p * E + xe];
        for (int i = u0; i < u1; i++)
            if ((smask[i] >> xe) & 1ull) {
                const int sl = i * K + kpos[i * E + xe];
                a.perm[pos] = sl;
                a.slot_pos[sl] = pos;
                pos++;
            }
    }
    RTL(5);
}

bool tok_ok(const RouterArgs& a) {
    return a.router_cm && a.dtype == 1 && a.E <= kTokMaxE && a.D % 256 == 0 && a.T >= 1 && a.T <= kTokMaxTokens &&
           a.K <= kMaxTopK && a.tile_cnt && a.done_counter;
}

bool wide_ok(const RouterArgs& a) {
    const size_t esz = a.dtype == 1 ? 2 : 4;
    return a.E <= kWideExperts && a.D % 4 == 0 && a.K * kWideTokens <= kWideTokens * kMaxTopK &&
           (reinterpret_cast<uintptr_t>(a.router) % (esz * 4)) == 0 && (reinterpret_cast<uintptr_t>(a.xb) % 16) == 0;
}

template <typename KernelT>
cudaError_t launch_with_smem(KernelT kernel, dim3 grid, size_t smem, const RouterArgs& a, cudaStream_t s) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    kernel<<<grid, kThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <typename WT>
cudaError_t launch_typed(const RouterArgs& a, cudaStream_t s, int* launches) {
    const int egroups = (a.E + kExpertsPerCta - 1) / kExpertsPerCta;
    *launches = 1;
    static const int mid_tokens = [] {
        const char* v = getenv("RBT_ROUTER_MID_TOKENS");  // tuning: the thread-per-chain kernel up to this T
        return v ? atoi(v) : kMidTokens;
    }();
    static const bool tok_on = [] {
        const char* v = getenv("RBT_ROUTER_TOK");  // RBT_ROUTER_TOK=0: without the token router
        return !(v && v[0] == '0');
    }();
    if (tok_on && tok_ok(a) && a.T <= mid_tokens) {
        // one CTA per token; rmsnorm (block form), softmax, top-k and the permutation
        // in the same launch
        return launch_with_smem(router_tok_kernel, dim3(a.T), tok_smem_bytes(a.D, a.E), a, s);
    }
    if (a.norm_w) {  // the block form's rmsnorm as its own launch, then the router on xb
        cudaError_t err = launch_rmsnorm(a.x_raw, a.norm_w, const_cast<float*>(a.xb), a.T, a.D, a.eps, s);
        if (err != cudaSuccess) return err;
        RouterArgs b = a;
        b.norm_w = nullptr;
        b.x_raw = nullptr;
        int inner = 0;
        err = launch_typed<WT>(b, s, &inner);
        *launches = inner + 1;
        return err;
    }
    if (a.T <= kSmallTokens || a.T <= mid_tokens) {
        // thread per chain: token tiles of 8 x expert groups of 8 (latency, not
        // issue rate, bounds a few hundred tokens)
        const size_t smem = 2ull * kExpertsPerCta * kSmallStride * sizeof(float);
        const int tiles = (a.T + kSmallTokens - 1) / kSmallTokens;
        RouterArgs b = a;
        b.tile_tokens = tiles > 1 ? kSmallTokens : 0;
        cudaError_t err = launch_with_smem(router_small_kernel<WT>, dim3(tiles, egroups), smem, b, s);
        if (err != cudaSuccess || tiles == 1) return err;
        *launches = 2;
        scatter_kernel<<<tiles, kThreads, 0, s>>>(b);
        return cudaGetLastError();
    }
    if (wide_ok(a)) {
        const int tiles = (a.T + kWideTokens - 1) / kWideTokens;
        RouterArgs b = a;
        b.tile_tokens = kWideTokens;
        cudaError_t err = launch_with_smem(router_wide_kernel<WT>, dim3(tiles), WideCfg<WT>::kSmem, b, s);
        if (err != cudaSuccess) return err;
        *launches = 2;
        scatter_kernel<<<tiles, kThreads, 0, s>>>(b);
        return cudaGetLastError();
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

// Token tiles any router variant uses for T tokens (sizes the per-tile arrays).
// (tiles of 8 tokens: at least as many as any variant uses, for every T' <= T)
int router_token_tiles(int T) { return T <= kSmallTokens ? 1 : (T + kSmallTokens - 1) / kSmallTokens; }

cudaError_t launch_route_given(const RouterArgs& a, cudaStream_t s, int* launches) {
    *launches = 0;
    if (a.T <= 0) return cudaSuccess;
    if (a.K > kMaxTopK || a.E > kMaxExperts) return cudaErrorInvalidValue;
    const int tiles = (a.T + kWideTokens - 1) / kWideTokens;
    RouterArgs b = a;
    b.tile_tokens = kWideTokens;
    route_given_kernel<<<tiles, kThreads, 0, s>>>(b);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    scatter_kernel<<<tiles, kThreads, 0, s>>>(b);
    *launches = 2;
    return cudaGetLastError();
}

cudaError_t launch_router(const RouterArgs& a, cudaStream_t s, int* launches) {
    *launches = 0;
    if (a.T <= 0) return cudaSuccess;
    RouterArgs b = a;
    b.expf_fma = host_expf_fma();
    return b.dtype == 1 ? launch_typed<uint16_t>(b, s, launches) : launch_typed<float>(b, s, launches);
}

bool router_chain_major_supported(int E, int D, int dtype) {
    return dtype == 1 && E > 0 && E <= kTokMaxE && D > 0 && D % 256 == 0;
}

cudaError_t router_to_chain_major(const void* router, int E, int D, void* out, cudaStream_t s) {
    if (!router_chain_major_supported(E, D, 1)) return cudaErrorInvalidValue;
    const size_t n = (size_t)E * D;
    const int grid = (int)((n + 255) / 256 < 2048 ? (n + 255) / 256 : 2048);
    router_cm_kernel<<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(router), E, D, static_cast<uint16_t*>(out));
    return cudaGetLastError();
}

// Loads every router kernel now (see preload_kernels in kernels.h).
void preload_router_kernels() {
    cudaFuncAttributes f;
    (void)cudaFuncGetAttributes(&f, router_tok_kernel);
    (void)cudaFuncGetAttributes(&f, router_small_kernel<uint16_t>);
    (void)cudaFuncGetAttributes(&f, router_small_kernel<float>);
    (void)cudaFuncGetAttributes(&f, router_wide_kernel<uint16_t>);
    (void)cudaFuncGetAttributes(&f, router_wide_kernel<float>);
    (void)cudaFuncGetAttributes(&f, router_large_kernel<uint16_t, 1>);
    (void)cudaFuncGetAttributes(&f, router_large_kernel<uint16_t, 2>);
    (void)cudaFuncGetAttributes(&f, router_large_kernel<uint16_t, 4>);
    (void)cudaFuncGetAttributes(&f, router_large_kernel<float, 1>);
    (void)cudaFuncGetAttributes(&f, router_large_kernel<float, 2>);
    (void)cudaFuncGetAttributes(&f, router_large_kernel<float, 4>);
    (void)cudaFuncGetAttributes(&f, scatter_kernel);
    (void)cudaFuncGetAttributes(&f, route_given_kernel);
    (void)cudaGetLastError();
}

}  // namespace rbt

#ifdef RBT_ROUTER_TIMELINE
extern "C" int rbt_router_timeline_read(void* host) {
    return cudaMemcpyFromSymbol(host, rbt::g_rtl, sizeof(rbt::g_rtl)) == cudaSuccess;
}
extern "C" int rbt_router_timeline_clear(void) {
    static unsigned long long zeros[4096 * 16];
    return cudaMemcpyToSymbol(rbt::g_rtl, zeros, sizeof(zeros)) == cudaSuccess;
}
#endif
