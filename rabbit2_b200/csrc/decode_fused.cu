// decode_fused.cu -- the whole MoE block for ONE token in one persistent kernel
// (bf16 models): rabbit2.c:512-542 -- RMSNorm, router, softmax, top-k, the k
// experts' SwiGLU FFNs, the weighted combine and the residual -- as a single
// cooperative launch of one CTA per SM.  Batch-1 decode is memory-bound on the
// K experts' weights (8 x 12 MB at OLMoE-1B-7B), so the kernel exists to keep
// HBM streaming: no launch gaps, no kernel-boundary drains, and every weight
// byte read exactly once in a single streaming phase.  Cross-CTA ordering is by
// words in global memory (release by atomics / __threadfence, acquire by
// ld.acquire), each wait bounded by %globaltimer; the launch is cooperative, so
// every CTA is resident and every wait ends.
//
//   0  every CTA: bulk-copies its router row(s) and ffn_norm into shared memory
//      (static weights, so before griddepcontrol.wait: this overlaps the
//      previous kernel's tail), then x; rmsnorm(x) for the block form with the
//      reference's sequential sum of squares (block_seq_sum), so every CTA holds
//      the reference's xb bits
//   1  CTAs compute router logits -- the four sequential chains of the
//      reference's scalar matvec (rabbit2.c:378-387), separately rounded
//      products and sums, (s0+s1)+(s2+s3) -- each expert by two CTAs when the
//      grid has room; a logit is published with its ready bit in one 64-bit word
//   2  every CTA, as soon as all E logits are published: softmax (the host's
//      expf, then the sequential sum in expert order, rabbit2.c:399-405) and top-k (selection
//      order = rank: higher probability, or equal and lower index); CTA 0
//      publishes the routing outputs
//   3  units of 8 hidden rows of one chosen expert, a contiguous range per CTA.
//      A unit is w1 and w3 rows [r, r+8) (two bulk copies) and the w2 part for
//      hidden rows [r, r+8): rows of the transposed copy (one bulk copy) or a
//      [D x 8] column tile of w2 itself (3-D TMA).  The units stream through a
//      2 x 96 KB shared-memory ring.  Warp w forms
//      h_w = silu(w1_w . xb) * (w3_w . xb) scaled by the expert's combine
//      weight; then each thread adds the w2 . h products to its 8 output rows.
//      The CTA's partial MoE output over all D rows stays in registers.
//   4  every CTA writes its partial [D]; one grid barrier; CTA b sums its band
//      of rows over all CTAs in a fixed order and writes out = x + moe
//      (rabbit2.c:539-542).  After the barrier CTA 0 clears the logit words and
//      the last CTA past it clears the barrier counters, and the next layer's
//      router row and ffn_norm are prefetched into L2.
#include <cuda_bf16.h>
#include <stdlib.h>

#ifdef RBT_DECODE_TIMELINE
// Optional phase timestamps (%globaltimer) of every CTA, read back with
// rbt_decode_timeline_read(); built only with -DRBT_DECODE_TIMELINE.
// Two buffers, alternating by launch, so consecutive launches can be compared.
namespace rbt {
__device__ unsigned long long g_timeline[2 * 256 * 32];
__device__ unsigned g_timeline_seq;
}  // namespace rbt
// block_seq_sum's own phases, slots 20..25 of both buffers (no load of the
// launch parity on the measured path: the stores are fire-and-forget)
#define RBT_SEQ_STAMP(i)                                                          \
    do {                                                                          \
        unsigned long long t_;                                                    \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                   \
        if (blockIdx.x < 256) {                                                   \
            ::rbt::g_timeline[blockIdx.x * 32 + 20 + (i)] = t_;                   \
            ::rbt::g_timeline[(256 + blockIdx.x) * 32 + 20 + (i)] = t_;           \
        }                                                                         \
    } while (0)
#endif

#include "common.cuh"
#include "exact_math.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rbt {
namespace {

using namespace tc;

constexpr int kWarps = 8;                  // consumer warps
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kSlot = 96 * 1024;           // ring slot: w1 rows | w3 rows | w2 part
constexpr int kSlots = 2;
constexpr int kGURows = 8;                 // hidden rows per unit (one per consumer warp)
constexpr int kMaxD = 2048;                // xb slices and output rows held in registers
constexpr int kRowsPerThread = kMaxD / kConsumers;
constexpr int kBoxRows = 256;              // rows of one w2 TMA box (the TMA limit)
constexpr uint64_t kWaitNs = 2000000000ull;
// phases 0-2 keep their staging in ring slot 0
constexpr int kXsOff = 0;                  // xb [D] f32
constexpr int kProdOff = 8 * 1024;         // router products, chain-major [4][D/4 + kProdPad] f32
constexpr int kProdPad = 4;                // floats between chains: the 4 chain lanes hit different banks
constexpr int kWrowOff = 24 * 1024;        // this CTA's router rows, bf16
constexpr int kWrowBytes = 64 * 1024;
constexpr int kNormOff = 88 * 1024;        // ffn_norm [D] f32

// sync words (a.sync, 32-bit): [0..1] unused, [2..3] the grid barrier's arrival
// count (64-bit), [4..31] unused, then one 64-bit word per expert at the start of
// its own 128-byte line (every CTA polls every word: separate lines spread the
// polls over the L2 slices): bit 32 = published, low 32 bits = the logit.
// The arrival count only grows: the n-th launch since the words were zeroed waits
// for n x G arrivals, which each CTA learns from the count its own arrival returns,
// so nothing has to reset it.  The logit words are zero between launches: CTA 0
// clears them after the barrier.
constexpr int kSyncHead = 32;
constexpr int kLogitStride = 16;  // 64-bit words between two experts' logit words

#ifdef RBT_DECODE_TIMELINE
#define TIMELINE(i)                                                                                   \
    do {                                                                                              \
        if (blockIdx.x < 256) g_timeline[(tl_par * 256 + blockIdx.x) * 32 + (i)] = globaltimer_ns(); \
    } while (0)
#else
#define TIMELINE(i) \
    do {            \
    } while (0)
#endif

__device__ __forceinline__ void record_error(unsigned* status, unsigned code) { atomicCAS(status, 0u, code); }

__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
// acc(lo,hi) += w(lo,hi) * x(lo,hi), two fp32 FMAs
__device__ __forceinline__ uint64_t ffma2(uint64_t w, uint64_t x, uint64_t acc) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(w), "l"(x), "l"(acc));
    return d;
}
__device__ __forceinline__ float f2sum(uint64_t v) {
    return __uint_as_float((uint32_t)v) + __uint_as_float((uint32_t)(v >> 32));
}
// bf16 pair (one 32-bit word) -> packed f32 pair
__device__ __forceinline__ uint64_t bf2(uint32_t w) { return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u)); }

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Spin (bounded by limit_ns) until *p >= target.
__device__ __forceinline__ bool wait_count(const unsigned long long* p, unsigned long long target, uint64_t limit_ns) {
    if (ld_acquire64(p) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire64(p) < target)
        if (globaltimer_ns() - t0 > limit_ns) return false;
    return true;
}

// Spin (bounded by limit_ns) until the logit word is published; returns the logit in *v.
__device__ __forceinline__ bool wait_logit(const unsigned long long* p, float* v, uint64_t limit_ns) {
    unsigned long long w = ld_acquire64(p);
    if (!(w >> 32)) {
        const uint64_t t0 = globaltimer_ns();
        while (!((w = ld_acquire64(p)) >> 32))
            if (globaltimer_ns() - t0 > limit_ns) return false;
    }
    *v = __uint_as_float((uint32_t)w);
    return true;
}

// Named barrier over n threads that also returns the OR of `pred` over them.
__device__ __forceinline__ bool named_sync_or(int id, int n, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

__host__ __device__ constexpr int w2_box_rows(int D) { return D < kBoxRows ? D : kBoxRows; }
__host__ __device__ constexpr int w2_boxes(int D) { return (D + w2_box_rows(D) - 1) / w2_box_rows(D); }
__host__ __device__ constexpr int w2_offset(int D) { return (2 * kGURows * D * 2 + 1023) / 1024 * 1024; }

// kW2T: the w2 part of a unit comes from the transposed copy a.w2t ([E][H][D],
// rows r..r+8 are one contiguous 8*D*2-byte run); otherwise from w2 itself as a
// [D x 8] column tile through w2map.  Shared memory then holds [8][D] or [D][8].
template <bool kW2T>
__global__ void __launch_bounds__(kThreads, 1)
    moe_decode_fused_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap w2map) {
    extern __shared__ __align__(1024) uint8_t ring[];
    __shared__ uint64_t full[kSlots], empty[kSlots], rbar, nbar;
    __shared__ int s_cnt[kThreads / 32];
    __shared__ unsigned long long s_seen;  // ranks given to chosen experts, one bit each
    __shared__ int32_t s_idx[kMaxTopK], s_act[kMaxTopK], s_kpos[kMaxTopK];
    __shared__ float s_p[kMaxTopK], s_wpos[kMaxTopK];
    __shared__ __align__(16) float s_prob[kMaxExperts];
    __shared__ __align__(16) float s_h[kSlots][kGURows];
    __shared__ float s_red[kThreads / 32];
    __shared__ int s_fail;
    __shared__ SeqSumSmem s_seq;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = a.D, H = a.H, E = a.E, K = a.K;
    const int G = gridDim.x, b = blockIdx.x;
#ifdef RBT_DECODE_TIMELINE
    const unsigned tl_par = *(volatile unsigned*)&g_timeline_seq & 1u;
#endif
    unsigned long long* bar_cnt = reinterpret_cast<unsigned long long*>(a.sync + 2);
    // waits on other CTAs end at this bound; waits on this CTA's own copies (which
    // always complete) keep kWaitNs, so a short bound never abandons a copy in flight
    const uint64_t peer_ns = a.peer_wait_ns ? a.peer_wait_ns : kWaitNs;
    unsigned long long* lword = reinterpret_cast<unsigned long long*>(a.sync + kSyncHead);
    float* xs = reinterpret_cast<float*>(ring + kXsOff);
    float* prods = reinterpret_cast<float*>(ring + kProdOff);
    uint16_t* wrow = reinterpret_cast<uint16_t*>(ring + kWrowOff);
    float* norm_s = reinterpret_cast<float*>(ring + kNormOff);
    TIMELINE(0);

    // router rows this CTA computes: two copies of every expert when the grid has room
    const bool dup = G >= 2 * E;
    const int e_first = dup ? (b < 2 * E ? b % E : E) : b;
    const int e_step = dup ? E : G;
    int n_rows = 0;
    for (int e = e_first; e < E; e += e_step) n_rows++;
    if (dup && n_rows > 1) n_rows = 1;

    if (tid == 0) {
        s_fail = 0;
        s_seen = 0ull;
        for (int s = 0; s < kSlots; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        mbar_init(&rbar, 1);
        mbar_init(&nbar, 1);
        fence_mbar_init();
        prefetch_tmap(&w2map);
        // static weights: no need to wait for the previous kernel
        if (n_rows > 0) {
            mbar_arrive_expect_tx(&rbar, (uint32_t)n_rows * D * 2);
            for (int j = 0; j < n_rows; j++)
                bulk_load(wrow + (size_t)j * D, a.router + (size_t)(e_first + j * e_step) * D, (uint32_t)D * 2, &rbar);
        }
        if (a.ffn_norm) {
            mbar_arrive_expect_tx(&nbar, (uint32_t)D * 4);
            bulk_load(norm_s, a.ffn_norm, (uint32_t)D * 4, &nbar);
        }
    }
    const uint64_t exp_tab = expf_tab_lane();  // the softmax's table entry of this lane
    // x, the sync words and every output may belong to the previous kernel in
    // the stream until this returns (programmatic dependent launch)
    pdl_wait();
    pdl_launch_dependents();
    // ---------------------------------------------------------------- phase 0
    // x straight from L2 (the previous kernel wrote it) into registers; for the block
    // form the squares go to shared memory (the products area, free until phase 1):
    // thread t holds the float4s t and t + kThreads (D <= 2048 = 2 x 4 x 288 - 256)
    const int n4 = D / 4;
    float4 xv[2];
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int i4 = tid + k * kThreads;
        xv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i4 < n4) {
            xv[k] = __ldcg(reinterpret_cast<const float4*>(a.x) + i4);
            if (a.ffn_norm)
                reinterpret_cast<float4*>(prods)[i4] =
                    make_float4(__fmul_rn(xv[k].x, xv[k].x), __fmul_rn(xv[k].y, xv[k].y),
                                __fmul_rn(xv[k].z, xv[k].z), __fmul_rn(xv[k].w, xv[k].w));
        }
    }
    if (tid == 0) TIMELINE(13);
    __syncthreads();  // the squares, and the mbarrier initialisation
    if (a.ffn_norm) {  // rmsnorm (rabbit2.c:392-397) with the reference's sequential sum of squares
        const float tot = block_seq_sum_l<kThreads, 8>(prods, D, s_seq);  // D <= 2048 <= 288 * 8
        if (tid == 0) TIMELINE(19);
        if (!mbar_wait_bounded(&nbar, 0, kWaitNs)) {
            record_error(a.status, 0x605);
            s_fail = 1;
        }
        const float inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, (float)D), a.eps));
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int i4 = tid + k * kThreads;
            if (i4 < n4) {
                const float4 nw = reinterpret_cast<const float4*>(norm_s)[i4];
                xv[k].x = __fmul_rn(__fmul_rn(xv[k].x, inv), nw.x);
                xv[k].y = __fmul_rn(__fmul_rn(xv[k].y, inv), nw.y);
                xv[k].z = __fmul_rn(__fmul_rn(xv[k].z, inv), nw.z);
                xv[k].w = __fmul_rn(__fmul_rn(xv[k].w, inv), nw.w);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int i4 = tid + k * kThreads;
        if (i4 < n4) reinterpret_cast<float4*>(xs)[i4] = xv[k];
    }
    TIMELINE(1);
    // ---------------------------------------------------------------- phase 1: exact router logits
    // The products w[i]*x[i] are independent: every thread rounds those of its own
    // float4s of xb into `prods`, laid out chain-major (chain c = i mod 4 holds its
    // D/4 products contiguously).  Lane c of warp 0 then runs chain c's D/4
    // dependent adds in order, reading 4 products per 16-byte load.
    for (int j = 0; j < n_rows; j++) {
        const int e = e_first + j * e_step;
        if (j == 0) {
            const bool got = mbar_wait_bounded(&rbar, 0, kWaitNs);
            if (!got) {
                record_error(a.status, 0x600);
                s_fail = 1;
            }
            if (tid == 0) TIMELINE(2);
        }
        const uint16_t* wr = wrow + (size_t)j * D;
        const int q = D / 4, qp = q + kProdPad;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int i4 = tid + k * kThreads;
            if (i4 < n4) {
                const uint2 w4 = *reinterpret_cast<const uint2*>(wr + 4 * i4);
                prods[i4] = __fmul_rn(__uint_as_float(w4.x << 16), xv[k].x);
                prods[qp + i4] = __fmul_rn(__uint_as_float(w4.x & 0xffff0000u), xv[k].y);
                prods[2 * qp + i4] = __fmul_rn(__uint_as_float(w4.y << 16), xv[k].z);
                prods[3 * qp + i4] = __fmul_rn(__uint_as_float(w4.y & 0xffff0000u), xv[k].w);
            }
        }
        __syncthreads();
        if (s_fail) break;
        if (tid == 0 && j == 0) TIMELINE(14);
        if (warp == 0) {
            float s = 0.0f;
            if (lane < 4) {
                // the dependent adds are the critical path (about 4.6 cycles per product)
                // (unrolled so that the 16-byte loads run well ahead of the adds)
                const float* pc = prods + lane * qp;
                const float4* pc4 = reinterpret_cast<const float4*>(pc);
                const int q4 = q >> 2;
#pragma unroll 8
                for (int i4 = 0; i4 < q4; i4++) {
                    const float4 v = pc4[i4];
                    s = __fadd_rn(s, v.x);
                    s = __fadd_rn(s, v.y);
                    s = __fadd_rn(s, v.z);
                    s = __fadd_rn(s, v.w);
                }
                for (int i = 4 * q4; i < q; i++) s = __fadd_rn(s, pc[i]);
            }
            const float s1 = __shfl_down_sync(FULL_MASK, s, 1);
            const float a01 = __fadd_rn(s, s1);
            const float a23 = __shfl_down_sync(FULL_MASK, a01, 2);
            if (lane == 0) {
                if (j == 0) TIMELINE(15);
                float logit = __fadd_rn(a01, a23);
                if (a.bias) logit = __fadd_rn(logit, a.bias[e]);
                // both copies publish the same bits (an exchange at L2 measured faster to
                // reach the pollers than a plain 64-bit store)
                atomicExch(lword + (size_t)e * kLogitStride, (1ull << 32) | (unsigned long long)__float_as_uint(logit));
            }
        }
        // the products are rewritten by the next row; after the last row nothing waits
        // here for the publishing warp (its exchange completes while the logits propagate)
        if (j + 1 < n_rows) __syncthreads();
    }
    if (n_rows == 0) __syncthreads();  // xs complete
    // consumer lanes keep their slices of xb (elements 8v..8v+8, v = lane + 32 j) in
    // registers from here on (loaded while the logits propagate); the ring region
    // holding xs is reused after routing
    const int nvx = D / 8;  // 16-byte bf16 vectors per w1/w3 row
    float xr[64];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int v = lane + 32 * j;
        float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
        if (warp < kWarps && v < nvx) {
            lo = reinterpret_cast<const float4*>(xs)[2 * v];
            hi = reinterpret_cast<const float4*>(xs)[2 * v + 1];
        }
        xr[8 * j] = lo.x; xr[8 * j + 1] = lo.y; xr[8 * j + 2] = lo.z; xr[8 * j + 3] = lo.w;
        xr[8 * j + 4] = hi.x; xr[8 * j + 5] = hi.y; xr[8 * j + 6] = hi.z; xr[8 * j + 7] = hi.w;
    }
    if (tid == 0) TIMELINE(3);
    // ---------------------------------------------------------------- phase 2: softmax, top-k, slot order
    // thread e < E owns expert e
    float lg = -INFINITY;
    bool ok2 = !s_fail;
    if (ok2 && tid < E) ok2 = wait_logit(lword + (size_t)tid * kLogitStride, &lg, peer_ns);
    if (!__syncthreads_and(ok2)) {
        if (tid == 0) {
            record_error(a.status, 0x601);
            s_fail = 1;
        }
    } else {
        if (tid == 0) TIMELINE(10);
        float mx = lg;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, o));
        if (lane == 0) s_red[warp] = mx;
        __syncthreads();
        if (tid == 0) TIMELINE(16);
        mx = s_red[0];
        for (int w = 1; w < (E + 31) / 32; w++) mx = fmaxf(mx, s_red[w]);
        // the host libm's expf (rabbit2.c:403), by whole warps
        float pe = 0.0f;
        if (warp < (E + 31) / 32) {
            const float v = expf_ref_warp(tid < E ? __fsub_rn(lg, mx) : 0.0f, a.expf_fma, exp_tab);
            if (tid < E) pe = v;
        }
        if (tid < E) s_prob[tid] = pe;
        __syncthreads();
        if (tid == 0) TIMELINE(17);
        if (tid == 0) {  // the sequential sum in expert order (rabbit2.c:403)
            float sum = 0.0f;
            int e = 0;
            for (; e + 4 <= E; e += 4) {
                const float4 v = *reinterpret_cast<const float4*>(s_prob + e);
                sum = __fadd_rn(sum, v.x);
                sum = __fadd_rn(sum, v.y);
                sum = __fadd_rn(sum, v.z);
                sum = __fadd_rn(sum, v.w);
            }
            for (; e < E; e++) sum = __fadd_rn(sum, s_prob[e]);
            s_red[0] = sum;
        }
        __syncthreads();
        if (tid == 0) TIMELINE(18);
        if (tid < E) {
            s_prob[tid] = __fdiv_rn(pe, s_red[0]);
            if (b == 0) a.logits[tid] = lg;
        }
        if (tid == 0) TIMELINE(11);
    }
    __syncthreads();
    // top-k by rank: expert e is chosen in round r when exactly r experts beat it
    // (higher probability, or equal probability and lower index) -- the order of
    // the reference's K rounds of strict-'>' scans (rabbit2.c:519-528).
    // 4 threads per expert (E <= 72; one per expert otherwise), each counting a
    // contiguous quarter of the rivals.  The chosen experts' position in expert
    // order (the unit order) comes from a ballot over the experts' first threads.
    // A consistent ranking gives ranks 0..K-1 to exactly K experts; a NaN
    // probability breaks the order (every comparison with it is false), and the
    // call then fails instead of indexing with an incomplete routing.
    {
        const int split = E <= kThreads / 4 ? 4 : 1;
        const int e = tid / split, part = tid % split;
        int r = 0;
        float pe = 0.0f;
        if (!s_fail && e < E) {
            pe = s_prob[e];
            const int f0 = part * E / split, f1 = (part + 1) * E / split;
            int f = f0;
            if ((f0 & 3) == 0)
                for (; f + 4 <= f1; f += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(s_prob + f);
                    r += (v.x > pe) || (v.x == pe && f < e);
                    r += (v.y > pe) || (v.y == pe && f + 1 < e);
                    r += (v.z > pe) || (v.z == pe && f + 2 < e);
                    r += (v.w > pe) || (v.w == pe && f + 3 < e);
                }
            for (; f < f1; f++) {
                const float pf = s_prob[f];
                r += (pf > pe) || (pf == pe && f < e);
            }
        }
        if (split == 4) {  // the 4 threads of an expert are adjacent lanes of one warp
            r += __shfl_xor_sync(FULL_MASK, r, 1);
            r += __shfl_xor_sync(FULL_MASK, r, 2);
        }
        const bool first = !s_fail && e < E && part == 0;
        const bool chosen = first && r < K;
        if (chosen) atomicOr(&s_seen, 1ull << r);
        const unsigned m = __ballot_sync(FULL_MASK, chosen);
        if (lane == 0) s_cnt[warp] = __popc(m);
        __syncthreads();
        if (tid == 0) TIMELINE(12);
        // chosen experts in the warps before this one, and in all warps: a scan of
        // the per-warp counts across lanes (lane w holds warp w's count)
        const int cw = lane < kThreads / 32 ? s_cnt[lane] : 0;
        int incl = cw;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(FULL_MASK, incl, o);
            if (lane >= o) incl += t;
        }
        const int n_chosen = __shfl_sync(FULL_MASK, incl, 31);
        const int warp_base = __shfl_sync(FULL_MASK, incl - cw, warp);
        const bool valid = !s_fail && n_chosen == K && s_seen == (K == 64 ? ~0ull : (1ull << K) - 1);
        if (valid && first) {
            const int below = warp_base + __popc(m & lanemask_lt());  // chosen experts with a lower index
            if (chosen) {
                s_idx[r] = e;
                s_p[r] = pe;
                s_act[below] = e;
                s_kpos[r] = below;
                s_wpos[below] = pe;
            }
            if (b == 0) {
                a.counts[e] = chosen ? 1 : 0;
                a.offsets[e] = below;
            }
        }
        // (a thread that reads the flag set here computes valid = false as well)
        if (!valid && tid == 0 && !s_fail) {
            record_error(a.status, 0x603);
            s_fail = 1;
        }
    }
    __syncthreads();
    if (a.norm_topk) {  // the sequential sum in selection order (rabbit2.c:529-531)
        if (warp == 0 && !s_fail) {
            float wsum = 0.0f;
            for (int k = 0; k < K; k++) wsum = __fadd_rn(wsum, s_p[k]);
            for (int k = lane; k < K; k += 32) s_wpos[s_kpos[k]] = __fdiv_rn(s_p[k], wsum);
        }
        __syncthreads();
    }
    const bool fail0 = s_fail != 0;
    if (warp == 0 && !fail0) {
        if (b == 0) {  // the routing outputs of the call (global memory only: no barrier after)
            for (int k = lane; k < K; k += 32) {
                const int pos = s_kpos[k];
                a.idx[k] = s_idx[k];
                a.wt[k] = s_wpos[pos];
                a.slot_pos[k] = pos;
                a.perm[pos] = k;
                a.active[pos] = s_idx[k];
                if (a.routing_out) a.routing_out[k] = s_idx[k];
            }
            if (lane == 0) {
                a.offsets[E] = K;
                *a.n_active = K;
            }
        }
    }
    if (tid == 0) TIMELINE(4);

    const uint32_t gu_half = (uint32_t)kGURows * D * 2;  // 8 rows of w1 (or w3)
    const int boxr = w2_box_rows(D), nbox = w2_boxes(D);
    const uint32_t w2_bytes = (uint32_t)nbox * boxr * kGURows * 2;  // whole boxes, zero-filled past D
    const int w2_off = w2_offset(D);
    const int units_per_e = H / kGURows;
    const int n_units = fail0 ? 0 : K * units_per_e;
    const int g0 = (int)((long)n_units * b / G), g1 = (int)((long)n_units * (b + 1) / G);

    if (warp == kWarps) {
        // ------------------------------------------------------------ producer
        // (an L2 prefetch of the CTA's later units measured slower: the ring alone
        // keeps enough bytes in flight)
        if (lane == 0) {
            int slot = 0;
            uint32_t ph = 0;
            int issued = 0;
            bool ok = true;
            for (int u = g0; ok && u < g1; u++) {
                if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, kWaitNs)) {
                    record_error(a.status, 0x611);
                    ok = false;
                    break;
                }
                const int e = s_act[u / units_per_e], r0 = (u % units_per_e) * kGURows;
                const uint8_t* w1 = a.experts + (size_t)e * a.stride + (size_t)r0 * D * 2;
                uint8_t* st = ring + slot * kSlot;
                mbar_arrive_expect_tx(&full[slot], 2 * gu_half + (kW2T ? gu_half : w2_bytes));
                bulk_load(st, w1, gu_half, &full[slot]);
                bulk_load(st + gu_half, w1 + (size_t)H * D * 2, gu_half, &full[slot]);
                if (kW2T)
                    bulk_load(st + w2_off, a.w2t + (size_t)e * a.w2t_stride + (size_t)r0 * D * 2, gu_half,
                              &full[slot]);
                else
                    for (int i = 0; i < nbox; i++)
                        tma_load_3d(st + w2_off + i * boxr * kGURows * 2, &w2map, &full[slot], r0, i * boxr, e);
                issued++;
                if (++slot == kSlots) { slot = 0; ph ^= 1u; }
            }
            TIMELINE(8);
            for (int i = 0; i < kSlots && i < issued; i++) {  // drain
                if (--slot < 0) { slot = kSlots - 1; ph ^= 1u; }
                if (!mbar_wait_bounded(&full[slot], ph, kWaitNs)) record_error(a.status, 0x613);
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        uint64_t acc[kRowsPerThread];
#pragma unroll
        for (int j = 0; j < kRowsPerThread; j++) acc[j] = 0;
        int slot = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int u = g0; u < g1; u++) {
            const bool got = __all_sync(FULL_MASK, mbar_wait_bounded(&full[slot], ph, kWaitNs));
            if (tid == 0 && u == g0) TIMELINE(9);
            if (!got && lane == 0) record_error(a.status, 0x621);
            const int pa = u / units_per_e;
            const uint8_t* st = ring + slot * kSlot;
            // gate/up: warp w forms hidden row r0 + w
            const uint4* w1 = reinterpret_cast<const uint4*>(st + warp * D * 2);
            const uint4* w3 = reinterpret_cast<const uint4*>(st + gu_half + warp * D * 2);
            uint64_t g[4] = {0, 0, 0, 0}, up[4] = {0, 0, 0, 0};
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = lane + 32 * j;
                if (got && v < nvx) {
                    const uint4 q1 = w1[v], q3 = w3[v];
                    const uint64_t x01 = f2(xr[8 * j], xr[8 * j + 1]), x23 = f2(xr[8 * j + 2], xr[8 * j + 3]);
                    const uint64_t x45 = f2(xr[8 * j + 4], xr[8 * j + 5]), x67 = f2(xr[8 * j + 6], xr[8 * j + 7]);
                    g[0] = ffma2(bf2(q1.x), x01, g[0]);
                    g[1] = ffma2(bf2(q1.y), x23, g[1]);
                    g[2] = ffma2(bf2(q1.z), x45, g[2]);
                    g[3] = ffma2(bf2(q1.w), x67, g[3]);
                    up[0] = ffma2(bf2(q3.x), x01, up[0]);
                    up[1] = ffma2(bf2(q3.y), x23, up[1]);
                    up[2] = ffma2(bf2(q3.z), x45, up[2]);
                    up[3] = ffma2(bf2(q3.w), x67, up[3]);
                }
            }
            const float gs = warp_sum((f2sum(g[0]) + f2sum(g[1])) + (f2sum(g[2]) + f2sum(g[3])));
            const float us = warp_sum((f2sum(up[0]) + f2sum(up[1])) + (f2sum(up[2]) + f2sum(up[3])));
            // silu(h1) * h3 (rabbit2.c:407, :536), times the expert's combine weight
            if (lane == 0) s_h[slot][warp] = __fmul_rn(__fmul_rn(silu_ref(gs, a.expf_fma), us), s_wpos[pa]);
            // every consumer warp reaches this barrier once per unit, and the
            // barrier's OR of the timeouts ends the loop in all of them together
            if (named_sync_or(1, kConsumers, !got)) {
                s_fail = 1;
                ok = false;
                break;
            }
            const float4 ha = *reinterpret_cast<const float4*>(&s_h[slot][0]);
            const float4 hb = *reinterpret_cast<const float4*>(&s_h[slot][4]);
            if (kW2T) {
                // down: this thread's output rows d = 8 tid .. 8 tid + 7, from the 8
                // transposed rows r0..r0+8 ([8][D] in shared memory)
                if (8 * tid < D) {
                    const float hv[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
                    const uint4* w2r = reinterpret_cast<const uint4*>(st + w2_off) + tid;
#pragma unroll
                    for (int r = 0; r < kGURows; r++) {
                        const uint4 q = w2r[r * (D / 8)];
                        const uint64_t hh = f2(hv[r], hv[r]);
                        acc[0] = ffma2(bf2(q.x), hh, acc[0]);
                        acc[1] = ffma2(bf2(q.y), hh, acc[1]);
                        acc[2] = ffma2(bf2(q.z), hh, acc[2]);
                        acc[3] = ffma2(bf2(q.w), hh, acc[3]);
                    }
                }
            } else {
                // down: this thread's output rows d = tid + 256 j, columns r0..r0+8 of w2
                const uint64_t h01 = f2(ha.x, ha.y), h23 = f2(ha.z, ha.w), h45 = f2(hb.x, hb.y),
                               h67 = f2(hb.z, hb.w);
                const uint4* w2c = reinterpret_cast<const uint4*>(st + w2_off);
#pragma unroll
                for (int j = 0; j < kRowsPerThread; j++) {
                    const int d = tid + kConsumers * j;
                    if (d < D) {
                        const uint4 q = w2c[d];
                        acc[j] = ffma2(bf2(q.x), h01, acc[j]);
                        acc[j] = ffma2(bf2(q.y), h23, acc[j]);
                        acc[j] = ffma2(bf2(q.z), h45, acc[j]);
                        acc[j] = ffma2(bf2(q.w), h67, acc[j]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == kSlots) { slot = 0; ph ^= 1u; }
        }
        if (tid == 0) TIMELINE(5);
        // this CTA's partial of the MoE output, every row (zeros if it had no units)
        float* part = a.partials + (size_t)b * D;
        if (kW2T) {
            // acc[i] holds rows (8 tid + 2i, 8 tid + 2i + 1)
            if (8 * tid < D) {
                float4* p4 = reinterpret_cast<float4*>(part + 8 * tid);
                p4[0] = make_float4(__uint_as_float((uint32_t)acc[0]), __uint_as_float((uint32_t)(acc[0] >> 32)),
                                    __uint_as_float((uint32_t)acc[1]), __uint_as_float((uint32_t)(acc[1] >> 32)));
                p4[1] = make_float4(__uint_as_float((uint32_t)acc[2]), __uint_as_float((uint32_t)(acc[2] >> 32)),
                                    __uint_as_float((uint32_t)acc[3]), __uint_as_float((uint32_t)(acc[3] >> 32)));
            }
        } else {
#pragma unroll
            for (int j = 0; j < kRowsPerThread; j++) {
                const int d = tid + kConsumers * j;
                if (d < D) part[d] = f2sum(acc[j]);
            }
        }
        if (!ok && lane == 0) s_fail = 1;
        // this CTA's band of output rows; the residual x of the band is read now, off
        // the critical path (only this CTA writes these rows, after the barrier)
        const int n4 = D / 4;
        const int c0 = (int)((long)n4 * b / G), c1 = (int)((long)n4 * (b + 1) / G);
        const int nc = c1 - c0;
        const int col = tid >> 3, grp = tid & 7;  // 32 float4 columns x 8 groups of CTAs per pass
        float4 xres = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.ffn_norm && grp == 0 && col < nc) xres = __ldcg(reinterpret_cast<const float4*>(a.x) + c0 + col);
        named_sync(1, kConsumers);
        if (tid == 0 && !s_fail) {
            // release: this CTA's partial (ordered before by the named barrier) is
            // visible at gpu scope before the arrival is
            // The count before this arrival is n G + m (m arrivals of this launch came
            // first), so the barrier completes at (n + 1) G; the last arrival needs no poll.
            unsigned long long before;
            asm volatile("atom.release.gpu.global.add.u64 %0, [%1], 1;" : "=l"(before) : "l"(bar_cnt) : "memory");
            const unsigned long long target = (before / (unsigned)G + 1) * (unsigned)G;
            if (before + 1 < target && !wait_count(bar_cnt, target, peer_ns)) {
                record_error(a.status, 0x602);
                s_fail = 1;
            }
        }
        named_sync(1, kConsumers);
        if (tid == 0) TIMELINE(6);
        if (!s_fail) {
            // every CTA has read the logits (before it arrived): clear them for the next launch
            if (b == 0)
                for (int e = tid; e < E; e += kConsumers) lword[(size_t)e * kLogitStride] = 0ull;
#ifdef RBT_DECODE_TIMELINE
            if (b == 0 && tid == 0) atomicAdd(&g_timeline_seq, 1u);
#endif
            // the next layer's router row and ffn_norm into L2 for its first phase
            if (tid == 32 && a.next_router && b < E)
                prefetch_l2(a.next_router + (size_t)b * D * 2, (uint32_t)D * 2);
            if (tid == 64 && a.next_norm && b == G - 1) prefetch_l2(a.next_norm, (uint32_t)D * 4);
        }
        // band reduction: float4 column c0 + col (4 rows) summed over the CTAs
        // g = grp, grp + 8, ... in order, then a fixed pairwise tree over the 8
        // groups; the loads of a pass are all in flight together
        constexpr int kLdR = 20;
        for (int cb = 0; !s_fail && cb < nc; cb += kConsumers / 8) {
            const int cc = cb + col;
            float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (cc < nc) {
                const float4* src = reinterpret_cast<const float4*>(a.partials) + c0 + cc;
                for (int gb = grp; gb < G; gb += 8 * kLdR) {
                    float4 v[kLdR];
#pragma unroll
                    for (int k = 0; k < kLdR; k++) {
                        const int g = gb + 8 * k;
                        v[k] = g < G ? __ldcg(src + (size_t)g * n4) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int k = 0; k < kLdR; k++) {
                        s4.x += v[k].x;
                        s4.y += v[k].y;
                        s4.z += v[k].z;
                        s4.w += v[k].w;
                    }
                }
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                s4.x += __shfl_xor_sync(FULL_MASK, s4.x, o);
                s4.y += __shfl_xor_sync(FULL_MASK, s4.y, o);
                s4.z += __shfl_xor_sync(FULL_MASK, s4.z, o);
                s4.w += __shfl_xor_sync(FULL_MASK, s4.w, o);
            }
            if (grp == 0 && cc < nc) {
                float4 xv = xres;
                if (cb > 0 && a.ffn_norm) xv = __ldcg(reinterpret_cast<const float4*>(a.x) + c0 + cc);
                float* o = a.out + 4 * (size_t)(c0 + cc);
                if (a.ffn_norm) {
                    o[0] = __fadd_rn(xv.x, s4.x);
                    o[1] = __fadd_rn(xv.y, s4.y);
                    o[2] = __fadd_rn(xv.z, s4.z);
                    o[3] = __fadd_rn(xv.w, s4.w);
                } else {
                    o[0] = s4.x;
                    o[1] = s4.y;
                    o[2] = s4.z;
                    o[3] = s4.w;
                }
            }
        }
    }
    if (tid == 0) TIMELINE(7);
}

// w2t[e][r][d] = w2[e][d][r]: one expert per blockIdx.z, 32 x 32 tiles through shared memory
__global__ void transpose_w2_kernel(const uint8_t* experts, size_t stride, int D, int H, uint16_t* w2t) {
    __shared__ uint16_t tile[32][33];
    const int e = blockIdx.z;
    const uint16_t* w2 = reinterpret_cast<const uint16_t*>(experts + (size_t)e * stride + (size_t)2 * H * D * 2);
    uint16_t* out = w2t + (size_t)e * H * D;
    const int r0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int d = d0 + j, r = r0 + threadIdx.x;
        if (d < D && r < H) tile[j][threadIdx.x] = w2[(size_t)d * H + r];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = r0 + j, d = d0 + threadIdx.x;
        if (d < D && r < H) out[(size_t)r * D + d] = tile[threadIdx.x][j];
    }
}

bool g_pdl_refused = false;

// RBT_MOE_DECODE_PDL=0 launches without programmatic dependent launch
bool decode_pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("RBT_MOE_DECODE_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

}  // namespace

int decode_sync_words(int E, int K) { return kSyncHead + 2 * kLogitStride * E + K; }

size_t decode_partials_bytes(int grid, int D) { return (size_t)grid * D * sizeof(float); }

cudaError_t transpose_w2(const void* experts, size_t stride, int D, int H, int E, void* w2t, cudaStream_t s) {
    if (E <= 0) return cudaSuccess;
    transpose_w2_kernel<<<dim3((H + 31) / 32, (D + 31) / 32, E), dim3(32, 8), 0, s>>>(
        static_cast<const uint8_t*>(experts), stride, D, H, static_cast<uint16_t*>(w2t));
    return cudaGetLastError();
}

bool decode_fused_supported(int T, int D, int H, int E, int K, int dtype, const void* experts, size_t stride,
                            const void* x, const void* router) {
    return T == 1 && dtype == 1 && D % 16 == 0 && D <= kMaxD && H % kGURows == 0 && E <= kMaxExperts &&
           K <= kMaxTopK && K <= E && w2_offset(D) + w2_boxes(D) * w2_box_rows(D) * kGURows * 2 <= kSlot &&
           stride % 16 == 0 && (reinterpret_cast<uintptr_t>(experts) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(x) % 16) == 0 && (reinterpret_cast<uintptr_t>(router) % 16) == 0;
}

bool make_decode_w2_map(CUtensorMap* map, const void* experts, int D, int H, int E, size_t stride) {
    // w2 of expert e is the row-major [D, H] matrix at experts + e*stride + 2*H*D*2;
    // a box is 8 columns (one unit's hidden rows) by up to 256 output rows
    const uint8_t* w2 = static_cast<const uint8_t*>(experts) + (size_t)2 * H * D * 2;
    return make_map_3d_plain(map, w2, H, D, E, stride, kGURows, w2_box_rows(D));
}

cudaError_t launch_decode_fused(const DecodeArgs& a, const CUtensorMap& w2map, int grid, cudaStream_t s) {
    const int rows_per_cta = (a.E + grid - 1) / grid;
    if ((size_t)rows_per_cta * a.D * 2 > (size_t)kWrowBytes || a.D * 4 > kProdOff - kXsOff ||
        (size_t)grid * ((a.D / 4 + grid - 1) / grid) * 16 > (size_t)kSlots * kSlot)
        return cudaErrorInvalidValue;
    auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) != 0; };
    // every pointer the kernel bulk-copies or prefetches from must be 16-byte aligned
    if ((a.w2t && (a.w2t_stride % 16 != 0 || misaligned(a.w2t))) || misaligned(a.ffn_norm) ||
        misaligned(a.next_router) || misaligned(a.next_norm) || misaligned(a.x) || misaligned(a.router) ||
        misaligned(a.experts))
        return cudaErrorMisalignedAddress;
    const size_t smem = (size_t)kSlots * kSlot;
    cudaError_t err = cudaFuncSetAttribute(moe_decode_fused_kernel<true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err == cudaSuccess)
        err = cudaFuncSetAttribute(moe_decode_fused_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (g_pdl_refused || !decode_pdl_enabled()) ? 1 : 2;
    auto kernel = a.w2t ? moe_decode_fused_kernel<true> : moe_decode_fused_kernel<false>;
    DecodeArgs b = a;
    b.expf_fma = host_expf_fma();
    err = cudaLaunchKernelEx(&cfg, kernel, b, w2map);
    if (err != cudaSuccess && cfg.numAttrs == 2) {
        // a driver that refuses the pair launches without the overlap
        (void)cudaGetLastError();
        g_pdl_refused = true;
        cfg.numAttrs = 1;
        err = cudaLaunchKernelEx(&cfg, kernel, b, w2map);
    }
    return err;
}

}  // namespace rbt

#ifdef RBT_DECODE_TIMELINE
extern "C" int rbt_decode_timeline_read(void* host) {
    return cudaMemcpyFromSymbol(host, rbt::g_timeline, sizeof(rbt::g_timeline)) == cudaSuccess;
}
extern "C" int rbt_decode_timeline_seq(void) {
    unsigned v = 0;
    cudaMemcpyFromSymbol(&v, rbt::g_timeline_seq, sizeof v);
    return (int)v;
}
#endif
