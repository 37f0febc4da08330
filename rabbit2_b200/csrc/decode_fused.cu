// decode_fused.cu -- the whole MoE block for ONE token in one persistent kernel
// (bf16 models): rabbit2.c:512-542 -- RMSNorm, router, softmax, top-k, the k
// experts' SwiGLU FFNs, the weighted combine and the residual -- as a single
// cooperative launch of one CTA per SM.  Batch-1 decode is memory-bound on the
// K experts' weights (8 x 12 MB at OLMoE-1B-7B), so the kernel exists to keep
// HBM streaming: no launch gaps and no kernel-boundary drains.  Cross-CTA
// ordering is by counters in global memory (release by __threadfence +
// atomic, acquire by ld.acquire), each wait bounded by %globaltimer; the launch
// is cooperative, so every CTA is resident and every wait ends.
//
//   0  every CTA: bulk-copies x (and, if it computes one, its router row) into
//      shared memory; rmsnorm(x) for the block form, the same fixed-order
//      reduction in every CTA so all hold the same xb
//   1  CTAs compute router logits -- the four sequential chains of the
//      reference's scalar matvec (rabbit2.c:378-387), separately rounded
//      products and sums, (s0+s1)+(s2+s3) -- each expert by two CTAs when the
//      grid has room; the first copy to finish publishes it (both are equal)
//   2  every CTA, as soon as all E logits are published: softmax and top-k
//      (selection order = rank: higher probability, or equal and lower index),
//      the K slots sorted by expert; CTA 0 publishes the routing outputs
//   3  gate/up: each CTA takes a contiguous range of units (8 rows of w1 and
//      the same 8 rows of w3); as soon as routing is known its producer thread
//      issues L2 prefetches for every weight byte the CTA will need (gate/up
//      units and its w2 rows), so HBM streams continuously while the
//      units pass through a 3 x 64 KB shared-memory ring (cp.async.bulk, now L2
//      hits); 8 consumer warps form h = silu(w1 . x) * (w3 . x) (packed
//      fma.rn.f32x2, x in registers)
//   -- grid barrier (consumer warps only; the producer keeps loading w2 rows)
//   4  down + combine: units of 2 output rows x the K experts; consumer warp w
//      keeps the h rows of chosen experts w and w+8 in registers; then
//      out[d] = x[d] + sum_k w_k y_k[d] in selection order (rabbit2.c:539-542)
// The last CTA to leave returns every counter to zero.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rbt {
namespace {

using namespace tc;

constexpr int kWarps = 8;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kSlot = 65536;       // ring slot bytes
constexpr int kSlots = 3;
constexpr int kGURows = 8;         // w1/w3 rows per gate-up unit
constexpr int kMaxH = 1024;        // a lane's slice of one h row stays in registers (H / 256 vectors)
constexpr int kDR = 2;             // w2 rows per down unit
constexpr uint64_t kWaitNs = 2000000000ull;

// sync words (a.sync): [0] CTAs done, [1] grid-barrier arrivals, [2..3] unused,
// [4, 4+E) logit published, [4+E, 4+E+K) unused
constexpr int kSyncHead = 4;

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

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Spin (bounded) until *p >= target.
__device__ __forceinline__ bool wait_count(const unsigned* p, unsigned target) {
    if (ld_acquire(p) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire(p) < target) {
        if (globaltimer_ns() - t0 > kWaitNs) return false;
        __nanosleep(32);
    }
    return true;
}

__global__ void __launch_bounds__(kThreads, 1) moe_decode_fused_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    float* ybuf = reinterpret_cast<float*>(smem + kSlots * kSlot);  // [band rows][K]
    __shared__ uint64_t full[kSlots], empty[kSlots], xbar, rbar;
    __shared__ int32_t s_idx[kMaxTopK], s_pos[kMaxTopK], s_act[kMaxTopK];
    __shared__ float s_p[kMaxTopK], s_w[kMaxTopK], s_prob[kMaxExperts];
    __shared__ float s_red[kThreads / 32];
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = a.D, H = a.H, E = a.E, K = a.K;
    const int G = gridDim.x, b = blockIdx.x;
    unsigned* done_cnt = a.sync;
    unsigned* bar_cnt = a.sync + 1;
    unsigned* lflag = a.sync + kSyncHead;
    float* xs = reinterpret_cast<float*>(ring);                   // phases 0-2: xb [D]
    uint16_t* wrow = reinterpret_cast<uint16_t*>(ring + kSlot);   // phase 1: this CTA's router rows

    // router rows this CTA computes: two copies of every expert when the grid has room
    const bool dup = G >= 2 * E;
    const int e_first = dup ? (b < 2 * E ? b % E : E) : b;
    const int e_step = dup ? E : G;
    int n_rows = 0;
    for (int e = e_first; e < E; e += e_step) n_rows++;
    if (dup && n_rows > 1) n_rows = 1;

    if (tid == 0) {
        s_fail = 0;
        for (int s = 0; s < kSlots; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        mbar_init(&xbar, 1);
        mbar_init(&rbar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&xbar, (uint32_t)D * 4);
        bulk_load(xs, a.x, (uint32_t)D * 4, &xbar);
        if (n_rows > 0) {
            mbar_arrive_expect_tx(&rbar, (uint32_t)n_rows * D * 2);
            for (int j = 0; j < n_rows; j++)
                bulk_load(wrow + (size_t)j * D, a.router + (size_t)(e_first + j * e_step) * D, (uint32_t)D * 2, &rbar);
        }
    }
    // ---------------------------------------------------------------- phase 0
    __syncthreads();
    if (!mbar_wait_bounded(&xbar, 0, kWaitNs)) {
        record_error(a.status, 0x604);
        s_fail = 1;
    }
    __syncthreads();
    if (a.ffn_norm) {  // rmsnorm, the same fixed-order reduction in every CTA
        float ss = 0.0f;
        for (int i = tid; i < D; i += kThreads) ss = fmaf(xs[i], xs[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int w = 0; w < kThreads / 32; w++) tot += s_red[w];
        const float inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tot, (float)D), a.eps));
        __syncthreads();
        for (int i = tid; i < D; i += kThreads) xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), a.ffn_norm[i]);
        __syncthreads();
    }
    // ---------------------------------------------------------------- phase 1: exact router logits
    // The products w[i]*x[i] are independent: every thread rounds its share of
    // them into `prods`, laid out chain-major (chain c = i mod 4 holds its D/4
    // products contiguously).  Lane c of warp 0 then runs chain c's D/4
    // dependent adds in order, reading 4 products per 16-byte load.
    float* prods = reinterpret_cast<float*>(ring + 2 * kSlot);  // [4][D/4]
    for (int j = 0; j < n_rows; j++) {
        const int e = e_first + j * e_step;
        if (j == 0) {
            const bool got = mbar_wait_bounded(&rbar, 0, kWaitNs);
            if (!got) {
                record_error(a.status, 0x600);
                s_fail = 1;
            }
        }
        __syncthreads();
        if (s_fail) break;
        const uint16_t* wr = wrow + (size_t)j * D;
        const int q = D / 4;
        for (int i = tid; i < 4 * q; i += kThreads)
            prods[(i & 3) * q + (i >> 2)] = __fmul_rn(bf16_bits_to_f32(wr[i]), xs[i]);
        __syncthreads();
        if (warp == 0) {
            float s = 0.0f;
            if (lane < 4) {
                const float* pc = prods + lane * q;
                int i = 0;
                for (; i + 4 <= q; i += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(pc + i);
                    s = __fadd_rn(s, v.x);
                    s = __fadd_rn(s, v.y);
                    s = __fadd_rn(s, v.z);
                    s = __fadd_rn(s, v.w);
                }
                for (; i < q; i++) s = __fadd_rn(s, pc[i]);
            }
            const float s1 = __shfl_down_sync(FULL_MASK, s, 1);
            const float a01 = __fadd_rn(s, s1);
            const float a23 = __shfl_down_sync(FULL_MASK, a01, 2);
            if (lane == 0) {
                float logit = __fadd_rn(a01, a23);
                if (a.bias) logit = __fadd_rn(logit, a.bias[e]);
                a.logits[e] = logit;  // both copies write the same bits
                __threadfence();
                atomicExch(lflag + e, 1u);
            }
        }
        __syncthreads();
    }
    // ---------------------------------------------------------------- phase 2: softmax, top-k, slot order
    if (warp == 0) {
        bool ok = true;
        for (int e = lane; e < E; e += 32) ok = ok && wait_count(lflag + e, 1u);
        if (!__all_sync(FULL_MASK, ok)) {
            if (lane == 0) {
                record_error(a.status, 0x601);
                s_fail = 1;
            }
        }
    }
    __syncthreads();
    if (warp == 0 && !s_fail) {
        constexpr int NJ = kMaxExperts / 32;
        const int nj = (E + 31) / 32;
        float l[NJ], p[NJ];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            l[j] = (j < nj && e < E) ? __ldcg(a.logits + e) : -INFINITY;
            mx = fmaxf(mx, l[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, o));
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            p[j] = (j < nj && e < E) ? (float)exp((double)__fsub_rn(l[j], mx)) : 0.0f;
        }
        // the sequential sum in expert order (rabbit2.c:403), values passed by shuffles
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            if (j < nj) {
#pragma unroll
                for (int src = 0; src < 32; src++) {
                    const float v = __shfl_sync(FULL_MASK, p[j], src);
                    if (32 * j + src < E) sum = __fadd_rn(sum, v);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            if (j < nj && e < E) s_prob[e] = __fdiv_rn(p[j], sum);
        }
    }
    __syncthreads();
    // top-k by rank: expert e is chosen in round r when exactly r experts beat it
    // (higher probability, or equal probability and lower index) -- the order of
    // the reference's K rounds of strict-'>' scans (rabbit2.c:519-528)
    if (!s_fail && tid < E) {
        const float pe = s_prob[tid];
        int r = 0;
        for (int f = 0; f < E; f++) {
            const float pf = s_prob[f];
            r += (pf > pe) || (pf == pe && f < tid);
        }
        if (r < K) {
            s_idx[r] = tid;
            s_p[r] = pe;
        }
    }
    __syncthreads();
    if (warp == 0 && !s_fail) {
        float wsum = 0.0f;
        for (int k = 0; k < K; k++) wsum = __fadd_rn(wsum, s_p[k]);
        for (int k = lane; k < K; k += 32) {
            s_w[k] = a.norm_topk ? __fdiv_rn(s_p[k], wsum) : s_p[k];
            int pos = 0;  // rank of this slot's expert among the chosen ones
            for (int j = 0; j < K; j++) pos += s_idx[j] < s_idx[k];
            s_pos[k] = pos;
            s_act[pos] = s_idx[k];
        }
        __syncwarp();
        if (b == 0) {  // the routing outputs of the call
            for (int k = lane; k < K; k += 32) {
                a.idx[k] = s_idx[k];
                a.wt[k] = s_w[k];
                a.slot_pos[k] = s_pos[k];
                a.perm[s_pos[k]] = k;
                a.active[s_pos[k]] = s_idx[k];
                if (a.routing_out) a.routing_out[k] = s_idx[k];
            }
            for (int e = lane; e < E; e += 32) {
                int c = 0, below = 0;
                for (int k = 0; k < K; k++) {
                    c += s_idx[k] == e;
                    below += s_idx[k] < e;
                }
                a.counts[e] = c;
                a.offsets[e] = below;
            }
            if (lane == 0) {
                a.offsets[E] = K;
                *a.n_active = K;
            }
        }
    }
    __syncthreads();
    const bool fail0 = s_fail != 0;

    const int nvx = D / 8;   // 16-byte vectors per w1/w3 row
    const int nvh = H / 8;   // per w2 row
    const uint32_t gu_half = (uint32_t)kGURows * D * 2;  // 8 rows of w1 (or w3)
    const uint32_t dn_rows = (uint32_t)kDR * H * 2;      // 2 rows of w2 of one expert
    const int units_per_e = H / kGURows;
    const int n_gu = fail0 ? 0 : K * units_per_e;
    const int g0 = (int)((long)n_gu * b / G), g1 = (int)((long)n_gu * (b + 1) / G);
    const int n_dn = fail0 ? 0 : D / kDR;
    const int d0 = (int)((long)n_dn * b / G), d1 = (int)((long)n_dn * (b + 1) / G);
    const int ups = (int)(kSlot / ((uint32_t)K * dn_rows)) >= 2 ? 2 : 1;  // down units per ring slot

    // consumer lanes keep their slice of xb in registers before the ring is reused
    float xr[64];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int v = lane + 32 * j;
#pragma unroll
        for (int q = 0; q < 8; q++) xr[8 * j + q] = (v < nvx) ? xs[v * 8 + q] : 0.0f;
    }
    __syncthreads();

    if (warp == kWarps) {
        // ------------------------------------------------------------ producer
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
                const int e = s_act[u / units_per_e], rg = u % units_per_e;
                const uint8_t* w1 = a.experts + (size_t)e * a.stride + (size_t)rg * gu_half;
                uint8_t* st = ring + slot * kSlot;
                mbar_arrive_expect_tx(&full[slot], 2 * gu_half);
                bulk_load(st, w1, gu_half, &full[slot]);
                bulk_load(st + gu_half, w1 + (size_t)H * D * 2, gu_half, &full[slot]);
                issued++;
                if (++slot == kSlots) { slot = 0; ph ^= 1u; }
                if (issued == kSlots || u + 1 == g1) {
                    // the ring is full: ask L2 for everything else this CTA will read,
                    // so HBM keeps streaming however long the ring takes to drain
                    for (int v = u + 1; v < g1; v++) {
                        const uint8_t* p1 = a.experts + (size_t)s_act[v / units_per_e] * a.stride +
                                            (size_t)(v % units_per_e) * gu_half;
                        prefetch_l2(p1, gu_half);
                        prefetch_l2(p1 + (size_t)H * D * 2, gu_half);
                    }
                    if (d1 > d0)
                        for (int pa = 0; pa < K; pa++)
                            prefetch_l2(a.experts + (size_t)s_act[pa] * a.stride + (size_t)2 * H * D * 2 +
                                            (size_t)d0 * dn_rows,
                                        (uint32_t)(d1 - d0) * dn_rows);
                }
            }
            for (int u = d0; ok && u < d1; u += ups) {  // down units, `ups` per slot
                if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, kWaitNs)) {
                    record_error(a.status, 0x612);
                    ok = false;
                    break;
                }
                const int nu = min(ups, d1 - u);
                uint8_t* st = ring + slot * kSlot;
                mbar_arrive_expect_tx(&full[slot], nu * K * dn_rows);
                for (int j = 0; j < nu; j++)
                    for (int pa = 0; pa < K; pa++) {
                        const uint8_t* src = a.experts + (size_t)s_act[pa] * a.stride + (size_t)2 * H * D * 2 +
                                             (size_t)(u + j) * dn_rows;
                        bulk_load(st + (j * K + pa) * dn_rows, src, dn_rows, &full[slot]);
                    }
                issued++;
                if (++slot == kSlots) { slot = 0; ph ^= 1u; }
            }
            for (int i = 0; i < kSlots && i < issued; i++) {  // drain
                if (--slot < 0) { slot = kSlots - 1; ph ^= 1u; }
                if (!mbar_wait_bounded(&full[slot], ph, kWaitNs)) record_error(a.status, 0x613);
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        int slot = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int u = g0; ok && u < g1; u++) {
            const bool got = mbar_wait_bounded(&full[slot], ph, kWaitNs);
            if (!__all_sync(FULL_MASK, got)) {
                record_error(a.status, 0x621);
                ok = false;
                break;
            }
            const int pa = u / units_per_e, r = (u % units_per_e) * kGURows + warp;
            const uint4* w1 = reinterpret_cast<const uint4*>(ring + slot * kSlot + warp * D * 2);
            const uint4* w3 = reinterpret_cast<const uint4*>(ring + slot * kSlot + gu_half + warp * D * 2);
            uint64_t g[4] = {0, 0, 0, 0}, up[4] = {0, 0, 0, 0};
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = lane + 32 * j;
                if (v < nvx) {
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
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            const float gs = warp_sum((f2sum(g[0]) + f2sum(g[1])) + (f2sum(g[2]) + f2sum(g[3])));
            const float us = warp_sum((f2sum(up[0]) + f2sum(up[1])) + (f2sum(up[2]) + f2sum(up[3])));
            if (lane == 0) a.h[(size_t)pa * H + r] = gs / (1.0f + expf(-gs)) * us;
            if (++slot == kSlots) { slot = 0; ph ^= 1u; }
        }
        // every CTA's h rows are written (and every CTA has read x) before any
        // CTA reads h or writes out
        if (!ok && lane == 0) s_fail = 1;
        named_sync(1, kWarps * 32);
        if (tid == 0 && !s_fail) {
            __threadfence();
            atomicAdd(bar_cnt, 1u);
            if (!wait_count(bar_cnt, (unsigned)G)) {
                record_error(a.status, 0x602);
                s_fail = 1;
            }
        }
        named_sync(1, kWarps * 32);
        // warp w owns the chosen experts w and w + 8: their h rows stay in registers
        // for the whole phase, so shared memory only streams weights
        float hr[2][32];
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const int pa = warp + kWarps * q;
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const int v = lane + 32 * m;
                float4 h0 = make_float4(0.f, 0.f, 0.f, 0.f), h1 = h0;
                if (!s_fail && pa < K && v < nvh) {
                    h0 = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)pa * H + v * 8));
                    h1 = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)pa * H + v * 8 + 4));
                }
                hr[q][8 * m] = h0.x; hr[q][8 * m + 1] = h0.y; hr[q][8 * m + 2] = h0.z; hr[q][8 * m + 3] = h0.w;
                hr[q][8 * m + 4] = h1.x; hr[q][8 * m + 5] = h1.y; hr[q][8 * m + 6] = h1.z; hr[q][8 * m + 7] = h1.w;
            }
        }
        // the per-expert results of the CTA's whole output band collect in ybuf
        // ([row][slot position]); one barrier, then one combine
        for (int u = d0; ok && !s_fail && u < d1; u += ups) {
            const bool got = mbar_wait_bounded(&full[slot], ph, kWaitNs);
            if (!__all_sync(FULL_MASK, got)) {
                record_error(a.status, 0x623);
                ok = false;
                break;
            }
            const int nu = min(ups, d1 - u);
            const uint8_t* st = ring + slot * kSlot;
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const int pa = warp + kWarps * q;
                if (pa >= K) continue;
                for (int j = 0; j < nu; j++) {
#pragma unroll
                    for (int rr = 0; rr < kDR; rr++) {
                        const uint4* w = reinterpret_cast<const uint4*>(st + (j * K + pa) * dn_rows + rr * H * 2);
                        uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int m = 0; m < 4; m++) {
                            const int v = lane + 32 * m;
                            if (v < nvh) {
                                const uint4 qv = w[v];
                                acc[0] = ffma2(bf2(qv.x), f2(hr[q][8 * m], hr[q][8 * m + 1]), acc[0]);
                                acc[1] = ffma2(bf2(qv.y), f2(hr[q][8 * m + 2], hr[q][8 * m + 3]), acc[1]);
                                acc[2] = ffma2(bf2(qv.z), f2(hr[q][8 * m + 4], hr[q][8 * m + 5]), acc[2]);
                                acc[3] = ffma2(bf2(qv.w), f2(hr[q][8 * m + 6], hr[q][8 * m + 7]), acc[3]);
                            }
                        }
                        const float sd = warp_sum((f2sum(acc[0]) + f2sum(acc[1])) + (f2sum(acc[2]) + f2sum(acc[3])));
                        if (lane == 0) ybuf[((u - d0 + j) * kDR + rr) * K + pa] = sd;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == kSlots) { slot = 0; ph ^= 1u; }
        }
        if (!ok && lane == 0) s_fail = 1;
        named_sync(1, kWarps * 32);
        const int nrows = (d1 - d0) * kDR;
        if (!s_fail && tid < nrows) {  // combine in selection order, then the residual
            const int d = d0 * kDR + tid;
            float mo = 0.0f;
            for (int k = 0; k < K; k++) mo = __fadd_rn(mo, __fmul_rn(s_w[k], ybuf[tid * K + s_pos[k]]));
            a.out[d] = a.ffn_norm ? __fadd_rn(a.x[d], mo) : mo;
        }
    }
    __syncthreads();
    if (tid == 0) {  // the last CTA out returns every counter to zero
        __threadfence();
        if (atomicAdd(done_cnt, 1u) == (unsigned)G - 1) {
            for (int i = 1; i < kSyncHead + E + K; i++) atomicExch(a.sync + i, 0u);
            __threadfence();
            atomicExch(done_cnt, 0u);
        }
    }
}

}  // namespace

int decode_sync_words(int E, int K) { return kSyncHead + E + K; }

bool decode_fused_supported(int T, int D, int H, int E, int K, int dtype, const void* experts, size_t stride,
                            const void* x, const void* router) {
    return T == 1 && dtype == 1 && D % 16 == 0 && D <= 2048 && H % kGURows == 0 && H % 8 == 0 && H <= kMaxH &&
           D % kDR == 0 && E <= kMaxExperts && K <= 2 * kWarps && 2 * kGURows * D * 2 <= kSlot &&
           K * kDR * H * 2 <= kSlot && stride % 16 == 0 &&
           (reinterpret_cast<uintptr_t>(experts) % 16) == 0 && (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(router) % 16) == 0;
}

cudaError_t launch_decode_fused(const DecodeArgs& a, int grid, cudaStream_t s) {
    // the output band of a CTA (ceil((D/2)/grid) units of 2 rows) times K results
    const size_t band_rows = (size_t)kDR * ((a.D / kDR + grid - 1) / grid);
    const size_t smem = (size_t)kSlots * kSlot + band_rows * a.K * 4;
    cudaError_t err = cudaFuncSetAttribute(moe_decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, moe_decode_fused_kernel, a);
}

}  // namespace rbt
