// decode_fused.cu -- the whole MoE block for ONE token in one persistent kernel
// (bf16 models): rabbit2.c:512-542 -- RMSNorm, router, softmax, top-k, the k
// experts' SwiGLU FFNs, the weighted combine and the residual -- as a single
// cooperative launch of one CTA per SM.  Batch-1 decode is memory-bound on the
// K experts' weights (8 x 12 MB at OLMoE-1B-7B), so the kernel exists to keep
// HBM streaming and to avoid launch gaps and cross-kernel drains.
//
// Phases (grid barriers are bounded spins on a global counter; the launch is
// cooperative, so every CTA is resident):
//   0  every CTA: x (and rmsnorm(x) for the block form) into shared memory --
//      the same deterministic reduction everywhere, so every CTA holds the same xb
//   1  CTA b computes router logits e = b, b+G, ...: the four sequential chains
//      of the reference's scalar matvec (rabbit2.c:378-387), separately rounded
//      products and sums, combined (s0+s1)+(s2+s3); logits to global
//   -- grid barrier 1
//   2  every CTA: softmax and top-k from the E logits (one warp, exactly as the
//      router kernel), the K slots sorted by expert; CTA 0 publishes routing
//   3  gate/up: the producer thread streams 8 rows of w1 and of w3 per unit with
//      cp.async.bulk into a 3 x 64 KB ring; 8 consumer warps form
//      h = silu(w1 . x) * (w3 . x) with packed fma.rn.f32x2 (x in registers)
//   -- grid barrier 2 (consumer warps only: the producer is already streaming
//      w2 rows into the ring, which do not depend on h)
//   4  down + combine + residual: h of the K slots in shared memory; units of
//      2 output rows x K experts; out[d] = x[d] + sum_k w_k y_k[d], k in
//      selection order (rabbit2.c:539-542)
// Every wait (mbarrier or grid barrier) is bounded by %globaltimer; a timeout
// records a code in `status` and the kernel unwinds.
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
constexpr int kDR = 2;             // w2 rows per down unit
constexpr int kHBuf = 32768;       // h of the K slots, bytes
constexpr uint64_t kWaitNs = 2000000000ull;

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

// One thread: publish this CTA's writes, arrive, and wait until `target` CTAs
// have arrived.  Returns false on timeout.
__device__ bool grid_arrive_wait(unsigned* counter, unsigned target) {
    __threadfence();
    atomicAdd(counter, 1u);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire(counter) < target) {
        if (globaltimer_ns() - t0 > kWaitNs) return false;
        __nanosleep(64);
    }
    return true;
}

__global__ void __launch_bounds__(kThreads, 1) moe_decode_fused_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    float* hbuf = reinterpret_cast<float*>(smem + kSlots * kSlot);        // [K][H]
    float* ybuf = hbuf + kHBuf / 4;                                       // [2 units][K][kDR]
    static_assert(kSlot >= kMaxExperts * 4, "softmax scratch lives in ring slot 2");
    __shared__ uint64_t full[kSlots], empty[kSlots], hbar;
    __shared__ int32_t s_idx[kMaxTopK], s_pos[kMaxTopK], s_act[kMaxTopK];
    __shared__ float s_p[kMaxTopK], s_w[kMaxTopK];
    __shared__ float s_red[kThreads / 32];
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = a.D, H = a.H, E = a.E, K = a.K;
    const int G = gridDim.x;
    float* xs = reinterpret_cast<float*>(ring);             // phase 0-2: xb [D]
    float* wrow = reinterpret_cast<float*>(ring + kSlot);   // phase 1: one router row as f32 [D]
    float* s_ex = reinterpret_cast<float*>(ring + 2 * kSlot);  // phase 2: exp(l - max) [E]

    if (tid == 0) {
        s_fail = 0;
        for (int s = 0; s < kSlots; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        mbar_init(&hbar, 1);
        fence_mbar_init();
    }
    // ---------------------------------------------------------------- phase 0
    for (int i = tid * 4; i < D; i += kThreads * 4) *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(a.x + i);
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
    for (int e = blockIdx.x; e < E; e += G) {
        for (int i = tid * 8; i < D; i += kThreads * 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(a.router + (size_t)e * D + i);
            float f[8];
            WeightTraits<uint16_t>::unpack(v, f);
            *reinterpret_cast<float4*>(wrow + i) = make_float4(f[0], f[1], f[2], f[3]);
            *reinterpret_cast<float4*>(wrow + i + 4) = make_float4(f[4], f[5], f[6], f[7]);
        }
        __syncthreads();
        if (warp == 0) {
            float s = 0.0f;
            if (lane < 4) {
                int i = lane;
                for (; i + 28 < D; i += 32) {
                    float w[8], x[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        w[u] = wrow[i + 4 * u];
                        x[u] = xs[i + 4 * u];
                    }
#pragma unroll
                    for (int u = 0; u < 8; u++) s = __fadd_rn(s, __fmul_rn(w[u], x[u]));
                }
                for (; i < D; i += 4) s = __fadd_rn(s, __fmul_rn(wrow[i], xs[i]));
            }
            const float s1 = __shfl_down_sync(FULL_MASK, s, 1);
            const float a01 = __fadd_rn(s, s1);
            const float a23 = __shfl_down_sync(FULL_MASK, a01, 2);
            if (lane == 0) {
                float logit = __fadd_rn(a01, a23);
                if (a.bias) logit = __fadd_rn(logit, a.bias[e]);
                a.logits[e] = logit;
            }
        }
        __syncthreads();
    }
    __syncthreads();
    if (tid == 0 && !grid_arrive_wait(a.bar, (unsigned)G)) {
        record_error(a.status, 0x601);
        s_fail = 1;
    }
    __syncthreads();
    // ---------------------------------------------------------------- phase 2: softmax, top-k, slot order
    if (warp == 0 && !s_fail) {
        constexpr int NJ = kMaxExperts / 32;
        float l[NJ], p[NJ];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            l[j] = (e < E) ? __ldcg(a.logits + e) : -INFINITY;
            mx = fmaxf(mx, l[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL_MASK, mx, o));
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            p[j] = (e < E) ? (float)exp((double)__fsub_rn(l[j], mx)) : 0.0f;
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
                s_p[k] = bp;
            }
        }
        __syncwarp();
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
        if (blockIdx.x == 0) {  // the routing outputs of the call
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
    const uint32_t gu_half = (uint32_t)kGURows * D * 2;         // 8 rows of w1 (or w3)
    const uint32_t dn_rows = (uint32_t)kDR * H * 2;             // 2 rows of w2 of one expert
    const int units_per_e = H / kGURows;
    const int n_gu = fail0 ? 0 : K * units_per_e;
    const int g0 = (int)((long)n_gu * blockIdx.x / G), g1 = (int)((long)n_gu * (blockIdx.x + 1) / G);
    const int n_dn = fail0 ? 0 : D / kDR;
    const int d0 = (int)((long)n_dn * blockIdx.x / G), d1 = (int)((long)n_dn * (blockIdx.x + 1) / G);

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
            }
            for (int u = d0; ok && u < d1; u += 2) {  // two down units per slot
                if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, kWaitNs)) {
                    record_error(a.status, 0x612);
                    ok = false;
                    break;
                }
                const int nu = min(2, d1 - u);
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
        // every CTA's h rows are written before any CTA reads h
        named_sync(1, kWarps * 32);
        if (tid == 0) {
            if (!ok || s_fail || !grid_arrive_wait(a.bar, (unsigned)(2 * G))) {
                if (ok && !s_fail) record_error(a.status, 0x602);
                s_fail = 1;
            } else {
                mbar_arrive_expect_tx(&hbar, (uint32_t)K * H * 4);
                bulk_load(hbuf, a.h, (uint32_t)K * H * 4, &hbar);
            }
        }
        named_sync(1, kWarps * 32);
        ok = ok && !s_fail;
        if (ok) {
            const bool got = mbar_wait_bounded(&hbar, 0, kWaitNs);
            if (!__all_sync(FULL_MASK, got)) {
                record_error(a.status, 0x622);
                ok = false;
            }
        }
        if (!ok && lane == 0) s_fail = 1;
        named_sync(1, kWarps * 32);
        // from here `ok` only changes through s_fail after a named barrier, so all
        // consumer warps take the same number of barriers
        for (int u = d0; !s_fail && u < d1; u += 2) {
            const bool got = mbar_wait_bounded(&full[slot], ph, kWaitNs);
            if (!__all_sync(FULL_MASK, got)) {
                record_error(a.status, 0x623);
                ok = false;
                if (lane == 0) s_fail = 1;
            }
            const int nu = min(2, d1 - u);
            const uint8_t* st = ring + slot * kSlot;
            if (ok) {
                for (int task = warp; task < nu * K * kDR; task += kWarps) {
                    const int jr = task / kDR, rr = task - jr * kDR;    // jr = j*K + pa
                    const int pa = jr % K;
                    const uint4* w = reinterpret_cast<const uint4*>(st + jr * dn_rows + rr * H * 2);
                    const float* hv = hbuf + (size_t)pa * H;
                    uint64_t acc[4] = {0, 0, 0, 0};
                    for (int v = lane; v < nvh; v += 32) {
                        const uint4 q = w[v];
                        const float4 h0 = *reinterpret_cast<const float4*>(hv + v * 8);
                        const float4 h1 = *reinterpret_cast<const float4*>(hv + v * 8 + 4);
                        acc[0] = ffma2(bf2(q.x), f2(h0.x, h0.y), acc[0]);
                        acc[1] = ffma2(bf2(q.y), f2(h0.z, h0.w), acc[1]);
                        acc[2] = ffma2(bf2(q.z), f2(h1.x, h1.y), acc[2]);
                        acc[3] = ffma2(bf2(q.w), f2(h1.z, h1.w), acc[3]);
                    }
                    const float s = warp_sum((f2sum(acc[0]) + f2sum(acc[1])) + (f2sum(acc[2]) + f2sum(acc[3])));
                    if (lane == 0) ybuf[jr * kDR + rr] = s;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == kSlots) { slot = 0; ph ^= 1u; }
            named_sync(1, kWarps * 32);
            ok = !s_fail;
            if (ok && tid < nu * kDR) {  // combine in selection order, then the residual
                const int j = tid / kDR, rr = tid - j * kDR;
                const int d = (u + j) * kDR + rr;
                float mo = 0.0f;
                for (int k = 0; k < K; k++) mo = __fadd_rn(mo, __fmul_rn(s_w[k], ybuf[(j * K + s_pos[k]) * kDR + rr]));
                a.out[d] = a.ffn_norm ? __fadd_rn(a.x[d], mo) : mo;
            }
            named_sync(1, kWarps * 32);
        }
    }
    __syncthreads();
    if (tid == 0) {  // the last CTA out returns the barrier counters to zero
        __threadfence();
        if (atomicAdd(a.bar + 1, 1u) == (unsigned)G - 1) {
            atomicExch(a.bar, 0u);
            atomicExch(a.bar + 1, 0u);
        }
    }
}

}  // namespace

bool decode_fused_supported(int T, int D, int H, int E, int K, int dtype, const void* experts, size_t stride,
                            const void* x, const void* router) {
    return T == 1 && dtype == 1 && D % 8 == 0 && D <= 2048 && H % kGURows == 0 && H % 8 == 0 && D % kDR == 0 &&
           E <= kMaxExperts && K <= kMaxTopK && (size_t)K * H * 4 <= (size_t)kHBuf &&
           2 * kGURows * D * 2 <= kSlot && 2 * K * kDR * H * 2 <= kSlot && stride % 16 == 0 &&
           (reinterpret_cast<uintptr_t>(experts) % 16) == 0 && (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
           (reinterpret_cast<uintptr_t>(router) % 16) == 0;
}

cudaError_t launch_decode_fused(const DecodeArgs& a, int grid, cudaStream_t s) {
    const size_t smem = (size_t)kSlots * kSlot + kHBuf + 2 * (size_t)a.K * kDR * 4;
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
