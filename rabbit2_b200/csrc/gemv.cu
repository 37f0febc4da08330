// gemv.cu -- K3: grouped expert GEMV for decode-sized batches (CUDA cores).
// Replaces the three matvec calls per chosen expert of rabbit2.c:534-538.
//
// Each warp owns one weight row at a time and applies it to every routed slot
// of that expert (up to kMaxTok at once), so each expert row streams from HBM
// once per call: 16-byte non-temporal loads, eight in flight per lane per
// matrix, fp32 accumulation.  Work is a flat list of (active expert, row) tasks
// striped over all warps of a grid sized to the SM count.
//
// Layouts (HBM): expert blob e at experts + e*stride holds w1[H,D] | w3[H,D] |
// w2[D,H] row-major -- the .rbt2 blob, uploaded unchanged.  h[p, H] and y[p, D]
// are indexed by the slot's position p in expert-grouped order.
#include "common.cuh"
#include "exact_math.cuh"
#include "kernels.h"

namespace rbt {
namespace {

constexpr int kThreads = 256;
// MT: routed slots applied per pass over a weight row (1 when T == 1, where
// every chosen expert has one token); UNR: 16-byte vectors per lane in flight.

// silu(g) * u (rabbit2.c:407, :536) with the host's expf
__device__ __forceinline__ float silu_mul(float g, float u, int fma) { return __fmul_rn(silu_ref(g, fma), u); }

// acc[i] += dot(w[V], x_i[V]) for the m slots of this pass.
template <int V, int MT>
__device__ __forceinline__ void fma_vec(float (&acc)[MT], const float* w, const float* const (&xrow)[MT], int col,
                                        int m) {
#pragma unroll
    for (int i = 0; i < MT; i++) {
        if (i < m) {
            const float* xp = xrow[i] + col;
#pragma unroll
            for (int q = 0; q < V; q += 4) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(xp + q));
                acc[i] = fmaf(w[q], x.x, acc[i]);
                acc[i] = fmaf(w[q + 1], x.y, acc[i]);
                acc[i] = fmaf(w[q + 2], x.z, acc[i]);
                acc[i] = fmaf(w[q + 3], x.w, acc[i]);
            }
        }
    }
}

// gate/up: h[p, r] = silu(w1[r,:] . x_p) * (w3[r,:] . x_p)
template <typename WT, bool kVecPath, int kMaxTok>
__global__ void __launch_bounds__(kThreads) gateup_gemv_kernel(GemvArgs a) {
    constexpr int V = kVecPath ? WeightTraits<WT>::kVec : 1;
    constexpr int kUnroll = kMaxTok == 1 ? 8 : 4;
    const int lane = threadIdx.x & 31;
    const long gw = ((long)blockIdx.x * kThreads + threadIdx.x) >> 5;
    const long nw = ((long)gridDim.x * kThreads) >> 5;
    const int na = *a.n_active;
    const int H = a.H, D = a.D, K = a.K;
    const int nvec = D / V;
    const long tasks = (long)na * H;
    for (long task = gw; task < tasks; task += nw) {
        const int ai = (int)(task / H), r = (int)(task - (long)ai * H);
        const int e = a.active[ai];
        const int p0 = a.offsets[e], p1 = a.offsets[e + 1];
        const WT* w1 = reinterpret_cast<const WT*>(a.experts + (size_t)e * a.stride) + (size_t)r * D;
        const WT* w3 = w1 + (size_t)H * D;
        for (int pb = p0; pb < p1; pb += kMaxTok) {
            const int m = min(kMaxTok, p1 - pb);
            const float* xrow[kMaxTok];
#pragma unroll
            for (int i = 0; i < kMaxTok; i++) xrow[i] = a.xb + (size_t)(a.perm[pb + (i < m ? i : 0)] / K) * D;
            float acc1[kMaxTok], acc3[kMaxTok];
#pragma unroll
            for (int i = 0; i < kMaxTok; i++) acc1[i] = acc3[i] = 0.0f;
            if (kVecPath) {
                for (int v0 = 0; v0 < nvec; v0 += 32 * kUnroll) {
                    uint4 q1[kUnroll], q3[kUnroll];
#pragma unroll
                    for (int u = 0; u < kUnroll; u++) {
                        const int v = v0 + u * 32 + lane;
                        if (v < nvec) {
                            q1[u] = ld_stream16(w1 + (size_t)v * V);
                            q3[u] = ld_stream16(w3 + (size_t)v * V);
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kUnroll; u++) {
                        const int v = v0 + u * 32 + lane;
                        if (v < nvec) {
                            float f[V];
                            WeightTraits<WT>::unpack(q1[u], f);
                            fma_vec<V, kMaxTok>(acc1, f, xrow, v * V, m);
                            WeightTraits<WT>::unpack(q3[u], f);
                            fma_vec<V, kMaxTok>(acc3, f, xrow, v * V, m);
                        }
                    }
                }
            } else {
                for (int c = lane; c < D; c += 32) {
                    const float g = WeightTraits<WT>::load1(w1 + c), u = WeightTraits<WT>::load1(w3 + c);
#pragma unroll
                    for (int i = 0; i < kMaxTok; i++) {
                        if (i < m) {
                            const float x = xrow[i][c];
                            acc1[i] = fmaf(g, x, acc1[i]);
                            acc3[i] = fmaf(u, x, acc3[i]);
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < kMaxTok; i++) {
                if (i < m) {
                    const float g = warp_sum(acc1[i]), u = warp_sum(acc3[i]);
                    if (lane == 0) a.h[(size_t)(pb + i) * H + r] = silu_mul(g, u, a.expf_fma);
                }
            }
        }
    }
}

// down: y[p, d] = w2[d,:] . h_p, two rows per task
template <typename WT, bool kVecPath, int kMaxTok>
__global__ void __launch_bounds__(kThreads) down_gemv_kernel(GemvArgs a) {
    constexpr int V = kVecPath ? WeightTraits<WT>::kVec : 1;
    constexpr int kUnroll = kMaxTok == 1 ? 4 : 2;
    constexpr int R = 2;
    const int lane = threadIdx.x & 31;
    const long gw = ((long)blockIdx.x * kThreads + threadIdx.x) >> 5;
    const long nw = ((long)gridDim.x * kThreads) >> 5;
    const int na = *a.n_active;
    const int H = a.H, D = a.D;
    const int nvec = H / V;
    const int pairs = (D + R - 1) / R;
    const long tasks = (long)na * pairs;
    for (long task = gw; task < tasks; task += nw) {
        const int ai = (int)(task / pairs), d0 = (int)(task - (long)ai * pairs) * R;
        const int e = a.active[ai];
        const int p0 = a.offsets[e], p1 = a.offsets[e + 1];
        const int nr = min(R, D - d0);
        const WT* w2 = reinterpret_cast<const WT*>(a.experts + (size_t)e * a.stride) + (size_t)2 * H * D +
                       (size_t)d0 * H;
        for (int pb = p0; pb < p1; pb += kMaxTok) {
            const int m = min(kMaxTok, p1 - pb);
            const float* hrow[kMaxTok];
#pragma unroll
            for (int i = 0; i < kMaxTok; i++) hrow[i] = a.h + (size_t)(pb + (i < m ? i : 0)) * H;
            float acc[R][kMaxTok];
#pragma unroll
            for (int rr = 0; rr < R; rr++)
#pragma unroll
                for (int i = 0; i < kMaxTok; i++) acc[rr][i] = 0.0f;
            if (kVecPath) {
                for (int v0 = 0; v0 < nvec; v0 += 32 * kUnroll) {
                    uint4 q[R][kUnroll];
#pragma unroll
                    for (int rr = 0; rr < R; rr++)
#pragma unroll
                        for (int u = 0; u < kUnroll; u++) {
                            const int v = v0 + u * 32 + lane;
                            if (rr < nr && v < nvec) q[rr][u] = ld_stream16(w2 + (size_t)rr * H + (size_t)v * V);
                        }
#pragma unroll
                    for (int rr = 0; rr < R; rr++)
#pragma unroll
                        for (int u = 0; u < kUnroll; u++) {
                            const int v = v0 + u * 32 + lane;
                            if (rr < nr && v < nvec) {
                                float f[V];
                                WeightTraits<WT>::unpack(q[rr][u], f);
                                fma_vec<V, kMaxTok>(acc[rr], f, hrow, v * V, m);
                            }
                        }
                }
            } else {
                for (int c = lane; c < H; c += 32) {
#pragma unroll
                    for (int rr = 0; rr < R; rr++) {
                        if (rr < nr) {
                            const float w = WeightTraits<WT>::load1(w2 + (size_t)rr * H + c);
#pragma unroll
                            for (int i = 0; i < kMaxTok; i++)
                                if (i < m) acc[rr][i] = fmaf(w, hrow[i][c], acc[rr][i]);
                        }
                    }
                }
            }
#pragma unroll
            for (int rr = 0; rr < R; rr++)
#pragma unroll
                for (int i = 0; i < kMaxTok; i++) {
                    if (rr < nr && i < m) {
                        const float s = warp_sum(acc[rr][i]);
                        if (lane == 0) a.y[(size_t)(pb + i) * D + d0 + rr] = s;
                    }
                }
        }
    }
}

// 16-byte vectors are usable when every row start is 16-byte aligned.
bool vec_ok(const GemvArgs& a) {
    const size_t esz = a.dtype == 1 ? 2 : 4;
    const size_t V = 16 / esz;
    return (reinterpret_cast<uintptr_t>(a.experts) % 16 == 0) && (reinterpret_cast<uintptr_t>(a.xb) % 16 == 0) &&
           (a.stride % 16 == 0) && (a.D % V == 0) && (a.H % V == 0);
}

template <typename KernelT>
cudaError_t launch_persistent(KernelT kernel, const GemvArgs& a, cudaStream_t s) {
    int per_sm = 0;
    cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0);
    if (err != cudaSuccess) return err;
    kernel<<<a.grid * (per_sm > 0 ? per_sm : 1), kThreads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

// a.grid = SM count; the launch fills every SM to its occupancy limit.
// Slots per pass: 1 for a single token, else 4.
#define RBT_GEMV_DISPATCH(KERNEL)                                                                       \
    const bool v = vec_ok(a);                                                                           \
    const bool one = a.T == 1;                                                                          \
    if (a.dtype == 1) {                                                                                 \
        if (v) return one ? launch_persistent(KERNEL<uint16_t, true, 1>, a, s)                          \
                          : launch_persistent(KERNEL<uint16_t, true, 4>, a, s);                         \
        return one ? launch_persistent(KERNEL<uint16_t, false, 1>, a, s)                                \
                   : launch_persistent(KERNEL<uint16_t, false, 4>, a, s);                               \
    }                                                                                                   \
    if (v) return one ? launch_persistent(KERNEL<float, true, 1>, a, s)                                 \
                      : launch_persistent(KERNEL<float, true, 4>, a, s);                                \
    return one ? launch_persistent(KERNEL<float, false, 1>, a, s) : launch_persistent(KERNEL<float, false, 4>, a, s);

cudaError_t launch_gateup_gemv(const GemvArgs& args, cudaStream_t s) {
    GemvArgs a = args;
    a.expf_fma = host_expf_fma();
    RBT_GEMV_DISPATCH(gateup_gemv_kernel)
}

cudaError_t launch_down_gemv(const GemvArgs& a, cudaStream_t s) { RBT_GEMV_DISPATCH(down_gemv_kernel) }

// Loads every CUDA-core GEMV kernel now (see preload_kernels in kernels.h).
void preload_gemv_kernels() {
    cudaFuncAttributes f;
#define RBT_PRELOAD_GEMV(WT, V, M)                                          \
    (void)cudaFuncGetAttributes(&f, gateup_gemv_kernel<WT, V, M>);          \
    (void)cudaFuncGetAttributes(&f, down_gemv_kernel<WT, V, M>);
    RBT_PRELOAD_GEMV(uint16_t, true, 1)
    RBT_PRELOAD_GEMV(uint16_t, true, 4)
    RBT_PRELOAD_GEMV(uint16_t, false, 1)
    RBT_PRELOAD_GEMV(uint16_t, false, 4)
    RBT_PRELOAD_GEMV(float, true, 1)
    RBT_PRELOAD_GEMV(float, true, 4)
    RBT_PRELOAD_GEMV(float, false, 1)
    RBT_PRELOAD_GEMV(float, false, 4)
#undef RBT_PRELOAD_GEMV
    (void)cudaGetLastError();
}

}  // namespace rbt
