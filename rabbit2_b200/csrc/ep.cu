// ep.cu -- expert parallelism across the GPUs of one node over NVLink peer
// memory: the dispatch plan, the push of each token's row to the GPUs that own
// its experts, the return of the partial outputs, and the fixed-order combine.
//
// GPU g owns experts [g*epr, (g+1)*epr).  A token goes to every GPU that owns at
// least one of its top-k experts, once per GPU (not once per expert), with its k
// expert ids made local to that GPU (-1 for the others) and its k combine weights;
// a token whose experts are all local never leaves its GPU.  The rows are stored
// straight into the owner's receive segment (plain stores to peer memory over
// NVLink, no TMA, no multicast), and a flag written with release semantics at
// system scope tells the owner they are complete.  Each owner returns one partial
// row per row it received (the sum over its own slots in selection order) into the
// sender's return segment, flagged the same way.  The sender adds the partials in
// ascending GPU order, then the residual: x + ((p_0 + p_1) + ...), deterministic
// for a given GPU count.  Flags carry epochs (one per layer call, counted on the
// device), so the whole layer can be captured in a CUDA graph; every wait is
// bounded by %globaltimer and leaves a status code (0x701 receive, 0x702 return,
// 0x703 a peer reported its own failure) instead of hanging.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace {

using rbt::FULL_MASK;
using rbt::lanemask_lt;
using rbt::EpArgs;
using rbt::tc::globaltimer_ns;

constexpr int kPlanThreads = 1024;
constexpr int kThreads = 256;
constexpr int kReturnRows = 8;  // received rows per CTA of the return kernel
constexpr unsigned long long kErrorBit = 1ull << 62;  // set in a flag by a GPU whose own waits failed
constexpr unsigned long long kEpochMask = kErrorBit - 1;

// One CTA per destination GPU g: pos[t, g] = rank of token t among the tokens
// sent to g (ascending t), or -1; counts[g] = tokens sent to g.  With a fixed
// capacity C >= T instead: pos[t, g] = t (or -1) and counts[g] = C, so every
// segment has the same, host-known size and no count needs to reach the host.
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int32_t* idx, int T, int K, int R, int epr,
                                                               int capacity, int32_t* pos, int32_t* counts) {
    __shared__ int s_warp[kPlanThreads / 32];
    const int g = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int base = 0;
    for (int c0 = 0; c0 < T; c0 += kPlanThreads) {
        const int t = c0 + tid;
        int flag = 0;
        if (t < T)
            for (int k = 0; k < K; k++) {
                const int e = idx[(size_t)t * K + k];
                flag |= e >= 0 && e / epr == g;
            }
        const unsigned bal = __ballot_sync(FULL_MASK, flag);
        if (lane == 0) s_warp[warp] = __popc(bal);
        __syncthreads();
        int pre = 0, tot = 0;
        for (int w = 0; w < kPlanThreads / 32; w++) {
            pre += w < warp ? s_warp[w] : 0;
            tot += s_warp[w];
        }
        if (t < T)
            pos[(size_t)t * R + g] = !flag ? -1 : capacity > 0 ? t : base + pre + __popc(bal & lanemask_lt());
        base += tot;
        __syncthreads();
    }
    if (tid == 0) counts[g] = capacity > 0 ? capacity : base;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void record(unsigned* status, unsigned code) { atomicCAS(status, 0u, code); }

// Wait (bounded) until the epoch in *p reaches e: 0 done, 1 timed out, 2 the
// writer reported a failure of its own.
__device__ int ep_wait(const unsigned long long* p, unsigned long long e, unsigned long long limit_ns) {
    unsigned long long v = ld_acquire_sys(p);
    if ((v & kEpochMask) < e) {
        const uint64_t t0 = globaltimer_ns();
        while (((v = ld_acquire_sys(p)) & kEpochMask) < e)
            if (globaltimer_ns() - t0 > limit_ns) return 1;
    }
    return (v & kErrorBit) ? 2 : 0;
}

// One CTA per local token (one CTA when there are none): its row, local ids and
// weights into every owning GPU's segment for this GPU, at its position there.
// The last CTA to finish writes the row counts and then the flags.
__global__ void __launch_bounds__(kThreads) ep_dispatch_kernel(EpArgs a, const float* xb, const int32_t* idx,
                                                                const float* wt, const int32_t* pos,
                                                                const int32_t* counts, int T) {
    const unsigned long long e = *a.epoch + 1;
    const int t = blockIdx.x, tid = threadIdx.x, D4 = a.D / 4;
    if (t < T) {
        for (int g = 0; g < a.R; g++) {
            const int p = pos[(size_t)t * a.R + g];
            if (p < 0) continue;
            const size_t row = (size_t)a.rank * a.cap + p;
            const float4* src = reinterpret_cast<const float4*>(xb + (size_t)t * a.D);
            float4* dst = reinterpret_cast<float4*>(a.peers.recv_rows[g] + row * a.D);
            for (int i = tid; i < D4; i += kThreads) dst[i] = src[i];
            for (int k = tid; k < a.K; k += kThreads) {
                const int ex = idx[(size_t)t * a.K + k];
                a.peers.recv_idx[g][row * a.K + k] = (ex >= 0 && ex / a.epr == g) ? ex - g * a.epr : -1;
                a.peers.recv_wt[g][row * a.K + k] = wt[(size_t)t * a.K + k];
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        if (atomicAdd(&a.done[0], 1u) == gridDim.x - 1) {
            __threadfence_system();
            for (int g = 0; g < a.R; g++) a.peers.recv_count[g][a.rank] = T > 0 ? counts[g] : 0;
            __threadfence_system();
            const unsigned long long f = e | (*(volatile unsigned*)a.status ? kErrorBit : 0ull);
            for (int g = 0; g < a.R; g++) st_release_sys(a.peers.flag_dispatch[g] + a.rank, f);
            a.done[0] = 0;
        }
    }
}

// One CTA per source GPU s: wait for its flag, then mark the rows of its segment
// beyond its count as holding no slot.  A source that never signals (or reports
// a failure) contributes no rows.
__global__ void __launch_bounds__(kThreads) ep_receive_kernel(EpArgs a) {
    __shared__ int s_n;
    const unsigned long long e = *a.epoch + 1;
    const int s = blockIdx.x;
    if (threadIdx.x == 0) {
        const int w = ep_wait(a.peers.flag_dispatch[a.rank] + s, e, a.timeout_ns);
        if (w) record(a.status, w == 1 ? 0x701u : 0x703u);
        int n = w ? 0 : *(volatile int32_t*)(a.peers.recv_count[a.rank] + s);
        n = n < 0 ? 0 : (n > a.cap ? a.cap : n);
        a.peers.recv_count[a.rank][s] = n;  // the count the return kernel uses
        s_n = n;
    }
    __syncthreads();
    int32_t* ids = a.peers.recv_idx[a.rank] + (size_t)s * a.cap * a.K;
    for (long i = (long)s_n * a.K + threadIdx.x; i < (long)a.cap * a.K; i += kThreads) ids[i] = -1;
}

// CTA (s, c): received rows [c*kReturnRows, ...) of source s's segment; each row's
// weighted sum over its local slots in selection order (rabbit2.c:539-540) goes
// straight into source s's return segment for this GPU.  The last CTA of a
// segment raises that source's flag.
__global__ void __launch_bounds__(kThreads) ep_return_kernel(EpArgs a, const float* y, const int32_t* slot_pos,
                                                              const float* rows, int chunks) {
    const unsigned long long e = *a.epoch + 1;
    const int s = blockIdx.x / chunks, c = blockIdx.x - s * chunks, tid = threadIdx.x, D4 = a.D / 4;
    const int n = a.peers.recv_count[a.rank][s];
    const float* wts = a.peers.recv_wt[a.rank];
    for (int r = c * kReturnRows; r < n && r < (c + 1) * kReturnRows; r++) {
        const size_t row = (size_t)s * a.cap + r;
        float4* dst = reinterpret_cast<float4*>(a.peers.back_rows[s] + ((size_t)a.rank * a.cap + r) * a.D);
        if (rows) {  // combined already (the streaming GEMV's down kernel)
            const float4* src = reinterpret_cast<const float4*>(rows + row * a.D);
            for (int d4 = tid; d4 < D4; d4 += kThreads) dst[d4] = src[d4];
            continue;
        }
        for (int d4 = tid; d4 < D4; d4 += kThreads) {
            float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k = 0; k < a.K; k++) {
                const int sp = slot_pos[row * a.K + k];
                if (sp < 0) continue;
                const float w = wts[row * a.K + k];
                const float4 v = reinterpret_cast<const float4*>(y + (size_t)sp * a.D)[d4];
                m.x = __fadd_rn(m.x, __fmul_rn(w, v.x));
                m.y = __fadd_rn(m.y, __fmul_rn(w, v.y));
                m.z = __fadd_rn(m.z, __fmul_rn(w, v.z));
                m.w = __fadd_rn(m.w, __fmul_rn(w, v.w));
            }
            dst[d4] = m;
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        if (atomicAdd(&a.done[2 + s], 1u) == (unsigned)chunks - 1) {
            __threadfence_system();
            st_release_sys(a.peers.flag_return[s] + a.rank, e | (*(volatile unsigned*)a.status ? kErrorBit : 0ull));
            a.done[2 + s] = 0;
        }
    }
}

// Wait for every GPU's return flag, then x[t] += ((p_0 + p_1) + ...) over the GPUs
// the token went to, in ascending order; the last CTA advances the epoch.
__global__ void __launch_bounds__(kThreads) ep_combine_kernel(EpArgs a, float* x, const int32_t* pos, int T) {
    __shared__ int s_bad;
    const unsigned long long e = *a.epoch + 1;
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();
    if (threadIdx.x < a.R) {
        const int w = ep_wait(a.peers.flag_return[a.rank] + threadIdx.x, e, a.timeout_ns);
        if (w) {
            record(a.status, w == 1 ? 0x702u : 0x703u);
            atomicOr(&s_bad, 1);
        }
    }
    __syncthreads();
    const float* back = a.peers.back_rows[a.rank];
    const int D4 = a.D / 4;
    if (!s_bad) {
        const long total = (long)T * D4;
        for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total; i += (long)gridDim.x * kThreads) {
            const int t = (int)(i / D4), d4 = (int)(i - (long)t * D4);
            float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int g = 0; g < a.R; g++) {
                const int p = pos[(size_t)t * a.R + g];
                if (p < 0) continue;
                const float4 v = reinterpret_cast<const float4*>(back + ((size_t)g * a.cap + p) * a.D)[d4];
                m.x = __fadd_rn(m.x, v.x);
                m.y = __fadd_rn(m.y, v.y);
                m.z = __fadd_rn(m.z, v.z);
                m.w = __fadd_rn(m.w, v.w);
            }
            float4* xr = reinterpret_cast<float4*>(x + (size_t)t * a.D) + d4;
            const float4 r = *xr;
            *xr = make_float4(__fadd_rn(r.x, m.x), __fadd_rn(r.y, m.y), __fadd_rn(r.z, m.z), __fadd_rn(r.w, m.w));
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(&a.done[1], 1u) == gridDim.x - 1) {
        *a.epoch = e;
        a.done[1] = 0;
    }
}

}  // namespace

namespace rbt {

cudaError_t launch_ep_plan(const int32_t* idx, int T, int K, int R, int epr, int32_t* pos, int32_t* counts,
                           cudaStream_t s) {
    ep_plan_kernel<<<R, kPlanThreads, 0, s>>>(idx, T, K, R, epr, 0, pos, counts);
    return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const EpArgs& a, const float* xb, const int32_t* idx, const float* wt,
                               const int32_t* pos, const int32_t* counts, int T, cudaStream_t s) {
    ep_dispatch_kernel<<<T > 0 ? T : 1, kThreads, 0, s>>>(a, xb, idx, wt, pos, counts, T);
    return cudaGetLastError();
}

cudaError_t launch_ep_receive(const EpArgs& a, cudaStream_t s) {
    ep_receive_kernel<<<a.R, kThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_return(const EpArgs& a, const float* y, const int32_t* slot_pos, const float* rows,
                             cudaStream_t s) {
    const int chunks = (a.cap + kReturnRows - 1) / kReturnRows;
    ep_return_kernel<<<a.R * chunks, kThreads, 0, s>>>(a, y, slot_pos, rows, chunks);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const EpArgs& a, float* x, const int32_t* pos, int T, cudaStream_t s) {
    const long work = (long)T * (a.D / 4);
    long blocks = (work + kThreads - 1) / kThreads;
    if (blocks < 1) blocks = 1;
    if (blocks > 148L * 8) blocks = 148L * 8;
    ep_combine_kernel<<<(int)blocks, kThreads, 0, s>>>(a, x, pos, T);
    return cudaGetLastError();
}

// Loads the expert-parallel kernels now (see preload_kernels in kernels.h).
void preload_ep_kernels() {
    cudaFuncAttributes f;
    (void)cudaFuncGetAttributes(&f, ep_plan_kernel);
    (void)cudaFuncGetAttributes(&f, ep_dispatch_kernel);
    (void)cudaFuncGetAttributes(&f, ep_receive_kernel);
    (void)cudaFuncGetAttributes(&f, ep_return_kernel);
    (void)cudaFuncGetAttributes(&f, ep_combine_kernel);
    (void)cudaGetLastError();
}

}  // namespace rbt

