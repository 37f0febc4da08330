// ep.cu -- expert parallelism across the GPUs of one node: the dispatch plan,
// the packing of token rows per destination GPU, and the fixed-order combine of
// the partial MoE outputs that come back.  The all-to-all exchanges themselves
// are NCCL collectives issued by the host (rabbit2_b200/ep.py); these kernels
// prepare and consume their buffers.
//
// GPU g owns experts [g*Epr, (g+1)*Epr).  A token goes to every GPU that owns
// at least one of its top-k experts, once per GPU (not once per expert), with
// its k expert ids made local to that GPU (-1 for the others) and its k combine
// weights.  Each GPU returns one partial row per token it received: the sum
// over its own slots in selection order.  The sender adds the partials in
// ascending GPU order, then the residual: moe = ((p_0 + p_1) + ...) and
// x + moe, deterministic for a given GPU count.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/rbt_moe.h"
#include "common.cuh"
#include "kernels.h"

namespace rbt {
void set_last_error(const char* msg);
}

namespace {

using rbt::FULL_MASK;
using rbt::lanemask_lt;

constexpr int kPlanThreads = 1024;
constexpr int kMaxRanks = 64;

int fail(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
int fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    fprintf(stderr, "rbt_ep: %s\n", buf);
    rbt::set_last_error(buf);
    return 0;
}

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

// One CTA per token: its row and routing go to every GPU it has a slot on, at
// (first row of that GPU's segment) + pos.
__global__ void __launch_bounds__(256) ep_pack_kernel(const float* xb, const int32_t* idx, const float* wt, int T,
                                                      int D, int K, int R, int epr, const int32_t* pos,
                                                      const int32_t* counts, float* send_rows, int32_t* send_idx,
                                                      float* send_wt) {
    __shared__ int s_off[kMaxRanks];
    const int t = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) {
        int run = 0;
        for (int g = 0; g < R; g++) {
            s_off[g] = run;
            run += counts[g];
        }
    }
    __syncthreads();
    for (int g = 0; g < R; g++) {
        const int p = pos[(size_t)t * R + g];
        if (p < 0) continue;
        const size_t row = (size_t)s_off[g] + p;
        const float4* src = reinterpret_cast<const float4*>(xb + (size_t)t * D);
        float4* dst = reinterpret_cast<float4*>(send_rows + row * D);
        for (int i = tid; i < D / 4; i += blockDim.x) dst[i] = src[i];
        for (int k = tid; k < K; k += blockDim.x) {
            const int e = idx[(size_t)t * K + k];
            send_idx[row * K + k] = (e >= 0 && e / epr == g) ? e - g * epr : -1;
            send_wt[row * K + k] = wt[(size_t)t * K + k];
        }
    }
}

// out[t] = (x[t] +) sum over GPUs g in ascending order of back[off_g + pos[t, g]].
__global__ void __launch_bounds__(256) ep_combine_kernel(const float* x, int T, int D, int R, const int32_t* pos,
                                                         const int32_t* counts, const float* back, float* out) {
    __shared__ int s_off[kMaxRanks];
    if (threadIdx.x == 0) {
        int run = 0;
        for (int g = 0; g < R; g++) {
            s_off[g] = run;
            run += counts[g];
        }
    }
    __syncthreads();
    const int D4 = D / 4;
    const long total = (long)T * D4;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int t = (int)(i / D4), d4 = (int)(i - (long)t * D4);
        float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int g = 0; g < R; g++) {
            const int p = pos[(size_t)t * R + g];
            if (p < 0) continue;
            const float4 v = reinterpret_cast<const float4*>(back + ((size_t)s_off[g] + p) * D)[d4];
            m.x = __fadd_rn(m.x, v.x);
            m.y = __fadd_rn(m.y, v.y);
            m.z = __fadd_rn(m.z, v.z);
            m.w = __fadd_rn(m.w, v.w);
        }
        if (x) {
            const float4 r = reinterpret_cast<const float4*>(x + (size_t)t * D)[d4];
            m = make_float4(__fadd_rn(r.x, m.x), __fadd_rn(r.y, m.y), __fadd_rn(r.z, m.z), __fadd_rn(r.w, m.w));
        }
        reinterpret_cast<float4*>(out + (size_t)t * D)[d4] = m;
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int rbt_ep_plan(const int32_t* d_idx, int n_tokens, int top_k, int n_ranks, int experts_per_rank, int capacity,
                int32_t* d_pos, int32_t* d_counts, void* stream) {
    if (n_ranks <= 0 || n_ranks > kMaxRanks || experts_per_rank <= 0 || top_k <= 0 || n_tokens < 0 ||
        (capacity > 0 && capacity < n_tokens))
        return fail("rbt_ep_plan: invalid sizes (n_ranks %d, experts_per_rank %d, top_k %d, n_tokens %d)", n_ranks,
                    experts_per_rank, top_k, n_tokens);
    if (!d_pos || !d_counts || (n_tokens > 0 && !d_idx)) return fail("rbt_ep_plan: null argument");
    ep_plan_kernel<<<n_ranks, kPlanThreads, 0, (cudaStream_t)stream>>>(d_idx, n_tokens, top_k, n_ranks,
                                                                       experts_per_rank, capacity, d_pos, d_counts);
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? 1 : fail("rbt_ep_plan: launch failed: %s", cudaGetErrorString(err));
}

int rbt_ep_pack(const float* d_xb, const int32_t* d_idx, const float* d_wt, int n_tokens, int dim, int top_k,
                int n_ranks, int experts_per_rank, const int32_t* d_pos, const int32_t* d_counts, float* d_send_rows,
                int32_t* d_send_idx, float* d_send_wt, void* stream) {
    if (n_tokens < 0 || dim <= 0 || dim % 4 || top_k <= 0 || n_ranks <= 0 || n_ranks > kMaxRanks ||
        experts_per_rank <= 0)
        return fail("rbt_ep_pack: invalid sizes");
    if (n_tokens == 0) return 1;
    if (!d_xb || !d_idx || !d_wt || !d_pos || !d_counts || !d_send_rows || !d_send_idx || !d_send_wt)
        return fail("rbt_ep_pack: null argument");
    if (!aligned16(d_xb) || !aligned16(d_send_rows)) return fail("rbt_ep_pack: rows must be 16-byte aligned");
    ep_pack_kernel<<<n_tokens, 256, 0, (cudaStream_t)stream>>>(d_xb, d_idx, d_wt, n_tokens, dim, top_k, n_ranks,
                                                               experts_per_rank, d_pos, d_counts, d_send_rows,
                                                               d_send_idx, d_send_wt);
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? 1 : fail("rbt_ep_pack: launch failed: %s", cudaGetErrorString(err));
}

int rbt_ep_combine(const float* d_x, int n_tokens, int dim, int n_ranks, const int32_t* d_pos,
                   const int32_t* d_counts, const float* d_back_rows, float* d_out, void* stream) {
    if (n_tokens < 0 || dim <= 0 || dim % 4 || n_ranks <= 0 || n_ranks > kMaxRanks)
        return fail("rbt_ep_combine: invalid sizes");
    if (n_tokens == 0) return 1;
    if (!d_pos || !d_counts || !d_out) return fail("rbt_ep_combine: null argument");
    if ((d_x && !aligned16(d_x)) || !aligned16(d_out) || (d_back_rows && !aligned16(d_back_rows)))
        return fail("rbt_ep_combine: rows must be 16-byte aligned");
    const long work = (long)n_tokens * (dim / 4);
    const int grid = (int)((work + 255) / 256 < 148L * 16 ? (work + 255) / 256 : 148L * 16);
    ep_combine_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(d_x, n_tokens, dim, n_ranks, d_pos, d_counts,
                                                              d_back_rows, d_out);
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? 1 : fail("rbt_ep_combine: launch failed: %s", cudaGetErrorString(err));
}

}  // extern "C"
