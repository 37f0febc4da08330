// gemv_stream.cu -- K3 (decode): expert weight streaming through shared memory
// with bulk asynchronous copies, for batches where each expert sees a few tokens.
// Replaces rabbit2.c:534-541 (three matvecs per chosen expert and the weighted
// combine) for bf16 models.
//
// Both kernels are persistent (one CTA per SM, 8 consumer warps + 1 producer
// warp).  The producer thread issues cp.async.bulk copies of whole weight rows
// (contiguous in the .rbt2 blob) into a ring of shared-memory stages guarded by
// mbarriers; the consumer warps compute dot products out of shared memory with
// fp32 FMA.  Work units are split into equal contiguous ranges per CTA.
//
//   gate/up: unit = 8 consecutive rows of w1 and the same 8 rows of w3 of one
//            expert (2 x 32 KB at D = 2048); consumer warp w owns row pair w and
//            writes h[p, r] = silu(w1_r . x_p) * (w3_r . x_p) for the expert's slots p.
//   down + combine: unit = 2 output rows d of w2 for every active expert (in
//            chunks of 8 experts per stage); per-slot results go to a small
//            shared buffer, then the unit's outputs are combined in selection
//            order, moe = sum_k w_k * y_k, and added to the residual: the y
//            scratch and the separate combine launch of the generic path vanish.
//
// Every mbarrier wait is bounded (2 s of %globaltimer); a timeout records a
// code in `status` and the kernel unwinds after draining its copies.
#include <cuda_bf16.h>

#include "common.cuh"
#include "exact_math.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rbt {
namespace {

using namespace tc;

constexpr int kWarps = 8;                   // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + producer warp
constexpr int kRows = 8;                    // gate/up row pairs per unit
constexpr int kStagesGU = 3;
constexpr int kDR = 2;                      // down rows per unit
constexpr int kExpChunk = 8;                // experts per down stage
constexpr int kStagesDN = 4;
constexpr int kMaxYbuf = 32768;             // bytes of per-slot down results per unit
constexpr uint64_t kWaitNs = 2000000000ull;

__device__ __forceinline__ void record_error(unsigned* status, unsigned code) { atomicCAS(status, 0u, code); }

__device__ __forceinline__ void unpack_bf16x8(const uint4& v, float* f) { WeightTraits<uint16_t>::unpack(v, f); }

// acc += w[8] . x[8] with x read from global (L1-resident activations)
__device__ __forceinline__ float dot8_global(const float* w, const float* x, float acc) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(x)), b = __ldg(reinterpret_cast<const float4*>(x + 4));
    acc = fmaf(w[0], a.x, acc);
    acc = fmaf(w[1], a.y, acc);
    acc = fmaf(w[2], a.z, acc);
    acc = fmaf(w[3], a.w, acc);
    acc = fmaf(w[4], b.x, acc);
    acc = fmaf(w[5], b.y, acc);
    acc = fmaf(w[6], b.z, acc);
    acc = fmaf(w[7], b.w, acc);
    return acc;
}

template <int MT, bool kXReg>
__global__ void __launch_bounds__(kThreads, 1) gateup_stream_kernel(StreamArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int D = a.D, H = a.H;
    const uint32_t row_bytes = (uint32_t)D * 2, half_bytes = kRows * row_bytes, stage_bytes = 2 * half_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStagesGU * stage_bytes);
    uint64_t* empty = full + kStagesGU;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesGU; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();  // routing and activations come from the preceding kernels
    const int units_per_e = H / kRows;
    const int n_units = *a.n_active * units_per_e;
    const int u0 = (int)((long)n_units * blockIdx.x / gridDim.x), u1 = (int)((long)n_units * (blockIdx.x + 1) / gridDim.x);
    if (warp == kWarps) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            for (int u = u0; u < u1; u++) {
                if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kWaitNs)) {
                    record_error(a.status, 0x401);
                    break;
                }
                const int ai = u / units_per_e, rg = u - ai * units_per_e;
                const uint8_t* w1 = a.experts + (size_t)a.active[ai] * a.stride + (size_t)rg * half_bytes;
                uint8_t* st = smem + stage * stage_bytes;
                mbar_arrive_expect_tx(&full[stage], stage_bytes);
                bulk_load(st, w1, half_bytes, &full[stage]);
                bulk_load(st + half_bytes, w1 + (size_t)H * row_bytes, half_bytes, &full[stage]);
                issued++;
                if (++stage == kStagesGU) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            // drain: the last min(issued, stages) copies have landed
            for (int i = 0; i < kStagesGU && i < issued; i++) {
                if (--stage < 0) {
                    stage = kStagesGU - 1;
                    phase ^= 1u;
                }
                if (!mbar_wait_bounded(&full[stage], phase, kWaitNs)) record_error(a.status, 0x402);
            }
        }
    } else {
        const int nv = D / 8;  // 16-byte vectors per row
        float xr[kXReg ? 64 : 1];
        if (kXReg) {  // one token (T == 1): its activations stay in registers
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = lane + 32 * j;
                if (v < nv) {
                    const float4 p = __ldg(reinterpret_cast<const float4*>(a.xb + v * 8));
                    const float4 q = __ldg(reinterpret_cast<const float4*>(a.xb + v * 8 + 4));
                    xr[8 * j] = p.x; xr[8 * j + 1] = p.y; xr[8 * j + 2] = p.z; xr[8 * j + 3] = p.w;
                    xr[8 * j + 4] = q.x; xr[8 * j + 5] = q.y; xr[8 * j + 6] = q.z; xr[8 * j + 7] = q.w;
                }
            }
        }
        int stage = 0;
        uint32_t phase = 0;
        for (int u = u0; u < u1; u++) {
            bool ok = mbar_wait_bounded(&full[stage], phase, kWaitNs);
            if (!__all_sync(FULL_MASK, ok)) {
                record_error(a.status, 0x403);
                break;
            }
            const int ai = u / units_per_e, rg = u - ai * units_per_e;
            const int e = a.active[ai];
            const int r = rg * kRows + warp;
            const int p0 = a.offsets[e], p1 = a.offsets[e + 1];
            const uint8_t* st = smem + stage * stage_bytes;
            const uint4* w1 = reinterpret_cast<const uint4*>(st + warp * row_bytes);
            const uint4* w3 = reinterpret_cast<const uint4*>(st + half_bytes + warp * row_bytes);
            for (int pb = p0; pb < p1; pb += MT) {
                const int m = min(MT, p1 - pb);
                const float* xrow[MT];
#pragma unroll
                for (int i = 0; i < MT; i++) xrow[i] = a.xb + (size_t)(a.perm[pb + (i < m ? i : 0)] / a.K) * D;
                float g[MT], up[MT];
#pragma unroll
                for (int i = 0; i < MT; i++) g[i] = up[i] = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int v = lane + 32 * j;
                    if (v >= nv) continue;
                    float f1[8], f3[8];
                    unpack_bf16x8(w1[v], f1);
                    unpack_bf16x8(w3[v], f3);
                    if (kXReg) {
#pragma unroll
                        for (int q = 0; q < 8; q++) {
                            g[0] = fmaf(f1[q], xr[8 * j + q], g[0]);
                            up[0] = fmaf(f3[q], xr[8 * j + q], up[0]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < MT; i++) {
                            if (i < m) {
                                g[i] = dot8_global(f1, xrow[i] + v * 8, g[i]);
                                up[i] = dot8_global(f3, xrow[i] + v * 8, up[i]);
                            }
                        }
                    }
                }
                for (int v = lane + 256; v < nv; v += 32) {  // rows longer than 2048 elements
                    float f1[8], f3[8];
                    unpack_bf16x8(w1[v], f1);
                    unpack_bf16x8(w3[v], f3);
#pragma unroll
                    for (int i = 0; i < MT; i++) {
                        if (i < m) {
                            g[i] = dot8_global(f1, xrow[i] + v * 8, g[i]);
                            up[i] = dot8_global(f3, xrow[i] + v * 8, up[i]);
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < MT; i++) {
                    if (i < m) {
                        const float gs = warp_sum(g[i]), us = warp_sum(up[i]);
                        if (lane == 0) a.h[(size_t)(pb + i) * H + r] = __fmul_rn(silu_ref(gs, a.expf_fma), us);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (++stage == kStagesGU) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
    __syncthreads();
    pdl_launch_dependents();
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1) down_combine_stream_kernel(StreamArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int D = a.D, H = a.H, K = a.K;
    const uint32_t rows_bytes = (uint32_t)kDR * H * 2;  // one expert's rows of a unit
    const uint32_t stage_bytes = kExpChunk * rows_bytes;
    float* ybuf = reinterpret_cast<float*>(smem + kStagesDN * stage_bytes);  // [S][kDR]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStagesDN * stage_bytes + kMaxYbuf);
    uint64_t* empty = full + kStagesDN;
    __shared__ int s_err;  // any consumer warp timed out: all consumer warps unwind together
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_err = 0;
        for (int s = 0; s < kStagesDN; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();
    const int na = *a.n_active;
    const int nch = (na + kExpChunk - 1) / kExpChunk;
    const int n_units = D / kDR;
    const int u0 = (int)((long)n_units * blockIdx.x / gridDim.x), u1 = (int)((long)n_units * (blockIdx.x + 1) / gridDim.x);
    if (warp == kWarps) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            for (int u = u0; ok && u < u1; u++) {
                for (int ch = 0; ch < nch; ch++) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kWaitNs)) {
                        record_error(a.status, 0x501);
                        ok = false;
                        break;
                    }
                    const int ne = min(kExpChunk, na - ch * kExpChunk);
                    uint8_t* st = smem + stage * stage_bytes;
                    mbar_arrive_expect_tx(&full[stage], ne * rows_bytes);
                    for (int j = 0; j < ne; j++) {
                        const int e = a.active[ch * kExpChunk + j];
                        const uint8_t* src = a.experts + (size_t)e * a.stride + (size_t)2 * H * D * 2 +
                                             (size_t)u * kDR * H * 2;
                        bulk_load(st + j * rows_bytes, src, rows_bytes, &full[stage]);
                    }
                    issued++;
                    if (++stage == kStagesDN) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            for (int i = 0; i < kStagesDN && i < issued; i++) {
                if (--stage < 0) {
                    stage = kStagesDN - 1;
                    phase ^= 1u;
                }
                if (!mbar_wait_bounded(&full[stage], phase, kWaitNs)) record_error(a.status, 0x502);
            }
        }
    } else {
        const int nv = H / 8;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int u = u0; ok && u < u1; u++) {
            const int d0 = u * kDR;
            for (int ch = 0; ch < nch; ch++) {
                const bool got = mbar_wait_bounded(&full[stage], phase, kWaitNs);
                if (!__all_sync(FULL_MASK, got)) {
                    record_error(a.status, 0x503);
                    if (lane == 0) s_err = 1;
                    ok = false;
                    break;
                }
                const int ne = min(kExpChunk, na - ch * kExpChunk);
                const uint8_t* st = smem + stage * stage_bytes;
                for (int task = warp; task < ne * kDR; task += kWarps) {
                    const int j = task / kDR, dr = task - j * kDR;
                    const int e = a.active[ch * kExpChunk + j];
                    const uint4* w = reinterpret_cast<const uint4*>(st + j * rows_bytes + dr * H * 2);
                    const int p0 = a.offsets[e], p1 = a.offsets[e + 1];
                    for (int pb = p0; pb < p1; pb += MT) {
                        const int m = min(MT, p1 - pb);
                        float acc[MT];
#pragma unroll
                        for (int i = 0; i < MT; i++) acc[i] = 0.0f;
                        for (int v = lane; v < nv; v += 32) {
                            float f[8];
                            unpack_bf16x8(w[v], f);
#pragma unroll
                            for (int i = 0; i < MT; i++)
                                if (i < m) acc[i] = dot8_global(f, a.h + (size_t)(pb + i) * H + v * 8, acc[i]);
                        }
#pragma unroll
                        for (int i = 0; i < MT; i++) {
                            if (i < m) {
                                const float s = warp_sum(acc[i]);
                                if (lane == 0) ybuf[(pb + i) * kDR + dr] = s;
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[stage]);
                if (++stage == kStagesDN) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            named_sync(1, kWarps * 32);
            ok = ok && !s_err;  // uniform across the consumer warps from here
            if (ok) {
                // combine in selection order, then the residual (rabbit2.c:539-542)
                for (int i = threadIdx.x; i < a.T * kDR; i += kWarps * 32) {
                    const int t = i / kDR, dr = i - t * kDR;
                    float mo = 0.0f;
                    for (int k = 0; k < K; k++) {
                        const int s = t * K + k, sp = a.slot_pos[s];
                        if (sp >= 0) mo = __fadd_rn(mo, __fmul_rn(a.wt[s], ybuf[sp * kDR + dr]));
                    }
                    const size_t o = (size_t)t * D + d0 + dr;
                    a.out[o] = a.resid ? __fadd_rn(a.resid[o], mo) : mo;
                }
            }
            named_sync(1, kWarps * 32);
        }
    }
    __syncthreads();
    pdl_launch_dependents();
}

template <typename KernelT>
cudaError_t launch_pdl(KernelT kernel, int grid, size_t smem, const StreamArgs& a, cudaStream_t s) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace

// Shapes the streaming kernels take: bf16 rows that fit the stages, aligned blobs.
bool stream_supported(const StreamArgs& a, int dtype) {
    const int S = a.T * a.K;
    return dtype == 1 && a.D % 8 == 0 && a.H % 8 == 0 && a.H % kRows == 0 && a.D % kDR == 0 &&
           2 * kRows * a.D * 2 <= 65536 && kExpChunk * kDR * a.H * 2 <= 65536 &&
           (size_t)S * kDR * 4 <= (size_t)kMaxYbuf && a.stride % 16 == 0 &&
           (reinterpret_cast<uintptr_t>(a.experts) % 16) == 0 && (reinterpret_cast<uintptr_t>(a.xb) % 16) == 0;
}

cudaError_t launch_gateup_stream(const StreamArgs& args, int grid, cudaStream_t s) {
    StreamArgs a = args;
    a.expf_fma = host_expf_fma();
    const size_t smem = (size_t)kStagesGU * 2 * kRows * a.D * 2 + 2 * kStagesGU * 8;
    if (a.T == 1 && a.D <= 2048 && a.D % 256 == 0)
        return launch_pdl(gateup_stream_kernel<1, true>, grid, smem, a, s);
    return launch_pdl(gateup_stream_kernel<4, false>, grid, smem, a, s);
}

cudaError_t launch_down_combine_stream(const StreamArgs& a, int grid, cudaStream_t s) {
    const size_t smem = (size_t)kStagesDN * kExpChunk * kDR * a.H * 2 + kMaxYbuf + 2 * kStagesDN * 8;
    if (a.T == 1) return launch_pdl(down_combine_stream_kernel<1>, grid, smem, a, s);
    return launch_pdl(down_combine_stream_kernel<4>, grid, smem, a, s);
}

// Loads the weight-streaming kernels now (see preload_kernels in kernels.h).
void preload_stream_kernels() {
    cudaFuncAttributes f;
    (void)cudaFuncGetAttributes(&f, gateup_stream_kernel<1, true>);
    (void)cudaFuncGetAttributes(&f, gateup_stream_kernel<4, false>);
    (void)cudaFuncGetAttributes(&f, down_combine_stream_kernel<1>);
    (void)cudaFuncGetAttributes(&f, down_combine_stream_kernel<4>);
    (void)cudaGetLastError();
}

}  // namespace rbt
