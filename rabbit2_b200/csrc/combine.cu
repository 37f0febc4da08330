// combine.cu -- K5: weighted combine of the k expert outputs of each token, plus
// the residual add of the block form (rabbit2.c:530-542), and the ffn RMSNorm
// that feeds the block form (rabbit2.c:512, rmsnorm at :392-397).
//
// Combine order follows the reference: moe = 0; moe += w_k * y_k for k in
// selection order (product rounded, then added); x += moe.  Each output element
// gathers its k inputs by slot position, so the result is deterministic (no
// floating-point atomics).
#include "common.cuh"
#include "exact_math.cuh"
#include "kernels.h"

namespace rbt {
namespace {

constexpr int kThreads = 256;
// the squares of one row in shared memory: dim <= 49152
constexpr size_t kRmsnormMaxSmem = 192 * 1024;

__global__ void __launch_bounds__(kThreads) combine_vec4_kernel(CombineArgs a) {
    const int D4 = a.D / 4;
    const long total = (long)a.T * D4;
    for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total; i += (long)gridDim.x * kThreads) {
        const int t = (int)(i / D4), d = (int)(i - (long)t * D4) * 4;
        float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < a.K; k++) {
            const int s = t * a.K + k, sp = a.slot_pos[s];
            if (sp < 0) continue;  // a slot another GPU computes (expert parallelism)
            const float w = a.wt[s];
            const float4 y = *reinterpret_cast<const float4*>(a.y + (size_t)sp * a.D + d);
            m.x = __fadd_rn(m.x, __fmul_rn(w, y.x));
            m.y = __fadd_rn(m.y, __fmul_rn(w, y.y));
            m.z = __fadd_rn(m.z, __fmul_rn(w, y.z));
            m.w = __fadd_rn(m.w, __fmul_rn(w, y.w));
        }
        if (a.resid) {
            const float4 x = *reinterpret_cast<const float4*>(a.resid + (size_t)t * a.D + d);
            m = make_float4(__fadd_rn(x.x, m.x), __fadd_rn(x.y, m.y), __fadd_rn(x.z, m.z), __fadd_rn(x.w, m.w));
        }
        *reinterpret_cast<float4*>(a.out + (size_t)t * a.D + d) = m;
    }
}

__global__ void __launch_bounds__(kThreads) combine_scalar_kernel(CombineArgs a) {
    const long total = (long)a.T * a.D;
    for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total; i += (long)gridDim.x * kThreads) {
        const int t = (int)(i / a.D), d = (int)(i - (long)t * a.D);
        float m = 0.0f;
        for (int k = 0; k < a.K; k++) {
            const int s = t * a.K + k, sp = a.slot_pos[s];
            if (sp >= 0) m = __fadd_rn(m, __fmul_rn(a.wt[s], a.y[(size_t)sp * a.D + d]));
        }
        if (a.resid) m = __fadd_rn(a.resid[(size_t)t * a.D + d], m);
        a.out[(size_t)t * a.D + d] = m;
    }
}

// out[t] = (x[t] * inv) * w, inv = 1 / sqrtf(mean(x^2) + eps); one CTA per token
// (rabbit2.c:392-397).  The sum of squares is the reference's sequential f32 sum,
// reproduced exactly by block_seq_sum over the squares staged in shared memory.
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const float* x, const float* w, float* out, int D,
                                                           float eps) {
    extern __shared__ float s_sq[];
    __shared__ SeqSumSmem s_seq;
    const float* xr = x + (size_t)blockIdx.x * D;
    for (int i = threadIdx.x; i < D; i += kThreads) s_sq[i] = __fmul_rn(xr[i], xr[i]);
    __syncthreads();
    const float ss = block_seq_sum<kThreads>(s_sq, D, s_seq);
    const float inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
    float* o = out + (size_t)blockIdx.x * D;
    for (int i = threadIdx.x; i < D; i += kThreads) o[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// The same rmsnorm for many tokens: one CTA per 32 rows, lane r of warp 0 running row r's
// sum of squares as the reference's plain sequential chain (products and sums
// separately rounded, in index order: the same bits as block_seq_sum), then the
// CTA's eight warps write the 32 normalised rows with coalesced stores.  At thousands of
// tokens the per-row parallel reproduction costs more issue slots than the chains'
// latency: one dependent add per element, 32 rows per warp, every SM streaming.
// The rows come through a shared-memory ring of kRowsStages chunks (32 rows x
// kRowsChunk floats), copied with coalesced cp.async (the warp moves one row's
// chunk per instruction), so that several chunks are in flight while the chains
// run; each row's chunk sits kRowsPitch bytes apart (16 bytes of padding keep the
// lanes' float4 reads on distinct banks).
constexpr int kRowsPerWarp = 32;
constexpr int kRowsMinTokens = 1024;
constexpr int kRowsChunk = 128;                      // floats per row per stage
constexpr int kRowsPitch = kRowsChunk * 4 + 16;      // bytes per row in a stage
constexpr int kRowsStages = 8;
constexpr int kRowsSmem = kRowsStages * kRowsPerWarp * kRowsPitch;
constexpr int kRowsWarps = 8;  // warp 0 runs the chains; all eight write the rows
constexpr int kRowsThreads = kRowsWarps * 32;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kRowsThreads) rmsnorm_rows_kernel(const float* x, const float* w, float* out, int T,
                                                                    int D, float eps) {
    extern __shared__ __align__(16) uint8_t ring[];
    __shared__ float s_inv[kRowsPerWarp];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, r0 = blockIdx.x * kRowsPerWarp;
    const int nrows = min(kRowsPerWarp, T - r0);
    const int n_chunks = D / kRowsChunk;
    // stage c % kRowsStages <- chunk c of every row (lane l copies bytes [16 l, 16 l + 16))
    auto load = [&](int c) {
        uint8_t* st = ring + (c % kRowsStages) * (kRowsPerWarp * kRowsPitch);
        if (c < n_chunks)
            for (int r = 0; r < nrows; r++)
                cp_async16(st + r * kRowsPitch + lane * 16, x + (size_t)(r0 + r) * D + c * kRowsChunk + lane * 4);
        cp_async_commit();  // (an empty group past the last chunk keeps the wait count uniform)
    };
    if (warp == 0) {  // the 32 chains
#pragma unroll 1
        for (int c = 0; c < kRowsStages - 1; c++) load(c);
        float ss = 0.0f;
#pragma unroll 1
        for (int c = 0; c < n_chunks; c++) {
            cp_async_wait<kRowsStages - 2>();  // chunk c has landed (this lane's copies)
            __syncwarp();                       // ... and every lane's
            if (lane < nrows) {
                const float4* v = reinterpret_cast<const float4*>(
                    ring + (c % kRowsStages) * (kRowsPerWarp * kRowsPitch) + lane * kRowsPitch);
#pragma unroll 8
                for (int i = 0; i < kRowsChunk / 4; i++) {
                    const float4 q = v[i];
                    ss = __fadd_rn(ss, __fmul_rn(q.x, q.x));
                    ss = __fadd_rn(ss, __fmul_rn(q.y, q.y));
                    ss = __fadd_rn(ss, __fmul_rn(q.z, q.z));
                    ss = __fadd_rn(ss, __fmul_rn(q.w, q.w));
                }
            }
            __syncwarp();  // every lane is done with the stage that chunk c + kRowsStages - 1 reuses
            load(c + kRowsStages - 1);
        }
        cp_async_wait<0>();
        s_inv[lane] = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
    }
    __syncthreads();
    // the normalised rows, every warp of the CTA: row r by warp r % kRowsWarps
    const int n4 = D / 4;
    for (int r = warp; r < nrows; r += kRowsWarps) {
        const float inv = s_inv[r];
        const float4* xr = reinterpret_cast<const float4*>(x + (size_t)(r0 + r) * D);
        float4* o = reinterpret_cast<float4*>(out + (size_t)(r0 + r) * D);
#pragma unroll 4
        for (int i4 = lane; i4 < n4; i4 += 32) {
            const float4 v = __ldg(xr + i4), ww = __ldg(reinterpret_cast<const float4*>(w) + i4);
            o[i4] = make_float4(__fmul_rn(__fmul_rn(v.x, inv), ww.x), __fmul_rn(__fmul_rn(v.y, inv), ww.y),
                                __fmul_rn(__fmul_rn(v.z, inv), ww.z), __fmul_rn(__fmul_rn(v.w, inv), ww.w));
        }
    }
}

}  // namespace

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t s) {
    if (a.T <= 0) return cudaSuccess;
    const bool vec = (a.D % 4 == 0) && (reinterpret_cast<uintptr_t>(a.out) % 16 == 0) &&
                     (!a.resid || reinterpret_cast<uintptr_t>(a.resid) % 16 == 0);
    const long work = vec ? (long)a.T * (a.D / 4) : (long)a.T * a.D;
    const long blocks = (work + kThreads - 1) / kThreads;
    const int grid = (int)(blocks < 148L * 16 ? blocks : 148L * 16);
    if (vec) combine_vec4_kernel<<<grid, kThreads, 0, s>>>(a);
    else combine_scalar_kernel<<<grid, kThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int T, int D, float eps, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    if (T >= kRowsMinTokens && D % kRowsChunk == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) {
        cudaError_t err = cudaFuncSetAttribute(rmsnorm_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kRowsSmem);
        if (err != cudaSuccess) return err;
        rmsnorm_rows_kernel<<<(T + kRowsPerWarp - 1) / kRowsPerWarp, kRowsThreads, kRowsSmem, s>>>(x, w, out, T, D,
                                                                                                 eps);
        return cudaGetLastError();
    }
    const size_t smem = (size_t)D * sizeof(float);
    if (smem > kRmsnormMaxSmem) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {  // the attribute belongs to the current device's context
        cudaError_t err = cudaFuncSetAttribute(rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)kRmsnormMaxSmem);
        if (err != cudaSuccess) return err;
    }
    rmsnorm_kernel<<<T, kThreads, smem, s>>>(x, w, out, D, eps);
    return cudaGetLastError();
}

// Loads the combine and rmsnorm kernels now (see preload_kernels in kernels.h).
void preload_combine_kernels() {
    cudaFuncAttributes f;
    (void)cudaFuncGetAttributes(&f, combine_vec4_kernel);
    (void)cudaFuncGetAttributes(&f, combine_scalar_kernel);
    (void)cudaFuncGetAttributes(&f, rmsnorm_kernel);
    (void)cudaFuncGetAttributes(&f, rmsnorm_rows_kernel);
    (void)cudaGetLastError();
}

}  // namespace rbt
