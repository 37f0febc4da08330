// selfcheck.cu -- device-pointer entry points that expose the two exact
// primitives of the routing arithmetic (exact_math.cuh) on their own, so that a
// test can hold them against the host: the libm's expf over any range of float
// bit patterns, and rmsnorm's sequential sum of squares over any rows.
#include <stdint.h>

#include "../../include/rbt_moe.h"
#include "common.cuh"
#include "exact_math.cuh"
#include "kernels.h"

namespace rbt {
void set_last_error(const char* msg);

namespace {

constexpr int kThreads = 256;

__global__ void expf_range_kernel(uint32_t first_bits, int64_t n, float* out, int fma) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = expf_ref(__uint_as_float(first_bits + (uint32_t)i), fma);
}

// one CTA per row: the squares (separately rounded products) staged in shared memory
__global__ void __launch_bounds__(kThreads) seq_sumsq_kernel(const float* x, int n, float* out) {
    extern __shared__ float s_sq[];
    __shared__ SeqSumSmem s_seq;
    const float* xr = x + (size_t)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += kThreads) s_sq[i] = __fmul_rn(xr[i], xr[i]);
    __syncthreads();
    const float r = block_seq_sum<kThreads>(s_sq, n, s_seq);
    if (threadIdx.x == 0) out[blockIdx.x] = r;
}

int fail_cuda(cudaError_t e) {
    set_last_error(cudaGetErrorString(e));
    return 0;
}

}  // namespace
}  // namespace rbt

extern "C" int rbt_expf_device(uint32_t first_bits, int64_t n, float* d_out, void* stream) {
    if (n < 0 || (n > 0 && !d_out) || (uint64_t)first_bits + (uint64_t)n > (1ull << 32)) {
        rbt::set_last_error("rbt_expf_device: bad range or null output");
        return 0;
    }
    if (n == 0) return 1;
    const int64_t blocks = (n + rbt::kThreads - 1) / rbt::kThreads;
    const int grid = (int)(blocks < 148 * 32 ? blocks : 148 * 32);
    rbt::expf_range_kernel<<<grid, rbt::kThreads, 0, (cudaStream_t)stream>>>(first_bits, n, d_out,
                                                                             rbt::host_expf_fma());
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : rbt::fail_cuda(e);
}

extern "C" int rbt_seq_sumsq_device(const float* d_x, int rows, int n, float* d_out, void* stream) {
    if (rows < 0 || n < 0 || n > 16384 || (rows > 0 && (!d_x || !d_out))) {
        rbt::set_last_error("rbt_seq_sumsq_device: bad shape (n <= 16384) or null pointer");
        return 0;
    }
    if (rows == 0) return 1;
    const size_t smem = (size_t)(n > 0 ? n : 1) * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(rbt::seq_sumsq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return rbt::fail_cuda(e);
    }
    rbt::seq_sumsq_kernel<<<rows, rbt::kThreads, smem, (cudaStream_t)stream>>>(d_x, n, d_out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : rbt::fail_cuda(e);
}

extern "C" int rbt_host_expf_variant(void) { return rbt::host_expf_fma(); }
