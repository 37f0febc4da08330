// kernels.h -- internal launch interface of the MoE kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rbt {

constexpr int kMaxExperts = 256;  // router/top-k keeps E logits per token in one warp
constexpr int kMaxTopK = 64;      // MAX_TOPK, rabbit2.c:59

// K1: router logits + softmax + top-k (+ the routed-slot permutation, done by
// the last CTA of the grid).
struct RouterArgs {
    const float* xb;          // [T, D] normalised MoE input
    int T, D, E, K;
    const void* router;       // [E, D] f32 or bf16 bits
    int dtype;                // 0 f32, 1 bf16
    const float* bias;        // [E] or nullptr
    int norm_topk;
    float* logits;            // [T, E] scratch
    int32_t* idx;             // [T*K] chosen experts, selection order
    float* wt;                // [T*K] combine weights (renormalised if norm_topk)
    int32_t* routing_out;     // [T, routing_stride] or nullptr
    int routing_stride;
    unsigned* tile_counter;   // [n_token_tiles], zero between calls
    unsigned* done_counter;   // [1], zero between calls
    int32_t* counts;          // [E] routed slots per expert
    int32_t* offsets;         // [E+1] exclusive prefix of counts
    int32_t* perm;            // [T*K] slot ids (t*K+k) grouped by expert, ascending within an expert
    int32_t* slot_pos;        // [T*K] inverse of perm
    int32_t* active;          // [E] experts with counts > 0, ascending
    int32_t* n_active;        // [1]
};
cudaError_t launch_router(const RouterArgs& a, cudaStream_t s);

// K3: grouped GEMV over the active experts (CUDA cores, fp32 accumulation).
struct GemvArgs {
    const float* xb;          // [T, D]
    const uint8_t* experts;   // E blobs, `stride` bytes apart: w1[H,D] | w3[H,D] | w2[D,H]
    size_t stride;
    int T, D, H, E, K, dtype;
    const int32_t* perm;
    const int32_t* offsets;
    const int32_t* active;
    const int32_t* n_active;
    float* h;                 // [T*K, H] SwiGLU activations, permuted order
    float* y;                 // [T*K, D] expert outputs, permuted order
    int grid;                 // CTAs to launch
};
cudaError_t launch_gateup_gemv(const GemvArgs& a, cudaStream_t s);
cudaError_t launch_down_gemv(const GemvArgs& a, cudaStream_t s);

// K5: weighted combine (+ residual) and the block form's RMSNorm.
struct CombineArgs {
    const float* resid;       // [T, D] or nullptr (ffn form)
    const float* y;           // [T*K, D] permuted expert outputs
    const float* wt;          // [T*K]
    const int32_t* slot_pos;  // [T*K]
    float* out;               // [T, D]
    int T, D, K;
};
cudaError_t launch_combine(const CombineArgs& a, cudaStream_t s);
cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int T, int D, float eps, cudaStream_t s);

}  // namespace rbt
