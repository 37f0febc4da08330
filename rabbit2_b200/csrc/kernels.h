// kernels.h -- internal launch interface of the MoE kernels (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rbt {

constexpr int kMaxExperts = 256;  // router/top-k keeps E logits per token in one warp
constexpr int kMaxTopK = 64;      // MAX_TOPK, rabbit2.c:59

// 1 when this process's libm expf is the FMA-contracted evaluation of the table
// method (exact_math.cuh), 0 for the separately rounded one; probed once on the
// host, so the GPU softmax reproduces the host's expf bit for bit.
int host_expf_fma();

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
    int32_t* tile_cnt;        // [n_tiles, E] routed slots per (token tile, expert)
    int32_t* tile_base;       // [n_tiles, E] first position of the tile's slots of each expert
    int32_t* slot_rank;       // [T*K] rank of a slot among its tile's slots of the same expert
    int tile_tokens;          // set by launch_router: tokens per tile of the per-tile permutation (0: one tile)
    const uint16_t* router_cm;  // the router in chain-major order (router_to_chain_major), or nullptr
    unsigned* status;         // error word (a bounded wait that ran out), or nullptr
    // block form: xb = rmsnorm(x_raw, norm_w) first (written to xb, which then must
    // not alias x_raw); the token router computes it itself, the others launch it
    const float* x_raw;       // [T, D] or nullptr (xb given)
    const float* norm_w;      // [D]
    float eps;
    int expf_fma;             // host_expf_fma(): which evaluation of expf the host's libm uses
};
// The token router's copy of a bf16 router [E, D]: chain-major, 16-byte groups
// (E <= 64, D % 256 == 0; E * D * 2 bytes at `out`).
bool router_chain_major_supported(int E, int D, int dtype);
cudaError_t router_to_chain_major(const void* router, int E, int D, void* out, cudaStream_t s);
// Kernels launched are reported in *launches (1 or 2).
cudaError_t launch_router(const RouterArgs& a, cudaStream_t s, int* launches);
// The permutation of given routing (a.idx in [0, a.E) or -1): counts, offsets,
// active list, perm and slot_pos (-1 for slots outside this GPU's experts).
cudaError_t launch_route_given(const RouterArgs& a, cudaStream_t s, int* launches);

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
    int expf_fma;             // set by the launchers: host_expf_fma()
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

// K3 (decode, bf16): bulk-copy weight streaming (gemv_stream.cu).
struct StreamArgs {
    const float* xb;          // [T, D] normalised input
    const float* resid;       // [T, D] residual (block form) or nullptr
    float* out;               // [T, D] output (may alias resid)
    const uint8_t* experts;
    size_t stride;
    int T, D, H, K;
    const int32_t* perm;
    const int32_t* offsets;
    const int32_t* active;
    const int32_t* n_active;
    const int32_t* slot_pos;
    const float* wt;
    float* h;                 // [T*K, H]
    unsigned* status;
    int expf_fma;             // set by the launchers: host_expf_fma()
};
bool stream_supported(const StreamArgs& a, int dtype);
cudaError_t launch_gateup_stream(const StreamArgs& a, int grid, cudaStream_t s);
cudaError_t launch_down_combine_stream(const StreamArgs& a, int grid, cudaStream_t s);

// Batch-1 decode: the whole MoE block in one cooperative kernel (decode_fused.cu).
struct DecodeArgs {
    const float* x;           // [D] residual stream (block form) or normalised input (ffn form)
    float* out;               // [D] output; equals x in the block form
    const float* ffn_norm;    // [D] for the block form, nullptr for the ffn form
    float eps;
    const uint16_t* router;   // [E, D] bf16
    const float* bias;        // [E] or nullptr
    const uint8_t* experts;
    size_t stride;
    int D, H, E, K, norm_topk;
    float* logits;            // [E] the router logits (written by CTA 0)
    float* partials;          // [grid, D] scratch: each CTA's partial MoE output
    const uint8_t* w2t;       // [E][H][D] bf16 transposed w2 (rows of a unit contiguous), or nullptr
    size_t w2t_stride;        // bytes per expert in w2t (H * D * 2)
    const uint8_t* next_router;  // [E, D] bf16 router of the layer that runs next (L2 prefetch), or nullptr
    const float* next_norm;      // [D] ffn_norm of the layer that runs next (L2 prefetch), or nullptr
    int32_t *idx, *counts, *offsets, *perm, *slot_pos, *active, *n_active;
    float* wt;
    int32_t* routing_out;     // [K] or nullptr
    unsigned* sync;           // [decode_sync_words(E, K)] cross-CTA counters, zero between calls
    unsigned* status;
    int expf_fma;             // host_expf_fma()
    unsigned long long peer_wait_ns;  // bound of the waits on other CTAs (logits, grid barrier); 0: 2 s
};
int decode_sync_words(int E, int K);
size_t decode_partials_bytes(int grid, int D);
bool decode_fused_supported(int T, int D, int H, int E, int K, int dtype, const void* experts, size_t stride,
                            const void* x, const void* router);
// the 3-D TMA map of every expert's w2 columns the kernel reads (8 columns x 256 rows per box)
bool make_decode_w2_map(CUtensorMap* map, const void* experts, int D, int H, int E, size_t stride);
cudaError_t launch_decode_fused(const DecodeArgs& a, const CUtensorMap& w2map, int grid, cudaStream_t s);
// w2t[e] = w2[e]^T for the E experts of a layer (bf16 [H, D] each)
cudaError_t transpose_w2(const void* experts, size_t stride, int D, int H, int E, void* w2t, cudaStream_t s);

// K4: tcgen05 grouped GEMM (gemm_tc.cu).
struct TcGemmArgs {
    const int32_t* tb_e;      // [n_tb] expert of each token block
    const int32_t* tb_p0;     // [n_tb] first slot position of the block
    const int32_t* tb_p1;     // [n_tb] end of the expert's slot range
    const int32_t* n_tb;      // [1]
    int BN;                   // routed tokens per tile: 32, 64 or 128
    int MB;                   // 128-row weight blocks per token block (H/128 gate/up, D/128 down)
    int KB;                   // 64-element K blocks (D/64 gate/up, H/64 down)
    int H, D;
    void* h_hi;               // [S_cap, H] bf16 (gate/up output)
    void* h_lo;
    float* y;                 // [S_cap, D] f32 (down output)
    unsigned* status;         // 0, or the code of a timed-out pipeline wait
    const float* bscale;      // [S_cap] power-of-two scale of each fp16 activation row (fp16 gate/up only)
    // dense projections (launch_tc_dense): dense_T > 0 rows, one weight matrix
    // (expert 0), token blocks of BN consecutive rows, y row pitch ldy, y += when
    // accumulate; 0 for the MoE GEMMs (schedule from tb_*, y pitch D)
    int dense_T;
    int ldy;
    int accumulate;
    // split K (dense only): ksplit slices of kb_per K blocks each, slice s's partial
    // rows into part[s][dense_T][D]; ksplit <= 1 writes y directly
    int ksplit;
    int kb_per;
    float* part;
};
int tc_block_n();
int tc_pick_bn(int T, int K, int E);
bool tc_supported(int D, int H, int dtype);
bool make_map_2d(CUtensorMap* map, const void* base, int cols, long rows, int box_rows);
// out[T, N] (row pitch ldy) (+)= (xhi + xlo)[T, K] (row pitch ld_in) . W[N, K]^T on the
// tensor cores, W bf16; cudaErrorNotSupported when the shape does not tile
// (N % 128, K % 64, ld_in % 8) so the caller takes its CUDA-core form
// part/part_bytes: f32 scratch for split-K partial sums at small T (may be null).
cudaError_t launch_tc_dense(const void* W, int N, int K, const void* xhi, const void* xlo, int ld_in, int T,
                            float* y, int ldy, bool accumulate, unsigned* status, float* part, size_t part_bytes,
                            int grid, cudaStream_t s);
// The MoE gate/up (gate_up) or down GEMM of a BN = 128 schedule with the slots as
// the MMA's M side (128 slots x 256 weight rows per tile); xhi/xlo: the input
// rows' 128-row maps (x for gate/up, h for down); w: the experts' 3-D map.
cudaError_t launch_tc_rows_moe(bool gate_up, const CUtensorMap& w, const CUtensorMap& xhi, const CUtensorMap& xlo,
                               const TcGemmArgs& t, int grid, cudaStream_t s);
// the scratch launch_tc_dense uses for T rows of N outputs (0: none)
size_t tc_dense_part_bytes(int N, int K, int T, int grid);
// bf16 tensor map of rank 2 or 3 (dims / byte strides of dims 1.. / box, innermost
// first) with 128-byte swizzling; the box's inner extent must be 64 elements
bool make_map_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                    const uint32_t* box);
// Causal attention of T query rows (positions pos0 .. pos0+T-1; q in the rows of
// qkv after RoPE) over the f32 KV cache positions [0, pos0 + T) of one layer
// ([n_kv][ctx][hd]) on the tensor cores (attn_tc.cu), hd 64 or 128, into ao
// [T][n_heads * hd]; scratch of attn_tc_scratch_bytes, 256-byte aligned.
size_t attn_tc_scratch_bytes(int T, int nq, int n_kv, int hd, int nk);
cudaError_t launch_attn_tc(const float* qkv, int nqkv, int n_heads, int n_kv, int hd, const float* kc,
                           const float* vc, int ctx, int pos0, int T, void* scratch, size_t scratch_bytes, float* ao,
                           unsigned* status, cudaStream_t s);
bool make_map_experts(CUtensorMap* map, const void* base, int cols, int rows, int E, size_t stride);
// bf16 [E][rows][cols] with row pitch cols*2 and matrix pitch `stride`, unswizzled boxes
bool make_map_3d_plain(CUtensorMap* map, const void* base, int cols, int rows, int E, size_t stride, int box_cols,
                       int box_rows);
cudaError_t launch_gather_split(const float* xb, const int32_t* perm, int S, const int32_t* n_slots, int D, int K,
                                void* xhi, void* xlo,
                                cudaStream_t s);
cudaError_t launch_tc_schedule(const int32_t* counts, const int32_t* offsets, int E, int bn, int32_t* tb_e,
                               int32_t* tb_p0, int32_t* tb_p1, int32_t* n_tb, cudaStream_t s);
cudaError_t launch_tc_gateup(const CUtensorMap& w, const CUtensorMap& xhi, const CUtensorMap& xlo,
                             const TcGemmArgs& a, int grid, cudaStream_t s);
// The gate/up GEMM with one fp16 MMA per K step: w16 maps the fp16 copy of w1|w3
// (convert_gateup_f16), xh the fp16 activation rows (launch_gather_f16).
cudaError_t launch_tc_gateup_f16(const CUtensorMap& w16, const CUtensorMap& xh, const TcGemmArgs& a, int grid,
                                 cudaStream_t s);
cudaError_t launch_gather_f16(const float* xb, const int32_t* perm, int S, const int32_t* n_slots, int D, int K,
                              void* xh, float* scale, cudaStream_t s);
cudaError_t convert_gateup_f16(const void* experts, size_t stride, int D, int H, int E, void* out, unsigned* overflow,
                               cudaStream_t s);
cudaError_t launch_tc_down(const CUtensorMap& w, const CUtensorMap& hhi, const CUtensorMap& hlo, const TcGemmArgs& a,
                           int grid, cudaStream_t s);

}  // namespace rbt

namespace rbt {

// ---- Expert parallelism over NVLink peer memory (ep.cu) ----
// GPU g of R owns experts [g*epr, (g+1)*epr).  Each GPU's EP block holds, per
// source GPU s, a segment of `cap` received rows (f32 [D]), their K expert ids
// local to this GPU (-1: another GPU's slot, or no row) and K combine weights, the
// row count, and a dispatch flag; and per destination GPU g a segment of `cap`
// returned partial rows and a return flag.  Flags hold epochs (one per layer call,
// counted on the device), so nothing is ever reset.
constexpr int kEpMaxRanks = 8;
struct EpPeers {
    float* recv_rows[kEpMaxRanks];                    // GPU g's [R][cap][D]
    int32_t* recv_idx[kEpMaxRanks];                   // GPU g's [R][cap][K]
    float* recv_wt[kEpMaxRanks];                      // GPU g's [R][cap][K]
    int32_t* recv_count[kEpMaxRanks];                 // GPU g's [R]
    unsigned long long* flag_dispatch[kEpMaxRanks];   // GPU g's [R], slot = source
    float* back_rows[kEpMaxRanks];                    // GPU g's [R][cap][D]
    unsigned long long* flag_return[kEpMaxRanks];     // GPU g's [R], slot = destination
};
struct EpArgs {
    EpPeers peers;            // every GPU's buffers (this GPU's own at [rank])
    int R, rank, epr, cap, D, K;
    unsigned long long* epoch;  // this GPU's last finished layer call (read by all, advanced by the combine)
    unsigned* done;           // [2 + R] zeroed tickets: dispatch, combine, return per source
    unsigned* status;         // this context's status word
    unsigned long long timeout_ns;
};
// route -> plan (ep_plan, positions of the T tokens among those sent to each GPU)
// -> dispatch (rows, ids, weights into the owners' segments; count and flag) ->
// receive (wait for every source's flag; clear the ids of unused rows) -> the
// experts on the R*cap received rows -> return (each valid row's weighted sum over
// its slots into its source's segment; flag) -> combine (wait for every GPU's
// return flag; x += partials in GPU order; advance the epoch).
cudaError_t launch_ep_plan(const int32_t* idx, int T, int K, int R, int epr, int32_t* pos, int32_t* counts,
                           cudaStream_t s);
cudaError_t launch_ep_dispatch(const EpArgs& a, const float* xb, const int32_t* idx, const float* wt,
                               const int32_t* pos, const int32_t* counts, int T, cudaStream_t s);
cudaError_t launch_ep_receive(const EpArgs& a, cudaStream_t s);
// rows != nullptr: each received row's combined partial is already there (rows [R*cap][D])
cudaError_t launch_ep_return(const EpArgs& a, const float* y, const int32_t* slot_pos, const float* rows,
                             cudaStream_t s);
cudaError_t launch_ep_combine(const EpArgs& a, float* x, const int32_t* pos, int T, cudaStream_t s);

// With lazy module loading (the CUDA 12 default) a kernel is loaded at its first
// launch, and that load can wait for kernels already running on the device.  An
// expert-parallel layer has kernels that wait for other GPUs: a first launch issued
// behind one of them could stall the host until the wait gives up, before the
// other GPUs' work is even launched (one host thread driving several GPUs).  These
// load every kernel of the expert-parallel path up front (cudaFuncGetAttributes),
// on the current device.
void preload_router_kernels();
void preload_gemm_kernels();
void preload_gemv_kernels();
void preload_stream_kernels();
void preload_combine_kernels();
void preload_attn_tc_kernels();
void preload_ep_kernels();

}  // namespace rbt
