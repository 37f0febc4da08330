// gemm_tc.cu -- K4: grouped expert GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA) for prefill-sized batches.  Replaces the per-token
// matvecs of rabbit2.c:534-538 when many tokens share an expert.
//
// Formulation ("swap AB"): the weight rows are the MMA's M = 128 side and the
// routed tokens of one expert are its N side, so an expert with few tokens
// wastes little work:
//   gate/up:  [W1; W3] rows (128 of H each)  x  X_e^T   -> two 128 x BN accumulators,
//             epilogue h = silu(g) * u, stored as bf16 hi + lo
//   down:     W2 rows (128 of D)             x  H_e^T   -> one 128 x BN accumulator,
//             epilogue y (f32)
// Precision: weights are bf16 as stored in the model file.  Activations are f32
// and are split into bf16 hi = rn(x) and lo = rn(x - hi) (16 significant bits);
// each K step issues two MMAs (hi and lo) into the same f32 accumulator.  One
// bf16 operand alone gives ~3e-3 relative error on this layer, over the 1e-3 bar.
// The gate/up GEMM can instead run one fp16 MMA per K step (kF16): an fp16 copy
// of w1/w3 (bf16 values convert exactly unless they are fp16-subnormal), and the
// activation row scaled by a power of two so its largest element is below 2^14,
// rounded once to fp16 (11 significant bits); the epilogue undoes the scale.
//
// Pipeline per CTA (persistent, one CTA per SM, 192 threads):
//   warp 0  TMA producer: weight tile via a 3-D map over the expert blobs
//           (x = K, y = row, z = expert; no multicast), token tiles via 2-D maps
//   warp 1  TMEM owner and MMA issuer (one thread), tcgen05.commit to mbarriers
//   warps 2-5  epilogue: tcgen05.ld 32x32b, SwiGLU / split / store
// Two TMEM accumulator buffers let the epilogue of tile i overlap the MMAs of
// tile i+1.  Every mbarrier wait is bounded by %globaltimer; on timeout the
// kernel records an error code in `status`, drains its in-flight copies and
// MMAs (again bounded), frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rbt {
namespace {

using namespace tc;

constexpr int kBM = 128;   // weight rows per tile (MMA M)
constexpr int kBK = 64;    // K elements per stage = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kTileBytes = kBM * kBK * 2;  // 16 KB weight tile
constexpr int kStageBudget = 200 * 1024;   // shared memory for the operand ring
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait

// BN: routed tokens per tile (the MMA's N), 32, 64 or 128.
template <bool kGateUp, int BN, bool kF16 = false>
struct Cfg {
    static constexpr int NA = kGateUp ? 2 : 1;                 // weight tiles per stage
    static constexpr int NB = kF16 ? 1 : 2;                    // token tiles per stage (hi, lo | fp16)
    static constexpr int kBTileBytes = BN * kBK * 2;           // one token tile
    static constexpr int kStageBytes = NA * kTileBytes + NB * kBTileBytes;
    static constexpr int kStages = kStageBudget / kStageBytes > 6 ? 6 : kStageBudget / kStageBytes;
    static constexpr int kAccCols = NA * BN;                   // TMEM columns per accumulator buffer
    static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;  // double buffered
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
    static_assert(kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation");
};

__device__ __forceinline__ void record_error(unsigned* status, unsigned code) {
    atomicCAS(status, 0u, code);
}

template <bool kGateUp, int BN, bool kF16>
__global__ void __launch_bounds__(kThreads, 1)
    moe_tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_bhi,
                       const __grid_constant__ CUtensorMap tm_blo, TcGemmArgs a) {
    using C = Cfg<kGateUp, BN, kF16>;
    static_assert(kGateUp || !kF16, "the fp16 form is the gate/up GEMM's");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
    uint64_t* full = bars;                       // [kStages] TMA landed
    uint64_t* empty = bars + C::kStages;         // [kStages] MMAs done reading
    uint64_t* tfull = bars + 2 * C::kStages;     // [2] accumulator ready
    uint64_t* tempty = tfull + 2;                // [2] accumulator drained
    uint64_t* done = tempty + 2;                 // [1] drain barrier for the MMA issuer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4 * 32);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        prefetch_tmap(&tm_w);
        prefetch_tmap(&tm_bhi);
        prefetch_tmap(&tm_blo);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // tile = (K slice, token block, weight block); one K slice except split-K dense calls
    const int n_blk = a.dense_T ? (a.dense_T + BN - 1) / BN : *a.n_tb;
    const int n_ks = a.ksplit > 1 ? a.ksplit : 1;
    const int kb_per = n_ks > 1 ? a.kb_per : a.KB;
    const int n_tiles = n_blk * a.MB * n_ks;
    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_parity[C::kStages];
        bool used[C::kStages];
        for (int s = 0; s < C::kStages; s++) used[s] = false;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
            const int ks = tile / (n_blk * a.MB), rem = tile - ks * n_blk * a.MB;
            const int tbi = rem / a.MB, mb = rem - tbi * a.MB;
            const int e = a.dense_T ? 0 : a.tb_e[tbi], p0 = a.dense_T ? tbi * BN : a.tb_p0[tbi];
            const int kb0 = ks * kb_per, kb1 = min(a.KB, kb0 + kb_per);
            for (int kb = kb0; kb < kb1; kb++) {
                if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kWaitNs)) {
                    record_error(a.status, 0x101);
                    ok = false;
                    break;
                }
                uint8_t* st = smem + stage * C::kStageBytes;
                mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
                tma_load_3d(st, &tm_w, &full[stage], kb * kBK, mb * kBM, e);
                if (kGateUp) tma_load_3d(st + kTileBytes, &tm_w, &full[stage], kb * kBK, a.H + mb * kBM, e);
                tma_load_2d(st + C::NA * kTileBytes, &tm_bhi, &full[stage], kb * kBK, p0);
                if (!kF16) tma_load_2d(st + C::NA * kTileBytes + C::kBTileBytes, &tm_blo, &full[stage], kb * kBK, p0);
                used[stage] = true;
                last_parity[stage] = phase;
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        // every copy this thread issued has landed before the CTA may exit
        for (int s = 0; s < C::kStages; s++)
            if (used[s] && !mbar_wait_bounded(&full[s], last_parity[s], kWaitNs)) record_error(a.status, 0x102);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------ MMA issuer
        constexpr uint32_t idesc = kF16 ? idesc_f16_f32(kBM, BN) : idesc_bf16_f32(kBM, BN);
        int stage = 0;
        uint32_t phase = 0;
        int buf = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
            if (!mbar_wait_bounded(&tempty[buf], acc_phase ^ 1u, kWaitNs)) {
                record_error(a.status, 0x201);
                break;
            }
            tc_fence_after();
            const uint32_t d1 = tmem_base + buf * C::kAccCols;
            const int ks = tile / (n_blk * a.MB);
            const int kb0 = ks * kb_per, kb1 = min(a.KB, kb0 + kb_per);
            for (int kb = kb0; kb < kb1; kb++) {
                if (!mbar_wait_bounded(&full[stage], phase, kWaitNs)) {
                    record_error(a.status, 0x202);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
                const uint32_t sbh = sa + C::NA * kTileBytes, sbl = sbh + C::kBTileBytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; kk++) {
                    const uint32_t koff = kk * 32;  // 16 bf16 = 32 bytes along K
                    const uint64_t bh = sw128_kmajor_desc(sbh + koff), bl = sw128_kmajor_desc(sbl + koff);
                    const uint64_t a1 = sw128_kmajor_desc(sa + koff);
                    const uint32_t acc = (kb != kb0 || kk != 0) ? 1u : 0u;
                    mma_bf16(d1, a1, bh, idesc, acc);
                    if (!kF16) mma_bf16(d1, a1, bl, idesc, 1u);
                    if (kGateUp) {
                        const uint64_t a3 = sw128_kmajor_desc(sa + kTileBytes + koff);
                        mma_bf16(d1 + BN, a3, bh, idesc, acc);
                        if (!kF16) mma_bf16(d1 + BN, a3, bl, idesc, 1u);
                    }
                }
                mma_commit(&empty[stage]);
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            mma_commit(&tfull[buf]);
            if (++buf == 2) {
                buf = 0;
                acc_phase ^= 1u;
            }
        }
        // all MMAs issued by this thread have completed before TMEM is freed
        mma_commit(done);
        if (!mbar_wait_bounded(done, 0, kWaitNs)) record_error(a.status, 0x203);
    } else if (warp >= 2) {
        // ------------------------------------------------ epilogue (4 warps = 128 TMEM lanes)
        const int q = warp & 3;          // TMEM lane quadrant this warp may access
        const int row = q * 32 + lane;   // weight row within the tile
        int buf = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            const int ks = tile / (n_blk * a.MB), rem = tile - ks * n_blk * a.MB;
            const int tbi = rem / a.MB, mb = rem - tbi * a.MB;
            const int p0 = a.dense_T ? tbi * BN : a.tb_p0[tbi], p1 = a.dense_T ? a.dense_T : a.tb_p1[tbi];
            const int ntok = min(BN, p1 - p0);
            bool ok = mbar_wait_bounded(&tfull[buf], acc_phase, kWaitNs);
            ok = __all_sync(FULL_MASK, ok);
            if (!ok) {
                record_error(a.status, 0x301);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * C::kAccCols;
            for (int j0 = 0; j0 < ntok; j0 += 32) {
                uint32_t g[32];
                tmem_ld_32x32b_x32(tbase + j0, g);
                if (kGateUp) {
                    uint32_t u[32];
                    tmem_ld_32x32b_x32(tbase + BN + j0, u);
                    tmem_ld_wait();
                    const int col = mb * kBM + row;
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) {
                        const int p = p0 + j0 + jj;
                        if (j0 + jj < ntok) {
                            float gv = __uint_as_float(g[jj]), uv = __uint_as_float(u[jj]);
                            if (kF16) {  // undo the activation row's power-of-two scale (exact)
                                const float sc = a.bscale[p];
                                gv *= sc;
                                uv *= sc;
                            }
                            const float hv = gv / (1.0f + expf(-gv)) * uv;
                            const __nv_bfloat16 hi = __float2bfloat16_rn(hv);
                            const __nv_bfloat16 lo = __float2bfloat16_rn(hv - __bfloat162float(hi));
                            static_cast<__nv_bfloat16*>(a.h_hi)[(size_t)p * a.H + col] = hi;
                            static_cast<__nv_bfloat16*>(a.h_lo)[(size_t)p * a.H + col] = lo;
                        }
                    }
                } else {
                    tmem_ld_wait();
                    const int col = mb * kBM + row;
                    const size_t ldy = a.ldy ? (size_t)a.ldy : (size_t)a.D;
                    if (n_ks > 1) {  // this K slice's partial sums, reduced by dense_reduce_kernel
                        float* part = a.part + (size_t)ks * a.dense_T * a.D + col;
#pragma unroll
                        for (int jj = 0; jj < 32; jj++)
                            if (j0 + jj < ntok) part[(size_t)(p0 + j0 + jj) * a.D] = __uint_as_float(g[jj]);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 32; jj++) {
                            const int p = p0 + j0 + jj;
                            if (j0 + jj < ntok) {
                                float* dst = a.y + (size_t)p * ldy + col;
                                *dst = a.accumulate ? *dst + __uint_as_float(g[jj]) : __uint_as_float(g[jj]);
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
            if (++buf == 2) {
                buf = 0;
                acc_phase ^= 1u;
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// ---------------------------------------------------------------- dense, rows as M
// A dense projection of many rows (T >= 128): the activation rows are the MMA's
// M side (128 per tile, hi and lo) and the weight rows its N side (256 per tile),
// D = 128 x 256 f32 in TMEM, two buffers (all 512 columns).  Per K step of 64 the
// CTA stages 32 KB of rows and 32 KB of weights for two 128x256x64 MMA groups:
// two thirds of the shared-memory traffic per MMA of the 128-row weight tiles
// above, whose N = 128 MMAs read as many operand bytes per cycle as the shared
// memory delivers.
constexpr int kRM = 128, kRN = 256;
constexpr int kRATile = kRM * kBK * 2;                  // 16 KB of rows (hi or lo)
constexpr int kRStageBytes = 2 * kRATile + kRN * kBK * 2;  // 64 KB
constexpr int kRStages = 3;
constexpr int kRSmemBytes = kRStages * kRStageBytes + 1024 + 256;

// kRowsDense: y[t, n] (+)= rows . W^T, one weight matrix (2-D map, 256-row box).
// kRowsGateUp / kRowsDown: the MoE GEMMs over routed slots in expert order, token
// blocks of up to 128 slots of one expert (tb_* from tc_schedule_kernel with 128),
// weights through the experts' 3-D maps (128-row boxes): gate/up tile nt = w1
// rows [128 nt, +128) and w3 rows [H + 128 nt, +128), epilogue h = silu(g) * u as
// bf16 hi + lo; down tile nt = w2 rows [256 nt, +256), epilogue y rows (f32).
constexpr int kRowsDense = 0, kRowsGateUp = 1, kRowsDown = 2;

struct RowsGemmArgs {
    int T, N, KB;             // dense: rows, outputs; every mode: 64-element K blocks
    float* y;                 // dense / down output rows
    int ldy;                  // dense: y row pitch
    int accumulate;           // dense: y +=
    unsigned* status;
    const int32_t* tb_e;      // MoE: token blocks (expert, first slot, end of the expert's slots)
    const int32_t* tb_p0;
    const int32_t* tb_p1;
    const int32_t* n_tb;
    int H, D;                 // MoE: expert hidden, model dim
    void* h_hi;               // gate/up output [S_cap, H] bf16
    void* h_lo;
};

template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    rows_gemm_kernel(const __grid_constant__ CUtensorMap tm_xhi, const __grid_constant__ CUtensorMap tm_xlo,
                     const __grid_constant__ CUtensorMap tm_w, RowsGemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRStages * kRStageBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + kRStages;
    uint64_t* tfull = bars + 2 * kRStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    constexpr int kCols = 2 * kRN;  // 512

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4 * 32);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        prefetch_tmap(&tm_xhi);
        prefetch_tmap(&tm_xlo);
        prefetch_tmap(&tm_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // tile = (row block, 256-column block of the output)
    const int NT = kMode == kRowsDense ? a.N / kRN : kMode == kRowsGateUp ? a.H / 128 : a.D / kRN;
    const int n_tiles = (kMode == kRowsDense ? (a.T + kRM - 1) / kRM : *a.n_tb) * NT;
    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_parity[kRStages];
        bool used[kRStages];
        for (int s = 0; s < kRStages; s++) used[s] = false;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
            const int mt = tile / NT, nt = tile - mt * NT;
            const int row0 = kMode == kRowsDense ? mt * kRM : a.tb_p0[mt];
            const int e = kMode == kRowsDense ? 0 : a.tb_e[mt];
            for (int kb = 0; kb < a.KB; kb++) {
                if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kWaitNs)) {
                    record_error(a.status, 0x111);
                    ok = false;
                    break;
                }
                uint8_t* st = smem + stage * kRStageBytes;
                mbar_arrive_expect_tx(&full[stage], kRStageBytes);
                tma_load_2d(st, &tm_xhi, &full[stage], kb * kBK, row0);
                tma_load_2d(st + kRATile, &tm_xlo, &full[stage], kb * kBK, row0);
                if (kMode == kRowsDense) {
                    tma_load_2d(st + 2 * kRATile, &tm_w, &full[stage], kb * kBK, nt * kRN);
                } else {
                    const int w0 = kMode == kRowsGateUp ? nt * 128 : nt * kRN;
                    const int w1 = kMode == kRowsGateUp ? a.H + nt * 128 : nt * kRN + 128;
                    tma_load_3d(st + 2 * kRATile, &tm_w, &full[stage], kb * kBK, w0, e);
                    tma_load_3d(st + 2 * kRATile + kTileBytes, &tm_w, &full[stage], kb * kBK, w1, e);
                }
                used[stage] = true;
                last_parity[stage] = phase;
                if (++stage == kRStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        for (int s = 0; s < kRStages; s++)
            if (used[s] && !mbar_wait_bounded(&full[s], last_parity[s], kWaitNs)) record_error(a.status, 0x112);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------ MMA issuer
        constexpr uint32_t idesc = idesc_bf16_f32(kRM, kRN);
        int stage = 0;
        uint32_t phase = 0;
        int buf = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
            if (!mbar_wait_bounded(&tempty[buf], acc_phase ^ 1u, kWaitNs)) {
                record_error(a.status, 0x211);
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + buf * kRN;
            for (int kb = 0; kb < a.KB; kb++) {
                if (!mbar_wait_bounded(&full[stage], phase, kWaitNs)) {
                    record_error(a.status, 0x212);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sh = smem_u32(smem + stage * kRStageBytes);
                const uint32_t sl = sh + kRATile, sw = sh + 2 * kRATile;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; kk++) {
                    const uint32_t koff = kk * 32;
                    const uint64_t bw = sw128_kmajor_desc(sw + koff);
                    mma_bf16(d, sw128_kmajor_desc(sh + koff), bw, idesc, (kb | kk) != 0);
                    mma_bf16(d, sw128_kmajor_desc(sl + koff), bw, idesc, 1u);
                }
                mma_commit(&empty[stage]);
                if (++stage == kRStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            mma_commit(&tfull[buf]);
            if (++buf == 2) {
                buf = 0;
                acc_phase ^= 1u;
            }
        }
        mma_commit(done);
        if (!mbar_wait_bounded(done, 0, kWaitNs)) record_error(a.status, 0x213);
    } else if (warp >= 2) {
        // ------------------------------------------------ epilogue: thread = one activation row
        const int q = warp & 3;
        int buf = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            const int mt = tile / NT, nt = tile - mt * NT;
            const int t = (kMode == kRowsDense ? mt * kRM : a.tb_p0[mt]) + q * 32 + lane;
            const int t_end = kMode == kRowsDense ? a.T : a.tb_p1[mt];
            bool ok = mbar_wait_bounded(&tfull[buf], acc_phase, kWaitNs);
            ok = __all_sync(FULL_MASK, ok);
            if (!ok) {
                record_error(a.status, 0x311);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * kRN;
            if (kMode == kRowsGateUp) {
                // columns [0, 128): gate, [128, 256): up, of hidden units 128 nt + c
                for (int c0 = 0; c0 < 128; c0 += 32) {
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(tbase + c0, g);
                    tmem_ld_32x32b_x32(tbase + 128 + c0, u);
                    tmem_ld_wait();
                    if (t < t_end) {
                        uint32_t hw[16], lw[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            float hv[2];
#pragma unroll
                            for (int k = 0; k < 2; k++) {
                                const float gv = __uint_as_float(g[2 * i + k]), uv = __uint_as_float(u[2 * i + k]);
                                hv[k] = gv / (1.0f + expf(-gv)) * uv;
                            }
                            const __nv_bfloat16 h0 = __float2bfloat16_rn(hv[0]), h1 = __float2bfloat16_rn(hv[1]);
                            const __nv_bfloat16 l0 = __float2bfloat16_rn(hv[0] - __bfloat162float(h0));
                            const __nv_bfloat16 l1 = __float2bfloat16_rn(hv[1] - __bfloat162float(h1));
                            hw[i] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
                            lw[i] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
                        }
                        const size_t o = (size_t)t * a.H + nt * 128 + c0;
                        uint4* dh = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.h_hi) + o);
                        uint4* dl = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.h_lo) + o);
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            dh[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
                            dl[i] = make_uint4(lw[4 * i], lw[4 * i + 1], lw[4 * i + 2], lw[4 * i + 3]);
                        }
                    }
                }
            } else {
            float* yrow = a.y + (size_t)t * (kMode == kRowsDense ? a.ldy : a.D) + nt * kRN;
            for (int c0 = 0; c0 < kRN; c0 += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + c0, v);
                tmem_ld_wait();
                if (t < t_end) {
                    float4* dst = reinterpret_cast<float4*>(yrow + c0);
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        float4 o = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                               __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
                        if (kMode == kRowsDense && a.accumulate) {
                            const float4 old = dst[i];
                            o.x += old.x;
                            o.y += old.y;
                            o.z += old.z;
                            o.w += old.w;
                        }
                        dst[i] = o;
                    }
                }
            }
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
            if (++buf == 2) {
                buf = 0;
                acc_phase ^= 1u;
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kCols);
    }
}

// y[t, n] (+)= sum over the K slices s of part[s][t][n], in slice order.
__global__ void __launch_bounds__(256) dense_reduce_kernel(const float* __restrict__ part, int S, int T, int N,
                                                           float* y, int ldy, int accumulate) {
    const int n4 = N / 4;
    const long total = (long)T * n4;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int t = (int)(i / n4), c = (int)(i - (long)t * n4) * 4;
        float4 acc = reinterpret_cast<const float4*>(part + (size_t)t * N + c)[0];
        for (int s = 1; s < S; s++) {
            const float4 v = reinterpret_cast<const float4*>(part + ((size_t)s * T + t) * N + c)[0];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        float4* dst = reinterpret_cast<float4*>(y + (size_t)t * ldy + c);
        if (accumulate) {
            const float4 old = *dst;
            acc.x += old.x;
            acc.y += old.y;
            acc.z += old.z;
            acc.w += old.w;
        }
        *dst = acc;
    }
}

// f32 rows of x, gathered into expert order, split into bf16 hi + lo.
// n_slots (device, or null for S): the routed slots to gather; fewer than S when
// some slots belong to experts on other GPUs.
__global__ void __launch_bounds__(256) gather_split_kernel(const float* __restrict__ xb, const int32_t* perm, int S,
                                                           const int32_t* n_slots, int D, int K,
                                                           __nv_bfloat16* xhi, __nv_bfloat16* xlo) {
    const int vpr = D / 8;
    if (n_slots) S = min(S, *n_slots);
    const long total = (long)S * vpr;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int p = (int)(i / vpr), v = (int)(i - (long)p * vpr);
        const int t = perm[p] / K;
        const float4* src = reinterpret_cast<const float4*>(xb + (size_t)t * D + v * 8);
        const float4 f0 = __ldg(src), f1 = __ldg(src + 1);
        const float f[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
        __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
            hi[q] = __float2bfloat16_rn(f[q]);
            lo[q] = __float2bfloat16_rn(f[q] - __bfloat162float(hi[q]));
        }
        *reinterpret_cast<uint4*>(xhi + (size_t)p * D + v * 8) = *reinterpret_cast<const uint4*>(hi);
        *reinterpret_cast<uint4*>(xlo + (size_t)p * D + v * 8) = *reinterpret_cast<const uint4*>(lo);
    }
}

// Token blocks of bn routed slots per active expert (one CTA, E <= 256).
__global__ void __launch_bounds__(256) tc_schedule_kernel(const int32_t* counts, const int32_t* offsets, int E,
                                                          int bn, int32_t* tb_e, int32_t* tb_p0, int32_t* tb_p1,
                                                          int32_t* n_tb) {
    __shared__ int32_t s_nt[kMaxExperts + 1];
    const int e = threadIdx.x;
    const int nt = (e < E) ? (counts[e] + bn - 1) / bn : 0;
    s_nt[e] = nt;
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int i = 0; i < E; i++) {
            const int c = s_nt[i];
            s_nt[i] = run;
            run += c;
        }
        s_nt[kMaxExperts] = run;
        *n_tb = run;
    }
    __syncthreads();
    if (e < E) {
        const int base = s_nt[e], p_end = offsets[e + 1];
        for (int j = 0; j < nt; j++) {
            tb_e[base + j] = e;
            tb_p0[base + j] = offsets[e] + j * bn;
            tb_p1[base + j] = p_end;
        }
    }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

template <bool kGateUp, int BN, bool kF16>
cudaError_t launch_gemm_bn(const CUtensorMap& w, const CUtensorMap& bhi, const CUtensorMap& blo,
                           const TcGemmArgs& a, int grid, cudaStream_t s) {
    using C = Cfg<kGateUp, BN, kF16>;
    cudaError_t err = cudaFuncSetAttribute(moe_tc_gemm_kernel<kGateUp, BN, kF16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (err != cudaSuccess) return err;
    moe_tc_gemm_kernel<kGateUp, BN, kF16><<<grid, kThreads, C::kSmemBytes, s>>>(w, bhi, blo, a);
    return cudaGetLastError();
}

template <bool kGateUp, bool kF16 = false>
cudaError_t launch_gemm(const CUtensorMap& w, const CUtensorMap& bhi, const CUtensorMap& blo, const TcGemmArgs& a,
                        int grid, cudaStream_t s) {
    switch (a.BN) {
        case 32: return launch_gemm_bn<kGateUp, 32, kF16>(w, bhi, blo, a, grid, s);
        case 64: return launch_gemm_bn<kGateUp, 64, kF16>(w, bhi, blo, a, grid, s);
        case 128: return launch_gemm_bn<kGateUp, 128, kF16>(w, bhi, blo, a, grid, s);
        default: return cudaErrorInvalidValue;
    }
}

// fp16 rows for the gate/up GEMM: one warp per routed slot; the row is scaled by
// 2^-s (s from its largest magnitude, so that every element is below 2^14) and
// rounded once to fp16; scale[p] = 2^s.
__global__ void __launch_bounds__(256) gather_f16_kernel(const float* __restrict__ xb, const int32_t* perm, int S,
                                                         const int32_t* n_slots, int D, int K, __half* xh,
                                                         float* scale) {
    if (n_slots) S = min(S, *n_slots);
    const int lane = threadIdx.x & 31;
    const int nw = gridDim.x * (blockDim.x >> 5);
    for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < S; p += nw) {
        const float4* src = reinterpret_cast<const float4*>(xb + (size_t)(perm[p] / K) * D);
        float mx = 0.0f;
        for (int v = lane; v < D / 4; v += 32) {
            const float4 f = __ldg(src + v);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // mx < 2^e for its binary exponent e (mx = m * 2^e, 0.5 <= m < 1): the
        // scaled row stays below 2^14
        int sexp = 0;
        if (mx > 0.0f) {
            int e;
            frexpf(mx, &e);
            sexp = e - 14;
        }
        if (lane == 0) scale[p] = ldexpf(1.0f, sexp);
        for (int v = lane; v < D / 4; v += 32) {
            const float4 f = __ldg(src + v);
            const __half2 h01 = __floats2half2_rn(ldexpf(f.x, -sexp), ldexpf(f.y, -sexp));
            const __half2 h23 = __floats2half2_rn(ldexpf(f.z, -sexp), ldexpf(f.w, -sexp));
            __half2* d = reinterpret_cast<__half2*>(xh + (size_t)p * D + v * 4);
            d[0] = h01;
            d[1] = h23;
        }
    }
}

// w1|w3 of every expert as one fp16 matrix [2H, D] per expert (rows w1 then w3),
// contiguous; *overflow is set if a value does not fit fp16.
__global__ void convert_gateup_f16_kernel(const uint8_t* experts, size_t stride, int D, int H, int E, __half* out,
                                          unsigned* overflow) {
    const size_t per = (size_t)2 * H * D;
    const size_t total = per * E;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t e = i / per, j = i - e * per;
        const uint16_t b = reinterpret_cast<const uint16_t*>(experts + e * stride)[j];
        const float f = __uint_as_float((uint32_t)b << 16);
        if (fabsf(f) > 65504.0f) atomicExch(overflow, 1u);
        out[i] = __float2half_rn(f);
    }
}

}  // namespace

int tc_block_n() { return 128; }

// Token-tile width for a call of T tokens: the MMA's N is wasted on empty
// columns when an expert sees fewer tokens than N (uniform routing gives
// T*K/E tokens per expert).
int tc_pick_bn(int T, int K, int E) {
    static const int forced = [] {
        const char* v = getenv("RBT_MOE_TC_BN");  // tuning: 32, 64 or 128 for every call
        const int n = v ? atoi(v) : 0;
        return (n == 32 || n == 64 || n == 128) ? n : 0;
    }();
    if (forced) return forced;
    // measured (16 layers, OLMoE shape): T = 64 (8 slots per expert) 3.12 / 3.27 ms per step
    // with 32- / 64-token blocks; T = 256 (32 per expert) 4.11 / 3.47 / 3.95 ms with 32 / 64 / 128
    const long per_expert = ((long)T * K + E - 1) / E;
    if (per_expert <= 8) return 32;
    if (per_expert <= 96) return 64;
    return 128;
}

bool tc_supported(int D, int H, int dtype) {
    return dtype == 1 && D % kBM == 0 && H % kBM == 0 && D % kBK == 0 && H % kBK == 0 && encode_fn() != nullptr;
}

// Row-major bf16 matrix [rows, cols] as a 2-D TMA map with a kBK x box_rows box.
bool make_map_2d(CUtensorMap* map, const void* base, int cols, long rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major bf16 matrix [rows, cols] with a row pitch of ld elements, kBK x box_rows box.
bool make_map_2d_ld(CUtensorMap* map, const void* base, int cols, int ld, long rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                    const uint32_t* box) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || rank < 2 || rank > 3 || box[0] != 64) return false;
    cuuint64_t d[3], st[2];
    cuuint32_t b[3], es[3] = {1, 1, 1};
    for (int i = 0; i < rank; i++) {
        d[i] = dims[i];
        b[i] = box[i];
    }
    for (int i = 0; i + 1 < rank; i++) st[i] = strides[i];
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, st, b, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per-expert row-major bf16 matrices [rows, cols] `stride` bytes apart as a 3-D
// map (x = column, y = row, z = expert) with a kBK x kBM x 1 box.
bool make_map_experts(CUtensorMap* map, const void* base, int cols, int rows, int E, size_t stride) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)E};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)stride};
    cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)kBM, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_3d_plain(CUtensorMap* map, const void* base, int cols, int rows, int E, size_t stride, int box_cols,
                       int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)E};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)stride};
    cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_gather_split(const float* xb, const int32_t* perm, int S, const int32_t* n_slots, int D, int K,
                                void* xhi, void* xlo, cudaStream_t s) {
    if (S <= 0) return cudaSuccess;
    const long total = (long)S * (D / 8);
    const long blocks = (total + 255) / 256;
    gather_split_kernel<<<(int)(blocks < 148L * 8 ? blocks : 148L * 8), 256, 0, s>>>(
        xb, perm, S, n_slots, D, K, static_cast<__nv_bfloat16*>(xhi), static_cast<__nv_bfloat16*>(xlo));
    return cudaGetLastError();
}

cudaError_t launch_tc_schedule(const int32_t* counts, const int32_t* offsets, int E, int bn, int32_t* tb_e,
                               int32_t* tb_p0, int32_t* tb_p1, int32_t* n_tb, cudaStream_t s) {
    tc_schedule_kernel<<<1, 256, 0, s>>>(counts, offsets, E, bn, tb_e, tb_p0, tb_p1, n_tb);
    return cudaGetLastError();
}

cudaError_t launch_tc_gateup(const CUtensorMap& w, const CUtensorMap& xhi, const CUtensorMap& xlo,
                             const TcGemmArgs& a, int grid, cudaStream_t s) {
    return launch_gemm<true>(w, xhi, xlo, a, grid, s);
}

cudaError_t launch_tc_gateup_f16(const CUtensorMap& w16, const CUtensorMap& xh, const TcGemmArgs& a, int grid,
                                 cudaStream_t s) {
    if (!a.bscale) return cudaErrorInvalidValue;
    return launch_gemm<true, true>(w16, xh, xh, a, grid, s);
}

cudaError_t launch_gather_f16(const float* xb, const int32_t* perm, int S, const int32_t* n_slots, int D, int K,
                              void* xh, float* scale, cudaStream_t s) {
    if (S <= 0) return cudaSuccess;
    const int blocks = (S + 7) / 8 < 148 * 16 ? (S + 7) / 8 : 148 * 16;
    gather_f16_kernel<<<blocks, 256, 0, s>>>(xb, perm, S, n_slots, D, K, static_cast<__half*>(xh), scale);
    return cudaGetLastError();
}

cudaError_t convert_gateup_f16(const void* experts, size_t stride, int D, int H, int E, void* out, unsigned* overflow,
                               cudaStream_t s) {
    convert_gateup_f16_kernel<<<148 * 8, 256, 0, s>>>(static_cast<const uint8_t*>(experts), stride, D, H, E,
                                                       static_cast<__half*>(out), overflow);
    return cudaGetLastError();
}

cudaError_t launch_tc_down(const CUtensorMap& w, const CUtensorMap& hhi, const CUtensorMap& hlo, const TcGemmArgs& a,
                           int grid, cudaStream_t s) {
    return launch_gemm<false>(w, hhi, hlo, a, grid, s);
}

// Dense projections: many rows (T >= 128, N % 256 == 0) take the rows-as-M
// kernel; fewer take the down GEMM's one-matrix case (the weight rows as M, the
// rows as N in blocks of BN consecutive rows, rows past T read as zeros), with K
// split over up to 8 CTAs per tile when the tiles alone would leave SMs idle.
struct DensePlan {
    bool rows;  // rows-as-M kernel
    int bn, ksplit, kb_per;
};

static DensePlan dense_plan(int N, int K, int T, int grid) {
    DensePlan p{false, 32, 1, K / kBK};
    if (T >= kRM && N % kRN == 0) {
        p.rows = true;
        return p;
    }
    p.bn = T > 64 ? 128 : T > 32 ? 64 : 32;
    const int KB = K / kBK, tiles = (N / kBM) * ((T + p.bn - 1) / p.bn);
    if (2 * tiles <= grid) {
        int S = grid / tiles < 8 ? grid / tiles : 8;
        S = S < KB ? S : KB;
        p.kb_per = (KB + S - 1) / S;
        p.ksplit = (KB + p.kb_per - 1) / p.kb_per;
    }
    return p;
}


size_t tc_dense_part_bytes(int N, int K, int T, int grid) {
    if (T <= 0 || N % kBM || K % kBK) return 0;
    const DensePlan p = dense_plan(N, K, T, grid);
    return p.rows || p.ksplit <= 1 ? 0 : (size_t)p.ksplit * T * N * 4;
}

cudaError_t launch_tc_dense(const void* W, int N, int K, const void* xhi, const void* xlo, int ld_in, int T,
                            float* y, int ldy, bool accumulate, unsigned* status, float* part, size_t part_bytes,
                            int grid, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    if (N % kBM || K % kBK || ld_in % 8 || ld_in < K || ldy % 4 || ldy < N ||
        ((uintptr_t)W | (uintptr_t)xhi | (uintptr_t)xlo | (uintptr_t)y) & 15 || !encode_fn())
        return cudaErrorNotSupported;
    DensePlan p = dense_plan(N, K, T, grid);
    if (p.rows) {
        CUtensorMap mh, ml, mw;
        if (!make_map_2d_ld(&mh, xhi, K, ld_in, T, kRM) || !make_map_2d_ld(&ml, xlo, K, ld_in, T, kRM) ||
            !make_map_2d_ld(&mw, W, K, K, N, kRN))
            return cudaErrorNotSupported;
        RowsGemmArgs a{};
        a.T = T;
        a.N = N;
        a.KB = K / kBK;
        a.y = y;
        a.ldy = ldy;
        a.accumulate = accumulate ? 1 : 0;
        a.status = status;
        cudaError_t err = cudaFuncSetAttribute(rows_gemm_kernel<kRowsDense>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kRSmemBytes);
        if (err != cudaSuccess) return err;
        const int tiles = ((T + kRM - 1) / kRM) * (N / kRN);
        rows_gemm_kernel<kRowsDense><<<tiles < grid ? tiles : grid, kThreads, kRSmemBytes, s>>>(mh, ml, mw, a);
        return cudaGetLastError();
    }
    if (p.ksplit > 1 && (!part || part_bytes < (size_t)p.ksplit * T * N * 4)) p.ksplit = 1;
    CUtensorMap mw, mh, ml;
    if (!make_map_experts(&mw, W, K, N, 1, (size_t)N * K * 2) || !make_map_2d_ld(&mh, xhi, K, ld_in, T, p.bn) ||
        !make_map_2d_ld(&ml, xlo, K, ld_in, T, p.bn))
        return cudaErrorNotSupported;
    TcGemmArgs a{};
    a.BN = p.bn;
    a.MB = N / kBM;
    a.KB = K / kBK;
    a.D = N;
    a.y = y;
    a.status = status;
    a.dense_T = T;
    a.ldy = ldy;
    a.accumulate = accumulate ? 1 : 0;
    if (p.ksplit > 1) {
        a.ksplit = p.ksplit;
        a.kb_per = p.kb_per;
        a.part = part;
    }
    const int tiles = a.MB * ((T + p.bn - 1) / p.bn) * (p.ksplit > 1 ? p.ksplit : 1);
    cudaError_t err = launch_gemm<false>(mw, mh, ml, a, tiles < grid ? tiles : grid, s);
    if (err != cudaSuccess || p.ksplit <= 1) return err;
    const long n4 = (long)T * (N / 4);
    const long blocks = (n4 + 255) / 256;
    dense_reduce_kernel<<<(int)(blocks < 148L * 4 ? blocks : 148L * 4), 256, 0, s>>>(part, p.ksplit, T, N, y, ldy,
                                                                                      a.accumulate);
    return cudaGetLastError();
}

// The MoE GEMMs of 128-slot token blocks (tc_pick_bn 128) with the activation
// slots as the MMA's M side: t, its BN = 128 schedule; xhi/xlo the 128-row maps
// of the gate/up input rows (h rows for down), w the experts' 3-D map.
cudaError_t launch_tc_rows_moe(bool gate_up, const CUtensorMap& w, const CUtensorMap& xhi, const CUtensorMap& xlo,
                               const TcGemmArgs& t, int grid, cudaStream_t s) {
    if (t.BN != kRM || (gate_up ? t.H % 128 : t.D % kRN)) return cudaErrorInvalidValue;
    RowsGemmArgs a{};
    a.KB = t.KB;
    a.y = t.y;
    a.status = t.status;
    a.tb_e = t.tb_e;
    a.tb_p0 = t.tb_p0;
    a.tb_p1 = t.tb_p1;
    a.n_tb = t.n_tb;
    a.H = t.H;
    a.D = t.D;
    a.h_hi = t.h_hi;
    a.h_lo = t.h_lo;
    cudaError_t err = cudaFuncSetAttribute(gate_up ? rows_gemm_kernel<kRowsGateUp> : rows_gemm_kernel<kRowsDown>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kRSmemBytes);
    if (err != cudaSuccess) return err;
    if (gate_up)
        rows_gemm_kernel<kRowsGateUp><<<grid, kThreads, kRSmemBytes, s>>>(xhi, xlo, w, a);
    else
        rows_gemm_kernel<kRowsDown><<<grid, kThreads, kRSmemBytes, s>>>(xhi, xlo, w, a);
    return cudaGetLastError();
}

// Loads every tensor-core path kernel now (see preload_kernels in kernels.h).
void preload_gemm_kernels() {
    cudaFuncAttributes f;
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<true, 32, false>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<true, 64, false>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<true, 128, false>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<false, 32, false>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<false, 64, false>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<false, 128, false>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<true, 32, true>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<true, 64, true>);
    (void)cudaFuncGetAttributes(&f, moe_tc_gemm_kernel<true, 128, true>);
    (void)cudaFuncGetAttributes(&f, gather_split_kernel);
    (void)cudaFuncGetAttributes(&f, gather_f16_kernel);
    (void)cudaFuncGetAttributes(&f, tc_schedule_kernel);
    (void)cudaFuncGetAttributes(&f, rows_gemm_kernel<kRowsDense>);
    (void)cudaFuncGetAttributes(&f, rows_gemm_kernel<kRowsGateUp>);
    (void)cudaFuncGetAttributes(&f, rows_gemm_kernel<kRowsDown>);
    (void)cudaFuncGetAttributes(&f, dense_reduce_kernel);
    (void)cudaGetLastError();
}

}  // namespace rbt
