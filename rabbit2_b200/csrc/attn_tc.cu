// attn_tc.cu -- causal attention of a whole prompt on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA), the bf16 models' batched prompt: for every head h
// and query row t (position pos0 + t) over the cache positions p <= pos0 + t,
//   att[p] = q . k[p] / sqrt(head_dim),  P = softmax(att),  out = sum_p P[p] v[p]
// as rabbit2.c:487-506 computes it one row at a time.
//
// One CTA per (head, 128 query rows); key positions in blocks of 64.  Precision:
// q, k, v, P are f32 values split into bf16 hi = rn(x) and lo = rn(x - hi); each
// product is hi.hi + hi.lo + lo.hi (three MMAs into one f32 accumulator; lo.lo is
// below f32 rounding of the sum).  One pass over the key blocks: S = Q K^T of a
// block into TMEM, p = exp(att - m) against the row's running max m, written as
// bf16 hi/lo rows of P into shared memory and summed in f32, and O += P V in TMEM;
// the epilogue divides O by the sum.  m moves only when a block's max exceeds it
// by enough to make p larger than 2^8, and then the row threads rescale O in TMEM
// between two blocks' P.V MMAs (rarely: a row's max settles within a few blocks).
//
// Roles (192 threads): warp 0 issues the TMA loads (Q once; K and V^T blocks in
// 2-slot rings); warp 1 owns TMEM and issues the
// MMAs; warps 2-5 (one thread per query row, TMEM lane quadrant warp % 4) run the
// softmax and the epilogue.  TMEM: two 64-column S buffers and the O accumulator.
// Every mbarrier wait is bounded by %globaltimer; a wait that runs out records a
// code in `status`, and every role unwinds (bounded) so the CTA frees TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace rbt {
namespace {

using namespace tc;

constexpr int kAQ = 128;  // query rows per CTA (MMA M)
constexpr int kAK = 64;   // key positions per block (S MMA N; P.V MMA K)
constexpr int kAThreads = 192;
constexpr uint64_t kAWaitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait
constexpr float kRescale = 8.0f;              // log2 of the largest p before the running max moves

template <int HD>
struct AttnCfg {
    static constexpr int kQChunk = kAQ * 128;              // 128 rows x 64 columns, 128-byte swizzle: 16 KB
    static constexpr int kQBytes = (HD / 64) * kQChunk;    // Q hi (or lo)
    static constexpr int kKChunk = kAK * 128;              // 64 keys x 64 columns: 8 KB
    static constexpr int kKBytes = (HD / 64) * kKChunk;    // K hi (or lo) of one block
    static constexpr int kVBytes = HD * 128;               // V^T hi (or lo): HD rows x 64 keys
    static constexpr int kPBytes = kAQ * 128;              // P hi (or lo): 128 rows x 64 keys
    static constexpr int oQ = 0;                           // Q hi, Q lo
    static constexpr int oK = 2 * kQBytes;                 // K ring [2] {hi, lo}
    static constexpr int oV = oK + 2 * 2 * kKBytes;        // V ring [2] {hi, lo}
    static constexpr int oP = oV + 2 * 2 * kVBytes;        // P hi, P lo
    static constexpr int oBar = oP + 2 * kPBytes;
    static constexpr int kSmem = oBar + 256 + 1024;
    static constexpr int kOCol = 2 * kAK;                  // O after the two S buffers
    static constexpr int kTmemCols = kOCol + HD <= 256 ? 256 : 512;
    static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
    static_assert(kSmem <= 232448, "shared memory per CTA");
};

struct AttnTcArgs {
    int T, pos0, nk, grp;  // query rows, first position, cache positions, heads per kv head
    float k2;              // 1/sqrt(head_dim) * log2(e)
    float* ao;             // [T][ld_ao], head h at columns h * HD
    int ld_ao;
    unsigned* status;
};

__device__ __forceinline__ void record(unsigned* status, unsigned code) { atomicCAS(status, 0u, code); }

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2^x of the MUFU unit (results below 2^-126 flush to 0: they are below the f32
// resolution of a softmax row whose largest term is 1)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 16-byte chunk `c` (of 8) of row `r` in a 128-byte-swizzled K-major tile
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

template <int HD>
__global__ void __launch_bounds__(kAThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_qh, const __grid_constant__ CUtensorMap tm_ql,
                   const __grid_constant__ CUtensorMap tm_kh, const __grid_constant__ CUtensorMap tm_kl,
                   const __grid_constant__ CUtensorMap tm_vh, const __grid_constant__ CUtensorMap tm_vl,
                   AttnTcArgs a) {
    using C = AttnCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::oBar);
    uint64_t* qfull = bars;        // Q landed
    uint64_t* kfull = bars + 1;    // [2] K block landed
    uint64_t* kempty = bars + 3;   // [2] S MMAs done reading it
    uint64_t* vfull = bars + 5;    // [2] V^T block landed
    uint64_t* vempty = bars + 7;   // [2] P.V MMAs done reading it
    uint64_t* sfull = bars + 9;    // [2] S buffer written
    uint64_t* sfree = bars + 11;   // [2] S buffer read by the 128 row threads
    uint64_t* pfull = bars + 13;   // P rows written by the 128 row threads
    uint64_t* pfree = bars + 14;   // P.V MMAs done reading P
    uint64_t* ofull = bars + 15;   // O complete
    uint64_t* done = bars + 16;    // drain barrier of the MMA issuer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, g = h / a.grp;
    const int q0 = (gridDim.y - 1 - blockIdx.y) * kAQ;  // the tiles with the most keys start first
    const int kend = min(a.nk, a.pos0 + q0 + kAQ);      // positions the tile's rows can see
    const int nblk = (kend + kAK - 1) / kAK;

    if (threadIdx.x == 0) {
        mbar_init(qfull, 1);
        for (int s = 0; s < 2; s++) {
            mbar_init(&kfull[s], 1);
            mbar_init(&kempty[s], 1);
            mbar_init(&vfull[s], 1);
            mbar_init(&vempty[s], 1);
            mbar_init(&sfull[s], 1);
            mbar_init(&sfree[s], kAQ);
        }
        mbar_init(pfull, kAQ);
        mbar_init(pfree, 1);
        mbar_init(ofull, 1);
        mbar_init(done, 1);
        fence_mbar_init();
        prefetch_tmap(&tm_qh);
        prefetch_tmap(&tm_ql);
        prefetch_tmap(&tm_kh);
        prefetch_tmap(&tm_kl);
        prefetch_tmap(&tm_vh);
        prefetch_tmap(&tm_vl);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        bool ok = true;
        bool kused[2] = {false, false}, vused[2] = {false, false};
        uint32_t kpar[2] = {0, 0}, vpar[2] = {0, 0};
        mbar_arrive_expect_tx(qfull, 2 * C::kQBytes);
#pragma unroll
        for (int c = 0; c < HD / 64; c++) {
            tma_load_2d(smem + C::oQ + c * C::kQChunk, &tm_qh, qfull, h * HD + c * 64, q0);
            tma_load_2d(smem + C::oQ + C::kQBytes + c * C::kQChunk, &tm_ql, qfull, h * HD + c * 64, q0);
        }
        for (int j = 0; j < nblk; j++) {
            const int ks = j & 1;
            if (!mbar_wait_bounded(&kempty[ks], ((j >> 1) & 1) ^ 1u, kAWaitNs)) {
                record(a.status, 0x121);
                ok = false;
                break;
            }
            uint8_t* st = smem + C::oK + ks * 2 * C::kKBytes;
            mbar_arrive_expect_tx(&kfull[ks], 2 * C::kKBytes);
#pragma unroll
            for (int c = 0; c < HD / 64; c++) {
                tma_load_3d(st + c * C::kKChunk, &tm_kh, &kfull[ks], c * 64, j * kAK, g);
                tma_load_3d(st + C::kKBytes + c * C::kKChunk, &tm_kl, &kfull[ks], c * 64, j * kAK, g);
            }
            kused[ks] = true;
            kpar[ks] = (j >> 1) & 1;
            const int vs = j & 1;
            if (!mbar_wait_bounded(&vempty[vs], ((j >> 1) & 1) ^ 1u, kAWaitNs)) {
                record(a.status, 0x122);
                ok = false;
                break;
            }
            uint8_t* sv = smem + C::oV + vs * 2 * C::kVBytes;
            mbar_arrive_expect_tx(&vfull[vs], 2 * C::kVBytes);
            tma_load_3d(sv, &tm_vh, &vfull[vs], j * kAK, 0, g);
            tma_load_3d(sv + C::kVBytes, &tm_vl, &vfull[vs], j * kAK, 0, g);
            vused[vs] = true;
            vpar[vs] = (j >> 1) & 1;
        }
        // every copy this thread issued has landed before the CTA may exit
        if (!mbar_wait_bounded(qfull, 0, kAWaitNs)) record(a.status, 0x123);
        for (int s = 0; s < 2; s++) {
            if (kused[s] && !mbar_wait_bounded(&kfull[s], kpar[s], kAWaitNs)) record(a.status, 0x123);
            if (vused[s] && !mbar_wait_bounded(&vfull[s], vpar[s], kAWaitNs)) record(a.status, 0x123);
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------ MMA issuer
        constexpr uint32_t idS = idesc_bf16_f32(kAQ, kAK);
        constexpr uint32_t idO = idesc_bf16_f32(kAQ, HD);
        const uint32_t sQh = smem_u32(smem + C::oQ), sQl = sQh + C::kQBytes;
        const uint32_t dO = tmem_base + C::kOCol;
        bool ok = mbar_wait_bounded(qfull, 0, kAWaitNs);
        if (!ok) record(a.status, 0x221);
        tc_fence_after();
        int kn = 0, sn = 0;
        // S[sn & 1] = Q . K^T of the next K block in the ring
        auto issue_s = [&]() -> bool {
            const int ks = kn & 1, sb = sn & 1;
            if (!mbar_wait_bounded(&kfull[ks], (kn >> 1) & 1, kAWaitNs)) {
                record(a.status, 0x222);
                return false;
            }
            if (!mbar_wait_bounded(&sfree[sb], ((sn >> 1) & 1) ^ 1u, kAWaitNs)) {
                record(a.status, 0x223);
                return false;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + sb * kAK;
            const uint32_t sKh = smem_u32(smem + C::oK + ks * 2 * C::kKBytes), sKl = sKh + C::kKBytes;
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++) {
                const uint32_t qo = (kk >> 2) * C::kQChunk + (kk & 3) * 32;
                const uint32_t ko = (kk >> 2) * C::kKChunk + (kk & 3) * 32;
                const uint64_t qh = sw128_kmajor_desc(sQh + qo), ql = sw128_kmajor_desc(sQl + qo);
                const uint64_t kh = sw128_kmajor_desc(sKh + ko), kl = sw128_kmajor_desc(sKl + ko);
                mma_bf16(d, qh, kh, idS, kk != 0);
                mma_bf16(d, qh, kl, idS, 1u);
                mma_bf16(d, ql, kh, idS, 1u);
            }
            mma_commit(&kempty[ks]);
            mma_commit(&sfull[sb]);
            kn++;
            sn++;
            return true;
        };
        if (ok) ok = issue_s();  // block 0
        for (int j = 0; ok && j < nblk; j++) {
            if (j + 1 < nblk && !(ok = issue_s())) break;  // S of block j+1 overlaps the softmax of j
            const int vs = j & 1;
            if (!mbar_wait_bounded(pfull, j & 1, kAWaitNs)) {
                record(a.status, 0x224);
                ok = false;
                break;
            }
            if (!mbar_wait_bounded(&vfull[vs], (j >> 1) & 1, kAWaitNs)) {
                record(a.status, 0x225);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sPh = smem_u32(smem + C::oP), sPl = sPh + C::kPBytes;
            const uint32_t sVh = smem_u32(smem + C::oV + vs * 2 * C::kVBytes), sVl = sVh + C::kVBytes;
#pragma unroll
            for (int kk = 0; kk < kAK / 16; kk++) {
                const uint32_t o = kk * 32;
                const uint64_t ph = sw128_kmajor_desc(sPh + o), pl = sw128_kmajor_desc(sPl + o);
                const uint64_t vh = sw128_kmajor_desc(sVh + o), vl = sw128_kmajor_desc(sVl + o);
                mma_bf16(dO, ph, vh, idO, (j | kk) != 0);
                mma_bf16(dO, ph, vl, idO, 1u);
                mma_bf16(dO, pl, vh, idO, 1u);
            }
            mma_commit(&vempty[vs]);
            mma_commit(pfree);
        }
        if (ok) mma_commit(ofull);
        // every MMA this thread issued has completed before TMEM is freed
        mma_commit(done);
        if (!mbar_wait_bounded(done, 0, kAWaitNs)) record(a.status, 0x226);
    } else if (warp >= 2) {
        // ------------------------------------------------ softmax + epilogue: thread = query row
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const int qpos = a.pos0 + q0 + r;  // this row's position (rows past T: never stored)
        const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16);
        const float k2 = a.k2;
        float m = -INFINITY, l = 0.0f;
        int sn = 0;
        bool ok = true;
        // the 64 scores of the next S buffer; false if the wait ran out
        auto load_s = [&](uint32_t (&v)[64]) -> bool {
            const int sb = sn & 1;
            bool w = mbar_wait_bounded(&sfull[sb], (sn >> 1) & 1, kAWaitNs);
            w = __all_sync(FULL_MASK, w);
            if (!w) {
                record(a.status, 0x321);
                return false;
            }
            tc_fence_after();
            tmem_ld_32x32b_x32(trow + sb * kAK, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            tmem_ld_32x32b_x32(trow + sb * kAK + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&sfree[sb]);
            sn++;
            return true;
        };
        // p = 2^(att k2 - m k2) as bf16 hi/lo rows of P for the P.V MMAs, and the row's
        // sum l of the f32 p in ascending position.  m is the row's running max, moved
        // only when a block's max exceeds it by more than 2^kRescale in p (p stays
        // below 2^kRescale): then O (in TMEM) and l are scaled by 2^((m_old - m) k2),
        // between the P.V MMAs of the previous block and those of this one.
        uint8_t* prow_h = smem + C::oP;
        uint8_t* prow_l = prow_h + C::kPBytes;
        for (int j = 0; ok && j < nblk; j++) {
            uint32_t v[64];
            if (!(ok = load_s(v))) break;
            const int lim = qpos - j * kAK;  // columns c <= lim are visible
            float bm = -INFINITY;
            if (lim >= kAK - 1) {
#pragma unroll
                for (int c = 0; c < 64; c++) bm = fmaxf(bm, __uint_as_float(v[c]));
            } else {
#pragma unroll
                for (int c = 0; c < 64; c++)
                    if (c <= lim) bm = fmaxf(bm, __uint_as_float(v[c]));
            }
            float alpha = 1.0f;
            const bool move = j == 0 ? true : (bm - m) * k2 > kRescale;
            if (move && bm > m) {
                if (j > 0) alpha = ex2_approx((m - bm) * k2);
                m = bm;
                l *= alpha;
            }
            const float mk = m * k2;
            uint32_t hw[32], lw[32];  // the row's P, packed bf16 pairs, before waiting for the P buffer
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const int c = 2 * i;
                const float p0 = c <= lim ? ex2_approx(fmaf(__uint_as_float(v[c]), k2, -mk)) : 0.0f;
                const float p1 = c + 1 <= lim ? ex2_approx(fmaf(__uint_as_float(v[c + 1]), k2, -mk)) : 0.0f;
                l += p0;
                l += p1;
                const __nv_bfloat162 hi = __floats2bfloat162_rn(p0, p1);
                const float2 hf = __bfloat1622float2(hi);
                const __nv_bfloat162 lo = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
                hw[i] = *reinterpret_cast<const uint32_t*>(&hi);
                lw[i] = *reinterpret_cast<const uint32_t*>(&lo);
            }
            if (j > 0) {  // the P.V MMAs of block j - 1 are done: P is free, O is stable
                bool w = mbar_wait_bounded(pfree, (j - 1) & 1, kAWaitNs);
                w = __all_sync(FULL_MASK, w);
                if (!w) {
                    record(a.status, 0x322);
                    ok = false;
                    break;
                }
                if (__any_sync(FULL_MASK, alpha != 1.0f)) {  // O *= alpha (1 on the rows that keep m)
                    tc_fence_after();
#pragma unroll 1
                    for (int c0 = 0; c0 < HD; c0 += 32) {
                        uint32_t o[32];
                        tmem_ld_32x32b_x32(trow + C::kOCol + c0, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st_32x32b_x32(trow + C::kOCol + c0, o);
                    }
                    tmem_st_wait();
                    tc_fence_before();
                }
            }
#pragma unroll
            for (int c8 = 0; c8 < 8; c8++) {
                const uint32_t off = sw128_offset(r, c8);
                *reinterpret_cast<uint4*>(prow_h + off) =
                    make_uint4(hw[4 * c8], hw[4 * c8 + 1], hw[4 * c8 + 2], hw[4 * c8 + 3]);
                *reinterpret_cast<uint4*>(prow_l + off) =
                    make_uint4(lw[4 * c8], lw[4 * c8 + 1], lw[4 * c8 + 2], lw[4 * c8 + 3]);
            }
            fence_proxy_async_smem();  // the generic-proxy writes, visible to the tensor cores
            mbar_arrive(pfull);
        }
        const float inv = 1.0f / l;
        if (ok) {
            bool w = mbar_wait_bounded(ofull, 0, kAWaitNs);
            w = __all_sync(FULL_MASK, w);
            if (!w) {
                record(a.status, 0x323);
            } else {
                tc_fence_after();
                const int t = q0 + r;
                float* orow = a.ao + (size_t)t * a.ld_ao + h * HD;
#pragma unroll
                for (int c0 = 0; c0 < HD; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld_32x32b_x32(trow + C::kOCol + c0, o);
                    tmem_ld_wait();
                    if (t < a.T) {
                        float4* dst = reinterpret_cast<float4*>(orow + c0);
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv, __uint_as_float(o[4 * i + 1]) * inv,
                                                 __uint_as_float(o[4 * i + 2]) * inv,
                                                 __uint_as_float(o[4 * i + 3]) * inv);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// q of every head of row t as bf16 hi / lo rows: qh, ql [T][nq]
__global__ void __launch_bounds__(256) split_q_rows_kernel(const float* __restrict__ qkv, int nqkv, int nq,
                                                           uint16_t* qh, uint16_t* ql) {
    const int t = blockIdx.x;
    const float* q = qkv + (size_t)t * nqkv;
    for (int j = threadIdx.x; j < nq; j += blockDim.x) {
        const float x = q[j];
        const __nv_bfloat16 hi = __float2bfloat16_rn(x);
        qh[(size_t)t * nq + j] = __bfloat16_as_ushort(hi);
        ql[(size_t)t * nq + j] = __bfloat16_as_ushort(__float2bfloat16_rn(x - __bfloat162float(hi)));
    }
}

// Cache positions [0, nk) of kv head blockIdx.y, 64 per CTA: k as bf16 hi / lo rows
// kh, kl [n_kv][nk][hd]; v transposed, vh, vl [n_kv][hd][ldv] (positions nk .. ldv
// of a row are zeros).
__global__ void __launch_bounds__(256) split_kv_t_kernel(const float* __restrict__ kc, const float* __restrict__ vc,
                                                         int ctx, int nk, int hd, int ldv, uint16_t* kh,
                                                         uint16_t* kl, uint16_t* vh, uint16_t* vl) {
    __shared__ float tile[kAK][128 + 1];
    const int g = blockIdx.y, p0 = blockIdx.x * kAK, hd4 = hd / 4;
    const float* ksrc = kc + (size_t)g * ctx * hd;
    const float* vsrc = vc + (size_t)g * ctx * hd;
    for (int i = threadIdx.x; i < kAK * hd4; i += blockDim.x) {  // float4 of position p, dims 4 d4 ..
        const int p = i / hd4, d = (i - p * hd4) * 4, pos = p0 + p;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (pos < nk) {
            const float4 k = *reinterpret_cast<const float4*>(ksrc + (size_t)pos * hd + d);
            const float ke[4] = {k.x, k.y, k.z, k.w};
            uint32_t hw[2], lw[2];
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const __nv_bfloat16 h0 = __float2bfloat16_rn(ke[2 * q]), h1 = __float2bfloat16_rn(ke[2 * q + 1]);
                const __nv_bfloat16 l0 = __float2bfloat16_rn(ke[2 * q] - __bfloat162float(h0));
                const __nv_bfloat16 l1 = __float2bfloat16_rn(ke[2 * q + 1] - __bfloat162float(h1));
                hw[q] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
                lw[q] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
            }
            const size_t o = ((size_t)g * nk + pos) * hd + d;
            *reinterpret_cast<uint2*>(kh + o) = make_uint2(hw[0], hw[1]);
            *reinterpret_cast<uint2*>(kl + o) = make_uint2(lw[0], lw[1]);
            v = *reinterpret_cast<const float4*>(vsrc + (size_t)pos * hd + d);
        }
        tile[p][d] = v.x;
        tile[p][d + 1] = v.y;
        tile[p][d + 2] = v.z;
        tile[p][d + 3] = v.w;
    }
    __syncthreads();
    constexpr int kP4 = kAK / 4;
    for (int i = threadIdx.x; i < hd * kP4; i += blockDim.x) {  // dim d, positions 4 p4 .. + 4
        const int d = i / kP4, p = (i - d * kP4) * 4, pos = p0 + p;
        if (pos >= ldv) continue;
        uint32_t hw[2], lw[2];
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const float x0 = tile[p + 2 * q][d], x1 = tile[p + 2 * q + 1][d];
            const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
            const __nv_bfloat16 l0 = __float2bfloat16_rn(x0 - __bfloat162float(h0));
            const __nv_bfloat16 l1 = __float2bfloat16_rn(x1 - __bfloat162float(h1));
            hw[q] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
            lw[q] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        }
        const size_t o = ((size_t)g * hd + d) * ldv + pos;
        *reinterpret_cast<uint2*>(vh + o) = make_uint2(hw[0], hw[1]);
        *reinterpret_cast<uint2*>(vl + o) = make_uint2(lw[0], lw[1]);
    }
}

size_t round1k(size_t b) { return (b + 1023) & ~size_t(1023); }

}  // namespace

size_t attn_tc_scratch_bytes(int T, int nq, int n_kv, int hd, int nk) {
    const size_t ldv = (size_t)((nk + kAK - 1) / kAK) * kAK;
    return 2 * round1k((size_t)T * nq * 2) + 2 * round1k((size_t)n_kv * nk * hd * 2) +
           2 * round1k((size_t)n_kv * hd * ldv * 2);
}

template <int HD>
static cudaError_t launch_hd(const CUtensorMap* maps, const AttnTcArgs& a, dim3 grid, cudaStream_t s) {
    using C = AttnCfg<HD>;
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attn_tc_kernel<HD><<<grid, kAThreads, C::kSmem, s>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], a);
    return cudaGetLastError();
}

cudaError_t launch_attn_tc(const float* qkv, int nqkv, int n_heads, int n_kv, int hd, const float* kc,
                           const float* vc, int ctx, int pos0, int T, void* scratch, size_t scratch_bytes, float* ao,
                           unsigned* status, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const int nq = n_heads * hd, nk = pos0 + T;
    if ((hd != 64 && hd != 128) || n_heads % n_kv || nk > ctx ||
        scratch_bytes < attn_tc_scratch_bytes(T, nq, n_kv, hd, nk) || (reinterpret_cast<uintptr_t>(scratch) & 255) ||
        (reinterpret_cast<uintptr_t>(ao) & 15))
        return cudaErrorInvalidValue;
    const int ldv = (nk + kAK - 1) / kAK * kAK;
    uint8_t* p = static_cast<uint8_t*>(scratch);
    uint16_t* qh = reinterpret_cast<uint16_t*>(p);
    uint16_t* ql = reinterpret_cast<uint16_t*>(p += round1k((size_t)T * nq * 2));
    uint16_t* kh = reinterpret_cast<uint16_t*>(p += round1k((size_t)T * nq * 2));
    uint16_t* kl = reinterpret_cast<uint16_t*>(p += round1k((size_t)n_kv * nk * hd * 2));
    uint16_t* vh = reinterpret_cast<uint16_t*>(p += round1k((size_t)n_kv * nk * hd * 2));
    uint16_t* vl = reinterpret_cast<uint16_t*>(p += round1k((size_t)n_kv * hd * ldv * 2));
    split_q_rows_kernel<<<T, 256, 0, s>>>(qkv, nqkv, nq, qh, ql);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    split_kv_t_kernel<<<dim3(ldv / kAK, n_kv), 256, 0, s>>>(kc, vc, ctx, nk, hd, ldv, kh, kl, vh, vl);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // Q rows [T][nq]; K [n_kv][nk][hd]; V^T [n_kv][hd][ldv]; 64-column boxes, 128-byte swizzle
    CUtensorMap maps[6];
    const uint64_t qd[2] = {(uint64_t)nq, (uint64_t)T}, qs[1] = {(uint64_t)nq * 2};
    const uint32_t qb[2] = {64, kAQ};
    const uint64_t kd[3] = {(uint64_t)hd, (uint64_t)nk, (uint64_t)n_kv};
    const uint64_t ks[2] = {(uint64_t)hd * 2, (uint64_t)nk * hd * 2};
    const uint32_t kb[3] = {64, kAK, 1};
    const uint64_t vd[3] = {(uint64_t)nk, (uint64_t)hd, (uint64_t)n_kv};
    const uint64_t vs[2] = {(uint64_t)ldv * 2, (uint64_t)hd * ldv * 2};
    const uint32_t vb[3] = {kAK, (uint32_t)hd, 1};
    if (!make_map_sw128(&maps[0], qh, 2, qd, qs, qb) || !make_map_sw128(&maps[1], ql, 2, qd, qs, qb) ||
        !make_map_sw128(&maps[2], kh, 3, kd, ks, kb) || !make_map_sw128(&maps[3], kl, 3, kd, ks, kb) ||
        !make_map_sw128(&maps[4], vh, 3, vd, vs, vb) || !make_map_sw128(&maps[5], vl, 3, vd, vs, vb))
        return cudaErrorNotSupported;
    AttnTcArgs a{T, pos0, nk, n_heads / n_kv, (1.0f / sqrtf((float)hd)) * 1.4426950408889634f, ao, nq, status};
    const dim3 grid(n_heads, (T + kAQ - 1) / kAQ);
    return hd == 128 ? launch_hd<128>(maps, a, grid, s) : launch_hd<64>(maps, a, grid, s);
}

void preload_attn_tc_kernels() {
    cudaFuncAttributes f;
    (void)cudaFuncGetAttributes(&f, attn_tc_kernel<64>);
    (void)cudaFuncGetAttributes(&f, attn_tc_kernel<128>);
    (void)cudaFuncGetAttributes(&f, split_q_rows_kernel);
    (void)cudaFuncGetAttributes(&f, split_kv_t_kernel);
    (void)cudaGetLastError();
}

}  // namespace rbt
