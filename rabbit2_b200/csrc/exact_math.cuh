// exact_math.cuh -- the two pieces of the reference's routing arithmetic that a
// GPU does not give for free, reproduced bit for bit:
//
//  * expf_ref(x): the host libm's expf.  The reference's softmax calls glibc's
//    expf (rabbit2.c:403), which since glibc 2.27 is Szabolcs Nagy's
//    table-plus-polynomial method from ARM optimized-routines: x * 32/ln2 is
//    split into an integer k and a remainder r (|r| <= 1/2) by adding the
//    1.5 * 2^52 rounding shift, 2^(k/32) comes from a 32-entry table of doubles
//    with the integer part of k/32 added into the exponent bits, and 2^(r/32) is
//    a degree-3 polynomial; everything is evaluated in double and rounded to
//    float once.  x86-64 glibc ships the same C source compiled twice, with and
//    without FMA contraction, and picks one at load time; the two differ on 2 of
//    the 2.24e9 floats in [-103.97, 88.72].  `fma` selects the contracted
//    evaluation; the host side probes which one its own libm resolved
//    (host_expf_fma()).  A correctly rounded exp differs from glibc's on 97,052
//    floats of the router's range (x <= 0), enough to swap near-tie experts.
//
//  * block_seq_sum(sq, n): the sequential f32 sum ((sq[0] + sq[1]) + sq[2]) + ...
//    of n non-negative floats -- the sum of squares of rmsnorm (rabbit2.c:394) --
//    computed by a whole CTA.  The dependent chain of n adds (about 4 us at
//    n = 2048) would sit on the critical path of every MoE block, so the CTA
//    reproduces its exact result in parallel:
//      1. P_i = sq[0] + ... + sq[i-1] by a block scan in f32 (all terms are
//         non-negative, so P_i is within 2^-19 of the real prefix sum);
//      2. the true running sum s_i of the chain is within i * 2^-24 * s_i of the
//         real prefix (each add rounds by at most 2^-24 of a sum <= s_i).
//         When that interval, and the one for s_i + sq[i], lie inside one binade
//         [2^e, 2^(e+1)), s_i is a multiple of q = 2^(e-23) and the add rounds
//         s_i + sq[i] to the nearest multiple of q: the increment is sq[i]
//         rounded to a multiple of q, known without s_i -- unless sq[i] is an odd
//         multiple of q/2 (a tie, resolved by the parity of s_i).  These exact
//         increments are summed as integers (a second block scan);
//      3. the first 32 adds (where the binade changes every few terms) run as
//         the plain chain in thread 0; every other add that is "sensitive" (near
//         a binade edge, or a tie) is replayed exactly, in order, by the same
//         thread: s_i is the last replayed sum plus the increments since (exact
//         in f32, see seq_replay), and the replayed add is a real __fadd_rn.
//    About 11 of the 2016 adds past the prefix are replayed for N(0,1) inputs
//    at n = 2048 (measured on a CPU model of these steps).  Non-finite or
//    near-overflow sums, and more than kSeqMaxSens sensitive adds, fall back to
//    the plain chain.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

// phase stamps of block_seq_sum (thread 0), for instrumented builds only
#ifndef RBT_SEQ_STAMP
#define RBT_SEQ_STAMP(i) \
    do {                 \
    } while (0)
#endif

namespace rbt {

// tab[i] = bits(2^(i/32) rounded to the nearest double) - (i << 47): adding
// k << 47 to tab[k mod 32] gives 2^(k/32) for any integer k.  Computed with
// 60-digit decimal arithmetic (tests/test_exact_math.py recomputes it).
static __constant__ uint64_t kExp2Tab32[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

// The method's constants: 32/ln2 (1/ln2 rounded to double, times 32), the
// round-to-integer shift, and the published minimax coefficients of 2^(r/32)
// (r^3, r^2 and r terms; the constant term is 1).
constexpr double kExpInvLn2N = 0x1.71547652b82fep+0 * 32.0;
constexpr double kExpShift = 0x1.8p+52;
constexpr double kExpC0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
constexpr double kExpC1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
constexpr double kExpC2 = 0x1.62e42ff0c52d6p-1 / 32.0;

// kShfl: the table entry comes from lane (k mod 32) of the warp, whose register
// tab_lane holds kExp2Tab32[lane] (expf_tab_lane(), loaded early): a shuffle in
// place of a divergent constant-memory read on the softmax's critical path.  All
// 32 lanes must then call it together.
template <bool kFma, bool kShfl>
__device__ __forceinline__ float expf_ref_t(float x, uint64_t tab_lane) {
    const double xd = (double)x;
    double kd, r;
    uint64_t ki;
    if (kFma) {
        kd = __fma_rn(kExpInvLn2N, xd, kExpShift);
        ki = (uint64_t)__double_as_longlong(kd);
        kd = __dsub_rn(kd, kExpShift);
        r = __fma_rn(kExpInvLn2N, xd, -kd);
    } else {
        const double z = __dmul_rn(kExpInvLn2N, xd);
        kd = __dadd_rn(z, kExpShift);
        ki = (uint64_t)__double_as_longlong(kd);
        kd = __dsub_rn(kd, kExpShift);
        r = __dsub_rn(z, kd);
    }
    uint64_t tk;
    if (kShfl) tk = __shfl_sync(0xffffffffu, tab_lane, (int)(ki & 31u));
    else tk = kExp2Tab32[ki & 31u];
    const double s = __longlong_as_double((long long)(tk + (ki << 47)));
    double y;
    if (kFma) {
        const double z = __fma_rn(kExpC0, r, kExpC1);
        const double r2 = __dmul_rn(r, r);
        y = __fma_rn(kExpC2, r, 1.0);
        y = __fma_rn(z, r2, y);
    } else {
        const double z = __dadd_rn(__dmul_rn(kExpC0, r), kExpC1);
        const double r2 = __dmul_rn(r, r);
        y = __dadd_rn(__dmul_rn(kExpC2, r), 1.0);
        y = __dadd_rn(__dmul_rn(z, r2), y);
    }
    float res = __double2float_rn(__dmul_rn(y, s));
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {                                   // |x| >= 88, inf or nan
        if (ux == 0xff800000u) res = 0.0f;                    // -inf
        else if (abstop >= 0x7f8u) res = x + x;               // +inf, nan
        else if (x > 0x1.62e42ep6f) res = __int_as_float(0x7f800000);  // overflows
        else if (x < -0x1.9fe368p6f) res = 0.0f;              // underflows to zero
    }
    return res;
}

__device__ __forceinline__ float expf_ref(float x, int fma) {
    return fma ? expf_ref_t<true, false>(x, 0) : expf_ref_t<false, false>(x, 0);
}
__device__ __forceinline__ uint64_t expf_tab_lane() { return kExp2Tab32[threadIdx.x & 31]; }
// warp-collective form (see expf_ref_t)
__device__ __forceinline__ float expf_ref_warp(float x, int fma, uint64_t tab_lane) {
    return fma ? expf_ref_t<true, true>(x, tab_lane) : expf_ref_t<false, true>(x, tab_lane);
}

// silu(x) = x / (1 + expf(-x)) (rabbit2.c:407) with the host's expf.
__device__ __forceinline__ float silu_ref(float x, int fma) {
    return __fdiv_rn(x, __fadd_rn(1.0f, expf_ref(-x, fma)));
}

// ---------------------------------------------------------------- sequential sum
constexpr int kSeqMaxSens = 256;  // replayed adds beyond the prefix; more fall back to the plain chain
constexpr int kSeqPrefix = 32;    // the first terms, summed by thread 0 as the plain chain

struct SeqSumSmem {
    float w_p[32];              // per-warp totals of the first scan
    long long w_s[32];          // and of the second
    int w_c[32];
    float result;
    float sens_a[kSeqMaxSens];  // replayed adds, ascending index: the term
    long long sens_ss[kSeqMaxSens];  // and the known increments before it (units of 2^(e_top - 60))
};

// Block-wide exclusive scan of non-negative floats over NT threads in thread
// order, with the total.  Exclusive values are sums of the inputs before them,
// never formed by a subtraction, so each carries a relative error below
// 2^-24 per add on its path (at most 5 + NT/32 + 1 adds).
template <int NT>
__device__ __forceinline__ float seq_scan_f(float v, float* w, float& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc = __fadd_rn(inc, y);
    }
    float exc = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) exc = 0.0f;
    if (lane == 31) w[warp] = inc;
    __syncthreads();
    float base = 0.0f, all = 0.0f;
#pragma unroll
    for (int k = 0; k < NT / 32; k++) {
        const float t = w[k];
        if (k < warp) base = __fadd_rn(base, t);
        all = __fadd_rn(all, t);
    }
    total = all;
    return __fadd_rn(base, exc);
}

// Exact block-wide exclusive scan of (int64, int) with the totals.
template <int NT>
__device__ __forceinline__ long long seq_scan_li(long long vd, int vi, SeqSumSmem& s, long long& td, int& ti,
                                                 int& ei) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    long long incd = vd;
    int inci = vi;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long yd = __shfl_up_sync(0xffffffffu, incd, o);
        const int yi = __shfl_up_sync(0xffffffffu, inci, o);
        if (lane >= o) {
            incd += yd;
            inci += yi;
        }
    }
    if (lane == 31) {
        s.w_s[warp] = incd;
        s.w_c[warp] = inci;
    }
    __syncthreads();
    long long based = 0, alld = 0;
    int basei = 0, alli = 0;
#pragma unroll
    for (int k = 0; k < NT / 32; k++) {
        const long long t = s.w_s[k];
        const int c = s.w_c[k];
        if (k < warp) {
            based += t;
            basei += c;
        }
        alld += t;
        alli += c;
    }
    td = alld;
    ti = alli;
    ei = basei + inci - vi;
    return based + incd - vd;
}

// Step classification (2. above), in integer arithmetic on float bit patterns and
// without branches.  P: the f32 prefix before term i (within 2^-19 of the real
// prefix sum), a > 0 the term, e_top the binade of the total.  Returns true when
// the add must be replayed; otherwise *inc is its exact increment in units of
// 2^(e_top - 60).  The margins, in units of 2^-23 relative: (i + 1) for the
// chain's own rounding (|s_i - real prefix| <= i * 2^-24 * s_i), 64 for the f32
// prefix, and a few more.
__device__ __forceinline__ bool seq_step_sensitive(float P, float a, int i, int e_top, long long* inc) {
    const uint32_t up = __float_as_uint(P);
    const int e = (int)(up >> 23) - 127;
    const uint32_t M = up & 0x7fffffu;
    const uint32_t slack = (uint32_t)(i + 1) + 64u + (uint32_t)(((long long)(i + 1) * (i + 1)) >> 22) + 2u;
    const uint32_t uq = __float_as_uint(__fadd_rn(P, a));
    const uint32_t ua = __float_as_uint(a);
    const int eb = (int)(ua >> 23);
    const uint32_t ma = eb ? ((ua & 0x7fffffu) | 0x800000u) : (ua & 0x7fffffu);
    // a / q = ma * 2^-shift, q = 2^(e - 23); clamped: 0 (a is a multiple of q) .. 25 (a < q / 2)
    const int sh = min(max(e - (eb ? eb - 127 : -126), 0), 25);
    const uint32_t half = sh ? 1u << (sh - 1) : 0u;
    const uint32_t low = ma & ((1u << sh) - 1u);
    const uint32_t k = (ma >> sh) + (low > half ? 1u : 0u);
    const int scale = e - e_top + 37;
    const bool sens = !(P >= 0x1p-125f)                                   // empty or subnormal prefix
                      | (M < slack)                                       // s_i may lie in the binade below
                      | ((int)(uq >> 23) - 127 != e)                      // s_i + a may reach the binade above
                      | ((uq & 0x7fffffu) + 1u + 2u * slack >= (1u << 23))
                      | (e > 125) | (scale < 0)                           // near overflow, below the unit
                      | (sh > 0 && low == half);                          // a tie: the parity of s_i decides
    *inc = sens ? 0ll : (long long)k << (scale < 0 ? 0 : scale);
    return sens;
}

// Thread 0's replay of the sensitive adds in index order (3. above), from the
// prefix sum s_pre; returns the final sum.  Between two replayed adds the running
// sum stays inside one binade (a step that could leave it is itself replayed), so
// the known increments D since the last replayed add sum to less than that
// binade's lower edge, on its grid: D has at most 23 significant bits, is exact as
// a float, and s_i = acc + D rounds to itself.  The chain is then two f32 adds
// per replayed term; the differences D are formed before it.
__device__ __forceinline__ float seq_replay(const SeqSumSmem& s, int ctot, float s_pre, long long SStot, float u) {
    float acc = s_pre;
    long long prev = 0;  // the prefix terms contribute no known increments
    int k = 0;
    for (; k + 4 <= ctot; k += 4) {
        float d[4], a[4];
#pragma unroll
        for (int v = 0; v < 4; v++) {
            const long long ss = s.sens_ss[k + v];
            d[v] = __fmul_rn(__ll2float_rn(ss - prev), u);
            a[v] = s.sens_a[k + v];
            prev = ss;
        }
#pragma unroll
        for (int v = 0; v < 4; v++) acc = __fadd_rn(__fadd_rn(acc, d[v]), a[v]);
    }
    for (; k < ctot; k++) {
        const long long ss = s.sens_ss[k];
        acc = __fadd_rn(__fadd_rn(acc, __fmul_rn(__ll2float_rn(ss - prev), u)), s.sens_a[k]);
        prev = ss;
    }
    return __fadd_rn(acc, __fmul_rn(__ll2float_rn(SStot - prev), u));
}

// Thread 0: the plain chain over the first np terms (np <= kSeqPrefix).
__device__ __forceinline__ float seq_prefix(const float* sq, int np) {
    float r = 0.0f;
    if (np == kSeqPrefix && (reinterpret_cast<uintptr_t>(sq) & 15u) == 0) {
        float4 v[kSeqPrefix / 4];  // the loads first, then the dependent adds
#pragma unroll
        for (int k = 0; k < kSeqPrefix / 4; k++) v[k] = reinterpret_cast<const float4*>(sq)[k];
#pragma unroll
        for (int k = 0; k < kSeqPrefix / 4; k++) {
            r = __fadd_rn(r, v[k].x);
            r = __fadd_rn(r, v[k].y);
            r = __fadd_rn(r, v[k].z);
            r = __fadd_rn(r, v[k].w);
        }
    } else {
        for (int i = 0; i < np; i++) r = __fadd_rn(r, sq[i]);
    }
    return r;
}

// The unit of the known increments: 2^(e_top - 60), e_top the binade of the total.
__device__ __forceinline__ int seq_e_top(float Ptot) {
    return Ptot >= 0x1p-125f ? (int)(__float_as_uint(Ptot) >> 23) - 127 : -126;
}
// The fast path needs a finite total below 2^125 and a unit 2^(e_top - 60) that is
// a normal float (totals of at least 2^-66).
__device__ __forceinline__ bool seq_fast_ok(float Ptot, int ctot) {
    return ctot <= kSeqMaxSens && isfinite(Ptot) && Ptot < 0x1p125f && Ptot >= 0x1p-66f;
}
__device__ __forceinline__ float seq_unit(int e_top) { return __int_as_float((e_top - 60 + 127) << 23); }

// The sequential f32 sum of sq[0..n) (non-negative floats in shared memory, 16-byte
// aligned), by all NT threads of the CTA; every thread gets the result.  Thread t
// owns terms [t*L, t*L + L) in registers; n <= NT * L.
template <int NT, int L>
__device__ float block_seq_sum_l(const float* sq, int n, SeqSumSmem& s) {
    static_assert(NT % 32 == 0 && NT <= 1024 && (L % 4 == 0 || L == 1) && L <= 8, "whole warps, float4 runs");
    const int tid = threadIdx.x;
    const int i0 = tid * L;
    float a[L];
#pragma unroll
    for (int j = 0; j < L; j++) a[j] = 0.0f;
    if (L % 4 == 0 && i0 + L <= n) {
#pragma unroll
        for (int j = 0; j < L; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(sq + i0 + j);
            a[j] = v.x;
            a[j + 1] = v.y;
            a[j + 2] = v.z;
            a[j + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < L; j++)
            if (i0 + j < n) a[j] = sq[i0 + j];
    }
    // thread 0: the first terms as the plain chain (most of the binade changes)
    const int np = n < kSeqPrefix ? n : kSeqPrefix;
    float s_pre = 0.0f;
    if (tid == 0) {
        s_pre = seq_prefix(sq, np);
        RBT_SEQ_STAMP(0);
    }
    float c[L];  // inclusive local prefix
    float run = 0.0f;
#pragma unroll
    for (int j = 0; j < L; j++) {
        run = __fadd_rn(run, a[j]);
        c[j] = run;
    }
    float Ptot;
    const float P0 = seq_scan_f<NT>(run, s.w_p, Ptot);
    if (tid == 0) RBT_SEQ_STAMP(1);
    const int e_top = seq_e_top(Ptot);
    long long r[L];
    unsigned sens = 0;
    long long rsum = 0;
#pragma unroll
    for (int j = 0; j < L; j++) {
        const int i = i0 + j;
        r[j] = 0;
        if (i >= np && i < n && a[j] != 0.0f) {
            const float P = j == 0 ? P0 : __fadd_rn(P0, c[j - 1]);
            if (seq_step_sensitive(P, a[j], i, e_top, &r[j])) sens |= 1u << j;
        }
        rsum += r[j];
    }
    if (tid == 0) RBT_SEQ_STAMP(2);
    long long SStot;
    int ctot, c0;
    const long long SS0 = seq_scan_li<NT>(rsum, __popc(sens), s, SStot, ctot, c0);
    if (tid == 0) RBT_SEQ_STAMP(3);
    const bool fast = seq_fast_ok(Ptot, ctot);
    if (fast && sens) {
        long long ss = SS0;
        int k = c0;
#pragma unroll
        for (int j = 0; j < L; j++) {
            if ((sens >> j) & 1u) {
                s.sens_a[k] = a[j];
                s.sens_ss[k] = ss;
                k++;
            }
            ss += r[j];
        }
    }
    __syncthreads();
    if (tid == 0) {
        RBT_SEQ_STAMP(4);
        float res;
        if (fast) {
            res = seq_replay(s, ctot, s_pre, SStot, seq_unit(e_top));
        } else {
            res = s_pre;
            for (int i = np; i < n; i++) res = __fadd_rn(res, sq[i]);
        }
        s.result = res;
        RBT_SEQ_STAMP(5);
    }
    __syncthreads();
    return s.result;
}

// Long rows (n > NT * 8): the same steps with runs of L = ceil(n / NT) terms read
// from shared memory in each pass instead of held in registers.
template <int NT>
__device__ float block_seq_sum_long(const float* sq, int n, SeqSumSmem& s) {
    const int tid = threadIdx.x;
    const int L = (n + NT - 1) / NT;
    const int i0 = min(tid * L, n), i1 = min(i0 + L, n);
    const int np = n < kSeqPrefix ? n : kSeqPrefix;
    float s_pre = 0.0f;
    if (tid == 0) s_pre = seq_prefix(sq, np);
    float run = 0.0f;
    for (int i = i0; i < i1; i++) run = __fadd_rn(run, sq[i]);
    float Ptot;
    const float P0 = seq_scan_f<NT>(run, s.w_p, Ptot);
    const int e_top = seq_e_top(Ptot);
    long long rsum = 0;
    int ns = 0;
    float P = P0;
    for (int i = i0; i < i1; i++) {
        const float a = sq[i];
        long long inc = 0;
        if (i >= np && a != 0.0f && seq_step_sensitive(P, a, i, e_top, &inc)) ns++;
        rsum += inc;
        P = __fadd_rn(P, a);
    }
    long long SStot;
    int ctot, c0;
    const long long SS0 = seq_scan_li<NT>(rsum, ns, s, SStot, ctot, c0);
    const bool fast = seq_fast_ok(Ptot, ctot);
    if (fast && ns > 0) {
        long long ss = SS0;
        int k = c0;
        P = P0;
        for (int i = i0; i < i1; i++) {
            const float a = sq[i];
            long long inc = 0;
            if (i >= np && a != 0.0f && seq_step_sensitive(P, a, i, e_top, &inc)) {
                s.sens_a[k] = a;
                s.sens_ss[k] = ss;
                k++;
            }
            ss += inc;
            P = __fadd_rn(P, a);
        }
    }
    __syncthreads();
    if (tid == 0) {
        float res;
        if (fast) {
            res = seq_replay(s, ctot, s_pre, SStot, seq_unit(e_top));
        } else {
            res = s_pre;
            for (int i = np; i < n; i++) res = __fadd_rn(res, sq[i]);
        }
        s.result = res;
    }
    __syncthreads();
    return s.result;
}

// Runtime n: register runs up to 8 terms per thread, shared-memory runs beyond.
template <int NT>
__device__ float block_seq_sum(const float* sq, int n, SeqSumSmem& s) {
    if (n <= NT) return block_seq_sum_l<NT, 1>(sq, n, s);
    if (n <= NT * 4) return block_seq_sum_l<NT, 4>(sq, n, s);
    if (n <= NT * 8) return block_seq_sum_l<NT, 8>(sq, n, s);
    return block_seq_sum_long<NT>(sq, n, s);
}

}  // namespace rbt
