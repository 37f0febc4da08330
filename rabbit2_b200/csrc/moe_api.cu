// moe_api.cu -- the C ABI of librbt_moe.so (include/rbt_moe.h): context,
// HBM-resident expert weights, workspace, and the per-call launch sequence
//
//   [rmsnorm] -> router/top-k/permute (K1) -> gate-up (K3|K4) -> down (K3|K4)
//   -> combine + residual (K5)
//
// Replaces, in the reference engine, the MoE block of forward()
// (rabbit2.c:511-542), the CPU matvec kernels it calls (:323-390) and the
// expert fetch seam get_expert()/ExpertCache (:83-94, :236-300).
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <new>
#include <vector>

#include "../../include/rbt_moe.h"
#include "kernels.h"

namespace rbt {
int router_token_tiles(int T);
}

namespace {

thread_local char g_err[512] = "";

int fail(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    fprintf(stderr, "rbt_moe: %s\n", g_err);
    return 0;
}

}  // namespace

namespace rbt {
// Sets the calling thread's rbt_moe_last_error() text (used by the entry points
// defined in other files of the library).
void set_last_error(const char* msg) { snprintf(g_err, sizeof g_err, "%s", msg); }
}  // namespace rbt

namespace {

#define CU(call)                                                                                  \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) return fail("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                           __FILE__, __LINE__);                                   \
    } while (0)

struct Layer {
    const float* ffn_norm = nullptr;
    const void* router = nullptr;
    const uint8_t* experts = nullptr;
    float* bias = nullptr;        // device [E] or null
    void* owned = nullptr;        // allocation made by rbt_moe_load_layer
    bool tc = false;              // tensor maps below are valid
    CUtensorMap w_gateup;         // [E][2H][D] bf16 rows (w1 then w3), 3-D
    CUtensorMap w_down;           // [E][D][H] bf16 rows (w2), 3-D
    bool dec = false;             // w2_cols is valid
    CUtensorMap w2_cols;          // w2 column tiles of the one-token kernel
    void* w2t = nullptr;          // [E][H][D] transposed w2 for the one-token kernel, owned (or null)
    void* w16 = nullptr;          // [E][2H][D] fp16 copy of w1|w3 for the fp16 gate/up GEMM, owned (or null)
    void* router_cm = nullptr;    // [E*D] bf16 chain-major copy of the router for the token router, owned (or null)
    CUtensorMap w_gateup16;       // its 3-D map (valid when w16 is set)
};

struct Workspace {
    int cap = 0;                  // tokens per call the buffers hold
    void* block = nullptr;
    float *xb, *logits, *wt, *h, *y, *hx, *hout, *partials, *bscale;
    int32_t *idx, *counts, *offsets, *perm, *slot_pos, *active, *n_active, *hrouting;
    int32_t *tile_cnt, *tile_base, *slot_rank;
    unsigned *tile_counter, *done_counter, *status, *gbar;
    // tcgen05 path: split-bf16 operands in expert order and the token-block list
    void *xhi, *xlo, *hhi, *hlo;
    int32_t *tb_e, *tb_p0, *tb_p1, *n_tb;
    bool tc_maps = false;
    CUtensorMap m_xhi[3], m_xlo[3], m_hhi[3], m_hlo[3];  // token-tile widths 32, 64, 128
    // host-pointer block calls of up to kStageTokens tokens: hx, hrouting and status are
    // one span of the block, returned by ONE copy into this pinned staging
    void* pinned = nullptr;
    size_t span = 0;              // bytes from hx to the end of status
};
constexpr int kStageTokens = 128;
// expert parallelism: received slots up to which the streaming GEMV beats the tensor cores
constexpr int kEpStreamSlots = 128;

}  // namespace

struct StageMark {
    int stage, ev_begin, ev_end;  // indices into the event pool
};

// Expert parallelism (rbt_moe_ep_*): this GPU's exported block of receive and
// return segments and flags, its local plan buffers, and every GPU's pointers.
struct EpState {
    int R = 0, rank = 0, epr = 0, cap = 0;
    void* block = nullptr;         // exported (IPC) or peer-read block
    size_t block_bytes = 0;
    size_t off_rows = 0, off_idx = 0, off_wt = 0, off_count = 0, off_fdisp = 0, off_back = 0, off_fret = 0;
    void* local = nullptr;         // pos [cap][R], counts [R], epoch, tickets
    int32_t *pos = nullptr, *counts = nullptr;
    unsigned long long* epoch = nullptr;
    unsigned* done = nullptr;
    rbt::EpPeers peers{};
    std::vector<void*> opened;     // peer blocks opened from IPC handles
    bool connected = false;
    unsigned long long timeout_ns = 2000000000ull;
};

struct RbtMoe {
    RbtMoeConfig cfg;
    bool timing = false;
    RbtMoeProfile prof{};
    std::vector<cudaEvent_t> ev_pool;  // timing events, created when timing is switched on
    int ev_used = 0;
    std::vector<StageMark> marks;      // stage intervals recorded since the last reset
    int device = 0;
    int sm_count = 0;
    int path = 0;
    int gemm_min_tokens = 2;   // automatic path: tensor-core GEMM from this many tokens (one token: fused decode)
    size_t esz = 2;
    int e0 = 0;                // expert parallelism: this context holds experts [e0, e0 + n_local)
    int n_local = 0;           // == cfg.n_experts unless rbt_moe_set_expert_range narrowed it
    cudaStream_t stream = nullptr;
    std::vector<Layer> layers;
    Workspace ws;
    unsigned long long ws_gen = 0;  // workspace allocations so far
    unsigned* h_status = nullptr;   // pinned host copy of the status word (host-pointer calls)
    int last_routed = 0;            // tokens the most recent routed call computed logits for
    unsigned long long peer_wait_ns = 0;  // the one-token kernel's bound on waits for other CTAs (0: 2 s)
    EpState ep;
};

namespace {

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int set_device(RbtMoe* m) {
    CU(cudaSetDevice(m->device));
    return 1;
}

// Grow the workspace to hold `T` tokens (allocates; not legal during capture).
int reserve(RbtMoe* m, int T) {
    if (T <= m->ws.cap) return 1;
    const RbtMoeConfig& c = m->cfg;
    const size_t D = c.dim, E = c.n_experts, K = c.top_k, H = c.expert_hidden, S = (size_t)T * K;
    const size_t tiles = (size_t)rbt::router_token_tiles(T) + 1;
    const size_t ntb = S / 32 + E + 1;  // token blocks at the narrowest tile width
    const bool tc = rbt::tc_supported(c.dim, c.expert_hidden, c.dtype);
    // split-bf16 operand rows: at least one full 128-row TMA box, whole boxes
    const size_t SB = tc ? ((S > 128 ? S : 128) + 127) / 128 * 128 : 0;
    struct Part { void** p; size_t bytes; };
    Workspace w;
    w.cap = T;
    std::vector<Part> parts = {
        {(void**)&w.xhi, SB * D * 2},            {(void**)&w.xlo, SB * D * 2},
        {(void**)&w.hhi, SB * H * 2},            {(void**)&w.hlo, SB * H * 2},
        {(void**)&w.tb_e, ntb * 4},              {(void**)&w.tb_p0, ntb * 4},
        {(void**)&w.tb_p1, ntb * 4},             {(void**)&w.n_tb, 4},
        {(void**)&w.gbar, (size_t)rbt::decode_sync_words((int)E, (int)K) * 4},
        // (the token router keeps one 64-bit expert mask per token in tile_cnt)
        {(void**)&w.tile_cnt, std::max(tiles * E * 4, (size_t)T * 8)}, {(void**)&w.tile_base, tiles * E * 4},
        {(void**)&w.slot_rank, S * 4},
        {(void**)&w.xb, (size_t)T * D * 4},      {(void**)&w.logits, (size_t)T * E * 4},
        {(void**)&w.wt, S * 4},                  {(void**)&w.h, S * H * 4},
        {(void**)&w.y, S * D * 4},
        {(void**)&w.hout, (size_t)T * D * 4},    {(void**)&w.idx, S * 4},
        {(void**)&w.counts, E * 4},              {(void**)&w.offsets, (E + 1) * 4},
        {(void**)&w.perm, S * 4},                {(void**)&w.slot_pos, S * 4},
        {(void**)&w.active, E * 4},              {(void**)&w.n_active, 4},
        {(void**)&w.tile_counter, tiles * 4},
        {(void**)&w.done_counter, 4},
        {(void**)&w.partials, rbt::decode_partials_bytes(m->sm_count, (int)D)},
        {(void**)&w.bscale, (SB > 0 ? SB : 1) * 4},
        // last, in this order: the one span a small host-pointer block call returns
        {(void**)&w.hx, (size_t)T * D * 4},      {(void**)&w.hrouting, S * 4},
        {(void**)&w.status, 4},
    };
    size_t total = 0;
    for (auto& p : parts) total = align_up(total, 256) + p.bytes;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    CU(cudaStreamIsCapturing(m->stream, &cs));
    if (cs != cudaStreamCaptureStatusNone)
        return fail("workspace for %d tokens must be reserved before stream capture (rbt_moe_reserve)", T);
    void* block = nullptr;
    CU(cudaMalloc(&block, total));
    size_t off = 0;
    for (auto& p : parts) {
        off = align_up(off, 256);
        *p.p = (char*)block + off;
        off += p.bytes;
    }
    // counters must start at zero; the kernels return them to zero after use
    CU(cudaMemsetAsync(w.tile_counter, 0, tiles * 4, m->stream));
    CU(cudaMemsetAsync(w.done_counter, 0, 4, m->stream));
    CU(cudaMemsetAsync(w.counts, 0, E * 4, m->stream));
    CU(cudaMemsetAsync(w.status, 0, 4, m->stream));
    CU(cudaMemsetAsync(w.gbar, 0, (size_t)rbt::decode_sync_words((int)E, (int)K) * 4, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    if (tc) {
        w.tc_maps = true;
        for (int i = 0; i < 3; i++) {
            const int bn = 32 << i;
            w.tc_maps = w.tc_maps && rbt::make_map_2d(&w.m_xhi[i], w.xhi, c.dim, (long)SB, bn) &&
                        rbt::make_map_2d(&w.m_xlo[i], w.xlo, c.dim, (long)SB, bn) &&
                        rbt::make_map_2d(&w.m_hhi[i], w.hhi, c.expert_hidden, (long)SB, bn) &&
                        rbt::make_map_2d(&w.m_hlo[i], w.hlo, c.expert_hidden, (long)SB, bn);
        }
    }
    w.span = (size_t)((char*)w.status - (char*)w.hx) + 4;
    if (T <= kStageTokens && cudaMallocHost(&w.pinned, w.span) != cudaSuccess) {
        (void)cudaGetLastError();
        w.pinned = nullptr;  // the calls then use one copy per output
    }
    if (m->ws.block) CU(cudaFree(m->ws.block));
    if (m->ws.pinned) cudaFreeHost(m->ws.pinned);
    w.block = block;
    m->ws = w;
    m->ws_gen++;  // captured graphs that use the old workspace are stale now
    return 1;
}

// RBT_MOE_TC_F16=1 (read when a layer is bound or loaded): the gate/up GEMM runs
// one fp16 MMA per K step on an fp16 copy of w1|w3 (+2*H*D*2 bytes per expert)
// with fp16 activations, ~3e-4 relative error on the OLMoE layer, 10-20% faster;
// by default it keeps the split-bf16 activations (two MMAs per K step, ~1e-5).
bool tc_f16_enabled() {
    const char* v = getenv("RBT_MOE_TC_F16");
    return v && v[0] == '1';
}

// RBT_MOE_DECODE_W2T=0: no transposed w2 copy (the one-token kernel then reads w2 as column tiles)
bool decode_w2t_enabled() {
    const char* v = getenv("RBT_MOE_DECODE_W2T");
    return !(v && v[0] == '0');
}

// Tensor maps of the layer's expert blobs for the tcgen05 path (bf16 only), and
// the one-token kernel's w2 map and transposed w2.
void layer_maps(RbtMoe* m, Layer& L) {
    const RbtMoeConfig& c = m->cfg;
    L.tc = false;
    if (L.w16) cudaFree(L.w16);
    L.w16 = nullptr;
    // the token router (2..256 tokens) reads the router in chain-major order: a
    // copy of E*D*2 bytes (256 KB at OLMoE), made once per binding
    if (L.router_cm) cudaFree(L.router_cm);
    L.router_cm = nullptr;
    if (L.router && rbt::router_chain_major_supported(c.n_experts, c.dim, c.dtype)) {
        void* p = nullptr;
        bool ok = cudaMalloc(&p, (size_t)c.n_experts * c.dim * 2) == cudaSuccess;
        // the router may still be in flight on another stream of the caller
        ok = ok && cudaDeviceSynchronize() == cudaSuccess &&
             rbt::router_to_chain_major(L.router, c.n_experts, c.dim, p, m->stream) == cudaSuccess &&
             cudaStreamSynchronize(m->stream) == cudaSuccess;
        if (ok) {
            L.router_cm = p;
        } else {  // without the copy the other router kernels run
            (void)cudaGetLastError();
            if (p) cudaFree(p);
        }
    }
    L.dec = m->n_local == c.n_experts && c.dtype == 1 && (c.expert_stride % 16) == 0 &&
            (reinterpret_cast<uintptr_t>(L.experts) % 16) == 0 &&
            (c.expert_hidden % 8) == 0 && c.dim <= 2048 &&
            rbt::make_decode_w2_map(&L.w2_cols, L.experts, c.dim, c.expert_hidden, c.n_experts, c.expert_stride);
    // the one-token kernel streams w2 fastest as rows of its transpose: one
    // contiguous run per unit instead of a tile of 16-byte pieces
    if (L.w2t) cudaFree(L.w2t);
    L.w2t = nullptr;
    if (L.dec && decode_w2t_enabled()) {
        const size_t bytes = (size_t)c.n_experts * c.expert_hidden * c.dim * 2;
        void* p = nullptr;
        bool ok = cudaMalloc(&p, bytes) == cudaSuccess;
        // the weights may still be in flight on another stream of the caller
        ok = ok && cudaDeviceSynchronize() == cudaSuccess &&
             rbt::transpose_w2(L.experts, c.expert_stride, c.dim, c.expert_hidden, c.n_experts, p, m->stream) ==
                 cudaSuccess &&
             cudaStreamSynchronize(m->stream) == cudaSuccess;
        if (ok) {
            L.w2t = p;
        } else {  // without the copy the kernel reads w2 as column tiles
            (void)cudaGetLastError();
            if (p) cudaFree(p);
        }
    }
    if (!rbt::tc_supported(c.dim, c.expert_hidden, c.dtype) || (c.expert_stride % 16) != 0 ||
        (reinterpret_cast<uintptr_t>(L.experts) % 16) != 0)
        return;
    L.tc = rbt::make_map_experts(&L.w_gateup, L.experts, c.dim, 2 * c.expert_hidden, m->n_local,
                                 c.expert_stride) &&
           rbt::make_map_experts(&L.w_down, L.experts + (size_t)2 * c.expert_hidden * c.dim * 2, c.expert_hidden,
                                 c.dim, m->n_local, c.expert_stride);
    if (L.tc && tc_f16_enabled()) {
        // fp16 copy of w1|w3; kept only if every value fits fp16
        const size_t per = (size_t)2 * c.expert_hidden * c.dim * 2;
        void* p = nullptr;
        unsigned* flag = nullptr;
        unsigned over = 1;
        bool ok = cudaMalloc(&p, per * m->n_local) == cudaSuccess && cudaMalloc(&flag, 4) == cudaSuccess &&
                  cudaMemset(flag, 0, 4) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
                  rbt::convert_gateup_f16(L.experts, c.expert_stride, c.dim, c.expert_hidden, m->n_local, p, flag,
                                          m->stream) == cudaSuccess &&
                  cudaMemcpyAsync(&over, flag, 4, cudaMemcpyDeviceToHost, m->stream) == cudaSuccess &&
                  cudaStreamSynchronize(m->stream) == cudaSuccess && over == 0 &&
                  rbt::make_map_experts(&L.w_gateup16, p, c.dim, 2 * c.expert_hidden, m->n_local, per);
        if (flag) cudaFree(flag);
        if (ok) {
            L.w16 = p;
        } else {  // without it the gate/up GEMM uses the split-bf16 activations
            (void)cudaGetLastError();
            if (p) cudaFree(p);
        }
    }
}

int check_layer(RbtMoe* m, int layer, bool need_norm) {
    if (!m) return fail("null context");
    if (layer < 0 || layer >= m->cfg.n_layers) return fail("layer %d out of range [0, %d)", layer, m->cfg.n_layers);
    const Layer& L = m->layers[layer];
    if (!L.router || !L.experts) return fail("layer %d has no weights (rbt_moe_load_layer / rbt_moe_bind_layer)", layer);
    if (need_norm && !L.ffn_norm) return fail("layer %d has no ffn_norm (needed by the block form)", layer);
    return 1;
}

// Stage bookkeeping: count every launch; with timing on, record an event at
// every stage boundary on the launching stream (cudaEventRecordExternal, so the
// records become graph nodes under stream capture).  Nothing waits here; the
// intervals are read by rbt_moe_profile.
struct StageClock {
    RbtMoe* m;
    cudaStream_t s;
    int open_stage = -1;
    int open_ev = -1;
    int mark() {
        if (m->ev_used >= (int)m->ev_pool.size()) return -1;  // pool exhausted: stop recording
        const int i = m->ev_used++;
        if (cudaEventRecordWithFlags(m->ev_pool[i], s, cudaEventRecordExternal) != cudaSuccess) return -1;
        return i;
    }
    int begin(int stage) {
        m->prof.launches++;
        m->prof.stage_launches[stage]++;
        if (!m->timing) return 1;
        const int e = mark();
        if (open_stage >= 0 && open_ev >= 0 && e >= 0) m->marks.push_back({open_stage, open_ev, e});
        open_stage = stage;
        open_ev = e;
        return 1;
    }
    int end() {
        if (!m->timing || open_stage < 0) return 1;
        const int e = mark();
        if (open_ev >= 0 && e >= 0) m->marks.push_back({open_stage, open_ev, e});
        open_stage = -1;
        return 1;
    }
};

rbt::StreamArgs sa_of(RbtMoe* m, const Layer& L, const float* xb, const float* x, float* out, int T, bool block) {
    const RbtMoeConfig& c = m->cfg;
    const Workspace& w = m->ws;
    rbt::StreamArgs a{};
    a.xb = xb; a.resid = block ? x : nullptr; a.out = block ? const_cast<float*>(x) : out;
    a.experts = L.experts; a.stride = c.expert_stride;
    a.T = T; a.D = c.dim; a.H = c.expert_hidden; a.K = c.top_k;
    a.perm = w.perm; a.offsets = w.offsets; a.active = w.active; a.n_active = w.n_active;
    a.slot_pos = w.slot_pos; a.wt = w.wt; a.h = w.h; a.status = w.status;
    return a;
}

// The whole MoE call on device pointers.  block: x is the residual stream,
// updated in place; otherwise out = moe(xb).
// given_idx / given_wt (expert parallelism): the routing comes from outside, with
// expert ids local to this context's range and -1 for slots computed elsewhere;
// x is then the router input itself (no norm, no router) and out = the weighted
// sum over the local slots.
int forward(RbtMoe* m, int layer, const float* x, float* out, int T, int32_t* routing, int routing_stride,
            cudaStream_t s, bool block, const int32_t* given_idx = nullptr, const float* given_wt = nullptr,
            bool ep_rows = false, bool* rows_combined = nullptr) {
    if (!check_layer(m, layer, block)) return 0;
    const bool given = given_idx != nullptr;
    if (!given && m->n_local != m->cfg.n_experts)
        return fail("this context holds experts [%d, %d) only (expert parallelism): use rbt_moe_ep_block_device",
                    m->e0, m->e0 + m->n_local);
    const int E_run = given ? m->n_local : m->cfg.n_experts;
    if (T < 0) return fail("n_tokens must be >= 0 (got %d)", T);
    if (T == 0) return 1;
    if (routing && routing_stride < m->cfg.top_k)
        return fail("routing_stride %d < top_k %d", routing_stride, m->cfg.top_k);
    if (!set_device(m) || !reserve(m, T)) return 0;
    const RbtMoeConfig& c = m->cfg;
    const Layer& L = m->layers[layer];
    Workspace& w = m->ws;
    StageClock clk{m, s};
    m->prof.calls++;
    if (!given) m->last_routed = T;
    if (!given && (m->path == 0 || m->path == 4) && L.dec &&
        (!block || (reinterpret_cast<uintptr_t>(L.ffn_norm) % 16) == 0) &&
        rbt::decode_fused_supported(T, c.dim, c.expert_hidden, c.n_experts, c.top_k, c.dtype, L.experts,
                                    c.expert_stride, x, L.router)) {
        rbt::DecodeArgs da{};
        da.x = x; da.out = block ? const_cast<float*>(x) : out; da.ffn_norm = block ? L.ffn_norm : nullptr;
        da.eps = c.rms_eps; da.router = static_cast<const uint16_t*>(L.router); da.bias = L.bias;
        da.experts = L.experts; da.stride = c.expert_stride;
        da.D = c.dim; da.H = c.expert_hidden; da.E = c.n_experts; da.K = c.top_k; da.norm_topk = c.norm_topk;
        da.logits = w.logits; da.partials = w.partials;
        da.w2t = static_cast<const uint8_t*>(L.w2t); da.w2t_stride = (size_t)c.expert_hidden * c.dim * 2;
        // decode runs the layers in order, and after the last comes the first of the next token
        const Layer& N = m->layers[(layer + 1) % c.n_layers];
        auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
        da.next_router = aligned(N.router) ? static_cast<const uint8_t*>(N.router) : nullptr;
        da.next_norm = aligned(N.ffn_norm) ? N.ffn_norm : nullptr; da.idx = w.idx; da.counts = w.counts; da.offsets = w.offsets;
        da.perm = w.perm; da.slot_pos = w.slot_pos; da.active = w.active; da.n_active = w.n_active; da.wt = w.wt;
        da.routing_out = routing; da.sync = w.gbar; da.status = w.status; da.peer_wait_ns = m->peer_wait_ns;
        if (!clk.begin(6)) return 0;
        CU(rbt::launch_decode_fused(da, L.w2_cols, m->sm_count, s));
        return clk.end();
    }
    if (m->path == 4 && !given)
        return fail("fused decode path requested but unavailable (needs T == 1, bf16, D <= 2048)");
    const float* xb = x;
    rbt::RouterArgs ra{};
    if (block && !given) {  // xb = rmsnorm(x), inside the router's launch where it can
        xb = w.xb;
        ra.x_raw = x;
        ra.norm_w = L.ffn_norm;
        ra.eps = c.rms_eps;
    }
    ra.xb = xb;
    ra.T = T; ra.D = c.dim; ra.E = c.n_experts; ra.K = c.top_k;
    ra.router = L.router; ra.dtype = c.dtype; ra.bias = L.bias; ra.norm_topk = c.norm_topk;
    ra.logits = w.logits; ra.idx = w.idx; ra.wt = w.wt;
    ra.routing_out = routing; ra.routing_stride = routing_stride;
    ra.tile_counter = w.tile_counter; ra.done_counter = w.done_counter;
    ra.counts = w.counts; ra.offsets = w.offsets; ra.perm = w.perm; ra.slot_pos = w.slot_pos;
    ra.active = w.active; ra.n_active = w.n_active;
    ra.tile_cnt = w.tile_cnt; ra.tile_base = w.tile_base; ra.slot_rank = w.slot_rank;
    ra.router_cm = static_cast<const uint16_t*>(L.router_cm); ra.status = w.status;
    if (!clk.begin(1)) return 0;
    int router_launches = 0;
    if (given) {  // the permutation of the given slots over the local experts
        ra.E = E_run;
        ra.idx = const_cast<int32_t*>(given_idx);
        ra.wt = const_cast<float*>(given_wt);
        ra.routing_out = nullptr;
        CU(rbt::launch_route_given(ra, s, &router_launches));
    } else {
        CU(rbt::launch_router(ra, s, &router_launches));
    }
    m->prof.launches += router_launches - 1;
    const float* wt = given ? given_wt : w.wt;

    // expert parallelism, few received rows: the weight-streaming GEMV, which also
    // combines each row's slots (into `out`); the caller returns rows instead of slots
    if (ep_rows && out && (m->path == 0 || m->path == 1) &&
        (size_t)T * c.top_k <= (size_t)kEpStreamSlots &&
        rbt::stream_supported(sa_of(m, L, xb, x, out, T, false), c.dtype)) {
        rbt::StreamArgs sa = sa_of(m, L, xb, x, out, T, false);
        sa.wt = wt;
        if (!clk.begin(2)) return 0;
        CU(rbt::launch_gateup_stream(sa, m->sm_count, s));
        if (!clk.begin(3)) return 0;
        CU(rbt::launch_down_combine_stream(sa, m->sm_count, s));
        if (rows_combined) *rows_combined = true;
        return clk.end();
    }
    // the split kernel reads xb with 16-byte vectors
    const bool tc_ready = L.tc && w.tc_maps && (reinterpret_cast<uintptr_t>(xb) % 16 == 0);
    if (m->path == 2 && !tc_ready)
        return fail("tensor-core path requested but unavailable (needs bf16 weights, D and H multiples of 128, "
                    "16-byte aligned input)");
    const bool use_tc = tc_ready && (m->path == 2 || (m->path == 0 && T >= m->gemm_min_tokens));
    if (use_tc) {
        const int S = T * c.top_k;
        const bool f16 = L.w16 != nullptr;
        if (!clk.begin(5)) return 0;
        if (f16)  // fp16 rows (in the hi buffer) and their scales
            CU(rbt::launch_gather_f16(xb, w.perm, S, given ? w.offsets + E_run : nullptr, c.dim, c.top_k, w.xhi,
                                      w.bscale, s));
        else
            CU(rbt::launch_gather_split(xb, w.perm, S, given ? w.offsets + E_run : nullptr, c.dim, c.top_k, w.xhi,
                                        w.xlo, s));
        const int bn = rbt::tc_pick_bn(T, c.top_k, E_run);
        const int bi = bn == 32 ? 0 : (bn == 64 ? 1 : 2);
        CU(rbt::launch_tc_schedule(w.counts, w.offsets, E_run, bn, w.tb_e, w.tb_p0, w.tb_p1, w.n_tb, s));
        m->prof.launches++;
        rbt::TcGemmArgs ta{};
        ta.BN = bn;
        ta.tb_e = w.tb_e; ta.tb_p0 = w.tb_p0; ta.tb_p1 = w.tb_p1; ta.n_tb = w.n_tb;
        ta.H = c.expert_hidden; ta.D = c.dim; ta.h_hi = w.hhi; ta.h_lo = w.hlo; ta.y = w.y; ta.status = w.status;
        ta.MB = c.expert_hidden / 128; ta.KB = c.dim / 64;
        ta.bscale = w.bscale;
        // 128-slot blocks: the slots as the MMA's M side against 256 weight rows per tile
        const bool rows = bn == 128 && c.dim % 256 == 0;
        if (!clk.begin(2)) return 0;
        if (f16)
            CU(rbt::launch_tc_gateup_f16(L.w_gateup16, w.m_xhi[bi], ta, m->sm_count, s));
        else if (rows)
            CU(rbt::launch_tc_rows_moe(true, L.w_gateup, w.m_xhi[bi], w.m_xlo[bi], ta, m->sm_count, s));
        else
            CU(rbt::launch_tc_gateup(L.w_gateup, w.m_xhi[bi], w.m_xlo[bi], ta, m->sm_count, s));
        ta.MB = c.dim / 128; ta.KB = c.expert_hidden / 64;
        if (!clk.begin(3)) return 0;
        if (rows)
            CU(rbt::launch_tc_rows_moe(false, L.w_down, w.m_hhi[bi], w.m_hlo[bi], ta, m->sm_count, s));
        else
            CU(rbt::launch_tc_down(L.w_down, w.m_hhi[bi], w.m_hlo[bi], ta, m->sm_count, s));
    } else if (!ep_rows && m->path != 3 &&
               rbt::stream_supported(sa_of(m, L, xb, x, out, T, block && !given), c.dtype)) {
        rbt::StreamArgs sa = sa_of(m, L, xb, x, out, T, block && !given);
        sa.wt = wt;
        if (!clk.begin(2)) return 0;
        CU(rbt::launch_gateup_stream(sa, m->sm_count, s));
        if (!clk.begin(3)) return 0;
        CU(rbt::launch_down_combine_stream(sa, m->sm_count, s));
        return clk.end();
    } else {
        rbt::GemvArgs ga{};
        ga.xb = xb; ga.experts = L.experts; ga.stride = c.expert_stride;
        ga.T = T; ga.D = c.dim; ga.H = c.expert_hidden; ga.E = E_run; ga.K = c.top_k; ga.dtype = c.dtype;
        ga.perm = w.perm; ga.offsets = w.offsets; ga.active = w.active; ga.n_active = w.n_active;
        ga.h = w.h; ga.y = w.y; ga.grid = m->sm_count;
        if (!clk.begin(2)) return 0;
        CU(rbt::launch_gateup_gemv(ga, s));
        if (!clk.begin(3)) return 0;
        CU(rbt::launch_down_gemv(ga, s));
    }
    if (ep_rows) return clk.end();  // the expert outputs go back to their GPUs (launch_ep_return)

    rbt::CombineArgs ca{};
    ca.resid = block && !given ? x : nullptr;
    ca.y = w.y; ca.wt = wt; ca.slot_pos = w.slot_pos;
    ca.out = block && !given ? const_cast<float*>(x) : out;
    ca.T = T; ca.D = c.dim; ca.K = c.top_k;
    if (!clk.begin(4)) return 0;
    CU(rbt::launch_combine(ca, s));
    return clk.end();
}

// A tensor-core pipeline wait that timed out leaves a code in the status word.
// The status word's value st (read by the caller): on a timed-out wait, clear the
// status and the one-token kernel's sync words, and report it.
int status_error(RbtMoe* m, unsigned st) {
    if (st) {
        CU(cudaMemset(m->ws.status, 0, 4));
        CU(cudaMemset(m->ws.gbar, 0, (size_t)rbt::decode_sync_words(m->cfg.n_experts, m->cfg.top_k) * 4));
        return fail("a bounded wait in the kernels timed out (code 0x%x)", st);
    }
    return 1;
}

int check_status(RbtMoe* m) {
    if (!m->ws.block) return 1;
    unsigned st = 0;
    CU(cudaMemcpy(&st, m->ws.status, 4, cudaMemcpyDeviceToHost));
    return status_error(m, st);
}

// Host-pointer wrapper: stage through the workspace's device buffers.
int forward_host(RbtMoe* m, int layer, const float* x, float* out, int T, int32_t* routing, int routing_stride,
                 bool block) {
    if (!m) return fail("null context");
    if (T < 0) return fail("n_tokens must be >= 0 (got %d)", T);
    if (T == 0) return 1;
    if (!x || !out) return fail("null input/output pointer");
    if (!set_device(m) || !reserve(m, T)) return 0;
    const RbtMoeConfig& c = m->cfg;
    Workspace& w = m->ws;
    const size_t bytes = (size_t)T * c.dim * sizeof(float);
    CU(cudaMemcpyAsync(w.hx, x, bytes, cudaMemcpyHostToDevice, m->stream));
    float* dout = block ? w.hx : w.hout;
    if (!forward(m, layer, w.hx, dout, T, routing ? w.hrouting : nullptr, c.top_k, m->stream, block)) return 0;
    if (block && w.pinned && T <= kStageTokens) {
        // x (in place), the routing rows and the status word: one span, one copy back
        CU(cudaMemcpyAsync(w.pinned, w.hx, w.span, cudaMemcpyDeviceToHost, m->stream));
        CU(cudaStreamSynchronize(m->stream));
        const char* base = static_cast<const char*>(w.pinned);
        memcpy(out, base, bytes);
        if (routing) {
            const int32_t* r = reinterpret_cast<const int32_t*>(base + ((char*)w.hrouting - (char*)w.hx));
            for (int t = 0; t < T; t++)
                memcpy(routing + (size_t)t * routing_stride, r + (size_t)t * c.top_k, sizeof(int32_t) * c.top_k);
        }
        unsigned st;
        memcpy(&st, base + ((char*)w.status - (char*)w.hx), sizeof st);
        return status_error(m, st);
    }
    CU(cudaMemcpyAsync(out, dout, bytes, cudaMemcpyDeviceToHost, m->stream));
    if (routing)
        CU(cudaMemcpy2DAsync(routing, (size_t)routing_stride * 4, w.hrouting, (size_t)c.top_k * 4,
                             (size_t)c.top_k * 4, T, cudaMemcpyDeviceToHost, m->stream));
    // the status word comes back with the results (one synchronisation per call)
    CU(cudaMemcpyAsync(m->h_status, w.status, sizeof(unsigned), cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return status_error(m, *m->h_status);
}

}  // namespace

namespace rbt {
// 1 if the context's kernels reported no timed-out wait since the last check,
// else 0 with the message set (for the whole-forward calls of model.cu)
int moe_status_ok(RbtMoe* m) { return check_status(m); }

// Changes whenever the workspace is reallocated (a larger call than any before):
// a CUDA graph captured with the block/ffn device calls holds workspace
// addresses and must be captured again after it changes.  (Used by model.cu.)
unsigned long long moe_workspace_generation(RbtMoe* m) { return m ? m->ws_gen : 0; }

// The device address of the status word (valid until the workspace generation
// changes), or nullptr before the first reservation.  (Used by model.cu.)
unsigned* moe_status_word(RbtMoe* m) { return m && m->ws.block ? m->ws.status : nullptr; }

// Rows an expert-parallel context's workspace must hold (every rank's max_tokens)
// once it is connected, else 0: the whole-forward calls then run each MoE block
// through the group (ep_block) instead of on this GPU alone.  (Used by model*.cu.)
int moe_ep_rows(RbtMoe* m) { return m && m->ep.connected ? m->ep.R * m->ep.cap : 0; }
int moe_ep_cap(RbtMoe* m) { return m && m->ep.connected ? m->ep.cap : 0; }
}  // namespace rbt

extern "C" {

const char* rbt_moe_last_error(void) { return g_err; }

int rbt_moe_create(RbtMoe** out, const RbtMoeConfig* cfg, int device) {
    if (!out || !cfg) return fail("null argument");
    *out = nullptr;
    const RbtMoeConfig& c = *cfg;
    if (c.dim <= 0 || c.expert_hidden <= 0 || c.n_layers <= 0 || c.n_experts <= 0 || c.top_k <= 0)
        return fail("invalid config: dims must be positive");
    if (c.top_k > c.n_experts || c.top_k > rbt::kMaxTopK)
        return fail("invalid config: top_k %d (n_experts %d, max %d)", c.top_k, c.n_experts, rbt::kMaxTopK);
    if (c.n_experts > rbt::kMaxExperts) return fail("n_experts %d above the supported %d", c.n_experts, rbt::kMaxExperts);
    if (c.dtype != RBT_MOE_DT_F32 && c.dtype != RBT_MOE_DT_BF16) return fail("dtype must be 0 (f32) or 1 (bf16)");
    const size_t esz = c.dtype == RBT_MOE_DT_BF16 ? 2 : 4;
    if (c.expert_stride < 3ull * c.expert_hidden * c.dim * esz) return fail("expert_stride smaller than one expert");
    int ndev = 0;
    CU(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail("device %d out of range (%d visible)", device, ndev);
    CU(cudaSetDevice(device));
    RbtMoe* m = new (std::nothrow) RbtMoe();
    if (!m) return fail("out of host memory");
    m->cfg = c;
    m->n_local = c.n_experts;
    m->device = device;
    m->esz = esz;
    if (const char* v = getenv("RBT_MOE_GEMM_MIN_TOKENS")) m->gemm_min_tokens = atoi(v);
    m->layers.resize(c.n_layers);
    bool ok = cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, device) == cudaSuccess &&
              cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaMallocHost((void**)&m->h_status, sizeof(unsigned)) == cudaSuccess;
    if (!ok) {
        if (m->stream) cudaStreamDestroy(m->stream);
        delete m;
        return fail("cannot initialise CUDA device %d", device);
    }
    *out = m;
    return 1;
}

void rbt_moe_destroy(RbtMoe* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    for (Layer& L : m->layers) {
        cudaFree(L.owned);
        cudaFree(L.bias);
        cudaFree(L.w2t);
        cudaFree(L.w16);
        cudaFree(L.router_cm);
    }
    cudaFree(m->ws.block);
    if (m->ws.pinned) cudaFreeHost(m->ws.pinned);
    for (void* p : m->ep.opened) cudaIpcCloseMemHandle(p);
    cudaFree(m->ep.block);
    cudaFree(m->ep.local);
    for (cudaEvent_t e : m->ev_pool) cudaEventDestroy(e);
    cudaStreamDestroy(m->stream);
    cudaFreeHost(m->h_status);
    delete m;
}

int rbt_moe_load_layer(RbtMoe* m, int layer, const float* ffn_norm, const void* router, const void* experts) {
    if (!m) return fail("null context");
    if (layer < 0 || layer >= m->cfg.n_layers) return fail("layer %d out of range", layer);
    if (!router || !experts) return fail("null router/experts pointer");
    if (!set_device(m)) return 0;
    const RbtMoeConfig& c = m->cfg;
    const size_t b_exp = (size_t)m->n_local * c.expert_stride;
    const size_t b_router = (size_t)c.n_experts * c.dim * m->esz;
    const size_t b_norm = (size_t)c.dim * 4;
    const size_t o_router = align_up(b_exp, 256), o_norm = align_up(o_router + b_router, 256);
    Layer& L = m->layers[layer];
    if (L.owned) CU(cudaFree(L.owned));
    L.owned = nullptr;
    void* p = nullptr;
    CU(cudaMalloc(&p, o_norm + b_norm));
    L.owned = p;
    CU(cudaMemcpy(p, experts, b_exp, cudaMemcpyHostToDevice));
    CU(cudaMemcpy((char*)p + o_router, router, b_router, cudaMemcpyHostToDevice));
    if (ffn_norm) CU(cudaMemcpy((char*)p + o_norm, ffn_norm, b_norm, cudaMemcpyHostToDevice));
    L.experts = (const uint8_t*)p;
    L.router = (char*)p + o_router;
    L.ffn_norm = ffn_norm ? (const float*)((char*)p + o_norm) : nullptr;
    layer_maps(m, L);
    return 1;
}

int rbt_moe_bind_layer(RbtMoe* m, int layer, const float* d_ffn_norm, const void* d_router, const void* d_experts) {
    if (!m) return fail("null context");
    if (layer < 0 || layer >= m->cfg.n_layers) return fail("layer %d out of range", layer);
    if (!d_router || !d_experts) return fail("null router/experts pointer");
    if (!set_device(m)) return 0;
    Layer& L = m->layers[layer];
    if (L.owned) CU(cudaFree(L.owned));
    L.owned = nullptr;
    L.ffn_norm = d_ffn_norm;
    L.router = d_router;
    L.experts = (const uint8_t*)d_experts;
    layer_maps(m, L);
    return 1;
}

int rbt_moe_set_router_bias(RbtMoe* m, int layer, const float* bias) {
    if (!m) return fail("null context");
    if (layer < 0 || layer >= m->cfg.n_layers) return fail("layer %d out of range", layer);
    if (!set_device(m)) return 0;
    Layer& L = m->layers[layer];
    if (!bias) {
        if (L.bias) CU(cudaFree(L.bias));
        L.bias = nullptr;
        return 1;
    }
    if (!L.bias) CU(cudaMalloc(&L.bias, (size_t)m->cfg.n_experts * 4));
    CU(cudaMemcpy(L.bias, bias, (size_t)m->cfg.n_experts * 4, cudaMemcpyHostToDevice));
    return 1;
}

int rbt_moe_reserve(RbtMoe* m, int n_tokens) {
    if (!m) return fail("null context");
    if (n_tokens < 0) return fail("n_tokens must be >= 0");
    return set_device(m) && reserve(m, n_tokens);
}

int rbt_moe_block(RbtMoe* m, int layer, float* x, int n_tokens, int32_t* routing_out, int routing_stride) {
    return forward_host(m, layer, x, x, n_tokens, routing_out, routing_stride, true);
}

int rbt_moe_ffn(RbtMoe* m, int layer, const float* xb, int n_tokens, float* moe_out, int32_t* routing_out,
                int routing_stride) {
    return forward_host(m, layer, xb, moe_out, n_tokens, routing_out, routing_stride, false);
}

int rbt_moe_block_device(RbtMoe* m, int layer, float* d_x, int n_tokens, int32_t* d_routing_out, int routing_stride,
                         void* stream) {
    if (!m) return fail("null context");
    if (!d_x && n_tokens > 0) return fail("null x");
    return forward(m, layer, d_x, d_x, n_tokens, d_routing_out, routing_stride, (cudaStream_t)stream, true);
}

int rbt_moe_ffn_device(RbtMoe* m, int layer, const float* d_xb, int n_tokens, float* d_moe_out,
                       int32_t* d_routing_out, int routing_stride, void* stream) {
    if (!m) return fail("null context");
    if ((!d_xb || !d_moe_out) && n_tokens > 0) return fail("null xb/moe_out");
    return forward(m, layer, d_xb, d_moe_out, n_tokens, d_routing_out, routing_stride, (cudaStream_t)stream, false);
}

// ---------------------------------------------------------------- expert parallelism

namespace {

// Narrow the context to experts [first_expert, first_expert + n_experts_local) (before any layer is bound).
int set_expert_range(RbtMoe* m, int first_expert, int n_experts_local) {
    if (!m) return fail("null context");
    const int E = m->cfg.n_experts;
    if (first_expert < 0 || n_experts_local <= 0 || first_expert + n_experts_local > E)
        return fail("expert range [%d, %d) outside [0, %d)", first_expert, first_expert + n_experts_local, E);
    for (const Layer& L : m->layers)
        if (L.experts) return fail("set the expert range before loading or binding any layer");
    m->e0 = first_expert;
    m->n_local = n_experts_local;
    return 1;
}

// The EP block's layout, the same on every GPU of a group (same config, R, cap).
void ep_layout(RbtMoe* m) {
    EpState& p = m->ep;
    const size_t R = p.R, cap = p.cap, D = m->cfg.dim, K = m->cfg.top_k;
    size_t o = 256;  // a header first: the block's shape, checked when peers connect
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes, 256);
        return at;
    };
    p.off_rows = take(R * cap * D * 4);
    p.off_back = take(R * cap * D * 4);
    p.off_idx = take(R * cap * K * 4);
    p.off_wt = take(R * cap * K * 4);
    p.off_count = take(R * 4);
    p.off_fdisp = take(R * 8);
    p.off_fret = take(R * 8);
    p.block_bytes = o;
}

// Pointers into GPU g's block (whose base in this process is `base`).
void ep_set_peer(EpState& p, int g, char* base) {
    p.peers.recv_rows[g] = reinterpret_cast<float*>(base + p.off_rows);
    p.peers.back_rows[g] = reinterpret_cast<float*>(base + p.off_back);
    p.peers.recv_idx[g] = reinterpret_cast<int32_t*>(base + p.off_idx);
    p.peers.recv_wt[g] = reinterpret_cast<float*>(base + p.off_wt);
    p.peers.recv_count[g] = reinterpret_cast<int32_t*>(base + p.off_count);
    p.peers.flag_dispatch[g] = reinterpret_cast<unsigned long long*>(base + p.off_fdisp);
    p.peers.flag_return[g] = reinterpret_cast<unsigned long long*>(base + p.off_fret);
}

// The header of an EP block: what every GPU of the group must agree on.
struct EpHeader {
    uint32_t magic, R, cap, D, K, E;
};
constexpr uint32_t kEpMagic = 0x52425445u;  // "ETBR"
EpHeader ep_header(const RbtMoe* m) {
    return EpHeader{kEpMagic, (uint32_t)m->ep.R, (uint32_t)m->ep.cap, (uint32_t)m->cfg.dim,
                    (uint32_t)m->cfg.top_k, (uint32_t)m->cfg.n_experts};
}

rbt::EpArgs ep_args(RbtMoe* m) {
    const EpState& p = m->ep;
    rbt::EpArgs a{};
    a.peers = p.peers;
    a.R = p.R; a.rank = p.rank; a.epr = p.epr; a.cap = p.cap; a.D = m->cfg.dim; a.K = m->cfg.top_k;
    a.epoch = p.epoch; a.done = p.done; a.status = m->ws.status; a.timeout_ns = p.timeout_ns;
    return a;
}

// One expert-parallel MoE block on this GPU: d_x [T, D] += MoE(rmsnorm(d_x)).
int ep_block(RbtMoe* m, int layer, float* d_x, int T, int32_t* d_routing, int routing_stride, cudaStream_t s) {
    EpState& p = m->ep;
    if (!p.connected) return fail("expert parallelism: rbt_moe_ep_connect (or _connect_local) first");
    if (T < 0 || T > p.cap) return fail("n_tokens %d outside [0, %d] (the max_tokens of rbt_moe_ep_init)", T, p.cap);
    if (T > 0 && !d_x) return fail("null input");
    if (d_routing && routing_stride < m->cfg.top_k)
        return fail("routing_stride %d < top_k %d", routing_stride, m->cfg.top_k);
    if (!check_layer(m, layer, true) || !set_device(m) || !reserve(m, p.R * p.cap)) return 0;
    const RbtMoeConfig& c = m->cfg;
    const Layer& L = m->layers[layer];
    Workspace& w = m->ws;
    StageClock clk{m, s};
    m->prof.calls++;
    if (T > 0) {  // rmsnorm + the whole router (global expert ids), bit-exact as on one GPU
        m->last_routed = T;
        rbt::RouterArgs ra{};
        ra.xb = w.xb; ra.x_raw = d_x; ra.norm_w = L.ffn_norm; ra.eps = c.rms_eps;
        ra.T = T; ra.D = c.dim; ra.E = c.n_experts; ra.K = c.top_k;
        ra.router = L.router; ra.dtype = c.dtype; ra.bias = L.bias; ra.norm_topk = c.norm_topk;
        ra.logits = w.logits; ra.idx = w.idx; ra.wt = w.wt;
        ra.routing_out = d_routing; ra.routing_stride = routing_stride;
        ra.tile_counter = w.tile_counter; ra.done_counter = w.done_counter;
        ra.counts = w.counts; ra.offsets = w.offsets; ra.perm = w.perm; ra.slot_pos = w.slot_pos;
        ra.active = w.active; ra.n_active = w.n_active;
        ra.tile_cnt = w.tile_cnt; ra.tile_base = w.tile_base; ra.slot_rank = w.slot_rank;
        ra.router_cm = static_cast<const uint16_t*>(L.router_cm); ra.status = w.status;
        if (!clk.begin(1)) return 0;
        int launches = 0;
        CU(rbt::launch_router(ra, s, &launches));
        m->prof.launches += launches - 1;
    }
    const rbt::EpArgs a = ep_args(m);
    if (!clk.begin(7)) return 0;
    CU(rbt::launch_ep_plan(w.idx, T, c.top_k, p.R, p.epr, p.pos, p.counts, s));
    m->prof.launches += 2;
    CU(rbt::launch_ep_dispatch(a, w.xb, w.idx, w.wt, p.pos, p.counts, T, s));
    CU(rbt::launch_ep_receive(a, s));
    // the experts of this GPU on every row it received ([R][cap], unused rows have no slots)
    char* own = static_cast<char*>(p.block);
    bool rows = false;
    if (!forward(m, layer, reinterpret_cast<const float*>(own + p.off_rows), w.hout, p.R * p.cap, nullptr,
                 c.top_k, s, false, reinterpret_cast<const int32_t*>(own + p.off_idx),
                 reinterpret_cast<const float*>(own + p.off_wt), true, &rows))
        return 0;
    if (!clk.begin(7)) return 0;
    CU(rbt::launch_ep_return(a, w.y, w.slot_pos, rows ? w.hout : nullptr, s));
    m->prof.launches++;
    CU(rbt::launch_ep_combine(a, d_x, p.pos, T, s));
    return clk.end();
}

}  // namespace

int rbt_moe_ep_init(RbtMoe* m, int rank, int n_ranks, int max_tokens) {
    if (!m) return fail("null context");
    const int E = m->cfg.n_experts;
    if (n_ranks < 1 || n_ranks > rbt::kEpMaxRanks || rank < 0 || rank >= n_ranks || E % n_ranks)
        return fail("expert parallelism: %d experts over %d GPUs (rank %d): need 1 <= n_ranks <= %d dividing the "
                    "experts", E, n_ranks, rank, rbt::kEpMaxRanks);
    if (max_tokens < 1) return fail("max_tokens must be >= 1");
    if (m->cfg.dim % 4) return fail("expert parallelism needs dim %% 4 == 0");
    if (m->ep.block) return fail("rbt_moe_ep_init was called already");
    if (!set_expert_range(m, rank * (E / n_ranks), E / n_ranks)) return 0;
    if (!set_device(m)) return 0;
    // every kernel of the layer loaded now, not at a first launch behind a waiting kernel
    rbt::preload_router_kernels();
    rbt::preload_gemm_kernels();
    rbt::preload_gemv_kernels();
    rbt::preload_stream_kernels();
    rbt::preload_combine_kernels();
    rbt::preload_attn_tc_kernels();
    rbt::preload_ep_kernels();
    EpState& p = m->ep;
    p.R = n_ranks; p.rank = rank; p.epr = E / n_ranks; p.cap = max_tokens;
    ep_layout(m);
    CU(cudaMalloc(&p.block, p.block_bytes));
    CU(cudaMemset(p.block, 0, p.block_bytes));
    const EpHeader hdr = ep_header(m);
    CU(cudaMemcpy(p.block, &hdr, sizeof hdr, cudaMemcpyHostToDevice));
    const size_t pos_b = align_up((size_t)max_tokens * n_ranks * 4, 256), cnt_b = 256, ep_b = 256;
    CU(cudaMalloc(&p.local, pos_b + cnt_b + ep_b + 256));
    CU(cudaMemset(p.local, 0, pos_b + cnt_b + ep_b + 256));
    char* l = static_cast<char*>(p.local);
    p.pos = reinterpret_cast<int32_t*>(l);
    p.counts = reinterpret_cast<int32_t*>(l + pos_b);
    p.epoch = reinterpret_cast<unsigned long long*>(l + pos_b + cnt_b);
    p.done = reinterpret_cast<unsigned*>(l + pos_b + cnt_b + ep_b);
    ep_set_peer(p, rank, static_cast<char*>(p.block));
    return 1;
}

int rbt_moe_ep_handle(RbtMoe* m, void* handle_out) {
    if (!m || !handle_out) return fail("null argument");
    if (!m->ep.block) return fail("rbt_moe_ep_init first");
    if (!set_device(m)) return 0;
    cudaIpcMemHandle_t h;
    CU(cudaIpcGetMemHandle(&h, m->ep.block));
    memcpy(handle_out, &h, sizeof h);
    return 1;
}

int rbt_moe_ep_connect(RbtMoe* m, const void* handles) {
    if (!m || !handles) return fail("null argument");
    EpState& p = m->ep;
    if (!p.block) return fail("rbt_moe_ep_init first");
    if (p.connected) return fail("already connected");
    if (!set_device(m)) return 0;
    for (int g = 0; g < p.R; g++) {
        if (g == p.rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + (size_t)g * sizeof h, sizeof h);
        void* base = nullptr;
        CU(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
        p.opened.push_back(base);
        EpHeader theirs{}, ours = ep_header(m);
        CU(cudaMemcpy(&theirs, base, sizeof theirs, cudaMemcpyDeviceToHost));
        if (memcmp(&theirs, &ours, sizeof ours) != 0)
            return fail("expert parallelism: rank %d's block has another shape (n_ranks %u, max_tokens %u, dim %u, "
                        "top_k %u, n_experts %u; here %u, %u, %u, %u, %u)", g, theirs.R, theirs.cap, theirs.D,
                        theirs.K, theirs.E, ours.R, ours.cap, ours.D, ours.K, ours.E);
        ep_set_peer(p, g, static_cast<char*>(base));
    }
    p.connected = true;
    return 1;
}

int rbt_moe_ep_connect_local(RbtMoe* const* ms, int n) {
    if (!ms || n < 1) return fail("null argument");
    for (int i = 0; i < n; i++) {
        if (!ms[i] || !ms[i]->ep.block) return fail("rbt_moe_ep_init every context first");
        if (ms[i]->ep.R != n || ms[i]->ep.rank != i) return fail("context %d is not rank %d of %d", i, i, n);
        const EpHeader a = ep_header(ms[i]), b = ep_header(ms[0]);
        if (memcmp(&a, &b, sizeof a) != 0) return fail("context %d's group shape differs from context 0's", i);
    }
    for (int i = 0; i < n; i++) {
        RbtMoe* m = ms[i];
        if (!set_device(m)) return 0;
        for (int j = 0; j < n; j++) {
            if (j == i) continue;
            if (ms[j]->device != m->device) {
                int can = 0;
                CU(cudaDeviceCanAccessPeer(&can, m->device, ms[j]->device));
                if (!can) return fail("GPU %d cannot access GPU %d's memory", m->device, ms[j]->device);
                const cudaError_t e = cudaDeviceEnablePeerAccess(ms[j]->device, 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) (void)cudaGetLastError();
                else if (e != cudaSuccess) return fail("cudaDeviceEnablePeerAccess: %s", cudaGetErrorString(e));
            }
            ep_set_peer(m->ep, j, static_cast<char*>(ms[j]->ep.block));
        }
        m->ep.connected = true;
    }
    return 1;
}

int rbt_moe_set_timeout(RbtMoe* m, uint64_t timeout_ns) {
    if (!m) return fail("null context");
    m->peer_wait_ns = timeout_ns;
    return 1;
}

int rbt_moe_ep_set_timeout(RbtMoe* m, uint64_t timeout_ns) {
    if (!m) return fail("null context");
    if (timeout_ns < 1000) return fail("timeout below 1 us");
    m->ep.timeout_ns = timeout_ns;
    return 1;
}

int rbt_moe_ep_block_device(RbtMoe* m, int layer, float* d_x, int n_tokens, int32_t* d_routing_out,
                            int routing_stride, void* stream) {
    if (!m) return fail("null context");
    return ep_block(m, layer, d_x, n_tokens, d_routing_out, routing_stride, (cudaStream_t)stream);
}

int rbt_moe_ep_block(RbtMoe* const* ms, int n, int layer, float* x, int n_tokens, int32_t* routing_out,
                     int routing_stride) {
    if (!ms || n < 1 || !ms[0]) return fail("null argument");
    RbtMoe* m0 = ms[0];
    if (n_tokens < 0) return fail("n_tokens must be >= 0 (got %d)", n_tokens);
    if (n_tokens == 0) return 1;
    if (!x) return fail("null x");
    if (n_tokens > m0->ep.cap) return fail("n_tokens %d above max_tokens %d", n_tokens, m0->ep.cap);
    for (int g = 0; g < n; g++)
        if (!set_device(ms[g]) || !reserve(ms[g], ms[g]->ep.R * ms[g]->ep.cap)) return 0;
    Workspace& w0 = m0->ws;
    const size_t bytes = (size_t)n_tokens * m0->cfg.dim * sizeof(float);
    if (!set_device(m0)) return 0;
    CU(cudaMemcpyAsync(w0.hx, x, bytes, cudaMemcpyHostToDevice, m0->stream));
    // every GPU runs the layer; GPU 0 holds the tokens, the others only their experts
    for (int g = 0; g < n; g++) {
        if (!set_device(ms[g])) return 0;
        if (!ep_block(ms[g], layer, g == 0 ? w0.hx : nullptr, g == 0 ? n_tokens : 0,
                      g == 0 && routing_out ? w0.hrouting : nullptr, m0->cfg.top_k, ms[g]->stream))
            return 0;
    }
    if (!set_device(m0)) return 0;
    CU(cudaMemcpyAsync(x, w0.hx, bytes, cudaMemcpyDeviceToHost, m0->stream));
    if (routing_out)
        CU(cudaMemcpy2DAsync(routing_out, (size_t)routing_stride * 4, w0.hrouting, (size_t)m0->cfg.top_k * 4,
                             (size_t)m0->cfg.top_k * 4, n_tokens, cudaMemcpyDeviceToHost, m0->stream));
    for (int g = 0; g < n; g++) {
        if (!set_device(ms[g])) return 0;
        CU(cudaStreamSynchronize(ms[g]->stream));
        if (!check_status(ms[g])) return fail("expert parallelism: GPU %d (rank %d) failed", ms[g]->device, g);
    }
    return 1;
}

int rbt_moe_status(RbtMoe* m, unsigned* status_out) {
    if (!m || !status_out) return fail("null argument");
    *status_out = 0;
    if (!m->ws.block) return 1;
    if (!set_device(m)) return 0;
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(status_out, m->ws.status, sizeof(unsigned), cudaMemcpyDeviceToHost));
    if (*status_out) {  // a failed call may leave the one-token kernel's words half set: clear them too
        CU(cudaMemset(m->ws.status, 0, 4));
        CU(cudaMemset(m->ws.gbar, 0, (size_t)rbt::decode_sync_words(m->cfg.n_experts, m->cfg.top_k) * 4));
    }
    return 1;
}

int rbt_moe_route_device(RbtMoe* m, int layer, const float* d_x, int n_tokens, int block, float* d_xb,
                         int32_t* d_idx, float* d_wt, void* stream) {
    if (!m) return fail("null context");
    if (n_tokens < 0) return fail("n_tokens must be >= 0 (got %d)", n_tokens);
    if (n_tokens == 0) return 1;
    if (!d_x || !d_xb || !d_idx || !d_wt) return fail("null argument");
    if (!check_layer(m, layer, block != 0) || !set_device(m) || !reserve(m, n_tokens)) return 0;
    const RbtMoeConfig& c = m->cfg;
    const Layer& L = m->layers[layer];
    Workspace& w = m->ws;
    cudaStream_t s = (cudaStream_t)stream;
    StageClock clk{m, s};
    m->prof.calls++;
    m->last_routed = n_tokens;
    if (block) {
        if (!clk.begin(0)) return 0;
        CU(rbt::launch_rmsnorm(d_x, L.ffn_norm, d_xb, n_tokens, c.dim, c.rms_eps, s));
    } else if (d_xb != d_x) {
        CU(cudaMemcpyAsync(d_xb, d_x, (size_t)n_tokens * c.dim * sizeof(float), cudaMemcpyDeviceToDevice, s));
    }
    rbt::RouterArgs ra{};
    ra.xb = d_xb;
    ra.T = n_tokens; ra.D = c.dim; ra.E = c.n_experts; ra.K = c.top_k;
    ra.router = L.router; ra.dtype = c.dtype; ra.bias = L.bias; ra.norm_topk = c.norm_topk;
    ra.logits = w.logits; ra.idx = d_idx; ra.wt = d_wt;
    ra.tile_counter = w.tile_counter; ra.done_counter = w.done_counter;
    ra.counts = w.counts; ra.offsets = w.offsets; ra.perm = w.perm; ra.slot_pos = w.slot_pos;
    ra.active = w.active; ra.n_active = w.n_active;
    ra.tile_cnt = w.tile_cnt; ra.tile_base = w.tile_base; ra.slot_rank = w.slot_rank;
    ra.router_cm = static_cast<const uint16_t*>(L.router_cm); ra.status = w.status;
    if (!clk.begin(1)) return 0;
    int launches = 0;
    CU(rbt::launch_router(ra, s, &launches));
    m->prof.launches += launches - 1;
    return clk.end();
}

int rbt_moe_expert_histogram(RbtMoe* m, int32_t* counts_out) {
    if (!m || !counts_out) return fail("null argument");
    if (!set_device(m)) return 0;
    if (!m->ws.block) {
        memset(counts_out, 0, sizeof(int32_t) * (size_t)m->cfg.n_experts);
        return 1;
    }
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(counts_out, m->ws.counts, sizeof(int32_t) * (size_t)m->cfg.n_experts, cudaMemcpyDeviceToHost));
    return 1;
}

int rbt_moe_router_logits(RbtMoe* m, float* logits_out, int n_tokens) {
    if (!m || !logits_out) return fail("null argument");
    if (n_tokens < 1 || n_tokens > m->last_routed)
        return fail("n_tokens %d outside [1, %d] (the tokens of the most recent routed call)", n_tokens,
                    m->last_routed);
    if (!set_device(m)) return 0;
    CU(cudaDeviceSynchronize());
    CU(cudaMemcpy(logits_out, m->ws.logits, sizeof(float) * (size_t)n_tokens * m->cfg.n_experts,
                  cudaMemcpyDeviceToHost));
    return 1;
}

int rbt_moe_profile(RbtMoe* m, int timing, int reset, RbtMoeProfile* out) {
    if (!m) return fail("null context");
    if (!set_device(m)) return 0;
    if (out) {
        *out = m->prof;
        for (int i = 0; i < RBT_MOE_STAGES; i++) out->stage_ms[i] = 0.0;
        for (const StageMark& k : m->marks) {
            // intervals whose events carry no timestamp yet (a captured graph not
            // replayed so far) contribute nothing
            float ms = 0.f;
            if (cudaEventSynchronize(m->ev_pool[k.ev_end]) != cudaSuccess ||
                cudaEventElapsedTime(&ms, m->ev_pool[k.ev_begin], m->ev_pool[k.ev_end]) != cudaSuccess) {
                (void)cudaGetLastError();
                continue;
            }
            out->stage_ms[k.stage] += ms;
        }
    }
    if (reset) {
        m->prof = RbtMoeProfile{};
        m->marks.clear();
        m->ev_used = 0;
    }
    if (timing >= 0) m->timing = timing != 0;
    if (m->timing && m->ev_pool.empty()) {
        m->ev_pool.resize(4096);
        for (cudaEvent_t& e : m->ev_pool) CU(cudaEventCreate(&e));
    }
    return 1;
}

int rbt_moe_set_path(RbtMoe* m, int path) {
    if (!m) return fail("null context");
    if (path < 0 || path > 4) return fail("path must be 0..4");
    m->path = path;
    return 1;
}

}  // extern "C"
