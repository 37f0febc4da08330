// decode_noalloc.cu -- rbt_moe_decode_noalloc: the one-token MoE block for
// callers that must not allocate GPU memory.
//
// Who needs it: code that runs inside a host framework which already owns the
// device memory (a caching allocator or an inference server that reserves most
// of HBM up front, where a cudaMalloc behind its back fails or fragments the
// pool), and latency-critical decode loops that cannot afford cudaMalloc's
// implicit device synchronisation.  The context API (rbt_moe_create) allocates
// its workspace with cudaMalloc; this entry point instead keeps its scratch in
// a fixed-size array in the library's own device memory, set aside when the
// library is loaded on a GPU, and allocates nothing per call.
//
// The array below is per GPU and lives until the process exits.  Host code may
// not use its name as a device address (on the host the name only stands in
// for the symbol), so set-up asks the runtime for the device address once per
// device and CUDA context, with that device current, and passes that pointer
// to the kernel.  A device reset destroys the context and may move the array;
// the next call sees a different current context and looks the address up
// again.
// All calls on a GPU share the array and find the previous call's contents in
// it: the counters that must start at zero are cleared on the caller's stream
// before every launch, and two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on the array.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "../../include/rbt_moe.h"
#include "kernels.h"

namespace rbt {
void set_last_error(const char* msg);
}

namespace {

constexpr size_t kScratchBytes = RBT_MOE_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DeviceSetup {
    void* scratch = nullptr;  // device address of g_noalloc_scratch on this GPU
    void* ctx = nullptr;      // the CUDA context that address belongs to
    int sm_count = 0;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mutex;

int fail(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
int fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    fprintf(stderr, "rbt_moe: %s\n", buf);
    rbt::set_last_error(buf);
    return 0;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// The calling thread's current CUDA context (driver API, through the runtime's
// entry-point query so that the library needs no link against libcuda).
void* current_context() {
    using Fn = CUresult (*)(CUcontext*);
    static Fn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (Fn) nullptr;
        return reinterpret_cast<Fn>(p);
    }();
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// Set-up for the current device (see above); false with the error recorded.
bool device_setup(DeviceSetup* out);

// Byte offsets of the scratch parts for one configuration; returns the total.
// The status word comes first, at the same place for every model, so that
// rbt_moe_decode_noalloc_status can read it without the call's configuration.
struct Layout {
    size_t logits, partials, idx, wt, counts, offsets, perm, slot_pos, active, n_active, sync, status, total;
};
Layout layout_for(int E, int K, int D, int grid) {
    Layout l{};
    size_t o = 0;
    l.status = o;     o = align256(o + sizeof(unsigned));
    l.sync = o;       o = align256(o + (size_t)rbt::decode_sync_words(E, K) * sizeof(unsigned));
    l.n_active = o;   o = align256(o + sizeof(int32_t));
    l.logits = o;     o = align256(o + (size_t)E * sizeof(float));
    l.counts = o;     o = align256(o + (size_t)E * sizeof(int32_t));
    l.offsets = o;    o = align256(o + ((size_t)E + 1) * sizeof(int32_t));
    l.idx = o;        o = align256(o + (size_t)K * sizeof(int32_t));
    l.wt = o;         o = align256(o + (size_t)K * sizeof(float));
    l.perm = o;       o = align256(o + (size_t)K * sizeof(int32_t));
    l.slot_pos = o;   o = align256(o + (size_t)K * sizeof(int32_t));
    l.active = o;     o = align256(o + (size_t)K * sizeof(int32_t));
    l.partials = o;   o = align256(o + rbt::decode_partials_bytes(grid, D));
    l.total = o;
    return l;
}

}  // namespace

extern "C" int rbt_moe_decode_noalloc(const RbtMoeConfig* cfg, const float* d_ffn_norm, const void* d_router,
                                      const float* d_router_bias, const void* d_experts, const float* d_x,
                                      float* d_out, int32_t* d_routing_out, void* stream) {
    if (!cfg || !d_router || !d_experts || !d_x || !d_out) return fail("rbt_moe_decode_noalloc: null argument");
    const RbtMoeConfig& c = *cfg;
    if (c.dim <= 0 || c.expert_hidden <= 0 || c.n_experts <= 0 || c.top_k <= 0 || c.top_k > c.n_experts)
        return fail("rbt_moe_decode_noalloc: invalid config");
    if (!rbt::decode_fused_supported(1, c.dim, c.expert_hidden, c.n_experts, c.top_k, c.dtype, d_experts,
                                     c.expert_stride, d_x, d_router))
        return fail("rbt_moe_decode_noalloc: unsupported model for the one-token kernel (needs bf16 weights, "
                    "dim <= 2048 and a multiple of 16, expert_hidden a multiple of 8, n_experts <= 256, "
                    "top_k <= 64, 16-byte aligned pointers)");
    if (d_out != d_x && (reinterpret_cast<uintptr_t>(d_out) % 4) != 0)
        return fail("rbt_moe_decode_noalloc: misaligned output");
    if ((reinterpret_cast<uintptr_t>(d_ffn_norm) % 16) != 0)
        return fail("rbt_moe_decode_noalloc: d_ffn_norm must be 16-byte aligned");

    DeviceSetup setup;
    if (!device_setup(&setup)) return 0;
    const Layout l = layout_for(c.n_experts, c.top_k, c.dim, setup.sm_count);
    if (l.total > kScratchBytes)
        return fail("rbt_moe_decode_noalloc: this model needs %zu bytes of scratch on this GPU (%d SMs x dim "
                    "%d partial sums), above the fixed %zu-byte buffer",
                    l.total, setup.sm_count, c.dim, kScratchBytes);
    CUtensorMap w2map;
    if (!rbt::make_decode_w2_map(&w2map, d_experts, c.dim, c.expert_hidden, c.n_experts, c.expert_stride))
        return fail("rbt_moe_decode_noalloc: cannot describe the w2 columns as a TMA tensor map");
    uint8_t* base = static_cast<uint8_t*>(setup.scratch);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the cross-CTA counters and the status word must start at zero
    cudaError_t err = cudaMemsetAsync(base, 0, l.logits, s);
    if (err != cudaSuccess) return fail("rbt_moe_decode_noalloc: cudaMemsetAsync failed: %s", cudaGetErrorString(err));

    rbt::DecodeArgs a{};
    a.x = d_x;
    a.out = d_out;
    a.ffn_norm = d_ffn_norm;
    a.eps = c.rms_eps;
    a.router = static_cast<const uint16_t*>(d_router);
    a.bias = d_router_bias;
    a.experts = static_cast<const uint8_t*>(d_experts);
    a.stride = c.expert_stride;
    a.D = c.dim;
    a.H = c.expert_hidden;
    a.E = c.n_experts;
    a.K = c.top_k;
    a.norm_topk = c.norm_topk;
    a.logits = reinterpret_cast<float*>(base + l.logits);
    a.partials = reinterpret_cast<float*>(base + l.partials);
    a.idx = reinterpret_cast<int32_t*>(base + l.idx);
    a.counts = reinterpret_cast<int32_t*>(base + l.counts);
    a.offsets = reinterpret_cast<int32_t*>(base + l.offsets);
    a.perm = reinterpret_cast<int32_t*>(base + l.perm);
    a.slot_pos = reinterpret_cast<int32_t*>(base + l.slot_pos);
    a.active = reinterpret_cast<int32_t*>(base + l.active);
    a.n_active = reinterpret_cast<int32_t*>(base + l.n_active);
    a.wt = reinterpret_cast<float*>(base + l.wt);
    a.routing_out = d_routing_out;
    a.sync = reinterpret_cast<unsigned*>(base + l.sync);
    a.status = reinterpret_cast<unsigned*>(base + l.status);
    err = rbt::launch_decode_fused(a, w2map, setup.sm_count, s);
    if (err != cudaSuccess) return fail("rbt_moe_decode_noalloc: launch failed: %s", cudaGetErrorString(err));
    return 1;
}

namespace {

bool device_setup(DeviceSetup* out) {
    // once per device and context, with that device current: the device address of the array
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return fail("rbt_moe_decode_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(err));
    if (dev < 0 || dev >= kMaxDevices) return fail("rbt_moe_decode_noalloc: device %d beyond %d", dev, kMaxDevices);
    // a runtime call first makes the device's primary context current
    int sms = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess)
        return fail("rbt_moe_decode_noalloc: cannot query device %d: %s", dev, cudaGetErrorString(err));
    void* ctx = current_context();
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_setup[dev].scratch || g_setup[dev].ctx != ctx) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess)
            return fail("rbt_moe_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                        cudaGetErrorString(err));
        g_setup[dev].scratch = p;
        g_setup[dev].ctx = ctx;
        g_setup[dev].sm_count = sms;
    }
    *out = g_setup[dev];
    return true;
}

}  // namespace

extern "C" int rbt_moe_decode_noalloc_status(void* stream, unsigned* status_out) {
    if (!status_out) return fail("rbt_moe_decode_noalloc_status: null argument");
    DeviceSetup setup;
    if (!device_setup(&setup)) return 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaMemcpyAsync(status_out, setup.scratch, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess)
        return fail("rbt_moe_decode_noalloc_status: reading the status word failed: %s", cudaGetErrorString(err));
    return 1;
}
