// gw_api.cu — the C-ABI declared in include/godwit_cuda.h.
//
// Host-side replacement for the reference's ExpertRunner / Router / the MoE
// half of TransformerLayer.forward, and for ExpertCache + ModelReader: the
// expert bank is resident in HBM, so a forward call never waits on storage.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/godwit_cuda.h"
#include "gw_internal.h"

namespace {

thread_local std::string g_last_error;

gw_status fail(gw_status code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

gw_status cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? GW_E_OOM : GW_E_CUDA, "%s: %s", what,
                cudaGetErrorString(e));
}

#define GW_CUDA(call)                                        \
    do {                                                     \
        cudaError_t _e = (call);                             \
        if (_e != cudaSuccess) return cuda_fail(_e, #call);  \
    } while (0)

// Device buffer that grows on demand and is released with its owner.
struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= n) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e == cudaSuccess) n = bytes;
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

struct gw_ctx {
    int device = 0;
    cudaStream_t own = nullptr;
    cudaStream_t cur = nullptr;
    std::recursive_mutex mu;
    DevBuf work;        // MoE scratch (MoeWork)
    DevBuf staging;     // inputs/outputs of the synchronous API
    DevBuf gemv_x;      // f16 x + block scales of GEMV calls
    unsigned* status = nullptr;  // sticky bits of bounded device waits that gave up
    int work_tcap = 0, work_H = 0, work_F = 0, work_E = 0, work_k = 0;
    gw::MoeWork w{};
    int sms = 148;          // persistent grid of the tensor-core expert kernels
    int mma_min_avg = 8;    // tensor-core expert path when T*k >= mma_min_avg * E
    int block_scaled = 0;   // tensor-core path: block-scaled MXFP4 x MXFP8 instead of exact f16
    int64_t launches = 0;
    // profiling (gw_profile_enable): event pairs per timed launch
    bool prof = false;
    struct Timed { int kind; cudaEvent_t a, b; int64_t units; };
    std::vector<Timed> timed;
    DevBuf nlog;              // nactive per profiled layer
    int nlog_used = 0;
    gw_profile acc{};
    // CUDA graph of the last stack forward (replayed while its inputs match)
    struct StackGraph {
        cudaGraphExec_t exec = nullptr;
        const void* bank = nullptr;
        const void* x = nullptr;
        const float* stream = nullptr;
        cudaStream_t on = nullptr;
        int T = 0, dtype = -1;
        int64_t kernels = 0;
        void* work = nullptr;
    } graph;
};

struct gw_bank {
    gw_ctx* ctx = nullptr;
    gw_bank_desc d{};
    int e_local = 0;
    std::vector<uint8_t*> layer_mem;  // [L] each E_local * stride bytes
    std::vector<uint8_t*> rowexp;     // [L] each E_local * (2F + H): largest scale exponent per row
    uint16_t* router_w = nullptr;     // [L][E][H]
    uint16_t* router_b = nullptr;     // [L][E]
    int64_t bytes = 0;
    DevBuf stage;                     // one stride in the reference layout (upload/download/fill)
};

namespace {

struct CtxLock {
    std::lock_guard<std::recursive_mutex> g;
    explicit CtxLock(gw_ctx* c) : g(c->mu) {}
};

gw_status set_device(gw_ctx* c) {
    GW_CUDA(cudaSetDevice(c->device));
    return GW_OK;
}

gw::MoeDims dims_of(const gw_bank* b) {
    gw::MoeDims m;
    m.H = b->d.hidden;
    m.F = b->d.intermediate;
    m.E = b->d.experts;
    m.k = b->d.top_k;
    m.act = b->d.activation;
    m.limit = b->d.limit;
    m.alpha = b->d.alpha;
    m.shard_rank = b->d.shard_rank;
    m.shard_count = b->d.shard_count;
    return m;
}

gw::LayerView layer_of(const gw_bank* b, int layer) {
    gw::LayerView v;
    v.base = b->layer_mem[layer];
    v.stride = b->d.expert_stride;
    for (int i = 0; i < 6; ++i) v.off[i] = b->d.section_offset[i];
    v.router_w = b->router_w + (int64_t)layer * b->d.experts * b->d.hidden;
    v.router_b = b->d.has_router_bias ? b->router_b + (int64_t)layer * b->d.experts : nullptr;
    v.rowexp = b->rowexp[layer];
    v.rowexp_stride = 2 * (int64_t)b->d.intermediate + b->d.hidden;
    return v;
}

// Carves the MoE scratch for T tokens out of one allocation.
gw_status ensure_work(gw_ctx* c, const gw_bank* b, int T) {
    const int H = b->d.hidden, F = b->d.intermediate, E = b->d.experts, k = b->d.top_k;
    if (c->w.logits && T <= c->work_tcap && H <= c->work_H && F <= c->work_F && E <= c->work_E &&
        k <= c->work_k)
        return GW_OK;
    const int tcap = std::max(T, std::max(c->work_tcap, 1));
    const int Hc = std::max(H, c->work_H), Fc = std::max(F, c->work_F);
    const int Ec = std::max(E, c->work_E), kc = std::max(k, c->work_k);
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
    const size_t o_xr = take((size_t)tcap * Hc * 2);
    const size_t o_x16 = take((size_t)tcap * Hc * 2);
    const size_t o_xmul = take((size_t)tcap * 4);
    const size_t o_logits = take((size_t)tcap * Ec * 4);
    const size_t o_experts = take((size_t)tcap * kc * 4);
    const size_t o_weights = take((size_t)tcap * kc * 4);
    const size_t o_counts = take((size_t)Ec * 4);
    const size_t o_active = take((size_t)Ec * 4);
    const size_t o_nactive = take(8);  // nactive, nextra
    const size_t o_extra = take(((size_t)tcap * kc / gw::kGemvPass + 1) * 4);
    const size_t o_lists = take((size_t)Ec * tcap * 4);
    const size_t o_act = take((size_t)tcap * kc * Fc * 2);
    const size_t o_ybuf = take((size_t)tcap * kc * Hc * 4);
    const size_t o_xg = take((size_t)tcap * kc * Hc * 2);
    const size_t o_xq = take((size_t)tcap * kc * Hc);
    const size_t o_xsf = take((size_t)tcap * kc * ((Hc + 127) / 128) * 4);
    const size_t o_aq = take((size_t)tcap * kc * Fc);
    const size_t o_asf = take((size_t)tcap * kc * ((Fc + 127) / 128) * 4);
    const size_t o_done = take((size_t)(tcap / 8 + 1) * 4);
    const size_t o_sched = take(8);
    cudaError_t e = c->work.ensure(off);
    if (e != cudaSuccess) return cuda_fail(e, "workspace allocation");
    char* base = static_cast<char*>(c->work.p);
    GW_CUDA(cudaMemsetAsync(base + o_done, 0, (size_t)(tcap / 8 + 1) * 4, c->cur));
    GW_CUDA(cudaMemsetAsync(base + o_nactive, 0, 8, c->cur));
    GW_CUDA(cudaMemsetAsync(base + o_counts, 0, (size_t)Ec * 4, c->cur));
    GW_CUDA(cudaMemsetAsync(base + o_sched, 0, 8, c->cur));
    gw::MoeWork& w = c->w;
    w.tcap = tcap;
    w.xr = base + o_xr;
    w.x16 = reinterpret_cast<__half*>(base + o_x16);
    w.xmul = reinterpret_cast<float*>(base + o_xmul);
    w.logits = reinterpret_cast<float*>(base + o_logits);
    w.experts = reinterpret_cast<int32_t*>(base + o_experts);
    w.weights = reinterpret_cast<float*>(base + o_weights);
    w.counts = reinterpret_cast<int32_t*>(base + o_counts);
    w.active = reinterpret_cast<int32_t*>(base + o_active);
    w.nactive = reinterpret_cast<int32_t*>(base + o_nactive);
    w.nextra = w.nactive + 1;
    w.extra = reinterpret_cast<int32_t*>(base + o_extra);
    w.lists = reinterpret_cast<int32_t*>(base + o_lists);
    w.act = reinterpret_cast<__half*>(base + o_act);
    w.ybuf = reinterpret_cast<float*>(base + o_ybuf);
    w.xg = reinterpret_cast<__half*>(base + o_xg);
    w.xq = reinterpret_cast<uint8_t*>(base + o_xq);
    w.xsf = reinterpret_cast<uint32_t*>(base + o_xsf);
    w.aq = reinterpret_cast<uint8_t*>(base + o_aq);
    w.asf = reinterpret_cast<uint32_t*>(base + o_asf);
    w.done = reinterpret_cast<unsigned*>(base + o_done);
    w.sched = reinterpret_cast<unsigned*>(base + o_sched);
    w.status = c->status;
    w.mma_min_avg = c->mma_min_avg;
    w.block_scaled = c->block_scaled;
    c->work_tcap = tcap;
    c->work_H = Hc;
    c->work_F = Fc;
    c->work_E = Ec;
    c->work_k = kc;
    return GW_OK;
}

gw_status count(gw_ctx* c, int n) {
    if (n < 0) return cuda_fail(cudaGetLastError(), "kernel launch");
    c->launches += n;
    return GW_OK;
}

gw_status check_bank(gw_bank* b, int layer) {
    if (!b || !b->ctx) return fail(GW_E_ARG, "null bank");
    if (layer < 0 || layer >= b->d.layers)
        return fail(GW_E_ARG, "layer %d out of range [0, %d)", layer, b->d.layers);
    return GW_OK;
}

// The expert kernels read activations and write outputs 16 bytes at a time.
gw_status check_align16(const void* p, const char* what) {
    if (reinterpret_cast<uintptr_t>(p) % 16)
        return fail(GW_E_ARG, "%s (%p) must be 16-byte aligned", what, p);
    return GW_OK;
}

gw_status check_dtype(int x_dtype) {
    if (x_dtype != GW_DTYPE_F16 && x_dtype != GW_DTYPE_BF16)
        return fail(GW_E_ARG, "x_dtype %d is neither GW_DTYPE_F16 nor GW_DTYPE_BF16", x_dtype);
    return GW_OK;
}

// Records an event pair around `launch` when profiling (kind: 0 gate_up,
// 1 down, 2 gemv, 3 router/grouping, 4 combine).
template <class F>
gw_status timed_launch(gw_ctx* c, int kind, int64_t units, F&& launch) {
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (c->prof) {
        GW_CUDA(cudaEventCreate(&e0));
        GW_CUDA(cudaEventCreate(&e1));
        GW_CUDA(cudaEventRecord(e0, c->cur));
    }
    gw_status st = count(c, launch());
    if (st) return st;
    if (c->prof) {
        GW_CUDA(cudaEventRecord(e1, c->cur));
        c->timed.push_back({kind, e0, e1, units});
    }
    return GW_OK;
}

// Appends this layer's number of active experts to the profile log.
gw_status log_nactive(gw_ctx* c) {
    const size_t need = (size_t)(c->nlog_used + 1) * 4;
    if (need > c->nlog.n) {
        DevBuf bigger;
        cudaError_t e = bigger.ensure(std::max<size_t>(need * 2, 4096));
        if (e != cudaSuccess) return cuda_fail(e, "profile log allocation");
        if (c->nlog_used)
            GW_CUDA(cudaMemcpyAsync(bigger.p, c->nlog.p, (size_t)c->nlog_used * 4,
                                    cudaMemcpyDeviceToDevice, c->cur));
        GW_CUDA(cudaStreamSynchronize(c->cur));
        c->nlog.release();
        c->nlog = bigger;
    }
    GW_CUDA(cudaMemcpyAsync(static_cast<int32_t*>(c->nlog.p) + c->nlog_used, c->w.nactive, 4,
                            cudaMemcpyDeviceToDevice, c->cur));
    c->nlog_used += 1;
    return GW_OK;
}

// Router + grouping (or grouping of a supplied routing), experts, combine —
// the device half of one MoE layer.  x_dev is [T][H] in x_dtype (f16 or
// bf16).  out (=, or += when accumulate) receives the weighted expert sum;
// if x_next is given it receives round(out) in x_dtype.
gw_status moe_layer_device(gw_ctx* c, gw_bank* b, int layer, const void* x_dev, int x_dtype,
                           int T, const int32_t* experts_in, const float* weights_in, float* out,
                           int accumulate, void* x_next, int64_t slots_hint = -1) {
    const gw::MoeDims d = dims_of(b);
    const gw::LayerView L = layer_of(b, layer);
    gw_status st = ensure_work(c, b, T);
    if (st) return st;
    gw::MoeWork& w = c->w;
    if (experts_in) {
        st = count(c, gw::launch_xprep(x_dev, x_dtype, T, d.H, w.x16, w.xmul, c->cur));
        if (st) return st;
        st = timed_launch(c, 3, 0, [&] { return gw::launch_group(d, experts_in, weights_in, T, w, c->cur); });
    }
    else
        st = timed_launch(c, 3, 0, [&] { return gw::launch_router(L, d, x_dev, x_dtype, T, w, c->cur); });
    if (st) return st;
    // Many tokens per expert: the tensor-core grouped GEMMs; few: the GEMV tiles.
    // the slots the layer will compute, at most T * k
    const int64_t slots = slots_hint >= 0 ? slots_hint : (int64_t)T * d.k;
    const bool mma = w.mma_min_avg > 0 && slots >= (int64_t)w.mma_min_avg * d.E &&
                     gw::grouped_supported(d, w);
    // A handful of slots (batch 1-2): the small-batch GEMV tiles, whose
    // launches start streaming sooner than the persistent TMA-fed kernel's.
    const bool small = !mma && slots <= gw::kSmallBatchSlots;
    if ((st = timed_launch(c, 0, 0, [&] {
             return mma     ? gw::launch_grouped(L, d, w, 0, c->sms, c->cur, x_dev, x_dtype)
                    : small ? gw::launch_gateup(L, d, x_dev, x_dtype, T, w, c->cur)
                            : gw::launch_expert_gemv(L, d, w, T, 0, c->cur);
         })))
        return st;
    if ((st = timed_launch(c, 1, 0, [&] {
             return mma     ? gw::launch_grouped(L, d, w, 1, c->sms, c->cur)
                    : small ? gw::launch_down(L, d, T, w, c->cur)
                            : gw::launch_expert_gemv(L, d, w, T, 1, c->cur);
         })))
        return st;
    if (c->prof && (st = log_nactive(c))) return st;
    return timed_launch(c, 4, 0, [&] {
        return gw::launch_combine(d, T, w, out, accumulate, x_next, x_dtype, c->cur);
    });
}

}  // namespace

// Staging area for the synchronous calls: carves consecutive device regions.
namespace {
size_t dtype_size(int) { return 2; }

struct Stage {
    gw_ctx* c;
    size_t off = 0;
    std::vector<std::pair<size_t, size_t>> regions;
    explicit Stage(gw_ctx* cc) : c(cc) {}
    size_t add(size_t bytes) {
        const size_t o = off;
        off += align256(bytes);
        return o;
    }
    cudaError_t alloc() { return c->staging.ensure(std::max<size_t>(off, 256)); }
    template <class T>
    T* at(size_t o) { return reinterpret_cast<T*>(static_cast<char*>(c->staging.p) + o); }
};
}  // namespace

// Destroys the recorded events (consecutive kernels share one) once each.
static void drop_timed(gw_ctx* c) {
    std::vector<cudaEvent_t> evs;
    for (auto& t : c->timed) { evs.push_back(t.a); evs.push_back(t.b); }
    std::sort(evs.begin(), evs.end());
    evs.erase(std::unique(evs.begin(), evs.end()), evs.end());
    for (auto e : evs) cudaEventDestroy(e);
    c->timed.clear();
}

extern "C" {

const char* gw_last_error(void) { return g_last_error.c_str(); }

int32_t gw_version(void) { return 200; }

gw_status gw_init(int32_t device, gw_ctx** out) {
    if (!out) return fail(GW_E_ARG, "null output pointer");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(GW_E_ARG, "device %d out of range [0, %d)", device, n);
    GW_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    GW_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(GW_E_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
    if (gw::configure_kernels() != 0 || gw::configure_grouped() != 0 || gw::configure_expert_gemv() != 0 ||
        gw::configure_int8() != 0)
        return cuda_fail(cudaGetLastError(), "kernel attributes");
    gw_ctx* c = new gw_ctx();
    c->device = device;
    c->sms = prop.multiProcessorCount;
    e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "cudaStreamCreate");
    }
    e = cudaMalloc(&c->status, 4);
    if (e == cudaSuccess) e = cudaMemset(c->status, 0, 4);
    if (e != cudaSuccess) {
        cudaStreamDestroy(c->own);
        if (c->status) cudaFree(c->status);
        delete c;
        return cuda_fail(e, "status word allocation");
    }
    c->cur = c->own;
    *out = c;
    g_last_error.clear();
    return GW_OK;
}

gw_status gw_shutdown(gw_ctx* c) {
    if (!c) return fail(GW_E_ARG, "null context");
    {
        CtxLock lk(c);
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->cur);
        drop_timed(c);
        if (c->graph.exec) cudaGraphExecDestroy(c->graph.exec);
        c->nlog.release();
        c->work.release();
        c->staging.release();
        c->gemv_x.release();
        if (c->status) cudaFree(c->status);
        cudaStreamDestroy(c->own);
    }
    delete c;
    return GW_OK;
}

gw_status gw_ctx_set_stream(gw_ctx* c, void* stream) {
    if (!c) return fail(GW_E_ARG, "null context");
    CtxLock lk(c);
    c->cur = stream ? static_cast<cudaStream_t>(stream) : c->own;
    return GW_OK;
}

gw_status gw_sync(gw_ctx* c) {
    if (!c) return fail(GW_E_ARG, "null context");
    CtxLock lk(c);
    GW_CUDA(cudaSetDevice(c->device));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    // a bounded wait inside one of the context's kernels ran out
    unsigned bits = 0;
    GW_CUDA(cudaMemcpy(&bits, c->status, 4, cudaMemcpyDeviceToHost));
    if (bits) {
        GW_CUDA(cudaMemset(c->status, 0, 4));
        return fail(GW_E_TIMEOUT, "a device-side wait gave up (status bits 0x%x)", bits);
    }
    return GW_OK;
}

gw_status gw_selftest_wait_timeout(gw_ctx* c, int64_t wait_cycles) {
    if (!c) return fail(GW_E_ARG, "null context");
    if (wait_cycles < 0 || wait_cycles > 100000000)
        return fail(GW_E_ARG, "wait_cycles %lld outside [0, 1e8]", (long long)wait_cycles);
    CtxLock lk(c);
    gw_status st = set_device(c);
    if (st) return st;
    return count(c, gw::launch_wait_probe(c->status, wait_cycles, c->cur));
}

gw_status gw_set_block_scaled(gw_ctx* c, int32_t enable) {
    if (!c) return fail(GW_E_ARG, "null context");
    CtxLock lk(c);
    c->block_scaled = enable != 0;
    c->w.block_scaled = c->block_scaled;
    if (c->graph.exec) {  // a captured stack forward baked the old choice in
        cudaGraphExecDestroy(c->graph.exec);
        c->graph = gw_ctx::StackGraph{};
    }
    return GW_OK;
}

gw_status gw_set_tensor_core_min_tokens(gw_ctx* c, int32_t min_avg) {
    if (!c) return fail(GW_E_ARG, "null context");
    if (min_avg < 0) return fail(GW_E_ARG, "min_avg must be >= 0");
    CtxLock lk(c);
    c->mma_min_avg = min_avg;
    c->w.mma_min_avg = min_avg;
    if (c->graph.exec) {  // a captured stack forward baked the old choice in
        cudaGraphExecDestroy(c->graph.exec);
        c->graph = gw_ctx::StackGraph{};
    }
    return GW_OK;
}

gw_status gw_profile_enable(gw_ctx* c, int32_t enable) {
    if (!c) return fail(GW_E_ARG, "null context");
    CtxLock lk(c);
    GW_CUDA(cudaSetDevice(c->device));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    drop_timed(c);
    c->nlog_used = 0;
    c->acc = gw_profile{};
    c->prof = enable != 0;
    return GW_OK;
}

gw_status gw_profile_read(gw_ctx* c, gw_profile* out) {
    if (!c || !out) return fail(GW_E_ARG, "null argument");
    CtxLock lk(c);
    GW_CUDA(cudaSetDevice(c->device));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    for (auto& t : c->timed) {
        float ms = 0.f;
        GW_CUDA(cudaEventElapsedTime(&ms, t.a, t.b));
        if (t.kind == 0) { c->acc.gateup_launches++; c->acc.gateup_ms += ms; }
        else if (t.kind == 1) { c->acc.down_launches++; c->acc.down_ms += ms; }
        else if (t.kind == 2) { c->acc.gemv_launches++; c->acc.gemv_ms += ms; c->acc.gemv_matrices += t.units; }
        else if (t.kind == 3) { c->acc.router_launches++; c->acc.router_ms += ms; }
        else { c->acc.combine_launches++; c->acc.combine_ms += ms; }
    }
    drop_timed(c);
    if (c->nlog_used) {
        std::vector<int32_t> h(c->nlog_used);
        GW_CUDA(cudaMemcpy(h.data(), c->nlog.p, h.size() * 4, cudaMemcpyDeviceToHost));
        for (int32_t v : h) c->acc.expert_passes += v;
        c->nlog_used = 0;
    }
    *out = c->acc;
    return GW_OK;
}

gw_status gw_last_launch_count(gw_ctx* c, int64_t* out) {
    if (!c || !out) return fail(GW_E_ARG, "null argument");
    *out = c->launches;
    return GW_OK;
}

gw_status gw_layout_default(int32_t hidden, int32_t intermediate, int32_t experts,
                            int32_t layers, int32_t top_k, int32_t activation,
                            gw_bank_desc* out) {
    if (!out) return fail(GW_E_ARG, "null output");
    if (hidden <= 0 || intermediate <= 0 || hidden % 32 || intermediate % 32)
        return fail(GW_E_ARG, "hidden (%d) and intermediate (%d) must be positive multiples of 32",
                    hidden, intermediate);
    std::memset(out, 0, sizeof *out);
    out->hidden = hidden;
    out->intermediate = intermediate;
    out->experts = experts;
    out->layers = layers;
    out->top_k = top_k;
    out->activation = activation;
    out->limit = 7.0f;
    out->alpha = 1.702f;
    out->has_router_bias = activation == GW_ACT_GPTOSS_CLAMPED ? 1 : 0;
    out->shard_rank = 0;
    out->shard_count = 1;
    // ExpertLayout.init (Install/InstallLayout.swift:56-91): six sections, each
    // starting on a 16 KiB page, stride rounded up to a page.
    const int64_t page = 16384;
    const int64_t gu_rows = 2LL * intermediate, dn_rows = hidden;
    const int64_t sizes[6] = {
        gu_rows * (hidden / 32) * 16, gu_rows * (hidden / 32),
        dn_rows * (intermediate / 32) * 16, dn_rows * (intermediate / 32),
        gu_rows * 2, dn_rows * 2};
    int64_t cursor = 0;
    for (int i = 0; i < 6; ++i) {
        cursor = (cursor + page - 1) / page * page;
        out->section_offset[i] = cursor;
        out->section_length[i] = sizes[i];
        cursor += sizes[i];
    }
    out->expert_stride = (cursor + page - 1) / page * page;
    return GW_OK;
}

gw_status gw_bank_create(gw_ctx* c, const gw_bank_desc* d, gw_bank** out) {
    if (!c || !d || !out) return fail(GW_E_ARG, "null argument");
    if (d->hidden <= 0 || d->hidden % 32 || d->intermediate <= 0 || d->intermediate % 32)
        return fail(GW_E_ARG, "hidden and intermediate must be positive multiples of 32");
    if (d->hidden > gw::kMaxGemvCols || d->intermediate > gw::kMaxGemvCols)
        return fail(GW_E_UNSUPPORTED, "hidden (%d) and intermediate (%d) above %d are not supported",
                    d->hidden, d->intermediate, gw::kMaxGemvCols);
    if (d->experts <= 0 || d->experts > gw::kMaxExperts)
        return fail(GW_E_ARG, "experts %d outside [1, %d]", d->experts, gw::kMaxExperts);
    if (d->top_k <= 0 || d->top_k > gw::kMaxTopK || d->top_k > d->experts)
        return fail(GW_E_ARG, "top_k %d outside [1, min(%d, experts)]", d->top_k, gw::kMaxTopK);
    if (d->layers <= 0) return fail(GW_E_ARG, "layers must be positive");
    if (d->activation != GW_ACT_GPTOSS_CLAMPED && d->activation != GW_ACT_SILU)
        return fail(GW_E_ARG, "unknown activation %d", d->activation);
    if (d->shard_count <= 0 || d->shard_rank < 0 || d->shard_rank >= d->shard_count)
        return fail(GW_E_ARG, "bad shard %d of %d", d->shard_rank, d->shard_count);
    const int64_t H = d->hidden, F = d->intermediate;
    const int64_t need[6] = {2 * F * (H / 32) * 16, 2 * F * (H / 32), H * (F / 32) * 16,
                             H * (F / 32), 2 * F * 2, H * 2};
    for (int i = 0; i < 6; ++i) {
        if (d->section_length[i] < need[i])
            return fail(GW_E_ARG, "section %d holds %lld bytes, needs %lld", i,
                        (long long)d->section_length[i], (long long)need[i]);
        if (d->section_offset[i] < 0 || d->section_offset[i] + need[i] > d->expert_stride)
            return fail(GW_E_ARG, "section %d does not fit in the %lld-byte stride", i,
                        (long long)d->expert_stride);
        if (d->section_offset[i] % 16)
            return fail(GW_E_ARG, "section %d offset %lld is not 16-byte aligned", i,
                        (long long)d->section_offset[i]);
    }
    if (d->expert_stride % 16) return fail(GW_E_ARG, "expert stride must be a multiple of 16");
    CtxLock lk(c);
    gw_status st = set_device(c);
    if (st) return st;
    gw_bank* b = new gw_bank();
    b->ctx = c;
    b->d = *d;
    b->e_local = (d->experts - d->shard_rank + d->shard_count - 1) / d->shard_count;
    const size_t per_layer = (size_t)b->e_local * d->expert_stride;
    const size_t rexp_layer = (size_t)b->e_local * (2 * F + H);
    b->layer_mem.assign(d->layers, nullptr);
    b->rowexp.assign(d->layers, nullptr);
    for (int l = 0; l < d->layers; ++l) {
        // 256 bytes of tail: the tensor-core path reads scale bytes in
        // aligned 16-byte windows that may reach past the last row
        cudaError_t e = cudaMalloc(&b->layer_mem[l], per_layer + 256);
        if (e == cudaSuccess) e = cudaMalloc(&b->rowexp[l], std::max<size_t>(rexp_layer, 256));
        if (e == cudaSuccess) e = cudaMemsetAsync(b->rowexp[l], 127, std::max<size_t>(rexp_layer, 256), c->cur);
        if (e != cudaSuccess) {
            gw_bank_destroy(b);
            return cuda_fail(e, "bank layer allocation");
        }
        b->bytes += per_layer + rexp_layer;
    }
    const size_t rw = (size_t)d->layers * d->experts * d->hidden * 2;
    const size_t rb = (size_t)d->layers * d->experts * 2;
    cudaError_t e = cudaMalloc(&b->router_w, rw);
    if (e == cudaSuccess) e = cudaMalloc(&b->router_b, rb);
    if (e != cudaSuccess) {
        gw_bank_destroy(b);
        return cuda_fail(e, "router allocation");
    }
    e = cudaMemsetAsync(b->router_b, 0, rb, c->cur);
    if (e == cudaSuccess) e = cudaMemsetAsync(b->router_w, 0, rw, c->cur);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->cur);
    if (e != cudaSuccess) {
        gw_bank_destroy(b);
        return cuda_fail(e, "router initialisation");
    }
    b->bytes += rw + rb;
    *out = b;
    return GW_OK;
}

gw_status gw_bank_destroy(gw_bank* b) {
    if (!b) return fail(GW_E_ARG, "null bank");
    if (b->ctx) {
        CtxLock lk(b->ctx);
        if (b->ctx->graph.bank == b) {
            if (b->ctx->graph.exec) cudaGraphExecDestroy(b->ctx->graph.exec);
            b->ctx->graph = gw_ctx::StackGraph{};
        }
        cudaSetDevice(b->ctx->device);
        cudaStreamSynchronize(b->ctx->cur);
        for (uint8_t* p : b->layer_mem)
            if (p) cudaFree(p);
        for (uint8_t* p : b->rowexp)
            if (p) cudaFree(p);
        if (b->router_w) cudaFree(b->router_w);
        if (b->router_b) cudaFree(b->router_b);
        b->stage.release();
    }
    delete b;
    return GW_OK;
}

static gw_status expert_ptr(gw_bank* b, int layer, int expert, uint8_t** out) {
    gw_status st = check_bank(b, layer);
    if (st) return st;
    if (expert < 0 || expert >= b->d.experts)
        return fail(GW_E_ARG, "expert %d out of range [0, %d)", expert, b->d.experts);
    if (expert % b->d.shard_count != b->d.shard_rank)
        return fail(GW_E_ARG, "expert %d is not resident on shard %d of %d", expert,
                    b->d.shard_rank, b->d.shard_count);
    *out = b->layer_mem[layer] + (int64_t)(expert / b->d.shard_count) * b->d.expert_stride;
    return GW_OK;
}

static uint8_t* rowexp_ptr(gw_bank* b, int layer, int expert) {
    return b->rowexp[layer] +
           (int64_t)(expert / b->d.shard_count) * (2 * (int64_t)b->d.intermediate + b->d.hidden);
}

// Converts one expert between the reference's installed stride (`ref`) and
// the bank's resident form (`bank`): the four MXFP4 sections in the tiled
// layout (tile_layout_offset in gw_device.cuh), the biases unchanged.
static gw_status relayout_expert(gw_bank* b, const uint8_t* src, uint8_t* dst, int to_tiled,
                                 uint8_t* rowexp = nullptr) {
    gw_ctx* c = b->ctx;
    const int H = b->d.hidden, F = b->d.intermediate;
    const int64_t* off = b->d.section_offset;
    if (rowexp) {  // per-row exponent maxima from the reference-layout scales
        gw_status st = count(c, gw::launch_rowexp(src + off[1], 2 * F, H, rowexp, c->cur));
        if (!st) st = count(c, gw::launch_rowexp(src + off[3], H, F, rowexp + 2 * F, c->cur));
        if (st) return st;
    }
    const int rows[4] = {2 * F, 2 * F, H, H}, cols[4] = {H, H, F, F}, is_scale[4] = {0, 1, 0, 1};
    for (int s = 0; s < 4; ++s) {
        gw_status st = count(c, gw::launch_tile_layout(src + off[s], dst + off[s], rows[s], cols[s],
                                                       is_scale[s], to_tiled, c->cur));
        if (st) return st;
    }
    for (int s = 4; s < 6; ++s)
        GW_CUDA(cudaMemcpyAsync(dst + off[s], src + off[s], b->d.section_length[s],
                                cudaMemcpyDeviceToDevice, c->cur));
    return GW_OK;
}

static gw_status bank_stage(gw_bank* b) {
    cudaError_t e = b->stage.ensure((size_t)b->d.expert_stride);
    if (e != cudaSuccess) return cuda_fail(e, "bank staging allocation");
    return GW_OK;
}

gw_status gw_bank_upload_expert(gw_bank* b, int32_t layer, int32_t expert, const void* bytes,
                                size_t len) {
    uint8_t* dst;
    gw_status st = expert_ptr(b, layer, expert, &dst);
    if (st) return st;
    if (!bytes) return fail(GW_E_ARG, "null stride bytes");
    if ((int64_t)len != b->d.expert_stride)
        return fail(GW_E_ARG, "stride is %zu bytes, the bank expects %lld", len,
                    (long long)b->d.expert_stride);
    CtxLock lk(b->ctx);
    if ((st = set_device(b->ctx)) || (st = bank_stage(b))) return st;
    uint8_t* stage = static_cast<uint8_t*>(b->stage.p);
    GW_CUDA(cudaMemcpyAsync(stage, bytes, len, cudaMemcpyHostToDevice, b->ctx->cur));
    if ((st = relayout_expert(b, stage, dst, 1, rowexp_ptr(b, layer, expert)))) return st;
    GW_CUDA(cudaStreamSynchronize(b->ctx->cur));
    return GW_OK;
}

gw_status gw_bank_download_expert(gw_bank* b, int32_t layer, int32_t expert, void* bytes,
                                  size_t len) {
    uint8_t* src;
    gw_status st = expert_ptr(b, layer, expert, &src);
    if (st) return st;
    if (!bytes || (int64_t)len != b->d.expert_stride)
        return fail(GW_E_ARG, "destination must hold exactly one stride");
    CtxLock lk(b->ctx);
    if ((st = set_device(b->ctx)) || (st = bank_stage(b))) return st;
    uint8_t* stage = static_cast<uint8_t*>(b->stage.p);
    if ((st = relayout_expert(b, src, stage, 0))) return st;
    GW_CUDA(cudaMemcpyAsync(bytes, stage, len, cudaMemcpyDeviceToHost, b->ctx->cur));
    GW_CUDA(cudaStreamSynchronize(b->ctx->cur));
    return GW_OK;
}

gw_status gw_bank_upload_router(gw_bank* b, int32_t layer, const uint16_t* w, const uint16_t* bias) {
    gw_status st = check_bank(b, layer);
    if (st) return st;
    if (!w) return fail(GW_E_ARG, "null router weight");
    CtxLock lk(b->ctx);
    if ((st = set_device(b->ctx))) return st;
    const size_t nw = (size_t)b->d.experts * b->d.hidden;
    GW_CUDA(cudaMemcpyAsync(b->router_w + layer * nw, w, nw * 2, cudaMemcpyHostToDevice, b->ctx->cur));
    uint16_t* bd = b->router_b + (size_t)layer * b->d.experts;
    if (bias)
        GW_CUDA(cudaMemcpyAsync(bd, bias, b->d.experts * 2, cudaMemcpyHostToDevice, b->ctx->cur));
    else
        GW_CUDA(cudaMemsetAsync(bd, 0, b->d.experts * 2, b->ctx->cur));
    GW_CUDA(cudaStreamSynchronize(b->ctx->cur));
    return GW_OK;
}

gw_status gw_bank_fill_synthetic(gw_bank* b, uint64_t seed) {
    if (!b || !b->ctx) return fail(GW_E_ARG, "null bank");
    CtxLock lk(b->ctx);
    gw_ctx* c = b->ctx;
    gw_status st = set_device(c);
    if (st) return st;
    if ((st = bank_stage(b))) return st;
    uint8_t* stage = static_cast<uint8_t*>(b->stage.p);
    const int kinds[6] = {gw::kFillCodes, gw::kFillScales, gw::kFillCodes, gw::kFillScales,
                          gw::kFillBf16Normal, gw::kFillBf16Normal};
    for (int l = 0; l < b->d.layers; ++l) {
        for (int e = b->d.shard_rank; e < b->d.experts; e += b->d.shard_count) {
            // generate the reference-layout stride, then lay it out in the bank
            uint8_t* ex = b->layer_mem[l] + (int64_t)(e / b->d.shard_count) * b->d.expert_stride;
            for (int s = 0; s < 6; ++s) {
                const uint64_t key = gw::mix64(seed ^ gw::mix64(((uint64_t)l << 40) |
                                                                ((uint64_t)e << 8) | (uint64_t)s));
                int kind = kinds[s];
                if (s >= 4 && b->d.activation == GW_ACT_SILU) kind = gw::kFillZero;
                if ((st = count(c, gw::launch_fill_bytes(stage + b->d.section_offset[s],
                                                         b->d.section_length[s], key, kind, c->cur))))
                    return st;
            }
            if ((st = relayout_expert(b, stage, ex, 1, rowexp_ptr(b, l, e)))) return st;
        }
        const uint64_t kw = gw::mix64(seed ^ gw::mix64(((uint64_t)l << 40) | (0xFFFFull << 8) | 6u));
        const uint64_t kb = gw::mix64(seed ^ gw::mix64(((uint64_t)l << 40) | (0xFFFFull << 8) | 7u));
        const size_t nw = (size_t)b->d.experts * b->d.hidden;
        if ((st = count(c, gw::launch_fill_bytes(reinterpret_cast<uint8_t*>(b->router_w + l * nw),
                                                 (int64_t)nw * 2, kw, gw::kFillBf16Normal, c->cur))))
            return st;
        if ((st = count(c, gw::launch_fill_bytes(
                 reinterpret_cast<uint8_t*>(b->router_b + (size_t)l * b->d.experts),
                 (int64_t)b->d.experts * 2, kb,
                 b->d.has_router_bias ? gw::kFillBf16Normal : gw::kFillZero, c->cur))))
            return st;
    }
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}

gw_status gw_bank_bytes(gw_bank* b, int64_t* out) {
    if (!b || !out) return fail(GW_E_ARG, "null argument");
    *out = b->bytes;
    return GW_OK;
}

// ---- device-pointer API ---------------------------------------------------

gw_status gw_moe_forward_async(gw_ctx* c, gw_bank* b, int32_t layer, const void* x_dev,
                               int32_t x_dtype, int32_t T, float* out_dev, int32_t* experts_dev,
                               float* weights_dev) {
    if (!c || !x_dev || !out_dev) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if ((st = check_align16(x_dev, "x_dev")) || (st = check_align16(out_dev, "out_dev"))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    st = moe_layer_device(c, b, layer, x_dev, x_dtype, T, nullptr, nullptr, out_dev, 0, nullptr);
    if (st) return st;
    const size_t nk = (size_t)T * b->d.top_k;
    if (experts_dev)
        GW_CUDA(cudaMemcpyAsync(experts_dev, c->w.experts, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    if (weights_dev)
        GW_CUDA(cudaMemcpyAsync(weights_dev, c->w.weights, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    return GW_OK;
}

gw_status gw_moe_stack_forward_async(gw_ctx* c, gw_bank* b, const void* x_dev, int32_t x_dtype,
                                     int32_t T, float* stream_dev) {
    if (!c || !x_dev || !stream_dev) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, 0);
    if (st || (st = check_dtype(x_dtype))) return st;
    if ((st = check_align16(x_dev, "x_dev")) || (st = check_align16(stream_dev, "stream_dev"))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    const int64_t n = (int64_t)T * b->d.hidden;
    // stream = x widened to fp32; then stream += moe_l(round(stream)) per layer.
    // Each layer's combine writes round(stream) into the workspace's x buffer,
    // which is the next layer's input.  The launch sequence is captured once
    // as a CUDA graph and replayed while the bank, buffers, stream and T are
    // unchanged (profiling runs launch eagerly so each kernel can be timed).
    if ((st = ensure_work(c, b, T))) return st;
    auto enqueue = [&]() -> gw_status {
        gw_status s2 = count(c, gw::launch_widen(x_dev, x_dtype, stream_dev, n, c->cur));
        if (s2) return s2;
        for (int l = 0; l < b->d.layers; ++l) {
            const void* src = (l == 0) ? x_dev : c->w.xr;
            void* next = (l + 1 < b->d.layers) ? c->w.xr : nullptr;
            s2 = moe_layer_device(c, b, l, src, x_dtype, T, nullptr, nullptr, stream_dev, 1, next);
            if (s2) return s2;
        }
        return GW_OK;
    };
    if (c->prof) return enqueue();
    auto& g = c->graph;
    const bool hit = g.exec && g.bank == b && g.x == x_dev && g.stream == stream_dev &&
                     g.on == c->cur && g.T == T && g.dtype == x_dtype && g.work == c->work.p;
    if (!hit) {
        if (g.exec) cudaGraphExecDestroy(g.exec);
        g.exec = nullptr;
        const int64_t before = c->launches;
        GW_CUDA(cudaStreamBeginCapture(c->cur, cudaStreamCaptureModeThreadLocal));
        st = enqueue();
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamEndCapture(c->cur, &graph);
        if (st) {
            if (graph) cudaGraphDestroy(graph);
            return st;
        }
        if (e != cudaSuccess) return cuda_fail(e, "stack graph capture");
        e = cudaGraphInstantiate(&g.exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) {
            g.exec = nullptr;
            return cuda_fail(e, "stack graph instantiation");
        }
        g.kernels = c->launches - before;
        c->launches = before;
        g.bank = b;
        g.x = x_dev;
        g.stream = stream_dev;
        g.on = c->cur;
        g.T = T;
        g.dtype = x_dtype;
        g.work = c->work.p;
    }
    GW_CUDA(cudaGraphLaunch(g.exec, c->cur));
    c->launches += g.kernels;
    return GW_OK;
}

gw_status gw_moe_apply_async(gw_ctx* c, gw_bank* b, int32_t layer, const void* x_dev,
                             int32_t x_dtype, int32_t T, const int32_t* experts_dev,
                             const float* weights_dev, float* out_dev, int32_t accumulate) {
    if (!c || !x_dev || !out_dev || !experts_dev || !weights_dev) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if ((st = check_align16(x_dev, "x_dev")) || (st = check_align16(out_dev, "out_dev"))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    // rows given to this entry point usually carry one expert each (the
    // per-rank half of expert parallelism), so the expert path is chosen as
    // for T slots rather than T * top_k
    return moe_layer_device(c, b, layer, x_dev, x_dtype, T, experts_dev, weights_dev, out_dev,
                            accumulate ? 1 : 0, nullptr, (int64_t)T);
}

gw_status gw_residual_round_async(gw_ctx* c, float* stream_dev, const float* delta_dev,
                                  void* x_out_dev, int32_t x_dtype, int64_t n) {
    if (!c || !stream_dev) return fail(GW_E_ARG, "null argument");
    gw_status st;
    if (x_out_dev && (st = check_dtype(x_dtype))) return st;
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    return count(c, gw::launch_residual_round(stream_dev, delta_dev, x_out_dev, x_dtype, n, c->cur));
}

// Argument checks shared by the RMSNorm entry points.
static gw_status check_norm(const void* stream, const void* weight, float eps, int32_t T, int32_t H) {
    if (!stream || !weight) return fail(GW_E_ARG, "null argument");
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    if (H <= 0 || H % 4) return fail(GW_E_ARG, "H = %d must be a positive multiple of 4", H);
    if (!(eps >= 0.f) || !std::isfinite(eps)) return fail(GW_E_ARG, "eps must be finite and >= 0");
    if (reinterpret_cast<uintptr_t>(stream) % 16 || reinterpret_cast<uintptr_t>(weight) % 8)
        return fail(GW_E_ARG, "stream must be 16-byte and weight 8-byte aligned");
    return GW_OK;
}

gw_status gw_rmsnorm_async(gw_ctx* c, const float* stream_dev, const uint16_t* weight_dev, float eps,
                           int32_t T, int32_t H, void* out_dev) {
    gw_status st = check_norm(stream_dev, weight_dev, eps, T, H);
    if (st) return st;
    if (!c || !out_dev) return fail(GW_E_ARG, "null argument");
    if (reinterpret_cast<uintptr_t>(out_dev) % 8) return fail(GW_E_ARG, "out must be 8-byte aligned");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    return count(c, gw::launch_rmsnorm(stream_dev, weight_dev, eps, T, H, static_cast<__half*>(out_dev),
                                       c->cur));
}

// The MoE half of TransformerLayer.forward on device memory: RMSNorm of the
// residual stream into the workspace's x buffer (f16), router + experts on
// it, and the combine adding the weighted expert sum into the stream.
static gw_status moe_block_device(gw_ctx* c, gw_bank* b, int layer, float* stream, const uint16_t* norm_w,
                                  float eps, int T) {
    gw_status st = ensure_work(c, b, T);
    if (st) return st;
    __half* xn = static_cast<__half*>(c->w.xr);
    if ((st = count(c, gw::launch_rmsnorm(stream, norm_w, eps, T, b->d.hidden, xn, c->cur)))) return st;
    return moe_layer_device(c, b, layer, xn, GW_DTYPE_F16, T, nullptr, nullptr, stream, 1, nullptr);
}

gw_status gw_moe_block_async(gw_ctx* c, gw_bank* b, int32_t layer, float* stream_dev,
                             const uint16_t* norm_w_dev, float eps, int32_t T, int32_t* experts_dev,
                             float* weights_dev) {
    if (!c) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_norm(stream_dev, norm_w_dev, eps, T, b->d.hidden))) return st;
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    if ((st = moe_block_device(c, b, layer, stream_dev, norm_w_dev, eps, T))) return st;
    const size_t nk = (size_t)T * b->d.top_k;
    if (experts_dev)
        GW_CUDA(cudaMemcpyAsync(experts_dev, c->w.experts, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    if (weights_dev)
        GW_CUDA(cudaMemcpyAsync(weights_dev, c->w.weights, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    return GW_OK;
}

gw_status gw_moe_block(gw_ctx* c, gw_bank* b, int32_t layer, float* stream, const uint16_t* norm_w,
                       float eps, int32_t T, int32_t* experts_out, float* weights_out) {
    if (!c || !stream || !norm_w) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st) return st;
    const int H = b->d.hidden;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    if (!(eps >= 0.f) || !std::isfinite(eps)) return fail(GW_E_ARG, "eps must be finite and >= 0");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    const size_t ns = (size_t)T * H * 4, nw = (size_t)H * 2, nk = (size_t)T * b->d.top_k;
    Stage sg(c);
    const size_t os = sg.add(ns), ow = sg.add(nw);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<float>(os), stream, ns, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<uint16_t>(ow), norm_w, nw, cudaMemcpyHostToDevice, c->cur));
    if ((st = moe_block_device(c, b, layer, sg.at<float>(os), sg.at<uint16_t>(ow), eps, T))) return st;
    GW_CUDA(cudaMemcpyAsync(stream, sg.at<float>(os), ns, cudaMemcpyDeviceToHost, c->cur));
    if (experts_out)
        GW_CUDA(cudaMemcpyAsync(experts_out, c->w.experts, nk * 4, cudaMemcpyDeviceToHost, c->cur));
    if (weights_out)
        GW_CUDA(cudaMemcpyAsync(weights_out, c->w.weights, nk * 4, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}

// GEMV over `count` matrices (device pointers).
static gw_status gemv_device(gw_ctx* c, int32_t count_m, const uint8_t* packed, int64_t ps,
                             const uint8_t* scales, int64_t ss, const uint16_t* bias, int64_t bs,
                             const void* x, int64_t x_stride, int32_t x_dtype, float* y,
                             int64_t ys, int32_t rows, int32_t cols) {
    const int nx = x_stride == 0 ? 1 : count_m;
    const size_t xbytes = align256((size_t)nx * cols * 2);
    cudaError_t e = c->gemv_x.ensure(xbytes + align256((size_t)nx * 4));
    if (e != cudaSuccess) return cuda_fail(e, "GEMV staging allocation");
    __half* x16 = static_cast<__half*>(c->gemv_x.p);
    float* xmul = reinterpret_cast<float*>(static_cast<char*>(c->gemv_x.p) + xbytes);
    return timed_launch(c, 2, count_m, [&] {
        return gw::launch_gemv_batched(count_m, packed, ps, scales, ss, bias, bs, x, x_stride,
                                       x_dtype, x16, xmul, y, ys, rows, cols, c->cur);
    });
}

gw_status gw_mxfp4_gemv_batched_async(gw_ctx* c, int32_t count_m, const uint8_t* packed,
                                      int64_t packed_stride, const uint8_t* scales,
                                      int64_t scale_stride, const uint16_t* bias,
                                      int64_t bias_stride, const void* x, int64_t x_stride,
                                      int32_t x_dtype, float* y, int64_t y_stride, int32_t rows,
                                      int32_t cols) {
    if (!c || !packed || !scales || !x || !y) return fail(GW_E_ARG, "null argument");
    gw_status st = check_dtype(x_dtype);
    if (st) return st;
    if (count_m <= 0 || rows <= 0 || cols <= 0 || cols % 32)
        return fail(GW_E_ARG, "need count > 0, rows > 0 and cols a positive multiple of 32");
    if (packed_stride % 16 || reinterpret_cast<uintptr_t>(packed) % 16)
        return fail(GW_E_ARG, "packed matrices must start on 16-byte boundaries");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    return gemv_device(c, count_m, packed, packed_stride, scales, scale_stride, bias, bias_stride,
                       x, x_stride, x_dtype, y, y_stride, rows, cols);
}

namespace {
gw_status check_int8(const void* codes, const void* meta, const void* x, const void* y, int T, int rows,
                     int cols, int y_dtype) {
    if (!codes || !meta || !x || !y) return fail(GW_E_ARG, "null argument");
    if (T <= 0 || rows <= 0 || cols <= 0 || cols % 64)
        return fail(GW_E_ARG, "need T > 0, rows > 0 and cols a positive multiple of 64 (got T=%d, %d x %d)",
                    T, rows, cols);
    if (cols > gw::kMaxInt8Cols) return fail(GW_E_ARG, "cols %d exceeds %d", cols, gw::kMaxInt8Cols);
    if (y_dtype != GW_DTYPE_F32 && y_dtype != GW_DTYPE_F16)
        return fail(GW_E_ARG, "y_dtype must be GW_DTYPE_F32 or GW_DTYPE_F16 (got %d)", y_dtype);
    return GW_OK;
}
}  // namespace

gw_status gw_int8_affine_gemv_async(gw_ctx* c, const uint8_t* codes, const uint16_t* meta,
                                    const uint16_t* bias, const uint16_t* x, int32_t T, int32_t rows,
                                    int32_t cols, void* y, int32_t y_dtype) {
    if (!c) return fail(GW_E_ARG, "null context");
    gw_status st = check_int8(codes, meta, x, y, T, rows, cols, y_dtype);
    if (st) return st;
    if ((st = check_align16(codes, "codes_dev")) || (st = check_align16(x, "x_dev"))) return st;
    if (reinterpret_cast<uintptr_t>(meta) % 4) return fail(GW_E_ARG, "meta_dev must be 4-byte aligned");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    return count(c, gw::launch_int8_gemv(codes, meta, bias, reinterpret_cast<const __half*>(x), T, rows, cols,
                                         y, y_dtype == GW_DTYPE_F16, c->cur));
}

gw_status gw_ep_dispatch_async(gw_ctx* c, gw_bank* b, const void* x, int32_t x_dtype, int32_t T,
                               const int32_t* experts, const float* weights, int32_t world, int32_t capacity,
                               void* send, int32_t* idx, int32_t* overflow) {
    if (!c || !b || !send || !idx || !overflow) return fail(GW_E_ARG, "null argument");
    gw_status st = check_dtype(x_dtype);
    if (st) return st;
    if (T < 0 || (T > 0 && (!x || !experts || !weights))) return fail(GW_E_ARG, "need T >= 0 and its inputs");
    if (world < 1 || world > gw::kMaxEpWorld || capacity < 1)
        return fail(GW_E_ARG, "need 1 <= world <= %d and capacity >= 1", gw::kMaxEpWorld);
    if ((T > 0 && (st = check_align16(x, "x_dev"))) || (st = check_align16(send, "send_dev"))) return st;
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    return count(c, gw::launch_ep_dispatch(x, T, b->d.hidden, experts, weights, b->d.top_k, world, capacity, send,
                                           idx, overflow, c->cur));
}

gw_status gw_ep_combine_async(gw_ctx* c, gw_bank* b, const float* back, const int32_t* idx, int32_t T, float* out) {
    if (!c || !b) return fail(GW_E_ARG, "null argument");
    if (T < 0 || (T > 0 && (!back || !idx || !out))) return fail(GW_E_ARG, "need T >= 0 and its buffers");
    gw_status st;
    if (T > 0 && ((st = check_align16(back, "back_dev")) || (st = check_align16(out, "out_dev")))) return st;
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    return count(c, gw::launch_ep_combine(back, idx, T, b->d.top_k, b->d.hidden, out, c->cur));
}

// ---- synchronous host-pointer API ------------------------------------------

gw_status gw_int8_affine_gemv(gw_ctx* c, const uint8_t* codes, const uint16_t* meta, const uint16_t* bias,
                              const uint16_t* x, int32_t T, int32_t rows, int32_t cols, void* y,
                              int32_t y_dtype) {
    if (!c) return fail(GW_E_ARG, "null context");
    gw_status st = check_int8(codes, meta, x, y, T, rows, cols, y_dtype);
    if (st) return st;
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    Stage sg(c);
    const size_t nc = (size_t)rows * cols, nm = (size_t)rows * (cols / 64) * 4, nx = (size_t)T * cols * 2;
    const size_t ny = (size_t)T * rows * (y_dtype == GW_DTYPE_F16 ? 2 : 4);
    const size_t oc = sg.add(nc), om = sg.add(nm), ob = sg.add(bias ? (size_t)rows * 2 : 0), ox = sg.add(nx),
                 oy = sg.add(ny);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(oc), codes, nc, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(om), meta, nm, cudaMemcpyHostToDevice, c->cur));
    if (bias) GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(ob), bias, (size_t)rows * 2, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(ox), x, nx, cudaMemcpyHostToDevice, c->cur));
    if ((st = count(c, gw::launch_int8_gemv(sg.at<uint8_t>(oc), sg.at<uint16_t>(om),
                                            bias ? sg.at<uint16_t>(ob) : nullptr, sg.at<__half>(ox), T, rows,
                                            cols, sg.at<void>(oy), y_dtype == GW_DTYPE_F16, c->cur))))
        return st;
    GW_CUDA(cudaMemcpyAsync(y, sg.at<uint8_t>(oy), ny, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}



gw_status gw_mxfp4_gemv(gw_ctx* c, const uint8_t* packed, const uint8_t* scales,
                        const uint16_t* bias, const void* x, int32_t x_dtype, float* y,
                        int32_t rows, int32_t cols) {
    if (!c || !packed || !scales || !x || !y) return fail(GW_E_ARG, "null argument");
    gw_status st = check_dtype(x_dtype);
    if (st) return st;
    if (rows <= 0 || cols <= 0 || cols % 32)
        return fail(GW_E_ARG, "rows must be positive and cols a positive multiple of 32 (got %d x %d)",
                    rows, cols);
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    Stage sg(c);
    const size_t np = (size_t)rows * cols / 2, ns = (size_t)rows * cols / 32;
    const size_t op = sg.add(np), os = sg.add(ns), ob = sg.add(bias ? rows * 2 : 0),
                 ox = sg.add((size_t)cols * 2), oy = sg.add((size_t)rows * 4);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(op), packed, np, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(os), scales, ns, cudaMemcpyHostToDevice, c->cur));
    if (bias) GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(ob), bias, rows * 2, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(ox), x, (size_t)cols * 2, cudaMemcpyHostToDevice, c->cur));
    st = gemv_device(c, 1, sg.at<uint8_t>(op), 0, sg.at<uint8_t>(os), 0,
                     bias ? sg.at<uint16_t>(ob) : nullptr, 0, sg.at<void>(ox), 0, x_dtype,
                     sg.at<float>(oy), 0, rows, cols);
    if (st) return st;
    GW_CUDA(cudaMemcpyAsync(y, sg.at<float>(oy), (size_t)rows * 4, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}

gw_status gw_mxfp4_dequant(gw_ctx* c, const uint8_t* packed, const uint8_t* scales, int32_t rows,
                           int32_t cols, float* w_out) {
    if (!c || !packed || !scales || !w_out) return fail(GW_E_ARG, "null argument");
    if (rows <= 0 || cols <= 0 || cols % 32)
        return fail(GW_E_ARG, "rows must be positive and cols a positive multiple of 32");
    CtxLock lk(c);
    gw_status st = set_device(c);
    if (st) return st;
    Stage sg(c);
    const size_t np = (size_t)rows * cols / 2, ns = (size_t)rows * cols / 32,
                 nw = (size_t)rows * cols * 4;
    const size_t op = sg.add(np), os = sg.add(ns), ow = sg.add(nw);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(op), packed, np, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<uint8_t>(os), scales, ns, cudaMemcpyHostToDevice, c->cur));
    if ((st = count(c, gw::launch_dequant(sg.at<uint8_t>(op), sg.at<uint8_t>(os), rows, cols,
                                          sg.at<float>(ow), c->cur))))
        return st;
    GW_CUDA(cudaMemcpyAsync(w_out, sg.at<float>(ow), nw, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}


gw_status gw_router_logits(gw_ctx* c, gw_bank* b, int32_t layer, const void* x, int32_t x_dtype,
                           int32_t T, float* logits) {
    if (!c || !x || !logits) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    if ((st = ensure_work(c, b, T))) return st;
    const size_t nx = (size_t)T * b->d.hidden * dtype_size(x_dtype);
    Stage sg(c);
    const size_t ox = sg.add(nx);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<void>(ox), x, nx, cudaMemcpyHostToDevice, c->cur));
    const gw::MoeDims d = dims_of(b);
    if ((st = count(c, gw::launch_router(layer_of(b, layer), d, sg.at<void>(ox), x_dtype, T, c->w,
                                         c->cur))))
        return st;
    GW_CUDA(cudaMemsetAsync(c->w.counts, 0, (size_t)d.E * 4, c->cur));
    GW_CUDA(cudaMemsetAsync(c->w.nactive, 0, 8, c->cur));  // and nextra
    GW_CUDA(cudaMemcpyAsync(logits, c->w.logits, (size_t)T * d.E * 4, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}

gw_status gw_route_async(gw_ctx* c, gw_bank* b, int32_t layer, const void* x_dev, int32_t x_dtype,
                         int32_t T, int32_t* experts_dev, float* weights_dev) {
    if (!c || !x_dev || !experts_dev || !weights_dev) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if ((st = check_align16(x_dev, "x_dev"))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    if ((st = ensure_work(c, b, T))) return st;
    const gw::MoeDims d = dims_of(b);
    if ((st = timed_launch(c, 3, 0, [&] {
             return gw::launch_router(layer_of(b, layer), d, x_dev, x_dtype, T, c->w, c->cur);
         })))
        return st;
    // the router also grouped the slots for the expert kernels: leave the
    // counts at zero for the next layer call, as the combine would
    GW_CUDA(cudaMemsetAsync(c->w.counts, 0, (size_t)d.E * 4, c->cur));
    GW_CUDA(cudaMemsetAsync(c->w.nactive, 0, 8, c->cur));  // and nextra
    const size_t nk = (size_t)T * d.k;
    GW_CUDA(cudaMemcpyAsync(experts_dev, c->w.experts, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(weights_dev, c->w.weights, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    return GW_OK;
}

gw_status gw_route(gw_ctx* c, gw_bank* b, int32_t layer, const void* x, int32_t x_dtype, int32_t T,
                   int32_t* experts_out, float* weights_out) {
    if (!c || !x || !experts_out || !weights_out) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    if ((st = ensure_work(c, b, T))) return st;
    const size_t nx = (size_t)T * b->d.hidden * dtype_size(x_dtype);
    Stage sg(c);
    const size_t ox = sg.add(nx);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<void>(ox), x, nx, cudaMemcpyHostToDevice, c->cur));
    const gw::MoeDims d = dims_of(b);
    if ((st = count(c, gw::launch_router(layer_of(b, layer), d, sg.at<void>(ox), x_dtype, T, c->w,
                                         c->cur))))
        return st;
    GW_CUDA(cudaMemsetAsync(c->w.counts, 0, (size_t)d.E * 4, c->cur));
    GW_CUDA(cudaMemsetAsync(c->w.nactive, 0, 8, c->cur));  // and nextra
    const size_t nk = (size_t)T * d.k;
    GW_CUDA(cudaMemcpyAsync(experts_out, c->w.experts, nk * 4, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaMemcpyAsync(weights_out, c->w.weights, nk * 4, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}

gw_status gw_moe_forward(gw_ctx* c, gw_bank* b, int32_t layer, const void* x, int32_t x_dtype,
                         int32_t T, const int32_t* experts_in, const float* weights_in, float* out,
                         int32_t* experts_out, float* weights_out) {
    if (!c || !x || !out) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    if ((experts_in == nullptr) != (weights_in == nullptr))
        return fail(GW_E_ARG, "experts_in and weights_in must both be given or both be NULL");
    const int k = b->d.top_k;
    if (experts_in) {
        for (int64_t i = 0; i < (int64_t)T * k; ++i) {
            if (experts_in[i] < 0 || experts_in[i] >= b->d.experts)
                return fail(GW_E_ARG, "routing entry %lld names expert %d, outside [0, %d)",
                            (long long)i, experts_in[i], b->d.experts);
            for (int64_t j = i - i % k; j < i; ++j)
                if (experts_in[j] == experts_in[i])
                    return fail(GW_E_ARG, "token %lld lists expert %d twice", (long long)(i / k),
                                experts_in[i]);
        }
    }
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    const size_t nx = (size_t)T * b->d.hidden * dtype_size(x_dtype), nk = (size_t)T * k,
                 no = (size_t)T * b->d.hidden * 4;
    Stage sg(c);
    const size_t ox = sg.add(nx), oe = sg.add(nk * 4), ow = sg.add(nk * 4), oo = sg.add(no);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<void>(ox), x, nx, cudaMemcpyHostToDevice, c->cur));
    if (experts_in) {
        GW_CUDA(cudaMemcpyAsync(sg.at<int32_t>(oe), experts_in, nk * 4, cudaMemcpyHostToDevice, c->cur));
        GW_CUDA(cudaMemcpyAsync(sg.at<float>(ow), weights_in, nk * 4, cudaMemcpyHostToDevice, c->cur));
    }
    st = moe_layer_device(c, b, layer, sg.at<void>(ox), x_dtype, T,
                          experts_in ? sg.at<int32_t>(oe) : nullptr,
                          experts_in ? sg.at<float>(ow) : nullptr, sg.at<float>(oo), 0, nullptr);
    if (st) return st;
    GW_CUDA(cudaMemcpyAsync(out, sg.at<float>(oo), no, cudaMemcpyDeviceToHost, c->cur));
    if (experts_out)
        GW_CUDA(cudaMemcpyAsync(experts_out, c->w.experts, nk * 4, cudaMemcpyDeviceToHost, c->cur));
    if (weights_out)
        GW_CUDA(cudaMemcpyAsync(weights_out, c->w.weights, nk * 4, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}

gw_status gw_expert_apply_batch(gw_ctx* c, gw_bank* b, int32_t layer, const void* x,
                                int32_t x_dtype, int32_t n, const int32_t* experts,
                                const float* weights, float* y) {
    if (!c || !x || !y || (n > 0 && (!experts || !weights))) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if (n < 0 || n > b->d.top_k)
        return fail(GW_E_ARG, "expert count %d outside [0, top_k=%d]", n, b->d.top_k);
    if (n == 0) {  // applyBatch returns zeros for an empty expert list
        std::memset(y, 0, (size_t)b->d.hidden * 4);
        return GW_OK;
    }
    // Pad the assignment to the bank's top-k with id -1 (skipped).
    int32_t ex[gw::kMaxTopK];
    float wt[gw::kMaxTopK];
    for (int j = 0; j < b->d.top_k; ++j) {
        ex[j] = j < n ? experts[j] : -1;
        wt[j] = j < n ? weights[j] : 0.f;
        if (j < n && (ex[j] < 0 || ex[j] >= b->d.experts))
            return fail(GW_E_ARG, "expert %d out of range [0, %d)", ex[j], b->d.experts);
        for (int i = 0; i < j && j < n; ++i)
            if (ex[i] == ex[j]) return fail(GW_E_ARG, "expert %d listed twice", ex[j]);
    }
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    const size_t nx = (size_t)b->d.hidden * 2, nk = (size_t)b->d.top_k, no = (size_t)b->d.hidden * 4;
    Stage sg(c);
    const size_t ox = sg.add(nx), oe = sg.add(nk * 4), ow = sg.add(nk * 4), oo = sg.add(no);
    cudaError_t e = sg.alloc();
    if (e != cudaSuccess) return cuda_fail(e, "staging allocation");
    GW_CUDA(cudaMemcpyAsync(sg.at<void>(ox), x, nx, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<int32_t>(oe), ex, nk * 4, cudaMemcpyHostToDevice, c->cur));
    GW_CUDA(cudaMemcpyAsync(sg.at<float>(ow), wt, nk * 4, cudaMemcpyHostToDevice, c->cur));
    st = moe_layer_device(c, b, layer, sg.at<void>(ox), x_dtype, 1, sg.at<int32_t>(oe),
                          sg.at<float>(ow), sg.at<float>(oo), 0, nullptr);
    if (st) return st;
    GW_CUDA(cudaMemcpyAsync(y, sg.at<float>(oo), no, cudaMemcpyDeviceToHost, c->cur));
    GW_CUDA(cudaStreamSynchronize(c->cur));
    return GW_OK;
}

gw_status gw_expert_apply(gw_ctx* c, gw_bank* b, int32_t layer, int32_t expert, const void* x,
                          int32_t x_dtype, float* y) {
    const float one = 1.0f;
    return gw_expert_apply_batch(c, b, layer, x, x_dtype, 1, &expert, &one, y);
}

}  // extern "C"

// ---- MoE layer without allocation ------------------------------------------
//
// For callers that cannot allocate device memory while they run a layer: an
// engine that plans all of its memory up front and forbids allocation in the
// serving loop, a caller running under a driver-level memory cap, or one that
// must not let a first-call allocation stall or fail mid-request.  Their layer
// scratch lives in this fixed device array instead of the context workspace.
// Every device that loads the library holds these bytes until the process
// exits.

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on `device` (current), resolved once.
gw_status noalloc_scratch(int device, void** out) {
    if (device < 0 || device >= kNoAllocMaxDevices)
        return fail(GW_E_UNSUPPORTED, "device %d beyond the no-allocation path's device table", device);
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
        g_noalloc_ptr[device] = p;
    }
    *out = g_noalloc_ptr[device];
    return GW_OK;
}

}  // namespace

extern "C" GW_API gw_status gw_moe_forward_noalloc_async(gw_ctx* c, gw_bank* b, int32_t layer,
                                                          const void* x_dev, int32_t x_dtype,
                                                          int32_t T, float* out_dev,
                                                          int32_t* experts_dev,
                                                          float* weights_dev) {
    if (!c || !x_dev || !out_dev) return fail(GW_E_ARG, "null argument");
    gw_status st = check_bank(b, layer);
    if (st || (st = check_dtype(x_dtype))) return st;
    if ((st = check_align16(x_dev, "x_dev")) || (st = check_align16(out_dev, "out_dev"))) return st;
    if (T <= 0) return fail(GW_E_ARG, "T must be positive");
    const int H = b->d.hidden, F = b->d.intermediate, E = b->d.experts, k = b->d.top_k;
    // the same scratch carve-up as the context workspace, sized for exactly T
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
    const size_t o_x16 = take((size_t)T * H * 2);
    const size_t o_xmul = take((size_t)T * 4);
    const size_t o_logits = take((size_t)T * E * 4);
    const size_t o_experts = take((size_t)T * k * 4);
    const size_t o_weights = take((size_t)T * k * 4);
    const size_t o_counts = take((size_t)E * 4);
    const size_t o_active = take((size_t)E * 4);
    const size_t o_nactive = take(8);  // nactive, nextra
    const size_t o_extra = take(((size_t)T * k / gw::kGemvPass + 1) * 4);
    const size_t o_lists = take((size_t)E * T * 4);
    const size_t o_act = take((size_t)T * k * F * 2);
    const size_t o_ybuf = take((size_t)T * k * H * 4);
    const size_t o_done = take((size_t)(T / 8 + 1) * 4);
    const size_t o_sched = take(8);
    if (off > kNoAllocScratchBytes)
        return fail(GW_E_ARG,
                    "T=%d needs %zu bytes of layer scratch; the no-allocation path holds %zu "
                    "(use gw_moe_forward_async, or fewer tokens per call)",
                    T, off, kNoAllocScratchBytes);
    CtxLock lk(c);
    if ((st = set_device(c))) return st;
    void* scratch = nullptr;
    if ((st = noalloc_scratch(c->device, &scratch))) return st;
    char* base = static_cast<char*>(scratch);
    gw::MoeWork w{};
    w.tcap = T;
    w.xr = nullptr;
    w.x16 = reinterpret_cast<__half*>(base + o_x16);
    w.xmul = reinterpret_cast<float*>(base + o_xmul);
    w.logits = reinterpret_cast<float*>(base + o_logits);
    w.experts = reinterpret_cast<int32_t*>(base + o_experts);
    w.weights = reinterpret_cast<float*>(base + o_weights);
    w.counts = reinterpret_cast<int32_t*>(base + o_counts);
    w.active = reinterpret_cast<int32_t*>(base + o_active);
    w.nactive = reinterpret_cast<int32_t*>(base + o_nactive);
    w.nextra = w.nactive + 1;
    w.extra = reinterpret_cast<int32_t*>(base + o_extra);
    w.lists = reinterpret_cast<int32_t*>(base + o_lists);
    w.act = reinterpret_cast<__half*>(base + o_act);
    w.ybuf = reinterpret_cast<float*>(base + o_ybuf);
    w.done = reinterpret_cast<unsigned*>(base + o_done);
    w.sched = reinterpret_cast<unsigned*>(base + o_sched);
    w.status = c->status;
    // The array keeps whatever the previous call left: clear the expert counts,
    // the active-expert count and the router completion counters.
    GW_CUDA(cudaMemsetAsync(base + o_counts, 0, (size_t)E * 4, c->cur));
    GW_CUDA(cudaMemsetAsync(base + o_nactive, 0, 8, c->cur));
    GW_CUDA(cudaMemsetAsync(base + o_done, 0, (size_t)(T / 8 + 1) * 4, c->cur));
    GW_CUDA(cudaMemsetAsync(base + o_sched, 0, 8, c->cur));
    const gw::MoeDims d = dims_of(b);
    const gw::LayerView L = layer_of(b, layer);
    if ((st = count(c, gw::launch_router(L, d, x_dev, x_dtype, T, w, c->cur)))) return st;
    if ((st = count(c, gw::launch_expert_gemv(L, d, w, T, 0, c->cur)))) return st;
    if ((st = count(c, gw::launch_expert_gemv(L, d, w, T, 1, c->cur)))) return st;
    if ((st = count(c, gw::launch_combine(d, T, w, out_dev, 0, nullptr, x_dtype, c->cur)))) return st;
    const size_t nk = (size_t)T * k;
    if (experts_dev)
        GW_CUDA(cudaMemcpyAsync(experts_dev, w.experts, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    if (weights_dev)
        GW_CUDA(cudaMemcpyAsync(weights_dev, w.weights, nk * 4, cudaMemcpyDeviceToDevice, c->cur));
    return GW_OK;
}
