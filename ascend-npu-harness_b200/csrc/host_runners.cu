// Host-buffer runners: copy inputs in, launch, copy outputs out, with the transfers of one
// chunk overlapping the kernel of the previous one.
//
// Mirrors the reference's host-pointer runner contract
// (ops/flash_attention_fwd_fused/runner/flash_attention_fwd_fused_runner.hpp:9-18 and the
// device branch of ops/elementwise_add/runner/elementwise_add_runner.cpp:16-38, which copies
// in, launches and copies out), with the difference that the device staging memory is a
// caller-owned workspace instead of per-call allocations.
#include <cuda_runtime.h>

#include <mutex>

#include "hc_internal.h"

namespace hc {
namespace {

// Three internal streams per device (copy-in, compute, copy-out) and the events that chain them;
// created on a device's first call and kept while the device's context lives.  `mu` serialises
// whole calls on one device: the events are shared, so two calls enqueuing at once could chain
// one call's copies to the other's start.
struct Pipe {
    std::mutex mu;
    uint64_t ctx = 0;  // context the handles belong to; a device reset makes them stale
    cudaStream_t in = nullptr, comp = nullptr, out = nullptr;
    cudaEvent_t in_done[2] = {nullptr, nullptr}, comp_done[2] = {nullptr, nullptr}, out_done[2] = {nullptr, nullptr};
    cudaEvent_t start = nullptr;
};

Pipe g_pipes[64];

// Returns the calling thread's device pipe with its mutex held in `lock`.
int get_pipe(Pipe** out, std::unique_lock<std::mutex>* lock) {
    int dev = 0;
    HC_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(HC_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    Pipe& p = g_pipes[dev];
    *lock = std::unique_lock<std::mutex>(p.mu);
    // A thread that has not used the runtime yet has no context bound (id 0); selecting the
    // current device binds its primary context, so the comparison below sees the real id.
    HC_CHECK_CUDA(cudaSetDevice(dev));
    const uint64_t ctx = current_context_id();
    if (p.ctx == 0 || ctx == 0 || p.ctx != ctx) {
        // First use on this device, or the device was reset since (the old handles died with the
        // old context and are dropped, not destroyed).
        p.ctx = 0;
        HC_CHECK_CUDA(cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking));
        HC_CHECK_CUDA(cudaStreamCreateWithFlags(&p.comp, cudaStreamNonBlocking));
        HC_CHECK_CUDA(cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking));
        for (int b = 0; b < 2; ++b) {
            HC_CHECK_CUDA(cudaEventCreateWithFlags(&p.in_done[b], cudaEventDisableTiming));
            HC_CHECK_CUDA(cudaEventCreateWithFlags(&p.comp_done[b], cudaEventDisableTiming));
            HC_CHECK_CUDA(cudaEventCreateWithFlags(&p.out_done[b], cudaEventDisableTiming));
        }
        HC_CHECK_CUDA(cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming));
        p.ctx = current_context_id();
    }
    *out = &p;
    return HC_OK;
}

struct FaChunking {
    uint64_t bh, heads_per_chunk, q_head_bytes, kv_head_bytes, o_head_bytes, lse_head_bytes, slot_bytes;
};

int fa_chunking(const flash_attention_fwd_fused_tiling_data* t, int dtype, FaChunking* c) {
    size_t es = dtype_size(dtype);
    if (es == 0 || dtype == HC_DTYPE_I32 || dtype == HC_DTYPE_I8 || dtype == HC_DTYPE_U8)
        return fail(HC_ERR_UNSUPPORTED, "flash_attention host runner: dtype %d", dtype);
    c->bh = static_cast<uint64_t>(t->B) * t->H;
    c->q_head_bytes = static_cast<uint64_t>(t->S_q) * t->D * es;
    c->kv_head_bytes = static_cast<uint64_t>(t->S_k) * t->D * es + static_cast<uint64_t>(t->S_k) * t->D_v * es;
    c->o_head_bytes = static_cast<uint64_t>(t->S_q) * t->D_v * es;
    c->lse_head_bytes = static_cast<uint64_t>(t->S_q) * sizeof(float);
    uint64_t per_head = c->q_head_bytes + c->kv_head_bytes;
    // ~96 MB of inputs per chunk: big enough to keep the copy engines streaming, small enough
    // that the first and last chunks (which cannot overlap) are a few percent of the job.
    uint64_t h = (96ull << 20) / (per_head ? per_head : 1);
    if (h < 1) h = 1;
    if (h > c->bh) h = c->bh;
    c->heads_per_chunk = h;
    auto align = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
    c->slot_bytes = align(h * c->q_head_bytes) + align(h * static_cast<uint64_t>(t->S_k) * t->D * es) +
                    align(h * static_cast<uint64_t>(t->S_k) * t->D_v * es) + align(h * c->o_head_bytes) +
                    align(h * c->lse_head_bytes);
    return HC_OK;
}

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_flash_attention_fwd_fused_host_workspace_size(const flash_attention_fwd_fused_tiling_data* t,
                                                                int dtype, size_t* bytes) {
    if (!t || !bytes) return fail(HC_ERR_INVALID, "flash_attention host workspace: null argument");
    FaChunking c;
    int rc = fa_chunking(t, dtype, &c);
    if (rc) return rc;
    *bytes = static_cast<size_t>(2 * c.slot_bytes);
    return ok();
}

extern "C" int hc_flash_attention_fwd_fused_host(const void* h_q, const void* h_k, const void* h_v, void* h_o,
                                                 float* h_lse, const flash_attention_fwd_fused_tiling_data* t,
                                                 int dtype, void* workspace, size_t workspace_bytes, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "flash_attention host: null tiling");
    if (!h_q || !h_k || !h_v || !h_o || !workspace) return fail(HC_ERR_INVALID, "flash_attention host: null pointer");
    int rc = fa_check_tiling(t, t->H, dtype);
    if (rc) return rc;
    FaChunking c;
    rc = fa_chunking(t, dtype, &c);
    if (rc) return rc;
    if (workspace_bytes < 2 * c.slot_bytes)
        return fail(HC_ERR_INVALID, "flash_attention host: workspace %zu B < required %llu B", workspace_bytes,
                    static_cast<unsigned long long>(2 * c.slot_bytes));
    if (c.bh == 0 || t->S_q == 0) return ok();
    Pipe* pp = nullptr;
    std::unique_lock<std::mutex> pipe_lock;
    rc = get_pipe(&pp, &pipe_lock);
    if (rc) return rc;
    Pipe& P = *pp;
    cudaStream_t user = static_cast<cudaStream_t>(stream);
    // Once anything is enqueued, an error return first waits for the work already queued on the
    // internal streams: the caller may free the workspace or reuse the host buffers as soon as
    // the call returns.
    auto join = [&](int status) {
        cudaStreamSynchronize(P.in);
        cudaStreamSynchronize(P.comp);
        cudaStreamSynchronize(P.out);
        cudaGetLastError();
        return status;
    };
#define HC_PIPE_CHECK(call)                                              \
    do {                                                                 \
        cudaError_t e__ = (call);                                        \
        if (e__ != cudaSuccess) return join(cuda_fail(e__, #call));      \
    } while (0)
    const size_t es = dtype_size(dtype);
    auto align = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
    const uint64_t h = c.heads_per_chunk;
    const uint64_t k_bytes_h = static_cast<uint64_t>(t->S_k) * t->D * es;
    const uint64_t v_bytes_h = static_cast<uint64_t>(t->S_k) * t->D_v * es;
    uint8_t* slot[2];
    slot[0] = static_cast<uint8_t*>(workspace);
    slot[1] = slot[0] + c.slot_bytes;
    HC_PIPE_CHECK(cudaEventRecord(P.start, user));
    HC_PIPE_CHECK(cudaStreamWaitEvent(P.in, P.start, 0));
    const uint64_t nchunks = (c.bh + h - 1) / h;
    for (uint64_t ci = 0; ci < nchunks; ++ci) {
        const int b = static_cast<int>(ci & 1);
        const uint64_t h0 = ci * h;
        const uint64_t hn = (h0 + h <= c.bh) ? h : (c.bh - h0);
        uint8_t* dq = slot[b];
        uint8_t* dk = dq + align(h * c.q_head_bytes);
        uint8_t* dv = dk + align(h * k_bytes_h);
        uint8_t* dO = dv + align(h * v_bytes_h);
        float* dl = reinterpret_cast<float*>(dO + align(h * c.o_head_bytes));
        // Copy-in of this chunk may start once the copy-out of the chunk that used this slot
        // two steps ago is finished (which also implies its kernel finished).
        if (ci >= 2) HC_PIPE_CHECK(cudaStreamWaitEvent(P.in, P.out_done[b], 0));
        if (fault_hit("memcpy")) return join(fail(HC_ERR_INJECTED, "flash_attention host: injected copy failure"));
        HC_PIPE_CHECK(cudaMemcpyAsync(dq, static_cast<const uint8_t*>(h_q) + h0 * c.q_head_bytes, hn * c.q_head_bytes,
                                      cudaMemcpyHostToDevice, P.in));
        HC_PIPE_CHECK(cudaMemcpyAsync(dk, static_cast<const uint8_t*>(h_k) + h0 * k_bytes_h, hn * k_bytes_h,
                                      cudaMemcpyHostToDevice, P.in));
        HC_PIPE_CHECK(cudaMemcpyAsync(dv, static_cast<const uint8_t*>(h_v) + h0 * v_bytes_h, hn * v_bytes_h,
                                      cudaMemcpyHostToDevice, P.in));
        HC_PIPE_CHECK(cudaEventRecord(P.in_done[b], P.in));
        HC_PIPE_CHECK(cudaStreamWaitEvent(P.comp, P.in_done[b], 0));
        flash_attention_fwd_fused_tiling_data tc = *t;
        tc.B = 1;
        tc.H = static_cast<uint32_t>(hn);
        rc = hc_flash_attention_fwd_fused_launch(dq, dk, dv, dO, h_lse ? dl : nullptr, &tc, dtype, P.comp);
        if (rc) return join(rc);
        HC_PIPE_CHECK(cudaEventRecord(P.comp_done[b], P.comp));
        HC_PIPE_CHECK(cudaStreamWaitEvent(P.out, P.comp_done[b], 0));
        HC_PIPE_CHECK(cudaMemcpyAsync(static_cast<uint8_t*>(h_o) + h0 * c.o_head_bytes, dO, hn * c.o_head_bytes,
                                      cudaMemcpyDeviceToHost, P.out));
        if (h_lse)
            HC_PIPE_CHECK(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(h_lse) + h0 * c.lse_head_bytes, dl,
                                          hn * c.lse_head_bytes, cudaMemcpyDeviceToHost, P.out));
        HC_PIPE_CHECK(cudaEventRecord(P.out_done[b], P.out));
    }
    HC_PIPE_CHECK(cudaStreamWaitEvent(user, P.out_done[(nchunks - 1) & 1], 0));
    HC_PIPE_CHECK(cudaStreamSynchronize(P.out));
#undef HC_PIPE_CHECK
    return hc_check_device_error();
}

// ------------------------------------------------------------------------------------------
// Allocation-free variant of the host-buffer flash-attention runner.
//
// Staging memory is a file-scope device array instead of a caller workspace, so the call makes
// no device allocation of any kind (no cudaMalloc / cudaFree, no allocating library routine) and
// creates no streams or events: everything runs in order on the caller's stream, one chunk of
// whole heads at a time (copy in, kernel, copy out).  For callers whose device memory is entirely
// owned by their own pool or budget, where an allocation inside the call could fail or would
// synchronise the device.
//   * Limit: kNoAllocScratchBytes per device.  One head's staging (q, k, v, o, lse) must fit;
//     larger heads, and every tiling the kernel would reject, are refused before any device work.
//   * The array is part of the library's device image: every device that loads the library
//     holds its 64 MiB until the process exits, whether or not this runner is ever called.
//   * The first call on a device looks the array's address up with cudaGetSymbolAddress (and
//     the kernel sets its attributes); make that first call before any stream capture.  The
//     address is kept per device context, so a device reset leads to a fresh lookup.
//   * The call waits for the caller's stream to drain before it returns, on success and on an
//     error after its first copy alike, so the host buffers are free again on return.
//   * Nothing in the scratch has to start at zero: every byte read is written earlier in the
//     same call.
//   * All calls on one device share the one array: calls that overlap in time (other threads,
//     other streams) race on it and must be serialised by the caller.
// ------------------------------------------------------------------------------------------
namespace hc {
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;  // 64 MiB per device
static __device__ __align__(256) uint8_t g_fa_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
struct ScratchAddr {
    uint64_t ctx = 0;
    void* ptr = nullptr;
};
ScratchAddr g_noalloc_addr[64];

int noalloc_scratch(void** out) {
    int dev = 0;
    HC_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(HC_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    ScratchAddr& a = g_noalloc_addr[dev];
    HC_CHECK_CUDA(cudaSetDevice(dev));  // binds the device's primary context to a thread new to the runtime
    const uint64_t ctx = current_context_id();
    if (!a.ptr || ctx == 0 || a.ctx != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_fa_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(flash-attention scratch)");
        a.ptr = p;
        a.ctx = current_context_id();  // the lookup binds the context if nothing had yet
    }
    *out = a.ptr;
    return HC_OK;
}

// Staging bytes of `h` consecutive heads: q, k, v, o, lse, each 256-byte aligned.
uint64_t noalloc_chunk_bytes(const flash_attention_fwd_fused_tiling_data* t, size_t es, uint64_t h) {
    auto align = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
    return align(h * t->S_q * t->D * es) + align(h * static_cast<uint64_t>(t->S_k) * t->D * es) +
           align(h * static_cast<uint64_t>(t->S_k) * t->D_v * es) + align(h * t->S_q * t->D_v * es) +
           align(h * t->S_q * sizeof(float));
}

}  // namespace
}  // namespace hc

extern "C" size_t hc_flash_attention_fwd_fused_host_noalloc_limit(void) { return hc::kNoAllocScratchBytes; }

extern "C" int hc_flash_attention_fwd_fused_host_noalloc(const void* h_q, const void* h_k, const void* h_v, void* h_o,
                                                         float* h_lse, const flash_attention_fwd_fused_tiling_data* t,
                                                         int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "flash_attention host (no-alloc): null tiling");
    if (!h_q || !h_k || !h_v || !h_o) return fail(HC_ERR_INVALID, "flash_attention host (no-alloc): null pointer");
    int rc = fa_check_tiling(t, t->H, dtype);
    if (rc) return rc;
    const size_t es = dtype_size(dtype);
    const uint64_t bh = static_cast<uint64_t>(t->B) * t->H;
    if (bh == 0 || t->S_q == 0) return ok();
    if (noalloc_chunk_bytes(t, es, 1) > kNoAllocScratchBytes)
        return fail(HC_ERR_UNSUPPORTED,
                    "flash_attention host (no-alloc): one head needs %llu B of staging, above the %zu B scratch",
                    static_cast<unsigned long long>(noalloc_chunk_bytes(t, es, 1)), kNoAllocScratchBytes);
    uint64_t h = kNoAllocScratchBytes / noalloc_chunk_bytes(t, es, 1);
    if (h > bh) h = bh;
    while (h > 1 && noalloc_chunk_bytes(t, es, h) > kNoAllocScratchBytes) --h;
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    auto align = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
    const uint64_t q_h = static_cast<uint64_t>(t->S_q) * t->D * es;
    const uint64_t k_h = static_cast<uint64_t>(t->S_k) * t->D * es;
    const uint64_t v_h = static_cast<uint64_t>(t->S_k) * t->D_v * es;
    const uint64_t o_h = static_cast<uint64_t>(t->S_q) * t->D_v * es;
    const uint64_t l_h = static_cast<uint64_t>(t->S_q) * sizeof(float);
    uint8_t* dq = static_cast<uint8_t*>(scratch);
    uint8_t* dk = dq + align(h * q_h);
    uint8_t* dv = dk + align(h * k_h);
    uint8_t* dO = dv + align(h * v_h);
    float* dl = reinterpret_cast<float*>(dO + align(h * o_h));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // An error after the first copy was queued waits for the stream before returning.
    auto drain = [&](int status) {
        cudaStreamSynchronize(s);
        cudaGetLastError();
        return status;
    };
#define HC_NOALLOC_CHECK(call)                                           \
    do {                                                                 \
        cudaError_t e__ = (call);                                        \
        if (e__ != cudaSuccess) return drain(cuda_fail(e__, #call));     \
    } while (0)
    for (uint64_t h0 = 0; h0 < bh; h0 += h) {
        const uint64_t hn = (h0 + h <= bh) ? h : (bh - h0);
        HC_NOALLOC_CHECK(cudaMemcpyAsync(dq, static_cast<const uint8_t*>(h_q) + h0 * q_h, hn * q_h,
                                         cudaMemcpyHostToDevice, s));
        HC_NOALLOC_CHECK(cudaMemcpyAsync(dk, static_cast<const uint8_t*>(h_k) + h0 * k_h, hn * k_h,
                                         cudaMemcpyHostToDevice, s));
        HC_NOALLOC_CHECK(cudaMemcpyAsync(dv, static_cast<const uint8_t*>(h_v) + h0 * v_h, hn * v_h,
                                         cudaMemcpyHostToDevice, s));
        flash_attention_fwd_fused_tiling_data tc = *t;
        tc.B = 1;
        tc.H = static_cast<uint32_t>(hn);
        rc = hc_flash_attention_fwd_fused_launch(dq, dk, dv, dO, h_lse ? dl : nullptr, &tc, dtype, s);
        if (rc) return drain(rc);
        HC_NOALLOC_CHECK(
            cudaMemcpyAsync(static_cast<uint8_t*>(h_o) + h0 * o_h, dO, hn * o_h, cudaMemcpyDeviceToHost, s));
        if (h_lse)
            HC_NOALLOC_CHECK(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(h_lse) + h0 * l_h, dl, hn * l_h,
                                             cudaMemcpyDeviceToHost, s));
    }
#undef HC_NOALLOC_CHECK
    HC_CHECK_CUDA(cudaStreamSynchronize(s));
    return hc_check_device_error();
}
