// Device context, buffers and fences: the part of the reference's D3D12Context the MoE path
// uses (include/gturbo/d3d12_context.hpp:22-54; src/d3d12_context.cpp), on the CUDA runtime.
//   create_uma_buffer            -> gtm_buffer_alloc (device memory, 64-bit addresses, so no
//                                   4 GB root-descriptor limit as in runner.cpp:330-333)
//   submit_command_list -> fence -> gtm_submit (a ticket = a monotonically increasing fence value)
//   wait_for_fence(INFINITE)     -> gtm_wait(ticket, timeout_ms): bounded, GTM_ERR_TIMEOUT on expiry
//   flush_gpu                    -> gtm_submit + gtm_wait
// One stream per context; a context is not thread-safe (as the reference's single generation).
#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <new>
#include <thread>

#include "gtm_internal.h"

namespace gtm {
namespace {

constexpr int kTicketRing = 64;   // fences kept; older tickets count as completed

struct Ctx {
    int device;
    cudaStream_t stream;
    cudaEvent_t ev[kTicketRing];
    uint64_t issued;   // last ticket handed out
};

Ctx* as_ctx(void* c) { return static_cast<Ctx*>(c); }

int activate(Ctx* c, const char* fn) {
    const cudaError_t e = cudaSetDevice(c->device);
    return e == cudaSuccess ? GTM_OK : set_cuda_error(fn, e);
}

}  // namespace
}  // namespace gtm

using namespace gtm;

extern "C" {

GTM_API int gtm_ctx_create(int device, void** ctx_out) {
    if (!ctx_out) return set_error(GTM_ERR_INVALID, "gtm_ctx_create: null ctx_out");
    *ctx_out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return set_cuda_error("gtm_ctx_create: cudaGetDeviceCount", e);
    if (device < 0 || device >= n) return set_error(GTM_ERR_INVALID, "gtm_ctx_create: device %d of %d", device, n);
    Ctx* c = new (std::nothrow) Ctx();
    if (!c) return set_error(GTM_ERR_INVALID, "gtm_ctx_create: out of host memory");
    c->device = device;
    c->issued = 0;
    e = cudaSetDevice(device);
    const bool have_stream = e == cudaSuccess && (e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) == cudaSuccess;
    int made = 0;
    while (e == cudaSuccess && made < kTicketRing) {
        e = cudaEventCreateWithFlags(&c->ev[made], cudaEventDisableTiming);
        if (e == cudaSuccess) ++made;
    }
    if (e != cudaSuccess) {
        for (int i = 0; i < made; ++i) cudaEventDestroy(c->ev[i]);
        if (have_stream) cudaStreamDestroy(c->stream);
        delete c;
        return set_cuda_error("gtm_ctx_create", e);
    }
    *ctx_out = c;
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_ctx_destroy(void* ctx) {
    Ctx* c = as_ctx(ctx);
    if (!c) return set_error(GTM_ERR_INVALID, "gtm_ctx_destroy: null ctx");
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (int i = 0; i < kTicketRing; ++i) cudaEventDestroy(c->ev[i]);
    cudaStreamDestroy(c->stream);
    delete c;
    clear_error();
    return GTM_OK;
}

GTM_API void* gtm_ctx_stream(void* ctx) { return ctx ? static_cast<void*>(as_ctx(ctx)->stream) : nullptr; }

GTM_API int gtm_buffer_alloc(void* ctx, uint64_t bytes, void** dev_out) {
    Ctx* c = as_ctx(ctx);
    if (!c || !dev_out || bytes == 0) return set_error(GTM_ERR_INVALID, "gtm_buffer_alloc: null argument or zero size");
    int rc = activate(c, "gtm_buffer_alloc");
    if (rc) return rc;
    const cudaError_t e = cudaMalloc(dev_out, bytes);
    if (e != cudaSuccess) { *dev_out = nullptr; return set_cuda_error("gtm_buffer_alloc", e); }
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_buffer_free(void* ctx, void* dev) {
    Ctx* c = as_ctx(ctx);
    if (!c) return set_error(GTM_ERR_INVALID, "gtm_buffer_free: null ctx");
    if (!dev) return GTM_OK;
    int rc = activate(c, "gtm_buffer_free");
    if (rc) return rc;
    const cudaError_t e = cudaFree(dev);
    if (e != cudaSuccess) return set_cuda_error("gtm_buffer_free", e);
    clear_error();
    return GTM_OK;
}

// Copies on the context's stream; complete after a gtm_wait on a later ticket.
GTM_API int gtm_buffer_upload(void* ctx, void* dev, uint64_t offset, const void* host, uint64_t bytes) {
    Ctx* c = as_ctx(ctx);
    if (!c || !dev || (!host && bytes)) return set_error(GTM_ERR_INVALID, "gtm_buffer_upload: null argument");
    int rc = activate(c, "gtm_buffer_upload");
    if (rc) return rc;
    const cudaError_t e = cudaMemcpyAsync(static_cast<char*>(dev) + offset, host, bytes, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_buffer_upload", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_buffer_download(void* ctx, void* host, const void* dev, uint64_t offset, uint64_t bytes) {
    Ctx* c = as_ctx(ctx);
    if (!c || !dev || (!host && bytes)) return set_error(GTM_ERR_INVALID, "gtm_buffer_download: null argument");
    int rc = activate(c, "gtm_buffer_download");
    if (rc) return rc;
    const cudaError_t e =
        cudaMemcpyAsync(host, static_cast<const char*>(dev) + offset, bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_buffer_download", e);
    clear_error();
    return GTM_OK;
}

GTM_API int gtm_submit(void* ctx, uint64_t* ticket_out) {
    Ctx* c = as_ctx(ctx);
    if (!c || !ticket_out) return set_error(GTM_ERR_INVALID, "gtm_submit: null argument");
    int rc = activate(c, "gtm_submit");
    if (rc) return rc;
    const uint64_t t = c->issued + 1;
    const cudaError_t e = cudaEventRecord(c->ev[t % kTicketRing], c->stream);
    if (e != cudaSuccess) return set_cuda_error("gtm_submit", e);
    c->issued = t;
    *ticket_out = t;
    clear_error();
    return GTM_OK;
}

// Waits until the work submitted up to `ticket` has finished, at most timeout_ms milliseconds.
GTM_API int gtm_wait(void* ctx, uint64_t ticket, uint32_t timeout_ms) {
    Ctx* c = as_ctx(ctx);
    if (!c) return set_error(GTM_ERR_INVALID, "gtm_wait: null ctx");
    if (ticket == 0 || ticket > c->issued)
        return set_error(GTM_ERR_INVALID, "gtm_wait: ticket %llu was not issued (last %llu)", (unsigned long long)ticket,
                         (unsigned long long)c->issued);
    if (c->issued - ticket >= (uint64_t)kTicketRing) {   // a newer fence on this stream has been recorded since
        const uint64_t newest_kept = c->issued - kTicketRing + 1;
        ticket = newest_kept;
    }
    int rc = activate(c, "gtm_wait");
    if (rc) return rc;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaEventQuery(c->ev[ticket % kTicketRing]);
        if (e == cudaSuccess) { clear_error(); return GTM_OK; }
        if (e != cudaErrorNotReady) return set_cuda_error("gtm_wait", e);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (ms >= (long long)timeout_ms)
            return set_error(GTM_ERR_TIMEOUT, "gtm_wait: ticket %llu not complete after %u ms", (unsigned long long)ticket,
                             timeout_ms);
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // extern "C"
