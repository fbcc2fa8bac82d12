// gtm_moe_decode_noalloc: the fused batch-1 decode of gtm_moe_decode with its scratch in a
// statically sized device array of this library instead of a workspace the caller allocates.
//
// Who needs it: callers that cannot allocate device memory. A host that reaches the library
// through a bare C/FFI binding holds device addresses of its weights and activations but has no
// device allocator of its own to create a workspace with; a serving process that reserves all
// device memory when it starts treats any later cudaMalloc as a failure (it would fragment or
// overrun its reservation). Both can still decode through this entry, which allocates nothing:
// the scratch is a file-scope __device__ array that exists on every GPU that loads the library,
// for as long as the process lives.
//
// Limits and rules:
//   * the scratch holds kScratchBytes (256 KB); the decode needs decode_workspace_bytes(), about
//     160 KB. A build whose decode needs more is rejected with GTM_ERR_UNSUPPORTED;
//   * one scratch per device, shared by every call: calls that overlap on one device (two
//     streams, or two host threads) race on it and must be serialised by the caller;
//   * the first call on each device looks the array's device address up (cudaGetSymbolAddress,
//     with that device current) and keeps it; make that first call before any stream capture.
//     The kept address belongs to the device's primary context as it was then: use the entry from
//     the primary context (the runtime's default), and do not reset the device
//     (cudaDeviceReset) after the first call, which unloads the module and leaves the kept
//     address pointing at nothing;
//   * what must start at zero: the barrier flags and the per-launch error word are cleared by
//     every call before its launch; the sticky error word starts at zero (static device storage
//     is zero-initialised at module load) and is cleared whenever it is read back;
//   * device-side timeouts are kept in that sticky word: calling with layers == NULL and
//     num_layers == 0 reads and clears it (synchronising `stream`) and returns GTM_OK or
//     GTM_ERR_TIMEOUT.
#include <cuda_runtime.h>

#include <mutex>

#include "gtm_internal.h"

namespace gtm {
namespace {

constexpr size_t kScratchBytes = 256 * 1024;
constexpr int kMaxDevices = 64;

// Host code must not hand this name to a kernel: on the host it is only a stand-in for the
// symbol. Its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the current device's scratch, looked up once per device.
int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode_noalloc: cudaGetDevice", e);
    if (dev < 0 || dev >= kMaxDevices)
        return set_error(GTM_ERR_UNSUPPORTED, "gtm_moe_decode_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) return set_cuda_error("gtm_moe_decode_noalloc: cudaGetSymbolAddress", e);
        if (!p) return set_error(GTM_ERR_CUDA, "gtm_moe_decode_noalloc: cudaGetSymbolAddress gave a null address");
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return GTM_OK;
}

}  // namespace
}  // namespace gtm

using namespace gtm;

extern "C" GTM_API int gtm_moe_decode_noalloc(const GtmDims* dims, const GtmLayer* layers, int num_layers,
                                              const GtmDecodeIO* io, void* stream) {
    const size_t need = decode_workspace_bytes();
    if (need > kScratchBytes)
        return set_error(GTM_ERR_UNSUPPORTED, "gtm_moe_decode_noalloc: the decode needs %zu bytes of scratch, the "
                                              "static scratch holds %zu", need, kScratchBytes);
    void* scratch = nullptr;
    const int rc = scratch_for_current_device(&scratch);
    if (rc != GTM_OK) return rc;
    if (layers == nullptr && num_layers == 0) return gtm_moe_decode_check(scratch, stream);
    return gtm_moe_decode(dims, layers, num_layers, io, scratch, kScratchBytes, stream);
}
