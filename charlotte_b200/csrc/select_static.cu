// Top-k selection and the draw for callers that cannot allocate device
// memory.
//
// cb_select_run needs scratch beside its inputs and outputs: each
// 1,024-logit tile's 64 candidates, and ticket words that find the tiles
// finishing last. Most callers hand in buffers they allocated once. Some
// cannot: a host that plans every byte of device memory up front and counts
// it against a budget (as Charlotte's residency plan does for every working
// buffer) and has no slot for a buffer this library asks for late; code that
// runs where cudaMalloc is not allowed or would stall the pipeline (it may
// synchronize the device); a plugin whose host owns the allocator. For them,
// cb_select_run_static keeps its scratch in a fixed array compiled into the
// library: 128 KiB of candidates (256 tiles, vocabularies up to 262,144)
// and its ticket words, held by every GPU that loads the library until the
// process exits. It allocates nothing.
//
// The first call on a device looks up the array's device address
// (cudaGetSymbolAddress, with that device current) and keeps it; make that
// first call before any stream capture. Every call shares the one array,
// which keeps the last call's contents: each call clears the tickets before
// its launch, and calls that overlap on the GPU (on two streams at once)
// race on the array — order them on one stream.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "api_common.h"
#include "charlotte_b200.h"
#include "kernels.h"

namespace {

constexpr uint32_t kStaticTiles = 256;                        // 262,144 logits
constexpr uint32_t kStaticCount = kStaticTiles * 1024u;
constexpr uint32_t kCandidateWords = kStaticTiles * 64u * 2u;   // (bits, token) pairs
constexpr uint32_t kTicketWord = kCandidateWords;             // after the candidates

// The scratch: every tile's candidates, then the tickets (at most 17 words
// of the 64).
static __device__ __align__(256) uint32_t g_select_scratch[kCandidateWords + 64u];

constexpr int kMaxDevices = 64;
uint32_t* g_scratch_address[kMaxDevices] = {nullptr};
std::mutex g_setup;

// The array's device address on the current device, looked up once.
int scratch_address(uint32_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cb::fail_cuda(e, "cb_select_run_static: no current device");
    if (dev < 0 || dev >= kMaxDevices) return cb::fail(CB_ERROR_STEP, "cb_select_run_static: device %d", dev);
    std::lock_guard<std::mutex> lock(g_setup);
    if (!g_scratch_address[dev]) {
        uint32_t* ptr = nullptr;
        e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_select_scratch);
        if (e != cudaSuccess) return cb::fail_cuda(e, "cb_select_run_static: cudaGetSymbolAddress");
        g_scratch_address[dev] = ptr;
    }
    *out = g_scratch_address[dev];
    return CB_OK;
}

}  // namespace

extern "C" {

int cb_select_run_static(const cb_select* s, uint32_t flags, void* stream) {
    if (int rc = cb::select_arguments(s, "cb_select_run_static", true)) return rc;
    if (s->partials || s->ticket)
        return cb::fail(CB_ERROR_INVALID,
                        "cb_select_run_static: partials and ticket must be NULL (this entry point uses its own scratch)");
    if (s->rows > 1)
        return cb::fail(CB_ERROR_INVALID, "cb_select_run_static: one row a call (its fixed scratch holds one selection)");
    if (s->count == 0 || s->count > kStaticCount)
        return cb::fail(CB_ERROR_INVALID, "cb_select_run_static: %u logits; its fixed scratch holds 1 to %u",
                        s->count, kStaticCount);
    uint32_t* base = nullptr;
    if (int rc = scratch_address(&base)) return rc;
    cb_select a = *s;
    a.partials = base;
    a.ticket = reinterpret_cast<unsigned int*>(base + kTicketWord);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(a.ticket, 0, cb_select_tickets(s->count) * sizeof(unsigned int), st);
    if (e != cudaSuccess) return cb::fail_cuda(e, "cb_select_run_static: clearing the tickets");
    e = cb::select_run(a, st, (flags & CB_RUN_PDL) != 0);
    return e == cudaSuccess ? CB_OK : cb::fail_cuda(e, "cb_select_run_static");
}

}  // extern "C"
