// kv800_decode_noalloc: the paged decode of kv800_decode for callers that must not allocate device memory at
// decode time.  Examples are a serving engine that plans every byte of the GPU up front, or a plugin host whose
// allocator is not reachable from the thread that calls this library.  Such a caller cannot provide the
// kv800_decode workspace.  This entry point uses a fixed scratch area built into the library instead: a file-scope
// __device__ array of NOALLOC_SCRATCH_BYTES (16 MiB) that every GPU loading the library holds until the process
// exits.
//
// Rules of use:
//   - the first call on a device looks up the array's device address (cudaGetSymbolAddress) with that device
//     current, so make the first call on each device before any stream capture;
//   - all calls share the one array and it keeps the last call's contents: calls that can overlap on the GPU (on
//     different streams, or different host threads) race on it and must be serialized by the caller;
//   - a decode whose scratch would exceed the array is rejected with KV800_ERR_RANGE (a larger spb needs less);
//   - nothing here calls cudaMalloc, cudaFree or any allocating routine.  The status word at the start of the array
//     and the per-row arrival counters are cleared on every call: by cudaMemsetAsync in the grid form (spb > 0) and
//     by the schedule kernel in the persistent form (spb <= 0 with quantized sub-blocks);
//   - the device range checks (offsets, tables, sinks, bounded waits) record into that status word like in
//     kv800_decode; kv800_decode_noalloc_status reads it back after a call.
#include <atomic>

#include "kv800_common.cuh"

namespace {
constexpr int64_t NOALLOC_SCRATCH_BYTES = 16ll << 20;
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// device address of g_noalloc_scratch per device ordinal (0 = not looked up yet)
std::atomic<uintptr_t> g_scratch_addr[MAX_DEVICES];
}  // namespace

// The scratch array's device address on the current device, looked up once per device (no allocation).
static int scratch_address(uintptr_t& addr, const char* who) {
    int dev = 0;
    int rc = kv800::cuda_status(cudaGetDevice(&dev), who);
    if (rc) return rc;
    if (dev < 0 || dev >= MAX_DEVICES) {
        kv800::set_error("%s: device ordinal %d above %d", who, dev, MAX_DEVICES - 1);
        return KV800_ERR_RANGE;
    }
    addr = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (addr == 0) {
        void* p = nullptr;
        rc = kv800::cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), who);
        if (rc) return rc;
        addr = reinterpret_cast<uintptr_t>(p);
        g_scratch_addr[dev].store(addr, std::memory_order_release);
    }
    return KV800_OK;
}

extern "C" int kv800_decode_noalloc(const kv800_paged* P, const uint16_t* q, const uint16_t* cos_t,
                                    const uint16_t* sin_t, int64_t npos, int64_t B, int64_t spb, uint16_t* out,
                                    void* stream) {
    if (!P) {
        kv800::set_error("kv800_decode_noalloc: null Paged record");
        return KV800_ERR_ARG;
    }
    const int64_t need = kv800_decode_workspace_size(B, P->nqmax, P->win, spb);
    if (need < 0) {
        kv800::set_error("kv800_decode_noalloc: negative batch");
        return KV800_ERR_ARG;
    }
    if (need > NOALLOC_SCRATCH_BYTES) {
        kv800::set_error("kv800_decode_noalloc: this decode needs %lld bytes of scratch, above the built-in %lld "
                         "(reduce the batch or raise spb)", (long long)need, (long long)NOALLOC_SCRATCH_BYTES);
        return KV800_ERR_RANGE;
    }
    uintptr_t addr = 0;
    const int rc = scratch_address(addr, "kv800_decode_noalloc: scratch array address");
    if (rc) return rc;
    return kv800_decode(P, q, cos_t, sin_t, npos, B, spb, out, reinterpret_cast<void*>(addr), NOALLOC_SCRATCH_BYTES,
                        stream);
}

// The status word of the last kv800_decode_noalloc call on the current device (the first int of the scratch array),
// read back like kv800_check_status: synchronizes `stream`, *host_value = the bits, KV800_ERR_DEVICE when nonzero.
extern "C" int kv800_decode_noalloc_status(int* host_value, void* stream) {
    uintptr_t addr = 0;
    const int rc = scratch_address(addr, "kv800_decode_noalloc_status: scratch array address");
    if (rc) return rc;
    return kv800_check_status(reinterpret_cast<const int*>(addr), host_value, stream);
}
