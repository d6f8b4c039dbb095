// Host side of the C ABI: error messages, status read-back, constants and version.
#include <cstdarg>
#include <cstdio>

#include "kv800_common.cuh"

namespace kv800 {
static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return KV800_OK;
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return KV800_ERR_CUDA;
}
}  // namespace kv800

extern "C" int kv800_abi_version(void) { return 1; }

extern "C" const char* kv800_last_error(void) { return kv800::g_err; }

extern "C" int kv800_constants(int64_t* blk, int64_t* sub, int64_t* lag, int64_t* nsink, int64_t* win) {
    if (blk) *blk = kv800::BLK;
    if (sub) *sub = kv800::SUB;
    if (lag) *lag = kv800::LAG;
    if (nsink) *nsink = kv800::NSINK;
    if (win) *win = kv800::WIN;
    return KV800_OK;
}

extern "C" int kv800_check_status(const int* status, int* host_value, void* stream) {
    if (!status || !host_value) {
        kv800::set_error("kv800_check_status: null pointer");
        return KV800_ERR_ARG;
    }
    cudaStream_t st = kv800::as_stream(stream);
    int rc = kv800::cuda_status(cudaMemcpyAsync(host_value, status, sizeof(int), cudaMemcpyDeviceToHost, st),
                                "kv800_check_status copy");
    if (rc) return rc;
    rc = kv800::cuda_status(cudaStreamSynchronize(st), "kv800_check_status sync");
    if (rc) return rc;
    if (*host_value) {
        kv800::set_error("device range check fired (status bits 0x%x: 1 qpool, 2 epool, 4 sinks, 8 tables, 16 timeout)",
                         *host_value);
        return KV800_ERR_DEVICE;
    }
    return KV800_OK;
}
