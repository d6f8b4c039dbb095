// 800h paged GQA decode on sm_100a: split partials over quantized sub-blocks (qdecode_mma.cuh) and over sinks +
// exact bf16 tokens (xdecode_tma.cuh for the reference's page layout, xdecode_mma.cuh for any other), all on the
// tensor cores, and the log-sum-exp merge with the in-register Hadamard (combine).
//
// Semantics follow the reference's torch decode (lfm3_kv800/torch_decode.py:16-80), including its two bf16 roundings
// of every key: the dequantized pre-RoPE key is rounded to bf16 (kv800.py:86) and the rotated key is rounded to bf16
// again (torch_decode.py:24).  Both are reproduced exactly: c * sc + lo is exact in fp32 for fp8 sc / lo and c <= 3,
// so one FMA gives the reference's fp32 value; k0 * cs and k2 * sn are exact in fp32 (bf16 x bf16), so
// fma(k0, cs, -(k2 * sn)) is the reference's fl(fl(k0 cs) - fl(k2 sn)).  Partials use the reference's split layout
// (kv800.py:362-383): per (row b, slot) m (log2 domain), l and acc (16 x 128, fp32); quantized slots keep V in the
// Hadamard domain and combine() rotates their weighted sum once (kv800.py:231-236).
#include "kv800_common.cuh"
#include "qdecode_mma.cuh"
#include "xdecode_mma.cuh"
#include "xdecode_tma.cuh"

#include <cudaTypedefs.h>

#include <atomic>

namespace kv800 {

// prefix[b] = sum over rows < b of clamp(min(NQ, nqmax), 0); prefix[B] = W.  One CTA of 1024 threads.  Also clears
// the workspace's status word and per-row arrival counters (zero[0 .. nzero)), so a persistent decode needs no
// separate reset: the kernels after it touch them only once this one has completed.
__global__ void __launch_bounds__(1024) qsched_kernel(const int32_t* NQ, int64_t nqmax, int64_t B, int64_t* prefix,
                                                      int* zero, int64_t nzero) {
    __shared__ int64_t wsum[32];
    __shared__ int64_t carry;
    pdl_launch_dependents();   // the quantized-partial kernel may place its CTAs now; it waits for this kernel
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int64_t i = tid; i < nzero; i += 1024) zero[i] = 0;
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < B; base += 1024) {
        int64_t v = 0;
        if (base + tid < B) {
            v = NQ[base + tid];
            if (v > nqmax) v = nqmax;
            if (v < 0) v = 0;
        }
        int64_t x = v;   // inclusive scan within the warp
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int64_t w = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            wsum[lane] = w;   // inclusive over warps
        }
        __syncthreads();
        const int64_t excl = carry + (warp ? wsum[warp - 1] : 0) + x - v;
        if (base + tid < B) prefix[base + tid] = excl;
        __syncthreads();
        if (tid == 0) carry += wsum[31];
        __syncthreads();
    }
    if (tid == 0) prefix[B] = carry;
}

// grid (B), block 128: warp h merges query rows 4 h .. 4 h + 3 of row blockIdx.x (combine.cuh).
__global__ void __launch_bounds__(128) combine_kernel(const float* mo, const float* lo, const float* ao, SlotMap sm,
                                                      uint16_t* out) {
    combine_head(mo, lo, ao, sm, out, blockIdx.x, threadIdx.x >> 5, threadIdx.x & 31);
}

}  // namespace kv800

using namespace kv800;

namespace {
constexpr int64_t MAX_B = 1 << 20;
constexpr int NX_DEFAULT = 4;                   // exact splits per row in kv800_decode
// exact splits per row of a window layer (no quantized sub-blocks): 3 keeps a 64-row layer's 768 one-warp CTAs in
// one wave on 148 SMs (18.5 us per decode as a CUDA graph, against 20.5 us with 4 splits and 22.0 / 22.5 with 6 / 8)
constexpr int NX_WIN = 3;
constexpr float SCALE = 0.12751743074602467f;   // 128^-0.5 * log2(e)
constexpr int MAX_DEV = 64;

// persistent CTAs of qdecode_mma on the current device: 3 per SM (its registers and shared-memory ring allow three)
int64_t persistent_ctas() {
    static int cache[MAX_DEV] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEV) return 3 * 148;
    if (!cache[dev]) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
        cache[dev] = sms;
    }
    return 3 * (int64_t)cache[dev];
}

int check_paged(const kv800_paged* P, const char* who) {
    if (!P || !P->epool || !P->eoff || !P->N || !P->NQ || P->ebs <= 0 || P->ebs > 0x7fffffffLL ||
        P->eoff_stride <= 0) {
        set_error("%s: null Paged record / epool / eoff / N / NQ, ebs outside [1, 2^31), or eoff_stride <= 0", who);
        return KV800_ERR_ARG;
    }
    if (P->win < 0 || P->nsink < 0 || P->nqmax < 0) {
        set_error("%s: negative win / nsink / nqmax", who);
        return KV800_ERR_ARG;
    }
    if (P->win == 0 && P->nqmax > 0 && (!P->qpool || !P->boff || P->boff_stride <= 0)) {
        set_error("%s: quantized layer with nqmax > 0 needs qpool and boff", who);
        return KV800_ERR_ARG;
    }
    if (P->win && P->sk && (!P->sv || !P->skoff || !P->svoff)) {
        set_error("%s: sinks need sk, sv, skoff and svoff", who);
        return KV800_ERR_ARG;
    }
    return KV800_OK;
}

// Workspace plan of kv800_decode.  spb > 0: grid splits of spb sub-blocks (ns per row, the reference's sizing);
// spb <= 0: persistent, G0 CTAs over the flattened sub-block list.  Layout: status word | arrival counters int32
// [B][4] (from byte 256: per (row, head) for the tensor-map form of the exact partials, per row (the first B) for the
// gather form; cleared with the status word before every decode) | prefix[B + 1] (persistent) |
// MO, LO [nslots][16] | AO [nslots][16][128], each 256-byte aligned.
struct Plan {
    bool persistent;
    int nx;   // exact splits per row
    int64_t ns, G0, nslots, cnt_off, prefix_off, mo_off, lo_off, ao_off, bytes;
};

int64_t up256(int64_t x) { return (x + 255) & ~(int64_t)255; }

Plan make_plan(int64_t B, int64_t nqmax, int64_t win, int64_t spb) {
    Plan p{};
    const int64_t nq = win ? 0 : nqmax;
    p.persistent = spb <= 0 && nq > 0;
    p.ns = (nq > 0 && !p.persistent) ? (nq + spb - 1) / spb : 0;
    p.G0 = p.persistent ? persistent_ctas() : 0;
    p.nx = win ? NX_WIN : NX_DEFAULT;
    p.nslots = p.persistent ? p.G0 + B + B * p.nx : B * (p.ns + p.nx);
    p.cnt_off = 256;
    p.prefix_off = up256(p.cnt_off + 4 * HEADS * B);
    p.mo_off = up256(p.prefix_off + (p.persistent ? (B + 1) * 8 : 0));
    p.lo_off = up256(p.mo_off + p.nslots * QROWS * 4);
    p.ao_off = up256(p.lo_off + p.nslots * QROWS * 4);
    p.bytes = up256(p.ao_off + p.nslots * QROWS * DIM * 4);
    return p;
}
}  // namespace

extern "C" int64_t kv800_decode_workspace_size(int64_t B, int64_t nqmax, int64_t win, int64_t spb) {
    if (B < 0) return -1;
    return make_plan(B, nqmax, win, spb).bytes;
}

// TMA descriptors of the quant pool as rows of 128 bytes: boxes of 64 rows with the 128-byte swizzle (kc rows and
// vb lines) and boxes of 16 rows without (the scale region).  The pool must start 16-byte aligned; a sub-block at an
// offset that is not a multiple of 128 is flagged and skipped by the kernel.
static int tensor_map_encoder(PFN_cuTensorMapEncodeTiled& out) {
    static PFN_cuTensorMapEncodeTiled encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult qres;
        void* fn = nullptr;
        const int rc = cuda_status(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres),
                                   "cuTensorMapEncodeTiled lookup");
        if (rc) return rc;
        if (qres != cudaDriverEntryPointSuccess || !fn) {
            set_error("cuTensorMapEncodeTiled is not available from the driver");
            return KV800_ERR_CUDA;
        }
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
    }
    out = encode;
    return KV800_OK;
}

static int make_qmaps(const uint8_t* qpool, int64_t qpool_bytes, QMArgs& qa) {
    PFN_cuTensorMapEncodeTiled encode = nullptr;
    const int rce = tensor_map_encoder(encode);
    if (rce) return rce;
    const int64_t rows = qpool_bytes / 128;
    if (!qpool || (reinterpret_cast<uintptr_t>(qpool) & 15u) || rows < 16 || rows > 0x7fffffffLL) {
        set_error("quant pool must be 16-byte aligned and hold between 2 KB and 2^31 x 128 bytes");
        return KV800_ERR_ARG;
    }
    cuuint64_t dims[2] = {128, (cuuint64_t)rows};
    cuuint64_t strides[1] = {128};
    cuuint32_t box_rows[2] = {128, 64}, box_sc[2] = {128, 16}, es[2] = {1, 1};
    CUresult r1 = encode(&qa.tm_rows, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(qpool), dims, strides,
                         box_rows, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = encode(&qa.tm_sc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(qpool), dims, strides,
                         box_sc, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d, %d)", (int)r1, (int)r2);
        return KV800_ERR_CUDA;
    }
    return KV800_OK;
}

// The kernels' shared-memory attributes are set once per device: cudaFuncSetAttribute applies to the current
// device's context, so a process that decodes on several GPUs sets them on each (flags per device ordinal).
static int set_smem_once(std::atomic<int>* flags, const char* what, int (*apply)()) {
    int dev = 0;
    int rc = cuda_status(cudaGetDevice(&dev), what);
    if (rc) return rc;
    if (dev < 0 || dev >= MAX_DEV) return apply();   // beyond the flag table: set it on every call
    if (flags[dev].load(std::memory_order_acquire)) return KV800_OK;
    rc = apply();
    if (!rc) flags[dev].store(1, std::memory_order_release);
    return rc;
}

static int qdecode_setup() {
    static std::atomic<int> done[MAX_DEV];
    return set_smem_once(done, "qdecode_mma smem attribute", [] {
        return cuda_status(cudaFuncSetAttribute(qdecode_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, QM_SMEM_TMA),
                           "qdecode_mma smem attribute");
    });
}

static int xdecode_setup() {
    static std::atomic<int> done[MAX_DEV];
    return set_smem_once(done, "xdecode_mma smem attribute", [] {
        int rc = cuda_status(cudaFuncSetAttribute(xdecode_mma<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  XM_SMEM),
                             "xdecode_mma smem attribute");
        if (rc) return rc;
        return cuda_status(cudaFuncSetAttribute(xdecode_mma<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, XM_SMEM),
                           "xdecode_mma smem attribute");
    });
}

// Launch the exact-token partials: with tables, or (both tables null) the no-rotation form of native sliding layers.
// Launch configuration of a 128-thread kernel; early = programmatic dependent launch (the kernel may start while the
// one before it in the stream still runs, and waits for it with griddepcontrol.wait where it reads its results).
struct LaunchCfg {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr;
    LaunchCfg(dim3 grid, size_t smem, cudaStream_t st, bool early, unsigned threads = 128) : cfg{}, attr{} {
        cfg.gridDim = grid;
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr.val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = early ? 1 : 0;
    }
};

// Stages of the tensor-map form's ring (one warp per CTA, 31.5 KB of shared memory with three stages).
constexpr int XT_S = 3;

static int xtma_setup() {
    static std::atomic<int> done[MAX_DEV];
    return set_smem_once(done, "xdecode_tma smem attribute", [] {
        int rc = cuda_status(cudaFuncSetAttribute(xdecode_tma<true, XT_S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  xt_smem<XT_S>()),
                             "xdecode_tma smem attribute");
        if (rc) return rc;
        return cuda_status(cudaFuncSetAttribute(xdecode_tma<false, XT_S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                xt_smem<XT_S>()),
                           "xdecode_tma smem attribute");
    });
}

// The tensor-map form applies to exact pools in the reference's page layout (K | V rows of 512 bytes per (head, slot),
// heads a whole number of rows apart, pages of a multiple of 16 slots) with at most 16 sinks; the tensor map is then
// the pool as rows of 256 bf16.  Other layouts take the gather form.
static bool xtma_layout(const kv800_paged& P) {
    const int64_t rows = P.epool_elems / 256;
    return P.e_ts == 256 && P.e_v == 128 && P.e_hs >= 0 && P.e_hs % 256 == 0 && P.ebs % 16 == 0 &&
           !(reinterpret_cast<uintptr_t>(P.epool) & 15u) && rows >= 16 && rows + 3 * (P.e_hs / 256) < 0x7fffffffLL &&
           (!P.sk || P.nsink <= XT_MAX_SINK);
}

static int make_emap(const kv800_paged& P, CUtensorMap& tm) {
    PFN_cuTensorMapEncodeTiled encode = nullptr;
    const int rce = tensor_map_encoder(encode);
    if (rce) return rce;
    cuuint64_t dims[2] = {256, (cuuint64_t)(P.epool_elems / 256)};
    cuuint64_t strides[1] = {512};
    cuuint32_t box[2] = {64, 16}, es[2] = {1, 1};
    const CUresult r = encode(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(P.epool), dims, strides,
                              box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (exact pool) failed (%d)", (int)r);
        return KV800_ERR_CUDA;
    }
    return KV800_OK;
}

// Host-side preparation of the exact partials (kernel attributes, and the exact pool's tensor map for the
// tensor-map form, whose encoding is host work of a few microseconds), done before a decode submits its first GPU
// operation so that its launches reach the stream back to back.
struct XPrep {
    bool tma = false;
    XTArgs ta{};
};
static int prepare_xdecode(const XMArgs& xa, XPrep& xp) {
    xp.tma = xtma_layout(xa.P);
    if (!xp.tma) return xdecode_setup();
    int rc = xtma_setup();
    if (rc) return rc;
    rc = make_emap(xa.P, xp.ta.tm);
    if (rc) return rc;
    xp.ta.x = xa;
    xp.ta.ehs_rows = xa.P.e_hs / 256;
    return KV800_OK;
}

// Launch the exact partials of B rows x nx splits: the tensor-map form (one warp per (row, split, head)) where the
// layout allows it, else the gather form (a 4-warp CTA per (row, split)).  early: the exact partials do not read the
// quantized ones (the row merge waits for them).
static void launch_xdecode_prepared(const XPrep& xp, const XMArgs& xa, int64_t B, int nx, cudaStream_t st,
                                    bool early) {
    if (xp.tma) {
        LaunchCfg lc(dim3((unsigned)B, (unsigned)nx, HEADS), xt_smem<XT_S>(), st, early, 32);
        if (xa.cos_t) cudaLaunchKernelEx(&lc.cfg, xdecode_tma<true, XT_S>, xp.ta);
        else cudaLaunchKernelEx(&lc.cfg, xdecode_tma<false, XT_S>, xp.ta);
        return;
    }
    LaunchCfg lc(dim3((unsigned)B, (unsigned)nx), XM_SMEM, st, early);
    if (xa.cos_t) cudaLaunchKernelEx(&lc.cfg, xdecode_mma<true>, xa);
    else cudaLaunchKernelEx(&lc.cfg, xdecode_mma<false>, xa);
}

static int launch_xdecode(const XMArgs& xa, int64_t B, int nx, cudaStream_t st, bool early = false) {
    XPrep xp;
    const int rc = prepare_xdecode(xa, xp);
    if (rc) return rc;
    launch_xdecode_prepared(xp, xa, B, nx, st, early);
    return KV800_OK;
}

// Tables: both given (16-byte aligned, npos > 0), or both null when nothing quantized is decoded (no rotation).
static int check_tables(const uint16_t* cos_t, const uint16_t* sin_t, int64_t npos, bool quantized, const char* who) {
    if (!cos_t && !sin_t) {
        if (quantized) {
            set_error("%s: quantized sub-blocks need the cos / sin tables (null tables mean no rotation, for layers "
                      "without quantized sub-blocks only)", who);
            return KV800_ERR_ARG;
        }
        return KV800_OK;
    }
    if (!cos_t || !sin_t || npos <= 0) {
        set_error("%s: give both cos / sin tables with npos > 0, or neither", who);
        return KV800_ERR_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(cos_t) | reinterpret_cast<uintptr_t>(sin_t)) & 15u) {
        set_error("%s: cos / sin tables must be 16-byte aligned", who);
        return KV800_ERR_ARG;
    }
    return KV800_OK;
}

// The decode of kv800_decode; ev (4 events or null) is recorded before the quantized partials, after them, after the
// exact partials and after the combine.
static int decode_core(const kv800_paged* P, const uint16_t* q, const uint16_t* cos_t, const uint16_t* sin_t,
                       int64_t npos, int64_t B, int64_t spb, uint16_t* out, void* workspace, int64_t workspace_bytes,
                       void* stream, cudaEvent_t* ev) {
    int rc = check_paged(P, "kv800_decode");
    if (rc) return rc;
    if (B < 0 || B > MAX_B) {
        set_error("kv800_decode: batch %lld outside [0, %lld]", (long long)B, (long long)MAX_B);
        return B < 0 ? KV800_ERR_ARG : KV800_ERR_RANGE;
    }
    if (B == 0) return KV800_OK;
    if (!q || !out || !workspace) {
        set_error("kv800_decode: null q / out / workspace");
        return KV800_ERR_ARG;
    }
    rc = check_tables(cos_t, sin_t, npos, P->win == 0 && P->nqmax > 0, "kv800_decode");
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(q) & 15u) {
        set_error("kv800_decode: q must be 16-byte aligned");
        return KV800_ERR_ARG;
    }
    if (reinterpret_cast<uintptr_t>(out) & 7u) {
        set_error("kv800_decode: out must be 8-byte aligned");
        return KV800_ERR_ARG;
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) {
        set_error("kv800_decode: workspace must be 256-byte aligned");
        return KV800_ERR_ARG;
    }
    const Plan pl = make_plan(B, P->nqmax, P->win, spb);
    if (pl.ns > 65535) {
        set_error("kv800_decode: %lld splits above the grid limit (raise spb)", (long long)pl.ns);
        return KV800_ERR_RANGE;
    }
    if (workspace_bytes < pl.bytes) {
        set_error("kv800_decode: workspace of %lld bytes, %lld needed", (long long)workspace_bytes,
                  (long long)pl.bytes);
        return KV800_ERR_RANGE;
    }
    cudaStream_t st = as_stream(stream);
    char* ws = static_cast<char*>(workspace);
    int* status = reinterpret_cast<int*>(ws);
    int64_t* prefix = reinterpret_cast<int64_t*>(ws + pl.prefix_off);
    float* mo = reinterpret_cast<float*>(ws + pl.mo_off);
    float* lo = reinterpret_cast<float*>(ws + pl.lo_off);
    float* ao = reinterpret_cast<float*>(ws + pl.ao_off);
    int* count = reinterpret_cast<int*>(ws + pl.cnt_off);
    // ---- host-side preparation first (kernel attributes, tensor maps, the slot map), so that the GPU work below
    // reaches the stream back to back and no device time waits on host encoding
    const bool needq = pl.persistent || pl.ns > 0;
    const int64_t rowslots = pl.ns + pl.nx;
    QMArgs qa{q, P->qpool, P->qpool_bytes, P->boff, P->boff_stride, P->NQ, P->nqmax, cos_t, sin_t, npos,
              mo, lo, ao, pl.persistent ? 0 : (int)rowslots, pl.persistent ? 0 : (int)spb, SCALE, status,
              pl.persistent ? prefix : nullptr, B, 0x40804080u};
    if (needq) {
        rc = qdecode_setup();
        if (rc) return rc;
        rc = make_qmaps(qa.qpool, qa.qpool_bytes, qa);
        if (rc) return rc;
    }
    SlotMap sm{};
    sm.nx = pl.nx;
    if (pl.persistent) {
        sm.prefix = prefix;
        sm.B = B;
        sm.G0 = pl.G0;
        sm.xbase = pl.G0 + B;
        sm.xstride = pl.nx;
    } else {
        sm.ns = (int)pl.ns;
        sm.qstride = rowslots;
        sm.xbase = pl.ns;
        sm.xstride = rowslots;
    }
    // the exact partials; the last of a row's pl.nx CTAs to finish also merges the row's partials into out
    XMArgs xa{q, *P, cos_t, sin_t, npos, mo, lo, ao, sm.xbase, sm.xstride, pl.nx, SCALE, status, count, sm, out};
    XPrep xp;
    rc = prepare_xdecode(xa, xp);
    if (rc) return rc;

    // ---- GPU work
    if (!pl.persistent) {   // (the persistent pass clears them in its schedule scan)
        rc = cuda_status(cudaMemsetAsync(status, 0, pl.cnt_off + 4 * HEADS * B, st),
                         "kv800_decode status / counter reset");
        if (rc) return rc;
    }
    if (ev) cudaEventRecord(ev[0], st);
    if (pl.persistent) {
        qsched_kernel<<<1, 1024, 0, st>>>(P->NQ, P->nqmax, B, prefix, status, (pl.cnt_off + 4 * HEADS * B) / 4);
        rc = cuda_status(cudaGetLastError(), "kv800_decode schedule");
        if (rc) return rc;
        {   // behind the schedule scan, early in untimed calls: the CTAs are placed while the scan runs and wait for
            // its prefix
            LaunchCfg lc(dim3((unsigned)pl.G0), QM_SMEM_TMA, st, !ev);
            cudaLaunchKernelEx(&lc.cfg, qdecode_mma, qa);
        }
        rc = cuda_status(cudaGetLastError(), "kv800_decode qdecode");
        if (rc) return rc;
    } else if (pl.ns > 0) {
        qdecode_mma<<<dim3((unsigned)B, (unsigned)pl.ns), 128, QM_SMEM_TMA, st>>>(qa);
        rc = cuda_status(cudaGetLastError(), "kv800_decode qdecode");
        if (rc) return rc;
    }
    if (ev) cudaEventRecord(ev[1], st);
    // early behind a persistent quantized pass (untimed calls): the exact partials fill the SMs its CTAs leave
    launch_xdecode_prepared(xp, xa, B, pl.nx, st, pl.persistent && !ev);
    rc = cuda_status(cudaGetLastError(), "kv800_decode xdecode");
    if (ev) cudaEventRecord(ev[2], st);
    if (ev) cudaEventRecord(ev[3], st);
    return rc;
}

extern "C" int kv800_decode(const kv800_paged* P, const uint16_t* q, const uint16_t* cos_t, const uint16_t* sin_t,
                            int64_t npos, int64_t B, int64_t spb, uint16_t* out, void* workspace,
                            int64_t workspace_bytes, void* stream) {
    return decode_core(P, q, cos_t, sin_t, npos, B, spb, out, workspace, workspace_bytes, stream, nullptr);
}

extern "C" int kv800_decode_timed(const kv800_paged* P, const uint16_t* q, const uint16_t* cos_t,
                                  const uint16_t* sin_t, int64_t npos, int64_t B, int64_t spb, uint16_t* out,
                                  void* workspace, int64_t workspace_bytes, void* stream, float* ms) {
    if (!ms) {
        set_error("kv800_decode_timed: null ms");
        return KV800_ERR_ARG;
    }
    cudaEvent_t ev[4];
    for (int i = 0; i < 4; i++) {
        const int rc = cuda_status(cudaEventCreate(&ev[i]), "kv800_decode_timed event");
        if (rc) {
            for (int j = 0; j < i; j++) cudaEventDestroy(ev[j]);
            return rc;
        }
    }
    int rc = decode_core(P, q, cos_t, sin_t, npos, B, spb, out, workspace, workspace_bytes, stream, ev);
    if (!rc) rc = cuda_status(cudaEventSynchronize(ev[3]), "kv800_decode_timed sync");
    for (int i = 0; i < 3 && !rc; i++) rc = cuda_status(cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]), "elapsed");
    for (int i = 0; i < 4; i++) cudaEventDestroy(ev[i]);
    return rc;
}

extern "C" int kv800_qdecode(const uint16_t* q, const uint8_t* qpool, int64_t qpool_bytes, const int64_t* boff,
                             int64_t boff_stride, const int32_t* NQ, const uint16_t* cos_t, const uint16_t* sin_t,
                             int64_t npos, float* mo, float* lo, float* ao, int64_t B, int64_t ns, int64_t spb,
                             int64_t nqmax, float scale, int* status, void* stream) {
    if (B < 0 || ns < 0 || spb <= 0) {
        set_error("kv800_qdecode: negative B / ns or spb <= 0");
        return KV800_ERR_ARG;
    }
    if (B == 0 || ns == 0) return KV800_OK;
    if (!q || !qpool || !boff || !NQ || !cos_t || !sin_t || !mo || !lo || !ao || boff_stride <= 0) {
        set_error("kv800_qdecode: null pointer or boff_stride <= 0");
        return KV800_ERR_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(cos_t) | reinterpret_cast<uintptr_t>(sin_t)) & 15u) {
        set_error("kv800_qdecode: cos / sin tables must be 16-byte aligned");
        return KV800_ERR_ARG;
    }
    if (B > MAX_B || ns > 65535) {
        set_error("kv800_qdecode: B %lld / ns %lld above the limits", (long long)B, (long long)ns);
        return KV800_ERR_RANGE;
    }
    int rc0 = qdecode_setup();
    if (rc0) return rc0;
    QMArgs qa{q, qpool, qpool_bytes, boff, boff_stride, NQ, nqmax, cos_t, sin_t, npos,
              mo, lo, ao, (int)(ns + 1), (int)spb, scale, status, nullptr, B, 0x40804080u};
    const int rcm = make_qmaps(qa.qpool, qa.qpool_bytes, qa);
    if (rcm) return rcm;
    qdecode_mma<<<dim3((unsigned)B, (unsigned)ns), 128, QM_SMEM_TMA, as_stream(stream)>>>(qa);
    return cuda_status(cudaGetLastError(), "kv800_qdecode launch");
}

extern "C" int kv800_xdecode(const uint16_t* q, const kv800_paged* P, const uint16_t* cos_t, const uint16_t* sin_t,
                             int64_t npos, float* mo, float* lo, float* ao, int64_t B, int64_t ns, float scale,
                             int* status, void* stream) {
    int rc = check_paged(P, "kv800_xdecode");
    if (rc) return rc;
    if (B < 0 || ns < 0) {
        set_error("kv800_xdecode: negative B / ns");
        return KV800_ERR_ARG;
    }
    if (B == 0) return KV800_OK;
    if (!q || !mo || !lo || !ao) {
        set_error("kv800_xdecode: null pointer");
        return KV800_ERR_ARG;
    }
    rc = check_tables(cos_t, sin_t, npos, false, "kv800_xdecode");
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(ao) & 15u) {
        set_error("kv800_xdecode: ao must be 16-byte aligned");
        return KV800_ERR_ARG;
    }
    if (B > MAX_B) {
        set_error("kv800_xdecode: B %lld above the limit", (long long)B);
        return KV800_ERR_RANGE;
    }
    XMArgs xa{q, *P, cos_t, sin_t, npos, mo, lo, ao, ns, ns + 1, 1, scale, status, nullptr, SlotMap{}, nullptr};
    const int rcx = launch_xdecode(xa, B, 1, as_stream(stream));
    if (rcx) return rcx;
    return cuda_status(cudaGetLastError(), "kv800_xdecode launch");
}

extern "C" int kv800_combine(const float* mo, const float* lo, const float* ao, int64_t B, int64_t ns, uint16_t* out,
                             void* stream) {
    if (B < 0 || ns < 0) {
        set_error("kv800_combine: negative B / ns");
        return KV800_ERR_ARG;
    }
    if (B == 0) return KV800_OK;
    if (!mo || !lo || !ao || !out) {
        set_error("kv800_combine: null pointer");
        return KV800_ERR_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(ao) & 15u) || (reinterpret_cast<uintptr_t>(out) & 7u)) {
        set_error("kv800_combine: ao must be 16-byte and out 8-byte aligned");
        return KV800_ERR_ARG;
    }
    SlotMap sm{};
    sm.ns = (int)ns;
    sm.qstride = ns + 1;
    sm.xbase = ns;
    sm.xstride = ns + 1;
    sm.nx = 1;
    combine_kernel<<<(unsigned)B, 128, 0, as_stream(stream)>>>(mo, lo, ao, sm, out);
    return cuda_status(cudaGetLastError(), "kv800_combine launch");
}
