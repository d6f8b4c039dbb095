// Device-side pieces of one vLLM step over the 800h caches (lfm3_kv800/vllm_attn.py:244-402), so that a step builds no
// index tensors and takes no host loop:
//   write_sinks     positions < 4 of a window layer into the aux area of the request's first quant page
//                   (vllm_attn.py:276-291)
//   decode_tables   N / NQ / EOFF / BOFF (and the sink offsets of window layers) of the decode rows from the block
//                   tables (vllm_attn.py:320-349)
//   prefill_kv      the K / V of a prefill or extend request in position order: dequantized history sub-blocks,
//                   sinks, exact window rows and the new chunk, K rotated (HF RoPE, bf16) unless the layer is a native
//                   sliding one, all bf16 (vllm_attn.py:355-388 and kv800.py:79-92).
// The exact-cache scatter (write_slots) and the flush (flush_step) live beside the quantizer in flush.cu.
#include <cstdint>

#include "hadamard.cuh"
#include "kv800_common.cuh"

namespace kv800 {

// request owning token i: the b with qsl[b] <= i < qsl[b + 1] (qsl non-decreasing, R + 1 entries)
__device__ __forceinline__ int64_t request_of(const int32_t* qsl, int64_t R, int64_t i) {
    int64_t lo = 0, hi = R;   // invariant: qsl[lo] <= i < qsl[hi]
    while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (qsl[mid] <= i) lo = mid;
        else hi = mid;
    }
    return lo;
}

// One warp per (token, head, K|V) row of 128 bf16.  The sink row of (position p < 4, head h) sits at element
// bt[b * bts] * s0 + aux + (p * 4 + h) * 128 of the host cache (bf16 view); K and V go to two different hosts.
__global__ void write_sinks_kernel(uint16_t* hk, int64_t hk_elems, int64_t hk_s0, int64_t hk_aux, const int32_t* hk_bt,
                                   int64_t hk_bts, uint16_t* hv, int64_t hv_elems, int64_t hv_s0, int64_t hv_aux,
                                   const int32_t* hv_bt, int64_t hv_bts, const uint16_t* k, const uint16_t* v,
                                   const int64_t* pos, const int64_t* slot, const int32_t* qsl, int64_t R, int64_t T,
                                   int* status) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= T * HEADS * 2) return;
    const int64_t i = row / (HEADS * 2);
    const int h = (int)((row / 2) % HEADS), isv = (int)(row & 1);
    const int64_t p = pos[i];
    if (p < 0 || p >= NSINK || slot[i] < 0 || i >= qsl[R]) return;
    const int64_t b = request_of(qsl, R, i);
    const int64_t o = isv ? (int64_t)hv_bt[b * hv_bts] * hv_s0 + hv_aux + (p * HEADS + h) * DIM
                          : (int64_t)hk_bt[b * hk_bts] * hk_s0 + hk_aux + (p * HEADS + h) * DIM;
    const int64_t lim = isv ? hv_elems : hk_elems;
    if (o < 0 || o + DIM > lim) {
        if (lane == 0) flag(status, ST_SINK);
        return;
    }
    const uint16_t* srow = (isv ? v : k) + (i * HEADS + h) * DIM;
    uint16_t* drow = (isv ? hv : hk) + o;
#pragma unroll
    for (int e = 0; e < 4; e++) drow[lane * 4 + e] = srow[lane * 4 + e];
}

struct TableArgs {
    const int32_t* seq_lens;   // [nd]
    int64_t nd;
    const int32_t* bt;         // exact block table, row stride bts
    int64_t bts, s0;
    int32_t* N;
    int32_t* NQ;
    int64_t* eoff;             // [nd, bts]
    const int32_t* qbt;        // quant block table (quantized layers), row stride qbts
    int64_t qbts, qs0, bsq, nqw;
    int64_t* boff;             // [nd, nqw]
    const int32_t* skbt;       // sink hosts' block tables (window layers)
    int64_t skbts, sk_s0, sk_aux;
    int64_t* skoff;            // [nd]
    const int32_t* svbt;
    int64_t svbts, sv_s0, sv_aux;
    int64_t* svoff;
};

// Grid-stride over nd x (bts + nqw + 1) outputs.  BOFF entries past a row's own NQ (or past its block table) are 0:
// the decode kernels never read them.
__global__ void decode_tables_kernel(TableArgs a) {
    const int64_t per = a.bts + a.nqw + 1;
    const int64_t total = a.nd * per;
    for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < total; x += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = x / per, c = x % per;
        const int64_t n = a.seq_lens[b];
        if (c < a.bts) {
            a.eoff[b * a.bts + c] = (int64_t)a.bt[b * a.bts + c] * a.s0;
        } else if (c < a.bts + a.nqw) {
            const int64_t j = c - a.bts;
            const int64_t nq = n > LAG ? (n - LAG) / BLK : 0;
            const int64_t tok0 = j * BLK;
            int64_t o = 0;
            if (j < nq && tok0 / a.bsq < a.qbts)
                o = (int64_t)a.qbt[b * a.qbts + tok0 / a.bsq] * a.qs0 + ((tok0 % a.bsq) / BLK) * SUB;
            a.boff[b * a.nqw + j] = o;
        } else {
            a.N[b] = (int32_t)n;
            a.NQ[b] = a.qbt ? (int32_t)(n > LAG ? (n - LAG) / BLK : 0) : 0;
            if (a.skoff) a.skoff[b] = (int64_t)a.skbt[b * a.skbts] * a.sk_s0 + a.sk_aux;
            if (a.svoff) a.svoff[b] = (int64_t)a.svbt[b * a.svbts] * a.sv_s0 + a.sv_aux;
        }
    }
}

// HF apply_rotary_pos_emb of one K row held by a lane as dims lane + 32 p (p = 0..3), in the reference's operation
// order (vllm_attn.py:162-165): kf * cos + rotate_half(kf) * sin as two fp32 products and one fp32 add, then bf16.
// cos / sin are [P, 32] bf16; the 128-dim tables repeat them for dims 0-31 and 64-95 and are 1 / 0 elsewhere.
__device__ __forceinline__ void rope_row(const float (&k)[4], float c, float s, uint16_t (&o)[4]) {
    o[0] = f2bf(__fadd_rn(__fmul_rn(k[0], c), __fmul_rn(-k[2], s)));
    o[1] = f2bf(__fadd_rn(__fmul_rn(k[1], 1.0f), __fmul_rn(-k[3], 0.0f)));
    o[2] = f2bf(__fadd_rn(__fmul_rn(k[2], c), __fmul_rn(k[0], s)));
    o[3] = f2bf(__fadd_rn(__fmul_rn(k[3], 1.0f), __fmul_rn(k[1], 0.0f)));
}

struct PrefillArgs {
    // quantized history: sub-blocks j < nqp of the request at qcache + qbt[(256 j) / bsq] * qs0 + ...
    const uint8_t* qcache;
    int64_t qcache_bytes, qs0, bsq;
    const int32_t* qbt;        // the request's row of the quant block table
    int64_t qbt_len, nqp;
    // sinks (window layers): ns rows, K at sk + (p * 4 + h) * 128, V at sv + ...
    const uint16_t* sk;
    const uint16_t* sv;
    int64_t ns;
    // exact rows [lo, n0): ecache + bt[p / ebs] * s0 + h * s1 + (p % ebs) * s2, V at + 128
    const uint16_t* ecache;
    int64_t ecache_elems, s0, s1, s2, ebs;
    const int32_t* bt;         // the request's row of the exact block table
    int64_t bt_len, lo, n0;
    // the new chunk: positions n0 .. n - 1, (n - n0, 4, 128) bf16
    const uint16_t* k;
    const uint16_t* v;
    int64_t n;
    const uint16_t* cos_t;     // [P, 32] bf16; nullptr = no rotation (native sliding layer)
    const uint16_t* sin_t;
    int64_t npos;
    uint16_t* kout;            // (S, 4, 128) bf16, S = 256 nqp + ns + (n0 - lo) + (n - n0)
    uint16_t* vout;
    int* status;
};

// Quantized history, grid (nqp, 8): 32 tokens per CTA, warp = 4 tokens.  K = bf16(code * ksc + klo) then RoPE; V =
// bf16 of the fp32 Hadamard rotation of bits * vsc + vlo (the dequantizer's exact arithmetic).
__global__ void __launch_bounds__(256) prefill_quant_kernel(PrefillArgs a) {
    const int64_t m = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t tok0 = m * BLK;
    if (tok0 / a.bsq >= a.qbt_len) {
        flag(a.status, ST_TABLE);
        return;
    }
    const int64_t off = (int64_t)a.qbt[tok0 / a.bsq] * a.qs0 + ((tok0 % a.bsq) / BLK) * SUB;
    if (off < 0 || off + SUB > a.qcache_bytes) {
        flag(a.status, ST_QPOOL);
        return;
    }
    const uint8_t* sb = a.qcache + off;
    __shared__ float vbuf[8][HEADS * DIM];
    float C[32];
    hadamard_signs(lane, C);
    for (int tt = 0; tt < 4; tt++) {
        const int t = blockIdx.y * 32 + warp * 4 + tt;
        const int64_t p = tok0 + t;
        float c = 1.f, s = 0.f;
        if (a.cos_t) {
            if (p >= a.npos) {
                flag(a.status, ST_TABLE);
                return;
            }
            c = bf2f(a.cos_t[p * 32 + lane]);
            s = bf2f(a.sin_t[p * 32 + lane]);
        }
#pragma unroll
        for (int h = 0; h < HEADS; h++) {
            const uint32_t byte = sb[KC_O + (t * HEADS + h) * 32 + lane];
            float kx[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int d = lane + 32 * q;
                const float sc = f8dec(sb[KSC_O + h * DIM + d]), lo = f8dec(sb[KLO_O + h * DIM + d]);
                kx[q] = bfround((float)((byte >> (2 * q)) & 3u) * sc + lo);
            }
            uint16_t o[4];
            if (a.cos_t) {
                rope_row(kx, c, s, o);
            } else {
#pragma unroll
                for (int q = 0; q < 4; q++) o[q] = f2bf(kx[q]);
            }
            uint16_t* kr = a.kout + (p * HEADS + h) * DIM;
#pragma unroll
            for (int q = 0; q < 4; q++) kr[lane + 32 * q] = o[q];
        }
#pragma unroll
        for (int h = 0; h < HEADS; h++) {
            const float vlo = f8dec(sb[VLO_O + t * 2 + (h >> 1)]), vsc = f8dec(sb[VSC_O + t * 2 + (h >> 1)]);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int d = lane + 32 * q;
                const uint32_t bit = (sb[VB_O + (t * HEADS + h) * 16 + (d & 15)] >> (d >> 4)) & 1u;
                vbuf[warp][h * DIM + d] = (float)bit * vsc + vlo;
            }
        }
        __syncwarp();
        float y[HEADS][4];
        hadamard_rows(vbuf[warp], C, y);
#pragma unroll
        for (int h = 0; h < HEADS; h++)
#pragma unroll
            for (int q = 0; q < 4; q++) a.vout[(p * HEADS + h) * DIM + lane + 32 * q] = f2bf(y[h][q]);
        __syncwarp();
    }
}

// Sinks, exact rows and the chunk: one warp per (row, head).  Row r < ns is sink position r; the next n0 - lo rows are
// exact positions lo ..; the last n - n0 are the chunk.  Output row = 256 nqp + r.
__global__ void prefill_rows_kernel(PrefillArgs a) {
    const int64_t rows = a.ns + (a.n0 - a.lo) + (a.n - a.n0);
    const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= rows * HEADS) return;
    const int64_t r = w / HEADS;
    const int h = (int)(w % HEADS);
    const uint16_t *kr = nullptr, *vr = nullptr;
    int64_t p;
    if (r < a.ns) {
        p = r;
        kr = a.sk + (p * HEADS + h) * DIM;
        vr = a.sv + (p * HEADS + h) * DIM;
    } else if (r < a.ns + (a.n0 - a.lo)) {
        p = a.lo + (r - a.ns);
        int64_t pg, sl;
        page_split(p, a.ebs, pg, sl);
        if (pg >= a.bt_len) {
            if (lane == 0) flag(a.status, ST_TABLE);
            return;
        }
        const int64_t o = (int64_t)a.bt[pg] * a.s0 + h * a.s1 + sl * a.s2;
        if (o < 0 || o + 128 + DIM > a.ecache_elems) {
            if (lane == 0) flag(a.status, ST_EPOOL);
            return;
        }
        kr = a.ecache + o;
        vr = a.ecache + o + 128;
    } else {
        const int64_t i = r - a.ns - (a.n0 - a.lo);
        p = a.n0 + i;
        kr = a.k + (i * HEADS + h) * DIM;
        vr = a.v + (i * HEADS + h) * DIM;
    }
    const int64_t orow = (a.nqp * BLK + r) * HEADS + h;
    float kx[4];
#pragma unroll
    for (int q = 0; q < 4; q++) kx[q] = bf2f(kr[lane + 32 * q]);
    uint16_t o[4];
    if (a.cos_t) {
        if (p >= a.npos) {
            if (lane == 0) flag(a.status, ST_TABLE);
            return;
        }
        rope_row(kx, bf2f(a.cos_t[p * 32 + lane]), bf2f(a.sin_t[p * 32 + lane]), o);
    } else {
#pragma unroll
        for (int q = 0; q < 4; q++) o[q] = f2bf(kx[q]);
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
        a.kout[orow * DIM + lane + 32 * q] = o[q];
        a.vout[orow * DIM + lane + 32 * q] = vr[lane + 32 * q];
    }
}

}  // namespace kv800

using namespace kv800;

extern "C" int kv800_write_sinks(uint16_t* hk, int64_t hk_elems, int64_t hk_s0, int64_t hk_aux, const int32_t* hk_bt,
                                 int64_t hk_bts, uint16_t* hv, int64_t hv_elems, int64_t hv_s0, int64_t hv_aux,
                                 const int32_t* hv_bt, int64_t hv_bts, const uint16_t* k, const uint16_t* v,
                                 const int64_t* positions, const int64_t* slot_mapping, const int32_t* query_start_loc,
                                 int64_t R, int64_t T, int* status, void* stream) {
    if (T < 0 || R < 0) {
        set_error("kv800_write_sinks: negative T or R");
        return KV800_ERR_ARG;
    }
    if (T == 0 || R == 0) return KV800_OK;
    if (!hk || !hv || !hk_bt || !hv_bt || !k || !v || !positions || !slot_mapping || !query_start_loc ||
        hk_bts <= 0 || hv_bts <= 0) {
        set_error("kv800_write_sinks: null pointer or empty block table");
        return KV800_ERR_ARG;
    }
    const int64_t blocks = (T * HEADS * 2 + 7) / 8;
    if (blocks > 0x7fffffffLL) {
        set_error("kv800_write_sinks: T = %lld too large", (long long)T);
        return KV800_ERR_RANGE;
    }
    write_sinks_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(hk, hk_elems, hk_s0, hk_aux, hk_bt, hk_bts, hv,
                                                                       hv_elems, hv_s0, hv_aux, hv_bt, hv_bts, k, v,
                                                                       positions, slot_mapping, query_start_loc, R, T,
                                                                       status);
    return cuda_status(cudaGetLastError(), "kv800_write_sinks launch");
}

extern "C" int kv800_decode_tables(const int32_t* seq_lens, int64_t nd, const int32_t* block_table, int64_t bt_stride,
                                   int64_t s0, int32_t* N, int32_t* NQ, int64_t* eoff, const int32_t* qblock_table,
                                   int64_t qbt_stride, int64_t qs0, int64_t bsq, int64_t nqw, int64_t* boff,
                                   const int32_t* sk_bt, int64_t sk_bts, int64_t sk_s0, int64_t sk_aux, int64_t* skoff,
                                   const int32_t* sv_bt, int64_t sv_bts, int64_t sv_s0, int64_t sv_aux, int64_t* svoff,
                                   void* stream) {
    if (nd < 0 || nqw < 0) {
        set_error("kv800_decode_tables: negative nd / nqw");
        return KV800_ERR_ARG;
    }
    if (nd == 0) return KV800_OK;
    if (!seq_lens || !block_table || bt_stride <= 0 || !N || !NQ || !eoff) {
        set_error("kv800_decode_tables: null pointer or empty exact block table");
        return KV800_ERR_ARG;
    }
    if (nqw > 0 && (!qblock_table || qbt_stride <= 0 || !boff || bsq <= 0 || bsq % BLK)) {
        set_error("kv800_decode_tables: BOFF requested without a quant block table (bsq a multiple of 256)");
        return KV800_ERR_ARG;
    }
    if ((skoff && (!sk_bt || sk_bts <= 0)) || (svoff && (!sv_bt || sv_bts <= 0))) {
        set_error("kv800_decode_tables: sink offsets requested without the hosts' block tables");
        return KV800_ERR_ARG;
    }
    TableArgs a{seq_lens, nd, block_table, bt_stride, s0, N, NQ, eoff, nqw > 0 ? qblock_table : nullptr, qbt_stride,
                qs0, bsq, nqw, boff, sk_bt, sk_bts, sk_s0, sk_aux, skoff, sv_bt, sv_bts, sv_s0, sv_aux, svoff};
    const int64_t total = nd * (bt_stride + nqw + 1);
    const int64_t want = (total + 255) / 256;
    const unsigned blocks = (unsigned)(want < 4096 ? want : 4096);
    decode_tables_kernel<<<blocks, 256, 0, as_stream(stream)>>>(a);
    return cuda_status(cudaGetLastError(), "kv800_decode_tables launch");
}

extern "C" int kv800_prefill_kv(const uint8_t* qcache, int64_t qcache_bytes, int64_t qs0, int64_t bsq,
                                const int32_t* qbt_row, int64_t qbt_len, int64_t nqp, const uint16_t* sk,
                                const uint16_t* sv, int64_t ns, const uint16_t* ecache, int64_t ecache_elems,
                                int64_t s0, int64_t s1, int64_t s2, int64_t ebs, const int32_t* bt_row, int64_t bt_len,
                                int64_t lo, int64_t n0, const uint16_t* k, const uint16_t* v, int64_t n,
                                const uint16_t* cos_t, const uint16_t* sin_t, int64_t npos, uint16_t* k_out,
                                uint16_t* v_out, int* status, void* stream) {
    if (nqp < 0 || ns < 0 || ns > NSINK || lo < 0 || n0 < lo || n < n0) {
        set_error("kv800_prefill_kv: need nqp >= 0, 0 <= ns <= 4, 0 <= lo <= n0 <= n");
        return KV800_ERR_ARG;
    }
    const int64_t rows = ns + (n0 - lo) + (n - n0);
    if (nqp + rows == 0) return KV800_OK;
    if (!k_out || !v_out || (nqp && (!qcache || !qbt_row || bsq <= 0 || bsq % BLK)) || (ns && (!sk || !sv)) ||
        (n0 > lo && (!ecache || !bt_row || ebs <= 0)) || (n > n0 && (!k || !v)) || ((cos_t == nullptr) != (sin_t == nullptr))) {
        set_error("kv800_prefill_kv: null pointer for a non-empty part, or bad bsq / ebs");
        return KV800_ERR_ARG;
    }
    if (nqp > 0x7fffffffLL || rows * HEADS / 8 + 1 > 0x7fffffffLL) {
        set_error("kv800_prefill_kv: too many rows");
        return KV800_ERR_RANGE;
    }
    PrefillArgs a{qcache, qcache_bytes, qs0, bsq, qbt_row, qbt_len, nqp, sk, sv, ns, ecache, ecache_elems, s0, s1, s2,
                  ebs, bt_row, bt_len, lo, n0, k, v, n, cos_t, sin_t, npos, k_out, v_out, status};
    cudaStream_t st = as_stream(stream);
    if (nqp) {
        prefill_quant_kernel<<<dim3((unsigned)nqp, 8), 256, 0, st>>>(a);
        const int rc = cuda_status(cudaGetLastError(), "kv800_prefill_kv quant launch");
        if (rc) return rc;
    }
    if (rows) {
        prefill_rows_kernel<<<(unsigned)((rows * HEADS + 7) / 8), 256, 0, st>>>(a);
        return cuda_status(cudaGetLastError(), "kv800_prefill_kv rows launch");
    }
    return KV800_OK;
}
