// 800h quantizer / flush on sm_100a: packs 256-token sub-blocks of bf16 K / V into the 51,200-byte layout, bit-exact
// with the reference torch quantizer (lfm3_kv800/kv800.py:56-76), plus the exact-page scatter of new tokens
// (kv800.py:423-428, vllm_attn.py:261-269).
//
// One launch covers M sub-blocks with grid (M, VSPLIT + HEADS); the long V CTAs come first in launch order:
//   blockIdx.y == 0..3     V part for 64 tokens: y = v @ H per head as the sequential fp32 FMA chain over i that the
//                          reference's CPU BLAS computes (bit-exact requirement), lo / hi per (token, 2-head group),
//                          1-bit codes, planar bytes.
//   blockIdx.y == 4..7     K part of head y - 4: 128 channels; lo / hi over the 256 tokens per channel, fp8 lo and
//                          scale (hi - lo) / 3, 2-bit codes (IEEE divide, round half to even), planar bytes.
// The V part is the arithmetic bound of the kernel (128 FMA per output element, 16.8 M FMA per sub-block); the K part
// streams 256 KB per sub-block twice (the second pass is served by L2), 32 tokens per thread per pass.
#include <cstdarg>
#include <cstdio>

#include "hadamard.cuh"
#include "kv800_common.cuh"

namespace kv800 {

// Where the 256 x 4 K / V rows of sub-block m come from and where its 51,200 bytes go.
// Row sources of the flush kernel.  kDirect: rows() is plain arithmetic, cheaper to evaluate per use than to
// broadcast; the paged sources look rows up through tables, so each warp resolves its rows once, one per lane.
struct ContigSrc {
    static constexpr bool kDirect = true;
    const uint16_t* k;
    const uint16_t* v;
    uint8_t* out;
    __device__ __forceinline__ bool rows(int64_t m, int t, int h, const uint16_t*& kr, const uint16_t*& vr) const {
        int64_t o = ((m * BLK + t) * HEADS + h) * DIM;
        kr = k + o;
        vr = v + o;
        return true;
    }
    __device__ __forceinline__ uint8_t* dst(int64_t m) const { return out + m * SUB; }
};

struct PagedSrc {
    static constexpr bool kDirect = false;
    const uint16_t* epool;
    int64_t epool_elems;
    const int64_t* eoff;
    int64_t eoff_stride, ebs, e_hs, e_ts, e_v;
    uint8_t* qpool;
    int64_t qpool_bytes;
    const int64_t* boff;
    int64_t boff_stride;
    const int32_t* seq;
    const int32_t* blk;
    int64_t nseq;
    int* status;
    __device__ __forceinline__ bool rows(int64_t m, int t, int h, const uint16_t*& kr, const uint16_t*& vr) const {
        int64_t b = seq[m], j = blk[m];
        int64_t p = j * BLK + t, pg, sl;
        page_split(p, ebs, pg, sl);
        if (b < 0 || b >= nseq || j < 0 || pg >= eoff_stride) {
            flag(status, ST_TABLE);
            return false;
        }
        int64_t o = eoff[b * eoff_stride + pg] + h * e_hs + sl * e_ts;
        if (o < 0 || o + DIM > epool_elems || o + e_v < 0 || o + e_v + DIM > epool_elems) {
            flag(status, ST_EPOOL);
            return false;
        }
        kr = epool + o;
        vr = epool + o + e_v;
        return true;
    }
    __device__ __forceinline__ uint8_t* dst(int64_t m) const {
        int64_t b = seq[m], j = blk[m];
        if (b < 0 || b >= nseq || j < 0 || j >= boff_stride) {
            flag(status, ST_TABLE);
            return nullptr;
        }
        int64_t o = boff[b * boff_stride + j];
        if (o < 0 || o + SUB > qpool_bytes) {
            flag(status, ST_QPOOL);
            return nullptr;
        }
        return qpool + o;
    }
};

// vLLM layout (vllm_attn.py:298-317): the exact cache is [blocks, 4, ebs, 256] bf16 addressed through a block
// table (row b of bt: block ids of request b), the quant cache is pages of qs0 bytes holding bsq / 256 sub-blocks each,
// addressed through qbt.  Sub-block m of the launch is pair m of a device-built list (request, sub-block index); CTAs
// past the list's count exit.
struct VllmSrc {
    static constexpr bool kDirect = false;
    const uint16_t* epool;
    int64_t epool_elems, s0, s1, s2, ebs;
    const int32_t* bt;
    int64_t bt_stride;
    uint8_t* qpool;
    int64_t qpool_bytes, qs0, bsq;
    const int32_t* qbt;
    int64_t qbt_stride;
    const int32_t* pairs;   // [2 * max] (request, sub-block)
    const int32_t* count;
    int64_t R;
    int* status;
    __device__ __forceinline__ bool rows(int64_t m, int t, int h, const uint16_t*& kr, const uint16_t*& vr) const {
        const int64_t b = pairs[2 * m], j = pairs[2 * m + 1];
        const int64_t p = j * BLK + t;
        int64_t pg, sl;
        page_split(p, ebs, pg, sl);
        if (b < 0 || b >= R || pg >= bt_stride) {
            flag(status, ST_TABLE);
            return false;
        }
        const int64_t blk = bt[b * bt_stride + pg];
        const int64_t o = blk * s0 + h * s1 + sl * s2;
        if (blk < 0 || o < 0 || o + 256 > epool_elems) {
            flag(status, ST_EPOOL);
            return false;
        }
        kr = epool + o;
        vr = epool + o + 128;
        return true;
    }
    __device__ __forceinline__ uint8_t* dst(int64_t m) const {
        if (m >= *count) return nullptr;
        const int64_t b = pairs[2 * m], j = pairs[2 * m + 1];
        const int64_t tok0 = j * BLK;
        if (b < 0 || b >= R || tok0 / bsq >= qbt_stride) {
            flag(status, ST_TABLE);
            return nullptr;
        }
        const int64_t blk = qbt[b * qbt_stride + tok0 / bsq];
        const int64_t o = blk * qs0 + ((tok0 % bsq) / BLK) * SUB;
        if (blk < 0 || o < 0 || o + SUB > qpool_bytes) {
            flag(status, ST_QPOOL);
            return nullptr;
        }
        return qpool + o;
    }
};

// Flush plan of one vLLM step on the device: request b (seq_len[b] tokens after the step, qlen[b] = qsl[b + 1] -
// qsl[b] of them new) owns sub-blocks j in [nq(seq_len[b] - qlen[b]), nq(seq_len[b])) with nq(n) = max(0, n - 128) /
// 256, the flush rule of vllm_attn.py:303-304; they are listed in request order as (b, j) pairs, at most max_pairs
// (more flags ST_TABLE and is cut).  One CTA of 1024 threads (block-wide scan); writes pairs [2 * max_pairs] and
// count.
__global__ void __launch_bounds__(1024) flush_plan_kernel(const int32_t* seq_len, const int32_t* qsl, int64_t R,
                                                          int64_t max_pairs, int32_t* pairs, int32_t* count,
                                                          int* status) {
    __shared__ int64_t wsum[32];
    __shared__ int64_t carry;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < R; base += 1024) {
        const int64_t b = base + tid;
        int64_t j0 = 0, n = 0;
        if (b < R) {
            const int64_t sl = seq_len[b], prev = sl - (int64_t)(qsl[b + 1] - qsl[b]);
            const int64_t a0 = prev > LAG ? (prev - LAG) / BLK : 0;
            const int64_t a1 = sl > LAG ? (sl - LAG) / BLK : 0;
            j0 = a0;
            n = a1 > a0 ? a1 - a0 : 0;
        }
        int64_t x = n;
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
            wsum[lane] = w;
        }
        __syncthreads();
        const int64_t start = carry + (warp ? wsum[warp - 1] : 0) + x - n;
        for (int64_t i = 0; i < n; i++) {
            if (start + i >= max_pairs) {
                flag(status, ST_TABLE);
                break;
            }
            pairs[2 * (start + i)] = (int32_t)b;
            pairs[2 * (start + i) + 1] = (int32_t)(j0 + i);
        }
        __syncthreads();
        if (tid == 0) carry += wsum[31];
        __syncthreads();
    }
    if (tid == 0) *count = (int32_t)(carry < max_pairs ? carry : max_pairs);
}

// Exact-cache scatter through vLLM's slot mapping (vllm_attn.py:261-269): token i goes to block slot[i] / ebs, row
// slot[i] % ebs; slot < 0 (padding) is skipped.  One warp per (token, head, K|V) row.
__global__ void write_slots_kernel(uint16_t* epool, int64_t epool_elems, int64_t s0, int64_t s1, int64_t s2,
                                   int64_t ebs, const uint16_t* k, const uint16_t* v, const int64_t* slot, int64_t T,
                                   int* status) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= T * HEADS * 2) return;
    const int64_t i = row / (HEADS * 2);
    const int h = (int)((row / 2) % HEADS), isv = (int)(row & 1);
    const int64_t sl = slot[i];
    if (sl < 0) return;
    int64_t blk, r;
    page_split(sl, ebs, blk, r);
    const int64_t o = blk * s0 + h * s1 + r * s2 + (isv ? 128 : 0);
    if (o < 0 || o + DIM > epool_elems) {
        if (lane == 0) flag(status, ST_EPOOL);
        return;
    }
    const uint16_t* srow = (isv ? v : k) + (i * HEADS + h) * DIM;
    uint16_t* drow = epool + o;
#pragma unroll
    for (int e = 0; e < 4; e++) drow[lane * 4 + e] = srow[lane * 4 + e];
}

constexpr int VSPLIT = 4;               // V-part CTAs per sub-block (64 tokens each)
constexpr int VTOK = BLK / VSPLIT;
static_assert(VTOK == 64, "the V part's 8 warps take 8 tokens each (row addresses resolved per lane)");

// 16 bf16 of a row at element offset e (e a multiple of 16), as fp32; vector loads when the row is 16-byte aligned.
__device__ __forceinline__ void load16(const uint16_t* row, int e, float* out) {
    const uint16_t* p = row + e;
    if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        uint4 a = *reinterpret_cast<const uint4*>(p);
        uint4 b = *reinterpret_cast<const uint4*>(p + 8);
        uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) out[i] = bf2f(p[i]);
    }
}


// 2-bit K code round(fl(d / sc)) clamped to [0, 3] (torch's .round().clamp(0, 3) of the IEEE quotient) from the
// cheap quotient q = d * (1 / sc), which is within 3 ulp of the IEEE one.  Only the rounding of quotients in
// [-0.5, 3.5] can change the clamped code, and there 3 ulp is below 1.5e-6: so where q is farther than 1.6e-5 from a
// half-integer both round alike, and near one the IEEE divide decides.  Non-finite q fail the distance test and
// clamp as the IEEE quotient does (NaN to 0, +inf to 3, -inf to 0).
__device__ __forceinline__ uint32_t code2(float d, float sc, float inv) {
    const float q = d * inv;
    const float r = rintf(q);
    if (fabsf(q - r) > 0.5f - 1.6e-5f) return round_clamp(__fdiv_rn(d, sc), 3.0f);
    return (uint32_t)fminf(fmaxf(r, 0.0f), 3.0f);
}

// 1-bit code round(fl(d / sc)) clamped to [0, 1], i.e. [fl(d / sc) > 1/2], from the cheap quotient as in code2.
__device__ __forceinline__ uint32_t code1(float d, float sc, float inv) {
    const float q = d * inv;
    const bool near = fabsf(q - 0.5f) <= 4e-6f * fmaxf(1.0f, fabsf(q)) || !isfinite(q);
    return near ? round_clamp(__fdiv_rn(d, sc), 1.0f) : (q > 0.5f ? 1u : 0u);
}

template <class Src>
__global__ void __launch_bounds__(256) flush_kernel(Src src) {
    const int64_t m = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t* out = src.dst(m);
    if (out == nullptr) return;

    if (blockIdx.y >= VSPLIT) {
        // ---------------- K part of head h = blockIdx.y - VSPLIT.  thread = (token group grp of 32 tokens, j):
        // channels j, j + 32, j + 64, j + 96 of the head for tokens 32 grp .. 32 grp + 31; per-channel lo / hi over
        // the 256 tokens through shared memory.
        __shared__ float slo[8][DIM], shi[8][DIM];
        const int h = blockIdx.y - VSPLIT, grp = warp, j = lane;
        float lo[4], hi[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            lo[p] = __int_as_float(0x7f800000);
            hi[p] = -__int_as_float(0x7f800000);
        }
        // the K row of token grp * 32 + i: for a table-driven source, lane i resolves it once and both passes
        // broadcast it
        const uint16_t *kr_l = nullptr, *vr_l = nullptr;
        uint32_t okm = 0u;
        if constexpr (!Src::kDirect) okm = __ballot_sync(0xffffffffu, src.rows(m, grp * 32 + lane, h, kr_l, vr_l));
        auto krow = [&](int i, bool& ok) -> const uint16_t* {
            if constexpr (Src::kDirect) {
                const uint16_t *kr, *vr;
                ok = src.rows(m, grp * 32 + i, h, kr, vr);
                return kr;
            } else {
                ok = (okm >> i) & 1u;
                return reinterpret_cast<const uint16_t*>(
                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(kr_l), i));
            }
        };
        {   // every K row of the warp's 32 tokens requested at once (an L2 prefetch of its two 128-byte lines per
            // lane): the token loops below keep only 4 tokens' loads in flight per warp, and without it the part
            // waits on DRAM latency
            const uint16_t *pk, *pv;
            bool pok;
            if constexpr (Src::kDirect) {
                pok = src.rows(m, grp * 32 + lane, h, pk, pv);
            } else {
                pk = kr_l;
                pok = (okm >> lane) & 1u;
            }
            if (pok) {
                asm volatile("prefetch.global.L2 [%0];" ::"l"(pk));
                asm volatile("prefetch.global.L2 [%0];" ::"l"(pk + 64));
            }
        }
#pragma unroll 4
        for (int i = 0; i < 32; i++) {
            bool ok;
            const uint16_t* kr = krow(i, ok);
            float x[4] = {0.f, 0.f, 0.f, 0.f};
            if (ok) {
#pragma unroll
                for (int p = 0; p < 4; p++) x[p] = bf2f(kr[j + 32 * p]);
            }
#pragma unroll
            for (int p = 0; p < 4; p++) {
                lo[p] = fminf(lo[p], x[p]);
                hi[p] = fmaxf(hi[p], x[p]);
            }
        }
#pragma unroll
        for (int p = 0; p < 4; p++) {
            slo[grp][j + 32 * p] = lo[p];
            shi[grp][j + 32 * p] = hi[p];
        }
        __syncthreads();
        float lof[4], scf[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int c = j + 32 * p;
            float l = slo[0][c], u = shi[0][c];
#pragma unroll
            for (int q = 1; q < 8; q++) {
                l = fminf(l, slo[q][c]);
                u = fmaxf(u, shi[q][c]);
            }
            uint32_t lo8 = f8enc(l);
            uint32_t sc8 = f8enc(clamp_min_1e8(__fdiv_rn(u - l, 3.0f)));
            lof[p] = f8dec(lo8);
            scf[p] = clamp_min_1e8(f8dec(sc8));
            if (grp == 0) {
                out[KLO_O + h * DIM + c] = (uint8_t)lo8;
                out[KSC_O + h * DIM + c] = (uint8_t)sc8;
            }
        }
        float inv[4];
#pragma unroll
        for (int p = 0; p < 4; p++) inv[p] = __frcp_rn(scf[p]);
#pragma unroll 4
        for (int i = 0; i < 32; i++) {
            const int t = grp * 32 + i;
            bool ok;
            const uint16_t* kr = krow(i, ok);
            float x[4] = {0.f, 0.f, 0.f, 0.f};
            if (ok) {
#pragma unroll
                for (int p = 0; p < 4; p++) x[p] = bf2f(kr[j + 32 * p]);
            }
            uint32_t byte = 0;
#pragma unroll
            for (int p = 0; p < 4; p++) byte |= code2(x[p] - lof[p], scf[p], inv[p]) << (2 * p);
            out[KC_O + (t * HEADS + h) * 32 + j] = (uint8_t)byte;
        }
        return;
    }

    // ---------------- V part: warp w handles tokens t0 + w, t0 + w + 8, ... of this CTA's 64-token slice.
    __shared__ float vbuf[8][HEADS * DIM];
    float C[32];
    hadamard_signs(lane, C);
    const int t0 = blockIdx.y * VTOK;
    // the V rows of this warp's 8 tokens x 4 heads: for a table-driven source, lane L resolves token
    // t0 + warp + 8 (L & 7), head L >> 3, once
    const uint16_t *kr_v = nullptr, *vr_v = nullptr;
    uint32_t okv = 0u;
    if constexpr (!Src::kDirect)
        okv = __ballot_sync(0xffffffffu, src.rows(m, t0 + warp + 8 * (lane & 7), lane >> 3, kr_v, vr_v));
    for (int tt = warp; tt < VTOK; tt += 8) {
        const int t = t0 + tt;
        // stage the 4 V rows (512 values) of token t as fp32: lane loads 16 values of head lane / 8
        {
            const int h = lane >> 3, e = (lane & 7) * 16;
            const uint16_t *kr, *vr;
            bool ok;
            if constexpr (Src::kDirect) {
                ok = src.rows(m, t, h, kr, vr);
            } else {
                const int from = (lane & 24) | (tt >> 3);
                vr = reinterpret_cast<const uint16_t*>(
                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(vr_v), from));
                ok = (okv >> from) & 1u;
            }
            float x[16];
            if (ok) load16(vr, e, x);
            else
#pragma unroll
                for (int i = 0; i < 16; i++) x[i] = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) vbuf[warp][h * DIM + e + i] = x[i];
        }
        __syncwarp();
        // per 2-head group: lo / hi over 256 dims, fp8 lo and scale hi - lo, 1-bit codes.  First from the fast
        // transform: every decision is taken at both ends of the error interval [y - E, y + E] (all of them are
        // monotone in y), and where both ends agree it is the decision the exact chain gives.  A token with an
        // undecided scale byte is redone with the exact chain; a token whose only undecided decisions are bits
        // redoes just those outputs with the chain (hadamard_one).
        uint32_t part[HEADS], lo8[2], sc8[2];
        {
            float y[HEADS][4], E[HEADS];
            bool ok = fwht_rows(vbuf[warp], y, E);   // finite inputs and the scale bytes decided
            uint32_t und = 0u;                        // this lane's undecided bits: bit 4 h + k
            float lofg[2], scfg[2];
#pragma unroll
            for (int h = 0; h < HEADS; h++) part[h] = 0;
#pragma unroll
            for (int g = 0; g < 2; g++) {
                const float Eg = fmaxf(E[2 * g], E[2 * g + 1]);
                float l = y[2 * g][0], u = y[2 * g][0];
#pragma unroll
                for (int hh = 0; hh < 2; hh++)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        l = fminf(l, y[2 * g + hh][k]);
                        u = fmaxf(u, y[2 * g + hh][k]);
                    }
#pragma unroll
                for (int o = 16; o; o >>= 1) {
                    l = fminf(l, __shfl_xor_sync(0xffffffffu, l, o));
                    u = fmaxf(u, __shfl_xor_sync(0xffffffffu, u, o));
                }
                const float l_lo = __fsub_rd(l, Eg), l_hi = __fadd_ru(l, Eg);
                const float u_lo = __fsub_rd(u, Eg), u_hi = __fadd_ru(u, Eg);
                lo8[g] = f8enc(l_lo);
                sc8[g] = f8enc(clamp_min_1e8(u_lo - l_hi));
                ok = ok && lo8[g] == f8enc(l_hi) && sc8[g] == f8enc(clamp_min_1e8(u_hi - l_lo));
                const float lof = f8dec(lo8[g]), scf = clamp_min_1e8(f8dec(sc8[g]));
                lofg[g] = lof;
                scfg[g] = scf;
                const float inv = __frcp_rn(scf);
                // bit = [fl(fl(y - lo8) / sc8) > 1/2] for the chain's y, which lies within Eg of the estimate:
                // decided when the estimate's quotient is farther from 1/2 than Eg / sc8 plus the quotient's own error
                const float tol = fmaf(Eg, inv * 1.01f, 4e-6f);
                // one compare per element: |q - 1/2| > 2 tol decides every q the test |q - 1/2| > tol max(1, |q|)
                // decides when tol < 1/4 (for |q| <= 2 its bound is at most 2 tol; for |q| > 2 both decide, as
                // |q - 1/2| > 3/2); for larger tol every element is left to the exact chain
                const float tol2 = tol < 0.25f ? 2.0f * tol : __int_as_float(0x7f800000);
#pragma unroll
                for (int hh = 0; hh < 2; hh++)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const float q = (y[2 * g + hh][k] - lof) * inv;
                        if (!(fabsf(q - 0.5f) > tol2)) und |= 1u << (4 * (2 * g + hh) + k);
                        part[2 * g + hh] |= (q > 0.5f ? 1u : 0u) << ((lane >> 4) + 2 * k);
                    }
            }
            if (!__all_sync(0xffffffffu, ok)) {
                hadamard_rows(vbuf[warp], C, y);
#pragma unroll
                for (int h = 0; h < HEADS; h++) part[h] = 0;
#pragma unroll
                for (int g = 0; g < 2; g++) {
                    float l = y[2 * g][0], u = y[2 * g][0];
#pragma unroll
                    for (int hh = 0; hh < 2; hh++)
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            l = fminf(l, y[2 * g + hh][k]);
                            u = fmaxf(u, y[2 * g + hh][k]);
                        }
#pragma unroll
                    for (int o = 16; o; o >>= 1) {
                        l = fminf(l, __shfl_xor_sync(0xffffffffu, l, o));
                        u = fmaxf(u, __shfl_xor_sync(0xffffffffu, u, o));
                    }
                    lo8[g] = f8enc(l);
                    sc8[g] = f8enc(clamp_min_1e8(u - l));
                    const float lof = f8dec(lo8[g]), scf = clamp_min_1e8(f8dec(sc8[g]));
#pragma unroll
                    for (int hh = 0; hh < 2; hh++)
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            part[2 * g + hh] |= round_clamp(__fdiv_rn(y[2 * g + hh][k] - lof, scf), 1.0f)
                                                << ((lane >> 4) + 2 * k);
                }
            } else if (__any_sync(0xffffffffu, und != 0u)) {
                // scale bytes decided, some bits not: the exact chain for just those outputs, then the bit as the
                // exact path takes it (IEEE divide)
                while (und) {
                    const int e = __ffs(und) - 1;
                    und &= und - 1u;
                    const int h = e >> 2, k = e & 3;
                    const float yc = hadamard_one(vbuf[warp] + h * DIM, C, k);
                    const float lof = (h >> 1) ? lofg[1] : lofg[0], scf = (h >> 1) ? scfg[1] : scfg[0];
                    const uint32_t m = 1u << ((lane >> 4) + 2 * k);
                    const uint32_t bit = round_clamp(__fdiv_rn(yc - lof, scf), 1.0f) ? m : 0u;
#pragma unroll
                    for (int hh = 0; hh < HEADS; hh++)
                        if (hh == h) part[hh] = (part[hh] & ~m) | bit;
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < 2; g++) {
                out[VLO_O + t * 2 + g] = (uint8_t)lo8[g];
                out[VSC_O + t * 2 + g] = (uint8_t)sc8[g];
            }
        }
        // byte j of (t, h) holds dims j + 16 i at bit i; lane (j, half) owns i = half + 2k
#pragma unroll
        for (int h = 0; h < HEADS; h++) {
            uint32_t byte = part[h] | __shfl_xor_sync(0xffffffffu, part[h], 16);
            if (lane < 16) out[VB_O + (t * HEADS + h) * 16 + lane] = (uint8_t)byte;
        }
    }
}


// Dequantizer (kv800.py:79-92): K (M, 256, 4, 128) bf16 = bf16(codes * ksc + klo) (exact in fp32, then rounded);
// V (M, 256, 4, 128) fp32 = (bits * vsc + vlo) @ H with the same FMA chain as the quantizer (bit-identical to the
// reference on CPU).  grid (M, 8): 32 tokens per CTA, warp = 4 tokens.
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* sb_all, uint16_t* kout, float* vout) {
    const int64_t m = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint8_t* sb = sb_all + m * SUB;
    __shared__ float vbuf[8][HEADS * DIM];
    float C[32];
    hadamard_signs(lane, C);
    for (int tt = 0; tt < 4; tt++) {
        const int t = blockIdx.y * 32 + warp * 4 + tt;
        // K: lane covers channel j = lane of each plane for the 4 heads
#pragma unroll
        for (int h = 0; h < HEADS; h++) {
            const uint32_t byte = sb[KC_O + (t * HEADS + h) * 32 + lane];
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const int d = lane + 32 * p;
                const float sc = f8dec(sb[KSC_O + h * DIM + d]), lo = f8dec(sb[KLO_O + h * DIM + d]);
                const float code = (float)((byte >> (2 * p)) & 3u);
                kout[((m * BLK + t) * HEADS + h) * DIM + d] = f2bf(code * sc + lo);
            }
        }
        // V in the Hadamard domain: y_d = bit_d * vsc + vlo, then rotated
#pragma unroll
        for (int h = 0; h < HEADS; h++) {
            const float vlo = f8dec(sb[VLO_O + t * 2 + (h >> 1)]), vsc = f8dec(sb[VSC_O + t * 2 + (h >> 1)]);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int d = lane + 32 * k;
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
            for (int k = 0; k < 4; k++) vout[((m * BLK + t) * HEADS + h) * DIM + lane + 32 * k] = y[h][k];
        __syncwarp();
    }
}

// ---- training-side fake quantization (lfm3_kv800/train.py:82-100): the cache's quantize -> dequantize round trip
// on fp32 activations without packing.
// K: x (G, 256, C) fp32, groups of 256 tokens per channel: lo / hi, fp8 lo and (hi - lo) / 3 scale, code =
// round((x - lo8) / sc8) in [0, 3], out = code * sc8 + lo8.  grid (G, ceil(C / 128)), thread = channel.
__global__ void __launch_bounds__(128) fake_quant_k_kernel(const float* x, int64_t C, float* out) {
    const int64_t g = blockIdx.x, c = (int64_t)blockIdx.y * 128 + threadIdx.x;
    if (c >= C) return;
    const float* col = x + g * BLK * C + c;
    float lo = __int_as_float(0x7f800000), hi = -__int_as_float(0x7f800000);
    for (int t = 0; t < BLK; t++) {
        const float v = col[(int64_t)t * C];
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
    }
    const float lof = f8dec(f8enc(lo));
    const float scq = f8dec(f8enc(clamp_min_1e8(__fdiv_rn(hi - lo, 3.0f))));
    const float scf = clamp_min_1e8(scq);
    float* oc = out + g * BLK * C + c;
    const float inv = __frcp_rn(scf);
    for (int t = 0; t < BLK; t++) {
        const float v = col[(int64_t)t * C];
        const float code = (float)code2(v - lof, scf, inv);
        oc[(int64_t)t * C] = fmaf(code, scq, lof);   // code * sc8 is exact, so this is the reference's mul + add
    }
}

// V: v (N, 4, 128) fp32 per token: y = v @ H per head (sequential FMA chain), per 2-head group lo / hi, fp8 lo and
// scale hi - lo, bit = round((y - lo8) / sc8) in [0, 1], out = (bit * sc8 + lo8) @ H.  Warp per token.
__global__ void __launch_bounds__(256) fake_quant_v_kernel(const float* v, int64_t N, float* out) {
    __shared__ float buf[8][HEADS * DIM];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t t = (int64_t)blockIdx.x * 8 + warp;
    if (t >= N) return;
    float C[32];
    hadamard_signs(lane, C);
    const float* row = v + t * HEADS * DIM;
#pragma unroll
    for (int i = 0; i < 16; i++) buf[warp][lane + 32 * i] = row[lane + 32 * i];
    __syncwarp();
    float y[HEADS][4];
    hadamard_rows(buf[warp], C, y);
    __syncwarp();
#pragma unroll
    for (int g2 = 0; g2 < 2; g2++) {
        float l = y[2 * g2][0], u = y[2 * g2][0];
#pragma unroll
        for (int hh = 0; hh < 2; hh++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                l = fminf(l, y[2 * g2 + hh][k]);
                u = fmaxf(u, y[2 * g2 + hh][k]);
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            l = fminf(l, __shfl_xor_sync(0xffffffffu, l, o));
            u = fmaxf(u, __shfl_xor_sync(0xffffffffu, u, o));
        }
        const float lof = f8dec(f8enc(l)), scq = f8dec(f8enc(clamp_min_1e8(u - l)));
        const float scf = clamp_min_1e8(scq);
        const float inv = __frcp_rn(scf);
#pragma unroll
        for (int hh = 0; hh < 2; hh++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float bit = (float)code1(y[2 * g2 + hh][k] - lof, scf, inv);
                buf[warp][(2 * g2 + hh) * DIM + lane + 32 * k] = fmaf(bit, scq, lof);
            }
    }
    __syncwarp();
    hadamard_rows(buf[warp], C, y);
    float* orow = out + t * HEADS * DIM;
#pragma unroll
    for (int h = 0; h < HEADS; h++)
#pragma unroll
        for (int k = 0; k < 4; k++) orow[h * DIM + lane + 32 * k] = y[h][k];
}

// Exact-page scatter: one warp per (token, head, K|V) row of 128 bf16 (256 B, 8 B per lane).
__global__ void write_exact_kernel(uint16_t* epool, int64_t epool_elems, const int64_t* eoff, int64_t eoff_stride,
                                   int64_t ebs, int64_t e_hs, int64_t e_ts, int64_t e_v, const uint16_t* k,
                                   const uint16_t* v, const int32_t* seq, const int64_t* pos, int64_t T, int64_t nseq,
                                   int* status) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= T * HEADS * 2) return;
    const int64_t i = row / (HEADS * 2);
    const int h = (int)((row / 2) % HEADS), isv = (int)(row & 1);
    const int64_t b = seq[i], p = pos[i];
    int64_t pg = 0, sl = 0;
    if (p >= 0) page_split(p, ebs, pg, sl);
    if (b < 0 || b >= nseq || p < 0 || pg >= eoff_stride) {
        if (lane == 0) flag(status, ST_TABLE);
        return;
    }
    const int64_t o = eoff[b * eoff_stride + pg] + h * e_hs + sl * e_ts + (isv ? e_v : 0);
    if (o < 0 || o + DIM > epool_elems) {
        if (lane == 0) flag(status, ST_EPOOL);
        return;
    }
    const uint16_t* srow = (isv ? v : k) + (i * HEADS + h) * DIM;
    uint16_t* drow = epool + o;
#pragma unroll
    for (int e = 0; e < 4; e++) drow[lane * 4 + e] = srow[lane * 4 + e];
}

}  // namespace kv800

using namespace kv800;

extern "C" int kv800_quantize_blocks(const uint16_t* k, const uint16_t* v, int64_t M, uint8_t* out, void* stream) {
    if (M < 0 || (M > 0 && (!k || !v || !out))) {
        set_error("kv800_quantize_blocks: null pointer or negative M (%lld)", (long long)M);
        return KV800_ERR_ARG;
    }
    if (M == 0) return KV800_OK;
    if (M > 0x7fffffffLL) {
        set_error("kv800_quantize_blocks: M = %lld above 2^31 - 1", (long long)M);
        return KV800_ERR_RANGE;
    }
    ContigSrc s{k, v, out};
    flush_kernel<ContigSrc><<<dim3((unsigned)M, HEADS + VSPLIT), 256, 0, as_stream(stream)>>>(s);
    return cuda_status(cudaGetLastError(), "kv800_quantize_blocks launch");
}

extern "C" int kv800_flush(const uint16_t* epool, int64_t epool_elems, const int64_t* eoff, int64_t eoff_stride,
                           int64_t ebs, int64_t e_hs, int64_t e_ts, int64_t e_v, uint8_t* qpool, int64_t qpool_bytes,
                           const int64_t* boff, int64_t boff_stride, const int32_t* seq, const int32_t* blk,
                           int64_t M, int64_t nseq, int* status, void* stream) {
    if (M < 0 || nseq < 0) {
        set_error("kv800_flush: negative M (%lld) or nseq (%lld)", (long long)M, (long long)nseq);
        return KV800_ERR_ARG;
    }
    if (M == 0) return KV800_OK;
    if (!epool || !eoff || !qpool || !boff || !seq || !blk || ebs <= 0 || eoff_stride <= 0 || boff_stride <= 0) {
        set_error("kv800_flush: null pointer or non-positive ebs / stride");
        return KV800_ERR_ARG;
    }
    if (M > 0x7fffffffLL) {
        set_error("kv800_flush: M = %lld above 2^31 - 1", (long long)M);
        return KV800_ERR_RANGE;
    }
    PagedSrc s{epool, epool_elems, eoff, eoff_stride, ebs, e_hs, e_ts, e_v, qpool, qpool_bytes,
               boff, boff_stride, seq, blk, nseq, status};
    flush_kernel<PagedSrc><<<dim3((unsigned)M, HEADS + VSPLIT), 256, 0, as_stream(stream)>>>(s);
    return cuda_status(cudaGetLastError(), "kv800_flush launch");
}

extern "C" int kv800_write_exact(uint16_t* epool, int64_t epool_elems, const int64_t* eoff, int64_t eoff_stride,
                                 int64_t ebs, int64_t e_hs, int64_t e_ts, int64_t e_v, const uint16_t* k,
                                 const uint16_t* v, const int32_t* seq, const int64_t* pos, int64_t T, int64_t nseq,
                                 int* status, void* stream) {
    if (T < 0) {
        set_error("kv800_write_exact: negative T (%lld)", (long long)T);
        return KV800_ERR_ARG;
    }
    if (T == 0) return KV800_OK;
    if (!epool || !eoff || !k || !v || !seq || !pos || ebs <= 0 || eoff_stride <= 0) {
        set_error("kv800_write_exact: null pointer or non-positive ebs / stride");
        return KV800_ERR_ARG;
    }
    const int64_t rows = T * HEADS * 2, per = 8;   // 8 warps per block
    const int64_t blocks = (rows + per - 1) / per;
    if (blocks > 0x7fffffffLL) {
        set_error("kv800_write_exact: T = %lld too large", (long long)T);
        return KV800_ERR_RANGE;
    }
    write_exact_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(epool, epool_elems, eoff, eoff_stride, ebs,
                                                                       e_hs, e_ts, e_v, k, v, seq, pos, T, nseq,
                                                                       status);
    return cuda_status(cudaGetLastError(), "kv800_write_exact launch");
}

extern "C" int kv800_dequantize_blocks(const uint8_t* sb, int64_t M, uint16_t* k_out, float* v_out, void* stream) {
    if (M < 0 || (M > 0 && (!sb || !k_out || !v_out))) {
        set_error("kv800_dequantize_blocks: null pointer or negative M (%lld)", (long long)M);
        return KV800_ERR_ARG;
    }
    if (M == 0) return KV800_OK;
    if (M > 0x7fffffffLL) {
        set_error("kv800_dequantize_blocks: M = %lld above 2^31 - 1", (long long)M);
        return KV800_ERR_RANGE;
    }
    dequant_kernel<<<dim3((unsigned)M, 8), 256, 0, as_stream(stream)>>>(sb, k_out, v_out);
    return cuda_status(cudaGetLastError(), "kv800_dequantize_blocks launch");
}

extern "C" int kv800_fake_quant_k(const float* x, int64_t G, int64_t C, float* out, void* stream) {
    if (G < 0 || C < 0 || ((G > 0 && C > 0) && (!x || !out))) {
        set_error("kv800_fake_quant_k: null pointer or negative size");
        return KV800_ERR_ARG;
    }
    if (G == 0 || C == 0) return KV800_OK;
    if (G > 0x7fffffffLL || (C + 127) / 128 > 65535) {
        set_error("kv800_fake_quant_k: G %lld / C %lld above the grid limits", (long long)G, (long long)C);
        return KV800_ERR_RANGE;
    }
    fake_quant_k_kernel<<<dim3((unsigned)G, (unsigned)((C + 127) / 128)), 128, 0, as_stream(stream)>>>(x, C, out);
    return cuda_status(cudaGetLastError(), "kv800_fake_quant_k launch");
}

extern "C" int kv800_fake_quant_v(const float* v, int64_t N, float* out, void* stream) {
    if (N < 0 || (N > 0 && (!v || !out))) {
        set_error("kv800_fake_quant_v: null pointer or negative N");
        return KV800_ERR_ARG;
    }
    if (N == 0) return KV800_OK;
    const int64_t blocks = (N + 7) / 8;
    if (blocks > 0x7fffffffLL) {
        set_error("kv800_fake_quant_v: N %lld too large", (long long)N);
        return KV800_ERR_RANGE;
    }
    fake_quant_v_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(v, N, out);
    return cuda_status(cudaGetLastError(), "kv800_fake_quant_v launch");
}

extern "C" int kv800_write_slots(uint16_t* ecache, int64_t ecache_elems, int64_t s0, int64_t s1, int64_t s2,
                                 int64_t ebs, const uint16_t* k, const uint16_t* v, const int64_t* slot_mapping,
                                 int64_t T, int* status, void* stream) {
    if (T < 0) {
        set_error("kv800_write_slots: negative T");
        return KV800_ERR_ARG;
    }
    if (T == 0) return KV800_OK;
    if (!ecache || !k || !v || !slot_mapping || ebs <= 0) {
        set_error("kv800_write_slots: null pointer or ebs <= 0");
        return KV800_ERR_ARG;
    }
    const int64_t blocks = (T * HEADS * 2 + 7) / 8;
    if (blocks > 0x7fffffffLL) {
        set_error("kv800_write_slots: T = %lld too large", (long long)T);
        return KV800_ERR_RANGE;
    }
    write_slots_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(ecache, ecache_elems, s0, s1, s2, ebs, k, v,
                                                                       slot_mapping, T, status);
    return cuda_status(cudaGetLastError(), "kv800_write_slots launch");
}

extern "C" int64_t kv800_flush_step_workspace_size(int64_t max_pairs) {
    if (max_pairs < 0) return -1;
    return 256 + ((max_pairs * 2 * 4 + 255) & ~(int64_t)255);
}

extern "C" int kv800_flush_step(const uint16_t* ecache, int64_t ecache_elems, int64_t s0, int64_t s1, int64_t s2,
                                int64_t ebs, const int32_t* block_table, int64_t bt_stride, uint8_t* qcache,
                                int64_t qcache_bytes, int64_t qs0, int64_t bsq, const int32_t* qblock_table,
                                int64_t qbt_stride, const int32_t* seq_lens, const int32_t* query_start_loc, int64_t R,
                                int64_t max_pairs, void* workspace, int64_t workspace_bytes, int* status,
                                void* stream) {
    if (R < 0 || max_pairs < 0) {
        set_error("kv800_flush_step: negative R / max_pairs");
        return KV800_ERR_ARG;
    }
    if (R == 0 || max_pairs == 0) return KV800_OK;
    if (!ecache || !block_table || !qcache || !qblock_table || !seq_lens || !query_start_loc || !workspace ||
        ebs <= 0 || bsq <= 0 || bsq % BLK || bt_stride <= 0 || qbt_stride <= 0) {
        set_error("kv800_flush_step: null pointer, or bad ebs / bsq (a multiple of 256) / table strides");
        return KV800_ERR_ARG;
    }
    const int64_t need = kv800_flush_step_workspace_size(max_pairs);
    if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
        set_error("kv800_flush_step: workspace of %lld bytes (256-aligned), %lld needed", (long long)workspace_bytes,
                  (long long)need);
        return KV800_ERR_RANGE;
    }
    if (max_pairs > 0x7fffffffLL || R > 0x7fffffffLL) {
        set_error("kv800_flush_step: R / max_pairs above 2^31 - 1");
        return KV800_ERR_RANGE;
    }
    cudaStream_t st = as_stream(stream);
    int32_t* count = static_cast<int32_t*>(workspace);
    int32_t* pairs = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + 256);
    flush_plan_kernel<<<1, 1024, 0, st>>>(seq_lens, query_start_loc, R, max_pairs, pairs, count, status);
    int rc = cuda_status(cudaGetLastError(), "kv800_flush_step plan");
    if (rc) return rc;
    VllmSrc src{ecache, ecache_elems, s0, s1, s2, ebs, block_table, bt_stride, qcache, qcache_bytes, qs0, bsq,
                qblock_table, qbt_stride, pairs, count, R, status};
    flush_kernel<VllmSrc><<<dim3((unsigned)max_pairs, HEADS + VSPLIT), 256, 0, st>>>(src);
    return cuda_status(cudaGetLastError(), "kv800_flush_step flush");
}
