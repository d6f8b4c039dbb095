// Exact-token decode partial on the tensor cores (mma.sync m16n8k16, bf16), sm_100a: the sinks and exact bf16 tokens
// of one (row b, split e), all 4 kv heads (warp = head), in 16-token tiles.
//
//   gather   per tile, 16 tokens x 4 heads x (K row, V row) of 256 B plus the tile's cos / sin rows (64 B) arrive
//            by bulk copies (cp.async.bulk, one per row, issued by the thread that owns the row) into a two-stage
//            shared-memory ring with one mbarrier per stage: every thread arrives once per phase with the bytes of its
//            own copies, so the phase completes when all of them have landed (bounded wait, flagged on time-out).
//            Rows sit at a 272-byte pitch, so the 8 rows an ldmatrix reads start in 8 different bank groups.  Rows
//            that fail the range / alignment checks, or lie past the split's list, are zero-filled by the thread.
//   QK       A = the tile's K rows via ldmatrix.x4 (dims on K); the RoPE dims (d, d + 64), d < 32, are rotated in
//            registers with the reference's roundings (torch_decode.py:16-24): fma.rn.f32.bf16 gives
//            fl32(k0 cs - k2 sn) exactly, cvt.rn.bf16x2 the bf16 rounding.  B = q (bf16, columns 4..7 zero).
//   PV       A = V^T via ldmatrix.x4.trans (dims on M, tokens on K), B = P transposed from the QK accumulator with
//            movmatrix, split into bf16 hi + lo (P - hi) so the products keep ~16 bits of P; fp32 accumulate.
// Online softmax in the log2 domain with a lazily moved reference point (as in qdecode_mma).  The partial (m, l, acc)
// goes to slot xbase + b xstride + e (the reference's slot ns of row b for the single-split form, kv800.py:224-228).
// With arrival counters (count != nullptr, zeroed before the launch; gridDim.y == nx), the CTA that completes a row's
// last exact partial merges all of the row's partials (the quantized ones come from the kernel launched before) into
// out with combine.cuh's warp merge: its stores are fenced before the counter's atomic add, and the merge reads through
// L2 after a fence, so a decode needs no separate merge launch.  Launched early behind the quantized-partial kernel
// (programmatic dependent launch), the CTAs fill the SMs that kernel's CTAs leave; the merge reduces the exact
// partials first and waits for the quantized ones (griddepcontrol.wait) only then.
// ROPE = false is the native sliding layers' form (keys stored post-RoPE, vllm_attn.py:256-257): the reference passes
// all-ones / all-zeros tables there, whose rotation returns every key unchanged, so this form drops the table copies
// and the rotation and gives the same scores.
#pragma once
#include "combine.cuh"
#include "qdecode_mma.cuh"

namespace kv800 {

struct XMArgs {
    const uint16_t* q;
    kv800_paged P;
    const uint16_t* cos_t;
    const uint16_t* sin_t;
    int64_t npos;
    float* mo;
    float* lo;
    float* ao;
    int64_t xbase;     // partial of split e of row b at slot xbase + b * xstride + e
    int64_t xstride;
    int nx;
    float scale;
    int* status;
    int* count;        // per-row arrival counters (nullptr: partials only, merged by a separate launch)
    SlotMap sm;        // with count: where the row's partials live, for the merge
    uint16_t* out;     // with count: (B, 16, 128) bf16 output
};

constexpr int XM_TILE = 16;
constexpr int XM_ROW = 272;                                  // pitch of a 256-byte K or V row in shared memory
constexpr int XM_HEAD_BYTES = XM_TILE * XM_ROW;              // one head's K (or V) rows of a tile
constexpr int XM_KV_BYTES = HEADS * XM_HEAD_BYTES;           // one of K / V for a tile: 17,408 B
constexpr int XM_CS_BYTES = XM_TILE * 64;                    // cos (or sin) rows of a tile
constexpr int XM_STAGE = 2 * XM_KV_BYTES + 2 * XM_CS_BYTES;  // 36,864 B
constexpr int XM_SMEM = 2 * XM_STAGE + 16;                   // two stages and their two mbarriers

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) completing on the mbarrier at bar
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
// this thread's arrival on the phase, announcing `bytes` of its bulk copies (0: a plain arrival)
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_init_count(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void zero_row(uint8_t* p, int bytes) {
    for (int o = 0; o < bytes; o += 16) *reinterpret_cast<uint4*>(p + o) = make_uint4(0u, 0u, 0u, 0u);
}

// RoPE of one register pair on the A fragment: k0 = (K[d], K[d+1]), k2 = (K[d+64], K[d+65]) of one token row,
// c / s = (cos, sin) of frequencies (d, d+1).  Returns kr0 pair in k0, kr2 pair in k2 (bf16, reference roundings).
__device__ __forceinline__ void rope_frag(uint32_t& k0, uint32_t& k2, uint32_t c, uint32_t s) {
    uint32_t r0, r2;
    asm("{\n\t.reg .b16 a0, a1, b0, b1, c0, c1, s0, s1;\n\t.reg .f32 t, x0, x1, y0, y1;\n\t"
        "mov.b32 {a0, a1}, %2;\n\tmov.b32 {b0, b1}, %3;\n\tmov.b32 {c0, c1}, %4;\n\tmov.b32 {s0, s1}, %5;\n\t"
        "fma.rn.f32.bf16 t, b0, s0, 0f00000000;\n\tneg.f32 t, t;\n\tfma.rn.f32.bf16 x0, a0, c0, t;\n\t"
        "fma.rn.f32.bf16 t, b1, s1, 0f00000000;\n\tneg.f32 t, t;\n\tfma.rn.f32.bf16 x1, a1, c1, t;\n\t"
        "fma.rn.f32.bf16 t, a0, s0, 0f00000000;\n\tfma.rn.f32.bf16 y0, b0, c0, t;\n\t"
        "fma.rn.f32.bf16 t, a1, s1, 0f00000000;\n\tfma.rn.f32.bf16 y1, b1, c1, t;\n\t"
        "cvt.rn.bf16x2.f32 %0, x1, x0;\n\tcvt.rn.bf16x2.f32 %1, y1, y0;\n\t}"
        : "=r"(r0), "=r"(r2)
        : "r"(k0), "r"(k2), "r"(c), "r"(s));
    k0 = r0;
    k2 = r2;
}

// smem byte offset of (row r, 16-byte chunk c) in a [16 rows][272 B] tile
__device__ __forceinline__ int xm_off(int r, int c) { return r * XM_ROW + (c << 4); }

// Shared-memory addressing of one head's 16 K and 16 V rows of a tile: the bulk-copy gather's rows at the 272-byte
// pitch, K and V in separate blocks.
struct PitchRows {
    uint32_t kb, vb;
    __device__ __forceinline__ uint32_t k(int r, int c) const { return kb + xm_off(r, c); }
    __device__ __forceinline__ uint32_t v(int r, int c) const { return vb + xm_off(r, c); }
};

// Online-softmax state of one warp (one kv head, its 4 query rows in MMA columns 0..3).
struct XMState {
    float m[2], l[2];
    float acc[8][4];
    __device__ __forceinline__ void init() {
        m[0] = m[1] = -1e30f;
        l[0] = l[1] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int k = 0; k < 4; k++) acc[i][k] = 0.f;
    }
};

// One 16-token tile of one head (warp): QK on the tensor cores with the in-register RoPE of dims (d, d + 64), d < 32,
// the masked online softmax (slot s takes part iff bit s of vmask is set) and PV with P split into bf16 hi + lo.
// cs / sn: the tile's cos / sin rows (16 x 64 B); rows: where the tile's K / V rows sit in shared memory.
template <bool ROPE, class Rows>
__device__ __forceinline__ void xm_tile(const Rows& rw, const uint32_t* cs, const uint32_t* sn, const uint32_t (&bq)[8][2],
                                        uint32_t vmask, float scale, XMState& S, int lane) {
    const int g = lane >> 2, tig = lane & 3, mi = lane >> 3, ri = lane & 7;
    // ---- QK: A fragments of the 8 K-steps (matrices: rows 0-7 / 8-15 x dims +0 / +8)
    uint32_t A[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
        const int r = (mi & 1) * 8 + ri, c = 2 * ks + (mi >> 1);
        ldsm_x4(rw.k(r, c), A[ks][0], A[ks][1], A[ks][2], A[ks][3]);
    }
    // RoPE on K-steps 0,1 (dims 0..31) with 4,5 (dims 64..95): regs 0 / 2 are token g, 1 / 3 token g + 8;
    // regs 0 / 1 cover dims 16 ks + 2 tig, regs 2 / 3 dims 16 ks + 8 + 2 tig
    if (ROPE) {
#pragma unroll
        for (int ks = 0; ks < 2; ks++)
#pragma unroll
            for (int rg = 0; rg < 4; rg++) {
                const int tok = g + 8 * (rg & 1);
                const int d = 16 * ks + 8 * (rg >> 1) + 2 * tig;   // even, < 32
                rope_frag(A[ks][rg], A[ks + 4][rg], cs[tok * 16 + (d >> 1)], sn[tok * 16 + (d >> 1)]);
            }
    }
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ks++) mma_bf16(sc, A[ks][0], A[ks][1], A[ks][2], A[ks][3], bq[ks][0], bq[ks][1]);
    // masked slots (past the list, outside the row's range, or without valid rows) get -inf by selection, so
    // whatever their rows hold never reaches the sums
    const bool va = (vmask >> g) & 1u, vb = (vmask >> (g + 8)) & 1u;
    float s2[4];
    s2[0] = va ? sc[0] * scale : -__int_as_float(0x7f800000);
    s2[1] = va ? sc[1] * scale : -__int_as_float(0x7f800000);
    s2[2] = vb ? sc[2] * scale : -__int_as_float(0x7f800000);
    s2[3] = vb ? sc[3] * scale : -__int_as_float(0x7f800000);
    // the row maxima are reduced across the 8 lanes of a row only when some score of the warp passes its row's
    // reference point by more than 2^6
    float lmx[2];
    bool need = false;
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        lmx[rr] = fmaxf(s2[rr], s2[rr + 2]);
        need |= lmx[rr] > S.m[rr] + 6.0f;
    }
    if (__any_sync(0xffffffffu, need)) {
        float alpha[2] = {1.f, 1.f};
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            float mx = lmx[rr];
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            if (mx > S.m[rr] + 6.0f) {
                alpha[rr] = fast_exp2(S.m[rr] - mx);
                S.m[rr] = mx;
            }
        }
        S.l[0] *= alpha[0];
        S.l[1] *= alpha[1];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            S.acc[i][0] *= alpha[0];
            S.acc[i][1] *= alpha[1];
            S.acc[i][2] *= alpha[0];
            S.acc[i][3] *= alpha[1];
        }
    }
    float p[4];
#pragma unroll
    for (int k = 0; k < 4; k++) p[k] = fast_exp2(s2[k] - S.m[k & 1]);
    S.l[0] += p[0] + p[2];
    S.l[1] += p[1] + p[3];
    // ---- PV: B = P^T (hi + lo bf16), A = V^T via ldmatrix.trans
    const uint32_t ha = pack_bf16(p[0], p[1]), hb = pack_bf16(p[2], p[3]);
    const uint32_t la = pack_bf16(p[0] - __uint_as_float(ha << 16), p[1] - __uint_as_float(ha & 0xffff0000u));
    const uint32_t lb = pack_bf16(p[2] - __uint_as_float(hb << 16), p[3] - __uint_as_float(hb & 0xffff0000u));
    const uint32_t bh0 = transpose8x8(ha), bh1 = transpose8x8(hb);
    const uint32_t bl0 = transpose8x8(la), bl1 = transpose8x8(lb);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        // matrices: (tokens 0-7, dims +0), (tokens 0-7, dims +8), (tokens 8-15, dims +0), (tokens 8-15, dims +8)
        const int r = (mi >> 1) * 8 + ri, c = 2 * i + (mi & 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(rw.v(r, c), v0, v1, v2, v3);
        mma_bf16(S.acc[i], v0, v1, v2, v3, bh0, bh1);
        mma_bf16(S.acc[i], v0, v1, v2, v3, bl0, bl1);
    }
}

// q B fragments of warp h (standard dims layout): b0 = q[g][16 ks + 2 tig ..], b1 = q[g][16 ks + 8 + 2 tig ..]
__device__ __forceinline__ void xm_load_q(const uint16_t* q, int b, int h, int lane, uint32_t (&bq)[8][2]) {
    const int g = lane >> 2, tig = lane & 3;
    const uint16_t* qr = q + ((int64_t)b * QROWS + h * 4 + (g & 3)) * DIM;
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
        const uint32_t v0 = *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 2 * tig);
        const uint32_t v1 = *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 8 + 2 * tig);
        bq[ks][0] = (g < 4) ? v0 : 0u;
        bq[ks][1] = (g < 4) ? v1 : 0u;
    }
}

// The partial of split e of row b (slot xbase + b xstride + e) for warp h's query rows: rows r = 2 tig, 2 tig + 1
// (valid for tig < 2); acc[i] rows d = 16 i + g, 16 i + g + 8.
__device__ __forceinline__ void xm_store_partial(const XMArgs& a, const XMState& S, int b, int e, int h, int lane) {
    const int g = lane >> 2, tig = lane & 3;
    float l[2];
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        float x = S.l[rr];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        l[rr] = x;
    }
    if (tig < 2) {
        const int64_t slot = a.xbase + (int64_t)b * a.xstride + e;
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const int64_t row = slot * QROWS + h * 4 + 2 * tig + rr;
            if (g == 0) {
                a.mo[row] = S.m[rr];
                a.lo[row] = l[rr];
            }
            float* o = a.ao + row * DIM;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                o[16 * i + g] = S.acc[i][rr];
                o[16 * i + g + 8] = S.acc[i][rr + 2];
            }
        }
    }
}

// Partial and merge of a 4-warp CTA (warp h = head h): with arrival counters (one per row, target nx) the last CTA of
// row b to arrive merges the row (warp h: query rows 4 h .. 4 h + 3).  Every thread of the CTA calls it.
__device__ __forceinline__ void xm_finish(const XMArgs& a, const XMState& S, int b, int e, int h, int lane) {
    xm_store_partial(a, S, b, e, h, lane);
    if (a.count) {
        __shared__ int last;
        __threadfence();
        __syncthreads();
        if (h == 0 && lane == 0) last = atomicAdd(a.count + b, 1) == a.nx - 1;
        __syncthreads();
        if (last) {   // (launched early behind the quantized-partial kernel: the merge waits for it after the exact
                      // group)
            __threadfence();
            combine_head(a.mo, a.lo, a.ao, a.sm, a.out, b, h, lane, true);
        }
    }
}

// Partial and merge of a one-warp CTA (row b, split e, head h): with arrival counters (one per (row, head), at
// b * 4 + h, target nx) the last warp of (b, h) to arrive merges head h's query rows of row b.
__device__ __forceinline__ void xm_finish_head(const XMArgs& a, const XMState& S, int b, int e, int h, int lane) {
    xm_store_partial(a, S, b, e, h, lane);
    if (a.count) {
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(a.count + (int64_t)b * HEADS + h, 1) == a.nx - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            combine_head(a.mo, a.lo, a.ao, a.sm, a.out, b, h, lane, true);
        }
    }
}

template <bool ROPE>
__global__ void __launch_bounds__(128, 3) xdecode_mma(XMArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];   // the same declaration as qdecode_mma's (one symbol per unit)
    const int b = blockIdx.x, e = blockIdx.y, tid = threadIdx.x;
    const int h = tid >> 5, lane = tid & 31;
    const kv800_paged& P = a.P;

    // ---- this split's token list: [s0, cnt) sinks, then exact positions lo_e + [x0, x1)
    const int64_t n = P.N[b], nqb = P.NQ[b];
    int64_t lo_e = nqb * BLK;
    if (P.win && n - P.win > lo_e) lo_e = n - P.win;
    int64_t cnt = 0;
    if (P.win && P.sk) {
        cnt = P.nsink;
        if (lo_e < cnt) cnt = lo_e;
        if (n < cnt) cnt = n;
        if (cnt < 0) cnt = 0;
    }
    const int64_t E = n > lo_e ? n - lo_e : 0;
    const int64_t ch = (E + a.nx - 1) / a.nx;
    const int64_t x0 = min((int64_t)e * ch, E), x1 = min(x0 + ch, E);
    const int64_t s0 = (e == 0) ? 0 : cnt;
    const int64_t nsk = cnt - s0;
    const int64_t total = nsk + (x1 - x0);
    const int ntiles = (int)((total + XM_TILE - 1) / XM_TILE);

    const uint32_t bar0 = smem_u32(smem + 2 * XM_STAGE);   // mbarrier of stage s at bar0 + 8 s
    // ---- issue the copies of tile `it` into stage `st` and arrive on its mbarrier; invalid rows are zero-filled
    // thread = (token tt = tid / 8, row role sub = tid % 8: head sub / 2, K (sub even) or V (odd)); threads < 32 also
    // copy one table row (token tid / 2, cos (tid even) or sin)
    auto issue = [&](int it, int st) {
        uint8_t* base = smem + st * XM_STAGE;
        const uint32_t bar = bar0 + 8 * st;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // earlier generic reads of the stage first
        const int tt = tid >> 3, sub = tid & 7, hh = sub >> 1, isv = sub & 1;
        const int64_t ti = (int64_t)it * XM_TILE + tt;
        const uint16_t* row = P.epool;
        bool ok = false;
        int64_t pos = 0;
        if (ti < total) {
            if (ti < nsk) {
                const int64_t t = s0 + ti;
                pos = t;
                const int64_t o = (isv ? P.svoff[b] : P.skoff[b]) + (t * HEADS + hh) * DIM;
                const int64_t lim = isv ? P.sv_elems : P.sk_elems;
                const uint16_t* pool = isv ? P.sv : P.sk;
                if (o >= 0 && o + DIM <= lim) {
                    row = pool + o;
                    ok = true;
                } else if (sub == 0) {
                    flag(a.status, ST_SINK);
                }
            } else {
                pos = lo_e + x0 + (ti - nsk);
                // positions are below 2^31 (N is int32) and 0 < ebs < 2^31 (checked by the host)
                const uint32_t eb = (uint32_t)P.ebs, pg = (uint32_t)pos / eb, sl = (uint32_t)pos - pg * eb;
                if (pg < P.eoff_stride) {
                    const int64_t o = P.eoff[(int64_t)b * P.eoff_stride + pg] + hh * P.e_hs + (int64_t)sl * P.e_ts +
                                      (isv ? P.e_v : 0);
                    if (o >= 0 && o + DIM <= P.epool_elems) {
                        row = P.epool + o;
                        ok = true;
                    } else if (sub == 0) {
                        flag(a.status, ST_EPOOL);
                    }
                } else if (sub == 0) {
                    flag(a.status, ST_TABLE);
                }
            }
            if (ROPE && ok && pos >= a.npos) {
                if (sub == 0) flag(a.status, ST_TABLE);
                ok = false;
            }
            if (ok && (reinterpret_cast<uintptr_t>(row) & 15u)) {
                if (sub == 0) flag(a.status, ST_EPOOL);
                ok = false;
            }
        }
        uint8_t* dst = base + isv * XM_KV_BYTES + hh * XM_HEAD_BYTES + tt * XM_ROW;
        uint32_t bytes = ok ? 2 * DIM : 0;
        // cos / sin rows of the tile's tokens: threads < 32, token tid / 2, cos (even) or sin (odd)
        const uint16_t* trow = nullptr;
        uint8_t* tdst = nullptr;
        if (ROPE && tid < 2 * XM_TILE) {
            const int tc = tid >> 1, which = tid & 1;
            const int64_t tj = (int64_t)it * XM_TILE + tc;
            int64_t pj = -1;
            if (tj < total) pj = (tj < nsk) ? (s0 + tj) : (lo_e + x0 + (tj - nsk));
            tdst = base + 2 * XM_KV_BYTES + which * XM_CS_BYTES + tc * 64;
            if (pj >= 0 && pj < a.npos) {
                trow = (which ? a.sin_t : a.cos_t) + pj * 32;
                bytes += 64;
            }
        }
        mbar_arrive_tx(bar, bytes);   // before the copies, so the phase cannot complete without them
        if (ok) bulk_g2s(smem_u32(dst), row, 2 * DIM, bar);
        else zero_row(dst, 2 * DIM);
        if (trow) bulk_g2s(smem_u32(tdst), trow, 64, bar);
        else if (tdst) zero_row(tdst, 64);
    };

    uint32_t bq[8][2];
    xm_load_q(a.q, b, h, lane, bq);
    if (tid == 0) {
        mbar_init_count(bar0, 128);
        mbar_init_count(bar0 + 8, 128);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (ntiles > 0) issue(0, 0);
    if (ntiles > 1) issue(1, 1);
    uint32_t phase = 0;      // bit s: parity of the next phase of stage s's mbarrier
    int timeouts = 0;

    XMState S;
    S.init();
    for (int it = 0; it < ntiles; it++) {
        const int st = it & 1;
        if (!mbar_wait(bar0 + 8 * st, (phase >> st) & 1u)) timeouts++;
        phase ^= 1u << st;
        __syncthreads();   // the zero-filled rows of other threads
        const uint8_t* base = smem + st * XM_STAGE;
        const PitchRows rw{smem_u32(base + h * XM_HEAD_BYTES), smem_u32(base + XM_KV_BYTES + h * XM_HEAD_BYTES)};
        const uint32_t* cs = reinterpret_cast<const uint32_t*>(base + 2 * XM_KV_BYTES);
        const uint32_t* sn = reinterpret_cast<const uint32_t*>(base + 2 * XM_KV_BYTES + XM_CS_BYTES);
        // slots past the list end are masked (zero-filled rows still give finite scores, but the list end is the
        // only place rows are missing when the tables are consistent)
        const int64_t left = total - (int64_t)it * XM_TILE;
        const uint32_t vmask = left >= XM_TILE ? 0xffffu : ((1u << left) - 1u);
        xm_tile<ROPE>(rw, cs, sn, bq, vmask, a.scale, S, lane);
        __syncthreads();
        if (it + 2 < ntiles) issue(it + 2, st);
    }
    if (timeouts && tid == 0) flag(a.status, ST_TIMEOUT);
    xm_finish(a, S, b, e, h, lane);
}

}  // namespace kv800
