// Quantized-split decode kernel on the tensor cores (mma.sync m16n8k16), sm_100a.
//
// Per (row b, split s) CTA of 4 warps, warp = kv head h, over sub-blocks [s spb, min((s + 1) spb, NQ[b], nqmax)):
//   QK   S[t, r] = sum_d Kr[t, d] q[r, d]: M = 16 tokens, N = 8 query columns (the head's 4 rows + 4 zero rows),
//        K = 16 dims per step, bf16 operands, fp32 accumulate.  The A fragments are the reference's keys exactly:
//        k = bf16(c sc + lo) (kv800.py:86) via one bf16x2 FMA per register pair (c sc + lo is exact before the single
//        rounding), and for the RoPE dims kr = bf16(fl32(k0 cs - k2 sn)) (torch_decode.py:16-24) in fp32.
//   PV   acc[d, r] += sum_t V^[t, d] P[t, r]: M = 16 dims (one bit plane of 16 V bytes), N = 8 columns, K = 16 tokens,
//        fp16 operands.  A = bit * 2^(i - 24) for bit plane i: the V byte sits in bits 0..7 of an fp16 lane, and
//        masking one bit leaves the fp16 subnormal of exactly that value (one AND per register, no offset).
//        B = fp16(p * vs), transposed from the QK accumulator layout with movmatrix.  sum_t B[t, r] bit[t, d] =
//        acc_i 2^(24 - i), carrying only the accumulation's own rounding.  (An offset encoding such as 0.5 + bit 2^k
//        with a constant tile subtracted at the end cancels a part of size 0.5 sum B against a result of size
//        ~ sum B / sqrt(tokens), and amplifies the accumulated fp32 rounding by up to 2^8 per plane: ~10 % rel-L2 at
//        32K tokens of random data.)
//   The exact V of a quantized token is bits * vs + vl in the Hadamard domain (kv800.py:87-91); vl enters through
//   lv = sum_t p vl, and combine() applies H once (kv800.py:231-236).
// Online softmax in the log2 domain per 32-token chunk; partial (m, l, acc + lv) written to the reference's slot
// layout.  Sub-block halves stream into a two-stage shared-memory ring by TMA (cp.async.bulk.tensor over the quant pool
// seen as 128-byte rows, the 128-byte swizzle putting chunk c of row t at c ^ (t & 7) so the fragment loads are
// bank-conflict free), one thread issuing and an mbarrier per stage signalling completion; per sub-block the CTA first
// decodes the fp8 scales once (hardware e4m3x2 -> f16x2 conversion) into bf16x2 dequant constants and (vl, vs) pairs
// in shared memory.
#pragma once
#include <cuda.h>

#include "kv800_common.cuh"

namespace kv800 {

struct QMArgs {
    const uint16_t* q;
    const uint8_t* qpool;
    int64_t qpool_bytes;
    const int64_t* boff;
    int64_t boff_stride;
    const int32_t* NQ;
    int64_t nqmax;
    const uint16_t* cos_t;
    const uint16_t* sin_t;
    int64_t npos;
    float* mo;
    float* lo;
    float* ao;
    int nslots;   // grid mode: slots per row (partial of split s of row b at slot b * nslots + s)
    int spb;      // grid mode: sub-blocks per split
    float scale;
    int* status;
    // persistent mode (prefix != nullptr): the rows' sub-block lists are flattened (prefix[b] = sum of
    // min(NQ, nqmax) over rows < b, prefix[B] = W) and cut into 2 W half sub-blocks; CTA c of G = min(gridDim.x, 2 W)
    // takes the halves [c 2W / G, (c + 1) 2W / G) and writes the partial of its segment of row b at slot c + b.
    const int64_t* prefix;
    int64_t B;
    // bf16x2 (4, 4), the base of the key code encoding.  Passed as a value: as a compile-time constant it becomes an
    // immediate that the packed-half instructions cannot encode next to the LOP3's mask, and the compiler
    // re-materializes it with an extra ALU instruction per use (~30 % of the kernel's ALU work).
    uint32_t kbase;
    // the quant pool as 128-byte rows, for the TMA loads of a sub-block half: tm_rows boxes of 64 rows with the
    // 128-byte swizzle (kc rows, vb lines), tm_sc boxes of 16 rows unswizzled (the scale region)
    CUtensorMap tm_rows, tm_sc;
};

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) { return (a & mask) | orv; }

__device__ __forceinline__ uint32_t hfma2_bf16(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hsub2_bf16(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// fp32 pair -> bf16x2 (RNE), lo in the low half.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
__device__ __forceinline__ uint32_t transpose8x8(uint32_t x) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(x));
    return d;
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// 2^x with the hardware approximation (relative error ~2^-22); arguments here are <= 6 (log2 domain, lazily moved
// max), and results below 2^-126 flush to 0, which drops nothing a softmax weight needs.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}


// Dims of register i (0..15) of a token's 16 A registers for thread tig (see the layout comment above the kernel).
__device__ __forceinline__ void reg_dims(int tig, int i, int& d0, int& d1) {
    if (i < 8) {
        const int j = 8 * tig + i;
        d0 = j;
        d1 = j + 64;
    } else {
        const int p = (i < 12) ? 1 : 3;
        const int pi = (i - 8) & 3;
        const int j = 8 * tig + ((pi & 1) | ((pi & 2) << 1));   // 0, 1, 4, 5
        d0 = 32 * p + j;
        d1 = 32 * p + j + 2;
    }
}

// Register layout of one token's QK A operand for thread tig (bytes J = 8 tig .. 8 tig + 7 of the kc row), in two
// halves so that only one is live at a time:
//   rotated  R[u], u < 8   (kr0_j, kr2_j), j = 8 tig + u              (RoPE dims j and j + 64)      K-steps 0..3
//   NoPE     R[pi]         (k1_j, k1_{j+2}), j = 8 tig + {0,1,4,5}[pi] (dims 32 + j, 32 + j + 2)     K-steps 4..7
//            R[4 + pi]     (k3_j, k3_{j+2})                            (dims 96 + j, 96 + j + 2)
// K-step ks of a half uses R[2 ks] for columns (2 tig, 2 tig + 1) and R[2 ks + 1] for columns (2 tig + 8, 2 tig + 9).
//
// Per-plane code encodings (bf16, code c at mantissa bits of the plane): x = 4 + c * 2^(2p - 5) for planes 0..2 and
// plane 3 shifted down by 4 bits (encoded like plane 1), so (x - 4) * (sc * 2^(5 - 2p)) = c * sc exactly and
// fma(x - 4, A, lo) = bf16(c sc + lo) with one rounding.  The per-sub-block constants (A, L) of a plane for the
// thread's 4 pairs are two 16-byte words in shared memory: (A0, L0, A1, L1), (A2, L2, A3, L3).

// RoPE of two key pairs with the reference's roundings, on packed bf16 operands (mixed-precision fma.rn.f32.bf16:
// bf16 x bf16 products are exact in fp32, so t = fma(k2, sn, 0) is k2 sn and fma(k0, cs, -t) is the reference's
// fl32(fl32(k0 cs) - fl32(k2 sn)); cvt.rn.bf16x2 is its second rounding).  k0 / k2 hold (byte j, byte j + 2) in
// (low, high); the cos / sin of j are in the half `odd` of word ca / sa, of j + 2 in word cb / sb.
// Ra = (kr0_j, kr2_j), Rb = (kr0_{j+2}, kr2_{j+2}).
__device__ __forceinline__ void rope_pairs(uint32_t k0, uint32_t k2, uint32_t ca, uint32_t cb, uint32_t sa, uint32_t sb,
                                           bool odd, uint32_t& Ra, uint32_t& Rb) {
    if (odd) {
        asm("{\n\t.reg .b16 k0a, k0b, k2a, k2b, x, csa, csb, sna, snb;\n\t.reg .f32 t, r0, r2;\n\t"
            "mov.b32 {k0a, k0b}, %2;\n\tmov.b32 {k2a, k2b}, %3;\n\t"
            "mov.b32 {x, csa}, %4;\n\tmov.b32 {x, csb}, %5;\n\tmov.b32 {x, sna}, %6;\n\tmov.b32 {x, snb}, %7;\n\t"
            "fma.rn.f32.bf16 t, k2a, sna, 0f00000000;\n\tneg.f32 t, t;\n\tfma.rn.f32.bf16 r0, k0a, csa, t;\n\t"
            "fma.rn.f32.bf16 t, k0a, sna, 0f00000000;\n\tfma.rn.f32.bf16 r2, k2a, csa, t;\n\t"
            "cvt.rn.bf16x2.f32 %0, r2, r0;\n\t"
            "fma.rn.f32.bf16 t, k2b, snb, 0f00000000;\n\tneg.f32 t, t;\n\tfma.rn.f32.bf16 r0, k0b, csb, t;\n\t"
            "fma.rn.f32.bf16 t, k0b, snb, 0f00000000;\n\tfma.rn.f32.bf16 r2, k2b, csb, t;\n\t"
            "cvt.rn.bf16x2.f32 %1, r2, r0;\n\t}"
            : "=r"(Ra), "=r"(Rb)
            : "r"(k0), "r"(k2), "r"(ca), "r"(cb), "r"(sa), "r"(sb));
    } else {
        asm("{\n\t.reg .b16 k0a, k0b, k2a, k2b, x, csa, csb, sna, snb;\n\t.reg .f32 t, r0, r2;\n\t"
            "mov.b32 {k0a, k0b}, %2;\n\tmov.b32 {k2a, k2b}, %3;\n\t"
            "mov.b32 {csa, x}, %4;\n\tmov.b32 {csb, x}, %5;\n\tmov.b32 {sna, x}, %6;\n\tmov.b32 {snb, x}, %7;\n\t"
            "fma.rn.f32.bf16 t, k2a, sna, 0f00000000;\n\tneg.f32 t, t;\n\tfma.rn.f32.bf16 r0, k0a, csa, t;\n\t"
            "fma.rn.f32.bf16 t, k0a, sna, 0f00000000;\n\tfma.rn.f32.bf16 r2, k2a, csa, t;\n\t"
            "cvt.rn.bf16x2.f32 %0, r2, r0;\n\t"
            "fma.rn.f32.bf16 t, k2b, snb, 0f00000000;\n\tneg.f32 t, t;\n\tfma.rn.f32.bf16 r0, k0b, csb, t;\n\t"
            "fma.rn.f32.bf16 t, k0b, snb, 0f00000000;\n\tfma.rn.f32.bf16 r2, k2b, csb, t;\n\t"
            "cvt.rn.bf16x2.f32 %1, r2, r0;\n\t}"
            : "=r"(Ra), "=r"(Rb)
            : "r"(k0), "r"(k2), "r"(ca), "r"(cb), "r"(sa), "r"(sb));
    }
}

// The rotated half of one token's A registers: planes 0 and 2 dequantized (KC = their constant words) and rotated.
// BASE = bf16x2 (4, 4) from the kernel arguments; w0 / w1 = the thread's 8 code bytes (pair words: byte pair (j,
// j + 2) at bits 0-7 / 16-23).
__device__ __forceinline__ void token_rope(uint32_t w0, uint32_t w1, const uint4& cw, const uint4& sw,
                                           const uint4 (&KC)[4], uint32_t (&R)[8], uint32_t BASE) {
    const uint32_t pw[4] = {w0, w0 >> 8, w1, w1 >> 8};
    const uint32_t cwv[4] = {cw.x, cw.y, cw.z, cw.w};   // cos of j = 8tig + {0,1}, {2,3}, {4,5}, {6,7}
    const uint32_t swv[4] = {sw.x, sw.y, sw.z, sw.w};
    // KC[0..1]: plane 0 (A, L) x 4 pairs, KC[2..3]: plane 2
    const uint32_t A0[4] = {KC[0].x, KC[0].z, KC[1].x, KC[1].z}, L0[4] = {KC[0].y, KC[0].w, KC[1].y, KC[1].w};
    const uint32_t A2[4] = {KC[2].x, KC[2].z, KC[3].x, KC[3].z}, L2[4] = {KC[2].y, KC[2].w, KC[3].y, KC[3].w};
#pragma unroll
    for (int pi = 0; pi < 4; pi++) {
        const uint32_t P = pw[pi];
        const uint32_t k0 = hfma2_bf16(hsub2_bf16(lop3_and_or(P, 0x00030003u, BASE), BASE), A0[pi], L0[pi]);
        const uint32_t k2 = hfma2_bf16(hsub2_bf16(lop3_and_or(P, 0x00300030u, BASE), BASE), A2[pi], L2[pi]);
        // the pair is (j, j + 2) with j = 8 tig + {0, 1, 4, 5}[pi]: cos / sin words {0,1} (pi < 2) or {2,3},
        // low halves for even j, high halves for odd j
        const int wi = (pi >> 1) * 2;
        const bool odd = (pi & 1) != 0;
        const int ua = (pi & 1) | ((pi & 2) << 1);   // u of byte j = 8 tig + u
        rope_pairs(k0, k2, cwv[wi], cwv[wi + 1], swv[wi], swv[wi + 1], odd, R[ua], R[ua + 2]);
    }
}

// The NoPE half: planes 1 and 3 (KC = their constant words) dequantized straight into A registers.
__device__ __forceinline__ void token_nope(uint32_t w0, uint32_t w1, const uint4 (&KC)[4], uint32_t (&R)[8],
                                           uint32_t BASE) {
    const uint32_t pw[4] = {w0, w0 >> 8, w1, w1 >> 8};
    const uint32_t A1[4] = {KC[0].x, KC[0].z, KC[1].x, KC[1].z}, L1[4] = {KC[0].y, KC[0].w, KC[1].y, KC[1].w};
    const uint32_t A3[4] = {KC[2].x, KC[2].z, KC[3].x, KC[3].z}, L3[4] = {KC[2].y, KC[2].w, KC[3].y, KC[3].w};
#pragma unroll
    for (int pi = 0; pi < 4; pi++) {
        const uint32_t P = pw[pi];
        R[pi] = hfma2_bf16(hsub2_bf16(lop3_and_or(P, 0x000c000cu, BASE), BASE), A1[pi], L1[pi]);
        R[4 + pi] = hfma2_bf16(hsub2_bf16(lop3_and_or(P >> 4, 0x000c000cu, BASE), BASE), A3[pi], L3[pi]);
    }
}

// ---- shared-memory staging of one sub-block half (TMA, 128-byte swizzle)
// kc region: token row t (128 B = 8 chunks): chunk c stored at c ^ (t & 7).  vb region: 128-B line L (2 tokens):
// chunk c stored at c ^ (L & 7).  A warp's fragment loads (8 tokens x one 8- or 2-byte piece of the same head) then
// hit 8 different bank groups.  Scale region linear.  Stages start 1024-byte aligned, as the swizzle requires.
// Stage unit = half a sub-block: the kc rows and vb lines of 128 tokens (+ the 2 KB scale region with the first half).
constexpr int QM_HALF = BLK / 2;
constexpr int QM_KC_BYTES = QM_HALF * 128;           // 16 KB of kc rows
constexpr int QM_VB_BYTES = QM_HALF * 64;            // 8 KB of vb lines
constexpr int QM_SC_BYTES = SUB - VLO_O;             // vlo | vsc | klo | ksc, 2 KB
constexpr int ST_VB = QM_KC_BYTES, ST_SC = QM_KC_BYTES + QM_VB_BYTES;
constexpr int QM_STAGE = QM_KC_BYTES + QM_VB_BYTES + QM_SC_BYTES;   // 26,624 B
constexpr int QM_CST_BYTES = HEADS * 4 * 4 * 4 * 8;  // [h][plane][tig][pair] x (A, L) bf16x2
constexpr int QM_VSL_BYTES = BLK * 2 * 8;            // [t][group] x (vl, vs) fp32
constexpr int QM_SMEM = 2 * QM_STAGE + QM_CST_BYTES + QM_VSL_BYTES;   // 59,392 B: three CTAs per SM

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

constexpr int QM_SMEM_TMA = 1024 + QM_SMEM + 16;   // 1 KB to align the stages for the swizzle, 2 mbarriers

__device__ __forceinline__ void mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* tm, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(0), "r"(y), "r"(bar) : "memory");
}
// issue the TMA loads of half `half` of the sub-block at byte offset off (a multiple of 128) into the stage at dst
// (1024-aligned): kc rows (2 boxes of 64 rows), vb lines (1 box), and with `sc` the scale region; one thread.
__device__ __forceinline__ void tma_half(const QMArgs& a, uint32_t dst, uint32_t bar, int64_t off, int half, bool sc) {
    const int row = (int)(off >> 7);
    const uint32_t bytes = QM_KC_BYTES + QM_VB_BYTES + (sc ? QM_SC_BYTES : 0);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    tma2d(dst, &a.tm_rows, row + half * 128, bar);
    tma2d(dst + 8192, &a.tm_rows, row + half * 128 + 64, bar);
    tma2d(dst + ST_VB, &a.tm_rows, row + (VB_O >> 7) + half * 64, bar);
    if (sc) tma2d(dst + ST_SC, &a.tm_sc, row + (VLO_O >> 7), bar);
}
// wait for the phase of the given parity of a stage's mbarrier, at most 2^18 polls; false on time-out
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < (1 << 18); i++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(bar), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// two e4m3 bytes (lo = first) -> two fp32, exact (hardware e4m3 -> f16 conversion)
__device__ __forceinline__ void e4m3x2_to_f32(uint32_t two, float& lo, float& hi) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((unsigned short)two));
    asm("{.reg .f16 l, h; mov.b32 {l, h}, %2; cvt.f32.f16 %0, l; cvt.f32.f16 %1, h;}" : "=f"(lo), "=f"(hi) : "r"(h2));
}

__device__ __forceinline__ bool sub_ok(const QMArgs& a, int b, int64_t jb, const uint8_t*& src) {
    if (jb >= a.boff_stride) return false;
    const int64_t off = a.boff[(int64_t)b * a.boff_stride + jb];
    src = a.qpool + off;
    return off >= 0 && off + SUB <= a.qpool_bytes && (off & 127) == 0 && (jb + 1) * BLK <= a.npos;
}

__global__ void __launch_bounds__(128, 3) qdecode_mma(const __grid_constant__ QMArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* raw0 = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);   // the 128-byte swizzle needs 1 KB alignment
    uint32_t* cst = reinterpret_cast<uint32_t*>(raw0 + 2 * QM_STAGE);
    float2* vsl = reinterpret_cast<float2*>(raw0 + 2 * QM_STAGE + QM_CST_BYTES);
    const uint32_t bar0 = smem_u32(raw0 + 2 * QM_STAGE + QM_CST_BYTES + QM_VSL_BYTES);   // 2 x 8-byte mbarriers

    const int tid = threadIdx.x;
    const int h = tid >> 5, lane = tid & 31, g = lane >> 2, tig = lane & 3;

    // ---- schedule: this CTA's half sub-blocks [h0, h1) (sub-block units h >> 1) and the row cursor of unit h0 >> 1
    int64_t h0, h1;          // halves of this CTA
    int64_t u0;              // unit of half h0
    int b0;                  // row of unit u0
    int64_t rs0, re0;        // global unit range of row b0 ([rs0, re0); grid mode: [0, nq))
    int slot_c;              // grid mode: slot = b * nslots + slot_c; persistent: slot = slot_c + b
    const bool persistent = a.prefix != nullptr;
    // the schedule prefix (and the cleared status word / counters) come from the kernel before this one, which may
    // still run; after it, the exact-partial kernel may start filling the SMs this grid leaves
    pdl_wait();
    pdl_launch_dependents();
    if (!persistent) {
        b0 = blockIdx.x;
        const int s = blockIdx.y;
        int64_t nq = a.NQ[b0];
        if (nq > a.nqmax) nq = a.nqmax;
        if (nq < 0) nq = 0;
        u0 = min((int64_t)s * a.spb, nq);
        h0 = 2 * u0;
        h1 = 2 * min(u0 + a.spb, nq);
        rs0 = 0;
        re0 = nq;
        slot_c = s;
    } else {
        const int64_t W2 = 2 * a.prefix[a.B];
        const int64_t G = min((int64_t)gridDim.x, W2);
        const int64_t c = blockIdx.x;
        if (c >= G) return;
        h0 = c * W2 / G;
        h1 = (c + 1) * W2 / G;
        u0 = h0 >> 1;
        // largest b with prefix[b] <= u0 and a nonempty row (prefix[b + 1] > u0)
        int64_t lo_b = 0, hi_b = a.B - 1;
        while (lo_b < hi_b) {
            const int64_t mid = (lo_b + hi_b + 1) >> 1;
            if (a.prefix[mid] <= u0) lo_b = mid; else hi_b = mid - 1;
        }
        b0 = (int)lo_b;
        rs0 = a.prefix[b0];
        re0 = a.prefix[b0 + 1];
        slot_c = (int)c;
    }
    const int n2 = (int)(h1 - h0);
    // unit u -> (row, sub-block) through a forward-only cursor
    struct Cursor {
        int b;
        int64_t rs, re;
    };
    auto advance = [&](Cursor& cu, int64_t u) {
        while (u >= cu.re) {
            cu.b++;
            cu.rs = cu.re;
            cu.re = a.prefix[cu.b + 1];
        }
    };
    Cursor cur{b0, rs0, re0}, pre{b0, rs0, re0};

    // ---- QK B fragments of row `row` (q is bf16 already): column n = g is query row r = g of this head, 0 for g >= 4
    uint32_t bq[8][2];
    auto load_q = [&](int row) {
        const uint16_t* qr = a.q + ((int64_t)row * QROWS + h * 4 + (g & 3)) * DIM;
#pragma unroll
        for (int ks = 0; ks < 8; ks++)
#pragma unroll
            for (int hl = 0; hl < 2; hl++) {
                int d0, d1;
                reg_dims(tig, 2 * ks + hl, d0, d1);
                const uint32_t v = (uint32_t)qr[d0] | ((uint32_t)qr[d1] << 16);
                bq[ks][hl] = (g < 4) ? v : 0u;
            }
    };
    if (tid == 0) {
        mbar_init(bar0);
        mbar_init(bar0 + 8);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    uint32_t phase = 0;      // bit s: parity of the next phase of stage s's mbarrier
    int timeouts = 0;
    int qrow = b0;
    load_q(qrow);
    // ---- prologue: the CTA's first two halves into the two stages (the first one with its sub-block's scales)
#pragma unroll 1
    for (int k = 0; k < 2 && k < n2; k++) {
        const int64_t hk = h0 + k;
        const uint8_t* src;
        if (persistent) advance(pre, hk >> 1);
        if (sub_ok(a, pre.b, (hk >> 1) - pre.rs, src) && tid == 0)
            tma_half(a, smem_u32(raw0 + k * QM_STAGE), bar0 + 8 * k, src - a.qpool, (int)(hk & 1),
                     k == 0 || (hk & 1) == 0);
    }

    // per-thread shared-memory offsets inside a 16-token tile starting at a multiple of 16 (the swizzle phase
    // (t & 7) / (L & 7) is then fixed per thread)
    const int cc_k = 2 * h + (tig >> 1);
    const int koff_a = g * 128 + ((cc_k ^ g) << 4) + (tig & 1) * 8;     // token t0 + g
    const int koff_b = koff_a + 8 * 128;                                 // token t0 + g + 8
    int voff[4];
#pragma unroll
    for (int q4 = 0; q4 < 4; q4++) {
        const int L = tig + 4 * (q4 >> 1);                               // line of token t0 + 2tig + (q4&1) + 8(q4>>1)
        const int cc = (q4 & 1) * 4 + h;
        voff[q4] = ST_VB + L * 128 + ((cc ^ L) << 4) + 2 * g;
    }
    const int vsl_a = 2 * g + (h >> 1), vsl_b = 2 * (g + 8) + (h >> 1);

    float m[2] = {-1e30f, -1e30f}, l_part[2] = {0.f, 0.f}, lv_part[2] = {0.f, 0.f};
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[i][e] = 0.f;

    // write the partial (m, l, acc + lv) of the current segment to `slot` and reset the accumulators
    auto flush_partial = [&](int64_t slot) {
        float l[2], lv[2];
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            float x = l_part[rr], y = lv_part[rr];
            x += __shfl_xor_sync(0xffffffffu, x, 4);
            x += __shfl_xor_sync(0xffffffffu, x, 8);
            x += __shfl_xor_sync(0xffffffffu, x, 16);
            y += __shfl_xor_sync(0xffffffffu, y, 4);
            y += __shfl_xor_sync(0xffffffffu, y, 8);
            y += __shfl_xor_sync(0xffffffffu, y, 16);
            l[rr] = x;
            lv[rr] = y;
        }
        if (tig < 2) {
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int r = 2 * tig + rr;
                const int64_t row = slot * QROWS + h * 4 + r;
                if (g == 0) {
                    a.mo[row] = m[rr];
                    a.lo[row] = l[rr];
                }
                float* o = a.ao + row * DIM;
#pragma unroll
                for (int i0 = 0; i0 < 8; i0++) {
                    const float f = __uint_as_float((uint32_t)(151 - i0) << 23);   // 2^(24 - i0)
                    o[2 * g + 16 * i0] = fmaf(acc[i0][rr], f, lv[rr]);
                    o[2 * g + 1 + 16 * i0] = fmaf(acc[i0][rr + 2], f, lv[rr]);
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            m[rr] = -1e30f;
            l_part[rr] = lv_part[rr] = 0.f;
        }
#pragma unroll
        for (int i9 = 0; i9 < 8; i9++)
#pragma unroll
            for (int e9 = 0; e9 < 4; e9++) acc[i9][e9] = 0.f;
    };
    auto slot_of = [&](int row) -> int64_t {
        return persistent ? (int64_t)slot_c + row : (int64_t)row * a.nslots + slot_c;
    };

    int b = 0;
    int64_t jb = 0;
    bool ok = false;
    for (int k = 0; k < n2; k++) {
        const int64_t u = (h0 + k) >> 1;
        const int half = (int)((h0 + k) & 1);
        const bool fresh = half == 0 || k == 0;   // first stage of a sub-block in this CTA: decode its scales
        if (fresh) {
            if (persistent) advance(cur, u);
            if (cur.b != qrow) {                 // segment boundary: the previous row's partial is complete
                flush_partial(slot_of(qrow));
                qrow = cur.b;
                load_q(qrow);
            }
            b = cur.b;
            jb = u - cur.rs;
            const uint8_t* src;
            ok = sub_ok(a, b, jb, src);
        }
        uint8_t* raw = raw0 + (k & 1) * QM_STAGE;
        if (ok) {   // every thread waits for the stage's TMA; the completed phase makes its bytes visible
            if (!mbar_wait(bar0 + 8 * (k & 1), (phase >> (k & 1)) & 1u)) timeouts++;
            phase ^= 1u << (k & 1);
        }
        if (fresh) {
            if (!ok) {
                if (tid == 0) flag(a.status, (jb >= a.boff_stride || (jb + 1) * BLK > a.npos) ? ST_TABLE : ST_QPOOL);
            } else {
                // ---- cooperative preprocessing: dequant constants and (vl, vs) of this sub-block
                const float pws[4] = {32.f, 8.f, 2.f, 8.f};   // 2^(5 - 2p); plane 3 is encoded like plane 1
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int idx = tid + 128 * e;             // (hh, p, tg, pi)
                    const int pi = idx & 3, tg = (idx >> 2) & 3, p = (idx >> 4) & 3, hh = idx >> 6;
                    const int j = 8 * tg + ((pi & 1) | ((pi & 2) << 1));
                    const uint8_t* sc = raw + ST_SC + (KSC_O - VLO_O) + hh * DIM + 32 * p + j;
                    const uint8_t* lo = raw + ST_SC + (KLO_O - VLO_O) + hh * DIM + 32 * p + j;
                    float s0, s1, l0, l1;
                    e4m3x2_to_f32((uint32_t)sc[0] | ((uint32_t)sc[2] << 8), s0, s1);
                    e4m3x2_to_f32((uint32_t)lo[0] | ((uint32_t)lo[2] << 8), l0, l1);
                    const float pw = (p == 0) ? pws[0] : (p == 2) ? pws[2] : pws[1];
                    cst[2 * idx] = pack_bf16(s0 * pw, s1 * pw);
                    cst[2 * idx + 1] = pack_bf16(l0, l1);
                }
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int t = tid + 128 * e;
                    float vl0, vl1, vs0, vs1;
                    e4m3x2_to_f32(*reinterpret_cast<const uint16_t*>(raw + ST_SC + 2 * t), vl0, vl1);
                    e4m3x2_to_f32(*reinterpret_cast<const uint16_t*>(raw + ST_SC + (VSC_O - VLO_O) + 2 * t), vs0,
                                  vs1);
                    vsl[2 * t] = make_float2(vl0, vs0);
                    vsl[2 * t + 1] = make_float2(vl1, vs1);
                }
            }
            __syncthreads();
        }
        if (ok) {
            // dequant constants stay in shared memory and are re-read for every 16-token tile (8 x 16 B per thread):
            // holding them in registers across the tile loop costs more in spills than the loads
            const uint4* cstp = reinterpret_cast<const uint4*>(cst);
            const int64_t pos0 = jb * BLK + half * QM_HALF;   // position of the half's first token
            const float2* vslh = vsl + 2 * half * QM_HALF;
            // cos / sin rows of the tile's tokens t0 + g and t0 + g + 8 (this thread's 8 frequencies; the 4 warps
            // read the same rows, served by L1)
            const uint16_t* crow0 = a.cos_t + (pos0 + g) * 32 + 8 * tig;
            const uint16_t* srow0 = a.sin_t + (pos0 + g) * 32 + 8 * tig;
            // table rows of the next tile, loaded right after the current tile's key registers are built so the
            // load latency overlaps the QK MMAs (and the softmax / PV at the chunk's end)
            uint4 nca = *reinterpret_cast<const uint4*>(crow0);
            uint4 nsa = *reinterpret_cast<const uint4*>(srow0);
            uint4 ncb = *reinterpret_cast<const uint4*>(crow0 + 8 * 32);
            uint4 nsb = *reinterpret_cast<const uint4*>(srow0 + 8 * 32);
#pragma unroll 1
            for (int c0 = 0; c0 < QM_HALF; c0 += 32) {
                float sc[2][4];
                float vsv[2][2], vlv[2][2];
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    const int t0 = c0 + 16 * mt;
                    // two accumulators (rotated half, NoPE half): the two chains of 4 MMAs do not wait for each
                    // other, which shortens the latency between the key registers and the scores
                    float sx[4] = {0.f, 0.f, 0.f, 0.f}, sy[4] = {0.f, 0.f, 0.f, 0.f};
                    {
                        const uint8_t* kt = raw + t0 * 128;
                        const uint2 kwa = *reinterpret_cast<const uint2*>(kt + koff_a);
                        const uint2 kwb = *reinterpret_cast<const uint2*>(kt + koff_b);
                        const uint4 ca = nca, sa = nsa, cb = ncb, sbw = nsb;
                        const uint4* cp = cstp + (h * 4 * 4 + tig) * 2;   // [plane p] at + p * 8
                        uint32_t Ra[8], Rb[8];
                        {
                            const uint4 KC[4] = {cp[0], cp[1], cp[16], cp[17]};   // planes 0, 2
                            token_rope(kwa.x, kwa.y, ca, sa, KC, Ra, a.kbase);
                            token_rope(kwb.x, kwb.y, cb, sbw, KC, Rb, a.kbase);
                        }
                        if (t0 + 16 < QM_HALF) {
                            const uint16_t* crow = crow0 + (t0 + 16) * 32;
                            const uint16_t* srow = srow0 + (t0 + 16) * 32;
                            nca = *reinterpret_cast<const uint4*>(crow);
                            nsa = *reinterpret_cast<const uint4*>(srow);
                            ncb = *reinterpret_cast<const uint4*>(crow + 8 * 32);
                            nsb = *reinterpret_cast<const uint4*>(srow + 8 * 32);
                        }
#pragma unroll
                        for (int ks = 0; ks < 4; ks++)
                            mma_bf16(sx, Ra[2 * ks], Rb[2 * ks], Ra[2 * ks + 1], Rb[2 * ks + 1], bq[ks][0], bq[ks][1]);
                        {
                            const uint4 KC[4] = {cp[8], cp[9], cp[24], cp[25]};   // planes 1, 3
                            token_nope(kwa.x, kwa.y, KC, Ra, a.kbase);
                            token_nope(kwb.x, kwb.y, KC, Rb, a.kbase);
                        }
#pragma unroll
                        for (int ks = 4; ks < 8; ks++)
                            mma_bf16(sy, Ra[2 * (ks - 4)], Rb[2 * (ks - 4)], Ra[2 * (ks - 4) + 1], Rb[2 * (ks - 4) + 1],
                                     bq[ks][0], bq[ks][1]);
                    }
#pragma unroll
                    for (int e = 0; e < 4; e++) sc[mt][e] = sx[e] + sy[e];
                    const float2 xa = vslh[2 * t0 + vsl_a], xb = vslh[2 * t0 + vsl_b];
                    vlv[mt][0] = xa.x; vsv[mt][0] = xa.y;
                    vlv[mt][1] = xb.x; vsv[mt][1] = xb.y;
                }
                // ---- online softmax over the 32 tokens for this thread's rows r = 2 tig, 2 tig + 1
                // lazy rescale: the reference point m moves only when a score exceeds it by more than 2^6, so p <= 64
                // and fp16(p * vs) <= 64 * 448 stays finite; the partial (m, l, acc) is exact for any m
                // the row maxima are reduced across the 8 lanes of a row only when some score of the warp passes its
                // row's reference point by more than 2^6 (rare after the first chunk)
                float lmx[2];
                bool need = false;
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    lmx[rr] = fmaxf(fmaxf(sc[0][rr], sc[0][rr + 2]), fmaxf(sc[1][rr], sc[1][rr + 2])) * a.scale;
                    need |= lmx[rr] > m[rr] + 6.0f;
                }
                if (__any_sync(0xffffffffu, need)) {
                    float alpha[2] = {1.f, 1.f};
#pragma unroll
                    for (int rr = 0; rr < 2; rr++) {
                        float mx = lmx[rr];
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                        if (mx > m[rr] + 6.0f) {
                            alpha[rr] = fast_exp2(m[rr] - mx);
                            m[rr] = mx;
                        }
                    }
#pragma unroll
                    for (int rr = 0; rr < 2; rr++) {
                        l_part[rr] *= alpha[rr];
                        lv_part[rr] *= alpha[rr];
                    }
#pragma unroll
                    for (int i9 = 0; i9 < 8; i9++) {
                        acc[i9][0] *= alpha[0];
                        acc[i9][1] *= alpha[1];
                        acc[i9][2] *= alpha[0];
                        acc[i9][3] *= alpha[1];
                    }
                }
                float p[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; mt++)
#pragma unroll
                    for (int e = 0; e < 4; e++) p[mt][e] = fast_exp2(fmaf(sc[mt][e], a.scale, -m[e & 1]));
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
#pragma unroll
                    for (int mt = 0; mt < 2; mt++) {
                        l_part[rr] += p[mt][rr] + p[mt][rr + 2];
                        lv_part[rr] = fmaf(p[mt][rr], vlv[mt][0], lv_part[rr]);
                        lv_part[rr] = fmaf(p[mt][rr + 2], vlv[mt][1], lv_part[rr]);
                    }
                }
                // ---- PV over the two 16-token K-steps
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    const int t0 = c0 + 16 * mt;
                    const uint32_t xa = pack_f16(p[mt][0] * vsv[mt][0], p[mt][1] * vsv[mt][0]);   // token g
                    const uint32_t xb = pack_f16(p[mt][2] * vsv[mt][1], p[mt][3] * vsv[mt][1]);   // token g + 8
                    const uint32_t b0 = transpose8x8(xa), b1 = transpose8x8(xb);
                    // V bytes (2g, 2g + 1) of head h for tokens t0 + 2tig, +1, +8, +9 (swizzled vb lines)
                    uint32_t v[4];
                    const uint8_t* vt = raw + t0 * 64;
#pragma unroll
                    for (int q4 = 0; q4 < 4; q4++) v[q4] = *reinterpret_cast<const uint16_t*>(vt + voff[q4]);
                    const uint32_t wa = __byte_perm(v[0], v[1], 0x2420);   // byte 2g of (t, t + 1), one per lane
                    const uint32_t wb = __byte_perm(v[0], v[1], 0x2521);   // byte 2g + 1
                    const uint32_t wc = __byte_perm(v[2], v[3], 0x2420);
                    const uint32_t wd = __byte_perm(v[2], v[3], 0x2521);
#pragma unroll
                    for (int i0 = 0; i0 < 8; i0++) {
                        const uint32_t msk = 0x00010001u << i0;
                        mma_f16(acc[i0], wa & msk, wb & msk, wc & msk, wd & msk, b0, b1);
                    }
                }
            }
        }
        __syncthreads();   // stage (k & 1) free again (and cst / vsl once the second half is done)
        if (k + 2 < n2) {
            const int64_t h2 = h0 + k + 2;
            const uint8_t* src2;
            if (persistent) advance(pre, h2 >> 1);
            if (sub_ok(a, pre.b, (h2 >> 1) - pre.rs, src2) && tid == 0)
                tma_half(a, smem_u32(raw), bar0 + 8 * (k & 1), src2 - a.qpool, (int)(h2 & 1), (h2 & 1) == 0);
        }
    }
    if (timeouts && tid == 0) flag(a.status, ST_TIMEOUT);
    flush_partial(slot_of(qrow));
}


}  // namespace kv800
