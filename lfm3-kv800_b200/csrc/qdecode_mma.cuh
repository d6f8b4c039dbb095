// Quantized-split decode kernel on the tensor cores (mma.sync m16n8k16), sm_100a.
//
// Per (row b, split s) CTA of 4 warps, warp = kv head h, over sub-blocks [s spb, min((s + 1) spb, NQ[b], nqmax)):
//   QK   S[t, r] = sum_d Kr[t, d] q[r, d]: M = 16 tokens, N = 8 query columns (the head's 4 rows + 4 zero rows),
//        K = 16 dims per step, bf16 operands, fp32 accumulate.  The A fragments are the reference's keys exactly:
//        k = bf16(c sc + lo) (kv800.py:86) via one bf16x2 FMA per register pair (c sc + lo is exact before the single
//        rounding), and for the RoPE dims kr = bf16(fl32(k0 cs - k2 sn)) (torch_decode.py:16-24) in fp32.
//   PV   acc[d, r] += sum_t V^[t, d] P[t, r]: M = 16 dims (one bit plane of 16 V bytes), N = 8 columns, K = 16 tokens,
//        fp16 operands.  A = 0.5 + bit * 2^(i - 8) for bit plane i (one LOP3 per register from the packed V bytes);
//        B = fp16(p * vs), transposed from the QK accumulator layout with movmatrix.  A ninth M-tile of constant 0.5
//        accumulates 0.5 sum_t B, so sum_t B[t, r] bit[t, d] = (acc_i - acc_S) 2^(8 - i) exactly up to fp32 rounding.
//   The exact V of a quantized token is bits * vs + vl in the Hadamard domain (kv800.py:87-91); vl enters through
//   lv = sum_t p vl, and combine() applies H once (kv800.py:231-236).
// Online softmax in the log2 domain per 32-token chunk; partial (m, l, acc + lv) written to the reference's slot
// layout.  Sub-blocks are prefetched into L2 by the TMA engine (cp.async.bulk.prefetch.L2) two ahead; fragments are
// then read with sector-exact global loads (each 32 B kc segment and 16 B vb segment once per head).
#pragma once
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
    int nslots;
    int spb;
    float scale;
    int* status;
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
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// bf16 bits of an fp8 e4m3fn byte scaled by 2^e (exact for the scalings used here).
__device__ __forceinline__ uint32_t f8_to_bf16_scaled(uint32_t b, float pw2) {
    return (uint32_t)f2bf(f8dec(b) * pw2);
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

// Register layout of one token's QK A operand for thread tig (bytes J = 8 tig .. 8 tig + 7 of the kc row):
//   R[u], u < 8      (kr0_j, kr2_j), j = 8 tig + u              (RoPE dims j and j + 64)
//   R[8 + pi]        (k1_j, k1_{j+2}), j = 8 tig + {0,1,4,5}[pi] (NoPE dims 32 + j, 32 + j + 2)
//   R[12 + pi]       (k3_j, k3_{j+2})                            (NoPE dims 96 + j, 96 + j + 2)
// K-step ks uses R[2 ks] for columns (2 tig, 2 tig + 1) and R[2 ks + 1] for columns (2 tig + 8, 2 tig + 9).
//
// Per-plane code encodings (bf16, code c at mantissa bits of the plane): x = 4 + c * 2^(2p - 5) for planes 0..2 and
// plane 3 shifted down by 4 bits (encoded like plane 1), so (x - 4) * (sc * 2^(5 - 2p)) = c * sc exactly and
// fma(x - 4, A, lo) = bf16(c sc + lo) with one rounding.
struct DequantConsts {
    uint32_t A[4][4];    // [plane][pair]: bf16x2 of sc_j * 2^(5 - 2p') for the pair (j, j + 2)
    uint32_t L[4][4];    // [plane][pair]: bf16x2 of lo_j, lo_{j+2}
};

__device__ __forceinline__ void token_regs(uint32_t w0, uint32_t w1, const uint4& cw, const uint4& sw,
                                           const DequantConsts& K, uint32_t (&R)[16]) {
    const uint32_t BASE = 0x40804080u;   // bf16x2 (4.0, 4.0)
    // pair words: byte pair (j, j + 2) at bits 0-7 / 16-23
    const uint32_t pw[4] = {w0, w0 >> 8, w1, w1 >> 8};
    const uint32_t cwv[4] = {cw.x, cw.y, cw.z, cw.w};   // cos of j = 8tig + {0,1}, {2,3}, {4,5}, {6,7}
    const uint32_t swv[4] = {sw.x, sw.y, sw.z, sw.w};
#pragma unroll
    for (int pi = 0; pi < 4; pi++) {
        const uint32_t P = pw[pi];
        // NoPE planes 1 and 3 -> A registers directly
        const uint32_t x1 = lop3_and_or(P, 0x000c000cu, BASE);
        R[8 + pi] = hfma2_bf16(hsub2_bf16(x1, BASE), K.A[1][pi], K.L[1][pi]);
        const uint32_t x3 = lop3_and_or(P >> 4, 0x000c000cu, BASE);
        R[12 + pi] = hfma2_bf16(hsub2_bf16(x3, BASE), K.A[3][pi], K.L[3][pi]);
        // RoPE planes 0 and 2: bf16 keys, then rotation in fp32 and the second rounding
        const uint32_t x0 = lop3_and_or(P, 0x00030003u, BASE);
        const uint32_t k0 = hfma2_bf16(hsub2_bf16(x0, BASE), K.A[0][pi], K.L[0][pi]);
        const uint32_t x2 = lop3_and_or(P, 0x00300030u, BASE);
        const uint32_t k2 = hfma2_bf16(hsub2_bf16(x2, BASE), K.A[2][pi], K.L[2][pi]);
        // the pair is (j, j + 2) with j = 8 tig + {0, 1, 4, 5}[pi]: cos word index (j - 8tig) / 2 and half (j & 1)
        const int wi = (pi >> 1) * 2;           // words {0,1} for pi < 2, {2,3} for pi >= 2
        const bool odd = (pi & 1) != 0;
        const float cs_a = __uint_as_float(odd ? (cwv[wi] & 0xffff0000u) : (cwv[wi] << 16));
        const float cs_b = __uint_as_float(odd ? (cwv[wi + 1] & 0xffff0000u) : (cwv[wi + 1] << 16));
        const float sn_a = __uint_as_float(odd ? (swv[wi] & 0xffff0000u) : (swv[wi] << 16));
        const float sn_b = __uint_as_float(odd ? (swv[wi + 1] & 0xffff0000u) : (swv[wi + 1] << 16));
        const float k0a = __uint_as_float(k0 << 16), k0b = __uint_as_float(k0 & 0xffff0000u);
        const float k2a = __uint_as_float(k2 << 16), k2b = __uint_as_float(k2 & 0xffff0000u);
        const float r0a = fmaf(k0a, cs_a, -(k2a * sn_a)), r2a = fmaf(k2a, cs_a, k0a * sn_a);
        const float r0b = fmaf(k0b, cs_b, -(k2b * sn_b)), r2b = fmaf(k2b, cs_b, k0b * sn_b);
        const int ua = (pi & 1) | ((pi & 2) << 1);   // u of byte j = 8 tig + u
        R[ua] = pack_bf16(r0a, r2a);
        R[ua + 2] = pack_bf16(r0b, r2b);
    }
}

__global__ void __launch_bounds__(128, 3) qdecode_mma(QMArgs a) {
    const int b = blockIdx.x, s = blockIdx.y;
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
    int64_t nq = a.NQ[b];
    if (nq > a.nqmax) nq = a.nqmax;
    const int64_t j0 = (int64_t)s * a.spb;
    const int64_t j1 = min(j0 + a.spb, nq);

    // ---- QK B fragments (q is bf16 already): column n = g is query row r = g of this head, zero for g >= 4
    uint32_t bq[8][2];
    {
        const uint16_t* qr = a.q + ((int64_t)b * QROWS + h * 4 + (g & 3)) * DIM;
#pragma unroll
        for (int ks = 0; ks < 8; ks++)
#pragma unroll
            for (int hl = 0; hl < 2; hl++) {
                int d0, d1;
                reg_dims(tig, 2 * ks + hl, d0, d1);
                const uint32_t v = (uint32_t)qr[d0] | ((uint32_t)qr[d1] << 16);
                bq[ks][hl] = (g < 4) ? v : 0u;
            }
    }
    // prefetch the first sub-blocks of this split into L2
    if (threadIdx.x == 0) {
        for (int64_t jb = j0; jb < min(j0 + 2, j1); jb++) {
            if (jb < a.boff_stride) {
                const int64_t off = a.boff[(int64_t)b * a.boff_stride + jb];
                if (off >= 0 && off + SUB <= a.qpool_bytes && ((off | reinterpret_cast<uintptr_t>(a.qpool)) & 15) == 0)
                    prefetch_l2(a.qpool + off, SUB);
            }
        }
    }

    float m[2] = {-1e30f, -1e30f}, l_part[2] = {0.f, 0.f}, lv_part[2] = {0.f, 0.f};
    float acc[9][4];
#pragma unroll
    for (int i = 0; i < 9; i++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[i][e] = 0.f;

    for (int64_t jb = j0; jb < j1; jb++) {
        if (jb >= a.boff_stride) {
            if (lane == 0) flag(a.status, ST_TABLE);
            break;
        }
        const int64_t off = a.boff[(int64_t)b * a.boff_stride + jb];
        const uint8_t* sb = a.qpool + off;
        if (off < 0 || off + SUB > a.qpool_bytes || (reinterpret_cast<uintptr_t>(sb) & 15u)) {
            if (lane == 0) flag(a.status, ST_QPOOL);
            continue;
        }
        if (threadIdx.x == 0 && jb + 2 < j1 && jb + 2 < a.boff_stride) {
            const int64_t off2 = a.boff[(int64_t)b * a.boff_stride + jb + 2];
            if (off2 >= 0 && off2 + SUB <= a.qpool_bytes && ((off2 | reinterpret_cast<uintptr_t>(a.qpool)) & 15) == 0)
                prefetch_l2(a.qpool + off2, SUB);
        }
        if ((jb + 1) * BLK > a.npos) {
            if (lane == 0) flag(a.status, ST_TABLE);
            break;
        }
        // ---- per-sub-block dequant constants for this thread's channels (bytes 8 tig .. 8 tig + 7, 4 planes)
        DequantConsts K;
        {
            const uint8_t* ksc = sb + KSC_O + h * DIM;
            const uint8_t* klo = sb + KLO_O + h * DIM;
            const float pw[4] = {32.f, 8.f, 2.f, 8.f};   // 2^(5 - 2p) per plane (plane 3 is encoded like plane 1)
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const uint2 scw = *reinterpret_cast<const uint2*>(ksc + 32 * p + 8 * tig);
                const uint2 low = *reinterpret_cast<const uint2*>(klo + 32 * p + 8 * tig);
                const uint32_t sbt[2] = {scw.x, scw.y}, lbt[2] = {low.x, low.y};
#pragma unroll
                for (int pi = 0; pi < 4; pi++) {
                    const int u = (pi & 1) | ((pi & 2) << 1);   // byte u and u + 2 of the 8
                    const uint32_t s0 = (sbt[u >> 2] >> (8 * (u & 3))) & 0xffu;
                    const uint32_t s1 = (sbt[(u + 2) >> 2] >> (8 * ((u + 2) & 3))) & 0xffu;
                    const uint32_t l0 = (lbt[u >> 2] >> (8 * (u & 3))) & 0xffu;
                    const uint32_t l1 = (lbt[(u + 2) >> 2] >> (8 * ((u + 2) & 3))) & 0xffu;
                    K.A[p][pi] = f8_to_bf16_scaled(s0, pw[p]) | (f8_to_bf16_scaled(s1, pw[p]) << 16);
                    K.L[p][pi] = f8_to_bf16_scaled(l0, 1.f) | (f8_to_bf16_scaled(l1, 1.f) << 16);
                }
            }
        }
        const int64_t pos0 = jb * BLK;
        // ---- 256 tokens in chunks of 32 (2 M-tiles)
#pragma unroll 1
        for (int c0 = 0; c0 < BLK; c0 += 32) {
            float sc[2][4];
            uint32_t P_lo[2], P_hi[2];
            float vsv[2][2];
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int t0 = c0 + 16 * mt;
                uint32_t R0[16], R1[16];
                {
                    const int ta = t0 + g, tb = t0 + g + 8;
                    const uint2 kwa = *reinterpret_cast<const uint2*>(sb + KC_O + (ta * HEADS + h) * 32 + 8 * tig);
                    const uint2 kwb = *reinterpret_cast<const uint2*>(sb + KC_O + (tb * HEADS + h) * 32 + 8 * tig);
                    const uint4 ca = *reinterpret_cast<const uint4*>(a.cos_t + (pos0 + ta) * 32 + 8 * tig);
                    const uint4 sa = *reinterpret_cast<const uint4*>(a.sin_t + (pos0 + ta) * 32 + 8 * tig);
                    const uint4 cb = *reinterpret_cast<const uint4*>(a.cos_t + (pos0 + tb) * 32 + 8 * tig);
                    const uint4 sbw = *reinterpret_cast<const uint4*>(a.sin_t + (pos0 + tb) * 32 + 8 * tig);
                    token_regs(kwa.x, kwa.y, ca, sa, K, R0);
                    token_regs(kwb.x, kwb.y, cb, sbw, K, R1);
                }
#pragma unroll
                for (int e = 0; e < 4; e++) sc[mt][e] = 0.f;
#pragma unroll
                for (int ks = 0; ks < 8; ks++)
                    mma_bf16(sc[mt], R0[2 * ks], R1[2 * ks], R0[2 * ks + 1], R1[2 * ks + 1], bq[ks][0], bq[ks][1]);
                // vl / vs of tokens t0 + g and t0 + g + 8
                vsv[mt][0] = f8dec(sb[VSC_O + (t0 + g) * 2 + (h >> 1)]);
                vsv[mt][1] = f8dec(sb[VSC_O + (t0 + g + 8) * 2 + (h >> 1)]);
                const float vla = f8dec(sb[VLO_O + (t0 + g) * 2 + (h >> 1)]);
                const float vlb = f8dec(sb[VLO_O + (t0 + g + 8) * 2 + (h >> 1)]);
                // stash vl in the P slots for now (used after the max is known)
                P_lo[mt] = __float_as_uint(vla);
                P_hi[mt] = __float_as_uint(vlb);
            }
            // ---- online softmax over the 32 tokens for this thread's rows r = 2 tig, 2 tig + 1
            float alpha[2];
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                float mx = fmaxf(fmaxf(sc[0][rr], sc[0][rr + 2]), fmaxf(sc[1][rr], sc[1][rr + 2])) * a.scale;
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float mn = fmaxf(m[rr], mx);
                alpha[rr] = exp2f(m[rr] - mn);
                m[rr] = mn;
            }
            float p[2][4];
#pragma unroll
            for (int mt = 0; mt < 2; mt++)
#pragma unroll
                for (int e = 0; e < 4; e++) p[mt][e] = exp2f(fmaf(sc[mt][e], a.scale, -m[e & 1]));
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                float ls = 0.f, lvs = 0.f;
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    ls += p[mt][rr] + p[mt][rr + 2];
                    lvs = fmaf(p[mt][rr], __uint_as_float(P_lo[mt]), lvs);
                    lvs = fmaf(p[mt][rr + 2], __uint_as_float(P_hi[mt]), lvs);
                }
                l_part[rr] = fmaf(l_part[rr], alpha[rr], ls);
                lv_part[rr] = fmaf(lv_part[rr], alpha[rr], lvs);
            }
#pragma unroll
            for (int i = 0; i < 9; i++) {
                acc[i][0] *= alpha[0];
                acc[i][1] *= alpha[1];
                acc[i][2] *= alpha[0];
                acc[i][3] *= alpha[1];
            }
            // ---- PV over the two 16-token K-steps
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int t0 = c0 + 16 * mt;
                // B = fp16(p * vs) transposed: rows r, tokens as K
                const uint32_t xa = pack_f16(p[mt][0] * vsv[mt][0], p[mt][1] * vsv[mt][0]);   // token g
                const uint32_t xb = pack_f16(p[mt][2] * vsv[mt][1], p[mt][3] * vsv[mt][1]);   // token g + 8
                const uint32_t b0 = transpose8x8(xa), b1 = transpose8x8(xb);
                // A: V bytes (2g, 2g + 1) of tokens t0 + 2tig, +1, +8, +9
                const uint16_t* vrow = reinterpret_cast<const uint16_t*>(sb + VB_O + h * 16 + 2 * g);
                const uint32_t v0 = vrow[(t0 + 2 * tig) * 32], v1 = vrow[(t0 + 2 * tig + 1) * 32];
                const uint32_t v2 = vrow[(t0 + 2 * tig + 8) * 32], v3 = vrow[(t0 + 2 * tig + 9) * 32];
                // byte 2g of (t, t+1) -> word A (dim row g), byte 2g+1 -> word B (dim row g + 8); shifted by 3
                // (bytes 2 and 3 of the zero-extended 16-bit loads are zero: selector 2 fills the gaps)
                const uint32_t wa = __byte_perm(v0, v1, 0x2420) << 3;   // (v0.b0, v1.b0)
                const uint32_t wb = __byte_perm(v0, v1, 0x2521) << 3;   // (v0.b1, v1.b1)
                const uint32_t wc = __byte_perm(v2, v3, 0x2420) << 3;
                const uint32_t wd = __byte_perm(v2, v3, 0x2521) << 3;
#pragma unroll
                for (int i0 = 0; i0 < 8; i0++) {
                    const uint32_t msk = 0x00080008u << i0;
                    mma_f16(acc[i0], lop3_and_or(wa, msk, 0x38003800u), lop3_and_or(wb, msk, 0x38003800u),
                            lop3_and_or(wc, msk, 0x38003800u), lop3_and_or(wd, msk, 0x38003800u), b0, b1);
                }
                mma_f16(acc[8], 0x38003800u, 0x38003800u, 0x38003800u, 0x38003800u, b0, b1);
            }
        }
    }
    // ---- finalize: rows r = 2 tig, 2 tig + 1 (valid for tig < 2)
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
        const int64_t slot = (int64_t)b * a.nslots + s;
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
                const float f = __uint_as_float((uint32_t)(135 - i0) << 23);   // 2^(8 - i0)
                o[2 * g + 16 * i0] = fmaf(acc[i0][rr] - acc[8][rr], f, lv[rr]);
                o[2 * g + 1 + 16 * i0] = fmaf(acc[i0][rr + 2] - acc[8][rr + 2], f, lv[rr]);
            }
        }
    }
}

}  // namespace kv800
