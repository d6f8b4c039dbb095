// Log-sum-exp merge of a row's split partials, with the in-register Hadamard for the quantized part (kv800.py:231-236).
// One warp merges the 4 query rows of one kv head; the standalone combine kernel runs it for every (row, head), and the
// exact-partial kernel runs it in the last CTA that finishes a row (or a (row, head)), so a decode needs no separate
// merge launch.
#pragma once
#include "kv800_common.cuh"

namespace kv800 {

constexpr float NEG_BIG = -1e30f;   // the reference's initial running max (kv800.py:127)

// Where the partials of row b live.  Quantized slots: grid mode (prefix == nullptr) b * qstride + s for s < ns;
// persistent mode c + b for the CTAs c whose range of half sub-blocks [c 2W / G, (c + 1) 2W / G) meets row b's
// halves [2 prefix[b], 2 prefix[b + 1]).  Exact slots: xbase + b * xstride + e for e < nx.
struct SlotMap {
    int ns;
    int64_t qstride;
    const int64_t* prefix;
    int64_t B;
    int64_t G0;
    int64_t xbase, xstride;
    int nx;
};

// Merge of query rows 4 h .. 4 h + 3 of row b by one warp, lane = dims 4 lane .. 4 lane + 3:
// o = (sum_{quantized} w_s acc_s) H + sum_{exact} w_s acc_s, w_s = exp2(m_s - max m), out = bf16(o / sum_s w_s l_s);
// a row with no keys at all gives zeros (torch_decode.py:71-72).  Each group of slots (exact, quantized) is reduced in
// one pass with a running maximum (a partial whose m exceeds it rescales the sums so far by exp2(M - m)), then the two
// groups are combined; with wait_quantized the exact group is reduced before waiting for the kernel that writes the
// quantized partials (programmatic dependent launch).  Partials are read through L2 (ld.global.cg): inside the kernel
// that wrote some of them, this SM's L1 may hold lines from before they were written.
__device__ __forceinline__ void combine_head(const float* mo, const float* lo, const float* ao, const SlotMap& sm,
                                             uint16_t* out, int b, int h, int lane, bool wait_quantized = false) {
    const int r0 = 4 * h;
    // one group of slots [s0, s0 + cnt) -> running max M, sum L, weighted acc o of this lane's dims
    auto reduce = [&](int64_t s0, int64_t cnt, float (&M)[4], float (&L)[4], float (&o)[4][4]) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            M[j] = NEG_BIG;
            L[j] = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) o[j][k] = 0.f;
        }
#pragma unroll 4
        for (int64_t i = 0; i < cnt; i++) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int64_t row = (s0 + i) * QROWS + r0 + j;
                const float m = __ldcg(mo + row), l = __ldcg(lo + row);
                const float4 x = __ldcg(reinterpret_cast<const float4*>(ao + row * DIM + 4 * lane));
                if (m > M[j]) {   // uniform across the warp: every lane reads the same m
                    const float sc = exp2f(M[j] - m);
                    L[j] *= sc;
#pragma unroll
                    for (int k = 0; k < 4; k++) o[j][k] *= sc;
                    M[j] = m;
                }
                const float w = exp2f(m - M[j]);
                L[j] = fmaf(w, l, L[j]);
                o[j][0] = fmaf(w, x.x, o[j][0]);
                o[j][1] = fmaf(w, x.y, o[j][1]);
                o[j][2] = fmaf(w, x.z, o[j][2]);
                o[j][3] = fmaf(w, x.w, o[j][3]);
            }
        }
    };
    float Mx[4], Lx[4], ox[4][4];
    reduce(sm.xbase + (int64_t)b * sm.xstride, sm.nx, Mx, Lx, ox);
    if (wait_quantized) pdl_wait();
    int64_t q0 = 0, nqs = 0;
    if (sm.prefix == nullptr) {
        q0 = (int64_t)b * sm.qstride;
        nqs = sm.ns;
    } else {
        const int64_t W2 = 2 * sm.prefix[sm.B];
        const int64_t rs = 2 * sm.prefix[b], re = 2 * sm.prefix[b + 1];   // the row's halves [rs, re)
        if (W2 > 0 && re > rs) {
            const int64_t G = min(sm.G0, W2);
            // CTA of half u: the c with floor(c W2 / G) <= u < floor((c + 1) W2 / G), i.e. ((u + 1) G - 1) / W2
            const int64_t cf = ((rs + 1) * G - 1) / W2, cl = (re * G - 1) / W2;
            q0 = cf + b;
            nqs = cl - cf + 1;
        }
    }
    float Mq[4], Lq[4], oq[4][4];
    reduce(q0, nqs, Mq, Lq, oq);
    if (nqs > 0) {
        // 128-point Sylvester Hadamard: dims d = 4 lane + e; stages 1, 2 in-lane, 4 .. 64 across lanes 1 .. 16
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float* v = oq[j];
            const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
            v[0] = a0 + a2;
            v[2] = a0 - a2;
            v[1] = a1 + a3;
            v[3] = a1 - a3;
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float other = __shfl_xor_sync(0xffffffffu, oq[j][e], o);
                    oq[j][e] = upper ? other - oq[j][e] : oq[j][e] + other;
                }
        }
    }
    const float c = 0.0883883461356163f;   // 128^-1/2
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float M = fmaxf(Mx[j], Mq[j]);
        const float sx = exp2f(Mx[j] - M), sq = exp2f(Mq[j] - M);
        const float L = fmaf(sx, Lx[j], sq * Lq[j]), cq = c * sq;
        uint16_t res[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float o = fmaf(oq[j][e], cq, sx * ox[j][e]);
            res[e] = (L > 0.f) ? f2bf(o / L) : (uint16_t)0;
        }
        uint2 pk;
        pk.x = (uint32_t)res[0] | ((uint32_t)res[1] << 16);
        pk.y = (uint32_t)res[2] | ((uint32_t)res[3] << 16);
        *reinterpret_cast<uint2*>(out + ((int64_t)b * QROWS + r0 + j) * DIM + 4 * lane) = pk;
    }
}

}  // namespace kv800
