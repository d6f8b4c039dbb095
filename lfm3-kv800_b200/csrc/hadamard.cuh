// The V rotation of the 800h quantizer: rows of 128 fp32 values times the Sylvester Hadamard matrix / sqrt(128),
// computed with the exact fp32 operation order of the reference's CPU BLAS (lfm3_kv800/kv800.py:43-46,66).
#pragma once
#include "kv800_common.cuh"

namespace kv800 {

// y[h][k] = (x_h @ H)[lane + 32 k] for the 4 rows x_h = rows[h * 128 .. h * 128 + 127] (fp32, shared memory), each
// output the sequential chain acc = fma(x_i, H[i][d], acc), i = 0 .. 127, from acc = 0: the arithmetic of the
// reference's CPU BLAS for v.float() @ H, so the result is bit-identical.  C[b] = +-c for the lane part of the sign
// (parity(b & lane)); the (a, k) part of the sign, parity(a & k) for i = 32 a + b and d = lane + 32 k, is folded
// into the operand at compile time.
__device__ __forceinline__ void hadamard_rows(const float* rows, const float (&C)[32], float (&y)[HEADS][4]) {
#pragma unroll
    for (int hp = 0; hp < 2; hp++) {
        float acc[2][4];
#pragma unroll
        for (int q = 0; q < 2; q++)
#pragma unroll
            for (int k = 0; k < 4; k++) acc[q][k] = 0.f;
        const float* v0 = rows + (2 * hp) * DIM;
        const float* v1 = rows + (2 * hp + 1) * DIM;
#pragma unroll
        for (int a = 0; a < 4; a++) {
#pragma unroll
            for (int b4 = 0; b4 < 32; b4 += 4) {
                float4 x0 = *reinterpret_cast<const float4*>(v0 + 32 * a + b4);
                float4 x1 = *reinterpret_cast<const float4*>(v1 + 32 * a + b4);
                float xs0[4] = {x0.x, x0.y, x0.z, x0.w}, xs1[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int u = 0; u < 4; u++) {
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const bool neg = (__builtin_popcount(a & k) & 1) != 0;
                        acc[0][k] = fmaf(neg ? -xs0[u] : xs0[u], C[b4 + u], acc[0][k]);
                        acc[1][k] = fmaf(neg ? -xs1[u] : xs1[u], C[b4 + u], acc[1][k]);
                    }
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            y[2 * hp][k] = acc[0][k];
            y[2 * hp + 1][k] = acc[1][k];
        }
    }
}

// One output of hadamard_rows: (x @ H)[lane + 32 k] of the 128 values at row, by the same sequential FMA chain in
// the same order and with the same operands, so the same bits.  For re-deciding a single element the fast estimate
// below could not decide.
__device__ __forceinline__ float hadamard_one(const float* row, const float (&C)[32], int k) {
    float acc = 0.f;
#pragma unroll
    for (int a = 0; a < 4; a++) {
        const bool neg = (__popc(a & k) & 1) != 0;
#pragma unroll
        for (int b4 = 0; b4 < 32; b4 += 4) {
            const float4 x = *reinterpret_cast<const float4*>(row + 32 * a + b4);
            const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int u = 0; u < 4; u++) acc = fmaf(neg ? -xs[u] : xs[u], C[b4 + u], acc);
        }
    }
    return acc;
}

// Fast estimate of the same rotation with a rigorous error bound, for decisions that only need the rotated value to
// within a tolerance (the quantizer's fp8 lo / scale bytes and 1-bit codes).  y[h][k] ~ (x_h @ H)[lane + 32 k] by a
// fast Walsh-Hadamard transform (7 butterfly levels, 2 in-lane, 5 across lanes) and one multiply by c, and E[h] bounds
// |y - y_chain| for every element of row h, y_chain being the sequential FMA chain of hadamard_rows:
//   chain:  rounding k (k = 1..128) is <= u |partial sum k| <= u c sum_{i<k} |x_i|, in total <= u c W with
//           W = sum_i (128 - i) |x_i| (element i is in the partial sums k > i)               (u = 2^-24)
//   FWHT:   each level's rounding errors sum to <= u S over the nodes feeding one output (7 levels, S = sum_i |x_i|),
//           plus the final multiply <= u c S,
// so |y - y_chain| <= u c (W + 8 S) (1 + 1e-5); E = (W + 8 S) * 1.02 u c + 1e-38 (the absolute term covers subnormal
// results).  A CPU sweep over 100 K rows of five distributions measured at most 19 u c S.
// Returns false when some S is not finite (NaN / inf inputs or overflow): the caller then needs the exact chain.
// Zero results are returned as +0, which is what the chain gives (its accumulator starts at +0).
__device__ __forceinline__ bool fwht_rows(const float* rows, float (&y)[HEADS][4], float (&E)[HEADS]) {
    const int lane = threadIdx.x & 31;
    const float c = 0.0883883461356163f;
    const float KE = 1.02f * 5.9604644775390625e-08f * 0.0883883461356163f;
    // this lane's dims d = lane + 32 k of every head, and its part of W + 8 S = sum of (W_i + 8) |x_i|
    float sl[HEADS];
#pragma unroll
    for (int h = 0; h < HEADS; h++) {
#pragma unroll
        for (int k = 0; k < 4; k++) y[h][k] = rows[h * DIM + lane + 32 * k];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 4; k++) s = fmaf((float)(136 - lane - 32 * k), fabsf(y[h][k]), s);
        sl[h] = s;
    }
    // the 4 sums over the warp in one transposed butterfly: after the xor-16 step a lane keeps heads 2 b4, 2 b4 + 1
    // (b4 = lane bit 4), after the xor-8 step head 2 b4 + b3, then three plain steps; head h's sum ends in lanes
    // 8 h .. 8 h + 7 and is broadcast from lane 8 h
    const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0;
    float k0 = b4 ? sl[2] : sl[0], k1 = b4 ? sl[3] : sl[1];
    k0 += __shfl_xor_sync(0xffffffffu, b4 ? sl[0] : sl[2], 16);
    k1 += __shfl_xor_sync(0xffffffffu, b4 ? sl[1] : sl[3], 16);
    float kk = b3 ? k1 : k0;
    kk += __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
    kk += __shfl_xor_sync(0xffffffffu, kk, 4);
    kk += __shfl_xor_sync(0xffffffffu, kk, 2);
    kk += __shfl_xor_sync(0xffffffffu, kk, 1);
    bool finite = true;
#pragma unroll
    for (int h = 0; h < HEADS; h++) {
        const float s = __shfl_sync(0xffffffffu, kk, 8 * h);
        float v[4] = {y[h][0], y[h][1], y[h][2], y[h][3]};
        // dims d = lane + 32 k: bits 5, 6 of d are k (in-lane levels), bits 0..4 are the lane (shuffle levels); a
        // butterfly is one FMA by +-1 (other - v = fma(v, -1, other), v + other = fma(v, 1, other), both exact
        // products with the one rounding of the sum)
        float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
        v[0] = a0 + a2;
        v[2] = a0 - a2;
        v[1] = a1 + a3;
        v[3] = a1 - a3;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float sg = (lane & o) ? -1.0f : 1.0f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float other = __shfl_xor_sync(0xffffffffu, v[k], o);
                v[k] = fmaf(v[k], sg, other);
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) y[h][k] = v[k] * c + 0.0f;
        finite = finite && isfinite(s);
        E[h] = fmaf(s, KE, 1e-38f);
    }
    return finite;
}

__device__ __forceinline__ void hadamard_signs(int lane, float (&C)[32]) {
    const float c = 0.0883883461356163f;   // fp32(1 / sqrt(128)), the entry magnitude of the reference's hadamard()
#pragma unroll
    for (int b = 0; b < 32; b++) C[b] = (__popc(b & lane) & 1) ? -c : c;
}

}  // namespace kv800
