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

__device__ __forceinline__ void hadamard_signs(int lane, float (&C)[32]) {
    const float c = 0.0883883461356163f;   // fp32(1 / sqrt(128)), the entry magnitude of the reference's hadamard()
#pragma unroll
    for (int b = 0; b < 32; b++) C[b] = (__popc(b & lane) & 1) ? -c : c;
}

}  // namespace kv800
