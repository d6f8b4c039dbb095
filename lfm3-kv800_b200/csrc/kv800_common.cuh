// Shared device helpers of the 800h CUDA library (sm_100a): layout constants, bf16 / fp8 e4m3fn conversions written
// from the format definitions, the device status word, and the host-side error plumbing of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/kv800_b200.h"

namespace kv800 {

// Sub-block byte map (lfm3_kv800/kv800.py:3-10,32-34).
constexpr int BLK = 256, LAG = 128, NSINK = 4, WIN = 256;
constexpr int SUB = 51200;
constexpr int KC_O = 0, VB_O = 32768, VLO_O = 49152, VSC_O = 49664, KLO_O = 50176, KSC_O = 50688;
constexpr int HEADS = 4, DIM = 128, QROWS = 16;

// Status bits written by the device-side range checks (first event wins for the index fields).
constexpr int ST_QPOOL = 1, ST_EPOOL = 2, ST_SINK = 4, ST_TABLE = 8, ST_TIMEOUT = 16;

__device__ __forceinline__ void flag(int* status, int bit) {
    if (status) atomicOr(status, bit);
}

// Programmatic dependent launch (a kernel launched with the programmatic-serialization attribute may start while the
// kernel before it in the stream still runs).  launch_dependents: this CTA allows the next kernel to start launching
// (it does once every CTA of this grid has allowed it or exited, so every CTA of this grid is resident by then).
// wait: block until the kernels this one depends on have completed and their writes are visible; a no-op in a kernel
// launched without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

// Page and slot of position p in pages of ebs tokens, (p / ebs, p % ebs) with C++'s semantics: in 32-bit unsigned
// arithmetic when 0 <= p, ebs < 2^31 (always, for real caches), in 64-bit otherwise.  A 64-bit division by a value
// known only at run time is emulated in software and costs several times the 32-bit one.
__device__ __forceinline__ void page_split(int64_t p, int64_t ebs, int64_t& pg, int64_t& sl) {
    if (((uint64_t)p | (uint64_t)ebs) <= 0x7fffffffull) {
        const uint32_t q = (uint32_t)p / (uint32_t)ebs;
        pg = q;
        sl = (uint32_t)p - q * (uint32_t)ebs;
    } else {
        pg = p / ebs;
        sl = p % ebs;
    }
}

// fp32 -> bf16 bits, round to nearest even (NaN kept quiet).
__device__ __forceinline__ uint16_t f2bf(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float bfround(float f) { return bf2f(f2bf(f)); }

// fp8 e4m3fn byte -> fp32, exact (bias 7, 3 mantissa bits; e = 0 is the subnormal grid m * 2^-9; 0x7f / 0xff NaN).
// The magnitude comes from the hardware e4m3 -> f16 conversion (exact: every e4m3 value is an f16 value) and the
// exact f16 -> f32 widening; the NaN bytes give the canonical quiet NaN and the sign is applied by negation, so -0 and
// the NaN bits are those of the format-definition decoder.
__device__ __forceinline__ float f8dec(uint32_t b) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((unsigned short)(b & 0x7fu)));
    float mag;
    asm("{.reg .f16 l, h;\n\tmov.b32 {l, h}, %1;\n\tcvt.f32.f16 %0, l;\n\t}" : "=f"(mag) : "r"(h2));
    if ((b & 0x7fu) == 0x7fu) mag = __uint_as_float(0x7fc00000u);
    return (b & 0x80u) ? -mag : mag;
}

// fp32 -> fp8 e4m3fn byte with the semantics of torch's non-saturating cast: round to nearest even (subnormals on
// the 2^-9 grid, normals to 3 mantissa bits with a carry into the exponent), magnitudes above 464 (those that would
// round past 448), infinities and NaN -> 0x7f with the sign kept.  The rounding is the hardware's RNE conversion
// (cvt.rn.satfinite, the same value converted into both bytes); it is the cast wherever |f| <= 464, where the result
// is at most 448 and saturation never acts, and the magnitudes above 464 and the NaN take the 0x7f byte explicitly.
__device__ __forceinline__ uint32_t f8enc(float f) {
    unsigned short two;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(two) : "f"(f));
    return (fabsf(f) <= 464.0f) ? (uint32_t)(two & 0xffu) : (((__float_as_uint(f) >> 24) & 0x80u) | 0x7fu);
}

// torch clamp_min(x, 1e-8): NaN propagates.
__device__ __forceinline__ float clamp_min_1e8(float x) { return (x != x) ? x : fmaxf(x, 1e-8f); }

// torch .round().clamp(0, hi).to(uint8) of an fp32 value: half to even, NaN -> 0.
__device__ __forceinline__ uint32_t round_clamp(float x, float hi) {
    if (x != x) return 0u;
    float r = fminf(fmaxf(rintf(x), 0.0f), hi);
    return (uint32_t)r;
}

}  // namespace kv800

// ------------------------------------------------------------------ host side of the C ABI
namespace kv800 {
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
}  // namespace kv800
