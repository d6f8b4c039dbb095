/*
 * kv800_oracle.c -- CPU restatement of the lfm3_kv800 800h hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA library in lfm3-kv800_b200/csrc.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may load it.  The product path never
 * calls it and has no CPU fallback.
 *
 * Every function restates the reference (riceharvest/lfm3-kv800 v0.1.1, Python/torch) in plain C, with the same
 * fp32 rounding steps where the packed bytes depend on them:
 *   - quantizer           lfm3_kv800/kv800.py:56-76   (quantize_blocks)
 *   - dequantizer         lfm3_kv800/kv800.py:79-92   (dequantize_blocks)
 *   - paged decode        lfm3_kv800/torch_decode.py:16-80
 *   - split combine       lfm3_kv800/kv800.py:231-236 (H applied to the quantized sum)
 *   - paged flush         lfm3_kv800/kv800.py:433-440 (PagedStore.append) and lfm3_kv800/vllm_attn.py:298-317
 * Parity of this file with the reference itself is pinned by tests/golden (fixtures made by importing the reference).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  Contraction must stay off: the reference rounds
 * every torch elementwise op separately, and the only fused multiply-adds are the explicit fmaf() calls below.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BLK 256
#define SUB 51200
#define KC_O 0
#define VB_O 32768
#define VLO_O 49152
#define VSC_O 49664
#define KLO_O 50176
#define KSC_O 50688
#define NSINK 4

/* ------------------------------------------------------------------ scalar formats */
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf16_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* fp32 -> bf16, round to nearest even (torch's Tensor.to(bfloat16)); NaN kept quiet. */
static inline uint16_t f32_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf16_round(float f) { return bf16_f32(f32_bf16(f)); }

/* fp32 -> fp8 e4m3fn, written from the format definition (bias 7, 3 mantissa bits, no infinities, 0x7f = NaN):
 * round to nearest even; magnitudes that round above 448 (i.e. > 464), infinities and NaN give 0x7f; the sign bit
 * is kept.  This is what torch's Tensor.to(float8_e4m3fn) does (non-saturating cast), as used at kv800.py:62,70. */
uint8_t orc_f8_encode(float f) {
    uint32_t u = f32_bits(f);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    uint32_t a = u & 0x7fffffffu;
    float af = bits_f32(a);
    if (a > 0x7f800000u || !(af <= 464.0f)) return (uint8_t)(sign | 0x7fu);   /* NaN, inf, overflow */
    if (af < 0.015625f) {                                                       /* below 2^-6: subnormal grid 2^-9 */
        float m = rintf(af * 512.0f);                                          /* exact scaling, RNE */
        return (uint8_t)(sign | (uint8_t)m);                                   /* m == 8 is the min normal 0x08 */
    }
    uint32_t r = a + 0x7ffffu + ((a >> 20) & 1u);                              /* RNE to 3 mantissa bits */
    int e = (int)(r >> 23) - 127 + 7;
    uint32_t m = (r >> 20) & 7u;
    return (uint8_t)(sign | (uint8_t)(e << 3) | (uint8_t)m);
}

/* fp8 e4m3fn -> fp32 (exact).  0x7f / 0xff decode to NaN. */
float orc_f8_decode(uint8_t b) {
    uint32_t e = (b >> 3) & 15u, m = b & 7u;
    float mag;
    if (e == 15u && m == 7u) mag = NAN;
    else if (e == 0u) mag = (float)m * 0.001953125f;
    else mag = bits_f32(((e + 120u) << 23) | (m << 20));
    return (b & 0x80u) ? -mag : mag;
}

/* torch's clamp_min(x, 1e-8) on fp32: NaN propagates (fmaxf would not). */
static inline float clamp_min_1e8(float x) { return (x != x) ? x : (x < 1e-8f ? 1e-8f : x); }

/* torch .round().clamp(0, hi).to(uint8): round half to even, NaN -> 0 (x86 float->uint8 cast of NaN). */
static inline uint8_t round_clamp_u8(float x, float hi) {
    if (x != x) return 0;
    float r = rintf(x);
    if (r < 0.f) r = 0.f;
    if (r > hi) r = hi;
    return (uint8_t)r;
}

/* The normalized Sylvester Hadamard entry H[i][d] = (+-1) / sqrt(128) in fp32 (kv800.py:43-46): sign is the parity
 * of popcount(i & d); the magnitude is fp32(1) / fp32(sqrt(128)) = 0x3db504f3. */
static inline float had(int i, int d) {
    static const float c = 0.0883883461356163f;
    return (__builtin_popcount((unsigned)(i & d)) & 1) ? -c : c;
}

/* ------------------------------------------------------------------ quantizer (kv800.py:56-76) */
/* k, v: [256][4][128] bf16 (pre-RoPE K, unrotated V) of one sub-block; out: 51,200 bytes. */
static void quantize_one(const uint16_t* k, const uint16_t* v, uint8_t* out) {
    /* K: per (head, channel) lo/hi over the 256 tokens, fp8 lo and scale (hi-lo)/3, 2-bit codes, planar packing */
    static __thread uint8_t codes[BLK * 512];
    for (int c = 0; c < 512; c++) {
        float lo = INFINITY, hi = -INFINITY;
        for (int t = 0; t < BLK; t++) {
            float x = bf16_f32(k[t * 512 + c]);
            lo = x < lo ? x : lo;
            hi = x > hi ? x : hi;
        }
        uint8_t lo8 = orc_f8_encode(lo);
        uint8_t sc8 = orc_f8_encode(clamp_min_1e8((hi - lo) / 3.0f));
        float lof = orc_f8_decode(lo8), scf = clamp_min_1e8(orc_f8_decode(sc8));
        for (int t = 0; t < BLK; t++) {
            float x = bf16_f32(k[t * 512 + c]);
            codes[t * 512 + c] = round_clamp_u8((x - lof) / scf, 3.0f);
        }
        out[KLO_O + c] = lo8;
        out[KSC_O + c] = sc8;
    }
    for (int t = 0; t < BLK; t++)
        for (int h = 0; h < 4; h++)
            for (int j = 0; j < 32; j++) {
                const uint8_t* cc = codes + t * 512 + h * 128;
                out[KC_O + (t * 4 + h) * 32 + j] =
                    (uint8_t)(cc[j] | (cc[j + 32] << 2) | (cc[j + 64] << 4) | (cc[j + 96] << 6));
            }
    /* V: y = v @ H per head (fp32, sequential FMA chain over i, which is what the CPU BLAS computes for this shape),
     * per (token, 2-head group) lo/hi over 256 dims, fp8 lo and scale hi-lo, 1-bit codes, planar packing */
    for (int t = 0; t < BLK; t++) {
        float y[512];
        for (int h = 0; h < 4; h++)
            for (int d = 0; d < 128; d++) {
                float acc = 0.0f;
                for (int i = 0; i < 128; i++) acc = fmaf(bf16_f32(v[t * 512 + h * 128 + i]), had(i, d), acc);
                y[h * 128 + d] = acc;
            }
        uint8_t bits[512];
        for (int g = 0; g < 2; g++) {
            float lo = INFINITY, hi = -INFINITY;
            for (int e = 0; e < 256; e++) {
                float x = y[g * 256 + e];
                lo = x < lo ? x : lo;
                hi = x > hi ? x : hi;
            }
            uint8_t lo8 = orc_f8_encode(lo);
            uint8_t sc8 = orc_f8_encode(clamp_min_1e8(hi - lo));
            float lof = orc_f8_decode(lo8), scf = clamp_min_1e8(orc_f8_decode(sc8));
            for (int e = 0; e < 256; e++) bits[g * 256 + e] = round_clamp_u8((y[g * 256 + e] - lof) / scf, 1.0f);
            out[VLO_O + t * 2 + g] = lo8;
            out[VSC_O + t * 2 + g] = sc8;
        }
        for (int h = 0; h < 4; h++)
            for (int j = 0; j < 16; j++) {
                unsigned byte = 0;
                for (int i = 0; i < 8; i++) byte |= (unsigned)bits[h * 128 + j + 16 * i] << i;
                out[VB_O + (t * 4 + h) * 16 + j] = (uint8_t)byte;
            }
    }
}

/* quantize_blocks(k, v, H): k, v (M, 256, 4, 128) bf16 -> (M, 51200) u8.  kv800.py:56 */
void orc_quantize_blocks(const uint16_t* k, const uint16_t* v, int64_t M, uint8_t* out, int nthreads) {
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(dynamic, 1)
    for (int64_t m = 0; m < M; m++)
        quantize_one(k + m * (int64_t)BLK * 512, v + m * (int64_t)BLK * 512, out + m * (int64_t)SUB);
}

/* dequantize_blocks(sb, H): K (M,256,4,128) bf16 = bf16(codes * ksc + klo) (mul, add, round: kv800.py:83-86);
 * V (M,256,4,128) fp32 = (bits * vsc + vlo) @ H (kv800.py:87-91).  v_hd (optional) gets the Hadamard-domain values
 * bits * vsc + vlo before the rotation. */
void orc_dequantize_blocks(const uint8_t* sb, int64_t M, uint16_t* k_out, float* v_out, float* v_hd) {
    for (int64_t m = 0; m < M; m++) {
        const uint8_t* s = sb + m * (int64_t)SUB;
        for (int t = 0; t < BLK; t++)
            for (int h = 0; h < 4; h++) {
                const uint8_t* kc = s + KC_O + (t * 4 + h) * 32;
                const uint8_t* vb = s + VB_O + (t * 4 + h) * 16;
                float vlo = orc_f8_decode(s[VLO_O + t * 2 + h / 2]), vsc = orc_f8_decode(s[VSC_O + t * 2 + h / 2]);
                float y[128];
                for (int d = 0; d < 128; d++) {
                    int code = (kc[d & 31] >> (2 * (d >> 5))) & 3;
                    float ksc = orc_f8_decode(s[KSC_O + h * 128 + d]), klo = orc_f8_decode(s[KLO_O + h * 128 + d]);
                    float prod = (float)code * ksc;
                    float kv = prod + klo;
                    int64_t o = ((m * BLK + t) * 4 + h) * 128 + d;
                    if (k_out) k_out[o] = f32_bf16(kv);
                    int bit = (vb[d & 15] >> (d >> 4)) & 1;
                    float bp = (float)bit * vsc;
                    y[d] = bp + vlo;
                    if (v_hd) v_hd[o] = y[d];
                }
                if (v_out)
                    for (int d = 0; d < 128; d++) {
                        float acc = 0.0f;
                        for (int i = 0; i < 128; i++) acc = fmaf(y[i], had(i, d), acc);
                        v_out[((m * BLK + t) * 4 + h) * 128 + d] = acc;
                    }
            }
    }
}

/* ------------------------------------------------------------------ paged flush (kv800.py:433-440) */
/* For each listed (sequence b, sub-block j): gather the 256 exact tokens of positions [256 j, 256 j + 256) from the
 * exact pages (K of head h, slot t at eoff[b][p / ebs] + h*e_hs + (p % ebs)*e_ts; V at + e_v), quantize, and write
 * the 51,200 bytes at qpool + boff[b][j]. */
void orc_flush(const uint16_t* epool, const int64_t* eoff, int64_t eoff_stride, int64_t ebs, int64_t e_hs,
               int64_t e_ts, int64_t e_v, uint8_t* qpool, const int64_t* boff, int64_t boff_stride,
               const int32_t* seq, const int32_t* blk, int64_t M, int nthreads) {
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(dynamic, 1)
    for (int64_t m = 0; m < M; m++) {
        uint16_t* kk = (uint16_t*)malloc(sizeof(uint16_t) * BLK * 512 * 2);
        uint16_t* vv = kk + BLK * 512;
        int64_t b = seq[m], j = blk[m];
        for (int t = 0; t < BLK; t++) {
            int64_t p = j * BLK + t;
            int64_t page = eoff[b * eoff_stride + p / ebs];
            for (int h = 0; h < 4; h++) {
                int64_t o = page + h * e_hs + (p % ebs) * e_ts;
                memcpy(kk + (t * 4 + h) * 128, epool + o, 256);
                memcpy(vv + (t * 4 + h) * 128, epool + o + e_v, 256);
            }
        }
        quantize_one(kk, vv, qpool + boff[b * boff_stride + j]);
        free(kk);
    }
}

/* ------------------------------------------------------------------ paged decode (torch_decode.py:27-80) */
/* RoPE of one pre-RoPE key row (torch_decode.py:16-24): dims (d, d + 64), d < 32, rotated in fp32 with separately
 * rounded mul / mul / sub (add), then the whole row is rounded to bf16. */
static inline void rope_row(const float* k, const uint16_t* cs_row, const uint16_t* sn_row, float* kr) {
    for (int d = 0; d < 128; d++) kr[d] = k[d];
    for (int d = 0; d < 32; d++) {
        float cs = bf16_f32(cs_row[d]), sn = bf16_f32(sn_row[d]);
        float k0 = k[d], k2 = k[d + 64];
        float a = k0 * cs, b = k2 * sn, c = k2 * cs, e = k0 * sn;
        kr[d] = a - b;
        kr[d + 64] = c + e;
    }
    for (int d = 0; d < 128; d++) kr[d] = bf16_round(kr[d]);
}

/*
 * One decode of the reference's kv800.decode(P, q, cos_t, sin_t, H) with torch_decode semantics, for every row b:
 *   quantized layer (win == 0): sub-blocks j < min(NQ[b], nqmax) from qpool + boff[b][j]; exact [256 NQ[b], n)
 *   window layer (win > 0): exact [max(256 NQ[b], n - win), n) + sinks (positions < min(4, lo, n)) when sk != NULL
 * q (B, 16, 128) bf16 post-RoPE; cos/sin (P, 32) bf16; out (B, 16, 128) bf16.  Quantized V is accumulated in the
 * Hadamard domain and rotated once per row (the reference kernels' order, kv800.py:235); the reference torch path
 * rotates per token first, which differs only by fp32 rounding.
 */
void orc_decode(const uint8_t* qpool, const int64_t* boff, int64_t boff_stride, const uint16_t* epool,
                const int64_t* eoff, int64_t eoff_stride, int64_t ebs, int64_t e_hs, int64_t e_ts, int64_t e_v,
                const uint16_t* sk, const uint16_t* sv, const int64_t* skoff, const int64_t* svoff,
                const int32_t* N, const int32_t* NQ, int64_t nqmax, int64_t win, const uint16_t* q,
                const uint16_t* cos_t, const uint16_t* sin_t, int64_t B, uint16_t* out, int nthreads) {
    const float scale = 0.08838834764831845f;   /* 128 ** -0.5 */
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(dynamic, 1)
    for (int64_t bh = 0; bh < B * 4; bh++) {
        int64_t b = bh / 4;
        int h = (int)(bh % 4);
        int64_t n = N[b], nqb = NQ[b];
        int64_t nq = win ? 0 : (nqb < nqmax ? nqb : nqmax);
        if (nq < 0) nq = 0;
        int64_t lo = nqb * BLK;
        if (win && n - win > lo) lo = n - win;
        int64_t cnt = 0;
        if (win && sk) {
            cnt = NSINK;
            if (lo < cnt) cnt = lo;
            if (n < cnt) cnt = n;
            if (cnt < 0) cnt = 0;
        }
        int64_t nex = n > lo ? n - lo : 0;
        int64_t S = nq * BLK + cnt + nex;
        float qf[4][128];
        for (int r = 0; r < 4; r++)
            for (int d = 0; d < 128; d++) qf[r][d] = bf16_f32(q[(b * 16 + h * 4 + r) * 128 + d]);
        if (S == 0) {
            for (int r = 0; r < 4; r++)
                for (int d = 0; d < 128; d++) out[(b * 16 + h * 4 + r) * 128 + d] = 0;
            continue;
        }
        float* sc = (float*)malloc(sizeof(float) * 4 * S);
        float kraw[128], kr[128];
        /* pass 1: scores */
        for (int64_t s = 0; s < S; s++) {
            int64_t pos;
            if (s < nq * BLK) {
                int64_t j = s / BLK, t = s % BLK;
                const uint8_t* sb = qpool + boff[b * boff_stride + j];
                const uint8_t* kc = sb + KC_O + (t * 4 + h) * 32;
                for (int d = 0; d < 128; d++) {
                    int code = (kc[d & 31] >> (2 * (d >> 5))) & 3;
                    float prod = (float)code * orc_f8_decode(sb[KSC_O + h * 128 + d]);
                    kraw[d] = bf16_round(prod + orc_f8_decode(sb[KLO_O + h * 128 + d]));
                }
                pos = s;
            } else if (s < nq * BLK + cnt) {
                int64_t t = s - nq * BLK;
                for (int d = 0; d < 128; d++) kraw[d] = bf16_f32(sk[skoff[b] + (t * 4 + h) * 128 + d]);
                pos = t;
            } else {
                pos = lo + (s - nq * BLK - cnt);
                int64_t o = eoff[b * eoff_stride + pos / ebs] + h * e_hs + (pos % ebs) * e_ts;
                for (int d = 0; d < 128; d++) kraw[d] = bf16_f32(epool[o + d]);
            }
            rope_row(kraw, cos_t + pos * 32, sin_t + pos * 32, kr);
            for (int r = 0; r < 4; r++) {
                float acc = 0.0f;
                for (int d = 0; d < 128; d++) acc += qf[r][d] * kr[d];
                sc[r * S + s] = acc * scale;
            }
        }
        /* softmax over all positions (fp32) */
        for (int r = 0; r < 4; r++) {
            float mx = -INFINITY, sum = 0.0f;
            for (int64_t s = 0; s < S; s++) mx = sc[r * S + s] > mx ? sc[r * S + s] : mx;
            for (int64_t s = 0; s < S; s++) {
                float e = expf(sc[r * S + s] - mx);
                sc[r * S + s] = e;
                sum += e;
            }
            for (int64_t s = 0; s < S; s++) sc[r * S + s] = sc[r * S + s] / sum;
        }
        /* pass 2: P @ V; quantized V in the Hadamard domain, rotated once */
        float accq[4][128], acce[4][128];
        memset(accq, 0, sizeof accq);
        memset(acce, 0, sizeof acce);
        for (int64_t s = 0; s < S; s++) {
            if (s < nq * BLK) {
                int64_t j = s / BLK, t = s % BLK;
                const uint8_t* sb = qpool + boff[b * boff_stride + j];
                const uint8_t* vb = sb + VB_O + (t * 4 + h) * 16;
                float vlo = orc_f8_decode(sb[VLO_O + t * 2 + h / 2]), vsc = orc_f8_decode(sb[VSC_O + t * 2 + h / 2]);
                for (int d = 0; d < 128; d++) {
                    int bit = (vb[d & 15] >> (d >> 4)) & 1;
                    float y = (float)bit * vsc + vlo;
                    for (int r = 0; r < 4; r++) accq[r][d] += sc[r * S + s] * y;
                }
            } else {
                const uint16_t* vr;
                if (s < nq * BLK + cnt) {
                    int64_t t = s - nq * BLK;
                    vr = sv + svoff[b] + (t * 4 + h) * 128;
                } else {
                    int64_t pos = lo + (s - nq * BLK - cnt);
                    vr = epool + eoff[b * eoff_stride + pos / ebs] + h * e_hs + (pos % ebs) * e_ts + e_v;
                }
                for (int d = 0; d < 128; d++) {
                    float vv = bf16_f32(vr[d]);
                    for (int r = 0; r < 4; r++) acce[r][d] += sc[r * S + s] * vv;
                }
            }
        }
        for (int r = 0; r < 4; r++)
            for (int d = 0; d < 128; d++) {
                float rot = 0.0f;
                if (nq)
                    for (int i = 0; i < 128; i++) rot = fmaf(accq[r][i], had(i, d), rot);
                out[(b * 16 + h * 4 + r) * 128 + d] = f32_bf16(acce[r][d] + rot);
            }
        free(sc);
    }
}

/* ------------------------------------------------------------------ training fake quant (train.py:82-100) */
/* fake_quant_k: x (G, 256, C) fp32 -> out: per (group, channel) lo / hi over the 256 tokens, lo8 = fp8(lo),
 * sc8 = fp8(max((hi - lo) / 3, 1e-8)), code = clamp(round((x - lo8) / max(sc8, 1e-8)), 0, 3), out = code * sc8 + lo8. */
void orc_fake_quant_k(const float* x, int64_t G, int64_t C, float* out, int nthreads) {
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(static)
    for (int64_t gc = 0; gc < G * C; gc++) {
        int64_t g = gc / C, c = gc % C;
        const float* col = x + g * BLK * C + c;
        float lo = INFINITY, hi = -INFINITY;
        for (int t = 0; t < BLK; t++) {
            float v = col[(int64_t)t * C];
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        float lof = orc_f8_decode(orc_f8_encode(lo));
        float scq = orc_f8_decode(orc_f8_encode(clamp_min_1e8((hi - lo) / 3.0f)));
        float scf = clamp_min_1e8(scq);
        for (int t = 0; t < BLK; t++) {
            float v = col[(int64_t)t * C];
            float code = (float)round_clamp_u8((v - lof) / scf, 3.0f);
            float prod = code * scq;
            out[g * BLK * C + (int64_t)t * C + c] = prod + lof;
        }
    }
}

/* fake_quant_v: v (N, 4, 128) fp32 -> ((v @ H) 1-bit quantized over 2-head groups of 256 dims, fp8 lo and scale
 * hi - lo, dequantized) @ H; both products as the sequential fp32 FMA chain. */
void orc_fake_quant_v(const float* v, int64_t N, float* out, int nthreads) {
#pragma omp parallel for num_threads(nthreads > 0 ? nthreads : 1) schedule(static)
    for (int64_t t = 0; t < N; t++) {
        const float* row = v + t * 512;
        float y[512], yq[512];
        for (int h = 0; h < 4; h++)
            for (int d = 0; d < 128; d++) {
                float acc = 0.0f;
                for (int i = 0; i < 128; i++) acc = fmaf(row[h * 128 + i], had(i, d), acc);
                y[h * 128 + d] = acc;
            }
        for (int g = 0; g < 2; g++) {
            float lo = INFINITY, hi = -INFINITY;
            for (int e = 0; e < 256; e++) {
                float x = y[g * 256 + e];
                lo = x < lo ? x : lo;
                hi = x > hi ? x : hi;
            }
            float lof = orc_f8_decode(orc_f8_encode(lo));
            float scq = orc_f8_decode(orc_f8_encode(clamp_min_1e8(hi - lo)));
            float scf = clamp_min_1e8(scq);
            for (int e = 0; e < 256; e++) {
                float bit = (float)round_clamp_u8((y[g * 256 + e] - lof) / scf, 1.0f);
                float prod = bit * scq;
                yq[g * 256 + e] = prod + lof;
            }
        }
        for (int h = 0; h < 4; h++)
            for (int d = 0; d < 128; d++) {
                float acc = 0.0f;
                for (int i = 0; i < 128; i++) acc = fmaf(yq[h * 128 + i], had(i, d), acc);
                out[t * 512 + h * 128 + d] = acc;
            }
    }
}

/* fp32 -> fp8 over an array (checks the encoder against torch on CPU). */
void orc_f8_encode_array(const float* x, int64_t n, uint8_t* out) {
    for (int64_t i = 0; i < n; i++) out[i] = orc_f8_encode(x[i]);
}

int orc_abi_version(void) { return 1; }
