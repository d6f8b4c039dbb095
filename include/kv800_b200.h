/*
 * kv800_b200.h -- C ABI of the B200 (sm_100a) implementation of lfm3_kv800's 800h hot path:
 *   the 800h quantizer / flush (256-token sub-blocks of 51,200 bytes: 2-bit pre-RoPE K per channel, 1-bit
 *   Hadamard-rotated V per token, fp8 e4m3 lo / scale) and paged GQA decode attention over those sub-blocks plus the
 *   exact bf16 tail (16 query heads, 4 KV heads, head_dim 128).
 *
 * Conventions (the reference's, lfm3_kv800/kv800.py:1-16):
 *   - every buffer is caller-owned device memory; the library allocates nothing (scratch is passed in);
 *   - pool offsets are int64 and relative to the pool pointer passed in: BOFF in BYTES from `qpool`, EOFF / SKOFF /
 *     SVOFF in bf16 ELEMENTS from `epool` / `sk` / `sv`;
 *   - exact page layout: K of (head h, slot t) at eoff + h*e_hs + t*e_ts, V at + e_v (elements);
 *   - bf16 tensors are passed as uint16_t bit patterns, fp8 bytes as uint8_t;
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream); every call only enqueues work on it;
 *   - return value: KV800_OK or an error code; kv800_last_error() gives a message for the calling host thread.
 * Device-side checks: each kernel compares every page / sub-block offset it reads against the pool extent passed in
 * (bytes / elements) and skips an out-of-range one instead of reading it; the first such event is recorded in the
 * status word of the workspace (decode) or reported through kv800_check_status (see below).
 */
#ifndef KV800_B200_H
#define KV800_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define KV800_API __attribute__((visibility("default")))
#else
#define KV800_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define KV800_OK 0
#define KV800_ERR_ARG 1      /* a null pointer, a negative size, a shape outside the supported set */
#define KV800_ERR_RANGE 2    /* a size above a stated maximum */
#define KV800_ERR_CUDA 3     /* a CUDA runtime error (launch, configuration) */
#define KV800_ERR_DEVICE 4   /* a device-side check fired: an offset outside its pool (see kv800_check_status) */

/* ABI revision of this header (bumped on any signature change). */
KV800_API int kv800_abi_version(void);

/* Message for the last error returned on the calling host thread ("" if none). */
KV800_API const char* kv800_last_error(void);

/* Layout constants (kv800.py:32-34): BLK 256, SUB 51200, LAG 128, NSINK 4, WIN 256. */
KV800_API int kv800_constants(int64_t* blk, int64_t* sub, int64_t* lag, int64_t* nsink, int64_t* win);

/*
 * kv800_quantize_blocks -- replaces kv800.quantize_blocks(k, v, H) (lfm3_kv800/kv800.py:56-76).
 * k, v: (M, 256, 4, 128) bf16, contiguous (pre-RoPE K, unrotated V); out: (M, 51200) u8.  Bit-exact with the
 * reference: K lo / hi over 256 tokens per (head, channel), fp8 lo and (hi - lo) / 3 scale, RNE codes; V rotated by
 * the normalized 128-point Hadamard as a sequential fp32 FMA chain, lo / hi per (token, 2-head group), 1-bit codes.
 */
KV800_API int kv800_quantize_blocks(const uint16_t* k, const uint16_t* v, int64_t M, uint8_t* out, void* stream);

/*
 * kv800_dequantize_blocks -- replaces kv800.dequantize_blocks(sb, H) (lfm3_kv800/kv800.py:79-92).
 * sb: (M, 51200) u8, contiguous; k_out: (M, 256, 4, 128) bf16 = bf16(codes * ksc + klo) (pre-RoPE);
 * v_out: (M, 256, 4, 128) f32 = (bits * vsc + vlo) @ H (unrotated V), the same FMA chain as the quantizer.
 */
KV800_API int kv800_dequantize_blocks(const uint8_t* sb, int64_t M, uint16_t* k_out, float* v_out, void* stream);

/*
 * kv800_fake_quant_k / kv800_fake_quant_v -- replace train.fake_quant_k(x) and train.fake_quant_v(v, H)
 * (lfm3_kv800/train.py:82-100): the cache's quantize -> dequantize round trip on fp32 training activations.
 * fake_quant_k: x (G, 256, C) fp32 (256-token groups on dim 1) -> out (G, 256, C) fp32 = code * sc8 + lo8 per
 * (group, channel).  fake_quant_v: v (N, 4, 128) fp32 -> out (N, 4, 128) fp32 = ((v @ H) quantized to 1 bit per dim
 * over 2-head groups, dequantized) @ H, with the same sequential FMA chain as the quantizer (bit-exact with the
 * reference on CPU).
 */
KV800_API int kv800_fake_quant_k(const float* x, int64_t G, int64_t C, float* out, void* stream);
KV800_API int kv800_fake_quant_v(const float* v, int64_t N, float* out, void* stream);

/*
 * kv800_flush -- replaces the flush of PagedStore.append (kv800.py:433-440) and of the vLLM backend
 * (vllm_attn.py:298-317): for m < M, gather the 256 exact tokens of sub-block blk[m] of sequence seq[m] (positions
 * [256 blk, 256 blk + 256)) from the exact pages, quantize them as kv800_quantize_blocks does, and write the 51,200
 * bytes at qpool + boff[seq * boff_stride + blk].  seq / blk are device int32 arrays of length M; nseq is the
 * number of rows of the eoff / boff tables (0 <= seq < nseq, 0 <= blk < boff_stride are checked on the device).
 * epool_elems / qpool_bytes: pool extents used by the device-side range checks.  status: optional device int
 * (NULL = none) set to nonzero when a range check fires.
 */
KV800_API int kv800_flush(const uint16_t* epool, int64_t epool_elems, const int64_t* eoff, int64_t eoff_stride, int64_t ebs,
                int64_t e_hs, int64_t e_ts, int64_t e_v, uint8_t* qpool, int64_t qpool_bytes, const int64_t* boff,
                int64_t boff_stride, const int32_t* seq, const int32_t* blk, int64_t M, int64_t nseq, int* status,
                void* stream);

/*
 * kv800_flush_step -- the flush of one vLLM step (vllm_attn.py:298-317) without a host loop.  The flush plan is built
 * on the device: request b (seq_lens[b] tokens after the step, query_start_loc[b + 1] - query_start_loc[b] of them new)
 * owns sub-blocks j in [nq(prev), nq(seq_lens[b])), nq(n) = max(0, n - 128) / 256, listed in request order (at most
 * max_pairs; more sets ST_TABLE in *status).  Each listed sub-block is gathered from the exact cache, quantized and
 * written to the quant cache in the same stream.  Replaces the reference's Python plan loop and per-element
 * index tensors (vllm_attn.py:300-317).
 *   exact cache  [blocks, 4, ebs, 256] bf16 with element strides s0 (block), s1 (head), s2 (row); K of (block, head,
 *                row) at blk * s0 + h * s1 + row * s2, V at + 128.  block_table: int32, row stride bt_stride, maps
 *                (request, position / ebs) to a block.
 *   quant cache  pages of qs0 bytes holding bsq / 256 sub-blocks of 51,200 B; qblock_table maps (request, 256 j / bsq)
 *                to a page.
 *   seq_lens, query_start_loc  int32 device arrays (R and R + 1 entries), as vLLM's attention metadata holds them.
 *   workspace    kv800_flush_step_workspace_size(max_pairs) bytes, 256-aligned (holds the plan).
 */
KV800_API int64_t kv800_flush_step_workspace_size(int64_t max_pairs);
KV800_API int kv800_flush_step(const uint16_t* ecache, int64_t ecache_elems, int64_t s0, int64_t s1, int64_t s2,
                               int64_t ebs, const int32_t* block_table, int64_t bt_stride, uint8_t* qcache,
                               int64_t qcache_bytes, int64_t qs0, int64_t bsq, const int32_t* qblock_table,
                               int64_t qbt_stride, const int32_t* seq_lens, const int32_t* query_start_loc, int64_t R,
                               int64_t max_pairs, void* workspace, int64_t workspace_bytes, int* status,
                               void* stream);

/*
 * kv800_write_sinks -- the sink write of a window layer (vllm_attn.py:276-291): token i with positions[i] < 4 (and
 * slot_mapping[i] >= 0) of request b (query_start_loc[b] <= i < query_start_loc[b + 1]) writes its K rows to
 * hk + hk_bt[b * hk_bts] * hk_s0 + hk_aux + (p * 4 + h) * 128 and its V rows likewise into hv (bf16 views of the two
 * host layers' quant caches; aux = the element offset of the page padding).  Out-of-range rows set ST_SINK.
 */
KV800_API int kv800_write_sinks(uint16_t* hk, int64_t hk_elems, int64_t hk_s0, int64_t hk_aux, const int32_t* hk_bt,
                                int64_t hk_bts, uint16_t* hv, int64_t hv_elems, int64_t hv_s0, int64_t hv_aux,
                                const int32_t* hv_bt, int64_t hv_bts, const uint16_t* k, const uint16_t* v,
                                const int64_t* positions, const int64_t* slot_mapping, const int32_t* query_start_loc,
                                int64_t R, int64_t T, int* status, void* stream);

/*
 * kv800_decode_tables -- the decode inputs of the first nd requests of a vLLM step (vllm_attn.py:320-349) in one
 * launch: N = seq_lens, NQ = max(0, N - 128) / 256 (0 when qblock_table is null), eoff[b, c] = block_table[b, c] * s0
 * ([nd, bt_stride] int64), boff[b, j] = qblock_table[b, 256 j / bsq] * qs0 + ((256 j % bsq) / 256) * 51200 for
 * j < NQ[b] and 0 beyond ([nd, nqw] int64), and for window layers skoff / svoff = host_bt[b, 0] * s0 + aux (pass null
 * to skip).
 */
KV800_API int kv800_decode_tables(const int32_t* seq_lens, int64_t nd, const int32_t* block_table, int64_t bt_stride,
                                  int64_t s0, int32_t* N, int32_t* NQ, int64_t* eoff, const int32_t* qblock_table,
                                  int64_t qbt_stride, int64_t qs0, int64_t bsq, int64_t nqw, int64_t* boff,
                                  const int32_t* sk_bt, int64_t sk_bts, int64_t sk_s0, int64_t sk_aux, int64_t* skoff,
                                  const int32_t* sv_bt, int64_t sv_bts, int64_t sv_s0, int64_t sv_aux, int64_t* svoff,
                                  void* stream);

/*
 * kv800_prefill_kv -- the K / V a prefill or extend request attends to, in position order (vllm_attn.py:355-388):
 * sub-blocks j < nqp dequantized from the quant cache (qbt_row: the request's quant block-table row), ns <= 4 sink
 * rows (sk / sv: (ns, 4, 128) bf16), exact rows of positions [lo, n0) from the exact cache (bt_row), and the chunk k / v
 * ((n - n0, 4, 128) bf16, positions n0 .. n - 1).  K is rotated with the [npos, 32] bf16 cos / sin tables (HF RoPE in
 * the reference's fp32 operation order, then bf16) unless cos_t and sin_t are null (native sliding layers); V is bf16.
 * k_out / v_out: (256 nqp + ns + (n0 - lo) + (n - n0), 4, 128) bf16.  Bit-identical to the reference's
 * dequantize_blocks + cat + _rope + bf16 casts.
 */
KV800_API int kv800_prefill_kv(const uint8_t* qcache, int64_t qcache_bytes, int64_t qs0, int64_t bsq,
                               const int32_t* qbt_row, int64_t qbt_len, int64_t nqp, const uint16_t* sk,
                               const uint16_t* sv, int64_t ns, const uint16_t* ecache, int64_t ecache_elems, int64_t s0,
                               int64_t s1, int64_t s2, int64_t ebs, const int32_t* bt_row, int64_t bt_len, int64_t lo,
                               int64_t n0, const uint16_t* k, const uint16_t* v, int64_t n, const uint16_t* cos_t,
                               const uint16_t* sin_t, int64_t npos, uint16_t* k_out, uint16_t* v_out, int* status,
                               void* stream);

/*
 * kv800_write_slots -- the exact-cache write of a vLLM step (vllm_attn.py:261-269): token i of k / v ((T, 4, 128)
 * bf16) goes to block slot_mapping[i] / ebs, row slot_mapping[i] % ebs of the [blocks, 4, ebs, 256] cache (element
 * strides s0, s1, s2; K at + 0, V at + 128); negative slots (padding) are skipped.
 */
KV800_API int kv800_write_slots(uint16_t* ecache, int64_t ecache_elems, int64_t s0, int64_t s1, int64_t s2,
                                int64_t ebs, const uint16_t* k, const uint16_t* v, const int64_t* slot_mapping,
                                int64_t T, int* status, void* stream);

/*
 * kv800_write_exact -- replaces the exact-page scatter of PagedStore.append (kv800.py:423-428) and of the vLLM
 * backend (vllm_attn.py:261-269): token i (i < T) of k / v ((T, 4, 128) bf16, contiguous) goes to sequence seq[i],
 * position pos[i]: K at epool + eoff[seq * eoff_stride + pos / ebs] + h*e_hs + (pos % ebs)*e_ts, V at + e_v.
 * seq (int32) and pos (int64) are device arrays of length T.
 */
KV800_API int kv800_write_exact(uint16_t* epool, int64_t epool_elems, const int64_t* eoff, int64_t eoff_stride, int64_t ebs,
                      int64_t e_hs, int64_t e_ts, int64_t e_v, const uint16_t* k, const uint16_t* v,
                      const int32_t* seq, const int64_t* pos, int64_t T, int64_t nseq, int* status, void* stream);

/*
 * Paged decode.  The record below carries the reference's Paged slots (kv800.py:239-248); pointers are device
 * pointers.  sk / sv / skoff / svoff may be NULL (no sinks).  win = 0: quantized layer, sub-blocks j < min(NQ[b],
 * nqmax) plus exact positions [256 NQ[b], N[b]); win > 0: window layer, exact positions [max(256 NQ[b], N[b] - win),
 * N[b]) plus the sinks (positions < min(nsink, lo, N[b])) when sk is set.  The quantized kernel reads sub-blocks by
 * TMA: qpool must start 16-byte aligned and BOFF entries be multiples of 128 (the reference's layouts use multiples
 * of 51,200); a sub-block at another offset is skipped and flagged in the status word.
 */
typedef struct kv800_paged {
    const uint8_t* qpool; int64_t qpool_bytes;
    const int64_t* boff; int64_t boff_stride;
    const uint16_t* epool; int64_t epool_elems;
    const int64_t* eoff; int64_t eoff_stride;
    int64_t ebs, e_hs, e_ts, e_v;
    const uint16_t* sk; const uint16_t* sv; int64_t sk_elems, sv_elems;
    const int64_t* skoff; const int64_t* svoff;
    const int32_t* N; const int32_t* NQ;
    int64_t nqmax;          /* host bound >= max(NQ) (the reference's host int) */
    int64_t win;            /* 0 or the window (256) */
    int64_t nsink;          /* sinks read when win > 0 and sk != NULL (the reference's NSINK = 4) */
} kv800_paged;

/*
 * kv800_decode -- replaces kv800.decode(P, q, cos_t, sin_t, H, spb, target) (kv800.py:330-383) with one CUDA
 * backend.  q: (B, 16, 128) bf16 post-RoPE; cos_t / sin_t: (npos, 32) bf16 tables of the 32 rotating frequency pairs
 * (dims d and d + 64 share frequency d, d < 32), or both NULL for a layer without quantized sub-blocks whose keys
 * need no rotation (native sliding layers); out: (B, 16, 128) bf16.  spb: sub-blocks per split (<= 0: chosen by
 * the library).  workspace: device scratch of kv800_decode_workspace_size(...) bytes, 256-byte aligned, any
 * contents (the decode clears what it needs); its first int is the device status word (0 = clean; set when a range
 * check fires).
 */
KV800_API int64_t kv800_decode_workspace_size(int64_t B, int64_t nqmax, int64_t win, int64_t spb);
KV800_API int kv800_decode(const kv800_paged* P, const uint16_t* q, const uint16_t* cos_t, const uint16_t* sin_t,
                 int64_t npos, int64_t B, int64_t spb, uint16_t* out, void* workspace, int64_t workspace_bytes,
                 void* stream);

/*
 * kv800_decode_noalloc -- has no counterpart in the reference.  The same decode as kv800_decode for callers that
 * cannot allocate device memory when they decode (an engine that budgets all GPU memory in advance, a host whose
 * allocator is out of reach on the decode thread), so they cannot pass a workspace.  The scratch is a 16 MiB array
 * inside the library (held on every GPU that loads it until exit); a decode that needs more (see
 * kv800_decode_workspace_size) is rejected with KV800_ERR_RANGE.  The first call on a device looks the array up
 * with that device current, so make it before any stream capture.  All calls share the array: calls that may run
 * at the same time on the GPU race and must be serialized by the caller.  The device range checks write their
 * status word into the array; read it with kv800_decode_noalloc_status.  Allocates nothing.
 */
KV800_API int kv800_decode_noalloc(const kv800_paged* P, const uint16_t* q, const uint16_t* cos_t,
                                   const uint16_t* sin_t, int64_t npos, int64_t B, int64_t spb, uint16_t* out,
                                   void* stream);

/*
 * kv800_decode_noalloc_status -- has no counterpart in the reference.  The device status word of the last
 * kv800_decode_noalloc call on the current device (it lives in the built-in scratch array, out of the caller's
 * reach): copies it to *host_value after synchronizing `stream`; returns KV800_ERR_DEVICE when a range check fired.
 */
KV800_API int kv800_decode_noalloc_status(int* host_value, void* stream);

/*
 * kv800_decode_timed -- has no counterpart in the reference: kv800_decode with CUDA events around its phases, for
 * benchmarks.  Blocks until the decode is done and writes ms[0] = the quantized partials (schedule + qdecode_mma),
 * ms[1] = the exact partials together with the merge of each row's partials, which the last exact-partial CTA of
 * each row (or (row, head)) performs, ms[2] = the gap after it (about zero), in milliseconds of device time.  A phase with no work
 * reports the gap between its two events (about zero).
 */
KV800_API int kv800_decode_timed(const kv800_paged* P, const uint16_t* q, const uint16_t* cos_t,
                                 const uint16_t* sin_t, int64_t npos, int64_t B, int64_t spb, uint16_t* out,
                                 void* workspace, int64_t workspace_bytes, void* stream, float* ms);

/*
 * The reference's three native decode ops (kv800::qdecode / xdecode / combine, csrc/kv800_sycl.sycl:554-561) with
 * the same argument meaning and partial layout: MO / LO (B, ns + 1, 16) f32, AO (B, ns + 1, 16, 128) f32; slots
 * [0, ns) are the quantized splits (V accumulated in the Hadamard domain), slot ns the sinks + exact tokens.
 * scale = 128^-0.5 * log2(e).  combine writes (B, 16, 128) bf16 into out.
 */
KV800_API int kv800_qdecode(const uint16_t* q, const uint8_t* qpool, int64_t qpool_bytes, const int64_t* boff,
                  int64_t boff_stride, const int32_t* NQ, const uint16_t* cos_t, const uint16_t* sin_t, int64_t npos,
                  float* mo, float* lo, float* ao, int64_t B, int64_t ns, int64_t spb, int64_t nqmax, float scale,
                  int* status, void* stream);
KV800_API int kv800_xdecode(const uint16_t* q, const kv800_paged* P, const uint16_t* cos_t, const uint16_t* sin_t,
                  int64_t npos, float* mo, float* lo, float* ao, int64_t B, int64_t ns, float scale, int* status,
                  void* stream);
KV800_API int kv800_combine(const float* mo, const float* lo, const float* ao, int64_t B, int64_t ns, uint16_t* out,
                  void* stream);

/* Copy the device status word at `status` to *host_value (synchronizes the stream). */
KV800_API int kv800_check_status(const int* status, int* host_value, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KV800_B200_H */
