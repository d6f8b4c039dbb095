// Exact-token decode partial, tensor-map form (sm_100a), for exact pools in the reference's page layout: a page of
// ebs slots holds, per kv head, ebs rows of 512 bytes (K dims 0..127 then V dims 0..127), so e_ts = 256, e_v = 128,
// e_hs a multiple of 256 and every page offset a multiple of 256 elements (kv800.py:387-441; vLLM's exact cache, the
// (blocks, 4, ebs, 256) tensor of vllm_attn.py).  The pool is then a 2-D tensor of 512-byte rows, and the rows of 16
// consecutive slots of one page and head are one box per 128-byte quarter of the row.
//
//   work     one warp per CTA, CTA (b, e, h) = row b, split e, kv head h: the warps of a row share nothing, so no
//            warp ever waits for another; each issues its own copies.
//   tiles    16-position groups [16 j, 16 j + 16) that meet the row's exact range [lo_e, n).  With ebs a multiple of
//            16 a group never crosses a page; slots outside the range are masked.  Split e of nx takes the tiles
//            [e T / nx, (e + 1) T / nx) of the row's T; split 0 also takes the sinks (at most 16) as one more tile.
//   tables   the page rows of a CTA's first XT_TAB tiles are looked up once, one per lane, at the start.
//   copies   lane 0 issues, per tile, 4 TMA boxes (the head's 4 quarters, 16 rows x 128 bytes, 128-byte swizzle) and
//            the tile's cos / sin rows (one bulk copy each) into an S-stage ring, one mbarrier per stage.  Rows past
//            the pool read as zeros (the tensor map's bounds); a tile whose page fails the checks gets no copies.
//            A page whose offset is not a multiple of 256 elements (but keeps the rows 16-byte aligned, all the
//            gather form needs) is not on the tensor's row grid: the warp loads that tile's rows with plain 16-byte
//            loads instead, so every page table the gather form accepts gives the same result here.
//   compute  xm_tile on the swizzled rows: 16-byte unit u of row r of a quarter sits at unit u ^ (r & 7), so the 8
//            rows an ldmatrix reads fall in 8 different bank groups.  V rows of masked slots are zeroed first (their
//            scores are masked by selection, but 0 x NaN would reach the PV sums).
//   sinks    the head's sink rows (separate pools, (token, head) rows of 128 elements) are loaded with plain loads
//            into the swizzled layout of the stage the sink tile uses.
//   merge    the partial goes to the row's slot (this head's 4 query rows); the last of the nx CTAs of (row, head) to
//            finish merges that head's rows of all the row's partials (per-(row, head) arrival counters).
#pragma once
#include "xdecode_mma.cuh"

namespace kv800 {

struct XTArgs {
    CUtensorMap tm;    // epool as rows of 256 bf16: dims {256, rows}, box {64, 16}, 128-byte swizzle
    XMArgs x;
    int64_t ehs_rows;  // e_hs / 256: rows between the heads of a page
};

constexpr int XT_BOX = 16 * 128;                           // one box: 16 rows x 128 bytes
constexpr int XT_KV = 4 * XT_BOX;                          // one head of a tile: K quarters 0, 1, V quarters 2, 3
constexpr int XT_STAGE = XT_KV + 2 * XM_CS_BYTES;          // + the tile's cos and sin rows: 10 KB, 1024-aligned
constexpr int XT_TAB = 64;                                 // tiles of a CTA whose page rows are looked up up front
constexpr int XT_MAX_SINK = 16;

template <int S>
constexpr int xt_smem() {
    return 1024 + S * XT_STAGE + XT_TAB * 8 + S * 8 + S * 8;
}

__device__ __forceinline__ void tma2d_xy(uint32_t dst, const CUtensorMap* tm, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar) : "memory");
}

// Shared-memory addressing of one head's rows in the swizzled layout: 16-byte column c (0..15) of K row r is in
// quarter c / 8 at unit (c % 8) ^ (r % 8); V the same from quarter 2.
struct SwzRows {
    uint32_t kb;
    __device__ __forceinline__ uint32_t k(int r, int c) const {
        return kb + ((c >> 3) << 11) + (r << 7) + ((((uint32_t)c & 7u) ^ ((uint32_t)r & 7u)) << 4);
    }
    __device__ __forceinline__ uint32_t v(int r, int c) const { return k(r, c) + 2 * XT_BOX; }
};

// Element offset of the row of head h, slot p0 % ebs of the page holding position p0 (a multiple of 256 when the page
// lies on the tensor's row grid), or -1 when the page table entry, the rows' 16-byte alignment or the rows used
// (slots [lo, hi) of the tile) fail the checks (status bit set).  Positions and page sizes are below 2^31 (N is
// int32, ebs checked by the host).
__device__ __forceinline__ int64_t xt_page_row(const kv800_paged& P, int64_t ehs_rows, int b, int h, uint32_t p0,
                                               int lo, int hi, int* status) {
    const uint32_t eb = (uint32_t)P.ebs, pg = p0 / eb, sl = p0 - pg * eb;
    if (pg >= P.eoff_stride) {
        flag(status, ST_TABLE);
        return -1;
    }
    const int64_t off = P.eoff[(int64_t)b * P.eoff_stride + pg] + (int64_t)h * ehs_rows * 256;
    // the rows of the slots used lie inside the pool
    if (off < 0 || (off & 7) || off + ((int64_t)sl + hi) * 256 > P.epool_elems || hi <= lo) {
        flag(status, ST_EPOOL);
        return -1;
    }
    return off + (int64_t)sl * 256;
}

// The K | V rows of a tile whose page is off the tensor's row grid, by plain 16-byte loads into the swizzled layout:
// slots [lo, hi) from src (slot s at src + 256 s), zeros elsewhere.  Kept out of line: it is the rare path, and
// inlined it would raise the register count of the whole loop.
__device__ __noinline__ void xt_fill_rows(uint8_t* base, const uint16_t* src, int lo, int hi, int lane) {
    for (int idx = lane; idx < 16 * 32; idx += 32) {
        const int s = idx >> 5, u = idx & 31;   // 512-byte K | V row: units 0..15 K, 16..31 V
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (s >= lo && s < hi) val = *reinterpret_cast<const uint4*>(src + s * 256 + 8 * u);
        *reinterpret_cast<uint4*>(base + (u >> 3) * XT_BOX + s * 128 + (((u & 7) ^ (s & 7)) << 4)) = val;
    }
    __syncwarp();
}

template <bool ROPE, int S>
__global__ void __launch_bounds__(32) xdecode_tma(const __grid_constant__ XTArgs t) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const XMArgs& a = t.x;
    const kv800_paged& P = a.P;
    const int b = blockIdx.x, e = blockIdx.y, h = blockIdx.z, lane = threadIdx.x;
    uint8_t* ring = smem + ((1024 - (smem_u32(smem) & 1023)) & 1023);   // stages 1024-aligned for the swizzle
    int64_t* tab = reinterpret_cast<int64_t*>(ring + S * XT_STAGE);   // page rows of the first XT_TAB tiles
    int64_t* srow = tab + XT_TAB;                                       // row offset of the tile in stage s
    const uint32_t bar0 = smem_u32(srow + S);                           // mbarrier of stage s at bar0 + 8 s

    uint32_t bq[8][2];
    xm_load_q(a.q, b, h, lane, bq);

    // ---- the row's exact range [lo_e, n) and sinks [0, cnt) (as in the gather form); positions below 2^31
    const int64_t n = P.N[b], nqb = P.NQ[b];
    int64_t lo_e = nqb * BLK;
    if (P.win && n - P.win > lo_e) lo_e = n - P.win;
    if (lo_e < 0) lo_e = 0;
    int cnt = 0;
    if (P.win && P.sk) {
        int64_t c = P.nsink;
        if (lo_e < c) c = lo_e;
        if (n < c) c = n;
        cnt = c < 0 ? 0 : (int)c;
    }
    const uint32_t j0 = (uint32_t)(lo_e >> 4), j1 = n > lo_e ? (uint32_t)((n + 15) >> 4) : j0;
    const uint32_t T = j1 - j0, nx = (uint32_t)a.nx;
    const uint32_t t0 = j0 + (uint32_t)e * T / nx, t1 = j0 + ((uint32_t)e + 1) * T / nx;   // this split's groups
    const int has_sink = (e == 0 && cnt > 0) ? 1 : 0;
    const int ntiles = (int)(t1 - t0) + has_sink;

    // slots [lo, hi) of group j that lie in [lo_e, n)
    auto slot_range = [&](uint32_t j, int& lo, int& hi) {
        const int64_t p0 = 16 * (int64_t)j;
        lo = (int)(lo_e > p0 ? lo_e - p0 : 0);
        hi = (int)(n < p0 + 16 ? n - p0 : 16);
    };
    auto page_row = [&](uint32_t j) {
        int lo, hi;
        slot_range(j, lo, hi);
        return xt_page_row(P, t.ehs_rows, b, h, 16 * j, lo, hi, a.status);
    };
    // copies of tile it (a page group, not the sink tile) into stage st; lane 0
    auto issue = [&](int it, int st, int64_t row) {
        const uint32_t p0 = 16 * (t0 + (uint32_t)(it - has_sink));
        uint8_t* base = ring + st * XT_STAGE;
        const uint32_t bar = bar0 + 8 * st;
        srow[st] = row;   // for the loop: written before the arrive, whose release the phase's waiters acquire
        const bool boxes = row >= 0 && !(row & 255);   // on the tensor's row grid (else plain loads in the loop)
        uint32_t bytes = boxes ? (uint32_t)XT_KV : 0u;
        int nt = 0;   // table rows copied (positions p0 .. p0 + nt - 1 below npos)
        if (ROPE && (int64_t)p0 < a.npos) nt = (int)min((int64_t)16, a.npos - p0);
        bytes += 2u * 64u * (uint32_t)nt;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_tx(bar, bytes);
        if (boxes) {
#pragma unroll
            for (int qq = 0; qq < 4; qq++)
                tma2d_xy(smem_u32(base + qq * XT_BOX), &t.tm, 64 * qq, (int)(row >> 8), bar);
        }
        if (nt > 0) {
            bulk_g2s(smem_u32(base + XT_KV), a.cos_t + (int64_t)p0 * 32, 64u * nt, bar);
            bulk_g2s(smem_u32(base + XT_KV + XM_CS_BYTES), a.sin_t + (int64_t)p0 * 32, 64u * nt, bar);
        }
    };

    // ---- page rows of the first tiles, one per lane; barriers; the first stages' copies
    const int ntab = min((int)(t1 - t0), XT_TAB);
    for (int k = lane; k < ntab; k += 32) tab[k] = page_row(t0 + (uint32_t)k);
    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init_count(bar0 + 8 * s, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (lane == 0)
        for (int it = has_sink; it < min(S, ntiles); it++) issue(it, it, tab[it - has_sink]);
    // ---- the sink tile (split 0): plain loads into stage 0's swizzled layout, zeros past cnt or for bad rows
    if (has_sink) {
        for (int idx = lane; idx < 16 * 2 * 16; idx += 32) {
            const int u = idx & 15, kv = (idx >> 4) & 1, s = idx >> 5;
            uint4 val = make_uint4(0u, 0u, 0u, 0u);
            if (s < cnt) {
                const int64_t o = (kv ? P.svoff[b] : P.skoff[b]) + ((int64_t)s * HEADS + h) * DIM;
                const int64_t lim = kv ? P.sv_elems : P.sk_elems;
                const uint16_t* pool = kv ? P.sv : P.sk;
                if (o >= 0 && o + DIM <= lim && !(reinterpret_cast<uintptr_t>(pool + o) & 15u))
                    val = *reinterpret_cast<const uint4*>(pool + o + 8 * u);
                else if (u == 0)
                    flag(a.status, ST_SINK);
            }
            const int qq = 2 * kv + (u >> 3);
            *reinterpret_cast<uint4*>(ring + qq * XT_BOX + s * 128 + (((u & 7) ^ (s & 7)) << 4)) = val;
        }
        if (ROPE) {   // cos / sin rows of positions 0 .. 15: 2 x 16 rows of 4 units
            for (int idx = lane; idx < 2 * 16 * 4; idx += 32) {
                const int u = idx & 3, s = (idx >> 2) & 15, which = idx >> 6;
                uint4 val = make_uint4(0u, 0u, 0u, 0u);
                if (s < cnt && s < a.npos)
                    val = *reinterpret_cast<const uint4*>((which ? a.sin_t : a.cos_t) + s * 32 + 8 * u);
                *reinterpret_cast<uint4*>(ring + XT_KV + which * XM_CS_BYTES + s * 64 + 16 * u) = val;
            }
        }
        __syncwarp();
    }

    XMState st_;
    st_.init();
    int timeouts = 0;
    for (int it = 0; it < ntiles; it++) {
        const int st = it % S;
        uint8_t* base = ring + st * XT_STAGE;
        uint32_t vmask;
        if (has_sink && it == 0) {
            vmask = (1u << cnt) - 1u;
            if (ROPE && cnt > a.npos) {
                vmask &= (1u << a.npos) - 1u;   // npos < cnt <= 16
                if (lane == 0) flag(a.status, ST_TABLE);
            }
        } else {
            const int use = it / S - ((has_sink && st == 0) ? 1 : 0);   // TMA fills of this stage before this one
            if (!mbar_wait(bar0 + 8 * st, (uint32_t)use & 1u)) timeouts++;
            const uint32_t j = t0 + (uint32_t)(it - has_sink);
            int lo, hi;
            slot_range(j, lo, hi);
            const int64_t row = srow[st];
            if (row >= 0 && (row & 255)) xt_fill_rows(base, P.epool + row, lo, hi, lane);   // off the row grid
            vmask = (row >= 0 && hi > lo) ? (((hi >= 16) ? 0xffffu : ((1u << hi) - 1u)) & ~((1u << lo) - 1u)) : 0u;
            if (ROPE && 16 * (int64_t)j + 16 > a.npos) {   // positions without a table row (flagged, as in the gather
                                                           // form)
                const int64_t ok = a.npos - 16 * (int64_t)j;
                const uint32_t tmask = ok <= 0 ? 0u : (ok >= 16 ? 0xffffu : ((1u << ok) - 1u));
                if ((vmask & ~tmask) && lane == 0) flag(a.status, ST_TABLE);
                vmask &= tmask;
            }
            if (vmask != 0xffffu) {   // zero the V rows of the masked slots (two 128-byte lines per row)
                for (int idx = lane; idx < 16 * 16; idx += 32) {
                    const int s = idx >> 4, u = idx & 15;
                    if (!((vmask >> s) & 1u))
                        *reinterpret_cast<uint4*>(base + (2 + (u >> 3)) * XT_BOX + s * 128 +
                                                  (((u & 7) ^ (s & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
                }
                __syncwarp();
            }
        }
        const SwzRows rw{smem_u32(base)};
        const uint32_t* cs = reinterpret_cast<const uint32_t*>(base + XT_KV);
        const uint32_t* sn = reinterpret_cast<const uint32_t*>(base + XT_KV + XM_CS_BYTES);
        xm_tile<ROPE>(rw, cs, sn, bq, vmask, a.scale, st_, lane);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // this lane's reads / zero-fills first
        __syncwarp();
        if (lane == 0 && it + S < ntiles) {
            const int nk = it + S - has_sink;
            issue(it + S, st, nk < XT_TAB ? tab[nk] : page_row(t0 + (uint32_t)nk));
        }
    }
    if (timeouts && lane == 0) flag(a.status, ST_TIMEOUT);
    xm_finish_head(a, st_, b, e, h, lane);
}

}  // namespace kv800
