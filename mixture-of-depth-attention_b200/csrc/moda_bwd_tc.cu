// MoDA backward on Blackwell tensor cores (sequence part) + a per-token CUDA-core
// kernel for the depth part.
//
// Gradients of the fused forward (moda/kernels/moda_naive.py:13-162 under torch
// autograd): with P = exp(scale*Q.K^T - lse) (row lse from the forward) and
// D = rowsum(dO * O),
//   dS = P * (dO.V^T - D),  dQ = scale*dS.K,  dK = scale*dS^T.Q,  dV = P^T.dO.
//
// Two launches of one kernel template, each a persistent TMA -> tcgen05.mma ->
// TMEM pipeline like the forward's:
//   MODE_DKDV  work item = 128 keys of one (batch, KV head). For every 128-row
//              query tile (token-major, the G query heads of the KV head) that
//              reaches those keys: S^T = K.Q^T and dP^T = V.dO^T into TMEM; four
//              warps (one key row per thread) form P^T and dS^T in 16-bit and
//              write them back into TMEM; dV += P^T.dO and dK += dS^T.Q take A
//              from TMEM. dK and dV accumulate in TMEM over all query tiles, so
//              the GQA sum over heads needs no atomics.
//   MODE_DQ    work item = one 128-row query tile. For every 128-key block up to
//              the diagonal: S = Q.K^T, dP = dO.V^T, dS (one query row per
//              thread), dQ += dS.K with A from TMEM.
// TMEM: [0,128) S or S^T, [128,256) dP or dP^T, then the d-column accumulators
// (dV, dK or dQ). The 16-bit P / dS overwrite the first 64 columns of the score
// block they come from, after the thread has read them.
//
// Warps: 0-3 elementwise (TMEM lane quarter w), 4 TMA producer, 5 TMEM allocator
// and MMA issuer (one thread). Every wait is bounded (status word, abort flag).
//
// The depth part (each token's own L rows, read only by that token's G query
// rows) is small: moda_bwd_depth_token_kernel stages one token's rows in shared
// memory and writes dK_depth, dV_depth and adds the depth term of dQ.
#include "moda_internal.h"

#include <cstdio>

namespace moda {

namespace {

constexpr int kBThreads = 192;
constexpr int kBRows = 128;      // rows per tile (query rows or keys)
constexpr int kWarpProd = 4, kWarpMma = 5;
constexpr int MODE_DKDV = 0, MODE_DQ = 1;

template <int HD>
struct BwdCfg {
    static constexpr int kTile = kBRows * HD * 2;          // one 128 x HD 16-bit tile
    static constexpr int kColBlocks = HD / 64;
    static constexpr int kStages = HD == 128 ? 2 : 4;      // ring of tile pairs
    static constexpr int kResOff = 0;                       // resident pair
    static constexpr int kRingOff = 2 * kTile;
    static constexpr int kStageOff = kRingOff + kStages * 2 * kTile;   // lse/D staging
    static constexpr int kBarOff = kStageOff + 2 * 2 * kBRows * 4;
    // res_full res_empty st_full_a pd_full_a acc_done acc_free end stage, ring_full[S]
    // ring_empty[S], st_full_b pd_full_b (a / b: the score tile's column halves)
    static constexpr int kNumBars = 10 + 2 * kStages;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kSmem = kMiscOff + 32 + 1024;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kAcc0 = 256, kAcc1 = 256 + HD;
};

}  // namespace

static __device__ int moda_bwd_status = 0;

MODA_DEV bool bwait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                *abort_flag = 1;
                atomicCAS(&moda_bwd_status, 0, 0x200 | site);
                return false;
            }
        }
    }
}

struct BwdItem {
    int b, hk;
    int res0;    // first token (DQ: query tile) or first key (DKDV: key tile)
    int first;   // first step index (DKDV: query tile, DQ: key tile)
    int nsteps;
};

template <int MODE>
MODA_DEV BwdItem bwd_item(const TcBwdParams& p, int item) {
    BwdItem it;
    const int bh = p.B * p.Hk;
    const int pos = item / bh, r = item % bh;
    it.b = r / p.Hk;
    it.hk = r % p.Hk;
    if (MODE == MODE_DKDV) {
        const int kt = pos;                          // ascending: most query tiles first
        it.res0 = kt * kBRows;
        it.first = it.res0 / p.n_tok;                // first query tile with a token >= res0
        it.nsteps = p.num_qtiles - it.first;
    } else {
        const int qt = p.num_qtiles - 1 - pos;       // descending: most key blocks first
        it.res0 = qt * p.n_tok;
        const int last_tok = min(p.T, it.res0 + p.n_tok) - 1;
        it.first = 0;
        it.nsteps = last_tok / kBRows + 1;
    }
    return it;
}

template <int HD, int FMT, int MODE>
__global__ void __launch_bounds__(kBThreads, 1) moda_bwd_tc_kernel(const __grid_constant__ TcBwdParams p) {
    using Cfg = BwdCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sRes = sbase + Cfg::kResOff;
    const uint32_t sRing = sbase + Cfg::kRingOff;
    const uint32_t bar0 = sbase + Cfg::kBarOff;
    const uint32_t res_full = bar0, res_empty = bar0 + 8, st_full = bar0 + 16, pd_full = bar0 + 24;
    const uint32_t acc_done = bar0 + 32, acc_free = bar0 + 40, end_bar = bar0 + 48;
    // DKDV: the four elementwise warps have staged their rows' lse and D for a step
    const uint32_t stage_bar = bar0 + 56;
    auto ring_full = [&](uint32_t i) { return bar0 + 8u * (8 + i); };
    auto ring_empty = [&](uint32_t i) { return bar0 + 8u * (8 + Cfg::kStages + i); };
    // per column half h of the 128-column score tiles: scores ready / P and dS written
    auto st_full_h = [&](int h) { return h == 0 ? st_full : bar0 + 8u * (8 + 2 * Cfg::kStages); };
    auto pd_full_h = [&](int h) { return h == 0 ? pd_full : bar0 + 8u * (9 + 2 * Cfg::kStages); };
    float* stage = reinterpret_cast<float*>(smem + Cfg::kStageOff);  // [2][2][128]: lse2, D
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOff);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kMiscOff + 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t kTile = Cfg::kTile;
    // Items (sorted heaviest first) in serpentine rounds: round r hands the CTAs items
    // [r*grid, (r+1)*grid) in CTA order for even r and in reverse for odd r, so no CTA
    // gets the heaviest item of every round. Every role walks the same sequence.
    auto round_item = [&](int round) {
        const int g = static_cast<int>(gridDim.x);
        return round * g + ((round & 1) ? g - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x));
    };

    if (threadIdx.x == 0) {
        mbar_init(res_full, 1);
        mbar_init(res_empty, 1);
        mbar_init(st_full, 1);
        mbar_init(pd_full, 4);
        mbar_init(st_full_h(1), 1);
        mbar_init(pd_full_h(1), 4);
        mbar_init(acc_done, 1);
        mbar_init(acc_free, 4);
        mbar_init(end_bar, 1);
        mbar_init(stage_bar, 4);
        for (int i = 0; i < Cfg::kStages; ++i) {
            mbar_init(ring_full(i), 1);
            mbar_init(ring_empty(i), 1);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(smem_u32(tmem_holder), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    // resident pair: DKDV (K, V) key tile, DQ (Q, dO) query tile; ring pairs the other way
    const CUtensorMap* res_m0 = MODE == MODE_DKDV ? &p.tm_k : &p.tm_q;
    const CUtensorMap* res_m1 = MODE == MODE_DKDV ? &p.tm_v : &p.tm_do;
    const CUtensorMap* ring_m0 = MODE == MODE_DKDV ? &p.tm_q : &p.tm_k;
    const CUtensorMap* ring_m1 = MODE == MODE_DKDV ? &p.tm_do : &p.tm_v;

    if (warp == kWarpProd) {
        if (lane == 0) {
            // ------------------------------------------------------------ TMA producer
            uint32_t f = 0, nres = 0;
            bool ok = true;
            // coordinates of a tile: key-like (d, row, hk, b), query-like (d, hk*G, tok, b)
            auto load_pair = [&](const CUtensorMap* m0, const CUtensorMap* m1, bool keylike, int row0,
                                 const BwdItem& it, uint32_t dst, uint32_t bar) {
                mbar_expect_tx(bar, 2 * kTile);
                for (int cb = 0; cb < Cfg::kColBlocks; ++cb) {
                    if (keylike) {
                        tma_load_4d(m0, dst + cb * 16384, bar, cb * 64, row0, it.hk, it.b);
                        tma_load_4d(m1, dst + kTile + cb * 16384, bar, cb * 64, row0, it.hk, it.b);
                    } else {
                        tma_load_4d(m0, dst + cb * 16384, bar, cb * 64, it.hk * p.G, row0, it.b);
                        tma_load_4d(m1, dst + kTile + cb * 16384, bar, cb * 64, it.hk * p.G, row0, it.b);
                    }
                }
            };
            for (int round = 0, item = round_item(0); item < p.num_items && ok; item = round_item(++round)) {
                const BwdItem it = bwd_item<MODE>(p, item);
                ok = bwait(res_empty, (nres & 1u) ^ 1u, abort_flag, 1);
                if (!ok) break;
                load_pair(res_m0, res_m1, MODE == MODE_DKDV, it.res0, it, sRes, res_full);
                ++nres;
                for (int s = 0; s < it.nsteps && ok; ++s) {
                    const uint32_t slot = f % Cfg::kStages;
                    ok = bwait(ring_empty(slot), ((f / Cfg::kStages) & 1u) ^ 1u, abort_flag, 2);
                    if (!ok) break;
                    const int idx = it.first + s;
                    if (MODE == MODE_DKDV)
                        load_pair(ring_m0, ring_m1, false, idx * p.n_tok, it, sRing + slot * 2 * kTile,
                                  ring_full(slot));
                    else
                        load_pair(ring_m0, ring_m1, true, idx * kBRows, it, sRing + slot * 2 * kTile,
                                  ring_full(slot));
                    ++f;
                }
            }
            // exit: loads in flight must land before shared memory goes away
            const uint32_t lo = f > Cfg::kStages ? f - Cfg::kStages : 0;
            for (uint32_t fi = lo; fi < f; ++fi)
                mbar_wait_drain(ring_full(fi % Cfg::kStages), (fi / Cfg::kStages) & 1u);
            if (nres > 0) mbar_wait_drain(res_full, (nres - 1) & 1u);
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            // Every step's 128-column score tiles are computed in two column halves (64
            // ring rows each). Issue order per step s:
            //   [S, dP half a(s); half b(s) -- issued during step s-1, or at item start]
            //   dV/dK (dQ) half a(s) once its P / dS are written
            //   S, dP half a(s+1): overwrite half a's columns after the MMAs above read them
            //   dV/dK (dQ) half b(s), then S, dP half b(s+1)
            // so the elementwise work on one half overlaps the tensor core on the other.
            constexpr uint32_t idesc_h = make_idesc(FMT, kBRows, kBRows / 2, 0);  // B K-major (d)
            constexpr uint32_t idesc_o = make_idesc(FMT, kBRows, HD, 1);         // B MN-major (d)
            constexpr uint32_t hi = desc_hi_sw128(1024);
            const uint32_t a0 = desc_lo(sRes, 16), a1 = desc_lo(sRes + kTile, 16);
            const uint32_t tS = tmem, tP = tmem + 128;
            uint32_t f = 0, nres = 0, nst = 0, nitems = 0;
            bool ok = true;
            // S (S^T) = res0 . ring0^T and dP (dP^T) = res1 . ring1^T for ring rows
            // [64h, 64h + 64), contraction over d, into score columns [64h, 64h + 64)
            auto issue_scores = [&](uint32_t rb, int h) {
                const uint32_t b0 = desc_lo(rb + h * 8192, 16), b1 = desc_lo(rb + kTile + h * 8192, 16);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                    mma_ss(tS + 64 * h, desc_join(a0 + off, hi), desc_join(b0 + off, hi), idesc_h, kk > 0);
                }
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                    mma_ss(tP + 64 * h, desc_join(a1 + off, hi), desc_join(b1 + off, hi), idesc_h, kk > 0);
                }
                mma_commit(st_full_h(h));
            };
            // contraction over ring rows [64h, 64h + 64) (MN-major B, d contiguous); the
            // 16-bit P / dS of half h sit in score columns [64h, 64h + 32)
            auto issue_acc = [&](uint32_t rb, int h, bool first) {
                const uint32_t v0 = desc_lo(rb, 16384), v1 = desc_lo(rb + kTile, 16384);
                if (MODE == MODE_DKDV) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)   // dV += P^T . dO
                        mma_ts(tmem + Cfg::kAcc0, tS + 64 * h + kk * 8,
                               desc_join(v1 + (((4 * h + kk) * 2048) >> 4), hi), idesc_o, (first && kk == 0) ? 0u : 1u);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)   // dK += dS^T . Q
                        mma_ts(tmem + Cfg::kAcc1, tP + 64 * h + kk * 8,
                               desc_join(v0 + (((4 * h + kk) * 2048) >> 4), hi), idesc_o, (first && kk == 0) ? 0u : 1u);
                } else {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)   // dQ += dS . K
                        mma_ts(tmem + Cfg::kAcc0, tS + 64 * h + kk * 8,
                               desc_join(v0 + (((4 * h + kk) * 2048) >> 4), hi), idesc_o, (first && kk == 0) ? 0u : 1u);
                }
            };
            for (int round = 0, item = round_item(0); item < p.num_items && ok; item = round_item(++round)) {
                const BwdItem it = bwd_item<MODE>(p, item);
                ok = bwait(res_full, nres & 1u, abort_flag, 3);
                if (!ok) break;
                ++nres;
                // the item's first step: both score halves
                ok = bwait(ring_full(f % Cfg::kStages), (f / Cfg::kStages) & 1u, abort_flag, 4);
                if (!ok) break;
                tc_fence_after();
                {
                    const uint32_t rb = sRing + (f % Cfg::kStages) * 2 * kTile;
                    issue_scores(rb, 0);
                    issue_scores(rb, 1);
                    if (it.nsteps == 1) mma_commit(res_empty);  // resident tiles no longer read
                }
                for (int s = 0; s < it.nsteps; ++s) {
                    const uint32_t slot = f % Cfg::kStages;
                    const uint32_t rb = sRing + slot * 2 * kTile;
                    const bool has_next = s + 1 < it.nsteps;
                    const uint32_t rb_next = sRing + ((f + 1) % Cfg::kStages) * 2 * kTile;
                    // half a of step s
                    ok = bwait(pd_full_h(0), nst & 1u, abort_flag, 5);
                    if (ok && s == 0 && nitems > 0) ok = bwait(acc_free, (nitems - 1) & 1u, abort_flag, 6);
                    if (!ok) break;
                    tc_fence_after();
                    issue_acc(rb, 0, s == 0);
                    if (has_next) {
                        ok = bwait(ring_full((f + 1) % Cfg::kStages), ((f + 1) / Cfg::kStages) & 1u, abort_flag, 4);
                        if (!ok) break;
                        tc_fence_after();
                        issue_scores(rb_next, 0);
                    }
                    // half b of step s
                    ok = bwait(pd_full_h(1), nst & 1u, abort_flag, 5);
                    if (!ok) break;
                    ++nst;
                    tc_fence_after();
                    issue_acc(rb, 1, false);
                    mma_commit(ring_empty(slot));
                    if (!has_next) mma_commit(acc_done);
                    if (has_next) {
                        issue_scores(rb_next, 1);
                        if (s + 2 == it.nsteps) mma_commit(res_empty);  // last scores of the item
                    }
                    ++f;
                }
                ++nitems;
            }
            mma_commit(end_bar);
            mbar_wait_drain(end_bar, 0);
        }
    } else {
        // ------------------------------------------------------------ elementwise warps
        const int wq = warp;  // TMEM lane quarter
        const int row = wq * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t tS = tmem + lane_off, tP = tmem + lane_off + 128;
        const float sc2 = p.sc;
        const int gsh = __ffs(p.G) - 1;  // G divides 128: a power of two
        uint32_t nst = 0, nitems = 0;
        bool ok = true;
        for (int round = 0, item = round_item(0); item < p.num_items && ok; item = round_item(++round)) {
            const BwdItem it = bwd_item<MODE>(p, item);
            // DQ: this thread's query row; its lse and D stay in registers
            int tok_r = 0;
            float lse2_r = INFINITY, D_r = 0.f;
            if (MODE == MODE_DQ) {
                tok_r = it.res0 + (row >> gsh);
                if (tok_r < p.T) {
                    const long long ri = (static_cast<long long>(it.b) * p.Hq + it.hk * p.G + (row & (p.G - 1))) * p.T + tok_r;
                    lse2_r = p.lse[ri] * kLog2e;
                    D_r = p.delta[ri];
                }
            }
            const int key_r = it.res0 + row;  // DKDV: this thread's key
            for (int s = 0; s < it.nsteps; ++s) {
                const int idx = it.first + s;
                float* st_lse = stage + (nst & 1u) * 256;
                float* st_D = st_lse + 128;
                int col0;       // DKDV: first query token of the tile; DQ: first key of the block
                bool need_mask;
                if (MODE == MODE_DKDV) {
                    col0 = idx * p.n_tok;
                    // stage lse and D of the tile's 128 query rows (column q <-> token q/G, head q%G)
                    const int tq = col0 + (row >> gsh);
                    float l2 = INFINITY, dd = 0.f;
                    if (tq < p.T) {
                        const long long ri = (static_cast<long long>(it.b) * p.Hq + it.hk * p.G + (row & (p.G - 1))) * p.T + tq;
                        l2 = p.lse[ri] * kLog2e;
                        dd = p.delta[ri];
                    }
                    st_lse[row] = l2;
                    st_D[row] = dd;
                    // all four warps staged (one phase per step; a warp reaches the next
                    // phase only after every warp arrived, so parities never alias)
                    __syncwarp();
                    if (lane == 0) mbar_arrive(stage_bar);
                    if (!bwait(stage_bar, nst & 1u, abort_flag, 9)) { ok = false; break; }
                    need_mask = col0 < it.res0 + kBRows;   // some token of the tile below some key
                } else {
                    col0 = idx * kBRows;
                    need_mask = col0 + kBRows - 1 > it.res0;  // some key above some token
                }
#pragma unroll 1
                for (int h = 0; h < 2 && ok; ++h) {  // the two column halves of the score tiles
                    if (!bwait(st_full_h(h), nst & 1u, abort_flag, 7)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 2 * h; c < 2 * h + 2; ++c) {
                        uint32_t sv[32], dv[32];
                        tmem_ld32(tS + 32 * c, sv);
                        tmem_ld32(tP + 32 * c, dv);
                        tmem_wait_ld();
                        tmem_reg_fence(sv);
                        tmem_reg_fence(dv);
                        uint32_t pk_p[16], pk_d[16];
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            float pr[2], ds[2];
#pragma unroll
                            for (int u = 0; u < 2; ++u) {
                                const int col = 32 * c + i + u;
                                float l2, dd;
                                bool valid;
                                if (MODE == MODE_DKDV) {
                                    l2 = st_lse[col];
                                    dd = st_D[col];
                                    valid = !need_mask || col0 + (col >> gsh) >= key_r;
                                } else {
                                    l2 = lse2_r;
                                    dd = D_r;
                                    valid = !need_mask || col0 + col <= tok_r;
                                }
                                const float e = ex2(fmaf(__uint_as_float(sv[i + u]), sc2, -l2));
                                pr[u] = valid ? e : 0.f;
                                ds[u] = pr[u] * (__uint_as_float(dv[i + u]) - dd);
                            }
                            pk_p[i >> 1] = FMT == 1 ? pack_bf16x2(pr[0], pr[1]) : pack_f16x2(pr[0], pr[1]);
                            pk_d[i >> 1] = FMT == 1 ? pack_bf16x2(ds[0], ds[1]) : pack_f16x2(ds[0], ds[1]);
                        }
                        // 16-bit results: half h's columns [64h, 64h + 32), already read
                        const uint32_t poff = 64 * h + 16 * (c - 2 * h);
                        if (MODE == MODE_DKDV) {
                            tmem_st16(tS + poff, pk_p);   // P^T
                            tmem_st16(tP + poff, pk_d);   // dS^T
                        } else {
                            tmem_st16(tS + poff, pk_d);   // dS
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(pd_full_h(h));
                }
                if (!ok) break;
                ++nst;
            }
            if (!ok) break;
            // ------------------------------------------------------------ epilogue
            if (!bwait(acc_done, nitems & 1u, abort_flag, 8)) { ok = false; break; }
            ++nitems;
            tc_fence_after();
            uint4* dst0;
            uint4* dst1 = nullptr;
            bool valid;
            if (MODE == MODE_DKDV) {
                valid = key_r < p.T;
                dst0 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.dv) + it.b * p.dv_sb + it.hk * p.dv_sh +
                                                static_cast<long long>(key_r) * p.dv_st);
                dst1 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.dk) + it.b * p.dk_sb + it.hk * p.dk_sh +
                                                static_cast<long long>(key_r) * p.dk_st);
            } else {
                valid = tok_r < p.T;
                const int head = it.hk * p.G + (row & (p.G - 1));
                dst0 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.dq) + it.b * p.dq_sb + head * p.dq_sh +
                                                static_cast<long long>(tok_r) * p.dq_st);
            }
#pragma unroll
            for (int a = 0; a < (MODE == MODE_DKDV ? 2 : 1); ++a) {
                const uint32_t tacc = tmem + lane_off + (a == 0 ? Cfg::kAcc0 : Cfg::kAcc1);
                // dV is P^T.dO as is; dK and dQ carry the softmax scale
                const float mul = (MODE == MODE_DKDV && a == 0) ? 1.f : p.scale;
                uint4* dst = a == 0 ? dst0 : dst1;
#pragma unroll
                for (int cb = 0; cb < HD; cb += 32) {
                    uint32_t ov[32];
                    tmem_ld32_sync(tacc + cb, ov);
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float x0 = __uint_as_float(ov[2 * i]) * mul, x1 = __uint_as_float(ov[2 * i + 1]) * mul;
                        pk[i] = FMT == 1 ? pack_bf16x2(x0, x1) : pack_f16x2(x0, x1);
                    }
                    if (valid) {
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch)
                            dst[(cb >> 3) + ch] = make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_free);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// ---------------------------------------------------------------- depth part
namespace {
template <typename T>
MODA_DEV float ldf(const T* p);
template <>
MODA_DEV float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
MODA_DEV float ldf<__half>(const __half* p) { return __half2float(*p); }
template <>
MODA_DEV float ldf<float>(const float* p) { return *p; }
template <typename T>
MODA_DEV void stf(T* p, float x);
template <>
MODA_DEV void stf<__nv_bfloat16>(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
template <>
MODA_DEV void stf<__half>(__half* p, float x) { *p = __float2half_rn(x); }
template <>
MODA_DEV void stf<float>(float* p, float x) { *p = x; }

template <typename T>
MODA_DEV T* rowp(const ModaTensor& t, int b, int h, long long r) {
    return static_cast<T*>(t.ptr) + b * t.strides[0] + h * t.strides[1] + r * t.strides[2];
}
}  // namespace

constexpr int kDepthChunk = 32;  // depth rows staged per pass

// One block per token (b, KV head, t): its G query rows against its L depth rows
// [t*L, (t+1)*L), in passes of kDepthChunk rows. Writes dK_depth, dV_depth for those
// rows and adds scale * sum_l dS_l kd_l to the token's dQ rows (which the sequence
// kernels wrote before this launch).
template <typename T>
__global__ void __launch_bounds__(128) moda_bwd_depth_token_kernel(const __grid_constant__ BwdParams p) {
    extern __shared__ float sm[];
    const int t = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
    const int G = p.G, L = p.L, d = p.d, dp1 = d + 1;
    const int LC = min(L, kDepthChunk);
    float* s_kd = sm;                  // [LC][d+1]
    float* s_vd = s_kd + LC * dp1;     // [LC][d+1]
    float* s_q = s_vd + LC * dp1;      // [G][d+1]
    float* s_do = s_q + G * dp1;       // [G][d+1]
    float* s_dq = s_do + G * dp1;      // [G][d]
    float* s_p = s_dq + G * d;         // [G][LC]
    float* s_ds = s_p + G * LC;        // [G][LC]
    float* s_lse = s_ds + G * LC;      // [G]
    float* s_D = s_lse + G;            // [G]
    const int tid = threadIdx.x, nth = blockDim.x;
    const float sc2 = p.scale * kLog2e;
    for (int i = tid; i < G * d; i += nth) {
        const int g = i / d, e = i % d, h = hk * G + g;
        s_q[g * dp1 + e] = ldf<T>(rowp<const T>(p.q, b, h, t) + e * p.q.strides[3]);
        s_do[g * dp1 + e] = ldf<T>(rowp<const T>(p.dout, b, h, t) + e * p.dout.strides[3]);
        s_dq[i] = 0.f;
    }
    for (int g = tid; g < G; g += nth) {
        const long long ri = (static_cast<long long>(b) * p.Hq + hk * G + g) * p.T + t;
        s_lse[g] = p.lse[ri] * kLog2e;
        s_D[g] = p.delta[ri];
    }
    for (int l0 = 0; l0 < L; l0 += LC) {
        const int nl = min(LC, L - l0);
        const long long r0 = static_cast<long long>(t) * L + l0;
        __syncthreads();  // previous pass done with the staged rows
        for (int i = tid; i < nl * d; i += nth) {
            const int l = i / d, e = i % d;
            s_kd[l * dp1 + e] = ldf<T>(rowp<const T>(p.kd, b, hk, r0 + l) + e * p.kd.strides[3]);
            s_vd[l * dp1 + e] = ldf<T>(rowp<const T>(p.vd, b, hk, r0 + l) + e * p.vd.strides[3]);
        }
        __syncthreads();
        for (int i = tid; i < G * nl; i += nth) {
            const int g = i / nl, l = i % nl;
            float s = 0.f, dp = 0.f;
            for (int e = 0; e < d; ++e) {
                s = fmaf(s_q[g * dp1 + e], s_kd[l * dp1 + e], s);
                dp = fmaf(s_do[g * dp1 + e], s_vd[l * dp1 + e], dp);
            }
            const float pr = ex2(fmaf(s, sc2, -s_lse[g]));
            s_p[g * LC + l] = pr;
            s_ds[g * LC + l] = pr * (dp - s_D[g]);
        }
        __syncthreads();
        for (int i = tid; i < nl * d; i += nth) {
            const int l = i / d, e = i % d;
            float ak = 0.f, av = 0.f;
            for (int g = 0; g < G; ++g) {
                ak = fmaf(s_ds[g * LC + l], s_q[g * dp1 + e], ak);
                av = fmaf(s_p[g * LC + l], s_do[g * dp1 + e], av);
            }
            stf<T>(rowp<T>(p.dkd, b, hk, r0 + l) + e * p.dkd.strides[3], ak * p.scale);
            stf<T>(rowp<T>(p.dvd, b, hk, r0 + l) + e * p.dvd.strides[3], av);
        }
        for (int i = tid; i < G * d; i += nth) {
            const int g = i / d, e = i % d;
            float a = s_dq[i];
            for (int l = 0; l < nl; ++l) a = fmaf(s_ds[g * LC + l], s_kd[l * dp1 + e], a);
            s_dq[i] = a;
        }
    }
    __syncthreads();
    for (int i = tid; i < G * d; i += nth) {
        const int g = i / d, e = i % d, h = hk * G + g;
        T* dq = rowp<T>(p.dq, b, h, t) + e * p.dq.strides[3];
        stf<T>(dq, ldf<T>(dq) + s_dq[i] * p.scale);
    }
}

// One warp per token (b, KV head, t); lane l owns depth rows t*L + l + 32j (j < J).
// The token's G query rows and dO rows are staged once in the warp's shared memory
// (fp32); each lane reads its own depth rows with 16-byte loads. Per lane:
//   s[j][g] = q_g . kd_r, dp[j][g] = dO_g . vd_r        (2*G*d FMA per row)
//   dK_depth[r] = scale * sum_g dS q_g, dV_depth[r] = sum_g P dO_g
// and the dQ term scale * sum_l dS_{g,l} kd_l goes through a shared-memory copy of
// dS (lanes then split d). No block-wide synchronisation.
constexpr int kDepthWarps = 4;

template <typename T, int HD, int G, int J>
__global__ void __launch_bounds__(kDepthWarps * 32) moda_bwd_depth_warp_kernel(const __grid_constant__ BwdParams p) {
    static_assert(sizeof(T) == 2, "16-bit inputs");
    __shared__ __align__(16) float s_q[kDepthWarps][G][HD];
    __shared__ __align__(16) float s_do[kDepthWarps][G][HD];
    __shared__ float s_ds[kDepthWarps][G][32 * J];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long tok_id = static_cast<long long>(blockIdx.x) * kDepthWarps + w;
    if (tok_id >= static_cast<long long>(p.B) * p.Hk * p.T) return;
    const int t = static_cast<int>(tok_id % p.T);
    const int hk = static_cast<int>((tok_id / p.T) % p.Hk);
    const int b = static_cast<int>(tok_id / (static_cast<long long>(p.T) * p.Hk));
    const int L = p.L;
    const float sc2 = p.scale * kLog2e;
    // stage q and dO rows of the G heads (lanes split d, 8 elements per 16-byte load)
    for (int i = lane; i < G * HD / 8; i += 32) {
        const int g = i / (HD / 8), e = (i % (HD / 8)) * 8, h = hk * G + g;
        const uint4 uq = *reinterpret_cast<const uint4*>(rowp<const T>(p.q, b, h, t) + e);
        const uint4 ug = *reinterpret_cast<const uint4*>(rowp<const T>(p.dout, b, h, t) + e);
        const T* tq = reinterpret_cast<const T*>(&uq);
        const T* tg = reinterpret_cast<const T*>(&ug);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            s_q[w][g][e + k] = ldf<T>(tq + k);
            s_do[w][g][e + k] = ldf<T>(tg + k);
        }
    }
    float lse2[G], dlt[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const long long ri = (static_cast<long long>(b) * p.Hq + hk * G + g) * p.T + t;
        lse2[g] = p.lse[ri] * kLog2e;
        dlt[g] = p.delta[ri];
    }
    __syncwarp();
    const long long r0 = static_cast<long long>(t) * L;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int l = lane + 32 * j;
        float s[G], dp[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = dp[g] = 0.f;
        if (l < L) {
            const T* kr = rowp<const T>(p.kd, b, hk, r0 + l);
            const T* vr = rowp<const T>(p.vd, b, hk, r0 + l);
#pragma unroll 4
            for (int e = 0; e < HD; e += 8) {
                const uint4 uk = *reinterpret_cast<const uint4*>(kr + e);
                const uint4 uv = *reinterpret_cast<const uint4*>(vr + e);
                const T* tk = reinterpret_cast<const T*>(&uk);
                const T* tv = reinterpret_cast<const T*>(&uv);
                float kf[8], vf[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    kf[k] = ldf<T>(tk + k);
                    vf[k] = ldf<T>(tv + k);
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 q0 = *reinterpret_cast<const float4*>(&s_q[w][g][e]);
                    const float4 q1 = *reinterpret_cast<const float4*>(&s_q[w][g][e + 4]);
                    const float4 g0 = *reinterpret_cast<const float4*>(&s_do[w][g][e]);
                    const float4 g1 = *reinterpret_cast<const float4*>(&s_do[w][g][e + 4]);
                    s[g] = fmaf(q0.x, kf[0], fmaf(q0.y, kf[1], fmaf(q0.z, kf[2], fmaf(q0.w, kf[3], s[g]))));
                    s[g] = fmaf(q1.x, kf[4], fmaf(q1.y, kf[5], fmaf(q1.z, kf[6], fmaf(q1.w, kf[7], s[g]))));
                    dp[g] = fmaf(g0.x, vf[0], fmaf(g0.y, vf[1], fmaf(g0.z, vf[2], fmaf(g0.w, vf[3], dp[g]))));
                    dp[g] = fmaf(g1.x, vf[4], fmaf(g1.y, vf[5], fmaf(g1.z, vf[6], fmaf(g1.w, vf[7], dp[g]))));
                }
            }
        }
        float pr[G], ds[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            pr[g] = l < L ? ex2(fmaf(s[g], sc2, -lse2[g])) : 0.f;
            ds[g] = pr[g] * (dp[g] - dlt[g]);
            s_ds[w][g][l] = ds[g];
        }
        if (l < L) {
            T* dkr = rowp<T>(p.dkd, b, hk, r0 + l);
            T* dvr = rowp<T>(p.dvd, b, hk, r0 + l);
#pragma unroll 2
            for (int e = 0; e < HD; e += 8) {
                float ak[8], av[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) ak[k] = av[k] = 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        ak[k] = fmaf(ds[g], s_q[w][g][e + k], ak[k]);
                        av[k] = fmaf(pr[g], s_do[w][g][e + k], av[k]);
                    }
                }
                uint4 ok, ov;
                T* tk = reinterpret_cast<T*>(&ok);
                T* tv = reinterpret_cast<T*>(&ov);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    stf<T>(tk + k, ak[k] * p.scale);
                    stf<T>(tv + k, av[k]);
                }
                *reinterpret_cast<uint4*>(dkr + e) = ok;
                *reinterpret_cast<uint4*>(dvr + e) = ov;
            }
        }
    }
    __syncwarp();
    // dQ_g[e] += scale * sum_l dS_{g,l} kd_l[e]: lanes split d (HD/32 elements each)
    constexpr int EPL = HD / 32;
    float acc[G][EPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int k = 0; k < EPL; ++k) acc[g][k] = 0.f;
    for (int l = 0; l < L; ++l) {
        const T* kr = rowp<const T>(p.kd, b, hk, r0 + l) + lane * EPL;
        float kf[EPL];
        if constexpr (EPL == 4) {
            const uint2 u = *reinterpret_cast<const uint2*>(kr);
            const T* tk = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) kf[k] = ldf<T>(tk + k);
        } else {
            const uint32_t u = *reinterpret_cast<const uint32_t*>(kr);
            const T* tk = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int k = 0; k < EPL; ++k) kf[k] = ldf<T>(tk + k);
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float dsv = s_ds[w][g][l];
#pragma unroll
            for (int k = 0; k < EPL; ++k) acc[g][k] = fmaf(dsv, kf[k], acc[g][k]);
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        T* dq = rowp<T>(p.dq, b, hk * G + g, t) + lane * EPL;
#pragma unroll
        for (int k = 0; k < EPL; ++k) stf<T>(dq + k, ldf<T>(dq + k) + acc[g][k] * p.scale);
    }
}

template <typename T, int HD>
static bool launch_depth_warp_hd(const BwdParams& p, cudaStream_t stream) {
    const long long n = static_cast<long long>(p.B) * p.Hk * p.T;
    const dim3 grid(static_cast<unsigned>((n + kDepthWarps - 1) / kDepthWarps)), block(kDepthWarps * 32);
#define MODA_DEPTH_CASE(GG, JJ)                                                              \
    if (p.G == GG && (p.L + 31) / 32 == JJ) {                                                 \
        moda_bwd_depth_warp_kernel<T, HD, GG, JJ><<<grid, block, 0, stream>>>(p);            \
        return true;                                                                          \
    }
    MODA_DEPTH_CASE(1, 1) MODA_DEPTH_CASE(2, 1) MODA_DEPTH_CASE(4, 1) MODA_DEPTH_CASE(8, 1)
    MODA_DEPTH_CASE(1, 2) MODA_DEPTH_CASE(2, 2) MODA_DEPTH_CASE(4, 2) MODA_DEPTH_CASE(8, 2)
#undef MODA_DEPTH_CASE
    return false;
}

// The warp-per-token kernel for 16-bit inputs with d in {64, 128}, G <= 8, L <= 64
// and 16-byte aligned unit-stride rows; false when it does not apply.
template <typename T>
static bool launch_depth_warp(const BwdParams& p, cudaStream_t stream) {
    if constexpr (sizeof(T) != 2) {
        return false;
    } else {
    if (p.L < 1 || p.L > 64) return false;
    const ModaTensor* ts[7] = {&p.q, &p.dout, &p.kd, &p.vd, &p.dkd, &p.dvd, &p.dq};
    for (const ModaTensor* x : ts) {
        if (x->strides[3] != 1 || reinterpret_cast<uintptr_t>(x->ptr) % 16 != 0) return false;
        for (int i = 0; i < 3; ++i)
            if (x->sizes[i] > 1 && (x->strides[i] * 2) % 16 != 0) return false;
    }
    if (p.d == 128) return launch_depth_warp_hd<T, 128>(p, stream);
    if (p.d == 64) return launch_depth_warp_hd<T, 64>(p, stream);
    return false;
    }
}

// ---------------------------------------------------------------- depth part, tensor cores
// One warp per 16-row block of query rows of one (batch, KV head): 16/G whole tokens
// (block row r is token t0 + r/G, query head hk*G + r%G). Per token of the block, with
// its depth rows staged in the warp's shared memory (cp.async) 32 at a time (P uses the
// forward's log-sum-exp, so key chunks are independent):
//   S = Q Kd^T, dP = dO Vd^T                 16 x 32, mma.sync m16n8k16, fp32 accumulate
//   P = exp(scale*S - lse), dS = P (dP - D)  the token's own rows; 0 for the others
//   dQ += scale * dS Kd                      added to the dQ the tcgen05 kernel wrote
//   dVd = P^T dO, dKd = scale * dS^T Q       32 x d (P and dS go through shared memory)
// Shared-memory rows of 128 bytes (64 columns) are stored with the 16-byte chunk index
// XORed with row % 8, so ldmatrix reads of 8 consecutive rows hit 8 different banks.
// Staging rows past a partial chunk are zeroed (their products must be finite).
constexpr int kDmWarps = 4;

template <int HD>
struct DmCfg {
    static constexpr int kBox16 = 16 * 128;             // 16 rows x 64 columns
    static constexpr int kBox32 = 32 * 128;             // 32 rows x 64 columns
    static constexpr int kQ = 0;                         // Q block   [HD/64][16][128 B]
    static constexpr int kDO = kQ + (HD / 64) * kBox16;  // dO block
    static constexpr int kK = kDO + (HD / 64) * kBox16;  // K_depth  [HD/64][32][128 B]
    static constexpr int kV = kK + (HD / 64) * kBox32;   // V_depth
    static constexpr int kP = kV + (HD / 64) * kBox32;   // P  [16][80 B] (32 keys, padded)
    static constexpr int kDS = kP + 16 * 80;             // dS
    static constexpr int kWarp = kDS + 16 * 80;          // bytes per warp
};

template <int FMT>
MODA_DEV void dm_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (FMT == 1)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7},"
            " {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7},"
            " {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
MODA_DEV void dm_ldsm(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
MODA_DEV void dm_ldsm_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
MODA_DEV uint32_t dm_sw(uint32_t base, int row, int chunk) {
    return base + row * 128 + (((chunk ^ row) & 7) << 4);
}
MODA_DEV void dm_cp16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
MODA_DEV void dm_cp_wait() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
template <int FMT>
MODA_DEV uint32_t dm_pack(float lo, float hi) {
    return FMT == 1 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}
template <int FMT>
MODA_DEV float2 dm_unpack(uint32_t w) {
    if constexpr (FMT == 1) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    return make_float2(__half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu))),
                       __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16))));
}

template <int HD, int FMT>
__global__ void __launch_bounds__(kDmWarps * 32) moda_bwd_depth_mma_kernel(const __grid_constant__ BwdParams p) {
    using C = DmCfg<HD>;
    extern __shared__ __align__(16) uint8_t dm_smem[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t base = smem_u32(dm_smem) + w * C::kWarp;
    const int G = p.G, L = p.L, T = p.T, Hk = p.Hk;
    const int tpg = 16 / G;
    const long long bpb = (static_cast<long long>(T) * G + 15) / 16;  // 16-row blocks per (b, KV head)
    const long long nblocks = static_cast<long long>(p.B) * Hk * bpb;
    const float sc2 = p.scale * kLog2e;
    for (int i = lane; i < (C::kP - C::kK) / 16; i += 32)
        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(base + C::kK + 16 * i), "r"(0u) : "memory");
    __syncwarp();
    const uint16_t* q = static_cast<const uint16_t*>(p.q.ptr);
    const uint16_t* dout = static_cast<const uint16_t*>(p.dout.ptr);
    const uint16_t* kd = static_cast<const uint16_t*>(p.kd.ptr);
    const uint16_t* vd = static_cast<const uint16_t*>(p.vd.ptr);
    uint16_t* dq = static_cast<uint16_t*>(p.dq.ptr);
    uint16_t* dkd = static_cast<uint16_t*>(p.dkd.ptr);
    uint16_t* dvd = static_cast<uint16_t*>(p.dvd.ptr);
    for (long long blk = static_cast<long long>(blockIdx.x) * kDmWarps + w; blk < nblocks;
         blk += static_cast<long long>(gridDim.x) * kDmWarps) {
        const int b = static_cast<int>(blk / (Hk * bpb));
        const int hk = static_cast<int>((blk / bpb) % Hk);
        const int t0 = static_cast<int>(blk % bpb) * tpg;
        // ---- stage the block's Q and dO rows
        for (int i = lane; i < 16 * (HD / 8); i += 32) {
            const int r = i / (HD / 8), ch = i % (HD / 8);
            int t = t0 + r / G;
            if (t >= T) t = t0;  // rows past T read a valid row and are never used
            const int h = hk * G + r % G;
            dm_cp16(dm_sw(base + C::kQ + (ch >> 3) * C::kBox16, r, ch & 7),
                    q + b * p.q.strides[0] + h * p.q.strides[1] + static_cast<long long>(t) * p.q.strides[2] + ch * 8);
            dm_cp16(dm_sw(base + C::kDO + (ch >> 3) * C::kBox16, r, ch & 7),
                    dout + b * p.dout.strides[0] + h * p.dout.strides[1] + static_cast<long long>(t) * p.dout.strides[2] + ch * 8);
        }
        // this thread's rows of the block: A = g, B = g + 8
        const int tA = t0 + g / G, tB = t0 + (g + 8) / G;
        const int hA = hk * G + g % G, hB = hk * G + (g + 8) % G;
        const bool vA = tA < T, vB = tB < T;
        const long long riA = (static_cast<long long>(b) * p.Hq + hA) * T + (vA ? tA : t0);
        const long long riB = (static_cast<long long>(b) * p.Hq + hB) * T + (vB ? tB : t0);
        const float lseA = p.lse[riA] * kLog2e, lseB = p.lse[riB] * kLog2e;
        const float dA = p.delta[riA], dB = p.delta[riB];
        for (int jc = 0; jc < tpg * ((L + 31) / 32); ++jc) {
            const int j = jc / ((L + 31) / 32);            // token of the block
            const int kc = 32 * (jc % ((L + 31) / 32));    // first depth row of the chunk
            const int t = t0 + j;
            if (t >= T) break;
            const int Lc = L - kc < 32 ? L - kc : 32;      // rows in this chunk
            const bool ownA = vA && g / G == j, ownB = vB && (g + 8) / G == j;
            // ---- stage the chunk's K_depth and V_depth rows (rows past Lc zeroed)
            const long long row0 = static_cast<long long>(t) * L + kc;
            if (Lc < 32) {
                for (int i = lane; i < (32 - Lc) * (HD / 8); i += 32) {
                    const int l = Lc + i / (HD / 8), ch = i % (HD / 8);
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dm_sw(base + C::kK + (ch >> 3) * C::kBox32, l, ch & 7)), "r"(0u) : "memory");
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dm_sw(base + C::kV + (ch >> 3) * C::kBox32, l, ch & 7)), "r"(0u) : "memory");
                }
            }
            for (int i = lane; i < Lc * (HD / 8); i += 32) {
                const int l = i / (HD / 8), ch = i % (HD / 8);
                dm_cp16(dm_sw(base + C::kK + (ch >> 3) * C::kBox32, l, ch & 7),
                        kd + b * p.kd.strides[0] + hk * p.kd.strides[1] + (row0 + l) * p.kd.strides[2] + ch * 8);
                dm_cp16(dm_sw(base + C::kV + (ch >> 3) * C::kBox32, l, ch & 7),
                        vd + b * p.vd.strides[0] + hk * p.vd.strides[1] + (row0 + l) * p.vd.strides[2] + ch * 8);
            }
            dm_cp_wait();
            __syncwarp();
            // ---- S = Q Kd^T and dP = dO Vd^T
            float sacc[4][4], pacc[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) sacc[nt][e] = pacc[nt][e] = 0.f;
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                uint32_t aq[4], ao[4];
                dm_ldsm(dm_sw(base + C::kQ + (ks >> 2) * C::kBox16, lane & 15, 2 * (ks & 3) + (lane >> 4)), aq);
                dm_ldsm(dm_sw(base + C::kDO + (ks >> 2) * C::kBox16, lane & 15, 2 * (ks & 3) + (lane >> 4)), ao);
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    if (16 * np >= Lc) break;
                    const int kr = 16 * np + (lane & 7) + 8 * (lane >> 4);
                    const int kc = 2 * (ks & 3) + ((lane >> 3) & 1);
                    uint32_t bk[4], bv[4];
                    dm_ldsm(dm_sw(base + C::kK + (ks >> 2) * C::kBox32, kr, kc), bk);
                    dm_ldsm(dm_sw(base + C::kV + (ks >> 2) * C::kBox32, kr, kc), bv);
                    dm_mma<FMT>(sacc[2 * np], aq, bk[0], bk[1]);
                    dm_mma<FMT>(sacc[2 * np + 1], aq, bk[2], bk[3]);
                    dm_mma<FMT>(pacc[2 * np], ao, bv[0], bv[1]);
                    dm_mma<FMT>(pacc[2 * np + 1], ao, bv[2], bv[3]);
                }
            }
            // ---- P and dS (the token's rows and keys < L only)
            uint32_t dsf[2][4];  // dS as 16-bit A fragments (keys 16u..16u+15)
            const uint32_t sP = base + C::kP, sDS = base + C::kDS;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                float pv[4], dv[4];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const bool ok = 8 * nt + 2 * c + e < Lc;
                    pv[e] = (ownA && ok) ? ex2(fmaf(sacc[nt][e], sc2, -lseA)) : 0.f;
                    pv[2 + e] = (ownB && ok) ? ex2(fmaf(sacc[nt][2 + e], sc2, -lseB)) : 0.f;
                    dv[e] = (ownA && ok) ? pv[e] * (pacc[nt][e] - dA) : 0.f;
                    dv[2 + e] = (ownB && ok) ? pv[2 + e] * (pacc[nt][2 + e] - dB) : 0.f;
                }
                dsf[nt >> 1][(nt & 1) * 2] = dm_pack<FMT>(dv[0], dv[1]);
                dsf[nt >> 1][(nt & 1) * 2 + 1] = dm_pack<FMT>(dv[2], dv[3]);
                const int col = 2 * (8 * nt + 2 * c);  // byte offset of keys 8nt + 2c, +1
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(sP + g * 80 + col), "r"(dm_pack<FMT>(pv[0], pv[1])) : "memory");
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(sP + (g + 8) * 80 + col), "r"(dm_pack<FMT>(pv[2], pv[3])) : "memory");
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(sDS + g * 80 + col), "r"(dsf[nt >> 1][(nt & 1) * 2]) : "memory");
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(sDS + (g + 8) * 80 + col), "r"(dsf[nt >> 1][(nt & 1) * 2 + 1]) : "memory");
            }
            __syncwarp();
            // ---- dQ += scale * dS Kd, 32 columns at a time
#pragma unroll
            for (int q4 = 0; q4 < HD / 32; ++q4) {
                float o[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    if (16 * u >= Lc) break;
#pragma unroll
                    for (int hp = 0; hp < 2; ++hp) {
                        const int ch = 4 * q4 + 2 * hp + (lane >> 4);
                        uint32_t bk[4];
                        dm_ldsm_t(dm_sw(base + C::kK + (ch >> 3) * C::kBox32, 16 * u + (lane & 7) + 8 * ((lane >> 3) & 1), ch & 7), bk);
                        dm_mma<FMT>(o[2 * hp], dsf[u], bk[0], bk[1]);
                        dm_mma<FMT>(o[2 * hp + 1], dsf[u], bk[2], bk[3]);
                    }
                }
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    if (!(rr == 0 ? ownA : ownB)) continue;
                    uint16_t* row = dq + b * p.dq.strides[0] + (rr == 0 ? hA : hB) * p.dq.strides[1] +
                                    static_cast<long long>(t) * p.dq.strides[2];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t* cell = reinterpret_cast<uint32_t*>(row + 8 * (4 * q4 + i) + 2 * c);
                        const float2 old = dm_unpack<FMT>(*cell);
                        *cell = dm_pack<FMT>(fmaf(o[i][2 * rr], p.scale, old.x), fmaf(o[i][2 * rr + 1], p.scale, old.y));
                    }
                }
            }
            // ---- dVd = P^T dO and dKd = scale * dS^T Q, keys 16m..16m+15
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                if (16 * m >= Lc) break;
                uint32_t pa[4], da[4];
                const int ar = (lane & 7) + 8 * (lane >> 4);
                const int ac = 2 * m + ((lane >> 3) & 1);
                dm_ldsm_t(sP + ar * 80 + ac * 16, pa);
                dm_ldsm_t(sDS + ar * 80 + ac * 16, da);
#pragma unroll
                for (int q4 = 0; q4 < HD / 32; ++q4) {
                    float ov[4][4], ok[4][4];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
#pragma unroll
                        for (int e = 0; e < 4; ++e) ov[i][e] = ok[i][e] = 0.f;
#pragma unroll
                    for (int hp = 0; hp < 2; ++hp) {
                        const int ch = 4 * q4 + 2 * hp + (lane >> 4);
                        const int br = (lane & 7) + 8 * ((lane >> 3) & 1);
                        uint32_t bo[4], bq[4];
                        dm_ldsm_t(dm_sw(base + C::kDO + (ch >> 3) * C::kBox16, br, ch & 7), bo);
                        dm_ldsm_t(dm_sw(base + C::kQ + (ch >> 3) * C::kBox16, br, ch & 7), bq);
                        dm_mma<FMT>(ov[2 * hp], pa, bo[0], bo[1]);
                        dm_mma<FMT>(ov[2 * hp + 1], pa, bo[2], bo[3]);
                        dm_mma<FMT>(ok[2 * hp], da, bq[0], bq[1]);
                        dm_mma<FMT>(ok[2 * hp + 1], da, bq[2], bq[3]);
                    }
                    // ov / ok [i]: keys 16m + g (0,1) and 16m + g + 8 (2,3), columns 8(4q4+i) + 2c, +1
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const int key = 16 * m + g + 8 * kk;
                        if (key >= Lc) continue;
                        uint16_t* vrow = dvd + b * p.dvd.strides[0] + hk * p.dvd.strides[1] + (row0 + key) * p.dvd.strides[2];
                        uint16_t* krow = dkd + b * p.dkd.strides[0] + hk * p.dkd.strides[1] + (row0 + key) * p.dkd.strides[2];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int col = 8 * (4 * q4 + i) + 2 * c;
                            *reinterpret_cast<uint32_t*>(vrow + col) = dm_pack<FMT>(ov[i][2 * kk], ov[i][2 * kk + 1]);
                            *reinterpret_cast<uint32_t*>(krow + col) =
                                dm_pack<FMT>(ok[i][2 * kk] * p.scale, ok[i][2 * kk + 1] * p.scale);
                        }
                    }
                }
            }
            __syncwarp();  // every lane is done with this token's staging before the next copies
        }
        __syncwarp();  // and with the block's Q / dO before the next block's copies
    }
}

template <int HD>
static bool launch_depth_mma_hd(const BwdParams& p, cudaStream_t stream) {
    using C = DmCfg<HD>;
    const long long bpb = (static_cast<long long>(p.T) * p.G + 15) / 16;
    const long long n = static_cast<long long>(p.B) * p.Hk * bpb;
    const long long want = (n + kDmWarps - 1) / kDmWarps;
    const int grid = static_cast<int>(want < 2LL * sm_count() ? want : 2LL * sm_count());
    const int smem = kDmWarps * C::kWarp;
    static std::atomic<uint64_t> done_bf16{0}, done_f16{0};
    auto launch = [&](auto kern, std::atomic<uint64_t>& done) {
        if (ensure_smem_attr(done, kern, smem) != cudaSuccess) return false;
        kern<<<grid, kDmWarps * 32, smem, stream>>>(p);
        return true;
    };
    return p.dtype == MODA_BF16 ? launch(moda_bwd_depth_mma_kernel<HD, 1>, done_bf16)
                                : launch(moda_bwd_depth_mma_kernel<HD, 0>, done_f16);
}

// The tensor-core depth kernel for 16-bit inputs with d in {64, 128}, whole tokens per
// 16-row block (16 % G == 0) and 16-byte aligned unit-stride rows; any L.
static bool launch_depth_mma(const BwdParams& p, cudaStream_t stream) {
    if (p.dtype != MODA_BF16 && p.dtype != MODA_F16) return false;
    if (p.L < 1 || p.G < 1 || 16 % p.G != 0) return false;
    const ModaTensor* ts[7] = {&p.q, &p.dout, &p.kd, &p.vd, &p.dkd, &p.dvd, &p.dq};
    for (const ModaTensor* x : ts) {
        if (x->strides[3] != 1 || reinterpret_cast<uintptr_t>(x->ptr) % 16 != 0) return false;
        for (int i = 0; i < 3; ++i)
            if (x->sizes[i] > 1 && (x->strides[i] * 2) % 16 != 0) return false;
    }
    if (p.d == 128) return launch_depth_mma_hd<128>(p, stream);
    if (p.d == 64) return launch_depth_mma_hd<64>(p, stream);
    return false;
}

// Zero gradient for depth rows the forward never reads (rows >= T*L).
template <typename T>
__global__ void moda_bwd_zero_rows_kernel(const __grid_constant__ BwdParams p, long long r_lo) {
    const long long r = r_lo + blockIdx.x;
    const int hk = blockIdx.y, b = blockIdx.z;
    for (int e = threadIdx.x; e < p.d; e += blockDim.x) {
        stf<T>(rowp<T>(p.dkd, b, hk, r) + e * p.dkd.strides[3], 0.f);
        stf<T>(rowp<T>(p.dvd, b, hk, r) + e * p.dvd.strides[3], 0.f);
    }
}

size_t depth_token_smem(int G, int L, int d) {
    const int LC = L < kDepthChunk ? L : kDepthChunk;
    return sizeof(float) * (static_cast<size_t>(2 * LC + 2 * G) * (d + 1) + static_cast<size_t>(G) * d +
                            2 * static_cast<size_t>(G) * LC + 2 * static_cast<size_t>(G));
}

template <typename T>
static int launch_depth_t(const BwdParams& p, cudaStream_t stream) {
    if (p.L > 0 && p.T > 0 && !launch_depth_mma(p, stream) && !launch_depth_warp<T>(p, stream)) {
        const size_t sm = depth_token_smem(p.G, p.L, p.d);
        if (sm > 48 * 1024 &&
            cudaFuncSetAttribute(moda_bwd_depth_token_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sm)) != cudaSuccess)
            return MODA_ERR_LAUNCH;
        moda_bwd_depth_token_kernel<T><<<dim3(p.T, p.Hk, p.B), 128, sm, stream>>>(p);
    }
    const long long used = static_cast<long long>(p.T) * p.L;
    if (p.R > used)
        moda_bwd_zero_rows_kernel<T><<<dim3(static_cast<unsigned>(p.R - used), p.Hk, p.B), 64, 0, stream>>>(p, used);
    return MODA_OK;
}

int launch_bwd_depth(const BwdParams& p, cudaStream_t stream) {
    switch (p.dtype) {
        case MODA_F32: return launch_depth_t<float>(p, stream);
        case MODA_BF16: return launch_depth_t<__nv_bfloat16>(p, stream);
        case MODA_F16: return launch_depth_t<__half>(p, stream);
        default: return MODA_ERR_DTYPE;
    }
}

bool bwd_depth_supported(const BwdParams& p) {
    return depth_token_smem(p.G, p.L, p.d) <= 200 * 1024 && p.R - static_cast<long long>(p.T) * p.L < (1LL << 31);
}

// ---------------------------------------------------------------- host side
bool tc_bwd_supports(const BwdParams& p, char* why, size_t whylen) {
    auto no = [&](const char* m) {
        snprintf(why, whylen, "%s", m);
        return false;
    };
    if (p.dtype != MODA_BF16 && p.dtype != MODA_F16) return no("tcgen05 backward needs bf16 or f16");
    if (p.d != 64 && p.d != 128) return no("tcgen05 backward needs head_dim 64 or 128");
    if (p.G < 1 || (128 % p.G) != 0) return no("tcgen05 backward needs H_q/H_k dividing 128");
    if (!bwd_depth_supported(p)) return no("depth part too large for the per-token kernel");
    if (!(p.scale > 0.f)) return no("tcgen05 backward needs a positive scale");
    const ModaTensor* ts[7] = {&p.q, &p.k, &p.v, &p.dout, &p.dq, &p.dk, &p.dv};
    for (const ModaTensor* t : ts) {
        if (t->strides[3] != 1) return no("tcgen05 backward needs unit stride along head_dim");
        if (reinterpret_cast<uintptr_t>(t->ptr) % 16 != 0) return no("tcgen05 backward needs 16-byte aligned tensors");
        for (int i = 0; i < 3; ++i)
            if (t->sizes[i] > 1 && (t->strides[i] * 2) % 16 != 0)
                return no("tcgen05 backward needs 16-byte multiple strides");
    }
    return true;
}

cudaError_t read_and_clear_bwd_status(cudaStream_t stream, int* value) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(value, moda_bwd_status, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && *value != 0) {
        static const int zero = 0;
        e = cudaMemcpyToSymbolAsync(moda_bwd_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                    stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    }
    return e;
}

template <int HD, int FMT, int MODE>
static int launch_bwd_inst(const TcBwdParams& tp, int items, cudaStream_t stream) {
    using Cfg = BwdCfg<HD>;
    auto kern = moda_bwd_tc_kernel<HD, FMT, MODE>;
    static std::atomic<uint64_t> attr_done{0};
    if (ensure_smem_attr(attr_done, kern, Cfg::kSmem) != cudaSuccess) return MODA_ERR_LAUNCH;
    if (items == 0) return MODA_OK;
    const int grid = items < sm_count() ? items : sm_count();
    kern<<<grid, kBThreads, Cfg::kSmem, stream>>>(tp);
    return MODA_OK;
}

template <int HD, int FMT>
static int launch_bwd_pair(TcBwdParams& tp, cudaStream_t stream) {
    const int bh = tp.B * tp.Hk;
    tp.num_items = tp.num_ktiles * bh;
    int r = launch_bwd_inst<HD, FMT, MODE_DKDV>(tp, tp.num_items, stream);
    if (r != MODA_OK) return r;
    tp.num_items = tp.num_qtiles * bh;
    return launch_bwd_inst<HD, FMT, MODE_DQ>(tp, tp.num_items, stream);
}

int launch_bwd_tc(const BwdParams& p, cudaStream_t stream, char* err, size_t errlen) {
    TcBwdParams tp;
    const CUtensorMapDataType dt =
        p.dtype == MODA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int n_tok = 128 / p.G;
    if (!encode_map(&tp.tm_q, p.q, p.T, true, 2, dt, p.G, n_tok, err, errlen, "Q") ||
        !encode_map(&tp.tm_do, p.dout, p.T, true, 2, dt, p.G, n_tok, err, errlen, "dO") ||
        !encode_map(&tp.tm_k, p.k, p.T, false, 2, dt, kBRows, 1, err, errlen, "K") ||
        !encode_map(&tp.tm_v, p.v, p.T, false, 2, dt, kBRows, 1, err, errlen, "V"))
        return MODA_ERR_LAUNCH;
    tp.lse = p.lse;
    tp.delta = p.delta;
    tp.dq = p.dq.ptr;
    tp.dq_sb = p.dq.strides[0]; tp.dq_sh = p.dq.strides[1]; tp.dq_st = p.dq.strides[2];
    tp.dk = p.dk.ptr;
    tp.dk_sb = p.dk.strides[0]; tp.dk_sh = p.dk.strides[1]; tp.dk_st = p.dk.strides[2];
    tp.dv = p.dv.ptr;
    tp.dv_sb = p.dv.strides[0]; tp.dv_sh = p.dv.strides[1]; tp.dv_st = p.dv.strides[2];
    tp.B = p.B; tp.Hq = p.Hq; tp.Hk = p.Hk; tp.G = p.G; tp.T = p.T;
    tp.n_tok = n_tok;
    tp.num_qtiles = (p.T + n_tok - 1) / n_tok;
    tp.num_ktiles = (p.T + kBRows - 1) / kBRows;
    tp.sc = p.scale * kLog2e;
    tp.scale = p.scale;
    const long long items = static_cast<long long>(tp.num_qtiles) * p.B * p.Hk;
    if (items > 0x7fffffffLL) {
        snprintf(err, errlen, "too many work items");
        return MODA_ERR_UNSUPPORTED;
    }
    if (p.d == 128)
        return p.dtype == MODA_BF16 ? launch_bwd_pair<128, 1>(tp, stream) : launch_bwd_pair<128, 0>(tp, stream);
    return p.dtype == MODA_BF16 ? launch_bwd_pair<64, 1>(tp, stream) : launch_bwd_pair<64, 0>(tp, stream);
}

}  // namespace moda
