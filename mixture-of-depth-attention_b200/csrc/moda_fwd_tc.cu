// Fused MoDA forward on Blackwell tensor cores: TMA -> tcgen05.mma -> TMEM.
//
// Semantics (moda/kernels/moda_naive.py:13-97): for query row (b, h, t)
//   out = softmax({scale*q.k_j : j <= t} U {scale*q.kd_{t*L+l} : l < L}) . [V ; V_depth]
// with KV head h / G. One online softmax covers both score sets.
//
// Work decomposition.
//   * A query tile is 128 rows of one (batch, KV head): n = 128/G tokens x the G
//     query heads of that KV head, token-major (row = token_local*G + head). The
//     TMA box (64, G, n) over the [d, H_q, T, B] view builds it, so every K/V
//     tile is used once by all G heads of its group -- GQA without
//     repeat_interleave.
//   * A work item is a pair of consecutive query tiles (A, B) of one (b, KV head).
//     The kernel is persistent: one CTA per SM walks the items, sorted heaviest
//     first (most causal blocks first), in serpentine rounds (see round_item), so
//     the producer already streams the next item while the current one drains.
//   * Each item walks one list of 128-row key blocks shared by both tiles:
//       - causal sequence blocks j = 0..S-1 (keys [128j, 128j+128)), masked on the
//         diagonal; both tiles read the same K/V fill;
//       - depth blocks k = 0..D-1: rows [t0*L + 128k, +128) of K_depth/V_depth,
//         i.e. only the rows of the tile's own tokens (chunk-aware: a tile of n
//         tokens touches n*L depth rows), masked so a row of token t keeps rows
//         t*L..t*L+L-1 (the paper's depth mask floor(row/G) == floor(j/L));
//     depth blocks are spread evenly between the causal blocks so the HBM-heavy
//     depth stream overlaps the compute-heavy causal part.
//   * Every block goes through the same two MMAs, S = Q K^T (A and B from shared
//     memory) and O += P V (P from tensor memory), and the same online softmax.
//
// Warp roles (640 threads = 5 warpgroups):
//   warps 0-7   softmax for tile A: warp w covers TMEM lane quarter w%4 (32 rows) and
//               score columns [64*(w/4), +64); the two warps of a quarter trade row
//               maxima and sums through shared memory (one named barrier per pair)
//   warps 8-15  the same for tile B
//   warp  16    TMA producer (Q tiles, then the K/V block ring)
//   warp  17    TMEM allocator and tcgen05.mma issuer for tile A (one thread)
//   warp  18    tcgen05.mma issuer for tile B (one thread)
//   warp  19    idle
// Two softmax warps per tile and lane quarter keep the MUFU (one ex2 per score)
// and the tensor core busy at the same time: a single warp per quarter is
// latency-bound. One MMA issuer per tile keeps each tile's barrier latencies off
// the other tile's critical path; an issuer checks the ring slots of its next
// MMAs while the softmax of the current block is still running.
// Registers: launched at 96 per thread; the producer/MMA warpgroup gives back to
// 56 and the four softmax warpgroups grow to 104 (4*128*104 + 128*56 <= 640*96).
//
// TMEM (512 columns): S_A [0,128) S_B [128,256) O_A [256,256+d) O_B [256+d,256+2d).
// P (16-bit) is written into the upper 64 columns of S and fed to the PV MMA
// straight from TMEM, so P never touches shared memory.
#include "moda_internal.h"

#include <cstdio>

namespace moda {

constexpr int kThreads = 640;
constexpr int kLaunchRegs = 96;    // 65536 / 640 rounded down to 8, enforced on the host
constexpr int kSoftmaxRegs = 104;
constexpr int kProducerRegs = 56;
static_assert(4 * 128 * kSoftmaxRegs + 128 * kProducerRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int kWarpProducer = 16, kWarpMmaA = 17, kWarpMmaB = 18;
constexpr int kBM = 128;  // query rows per tile
constexpr int kBN = 128;  // key rows per block

template <int HD>
struct TcCfg {
    static constexpr int kTileBytes = kBM * HD * 2;       // one 128 x HD 16-bit tile
    static constexpr int kColBlocks = HD / 64;            // 128-byte swizzle atoms across d
    static constexpr int kStages = (HD == 128) ? 4 : 10;  // K/V ring depth
    static constexpr int kQOff = 0;
    static constexpr int kRingOff = 2 * kTileBytes;
    static constexpr int kBarOff = kRingOff + kStages * kTileBytes;
    // barriers: q_full[2] q_empty[2] s_full[2] p_full[2] o_done[2] o_free[2] end[2],
    //           slot_full[S] slot_empty_A[S] slot_empty_B[S]
    static constexpr int kNumBars = 14 + 3 * kStages;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    // row-max exchange [tile][block parity][half][row] and row-sum exchange [tile][half][row]
    static constexpr int kXmaxOff = (kMiscOff + 48 + 15) & ~15;
    static constexpr int kXsumOff = kXmaxOff + 2 * 2 * 2 * 128 * 4;
    static constexpr int kSmemBytes = kXsumOff + 2 * 2 * 128 * 4 + 1024;  // + alignment slack
    static constexpr uint32_t kTmemCols = 512;
    static constexpr uint32_t kOCol = 256;
};

struct TileInfo {
    int t0;    // first token
    int tend;  // one past the last valid token (<= T)
    int ndep;  // depth blocks
    int nseq;  // causal sequence blocks
    __device__ int len() const { return ndep + nseq; }
};

__device__ __forceinline__ TileInfo tile_info(const TcParams& p, int pair, int x) {
    TileInfo ti;
    ti.t0 = (pair * 2 + x) * p.n_tok;
    if (ti.t0 >= p.T) {
        ti.tend = ti.t0;
        ti.ndep = ti.nseq = 0;
        return ti;
    }
    ti.tend = min(p.T, ti.t0 + p.n_tok);
    ti.nseq = (ti.tend + kBN - 1) / kBN;
    ti.ndep = static_cast<int>(((static_cast<long long>(ti.tend - ti.t0) * p.L) + kBN - 1) / kBN);
    return ti;
}

struct Item {
    int b, hk;
    TileInfo t[2];
    int S, D;  // causal / depth blocks of the item (max over its tiles)
    __device__ int nsteps() const { return S + D; }
};

__device__ __forceinline__ Item item_info(const TcParams& p, int item) {
    Item it;
    const int bh_count = p.B * p.Hk;
    const int pair = p.num_pairs - 1 - item / bh_count;  // heaviest pairs first
    const int bh = item % bh_count;
    it.b = bh / p.Hk;
    it.hk = bh % p.Hk;
    it.t[0] = tile_info(p, pair, 0);
    it.t[1] = tile_info(p, pair, 1);
    it.S = max(it.t[0].nseq, it.t[1].nseq);
    it.D = max(it.t[0].ndep, it.t[1].ndep);
    return it;
}

// One step of an item's block list. Depth block k is placed before causal block j
// when k/D <= j/S, which spreads the D depth blocks evenly over the S causal ones.
struct Step {
    bool dep;
    int idx;
    bool has[2];
};

struct StepWalker {
    int S, D, j, k;
    __device__ StepWalker(const Item& it) : S(it.S), D(it.D), j(0), k(0) {}
    __device__ Step next(const Item& it) {
        Step st;
        st.dep = k < D && (j >= S || static_cast<long long>(k) * S <= static_cast<long long>(j) * D);
        st.idx = st.dep ? k++ : j++;
        for (int x = 0; x < 2; ++x)
            st.has[x] = st.dep ? st.idx < it.t[x].ndep : st.idx < it.t[x].nseq;
        return st;
    }
};

// Ring fills of one step, in fill order K_A, K_B, V_A, V_B; a causal block read
// by both tiles is filled once.
struct Fills {
    bool shared;
    uint32_t k[2], v[2], n;
};

__device__ __forceinline__ Fills step_fills(const Step& st, uint32_t base) {
    Fills r;
    r.shared = !st.dep && st.has[0] && st.has[1];
    uint32_t f = base;
    r.k[0] = r.k[1] = r.v[0] = r.v[1] = 0;
    if (st.has[0]) r.k[0] = f++;
    if (st.has[1]) r.k[1] = r.shared ? r.k[0] : f++;
    if (st.has[0]) r.v[0] = f++;
    if (st.has[1]) r.v[1] = r.shared ? r.v[0] : f++;
    r.n = f - base;
    return r;
}

// DG: width of the column groups a depth window is picked by (16, or 8 for L a multiple
// of 8 but not of 16, so that such L also avoid the per-score depth mask).
template <int HD, int FMT, int DG>
__global__ void __launch_bounds__(kThreads, 1) moda_fwd_tc_kernel(const __grid_constant__ TcParams p) {
    using Cfg = TcCfg<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sQ = sbase + Cfg::kQOff;
    const uint32_t sRing = sbase + Cfg::kRingOff;
    const uint32_t bar0 = sbase + Cfg::kBarOff;
    auto q_full = [&](int x) { return bar0 + 8u * x; };
    auto q_empty = [&](int x) { return bar0 + 8u * (2 + x); };
    auto s_full = [&](int x) { return bar0 + 8u * (4 + x); };
    auto p_full = [&](int x) { return bar0 + 8u * (6 + x); };
    auto o_done = [&](int x) { return bar0 + 8u * (8 + x); };
    auto o_free = [&](int x) { return bar0 + 8u * (10 + x); };
    auto end_bar = [&](int x) { return bar0 + 8u * (12 + x); };
    auto slot_full = [&](uint32_t i) { return bar0 + 8u * (14 + i); };
    // released by tile x's issuer once its MMAs reading the slot have completed
    auto slot_empty = [&](int x, uint32_t i) { return bar0 + 8u * (14 + (1 + x) * Cfg::kStages + i); };
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOff);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kMiscOff + 8);
    // Fills whose TMA loads the producer has started. An issuer looks at a slot's
    // barrier only for an issued fill: then the slot's previous fill has landed
    // and been released, so the barrier is exactly at this fill's phase (the
    // 1-bit parity cannot alias a fill two phases old).
    volatile uint32_t* issued = reinterpret_cast<volatile uint32_t*>(smem + Cfg::kMiscOff + 16);
    // Exponential-phase turns of the two tiles: 8 increments (one per softmax warp) per
    // block whose exponentials are done. A tile starts the exponentials of a block once
    // the other tile has finished every block that precedes it in the item's step order,
    // so the two tiles take turns on the MUFU while the tensor core runs the other tile.
    // Purely a scheduling hint: the result does not depend on it.
    uint32_t* exp_turns = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOff + 24);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // Items in serpentine order: round r hands the CTAs items [r*grid, (r+1)*grid) in
    // CTA order for even r and in reverse for odd r. Items are sorted heaviest first, so
    // a fixed stride would give CTA 0 the heaviest item of every round; alternating the
    // direction pairs a heavier item with a lighter one. Every role of the CTA walks the
    // same sequence.
    auto round_item = [&](int round) {
        const int g = static_cast<int>(gridDim.x);
        return round * g + ((round & 1) ? g - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x));
    };

    if (threadIdx.x == 0) {
        for (int x = 0; x < 2; ++x) {
            mbar_init(q_full(x), 1);
            mbar_init(q_empty(x), 1);
            mbar_init(s_full(x), 1);
            mbar_init(p_full(x), 2 * kBM);
            mbar_init(o_done(x), 1);
            mbar_init(o_free(x), 2 * kBM);
        }
        mbar_init(end_bar(0), 1);
        mbar_init(end_bar(1), 1);
        for (int i = 0; i < Cfg::kStages; ++i) {
            mbar_init(slot_full(i), 1);
            mbar_init(slot_empty(0, i), 1);
            mbar_init(slot_empty(1, i), 1);
        }
        *abort_flag = 0;
        *issued = 0;
        exp_turns[0] = 0;
        exp_turns[1] = 0;
        fence_barrier_init();
    }
    if (warp == kWarpMmaA) {
        tmem_alloc(smem_u32(tmem_holder), Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == kWarpProducer && lane == 0) {
        tma_prefetch_desc(&p.tm_q);
        tma_prefetch_desc(&p.tm_k);
        tma_prefetch_desc(&p.tm_v);
        tma_prefetch_desc(&p.tm_kd);
        tma_prefetch_desc(&p.tm_vd);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    constexpr uint32_t kBytes = Cfg::kTileBytes;

    if (warp >= kWarpProducer) {
        reg_dealloc<kProducerRegs>();
        if (warp == kWarpProducer && lane == 0) {
            // ------------------------------------------------------------ TMA producer
            uint32_t f = 0;          // fills issued (ring position)
            uint32_t quse[2] = {0, 0};
            // per slot: which tiles read its current fill (2 bits), and the parity of
            // the next release to wait for from each tile (1 bit per slot)
            uint32_t cons = 0, par_a = 0, par_b = 0;
            bool ok = true;
            for (int round = 0, item = round_item(0); item < p.num_items && ok; item = round_item(++round)) {
                const Item it = item_info(p, item);
#pragma unroll
                for (int x = 0; x < 2; ++x) {
                    if (!ok || it.t[x].len() == 0) continue;
                    ok = mbar_wait(q_empty(x), (quse[x] & 1u) ^ 1u, abort_flag, 1);
                    if (!ok) continue;
                    mbar_expect_tx(q_full(x), kBytes);
                    for (int cb = 0; cb < Cfg::kColBlocks; ++cb)
                        tma_load_4d(&p.tm_q, sQ + x * kBytes + cb * 16384, q_full(x), cb * 64,
                                    it.hk * p.G, it.t[x].t0, it.b);
                    ++quse[x];
                }
                StepWalker w(it);
                for (int s = 0; s < it.nsteps() && ok; ++s) {
                    const Step st = w.next(it);
                    const Fills fl = step_fills(st, f);
                    // fill order: K_A, K_B, V_A, V_B (a shared causal block is filled once)
#pragma unroll
                    for (int kv = 0; kv < 2; ++kv) {
#pragma unroll
                        for (int x = 0; x < 2; ++x) {
                            if (!ok || !st.has[x] || (x == 1 && fl.shared)) continue;
                            const uint32_t fi = kv == 0 ? fl.k[x] : fl.v[x];
                            const uint32_t slot = fi % Cfg::kStages;
                            // wait until every tile that read the slot's previous fill released it
                            const uint32_t prev = (cons >> (2 * slot)) & 3u;
                            if (prev & 1u) {
                                ok = ok && mbar_wait(slot_empty(0, slot), (par_a >> slot) & 1u, abort_flag, 2);
                                par_a ^= 1u << slot;
                            }
                            if (prev & 2u) {
                                ok = ok && mbar_wait(slot_empty(1, slot), (par_b >> slot) & 1u, abort_flag, 2);
                                par_b ^= 1u << slot;
                            }
                            if (!ok) continue;
                            const uint32_t readers = fl.shared ? 3u : (1u << x);
                            cons = (cons & ~(3u << (2 * slot))) | (readers << (2 * slot));
                            const CUtensorMap* m;
                            int row0;
                            if (st.dep) {
                                m = kv == 0 ? &p.tm_kd : &p.tm_vd;
                                row0 = it.t[x].t0 * p.L + kBN * st.idx;
                            } else {
                                m = kv == 0 ? &p.tm_k : &p.tm_v;
                                row0 = kBN * st.idx;
                            }
                            mbar_expect_tx(slot_full(slot), kBytes);
                            for (int cb = 0; cb < Cfg::kColBlocks; ++cb)
                                tma_load_4d(m, sRing + slot * kBytes + cb * 16384, slot_full(slot),
                                            cb * 64, row0, it.hk, it.b);
                            *issued = fi + 1;
                        }
                    }
                    if (ok) f += fl.n;
                }
            }
            // Exit path: loads still in flight must land before shared memory is released
            // (a no-op when everything was consumed).
            const uint32_t first = f > Cfg::kStages ? f - Cfg::kStages : 0;
            for (uint32_t fi = first; fi < f; ++fi)
                mbar_wait_drain(slot_full(fi % Cfg::kStages), (fi / Cfg::kStages) & 1u);
            for (int x = 0; x < 2; ++x)
                if (quse[x] > 0) mbar_wait_drain(q_full(x), (quse[x] - 1) & 1u);
        } else if ((warp == kWarpMmaA || warp == kWarpMmaB) && lane == 0) {
            // ------------------------------------------------------------ MMA issuer (tile x)
            const int x = warp - kWarpMmaA;
            constexpr uint32_t idesc_s = make_idesc(FMT, kBM, kBN, 0);
            constexpr uint32_t idesc_pv = make_idesc(FMT, kBM, HD, 1);
            // Descriptors are built once; each MMA advances the start address with a
            // single 32-bit add (K-major Q/K: 32 B per 16-wide k step inside a 128-byte
            // swizzle atom, 16 KB per atom; V MN-major: 2 KB per 16 key rows).
            constexpr uint32_t hi = desc_hi_sw128(1024);
            const uint32_t qa = desc_lo(sQ + x * kBytes, 16);
            const uint32_t ring_lo_k = desc_lo(sRing, 16);
            const uint32_t ring_lo_v = desc_lo(sRing, 128 * 128);
            constexpr uint32_t kSlotStep = kBytes >> 4;  // descriptor units per ring slot
            const uint32_t s_tm = tmem + x * 128;
            const uint32_t p_tm = s_tm + 64;
            const uint32_t o_tm = tmem + Cfg::kOCol + x * HD;
            const uint32_t rel_bar0 = slot_empty(x, 0);

            auto wait_issued = [&](uint32_t fi) {
                if (*issued > fi) return true;
                const long long t0 = clock64();
                for (uint32_t i = 1;; ++i) {
                    if (*issued > fi) return true;
                    if ((i & 255u) == 0) {
                        if (*abort_flag) return false;
                        if (clock64() - t0 > kWaitLimitCycles) {
                            *abort_flag = 1;
                            atomicCAS(&moda_dev_status, 0, 0x100 | 11);
                            return false;
                        }
                    }
                }
            };
            auto wait_full = [&](uint32_t fi) {
                return wait_issued(fi) &&
                       mbar_wait(slot_full(fi % Cfg::kStages), (fi / Cfg::kStages) & 1u, abort_flag, 3);
            };
            auto issue_s = [&](uint32_t fi) {
                const uint32_t kb = ring_lo_k + (fi % Cfg::kStages) * kSlotStep;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                    mma_ss(s_tm, desc_join(qa + off, hi), desc_join(kb + off, hi), idesc_s, kk > 0);
                }
                mma_commit(s_full(x));
                mma_commit(rel_bar0 + 8u * (fi % Cfg::kStages));
            };
            auto issue_pv = [&](uint32_t fi, bool first) {
                const uint32_t vb = ring_lo_v + (fi % Cfg::kStages) * kSlotStep;
                mma_ts(o_tm, p_tm, desc_join(vb, hi), idesc_pv, first ? 0u : 1u);
#pragma unroll
                for (int kk = 1; kk < kBN / 16; ++kk)
                    mma_ts(o_tm, p_tm + kk * 8, desc_join(vb + ((kk * 2048) >> 4), hi), idesc_pv, 1u);
                mma_commit(rel_bar0 + 8u * (fi % Cfg::kStages));
            };

            uint32_t f = 0;       // ring position (same fill sequence as the producer)
            uint32_t pcnt = 0;    // P blocks consumed
            uint32_t items = 0;   // items of this tile started
            bool ok = true;
            for (int round = 0, item = round_item(0); item < p.num_items && ok; item = round_item(++round)) {
                const Item it = item_info(p, item);
                const TileInfo ti = x == 0 ? it.t[0] : it.t[1];
                if (ti.len() == 0) {
                    // still walk the fills so the ring position stays in step with the producer
                    StepWalker w(it);
                    for (int s = 0; s < it.nsteps(); ++s) f += step_fills(w.next(it), f).n;
                    continue;
                }
                // Blocks of this tile in step order; the walker runs one block ahead.
                StepWalker w(it);
                uint32_t fcur = f;
                Step st;
                Fills fl;
                // advance to this tile's first block
                do {
                    st = w.next(it);
                    fl = step_fills(st, fcur);
                    if (!(x == 0 ? st.has[0] : st.has[1])) fcur += fl.n;
                } while (!(x == 0 ? st.has[0] : st.has[1]));
                int steps_left = it.nsteps() - (w.j + w.k);
                uint32_t kf = x == 0 ? fl.k[0] : fl.k[1];
                uint32_t vf = x == 0 ? fl.v[0] : fl.v[1];
                ok = mbar_wait(q_full(x), items & 1u, abort_flag, 5) && wait_full(kf);
                if (!ok) break;
                tc_fence_after();
                issue_s(kf);
                fcur += fl.n;
                for (int b = 0; b < ti.len() && ok; ++b) {
                    // find the next block of this tile (if any) and its fills
                    bool has_next = false;
                    uint32_t kf_next = 0, vf_next = 0;
                    while (steps_left > 0) {
                        const Step sn = w.next(it);
                        const Fills fn = step_fills(sn, fcur);
                        --steps_left;
                        fcur += fn.n;
                        if (x == 0 ? sn.has[0] : sn.has[1]) {
                            has_next = true;
                            kf_next = x == 0 ? fn.k[0] : fn.k[1];
                            vf_next = x == 0 ? fn.v[0] : fn.v[1];
                            break;
                        }
                    }
                    // This block's V slot first (normally loaded long ago), then the softmax's
                    // P. The next K slot is only probed here: blocking on it before the PV
                    // below releases this block's V slot could deadlock the ring when the
                    // next block is more than a ring's length of fills ahead.
                    ok = wait_full(vf);
                    const bool k_ready = ok && has_next && *issued > kf_next &&
                                         mbar_test(slot_full(kf_next % Cfg::kStages),
                                                   (kf_next / Cfg::kStages) & 1u);
                    ok = ok && mbar_wait_hot(p_full(x), pcnt & 1u, abort_flag, 6);
                    if (!ok) break;
                    ++pcnt;
                    if (b == 0 && items > 0) {
                        // the epilogue of this tile's previous item must have read O
                        ok = mbar_wait(o_free(x), (items - 1) & 1u, abort_flag, 7);
                        if (!ok) break;
                    }
                    tc_fence_after();
                    issue_pv(vf, b == 0);
                    if (has_next) {
                        if (!k_ready) {
                            ok = wait_full(kf_next);
                            if (!ok) break;
                            tc_fence_after();
                        }
                        issue_s(kf_next);
                        vf = vf_next;
                    } else {
                        mma_commit(o_done(x));   // the item's last PV: epilogue may read O
                        mma_commit(q_empty(x));  // and every S of the item is complete
                    }
                }
                // walk the remaining steps of the item (fills of the other tile only)
                while (steps_left > 0) {
                    fcur += step_fills(w.next(it), fcur).n;
                    --steps_left;
                }
                f = fcur;
                ++items;
            }
            // every MMA issued above has completed once end_bar flips
            mma_commit(end_bar(x));
            mbar_wait_drain(end_bar(x), 0);
        }
    } else {
        reg_alloc<kSoftmaxRegs>();
        // ------------------------------------------------------------ softmax warpgroups
        const int x = warp >> 3;        // tile
        const int half = (warp >> 2) & 1;  // score columns [64*half, 64*half + 64)
        const int wq = warp & 3;        // TMEM lane quarter of this warp
        const int row = wq * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t tS = tmem + lane_off + x * 128 + 64 * half;
        const uint32_t tP = tmem + lane_off + x * 128 + 64 + 32 * half;
        constexpr int kHalfD = HD / 2;
        const uint32_t tO = tmem + lane_off + Cfg::kOCol + x * HD + kHalfD * half;
        const int pair_bar = 1 + x * 4 + wq;  // named barrier of the two warps of this quarter
        float* xmax = reinterpret_cast<float*>(smem + Cfg::kXmaxOff) + x * 512;  // [parity][half][row]
        float* xsum = reinterpret_cast<float*>(smem + Cfg::kXsumOff) + x * 256;  // [half][row]
        const float sc = p.sc;
        uint32_t nblk = 0;   // blocks processed by this tile slot (s_full / p_full phase)
        uint32_t nitem = 0;  // items finished by this tile slot (o_done / o_free phase)
        uint32_t other_before = 0;  // blocks of the other tile in earlier items
        volatile uint32_t* other_turns = exp_turns + (x ^ 1);
        bool ok = true;
        for (int round = 0, item = round_item(0); item < p.num_items && ok; item = round_item(++round)) {
            const Item it = item_info(p, item);
            const TileInfo ti = x == 0 ? it.t[0] : it.t[1];
            const int other_len = x == 0 ? it.t[1].len() : it.t[0].len();
            if (ti.len() == 0) {
                other_before += other_len;
                continue;
            }
            uint32_t other_seen = other_before;  // other-tile blocks at earlier steps of this item
            const int tok = ti.t0 + row / p.G;
            float m_run = -INFINITY, l_run = 0.f;  // l_run: this half's share of the row sum
            StepWalker w(it);
            int done = 0;
            for (int s = 0; s < it.nsteps(); ++s) {
                const Step st = w.next(it);
                const bool mine = x == 0 ? st.has[0] : st.has[1];
                const bool theirs = x == 0 ? st.has[1] : st.has[0];
                // tile A goes first within a step, tile B follows A's block of the same step
                if (x == 1 && theirs) ++other_seen;
                const uint32_t turn_target = other_seen;
                if (x == 0 && theirs) ++other_seen;
                if (!mine) continue;
                if (!mbar_wait_hot(s_full(x), nblk & 1u, abort_flag, 8)) { ok = false; break; }
                tc_fence_after();
                uint32_t sv[64];
                {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(tS, r0);
                    tmem_ld32(tS + 32, r1);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        sv[i] = r0[i];
                        sv[32 + i] = r1[i];
                    }
                }
                // keep columns c (of the 128-wide block) with lo <= c < hi
                int lo = 0, hi = kBN;
                bool need_mask;
                if (st.dep) {
                    lo = (tok - ti.t0) * p.L - kBN * st.idx;
                    hi = lo + p.L;
                    need_mask = true;
                } else {
                    const int j0 = kBN * st.idx;
                    hi = tok - j0 + 1;
                    need_mask = (j0 + kBN - 1) > ti.t0;
                }
                lo -= 64 * half;  // into this warp's column range
                hi -= 64 * half;
                const bool live = !need_mask || (lo < hi && hi > 0 && lo < 64);
                // With L a multiple of DG a depth block's window [lo, hi) covers whole
                // DG-column groups: pick groups per row instead of masking each score.
                constexpr int kNG = 64 / DG;  // groups in this warp's 64 columns
                const bool chunked = st.dep && (p.L % DG) == 0;
                bool ok[kNG];
#pragma unroll
                for (int k = 0; k < kNG; ++k) ok[k] = lo <= DG * k && hi >= DG * k + DG;
                float mx = -INFINITY;
                if (__any_sync(0xffffffffu, live)) {
                    if (need_mask && !chunked) {
                        if (st.dep) {
#pragma unroll
                            for (int c = 0; c < 64; ++c) {
                                const bool keep = (c >= lo) && (c < hi);
                                sv[c] = keep ? sv[c] : __float_as_uint(-INFINITY);
                            }
                        } else {  // causal diagonal: lo <= 0, only the upper bound bites
#pragma unroll
                            for (int c = 0; c < 64; ++c)
                                sv[c] = c < hi ? sv[c] : __float_as_uint(-INFINITY);
                        }
                    }
                    if constexpr (DG == 16) {
                        float mx4[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            float a = __uint_as_float(sv[16 * k]);
#pragma unroll
                            for (int i = 1; i < 15; i += 2)
                                a = fmax3(a, __uint_as_float(sv[16 * k + i]), __uint_as_float(sv[16 * k + i + 1]));
                            mx4[k] = fmaxf(a, __uint_as_float(sv[16 * k + 15]));
                        }
                        if (chunked)
                            mx = fmaxf(fmaxf(ok[0] ? mx4[0] : -INFINITY, ok[1] ? mx4[1] : -INFINITY),
                                       fmaxf(ok[2] ? mx4[2] : -INFINITY, ok[3] ? mx4[3] : -INFINITY));
                        else
                            mx = fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]);
                    } else {
                        float m8[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            float a = fmax3(__uint_as_float(sv[8 * k]), __uint_as_float(sv[8 * k + 1]),
                                            __uint_as_float(sv[8 * k + 2]));
                            a = fmax3(a, __uint_as_float(sv[8 * k + 3]), __uint_as_float(sv[8 * k + 4]));
                            a = fmax3(a, __uint_as_float(sv[8 * k + 5]), __uint_as_float(sv[8 * k + 6]));
                            m8[k] = fmaxf(a, __uint_as_float(sv[8 * k + 7]));
                        }
                        if (chunked) {
#pragma unroll
                            for (int k = 0; k < 8; ++k) m8[k] = ok[k] ? m8[k] : -INFINITY;
                        }
                        mx = fmaxf(fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), m8[6]), m8[7]);
                    }
                }
                // trade partial row maxima with the partner warp (double-buffered by block parity)
                float* xm = xmax + (nblk & 1u) * 256;
                xm[half * 128 + row] = mx;
                named_bar_sync(pair_bar, 64);
                mx = fmaxf(mx, xm[(half ^ 1) * 128 + row]);
                const float m_new = fmaxf(m_run, mx * sc);
                // lazy rescale: keep the stale max unless it grew by more than 2^8
                const bool rescale = m_new > m_run + 8.0f;
                const float m_use = rescale ? m_new : m_run;
                const float alpha = rescale ? ex2(m_run - m_use) : 1.0f;
                m_run = m_use;
                // wait for the other tile's turn to end (bounded; skipped after an abort)
                // (a hint only: at most 2^20 polls, and no clock read on this hot path).
                // Every lane polls the same words, so the warp never diverges here.
                {
                    const uint32_t need = 8u * turn_target;
                    for (uint32_t it = 0; it < (1u << 20) && *other_turns < need && !*abort_flag; ++it) {
                    }
                }
                if (__any_sync(0xffffffffu, live)) {
                    const float m_base = (m_use == -INFINITY) ? 0.f : m_use;
                    const uint64_t sc2 = f2_pack(sc, sc);
                    uint64_t acc[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) acc[k] = 0ull;
#pragma unroll
                    for (int q4 = 0; q4 < 2; ++q4) {
                        uint32_t pk[16];
                        // a group outside the row's depth window gives exp2(-inf) = 0
                        constexpr int kGq = 32 / DG;  // groups in these 32 columns
                        uint64_t nmg[kGq];
#pragma unroll
                        for (int k = 0; k < kGq; ++k) {
                            const float nb = (chunked && !ok[kGq * q4 + k]) ? -INFINITY : -m_base;
                            nmg[k] = f2_pack(nb, nb);
                        }
#pragma unroll
                        for (int c = 0; c < 32; c += 2) {
                            const int cc = 32 * q4 + c;
                            const uint64_t xx = f2_fma(
                                f2_pack(__uint_as_float(sv[cc]), __uint_as_float(sv[cc + 1])), sc2,
                                nmg[c / DG]);
                            float x0, x1;
                            f2_unpack(xx, x0, x1);
                            const float p0 = ex2(x0), p1 = ex2(x1);
                            acc[(c >> 1) & 3] = f2_add(acc[(c >> 1) & 3], f2_pack(p0, p1));
                            pk[c >> 1] = FMT == 1 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
                        }
                        tmem_st16(tP + 16 * q4, pk);
                    }
                    float s0, s1;
                    f2_unpack(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), s0, s1);
                    l_run = fmaf(l_run, alpha, s0 + s1);
                } else {
                    uint32_t z[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) z[i] = 0u;
                    tmem_st16(tP, z);
                    tmem_st16(tP + 16, z);
                    l_run *= alpha;
                }
                __syncwarp();
                if (lane == 0) atomicAdd(exp_turns + x, 1u);  // this warp's exponentials are done
                if (done > 0 && __any_sync(0xffffffffu, rescale)) {
                    // This half's O columns hold the previous blocks' sum. Their PV has
                    // completed: the S just read was issued after it by the same thread,
                    // and its commit covers both.
                    const uint64_t al2 = f2_pack(alpha, alpha);
#pragma unroll
                    for (int cb = 0; cb < kHalfD; cb += 32) {
                        uint32_t ov[32];
                        tmem_ld32(tO + cb, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            float a, c;
                            f2_unpack(f2_mul(f2_pack(__uint_as_float(ov[i]), __uint_as_float(ov[i + 1])), al2), a, c);
                            ov[i] = __float_as_uint(a);
                            ov[i + 1] = __float_as_uint(c);
                        }
                        tmem_st32(tO + cb, ov);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(p_full(x));
                ++nblk;
                ++done;
            }
            other_before += other_len;
            if (!ok) break;
            // ------------------------------------------------------------ epilogue
            // O = sum / l for this half's columns, straight from TMEM to global memory.
            if (!mbar_wait(o_done(x), nitem & 1u, abort_flag, 10)) { ok = false; break; }
            ++nitem;
            tc_fence_after();
            xsum[half * 128 + row] = l_run;
            named_bar_sync(pair_bar, 64);
            float l_tot = l_run + xsum[(half ^ 1) * 128 + row];
            named_bar_sync(pair_bar, 64);  // both read before the next item overwrites
            float m_fin = m_run, o_scale = 1.f;
            if (p.zero_rows > 0) {  // zero_rows more keys of score 0 whose values are 0
                m_fin = fmaxf(m_run, 0.f);
                o_scale = exp2f(m_run - m_fin);
                l_tot = fmaf(l_tot, o_scale, static_cast<float>(p.zero_rows) * exp2f(-m_fin));
            }
            const float inv = l_tot > 0.f ? o_scale / l_tot : 0.f;
            const bool valid = tok < ti.tend;
            const int head = it.hk * p.G + row % p.G;
            if (p.lse && half == 0 && valid)  // natural log of sum_j exp(scale * q.k_j)
                p.lse[it.b * p.lse_sb + head * p.lse_sh + tok] = (m_fin + __log2f(l_tot)) * kLn2;
            uint4* dst = reinterpret_cast<uint4*>(
                static_cast<uint16_t*>(p.o) + it.b * p.o_sb + head * p.o_sh +
                static_cast<long long>(tok) * p.o_st + kHalfD * half);
#pragma unroll
            for (int cb = 0; cb < kHalfD; cb += 32) {
                uint32_t ov[32];
                tmem_ld32(tO + cb, ov);
                tmem_wait_ld();
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float a = __uint_as_float(ov[2 * i]) * inv;
                    const float c = __uint_as_float(ov[2 * i + 1]) * inv;
                    pk[i] = FMT == 1 ? pack_bf16x2(a, c) : pack_f16x2(a, c);
                }
                if (valid) {
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch)
                        dst[(cb >> 3) + ch] = make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
                }
            }
            tc_fence_before();
            mbar_arrive(o_free(x));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMmaA) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// ---------------------------------------------------------------- host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// Byte stride for a TMA dimension; a size-1 dimension is never stepped, so any
// legal (16-byte multiple) stride works for it.
static cuuint64_t tma_stride(int64_t size, int64_t stride_elems, int esz) {
    if (size <= 1) return 256;
    return static_cast<cuuint64_t>(stride_elems) * esz;
}

// Map over a [B, H, rows, d] view with dimension order (d, a, c, B) where a/c are
// either (rows, H) for key-like tensors or (H, rows) for query-like tensors.
bool encode_map(CUtensorMap* m, const ModaTensor& t, int rows, bool head_inner, int esz,
                       CUtensorMapDataType dt, uint32_t box1, uint32_t box2, char* err,
                       size_t errlen, const char* name) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) {
        snprintf(err, errlen, "cuTensorMapEncodeTiled unavailable from the CUDA driver");
        return false;
    }
    const int64_t B = t.sizes[0], H = t.sizes[1], d = t.sizes[3];
    cuuint64_t dims[4], strides[3];
    dims[0] = static_cast<cuuint64_t>(d);
    if (head_inner) {
        dims[1] = H;
        dims[2] = rows;
        strides[0] = tma_stride(H, t.strides[1], esz);
        strides[1] = tma_stride(rows, t.strides[2], esz);
    } else {
        dims[1] = rows;
        dims[2] = H;
        strides[0] = tma_stride(rows, t.strides[2], esz);
        strides[1] = tma_stride(H, t.strides[1], esz);
    }
    dims[3] = B;
    strides[2] = tma_stride(B, t.strides[0], esz);
    const cuuint32_t box[4] = {64, box1, box2, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, dt, 4, t.ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(err, errlen, "cuTensorMapEncodeTiled failed for %s (CUresult %d)", name,
                 static_cast<int>(r));
        return false;
    }
    return true;
}

cudaError_t read_and_clear_status(cudaStream_t stream, int* value) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(value, moda_dev_status, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && *value != 0) {
        static const int zero = 0;
        e = cudaMemcpyToSymbolAsync(moda_dev_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                    stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    }
    return e;
}

bool tc_supports(const FwdParams& p, char* why, size_t whylen) {
    auto no = [&](const char* s) {
        snprintf(why, whylen, "%s", s);
        return false;
    };
    if (p.dtype != MODA_BF16 && p.dtype != MODA_F16) return no("tcgen05 path needs bf16 or f16");
    if (p.d != 64 && p.d != 128) return no("tcgen05 path needs head_dim 64 or 128");
    // G dividing 128: one launch, 128 / G tokens x G heads per query tile; any other
    // G <= 128: G launches with G = 1 (launch_fwd_tc)
    if (p.G < 1 || p.G > 128) return no("tcgen05 path needs 1 <= H_q/H_k <= 128");
    if (!(p.scale > 0.f)) return no("tcgen05 path needs a positive scale");
    if (static_cast<long long>(p.T) * p.L >= (1LL << 31)) return no("T*L too large for TMA coordinates");
    const ModaTensor* ts[6] = {&p.q, &p.k, &p.v, &p.o, &p.kd, &p.vd};
    const int nts = p.L > 0 ? 6 : 4;  // depth tensors are never read when L == 0
    for (int i = 0; i < nts; ++i) {
        const ModaTensor* t = ts[i];
        if (t->strides[3] != 1) return no("tcgen05 path needs unit stride along head_dim");
        if (reinterpret_cast<uintptr_t>(t->ptr) % 16 != 0) return no("tcgen05 path needs 16-byte aligned tensors");
        for (int i = 0; i < 3; ++i)
            if (t->sizes[i] > 1 && (t->strides[i] * 2) % 16 != 0)
                return no("tcgen05 path needs 16-byte multiple strides");
    }
    return true;
}

template <int HD, int FMT, int DG>
static int launch_tc_inst(const TcParams& tp, int grid, cudaStream_t stream) {
    using Cfg = TcCfg<HD>;
    auto kern = moda_fwd_tc_kernel<HD, FMT, DG>;
    static std::atomic<uint64_t> attr_done{0};
    static std::atomic<int> num_regs{0};  // registers per thread of the compiled kernel, once known
    int nr = num_regs.load(std::memory_order_relaxed);
    if (nr == 0) {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return MODA_ERR_UNSUPPORTED;
        nr = fa.numRegs;
        num_regs.store(nr, std::memory_order_relaxed);
    }
    // The setmaxnreg split assumes exactly kLaunchRegs registers per thread at
    // launch; with fewer, the softmax warpgroups' increase could never be granted.
    if (nr != kLaunchRegs) return MODA_ERR_UNSUPPORTED;
    if (ensure_smem_attr(attr_done, kern, Cfg::kSmemBytes) != cudaSuccess) return MODA_ERR_LAUNCH;
    kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(tp);
    return MODA_OK;
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 148;
    return n;
}

static int launch_fwd_tc_one(const FwdParams& p, float* lse, long long lse_sb, long long lse_sh,
                             cudaStream_t stream, char* err, size_t errlen) {
    TcParams tp;
    const CUtensorMapDataType dt =
        p.dtype == MODA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int n_tok = 128 / p.G;
    const int rows_depth = p.T * p.L;
    if (!encode_map(&tp.tm_q, p.q, p.T, true, 2, dt, p.G, n_tok, err, errlen, "Q") ||
        !encode_map(&tp.tm_k, p.k, p.T, false, 2, dt, kBN, 1, err, errlen, "K") ||
        !encode_map(&tp.tm_v, p.v, p.T, false, 2, dt, kBN, 1, err, errlen, "V") ||
        !encode_map(&tp.tm_kd, rows_depth > 0 ? p.kd : p.k, rows_depth > 0 ? rows_depth : p.T,
                    false, 2, dt, kBN, 1, err, errlen, "K_depth") ||
        !encode_map(&tp.tm_vd, rows_depth > 0 ? p.vd : p.v, rows_depth > 0 ? rows_depth : p.T,
                    false, 2, dt, kBN, 1, err, errlen, "V_depth"))
        return MODA_ERR_LAUNCH;  // with L == 0 the depth maps are placeholders, never loaded
    tp.o = p.o.ptr;
    tp.o_sb = p.o.strides[0];
    tp.o_sh = p.o.strides[1];
    tp.o_st = p.o.strides[2];
    tp.B = p.B;
    tp.Hq = p.Hq;
    tp.Hk = p.Hk;
    tp.G = p.G;
    tp.T = p.T;
    tp.L = p.L;
    tp.n_tok = n_tok;
    tp.num_pairs = (p.T + 2 * n_tok - 1) / (2 * n_tok);
    tp.sc = p.scale * kLog2e;
    tp.lse = lse;
    tp.lse_sb = lse_sb;
    tp.lse_sh = lse_sh;
    tp.zero_rows = p.zero_rows;
    const long long items = static_cast<long long>(tp.num_pairs) * p.B * p.Hk;
    if (items == 0) return MODA_OK;
    if (items > 0x7fffffffLL) {
        snprintf(err, errlen, "too many work items");
        return MODA_ERR_UNSUPPORTED;
    }
    tp.num_items = static_cast<int>(items);
    const int g = static_cast<int>(items < sm_count() ? items : sm_count());
    // 8-column depth groups only where 16 would not divide L: finer groups cost every
    // block a little (more group maxima and biases), so L % 16 == 0 keeps 16.
    const bool g8 = p.L % 16 != 0 && p.L % 8 == 0;
    if (p.d == 128) {
        if (p.dtype == MODA_BF16)
            return g8 ? launch_tc_inst<128, 1, 8>(tp, g, stream) : launch_tc_inst<128, 1, 16>(tp, g, stream);
        return g8 ? launch_tc_inst<128, 0, 8>(tp, g, stream) : launch_tc_inst<128, 0, 16>(tp, g, stream);
    }
    if (p.dtype == MODA_BF16)
        return g8 ? launch_tc_inst<64, 1, 8>(tp, g, stream) : launch_tc_inst<64, 1, 16>(tp, g, stream);
    return g8 ? launch_tc_inst<64, 0, 8>(tp, g, stream) : launch_tc_inst<64, 0, 16>(tp, g, stream);
}


// H_q / H_k = G with 128 % G != 0 (3, 5, 6, 12, ...): a query tile cannot hold whole
// tokens of all G heads, so run G problems with G = 1. Problem c takes query heads
// hk*G + c of every KV head -- one stride, G times the head stride, in Q, O and the
// log-sum-exp rows -- against the same K, V and depth rows. The K/V tiles are then read
// G times, once per problem.
int launch_fwd_tc(const FwdParams& p, cudaStream_t stream, char* err, size_t errlen) {
    const long long lse_sb = static_cast<long long>(p.Hq) * p.T, lse_sh = p.T;
    if (128 % p.G == 0) return launch_fwd_tc_one(p, p.lse, lse_sb, lse_sh, stream, err, errlen);
    const int esz = 2;  // bf16 / f16
    for (int c = 0; c < p.G; ++c) {
        FwdParams pc = p;
        pc.q.ptr = static_cast<char*>(p.q.ptr) + static_cast<long long>(c) * p.q.strides[1] * esz;
        pc.q.sizes[1] = p.Hk;
        pc.q.strides[1] = p.q.strides[1] * p.G;
        pc.o.ptr = static_cast<char*>(p.o.ptr) + static_cast<long long>(c) * p.o.strides[1] * esz;
        pc.o.sizes[1] = p.Hk;
        pc.o.strides[1] = p.o.strides[1] * p.G;
        pc.Hq = p.Hk;
        pc.G = 1;
        const int r = launch_fwd_tc_one(pc, p.lse ? p.lse + static_cast<long long>(c) * p.T : nullptr,
                                        lse_sb, lse_sh * p.G, stream, err, errlen);
        if (r != MODA_OK) return r;
    }
    return MODA_OK;
}
}  // namespace moda
