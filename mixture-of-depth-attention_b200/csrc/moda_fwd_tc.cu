// Fused MoDA forward on Blackwell tensor cores: TMA -> tcgen05.mma -> TMEM.
//
// Semantics (moda/kernels/moda_naive.py:13-97): for query row (b, h, t)
//   out = softmax({scale*q.k_j : j <= t} U {scale*q.kd_{t*L+l} : l < L}) . [V ; V_depth]
// with KV head h / G. One online softmax covers both score sets.
//
// Tiling.
//   * A query tile is 128 rows of one (batch, KV head): n = 128/G tokens x the G
//     query heads of that KV head, token-major (row = token_local*G + head). The
//     TMA box (64, G, n) over the [d, H_q, T, B] view builds it, so every K/V
//     tile is used once by all G heads of its group -- GQA without
//     repeat_interleave.
//   * A CTA owns two consecutive query tiles (A, B) of the same (b, KV head) and
//     ping-pongs them on the tensor core: while softmax warpgroup A works on
//     S_A, the tensor core runs tile B's MMAs, and vice versa.
//   * Each tile walks a list of 128-row key blocks:
//       - depth blocks: rows [t0*L + 128i, +128) of K_depth/V_depth, exactly the
//         rows of the tile's own tokens (chunk-aware: a tile of n tokens touches
//         n*L depth rows), masked so row (token t) keeps rows t*L..t*L+L-1;
//       - causal sequence blocks 0..ceil((t0+n)/128)-1, masked on the diagonal.
//     Both kinds go through the same TMA ring and the same two MMAs
//     (S = Q K^T, O += P V), i.e. the depth phase of the paper's algorithm
//     (group-aware indexing, depth mask floor(row/G) == floor(j/L)).
//
// Warp roles (320 threads):
//   warps 0-3  softmax + correction + epilogue for tile A (thread = TMEM lane = row)
//   warps 4-7  the same for tile B
//   warp  8    TMA producer (Q tiles, then the K/V block ring)
//   warp  9    TMEM allocator and single-thread tcgen05.mma issuer
//
// TMEM (512 columns): S_A [0,128) S_B [128,256) O_A [256,256+d) O_B [256+d,256+2d).
// P (bf16/f16) is written into the upper 64 columns of S and fed to the PV MMA
// straight from TMEM (A operand in tensor memory), so P never touches shared memory.
#include "moda_internal.h"

#include <cstdio>

namespace moda {

constexpr int kThreads = 320;
constexpr int kBM = 128;  // query rows per tile
constexpr int kBN = 128;  // key rows per block

template <int HD>
struct TcCfg {
    static constexpr int kTileBytes = kBM * HD * 2;       // one 128 x HD 16-bit tile
    static constexpr int kColBlocks = HD / 64;            // 128-byte swizzle atoms across d
    static constexpr int kStages = (HD == 128) ? 4 : 8;   // K/V ring depth
    static constexpr int kQOff = 0;
    static constexpr int kRingOff = 2 * kTileBytes;
    static constexpr int kBarOff = kRingOff + kStages * kTileBytes;
    // barriers: q_full[2], s_full[2], p_full[2], o_done[2], end, slot_full[S], slot_empty[S]
    static constexpr int kNumBars = 9 + 2 * kStages;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kSmemBytes = kMiscOff + 64 + 1024;  // + alignment slack
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

// Per step s of a tile: which block. Depth blocks first, then causal blocks.
__device__ __forceinline__ bool is_depth(const TileInfo& ti, int s) { return s < ti.ndep; }

// Ring bookkeeping shared by producer and consumer: the blocks of step s are
// filled in the order K_A, K_B, V_A, V_B, where K_B / V_B are skipped when both
// tiles read the same causal block (then one fill serves both).
struct StepSlots {
    bool hasA, hasB, shared;
    uint32_t kA, kB, vA, vB;  // fill indices
    uint32_t nfill;
};

__device__ __forceinline__ StepSlots step_slots(const TileInfo& A, const TileInfo& Bt, int s,
                                                uint32_t base) {
    StepSlots r;
    r.hasA = s < A.len();
    r.hasB = s < Bt.len();
    r.shared = r.hasA && r.hasB && !is_depth(A, s) && !is_depth(Bt, s) &&
               (s - A.ndep) == (s - Bt.ndep);
    uint32_t f = base;
    if (r.hasA) r.kA = f++;
    if (r.hasB) r.kB = r.shared ? r.kA : f++;
    if (r.hasA) r.vA = f++;
    if (r.hasB) r.vB = r.shared ? r.vA : f++;
    r.nfill = f - base;
    return r;
}

template <int HD, int FMT>
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
    auto s_full = [&](int x) { return bar0 + 8u * (2 + x); };
    auto p_full = [&](int x) { return bar0 + 8u * (4 + x); };
    auto o_done = [&](int x) { return bar0 + 8u * (6 + x); };
    const uint32_t end_bar = bar0 + 8u * 8;
    auto slot_full = [&](uint32_t i) { return bar0 + 8u * (9 + i); };
    auto slot_empty = [&](uint32_t i) { return bar0 + 8u * (9 + Cfg::kStages + i); };
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOff);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kMiscOff + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // heavy pairs (more causal blocks) first
    const int bh_count = p.B * p.Hk;
    const int pair = p.num_pairs - 1 - static_cast<int>(blockIdx.x) / bh_count;
    const int bh = static_cast<int>(blockIdx.x) % bh_count;
    const int b = bh / p.Hk;
    const int hk = bh % p.Hk;
    const TileInfo tA = tile_info(p, pair, 0);
    const TileInfo tB = tile_info(p, pair, 1);
    const int nsteps = max(tA.len(), tB.len());

    if (threadIdx.x == 0) {
        for (int i = 0; i < 8; ++i) mbar_init(bar0 + 8u * i, (i == 4 || i == 5) ? kBM : 1);
        mbar_init(end_bar, 1);
        for (int i = 0; i < Cfg::kStages; ++i) {
            mbar_init(slot_full(i), 1);
            mbar_init(slot_empty(i), 1);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 9) {
        tmem_alloc(smem_u32(tmem_holder), Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 8 && lane == 0) {
        tma_prefetch_desc(&p.tm_q);
        tma_prefetch_desc(&p.tm_k);
        tma_prefetch_desc(&p.tm_v);
        tma_prefetch_desc(&p.tm_kd);
        tma_prefetch_desc(&p.tm_vd);
        tma_prefetch_desc(&p.tm_o);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 8) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            constexpr uint32_t kBytes = Cfg::kTileBytes;
            const int head0 = hk * p.G;
            if (tA.len() > 0) {
                mbar_expect_tx(q_full(0), kBytes);
                for (int cb = 0; cb < Cfg::kColBlocks; ++cb)
                    tma_load_4d(&p.tm_q, sQ + cb * 16384, q_full(0), cb * 64, head0, tA.t0, b);
            }
            if (tB.len() > 0) {
                mbar_expect_tx(q_full(1), kBytes);
                for (int cb = 0; cb < Cfg::kColBlocks; ++cb)
                    tma_load_4d(&p.tm_q, sQ + kBytes + cb * 16384, q_full(1), cb * 64, head0,
                                tB.t0, b);
            }
            uint32_t base = 0;
            bool ok = true;
            auto fill = [&](uint32_t f, const CUtensorMap* map, int row0) {
                const uint32_t slot = f % Cfg::kStages;
                const uint32_t use = f / Cfg::kStages;
                if (!mbar_wait(slot_empty(slot), (use & 1u) ^ 1u, abort_flag, 1)) return false;
                mbar_expect_tx(slot_full(slot), kBytes);
                const uint32_t dst = sRing + slot * kBytes;
                for (int cb = 0; cb < Cfg::kColBlocks; ++cb)
                    tma_load_4d(map, dst + cb * 16384, slot_full(slot), cb * 64, row0, hk, b);
                return true;
            };
            auto k_src = [&](const TileInfo& ti, int s, int& row0) -> const CUtensorMap* {
                if (is_depth(ti, s)) {
                    row0 = ti.t0 * p.L + kBN * s;
                    return &p.tm_kd;
                }
                row0 = kBN * (s - ti.ndep);
                return &p.tm_k;
            };
            auto v_src = [&](const TileInfo& ti, int s, int& row0) -> const CUtensorMap* {
                if (is_depth(ti, s)) {
                    row0 = ti.t0 * p.L + kBN * s;
                    return &p.tm_vd;
                }
                row0 = kBN * (s - ti.ndep);
                return &p.tm_v;
            };
            uint32_t issued = 0;  // fills whose TMA loads were started
            for (int s = 0; s < nsteps && ok; ++s) {
                const StepSlots st = step_slots(tA, tB, s, base);
                int row0;
                const CUtensorMap* m;
                if (st.hasA) { m = k_src(tA, s, row0); ok = fill(st.kA, m, row0); issued += ok; }
                if (ok && st.hasB && !st.shared) { m = k_src(tB, s, row0); ok = fill(st.kB, m, row0); issued += ok; }
                if (ok && st.hasA) { m = v_src(tA, s, row0); ok = fill(st.vA, m, row0); issued += ok; }
                if (ok && st.hasB && !st.shared) { m = v_src(tB, s, row0); ok = fill(st.vB, m, row0); issued += ok; }
                base += st.nfill;
            }
            // Exit path: the last loads of every slot must have landed before the
            // CTA's shared memory is released (already true when all went well).
            const uint32_t first = issued > Cfg::kStages ? issued - Cfg::kStages : 0;
            for (uint32_t f = first; f < issued; ++f)
                mbar_wait_drain(slot_full(f % Cfg::kStages), (f / Cfg::kStages) & 1u);
            if (tA.len() > 0) mbar_wait_drain(q_full(0), 0);
            if (tB.len() > 0) mbar_wait_drain(q_full(1), 0);
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = make_idesc(FMT, kBM, kBN, 0);
            constexpr uint32_t idesc_pv = make_idesc(FMT, kBM, HD, 1);
            constexpr uint32_t kBytes = Cfg::kTileBytes;
            bool ok = true;
            // Q tiles are needed by the first S MMA of each tile.
            if (tA.len() > 0) ok = ok && mbar_wait(q_full(0), 0, abort_flag, 2);
            if (ok && tB.len() > 0) ok = mbar_wait(q_full(1), 0, abort_flag, 2);

            auto issue_s = [&](int x, uint32_t f) {
                const uint32_t slot = f % Cfg::kStages;
                if (!mbar_wait(slot_full(slot), (f / Cfg::kStages) & 1u, abort_flag, 3)) return false;
                tc_fence_after();
                const uint32_t qa = sQ + x * kBytes;
                const uint32_t kb = sRing + slot * kBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    mma_ss(tmem + x * 128, smem_desc_sw128(qa + off, 16, 1024),
                           smem_desc_sw128(kb + off, 16, 1024), idesc_s, kk > 0);
                }
                mma_commit(s_full(x));
                return true;
            };
            auto issue_pv = [&](int x, uint32_t f, bool first) {
                const uint32_t slot = f % Cfg::kStages;
                if (!mbar_wait(slot_full(slot), (f / Cfg::kStages) & 1u, abort_flag, 4)) return false;
                tc_fence_after();
                const uint32_t vb = sRing + slot * kBytes;
                const uint32_t ptm = tmem + x * 128 + 64;
                const uint32_t otm = tmem + Cfg::kOCol + x * HD;
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                    mma_ts(otm, ptm + kk * 8, smem_desc_sw128(vb + kk * 2048, 128 * 128, 1024),
                           idesc_pv, (first && kk == 0) ? 0u : 1u);
                }
                mma_commit(o_done(x));
                return true;
            };

            StepSlots cur = step_slots(tA, tB, 0, 0);
            uint32_t base_next = cur.nfill;
            // prologue: S of step 0 for both tiles
            if (ok && cur.hasA) {
                ok = issue_s(0, cur.kA);
                if (ok && !cur.shared) mma_commit(slot_empty(cur.kA % Cfg::kStages));
            }
            if (ok && cur.hasB) {
                ok = issue_s(1, cur.kB);
                if (ok) mma_commit(slot_empty(cur.kB % Cfg::kStages));
            }
            for (int s = 0; s < nsteps && ok; ++s) {
                const StepSlots nxt = step_slots(tA, tB, s + 1, base_next);
                if (cur.hasA) {
                    ok = mbar_wait(p_full(0), s & 1, abort_flag, 5);
                    if (!ok) break;
                    tc_fence_after();
                    ok = issue_pv(0, cur.vA, s == 0);
                    if (!ok) break;
                    if (!cur.shared) mma_commit(slot_empty(cur.vA % Cfg::kStages));
                    if (nxt.hasA) {
                        ok = issue_s(0, nxt.kA);
                        if (!ok) break;
                        if (!nxt.shared) mma_commit(slot_empty(nxt.kA % Cfg::kStages));
                    }
                }
                if (cur.hasB) {
                    ok = mbar_wait(p_full(1), s & 1, abort_flag, 6);
                    if (!ok) break;
                    tc_fence_after();
                    ok = issue_pv(1, cur.vB, s == 0);
                    if (!ok) break;
                    mma_commit(slot_empty(cur.vB % Cfg::kStages));
                    if (nxt.hasB) {
                        ok = issue_s(1, nxt.kB);
                        if (!ok) break;
                        mma_commit(slot_empty(nxt.kB % Cfg::kStages));
                    }
                }
                cur = nxt;
                base_next += nxt.nfill;
            }
            // every MMA issued above has completed once end_bar flips
            mma_commit(end_bar);
            mbar_wait_drain(end_bar, 0);
        }
    } else {
        // ------------------------------------------------------------ softmax warpgroups
        const int x = warp >> 2;  // tile
        const TileInfo ti = x == 0 ? tA : tB;
        const int row = threadIdx.x & 127;
        const int wq = warp & 3;  // TMEM lane quarter of this warp
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t tS = tmem + lane_off + x * 128;
        const uint32_t tP = tS + 64;
        const uint32_t tO = tmem + lane_off + Cfg::kOCol + x * HD;
        const int tok = ti.t0 + row / p.G;
        const float sc = p.sc;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        const int len = ti.len();
        for (int s = 0; s < len; ++s) {
            if (!mbar_wait(s_full(x), s & 1, abort_flag, 8)) { ok = false; break; }
            tc_fence_after();
            uint32_t sv[128];
            {
                uint32_t (&c0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[0]);
                uint32_t (&c1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[32]);
                uint32_t (&c2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[64]);
                uint32_t (&c3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[96]);
                tmem_ld32(tS + 0, c0);
                tmem_ld32(tS + 32, c1);
                tmem_ld32(tS + 64, c2);
                tmem_ld32(tS + 96, c3);
                tmem_wait_ld();
            }
            // mask: keep columns c with lo <= c < hi
            int lo = 0, hi = kBN;
            bool need_mask;
            if (is_depth(ti, s)) {
                lo = (tok - ti.t0) * p.L - kBN * s;
                hi = lo + p.L;
                need_mask = true;
            } else {
                const int j0 = kBN * (s - ti.ndep);
                hi = tok - j0 + 1;
                need_mask = (j0 + kBN - 1) > ti.t0;
            }
            float mx = -INFINITY;
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    const bool keep = (c >= lo) && (c < hi);
                    float v = keep ? __uint_as_float(sv[c]) : -INFINITY;
                    sv[c] = __float_as_uint(v);
                    mx = fmaxf(mx, v);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 128; ++c) mx = fmaxf(mx, __uint_as_float(sv[c]));
            }
            const float m_blk = mx * sc;
            const float m_new = fmaxf(m_run, m_blk);
            // lazy rescale: keep the stale max unless it grew by more than 2^8
            const bool rescale = m_new > m_run + 8.0f;
            const float m_use = rescale ? m_new : m_run;
            const float alpha = rescale ? ex2(m_run - m_use) : 1.0f;
            const float m_base = (m_use == -INFINITY) ? 0.f : m_use;
            float sum = 0.f;
            uint32_t pk[64];
#pragma unroll
            for (int c = 0; c < 128; c += 2) {
                const float p0 = ex2(fmaf(__uint_as_float(sv[c]), sc, -m_base));
                const float p1 = ex2(fmaf(__uint_as_float(sv[c + 1]), sc, -m_base));
                sum += p0 + p1;
                pk[c >> 1] = FMT == 1 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
            }
            l_run = fmaf(l_run, alpha, sum);
            m_run = m_use;
            tmem_st32(tP, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
            tmem_st32(tP + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
            if (s > 0 && __any_sync(0xffffffffu, rescale)) {
                if (!mbar_wait(o_done(x), (s - 1) & 1, abort_flag, 9)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int cb = 0; cb < HD; cb += 32) {
                    uint32_t ov[32];
                    tmem_ld32(tO + cb, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                    tmem_st32(tO + cb, ov);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_full(x));
        }
        // ------------------------------------------------------------ epilogue
        // Runs whenever the tile has work, even after an abort (then the output is
        // garbage and the host sees the status word): the named barrier below
        // needs all four warps of the warpgroup.
        if (len > 0) {
            if (ok) mbar_wait(o_done(x), (len - 1) & 1, abort_flag, 10);
            tc_fence_after();
            const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
            const uint32_t tile = sQ + x * Cfg::kTileBytes;  // Q tile is free: reuse as staging
#pragma unroll
            for (int cb = 0; cb < HD; cb += 32) {
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
                const int colblk = cb >> 6;
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    const int chunk = ((cb & 63) >> 3) + ch;  // 16-byte chunk within the 128-byte row
                    const uint32_t addr = tile + colblk * 16384 + row * 128 + ((chunk ^ (row & 7)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                                 "r"(pk[4 * ch]), "r"(pk[4 * ch + 1]), "r"(pk[4 * ch + 2]),
                                 "r"(pk[4 * ch + 3])
                                 : "memory");
                }
            }
            fence_proxy_async_smem();
            named_bar_sync(1 + x, 128);
            if (row == 0) {
                for (int cb = 0; cb < Cfg::kColBlocks; ++cb)
                    tma_store_4d(&p.tm_o, tile + cb * 16384, cb * 64, hk * p.G, ti.t0, b);
                bulk_commit();
                bulk_wait0();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
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
static bool encode_map(CUtensorMap* m, const ModaTensor& t, int rows, bool head_inner, int esz,
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
    if (p.G < 1 || p.G > 128 || (128 % p.G) != 0) return no("tcgen05 path needs H_q/H_k dividing 128");
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

template <int HD, int FMT>
static int launch_tc_inst(const TcParams& tp, int grid, cudaStream_t stream) {
    using Cfg = TcCfg<HD>;
    auto kern = moda_fwd_tc_kernel<HD, FMT>;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Cfg::kSmemBytes) != cudaSuccess)
            return MODA_ERR_LAUNCH;
        attr_set = true;
    }
    kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(tp);
    return MODA_OK;
}

int launch_fwd_tc(const FwdParams& p, cudaStream_t stream, char* err, size_t errlen) {
    TcParams tp;
    const CUtensorMapDataType dt =
        p.dtype == MODA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int n_tok = 128 / p.G;
    const int rows_depth = p.T * p.L;
    if (!encode_map(&tp.tm_q, p.q, p.T, true, 2, dt, p.G, n_tok, err, errlen, "Q") ||
        !encode_map(&tp.tm_o, p.o, p.T, true, 2, dt, p.G, n_tok, err, errlen, "O") ||
        !encode_map(&tp.tm_k, p.k, p.T, false, 2, dt, kBN, 1, err, errlen, "K") ||
        !encode_map(&tp.tm_v, p.v, p.T, false, 2, dt, kBN, 1, err, errlen, "V") ||
        !encode_map(&tp.tm_kd, rows_depth > 0 ? p.kd : p.k, rows_depth > 0 ? rows_depth : p.T,
                    false, 2, dt, kBN, 1, err, errlen, "K_depth") ||
        !encode_map(&tp.tm_vd, rows_depth > 0 ? p.vd : p.v, rows_depth > 0 ? rows_depth : p.T,
                    false, 2, dt, kBN, 1, err, errlen, "V_depth"))
        return MODA_ERR_LAUNCH;  // with L == 0 the depth maps are placeholders, never loaded
    tp.B = p.B;
    tp.Hq = p.Hq;
    tp.Hk = p.Hk;
    tp.G = p.G;
    tp.T = p.T;
    tp.L = p.L;
    tp.n_tok = n_tok;
    tp.num_pairs = (p.T + 2 * n_tok - 1) / (2 * n_tok);
    tp.sc = p.scale * kLog2e;
    const long long grid = static_cast<long long>(tp.num_pairs) * p.B * p.Hk;
    if (grid == 0) return MODA_OK;
    if (grid > 0x7fffffffLL) {
        snprintf(err, errlen, "grid too large");
        return MODA_ERR_UNSUPPORTED;
    }
    const int g = static_cast<int>(grid);
    if (p.d == 128) return p.dtype == MODA_BF16 ? launch_tc_inst<128, 1>(tp, g, stream)
                                                : launch_tc_inst<128, 0>(tp, g, stream);
    return p.dtype == MODA_BF16 ? launch_tc_inst<64, 1>(tp, g, stream)
                                : launch_tc_inst<64, 0>(tp, g, stream);
}

}  // namespace moda
