// MoDA backward on CUDA cores in fp32 arithmetic, tiled like the fp32 forward
// (moda_fwd_simt.cu): fp32 inputs, and bf16 / f16 inputs of the shapes the tensor-core
// backward does not take (head_dim outside {64, 128}, H_q / H_k not dividing 128).
// 16-bit rows are staged raw by cp.async and converted once per tile into the fp32
// tiles; gradients are rounded to the input dtype on store.
//
// The gradients are those of moda_bwd.cu's row kernels -- torch autograd of
// moda_attention_naive (moda/kernels/moda_naive.py:13-162) -- computed from shared-memory
// tiles so that every staged value feeds several FMAs (the row kernels re-read every key
// for each query row and every query row for each key):
//   dq     CTA per 64 query rows of one head; for each causal 64-key tile
//          S = Q K^T and dP = dO V^T (4 x 4 per thread), dS = P (dP - D) through shared
//          memory, dQ += dS K;
//   dkdv   CTA per 64-key tile of one KV head; for each 64-token query tile of each of
//          its G heads (tokens from the key tile's first one on) S^T = K Q^T and
//          dP^T = V dO^T, P^T and dS^T through shared memory, dV += P^T dO, dK += dS^T Q;
//   depth  CTA per token of one KV head: the token's G query rows and its depth rows (32
//          at a time) in shared memory; one thread per (depth row, head) dot product,
//          then dK_depth and dV_depth by (row, 4 columns), and the depth part of dQ,
//          added to what the dq kernel wrote;
//   zero   depth rows at or past T*L (never read by the forward) get zero gradient.
// Every output element has one writer per launch; fp32 FMA throughout.
//
// dq / dkdv thread layout (256 threads): ty = tid / 16, tx = tid % 16; a thread owns
// tile rows ty + 16i (i < 4), tile columns tx + 16j (j < 4), and output columns in groups
// of VW adjacent ones at g*16*VW + tx*VW. The two rows of a warp are adjacent, so row
// reads are two broadcast addresses; Q/K/V/dO rows are padded by 4 floats and P/dS rows
// by 16, which keeps every shared-memory access free of bank conflicts.
#include "moda_internal.h"

#include <algorithm>
#include <type_traits>

namespace moda {

constexpr int kB32Tile = 64, kB32Threads = 256;
constexpr int kB32DepthThreads = 128, kB32DepthRows = 32;

template <int HD>
struct B32Cfg {
    static constexpr int kStride = HD + 4;               // floats per staged row
    static constexpr int kPStride = kB32Tile + 16;       // floats per P / dS row
    static constexpr int kRowTile = kB32Tile * kStride;  // one [64][HD+4] array
    static constexpr int kPTile = kB32Tile * kPStride;   // one [64][64+16] array
    static constexpr int kDqBytes = (4 * kRowTile + kPTile) * 4;        // Q dO K V dS
    static constexpr int kDkvBytes = (4 * kRowTile + 2 * kPTile) * 4;   // K V Q dO P^T dS^T
};

namespace {

// 4 elements into 4 floats of shared memory (zeros when !ok): fp32 by cp.async, 16-bit
// by one 8-byte load and a conversion
template <typename T>
MODA_DEV void b32_stage4(float* dst, const T* src, bool ok) {
    if constexpr (kIsF32<T>) {
        f32_cp16(dst, src, ok ? 16 : 0);
    } else {
        *reinterpret_cast<float4*>(dst) = ok ? b32_ld4<T>(src) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// raw 16-bit tiles of this file's 64 rows with its 256 threads
template <typename T, int HD>
MODA_DEV void b16_stage(T* dst, const T* base, int64_t rstride, int row0, int limit, int d, int tid) {
    raw16_stage<T, HD, kB32Tile, kB32Threads>(dst, base, rstride, row0, limit, d, tid);
}
template <typename T, int HD>
MODA_DEV void b16_convert(float* dst, const T* raw, int tid) {
    raw16_convert<T, HD, kB32Tile, kB32Threads>(dst, raw, tid);
}

// 64 rows of a [.., rows, d] fp32 view, from row0, into dst [64][HD+4] by cp.async
// (zeros for rows at or past `limit` and for columns at or past d)
template <int HD>
MODA_DEV void b32_stage(float* dst, const float* base, int64_t rstride, int row0, int limit, int d,
                        int tid) {
    for (int i = tid; i < kB32Tile * (HD / 4); i += kB32Threads) {
        const int r = i / (HD / 4), c4 = i % (HD / 4);
        const bool ok = row0 + r < limit && 4 * c4 < d;
        const float* src = ok ? base + static_cast<int64_t>(row0 + r) * rstride + 4 * c4 : base;
        f32_cp16(dst + r * (HD + 4) + 4 * c4, src, ok ? 16 : 0);
    }
}

// s[i][j] = A[ty + 16i] . B[tx + 16j] over HD columns of two [64][HD+4] arrays
template <int HD>
MODA_DEV void b32_abt(float (&s)[4][4], const float* A, const float* Bm, int ty, int tx) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int c = 0; c < HD; c += 4) {
        float4 a[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(A + (ty + 16 * i) * (HD + 4) + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = *reinterpret_cast<const float4*>(Bm + (tx + 16 * j) * (HD + 4) + c);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                s[i][j] = fmaf(a[i].x, bv[j].x, s[i][j]);
                s[i][j] = fmaf(a[i].y, bv[j].y, s[i][j]);
                s[i][j] = fmaf(a[i].z, bv[j].z, s[i][j]);
                s[i][j] = fmaf(a[i].w, bv[j].w, s[i][j]);
            }
    }
}

// acc[i][.] += sum_k P[ty + 16i][k] * M[k][this thread's columns], k < 64; P is
// [64][64+16], M is [64][HD+4]
template <int HD>
MODA_DEV void b32_pm(float (&acc)[4][HD / 16], const float* P, const float* M, int ty, int tx) {
    constexpr int OC = HD / 16, VW = OC >= 4 ? 4 : 2, NG = OC / VW;
#pragma unroll 2
    for (int k = 0; k < kB32Tile; k += 4) {
        float4 pv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            pv[i] = *reinterpret_cast<const float4*>(P + (ty + 16 * i) * B32Cfg<HD>::kPStride + k);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const float* mr = M + (k + kk) * (HD + 4) + tx * VW;
            float mv[OC];
#pragma unroll
            for (int g = 0; g < NG; ++g) f32_ldv<VW>(mv + g * VW, mr + g * 16 * VW);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pk = kk == 0 ? pv[i].x : kk == 1 ? pv[i].y : kk == 2 ? pv[i].z : pv[i].w;
#pragma unroll
                for (int c = 0; c < OC; ++c) acc[i][c] = fmaf(pk, mv[c], acc[i][c]);
            }
        }
    }
}

// rows row0 + ty + 16i (those below `rows`) of acc * s into out, this thread's columns
template <typename T, int HD>
MODA_DEV void b32_store(const ModaTensor& t, int b, int h, int row0, int rows, int d,
                        const float (&acc)[4][HD / 16], float s, int ty, int tx) {
    constexpr int OC = HD / 16, VW = OC >= 4 ? 4 : 2, NG = OC / VW;
    T* base = static_cast<T*>(t.ptr) + b * t.strides[0] + h * t.strides[1];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = row0 + ty + 16 * i;
        if (r >= rows) continue;
        T* row = base + static_cast<int64_t>(r) * t.strides[2] + tx * VW;
#pragma unroll
        for (int g = 0; g < NG; ++g) {  // d is a multiple of 4: a group starting below d is inside it
            if (tx * VW + g * 16 * VW >= d) continue;
            const float* a = acc[i] + g * VW;
            if constexpr (VW == 4)
                b32_st4<T>(row + g * 16 * VW, make_float4(a[0], a[1], a[2], a[3]), s);
            else if constexpr (kIsF32<T>)
                f32_stv<2>(row + g * 16 * VW, a, s);
            else
                *reinterpret_cast<uint32_t*>(row + g * 16 * VW) = pack2<T>(a[0] * s, a[1] * s);
        }
    }
}

template <typename T>
MODA_DEV const T* b32_head(const ModaTensor& t, int b, int h) {
    return static_cast<const T*>(t.ptr) + b * t.strides[0] + h * t.strides[1];
}

}  // namespace

template <typename T, int HD>
__global__ void __launch_bounds__(kB32Threads, 1) moda_bwd_f32_dq_kernel(const __grid_constant__ BwdParams p) {
    using C = B32Cfg<HD>;
    constexpr int OC = HD / 16;
    extern __shared__ __align__(16) float b32_smem[];
    float* sQ = b32_smem;
    float* sdO = sQ + C::kRowTile;
    float* sK = sdO + C::kRowTile;
    float* sV = sK + C::kRowTile;
    float* sdS = sV + C::kRowTile;
    T* rK = reinterpret_cast<T*>(sdS + C::kPTile);  // 16-bit only: raw K and V tiles
    T* rV = rK + kB32Tile * HD;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int ntiles = (p.T + kB32Tile - 1) / kB32Tile;
    // grid (H_q * B, tiles): every head's heaviest tile (the last 64 tokens) goes first
    const int t0 = (ntiles - 1 - static_cast<int>(blockIdx.y)) * kB32Tile;
    const int h = blockIdx.x % p.Hq, b = blockIdx.x / p.Hq, hk = h / p.G, d = p.d;
    const T* kb = b32_head<T>(p.k, b, hk);
    const T* vb = b32_head<T>(p.v, b, hk);
    const float sc2 = p.scale * kLog2e;

    if constexpr (kIsF32<T>) {
        b32_stage<HD>(sQ, b32_head<float>(p.q, b, h), p.q.strides[2], t0, p.T, d, tid);
        b32_stage<HD>(sdO, b32_head<float>(p.dout, b, h), p.dout.strides[2], t0, p.T, d, tid);
        f32_cp_commit();
        b32_stage<HD>(sV, vb, p.v.strides[2], 0, p.T, d, tid);
        f32_cp_commit();
        b32_stage<HD>(sK, kb, p.k.strides[2], 0, p.T, d, tid);
        f32_cp_commit();
    } else {  // Q and dO through the raw K / V tiles, then K and V of the first key tile
        b16_stage<T, HD>(rK, b32_head<T>(p.q, b, h), p.q.strides[2], t0, p.T, d, tid);
        b16_stage<T, HD>(rV, b32_head<T>(p.dout, b, h), p.dout.strides[2], t0, p.T, d, tid);
        f32_cp_commit();
        f32_cp_wait<0>();
        __syncthreads();
        b16_convert<T, HD>(sQ, rK, tid);
        b16_convert<T, HD>(sdO, rV, tid);
        __syncthreads();
        b16_stage<T, HD>(rV, vb, p.v.strides[2], 0, p.T, d, tid);
        f32_cp_commit();
        b16_stage<T, HD>(rK, kb, p.k.strides[2], 0, p.T, d, tid);
        f32_cp_commit();
    }

    // rows past T: lse = +inf makes their P (and dS) zero
    float lse2[4], del[4];
    const int64_t rbase = (static_cast<int64_t>(b) * p.Hq + h) * p.T;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty + 16 * i;
        lse2[i] = t < p.T ? p.lse[rbase + t] * kLog2e : INFINITY;
        del[i] = t < p.T ? p.delta[rbase + t] : 0.f;
    }
    float acc[4][OC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < OC; ++c) acc[i][c] = 0.f;

    const int kmax = min(t0 + kB32Tile, p.T);
    const int nkt = (kmax + kB32Tile - 1) / kB32Tile;
#pragma unroll 1
    for (int kt = 0; kt < nkt; ++kt) {
        f32_cp_wait<1>();  // this V (this K may still be in flight)
        __syncthreads();
        if constexpr (!kIsF32<T>) {
            b16_convert<T, HD>(sV, rV, tid);
            __syncthreads();
            if (kt + 1 < nkt) b16_stage<T, HD>(rV, vb, p.v.strides[2], (kt + 1) * kB32Tile, p.T, d, tid);
            f32_cp_commit();
        }
        float dp[4][4];
        b32_abt<HD>(dp, sdO, sV, ty, tx);
        if constexpr (kIsF32<T>) {
            f32_cp_wait<0>();  // this K
            __syncthreads();   // and every thread is done with V
            if (kt + 1 < nkt) b32_stage<HD>(sV, vb, p.v.strides[2], (kt + 1) * kB32Tile, p.T, d, tid);
            f32_cp_commit();
        } else {
            f32_cp_wait<1>();  // this K (the next V may still be in flight)
            __syncthreads();
            b16_convert<T, HD>(sK, rK, tid);
            __syncthreads();
            if (kt + 1 < nkt) b16_stage<T, HD>(rK, kb, p.k.strides[2], (kt + 1) * kB32Tile, p.T, d, tid);
            f32_cp_commit();
        }
        float s[4][4];
        b32_abt<HD>(s, sQ, sK, ty, tx);
        // keys after a row's token are masked (this covers keys at or past T for rows < T)
        const bool diag = kt * kB32Tile + kB32Tile - 1 > t0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int ti = t0 + ty + 16 * i;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kj = kt * kB32Tile + tx + 16 * j;
                const float pr = (diag && kj > ti) ? 0.f : ex2(fmaf(s[i][j], sc2, -lse2[i]));
                sdS[(ty + 16 * i) * C::kPStride + tx + 16 * j] = pr * (dp[i][j] - del[i]);
            }
        }
        __syncthreads();
        b32_pm<HD>(acc, sdS, sK, ty, tx);
        __syncthreads();  // every thread is done with K and dS
        if constexpr (kIsF32<T>) {
            if (kt + 1 < nkt) b32_stage<HD>(sK, kb, p.k.strides[2], (kt + 1) * kB32Tile, p.T, d, tid);
            f32_cp_commit();
        }
    }
    f32_cp_wait<0>();
    b32_store<T, HD>(p.dq, b, h, t0, p.T, d, acc, p.scale, ty, tx);
}

template <typename T, int HD>
__global__ void __launch_bounds__(kB32Threads, 1) moda_bwd_f32_dkdv_kernel(const __grid_constant__ BwdParams p) {
    using C = B32Cfg<HD>;
    constexpr int OC = HD / 16;
    extern __shared__ __align__(16) float b32_smem[];
    float* sK = b32_smem;
    float* sV = sK + C::kRowTile;
    float* sQ = sV + C::kRowTile;
    float* sdO = sQ + C::kRowTile;
    float* sP = sdO + C::kRowTile;
    float* sdS = sP + C::kPTile;
    T* rQ = reinterpret_cast<T*>(sdS + C::kPTile);  // 16-bit only: raw Q and dO tiles
    T* rO = rQ + kB32Tile * HD;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    // grid (H_k * B, tiles): every KV head's heaviest tile (the first 64 keys, read by
    // every query tile) goes first
    const int k0 = blockIdx.y * kB32Tile;
    const int hk = blockIdx.x % p.Hk, b = blockIdx.x / p.Hk, d = p.d, G = p.G;
    const float sc2 = p.scale * kLog2e;

    // query tile idx: tokens tq0 = k0 + (idx / G) * 64 of head hk*G + idx % G
    const int nq = (p.T - k0 + kB32Tile - 1) / kB32Tile * G;
    auto stage_q = [&](float* dst, T* raw, const ModaTensor& t, int idx) {
        const T* base = b32_head<T>(t, b, hk * G + idx % G);
        const int row0 = k0 + idx / G * kB32Tile;
        if constexpr (kIsF32<T>) b32_stage<HD>(dst, base, t.strides[2], row0, p.T, d, tid);
        else b16_stage<T, HD>(raw, base, t.strides[2], row0, p.T, d, tid);
    };
    if constexpr (kIsF32<T>) {
        b32_stage<HD>(sK, b32_head<float>(p.k, b, hk), p.k.strides[2], k0, p.T, d, tid);
        b32_stage<HD>(sV, b32_head<float>(p.v, b, hk), p.v.strides[2], k0, p.T, d, tid);
        f32_cp_commit();
    } else {  // K and V through the raw Q / dO tiles
        b16_stage<T, HD>(rQ, b32_head<T>(p.k, b, hk), p.k.strides[2], k0, p.T, d, tid);
        b16_stage<T, HD>(rO, b32_head<T>(p.v, b, hk), p.v.strides[2], k0, p.T, d, tid);
        f32_cp_commit();
        f32_cp_wait<0>();
        __syncthreads();
        b16_convert<T, HD>(sK, rQ, tid);
        b16_convert<T, HD>(sV, rO, tid);
        __syncthreads();
    }
    stage_q(sdO, rO, p.dout, 0);
    f32_cp_commit();
    stage_q(sQ, rQ, p.q, 0);
    f32_cp_commit();

    float dk[4][OC], dv[4][OC];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < OC; ++c) dk[i][c] = dv[i][c] = 0.f;

#pragma unroll 1
    for (int idx = 0; idx < nq; ++idx) {
        const int tq0 = k0 + idx / G * kB32Tile, h = hk * G + idx % G;
        // this tile's query columns: lse = +inf past T makes their P (and dS) zero
        float lse2[4], del[4];
        const int64_t rbase = (static_cast<int64_t>(b) * p.Hq + h) * p.T;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int tq = tq0 + tx + 16 * j;
            lse2[j] = tq < p.T ? p.lse[rbase + tq] * kLog2e : INFINITY;
            del[j] = tq < p.T ? p.delta[rbase + tq] : 0.f;
        }
        f32_cp_wait<1>();  // this dO (this Q may still be in flight)
        __syncthreads();
        if constexpr (!kIsF32<T>) {
            b16_convert<T, HD>(sdO, rO, tid);
            __syncthreads();
            if (idx + 1 < nq) stage_q(sdO, rO, p.dout, idx + 1);
            f32_cp_commit();
        }
        float dpt[4][4];
        b32_abt<HD>(dpt, sV, sdO, ty, tx);
        if constexpr (kIsF32<T>) {
            f32_cp_wait<0>();  // this Q
            __syncthreads();
        } else {
            f32_cp_wait<1>();  // this Q (the next dO may still be in flight)
            __syncthreads();
            b16_convert<T, HD>(sQ, rQ, tid);
            __syncthreads();
            if (idx + 1 < nq) stage_q(sQ, rQ, p.q, idx + 1);
            f32_cp_commit();
        }
        float st[4][4];
        b32_abt<HD>(st, sK, sQ, ty, tx);
        // queries before a key are masked: only the first token tile (tq0 == k0) has them,
        // and it also covers keys at or past T for queries < T
        const bool diag = tq0 == k0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int kj = k0 + ty + 16 * i;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int tq = tq0 + tx + 16 * j;
                const float pr = (diag && tq < kj) ? 0.f : ex2(fmaf(st[i][j], sc2, -lse2[j]));
                sP[(ty + 16 * i) * C::kPStride + tx + 16 * j] = pr;
                sdS[(ty + 16 * i) * C::kPStride + tx + 16 * j] = pr * (dpt[i][j] - del[j]);
            }
        }
        __syncthreads();
        b32_pm<HD>(dv, sP, sdO, ty, tx);
        if constexpr (kIsF32<T>) {
            __syncthreads();  // every thread is done with dO and P
            if (idx + 1 < nq) stage_q(sdO, rO, p.dout, idx + 1);
            f32_cp_commit();
        }
        b32_pm<HD>(dk, sdS, sQ, ty, tx);
        __syncthreads();  // every thread is done with Q, dO, P and dS
        if constexpr (kIsF32<T>) {
            if (idx + 1 < nq) stage_q(sQ, rQ, p.q, idx + 1);
            f32_cp_commit();
        }
    }
    f32_cp_wait<0>();
    b32_store<T, HD>(p.dk, b, hk, k0, p.T, d, dk, p.scale, ty, tx);
    b32_store<T, HD>(p.dv, b, hk, k0, p.T, d, dv, 1.f, ty, tx);
}

// Shared memory of the depth kernel, in floats: depth K and V rows [32][d+4], the token's
// query and dO rows [G][d+4], the depth part of dQ [G][d], two [32][gs] score arrays
// (gs = G rounded up to odd, so a warp's 32 rows at one head hit 32 banks), lse and D.
static int b32_depth_floats(int G, int d) {
    const int ds = d + 4, gs = G | 1;
    return 2 * kB32DepthRows * ds + 2 * G * ds + G * d + 2 * kB32DepthRows * gs + 2 * G;
}

template <typename T>
__global__ void __launch_bounds__(kB32DepthThreads) moda_bwd_f32_depth_kernel(const __grid_constant__ BwdParams p) {
    extern __shared__ __align__(16) float b32_smem[];
    const int t = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
    const int G = p.G, d = p.d, ds = d + 4, d4 = d / 4, gs = G | 1;
    float* sKd = b32_smem;
    float* sVd = sKd + kB32DepthRows * ds;
    float* sQ = sVd + kB32DepthRows * ds;
    float* sdO = sQ + G * ds;
    float* sDq = sdO + G * ds;
    float* sA = sDq + G * d;               // scores, then P
    float* sB = sA + kB32DepthRows * gs;   // dO . V_depth, then dS
    float* sLse2 = sB + kB32DepthRows * gs;
    float* sDel = sLse2 + G;
    const int tid = threadIdx.x;
    const float sc2 = p.scale * kLog2e;

    for (int i = tid; i < G * d4; i += kB32DepthThreads) {
        const int g = i / d4, c4 = i % d4, h = hk * G + g;
        b32_stage4<T>(sQ + g * ds + 4 * c4, b32_head<T>(p.q, b, h) + static_cast<int64_t>(t) * p.q.strides[2] + 4 * c4,
                      true);
        b32_stage4<T>(sdO + g * ds + 4 * c4,
                      b32_head<T>(p.dout, b, h) + static_cast<int64_t>(t) * p.dout.strides[2] + 4 * c4, true);
    }
    f32_cp_commit();
    for (int i = tid; i < G * d; i += kB32DepthThreads) sDq[i] = 0.f;
    for (int g = tid; g < G; g += kB32DepthThreads) {
        const int64_t ri = (static_cast<int64_t>(b) * p.Hq + hk * G + g) * p.T + t;
        sLse2[g] = p.lse[ri] * kLog2e;
        sDel[g] = p.delta[ri];
    }
    const T* kdb = b32_head<T>(p.kd, b, hk);
    const T* vdb = b32_head<T>(p.vd, b, hk);
    T* dkdb = static_cast<T*>(p.dkd.ptr) + b * p.dkd.strides[0] + hk * p.dkd.strides[1];
    T* dvdb = static_cast<T*>(p.dvd.ptr) + b * p.dvd.strides[0] + hk * p.dvd.strides[1];
    const int64_t r0 = static_cast<int64_t>(t) * p.L;

#pragma unroll 1
    for (int l0 = 0; l0 < p.L; l0 += kB32DepthRows) {
        const int nr = min(kB32DepthRows, p.L - l0);
        for (int i = tid; i < kB32DepthRows * d4; i += kB32DepthThreads) {
            const int r = i / d4, c4 = i % d4;
            const bool ok = r < nr;
            const int64_t row = r0 + l0 + r;
            b32_stage4<T>(sKd + r * ds + 4 * c4, ok ? kdb + row * p.kd.strides[2] + 4 * c4 : kdb, ok);
            b32_stage4<T>(sVd + r * ds + 4 * c4, ok ? vdb + row * p.vd.strides[2] + 4 * c4 : vdb, ok);
        }
        f32_cp_commit();
        f32_cp_wait<0>();
        __syncthreads();
        // dot products: item (row r, head g, which) -- a warp shares g and which, its
        // lanes take 32 rows
        for (int it = tid; it < 2 * kB32DepthRows * G; it += kB32DepthThreads) {
            const int r = it & (kB32DepthRows - 1), rest = it / kB32DepthRows;
            const int g = rest % G, which = rest / G;
            const float* a = (which ? sVd : sKd) + r * ds;
            const float* q = (which ? sdO : sQ) + g * ds;
            float acc = 0.f;
            for (int c = 0; c < d; c += 4) {
                const float4 av = *reinterpret_cast<const float4*>(a + c);
                const float4 qv = *reinterpret_cast<const float4*>(q + c);
                acc = fmaf(av.x, qv.x, acc);
                acc = fmaf(av.y, qv.y, acc);
                acc = fmaf(av.z, qv.z, acc);
                acc = fmaf(av.w, qv.w, acc);
            }
            (which ? sB : sA)[r * gs + g] = acc;
        }
        __syncthreads();
        for (int it = tid; it < kB32DepthRows * G; it += kB32DepthThreads) {
            const int r = it / G, g = it % G;
            const float pr = r < nr ? ex2(fmaf(sA[r * gs + g], sc2, -sLse2[g])) : 0.f;
            sA[r * gs + g] = pr;
            sB[r * gs + g] = pr * (sB[r * gs + g] - sDel[g]);
        }
        __syncthreads();
        // dK_depth = scale * sum_g dS q_g and dV_depth = sum_g P dO_g, by (row, 4 columns)
        for (int it = tid; it < nr * d4; it += kB32DepthThreads) {
            const int r = it / d4, c4 = it % d4;
            float dk4[4] = {0.f, 0.f, 0.f, 0.f}, dv4[4] = {0.f, 0.f, 0.f, 0.f};
            for (int g = 0; g < G; ++g) {
                const float dsv = sB[r * gs + g], pv = sA[r * gs + g];
                const float4 qv = *reinterpret_cast<const float4*>(sQ + g * ds + 4 * c4);
                const float4 ov = *reinterpret_cast<const float4*>(sdO + g * ds + 4 * c4);
                dk4[0] = fmaf(dsv, qv.x, dk4[0]);
                dk4[1] = fmaf(dsv, qv.y, dk4[1]);
                dk4[2] = fmaf(dsv, qv.z, dk4[2]);
                dk4[3] = fmaf(dsv, qv.w, dk4[3]);
                dv4[0] = fmaf(pv, ov.x, dv4[0]);
                dv4[1] = fmaf(pv, ov.y, dv4[1]);
                dv4[2] = fmaf(pv, ov.z, dv4[2]);
                dv4[3] = fmaf(pv, ov.w, dv4[3]);
            }
            const int64_t row = r0 + l0 + r;
            b32_st4<T>(dkdb + row * p.dkd.strides[2] + 4 * c4, make_float4(dk4[0], dk4[1], dk4[2], dk4[3]), p.scale);
            b32_st4<T>(dvdb + row * p.dvd.strides[2] + 4 * c4, make_float4(dv4[0], dv4[1], dv4[2], dv4[3]), 1.f);
        }
        // the depth part of dQ: sum over this chunk's rows of dS K_depth, by (head, 4 columns)
        for (int it = tid; it < G * d4; it += kB32DepthThreads) {
            const int g = it / d4, c4 = it % d4;
            float4 a = *reinterpret_cast<const float4*>(sDq + g * d + 4 * c4);
            for (int r = 0; r < nr; ++r) {
                const float dsv = sB[r * gs + g];
                const float4 kv = *reinterpret_cast<const float4*>(sKd + r * ds + 4 * c4);
                a.x = fmaf(dsv, kv.x, a.x);
                a.y = fmaf(dsv, kv.y, a.y);
                a.z = fmaf(dsv, kv.z, a.z);
                a.w = fmaf(dsv, kv.w, a.w);
            }
            *reinterpret_cast<float4*>(sDq + g * d + 4 * c4) = a;
        }
        __syncthreads();  // before the next chunk restages the rows and rewrites the scores
    }
    // dQ (the sequence part, from the dq kernel) += scale * the depth part
    for (int it = tid; it < G * d4; it += kB32DepthThreads) {
        const int g = it / d4, c4 = it % d4;
        T* dqr = static_cast<T*>(p.dq.ptr) + b * p.dq.strides[0] + (hk * G + g) * p.dq.strides[1] +
                     static_cast<int64_t>(t) * p.dq.strides[2] + 4 * c4;
        float4 cur = b32_ld4<T>(dqr);
        const float4 a = *reinterpret_cast<const float4*>(sDq + g * d + 4 * c4);
        cur.x = fmaf(p.scale, a.x, cur.x);
        cur.y = fmaf(p.scale, a.y, cur.y);
        cur.z = fmaf(p.scale, a.z, cur.z);
        cur.w = fmaf(p.scale, a.w, cur.w);
        b32_st4<T>(dqr, cur, 1.f);
    }
}

// depth rows [T*L, R) of dK_depth and dV_depth: never read by the forward, zero gradient
template <typename T>
__global__ void moda_bwd_f32_depth_zero_kernel(const __grid_constant__ BwdParams p) {
    const int hk = blockIdx.y, b = blockIdx.z;
    const int64_t first = static_cast<int64_t>(p.T) * p.L;
    const int64_t n = (p.R - first) * p.d;
    T* dk = static_cast<T*>(p.dkd.ptr) + b * p.dkd.strides[0] + hk * p.dkd.strides[1];
    T* dv = static_cast<T*>(p.dvd.ptr) + b * p.dvd.strides[0] + hk * p.dvd.strides[1];
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = first + i / p.d, c = i % p.d;
        dk[r * p.dkd.strides[2] + c * p.dkd.strides[3]] = T{};
        dv[r * p.dvd.strides[2] + c * p.dvd.strides[3]] = T{};
    }
}

// fp32 or 16-bit with d a multiple of 4 up to 128, G <= 32 and unit-stride, 16-byte
// aligned rows (16-byte copies) in every tensor the kernels read or write with vectors.
bool bwd_tiled_ok(const BwdParams& p) {
    const int esz = p.dtype == MODA_F32 ? 4 : (p.dtype == MODA_BF16 || p.dtype == MODA_F16) ? 2 : 0;
    if (esz == 0 || p.d % 4 != 0 || p.d > 128 || p.G > 32) return false;
    if ((p.T + kB32Tile - 1) / kB32Tile > 65535 || static_cast<int64_t>(p.Hq) * p.B > INT32_MAX) return false;
    const ModaTensor* ts[11] = {&p.q, &p.k, &p.v, &p.dout, &p.dq, &p.dk, &p.dv, &p.kd, &p.vd, &p.dkd, &p.dvd};
    const int nts = p.L > 0 ? 11 : 7;
    for (int i = 0; i < nts; ++i) {
        const ModaTensor* t = ts[i];
        if (t->strides[3] != 1 || reinterpret_cast<uintptr_t>(t->ptr) % 16 != 0) return false;
        for (int j = 0; j < 3; ++j)
            if (t->sizes[j] > 1 && (t->strides[j] * esz) % 16 != 0) return false;
    }
    return true;
}

template <typename T, int HD>
static int launch_b32_hd(const BwdParams& p, cudaStream_t stream) {
    using C = B32Cfg<HD>;
    constexpr int raw = kIsF32<T> ? 0 : 2 * kB32Tile * HD * 2;  // two raw 16-bit tiles
    constexpr int dq_bytes = C::kDqBytes + raw, dkv_bytes = C::kDkvBytes + raw;
    static std::atomic<uint64_t> dq_attr{0}, dkv_attr{0};
    if (ensure_smem_attr(dq_attr, moda_bwd_f32_dq_kernel<T, HD>, dq_bytes) != cudaSuccess ||
        ensure_smem_attr(dkv_attr, moda_bwd_f32_dkdv_kernel<T, HD>, dkv_bytes) != cudaSuccess)
        return MODA_ERR_LAUNCH;
    const unsigned tiles = static_cast<unsigned>((p.T + kB32Tile - 1) / kB32Tile);
    moda_bwd_f32_dq_kernel<T, HD><<<dim3(p.Hq * p.B, tiles), kB32Threads, dq_bytes, stream>>>(p);
    moda_bwd_f32_dkdv_kernel<T, HD><<<dim3(p.Hk * p.B, tiles), kB32Threads, dkv_bytes, stream>>>(p);
    return MODA_OK;
}

// dq, dkdv, then depth (which adds into dq) and the zero rows; rowsum(dO * O) is already
// in p.delta.
template <typename T>
static int launch_tiled_t(const BwdParams& p, cudaStream_t stream) {
    if (p.T > 0) {
        const int r = p.d <= 32 ? launch_b32_hd<T, 32>(p, stream)
                      : p.d <= 64 ? launch_b32_hd<T, 64>(p, stream)
                                  : launch_b32_hd<T, 128>(p, stream);
        if (r != MODA_OK) return r;
        if (p.L > 0) {
            static std::atomic<uint64_t> depth_attr{0};
            const int bytes = b32_depth_floats(p.G, p.d) * 4;
            // one opt-in at the largest size any G <= 32, d <= 128 needs
            if (ensure_smem_attr(depth_attr, moda_bwd_f32_depth_kernel<T>, b32_depth_floats(32, 128) * 4) !=
                cudaSuccess)
                return MODA_ERR_LAUNCH;
            moda_bwd_f32_depth_kernel<T><<<dim3(p.T, p.Hk, p.B), kB32DepthThreads, bytes, stream>>>(p);
        }
    }
    const int64_t extra = p.R - static_cast<int64_t>(p.T) * p.L;
    if (extra > 0) {
        const int64_t n = extra * p.d;
        const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 1024));
        moda_bwd_f32_depth_zero_kernel<T><<<dim3(blocks, p.Hk, p.B), 256, 0, stream>>>(p);
    }
    return MODA_OK;
}

int launch_bwd_tiled(const BwdParams& p, cudaStream_t stream) {
    switch (p.dtype) {
        case MODA_F32: return launch_tiled_t<float>(p, stream);
        case MODA_BF16: return launch_tiled_t<__nv_bfloat16>(p, stream);
        case MODA_F16: return launch_tiled_t<__half>(p, stream);
        default: return MODA_ERR_DTYPE;
    }
}

}  // namespace moda
