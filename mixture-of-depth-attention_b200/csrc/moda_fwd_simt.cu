// CUDA-core MoDA forward: any dtype (f32 / bf16 / f16), fp32 FMA throughout.
//
// This is the path for fp32 inputs, whose tolerance (1e-4 relative) tensor-core
// bf16/tf32 products cannot meet, and for the shapes the tcgen05 kernel does not tile
// (16-bit head_dim outside {64, 128}, more than 128 query heads per KV head, layouts
// TMA cannot describe). Two kernels: a tiled one (below) for d a multiple of 4 up to
// 128 with 16-byte aligned rows, and a warp-per-row one for everything else (any
// strides, d <= 256).
//
// Warp-per-row kernel: one warp owns one query row (b, h, t). Lanes split the head dimension; every
// key is one warp-wide dot product, folded into a single online softmax that
// runs over the causal keys 0..t and then over the L depth rows t*L..t*L+L-1
// of the same KV head -- the combined softmax of moda_attention_naive
// (moda/kernels/moda_naive.py:61-95), in streaming form.
#include "moda_internal.h"

namespace moda {

template <typename T>
MODA_DEV float to_f(T x);
template <>
MODA_DEV float to_f<float>(float x) { return x; }
template <>
MODA_DEV float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
MODA_DEV float to_f<__half>(__half x) { return __half2float(x); }

template <typename T>
MODA_DEV T from_f(float x);
template <>
MODA_DEV float from_f<float>(float x) { return x; }
template <>
MODA_DEV __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
MODA_DEV __half from_f<__half>(float x) { return __float2half_rn(x); }

constexpr int kSimtRows = 4;   // warps (query rows) per block
constexpr int kSimtMaxChunks = 8;  // d <= 256

template <typename T>
__global__ void __launch_bounds__(kSimtRows * 32)
    moda_fwd_simt_kernel(const FwdParams p) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * kSimtRows + warp;
    const int h = blockIdx.y;
    const int b = blockIdx.z;
    if (t >= p.T) return;
    const int hk = h / p.G;
    const int d = p.d;

    const T* q = static_cast<const T*>(p.q.ptr) + b * p.q.strides[0] + h * p.q.strides[1] +
                 static_cast<int64_t>(t) * p.q.strides[2];
    float qr[kSimtMaxChunks], acc[kSimtMaxChunks];
#pragma unroll
    for (int i = 0; i < kSimtMaxChunks; ++i) {
        const int c = lane + 32 * i;
        qr[i] = (c < d) ? to_f<T>(q[c * p.q.strides[3]]) : 0.f;
        acc[i] = 0.f;
    }
    const float sc = p.scale * kLog2e;
    float m = -INFINITY, l = 0.f;

    auto consume = [&](const T* krow, int64_t ks, const T* vrow, int64_t vs) {
        float part = 0.f;
#pragma unroll
        for (int i = 0; i < kSimtMaxChunks; ++i) {
            const int c = lane + 32 * i;
            if (c < d) part = fmaf(qr[i], to_f<T>(krow[c * ks]), part);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const float s = part * sc;
        const float m_new = fmaxf(m, s);
        const float alpha = ex2(m - m_new);
        const float pw = ex2(s - m_new);
        l = fmaf(l, alpha, pw);
#pragma unroll
        for (int i = 0; i < kSimtMaxChunks; ++i) {
            const int c = lane + 32 * i;
            const float vv = (c < d) ? to_f<T>(vrow[c * vs]) : 0.f;
            acc[i] = fmaf(acc[i], alpha, pw * vv);
        }
        m = m_new;
    };

    const T* kb = static_cast<const T*>(p.k.ptr) + b * p.k.strides[0] + hk * p.k.strides[1];
    const T* vb = static_cast<const T*>(p.v.ptr) + b * p.v.strides[0] + hk * p.v.strides[1];
    for (int j = 0; j <= t; ++j)
        consume(kb + j * p.k.strides[2], p.k.strides[3], vb + j * p.v.strides[2], p.v.strides[3]);

    const T* kdb = static_cast<const T*>(p.kd.ptr) + b * p.kd.strides[0] + hk * p.kd.strides[1];
    const T* vdb = static_cast<const T*>(p.vd.ptr) + b * p.vd.strides[0] + hk * p.vd.strides[1];
    const int64_t r0 = static_cast<int64_t>(t) * p.L;
    for (int li = 0; li < p.L; ++li)
        consume(kdb + (r0 + li) * p.kd.strides[2], p.kd.strides[3], vdb + (r0 + li) * p.vd.strides[2],
                p.vd.strides[3]);

    if (p.zero_rows > 0) {  // zero_rows more keys of score 0 whose values are 0
        const float m_new = fmaxf(m, 0.f);
        const float alpha = ex2(m - m_new);
        l = fmaf(l, alpha, static_cast<float>(p.zero_rows) * ex2(-m_new));
#pragma unroll
        for (int i = 0; i < kSimtMaxChunks; ++i) acc[i] *= alpha;
        m = m_new;
    }
    const float inv = 1.f / l;
    if (p.lse && lane == 0)  // natural log of sum_j exp(scale * q.k_j)
        p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.T + t] = (m + __log2f(l)) * kLn2;
    T* o = static_cast<T*>(p.o.ptr) + b * p.o.strides[0] + h * p.o.strides[1] +
           static_cast<int64_t>(t) * p.o.strides[2];
#pragma unroll
    for (int i = 0; i < kSimtMaxChunks; ++i) {
        const int c = lane + 32 * i;
        if (c < d) o[c * p.o.strides[3]] = from_f<T>(acc[i] * inv);
    }
}

// ---------------------------------------------------------------- fp32, tiled
// The fp32 forward on CUDA cores, tiled like a GEMM so that every value read from
// shared memory feeds several FMAs (the warp-per-row kernel above re-reads each key for
// every query row and reduces every dot product across a warp). fp32 FMA throughout, so
// the fp32 tolerance holds; only the summation order differs from the row kernel.
//
// A CTA (256 threads) takes 128 consecutive tokens of one query head. Thread (ty, tx),
// ty = tid / 16, tx = tid % 16, owns query rows ty + 16i (i < 8) and, of each 64-key
// tile, keys tx + 16j (j < 4); of the output it owns OC = HD / 16 columns, in groups of
// VW = 4 adjacent ones (2 when HD = 32) at column g*16*VW + tx*VW, so the 16 threads of a
// row read one contiguous segment of a V row per access. The 16 threads of a row sit in
// one half-warp, so row maxima and sums are 4 shuffles. Per CTA:
//   1. the depth rows first: for each of its rows, the row's 16 threads take L depth rows
//      (two per thread per 32-row chunk), compute their scores against Q from shared
//      memory, softmax them, and accumulate P.V_depth straight into their own O columns;
//      this seeds the online softmax (m, l, O);
//   2. the causal keys in 64-key tiles: S = Q K^T from shared memory (8 x 4 per thread),
//      the diagonal tiles masked, online softmax, P through shared memory, O += P V.
//      K and V tiles arrive by cp.async; the next tile's K is copied during the softmax
//      and P.V of this one, the next V during the next S.
// Q, K and V rows in shared memory are padded by 4 floats, so the 16 rows a half-warp
// reads at one column fall into different banks; P rows by 16, so the two rows a warp
// writes at one key do too.
constexpr int kF32Rows = 128, kF32Keys = 64;
constexpr int kF32RowsPerThread = 8;  // query rows of a thread's 8 x 4 score block
__host__ __device__ constexpr int f32_threads(int rpt) { return kF32Rows / rpt * 16; }

template <int HD>
struct F32Cfg {
    static constexpr int kStride = HD + 4;                     // floats per staged row
    static constexpr int kQ = 0;                                // Q   [128][HD+4]
    static constexpr int kK = kQ + kF32Rows * kStride;          // K   [64][HD+4]
    static constexpr int kV = kK + kF32Keys * kStride;          // V   [64][HD+4]
    static constexpr int kPStride = kF32Keys + 16;             // a warp's two P rows 16 banks apart
    static constexpr int kP = kV + kF32Keys * kStride;          // P   [128][64+16]
    static constexpr int kFloats = kP + kF32Rows * kPStride;
    static constexpr int kBytes = kFloats * 4;
};

template <typename T, int HD, int RPT>
__global__ void __launch_bounds__(f32_threads(RPT), 1) moda_fwd_f32_tiled_kernel(const FwdParams p) {
    using C = F32Cfg<HD>;
    // RPT query rows per thread, RS apart (RS = 128 / RPT threads per key column)
    constexpr int NT = f32_threads(RPT), RS = kF32Rows / RPT;
    // a thread's OC output columns: NG groups of VW adjacent columns, group g at column
    // g*16*VW + tx*VW, so the 16 threads of a row read one contiguous V segment per access
    constexpr int OC = HD / 16;
    constexpr int VW = OC >= 4 ? 4 : 2;
    constexpr int NG = OC / VW;
    extern __shared__ __align__(16) float f32_smem[];
    float* sQ = f32_smem + C::kQ;
    float* sK = f32_smem + C::kK;
    float* sV = f32_smem + C::kV;
    float* sP = f32_smem + C::kP;
    T* rK = reinterpret_cast<T*>(f32_smem + C::kFloats);  // 16-bit only: raw K and V tiles
    T* rV = rK + kF32Keys * HD;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int ntiles = (p.T + kF32Rows - 1) / kF32Rows;
    // grid (H_q * B, tiles): dispatch runs x fastest, so every head's heaviest tile (the
    // last 128 tokens) goes first, then every head's next one
    const int t0 = (ntiles - 1 - static_cast<int>(blockIdx.y)) * kF32Rows;
    const int h = blockIdx.x % p.Hq, b = blockIdx.x / p.Hq, hk = h / p.G;
    const int d = p.d;
    const T* qb = static_cast<const T*>(p.q.ptr) + b * p.q.strides[0] + h * p.q.strides[1];
    const T* kb = static_cast<const T*>(p.k.ptr) + b * p.k.strides[0] + hk * p.k.strides[1];
    const T* vb = static_cast<const T*>(p.v.ptr) + b * p.v.strides[0] + hk * p.v.strides[1];
    const float sc = p.scale * kLog2e;

    // fp32: stage `rows` rows starting at row0 of a [.., rows, d] view into dst (zeros
    // past T or d); 16-bit rows go through the raw tiles (raw16_stage, raw16_convert)
    auto stage = [&](float* dst, const float* base, int64_t rstride, int row0, int rows, int limit) {
        for (int i = tid; i < rows * (HD / 4); i += NT) {
            const int r = i / (HD / 4), c4 = i % (HD / 4);
            const bool ok = row0 + r < limit && 4 * c4 < d;
            const float* src = ok ? base + static_cast<int64_t>(row0 + r) * rstride + 4 * c4 : base;
            f32_cp16(dst + r * C::kStride + 4 * c4, src, ok ? 16 : 0);
        }
    };
    const int kmax = min(t0 + kF32Rows, p.T);           // keys [0, kmax) are needed
    const int nkt = (kmax + kF32Keys - 1) / kF32Keys;    // causal key tiles
    if constexpr (kIsF32<T>) {
        stage(sQ, qb, p.q.strides[2], t0, kF32Rows, p.T);
        f32_cp_commit();
        stage(sK, kb, p.k.strides[2], 0, kF32Keys, p.T);
        f32_cp_commit();
        stage(sV, vb, p.v.strides[2], 0, kF32Keys, p.T);
        f32_cp_commit();
    } else {  // Q in two 64-row halves through the raw K / V tiles, then the first K and V
        raw16_stage<T, HD, kF32Keys, NT>(rK, qb, p.q.strides[2], t0, p.T, d, tid);
        raw16_stage<T, HD, kF32Keys, NT>(rV, qb, p.q.strides[2], t0 + kF32Keys, p.T, d, tid);
        f32_cp_commit();
        f32_cp_wait<0>();
        __syncthreads();
        raw16_convert<T, HD, kF32Keys, NT>(sQ, rK, tid);
        raw16_convert<T, HD, kF32Keys, NT>(sQ + kF32Keys * C::kStride, rV, tid);
        __syncthreads();
        raw16_stage<T, HD, kF32Keys, NT>(rK, kb, p.k.strides[2], 0, p.T, d, tid);
        f32_cp_commit();
        raw16_stage<T, HD, kF32Keys, NT>(rV, vb, p.v.strides[2], 0, p.T, d, tid);
        f32_cp_commit();
    }

    float o[RPT][OC], m[RPT], l[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < OC; ++c) o[i][c] = 0.f;
    }
    f32_cp_wait<2>();  // Q
    __syncthreads();

    // ---- 1. depth rows: row ty + RS*i is token t0 + ty + RS*i; its 16 threads split the L rows
    if (p.L > 0) {
        const T* kdb = static_cast<const T*>(p.kd.ptr) + b * p.kd.strides[0] + hk * p.kd.strides[1];
        const T* vdb = static_cast<const T*>(p.vd.ptr) + b * p.vd.strides[0] + hk * p.vd.strides[1];
#pragma unroll
        for (int i = 0; i < RPT; ++i) {  // unrolled: o, m and l stay in registers
            const int r = ty + RS * i, t = t0 + r;
            // rows past T (last tile) run the same shuffles with nothing read or kept: the
            // two rows of a warp must stay converged
            const bool valid = t < p.T;
            const float* qr = sQ + r * C::kStride;
            const int64_t row0 = static_cast<int64_t>(valid ? t : 0) * p.L;
#pragma unroll 1
            for (int l0 = 0; l0 < p.L; l0 += 32) {
                // scores of depth rows l0 .. l0 + nrows - 1: the row's 16 threads split each
                // depth row's columns like their O columns (one contiguous segment per
                // access) and sum the partial dot products over the half-warp; depth row u
                // stays with thread u % 16, slot u / 16 (a past-T row reads token 0's rows
                // and keeps nothing)
                const int nrows = min(32, p.L - l0);
                float qa[OC];
#pragma unroll
                for (int g = 0; g < NG; ++g) f32_ldv<VW>(qa + g * VW, qr + g * 16 * VW + tx * VW);
                float s2[2] = {-INFINITY, -INFINITY};
                // 8 depth rows per step: their loads are issued before any of them is used
#pragma unroll 1
                for (int u0 = 0; u0 < nrows; u0 += 8) {
                    float kv[8][OC];
#pragma unroll
                    for (int uu = 0; uu < 8; ++uu) {
                        const bool okr = u0 + uu < nrows;  // the same for the whole warp
                        const T* kr = kdb + (row0 + l0 + (okr ? u0 + uu : 0)) * p.kd.strides[2] + tx * VW;
#pragma unroll
                        for (int g = 0; g < NG; ++g) {
                            if (okr && tx * VW + g * 16 * VW < d) ldv_as_f32<T, VW>(kv[uu] + g * VW, kr + g * 16 * VW);
                            else
#pragma unroll
                                for (int w = 0; w < VW; ++w) kv[uu][g * VW + w] = 0.f;
                        }
                    }
                    float part[8];
#pragma unroll
                    for (int uu = 0; uu < 8; ++uu) {
                        part[uu] = 0.f;
#pragma unroll
                        for (int c = 0; c < OC; ++c) part[uu] = fmaf(qa[c], kv[uu][c], part[uu]);
                    }
#pragma unroll
                    for (int off = 1; off < 16; off <<= 1)
#pragma unroll
                        for (int uu = 0; uu < 8; ++uu) part[uu] += __shfl_xor_sync(0xffffffffu, part[uu], off);
#pragma unroll
                    for (int uu = 0; uu < 8; ++uu) {
                        const int u = u0 + uu;
                        if (u < nrows && u == tx) s2[0] = part[uu] * sc;
                        if (u < nrows && u == tx + 16) s2[1] = part[uu] * sc;
                    }
                }
                float mx = fmaxf(s2[0], s2[1]);
#pragma unroll
                for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                // finite for a valid row: the chunk has >= 1 depth row
                const float m_new = valid ? fmaxf(m[i], mx) : 0.f;
                const float alpha = valid ? ex2(m[i] - m_new) : 1.f;
                const float p0 = valid ? ex2(s2[0] - m_new) : 0.f, p1 = valid ? ex2(s2[1] - m_new) : 0.f;
                l[i] = fmaf(l[i], alpha, p0 + p1);  // this thread's share of the row sum
                if (valid) m[i] = m_new;
#pragma unroll
                for (int c = 0; c < OC; ++c) o[i][c] *= alpha;
#pragma unroll 1
                for (int u0 = 0; u0 < nrows; u0 += 8) {
                    float vv[8][OC];
#pragma unroll
                    for (int uu = 0; uu < 8; ++uu) {
                        const bool okr = valid && u0 + uu < nrows;
                        const T* vr = vdb + (row0 + l0 + (okr ? u0 + uu : 0)) * p.vd.strides[2] + tx * VW;
#pragma unroll
                        for (int g = 0; g < NG; ++g) {
                            if (okr && tx * VW + g * 16 * VW < d) ldv_as_f32<T, VW>(vv[uu] + g * VW, vr + g * 16 * VW);
                            else
#pragma unroll
                                for (int w = 0; w < VW; ++w) vv[uu][g * VW + w] = 0.f;
                        }
                    }
#pragma unroll
                    for (int uu = 0; uu < 8; ++uu) {
                        // p of depth row u lives in thread (u % 16), slot u / 16 of this
                        // half-warp; rows at or past nrows have p = 0 and zero values
                        const int u = u0 + uu;
                        const float pu = __shfl_sync(0xffffffffu, u < 16 ? p0 : p1, (tid & 16) + (u & 15));
#pragma unroll
                        for (int c = 0; c < OC; ++c) o[i][c] = fmaf(pu, vv[uu][c], o[i][c]);
                    }
                }
            }
        }
    }

    // ---- 2. causal key tiles
#pragma unroll 1
    for (int kt = 0; kt < nkt; ++kt) {
        f32_cp_wait<1>();  // this tile's K (its V may still be in flight)
        __syncthreads();
        if constexpr (!kIsF32<T>) {
            raw16_convert<T, HD, kF32Keys, NT>(sK, rK, tid);
            __syncthreads();
            if (kt + 1 < nkt) raw16_stage<T, HD, kF32Keys, NT>(rK, kb, p.k.strides[2], (kt + 1) * kF32Keys, p.T, d, tid);
            f32_cp_commit();
        }
        float s[RPT][4];
#pragma unroll
        for (int i = 0; i < RPT; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
        for (int c = 0; c < HD; c += 4) {
            float4 qv[RPT], kv[4];
#pragma unroll
            for (int i = 0; i < RPT; ++i) qv[i] = *reinterpret_cast<const float4*>(sQ + (ty + RS * i) * C::kStride + c);
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(sK + (tx + 16 * j) * C::kStride + c);
#pragma unroll
            for (int i = 0; i < RPT; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
                    s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
                    s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
                    s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
                }
        }
        if constexpr (kIsF32<T>) {
            __syncthreads();  // every thread is done with this K tile
            if (kt + 1 < nkt) stage(sK, kb, p.k.strides[2], (kt + 1) * kF32Keys, kF32Keys, p.T);
            f32_cp_commit();
        }
        // online softmax over this tile; keys after the row's token are masked
        const bool diag = kt * kF32Keys + kF32Keys - 1 > t0;
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int ti = t0 + ty + RS * i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kj = kt * kF32Keys + tx + 16 * j;
                s[i][j] = (diag && kj > ti) ? -INFINITY : s[i][j] * sc;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m[i], mx);
            const float mb = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = ex2(m[i] - mb);
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float pj = ex2(s[i][j] - mb);
                ps += pj;
                sP[(ty + RS * i) * C::kPStride + tx + 16 * j] = pj;
            }
            l[i] = fmaf(l[i], alpha, ps);
            m[i] = m_new;
#pragma unroll
            for (int c = 0; c < OC; ++c) o[i][c] *= alpha;
        }
        f32_cp_wait<1>();  // this tile's V (the next K may still be in flight)
        __syncthreads();   // and P from every thread
        if constexpr (!kIsF32<T>) {
            raw16_convert<T, HD, kF32Keys, NT>(sV, rV, tid);
            __syncthreads();
            if (kt + 1 < nkt) raw16_stage<T, HD, kF32Keys, NT>(rV, vb, p.v.strides[2], (kt + 1) * kF32Keys, p.T, d, tid);
            f32_cp_commit();
        }
#pragma unroll 2
        for (int k = 0; k < kF32Keys; k += 4) {
            float4 pv[RPT];
#pragma unroll
            for (int i = 0; i < RPT; ++i) pv[i] = *reinterpret_cast<const float4*>(sP + (ty + RS * i) * C::kPStride + k);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float* vr = sV + (k + kk) * C::kStride + tx * VW;
                float vv[OC];
#pragma unroll
                for (int g = 0; g < NG; ++g) f32_ldv<VW>(vv + g * VW, vr + g * 16 * VW);
#pragma unroll
                for (int i = 0; i < RPT; ++i) {
                    const float pk = kk == 0 ? pv[i].x : kk == 1 ? pv[i].y : kk == 2 ? pv[i].z : pv[i].w;
#pragma unroll
                    for (int c = 0; c < OC; ++c) o[i][c] = fmaf(pk, vv[c], o[i][c]);
                }
            }
        }
        if constexpr (kIsF32<T>) {
            __syncthreads();  // every thread is done with this V tile and with P
            if (kt + 1 < nkt) stage(sV, vb, p.v.strides[2], (kt + 1) * kF32Keys, kF32Keys, p.T);
            f32_cp_commit();
        }  // 16-bit: the next tile's first barrier orders its K conversion after this P V
    }
    f32_cp_wait<0>();

    // ---- epilogue: O / l, the zero_rows keys, the log-sum-exp
    T* obase = static_cast<T*>(p.o.ptr) + b * p.o.strides[0] + h * p.o.strides[1];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        float lt = l[i];
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
        float mf = m[i], a = 1.f;
        if (p.zero_rows > 0) {  // zero_rows more keys of score 0 whose values are 0
            mf = fmaxf(m[i], 0.f);
            a = ex2(m[i] - mf);
            lt = fmaf(lt, a, static_cast<float>(p.zero_rows) * ex2(-mf));
        }
        const int t = t0 + ty + RS * i;
        if (t >= p.T) continue;
        const float inv = a / lt;
        if (p.lse && tx == 0)  // natural log of sum_j exp(scale * q.k_j)
            p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.T + t] = (mf + __log2f(lt)) * kLn2;
        T* orow = obase + static_cast<int64_t>(t) * p.o.strides[2] + tx * VW;
#pragma unroll
        for (int g = 0; g < NG; ++g)
            if (tx * VW + g * 16 * VW < d) stv_from_f32<T, VW>(orow + g * 16 * VW, o[i] + g * VW, inv);
    }
}

// The tiled kernel serves fp32, and bf16 / f16 that the tensor-core kernel does not take,
// with d a multiple of 4 up to 128 and unit-stride, 16-byte aligned rows (16-byte
// copies); everything else takes the row kernel.
static bool tiled_ok(const FwdParams& p) {
    const int esz = p.dtype == MODA_F32 ? 4 : (p.dtype == MODA_BF16 || p.dtype == MODA_F16) ? 2 : 0;
    if (esz == 0 || p.d % 4 != 0 || p.d > 128) return false;
    if ((p.T + kF32Rows - 1) / kF32Rows > 65535 || static_cast<int64_t>(p.Hq) * p.B > INT32_MAX) return false;
    const ModaTensor* ts[6] = {&p.q, &p.k, &p.v, &p.o, &p.kd, &p.vd};
    const int nts = p.L > 0 ? 6 : 4;
    for (int i = 0; i < nts; ++i) {
        const ModaTensor* t = ts[i];
        if (t->strides[3] != 1 || reinterpret_cast<uintptr_t>(t->ptr) % 16 != 0) return false;
        for (int j = 0; j < 3; ++j)
            if (t->sizes[j] > 1 && (t->strides[j] * esz) % 16 != 0) return false;
    }
    return true;
}

template <typename T, int HD>
static int launch_tiled_hd(const FwdParams& p, cudaStream_t stream) {
    using C = F32Cfg<HD>;
    static std::atomic<uint64_t> attr_done{0};
    constexpr int RPT = kF32RowsPerThread;
    constexpr int bytes = C::kBytes + (kIsF32<T> ? 0 : 2 * kF32Keys * HD * 2);  // + raw K, V tiles
    if (ensure_smem_attr(attr_done, moda_fwd_f32_tiled_kernel<T, HD, RPT>, bytes) != cudaSuccess)
        return MODA_ERR_LAUNCH;
    const dim3 grid(p.Hq * p.B, (p.T + kF32Rows - 1) / kF32Rows);
    moda_fwd_f32_tiled_kernel<T, HD, RPT><<<grid, f32_threads(RPT), bytes, stream>>>(p);
    return MODA_OK;
}

template <typename T>
static int launch_tiled_t(const FwdParams& p, cudaStream_t stream) {
    if (p.d <= 32) return launch_tiled_hd<T, 32>(p, stream);
    if (p.d <= 64) return launch_tiled_hd<T, 64>(p, stream);
    return launch_tiled_hd<T, 128>(p, stream);
}

int launch_fwd_simt(const FwdParams& p, cudaStream_t stream) {
    if (tiled_ok(p)) {
        if (p.dtype == MODA_F32) return launch_tiled_t<float>(p, stream);
        if (p.dtype == MODA_BF16) return launch_tiled_t<__nv_bfloat16>(p, stream);
        return launch_tiled_t<__half>(p, stream);
    }
    const dim3 grid((p.T + kSimtRows - 1) / kSimtRows, p.Hq, p.B);
    const dim3 block(kSimtRows * 32);
    switch (p.dtype) {
        case MODA_F32: moda_fwd_simt_kernel<float><<<grid, block, 0, stream>>>(p); break;
        case MODA_BF16: moda_fwd_simt_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(p); break;
        case MODA_F16: moda_fwd_simt_kernel<__half><<<grid, block, 0, stream>>>(p); break;
        default: return MODA_ERR_DTYPE;
    }
    return MODA_OK;
}

// ---------------------------------------------------------------- depth append
// k_cache[b,h,t*L+layer,:] = k_src[b,h,t,:] (and v), both tensors in one launch:
// blockIdx.y selects k (0) or v (1). Rows move as 16-byte vectors when every
// row start is 16-byte aligned, else element by element.
template <int ESZ, bool VEC16>
__global__ void moda_depth_append_kernel(const AppendParams p) {
    const ModaTensor& src = blockIdx.y == 0 ? p.k_src : p.v_src;
    const ModaTensor& dst = blockIdx.y == 0 ? p.k_cache : p.v_cache;
    const int units_per_row = VEC16 ? (p.d * ESZ) / 16 : p.d;
    const int64_t total = static_cast<int64_t>(p.B) * p.H * p.T * units_per_row;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int u = static_cast<int>(i % units_per_row);
        int64_t r = i / units_per_row;
        const int t = static_cast<int>(r % p.T);
        r /= p.T;
        const int h = static_cast<int>(r % p.H);
        const int b = static_cast<int>(r / p.H);
        const int64_t drow = static_cast<int64_t>(t) * p.L + p.layer;
        const char* s = static_cast<const char*>(src.ptr) +
                        ESZ * (b * src.strides[0] + h * src.strides[1] + t * src.strides[2]);
        char* dd = static_cast<char*>(dst.ptr) +
                   ESZ * (b * dst.strides[0] + h * dst.strides[1] + drow * dst.strides[2]);
        if constexpr (VEC16) {
            reinterpret_cast<uint4*>(dd)[u] = reinterpret_cast<const uint4*>(s)[u];
        } else {
            const int64_t so = u * src.strides[3] * ESZ, dof = u * dst.strides[3] * ESZ;
            if constexpr (ESZ == 4)
                *reinterpret_cast<uint32_t*>(dd + dof) = *reinterpret_cast<const uint32_t*>(s + so);
            else
                *reinterpret_cast<uint16_t*>(dd + dof) = *reinterpret_cast<const uint16_t*>(s + so);
        }
    }
}

int launch_depth_append(const AppendParams& p, bool vec16, cudaStream_t stream) {
    const int esz = p.dtype == MODA_F32 ? 4 : 2;
    const int units = vec16 ? (p.d * esz) / 16 : p.d;
    const int64_t total = static_cast<int64_t>(p.B) * p.H * p.T * units;
    if (total == 0) return MODA_OK;
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    const dim3 grid(static_cast<unsigned>(blocks), 2);
    if (esz == 4) {
        if (vec16) moda_depth_append_kernel<4, true><<<grid, threads, 0, stream>>>(p);
        else moda_depth_append_kernel<4, false><<<grid, threads, 0, stream>>>(p);
    } else {
        if (vec16) moda_depth_append_kernel<2, true><<<grid, threads, 0, stream>>>(p);
        else moda_depth_append_kernel<2, false><<<grid, threads, 0, stream>>>(p);
    }
    return MODA_OK;
}

}  // namespace moda
