// MoDA backward on CUDA cores: gradients of the fused sequence + depth attention.
//
// The reference trains through torch autograd of moda_attention_naive
// (moda/kernels/moda_naive.py:13-162; its tests differentiate through it,
// tests/test_kernel.py:106-119). For query row i with key set
// {causal keys j <= t} U {own depth rows t*L + l}:
//   P_ij = exp(scale*q_i.k_j - lse_i)           (lse from the forward)
//   dP_ij = dO_i.v_j,  D_i = dO_i.O_i,  dS_ij = P_ij (dP_ij - D_i)
//   dQ_i = scale * sum_j dS_ij k_j
//   dK_j = scale * sum_i dS_ij q_i,  dV_j = sum_i P_ij dO_i
// where the sums over i run over every query row that attends j: all G query
// heads of the KV head (GQA) and, for a depth row, only the rows of its token.
//
// Four launches, no atomics (every output element has one writer):
//   delta   one warp per query row: D_i into the caller's workspace;
//   dq      one warp per query row; keys in groups of 32, one lane per key for
//           the two dot products (q.k, dO.v), then the warp folds dS_ij k_j into
//           the row (lanes split d);
//   dkdv    one warp per sequence key row; its query rows (tokens >= j, all G
//           heads) in groups of 32, one lane per row, then the warp folds
//           dS q and P dO into the key row;
//   ddepth  one warp per depth row; the G query rows of its token. Rows at or
//           beyond T*L are never read by the forward and get zero gradient.
// fp32 arithmetic throughout; inputs and gradients in the forward's dtype.
#include "moda_internal.h"

namespace moda {

namespace {

template <typename T>
MODA_DEV float ld(const T* p);
template <>
MODA_DEV float ld<float>(const float* p) { return *p; }
template <>
MODA_DEV float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
MODA_DEV float ld<__half>(const __half* p) { return __half2float(*p); }

template <typename T>
MODA_DEV void st(T* p, float x);
template <>
MODA_DEV void st<float>(float* p, float x) { *p = x; }
template <>
MODA_DEV void st<__nv_bfloat16>(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
template <>
MODA_DEV void st<__half>(__half* p, float x) { *p = __float2half_rn(x); }

constexpr int kRows = 4;       // warps per block
constexpr int kMaxD = 256;
constexpr int kChunks = kMaxD / 32;

// Row base pointer of a [B, H, rows, d] view.
template <typename T>
MODA_DEV T* row_ptr(const ModaTensor& t, int b, int h, int64_t r) {
    return static_cast<T*>(t.ptr) + b * t.strides[0] + h * t.strides[1] + r * t.strides[2];
}

// sum_e a[e] * row[e*s3] with a[] in shared memory (broadcast reads).
template <typename T>
MODA_DEV float dot_row(const float* a, const T* row, int64_t s3, int d) {
    float acc0 = 0.f, acc1 = 0.f;
    int e = 0;
    for (; e + 1 < d; e += 2) {
        acc0 = fmaf(a[e], ld<T>(row + e * s3), acc0);
        acc1 = fmaf(a[e + 1], ld<T>(row + (e + 1) * s3), acc1);
    }
    if (e < d) acc0 = fmaf(a[e], ld<T>(row + e * s3), acc0);
    return acc0 + acc1;
}

// Copy one row into shared memory as fp32 (lanes split d).
template <typename T>
MODA_DEV void stage_row(float* dst, const T* row, int64_t s3, int d, int lane) {
    for (int e = lane; e < d; e += 32) dst[e] = ld<T>(row + e * s3);
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kRows * 32) moda_bwd_delta_kernel(const __grid_constant__ BwdParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kRows + warp, h = blockIdx.y, b = blockIdx.z;
    if (t >= p.T) return;
    const T* o = row_ptr<const T>(p.o, b, h, t);
    const T* g = row_ptr<const T>(p.dout, b, h, t);
    float acc = 0.f;
    for (int e = lane; e < p.d; e += 32)
        acc = fmaf(ld<T>(o + e * p.o.strides[3]), ld<T>(g + e * p.dout.strides[3]), acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) p.delta[(static_cast<int64_t>(b) * p.Hq + h) * p.T + t] = acc;
}

template <typename T>
__global__ void __launch_bounds__(kRows * 32) moda_bwd_dq_kernel(const __grid_constant__ BwdParams p) {
    __shared__ float s_q[kRows][kMaxD], s_do[kRows][kMaxD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kRows + warp, h = blockIdx.y, b = blockIdx.z;
    if (t >= p.T) return;
    const int hk = h / p.G, d = p.d;
    stage_row<T>(s_q[warp], row_ptr<const T>(p.q, b, h, t), p.q.strides[3], d, lane);
    stage_row<T>(s_do[warp], row_ptr<const T>(p.dout, b, h, t), p.dout.strides[3], d, lane);
    __syncwarp();
    const int64_t ri = (static_cast<int64_t>(b) * p.Hq + h) * p.T + t;
    const float lse2 = p.lse[ri] * kLog2e, delta = p.delta[ri], sc2 = p.scale * kLog2e;
    float acc[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) acc[c] = 0.f;

    // n <= 32 keys starting at row r0 of (kt, vt): one lane per key for the dot
    // products, then every lane folds dS_j * k_j into its slice of d.
    auto group = [&](const ModaTensor& kt, const ModaTensor& vt, int64_t r0, int n) {
        float ds = 0.f;
        if (lane < n) {
            const float s = dot_row<T>(s_q[warp], row_ptr<const T>(kt, b, hk, r0 + lane), kt.strides[3], d);
            const float dp = dot_row<T>(s_do[warp], row_ptr<const T>(vt, b, hk, r0 + lane), vt.strides[3], d);
            const float pr = ex2(fmaf(s, sc2, -lse2));
            ds = pr * (dp - delta);
        }
        for (int j = 0; j < n; ++j) {
            const float dsj = __shfl_sync(0xffffffffu, ds, j);
            const T* kr = row_ptr<const T>(kt, b, hk, r0 + j);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                const int e = lane + 32 * c;
                if (e < d) acc[c] = fmaf(dsj, ld<T>(kr + e * kt.strides[3]), acc[c]);
            }
        }
    };
    for (int j0 = 0; j0 <= t; j0 += 32) group(p.k, p.v, j0, min(32, t + 1 - j0));
    const int64_t d0 = static_cast<int64_t>(t) * p.L;
    for (int l0 = 0; l0 < p.L; l0 += 32) group(p.kd, p.vd, d0 + l0, min(32, p.L - l0));

    T* dq = row_ptr<T>(p.dq, b, h, t);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        const int e = lane + 32 * c;
        if (e < d) st<T>(dq + e * p.dq.strides[3], acc[c] * p.scale);
    }
}

// Key-row gradients. DEPTH = false: sequence key j, query rows (t >= j, all G heads).
// DEPTH = true: depth row r of token r / L, query rows (that token, all G heads).
template <typename T, bool DEPTH>
__global__ void __launch_bounds__(kRows * 32) moda_bwd_dkdv_kernel(const __grid_constant__ BwdParams p) {
    __shared__ float s_k[kRows][kMaxD], s_v[kRows][kMaxD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * kRows + warp;
    const int hk = blockIdx.y, b = blockIdx.z, d = p.d;
    const ModaTensor& kt = DEPTH ? p.kd : p.k;
    const ModaTensor& vt = DEPTH ? p.vd : p.v;
    const ModaTensor& dkt = DEPTH ? p.dkd : p.dk;
    const ModaTensor& dvt = DEPTH ? p.dvd : p.dv;
    const int64_t rows = DEPTH ? p.R : p.T;
    if (r >= rows) return;
    T* dk = row_ptr<T>(dkt, b, hk, r);
    T* dv = row_ptr<T>(dvt, b, hk, r);
    if (DEPTH && r >= static_cast<int64_t>(p.T) * p.L) {  // never read by the forward
        for (int e = lane; e < d; e += 32) {
            st<T>(dk + e * dkt.strides[3], 0.f);
            st<T>(dv + e * dvt.strides[3], 0.f);
        }
        return;
    }
    stage_row<T>(s_k[warp], row_ptr<const T>(kt, b, hk, r), kt.strides[3], d, lane);
    stage_row<T>(s_v[warp], row_ptr<const T>(vt, b, hk, r), vt.strides[3], d, lane);
    __syncwarp();
    const float sc2 = p.scale * kLog2e;
    float ak[kChunks], av[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) ak[c] = av[c] = 0.f;
    // query rows: index n -> token t0 + n / G, head hk*G + n % G
    const int t0 = DEPTH ? static_cast<int>(r / p.L) : static_cast<int>(r);
    const int ntok = DEPTH ? 1 : p.T - t0;
    const int nrows = ntok * p.G;
    for (int n0 = 0; n0 < nrows; n0 += 32) {
        const int n = min(32, nrows - n0);
        float ds = 0.f, pr = 0.f;
        if (lane < n) {
            const int t = t0 + (n0 + lane) / p.G, h = hk * p.G + (n0 + lane) % p.G;
            const float s = dot_row<T>(s_k[warp], row_ptr<const T>(p.q, b, h, t), p.q.strides[3], d);
            const float dp = dot_row<T>(s_v[warp], row_ptr<const T>(p.dout, b, h, t), p.dout.strides[3], d);
            const int64_t ri = (static_cast<int64_t>(b) * p.Hq + h) * p.T + t;
            pr = ex2(fmaf(s, sc2, -p.lse[ri] * kLog2e));
            ds = pr * (dp - p.delta[ri]);
        }
        for (int j = 0; j < n; ++j) {
            const float dsj = __shfl_sync(0xffffffffu, ds, j);
            const float prj = __shfl_sync(0xffffffffu, pr, j);
            const int t = t0 + (n0 + j) / p.G, h = hk * p.G + (n0 + j) % p.G;
            const T* qr = row_ptr<const T>(p.q, b, h, t);
            const T* gr = row_ptr<const T>(p.dout, b, h, t);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                const int e = lane + 32 * c;
                if (e < d) {
                    ak[c] = fmaf(dsj, ld<T>(qr + e * p.q.strides[3]), ak[c]);
                    av[c] = fmaf(prj, ld<T>(gr + e * p.dout.strides[3]), av[c]);
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        const int e = lane + 32 * c;
        if (e < d) {
            st<T>(dk + e * dkt.strides[3], ak[c] * p.scale);
            st<T>(dv + e * dvt.strides[3], av[c]);
        }
    }
}

template <typename T>
static void launch_bwd_t(const BwdParams& p, cudaStream_t stream) {
    const dim3 block(kRows * 32);
    const dim3 gq((p.T + kRows - 1) / kRows, p.Hq, p.B);
    moda_bwd_delta_kernel<T><<<gq, block, 0, stream>>>(p);
    moda_bwd_dq_kernel<T><<<gq, block, 0, stream>>>(p);
    const dim3 gk((p.T + kRows - 1) / kRows, p.Hk, p.B);
    moda_bwd_dkdv_kernel<T, false><<<gk, block, 0, stream>>>(p);
    if (p.R > 0) {
        const dim3 gd(static_cast<unsigned>((p.R + kRows - 1) / kRows), p.Hk, p.B);
        moda_bwd_dkdv_kernel<T, true><<<gd, block, 0, stream>>>(p);
    }
}

// Scratch for moda_bwd_noalloc: rowsum(dO * O) of up to MODA_NOALLOC_ROWS query rows,
// part of the library image, so that entry point allocates nothing.
static __device__ __align__(256) float g_noalloc_delta[MODA_NOALLOC_ROWS];

// Looked up on every call (cheap next to the launches): an address kept from an earlier
// call would dangle after the context that loaded the module is reset or recreated.
cudaError_t noalloc_scratch(void** ptr) {
    return cudaGetSymbolAddress(ptr, g_noalloc_delta);
}

template <typename T>
static void launch_delta_t(const BwdParams& p, cudaStream_t stream) {
    const dim3 gq((p.T + kRows - 1) / kRows, p.Hq, p.B);
    moda_bwd_delta_kernel<T><<<gq, dim3(kRows * 32), 0, stream>>>(p);
}

// bf16/f16 with d in {64, 128}, H_q/H_k dividing 128 and TMA-friendly layouts: the
// sequence part on tensor cores (moda_bwd_tc.cu) and the depth part per token;
// the rest with d <= 128 (d % 4 == 0), G <= 32 and 16-byte aligned rows (fp32, and 16-bit
// shapes the tensor-core kernels do not take) in CUDA-core tiles (moda_bwd_f32.cu);
// everything else on the CUDA-core row kernels above.
int launch_bwd(const BwdParams& p, cudaStream_t stream, char* err, size_t errlen) {
    char why[160];
    if (tc_bwd_supports(p, why, sizeof(why))) {
        if (p.dtype == MODA_BF16) launch_delta_t<__nv_bfloat16>(p, stream);
        else launch_delta_t<__half>(p, stream);
        int r = launch_bwd_tc(p, stream, err, errlen);
        if (r != MODA_OK) return r;
        return launch_bwd_depth(p, stream);
    }
    if (bwd_tiled_ok(p)) {  // CUDA-core tiles (moda_bwd_f32.cu)
        if (p.T > 0) {
            if (p.dtype == MODA_F32) launch_delta_t<float>(p, stream);
            else if (p.dtype == MODA_BF16) launch_delta_t<__nv_bfloat16>(p, stream);
            else launch_delta_t<__half>(p, stream);
        }
        return launch_bwd_tiled(p, stream);
    }
    switch (p.dtype) {
        case MODA_F32: launch_bwd_t<float>(p, stream); break;
        case MODA_BF16: launch_bwd_t<__nv_bfloat16>(p, stream); break;
        case MODA_F16: launch_bwd_t<__half>(p, stream); break;
        default: return MODA_ERR_DTYPE;
    }
    return MODA_OK;
}

}  // namespace moda
