// CUDA-core MoDA forward: any dtype (f32 / bf16 / f16), any strides, d <= 256.
//
// This is the exact-arithmetic path (fp32 FMA throughout) used for fp32 inputs,
// whose tolerance (1e-4 relative) tensor-core bf16/tf32 products cannot meet,
// and for shapes the tcgen05 kernel does not tile (d not in {64,128}, G not
// dividing 128, unaligned strides).
//
// One warp owns one query row (b, h, t). Lanes split the head dimension; every
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

int launch_fwd_simt(const FwdParams& p, cudaStream_t stream) {
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
