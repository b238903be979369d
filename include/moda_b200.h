/*
 * moda_b200.h - C ABI of the B200 (sm_100a) fused MoDA attention library
 * (forward, backward, depth-cache append).
 *
 * Plain pointers and sizes only: no PyTorch types cross this boundary. The
 * caller owns every buffer; the library never allocates device memory on the
 * compute path. Kernels launch on the caller's stream; no call synchronizes
 * the host.
 *
 * Each entry point names the reference interface it replaces
 * (sahilmalik27/mixture-of-depth-attention, paths relative to that project).
 */
#ifndef MODA_B200_H_
#define MODA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A rank-4 strided view. sizes/strides are in elements, outermost first,
 * exactly torch.Tensor.size()/.stride() of a [B, H, rows, d] tensor. */
typedef struct ModaTensor {
    void* ptr;
    int64_t sizes[4];
    int64_t strides[4];
} ModaTensor;

typedef void* moda_stream_t; /* a cudaStream_t (torch.cuda.current_stream().cuda_stream) */

enum ModaDtype { MODA_F32 = 0, MODA_BF16 = 1, MODA_F16 = 2 };

enum ModaStatus {
    MODA_OK = 0,
    MODA_ERR_ARG = -1,        /* null pointer, bad num_layers / scale / layer index */
    MODA_ERR_SHAPE = -2,      /* inconsistent B, H, T or d between tensors */
    MODA_ERR_DEPTH_ROWS = -3, /* depth buffer holds fewer than T*num_layers rows */
    MODA_ERR_DTYPE = -4,      /* unknown dtype code */
    MODA_ERR_LAUNCH = -5,     /* CUDA reported an error at launch */
    MODA_ERR_UNSUPPORTED = -6 /* a forced kernel cannot run this shape/layout */
};

/* Kernel selection for moda_fwd_ex (moda_fwd uses MODA_KERNEL_AUTO). */
enum ModaKernel {
    MODA_KERNEL_AUTO = 0, /* tcgen05 path when the shape allows it, else SIMT */
    MODA_KERNEL_TC = 1,   /* TMA + tcgen05/TMEM fused kernel (bf16/f16, d in {64,128}) */
    MODA_KERNEL_SIMT = 2  /* CUDA-core kernel: any dtype, any strides, d <= 256 */
};

/*
 * Fused sequence + depth attention forward:
 *   O[b,h,t] = softmax over { scale*q.k_j : j <= t }  U  { scale*q.kd_{t*L+l} : l < L }
 *              applied to the matching V / V_depth rows, with KV head h / (H_q/H_k).
 * q [B,H_q,T,d]; k, v [B,H_k,T,d]; kd, vd [B,H_k,R,d] with R >= T*num_layers
 * (only rows [0, T*num_layers) are read); o [B,H_q,T,d] written in full.
 * scale <= 0 selects d^-0.5. chunk_size is accepted for signature parity and
 * does not change the result (the function is chunk-invariant); pass 0 for none.
 *
 * Replaces moda_attention_triton (moda/kernels/moda_triton.py:218-297) and
 * moda_attention_naive (moda/kernels/moda_naive.py:13-97), reached from
 * MoDAAttention.forward (moda/attention.py:85-93).
 */
int moda_fwd(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v, const ModaTensor* kd,
             const ModaTensor* vd, const ModaTensor* o, int num_layers, float scale,
             int chunk_size, int dtype, moda_stream_t stream);

/* moda_fwd with an explicit kernel choice (ModaKernel). Same reference counterpart. */
int moda_fwd_ex(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o, int num_layers,
                float scale, int chunk_size, int dtype, int kernel, moda_stream_t stream);

/* moda_fwd_ex that also writes the row log-sum-exp the backward pass needs:
 * lse[(b*H_q + h)*T + t] = log(sum over the row's keys of exp(scale*q.k)), natural log,
 * float32, contiguous [B, H_q, T]. Same result O as moda_fwd_ex.
 * Reference counterpart: the forward half of autograd through moda_attention_naive
 * (moda/kernels/moda_naive.py:13-97), which keeps the softmax for its backward. */
int moda_fwd_lse(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                 const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o, float* lse,
                 int num_layers, float scale, int chunk_size, int dtype, int kernel,
                 moda_stream_t stream);

/* Forward whose depth part is known to be all zeros: every row's softmax holds its
 * causal keys plus zero_rows keys of score 0 whose values are 0, and nothing is read
 * for them. Equals moda_fwd_lse with kd = vd = zeros [B,H_k,T*zero_rows,d] and
 * num_layers = zero_rows, up to rounding. lse as in moda_fwd_lse, or NULL.
 * The first layer of MoDAModel reads a freshly zero-filled cache (moda/model.py:
 * 143-151, moda/cache.py:40-47, moda/attention.py:85-93); its opt-in lean cache
 * lifecycle calls this instead of reading those zeros. No reference counterpart. */
int moda_fwd_zero_depth(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                        const ModaTensor* o, float* lse, int zero_rows, float scale, int dtype,
                        int kernel, moda_stream_t stream);

/* Bytes of device workspace moda_bwd needs (one float per query row), or -1 for
 * negative sizes. No reference counterpart. */
int64_t moda_bwd_workspace_size(int64_t batch, int64_t num_q_heads, int64_t seq_len);

/*
 * Backward of moda_fwd: given dout = dL/dO and the forward's o and lse, writes
 *   dq [B,H_q,T,d], dk, dv [B,H_k,T,d], dkd, dvd [B,H_k,R,d]
 * in full (each shaped like its input; depth rows at or beyond T*num_layers, which
 * the forward never reads, get zero). GQA gradients are summed over the G query
 * heads of each KV head. workspace: device memory of at least
 * moda_bwd_workspace_size(B, H_q, T) bytes, used for rowsum(dO*O); nothing is
 * allocated. Any strides; fp32 arithmetic.
 * Replaces torch autograd through moda_attention_naive (moda/kernels/moda_naive.py:
 * 13-162), which the reference trains with (tests/test_kernel.py:106-119,
 * tests/test_attention.py:57-71).
 */
int moda_bwd(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v, const ModaTensor* kd,
             const ModaTensor* vd, const ModaTensor* o, const ModaTensor* dout, const float* lse,
             const ModaTensor* dq, const ModaTensor* dk, const ModaTensor* dv,
             const ModaTensor* dkd, const ModaTensor* dvd, void* workspace,
             int64_t workspace_bytes, int num_layers, float scale, int dtype,
             moda_stream_t stream);

/* Largest B*H_q*T that moda_bwd_noalloc accepts. */
#define MODA_NOALLOC_ROWS (1 << 20)

/* moda_bwd without any workspace argument: the rowsum(dO*O) scratch is a fixed
 * array compiled into the library (MODA_NOALLOC_ROWS floats per device, its address
 * resolved once per device), so the call allocates nothing and needs no buffer from
 * the caller. B*H_q*T > MODA_NOALLOC_ROWS is rejected with MODA_ERR_UNSUPPORTED
 * before anything else (each of B, H_q and T is bounded before they are multiplied).
 * The array is shared by all calls on a device: such calls must not overlap in time
 * (issue them on one stream, or synchronize). The address is resolved on the first
 * call on each device and kept for the life of the process; cudaDeviceReset (or any
 * other teardown of the device's primary context) between calls is not supported,
 * since the kept address would then be stale.
 * No reference counterpart (the reference's autograd allocates through torch). */
int moda_bwd_noalloc(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                     const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o,
                     const ModaTensor* dout, const float* lse, const ModaTensor* dq,
                     const ModaTensor* dk, const ModaTensor* dv, const ModaTensor* dkd,
                     const ModaTensor* dvd, int num_layers, float scale, int dtype,
                     moda_stream_t stream);

/* Which kernel moda_fwd_ex would launch for these arguments (ModaKernel value,
 * or a negative ModaStatus). Host-only: validates and plans, launches nothing.
 * No reference counterpart (the reference picks its path in Python,
 * moda/attention.py:48,87). */
int moda_fwd_plan(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                  const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o, int num_layers,
                  int dtype, int kernel);

/*
 * Depth-cache append: k_cache[b,h,t*L + layer_idx,:] = k_src[b,h,t,:] for t < seq_len,
 * and the same for v, in one launch. k_src/v_src [B,H_k,>=seq_len,d];
 * caches [B,H_k,>=seq_len*L,d]; any strides.
 * Replaces DepthKVCache.write (moda/cache.py:52-74).
 */
int moda_depth_append(const ModaTensor* k_src, const ModaTensor* v_src, const ModaTensor* k_cache,
                      const ModaTensor* v_cache, int layer_idx, int num_layers, int seq_len,
                      int dtype, moda_stream_t stream);

/*
 * Depth-write projection with the depth-cache append in its epilogue:
 *   y = x . w^T, x [B,1,T,D], w [1,1,2*H_k*d,D] (the H_k*d k rows, then the v rows);
 *   k_cache[b,h,t*L + layer_idx,:] = y[b,t,h*d : (h+1)*d]
 *   v_cache[b,h,t*L + layer_idx,:] = y[b,t,(H_k+h)*d : (H_k+h+1)*d]   for t < seq_len.
 * H_k and d come from the caches [B,H_k,>=seq_len*L,d]; no other cache row is touched.
 * bf16/f16 with fp32 accumulation (tcgen05); needs d a multiple of 32, D a multiple of
 * 8, unit stride along the last dimension and 16-byte aligned strides, else
 * MODA_ERR_UNSUPPORTED before any launch.
 * Replaces k_depth_proj / v_depth_proj (moda/attention.py:81-82) or ffn_k_depth_proj /
 * ffn_v_depth_proj (moda/model.py:78-81, 92-95) followed by DepthKVCache.write
 * (moda/cache.py:52-74).
 */
int moda_depth_proj_append(const ModaTensor* x, const ModaTensor* w, const ModaTensor* k_cache,
                           const ModaTensor* v_cache, int layer_idx, int num_layers, int seq_len,
                           int dtype, moda_stream_t stream);

/*
 * The attention's three input projections as one GEMM whose epilogue writes Q, K and V
 * head-major: y = x . w^T with x [B,1,T,D] and w [1,1,(H_q+2*H_k)*d,D] (the H_q*d rows
 * of W_q, then W_k, then W_v);
 *   q[b,h,t,:] = y[b,t,h*d : (h+1)*d]                     (q [B,H_q,T,d])
 *   k[b,h,t,:] = y[b,t,(H_q+h)*d : ...], v likewise after k (k, v [B,H_k,T,d]).
 * Any output strides with unit stride along d (16-byte aligned). bf16/f16 with fp32
 * accumulation (tcgen05); needs d a multiple of 32 and D a multiple of 8, else
 * MODA_ERR_UNSUPPORTED before any launch.
 * Replaces q_proj / k_proj / v_proj and their view(B,T,H,d).transpose(1,2)
 * (moda/attention.py:77-79).
 */
int moda_qkv_proj(const ModaTensor* x, const ModaTensor* w, const ModaTensor* q,
                  const ModaTensor* k, const ModaTensor* v, int dtype, moda_stream_t stream);

/* Text of the last error on the calling thread ("" if none). Thread-local. */
const char* moda_last_error(void);

/* Reads and clears the device status word kernels set when a bounded wait
 * times out (0 = none). Synchronizes `stream`. No reference counterpart. */
int moda_device_status(moda_stream_t stream);

/* Library version (major*10000 + minor*100 + patch). */
int moda_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MODA_B200_H_ */
