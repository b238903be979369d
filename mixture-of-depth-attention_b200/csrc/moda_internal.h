// Internal declarations shared by the MoDA CUDA sources (not part of the C ABI).
#pragma once

#include "../../include/moda_b200.h"
#include "moda_common.cuh"

#include <atomic>
#include <cstdint>

namespace moda {

// Validated forward problem. Strides are in elements.
struct FwdParams {
    ModaTensor q, k, v, kd, vd, o;
    float* lse;  // optional [B, H_q, T] fp32, contiguous: natural log-sum-exp per row
    int B, Hq, Hk, G, T, d, L;
    int zero_rows;  // implicit depth rows per token with k = v = 0 (never read from memory)
    float scale;
    int dtype;
};

// Validated backward problem (tensors as in FwdParams, gradients shaped like
// their inputs). delta is the caller's workspace, [B, H_q, T] fp32.
struct BwdParams {
    ModaTensor q, k, v, kd, vd, o, dout, dq, dk, dv, dkd, dvd;
    const float* lse;
    float* delta;
    int B, Hq, Hk, G, T, d, L;
    long long R;  // depth rows of kd / dkd (>= T*L)
    float scale;
    int dtype;
};

struct AppendParams {
    ModaTensor k_src, v_src, k_cache, v_cache;
    int B, H, T, d, L, layer;
    int dtype;
};

// Parameters of the tcgen05 kernel. Tensor maps first (64-byte aligned).
struct TcParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_kd, tm_vd;
    void* o;                      // output [B, H_q, T, d], unit stride along d
    long long o_sb, o_sh, o_st;   // output strides in elements
    int B, Hq, Hk, G, T, L;
    int n_tok;      // tokens per 128-row query tile (128 / G)
    int num_pairs;  // tile pairs per (b, kv head)
    int num_items;  // num_pairs * B * Hk work items
    float sc;       // scale * log2(e)
    float* lse;     // optional fp32 log-sum-exp output: row (b, head, t) at
    long long lse_sb, lse_sh;  // lse[b * lse_sb + head * lse_sh + t]
    int zero_rows;  // implicit all-zero depth rows per token (score 0, value 0)
};

// Projection GEMM y = x . W^T whose epilogue stores column segments of y into up to
// three head-major outputs: x [B, 1, T, D], w [1, 1, N, D]; segment s covers columns
// [seg_start, seg_start + heads[s]*d) and stores row t, head h into
// out[s][b, h, t*L + slot, :] for t < n_write. moda_depth_proj_append: two outputs (the
// k and v caches, L = cache layers, slot = layer); moda_qkv_proj: three outputs (Q, K,
// V in [B, H, T, d], L = 1, slot = 0).
struct ProjProblem {
    ModaTensor x, w, out[3];
    int nout;
    int heads[3];
    int B, T, D, N, d, L, slot, n_write;
    int dtype;
};

struct ProjParams {
    CUtensorMap tm_x, tm_w;  // first: 64-byte aligned
    void* out0;
    void* out1;
    void* out2;
    long long o_sb[3], o_sh[3], o_sr[3];  // output strides (elements)
    int seg_end[3];                       // exclusive column end of each output's segment
    int B, T, K, N, d, Lc, slot, n_write;
    int m_tiles_per_batch, n_tiles, num_tiles;
};

bool proj_supports(const ProjProblem& q, char* why, size_t whylen);
int launch_proj_append(const ProjProblem& q, cudaStream_t stream, char* err, size_t errlen);
cudaError_t read_and_clear_proj_status(cudaStream_t stream, int* value);

// TMA map over a [B, H, rows, d] view (128-byte swizzle, box (64, box1, box2, 1)),
// dimension order (d, H, rows, B) when head_inner (query-like tensors: box (64, G, n)
// is a token-major tile of G heads x n tokens), else (d, rows, H, B).
bool encode_map(CUtensorMap* m, const ModaTensor& t, int rows, bool head_inner, int esz,
                CUtensorMapDataType dt, uint32_t box1, uint32_t box2, char* err, size_t errlen,
                const char* name);
int sm_count();

int launch_fwd_simt(const FwdParams& p, cudaStream_t stream);
int launch_fwd_tc(const FwdParams& p, cudaStream_t stream, char* err, size_t errlen);
bool tc_supports(const FwdParams& p, char* why, size_t whylen);
int launch_depth_append(const AppendParams& p, bool vec16, cudaStream_t stream);
// Parameters of the tcgen05 backward kernels. Tensor maps first (64-byte aligned).
struct TcBwdParams {
    CUtensorMap tm_q, tm_do, tm_k, tm_v;
    const float* lse;
    const float* delta;
    void* dq;
    long long dq_sb, dq_sh, dq_st;
    void* dk;
    long long dk_sb, dk_sh, dk_st;
    void* dv;
    long long dv_sb, dv_sh, dv_st;
    int B, Hq, Hk, G, T;
    int n_tok;       // tokens per 128-row query tile (128 / G)
    int num_qtiles;  // query tiles per (b, kv head)
    int num_ktiles;  // 128-key tiles per (b, kv head)
    int num_items;
    float sc;        // scale * log2(e)
    float scale;
};

int launch_bwd(const BwdParams& p, cudaStream_t stream, char* err, size_t errlen);
bool tc_bwd_supports(const BwdParams& p, char* why, size_t whylen);
int launch_bwd_tc(const BwdParams& p, cudaStream_t stream, char* err, size_t errlen);
int launch_bwd_depth(const BwdParams& p, cudaStream_t stream);
bool bwd_tiled_ok(const BwdParams& p);
int launch_bwd_tiled(const BwdParams& p, cudaStream_t stream);
cudaError_t read_and_clear_bwd_status(cudaStream_t stream, int* value);
constexpr int kMaxDevices = 64;
// Device address of the library's fixed backward scratch on the current device.
cudaError_t noalloc_scratch(void** ptr);
cudaError_t read_and_clear_status(cudaStream_t stream, int* value);

// One-time opt-in of a kernel's dynamic shared memory on the current device (function
// attributes are per device). `done` is the kernel's own bitmask of devices already set
// up; devices past 63 are set up on every call.
template <typename Kernel>
cudaError_t ensure_smem_attr(std::atomic<uint64_t>& done, Kernel kern, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_release);
    return e;
}

}  // namespace moda
