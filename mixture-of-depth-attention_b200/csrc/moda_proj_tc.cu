// Projection GEMM with the head-major scatter in its epilogue (tcgen05 / TMA / TMEM).
//
//   y[b, t, :] = x[b, t, :] . W^T          W [N, D], N = (sum of the outputs' heads) * d
//   out_s[b, h, t*L + slot, :] = y[b, t, c_s + h*d : c_s + (h+1)*d]     for t < n_write
//
// with c_s the first column of output s. Two uses:
// * the depth writes (moda_depth_proj_append): W = [W_k; W_v], outputs the k and v
//   caches, L = the cache's layers, slot = the writing layer. The reference computes
//   the two depth projections with nn.Linear (moda/attention.py:81-82 for the
//   attention's writes, moda/model.py:78-81 for the FFN's) and copies them into the
//   cache with a strided slice assignment (moda/cache.py:73-74);
// * the attention's input projections (moda_qkv_proj): W = [W_q; W_k; W_v], outputs Q,
//   K, V in [B, H, T, d] (L = 1, slot = 0), the layout the attention kernel reads; the
//   reference runs three nn.Linear and views them as transposes (moda/attention.py:77-79).
// In both, one GEMM stores its tiles straight into the destination rows, so y never
// exists in memory.
//
// Tiling: a CTA tile is 256 rows (tokens of one batch) x 256 columns, K in steps of 64.
// Both 128-row halves of the A tile share the B tile (two M = 128, N = 256 MMAs per
// 16-wide k step into two TMEM accumulators of 256 columns), which halves the B bytes
// per FLOP against a 128-row tile -- the operand feed from L2 is what bounds a
// single-CTA tile. Persistent CTAs (one per SM) walk the tiles with a fixed stride;
// consecutive tiles share their A rows, so x is read from HBM about once.
//
// Warps (320 threads): 0 TMA producer, 1 TMEM allocator + MMA issuer, 2-9 epilogue
// (warp w reads TMEM lane quarter w % 4 of accumulator (w - 2) / 4). The accumulators
// are single-buffered: the issuer starts a tile's MMAs once the epilogue has loaded
// the previous tile out of TMEM (the stores to the cache then overlap the next MMAs).
#include "moda_internal.h"

#include <cstdio>

namespace moda {

namespace {

constexpr int kPThreads = 320;
constexpr int kPBM = 256, kPBN = 256, kPBK = 64, kPStages = 3;
constexpr int kPABytes = kPBM * kPBK * 2;
constexpr int kPBBytes = kPBN * kPBK * 2;
constexpr int kPStageBytes = kPABytes + kPBBytes;
constexpr int kPBarOff = kPStages * kPStageBytes;
constexpr int kPNumBars = 2 * kPStages + 3;  // full[S] empty[S] acc_full acc_empty end
constexpr int kPMiscOff = kPBarOff + kPNumBars * 8;
constexpr int kPSmemBytes = kPMiscOff + 32 + 1024;  // + alignment slack

struct PTile {
    int b, t0, n0;
};

__device__ __forceinline__ PTile ptile(const ProjParams& p, int tile) {
    PTile r;
    const int m = tile / p.n_tiles;
    r.n0 = (tile % p.n_tiles) * kPBN;
    r.b = m / p.m_tiles_per_batch;
    r.t0 = (m % p.m_tiles_per_batch) * kPBM;
    return r;
}

template <int FMT>
__global__ void __launch_bounds__(kPThreads, 1)
    moda_proj_append_kernel(const __grid_constant__ ProjParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + kPBarOff;
    auto full = [&](uint32_t s) { return bar0 + 8u * s; };
    auto empty = [&](uint32_t s) { return bar0 + 8u * (kPStages + s); };
    const uint32_t acc_full = bar0 + 8u * (2 * kPStages);
    const uint32_t acc_empty = bar0 + 8u * (2 * kPStages + 1);
    const uint32_t end_bar = bar0 + 8u * (2 * kPStages + 2);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kPMiscOff);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kPMiscOff + 8);
    auto sA = [&](uint32_t s) { return sbase + s * kPStageBytes; };
    auto sB = [&](uint32_t s) { return sbase + s * kPStageBytes + kPABytes; };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nk = (p.K + kPBK - 1) / kPBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 8);  // one arrival per epilogue warp
        mbar_init(end_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&p.tm_x);
        tma_prefetch_desc(&p.tm_w);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------------- TMA producer
            uint32_t fill = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                const PTile tl = ptile(p, tile);
                for (int kb = 0; kb < nk; ++kb, ++fill) {
                    const uint32_t s = fill % kPStages;
                    if (fill >= kPStages &&
                        !mbar_wait(empty(s), ((fill / kPStages) + 1) & 1u, abort_flag, 1)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full(s), kPStageBytes);
                    tma_load_4d(&p.tm_x, sA(s), full(s), kb * kPBK, tl.t0, 0, tl.b);
                    tma_load_4d(&p.tm_w, sB(s), full(s), kb * kPBK, tl.n0, 0, 0);
                }
            }
            // let every load in flight land before the CTA's shared memory goes away
            const uint32_t first = fill > kPStages ? fill - kPStages : 0;
            for (uint32_t f = first; f < fill; ++f)
                mbar_wait_drain(full(f % kPStages), (f / kPStages) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------------------- MMA issuer
            constexpr uint32_t idesc = make_idesc(FMT, 128, kPBN, 0);
            constexpr uint32_t hi = desc_hi_sw128(1024);
            uint32_t fill = 0, tcount = 0;
            bool ok = true, issued = false;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++tcount) {
                if (tcount > 0 && !mbar_wait(acc_empty, (tcount + 1) & 1u, abort_flag, 2)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < nk; ++kb, ++fill) {
                    const uint32_t s = fill % kPStages;
                    if (!mbar_wait(full(s), (fill / kPStages) & 1u, abort_flag, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_lo = desc_lo(sA(s), 16);
                    const uint32_t b_lo = desc_lo(sB(s), 16);
#pragma unroll
                    for (int kk = 0; kk < kPBK / 16; ++kk) {
                        const uint32_t off = (kk * 32) >> 4;
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        mma_ss(tmem, desc_join(a_lo + off, hi), desc_join(b_lo + off, hi), idesc, acc);
                        mma_ss(tmem + kPBN, desc_join(a_lo + (16384 >> 4) + off, hi),
                               desc_join(b_lo + off, hi), idesc, acc);
                    }
                    issued = true;
                    mma_commit(empty(s));
                }
                if (!ok) break;
                mma_commit(acc_full);
            }
            if (issued) {  // every MMA issued has completed before TMEM is released
                mma_commit(end_bar);
                mbar_wait_drain(end_bar, 0);
            }
        }
    } else {
        // -------------------------------------------------------------------- epilogue
        const int q = warp & 3;               // TMEM lane quarter
        const int half = (warp - 2) >> 2;     // accumulator: rows [128*half, +128) of the tile
        const uint32_t t_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + half * kPBN;
        uint32_t tcount = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++tcount) {
            const PTile tl = ptile(p, tile);
            if (!mbar_wait(acc_full, tcount & 1u, abort_flag, 4)) break;
            tc_fence_after();
            const int t = tl.t0 + half * 128 + q * 32 + lane;
            const bool row_ok = t < p.n_write;
            const long long crow = static_cast<long long>(t) * p.Lc + p.slot;
#pragma unroll 1
            for (int c = 0; c < kPBN / 32; ++c) {
                uint32_t v[32];
                tmem_ld32(t_base + c * 32, v);
                tmem_wait_ld();
                if (c == kPBN / 32 - 1) {  // the accumulators are free for the next tile
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acc_empty);
                }
                const int n = tl.n0 + c * 32;
                if (!row_ok || n >= p.N) continue;
                // the output segment holding column n (32-column chunks never straddle a head)
                const int sg = n < p.seg_end[0] ? 0 : (n < p.seg_end[1] ? 1 : 2);
                const int nn = n - (sg == 0 ? 0 : p.seg_end[sg - 1]);
                const int h = nn / p.d, col = nn % p.d;
                uint16_t* base = static_cast<uint16_t*>(sg == 0 ? p.out0 : (sg == 1 ? p.out1 : p.out2));
                const long long off = p.o_sb[sg] * tl.b + p.o_sh[sg] * h + p.o_sr[sg] * crow + col;
                uint4* dst = reinterpret_cast<uint4*>(base + off);
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float a = __uint_as_float(v[2 * i]);
                    const float b = __uint_as_float(v[2 * i + 1]);
                    pk[i] = FMT == 1 ? pack_bf16x2(a, b) : pack_f16x2(a, b);
                }
#pragma unroll
                for (int ch = 0; ch < 4; ++ch)
                    dst[ch] = make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// One shared-memory opt-in per instantiation and device (each instantiation has its own mask).
template <int FMT>
int launch_proj_inst(const ProjParams& p, int grid, cudaStream_t stream) {
    static std::atomic<uint64_t> attr_done{0};
    if (ensure_smem_attr(attr_done, moda_proj_append_kernel<FMT>, kPSmemBytes) != cudaSuccess)
        return MODA_ERR_LAUNCH;
    moda_proj_append_kernel<FMT><<<grid, kPThreads, kPSmemBytes, stream>>>(p);
    return MODA_OK;
}

}  // namespace

cudaError_t read_and_clear_proj_status(cudaStream_t stream, int* value) {
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

bool proj_supports(const ProjProblem& q, char* why, size_t whylen) {
    auto no = [&](const char* s) {
        snprintf(why, whylen, "%s", s);
        return false;
    };
    if (q.dtype != MODA_BF16 && q.dtype != MODA_F16) return no("needs bf16 or f16");
    if (q.d % 32 != 0) return no("needs head_dim a multiple of 32");
    const ModaTensor* ts[5] = {&q.x, &q.w, &q.out[0], &q.out[1], &q.out[2]};
    for (int i = 0; i < 2 + q.nout; ++i) {
        const ModaTensor* t = ts[i];
        if (t->strides[3] != 1) return no("needs unit stride along the feature dimension");
        if (reinterpret_cast<uintptr_t>(t->ptr) % 16 != 0) return no("needs 16-byte aligned tensors");
        for (int j = 0; j < 3; ++j)
            if (t->sizes[j] > 1 && (t->strides[j] * 2) % 16 != 0)
                return no("needs 16-byte multiple strides");
    }
    if (q.D % 8 != 0) return no("needs D a multiple of 8");
    return true;
}

int launch_proj_append(const ProjProblem& q, cudaStream_t stream, char* err, size_t errlen) {
    ProjParams p;
    const CUtensorMapDataType dt =
        q.dtype == MODA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (!encode_map(&p.tm_x, q.x, q.T, false, 2, dt, kPBM, 1, err, errlen, "x") ||
        !encode_map(&p.tm_w, q.w, q.N, false, 2, dt, kPBN, 1, err, errlen, "W"))
        return MODA_ERR_LAUNCH;
    void* outs[3] = {nullptr, nullptr, nullptr};
    int end = 0;
    for (int i = 0; i < 3; ++i) {
        if (i < q.nout) {
            outs[i] = q.out[i].ptr;
            p.o_sb[i] = q.out[i].strides[0];
            p.o_sh[i] = q.out[i].strides[1];
            p.o_sr[i] = q.out[i].strides[2];
            end += q.heads[i] * q.d;
        } else {
            p.o_sb[i] = p.o_sh[i] = p.o_sr[i] = 0;
        }
        p.seg_end[i] = end;  // a missing segment is empty (end repeats)
    }
    p.out0 = outs[0];
    p.out1 = outs[1];
    p.out2 = outs[2];
    p.B = q.B;
    p.T = q.T;
    p.K = q.D;
    p.N = q.N;
    p.d = q.d;
    p.Lc = q.L;
    p.slot = q.slot;
    p.n_write = q.n_write;
    // tiles past the last written token are skipped
    p.m_tiles_per_batch = (q.n_write + kPBM - 1) / kPBM;
    p.n_tiles = (q.N + kPBN - 1) / kPBN;
    const long long tiles = static_cast<long long>(p.m_tiles_per_batch) * q.B * p.n_tiles;
    if (tiles == 0) return MODA_OK;
    if (tiles > 0x7fffffffLL) {
        snprintf(err, errlen, "too many tiles");
        return MODA_ERR_UNSUPPORTED;
    }
    p.num_tiles = static_cast<int>(tiles);
    const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
    return q.dtype == MODA_BF16 ? launch_proj_inst<1>(p, grid, stream)
                                : launch_proj_inst<0>(p, grid, stream);
}

}  // namespace moda
