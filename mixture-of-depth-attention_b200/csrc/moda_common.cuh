// Shared device helpers for the MoDA forward kernels (sm_100a).
//
// Everything here is a thin, hand-written wrapper over one PTX instruction:
// mbarriers, TMA (cp.async.bulk.tensor), tcgen05 (TMEM alloc, MMA, commit,
// ld/st, fences). Every spin-wait is bounded: a wait that runs out of time
// records an error code in `moda_dev_status` and returns false, so a kernel
// whose producer died returns instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

namespace moda {

// Error word written by kernels (0 = fine): 0x100 | site for a wait that timed
// out. One copy per translation unit; the tcgen05 unit's copy is read and
// cleared by the host through moda_device_status().
static __device__ int moda_dev_status = 0;

#define MODA_DEV __device__ __forceinline__

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ------------------------------------------------------------------ basics
MODA_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

MODA_DEV float ex2(float x) {  // hardware base-2 exponential (MUFU.EX2)
    float y;
    asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

MODA_DEV uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

MODA_DEV uint32_t pack_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Packed fp32 pair arithmetic (sm_100 FFMA2 / FADD2 / FMUL2): one instruction, two lanes of math.
MODA_DEV uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
MODA_DEV void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
MODA_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
MODA_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
MODA_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
MODA_DEV float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// ------------------------------------------------------------------ mbarrier
MODA_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

MODA_DEV void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

MODA_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

MODA_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

MODA_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Non-blocking probe of a phase (no suspension): true if it has completed.
MODA_DEV bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait. `abort_flag` lives in shared memory and is shared by all warps
// of the CTA: once any wait times out, every later wait returns false at once,
// so all roles drain to the common exit (TMEM free) instead of spinning.
constexpr long long kWaitLimitCycles = 4000000000LL;  // about 2 s at 1.9 GHz

#ifndef MODA_WAIT_SLEEP_NS
#define MODA_WAIT_SLEEP_NS 20
#endif
// Back-off of a waiting warp between polls (nanoseconds): a sleeping warp takes no
// issue slots from the working warps of its scheduler partition (measured 2-5 % faster
// forward at the kernel-only shape than polling without a pause).
MODA_DEV void wait_backoff() {
    if (MODA_WAIT_SLEEP_NS > 0) __nanosleep(MODA_WAIT_SLEEP_NS);
}

MODA_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        wait_backoff();
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                *abort_flag = 1;
                atomicCAS(&moda_dev_status, 0, 0x100 | site);
                return false;
            }
        }
    }
}

// The same bounded wait without the back-off, for the waits on a softmax step's critical
// path (scores ready, P ready): there the wake-up latency matters more than issue slots.
MODA_DEV bool mbar_wait_hot(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                *abort_flag = 1;
                atomicCAS(&moda_dev_status, 0, 0x100 | site);
                return false;
            }
        }
    }
}

// Bounded wait that ignores the abort flag: used only on the exit path to let
// copies and MMAs already in flight land before shared memory / TMEM are released.
MODA_DEV bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitLimitCycles / 4) return false;
    }
    return true;
}

// Warpgroup register reallocation (all 4 warps of a warpgroup execute it).
template <uint32_t N>
MODA_DEV void reg_dealloc() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <uint32_t N>
MODA_DEV void reg_alloc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }

// ------------------------------------------------------------------ TMA
MODA_DEV void tma_prefetch_desc(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

MODA_DEV void tma_load_4d(const CUtensorMap* m, uint32_t dst, uint32_t bar, int c0, int c1, int c2,
                          int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

MODA_DEV void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------ tcgen05
MODA_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
MODA_DEV void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MODA_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

MODA_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MODA_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T   (kind::f16, fp32 accumulate)
MODA_DEV void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]
MODA_DEV void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread has completed.
MODA_DEV void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

MODA_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Emits nothing. The registers of a tcgen05.ld are valid only after tcgen05.wait::ld;
// passing them through this volatile asm (ordered after the wait) makes every later
// use depend on a definition that follows the wait, so no computation on them can be
// scheduled before it.
MODA_DEV void tmem_reg_fence(uint32_t (&r)[32]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31]));
}
MODA_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns; thread i <-> lane (base lane + i).
MODA_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
        "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// tcgen05.ld of 32 columns followed by the wait and the register fence.
MODA_DEV void tmem_ld32_sync(uint32_t taddr, uint32_t (&r)[32]) {
    tmem_ld32(taddr, r);
    tmem_wait_ld();
    tmem_reg_fence(r);
}

MODA_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

MODA_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

// ------------------------------------------------------------------ cp.async, vectors
// 16-byte cp.async; src_bytes 0 writes zeros and reads nothing
MODA_DEV void f32_cp16(float* dst, const float* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
MODA_DEV void f32_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MODA_DEV void f32_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// W consecutive floats (W = 2 or 4) through one 8- or 16-byte access
template <int W>
MODA_DEV void f32_ldv(float* dst, const float* src) {
    if constexpr (W == 4) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        dst[0] = v.x, dst[1] = v.y, dst[2] = v.z, dst[3] = v.w;
    } else {
        const float2 v = *reinterpret_cast<const float2*>(src);
        dst[0] = v.x, dst[1] = v.y;
    }
}
template <int W>
MODA_DEV void f32_stv(float* dst, const float* src, float s) {
    if constexpr (W == 4)
        *reinterpret_cast<float4*>(dst) = make_float4(src[0] * s, src[1] * s, src[2] * s, src[3] * s);
    else
        *reinterpret_cast<float2*>(dst) = make_float2(src[0] * s, src[1] * s);
}

// ------------------------------------------------------------------ fp32 / 16-bit values
template <typename T>
constexpr bool kIsF32 = std::is_same<T, float>::value;

template <typename T>
MODA_DEV float2 unpack2(uint32_t w);  // two 16-bit values, low half first
template <>
MODA_DEV float2 unpack2<__nv_bfloat16>(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
MODA_DEV float2 unpack2<__half>(uint32_t w) {
    return make_float2(__half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu))),
                       __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16))));
}
template <typename T>
MODA_DEV uint32_t pack2(float lo, float hi);
template <>
MODA_DEV uint32_t pack2<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <>
MODA_DEV uint32_t pack2<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }

// 4 consecutive elements as floats / from floats times s (16-bit: one 8-byte access)
template <typename T>
MODA_DEV float4 b32_ld4(const T* src) {
    if constexpr (kIsF32<T>) {
        return *reinterpret_cast<const float4*>(src);
    } else {
        const uint2 w = *reinterpret_cast<const uint2*>(src);
        const float2 a = unpack2<T>(w.x), c = unpack2<T>(w.y);
        return make_float4(a.x, a.y, c.x, c.y);
    }
}
template <typename T>
MODA_DEV void b32_st4(T* dst, float4 v, float s) {
    if constexpr (kIsF32<T>)
        *reinterpret_cast<float4*>(dst) = make_float4(v.x * s, v.y * s, v.z * s, v.w * s);
    else
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack2<T>(v.x * s, v.y * s), pack2<T>(v.z * s, v.w * s));
}

// ROWS rows of a [.., rows, d] 16-bit view, from row0, into a raw [ROWS][HD] tile by
// cp.async, NT threads (16 bytes = 8 elements per copy; zeros for rows at or past
// `limit` and for columns at or past d, which must be a multiple of 4)
template <typename T, int HD, int ROWS, int NT>
MODA_DEV void raw16_stage(T* dst, const T* base, int64_t rstride, int row0, int limit, int d, int tid) {
    for (int i = tid; i < ROWS * (HD / 8); i += NT) {
        const int r = i / (HD / 8), col = 8 * (i % (HD / 8));
        const int n = row0 + r < limit && col < d ? min(8, d - col) : 0;  // elements to copy
        const T* src = n ? base + static_cast<int64_t>(row0 + r) * rstride + col : base;
        f32_cp16(reinterpret_cast<float*>(dst + r * HD + col), reinterpret_cast<const float*>(src), 2 * n);
    }
}

// raw [ROWS][HD] 16-bit tile -> fp32 [ROWS][HD+4] tile, NT threads
template <typename T, int HD, int ROWS, int NT>
MODA_DEV void raw16_convert(float* dst, const T* raw, int tid) {
    for (int i = tid; i < ROWS * (HD / 8); i += NT) {
        const int r = i / (HD / 8), col = 8 * (i % (HD / 8));
        const uint4 w = *reinterpret_cast<const uint4*>(raw + r * HD + col);
        const float2 a = unpack2<T>(w.x), b = unpack2<T>(w.y), c = unpack2<T>(w.z), e = unpack2<T>(w.w);
        *reinterpret_cast<float4*>(dst + r * (HD + 4) + col) = make_float4(a.x, a.y, b.x, b.y);
        *reinterpret_cast<float4*>(dst + r * (HD + 4) + col + 4) = make_float4(c.x, c.y, e.x, e.y);
    }
}

// W consecutive elements (W = 2 or 4) as floats / from floats times s, one access
template <typename T, int W>
MODA_DEV void ldv_as_f32(float* dst, const T* src) {
    if constexpr (kIsF32<T>) {
        f32_ldv<W>(dst, src);
    } else if constexpr (W == 4) {
        const float4 v = b32_ld4<T>(src);
        dst[0] = v.x, dst[1] = v.y, dst[2] = v.z, dst[3] = v.w;
    } else {
        const float2 v = unpack2<T>(*reinterpret_cast<const uint32_t*>(src));
        dst[0] = v.x, dst[1] = v.y;
    }
}
template <typename T, int W>
MODA_DEV void stv_from_f32(T* dst, const float* src, float s) {
    if constexpr (kIsF32<T>)
        f32_stv<W>(dst, src, s);
    else if constexpr (W == 4)
        b32_st4<T>(dst, make_float4(src[0], src[1], src[2], src[3]), s);
    else
        *reinterpret_cast<uint32_t*>(dst) = pack2<T>(src[0] * s, src[1] * s);
}

// ------------------------------------------------------------------ UMMA descriptors
// Shared-memory matrix descriptor (sm_100 format, version 1), 128-byte swizzle:
//   bits  0-13 start address >> 4     bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4 bits 46-47 version (1)
//   bits 61-63 layout (2 = 128B swizzle)
// Built as two 32-bit words, so the issue loop advances the
// start address with one 32-bit add: lo = (addr >> 4) | (lbo >> 4) << 16,
// hi = (sbo >> 4) | version << 14 | layout << 29. Valid while addr < 256 KB.
__host__ __device__ constexpr uint32_t desc_hi_sw128(uint32_t sbo_bytes) {
    return ((sbo_bytes >> 4) & 0x3FFFu) | (1u << 14) | (2u << 29);
}
MODA_DEV uint32_t desc_lo(uint32_t addr, uint32_t lbo_bytes) {
    return ((addr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}
MODA_DEV uint64_t desc_join(uint32_t lo, uint32_t hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (0 = f16, 1 = bf16),
//   bit 15 A major (0 = K), bit 16 B major (1 = MN), bits 17-22 N >> 3, bits 24-28 M >> 4.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_fmt, uint32_t M, uint32_t N,
                                                  uint32_t b_mn_major) {
    return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (b_mn_major << 16) | ((N >> 3) << 17) |
           ((M >> 4) << 24);
}

}  // namespace moda
