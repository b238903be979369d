// C ABI of the MoDA B200 library: argument validation, kernel planning, launch.
//
// All checks run on the host before any launch; a rejected call returns a
// negative ModaStatus and leaves its text in a thread-local buffer
// (moda_last_error). Nothing here allocates device memory.
#include "moda_internal.h"

#include <cstdarg>
#include <cstdio>
#include <cstring>

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

bool dtype_ok(int dtype) { return dtype == MODA_F32 || dtype == MODA_BF16 || dtype == MODA_F16; }

// Validation mirrors what moda_attention_naive (moda/kernels/moda_naive.py:44-59)
// needs to produce a result, plus the explicit depth-row check that the
// reference leaves to a late shape error (moda_naive.py:137-149).
int validate_fwd(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                 const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o, int num_layers,
                 float scale, int dtype, moda::FwdParams* out) {
    if (!q || !k || !v || !kd || !vd || !o) return fail(MODA_ERR_ARG, "null tensor descriptor");
    if (!dtype_ok(dtype)) return fail(MODA_ERR_DTYPE, "unknown dtype code %d", dtype);
    const ModaTensor* all[6] = {q, k, v, kd, vd, o};
    const char* names[6] = {"Q", "K", "V", "K_depth", "V_depth", "O"};
    for (int i = 0; i < 6; ++i) {
        for (int j = 0; j < 4; ++j)
            if (all[i]->sizes[j] < 0) return fail(MODA_ERR_SHAPE, "%s has a negative size", names[i]);
    }
    const int64_t B = q->sizes[0], Hq = q->sizes[1], T = q->sizes[2], d = q->sizes[3];
    const int64_t Hk = k->sizes[1];
    if (num_layers < 0) return fail(MODA_ERR_ARG, "num_layers must be >= 0, got %d", num_layers);
    if (Hk <= 0 || Hq % Hk != 0)
        return fail(MODA_ERR_SHAPE, "H_q (%lld) must be a multiple of H_k (%lld)", (long long)Hq,
                    (long long)Hk);
    if (d <= 0 || d > 256) return fail(MODA_ERR_SHAPE, "head_dim must be in [1, 256], got %lld", (long long)d);
    auto same = [&](const ModaTensor* t, const char* n, int64_t b, int64_t h, int64_t rows_min,
                    bool exact_rows) -> int {
        if (t->sizes[0] != b || t->sizes[1] != h || t->sizes[3] != d)
            return fail(MODA_ERR_SHAPE, "%s has shape [%lld,%lld,%lld,%lld], expected [%lld,%lld,*,%lld]",
                        n, (long long)t->sizes[0], (long long)t->sizes[1], (long long)t->sizes[2],
                        (long long)t->sizes[3], (long long)b, (long long)h, (long long)d);
        if (exact_rows ? t->sizes[2] != rows_min : t->sizes[2] < rows_min)
            return fail(MODA_ERR_SHAPE, "%s has %lld rows, expected %s%lld", n,
                        (long long)t->sizes[2], exact_rows ? "" : ">= ", (long long)rows_min);
        return MODA_OK;
    };
    int r;
    if ((r = same(k, "K", B, Hk, T, true)) || (r = same(v, "V", B, Hk, T, true)) ||
        (r = same(o, "O", B, Hq, T, true)))
        return r;
    const int64_t need = T * static_cast<int64_t>(num_layers);
    for (int i = 3; i < 5; ++i) {
        const ModaTensor* t = all[i];
        if (t->sizes[0] != B || t->sizes[1] != Hk || t->sizes[3] != d)
            return fail(MODA_ERR_SHAPE, "%s has shape [%lld,%lld,%lld,%lld], expected [%lld,%lld,>=T*L,%lld]",
                        names[i], (long long)t->sizes[0], (long long)t->sizes[1],
                        (long long)t->sizes[2], (long long)t->sizes[3], (long long)B,
                        (long long)Hk, (long long)d);
        if (t->sizes[2] < need)
            return fail(MODA_ERR_DEPTH_ROWS,
                        "%s holds %lld rows but T*num_layers = %lld*%d = %lld rows are addressed",
                        names[i], (long long)t->sizes[2], (long long)T, num_layers, (long long)need);
    }
    const int64_t numel = B * Hq * T * d;
    for (int i = 0; i < 6; ++i) {
        int64_t n = 1;
        for (int j = 0; j < 4; ++j) n *= all[i]->sizes[j];
        if (n > 0 && !all[i]->ptr) return fail(MODA_ERR_ARG, "%s has a null data pointer", names[i]);
    }
    if (B > 65535 || Hq > 65535)
        return fail(MODA_ERR_SHAPE, "batch and head counts must be <= 65535");
    if (T > 0x7fffffff || need > 0x7fffffffLL)
        return fail(MODA_ERR_SHAPE, "T and T*num_layers must fit in 31 bits");
    (void)numel;
    out->q = *q;
    out->k = *k;
    out->v = *v;
    out->kd = *kd;
    out->vd = *vd;
    out->o = *o;
    out->B = static_cast<int>(B);
    out->Hq = static_cast<int>(Hq);
    out->Hk = static_cast<int>(Hk);
    out->G = static_cast<int>(Hq / Hk);
    out->T = static_cast<int>(T);
    out->d = static_cast<int>(d);
    out->L = num_layers;
    out->zero_rows = 0;
    out->scale = scale > 0.f ? scale : 1.0f / sqrtf(static_cast<float>(d));
    out->lse = nullptr;
    out->dtype = dtype;
    return MODA_OK;
}

int plan_kernel(const moda::FwdParams& p, int kernel) {
    char why[256];
    switch (kernel) {
        case MODA_KERNEL_SIMT: return MODA_KERNEL_SIMT;
        case MODA_KERNEL_TC:
            if (!moda::tc_supports(p, why, sizeof(why)))
                return fail(MODA_ERR_UNSUPPORTED, "tcgen05 kernel forced but %s", why);
            return MODA_KERNEL_TC;
        case MODA_KERNEL_AUTO:
            return moda::tc_supports(p, why, sizeof(why)) ? MODA_KERNEL_TC : MODA_KERNEL_SIMT;
        default: return fail(MODA_ERR_ARG, "unknown kernel selector %d", kernel);
    }
}

int launch_validated(const moda::FwdParams& p, int kernel, cudaStream_t st) {
    const int which = plan_kernel(p, kernel);
    if (which < 0) return which;
    if (static_cast<int64_t>(p.B) * p.Hq * p.T * p.d == 0) return MODA_OK;  // nothing to write
    cudaGetLastError();  // clear a stale error so the check below is ours
    int r;
    if (which == MODA_KERNEL_TC) {
        char err[256] = "";
        r = moda::launch_fwd_tc(p, st, err, sizeof(err));
        if (r != MODA_OK) return fail(r, "%s", err[0] ? err : "tcgen05 launch failed");
    } else {
        r = moda::launch_fwd_simt(p, st);
        if (r != MODA_OK) return fail(r, "SIMT launch rejected");
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MODA_ERR_LAUNCH, "CUDA launch error: %s", cudaGetErrorString(e));
    return MODA_OK;
}

}  // namespace

extern "C" {

int moda_fwd_plan(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                  const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o, int num_layers,
                  int dtype, int kernel) {
    g_err[0] = 0;
    moda::FwdParams p;
    int r = validate_fwd(q, k, v, kd, vd, o, num_layers, 0.f, dtype, &p);
    if (r != MODA_OK) return r;
    return plan_kernel(p, kernel);
}

int moda_fwd_lse(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                 const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o, float* lse,
                 int num_layers, float scale, int chunk_size, int dtype, int kernel,
                 moda_stream_t stream) {
    g_err[0] = 0;
    if (chunk_size < 0) return fail(MODA_ERR_ARG, "chunk_size must be >= 0 (0 = none), got %d", chunk_size);
    moda::FwdParams p;
    int r = validate_fwd(q, k, v, kd, vd, o, num_layers, scale, dtype, &p);
    if (r != MODA_OK) return r;
    if (!lse && static_cast<int64_t>(p.B) * p.Hq * p.T > 0)
        return fail(MODA_ERR_ARG, "lse must point to B*H_q*T floats");
    p.lse = lse;
    return launch_validated(p, kernel, static_cast<cudaStream_t>(stream));
}

int moda_fwd_zero_depth(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                        const ModaTensor* o, float* lse, int zero_rows, float scale, int dtype,
                        int kernel, moda_stream_t stream) {
    g_err[0] = 0;
    if (zero_rows < 0) return fail(MODA_ERR_ARG, "zero_rows must be >= 0, got %d", zero_rows);
    if (!q || !k) return fail(MODA_ERR_ARG, "null tensor descriptor");
    // No depth tensor: empty [B, H_k, 0, d] descriptors that nothing reads.
    ModaTensor none;
    memset(&none, 0, sizeof(none));
    none.sizes[0] = q->sizes[0];
    none.sizes[1] = k->sizes[1];
    none.sizes[3] = q->sizes[3];
    none.strides[3] = 1;
    moda::FwdParams p;
    int r = validate_fwd(q, k, v, &none, &none, o, 0, scale, dtype, &p);
    if (r != MODA_OK) return r;
    p.lse = lse;
    p.zero_rows = zero_rows;
    return launch_validated(p, kernel, static_cast<cudaStream_t>(stream));
}

int moda_fwd_ex(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o, int num_layers,
                float scale, int chunk_size, int dtype, int kernel, moda_stream_t stream) {
    g_err[0] = 0;
    if (chunk_size < 0) return fail(MODA_ERR_ARG, "chunk_size must be >= 0 (0 = none), got %d", chunk_size);
    moda::FwdParams p;
    int r = validate_fwd(q, k, v, kd, vd, o, num_layers, scale, dtype, &p);
    if (r != MODA_OK) return r;
    p.lse = nullptr;
    return launch_validated(p, kernel, static_cast<cudaStream_t>(stream));
}

int64_t moda_bwd_workspace_size(int64_t batch, int64_t num_q_heads, int64_t seq_len) {
    if (batch < 0 || num_q_heads < 0 || seq_len < 0) return -1;
    return batch * num_q_heads * seq_len * static_cast<int64_t>(sizeof(float));
}

int moda_bwd_noalloc(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v,
                     const ModaTensor* kd, const ModaTensor* vd, const ModaTensor* o,
                     const ModaTensor* dout, const float* lse, const ModaTensor* dq,
                     const ModaTensor* dk, const ModaTensor* dv, const ModaTensor* dkd,
                     const ModaTensor* dvd, int num_layers, float scale, int dtype,
                     moda_stream_t stream) {
    g_err[0] = 0;
    // Size check first, before anything else touches the descriptors or CUDA.
    if (!q) return fail(MODA_ERR_ARG, "null tensor descriptor");
    // Each factor is checked before it is multiplied, so no product can overflow or
    // wrap back under the limit.
    int64_t rows = 1;
    for (int i = 0; i < 3; ++i) {
        if (q->sizes[i] < 0)
            return fail(MODA_ERR_SHAPE, "negative size %lld in dimension %d of q",
                        (long long)q->sizes[i], i);
        if (q->sizes[i] > MODA_NOALLOC_ROWS || __builtin_mul_overflow(rows, q->sizes[i], &rows) ||
            rows > MODA_NOALLOC_ROWS) {
            rows = -1;
            break;
        }
    }
    if (rows < 0 && q->sizes[0] != 0 && q->sizes[1] != 0 && q->sizes[2] != 0)
        return fail(MODA_ERR_UNSUPPORTED,
                    "moda_bwd_noalloc handles up to %d query rows (B*H_q*T), got %lld x %lld x %lld",
                    MODA_NOALLOC_ROWS, (long long)q->sizes[0], (long long)q->sizes[1],
                    (long long)q->sizes[2]);
    if (rows < 0) rows = 0;  // an empty dimension (with an oversize one): no rows
    void* scratch = nullptr;
    if (rows > 0 && moda::noalloc_scratch(&scratch) != cudaSuccess)
        return fail(MODA_ERR_LAUNCH, "could not resolve the library's backward scratch");
    return moda_bwd(q, k, v, kd, vd, o, dout, lse, dq, dk, dv, dkd, dvd, scratch,
                    static_cast<int64_t>(MODA_NOALLOC_ROWS) * static_cast<int64_t>(sizeof(float)),
                    num_layers, scale, dtype, stream);
}

int moda_bwd(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v, const ModaTensor* kd,
             const ModaTensor* vd, const ModaTensor* o, const ModaTensor* dout, const float* lse,
             const ModaTensor* dq, const ModaTensor* dk, const ModaTensor* dv,
             const ModaTensor* dkd, const ModaTensor* dvd, void* workspace,
             int64_t workspace_bytes, int num_layers, float scale, int dtype,
             moda_stream_t stream) {
    g_err[0] = 0;
    moda::FwdParams f;
    int r = validate_fwd(q, k, v, kd, vd, o, num_layers, scale, dtype, &f);
    if (r != MODA_OK) return r;
    if (!dout || !dq || !dk || !dv || !dkd || !dvd) return fail(MODA_ERR_ARG, "null gradient descriptor");
    const ModaTensor* like[5][2] = {{dout, o}, {dq, q}, {dk, k}, {dv, v}, {dkd, kd}};
    const char* names[5] = {"dO", "dQ", "dK", "dV", "dK_depth"};
    for (int i = 0; i < 5; ++i)
        for (int j = 0; j < 4; ++j)
            if (like[i][0]->sizes[j] != like[i][1]->sizes[j])
                return fail(MODA_ERR_SHAPE, "%s must have the shape of its tensor (dim %d: %lld vs %lld)",
                            names[i], j, (long long)like[i][0]->sizes[j], (long long)like[i][1]->sizes[j]);
    for (int j = 0; j < 4; ++j)
        if (dvd->sizes[j] != vd->sizes[j])
            return fail(MODA_ERR_SHAPE, "dV_depth must have the shape of V_depth");
    if (kd->sizes[2] != vd->sizes[2])
        return fail(MODA_ERR_SHAPE, "K_depth and V_depth must have the same number of rows");
    const int64_t rows = static_cast<int64_t>(f.B) * f.Hq * f.T;
    if (rows > 0 && !lse) return fail(MODA_ERR_ARG, "lse must point to B*H_q*T floats");
    if (workspace_bytes < moda_bwd_workspace_size(f.B, f.Hq, f.T) || (rows > 0 && !workspace))
        return fail(MODA_ERR_ARG, "workspace needs %lld bytes, got %lld",
                    (long long)moda_bwd_workspace_size(f.B, f.Hq, f.T), (long long)workspace_bytes);
    const ModaTensor* outs[5] = {dq, dk, dv, dkd, dvd};
    for (const ModaTensor* t : outs) {
        int64_t n = 1;
        for (int j = 0; j < 4; ++j) n *= t->sizes[j];
        if (n > 0 && !t->ptr) return fail(MODA_ERR_ARG, "a gradient tensor has a null data pointer");
    }
    if (dout->sizes[0] * dout->sizes[1] * dout->sizes[2] * dout->sizes[3] > 0 && !dout->ptr)
        return fail(MODA_ERR_ARG, "dO has a null data pointer");
    if (kd->sizes[2] > 0x7fffffffLL * 4)
        return fail(MODA_ERR_SHAPE, "depth buffer too large");
    moda::BwdParams p;
    p.q = *q; p.k = *k; p.v = *v; p.kd = *kd; p.vd = *vd; p.o = *o; p.dout = *dout;
    p.dq = *dq; p.dk = *dk; p.dv = *dv; p.dkd = *dkd; p.dvd = *dvd;
    p.lse = lse;
    p.delta = static_cast<float*>(workspace);
    p.B = f.B; p.Hq = f.Hq; p.Hk = f.Hk; p.G = f.G; p.T = f.T; p.d = f.d; p.L = f.L;
    p.R = kd->sizes[2];
    p.scale = f.scale;
    p.dtype = dtype;
    if (static_cast<int64_t>(p.B) * p.Hk * (p.T + p.R) * p.d == 0) return MODA_OK;
    cudaGetLastError();
    char err[256] = "";
    r = moda::launch_bwd(p, static_cast<cudaStream_t>(stream), err, sizeof(err));
    if (r != MODA_OK) return fail(r, "%s", err[0] ? err : "backward launch rejected");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MODA_ERR_LAUNCH, "CUDA launch error: %s", cudaGetErrorString(e));
    return MODA_OK;
}

int moda_fwd(const ModaTensor* q, const ModaTensor* k, const ModaTensor* v, const ModaTensor* kd,
             const ModaTensor* vd, const ModaTensor* o, int num_layers, float scale,
             int chunk_size, int dtype, moda_stream_t stream) {
    return moda_fwd_ex(q, k, v, kd, vd, o, num_layers, scale, chunk_size, dtype, MODA_KERNEL_AUTO,
                       stream);
}

int moda_depth_append(const ModaTensor* k_src, const ModaTensor* v_src, const ModaTensor* k_cache,
                      const ModaTensor* v_cache, int layer_idx, int num_layers, int seq_len,
                      int dtype, moda_stream_t stream) {
    g_err[0] = 0;
    if (!k_src || !v_src || !k_cache || !v_cache) return fail(MODA_ERR_ARG, "null tensor descriptor");
    if (!dtype_ok(dtype)) return fail(MODA_ERR_DTYPE, "unknown dtype code %d", dtype);
    if (num_layers <= 0) return fail(MODA_ERR_ARG, "num_layers must be > 0, got %d", num_layers);
    if (layer_idx < 0 || layer_idx >= num_layers)
        return fail(MODA_ERR_ARG, "layer_idx %d outside [0, %d)", layer_idx, num_layers);
    if (seq_len < 0) return fail(MODA_ERR_ARG, "seq_len must be >= 0");
    const int64_t B = k_cache->sizes[0], H = k_cache->sizes[1], d = k_cache->sizes[3];
    const ModaTensor* src[2] = {k_src, v_src};
    const ModaTensor* dst[2] = {k_cache, v_cache};
    for (int i = 0; i < 2; ++i) {
        if (src[i]->sizes[0] != B || src[i]->sizes[1] != H || src[i]->sizes[3] != d ||
            dst[i]->sizes[0] != B || dst[i]->sizes[1] != H || dst[i]->sizes[3] != d)
            return fail(MODA_ERR_SHAPE, "depth append: batch/head/head_dim mismatch");
        if (src[i]->sizes[2] < seq_len)
            return fail(MODA_ERR_SHAPE, "depth append: source has %lld rows < seq_len %d",
                        (long long)src[i]->sizes[2], seq_len);
        if (dst[i]->sizes[2] < static_cast<int64_t>(seq_len) * num_layers)
            return fail(MODA_ERR_DEPTH_ROWS, "depth append: cache has %lld rows < seq_len*L = %lld",
                        (long long)dst[i]->sizes[2], (long long)seq_len * num_layers);
    }
    if (B * H * seq_len * d == 0) return MODA_OK;
    moda::AppendParams p;
    p.k_src = *k_src;
    p.v_src = *v_src;
    p.k_cache = *k_cache;
    p.v_cache = *v_cache;
    p.B = static_cast<int>(B);
    p.H = static_cast<int>(H);
    p.T = seq_len;
    p.d = static_cast<int>(d);
    p.L = num_layers;
    p.layer = layer_idx;
    p.dtype = dtype;
    const int esz = dtype == MODA_F32 ? 4 : 2;
    bool vec16 = (d * esz) % 16 == 0;
    for (int i = 0; i < 2 && vec16; ++i) {
        const ModaTensor* ts[2] = {src[i], dst[i]};
        for (const ModaTensor* t : ts) {
            if (t->strides[3] != 1 || reinterpret_cast<uintptr_t>(t->ptr) % 16 != 0) vec16 = false;
            for (int j = 0; j < 3; ++j)
                if ((t->strides[j] * esz) % 16 != 0) vec16 = false;
        }
    }
    cudaGetLastError();
    int r = moda::launch_depth_append(p, vec16, static_cast<cudaStream_t>(stream));
    if (r != MODA_OK) return fail(r, "depth append launch rejected");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MODA_ERR_LAUNCH, "CUDA launch error: %s", cudaGetErrorString(e));
    return MODA_OK;
}

const char* moda_last_error(void) { return g_err; }

int moda_device_status(moda_stream_t stream) {
    int v = 0, w = 0, x = 0;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (moda::read_and_clear_status(st, &v) != cudaSuccess ||
        moda::read_and_clear_bwd_status(st, &w) != cudaSuccess ||
        moda::read_and_clear_proj_status(st, &x) != cudaSuccess)
        return fail(MODA_ERR_LAUNCH, "could not read the device status word");
    return v ? v : (w ? w : x);
}

int moda_depth_proj_append(const ModaTensor* x, const ModaTensor* w, const ModaTensor* k_cache,
                           const ModaTensor* v_cache, int layer_idx, int num_layers, int seq_len,
                           int dtype, moda_stream_t stream) {
    g_err[0] = 0;
    if (!x || !w || !k_cache || !v_cache) return fail(MODA_ERR_ARG, "null tensor descriptor");
    if (!dtype_ok(dtype)) return fail(MODA_ERR_DTYPE, "unknown dtype code %d", dtype);
    if (num_layers <= 0) return fail(MODA_ERR_ARG, "num_layers must be > 0, got %d", num_layers);
    if (layer_idx < 0 || layer_idx >= num_layers)
        return fail(MODA_ERR_ARG, "layer_idx %d outside [0, %d)", layer_idx, num_layers);
    const ModaTensor* all[4] = {x, w, k_cache, v_cache};
    for (const ModaTensor* t : all)
        for (int j = 0; j < 4; ++j)
            if (t->sizes[j] < 0) return fail(MODA_ERR_SHAPE, "negative size");
    const int64_t B = x->sizes[0], T = x->sizes[2], D = x->sizes[3];
    const int64_t Hk = k_cache->sizes[1], d = k_cache->sizes[3];
    if (x->sizes[1] != 1) return fail(MODA_ERR_SHAPE, "x must be [B, 1, T, D]");
    if (w->sizes[0] != 1 || w->sizes[1] != 1 || w->sizes[2] != 2 * Hk * d || w->sizes[3] != D)
        return fail(MODA_ERR_SHAPE, "w has shape [%lld,%lld,%lld,%lld], expected [1,1,2*H_k*d = %lld,%lld]",
                    (long long)w->sizes[0], (long long)w->sizes[1], (long long)w->sizes[2],
                    (long long)w->sizes[3], (long long)(2 * Hk * d), (long long)D);
    for (const ModaTensor* c : {k_cache, v_cache}) {
        if (c->sizes[0] != B || c->sizes[1] != Hk || c->sizes[3] != d)
            return fail(MODA_ERR_SHAPE, "k_cache and v_cache must both be [B, H_k, rows, d]");
    }
    if (seq_len < 0 || seq_len > T) return fail(MODA_ERR_ARG, "seq_len %d outside [0, T = %lld]", seq_len, (long long)T);
    for (const ModaTensor* c : {k_cache, v_cache})
        if (c->sizes[2] < static_cast<int64_t>(seq_len) * num_layers)
            return fail(MODA_ERR_DEPTH_ROWS, "cache has %lld rows < seq_len*L = %lld",
                        (long long)c->sizes[2], (long long)seq_len * num_layers);
    if (B > 65535 || T > 0x7fffffff || D > 0x7fffffff || 2 * Hk * d > 0x7fffffff)
        return fail(MODA_ERR_SHAPE, "sizes too large");
    for (const ModaTensor* t : all) {
        int64_t n = 1;
        for (int j = 0; j < 4; ++j) n *= t->sizes[j];
        if (n > 0 && !t->ptr) return fail(MODA_ERR_ARG, "null data pointer");
    }
    moda::ProjProblem q;
    q.x = *x;
    q.w = *w;
    q.out[0] = *k_cache;
    q.out[1] = *v_cache;
    q.out[2] = *v_cache;  // unused (nout = 2)
    q.nout = 2;
    q.heads[0] = q.heads[1] = static_cast<int>(Hk);
    q.heads[2] = 0;
    q.B = static_cast<int>(B);
    q.T = static_cast<int>(T);
    q.D = static_cast<int>(D);
    q.N = static_cast<int>(2 * Hk * d);
    q.d = static_cast<int>(d);
    q.L = num_layers;
    q.slot = layer_idx;
    q.n_write = seq_len;
    q.dtype = dtype;
    char why[256];
    if (!moda::proj_supports(q, why, sizeof(why)))
        return fail(MODA_ERR_UNSUPPORTED, "fused depth projection %s", why);
    if (B * Hk * static_cast<int64_t>(seq_len) * d == 0 || D == 0) {
        if (D == 0 && B * seq_len > 0)
            return fail(MODA_ERR_UNSUPPORTED, "fused depth projection needs D > 0");
        return MODA_OK;
    }
    cudaGetLastError();
    char err[256] = "";
    const int r = moda::launch_proj_append(q, static_cast<cudaStream_t>(stream), err, sizeof(err));
    if (r != MODA_OK) return fail(r, "%s", err[0] ? err : "projection launch failed");
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MODA_ERR_LAUNCH, "CUDA launch error: %s", cudaGetErrorString(e));
    return MODA_OK;
}

int moda_qkv_proj(const ModaTensor* x, const ModaTensor* w, const ModaTensor* q_out,
                  const ModaTensor* k_out, const ModaTensor* v_out, int dtype, moda_stream_t stream) {
    g_err[0] = 0;
    if (!x || !w || !q_out || !k_out || !v_out) return fail(MODA_ERR_ARG, "null tensor descriptor");
    if (!dtype_ok(dtype)) return fail(MODA_ERR_DTYPE, "unknown dtype code %d", dtype);
    const ModaTensor* all[5] = {x, w, q_out, k_out, v_out};
    for (const ModaTensor* t : all)
        for (int j = 0; j < 4; ++j)
            if (t->sizes[j] < 0) return fail(MODA_ERR_SHAPE, "negative size");
    const int64_t B = x->sizes[0], T = x->sizes[2], D = x->sizes[3];
    const int64_t Hq = q_out->sizes[1], Hk = k_out->sizes[1], d = q_out->sizes[3];
    if (x->sizes[1] != 1) return fail(MODA_ERR_SHAPE, "x must be [B, 1, T, D]");
    if (q_out->sizes[0] != B || q_out->sizes[2] != T)
        return fail(MODA_ERR_SHAPE, "q must be [B, H_q, T, d] with x's B and T");
    for (const ModaTensor* o : {k_out, v_out})
        if (o->sizes[0] != B || o->sizes[1] != Hk || o->sizes[2] != T || o->sizes[3] != d)
            return fail(MODA_ERR_SHAPE, "k and v must both be [B, H_k, T, d] (d of q)");
    const int64_t N = (Hq + 2 * Hk) * d;
    if (w->sizes[0] != 1 || w->sizes[1] != 1 || w->sizes[2] != N || w->sizes[3] != D)
        return fail(MODA_ERR_SHAPE, "w has shape [%lld,%lld,%lld,%lld], expected [1,1,(H_q+2*H_k)*d = %lld,%lld]",
                    (long long)w->sizes[0], (long long)w->sizes[1], (long long)w->sizes[2],
                    (long long)w->sizes[3], (long long)N, (long long)D);
    if (B > 65535 || T > 0x7fffffff || D > 0x7fffffff || N > 0x7fffffff)
        return fail(MODA_ERR_SHAPE, "sizes too large");
    for (const ModaTensor* t : all) {
        int64_t n = 1;
        for (int j = 0; j < 4; ++j) n *= t->sizes[j];
        if (n > 0 && !t->ptr) return fail(MODA_ERR_ARG, "null data pointer");
    }
    moda::ProjProblem q;
    q.x = *x;
    q.w = *w;
    q.out[0] = *q_out;
    q.out[1] = *k_out;
    q.out[2] = *v_out;
    q.nout = 3;
    q.heads[0] = static_cast<int>(Hq);
    q.heads[1] = q.heads[2] = static_cast<int>(Hk);
    q.B = static_cast<int>(B);
    q.T = static_cast<int>(T);
    q.D = static_cast<int>(D);
    q.N = static_cast<int>(N);
    q.d = static_cast<int>(d);
    q.L = 1;
    q.slot = 0;
    q.n_write = static_cast<int>(T);
    q.dtype = dtype;
    char why[256];
    if (!moda::proj_supports(q, why, sizeof(why)))
        return fail(MODA_ERR_UNSUPPORTED, "fused QKV projection %s", why);
    if (B * T * N == 0) return MODA_OK;
    if (D == 0) return fail(MODA_ERR_UNSUPPORTED, "fused QKV projection needs D > 0");
    cudaGetLastError();
    char err[256] = "";
    const int r = moda::launch_proj_append(q, static_cast<cudaStream_t>(stream), err, sizeof(err));
    if (r != MODA_OK) return fail(r, "%s", err[0] ? err : "projection launch failed");
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MODA_ERR_LAUNCH, "CUDA launch error: %s", cudaGetErrorString(e));
    return MODA_OK;
}

int moda_version(void) { return 200; }

}  // extern "C"
