// extern "C" entry points of libsaeflow_b200.so: argument validation, workspace layout,
// kernel selection. The entry points mirror the host wrappers of saeflow/kernels
// (encode.py:97-139, decode.py:77-126) one level down: the caller owns every buffer.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "sf_common.cuh"
#include "sf_internal.h"

namespace sf {

// Defined in sparse.cu
int launch_row_nnz(const sf_matrix &f, int32_t *row_nnz, cudaStream_t s);
int launch_indptr(const int32_t *cnt, int64_t M, int64_t *indptr, cudaStream_t s, const unsigned *skip = nullptr);
int launch_compact(const sf_matrix &f, const int64_t *indptr, int32_t *indices, void *values, int vdt,
                   cudaStream_t s);
int launch_decode(const int64_t *indptr, int64_t M, const int32_t *indices, const void *values, int vdt,
                  const sf_matrix &W, const sf_vector *b, const sf_matrix &out, cudaStream_t s);
int launch_topk_merge(const unsigned long long *cand, int64_t M, int ncand, int k, int32_t *out_idx, void *out_val,
                      int vdt, cudaStream_t s);
int launch_topk_rows(const sf_matrix &f, int k, int32_t *out_idx, void *out_val, int vdt, cudaStream_t s);
int launch_csr_place(const int32_t *tile_cnt, const int32_t *tile_off, int64_t n_tiles, const int32_t *stage_idx,
                     const void *stage_val, int64_t stage_cap, int vdt, const int64_t *indptr, int64_t M,
                     int32_t *indices, void *values, cudaStream_t s, const unsigned *skip = nullptr);

namespace {
thread_local char g_last_error[512] = "";

// One error word per device, read back by sf_device_error().
__device__ unsigned g_error_word;

constexpr int kMaxDevices = 64;
unsigned *g_error_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
std::mutex g_dev_mu;

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}
}  // namespace

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int check_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return SF_OK;
    return set_error(SF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t dtype_size(int dtype) { return dtype == SF_F32 ? 4 : 2; }
bool valid_dtype(int dtype) { return dtype == SF_F32 || dtype == SF_BF16 || dtype == SF_F16; }

unsigned *device_error_word() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!g_error_ptr[d]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_error_word) == cudaSuccess) g_error_ptr[d] = static_cast<unsigned *>(p);
    }
    return g_error_ptr[d];
}

int num_sms() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return 148;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!g_sms[d]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) n = 148;
        g_sms[d] = n;
    }
    return g_sms[d];
}

namespace {

// ------------------------------------------------------------------ pre-pass kernels
// xs[m, k] = MT(float(x[m, k]) - float(b_dec[k])) for k < K, 0 for K <= k < pitch.
// Rounding to the MMA dtype after an fp32 subtraction is the reference prologue
// (saeflow/kernels/encode.py:72 of _encode_kernel).
template <typename XT, typename MT>
__global__ void shift_convert_kernel(const XT *__restrict__ x, int64_t M, int64_t K, int64_t sxm, int64_t sxk,
                                     const void *b_dec, int b_dtype, int64_t b_stride, MT *__restrict__ xs,
                                     int64_t pitch, const unsigned *gate) {
    if (gate != nullptr && *reinterpret_cast<const volatile unsigned *>(gate) == 0u) return;
    constexpr int EPV = 16 / sizeof(MT);
    const int64_t vec_per_row = pitch / EPV;
    const int64_t total = M * vec_per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / vec_per_row;
        const int64_t k0 = (i - m * vec_per_row) * EPV;
        uint4 pk;
        MT *o = reinterpret_cast<MT *>(&pk);
        const XT *xr = x + m * sxm;
#pragma unroll
        for (int e = 0; e < EPV; ++e) {
            const int64_t k = k0 + e;
            float v = 0.f;
            if (k < K) {
                v = to_f32(xr[k * sxk]);
                if (b_dec) v -= load_as_f32(b_dec, b_dtype, k * b_stride);
            }
            o[e] = from_f32<MT>(k < K ? v : 0.f);
        }
        *reinterpret_cast<uint4 *>(xs + m * pitch + k0) = pk;
    }
}

// Contiguous fast path: 16-byte loads of x (x rows contiguous, K multiple of EPV_X).
template <typename XT, typename MT>
__global__ void shift_convert_vec_kernel(const XT *__restrict__ x, int64_t M, int64_t K, int64_t sxm,
                                         const void *b_dec, int b_dtype, int64_t b_stride, MT *__restrict__ xs,
                                         int64_t pitch, const unsigned *gate) {
    if (gate != nullptr && *reinterpret_cast<const volatile unsigned *>(gate) == 0u) return;
    constexpr int EPV = 8;  // elements per work item (16 B of 16-bit, 32 B of fp32)
    const int64_t items_per_row = pitch / EPV;
    const int64_t total = M * items_per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / items_per_row;
        const int64_t k0 = (i - m * items_per_row) * EPV;
        float v[EPV];
        if (k0 + EPV <= K) {
            const XT *src = x + m * sxm + k0;
            if (sizeof(XT) == 2) {
                const uint4 q = __ldg(reinterpret_cast<const uint4 *>(src));
                const XT *e = reinterpret_cast<const XT *>(&q);
#pragma unroll
                for (int t = 0; t < EPV; ++t) v[t] = to_f32(e[t]);
            } else {
                const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(src));
                const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(src) + 1);
                const XT *e0 = reinterpret_cast<const XT *>(&q0);
                const XT *e1 = reinterpret_cast<const XT *>(&q1);
#pragma unroll
                for (int t = 0; t < 4; ++t) v[t] = to_f32(e0[t]), v[t + 4] = to_f32(e1[t]);
            }
#pragma unroll
            for (int t = 0; t < EPV; ++t)
                if (b_dec) v[t] -= load_as_f32(b_dec, b_dtype, (k0 + t) * b_stride);
        } else {
#pragma unroll
            for (int t = 0; t < EPV; ++t) {
                const int64_t k = k0 + t;
                v[t] = k < K ? to_f32(x[m * sxm + k]) - (b_dec ? load_as_f32(b_dec, b_dtype, k * b_stride) : 0.f)
                             : 0.f;
            }
        }
        MT *dst = xs + m * pitch + k0;
        if (sizeof(MT) == 2) {
            uint4 pk;
            MT *o = reinterpret_cast<MT *>(&pk);
#pragma unroll
            for (int t = 0; t < EPV; ++t) o[t] = from_f32<MT>(v[t]);
            *reinterpret_cast<uint4 *>(dst) = pk;
        } else {
            float4 *d4 = reinterpret_cast<float4 *>(dst);
            d4[0] = make_float4(v[0], v[1], v[2], v[3]);
            d4[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    }
}

// wp[k, n] = W[k, n] (row pitch `pitch`, zero padding) — makes any W_enc layout TMA-readable.
template <typename T>
__global__ void repack_kernel(const T *__restrict__ W, int64_t K, int64_t N, int64_t swk, int64_t swn,
                              T *__restrict__ wp, int64_t pitch) {
    const int64_t total = K * pitch;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = i / pitch, n = i - k * pitch;
        wp[i] = n < N ? W[k * swk + n * swn] : from_f32<T>(0.f);
    }
}

// wt[n, k] = W[k, n] (row pitch `pitch` >= K, zero padding): K-major copy of W_enc for
// the TF32 path, whose 32-bit operands the tensor cores read K-major. 32 x 32 tiles
// through shared memory so both the read and the write are coalesced.
template <typename T>
__global__ void repack_t_kernel(const T *__restrict__ W, int64_t K, int64_t N, int64_t swk, int64_t swn,
                                T *__restrict__ wt, int64_t pitch) {
    __shared__ T tile[32][33];
    const int64_t n0 = (int64_t)blockIdx.x * 32, k0 = (int64_t)blockIdx.y * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    for (int i = ty; i < 32; i += 8) {
        const int64_t k = k0 + i, n = n0 + tx;
        tile[i][tx] = (k < K && n < N) ? W[k * swk + n * swn] : from_f32<T>(0.f);
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int64_t n = n0 + i, k = k0 + tx;
        if (n < N && k < pitch) wt[n * pitch + k] = tile[tx][i];
    }
}

template <typename F>
int by_dtype2(int dt, F &&f) {
    if (dt == SF_F32) return f(float{});
    if (dt == SF_BF16) return f(__nv_bfloat16{});
    return f(__half{});
}

unsigned grid_for(int64_t items) {
    const int64_t per = 256;
    int64_t blocks = (items + per - 1) / per;
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// ------------------------------------------------------------------ validation
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_matrix(const sf_matrix *m, const char *name) {
    if (!m) return set_error(SF_ERR_INVALID, "%s is NULL", name);
    if (!valid_dtype(m->dtype)) return set_error(SF_ERR_INVALID, "%s has unsupported dtype code %d", name, m->dtype);
    if (m->rows < 0 || m->cols < 0) return set_error(SF_ERR_INVALID, "%s has a negative extent", name);
    if (m->rows > 0 && m->cols > 0 && !m->data) return set_error(SF_ERR_INVALID, "%s has no data", name);
    if (m->rows > (int64_t)INT32_MAX || m->cols > (int64_t)INT32_MAX)
        return set_error(SF_ERR_UNSUPPORTED, "%s extent exceeds 2^31-1", name);
    return SF_OK;
}

int check_vector(const sf_vector *v, int64_t len, const char *name, bool optional) {
    if (!v || !v->data) {
        if (optional) return SF_OK;
        return set_error(SF_ERR_INVALID, "%s is required", name);
    }
    if (!valid_dtype(v->dtype)) return set_error(SF_ERR_INVALID, "%s has unsupported dtype code %d", name, v->dtype);
    if (v->len != len)
        return set_error(SF_ERR_INVALID, "%s has length %lld, expected %lld", name, (long long)v->len, (long long)len);
    return SF_OK;
}

// MMA type from W_enc's dtype and the TF32 switch (encode.py:118-120: fp32 inputs use
// IEEE products unless TF32 is allowed; any 16-bit input forces the tensor-core path).
struct EncodePlan {
    bool tensor_cores;
    int ab_fmt;      // 0 f16, 1 bf16, 2 tf32
    int mma_dtype;   // storage dtype of the shifted x copy
    int64_t a_pitch;
    bool w_direct;   // TMA reads W_enc in place
    bool b_mn;
    int64_t w_pitch; // pitch of W_enc as TMA sees it (elements)
    size_t xs_bytes, wp_bytes;
    bool fused_x;    // the CTA-pair kernel's converter warps read x itself and shift it (no copy)
    // IEEE fp32 on the bf16 tensor cores (emulate.cu), in nkc K ranges of kc columns of x
    // (the last one shorter). Workspace: the split x of one range [M, 3 kp] bf16, then (at
    // xs32_off) the fp32 shifted x of the non-finite fallback, the fallback flag (at
    // flag_off), with more than one range the fp32 partial sums [M, part_pitch] (at
    // part_off), then the split W_enc of one range [3 kp, w_pitch] bf16.
    bool emulate;
    int nkc;
    int64_t kc, kp, xs32_pitch, part_pitch;
    size_t xs32_off, flag_off, part_off;
};

int plan_encode(const sf_matrix *x, const sf_matrix *W, int allow_tf32, int variant, EncodePlan *pl) {
    const int64_t M = x->rows, K = x->cols, N = W->cols;
    const int wdt = W->dtype;
    if (variant < SF_VARIANT_AUTO || variant > SF_VARIANT_TCGEN05_SINGLE)
        return set_error(SF_ERR_INVALID, "unknown encode variant %d", variant);
    bool tc;
    pl->emulate = false;
    if (wdt == SF_F32) {
        // IEEE products (fp32 x, TF32 not allowed) run split-precision on the bf16 tensor
        // cores unless the CUDA-core kernel is asked for; TF32 products on the tensor cores.
        const bool ieee = !allow_tf32 && x->dtype == SF_F32;
        tc = variant != SF_VARIANT_SIMT;
        pl->emulate = ieee && tc;
    } else {
        tc = true;
        if (variant == SF_VARIANT_SIMT)
            return set_error(SF_ERR_UNSUPPORTED, "the CUDA-core encode kernel is fp32 only");
    }
    pl->tensor_cores = tc;
    pl->mma_dtype = wdt;
    pl->ab_fmt = wdt == SF_F32 ? 2 : (wdt == SF_BF16 ? 1 : 0);
    const int64_t es = (int64_t)dtype_size(wdt);
    const int64_t epv = 16 / es;
    // Shifted x: rows padded to 16 B (vector kernel writes 8 elements per item).
    pl->a_pitch = round_up(K > 0 ? K : 1, 8);
    pl->xs_bytes = (size_t)(M * pl->a_pitch * es);
    // Fused shift: 16-bit operands on the CTA-pair kernel (M > 128 rows) with x in W_enc's
    // dtype, K-contiguous, 16-byte-aligned rows and d_in a multiple of 8 (whole 16-byte
    // chunks). Otherwise the shift pass writes the shifted copy the kernel reads.
    pl->fused_x = kFusedShift && tc && wdt != SF_F32 && M > 128 && variant != SF_VARIANT_TCGEN05_SINGLE &&
                  x->dtype == wdt && x->stride_col == 1 && (x->stride_row % 8) == 0 && x->stride_row >= K &&
                  aligned16(x->data) && (K % 8) == 0;
    if (pl->fused_x) pl->xs_bytes = 0;
    pl->wp_bytes = 0;
    pl->w_direct = true;
    pl->b_mn = true;
    pl->w_pitch = 0;
    if (pl->emulate) {
        pl->ab_fmt = 1;
        pl->mma_dtype = SF_BF16;
        const int64_t k1 = K > 0 ? K : 1;
        const int64_t ranges = (k1 + kEmuMaxRangeK - 1) / kEmuMaxRangeK;
        pl->kc = ranges == 1 ? k1 : round_up((k1 + ranges - 1) / ranges, kEmuKBlock);
        pl->nkc = (int)((k1 + pl->kc - 1) / pl->kc);
        pl->kp = round_up(pl->kc, kEmuKBlock);
        pl->a_pitch = 3 * pl->kp;
        pl->xs32_pitch = round_up(k1, 8);
        pl->xs32_off = (size_t)round_up(M * pl->a_pitch * 2, 256);
        pl->flag_off = pl->xs32_off + (size_t)round_up(M * pl->xs32_pitch * 4, 256);
        pl->part_off = pl->flag_off + 256;
        pl->part_pitch = round_up(N > 0 ? N : 1, kCsrTile);  // whole 256-column tiles
        pl->xs_bytes = pl->part_off + (pl->nkc > 1 ? (size_t)round_up(M * pl->part_pitch * 4, 256) : 0);
        pl->w_direct = false;
        pl->b_mn = true;
        pl->w_pitch = round_up(N > 0 ? N : 1, 8);
        pl->wp_bytes = (size_t)(3 * pl->kp * pl->w_pitch * 2);
        return SF_OK;
    }
    if (tc && wdt == SF_F32) {
        // 32-bit operands: feed W_enc K-major (in place when it is column-major).
        pl->b_mn = false;
        if (W->stride_row == 1 && (W->stride_col * es) % 16 == 0 && aligned16(W->data) && W->stride_col >= K) {
            pl->w_pitch = W->stride_col;
        } else {
            pl->w_direct = false;
            pl->w_pitch = round_up(K > 0 ? K : 1, epv);
            pl->wp_bytes = (size_t)(N * pl->w_pitch * es);
        }
    } else if (tc) {
        const bool al = aligned16(W->data);
        if (W->stride_col == 1 && (W->stride_row * es) % 16 == 0 && al && W->stride_row >= N) {
            pl->b_mn = true;
            pl->w_pitch = W->stride_row;
        } else if (W->stride_row == 1 && (W->stride_col * es) % 16 == 0 && al && W->stride_col >= K) {
            pl->b_mn = false;
            pl->w_pitch = W->stride_col;
        } else {
            pl->w_direct = false;
            pl->b_mn = true;
            pl->w_pitch = round_up(N > 0 ? N : 1, epv);
            pl->wp_bytes = (size_t)(K * pl->w_pitch * es);
        }
    }
    return SF_OK;
}

size_t plan_workspace(const EncodePlan &pl) { return round_up((int64_t)pl.xs_bytes, 256) + pl.wp_bytes; }

// The GEMM's A operand: x itself with b_dec for the converter warps (fused shift), or the
// shifted copy `xs` that run_shift_convert wrote.
void set_a_operand(GemmOperands &g, const EncodePlan &pl, const sf_matrix *x, const sf_vector *b_dec, void *xs) {
    g.bdec = nullptr;
    g.bdec_mode = 0;
    if (!pl.fused_x) {
        g.a = xs;
        g.a_pitch = pl.a_pitch;
        return;
    }
    g.a = x->data;
    g.a_pitch = x->stride_row;
    if (b_dec && b_dec->data) {
        g.bdec = b_dec->data;
        g.bdec_dtype = b_dec->dtype;
        g.bdec_stride = b_dec->stride;
        const bool packed = b_dec->stride == 1 && aligned16(b_dec->data);
        g.bdec_mode = !packed ? 3 : (b_dec->dtype == SF_F32 ? 2 : 1);
    }
}

// gate: non-null makes the pass a no-op unless *gate is nonzero at run time.
int run_shift_convert(const sf_matrix *x, const sf_vector *b_dec, int mdt, void *xs, int64_t pitch, cudaStream_t s,
                      const unsigned *gate = nullptr) {
    const int64_t M = x->rows, K = x->cols;
    if (M == 0) return SF_OK;
    const void *bp = (b_dec && b_dec->data) ? b_dec->data : nullptr;
    const int bdt = bp ? b_dec->dtype : 0;
    const int64_t bs = bp ? b_dec->stride : 0;
    return by_dtype2(x->dtype, [&](auto xtag) {
        using XT = decltype(xtag);
        return by_dtype2(mdt, [&](auto mtag) {
            using MT = decltype(mtag);
            const int64_t xe = sizeof(XT);
            const bool vec = x->stride_col == 1 && (x->stride_row * xe) % 16 == 0 && aligned16(x->data) &&
                             (K % (16 / xe)) == 0;
            // A gated pass (a no-op unless a flag is set) runs on one CTA per SM, grid-stride.
            auto grid = [&](int64_t items) { return gate ? std::min<unsigned>(grid_for(items), num_sms()) : grid_for(items); };
            if (vec) {
                const int64_t items = M * (pitch / 8);
                shift_convert_vec_kernel<XT, MT><<<grid(items), 256, 0, s>>>(
                    reinterpret_cast<const XT *>(x->data), M, K, x->stride_row, bp, bdt, bs,
                    reinterpret_cast<MT *>(xs), pitch, gate);
            } else {
                const int64_t items = M * (pitch / (16 / (int64_t)sizeof(MT)));
                shift_convert_kernel<XT, MT><<<grid(items), 256, 0, s>>>(
                    reinterpret_cast<const XT *>(x->data), M, K, x->stride_row, x->stride_col, bp, bdt, bs,
                    reinterpret_cast<MT *>(xs), pitch, gate);
            }
            return check_cuda(cudaGetLastError(), "shift_convert launch");
        });
    });
}

int run_repack(const sf_matrix *W, void *wp, int64_t pitch, bool mn_major, cudaStream_t s) {
    const int64_t K = W->rows, N = W->cols;
    return by_dtype2(W->dtype, [&](auto tag) {
        using T = decltype(tag);
        if (!mn_major) {
            dim3 grid((unsigned)((N + 31) / 32), (unsigned)((pitch + 31) / 32));
            repack_t_kernel<T><<<grid, dim3(32, 8), 0, s>>>(reinterpret_cast<const T *>(W->data), K, N,
                                                            W->stride_row, W->stride_col, reinterpret_cast<T *>(wp),
                                                            pitch);
            return check_cuda(cudaGetLastError(), "repack launch");
        }
        repack_kernel<T><<<grid_for(K * pitch), 256, 0, s>>>(reinterpret_cast<const T *>(W->data), K, N,
                                                             W->stride_row, W->stride_col, reinterpret_cast<T *>(wp),
                                                             pitch);
        return check_cuda(cudaGetLastError(), "repack launch");
    });
}

// Pre-passes of a tensor-core plan and the GEMM operands they leave in the workspace: the
// operand split (split-precision fp32), or the shifted copy of x and, when TMA cannot read
// W_enc in place, its repacked copy.
int prepare_tc(const EncodePlan &pl, const sf_matrix *x, const sf_matrix *W, const sf_vector *b_dec, uint8_t *ws,
               cudaStream_t s, GemmOperands &g, int range = 0) {
    g = GemmOperands{};
    g.M = x->rows;
    g.N = W->cols;
    void *wp = ws + round_up((int64_t)pl.xs_bytes, 256);
    if (pl.emulate) {
        // K range `range`: columns [k0, k0 + kc) of x and rows of W_enc
        const int64_t k0 = range * pl.kc;
        const int64_t kr = std::min<int64_t>(pl.kc, x->cols - k0);
        EmuOperands e{};
        e.x = static_cast<const float *>(x->data) + k0 * x->stride_col;
        e.M = x->rows;
        e.K = kr;
        e.sxm = x->stride_row;
        e.sxk = x->stride_col;
        if (b_dec && b_dec->data) {
            e.b_dec = static_cast<const uint8_t *>(b_dec->data) + k0 * b_dec->stride * (int64_t)dtype_size(b_dec->dtype);
            e.b_dtype = b_dec->dtype;
            e.b_stride = b_dec->stride;
        }
        e.W = static_cast<const float *>(W->data) + k0 * W->stride_row;
        e.N = W->cols;
        e.swk = W->stride_row;
        e.swn = W->stride_col;
        e.a = reinterpret_cast<__nv_bfloat16 *>(ws);
        e.b = static_cast<__nv_bfloat16 *>(wp);
        e.kp = pl.kp;
        e.b_pitch = pl.w_pitch;
        e.flag = reinterpret_cast<unsigned *>(ws + pl.flag_off);
        e.reset_flag = range == 0;
        const int st = emu_split_operands(e, s);
        if (st) return st;
        g.a = ws;
        g.a_pitch = pl.a_pitch;
        g.b = wp;
        g.b_pitch = pl.w_pitch;
        g.b_mn_major = true;
        g.ab_fmt = 1;
        g.K = 3 * pl.kp;
        g.seg_kb = (int)(pl.kp / kEmuKBlock);
        g.seg_a = kEmuSegA;
        g.seg_b = kEmuSegB;
        g.skip = e.flag;
        return SF_OK;
    }
    if (!pl.fused_x) {
        const int st = run_shift_convert(x, b_dec, pl.mma_dtype, ws, pl.a_pitch, s);
        if (st) return st;
    }
    set_a_operand(g, pl, x, b_dec, ws);
    g.ab_fmt = pl.ab_fmt;
    g.K = x->cols;
    g.b_mn_major = pl.b_mn;
    if (pl.w_direct) {
        g.b = W->data;
        g.b_pitch = pl.w_pitch;
        return SF_OK;
    }
    const int st = run_repack(W, wp, pl.w_pitch, pl.b_mn, s);
    if (st) return st;
    g.b = wp;
    g.b_pitch = pl.w_pitch;
    return SF_OK;
}

// The split-precision encode over its K ranges: ranges before the last store (the first) or
// add to (the others) the fp32 partial sums with the raw epilogue; the last runs `final`
// (the dense or CSR epilogue) with those partial sums added to its accumulators.
template <typename Final>
int run_emulated(const EncodePlan &pl, const sf_matrix *x, const sf_matrix *W, const sf_vector *b_dec,
                 const sf_vector *b_enc, uint8_t *ws, int variant, cudaStream_t s, Final final) {
    float *part = reinterpret_cast<float *>(ws + pl.part_off);
    for (int r = 0; r < pl.nkc; ++r) {
        GemmOperands g;
        int st = prepare_tc(pl, x, W, b_dec, ws, s, g, r);
        if (st) return st;
        if (r + 1 == pl.nkc) return final(g, pl.nkc > 1 ? part : nullptr, pl.part_pitch);
        EpilogueArgs raw{};
        raw.b_enc = b_enc->data;  // staged by the epilogue, unused by a raw pass
        raw.b_enc_dtype = b_enc->dtype;
        raw.b_enc_stride = b_enc->stride;
        raw.activation = SF_ACT_RELU;
        raw.out = part;
        raw.out_dtype = SF_F32;
        raw.out_sm = pl.part_pitch;
        raw.out_sn = 1;
        raw.out_vec = 1;
        raw.raw = 1;
        raw.c_in = r > 0 ? part : nullptr;
        raw.c_in_pitch = pl.part_pitch;
        st = encode_tc_dense(g, raw, variant, s);
        if (st) return st;
    }
    return SF_OK;
}

// Behind a split-precision GEMM: when the split found an inf or NaN operand (the GEMM then
// exited at once), the shifted fp32 x and the CUDA-core IEEE kernel compute the call; both
// launches are no-ops otherwise.
int run_emu_fallback(const EncodePlan &pl, const sf_matrix *x, const sf_matrix *W, const sf_vector *b_dec,
                     uint8_t *ws, const EpilogueArgs &ep, const CsrArgs *csr, cudaStream_t s) {
    const unsigned *flag = reinterpret_cast<const unsigned *>(ws + pl.flag_off);
    float *xs32 = reinterpret_cast<float *>(ws + pl.xs32_off);
    const int st = run_shift_convert(x, b_dec, SF_F32, xs32, pl.xs32_pitch, s, flag);
    if (st) return st;
    return encode_simt_f32(xs32, pl.xs32_pitch, static_cast<const float *>(W->data), W->stride_row, W->stride_col,
                           x->rows, W->cols, x->cols, ep, s, csr, flag);
}

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

const char *sf_last_error(void) { return g_last_error; }

int sf_abi_version(void) { return SF_ABI_VERSION; }

int sf_device_error(uint32_t *code) {
    if (!code) return set_error(SF_ERR_INVALID, "code is NULL");
    *code = 0;
    unsigned *w = device_error_word();
    if (!w) return set_error(SF_ERR_CUDA, "device error word unavailable");
    int st = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    if (st) return st;
    unsigned v = 0;
    st = check_cuda(cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost), "read device error word");
    if (st) return st;
    const unsigned zero = 0;
    st = check_cuda(cudaMemcpy(w, &zero, sizeof(zero), cudaMemcpyHostToDevice), "clear device error word");
    if (st) return st;
    *code = v;
    return SF_OK;
}

int sf_fused_encode_workspace(const sf_matrix *x, const sf_matrix *W_enc, int allow_tf32, int variant,
                              size_t *bytes) {
    if (!bytes) return set_error(SF_ERR_INVALID, "bytes is NULL");
    *bytes = 0;
    int st = check_matrix(x, "x");
    if (!st) st = check_matrix(W_enc, "W_enc");
    if (st) return st;
    if (x->cols != W_enc->rows)
        return set_error(SF_ERR_INVALID, "x has d_in=%lld but W_enc has d_in=%lld", (long long)x->cols,
                         (long long)W_enc->rows);
    EncodePlan pl;
    st = plan_encode(x, W_enc, allow_tf32, variant, &pl);
    if (st) return st;
    *bytes = plan_workspace(pl);
    return SF_OK;
}

int sf_fused_encode(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc, const sf_vector *b_dec,
                    const sf_vector *threshold, int activation, const sf_matrix *out, int32_t *row_nnz,
                    int allow_tf32, int variant, void *workspace, size_t workspace_bytes, sf_stream stream) {
    int st = check_matrix(x, "x");
    if (!st) st = check_matrix(W_enc, "W_enc");
    if (!st) st = check_matrix(out, "out");
    if (st) return st;
    const int64_t M = x->rows, K = x->cols, N = W_enc->cols;
    if (activation != SF_ACT_RELU && activation != SF_ACT_JUMPRELU)
        return set_error(SF_ERR_INVALID, "unknown activation code %d", activation);
    if (K != W_enc->rows)
        return set_error(SF_ERR_INVALID, "x has d_in=%lld but W_enc has d_in=%lld", (long long)K,
                         (long long)W_enc->rows);
    if (out->rows != M || out->cols != N)
        return set_error(SF_ERR_INVALID, "out must be [%lld, %lld]", (long long)M, (long long)N);
    st = check_vector(b_enc, N, "b_enc", false);
    if (!st) st = check_vector(b_dec, K, "b_dec", true);
    if (!st) st = check_vector(threshold, N, "threshold", activation != SF_ACT_JUMPRELU);
    if (st) return st;
    if (M == 0 || N == 0) return SF_OK;

    EncodePlan pl;
    st = plan_encode(x, W_enc, allow_tf32, variant, &pl);
    if (st) return st;
    const size_t need = plan_workspace(pl);
    if (workspace_bytes < need || (!workspace && need))
        return set_error(SF_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    if (!aligned16(workspace)) return set_error(SF_ERR_WORKSPACE, "workspace must be 16-byte aligned");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

    uint8_t *ws = static_cast<uint8_t *>(workspace);

    EpilogueArgs ep{};
    ep.b_enc = b_enc->data;
    ep.b_enc_dtype = b_enc->dtype;
    ep.b_enc_stride = b_enc->stride;
    if (threshold && threshold->data) {
        ep.thr = threshold->data;
        ep.thr_dtype = threshold->dtype;
        ep.thr_stride = threshold->stride;
    }
    ep.activation = activation;
    ep.out = const_cast<void *>(out->data);
    ep.out_dtype = out->dtype;
    ep.out_sm = out->stride_row;
    ep.out_sn = out->stride_col;
    ep.out_vec = (out->stride_col == 1 && (out->stride_row * (int64_t)dtype_size(out->dtype)) % 16 == 0 &&
                  aligned16(out->data))
                     ? 1
                     : 0;
    ep.row_nnz = row_nnz;

    if (!pl.tensor_cores) {
        st = run_shift_convert(x, b_dec, pl.mma_dtype, ws, pl.a_pitch, s);
        if (st) return st;
        return encode_simt_f32(reinterpret_cast<const float *>(ws), pl.a_pitch,
                               static_cast<const float *>(W_enc->data), W_enc->stride_row, W_enc->stride_col, M, N,
                               K, ep, s);
    }
    if (pl.emulate) {
        st = run_emulated(pl, x, W_enc, b_dec, b_enc, ws, variant, s,
                          [&](const GemmOperands &g, const float *part, int64_t pitch) {
                              EpilogueArgs e = ep;
                              e.c_in = part;
                              e.c_in_pitch = pitch;
                              return encode_tc_dense(g, e, variant, s);
                          });
        if (st) return st;
        return run_emu_fallback(pl, x, W_enc, b_dec, ws, ep, nullptr, s);
    }
    GemmOperands g;
    st = prepare_tc(pl, x, W_enc, b_dec, ws, s, g);
    if (st) return st;
    return encode_tc_dense(g, ep, variant, s);
}

int sf_encode_csr_stage(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc, const sf_vector *b_dec,
                        const sf_vector *threshold, int activation, int values_dtype, int32_t *row_nnz,
                        int32_t *tile_counts, int32_t *tile_offsets, int32_t *stage_indices, void *stage_values,
                        int64_t stage_capacity, uint32_t *state, int allow_tf32, void *workspace,
                        size_t workspace_bytes, sf_stream stream) {
    int st = check_matrix(x, "x");
    if (!st) st = check_matrix(W_enc, "W_enc");
    if (st) return st;
    const int64_t M = x->rows, K = x->cols, N = W_enc->cols;
    if (activation != SF_ACT_RELU && activation != SF_ACT_JUMPRELU)
        return set_error(SF_ERR_INVALID, "unknown activation code %d", activation);
    if (K != W_enc->rows)
        return set_error(SF_ERR_INVALID, "x has d_in=%lld but W_enc has d_in=%lld", (long long)K,
                         (long long)W_enc->rows);
    if (!valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad values dtype %d", values_dtype);
    st = check_vector(b_enc, N, "b_enc", false);
    if (!st) st = check_vector(b_dec, K, "b_dec", true);
    if (!st) st = check_vector(threshold, N, "threshold", activation != SF_ACT_JUMPRELU);
    if (st) return st;
    if (stage_capacity < 0 || stage_capacity > 2147483647ll)
        return set_error(SF_ERR_INVALID, "stage_capacity must be in [0, 2^31)");
    if (M == 0 || N == 0) return SF_OK;
    if (!tile_counts || !tile_offsets || !state || (stage_capacity > 0 && (!stage_indices || !stage_values)))
        return set_error(SF_ERR_INVALID, "NULL staging pointer");
    EncodePlan pl;
    st = plan_encode(x, W_enc, allow_tf32, SF_VARIANT_AUTO, &pl);
    if (st) return st;
    const size_t need = plan_workspace(pl);
    if (workspace_bytes < need || (!workspace && need))
        return set_error(SF_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    if (!aligned16(workspace)) return set_error(SF_ERR_WORKSPACE, "workspace must be 16-byte aligned");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    EpilogueArgs ep{};
    ep.b_enc = b_enc->data;
    ep.b_enc_dtype = b_enc->dtype;
    ep.b_enc_stride = b_enc->stride;
    if (threshold && threshold->data) {
        ep.thr = threshold->data;
        ep.thr_dtype = threshold->dtype;
        ep.thr_stride = threshold->stride;
    }
    ep.activation = activation;
    ep.out_dtype = values_dtype;
    ep.row_nnz = row_nnz;
    CsrArgs csr{tile_counts, tile_offsets, stage_indices, stage_values, state, (unsigned)stage_capacity};
    if (!pl.tensor_cores) {
        // the CUDA-core IEEE encoder with the same CSR staging epilogue
        st = run_shift_convert(x, b_dec, pl.mma_dtype, ws, pl.a_pitch, s);
        if (st) return st;
        return encode_simt_f32(reinterpret_cast<const float *>(ws), pl.a_pitch,
                               static_cast<const float *>(W_enc->data), W_enc->stride_row, W_enc->stride_col, M, N,
                               K, ep, s, &csr);
    }
    if (pl.emulate) {
        st = run_emulated(pl, x, W_enc, b_dec, b_enc, ws, SF_VARIANT_AUTO, s,
                          [&](const GemmOperands &g, const float *part, int64_t pitch) {
                              EpilogueArgs e = ep;
                              e.c_in = part;
                              e.c_in_pitch = pitch;
                              return encode_tc_csr(g, e, csr, s);
                          });
        if (st) return st;
        return run_emu_fallback(pl, x, W_enc, b_dec, ws, ep, &csr, s);
    }
    GemmOperands g;
    st = prepare_tc(pl, x, W_enc, b_dec, ws, s, g);
    if (st) return st;
    return encode_tc_csr(g, ep, csr, s);
}

int sf_csr_place(const int32_t *tile_counts, const int32_t *tile_offsets, int64_t M, int64_t d_sae,
                 const int32_t *stage_indices, const void *stage_values, int64_t stage_capacity, int values_dtype,
                 const int64_t *indptr, int32_t *indices, void *values, sf_stream stream) {
    if (M < 0 || d_sae < 0 || stage_capacity < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (!valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad values dtype %d", values_dtype);
    if (M == 0) return SF_OK;
    if (!tile_counts || !tile_offsets || !indptr) return set_error(SF_ERR_INVALID, "NULL pointer");
    const int64_t n_tiles = (d_sae + kCsrTile - 1) / kCsrTile;
    return launch_csr_place(tile_counts, tile_offsets, n_tiles, stage_indices, stage_values, stage_capacity,
                            values_dtype, indptr, M, indices, values, reinterpret_cast<cudaStream_t>(stream));
}

int sf_csr_finish_async(const int32_t *row_nnz, const int32_t *tile_counts, const int32_t *tile_offsets, int64_t M,
                        int64_t d_sae, const int32_t *stage_indices, const void *stage_values,
                        int64_t stage_capacity, int values_dtype, const uint32_t *state, int64_t *indptr,
                        int32_t *indices, void *values, sf_stream stream) {
    if (M < 0 || d_sae < 0 || stage_capacity < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (!valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad values dtype %d", values_dtype);
    if (!indptr || !state) return set_error(SF_ERR_INVALID, "NULL pointer");
    if (M > 0 && (!row_nnz || !tile_counts || !tile_offsets))
        return set_error(SF_ERR_INVALID, "NULL pointer");
    if (stage_capacity > 0 && (!stage_indices || !stage_values || !indices || !values))
        return set_error(SF_ERR_INVALID, "NULL staging or output pointer");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const unsigned *overflow = reinterpret_cast<const unsigned *>(state) + 1;
    int st = launch_indptr(row_nnz, M, indptr, s, overflow);
    if (st || M == 0) return st;
    const int64_t n_tiles = (d_sae + kCsrTile - 1) / kCsrTile;
    return launch_csr_place(tile_counts, tile_offsets, n_tiles, stage_indices, stage_values, stage_capacity,
                            values_dtype, indptr, M, indices, values, s, overflow);
}

int sf_row_nnz(const sf_matrix *f, int32_t *row_nnz, sf_stream stream) {
    int st = check_matrix(f, "f");
    if (st) return st;
    if (f->rows > 0 && !row_nnz) return set_error(SF_ERR_INVALID, "row_nnz is NULL");
    if (f->cols == 0) {
        if (f->rows) {
            st = check_cuda(cudaMemsetAsync(row_nnz, 0, (size_t)f->rows * 4, reinterpret_cast<cudaStream_t>(stream)),
                            "memset row_nnz");
        }
        return st;
    }
    return launch_row_nnz(*f, row_nnz, reinterpret_cast<cudaStream_t>(stream));
}

int sf_csr_indptr(const int32_t *row_nnz, int64_t M, int64_t *indptr, sf_stream stream) {
    if (M < 0) return set_error(SF_ERR_INVALID, "M is negative");
    if (!indptr || (M > 0 && !row_nnz)) return set_error(SF_ERR_INVALID, "NULL pointer");
    return launch_indptr(row_nnz, M, indptr, reinterpret_cast<cudaStream_t>(stream));
}

int sf_dense_to_csr(const sf_matrix *f, const int64_t *indptr, int32_t *indices, void *values, int values_dtype,
                    sf_stream stream) {
    int st = check_matrix(f, "f");
    if (st) return st;
    if (!valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad values dtype %d", values_dtype);
    if (f->rows > 0 && !indptr) return set_error(SF_ERR_INVALID, "indptr is NULL");
    if (f->rows == 0 || f->cols == 0) return SF_OK;
    return launch_compact(*f, indptr, indices, values, values_dtype, reinterpret_cast<cudaStream_t>(stream));
}

int sf_sparse_decode(const int64_t *indptr, int64_t M, const int32_t *indices, const void *values, int values_dtype,
                     const sf_matrix *W_dec, const sf_vector *b_dec, const sf_matrix *out, sf_stream stream) {
    int st = check_matrix(W_dec, "W_dec");
    if (!st) st = check_matrix(out, "out");
    if (st) return st;
    if (M < 0) return set_error(SF_ERR_INVALID, "M is negative");
    if (!valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad values dtype %d", values_dtype);
    if (out->rows != M || out->cols != W_dec->cols)
        return set_error(SF_ERR_INVALID, "out must be [%lld, %lld]", (long long)M, (long long)W_dec->cols);
    st = check_vector(b_dec, W_dec->cols, "b_dec", true);
    if (st) return st;
    if (M > 0 && !indptr) return set_error(SF_ERR_INVALID, "indptr is NULL");
    const sf_vector *b = (b_dec && b_dec->data) ? b_dec : nullptr;
    return launch_decode(indptr, M, indices, values, values_dtype, *W_dec, b, *out,
                         reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace sf {
namespace {

constexpr int kTopkDenseMaxK = 200;         // shared-memory bound of topk_rows_kernel
constexpr int64_t kTopkDenseChunk = 256ll << 20;  // bytes of dense features per row chunk

// The fused epilogue selects on tensor-core products: 16-bit operands, or fp32 with TF32
// allowed (or non-fp32 x, the reference's own rule, encode.py:118-120). fp32 with IEEE
// products, and k beyond the epilogue's limit, take the dense route: encode a chunk of
// rows (CUDA-core kernel for IEEE fp32), then select per row from the stored values.
bool topk_fused(const sf_matrix *x, const sf_matrix *W, int k, int allow_tf32) {
    if (k > kTopkMaxK) return false;
    if (W->dtype != SF_F32) return true;
    return allow_tf32 || x->dtype != SF_F32;
}

int64_t topk_chunk_rows(const sf_matrix *x, const sf_matrix *W) {
    const int64_t per_row = W->cols * (int64_t)dtype_size(x->dtype);
    int64_t r = kTopkDenseChunk / (per_row > 0 ? per_row : 1);
    if (r < 1) r = 1;
    return r < x->rows ? r : x->rows;
}

// Rows per launch of the fused top-k encoder. Measured on B200 at config 4 (32768 x 4096 ->
// 131072, k = 32, at the 1000 W power cap): the same tokens through 8192-row launches ran
// faster than through one launch of every row, and the W_enc re-read each launch costs
// (1 GB, ~0.15 ms) is small beside ~8 ms of GEMM. 0: one launch.
#ifndef SF_TOPK_LAUNCH_ROWS
#define SF_TOPK_LAUNCH_ROWS 8192
#endif
int64_t topk_launch_rows(int64_t M) {
    return (SF_TOPK_LAUNCH_ROWS > 0 && M > SF_TOPK_LAUNCH_ROWS) ? (int64_t)SF_TOPK_LAUNCH_ROWS : M;
}

// Workspace of one fused top-k launch over `rows` rows of x: the encoder's plan, then the
// candidate lists [rows, chunks, k].
int topk_launch_workspace(const sf_matrix *x, const sf_matrix *W, int k, int64_t rows, size_t *bytes) {
    sf_matrix xr = *x;
    xr.rows = rows;
    EncodePlan pl;
    int st = plan_encode(&xr, W, 1, SF_VARIANT_TCGEN05, &pl);
    if (st) return st;
    const int chunks = topk_chunks(rows, W->cols);
    *bytes = (size_t)round_up((int64_t)plan_workspace(pl), 256) +
             (size_t)rows * chunks * k * sizeof(unsigned long long);
    return SF_OK;
}

int topk_workspace(const sf_matrix *x, const sf_matrix *W, int k, int allow_tf32, size_t *bytes) {
    if (topk_fused(x, W, k, allow_tf32)) {
        // the largest of a full launch and the last, shorter one
        const int64_t R = topk_launch_rows(x->rows), tail = R > 0 ? x->rows % R : 0;
        int st = topk_launch_workspace(x, W, k, R, bytes);
        if (st || tail == 0) return st;
        size_t t = 0;
        st = topk_launch_workspace(x, W, k, tail, &t);
        if (t > *bytes) *bytes = t;
        return st;
    }
    if (k > kTopkDenseMaxK) return set_error(SF_ERR_UNSUPPORTED, "top-k supports k <= %d", kTopkDenseMaxK);
    sf_matrix xr = *x;
    xr.rows = topk_chunk_rows(x, W);
    size_t enc = 0;
    int st = sf_fused_encode_workspace(&xr, W, allow_tf32, SF_VARIANT_AUTO, &enc);
    if (st) return st;
    *bytes = (size_t)round_up((int64_t)enc, 256) + (size_t)xr.rows * W->cols * dtype_size(x->dtype);
    return SF_OK;
}

}  // namespace
}  // namespace sf

extern "C" {

int sf_topk_encode_workspace(const sf_matrix *x, const sf_matrix *W_enc, int k, int allow_tf32, size_t *bytes) {
    if (!bytes) return set_error(SF_ERR_INVALID, "bytes is NULL");
    *bytes = 0;
    int st = check_matrix(x, "x");
    if (!st) st = check_matrix(W_enc, "W_enc");
    if (st) return st;
    if (x->cols != W_enc->rows)
        return set_error(SF_ERR_INVALID, "x has d_in=%lld but W_enc has d_in=%lld", (long long)x->cols,
                         (long long)W_enc->rows);
    if (k < 1 || k > W_enc->cols)
        return set_error(SF_ERR_INVALID, "k=%d must be in [1, d_sae=%lld]", k, (long long)W_enc->cols);
    return topk_workspace(x, W_enc, k, allow_tf32, bytes);
}

int sf_topk_encode(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc, const sf_vector *b_dec, int k,
                   int32_t *indices, void *values, int values_dtype, int allow_tf32, void *workspace,
                   size_t workspace_bytes, sf_stream stream) {
    int st = check_matrix(x, "x");
    if (!st) st = check_matrix(W_enc, "W_enc");
    if (st) return st;
    const int64_t M = x->rows, K = x->cols, N = W_enc->cols;
    if (K != W_enc->rows)
        return set_error(SF_ERR_INVALID, "x has d_in=%lld but W_enc has d_in=%lld", (long long)K,
                         (long long)W_enc->rows);
    if (k < 1 || k > N) return set_error(SF_ERR_INVALID, "k=%d must be in [1, d_sae=%lld]", k, (long long)N);
    if (!valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad values dtype %d", values_dtype);
    st = check_vector(b_enc, N, "b_enc", false);
    if (!st) st = check_vector(b_dec, K, "b_dec", true);
    if (st) return st;
    if (M == 0) return SF_OK;
    if (!indices || !values) return set_error(SF_ERR_INVALID, "indices/values are NULL");
    size_t need = 0;
    st = topk_workspace(x, W_enc, k, allow_tf32, &need);
    if (st) return st;
    if (workspace_bytes < need || !workspace)
        return set_error(SF_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    if (!aligned16(workspace)) return set_error(SF_ERR_WORKSPACE, "workspace must be 16-byte aligned");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);

    if (!topk_fused(x, W_enc, k, allow_tf32)) {
        // Dense route: the stored ReLU output (in the values dtype, as the reference's
        // fused_encode(..., "relu") stores it in x's dtype) is selected row by row.
        const int64_t R = topk_chunk_rows(x, W_enc);
        sf_matrix xr = *x;
        xr.rows = R;
        size_t enc = 0;
        st = sf_fused_encode_workspace(&xr, W_enc, allow_tf32, SF_VARIANT_AUTO, &enc);
        if (st) return st;
        uint8_t *fbuf = ws + round_up((int64_t)enc, 256);
        const size_t xes = dtype_size(x->dtype), ves = dtype_size(values_dtype);
        for (int64_t r0 = 0; r0 < M; r0 += R) {
            const int64_t rr = (M - r0) < R ? (M - r0) : R;
            xr.data = static_cast<const uint8_t *>(x->data) + r0 * x->stride_row * (int64_t)xes;
            xr.rows = rr;
            sf_matrix fr{fbuf, values_dtype, 0, rr, N, N, 1};
            st = sf_fused_encode(&xr, W_enc, b_enc, b_dec, nullptr, SF_ACT_RELU, &fr, nullptr, allow_tf32,
                                 SF_VARIANT_AUTO, ws, enc, stream);
            if (st) return st;
            st = launch_topk_rows(fr, k, indices + r0 * k, static_cast<uint8_t *>(values) + r0 * k * (int64_t)ves,
                                  values_dtype, s);
            if (st) return st;
        }
        return SF_OK;
    }

    // Launches of at most topk_launch_rows rows, each with its own candidate lists and merge.
    const int64_t R = topk_launch_rows(M);
    const size_t xes = dtype_size(x->dtype), ves = dtype_size(values_dtype);
    for (int64_t r0 = 0; r0 < M; r0 += R) {
        sf_matrix xr = *x;
        xr.data = static_cast<const uint8_t *>(x->data) + r0 * x->stride_row * (int64_t)xes;
        xr.rows = (M - r0) < R ? (M - r0) : R;
        EncodePlan pl;
        st = plan_encode(&xr, W_enc, 1, SF_VARIANT_TCGEN05, &pl);
        if (st) return st;
        const int chunks = topk_chunks(xr.rows, N);
        const size_t cand_off = (size_t)round_up((int64_t)plan_workspace(pl), 256);
        auto *cand = reinterpret_cast<unsigned long long *>(ws + cand_off);
        GemmOperands g;
        st = prepare_tc(pl, &xr, W_enc, b_dec, ws, s, g);
        if (st) return st;
        TopkArgs tk{};
        tk.b_enc = b_enc->data;
        tk.b_enc_dtype = b_enc->dtype;
        tk.b_enc_stride = b_enc->stride;
        tk.k = k;
        tk.values_dtype = values_dtype;
        tk.n_chunks = chunks;
        tk.cand = cand;
        st = encode_tc_topk(g, tk, s);
        if (st) return st;
        st = launch_topk_merge(cand, xr.rows, chunks * k, k, indices + r0 * k,
                               static_cast<uint8_t *>(values) + r0 * k * (int64_t)ves, values_dtype, s);
        if (st) return st;
    }
    return SF_OK;
}

}  // extern "C"
