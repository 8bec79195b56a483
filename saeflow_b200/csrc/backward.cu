// Backward of the sparse SAE forward, for training on sparse features (saeflow's roadmap,
// README.md:244; the reference itself has no backward kernels).
//
//   forward:  pre = (x - b_dec) @ W_enc + b_enc ; f = act(pre) as CSR ; x_hat = f @ W_dec + b_dec
//   backward, given g = dL/dx_hat [M, d_in]:
//     dpre[e]  = g[row(e)] . W_dec[col(e)]            for each CSR entry e with f_e != 0   (sddmm)
//     dW_dec[j] = sum_{e in column j} f_e * g[row(e)]                                        (csc accumulate)
//     dW_enc^T[j] = sum_{e in column j} dpre_e * xs[row(e)],   db_enc[j] = sum dpre_e        (csc accumulate)
//     dx = dpre @ W_enc^T (a CSR decode against W_enc^T),       db_dec = sum_m (g[m] - dx[m])
// The gradient reaches only the active features: ReLU and JumpReLU pass it where f != 0,
// TopK where a selected value is positive. (The JumpReLU threshold gets none here.)
//
// Column-wise work needs the CSR transposed: a column count (atomics), the indptr scan of
// sparse.cu, and a scatter that records each entry's row and its CSR position. The scatter's
// order within a column depends on atomic timing, so the per-column sums accumulate in fp64:
// rounding the fp64 sum to fp32 makes the result independent of that order (barring a sum
// within one fp64 ulp of an fp32 rounding boundary).
#include <algorithm>

#include "sf_common.cuh"
#include "sf_internal.h"

namespace sf {

int launch_indptr(const int32_t *cnt, int64_t M, int64_t *indptr, cudaStream_t s, const unsigned *skip);

namespace {

// ------------------------------------------------------------------ CSR -> CSC
__global__ void csr_col_count_kernel(const int32_t *__restrict__ indices, int64_t nnz, int64_t n_cols,
                                     int32_t *__restrict__ cnt, unsigned *err) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz; e += (int64_t)gridDim.x * blockDim.x) {
        const int32_t j = indices[e];
        if (j < 0 || (int64_t)j >= n_cols) {
            atomicOr(err, kErrIndex);
            continue;
        }
        atomicAdd(cnt + j, 1);
    }
}

// One warp per CSR row: each entry takes the next slot of its column.
__global__ void csr_to_csc_kernel(const int64_t *__restrict__ indptr, int64_t M, const int32_t *__restrict__ indices,
                                  int64_t n_cols, const int64_t *__restrict__ col_ptr, int32_t *__restrict__ cursor,
                                  int32_t *__restrict__ row_idx, int64_t *__restrict__ perm) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = lane_id();
    const int64_t start = indptr[row], end = indptr[row + 1];
    for (int64_t e = start + lane; e < end; e += 32) {
        const int32_t j = indices[e];
        if (j < 0 || (int64_t)j >= n_cols) continue;  // reported by the count kernel
        const int64_t pos = col_ptr[j] + atomicAdd(cursor + j, 1);
        if (pos < col_ptr[j + 1]) {
            row_idx[pos] = (int32_t)row;
            perm[pos] = e;
        }
    }
}

// Column order for the accumulation: columns with more than kHotEntries entries first (they
// are the long-running warps; started last they would form the kernel's tail), the rest after.
constexpr int64_t kHotEntries = 256;
__global__ void csc_order_kernel(const int64_t *__restrict__ col_ptr, int64_t n_cols, int32_t *__restrict__ order,
                                 int32_t *__restrict__ counters) {
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n_cols; j += (int64_t)gridDim.x * blockDim.x) {
        const bool hot = col_ptr[j + 1] - col_ptr[j] > kHotEntries;
        const int64_t pos = hot ? atomicAdd(counters, 1) : n_cols - 1 - atomicAdd(counters + 1, 1);
        order[pos] = (int32_t)j;
    }
}

__global__ void csc_hot_count_kernel(const int32_t *__restrict__ counters, int32_t *__restrict__ order,
                                     int64_t n_cols) {
    order[n_cols] = counters[0];
}

// ------------------------------------------------------------------ per-column accumulation
// out[j, d] = sum_{p in column j} values[perm[p]] * R[row_idx[p], d]; col_sums[j] = sum values.
// Work items (one warp each): a light column (<= kHotEntries entries) is one item over the
// whole row width, holding its (row, value) pairs in registers across the D-slices; a hot
// column is split into one item per 32x16-byte D-slice so several warps share it. Hot items
// come first (col_order from sf_csr_transpose lists hot columns first and stores their count
// after the n_cols entries). Rows are gathered as coalesced 16-byte segments, kInflight at a
// time; sums in fp64.
constexpr int kInflight = 4;
#ifdef SF_ACC_FP32
using AccT = float;
#else
using AccT = double;
#endif
constexpr int kLightChunks = (int)(kHotEntries / 32);

template <typename RT>
__device__ __forceinline__ void gather_rows(const RT *__restrict__ R, int64_t ldr, int64_t dl, int64_t D, int vec,
                                            int my_row, float my_val, int n, AccT (&acc)[16 / sizeof(RT)]) {
    constexpr int EPV = 16 / sizeof(RT);
    int t = 0;
    if (vec) {  // D % EPV == 0: a lane's vector is wholly inside the row or wholly past it
        const bool in = dl < D;
        for (; t + kInflight <= n; t += kInflight) {
            uint4 u[kInflight];
            AccT a[kInflight];
#pragma unroll
            for (int i = 0; i < kInflight; ++i) {
                const int r = __shfl_sync(0xffffffffu, my_row, t + i);
                a[i] = (AccT)__shfl_sync(0xffffffffu, my_val, t + i);
                u[i] = in ? __ldg(reinterpret_cast<const uint4 *>(R + (int64_t)r * ldr + dl)) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int i = 0; i < kInflight; ++i) {
                const RT *el = reinterpret_cast<const RT *>(&u[i]);
#pragma unroll
                for (int e = 0; e < EPV; ++e) acc[e] += a[i] * (AccT)to_f32(el[e]);
            }
        }
        for (; t < n; ++t) {
            const int r = __shfl_sync(0xffffffffu, my_row, t);
            const AccT a = (AccT)__shfl_sync(0xffffffffu, my_val, t);
            if (in) {
                const uint4 u = __ldg(reinterpret_cast<const uint4 *>(R + (int64_t)r * ldr + dl));
                const RT *el = reinterpret_cast<const RT *>(&u);
#pragma unroll
                for (int e = 0; e < EPV; ++e) acc[e] += a * (AccT)to_f32(el[e]);
            }
        }
        return;
    }
    for (; t < n; ++t) {
        const int r = __shfl_sync(0xffffffffu, my_row, t);
        const AccT a = (AccT)__shfl_sync(0xffffffffu, my_val, t);
        const RT *src = R + (int64_t)r * ldr;
#pragma unroll
        for (int e = 0; e < EPV; ++e)
            if (dl + e < D) acc[e] += a * (AccT)to_f32(src[dl + e]);
    }
}

template <typename RT, typename VT>
__global__ void __launch_bounds__(128, 5) csc_accumulate_kernel(const int64_t *__restrict__ col_ptr, int64_t n_cols,
                                                                const int32_t *__restrict__ order,
                                                                const int32_t *__restrict__ row_idx,
                                                                const int64_t *__restrict__ perm,
                                                                const VT *__restrict__ values,
                                                                const RT *__restrict__ R, int64_t ldr, int64_t M,
                                                                int64_t D, float *__restrict__ out, int64_t ldo,
                                                                float *__restrict__ col_sums, int vec, unsigned *err) {
    constexpr int EPV = 16 / sizeof(RT);
    constexpr int SLICE = 32 * EPV;
    const int64_t n_slices = (D + SLICE - 1) / SLICE;
    const int64_t w = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int64_t n_hot = order != nullptr ? (int64_t)order[n_cols] : 0;
    int64_t col, s_first, s_last;
    if (w < n_hot * n_slices) {
        col = order[w / n_slices];
        s_first = w % n_slices;
        s_last = s_first + 1;
    } else {
        const int64_t li = w - n_hot * n_slices;
        if (li >= n_cols - n_hot) return;
        col = order != nullptr ? (int64_t)order[n_hot + li] : li;
        s_first = 0;
        s_last = n_slices;
    }
    const int lane = lane_id();
    const int64_t p0 = col_ptr[col], p1 = col_ptr[col + 1];
    bool bad = false;
    double vsum = 0.0;
    auto entry = [&](int64_t q, int &r, float &v) {
        r = 0;
        v = 0.f;
        if (q < p1) {
            r = row_idx[q];
            v = to_f32(values[perm[q]]);
            if (r < 0 || (int64_t)r >= M) {
                bad = true;
                r = 0;
                v = 0.f;
            }
        }
    };
    auto store = [&](int64_t s, const AccT(&acc)[EPV]) {
        const int64_t dl = s * SLICE + (int64_t)lane * EPV;
#pragma unroll
        for (int e = 0; e < EPV; ++e)
            if (dl + e < D) out[col * ldo + dl + e] = (float)acc[e];
    };

    if (p1 - p0 <= kHotEntries) {
        // Light column: its (row, value) pairs stay in registers across the slices.
        int rows[kLightChunks];
        float vals[kLightChunks];
#pragma unroll
        for (int c = 0; c < kLightChunks; ++c) {
            entry(p0 + c * 32 + lane, rows[c], vals[c]);
            vsum += (double)vals[c];
        }
        for (int64_t s = s_first; s < s_last; ++s) {
            AccT acc[EPV];
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[e] = 0.0;
            const int64_t dl = s * SLICE + (int64_t)lane * EPV;
#pragma unroll
            for (int c = 0; c < kLightChunks; ++c) {
                const int64_t left = p1 - p0 - c * 32;
                if (left > 0) gather_rows<RT>(R, ldr, dl, D, vec, rows[c], vals[c], left < 32 ? (int)left : 32, acc);
            }
            store(s, acc);
        }
    } else {
        for (int64_t s = s_first; s < s_last; ++s) {
            AccT acc[EPV];
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[e] = 0.0;
            const int64_t dl = s * SLICE + (int64_t)lane * EPV;
            for (int64_t q0 = p0; q0 < p1; q0 += 32) {
                int r;
                float v;
                entry(q0 + lane, r, v);
                if (s == 0) vsum += (double)v;
                const int64_t left = p1 - q0;
                gather_rows<RT>(R, ldr, dl, D, vec, r, v, left < 32 ? (int)left : 32, acc);
            }
            store(s, acc);
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(err, kErrIndex);
    if (col_sums != nullptr && s_first == 0) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) vsum += __shfl_xor_sync(0xffffffffu, vsum, off);
        if (lane == 0) col_sums[col] = (float)vsum;
    }
}

// ------------------------------------------------------------------ sampled dot products
// out[e] = (values[e] != 0) * sum_d G[row(e), d] * W[indices[e], d], one warp per CSR row:
// the row of G stays in L1 while the warp walks the row's entries, each W row read as
// coalesced 16-byte segments; fp32 accumulation, warp-shuffle reduction.
template <typename T, typename VT>
__global__ void __launch_bounds__(128) csr_sddmm_kernel(const int64_t *__restrict__ indptr, int64_t M,
                                                        const int32_t *__restrict__ indices, int64_t n_cols,
                                                        const T *__restrict__ G, int64_t ldg,
                                                        const T *__restrict__ W, int64_t ldw, int64_t D,
                                                        const VT *__restrict__ values, float *__restrict__ out,
                                                        int vec, unsigned *err) {
    constexpr int EPV = 16 / sizeof(T);
    const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = lane_id();
    const int64_t start = indptr[row], end = indptr[row + 1];
    const T *g = G + row * ldg;
    bool bad = false;
    for (int64_t e = start; e < end; ++e) {
        const int32_t j = indices[e];
        if (j < 0 || (int64_t)j >= n_cols) {
            bad = true;
            if (lane == 0) out[e] = 0.f;
            continue;
        }
        const T *w = W + (int64_t)j * ldw;
        float s = 0.f;
        if (vec) {
            for (int64_t d = (int64_t)lane * EPV; d < D; d += 32 * EPV) {
                const uint4 ug = __ldg(reinterpret_cast<const uint4 *>(g + d));
                const uint4 uw = __ldg(reinterpret_cast<const uint4 *>(w + d));
                const T *eg = reinterpret_cast<const T *>(&ug);
                const T *ew = reinterpret_cast<const T *>(&uw);
#pragma unroll
                for (int k = 0; k < EPV; ++k) s = fmaf(to_f32(eg[k]), to_f32(ew[k]), s);
            }
        } else {
            for (int64_t d = lane; d < D; d += 32) s = fmaf(to_f32(g[d]), to_f32(w[d]), s);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) out[e] = (to_f32(values[e]) != 0.f) ? s : 0.f;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(err, kErrIndex);
}

// ------------------------------------------------------------------ transpose + convert
// out[j, i] = in[i, j] converted to out's dtype, through 32 x 33 shared-memory tiles so both the
// reads and the writes are row-contiguous (W_enc -> W_enc^T for dx, dW_enc^T -> dW_enc).
template <typename IT, typename OT>
__global__ void __launch_bounds__(256) transpose_kernel(const IT *__restrict__ in, int64_t rows, int64_t cols,
                                                        int64_t ldi, OT *__restrict__ out, int64_t ldo) {
    __shared__ float tile[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int64_t r = r0 + ty + k, c = c0 + tx;
        tile[ty + k][tx] = (r < rows && c < cols) ? to_f32(in[r * ldi + c]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int64_t oc = r0 + tx, orow = c0 + ty + k;  // out is [cols, rows]
        if (orow < cols && oc < rows) out[orow * ldo + oc] = from_f32<OT>(tile[tx][ty + k]);
    }
}

template <typename F>
int by_dtype(int dt, F &&f) {
    if (dt == SF_F32) return f(float{});
    if (dt == SF_BF16) return f(__nv_bfloat16{});
    return f(__half{});
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

int sf_csr_transpose_workspace(int64_t n_cols, size_t *bytes) {
    if (!bytes) return set_error(SF_ERR_INVALID, "bytes is NULL");
    if (n_cols < 0) return set_error(SF_ERR_INVALID, "n_cols is negative");
    *bytes = (size_t)(2 * n_cols + 64) * sizeof(int32_t);  // counts, cursors, two order counters
    return SF_OK;
}

int sf_csr_transpose(const int64_t *indptr, int64_t M, const int32_t *indices, int64_t nnz, int64_t n_cols,
                     int64_t *col_ptr, int32_t *row_idx, int64_t *perm, int32_t *col_order, void *workspace,
                     size_t workspace_bytes, sf_stream stream) {
    if (M < 0 || nnz < 0 || n_cols < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (n_cols > (int64_t)INT32_MAX) return set_error(SF_ERR_UNSUPPORTED, "n_cols exceeds 2^31-1");
    if (!col_ptr || (M > 0 && !indptr)) return set_error(SF_ERR_INVALID, "NULL pointer");
    if (nnz > 0 && (!indices || !row_idx || !perm)) return set_error(SF_ERR_INVALID, "NULL pointer");
    size_t need = 0;
    sf_csr_transpose_workspace(n_cols, &need);
    if (!workspace || workspace_bytes < need)
        return set_error(SF_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes, need);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t *cnt = static_cast<int32_t *>(workspace);
    int32_t *cursor = cnt + n_cols;
    int32_t *order_counters = cursor + n_cols;
    int st = check_cuda(cudaMemsetAsync(cnt, 0, (size_t)(2 * n_cols + 2) * sizeof(int32_t), s), "memset counts");
    if (st) return st;
    if (nnz > 0) {
        const unsigned blocks = (unsigned)std::min<int64_t>((nnz + 255) / 256, 4096);
        csr_col_count_kernel<<<blocks, 256, 0, s>>>(indices, nnz, n_cols, cnt, device_error_word());
        st = check_cuda(cudaGetLastError(), "column count launch");
        if (st) return st;
    }
    st = launch_indptr(cnt, n_cols, col_ptr, s, nullptr);
    if (st) return st;
    if (col_order != nullptr && n_cols > 0) {
        const unsigned blocks = (unsigned)std::min<int64_t>((n_cols + 255) / 256, 4096);
        csc_order_kernel<<<blocks, 256, 0, s>>>(col_ptr, n_cols, col_order, order_counters);
        csc_hot_count_kernel<<<1, 1, 0, s>>>(order_counters, col_order, n_cols);
        st = check_cuda(cudaGetLastError(), "column order launch");
        if (st) return st;
    }
    if (M == 0 || nnz == 0) return st;
    csr_to_csc_kernel<<<(unsigned)((M + 7) / 8), 256, 0, s>>>(indptr, M, indices, n_cols, col_ptr, cursor, row_idx,
                                                               perm);
    return check_cuda(cudaGetLastError(), "csc scatter launch");
}

int sf_csc_accumulate(const int64_t *col_ptr, int64_t n_cols, const int32_t *col_order, int64_t nnz,
                      const int32_t *row_idx, const int64_t *perm, const void *values, int values_dtype,
                      const sf_matrix *R, float *out, int64_t ld_out, float *col_sums, sf_stream stream) {
    if (!R) return set_error(SF_ERR_INVALID, "R is NULL");
    if (!valid_dtype(R->dtype) || !valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad dtype");
    if (n_cols < 0 || nnz < 0 || R->rows < 0 || R->cols < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (n_cols == 0 || R->cols == 0) return SF_OK;
    if (!col_ptr || !out || ld_out < R->cols) return set_error(SF_ERR_INVALID, "bad output or col_ptr");
    if (nnz > 0 && (!row_idx || !perm || !values)) return set_error(SF_ERR_INVALID, "NULL entry arrays");
    if (R->stride_col != 1) return set_error(SF_ERR_UNSUPPORTED, "R must have unit column stride");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t D = R->cols;
    return by_dtype(R->dtype, [&](auto rtag) {
        using RT = decltype(rtag);
        constexpr int EPV = 16 / sizeof(RT);
        const int vec =
            (aligned16(R->data) && (R->stride_row * (int64_t)sizeof(RT)) % 16 == 0 && D % EPV == 0) ? 1 : 0;
        const int64_t n_slices = (D + 32 * EPV - 1) / (32 * EPV);
        // Work items: light columns one each, hot columns one per slice; at most nnz / 257
        // columns can be hot.
        const int64_t hot_max = col_order ? std::min<int64_t>(n_cols, nnz / (kHotEntries + 1)) : 0;
        const int64_t items = n_cols + hot_max * (n_slices - 1);
        if ((items + 3) / 4 > (int64_t)INT32_MAX) return set_error(SF_ERR_UNSUPPORTED, "too many columns");
        return by_dtype(values_dtype, [&](auto vtag) {
            using VT = decltype(vtag);
            csc_accumulate_kernel<RT, VT><<<(unsigned)((items + 3) / 4), 128, 0, s>>>(
                col_ptr, n_cols, col_order, row_idx, perm, reinterpret_cast<const VT *>(values),
                reinterpret_cast<const RT *>(R->data), R->stride_row, R->rows, D, out, ld_out, col_sums, vec,
                device_error_word());
            return check_cuda(cudaGetLastError(), "csc accumulate launch");
        });
    });
}

int sf_transpose(const sf_matrix *in, const sf_matrix *out, sf_stream stream) {
    if (!in || !out) return set_error(SF_ERR_INVALID, "NULL matrix");
    if (!valid_dtype(in->dtype) || !valid_dtype(out->dtype)) return set_error(SF_ERR_INVALID, "bad dtype");
    if (out->rows != in->cols || out->cols != in->rows)
        return set_error(SF_ERR_INVALID, "out must be [%lld, %lld]", (long long)in->cols, (long long)in->rows);
    if (in->stride_col != 1 || out->stride_col != 1) return set_error(SF_ERR_UNSUPPORTED, "unit column strides required");
    if (in->rows == 0 || in->cols == 0) return SF_OK;
    if ((in->cols + 31) / 32 > (int64_t)INT32_MAX || (in->rows + 31) / 32 > 65535)
        return set_error(SF_ERR_UNSUPPORTED, "transpose grid too large");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    dim3 grid((unsigned)((in->cols + 31) / 32), (unsigned)((in->rows + 31) / 32));
    return by_dtype(in->dtype, [&](auto itag) {
        using IT = decltype(itag);
        return by_dtype(out->dtype, [&](auto otag) {
            using OT = decltype(otag);
            transpose_kernel<IT, OT><<<grid, 256, 0, s>>>(reinterpret_cast<const IT *>(in->data), in->rows, in->cols,
                                                          in->stride_row,
                                                          reinterpret_cast<OT *>(const_cast<void *>(out->data)),
                                                          out->stride_row);
            return check_cuda(cudaGetLastError(), "transpose launch");
        });
    });
}

int sf_csr_sddmm(const int64_t *indptr, int64_t M, const int32_t *indices, const sf_matrix *G, const sf_matrix *W,
                 const void *values, int values_dtype, float *out, sf_stream stream) {
    if (!G || !W) return set_error(SF_ERR_INVALID, "G and W are required");
    if (!valid_dtype(G->dtype) || !valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad dtype");
    if (G->dtype != W->dtype) return set_error(SF_ERR_UNSUPPORTED, "G and W must have one dtype");
    if (M < 0 || G->rows != M || G->cols != W->cols)
        return set_error(SF_ERR_INVALID, "G must be [M, d_in] and W [d_sae, d_in]");
    if (G->stride_col != 1 || W->stride_col != 1) return set_error(SF_ERR_UNSUPPORTED, "unit column strides required");
    if (M == 0) return SF_OK;
    if (!indptr || !out) return set_error(SF_ERR_INVALID, "NULL pointer");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    return by_dtype(G->dtype, [&](auto tag) {
        using T = decltype(tag);
        const int64_t es = (int64_t)sizeof(T);
        const int vec = (aligned16(G->data) && aligned16(W->data) && (G->stride_row * es) % 16 == 0 &&
                         (W->stride_row * es) % 16 == 0 && (G->cols * es) % 16 == 0)
                            ? 1
                            : 0;
        return by_dtype(values_dtype, [&](auto vtag) {
            using VT = decltype(vtag);
            csr_sddmm_kernel<T, VT><<<(unsigned)((M + 3) / 4), 128, 0, s>>>(
                indptr, M, indices, W->rows, reinterpret_cast<const T *>(G->data), G->stride_row,
                reinterpret_cast<const T *>(W->data), W->stride_row, G->cols, reinterpret_cast<const VT *>(values),
                out, vec, device_error_word());
            return check_cuda(cudaGetLastError(), "sddmm launch");
        });
    });
}

}  // extern "C"
