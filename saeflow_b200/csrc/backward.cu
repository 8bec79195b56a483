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

// ------------------------------------------------------------------ per-column accumulation
// out[j, d] = sum_{p in column j} values[perm[p]] * R[row_idx[p], d]; col_sums[j] = sum values.
// One warp per (column, D-slice); lane l owns V 16-byte vectors at slice + (v*32 + l)*EPV, so
// each gathered row of R is read as coalesced 16-byte segments; fp64 accumulators.
template <typename RT, typename VT, int V>
__global__ void __launch_bounds__(128) csc_accumulate_kernel(const int64_t *__restrict__ col_ptr, int64_t n_cols,
                                                             const int32_t *__restrict__ row_idx,
                                                             const int64_t *__restrict__ perm,
                                                             const VT *__restrict__ values, const RT *__restrict__ R,
                                                             int64_t ldr, int64_t M, int64_t D, float *__restrict__ out,
                                                             int64_t ldo, float *__restrict__ col_sums, int vec,
                                                             unsigned *err) {
    constexpr int EPV = 16 / sizeof(RT);
    constexpr int SLICE = 32 * V * EPV;
    const int64_t col = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (col >= n_cols) return;
    const int lane = lane_id();
    const int64_t d0 = (int64_t)blockIdx.y * SLICE;
    const int64_t p0 = col_ptr[col], p1 = col_ptr[col + 1];

    double acc[V][EPV];
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[v][e] = 0.0;
    double vsum = 0.0;
    bool bad = false;

    for (int64_t q0 = p0; q0 < p1; q0 += 32) {
        const int64_t q = q0 + lane;
        int32_t my_row = 0;
        float my_val = 0.f;
        if (q < p1) {
            my_row = row_idx[q];
            my_val = to_f32(values[perm[q]]);
            if (my_row < 0 || (int64_t)my_row >= M) {
                bad = true;
                my_row = 0;
                my_val = 0.f;
            }
        }
        vsum += (double)my_val;
        const int n = (p1 - q0) < 32 ? (int)(p1 - q0) : 32;
        for (int t = 0; t < n; ++t) {
            const int r = __shfl_sync(0xffffffffu, my_row, t);
            const double a = (double)__shfl_sync(0xffffffffu, my_val, t);
            const RT *src = R + (int64_t)r * ldr + d0;
#pragma unroll
            for (int v = 0; v < V; ++v) {
                const int64_t d = (int64_t)(v * 32 + lane) * EPV;
                if (d0 + d >= D) continue;
                if (vec && d0 + d + EPV <= D) {
                    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(src + d));
                    const RT *el = reinterpret_cast<const RT *>(&u);
#pragma unroll
                    for (int e = 0; e < EPV; ++e) acc[v][e] += a * (double)to_f32(el[e]);
                } else {
#pragma unroll
                    for (int e = 0; e < EPV; ++e)
                        if (d0 + d + e < D) acc[v][e] += a * (double)to_f32(src[d + e]);
                }
            }
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(err, kErrIndex);
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const int64_t d = (int64_t)(v * 32 + lane) * EPV;
#pragma unroll
        for (int e = 0; e < EPV; ++e)
            if (d0 + d + e < D) out[col * ldo + d0 + d + e] = (float)acc[v][e];
    }
    if (col_sums != nullptr && blockIdx.y == 0) {
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

template <typename F>
int by_dtype(int dt, F &&f) {
    if (dt == SF_F32) return f(float{});
    if (dt == SF_BF16) return f(__nv_bfloat16{});
    return f(__half{});
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Bytes of the gathered matrix one accumulation slice may span over all rows (half the L2).
constexpr int64_t kAccL2Budget = 64ll << 20;

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

int sf_csr_transpose_workspace(int64_t n_cols, size_t *bytes) {
    if (!bytes) return set_error(SF_ERR_INVALID, "bytes is NULL");
    if (n_cols < 0) return set_error(SF_ERR_INVALID, "n_cols is negative");
    *bytes = (size_t)(2 * n_cols + 64) * sizeof(int32_t);
    return SF_OK;
}

int sf_csr_transpose(const int64_t *indptr, int64_t M, const int32_t *indices, int64_t nnz, int64_t n_cols,
                     int64_t *col_ptr, int32_t *row_idx, int64_t *perm, void *workspace, size_t workspace_bytes,
                     sf_stream stream) {
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
    int st = check_cuda(cudaMemsetAsync(cnt, 0, (size_t)2 * n_cols * sizeof(int32_t), s), "memset counts");
    if (st) return st;
    if (nnz > 0) {
        const unsigned blocks = (unsigned)std::min<int64_t>((nnz + 255) / 256, 4096);
        csr_col_count_kernel<<<blocks, 256, 0, s>>>(indices, nnz, n_cols, cnt, device_error_word());
        st = check_cuda(cudaGetLastError(), "column count launch");
        if (st) return st;
    }
    st = launch_indptr(cnt, n_cols, col_ptr, s, nullptr);
    if (st || M == 0 || nnz == 0) return st;
    csr_to_csc_kernel<<<(unsigned)((M + 7) / 8), 256, 0, s>>>(indptr, M, indices, n_cols, col_ptr, cursor, row_idx,
                                                               perm);
    return check_cuda(cudaGetLastError(), "csc scatter launch");
}

int sf_csc_accumulate(const int64_t *col_ptr, int64_t n_cols, const int32_t *row_idx, const int64_t *perm,
                      const void *values, int values_dtype, const sf_matrix *R, float *out, int64_t ld_out,
                      float *col_sums, sf_stream stream) {
    if (!R) return set_error(SF_ERR_INVALID, "R is NULL");
    if (!valid_dtype(R->dtype) || !valid_dtype(values_dtype)) return set_error(SF_ERR_INVALID, "bad dtype");
    if (n_cols < 0 || R->rows < 0 || R->cols < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (n_cols == 0 || R->cols == 0) return SF_OK;
    if (!col_ptr || !out || ld_out < R->cols) return set_error(SF_ERR_INVALID, "bad output or col_ptr");
    if (R->stride_col != 1) return set_error(SF_ERR_UNSUPPORTED, "R must have unit column stride");
    if (n_cols > 4 * (int64_t)INT32_MAX) return set_error(SF_ERR_UNSUPPORTED, "too many columns");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t D = R->cols;
    return by_dtype(R->dtype, [&](auto rtag) {
        using RT = decltype(rtag);
        constexpr int EPV = 16 / sizeof(RT);
        const int vec = (aligned16(R->data) && (R->stride_row * (int64_t)sizeof(RT)) % 16 == 0) ? 1 : 0;
        return by_dtype(values_dtype, [&](auto vtag) {
            using VT = decltype(vtag);
            // Two 16-byte vectors per lane when the gathered rows' slice fits half the L2, else one.
            const int64_t row_bytes_budget = kAccL2Budget / std::max<int64_t>(R->rows, 1);
            const bool two = row_bytes_budget >= 2 * 32 * 16;
            const int64_t slice = 32 * (two ? 2 : 1) * EPV;
            dim3 grid((unsigned)((n_cols + 3) / 4), (unsigned)((D + slice - 1) / slice));
            if (two)
                csc_accumulate_kernel<RT, VT, 2><<<grid, 128, 0, s>>>(
                    col_ptr, n_cols, row_idx, perm, reinterpret_cast<const VT *>(values),
                    reinterpret_cast<const RT *>(R->data), R->stride_row, R->rows, D, out, ld_out, col_sums, vec,
                    device_error_word());
            else
                csc_accumulate_kernel<RT, VT, 1><<<grid, 128, 0, s>>>(
                    col_ptr, n_cols, row_idx, perm, reinterpret_cast<const VT *>(values),
                    reinterpret_cast<const RT *>(R->data), R->stride_row, R->rows, D, out, ld_out, col_sums, vec,
                    device_error_word());
            return check_cuda(cudaGetLastError(), "csc accumulate launch");
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
