/*
 * saeflow_b200 — C ABI of the B200 (sm_100a) SAE hot path:
 *
 *     fused encode  ->  dense -> CSR compaction  ->  CSR sparse decode
 *
 * Every entry point takes plain device pointers, element strides, dtype codes and a
 * CUDA stream, launches its kernels on that stream and returns an sf_status code.
 * Nothing here synchronises the stream except sf_device_error(). No torch types cross
 * this boundary; the Python layer in saeflow_b200/kernels binds it with ctypes.
 *
 * The reference interfaces these replace are the Triton host wrappers of saeflow:
 *   saeflow/kernels/encode.py:97-139   fused_encode
 *   saeflow/kernels/decode.py:77-94    dense_to_csr  (count, cumsum, host sync, compaction)
 *   saeflow/kernels/decode.py:97-120   sparse_decode
 *   saeflow/ops.py:12-16,29-36         TopK encode (dense ReLU encode + torch.topk)
 * Each declaration below names the line range it replaces.
 */
#ifndef SAEFLOW_B200_H
#define SAEFLOW_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SF_ABI_VERSION 1

/* The library is built with hidden visibility; only these entry points are exported. */
#if defined(__GNUC__)
#define SF_API __attribute__((visibility("default")))
#else
#define SF_API
#endif

/* A cudaStream_t; 0 is the legacy default stream. */
typedef struct CUstream_st *sf_stream;

/* Element types. Codes are stable ABI. */
enum sf_dtype { SF_F32 = 0, SF_BF16 = 1, SF_F16 = 2 };

/* Activations of fused_encode (saeflow/kernels/encode.py:16 ACTIVATIONS). */
enum sf_activation { SF_ACT_RELU = 0, SF_ACT_JUMPRELU = 1 };

/* Return codes. SF_ERR_INVALID maps to Python ValueError, the rest to RuntimeError. */
enum sf_status {
    SF_OK = 0,
    SF_ERR_INVALID = 1,      /* bad shape / dtype / pointer / stride combination     */
    SF_ERR_UNSUPPORTED = 2,  /* valid request this build has no kernel for            */
    SF_ERR_CUDA = 3,         /* a CUDA runtime or driver call failed                  */
    SF_ERR_WORKSPACE = 4,    /* workspace pointer missing or smaller than required    */
    SF_ERR_DEVICE = 5        /* a kernel reported a device-side error (sf_device_error) */
};

/* Encode variant selector (the `config=` kwarg of fused_encode).                  */
enum sf_encode_variant {
    SF_VARIANT_AUTO = 0,     /* the tcgen05/TMEM kernel for every dtype (IEEE fp32: split operands) */
    SF_VARIANT_TCGEN05 = 1,  /* force the tcgen05/TMEM kernel (CTA pairs when M > 128) */
    SF_VARIANT_SIMT = 2,     /* force the CUDA-core kernel (fp32 W_enc only)          */
    SF_VARIANT_TCGEN05_SINGLE = 3  /* tcgen05 kernel on single CTAs (128 x 256 tiles)  */
};

/* A strided 2-D tensor: element (i, j) is at data + (i*stride_row + j*stride_col)*size. */
typedef struct sf_matrix {
    const void *data;
    int32_t dtype;           /* enum sf_dtype */
    int32_t reserved;
    int64_t rows, cols;
    int64_t stride_row, stride_col;   /* in elements */
} sf_matrix;

/* A strided 1-D tensor; data == NULL means "absent" where the argument is optional. */
typedef struct sf_vector {
    const void *data;
    int32_t dtype;
    int32_t reserved;
    int64_t len;
    int64_t stride;          /* in elements */
} sf_vector;

/* Message of the last failing call on this host thread ("" if none). */
SF_API const char *sf_last_error(void);

/* ABI version (SF_ABI_VERSION) of the loaded library. */
SF_API int sf_abi_version(void);

/*
 * Device-side error word of the current device: kernels never trap; a bounded wait
 * that runs out, or an out-of-range CSR index, ORs a code into this word. The call
 * synchronises the device, stores the word in *code and clears it.
 * Bits: 1 = pipeline wait timed out, 2 = CSR index out of range, 4 = bad indptr.
 */
SF_API int sf_device_error(uint32_t *code);

/*
 * Workspace bytes sf_fused_encode needs for these operands (the b_dec-shifted,
 * dtype-converted copy of x, plus a repacked W_enc when its layout cannot be read by
 * TMA; for IEEE fp32 on the tensor cores the three-part bf16 splits of the shifted x and of
 * W_enc for one K range, 6 k' bytes per row and 6 k' bytes per feature with k' = the range
 * (d_in up to 1024, else d_in split evenly into ranges of at most 1024) rounded up to 64,
 * 4 d_in bytes per row for the non-finite fallback and, with more than one range, 4 bytes
 * per (row, feature rounded up to 256) of fp32 partial sums). Replaces the
 * allocation-free Triton launch of saeflow/kernels/encode.py:115-139.
 */
SF_API int sf_fused_encode_workspace(const sf_matrix *x, const sf_matrix *W_enc, int allow_tf32,
                              int variant, size_t *bytes);

/*
 * out = act((x - b_dec) @ W_enc + b_enc), fp32 accumulation.
 * Replaces saeflow/kernels/encode.py:97-139 (+ _encode_kernel :36-91).
 *   x      [M, d_in]  f32/bf16/f16, any strides
 *   W_enc  [d_in, d_sae], any strides; its dtype picks the MMA type (encode.py:72)
 *   b_enc, b_dec, threshold: vectors (threshold only for SF_ACT_JUMPRELU)
 *   out    [M, d_sae] in out->dtype, any strides (data is written through)
 *   row_nnz: NULL or int32 [M]; each row's count of stored nonzeros is ADDED
 *            (encode.py:89-91; the buffer is caller-zeroed)
 *   allow_tf32: fp32 W_enc only; 0 = IEEE fp32 products (encode.py:118-120). With fp32 x
 *            too these run on the bf16 tensor cores by default: both operands split into
 *            three bf16 parts (Henry, Tang & Heinecke, ARITH 2019), the six partial products
 *            above 2^-23 summed smallest first in the fp32 accumulator. The tensor cores
 *            round that sum toward zero once per 16 products, an error growing with the K
 *            range, so d_in runs in ranges of at most 1024 whose sums are added in fp32
 *            round-to-nearest: errors of the order of fp32 FMA chains (measured at d_in 768
 *            and 2304). SF_VARIANT_SIMT pins the CUDA-core IEEE kernel. An inf or NaN operand
 *            makes the call run on the CUDA-core kernel instead (decided on the device, no
 *            sync).
 */
SF_API int sf_fused_encode(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc,
                    const sf_vector *b_dec, const sf_vector *threshold, int activation,
                    const sf_matrix *out, int32_t *row_nnz, int allow_tf32, int variant,
                    void *workspace, size_t workspace_bytes, sf_stream stream);

/* Columns per (row, tile) cell of the encode-straight-to-CSR staging. */
#define SF_CSR_TILE 256

/*
 * Encode straight to CSR, step 1: the encoder GEMM without its dense [M, d_sae] output.
 * For every (row, SF_CSR_TILE-column tile) the epilogue writes the count of stored nonzeros
 * to tile_counts [M, ceil(d_sae / SF_CSR_TILE)] and, where nonzero, the staging offset of the
 * tile's (column, value) pairs to tile_offsets; the pairs go to stage_indices / stage_values
 * (stage_capacity entries, values in values_dtype) in column order; each row's count is added
 * to row_nnz (caller-zeroed). state[0] (staging cursor) and state[1] (overflow flag) must be
 * zero on entry; state[1] != 0 afterwards means stage_capacity was too small and the staged
 * pairs are incomplete. Workspace: sf_fused_encode_workspace. Every dtype on the tensor
 * cores (IEEE fp32 from split operands, with the CUDA-core fallback for non-finite ones).
 * With sf_csr_indptr and sf_csr_place this replaces saeflow/ops.py:36-39 (fused_encode with
 * row_nnz, then dense_to_csr, decode.py:77-94), producing the identical canonical CSR.
 */
SF_API int sf_encode_csr_stage(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc,
                               const sf_vector *b_dec, const sf_vector *threshold, int activation,
                               int values_dtype, int32_t *row_nnz, int32_t *tile_counts, int32_t *tile_offsets,
                               int32_t *stage_indices, void *stage_values, int64_t stage_capacity, uint32_t *state,
                               int allow_tf32, void *workspace, size_t workspace_bytes, sf_stream stream);

/*
 * Encode straight to CSR, step 2 (after sf_csr_indptr on row_nnz and a read of indptr[M] to
 * size indices / values): moves the staged pairs into canonical CSR order. A cell whose count
 * or offset is inconsistent (outside [0, SF_CSR_TILE] or the staging capacity) is skipped
 * and sets bit 4 of the device error.
 */
SF_API int sf_csr_place(const int32_t *tile_counts, const int32_t *tile_offsets, int64_t M, int64_t d_sae,
                        const int32_t *stage_indices, const void *stage_values, int64_t stage_capacity,
                        int values_dtype, const int64_t *indptr, int32_t *indices, void *values, sf_stream stream);

/*
 * Encode straight to CSR, step 2 with no host sync, for a CSR consumed on the device (the
 * forward pass decodes it right away): sf_csr_indptr on row_nnz followed by sf_csr_place,
 * with indices / values sized by the staging capacity instead of by nnz (every placed pair
 * comes from the staging, so nnz <= stage_capacity). If the staging overflowed (state[1] != 0,
 * as written by sf_encode_csr_stage), indptr is written all zero and nothing is placed, so a
 * decode that follows on the stream reads no entries; the caller reads state[1] after the
 * stream work and redoes those rows through the dense route.
 * Replaces the host sync of saeflow/kernels/decode.py:88 for device-side consumers
 * (saeflow/ops.py:47-49 forward = decode_sparse(encode_sparse(x))).
 */
SF_API int sf_csr_finish_async(const int32_t *row_nnz, const int32_t *tile_counts, const int32_t *tile_offsets,
                               int64_t M, int64_t d_sae, const int32_t *stage_indices, const void *stage_values,
                               int64_t stage_capacity, int values_dtype, const uint32_t *state, int64_t *indptr,
                               int32_t *indices, void *values, sf_stream stream);

/*
 * row_nnz[m] = number of f[m, :] != 0 (NaN counts, -0.0 does not). Overwrites.
 * Replaces torch.count_nonzero at saeflow/kernels/decode.py:85.
 */
SF_API int sf_row_nnz(const sf_matrix *f, int32_t *row_nnz, sf_stream stream);

/*
 * indptr[0] = 0, indptr[m+1] = sum_{i<=m} row_nnz[i] (int64).
 * Replaces saeflow/kernels/decode.py:86-87 (zeros + cumsum).
 */
SF_API int sf_csr_indptr(const int32_t *row_nnz, int64_t M, int64_t *indptr, sf_stream stream);

/*
 * Canonical (column-sorted) CSR of the nonzeros of f, given its indptr.
 * indices int32 [nnz], values [nnz] in values_dtype (conversion from f's dtype if it
 * differs). Replaces _compact_kernel, saeflow/kernels/decode.py:61-74,93.
 */
SF_API int sf_dense_to_csr(const sf_matrix *f, const int64_t *indptr, int32_t *indices, void *values,
                    int values_dtype, sf_stream stream);

/*
 * out[m, :] = b_dec + sum_{j in row m} values[j] * W_dec[indices[j], :], fp32 accumulation.
 * Replaces saeflow/kernels/decode.py:97-120 (+ _decode_kernel :28-55).
 *   indptr int64 [M+1], indices int32 [nnz], values [nnz] (values_dtype)
 *   W_dec [d_sae, d_in] any strides; b_dec NULL data = no bias; out [M, d_in] any strides.
 * An index outside [0, d_sae) contributes nothing and sets bit 2 of the device error.
 */
SF_API int sf_sparse_decode(const int64_t *indptr, int64_t M, const int32_t *indices, const void *values,
                     int values_dtype, const sf_matrix *W_dec, const sf_vector *b_dec,
                     const sf_matrix *out, sf_stream stream);

/*
 * sf_fused_encode without a caller-supplied workspace, for callers that cannot allocate
 * device memory: a foreign-language host handed only input/output buffers by the
 * framework that owns the GPU, a process whose caching allocator already holds nearly
 * all device memory, or a loop that cannot take cudaMalloc's implicit synchronisation.
 * It has no counterpart in the reference (whose Triton launch needs no workspace).
 *
 * The workspace is a 16 MiB array in the library's device image (held by every GPU that
 * loads the library's device code, until exit); this call allocates nothing. Operands
 * whose sf_fused_encode_workspace exceeds 16 MiB are rejected with SF_ERR_WORKSPACE
 * (e.g. bf16 x with d_in=2304: at most 3640 rows per call). W_enc must be readable in
 * place: a 16-bit W_enc contiguous along one dimension with a 16-byte-aligned base and
 * row pitch, or on the TF32 path an fp32 W_enc in column-major layout; other layouts need a
 * repacked copy of W_enc that the scratch cannot hold, and are rejected with their own
 * message. IEEE fp32 (fp32 x and W_enc, allow_tf32 0) with SF_VARIANT_AUTO runs on the
 * CUDA-core kernel here, which reads W_enc in place: the tensor-core route's split copy of
 * W_enc does not fit the scratch. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) and should come
 * before any stream capture; the address is kept for the process's life, so calls after
 * a cudaDeviceReset of that device are unsupported. Every call on a device shares the one
 * array: calls whose kernels overlap on the GPU (other streams, other host threads) race
 * on it; serialise them. Arguments and results are those of sf_fused_encode.
 */
SF_API int sf_fused_encode_noalloc(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc,
                                   const sf_vector *b_dec, const sf_vector *threshold, int activation,
                                   const sf_matrix *out, int32_t *row_nnz, int allow_tf32, int variant,
                                   sf_stream stream);

/*
 * Workspace bytes for sf_topk_encode.
 */
SF_API int sf_topk_encode_workspace(const sf_matrix *x, const sf_matrix *W_enc, int k, int allow_tf32,
                             size_t *bytes);

/*
 * TopK SAE encode without the dense [M, d_sae] output: per row the k largest values of
 * relu((x - b_dec) @ W_enc + b_enc), rounded to values_dtype, selected inside the GEMM
 * epilogue. Output is fixed width: indices int32 [M, k], values [M, k], each row sorted
 * by value descending, ties by lower feature index.
 * Replaces saeflow/ops.py:12-16 (_topk) and :32-36 (TopK branch of encode_sparse).
 */
SF_API int sf_topk_encode(const sf_matrix *x, const sf_matrix *W_enc, const sf_vector *b_enc,
                   const sf_vector *b_dec, int k, int32_t *indices, void *values,
                   int values_dtype, int allow_tf32, void *workspace, size_t workspace_bytes,
                   sf_stream stream);

/* ------------------------------------------------------------------------------------
 * Backward of the sparse forward (training on sparse features). The reference has no
 * backward kernels; these implement its roadmap item (README.md:244). With the forward
 * f = act((x - b_dec) @ W_enc + b_enc) as CSR and x_hat = f @ W_dec + b_dec, and
 * g = dL/dx_hat: the column view of the CSR from sf_csr_transpose; dW_dec and dpre in one
 * sf_csc_gather(values = f, R = g, W = W_dec); dW_enc^T and db_enc from
 * sf_csc_gather(values = dpre, R = x - b_dec); dx from sf_sparse_decode of dpre against
 * W_enc^T. sf_csr_sddmm computes dpre alone on the CSR pattern.
 */

/* out[j, i] = in[i, j], converted to out's dtype (W_enc^T for dx; dW_enc from dW_enc^T). */
SF_API int sf_transpose(const sf_matrix *in, const sf_matrix *out, sf_stream stream);

/* Bytes of workspace sf_csr_transpose needs for n_cols columns and nnz entries. */
SF_API int sf_csr_transpose_workspace(int64_t n_cols, int64_t nnz, size_t *bytes);

/*
 * Column view of a CSR pattern (the CSR of its transpose): col_ptr int64 [n_cols+1], and for
 * each column's entries, rows ascending, row_idx int32 [nnz] (the entry's row), perm int64 [nnz]
 * (its position in the CSR) and col_idx int32 [nnz] (its column; optional, may be NULL; required
 * by sf_csc_gather). An index outside [0, n_cols) is skipped and sets bit 2 of the device error;
 * a (row, column) pair present twice sets bit 4.
 */
SF_API int sf_csr_transpose(const int64_t *indptr, int64_t M, const int32_t *indices, int64_t nnz, int64_t n_cols,
                            int64_t *col_ptr, int32_t *row_idx, int64_t *perm, int32_t *col_idx,
                            void *workspace, size_t workspace_bytes, sf_stream stream);

/*
 * Sampled dot products on a CSR pattern:
 *   out[e] = (values[e] != 0) * sum_d G[row(e), d] * W[indices[e], d]      (fp32 accumulation)
 * G [M, D] and W [n, D] of one dtype with unit column stride; values (values_dtype) masks
 * entries whose forward value is zero (TopK's non-positive picks).
 */
SF_API int sf_csr_sddmm(const int64_t *indptr, int64_t M, const int32_t *indices, const sf_matrix *G,
                        const sf_matrix *W, const void *values, int values_dtype, float *out, sf_stream stream);

/*
 * y[i] = sum_j A[i, j] * x[j] with fp32 x and y, fp32 sums in a fixed order; A [rows, cols] any
 * dtype with unit column stride. With A = W_enc and x = the per-feature sums of dpre (db_enc),
 * y is the sum of dx over the tokens, which db_dec needs, without forming dx.
 */
SF_API int sf_matvec(const sf_matrix *A, const float *x, float *y, sf_stream stream);

/* Bytes of workspace sf_csc_gather needs for nnz entries gathering rows of R (0 when it needs none). */
SF_API int sf_csc_gather_workspace(int64_t nnz, const sf_matrix *R, size_t *bytes);

/*
 * Per-column gather over the column view of sf_csr_transpose (p runs over column j's entries
 * in the view's order, rows ascending):
 *   out[j, :]     = sum_p values[perm[p]] * R[row_idx[p], :]            (fp32 sums, out's dtype)
 *   col_sums[j]   = sum_p values[perm[p]]                                (optional, may be NULL)
 *   dots[perm[p]] = (values[perm[p]] != 0) * R[row_idx[p], :] . W[j, :]  (optional: W NULL or
 *                                                                         W->data NULL skips it)
 * R [M, D] and W [n_cols, D] of one dtype with unit column stride; out [n_cols, D] in any
 * dtype; values in values_dtype, indexed by CSR position. Rows whose byte width and pitch are
 * multiples of 16 go through the shared-memory bulk-copy kernel, others through a plain one.
 */
SF_API int sf_csc_gather(const int64_t *col_ptr, int64_t n_cols, const int32_t *col_idx, int64_t nnz,
                         const int32_t *row_idx, const int64_t *perm, const void *values, int values_dtype,
                         const sf_matrix *R, const sf_matrix *W, float *dots, const sf_matrix *out,
                         float *col_sums, void *workspace, size_t workspace_bytes, sf_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* SAEFLOW_B200_H */
