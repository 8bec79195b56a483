// Host-side interfaces between the saeflow_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sf {

// GEMM operands as the tensor-core kernel reads them through TMA.
//   A: [M, K] K-contiguous, row pitch a_pitch elements (16-byte multiple), MMA dtype.
//   B: W_enc as [K, N]; b_mn_major: element (k, n) at b[k*b_pitch + n] (N-contiguous),
//      else at b[n*b_pitch + k] (K-contiguous).
struct GemmOperands {
    const void *a;
    int64_t a_pitch;
    const void *b;
    int64_t b_pitch;
    bool b_mn_major;
    int ab_fmt;  // 0 fp16, 1 bf16, 2 tf32 (fp32 storage)
    int64_t M, N, K;
    // Fused shift (16-bit CTA-pair kernel, kFusedShift): the kernel's converter warps read A
    // rows from `a` (K-contiguous, pitch a_pitch elements, 16-byte aligned, K % 8 == 0) and
    // subtract `bdec` in fp32 before rounding to the MMA dtype. bdec_mode: 0 no shift (the
    // rows are already shifted), 1 contiguous 16-byte-aligned 16-bit, 2 contiguous
    // 16-byte-aligned fp32, 3 any dtype and stride.
    const void *bdec;
    int bdec_dtype;
    int64_t bdec_stride;
    int bdec_mode;
};

// 1: the CTA-pair kernel for 16-bit operands builds its A tiles with converter warps that
// read x itself and subtract b_dec on the way (no shifted copy of x in HBM, no shift pass).
// 0 (default): a separate pass writes the shifted copy and TMA loads it. Measured on B200
// at config 2 (16384 x 2304 -> 65536 bf16), the converter warps cannot keep enough loads
// in flight beside the epilogue's registers (warps stalled on L2 latency, tensor pipe 19%
// busy against 81%): encode 12.07 ms against 3.55 ms for the pass + TMA, whose shift pass
// costs 38 us.
#ifndef SF_FUSED_SHIFT
#define SF_FUSED_SHIFT 0
#endif
constexpr bool kFusedShift = SF_FUSED_SHIFT != 0;

struct EpilogueArgs {
    const void *b_enc;
    int b_enc_dtype;
    int64_t b_enc_stride;
    const void *thr;
    int thr_dtype;
    int64_t thr_stride;
    int activation;
    void *out;
    int out_dtype;
    int64_t out_sm, out_sn;
    int out_vec;
    int32_t *row_nnz;
};

struct TopkArgs {
    const void *b_enc;
    int b_enc_dtype;
    int64_t b_enc_stride;
    int k;
    int values_dtype;
    int n_chunks;
    unsigned long long *cand;  // [M, n_chunks, k]
};

// Staging of the encode-straight-to-CSR path.
struct CsrArgs {
    int32_t *tile_cnt;   // [M, n_tiles]
    int32_t *tile_off;   // [M, n_tiles]
    int32_t *stage_idx;  // [cap]
    void *stage_val;     // [cap]
    unsigned *state;     // [0] cursor, [1] overflow
    unsigned cap;
};
constexpr int kCsrTile = 256;  // columns per (row, tile) count cell

int encode_tc_dense(const GemmOperands &g, const EpilogueArgs &ep, int variant, cudaStream_t stream);
int encode_tc_csr(const GemmOperands &g, const EpilogueArgs &ep, const CsrArgs &csr, cudaStream_t stream);
int pair_slots(const void *kern, const cudaLaunchConfig_t &cfg);
int encode_tc_topk(const GemmOperands &g, const TopkArgs &tk, cudaStream_t stream);
int topk_chunks(int64_t M, int64_t N);
constexpr int kTopkMaxK = 112;  // shared-memory bound of the fused top-k lists and candidate buffers

// IEEE fp32 encoder on the CUDA cores: dense output (csr == nullptr) or the CSR staging of
// encode_tc_csr (same tile counts, offsets and column-ordered runs).
int encode_simt_f32(const float *xs, int64_t xs_pitch, const float *W, int64_t swk, int64_t swn, int64_t M,
                    int64_t N, int64_t K, const EpilogueArgs &ep, cudaStream_t stream, const CsrArgs *csr = nullptr);

}  // namespace sf
