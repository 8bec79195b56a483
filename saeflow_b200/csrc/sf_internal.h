// Host-side interfaces between the saeflow_b200 translation units.
#pragma once

#include <cuda_bf16.h>
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
    // Split-operand K schedule (IEEE-grade fp32 on bf16 tensor cores, emulate.cu): when
    // seg_kb > 0, A and B each hold 3 segments of seg_kb K blocks and the kernel runs
    // kEmuPairs segment pairs, pair s reading A segment (seg_a >> 4s) & 15 against B segment
    // (seg_b >> 4s) & 15. K is then the extent of the stored segments (3 seg_kb blocks).
    int seg_kb;
    uint32_t seg_a, seg_b;
    // When non-null and nonzero at launch, the kernel exits without touching any output.
    const unsigned *skip;
};

// Operands of the split-precision fp32 encode (emulate.cu): x (fp32, any strides) minus
// b_dec into a = [x0 | x1 | x2] ([M, 3 kp] bf16), W_enc (fp32 [K, N], any strides) into
// b = [W0 ; W1 ; W2] ([3 kp, N] bf16, row pitch b_pitch); *flag = 1 if any operand is not
// finite.
struct EmuOperands {
    const float *x;
    int64_t M, K, sxm, sxk;
    const void *b_dec;
    int b_dtype;
    int64_t b_stride;
    const float *W;
    int64_t N, swk, swn;
    __nv_bfloat16 *a;
    __nv_bfloat16 *b;
    int64_t kp, b_pitch;
    unsigned *flag;
    bool reset_flag;  // zero *flag first (the first K range of a call)
};
constexpr int kEmuKBlock = 64;  // bf16 elements per GEMM K block: the segment padding
constexpr int kEmuPairs = 6;
// (a segment, b segment) pairs, smallest products first: (x2,W0) (x1,W1) (x0,W2) (x1,W0) (x0,W1) (x0,W0)
constexpr uint32_t kEmuSegA = 0x001012u;  // nibble s = A segment of pair s
constexpr uint32_t kEmuSegB = 0x010210u;  // nibble s = B segment of pair s
int emu_split_operands(const EmuOperands &e, cudaStream_t s);
// Largest K range one split-precision GEMM accumulates. Its partial products are exact, but
// the tensor cores round the running fp32 sum once per 16-product MMA, toward zero, so the
// error of the large (x0, W0) term grows with the range / 16 (a bias, not a random walk):
// measured on B200 against float64, max |error| 7.8e-6 at d_in 768 (the CUDA-core IEEE
// kernel: 7.1e-6), within the fp32 contract (rtol 1e-5, atol 1e-5) at 2304, 89 of 51200
// features outside it at 4096 in one range (worst 1.6e-5). Up to 1024 the bound
// range/16 * 2^-24 (3.8e-6 relative) leaves a 2.6x margin, so a larger d_in runs as K ranges
// of at most this size, each accumulated from zero and added to the partial sum of the
// earlier ranges in fp32 round-to-nearest (EpilogueArgs::c_in).
constexpr int64_t kEmuMaxRangeK = 1024;

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
    // K-range partial sums of the split-precision route (tensor-core kernels): c_in (fp32,
    // row pitch c_in_pitch, padded to whole 256-column tiles) is added to the accumulators
    // before anything else; raw (dense kernel only) stores the sums themselves to `out` (the
    // same padded fp32 layout) with no bias, activation or count. c_in may equal out.
    const float *c_in;
    int64_t c_in_pitch;
    int raw;
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
// A non-null `gate` makes the launch a no-op unless *gate is nonzero (the non-finite-operand
// fallback of the split-precision encode).
int encode_simt_f32(const float *xs, int64_t xs_pitch, const float *W, int64_t swk, int64_t swn, int64_t M,
                    int64_t N, int64_t K, const EpilogueArgs &ep, cudaStream_t stream, const CsrArgs *csr = nullptr,
                    const unsigned *gate = nullptr);

}  // namespace sf
