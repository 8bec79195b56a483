// IEEE-grade fp32 encode on the bf16 tensor cores: operand splitting.
//
// The reference computes fp32 x with fp32 W_enc at `input_precision="ieee"` unless TF32 is
// allowed (saeflow/kernels/encode.py:118-120). On B200 the CUDA cores give 74 TFLOP/s of
// fp32 FMA; the bf16 tensor cores give ~1.6 PFLOP/s. This file writes the operands of the
// split-precision product of Henry, Tang & Heinecke ("Leveraging the bfloat16 Artificial
// Intelligence Datatype for Higher-Precision Computations", ARITH 2019):
//
//   v = v0 + v1 + v2,  v0 = bf16_rn(v), v1 = bf16_rn(v - v0), v2 = bf16_rn(v - v0 - v1)
//
// Both differences are exact in fp32 and v2 holds the last <= 8 significant bits, so the
// three terms represent a normal fp32 value exactly. x·w is then the sum of the six products
// vi·wj with i + j <= 2; the three dropped ones are below 2^-23 |x w|. Each bf16 x bf16
// product is exact in the fp32 accumulator. The tensor cores accumulate with less than
// round-to-nearest care, so the GEMM issues the products smallest first — (x2,W0), (x1,W1),
// (x0,W2), then (x1,W0), (x0,W1), then (x0,W0) — and the large terms meet an accumulator
// that already holds the small ones (issuing them largest first measured ~7x the error).
//
// Layout: a = [x0 | x1 | x2] as one [M, 3 kp] bf16 matrix and b = [W0 ; W1 ; W2] as one
// [3 kp, N] N-contiguous bf16 matrix, kp = the K range rounded up to the GEMM's 64-element
// K block with zero padding, so every K block lies inside one segment. The GEMM's TMA
// producer maps its 6 kp/64 K blocks onto (a segment, b segment) pairs: nothing is stored
// twice. A d_in above kEmuMaxRangeK is split into K ranges, one split and one GEMM each.
//
// Non-finite operands: an inf or NaN in x - b_dec or in W_enc would meet the zero parts of
// the other operand (inf * 0 = NaN where IEEE gives inf * w = inf). The split kernels raise a
// flag for them; the tensor-core kernel then exits at once and the CUDA-core IEEE kernel,
// launched behind it and gated on the same flag, computes the call. No host sync.
#include "sf_common.cuh"
#include "sf_internal.h"

namespace sf {

namespace {

struct Split3 {
    __nv_bfloat16 p[3];
};

// Parts of v, high to low. A finite v whose bf16 rounding overflows (|v| above the largest
// bf16) takes its high part truncated, so the remainder stays exact.
__device__ __forceinline__ Split3 split3(float v, bool &bad) {
    Split3 s;
    const __nv_bfloat16 zero = __float2bfloat16_rn(0.f);
    if (!isfinite(v)) {
        bad = true;
        s.p[0] = __float2bfloat16_rn(v);
        s.p[1] = zero;
        s.p[2] = zero;
        return s;
    }
    __nv_bfloat16 a = __float2bfloat16_rn(v);
    if (__hisinf(a)) a = __float2bfloat16_rz(v);
    const float r = v - __bfloat162float(a);
    const __nv_bfloat16 b = __float2bfloat16_rn(r);
    s.p[0] = a;
    s.p[1] = b;
    s.p[2] = __float2bfloat16_rn(r - __bfloat162float(b));
    return s;
}

__device__ __forceinline__ void raise_flag(bool bad, unsigned *flag) {
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1u);
}

// a[m, s kp + k] = part s of (x[m, k] - b_dec[k]); zero for K <= k < kp. Eight elements per
// item: 2 x 16 B loads of x where rows are contiguous and 16-byte aligned, 3 x 16 B stores.
template <bool VEC>
__global__ void split_x_kernel(const float *__restrict__ x, int64_t M, int64_t K, int64_t sxm, int64_t sxk,
                               const void *b_dec, int b_dtype, int64_t b_stride, __nv_bfloat16 *__restrict__ a,
                               int64_t kp, unsigned *flag) {
    const int64_t items_per_row = kp / 8;
    const int64_t total = M * items_per_row;
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / items_per_row;
        const int64_t k0 = (i - m * items_per_row) * 8;
        float v[8];
        if (VEC && k0 + 8 <= K) {
            const float4 *src = reinterpret_cast<const float4 *>(x + m * sxm + k0);
            const float4 q0 = __ldg(src), q1 = __ldg(src + 1);
            v[0] = q0.x, v[1] = q0.y, v[2] = q0.z, v[3] = q0.w;
            v[4] = q1.x, v[5] = q1.y, v[6] = q1.z, v[7] = q1.w;
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = (k0 + t < K) ? x[m * sxm + (k0 + t) * sxk] : 0.f;
        }
        if (b_dec) {
#pragma unroll
            for (int t = 0; t < 8; ++t)
                if (k0 + t < K) v[t] -= load_as_f32(b_dec, b_dtype, (k0 + t) * b_stride);
        }
        uint4 out[3];
        __nv_bfloat16 *o[3] = {reinterpret_cast<__nv_bfloat16 *>(&out[0]), reinterpret_cast<__nv_bfloat16 *>(&out[1]),
                               reinterpret_cast<__nv_bfloat16 *>(&out[2])};
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const Split3 s = split3(v[t], bad);
            o[0][t] = s.p[0];
            o[1][t] = s.p[1];
            o[2][t] = s.p[2];
        }
        __nv_bfloat16 *dst = a + m * 3 * kp + k0;
#pragma unroll
        for (int s = 0; s < 3; ++s) *reinterpret_cast<uint4 *>(dst + s * kp) = out[s];
    }
    raise_flag(bad, flag);
}

// b[(s kp + k) * pitch + n] = part s of W[k, n]; zero rows for K <= k < kp. Row-major W
// (n contiguous, 16-byte aligned rows, N a multiple of 8): eight columns per item.
__global__ void split_w_rows_kernel(const float *__restrict__ W, int64_t K, int64_t N, int64_t swk,
                                    __nv_bfloat16 *__restrict__ b, int64_t kp, int64_t pitch, unsigned *flag) {
    const int64_t items_per_row = N / 8;
    const int64_t total = kp * items_per_row;
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = i / items_per_row;
        const int64_t n0 = (i - k * items_per_row) * 8;
        float v[8];
        if (k < K) {
            const float4 *src = reinterpret_cast<const float4 *>(W + k * swk + n0);
            const float4 q0 = __ldg(src), q1 = __ldg(src + 1);
            v[0] = q0.x, v[1] = q0.y, v[2] = q0.z, v[3] = q0.w;
            v[4] = q1.x, v[5] = q1.y, v[6] = q1.z, v[7] = q1.w;
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = 0.f;
        }
        uint4 out[3];
        __nv_bfloat16 *o[3] = {reinterpret_cast<__nv_bfloat16 *>(&out[0]), reinterpret_cast<__nv_bfloat16 *>(&out[1]),
                               reinterpret_cast<__nv_bfloat16 *>(&out[2])};
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const Split3 s = split3(v[t], bad);
            o[0][t] = s.p[0];
            o[1][t] = s.p[1];
            o[2][t] = s.p[2];
        }
#pragma unroll
        for (int s = 0; s < 3; ++s) *reinterpret_cast<uint4 *>(b + (s * kp + k) * pitch + n0) = out[s];
    }
    raise_flag(bad, flag);
}

// Any strides: 32 x 32 tiles through shared memory, read along whichever of k and n is the
// unit stride, written along n.
__global__ void split_w_tiled_kernel(const float *__restrict__ W, int64_t K, int64_t N, int64_t swk, int64_t swn,
                                     __nv_bfloat16 *__restrict__ b, int64_t kp, int64_t pitch, unsigned *flag) {
    __shared__ float tile[32][33];  // [k][n]
    const int64_t n0 = (int64_t)blockIdx.x * 32, k0 = (int64_t)blockIdx.y * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const bool k_unit = swk == 1 && swn != 1;
    for (int i = ty; i < 32; i += 8) {
        const int kk = k_unit ? tx : i, nn = k_unit ? i : tx;
        const int64_t k = k0 + kk, n = n0 + nn;
        tile[kk][nn] = (k < K && n < N) ? W[k * swk + n * swn] : 0.f;
    }
    __syncthreads();
    bool bad = false;
    for (int i = ty; i < 32; i += 8) {
        const int64_t k = k0 + i, n = n0 + tx;
        const Split3 s = split3(tile[i][tx], bad);
        if (k < kp && n < N) {
#pragma unroll
            for (int p = 0; p < 3; ++p) b[(p * kp + k) * pitch + n] = s.p[p];
        }
    }
    raise_flag(bad, flag);
}

unsigned blocks_for(int64_t items) {
    int64_t blocks = (items + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

bool aligned16_ptr(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int emu_split_operands(const EmuOperands &e, cudaStream_t s) {
    int st = SF_OK;
    if (e.reset_flag) st = check_cuda(cudaMemsetAsync(e.flag, 0, sizeof(unsigned), s), "emulated encode flag reset");
    if (st) return st;
    if (e.M > 0) {
        const bool xvec = e.sxk == 1 && (e.sxm % 4) == 0 && aligned16_ptr(e.x);
        const int64_t items = e.M * (e.kp / 8);
        if (xvec)
            split_x_kernel<true><<<blocks_for(items), 256, 0, s>>>(e.x, e.M, e.K, e.sxm, e.sxk, e.b_dec, e.b_dtype,
                                                                  e.b_stride, e.a, e.kp, e.flag);
        else
            split_x_kernel<false><<<blocks_for(items), 256, 0, s>>>(e.x, e.M, e.K, e.sxm, e.sxk, e.b_dec, e.b_dtype,
                                                                   e.b_stride, e.a, e.kp, e.flag);
        st = check_cuda(cudaGetLastError(), "split_x launch");
        if (st) return st;
    }
    if (e.swn == 1 && (e.N % 8) == 0 && (e.swk % 4) == 0 && aligned16_ptr(e.W)) {
        split_w_rows_kernel<<<blocks_for(e.kp * (e.N / 8)), 256, 0, s>>>(e.W, e.K, e.N, e.swk, e.b, e.kp, e.b_pitch,
                                                                        e.flag);
    } else {
        dim3 grid((unsigned)((e.N + 31) / 32), (unsigned)((e.kp + 31) / 32));
        split_w_tiled_kernel<<<grid, dim3(32, 8), 0, s>>>(e.W, e.K, e.N, e.swk, e.swn, e.b, e.kp, e.b_pitch, e.flag);
    }
    return check_cuda(cudaGetLastError(), "split_w launch");
}

}  // namespace sf
