// fp32 SAE encoder on the CUDA cores, IEEE fp32 products and fp32 accumulation.
//
// The reference computes fp32 inputs with `input_precision="ieee"` unless TF32 is
// allowed (saeflow/kernels/encode.py:118-120); this kernel is that path. Epilogue
// semantics are identical to the tensor-core kernel (encode.py:77-91), including the
// encode-straight-to-CSR staging epilogue (CSR = true).
//
// 128 x (64*NF) output tile per CTA, K in steps of 8 through double-buffered shared memory,
// 256 threads each owning an 8 x (4*NF) register block (rows {4ty..4ty+3, 64+4ty..}, columns
// {64q+4tx..64q+4tx+3 : q < NF}) so the shared-memory reads are conflict-free float4
// broadcasts. NF=4 (128 x 256 tiles, 128 accumulators per thread) is the default: per K step
// a thread issues 6 shared loads for 128 FMAs (4 for 64 with NF=2), which moved the FMA pipe
// from 62% busy (instruction-issue bound) toward its peak; NF=2 serves d_sae < 256.
#include "sf_common.cuh"
#include "sf_internal.h"

namespace sf {

namespace {

constexpr int SB_M = 128, SB_K = 8, SB_T = 256;
// K steps of one shared-memory tile unrolled at once: each is 8 x 4NF FMAs, and the fully
// unrolled tile body (8 steps, ~1000 FMAs) overflows the instruction cache.
#ifndef SF_SIMT_KK_UNROLL
#define SF_SIMT_KK_UNROLL 8
#endif
constexpr int kKkUnroll = SF_SIMT_KK_UNROLL;

template <typename OT>
__device__ __forceinline__ void simt_store4(void *out, int64_t sm, int64_t sn, int vec, int64_t N, int row, int col,
                                            const float (&v)[4]) {
    OT *base = reinterpret_cast<OT *>(out) + (int64_t)row * sm;
    if (vec && col + 4 <= N && sizeof(OT) == 4) {
        *reinterpret_cast<float4 *>(base + col) = make_float4(v[0], v[1], v[2], v[3]);
        return;
    }
    if (vec && col + 4 <= N && sizeof(OT) == 2) {
        uint2 pk;
        OT *e = reinterpret_cast<OT *>(&pk);
#pragma unroll
        for (int j = 0; j < 4; ++j) e[j] = from_f32<OT>(v[j]);
        *reinterpret_cast<uint2 *>(base + col) = pk;
        return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (col + j < N) base[(int64_t)(col + j) * sn] = from_f32<OT>(v[j]);
}

// Inclusive sum over the 16 lanes of this half-warp (lanes 0-15 or 16-31).
__device__ __forceinline__ int half_warp_inclusive_scan(int v, int tx) {
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, off, 16);
        if (tx >= off) v += t;
    }
    return v;
}

// Encode straight to CSR (256-column tiles): for each of its 8 rows a thread holds 16
// stored values (columns 64h + 4tx + j); the 16 threads of a row are one half-warp. Nonzero
// masks are taken on the stored value, as the dense route counts them. Within a row, offsets
// follow column order (h, then tx, then j) by four half-warp scans; one atomicAdd per warp
// reserves staging space for its 16 rows (ordered i, half), and each (row, tile) cell gets its
// count and, when nonzero, its staging offset: the staging contract of the tensor-core
// kernel's CSR epilogue, consumed by the same placement kernel.
template <typename VT>
__device__ __forceinline__ void simt_csr_epilogue(const float (&o)[8][16], int m0, int n0, int M, int N, int tx,
                                                  int ty, const EpilogueArgs &ep, const CsrArgs &csr,
                                                  int n_tiles) {
    const int lane = threadIdx.x & 31;
    const int tile = n0 / kCsrTile;
    int tot[8], pre[8][4];
    uint32_t mask[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int row = m0 + ((i < 4) ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        uint32_t m = 0;
#pragma unroll
        for (int h = 0; h < 4; ++h)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                m |= ((o[i][h * 4 + j] != 0.f && n0 + h * 64 + tx * 4 + j < N && row < M) ? 1u : 0u)
                     << (h * 4 + j);
        mask[i] = m;
        int run = 0;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const int c = __popc((m >> (h * 4)) & 0xFu);
            const int incl = half_warp_inclusive_scan(c, tx);
            pre[i][h] = run + incl - c;
            run += __shfl_sync(0xffffffffu, incl, 15, 16);
        }
        tot[i] = run;
    }
    // One reservation per warp: its rows ordered (i, half), half = lane / 16.
    const int half = lane >> 4;
    int warp_total = 0, my_off[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int t0 = __shfl_sync(0xffffffffu, tot[i], 0);
        const int t1 = __shfl_sync(0xffffffffu, tot[i], 16);
        my_off[i] = warp_total + (half ? t0 : 0);
        warp_total += t0 + t1;
    }
    unsigned base = 0;
    if (lane == 0 && warp_total > 0) base = atomicAdd(&csr.state[0], (unsigned)warp_total);
    base = __shfl_sync(0xffffffffu, base, 0);
    const bool fits = (unsigned long long)base + (unsigned long long)warp_total <= (unsigned long long)csr.cap;
    if (lane == 0 && warp_total > 0 && !fits) atomicOr(&csr.state[1], 1u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int row = m0 + ((i < 4) ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        const unsigned row_off = base + (unsigned)my_off[i];
        if (tx == 0 && row < M) {
            const int64_t cell = (int64_t)row * n_tiles + tile;
            csr.tile_cnt[cell] = tot[i];
            if (tot[i]) csr.tile_off[cell] = (int)row_off;
            if (ep.row_nnz != nullptr && tot[i]) atomicAdd(ep.row_nnz + row, tot[i]);
        }
        if (!fits || mask[i] == 0) continue;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            unsigned at = row_off + (unsigned)pre[i][h];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (mask[i] & (1u << (h * 4 + j))) {
                    csr.stage_idx[at] = n0 + h * 64 + tx * 4 + j;
                    reinterpret_cast<VT *>(csr.stage_val)[at] = from_f32<VT>(o[i][h * 4 + j]);
                    ++at;
                }
            }
        }
    }
}

// One 128 x (64 NF) output tile at (m0, n0).
template <int NF, bool CSR>
__device__ __forceinline__ void simt_tile(const float *__restrict__ xs, int64_t ldx, const float *__restrict__ W,
                                          int64_t swk, int64_t swn, int M, int N, int K, const EpilogueArgs &ep,
                                          int w_vec, const CsrArgs &csr, int n_tiles, int m0, int n0) {
    constexpr int SB_N = 64 * NF;
    constexpr int BQ = NF / 2;  // float4 loads of the B tile per thread per K step
    __shared__ __align__(16) float As[2][SB_K][SB_M + 4];
    __shared__ __align__(16) float Bs[2][SB_K][SB_N + 4];
    __shared__ float s_bias[SB_N], s_thr[SB_N];

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;

    for (int j = tid; j < SB_N; j += SB_T) {
        const int col = n0 + j;
        s_bias[j] = col < N ? load_as_f32(ep.b_enc, ep.b_enc_dtype, (int64_t)col * ep.b_enc_stride) : 0.f;
        s_thr[j] = (col < N && ep.activation == SF_ACT_JUMPRELU)
                       ? load_as_f32(ep.thr, ep.thr_dtype, (int64_t)col * ep.thr_stride)
                       : 0.f;
    }

    // Global -> register staging: A: row = tid/2, k-quad = tid%2; B: k = tid/32, n-quads
    // (tid%32)*4 + 128q.
    const int a_row = tid >> 1, a_kq = (tid & 1) * 4;
    const int b_k = tid >> 5, b_nq = (tid & 31) * 4;
    float4 ra;
    float rb[BQ][4];

    auto load_tile = [&](int k0) {
        const int gr = m0 + a_row, gk = k0 + a_kq;
        // xs rows are zero-padded to a multiple of 4 columns, so a quad never straddles K.
        ra = (gr < M && gk < K) ? *reinterpret_cast<const float4 *>(xs + (int64_t)gr * ldx + gk)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        const int kk = k0 + b_k;
#pragma unroll
        for (int q = 0; q < BQ; ++q) {
            const int nn = n0 + b_nq + q * 128;
            if (w_vec && kk < K && nn + 4 <= N) {
                const float4 t = *reinterpret_cast<const float4 *>(W + (int64_t)kk * swk + nn);
                rb[q][0] = t.x, rb[q][1] = t.y, rb[q][2] = t.z, rb[q][3] = t.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    rb[q][j] = (kk < K && nn + j < N) ? __ldg(W + (int64_t)kk * swk + (int64_t)(nn + j) * swn) : 0.f;
            }
        }
    };
    auto store_tile = [&](int buf) {
        As[buf][a_kq + 0][a_row] = ra.x;
        As[buf][a_kq + 1][a_row] = ra.y;
        As[buf][a_kq + 2][a_row] = ra.z;
        As[buf][a_kq + 3][a_row] = ra.w;
#pragma unroll
        for (int q = 0; q < BQ; ++q)
            *reinterpret_cast<float4 *>(&Bs[buf][b_k][b_nq + q * 128]) =
                make_float4(rb[q][0], rb[q][1], rb[q][2], rb[q][3]);
    };

    float acc[8][4 * NF];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4 * NF; ++j) acc[i][j] = 0.f;

    const int nk = (K + SB_K - 1) / SB_K;
    load_tile(0);
    store_tile(0);
    __syncthreads();
    for (int kt = 0; kt < nk; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < nk) load_tile((kt + 1) * SB_K);
#pragma unroll kKkUnroll
        for (int kk = 0; kk < SB_K; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float b[4 * NF];
#pragma unroll
            for (int q = 0; q < NF; ++q) {
                const float4 bq = *reinterpret_cast<const float4 *>(&Bs[buf][kk][q * 64 + tx * 4]);
                b[4 * q + 0] = bq.x, b[4 * q + 1] = bq.y, b[4 * q + 2] = bq.z, b[4 * q + 3] = bq.w;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4 * NF; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < nk) store_tile(buf ^ 1);
        __syncthreads();
    }

    if constexpr (CSR) {
        static_assert(NF == 4, "CSR staging needs 256-column tiles");
        // bias, activation and rounding in place, then the staging epilogue
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int h = 0; h < NF; ++h)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int c = h * 64 + tx * 4 + j;
                    const float pre = acc[i][h * 4 + j] + s_bias[c];
                    float o = fmaxf(pre, 0.f);
                    if (ep.activation == SF_ACT_JUMPRELU) o = (pre > s_thr[c]) ? o : 0.f;
                    acc[i][h * 4 + j] = round_to(o, ep.out_dtype);
                }
        if (ep.out_dtype == SF_F32)
            simt_csr_epilogue<float>(acc, m0, n0, M, N, tx, ty, ep, csr, n_tiles);
        else if (ep.out_dtype == SF_BF16)
            simt_csr_epilogue<__nv_bfloat16>(acc, m0, n0, M, N, tx, ty, ep, csr, n_tiles);
        else
            simt_csr_epilogue<__half>(acc, m0, n0, M, N, tx, ty, ep, csr, n_tiles);
        return;
    } else {

    // Epilogue: bias, activation, rounding to the output dtype, count, store.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = (i < 4) ? ty * 4 + i : 64 + ty * 4 + (i - 4);
        const int row = m0 + r;
        int cnt = 0;
#pragma unroll
        for (int h = 0; h < NF; ++h) {
            const int c = h * 64 + tx * 4;
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float pre = acc[i][h * 4 + j] + s_bias[c + j];
                float o = fmaxf(pre, 0.f);
                if (ep.activation == SF_ACT_JUMPRELU) o = (pre > s_thr[c + j]) ? o : 0.f;
                o = round_to(o, ep.out_dtype);
                v[j] = o;
                cnt += (o != 0.f && n0 + c + j < N) ? 1 : 0;
            }
            if (row < M) {
                if (ep.out_dtype == SF_F32)
                    simt_store4<float>(ep.out, ep.out_sm, ep.out_sn, ep.out_vec, N, row, n0 + c, v);
                else if (ep.out_dtype == SF_BF16)
                    simt_store4<__nv_bfloat16>(ep.out, ep.out_sm, ep.out_sn, ep.out_vec, N, row, n0 + c, v);
                else
                    simt_store4<__half>(ep.out, ep.out_sm, ep.out_sn, ep.out_vec, N, row, n0 + c, v);
            }
        }
        // The 16 threads sharing these rows are 16 consecutive lanes (same ty).
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
        if (tx == 0 && ep.row_nnz != nullptr && row < M && cnt != 0) atomicAdd(ep.row_nnz + row, cnt);
    }
    }  // dense epilogue
}

// Tiles in row-major order over (m-tile, n-tile), n fastest. LOOP = false: one tile per CTA
// (the grid covers them all). LOOP = true: the gated launch, one CTA per SM looping over the
// tiles, so that skipping it costs one short wave (the loop costs the CSR variant a few
// spilled registers, which only the rare non-finite fallback pays).
template <int NF, bool CSR, bool LOOP>
__global__ void __launch_bounds__(SB_T, 1)
    encode_simt_kernel(const float *__restrict__ xs, int64_t ldx, const float *__restrict__ W, int64_t swk,
                       int64_t swn, int M, int N, int K, EpilogueArgs ep, int w_vec, CsrArgs csr, int n_tiles,
                       int tiles_n, int64_t tiles, const unsigned *gate) {
    if (gate != nullptr && *reinterpret_cast<const volatile unsigned *>(gate) == 0u) return;
    if constexpr (LOOP) {
        for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
            const int m0 = (int)(t / tiles_n) * SB_M, n0 = (int)(t % tiles_n) * (64 * NF);
            simt_tile<NF, CSR>(xs, ldx, W, swk, swn, M, N, K, ep, w_vec, csr, n_tiles, m0, n0);
            __syncthreads();  // the next tile reuses the shared operand and bias arrays
        }
    } else {  // grid (n-tiles, m-tiles)
        simt_tile<NF, CSR>(xs, ldx, W, swk, swn, M, N, K, ep, w_vec, csr, n_tiles, blockIdx.y * SB_M,
                           blockIdx.x * (64 * NF));
    }
}

}  // namespace

int encode_simt_f32(const float *xs, int64_t xs_pitch, const float *W, int64_t swk, int64_t swn, int64_t M,
                    int64_t N, int64_t K, const EpilogueArgs &ep, cudaStream_t stream, const CsrArgs *csr,
                    const unsigned *gate) {
    const bool wide = N >= 256 || csr != nullptr;  // CSR staging needs whole 256-column tiles
    const int64_t sb_n = wide ? 256 : 128;
    const int64_t tiles_n = (N + sb_n - 1) / sb_n, tiles_m = (M + SB_M - 1) / SB_M, tiles = tiles_n * tiles_m;
    const int w_vec = (swn == 1 && (swk % 4) == 0 && (reinterpret_cast<uintptr_t>(W) & 15u) == 0) ? 1 : 0;
    // One CTA per tile on a (n-tiles, m-tiles) grid; a gated launch (a no-op unless the split
    // found a non-finite operand) takes one CTA per SM looping over the tiles, so that
    // skipping it costs one short wave.
    const bool loop = gate != nullptr && tiles > num_sms();
    if (!loop && (tiles_n > 2147483647ll || tiles_m > 65535))
        return set_error(SF_ERR_UNSUPPORTED, "SIMT encode grid too large (M=%lld N=%lld)", (long long)M, (long long)N);
    const dim3 grid = loop ? dim3((unsigned)num_sms()) : dim3((unsigned)tiles_n, (unsigned)tiles_m);
    const int n_tiles = (int)((N + kCsrTile - 1) / kCsrTile);
    const CsrArgs c = csr ? *csr : CsrArgs{};
    auto launch = [&](auto kern) {
        kern<<<grid, SB_T, 0, stream>>>(xs, xs_pitch, W, swk, swn, (int)M, (int)N, (int)K, ep, w_vec, c, n_tiles,
                                        (int)tiles_n, tiles, gate);
    };
    if (csr)
        loop ? launch(encode_simt_kernel<4, true, true>) : launch(encode_simt_kernel<4, true, false>);
    else if (wide)
        loop ? launch(encode_simt_kernel<4, false, true>) : launch(encode_simt_kernel<4, false, false>);
    else
        loop ? launch(encode_simt_kernel<2, false, true>) : launch(encode_simt_kernel<2, false, false>);
    return check_cuda(cudaGetLastError(), "encode_simt launch");
}

}  // namespace sf
