// CSR side of the SAE hot path: nonzero counting, indptr scan, dense -> CSR compaction,
// CSR sparse decode, and the final merge of the fused top-k candidates. All HBM-bound.
//
//   row_nnz_kernel     replaces torch.count_nonzero    (saeflow/kernels/decode.py:85)
//   indptr_scan_kernel replaces zeros + cumsum          (decode.py:86-87)
//   compact_kernel     replaces _compact_kernel         (decode.py:61-74)
//   decode_kernel      replaces _decode_kernel          (decode.py:28-55)
//   topk_merge_kernel  replaces torch.topk on the dense ReLU output (saeflow/ops.py:12-16)
#include <algorithm>

#include <cstring>
#include <type_traits>

#include "sf_common.cuh"
#include "sf_internal.h"

namespace sf {

namespace {

// Nonzero test on raw bits, as `f != 0.0` (NaN counts, -0.0 does not).
__device__ __forceinline__ bool nz_bits16(uint32_t h) { return (h & 0x7FFFu) != 0u; }
__device__ __forceinline__ bool nz_bits32(uint32_t w) { return (w & 0x7FFFFFFFu) != 0u; }

template <typename T>
__device__ __forceinline__ bool elem_nonzero(T v);
template <>
__device__ __forceinline__ bool elem_nonzero<float>(float v) {
    return nz_bits32(__float_as_uint(v));
}
template <>
__device__ __forceinline__ bool elem_nonzero<__nv_bfloat16>(__nv_bfloat16 v) {
    return nz_bits16(__bfloat16_as_ushort(v));
}
template <>
__device__ __forceinline__ bool elem_nonzero<__half>(__half v) {
    return nz_bits16(__half_as_ushort(v));
}

// Nonzero mask of the elements packed in a 16-byte vector, bit e = element e.
template <typename T>
__device__ __forceinline__ uint32_t vec_mask(const uint4 &q) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t m = 0;
    if (sizeof(T) == 4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) m |= nz_bits32(w[i]) ? (1u << i) : 0u;
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            m |= nz_bits16(w[i] & 0xFFFFu) ? (1u << (2 * i)) : 0u;
            m |= nz_bits16(w[i] >> 16) ? (1u << (2 * i + 1)) : 0u;
        }
    }
    return m;
}

// Streaming 16-byte load: no L1 allocation, L2 evict-first (the dense features are read once).
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
    uint4 r;
    asm volatile(
        "{\n\t.reg .b64 pol;\n\t"
        "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
        "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], pol;\n\t}"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__device__ __forceinline__ int warp_inclusive_scan(int v) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, off);
        if ((int)lane_id() >= off) v += t;
    }
    return v;
}

// ------------------------------------------------------------------ row counts
// One warp per row. VEC: rows contiguous and 16-byte aligned.
template <typename T, bool VEC>
__global__ void row_nnz_kernel(const T *__restrict__ f, int64_t M, int64_t N, int64_t sm, int64_t sn,
                               int32_t *__restrict__ row_nnz) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = lane_id();
    const T *rp = f + row * sm;
    int cnt = 0;
    if (VEC) {
        constexpr int EPV = 16 / sizeof(T);
        const int64_t nv = N / EPV;
        for (int64_t v = lane; v < nv; v += 32) cnt += __popc(vec_mask<T>(ld_stream_v4(rp + v * EPV)));
        for (int64_t c = nv * EPV + lane; c < N; c += 32) cnt += elem_nonzero<T>(rp[c]) ? 1 : 0;
    } else {
        for (int64_t c = lane; c < N; c += 32) cnt += elem_nonzero<T>(rp[c * sn]) ? 1 : 0;
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    if (lane == 0) row_nnz[row] = cnt;
}

// ------------------------------------------------------------------ indptr scan
// Single CTA of 1024 threads; tiles of 4096 counts, carry in a register.
// `skip` (may be NULL): when *skip is nonzero every row is written empty (indptr = 0), so a
// decode that follows on the stream reads no entries (the CSR staging overflowed).
__global__ void __launch_bounds__(1024) indptr_scan_kernel(const int32_t *__restrict__ cnt, int64_t M,
                                                           int64_t *__restrict__ indptr, unsigned *err,
                                                           const unsigned *__restrict__ skip) {
    __shared__ long long warp_sums[32];
    __shared__ long long carry_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (skip != nullptr && *skip != 0u) {
        for (int64_t i = tid; i <= M; i += blockDim.x) indptr[i] = 0;
        return;
    }
    if (tid == 0) {
        carry_s = 0;
        indptr[0] = 0;
    }
    __syncthreads();
    for (int64_t base = 0; base < M; base += 4096) {
        long long v[4];
        long long local = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t idx = base + tid * 4 + i;
            int c = idx < M ? cnt[idx] : 0;
            if (c < 0) {
                atomicOr(err, kErrIndptr);
                c = 0;
            }
            local += c;
            v[i] = local;
        }
        // inclusive scan of `local` across the block
        long long s = local;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long t = __shfl_up_sync(0xffffffffu, s, off);
            if (lane >= off) s += t;
        }
        if (lane == 31) warp_sums[warp] = s;
        __syncthreads();
        if (warp == 0) {
            long long w = warp_sums[lane];
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const long long t = __shfl_up_sync(0xffffffffu, w, off);
                if (lane >= off) w += t;
            }
            warp_sums[lane] = w;
        }
        __syncthreads();
        const long long prefix = carry_s + (warp > 0 ? warp_sums[warp - 1] : 0) + (s - local);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t idx = base + tid * 4 + i;
            if (idx < M) indptr[idx + 1] = prefix + v[i];
        }
        __syncthreads();
        if (tid == 0) carry_s += warp_sums[31];
        __syncthreads();
    }
}

// ------------------------------------------------------------------ compaction
// One warp per row, single pass in column order: each lane takes one 16-byte vector
// per step (or one element when the row is strided), a warp prefix sum of the per-lane
// counts gives every nonzero its slot, so the CSR comes out column-sorted. Steps whose
// vectors are all zero (the common case at SAE sparsity) cost one ballot.
template <typename T, typename VT, bool VEC>
__global__ void compact_kernel(const T *__restrict__ f, int64_t M, int64_t N, int64_t sm, int64_t sn,
                               const int64_t *__restrict__ indptr, int32_t *__restrict__ indices,
                               VT *__restrict__ values, unsigned *err) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = lane_id();
    const T *rp = f + row * sm;
    int64_t slot = indptr[row];
    const int64_t end = indptr[row + 1];
    if (VEC) {
        constexpr int EPV = 16 / sizeof(T);
        constexpr int UNROLL = 4;
        const int64_t nv = N / EPV;
        for (int64_t v0 = 0; v0 < nv; v0 += 32 * UNROLL) {
            uint4 q[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const int64_t v = v0 + u * 32 + lane;
                q[u] = v < nv ? ld_stream_v4(rp + v * EPV) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                const uint32_t m = vec_mask<T>(q[u]);
                if (__ballot_sync(0xffffffffu, m != 0) == 0) continue;
                const int c = __popc(m);
                const int incl = warp_inclusive_scan(c);
                int64_t s = slot + incl - c;
                const int64_t col0 = (v0 + u * 32 + lane) * EPV;
                const T *e = reinterpret_cast<const T *>(&q[u]);
#pragma unroll
                for (int t = 0; t < EPV; ++t) {
                    if (m & (1u << t)) {
                        if (s < end) {
                            indices[s] = (int32_t)(col0 + t);
                            values[s] = from_f32<VT>(to_f32(e[t]));
                        }
                        ++s;
                    }
                }
                slot += __shfl_sync(0xffffffffu, incl, 31);
            }
        }
        // Ragged tail (N not a multiple of the vector width): one element per lane.
        for (int64_t c0 = nv * EPV; c0 < N; c0 += 32) {
            const int64_t c = c0 + lane;
            const bool nz = c < N && elem_nonzero<T>(rp[c]);
            const uint32_t b = __ballot_sync(0xffffffffu, nz);
            if (nz) {
                const int64_t s = slot + __popc(b & ((1u << lane) - 1u));
                if (s < end) {
                    indices[s] = (int32_t)c;
                    values[s] = from_f32<VT>(to_f32(rp[c]));
                }
            }
            slot += __popc(b);
        }
    } else {
        for (int64_t c0 = 0; c0 < N; c0 += 32) {
            const int64_t c = c0 + lane;
            T x{};
            const bool nz = c < N && elem_nonzero<T>(x = rp[c * sn]);
            const uint32_t b = __ballot_sync(0xffffffffu, nz);
            if (nz) {
                const int64_t s = slot + __popc(b & ((1u << lane) - 1u));
                if (s < end) {
                    indices[s] = (int32_t)c;
                    values[s] = from_f32<VT>(to_f32(x));
                }
            }
            slot += __popc(b);
        }
    }
    if (lane == 0 && slot != end) atomicOr(err, kErrIndptr);
}

// ------------------------------------------------------------------ sparse decode
// out[m, d] = b_dec[d] + sum_j val[j] * W[idx[j], d]
// One warp per (row, D-slice). Lane l owns V 16-byte vectors of the slice at
// slice_start + (v*32 + l)*EPV, so each gathered W row is read as 32 x 16 B coalesced
// segments; the row's (index, value) pairs are read 32 at a time and broadcast with
// shuffles, and two W rows are kept in flight per step.
// The slice width is chosen on the host so that one slice of every W_dec row fits in L2
// (kDecodeL2Budget); the grid runs all rows of slice 0, then slice 1, ..., so each W_dec
// row slice comes from HBM about once and its other uses hit L2.
// The kernel is bound by instruction issue, not by L2 (ncu at config 2, 4096 tokens:
// issue slots 75% busy, L2 throughput 37% of peak), so the per-element work is kept to
// the fewest instructions: accumulators are fp32 pairs updated by one packed FMA
// (__ffma2_rn, two IEEE fp32 FMAs, each bit-identical to fmaf) per two W elements, and
// bf16 elements are widened by placing their bits in the high half of a 32-bit word (exact).
#ifndef SF_DECODE_WPOL
#define SF_DECODE_WPOL 0  // W_dec loads: 0 default L2 policy, 1 evict_last
#endif
#ifndef SF_DECODE_OPOL
#define SF_DECODE_OPOL 1  // output stores: 0 default L2 policy, 1 evict_first
#endif
#ifndef SF_DECODE_MATH
#define SF_DECODE_MATH 1  // 0 scalar fmaf per element; 1 packed fp32 FMA per element pair
#endif
__device__ __forceinline__ uint4 ld_w_v4(const void *p, uint64_t pol) {
    if (SF_DECODE_WPOL) return ld_nc_v4_hint(p, pol);
    return __ldg(reinterpret_cast<const uint4 *>(p));
}

// The two W elements of 32-bit word `w` of a gathered 16-bit vector, widened to fp32 (exact).
template <typename WT>
__device__ __forceinline__ float2 widen_pair(uint32_t w) {
    if constexpr (std::is_same<WT, __nv_bfloat16>::value) {
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    } else {
        __half2 h;
        memcpy(&h, &w, 4);
        return __half22float2(h);
    }
}

// acc[v][i] += a * (elements 2i, 2i+1 of vector q[v]).
template <typename WT, int V, int NP>
__device__ __forceinline__ void fma_vectors(float2 (&acc)[V][NP], float a, const uint4 (&q)[V],
                                            const bool (&active)[V]) {
    const float2 aa = make_float2(a, a);
#pragma unroll
    for (int v = 0; v < V; ++v) {
        if (!active[v]) continue;
        const uint32_t w[4] = {q[v].x, q[v].y, q[v].z, q[v].w};
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            float2 wf;
            if constexpr (sizeof(WT) == 4)
                wf = make_float2(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1]));
            else
                wf = widen_pair<WT>(w[i]);
            if (SF_DECODE_MATH == 1) {
                acc[v][i] = __ffma2_rn(aa, wf, acc[v][i]);
            } else {
                acc[v][i].x = fmaf(a, wf.x, acc[v][i].x);
                acc[v][i].y = fmaf(a, wf.y, acc[v][i].y);
            }
        }
    }
}

#ifndef SF_DECODE_MIN_BLOCKS
#define SF_DECODE_MIN_BLOCKS 1  // V <= 2: resident 128-thread blocks per SM the register budget must allow
#endif
template <typename WT, typename VT, typename OT, int V>
__global__ void __launch_bounds__(128, V <= 2 ? SF_DECODE_MIN_BLOCKS : 1) decode_vec_kernel(const int64_t *__restrict__ indptr,
                                                         const int32_t *__restrict__ indices,
                                                         const VT *__restrict__ values, const WT *__restrict__ W,
                                                         int64_t ldw, int64_t d_sae, const void *b_dec, int b_dtype,
                                                         int64_t b_stride, OT *__restrict__ out, int64_t ldo,
                                                         int64_t M, int64_t D, int out_vec, unsigned *err) {
    constexpr int EPV = 16 / sizeof(WT);
    constexpr int NP = EPV / 2;  // element pairs per vector
    constexpr int SLICE = 32 * V * EPV;
    const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = lane_id();
    const int64_t d0 = (int64_t)blockIdx.y * SLICE;
    const int64_t start = indptr[row], end = indptr[row + 1];

    float2 acc[V][NP];
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
        for (int i = 0; i < NP; ++i) acc[v][i] = make_float2(0.f, 0.f);

    bool active[V];
#pragma unroll
    for (int v = 0; v < V; ++v) active[v] = d0 + (int64_t)(v * 32 + lane) * EPV < D;
    const uint64_t wpol = SF_DECODE_WPOL ? l2_policy_evict_last() : 0ull;

    bool bad = false;
    for (int64_t j0 = start; j0 < end; j0 += 32) {
        const int64_t j = j0 + lane;
        int32_t my_idx = 0;
        float my_val = 0.f;
        if (j < end) {
            my_idx = __ldg(indices + j);
            my_val = to_f32(values[j]);
            if (my_idx < 0 || (int64_t)my_idx >= d_sae) {
                bad = true;
                my_idx = 0;
                my_val = 0.f;
            }
        }
        const int n = (end - j0) < 32 ? (int)(end - j0) : 32;
        int t = 0;
        for (; t + 2 <= n; t += 2) {
            const int i0 = __shfl_sync(0xffffffffu, my_idx, t);
            const int i1 = __shfl_sync(0xffffffffu, my_idx, t + 1);
            const float a0 = __shfl_sync(0xffffffffu, my_val, t);
            const float a1 = __shfl_sync(0xffffffffu, my_val, t + 1);
            const WT *r0 = W + (int64_t)i0 * ldw + d0 + lane * EPV;
            const WT *r1 = W + (int64_t)i1 * ldw + d0 + lane * EPV;
            uint4 q0[V], q1[V];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                q0[v] = active[v] ? ld_w_v4(r0 + v * 32 * EPV, wpol) : make_uint4(0, 0, 0, 0);
                q1[v] = active[v] ? ld_w_v4(r1 + v * 32 * EPV, wpol) : make_uint4(0, 0, 0, 0);
            }
            fma_vectors<WT, V, NP>(acc, a0, q0, active);
            fma_vectors<WT, V, NP>(acc, a1, q1, active);
        }
        if (t < n) {
            const int i0 = __shfl_sync(0xffffffffu, my_idx, t);
            const float a0 = __shfl_sync(0xffffffffu, my_val, t);
            const WT *r0 = W + (int64_t)i0 * ldw + d0 + lane * EPV;
            uint4 q0[V];
#pragma unroll
            for (int v = 0; v < V; ++v) q0[v] = active[v] ? ld_w_v4(r0 + v * 32 * EPV, wpol) : make_uint4(0, 0, 0, 0);
            fma_vectors<WT, V, NP>(acc, a0, q0, active);
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(err, kErrIndex);

#pragma unroll
    for (int v = 0; v < V; ++v) {
        if (!active[v]) continue;
        const int64_t d = d0 + (int64_t)(v * 32 + lane) * EPV;
        float r[EPV];
#pragma unroll
        for (int e = 0; e < EPV; ++e)
            r[e] = ((e & 1) ? acc[v][e / 2].y : acc[v][e / 2].x) +
                   (b_dec ? load_as_f32(b_dec, b_dtype, (d + e) * b_stride) : 0.f);
        OT *dst = out + row * ldo + d;
        if (out_vec && sizeof(OT) * EPV >= 8) {
            if (sizeof(OT) == sizeof(WT)) {
                uint4 pk;
                OT *o = reinterpret_cast<OT *>(&pk);
#pragma unroll
                for (int e = 0; e < EPV; ++e) o[e] = from_f32<OT>(r[e]);
                if (SF_DECODE_OPOL)
                    st_global_v4_hint(dst, pk, l2_policy_evict_first());
                else
                    *reinterpret_cast<uint4 *>(dst) = pk;
            } else {
#pragma unroll
                for (int e = 0; e < EPV; ++e) dst[e] = from_f32<OT>(r[e]);
            }
        } else {
#pragma unroll
            for (int e = 0; e < EPV; ++e) dst[e] = from_f32<OT>(r[e]);
        }
    }
}

// Generic strided decode: one warp per (row, 32-column block group), scalar loads.
template <typename WT, typename VT, typename OT>
__global__ void __launch_bounds__(128) decode_generic_kernel(const int64_t *__restrict__ indptr,
                                                             const int32_t *__restrict__ indices,
                                                             const VT *__restrict__ values, const WT *__restrict__ W,
                                                             int64_t swn, int64_t swd, int64_t d_sae, const void *b_dec,
                                                             int b_dtype, int64_t b_stride, OT *__restrict__ out,
                                                             int64_t som, int64_t sod, int64_t M, int64_t D,
                                                             unsigned *err) {
    constexpr int PER_LANE = 8;
    const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (row >= M) return;
    const int lane = lane_id();
    const int64_t d0 = (int64_t)blockIdx.y * 32 * PER_LANE;
    const int64_t start = indptr[row], end = indptr[row + 1];
    float acc[PER_LANE];
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) acc[i] = 0.f;
    bool bad = false;
    for (int64_t j = start; j < end; ++j) {
        int64_t idx = __ldg(indices + j);
        float a = to_f32(values[j]);
        if (idx < 0 || idx >= d_sae) {
            bad = true;
            continue;
        }
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i) {
            const int64_t d = d0 + i * 32 + lane;
            if (d < D) acc[i] = fmaf(a, to_f32(W[idx * swn + d * swd]), acc[i]);
        }
    }
    if (bad && lane == 0) atomicOr(err, kErrIndex);
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const int64_t d = d0 + i * 32 + lane;
        if (d < D) {
            const float b = b_dec ? load_as_f32(b_dec, b_dtype, d * b_stride) : 0.f;
            out[row * som + d * sod] = from_f32<OT>(acc[i] + b);
        }
    }
}

// ------------------------------------------------------------------ CSR placement
// Moves the staged (column, value) pairs of the encode-straight-to-CSR path into canonical
// CSR: one warp per row scans the row's per-tile counts (tiles in column order) to find
// each tile's output slot and copies the tile's staged run there.
template <typename VT>
__global__ void csr_place_kernel(const int32_t *__restrict__ tile_cnt, const int32_t *__restrict__ tile_off,
                                 int64_t n_tiles, const int32_t *__restrict__ stage_idx,
                                 const VT *__restrict__ stage_val, int64_t stage_cap,
                                 const int64_t *__restrict__ indptr, int64_t M, int32_t *__restrict__ indices,
                                 VT *__restrict__ values, unsigned *err, const unsigned *__restrict__ skip) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= M) return;
    if (skip != nullptr && *skip != 0u) return;  // staging overflowed: nothing to place
    const int lane = lane_id();
    const int64_t start = indptr[row], end = indptr[row + 1];
    int64_t run = start;
    bool bad = false;
    for (int64_t t0 = 0; t0 < n_tiles; t0 += 32) {
        const int64_t t = t0 + lane;
        int c = t < n_tiles ? tile_cnt[row * n_tiles + t] : 0;
        if (c < 0 || c > kCsrTile) {  // a cell the encoder did not write: report, never follow
            bad = true;
            c = 0;
        }
        const int incl = warp_inclusive_scan(c);
        if (c > 0) {
            const int64_t dst = run + incl - c;
            const int64_t src = tile_off[row * n_tiles + t];
            if (dst + c > end || src < 0 || src + c > stage_cap) {
                bad = true;
            } else {
                for (int j = 0; j < c; ++j) {
                    indices[dst + j] = stage_idx[src + j];
                    values[dst + j] = stage_val[src + j];
                }
            }
        }
        run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (__any_sync(0xffffffffu, bad || run != end) && lane == 0) atomicOr(err, kErrIndptr);
}

// ------------------------------------------------------------------ top-k merge
// One warp per row: k rounds of a warp-wide max over the row's n_chunks*k packed
// (value, ~index) keys; the winner is removed from its lane's registers... kept in
// shared memory so any candidate count works.
template <typename VT>
__global__ void __launch_bounds__(128) topk_merge_kernel(const unsigned long long *__restrict__ cand, int64_t M,
                                                         int ncand, int k, int32_t *__restrict__ out_idx,
                                                         VT *__restrict__ out_val) {
    extern __shared__ unsigned long long s_cand[];  // [4 warps][ncand]
    const int w = threadIdx.x >> 5;
    const int lane = lane_id();
    const int64_t row = (int64_t)blockIdx.x * 4 + w;
    if (row >= M) return;
    unsigned long long *my = s_cand + (size_t)w * ncand;
    const unsigned long long *src = cand + row * ncand;
    for (int i = lane; i < ncand; i += 32) my[i] = src[i];
    __syncwarp();
    for (int r = 0; r < k; ++r) {
        unsigned long long best = 0;
        int best_pos = -1;
        for (int i = lane; i < ncand; i += 32) {
            const unsigned long long q = my[i];
            if (best_pos < 0 || q > best) {
                best = q;
                best_pos = i;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int op = __shfl_xor_sync(0xffffffffu, best_pos, off);
            if (op >= 0 && (best_pos < 0 || ob > best)) {
                best = ob;
                best_pos = op;
            }
        }
        if (lane == 0) {
            my[best_pos] = 0ull;
            const uint32_t col = 0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull);
            const float val = __uint_as_float(static_cast<uint32_t>(best >> 32));
            out_idx[row * k + r] = (int32_t)col;
            out_val[row * k + r] = from_f32<VT>(val);
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------ dense-row top-k
// One CTA of 128 threads per row of a dense ReLU output f (values >= 0): each thread keeps
// the k largest packed (value, ~column) keys of its columns in shared memory, sorts them,
// and k rounds of a block-wide max emit the row's top-k sorted by value descending, ties
// by lower column. Used for fp32 IEEE TopK and for k beyond the fused epilogue's limit.
template <typename T, typename VT>
__global__ void __launch_bounds__(128) topk_rows_kernel(const T *__restrict__ f, int64_t N, int64_t ld, int k,
                                                        int32_t *__restrict__ out_idx, VT *__restrict__ out_val) {
    extern __shared__ unsigned long long lists[];  // [k][128]
    __shared__ unsigned long long warp_best[4];
    __shared__ unsigned long long winner;
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    const int64_t row = blockIdx.x;
    const T *rp = f + row * ld;
    for (int s = 0; s < k; ++s) lists[s * 128 + t] = 0ull;
    unsigned long long min_key = 0;
    int min_slot = 0;
    for (int64_t c = t; c < N; c += 128) {
        const uint32_t bits = __float_as_uint(to_f32(rp[c])) & 0x7FFFFFFFu;
        const unsigned long long key =
            (static_cast<unsigned long long>(bits) << 32) | (0xFFFFFFFFull - static_cast<unsigned long long>(c));
        if (key > min_key) {
            lists[min_slot * 128 + t] = key;
            min_key = ~0ull;
            for (int s = 0; s < k; ++s) {
                const unsigned long long q = lists[s * 128 + t];
                if (q < min_key) {
                    min_key = q;
                    min_slot = s;
                }
            }
        }
    }
    // sort this thread's list descending (insertion sort, k <= a few hundred)
    for (int i = 1; i < k; ++i) {
        const unsigned long long v = lists[i * 128 + t];
        int j = i - 1;
        while (j >= 0 && lists[j * 128 + t] < v) {
            lists[(j + 1) * 128 + t] = lists[j * 128 + t];
            --j;
        }
        lists[(j + 1) * 128 + t] = v;
    }
    int head = 0;
    for (int r = 0; r < k; ++r) {
        unsigned long long mine = head < k ? lists[head * 128 + t] : 0ull;
        unsigned long long best = mine;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
            best = o > best ? o : best;
        }
        if (lane == 0) warp_best[w] = best;
        __syncthreads();
        if (t == 0) {
            unsigned long long b = warp_best[0];
            for (int i = 1; i < 4; ++i) b = warp_best[i] > b ? warp_best[i] : b;
            winner = b;
            const uint32_t col = 0xFFFFFFFFu - static_cast<uint32_t>(b & 0xFFFFFFFFull);
            out_idx[row * k + r] = (int32_t)col;
            out_val[row * k + r] = from_f32<VT>(__uint_as_float(static_cast<uint32_t>(b >> 32)));
        }
        __syncthreads();
        if (head < k && mine == winner && mine != 0ull) ++head;
    }
}

template <typename F>
int by_dtype(int dt, F &&f) {
    if (dt == SF_F32) return f(float{});
    if (dt == SF_BF16) return f(__nv_bfloat16{});
    return f(__half{});
}

}  // namespace

// =======================================================================================
// Launchers (called from api.cu)

int launch_row_nnz(const sf_matrix &f, int32_t *row_nnz, cudaStream_t s) {
    const int64_t M = f.rows;
    if (M == 0) return SF_OK;
    const unsigned blocks = (unsigned)((M + 7) / 8);
    return by_dtype(f.dtype, [&](auto tag) {
        using T = decltype(tag);
        const T *p = reinterpret_cast<const T *>(f.data);
        const bool vec = f.stride_col == 1 && ((f.stride_row * (int64_t)sizeof(T)) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
        if (vec)
            row_nnz_kernel<T, true><<<blocks, 256, 0, s>>>(p, M, f.cols, f.stride_row, f.stride_col, row_nnz);
        else
            row_nnz_kernel<T, false><<<blocks, 256, 0, s>>>(p, M, f.cols, f.stride_row, f.stride_col, row_nnz);
        return check_cuda(cudaGetLastError(), "row_nnz launch");
    });
}

int launch_indptr(const int32_t *cnt, int64_t M, int64_t *indptr, cudaStream_t s, const unsigned *skip) {
    indptr_scan_kernel<<<1, 1024, 0, s>>>(cnt, M, indptr, device_error_word(), skip);
    return check_cuda(cudaGetLastError(), "indptr scan launch");
}

int launch_compact(const sf_matrix &f, const int64_t *indptr, int32_t *indices, void *values, int vdt,
                   cudaStream_t s) {
    const int64_t M = f.rows;
    if (M == 0) return SF_OK;
    const unsigned blocks = (unsigned)((M + 7) / 8);
    unsigned *err = device_error_word();
    return by_dtype(f.dtype, [&](auto tag) {
        using T = decltype(tag);
        const T *p = reinterpret_cast<const T *>(f.data);
        const bool vec = f.stride_col == 1 && ((f.stride_row * (int64_t)sizeof(T)) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
        return by_dtype(vdt, [&](auto vtag) {
            using VT = decltype(vtag);
            VT *vals = reinterpret_cast<VT *>(values);
            if (vec)
                compact_kernel<T, VT, true>
                    <<<blocks, 256, 0, s>>>(p, M, f.cols, f.stride_row, f.stride_col, indptr, indices, vals, err);
            else
                compact_kernel<T, VT, false>
                    <<<blocks, 256, 0, s>>>(p, M, f.cols, f.stride_row, f.stride_col, indptr, indices, vals, err);
            return check_cuda(cudaGetLastError(), "compact launch");
        });
    });
}

// Bytes of W_dec one decode slice may span over all d_sae rows: half of the 126 MB L2, the
// rest left to the CSR, the output stream and the other slice in flight at slice boundaries.
constexpr int64_t kDecodeL2Budget = 64ll << 20;

template <typename WT, typename VT, typename OT, int V>
static int launch_decode_v(const int64_t *indptr, const int32_t *indices, const VT *values, const sf_matrix &W,
                           const sf_vector *b, const sf_matrix &out, int64_t M, int out_vec, cudaStream_t s) {
    constexpr int EPV = 16 / sizeof(WT);
    const int64_t D = W.cols;
    const int64_t slice = 32 * V * EPV;
    dim3 grid((unsigned)((M + 3) / 4), (unsigned)((D + slice - 1) / slice));
    decode_vec_kernel<WT, VT, OT, V><<<grid, 128, 0, s>>>(
        indptr, indices, values, reinterpret_cast<const WT *>(W.data), W.stride_row, W.rows,
        b ? b->data : nullptr, b ? b->dtype : 0, b ? b->stride : 0, reinterpret_cast<OT *>(const_cast<void *>(out.data)),
        out.stride_row, M, D, out_vec, device_error_word());
    return check_cuda(cudaGetLastError(), "decode launch");
}

int launch_decode(const int64_t *indptr, int64_t M, const int32_t *indices, const void *values, int vdt,
                  const sf_matrix &W, const sf_vector *b, const sf_matrix &out, cudaStream_t s) {
    if (M == 0 || W.cols == 0) return SF_OK;
    const int64_t D = W.cols;
    return by_dtype(W.dtype, [&](auto wtag) {
        using WT = decltype(wtag);
        constexpr int EPV = 16 / sizeof(WT);
        return by_dtype(vdt, [&](auto vtag) {
            using VT = decltype(vtag);
            const VT *vals = reinterpret_cast<const VT *>(values);
            return by_dtype(out.dtype, [&](auto otag) {
                using OT = decltype(otag);
                const bool vec = W.stride_col == 1 && (W.stride_row % EPV) == 0 && (D % EPV) == 0 &&
                                 (reinterpret_cast<uintptr_t>(W.data) & 15u) == 0 && out.stride_col == 1;
                if (vec) {
                    const int out_vec = ((out.stride_row * (int64_t)sizeof(OT)) % 16 == 0) &&
                                        (reinterpret_cast<uintptr_t>(out.data) & 15u) == 0;
                    // Vectors per lane: the widest slice (<= 8 vectors per lane) whose bytes
                    // over all d_sae rows of W_dec fit the L2 budget (at least 1 vector),
                    // then spread evenly over the slices that width needs.
                    const int64_t nvec = D / EPV;
                    const int64_t row_slice_budget = kDecodeL2Budget / std::max<int64_t>(W.rows, 1);
                    const int64_t vmax = std::min<int64_t>(8, std::max<int64_t>(1, row_slice_budget / (32 * 16)));
                    const int64_t slices = (nvec + 32 * vmax - 1) / (32 * vmax);
#ifdef SF_DECODE_V
                    const int V = SF_DECODE_V;  // tuning builds only
#else
                    const int V = (int)((nvec + 32 * slices - 1) / (32 * slices));
#endif
                    switch (V) {
                        case 1: return launch_decode_v<WT, VT, OT, 1>(indptr, indices, vals, W, b, out, M, out_vec, s);
                        case 2: return launch_decode_v<WT, VT, OT, 2>(indptr, indices, vals, W, b, out, M, out_vec, s);
                        case 3: return launch_decode_v<WT, VT, OT, 3>(indptr, indices, vals, W, b, out, M, out_vec, s);
                        case 4: return launch_decode_v<WT, VT, OT, 4>(indptr, indices, vals, W, b, out, M, out_vec, s);
                        case 5: return launch_decode_v<WT, VT, OT, 5>(indptr, indices, vals, W, b, out, M, out_vec, s);
                        case 6: return launch_decode_v<WT, VT, OT, 6>(indptr, indices, vals, W, b, out, M, out_vec, s);
                        case 7: return launch_decode_v<WT, VT, OT, 7>(indptr, indices, vals, W, b, out, M, out_vec, s);
                        default: return launch_decode_v<WT, VT, OT, 8>(indptr, indices, vals, W, b, out, M, out_vec, s);
                    }
                }
                dim3 grid((unsigned)((M + 3) / 4), (unsigned)((D + 255) / 256));
                decode_generic_kernel<WT, VT, OT><<<grid, 128, 0, s>>>(
                    indptr, indices, vals, reinterpret_cast<const WT *>(W.data), W.stride_row, W.stride_col, W.rows,
                    b ? b->data : nullptr, b ? b->dtype : 0, b ? b->stride : 0,
                    reinterpret_cast<OT *>(const_cast<void *>(out.data)), out.stride_row, out.stride_col, M, D,
                    device_error_word());
                return check_cuda(cudaGetLastError(), "decode launch");
            });
        });
    });
}

int launch_topk_merge(const unsigned long long *cand, int64_t M, int ncand, int k, int32_t *out_idx, void *out_val,
                      int vdt, cudaStream_t s) {
    if (M == 0) return SF_OK;
    const size_t smem = (size_t)4 * ncand * sizeof(unsigned long long);
    return by_dtype(vdt, [&](auto vtag) {
        using VT = decltype(vtag);
        auto kern = topk_merge_kernel<VT>;
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(topk_merge)");
        }
        kern<<<(unsigned)((M + 3) / 4), 128, smem, s>>>(cand, M, ncand, k, out_idx, reinterpret_cast<VT *>(out_val));
        return check_cuda(cudaGetLastError(), "topk merge launch");
    });
}

}  // namespace sf

namespace sf {
int launch_topk_rows(const sf_matrix &f, int k, int32_t *out_idx, void *out_val, int vdt, cudaStream_t s) {
    if (f.rows == 0) return SF_OK;
    const size_t smem = (size_t)k * 128 * sizeof(unsigned long long);
    return by_dtype(f.dtype, [&](auto tag) {
        using T = decltype(tag);
        return by_dtype(vdt, [&](auto vtag) {
            using VT = decltype(vtag);
            auto kern = topk_rows_kernel<T, VT>;
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(topk_rows)");
            kern<<<(unsigned)f.rows, 128, smem, s>>>(reinterpret_cast<const T *>(f.data), f.cols, f.stride_row, k,
                                                     out_idx, reinterpret_cast<VT *>(out_val));
            return check_cuda(cudaGetLastError(), "topk rows launch");
        });
    });
}
}  // namespace sf

namespace sf {
int launch_csr_place(const int32_t *tile_cnt, const int32_t *tile_off, int64_t n_tiles, const int32_t *stage_idx,
                     const void *stage_val, int64_t stage_cap, int vdt, const int64_t *indptr, int64_t M,
                     int32_t *indices, void *values, cudaStream_t s, const unsigned *skip) {
    if (M == 0) return SF_OK;
    return by_dtype(vdt, [&](auto tag) {
        using VT = decltype(tag);
        csr_place_kernel<VT><<<(unsigned)((M + 7) / 8), 256, 0, s>>>(
            tile_cnt, tile_off, n_tiles, stage_idx, reinterpret_cast<const VT *>(stage_val), stage_cap, indptr, M,
            indices, reinterpret_cast<VT *>(values), device_error_word(), skip);
        return check_cuda(cudaGetLastError(), "csr place launch");
    });
}
}  // namespace sf
