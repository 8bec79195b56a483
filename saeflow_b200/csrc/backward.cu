// Backward of the sparse SAE forward, for training on sparse features (saeflow's roadmap,
// README.md:244; the reference itself has no backward kernels).
//
//   forward:  pre = (x - b_dec) @ W_enc + b_enc ; f = act(pre) as CSR ; x_hat = f @ W_dec + b_dec
//   backward, given g = dL/dx_hat [M, d_in]:
//     dpre[e]  = g[row(e)] . W_dec[col(e)]            for each CSR entry e with f_e != 0
//     dW_dec[j] = sum_{e in column j} f_e * g[row(e)]
//     dW_enc^T[j] = sum_{e in column j} dpre_e * xs[row(e)],   db_enc[j] = sum dpre_e
//     dx = dpre @ W_enc^T (a CSR decode against W_enc^T),       db_dec = sum_m (g[m] - dx[m])
// The gradient reaches only the active features: ReLU and JumpReLU pass it where f != 0,
// TopK where a selected value is positive. (The JumpReLU threshold gets none here.)
//
// Column-wise work runs on the CSR transposed: a column count (atomics), the indptr scan of
// sparse.cu, a scatter that records each entry's row and CSR position, and a sort of each
// column's entries by row, so the column view is canonical (the CSR of the transpose) and the
// per-column sums are taken in one fixed order.
//
// The column gather (dW_dec with dpre fused into the same pass, then dW_enc^T) is
// csc_gather_kernel: rows of R stream into shared memory by cp.async.bulk, one copy per
// gathered row, so the bytes in flight are bounded by shared memory rather than registers.
#include <algorithm>
#include <climits>
#include <type_traits>

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

// Rows ascending within each column, so the column view (and every sum taken over it in
// order) does not depend on the scatter's atomic timing. A column of at most 128 entries is
// ranked by one warp: each lane holds up to four of its rows and counts the smaller rows of the
// column, broadcast one at a time by shuffles. Longer columns are queued for
// csc_sort_large_kernel.
constexpr int kSortWarpMax = 128;
__global__ void csc_sort_small_kernel(const int64_t *__restrict__ col_ptr, int64_t n_cols,
                                      const int32_t *__restrict__ trow, const int64_t *__restrict__ tperm,
                                      int32_t *__restrict__ row_idx, int64_t *__restrict__ perm,
                                      int32_t *__restrict__ col_idx, int32_t *__restrict__ large) {
    constexpr int Q = kSortWarpMax / 32;
    const int lane = lane_id();
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t j = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); j < n_cols; j += warps) {
        const int64_t p0 = col_ptr[j];
        const int n = (int)min(col_ptr[j + 1] - p0, (int64_t)kSortWarpMax + 1);
        if (n > kSortWarpMax) {
            if (lane == 0) large[1 + atomicAdd(large, 1)] = (int32_t)j;
            continue;
        }
        int32_t r[Q];
        int rank[Q];
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const int i = q * 32 + lane;
            r[q] = i < n ? trow[p0 + i] : INT32_MAX;
            rank[q] = 0;
        }
#pragma unroll
        for (int qt = 0; qt < Q; ++qt) {
            if (qt * 32 >= n) break;
            const int m = min(32, n - qt * 32);
            for (int t = 0; t < m; ++t) {
                const int32_t rt = __shfl_sync(0xffffffffu, r[qt], t);
                const int it = qt * 32 + t;
#pragma unroll
                for (int q = 0; q < Q; ++q) rank[q] += (rt < r[q] || (rt == r[q] && it < q * 32 + lane)) ? 1 : 0;
            }
        }
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const int i = q * 32 + lane;
            if (i < n) {
                row_idx[p0 + rank[q]] = r[q];
                perm[p0 + rank[q]] = tperm[p0 + i];
                if (col_idx != nullptr) col_idx[p0 + rank[q]] = (int32_t)j;
            }
        }
    }
}

// Columns of more than kSortWarpMax entries, one CTA each: mark the column's rows in a shared-memory
// bitmap (a window of up to 32 * words rows at a time), prefix-count the bitmap's words, and
// place each entry at its row's rank. A row present twice in a column (a malformed CSR) sets
// bit 4 of the device error; the placement then stays inside the column.
constexpr int kSortThreads = 256;
__global__ void __launch_bounds__(kSortThreads) csc_sort_large_kernel(
    const int64_t *__restrict__ col_ptr, const int32_t *__restrict__ trow, const int64_t *__restrict__ tperm,
    int32_t *__restrict__ row_idx, int64_t *__restrict__ perm, int32_t *__restrict__ col_idx,
    const int32_t *__restrict__ large, int words, unsigned *err) {
    extern __shared__ uint32_t sm_words[];
    uint32_t *bm = sm_words;                                        // [words]
    int32_t *pre = reinterpret_cast<int32_t *>(sm_words + words);  // [words]
    __shared__ int32_t red[2][kSortThreads / 32];
    __shared__ int32_t scan[kSortThreads / 32];
    const int tid = threadIdx.x, lane = lane_id(), wid = tid >> 5;
    const int n_large = large[0];
    for (int li = blockIdx.x; li < n_large; li += gridDim.x) {
        const int64_t j = large[1 + li];
        const int64_t p0 = col_ptr[j], n = col_ptr[j + 1] - p0;
        int32_t lo = INT32_MAX, hi = -1;
        for (int64_t i = tid; i < n; i += kSortThreads) {
            const int32_t r = trow[p0 + i];
            lo = min(lo, r);
            hi = max(hi, r);
        }
        lo = __reduce_min_sync(0xffffffffu, lo);
        hi = __reduce_max_sync(0xffffffffu, hi);
        if (lane == 0) red[0][wid] = lo, red[1][wid] = hi;
        __syncthreads();
        lo = red[0][0];
        hi = red[1][0];
        for (int w = 1; w < kSortThreads / 32; ++w) lo = min(lo, red[0][w]), hi = max(hi, red[1][w]);
        __syncthreads();
        int64_t base = 0;  // entries placed by earlier windows
        for (int64_t w0 = (int64_t)(lo & ~31); w0 <= hi; w0 += (int64_t)words * 32) {
            const int nw = (int)min((int64_t)words, ((int64_t)hi - w0) / 32 + 1);
            for (int w = tid; w < nw; w += kSortThreads) bm[w] = 0u;
            __syncthreads();
            for (int64_t i = tid; i < n; i += kSortThreads) {
                const int64_t r = trow[p0 + i] - w0;
                if (r >= 0 && r < (int64_t)nw * 32) {
                    const uint32_t bit = 1u << (r & 31);
                    if (atomicOr(&bm[r >> 5], bit) & bit) atomicOr(err, kErrIndptr);
                }
            }
            __syncthreads();
            // exclusive prefix of popc over the window's words: contiguous chunks per thread
            const int per = (nw + kSortThreads - 1) / kSortThreads;
            const int wb = min(nw, tid * per), we = min(nw, wb + per);
            int sum = 0;
            for (int w = wb; w < we; ++w) sum += __popc(bm[w]);
            int incl = sum;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += t;
            }
            if (lane == 31) scan[wid] = incl;
            __syncthreads();
            int before = incl - sum;
            for (int w = 0; w < wid; ++w) before += scan[w];
            int total = 0;
            for (int w = 0; w < kSortThreads / 32; ++w) total += scan[w];
            for (int w = wb; w < we; ++w) {
                pre[w] = before;
                before += __popc(bm[w]);
            }
            __syncthreads();
            for (int64_t i = tid; i < n; i += kSortThreads) {
                const int32_t r = trow[p0 + i];
                const int64_t rr = (int64_t)r - w0;
                if (rr >= 0 && rr < (int64_t)nw * 32) {
                    const int w = (int)(rr >> 5);
                    const int64_t rank = base + pre[w] + __popc(bm[w] & ((1u << (rr & 31)) - 1u));
                    if (rank < n) {
                        row_idx[p0 + rank] = r;
                        perm[p0 + rank] = tperm[p0 + i];
                        if (col_idx != nullptr) col_idx[p0 + rank] = (int32_t)j;
                    }
                }
            }
            base += total;
            __syncthreads();
        }
    }
}

// ------------------------------------------------------------------ output stores
// EPV consecutive elements of an output row in a runtime dtype; `vec` when the row start is
// 16-byte aligned (the element offset i is a multiple of EPV).
template <int EPV>
__device__ __forceinline__ void store_chunk(void *out, int odt, int64_t i, const float (&f)[EPV], bool vec) {
    if (odt == SF_F32) {
        float *o = reinterpret_cast<float *>(out) + i;
        if (vec) {
#pragma unroll
            for (int e = 0; e < EPV; e += 4)
                *reinterpret_cast<float4 *>(o + e) = make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]);
        } else {
#pragma unroll
            for (int e = 0; e < EPV; ++e) o[e] = f[e];
        }
        return;
    }
    uint32_t w[EPV / 2];
#pragma unroll
    for (int e = 0; e < EPV; e += 2) {
        if (odt == SF_BF16) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(f[e], f[e + 1]);
            w[e / 2] = *reinterpret_cast<const uint32_t *>(&h);
        } else {
            const __half2 h = __floats2half2_rn(f[e], f[e + 1]);
            w[e / 2] = *reinterpret_cast<const uint32_t *>(&h);
        }
    }
    uint16_t *o = reinterpret_cast<uint16_t *>(out) + i;
    if (vec) {
        if constexpr (EPV == 8) {
            *reinterpret_cast<uint4 *>(o) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
            *reinterpret_cast<uint2 *>(o) = make_uint2(w[0], w[1]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < EPV; e += 2) {
            o[e] = (uint16_t)(w[e / 2] & 0xffffu);
            o[e + 1] = (uint16_t)(w[e / 2] >> 16);
        }
    }
}

__device__ __forceinline__ void store_one(void *out, int odt, int64_t i, float v) {
    if (odt == SF_F32) {
        reinterpret_cast<float *>(out)[i] = v;
    } else if (odt == SF_BF16) {
        reinterpret_cast<__nv_bfloat16 *>(out)[i] = __float2bfloat16_rn(v);
    } else {
        reinterpret_cast<__half *>(out)[i] = __float2half_rn(v);
    }
}

// One contiguous global -> shared copy completing on `bar` (16-byte aligned ends, size a
// multiple of 16).
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_count(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// mbar_wait for short hand-overs: each try_wait may suspend the warp (until the phase
// completes, or for at most kSuspendNs), so a warp that runs ahead does not take issue slots
// from the warps it waits for. Same time limit and abort protocol as mbar_wait.
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_wait_suspend(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                                  unsigned *err_word) {
    const uint32_t a = smem_u32(bar);
    unsigned long long t0 = 0;
    for (uint32_t i = 0;; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred P;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
            "selp.b32 %0, 1, 0, P;\n\t}"
            : "=r"(ok)
            : "r"(a), "r"(parity), "r"(kSuspendNs)
            : "memory");
        if (ok) return true;
        if (*abort_flag) return false;
        const unsigned long long t = global_timer_ns();
        if (i == 0) {
            t0 = t;
        } else if (t - t0 > kWaitLimitNs) {
            atomicOr(err_word, kErrTimeout);
            *abort_flag = 1;
            return false;
        }
    }
}

// ------------------------------------------------------------------ bulk-copy column gather
// out[j, :]  = sum_{p in column j} values[perm[p]] * R[row_idx[p], :]     (fp32, rows ascending)
// sums[j]    = sum_{p in column j} values[perm[p]]                         (optional, fp64 sums)
// dots[perm[p]] = (values[perm[p]] != 0) * R[row_idx[p], :] . W[j, :]    (optional, fp32)
//
// Work is split by entries, not columns: range c takes the column-ordered entries [a, b) of an
// equal share, so a column active in every row costs no more than its share of entries. Warp 0
// streams each entry's row of R (one D-piece, blockIdx.y) into a ring of shared-memory slots, one
// cp.async.bulk per row; with dots, the column's row of W enters the ring ahead of its entries.
// The slots are grouped into stages of G rows that share one "full" mbarrier (the copies'
// bytes) and one "empty" mbarrier (one arrival per consumer warp), so the hand-over costs
// are paid once per G rows; the producer's lanes hand over a stage's rows in parallel (each
// lane writes one slot's metadata and issues its copy). Each consumer thread owns 16-byte
// chunks of the piece and accumulates them in fp32 registers, in the column view's fixed
// (row-ascending) order; a column's sums leave the registers when the stream moves on to the
// next column. The first and the last column of a range can continue in the neighbouring
// range: their partial sums go to the carry workspace and csc_carry_kernel adds the parts in
// range order. A column without entries is written as zeros by the range in which its (empty)
// entry span starts.
constexpr int kGatherMaxPieceBytes = 16384;
constexpr int kGatherSmemPerSm = 192 * 1024;  // rings of the three CTAs an SM holds
constexpr int kGatherStages = 2;
constexpr int kGatherMaxWarps = 16;    // consumer warps
constexpr int kGatherMinEntries = 64;  // entries per range at least

struct __align__(16) GatherSlot {
    float v;       // the entry's value
    int32_t col;   // its column
    int32_t kind;  // 0 entry, 1 row of W, 2 end of the stream
    int32_t row;   // the gathered row of R
    int64_t pos;   // CSR position of the entry (dots), -1 if none
    int64_t pad;
};

struct GatherArgs {
    const int32_t *col_idx;
    const int32_t *row_idx;
    const int64_t *perm;
    const void *values;
    int values_dtype;
    const void *R;
    int64_t ldr;
    const void *W;
    int64_t ldw;
    float *dots;
    void *out;
    int out_dtype;
    int64_t ldo;
    int out_vec;
    float *col_sums;
    double *carry;  // [n_ranges][n_pieces][2][carry_stride]
    int32_t *info;  // [n_ranges][4]: first column, last column, head, tail
    int64_t n_cols, nnz, M, D;
    int64_t per_range, piece_elems, carry_stride;
    int n_ranges, slots, group, consumer_warps;
    uint32_t slot_stride;
    unsigned *err;
};

// Shared memory ahead of the ring: full and empty barriers, slot metadata, dot partials, the
// abort flag, and the producer's item list of one batch (at most 64 items: 32 entries, 32 W rows).
__host__ __device__ constexpr size_t gather_header_bytes(int slots) {
    return ((size_t)slots * (16 + sizeof(GatherSlot) + 4 * kGatherMaxWarps) + 16 + 64 * sizeof(GatherSlot) + 127) /
           128 * 128;
}

// The EPV elements of a 16-byte chunk as fp32. A bf16 is the upper half of its fp32 value, so
// each conversion is one shift or mask of the 32-bit word holding two of them.
template <typename RT>
__device__ __forceinline__ void chunk_to_f32(const uint4 &u, float (&x)[16 / sizeof(RT)]) {
    if constexpr (sizeof(RT) == 4) {
        x[0] = __uint_as_float(u.x), x[1] = __uint_as_float(u.y);
        x[2] = __uint_as_float(u.z), x[3] = __uint_as_float(u.w);
    } else if constexpr (std::is_same<RT, __nv_bfloat16>::value) {
        x[0] = __uint_as_float(u.x << 16), x[1] = __uint_as_float(u.x & 0xffff0000u);
        x[2] = __uint_as_float(u.y << 16), x[3] = __uint_as_float(u.y & 0xffff0000u);
        x[4] = __uint_as_float(u.z << 16), x[5] = __uint_as_float(u.z & 0xffff0000u);
        x[6] = __uint_as_float(u.w << 16), x[7] = __uint_as_float(u.w & 0xffff0000u);
    } else {
        const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    }
}

// 1: the consumers update their row accumulators two at a time with the packed fp32 FMA of
// sm_100 (__ffma2_rn); 0: one fmaf each. Same bits either way.
#ifndef SF_GATHER_FMA2
#define SF_GATHER_FMA2 1
#endif
constexpr bool kGatherFma2 = SF_GATHER_FMA2 != 0;

// Consumer warps a launch may have: with 3 or 4 chunks per thread the register budget allows 8.
__host__ __device__ constexpr int gather_max_warps(int cpt) { return cpt >= 3 ? 8 : kGatherMaxWarps; }

template <typename RT, int CPT, bool DOT>
__global__ void __launch_bounds__(32 * (1 + gather_max_warps(CPT)), 1) csc_gather_kernel(const GatherArgs g) {
    constexpr int EPV = 16 / sizeof(RT);
    extern __shared__ __align__(128) unsigned char smem[];
    const int S = g.slots, G = g.group, NS = S / G;  // slots, rows per stage, stages
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + S;
    GatherSlot *meta = reinterpret_cast<GatherSlot *>(empty + S);
    float *dotp = reinterpret_cast<float *>(meta + S);  // [S][kGatherMaxWarps]
    volatile int *abort_flag = reinterpret_cast<volatile int *>(dotp + (size_t)S * kGatherMaxWarps);
    GatherSlot *items = reinterpret_cast<GatherSlot *>(dotp + (size_t)S * kGatherMaxWarps + 4);
    unsigned char *ring = smem + gather_header_bytes(S);

    const int64_t c = blockIdx.x, q = blockIdx.y;
    const int64_t a = c * g.per_range, b = min(g.nnz, a + g.per_range);
    const int64_t d0 = q * g.piece_elems;
    const int64_t pe = min(g.piece_elems, g.D - d0);
    const uint32_t piece_bytes = (uint32_t)(pe * (int64_t)sizeof(RT));
    const int n_chunks = (int)(pe / EPV);
    const int warp = threadIdx.x >> 5, lane = lane_id();

    auto col_at = [&](int64_t p) {
        const int32_t j = g.col_idx[p];
        return (j < 0 || (int64_t)j >= g.n_cols) ? 0 : j;
    };
    const int32_t first_col = col_at(a), last_col = col_at(b - 1);
    const bool head = a > 0 && col_at(a - 1) == first_col;
    const bool tail = b < g.nnz && col_at(b) == last_col;

    if (piece_bytes < g.slot_stride) {  // zero the slot padding (the copies never write it)
        const uint32_t pad = g.slot_stride - piece_bytes;
        for (uint32_t i = threadIdx.x * 4; i < (uint32_t)S * pad; i += blockDim.x * 4) {
            const uint32_t sl = i / pad, o = i - sl * pad;
            *reinterpret_cast<uint32_t *>(ring + (size_t)sl * g.slot_stride + piece_bytes + o) = 0u;
        }
    }
    if (threadIdx.x == 0) {
        for (int st = 0; st < NS; ++st) {
            mbar_init(&full[st], G);
            mbar_init(&empty[st], g.consumer_warps);
        }
        *abort_flag = 0;
        fence_mbar_init();
        if (q == 0) {
            int32_t *inf = g.info + 4 * c;
            inf[0] = first_col;
            inf[1] = last_col;
            inf[2] = head;
            inf[3] = tail;
        }
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------- producer
        const uint64_t keep = l2_policy_evict_last(), once = l2_policy_evict_first();
        const RT *R = reinterpret_cast<const RT *>(g.R);
        const RT *W = reinterpret_cast<const RT *>(g.W);
        int64_t staged = 0;  // stages handed to the consumers
        int stage = 0, fill = 0;
        uint32_t phase = 0;  // ring lap parity of `stage`
        bool ok = true;
        int32_t prev_col = -1;
        // Dot products of the entries stage st held (lane i: slot i), up to an end marker.
        auto finalize = [&](int st) {
            if constexpr (DOT) {
                const int s = st * G + lane;
                GatherSlot m{};
                m.kind = 1;
                if (lane < G) m = meta[s];
                const unsigned ends = __ballot_sync(0xffffffffu, lane < G && m.kind == 2);
                if (lane < G && m.kind == 0 && m.pos >= 0 && (ends & ((2u << lane) - 1u)) == 0) {
                    float sum = 0.f;
                    for (int w = 0; w < g.consumer_warps; ++w) sum += dotp[s * kGatherMaxWarps + w];
                    g.dots[m.pos] = m.v != 0.f ? sum : 0.f;
                }
            }
        };
        // Start of a stage: its previous lap must have been consumed.
        auto claim = [&]() {
            if (fill == 0 && staged >= NS) {
                if (!mbar_wait_suspend(&empty[stage], phase ^ 1u, abort_flag, g.err)) return false;
                finalize(stage);
            }
            return true;
        };
        auto advance = [&]() {
            fill = 0;
            ++staged;
            if (++stage == NS) stage = 0, phase ^= 1u;
        };
        // Entry metadata runs two batches of 32 ahead of the copies: (column, row, position) of
        // batch i+2 and the value of batch i+1 are loaded before batch i's copies are issued.
        auto load_meta = [&](int64_t base, int32_t &col, int32_t &r, int64_t &pos) {
            const int64_t p = base + lane;
            col = 0;
            r = 0;
            pos = -1;
            if (p < b) {
                col = g.col_idx[p];
                r = g.row_idx[p];
                pos = g.perm[p];
            }
        };
        auto load_value = [&](int64_t pos) {
            return (pos >= 0 && pos < g.nnz) ? load_as_f32(g.values, g.values_dtype, pos) : 0.f;
        };
        int32_t col0, r0, col1, r1;
        int64_t pos0, pos1;
        load_meta(a, col0, r0, pos0);
        load_meta(a + 32, col1, r1, pos1);
        float v0 = load_value(pos0);
        for (int64_t base = a; base < b && ok; base += 32) {
            const float v1 = load_value(pos1);
            int32_t col2, r2;
            int64_t pos2;
            load_meta(base + 64, col2, r2, pos2);
            const int n = (int)min((int64_t)32, b - base);
            const bool mine = lane < n;
            if (mine) {
                bool bad = false;
                if (col0 < 0 || (int64_t)col0 >= g.n_cols) bad = true, col0 = 0;
                if (r0 < 0 || (int64_t)r0 >= g.M) bad = true, r0 = 0;
                if (pos0 < 0 || pos0 >= g.nnz) bad = true, pos0 = -1;
                if (bad) {
                    atomicOr(g.err, kErrIndex);
                    v0 = 0.f;
                }
            }
            // This batch's items in stream order: with dots, a column's row of W precedes its
            // first entry in the batch when the column differs from the previous entry's.
            const int32_t up = __shfl_up_sync(0xffffffffu, col0, 1);
            const bool newc = DOT && mine && col0 != (lane == 0 ? prev_col : up);
            const unsigned nb = __ballot_sync(0xffffffffu, newc);
            const int k = lane + __popc(nb & ((1u << lane) - 1u)) + (newc ? 1 : 0);
            if (newc) {
                GatherSlot &it = items[k - 1];
                it.v = 0.f;
                it.col = col0;
                it.kind = 1;
                it.row = 0;
                it.pos = -1;
            }
            if (mine) {
                GatherSlot &it = items[k];
                it.v = v0;
                it.col = col0;
                it.kind = 0;
                it.row = r0;
                it.pos = pos0;
            }
            if (DOT) prev_col = __shfl_sync(0xffffffffu, col0, n - 1);
            const int n_items = n + __popc(nb);
            __syncwarp();
            for (int k0 = 0; k0 < n_items;) {
                if (!claim()) {
                    ok = false;
                    break;
                }
                const int m = min(G - fill, n_items - k0);
                if (lane < m) {
                    const GatherSlot it = items[k0 + lane];
                    const int s = stage * G + fill + lane;
                    meta[s] = it;
                    const RT *src = it.kind == 1 ? W + (int64_t)it.col * g.ldw + d0 : R + (int64_t)it.row * g.ldr + d0;
                    mbar_arrive_expect_tx(&full[stage], piece_bytes);  // release: the slot's metadata
                    bulk_load(ring + (size_t)s * g.slot_stride, src, piece_bytes, &full[stage],
                              it.kind == 1 ? once : keep);
                }
                k0 += m;
                fill += m;
                if (fill == G) advance();
            }
            __syncwarp();  // the item list is rewritten by the next batch
            col0 = col1, r0 = r1, pos0 = pos1, v0 = v1;
            col1 = col2, r1 = r2, pos1 = pos2;
        }
        if (ok) ok = claim();
        if (ok) {
            if (lane == 0) {
                GatherSlot &m = meta[stage * G + fill];
                m.pos = -1;
                m.kind = 2;
                mbar_arrive_count(&full[stage], (uint32_t)(G - fill));
            }
            __syncwarp();
            advance();
        }
        // A failed claim() waited at the start of a stage, so every stage with copies in flight
        // was handed over. Finish the dots of the stages still in the ring; after a time-out,
        // let the copies in flight land.
        bool aborted = !ok;
        const int back = (int)min(staged, (int64_t)NS);  // the last `back` stages, oldest first
        int st = stage - back;
        uint32_t par = phase;
        if (st < 0) st += NS, par ^= 1u;
        for (int i = 0; i < back; ++i, ++st) {
            if (st == NS) st = 0, par ^= 1u;
            if (!aborted) {
                if (mbar_wait_suspend(&empty[st], par, abort_flag, g.err)) {
                    finalize(st);
                    continue;
                }
                aborted = true;
            }
            mbar_wait_drain(&full[st], par, g.err);
        }
        return;
    }

    // ---------------- consumers
    const int cw = warp - 1;
    const int ct = threadIdx.x - 32;
    const int nct = g.consumer_warps * 32;
    float acc[CPT][EPV];
    float wv[DOT ? CPT : 1][DOT ? EPV : 1];
    double vsum = 0.0;
    int32_t cur = -1;
    char *out = reinterpret_cast<char *>(g.out);
    const size_t oes = g.out_dtype == SF_F32 ? 4 : 2;
    const bool sums = g.col_sums != nullptr;  // the carry holds them for the range's end columns
    const bool write_sums = sums && q == 0;
    const bool vec = g.out_vec != 0;

    auto zero_cols = [&](int64_t lo, int64_t hi) {  // columns [lo, hi) have no entries
        float z[EPV];
#pragma unroll
        for (int e = 0; e < EPV; ++e) z[e] = 0.f;
        for (int64_t j = lo; j < hi; ++j) {
#pragma unroll
            for (int k = 0; k < CPT; ++k) {
                const int ch = ct + k * nct;
                if (ch < n_chunks) store_chunk<EPV>(out + (size_t)j * g.ldo * oes, g.out_dtype, d0 + ch * EPV, z, vec);
            }
            if (write_sums && ct == 0) g.col_sums[j] = 0.f;
        }
    };
    auto flush = [&](int32_t col) {
        const int which = (head && col == first_col) ? 0 : ((tail && col == last_col) ? 1 : -1);
        if (which >= 0) {
            double *dst = g.carry + ((c * gridDim.y + q) * 2 + which) * g.carry_stride;
#pragma unroll
            for (int k = 0; k < CPT; ++k) {
                const int ch = ct + k * nct;
                if (ch < n_chunks) {
#pragma unroll
                    for (int e = 0; e < EPV; ++e) dst[ch * EPV + e] = acc[k][e];
                }
            }
            if (ct == 0) dst[g.piece_elems] = vsum;
            return;
        }
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int ch = ct + k * nct;
            if (ch < n_chunks) store_chunk<EPV>(out + (size_t)col * g.ldo * oes, g.out_dtype, d0 + ch * EPV, acc[k], vec);
        }
        if (write_sums && ct == 0) g.col_sums[col] = (float)vsum;
    };

    // Empty columns whose entry span starts at a: those after the previous range's last column.
    if (a == 0) {
        zero_cols(0, first_col);
    } else if (!head) {
        zero_cols((int64_t)col_at(a - 1) + 1, first_col);
    }
    // A stage's rows have all landed once its full barrier completes, so the loop loads the
    // next slot's metadata and chunks before working on the current one, alternating between
    // two register sets.
    auto load = [&](int s, int4 &m, uint4 (&u)[CPT]) {
        m = *reinterpret_cast<const int4 *>(&meta[s]);  // v, col, kind, row
        const uint4 *src = reinterpret_cast<const uint4 *>(ring + (size_t)s * g.slot_stride);
#pragma unroll
        for (int k = 0; k < CPT; ++k) u[k] = src[ct + k * nct];
    };
    auto work = [&](const int4 &m, const uint4 (&u)[CPT]) -> float {  // the lane's dot product part
        const int32_t mcol = m.y;
        if (mcol != cur) {
            if (cur >= 0) {
                flush(cur);
                zero_cols((int64_t)cur + 1, mcol);
            }
            cur = mcol;
#pragma unroll
            for (int k = 0; k < CPT; ++k)
#pragma unroll
                for (int e = 0; e < EPV; ++e) acc[k][e] = 0.f;
            vsum = 0.0;
        }
        if constexpr (DOT) {  // only the dot products put rows of W in the stream
            if (m.z == 1) {
#pragma unroll
                for (int k = 0; k < CPT; ++k) chunk_to_f32<RT>(u[k], wv[k]);
                return 0.f;
            }
        }
        const float vf = __int_as_float(m.x);
        float dp = 0.f;
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            float x[EPV];
            chunk_to_f32<RT>(u[k], x);
            if constexpr (kGatherFma2) {
                // two accumulators per packed FMA (each lane bit-identical to fmaf); the dot
                // product keeps its one scalar chain, so its summation order is unchanged
#pragma unroll
                for (int e = 0; e < EPV; e += 2) {
                    const float2 r = __ffma2_rn(make_float2(vf, vf), make_float2(x[e], x[e + 1]),
                                                make_float2(acc[k][e], acc[k][e + 1]));
                    acc[k][e] = r.x;
                    acc[k][e + 1] = r.y;
                }
                if constexpr (DOT) {
#pragma unroll
                    for (int e = 0; e < EPV; ++e) dp = fmaf(x[e], wv[k][e], dp);
                }
            } else {
#pragma unroll
                for (int e = 0; e < EPV; ++e) {
                    acc[k][e] = fmaf(vf, x[e], acc[k][e]);
                    if constexpr (DOT) dp = fmaf(x[e], wv[k][e], dp);
                }
            }
        }
        if (sums) vsum += (double)vf;
        return dp;
    };
    // Warp sums of the dot product parts of one slot, or of two at once: the first butterfly
    // step sends each half-warp the other slot's parts, so two slots cost five shuffles.
    auto reduce1 = [&](float d, int s) {
        if constexpr (DOT) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            if (lane == 0) dotp[s * kGatherMaxWarps + cw] = d;
        }
    };
    auto reduce2 = [&](float da, int sa, float db, int sb) {
        if constexpr (DOT) {
            const bool lo = lane < 16;
            float d = (lo ? da : db) + __shfl_xor_sync(0xffffffffu, lo ? db : da, 16);
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
            if (lane == 0) dotp[sa * kGatherMaxWarps + cw] = d;
            if (lane == 16) dotp[sb * kGatherMaxWarps + cw] = d;
        }
    };
    bool end = false;
    for (int st = 0, phase = 0; !end; ++st) {
        if (st == NS) st = 0, phase ^= 1;
        if (!mbar_wait_suspend(&full[st], (uint32_t)phase, abort_flag, g.err)) return;
        const int s0 = st * G;
        int4 ma, mb;
        uint4 ua[CPT], ub[CPT];
        load(s0, ma, ua);
        for (int i = 0; i < G; i += 2) {
            if (ma.z == 2) {
                end = true;
                break;
            }
            if (i + 1 < G) load(s0 + i + 1, mb, ub);
            const float da = work(ma, ua);
            if (i + 1 >= G || mb.z == 2) {
                reduce1(da, s0 + i);
                end = i + 1 < G;
                break;
            }
            if (i + 2 < G) load(s0 + i + 2, ma, ua);
            const float db = work(mb, ub);
            reduce2(da, s0 + i, db, s0 + i + 1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (cur >= 0) flush(cur);
    if (b == g.nnz) zero_cols((int64_t)last_col + 1, g.n_cols);
}

// Columns that continue across ranges: the range in which a column starts (its tail part)
// adds the head parts of the following ranges, in range order, and writes the column.
__global__ void __launch_bounds__(256) csc_carry_kernel(const GatherArgs g) {
    const int64_t c = blockIdx.x, q = blockIdx.y;
    const int32_t *inf = g.info + 4 * c;
    const int32_t last = inf[1];
    if (!inf[3] || (inf[2] && inf[0] == last)) return;  // no tail, or not the range it starts in
    const int64_t d0 = q * g.piece_elems;
    const int64_t pe = min(g.piece_elems, g.D - d0);
    const size_t oes = g.out_dtype == SF_F32 ? 4 : 2;
    char *out = reinterpret_cast<char *>(g.out) + (size_t)last * g.ldo * oes;
    for (int64_t d = threadIdx.x; d <= pe; d += blockDim.x) {
        const int64_t at = d < pe ? d : g.piece_elems;
        double total = g.carry[((c * gridDim.y + q) * 2 + 1) * g.carry_stride + at];
        for (int64_t c2 = c + 1; c2 < g.n_ranges; ++c2) {
            const int32_t *i2 = g.info + 4 * c2;
            if (!i2[2] || i2[0] != last) break;
            total += g.carry[((c2 * gridDim.y + q) * 2 + 0) * g.carry_stride + at];
            if (!(i2[3] && i2[1] == last)) break;
        }
        if (d < pe) {
            store_one(out, g.out_dtype, d0 + d, (float)total);
        } else if (g.col_sums != nullptr && q == 0) {
            g.col_sums[last] = (float)total;
        }
    }
}

// ------------------------------------------------------------------ fallbacks (unaligned rows)
// One warp per column, 32 output elements at a time, entries 32 at a time broadcast by
// shuffle; fp64 sums in the column view's order. Used when a row of R is not a whole number of
// 16-byte chunks.
template <typename RT>
__global__ void __launch_bounds__(128) csc_accumulate_kernel(const int64_t *__restrict__ col_ptr, int64_t n_cols,
                                                             const int32_t *__restrict__ row_idx,
                                                             const int64_t *__restrict__ perm, int64_t nnz,
                                                             const void *values, int values_dtype,
                                                             const RT *__restrict__ R, int64_t ldr, int64_t M,
                                                             int64_t D, void *out, int odt, int64_t ldo,
                                                             float *__restrict__ col_sums, unsigned *err) {
    const int64_t col = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (col >= n_cols) return;
    const int lane = lane_id();
    const int64_t p0 = col_ptr[col], p1 = col_ptr[col + 1];
    bool bad = false;
    auto entry = [&](int64_t q, int &r, float &v) {
        r = 0;
        v = 0.f;
        if (q < p1) {
            const int32_t rr = row_idx[q];
            const int64_t pos = perm[q];
            if (rr < 0 || (int64_t)rr >= M || pos < 0 || pos >= nnz) {
                bad = true;
            } else {
                r = rr;
                v = load_as_f32(values, values_dtype, pos);
            }
        }
    };
    if (col_sums != nullptr) {
        double vsum = 0.0;
        for (int64_t q0 = p0; q0 < p1; q0 += 32) {
            int r;
            float v;
            entry(q0 + lane, r, v);
            vsum += (double)v;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) vsum += __shfl_xor_sync(0xffffffffu, vsum, off);
        if (lane == 0) col_sums[col] = (float)vsum;
    }
    for (int64_t dc = 0; dc < D; dc += 32) {
        const int64_t d = dc + lane;
        double acc = 0.0;
        for (int64_t q0 = p0; q0 < p1; q0 += 32) {
            int r;
            float v;
            entry(q0 + lane, r, v);
            const int n = (int)min((int64_t)32, p1 - q0);
            for (int t = 0; t < n; ++t) {
                const int rt = __shfl_sync(0xffffffffu, r, t);
                const float vt = __shfl_sync(0xffffffffu, v, t);
                if (d < D) acc = fma((double)vt, (double)to_f32(R[(int64_t)rt * ldr + d]), acc);
            }
        }
        if (d < D) store_one(out, odt, col * ldo + d, (float)acc);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(err, kErrIndex);
}

// dots[perm[p]] = (v != 0) * R[row_idx[p]] . W[col_idx[p]], one warp per column-ordered entry.
template <typename RT>
__global__ void __launch_bounds__(128) csc_dot_kernel(const int32_t *__restrict__ col_idx,
                                                      const int32_t *__restrict__ row_idx,
                                                      const int64_t *__restrict__ perm, int64_t nnz,
                                                      const void *values, int values_dtype,
                                                      const RT *__restrict__ R, int64_t ldr, int64_t M,
                                                      const RT *__restrict__ W, int64_t ldw, int64_t n_cols,
                                                      int64_t D, float *__restrict__ dots, unsigned *err) {
    const int64_t p = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (p >= nnz) return;
    const int lane = lane_id();
    const int32_t r = row_idx[p], j = col_idx[p];
    const int64_t pos = perm[p];
    if (r < 0 || (int64_t)r >= M || j < 0 || (int64_t)j >= n_cols || pos < 0 || pos >= nnz) {
        if (lane == 0) atomicOr(err, kErrIndex);
        return;
    }
    float s = 0.f;
    for (int64_t d = lane; d < D; d += 32)
        s = fmaf(to_f32(R[(int64_t)r * ldr + d]), to_f32(W[(int64_t)j * ldw + d]), s);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) dots[pos] = load_as_f32(values, values_dtype, pos) != 0.f ? s : 0.f;
}

__global__ void zero_rows_kernel(void *out, int odt, int64_t rows, int64_t cols, int64_t ldo, float *col_sums) {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        store_one(out, odt, (i / cols) * ldo + i % cols, 0.f);
    if (col_sums != nullptr)
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x)
            col_sums[i] = 0.f;
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

// The same on 64 x 64 tiles with two elements per thread along the contiguous dimension, for
// even extents and pitches: each warp reads and writes 64 consecutive elements (128 bytes of a
// 16-bit matrix) per row instead of 32.
template <typename T>
struct Pair;
template <>
struct Pair<float> {
    using V = float2;
    static __device__ __forceinline__ void get(const V &v, float &a, float &b) { a = v.x, b = v.y; }
    static __device__ __forceinline__ V make(float a, float b) { return make_float2(a, b); }
};
template <>
struct Pair<__nv_bfloat16> {
    using V = __nv_bfloat162;
    static __device__ __forceinline__ void get(const V &v, float &a, float &b) {
        a = __low2float(v), b = __high2float(v);
    }
    static __device__ __forceinline__ V make(float a, float b) { return __floats2bfloat162_rn(a, b); }
};
template <>
struct Pair<__half> {
    using V = __half2;
    static __device__ __forceinline__ void get(const V &v, float &a, float &b) {
        a = __low2float(v), b = __high2float(v);
    }
    static __device__ __forceinline__ V make(float a, float b) { return __floats2half2_rn(a, b); }
};

template <typename IT, typename OT>
__global__ void __launch_bounds__(256) transpose2_kernel(const IT *__restrict__ in, int64_t rows, int64_t cols,
                                                         int64_t ldi, OT *__restrict__ out, int64_t ldo) {
    __shared__ float tile[64][65];
    const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads, 2 elements each
#pragma unroll
    for (int k = 0; k < 64; k += 8) {
        const int64_t r = r0 + ty + k, c = c0 + 2 * tx;
        float a = 0.f, b = 0.f;
        if (r < rows && c < cols)  // cols is even, so c + 1 < cols too
            Pair<IT>::get(*reinterpret_cast<const typename Pair<IT>::V *>(in + r * ldi + c), a, b);
        tile[ty + k][2 * tx] = a;
        tile[ty + k][2 * tx + 1] = b;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 64; k += 8) {
        const int64_t orow = c0 + ty + k, oc = r0 + 2 * tx;  // out is [cols, rows]
        if (orow < cols && oc < rows)  // rows is even
            *reinterpret_cast<typename Pair<OT>::V *>(out + orow * ldo + oc) =
                Pair<OT>::make(tile[2 * tx][ty + k], tile[2 * tx + 1][ty + k]);
    }
}

// y[i] = sum_j A[i, j] * x[j] (fp32 x, fp32 sums in a fixed order): one CTA per row of A,
// 16-byte loads when the rows allow them. With A = W_enc and x = the column sums of dpre it gives
// sum over tokens of dx without forming dx.
template <typename T>
__global__ void __launch_bounds__(256) matvec_kernel(const T *__restrict__ A, int64_t rows, int64_t cols, int64_t lda,
                                                     const float *__restrict__ x, float *__restrict__ y, int vec) {
    constexpr int EPV = 16 / sizeof(T);
    __shared__ float part[8];
    const int64_t i = blockIdx.x;
    const T *a = A + i * lda;
    float sum = 0.f;
    if (vec) {  // four 16-byte chunks of the row (and their x) in flight per thread
        constexpr int U = 4;
        int64_t c = (int64_t)threadIdx.x * EPV;
        for (; c + (U - 1) * 256 * EPV < cols; c += U * 256 * EPV) {
            uint4 ua[U];
            float4 xa[U][EPV / 4];
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const int64_t ck = c + (int64_t)k * 256 * EPV;
                ua[k] = __ldg(reinterpret_cast<const uint4 *>(a + ck));
#pragma unroll
                for (int h = 0; h < EPV / 4; ++h) xa[k][h] = __ldg(reinterpret_cast<const float4 *>(x + ck) + h);
            }
#pragma unroll
            for (int k = 0; k < U; ++k) {
                float v[EPV];
                chunk_to_f32<T>(ua[k], v);
                const float *xv = reinterpret_cast<const float *>(xa[k]);
#pragma unroll
                for (int e = 0; e < EPV; ++e) sum = fmaf(v[e], xv[e], sum);
            }
        }
        for (; c < cols; c += 256 * EPV) {
            float v[EPV];
            chunk_to_f32<T>(__ldg(reinterpret_cast<const uint4 *>(a + c)), v);
#pragma unroll
            for (int e = 0; e < EPV; ++e) sum = fmaf(v[e], __ldg(x + c + e), sum);
        }
    } else {
        for (int64_t c = threadIdx.x; c < cols; c += 256) sum = fmaf(to_f32(a[c]), __ldg(x + c), sum);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane_id() == 0) part[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < 8; ++w) t += part[w];
        y[i] = t;
    }
}

// 16-bit to 16-bit on 64 x 64 tiles with 16-byte loads and stores (extents and pitches
// multiples of 8, 16-byte aligned): each thread moves two 8-element chunks each way.
__device__ __forceinline__ float half_bits_to_f32(uint16_t h, bool bf) {
    return bf ? __uint_as_float((uint32_t)h << 16) : __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint32_t pack_f32_pair(float a, float b, bool bf) {
    if (bf) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&v);
    }
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&v);
}
__global__ void __launch_bounds__(256) transpose16_kernel(const uint16_t *__restrict__ in, int64_t rows, int64_t cols,
                                                          int64_t ldi, bool in_bf, uint16_t *__restrict__ out,
                                                          int64_t ldo, bool out_bf) {
    __shared__ float tile[64][65];
    const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
    const int t = threadIdx.x, q = t & 7, rr = t >> 3;  // chunk q of row rr (and rr + 32)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int lr = rr + 32 * k;
        const int64_t r = r0 + lr, c = c0 + 8 * q;
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (r < rows && c < cols) u = __ldg(reinterpret_cast<const uint4 *>(in + r * ldi + c));
        tile[lr][8 * q + 0] = half_bits_to_f32((uint16_t)(u.x & 0xffffu), in_bf);
        tile[lr][8 * q + 1] = half_bits_to_f32((uint16_t)(u.x >> 16), in_bf);
        tile[lr][8 * q + 2] = half_bits_to_f32((uint16_t)(u.y & 0xffffu), in_bf);
        tile[lr][8 * q + 3] = half_bits_to_f32((uint16_t)(u.y >> 16), in_bf);
        tile[lr][8 * q + 4] = half_bits_to_f32((uint16_t)(u.z & 0xffffu), in_bf);
        tile[lr][8 * q + 5] = half_bits_to_f32((uint16_t)(u.z >> 16), in_bf);
        tile[lr][8 * q + 6] = half_bits_to_f32((uint16_t)(u.w & 0xffffu), in_bf);
        tile[lr][8 * q + 7] = half_bits_to_f32((uint16_t)(u.w >> 16), in_bf);
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int lc = rr + 32 * k;  // the input column = the output row
        const int64_t orow = c0 + lc, oc = r0 + 8 * q;
        if (orow < cols && oc < rows) {
            uint4 v;
            v.x = pack_f32_pair(tile[8 * q + 0][lc], tile[8 * q + 1][lc], out_bf);
            v.y = pack_f32_pair(tile[8 * q + 2][lc], tile[8 * q + 3][lc], out_bf);
            v.z = pack_f32_pair(tile[8 * q + 4][lc], tile[8 * q + 5][lc], out_bf);
            v.w = pack_f32_pair(tile[8 * q + 6][lc], tile[8 * q + 7][lc], out_bf);
            *reinterpret_cast<uint4 *>(out + orow * ldo + oc) = v;
        }
    }
}

template <typename F>
int by_dtype(int dt, F &&f) {
    if (dt == SF_F32) return f(float{});
    if (dt == SF_BF16) return f(__nv_bfloat16{});
    return f(__half{});
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch shape of csc_gather_kernel for nnz entries gathering D-element rows of es bytes each.
struct GatherPlan {
    bool bulk;
    int64_t piece_elems, n_pieces, per_range, n_ranges, carry_stride;
    int cpt, consumer_warps, slots, group;
    uint32_t slot_stride;
    size_t smem, carry_bytes, info_bytes;
};

GatherPlan plan_gather(int64_t nnz, int64_t D, size_t es, bool aligned) {
    GatherPlan p{};
    p.bulk = aligned && nnz > 0 && D > 0 && (D * (int64_t)es) % 16 == 0;
    if (!p.bulk) return p;
    const int64_t epv = 16 / (int64_t)es;
    const int64_t row_bytes = D * (int64_t)es;
    const int64_t pieces = (row_bytes + kGatherMaxPieceBytes - 1) / kGatherMaxPieceBytes;
    p.piece_elems = ((D + pieces - 1) / pieces + epv - 1) / epv * epv;
    p.n_pieces = (D + p.piece_elems - 1) / p.piece_elems;
    const int64_t chunks = p.piece_elems / epv;
    // 16-byte chunks per consumer thread. Every consumer warp walks every row in the ring, so
    // fewer, wider warps cut the per-row overhead: the fewest warps that leave under a quarter
    // of the lanes idle.
    p.cpt = 1;
    for (int cpt = 2; cpt <= 4; ++cpt) {
        const int64_t warps = (chunks + 32 * cpt - 1) / (32 * cpt);
        if (warps <= gather_max_warps(cpt) && warps * 32 * cpt * 3 < chunks * 4) p.cpt = cpt;
    }
    while ((chunks + 32 * p.cpt - 1) / (32 * p.cpt) > gather_max_warps(p.cpt)) ++p.cpt;
    p.consumer_warps = (int)((chunks + 32 * p.cpt - 1) / (32 * p.cpt));
    // A slot spans every consumer thread's chunks; the bytes past the row piece stay zero, so
    // the consumers read their chunks unconditionally.
    p.slot_stride = (uint32_t)((std::max<int64_t>(p.piece_elems * (int64_t)es, (int64_t)p.consumer_warps * 32 * p.cpt * 16) + 127) /
                               128 * 128);
    int slots = 2;
    const int ctas_per_sm = 3;
    const size_t ring_bytes = (size_t)kGatherSmemPerSm / ctas_per_sm;
    while (slots < 64 && gather_header_bytes(slots + 1) + (size_t)(slots + 1) * p.slot_stride <= ring_bytes) ++slots;
    p.group = std::min(32, std::max(1, slots / kGatherStages));
    p.slots = slots / p.group * p.group;
    p.smem = gather_header_bytes(p.slots) + (size_t)p.slots * p.slot_stride;
    const int64_t max_ranges = ctas_per_sm * (int64_t)num_sms();
    int64_t ranges = std::min<int64_t>(max_ranges, (nnz + kGatherMinEntries - 1) / kGatherMinEntries);
    ranges = std::max<int64_t>(ranges, 1);
    p.per_range = (nnz + ranges - 1) / ranges;
    p.n_ranges = (nnz + p.per_range - 1) / p.per_range;
    p.carry_stride = p.piece_elems + 2;
    p.carry_bytes = (size_t)(p.n_ranges * p.n_pieces * 2 * p.carry_stride) * sizeof(double);
    p.info_bytes = (size_t)p.n_ranges * 4 * sizeof(int32_t);
    return p;
}

// Workspace of sf_csr_transpose: column counts, cursors and the long-column list (int32), then
// the unsorted scatter (int64 positions, int32 rows) that the in-column sort reads.
size_t transpose_ints(int64_t n_cols) { return ((size_t)(3 * n_cols + 64) * sizeof(int32_t) + 15) / 16 * 16; }

}  // namespace
}  // namespace sf

using namespace sf;

extern "C" {

int sf_csr_transpose_workspace(int64_t n_cols, int64_t nnz, size_t *bytes) {
    if (!bytes) return set_error(SF_ERR_INVALID, "bytes is NULL");
    if (n_cols < 0 || nnz < 0) return set_error(SF_ERR_INVALID, "negative extent");
    *bytes = transpose_ints(n_cols) + (size_t)nnz * (sizeof(int64_t) + sizeof(int32_t)) + 16;
    return SF_OK;
}

int sf_csr_transpose(const int64_t *indptr, int64_t M, const int32_t *indices, int64_t nnz, int64_t n_cols,
                     int64_t *col_ptr, int32_t *row_idx, int64_t *perm, int32_t *col_idx, void *workspace,
                     size_t workspace_bytes, sf_stream stream) {
    if (M < 0 || nnz < 0 || n_cols < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (n_cols > (int64_t)INT32_MAX || M > (int64_t)INT32_MAX)
        return set_error(SF_ERR_UNSUPPORTED, "n_cols and M must be below 2^31");
    if (!col_ptr || (M > 0 && !indptr)) return set_error(SF_ERR_INVALID, "NULL pointer");
    if (nnz > 0 && (!indices || !row_idx || !perm)) return set_error(SF_ERR_INVALID, "NULL pointer");
    size_t need = 0;
    sf_csr_transpose_workspace(n_cols, nnz, &need);
    if (!workspace || workspace_bytes < need)
        return set_error(SF_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes, need);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t *cnt = static_cast<int32_t *>(workspace);
    int32_t *cursor = cnt + n_cols;
    int32_t *large = cursor + n_cols;  // [0] count, [1..] columns csc_sort_small_kernel leaves
    int64_t *tperm = reinterpret_cast<int64_t *>(static_cast<char *>(workspace) + transpose_ints(n_cols));
    int32_t *trow = reinterpret_cast<int32_t *>(tperm + nnz);
    int st = check_cuda(cudaMemsetAsync(cnt, 0, (size_t)(2 * n_cols + 1) * sizeof(int32_t), s), "memset counts");
    if (st) return st;
    if (nnz > 0) {
        const unsigned blocks = (unsigned)std::min<int64_t>((nnz + 255) / 256, 4096);
        csr_col_count_kernel<<<blocks, 256, 0, s>>>(indices, nnz, n_cols, cnt, device_error_word());
        st = check_cuda(cudaGetLastError(), "column count launch");
        if (st) return st;
    }
    st = launch_indptr(cnt, n_cols, col_ptr, s, nullptr);
    if (st) return st;
    if (M == 0 || nnz == 0) return st;
    csr_to_csc_kernel<<<(unsigned)((M + 7) / 8), 256, 0, s>>>(indptr, M, indices, n_cols, col_ptr, cursor, trow,
                                                               tperm);
    st = check_cuda(cudaGetLastError(), "csc scatter launch");
    if (st) return st;
    const unsigned sblocks = (unsigned)std::min<int64_t>((n_cols + 7) / 8, 8192);
    csc_sort_small_kernel<<<sblocks, 256, 0, s>>>(col_ptr, n_cols, trow, tperm, row_idx, perm, col_idx, large);
    st = check_cuda(cudaGetLastError(), "csc sort launch");
    if (st) return st;
    const int words = (int)std::min<int64_t>((M + 31) / 32 + 1, 16384);
    const size_t smem = (size_t)words * 2 * sizeof(uint32_t);
    st = check_cuda(cudaFuncSetAttribute(csc_sort_large_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "csc sort smem attribute");
    if (st) return st;
    csc_sort_large_kernel<<<(unsigned)(2 * num_sms()), kSortThreads, smem, s>>>(col_ptr, trow, tperm, row_idx, perm,
                                                                               col_idx, large, words,
                                                                               device_error_word());
    return check_cuda(cudaGetLastError(), "csc sort launch");
}

int sf_csc_gather_workspace(int64_t nnz, const sf_matrix *R, size_t *bytes) {
    if (!R || !bytes) return set_error(SF_ERR_INVALID, "NULL argument");
    if (!valid_dtype(R->dtype)) return set_error(SF_ERR_INVALID, "bad dtype");
    if (nnz < 0 || R->cols < 0) return set_error(SF_ERR_INVALID, "negative extent");
    const GatherPlan p = plan_gather(nnz, R->cols, dtype_size(R->dtype), true);
    *bytes = p.bulk ? p.carry_bytes + p.info_bytes : 0;
    return SF_OK;
}

int sf_csc_gather(const int64_t *col_ptr, int64_t n_cols, const int32_t *col_idx, int64_t nnz,
                  const int32_t *row_idx, const int64_t *perm, const void *values, int values_dtype,
                  const sf_matrix *R, const sf_matrix *W, float *dots, const sf_matrix *out, float *col_sums,
                  void *workspace, size_t workspace_bytes, sf_stream stream) {
    if (!R || !out) return set_error(SF_ERR_INVALID, "R and out are required");
    const bool dot = W != nullptr && W->data != nullptr;
    if (!valid_dtype(R->dtype) || !valid_dtype(values_dtype) || !valid_dtype(out->dtype))
        return set_error(SF_ERR_INVALID, "bad dtype");
    if (n_cols < 0 || nnz < 0 || R->rows < 0 || R->cols < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (out->rows != n_cols || out->cols != R->cols) return set_error(SF_ERR_INVALID, "out must be [n_cols, R.cols]");
    if (R->stride_col != 1 || out->stride_col != 1 || out->stride_row < out->cols)
        return set_error(SF_ERR_UNSUPPORTED, "R and out need unit column strides and non-overlapping rows");
    if (dot) {
        if (W->dtype != R->dtype) return set_error(SF_ERR_UNSUPPORTED, "W and R must have one dtype");
        if (W->rows != n_cols || W->cols != R->cols) return set_error(SF_ERR_INVALID, "W must be [n_cols, R.cols]");
        if (W->stride_col != 1) return set_error(SF_ERR_UNSUPPORTED, "W needs a unit column stride");
        if (nnz > 0 && !dots) return set_error(SF_ERR_INVALID, "dots is NULL");
    }
    if (n_cols == 0) return SF_OK;
    if (!col_ptr || !out->data) return set_error(SF_ERR_INVALID, "NULL pointer");
    if (nnz > 0 && (!row_idx || !perm || !values || !col_idx)) return set_error(SF_ERR_INVALID, "NULL entry arrays");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    void *outp = const_cast<void *>(out->data);
    const int64_t D = R->cols;
    if (nnz == 0) {
        const unsigned blocks = (unsigned)std::min<int64_t>((n_cols * std::max<int64_t>(D, 1) + 255) / 256, 4096);
        zero_rows_kernel<<<blocks, 256, 0, s>>>(outp, out->dtype, n_cols, D, out->stride_row, col_sums);
        return check_cuda(cudaGetLastError(), "zero fill launch");
    }
    const size_t es = dtype_size(R->dtype), oes = dtype_size(out->dtype);
    const bool aligned = aligned16(R->data) && (R->stride_row * (int64_t)es) % 16 == 0 &&
                         (!dot || (aligned16(W->data) && (W->stride_row * (int64_t)es) % 16 == 0));
    const GatherPlan p = plan_gather(nnz, D, es, aligned);
    return by_dtype(R->dtype, [&](auto rtag) {
        using RT = decltype(rtag);
        if (!p.bulk) {
            if ((n_cols + 3) / 4 > (int64_t)INT32_MAX || (nnz + 3) / 4 > (int64_t)INT32_MAX)
                return set_error(SF_ERR_UNSUPPORTED, "grid too large");
            csc_accumulate_kernel<RT><<<(unsigned)((n_cols + 3) / 4), 128, 0, s>>>(
                col_ptr, n_cols, row_idx, perm, nnz, values, values_dtype, reinterpret_cast<const RT *>(R->data),
                R->stride_row, R->rows, D, outp, out->dtype, out->stride_row, col_sums, device_error_word());
            int st = check_cuda(cudaGetLastError(), "csc accumulate launch");
            if (st || !dot) return st;
            csc_dot_kernel<RT><<<(unsigned)((nnz + 3) / 4), 128, 0, s>>>(
                col_idx, row_idx, perm, nnz, values, values_dtype, reinterpret_cast<const RT *>(R->data),
                R->stride_row, R->rows, reinterpret_cast<const RT *>(W->data), W->stride_row, n_cols, D, dots,
                device_error_word());
            return check_cuda(cudaGetLastError(), "csc dot launch");
        }
        if (p.n_ranges > (int64_t)INT32_MAX || p.n_pieces > 65535 || (nnz + 3) / 4 > (int64_t)INT32_MAX)
            return set_error(SF_ERR_UNSUPPORTED, "grid too large");
        if (!workspace || workspace_bytes < p.carry_bytes + p.info_bytes)
            return set_error(SF_ERR_WORKSPACE, "workspace of %zu bytes, need %zu", workspace_bytes,
                             p.carry_bytes + p.info_bytes);
        const bool fuse_dot = dot && p.n_pieces == 1;
        GatherArgs g{};
        g.col_idx = col_idx;
        g.row_idx = row_idx;
        g.perm = perm;
        g.values = values;
        g.values_dtype = values_dtype;
        g.R = R->data;
        g.ldr = R->stride_row;
        g.W = fuse_dot ? W->data : nullptr;
        g.ldw = fuse_dot ? W->stride_row : 0;
        g.dots = fuse_dot ? dots : nullptr;
        g.out = outp;
        g.out_dtype = out->dtype;
        g.ldo = out->stride_row;
        g.out_vec = aligned16(outp) && (out->stride_row * (int64_t)oes) % 16 == 0;
        g.col_sums = col_sums;
        g.carry = static_cast<double *>(workspace);
        g.info = reinterpret_cast<int32_t *>(static_cast<char *>(workspace) + p.carry_bytes);
        g.n_cols = n_cols;
        g.nnz = nnz;
        g.M = R->rows;
        g.D = D;
        g.per_range = p.per_range;
        g.piece_elems = p.piece_elems;
        g.carry_stride = p.carry_stride;
        g.n_ranges = (int)p.n_ranges;
        g.slots = p.slots;
        g.group = p.group;
        g.consumer_warps = p.consumer_warps;
        g.slot_stride = p.slot_stride;
        g.err = device_error_word();
        const void *kern;
        switch (p.cpt * 2 + (fuse_dot ? 1 : 0)) {
            case 2: kern = (const void *)csc_gather_kernel<RT, 1, false>; break;
            case 3: kern = (const void *)csc_gather_kernel<RT, 1, true>; break;
            case 4: kern = (const void *)csc_gather_kernel<RT, 2, false>; break;
            case 5: kern = (const void *)csc_gather_kernel<RT, 2, true>; break;
            case 6: kern = (const void *)csc_gather_kernel<RT, 3, false>; break;
            case 7: kern = (const void *)csc_gather_kernel<RT, 3, true>; break;
            case 8: kern = (const void *)csc_gather_kernel<RT, 4, false>; break;
            default: kern = (const void *)csc_gather_kernel<RT, 4, true>; break;
        }
        int st = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem),
                            "gather smem attribute");
        if (st) return st;
        const dim3 grid((unsigned)p.n_ranges, (unsigned)p.n_pieces);
        const dim3 block(32u * (1u + (unsigned)p.consumer_warps));
        void *args[] = {&g};
        st = check_cuda(cudaLaunchKernel(kern, grid, block, args, p.smem, s), "csc gather launch");
        if (st) return st;
        csc_carry_kernel<<<grid, 256, 0, s>>>(g);
        st = check_cuda(cudaGetLastError(), "csc carry launch");
        if (st || !dot || fuse_dot) return st;
        csc_dot_kernel<RT><<<(unsigned)((nnz + 3) / 4), 128, 0, s>>>(
            col_idx, row_idx, perm, nnz, values, values_dtype, reinterpret_cast<const RT *>(R->data), R->stride_row,
            R->rows, reinterpret_cast<const RT *>(W->data), W->stride_row, n_cols, D, dots, device_error_word());
        return check_cuda(cudaGetLastError(), "csc dot launch");
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
    const size_t ies = dtype_size(in->dtype), oes = dtype_size(out->dtype);
    const bool pairs = in->rows % 2 == 0 && in->cols % 2 == 0 && in->stride_row % 2 == 0 && out->stride_row % 2 == 0 &&
                       (reinterpret_cast<uintptr_t>(in->data) % (2 * ies)) == 0 &&
                       (reinterpret_cast<uintptr_t>(out->data) % (2 * oes)) == 0 && (in->rows + 63) / 64 <= 65535;
    const bool chunks16 = ies == 2 && oes == 2 && in->rows % 8 == 0 && in->cols % 8 == 0 && in->stride_row % 8 == 0 &&
                          out->stride_row % 8 == 0 && aligned16(in->data) && aligned16(out->data) &&
                          (in->rows + 63) / 64 <= 65535;
    if (chunks16) {
        const dim3 g16((unsigned)((in->cols + 63) / 64), (unsigned)((in->rows + 63) / 64));
        transpose16_kernel<<<g16, 256, 0, s>>>(static_cast<const uint16_t *>(in->data), in->rows, in->cols,
                                               in->stride_row, in->dtype == SF_BF16,
                                               static_cast<uint16_t *>(const_cast<void *>(out->data)),
                                               out->stride_row, out->dtype == SF_BF16);
        return check_cuda(cudaGetLastError(), "transpose launch");
    }
    dim3 grid((unsigned)((in->cols + 31) / 32), (unsigned)((in->rows + 31) / 32));
    if (pairs) grid = dim3((unsigned)((in->cols + 63) / 64), (unsigned)((in->rows + 63) / 64));
    return by_dtype(in->dtype, [&](auto itag) {
        using IT = decltype(itag);
        return by_dtype(out->dtype, [&](auto otag) {
            using OT = decltype(otag);
            if (pairs) {
                transpose2_kernel<IT, OT><<<grid, 256, 0, s>>>(reinterpret_cast<const IT *>(in->data), in->rows,
                                                               in->cols, in->stride_row,
                                                               reinterpret_cast<OT *>(const_cast<void *>(out->data)),
                                                               out->stride_row);
                return check_cuda(cudaGetLastError(), "transpose launch");
            }
            transpose_kernel<IT, OT><<<grid, 256, 0, s>>>(reinterpret_cast<const IT *>(in->data), in->rows, in->cols,
                                                          in->stride_row,
                                                          reinterpret_cast<OT *>(const_cast<void *>(out->data)),
                                                          out->stride_row);
            return check_cuda(cudaGetLastError(), "transpose launch");
        });
    });
}

int sf_matvec(const sf_matrix *A, const float *x, float *y, sf_stream stream) {
    if (!A) return set_error(SF_ERR_INVALID, "A is NULL");
    if (!valid_dtype(A->dtype)) return set_error(SF_ERR_INVALID, "bad dtype");
    if (A->rows < 0 || A->cols < 0) return set_error(SF_ERR_INVALID, "negative extent");
    if (A->stride_col != 1) return set_error(SF_ERR_UNSUPPORTED, "A needs a unit column stride");
    if (A->rows == 0) return SF_OK;
    if (!y || (A->cols > 0 && (!x || !A->data))) return set_error(SF_ERR_INVALID, "NULL pointer");
    if (A->rows > (int64_t)INT32_MAX) return set_error(SF_ERR_UNSUPPORTED, "too many rows");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    return by_dtype(A->dtype, [&](auto tag) {
        using T = decltype(tag);
        const int64_t es = (int64_t)sizeof(T);
        const int vec = (aligned16(A->data) && aligned16(x) && (A->stride_row * es) % 16 == 0 && (A->cols * es) % 16 == 0)
                            ? 1
                            : 0;
        matvec_kernel<T><<<(unsigned)A->rows, 256, 0, s>>>(reinterpret_cast<const T *>(A->data), A->rows, A->cols,
                                                          A->stride_row, x, y, vec);
        return check_cuda(cudaGetLastError(), "matvec launch");
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
