// Fused SAE encoder on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   out = act((x - b_dec) @ W_enc + b_enc)       fp32 accumulation in TMEM
//
// Follows the semantics of saeflow/kernels/encode.py:36-91 (_encode_kernel): the b_dec
// shift is applied in fp32 and rounded to W_enc's dtype before the product (encode.py:72
// of the kernel body, line 189 of the file), bias + ReLU / JumpReLU (strict `pre > thr`)
// run on the fp32 accumulator (:195-199), and the epilogue adds each row's count of
// stored nonzeros into row_nnz (:206-208). The count is taken on the value as stored
// (after rounding to the output dtype), so it always equals count_nonzero(out).
//
// Two persistent, warp-specialised kernels (192 threads, one CTA per SM):
//   warp 0      TMA producer: operand tiles of 128 B rows, SWIZZLE_128B, mbarrier ring.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer; fp32 accumulators
//               double-buffered in TMEM (2 x 256 columns) so the epilogue of one tile
//               overlaps the MMAs of the next.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, bias/activation in fp32,
//               rounding, nonzero count, 16-byte streaming stores (L2 evict_first).
//               In TOPK mode they instead keep a per-row running top-k in shared memory
//               and write k candidates per (row, column chunk); see topk_merge_kernel.
//
// encode_tc2_kernel (the default for M > 128) runs on CTA pairs (cluster of 2,
// tcgen05 cta_group::2): the pair computes a 256 x 256 tile, each CTA loading its 128 rows
// of x and 128 columns of W_enc, so each SM pulls 64 B of operands per MMA clock instead
// of the 96 B of the single-CTA 128 x 256 tile (encode_tc_kernel), which starves the tensor
// cores on L2 bandwidth. Both CTAs' TMA loads complete on the leader CTA's barrier; the
// leader's MMA thread signals each CTA's barriers with its own commit.
//
// The x operand is a pre-shifted copy (x - b_dec, rounded to the MMA dtype) made by
// shift_convert_kernel: a separate HBM pass costs <1% of the GEMM, whereas shifting in
// shared memory would compete with the tensor cores for shared-memory bandwidth.
#include <algorithm>
#include <cstddef>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "sf_common.cuh"
#include "sf_internal.h"

namespace sf {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kThreads = 192;
constexpr int kAccCols = 256;
constexpr int kTmemCols = 512;
constexpr int kTileABytes = kBM * 128;  // 128 rows x 128 B
constexpr size_t kSmemOptin = 232448;   // opt-in shared memory per block on sm_100 (227 KB)
constexpr int kTileBBytes = kBN * 128;  // 256 rows (or MN chunks) x 128 B
constexpr int kStageBytes = kTileABytes + kTileBBytes;

enum Mode { kDense = 0, kTopk = 1, kCsr = 2 };

// Bytes of x a raster group of m-tiles may span: the group's m-tiles run side by side over
// each W_enc n-tile, so W_enc is read from HBM once per group while the group's x stays in L2.
#ifndef SF_RASTER_GROUP_MB
#define SF_RASTER_GROUP_MB 32
#endif
constexpr long long kRasterGroupBytes = (long long)SF_RASTER_GROUP_MB << 20;

struct TcParams {
    int M, N, K;
    int bm;               // rows per tile: 128 (single CTA) or 256 (CTA pair)
    int num_m_tiles, num_n_tiles;
    int num_kb;
    int group_m;          // raster group height in m-tiles
    int num_units;        // dense: tiles; topk: m_tiles * n_chunks
    int n_chunks, tiles_per_chunk;
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
    unsigned *err;
    // topk
    int k;
    int topk_buf;              // candidate buffer depth per row (entries)
    int values_dtype;
    unsigned long long *cand;  // [M, n_chunks, k] packed keys
    // csr (encode straight to CSR staging)
    int32_t *tile_cnt;         // [M, num_n_tiles] nonzeros of each (row, n-tile)
    int32_t *tile_off;         // [M, num_n_tiles] their staging offset (where the count is > 0)
    int32_t *stage_idx;        // [stage_cap] feature ids
    void *stage_val;           // [stage_cap] values in out_dtype
    unsigned *csr_state;       // [0] staging cursor, [1] overflow flag
    unsigned stage_cap;
    // A operand of the converter warps (see GemmOperands)
    const void *xa;
    int64_t xa_pitch;
    const void *bdec;
    int bdec_dtype;
    int64_t bdec_stride;
    int bdec_mode;
    // split-operand K schedule and the early-exit flag (see GemmOperands)
    int seg_kb;
    uint32_t seg_a, seg_b;
    const unsigned *skip;
    // K-range partial sums (see EpilogueArgs): c_in added to the accumulators; raw: store them
    const float *c_in;
    int64_t c_in_pitch;
    int raw;
};

// TMEM accumulators of 32 columns at (row, col0) plus the partial sum of the earlier K ranges
// (fp32, round to nearest); the partial buffer is padded to whole tiles, so every column of
// a tile is in bounds.
// PART: instantiated only for the split-precision route (a runtime test in every epilogue
// cost the 16-bit kernels ~5% at config 2 through register pressure).
template <bool PART>
__device__ __forceinline__ void add_partial(const TcParams &p, int row, int col0, uint32_t (&r)[32]) {
    if constexpr (!PART) return;
    if (p.c_in == nullptr || row >= p.M) return;
    // plain loads: a raw pass reads and then rewrites these same addresses
    const float4 *src = reinterpret_cast<const float4 *>(p.c_in + (int64_t)row * p.c_in_pitch + col0);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 v = src[j / 4];
        r[j + 0] = __float_as_uint(__uint_as_float(r[j + 0]) + v.x);
        r[j + 1] = __float_as_uint(__uint_as_float(r[j + 1]) + v.y);
        r[j + 2] = __float_as_uint(__uint_as_float(r[j + 2]) + v.z);
        r[j + 3] = __float_as_uint(__uint_as_float(r[j + 3]) + v.w);
    }
}

// Raw epilogue of one 32-column chunk: the fp32 sums themselves (no bias, no activation) to
// the partial buffer, whole chunks (the buffer is padded to whole tiles).
__device__ __forceinline__ void raw_chunk(const TcParams &p, const uint32_t (&r)[32], int row, int col0) {
    if (row >= p.M) return;
    uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<float *>(p.out) + (int64_t)row * p.out_sm + col0);
#pragma unroll
    for (int j = 0; j < 32; j += 4) dst[j / 4] = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
}

// TMA K coordinates of K block kb in A and in B. Plain GEMM: both kb * bk. Split-operand
// schedule: block kb lies in segment pair s = kb / seg_kb, whose A and B segments come from
// the seg_a / seg_b nibbles.
__device__ __forceinline__ void k_coords(const TcParams &p, int kb, int bk, int &ka, int &kw) {
    if (p.seg_kb == 0) {
        ka = kw = kb * bk;
        return;
    }
    const int s = kb / p.seg_kb;
    const int off = (kb - s * p.seg_kb) * bk;
    const int span = p.seg_kb * bk;
    ka = (int)((p.seg_a >> (4 * s)) & 15u) * span + off;
    kw = (int)((p.seg_b >> (4 * s)) & 15u) * span + off;
}

// The split-precision encode's non-finite fallback: set before launch by the operand split.
__device__ __forceinline__ bool skip_launch(const TcParams &p) {
    return p.skip != nullptr && *reinterpret_cast<const volatile unsigned *>(p.skip) != 0u;
}

// The staged bias / cut arrays are read as float4: they must start on 16-byte boundaries.
struct __align__(16) TcShared {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    alignas(16) float bias[2][kBN];
    alignas(16) float thr[2][kBN];
};
static_assert(offsetof(TcShared, bias) % 16 == 0 && offsetof(TcShared, thr) % 16 == 0, "float4 staging");

// Unit u -> (m_blk, first n_blk, n-tile count).
struct Unit {
    int m_blk, n_first, n_count, chunk;
};

__device__ __forceinline__ Unit unit_coords(const TcParams &p, int u, int mode) {
    Unit r;
    if (mode != kTopk) {
        // One tile per unit, grouped raster: group_m m-tiles share each W n-tile in L2.
        const int per_group = p.group_m * p.num_n_tiles;
        const int g = u / per_group;
        const int first_m = g * p.group_m;
        const int gm = min(p.num_m_tiles - first_m, p.group_m);
        const int local = u - g * per_group;
        r.m_blk = first_m + local % gm;
        r.n_first = local / gm;
        r.n_count = 1;
        r.chunk = 0;
    } else {
        // Grouped raster over (m-tile, column chunk) units, m fastest: the units running at
        // once are group_m m-tiles on each of a few chunks, so each W_enc tile of a chunk is
        // fetched from HBM once per group (its other group_m - 1 uses hit L2) and each x
        // tile is shared by the chunks in flight. An m-tile-major order would instead pull
        // all of W_enc from HBM once per m-tile.
        const int per_group = p.group_m * p.n_chunks;
        const int g = u / per_group;
        const int first_m = g * p.group_m;
        const int gm = min(p.num_m_tiles - first_m, p.group_m);
        const int local = u - g * per_group;
        r.m_blk = first_m + local % gm;
        r.chunk = local / gm;
        r.n_first = r.chunk * p.tiles_per_chunk;
        r.n_count = min(p.tiles_per_chunk, p.num_n_tiles - r.n_first);
    }
    return r;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Largest fp32 value that rounds to zero when stored in `dtype` (round to nearest even):
// half the smallest subnormal of bf16 (2^-134) and fp16 (2^-25), 0 for fp32.
__device__ __forceinline__ float zero_cut(int dtype) {
    if (dtype == SF_BF16) return __uint_as_float(0x00008000u);  // 2^-134 (an fp32 subnormal)
    if (dtype == SF_F16) return __uint_as_float(0x33000000u);   // 2^-25
    return 0.f;
}

// Stage this tile's b_enc / threshold in fp32 (double-buffered by tile parity). In CSR mode
// the second array holds the cut: a stored value is nonzero exactly when pre > cut, with
// cut = max(threshold, zero_cut) for JumpReLU (never for a NaN threshold) and zero_cut for
// ReLU, since v = relu(pre) (or 0 unless pre > threshold) rounds to zero iff v <= zero_cut.
__device__ __forceinline__ void stage_bias(const TcParams &p, TcShared *sh, int mode, int et, int n_blk, int buf) {
    const float zc = zero_cut(p.out_dtype);
    for (int j = et; j < kBN; j += 128) {
        const int col = n_blk * kBN + j;
        float b = 0.f, t = 0.f;
        if (col < p.N) {
            b = load_as_f32(p.b_enc, p.b_enc_dtype, (int64_t)col * p.b_enc_stride);
            if (mode != kTopk && p.activation == SF_ACT_JUMPRELU)
                t = load_as_f32(p.thr, p.thr_dtype, (int64_t)col * p.thr_stride);
            if (mode == kCsr) t = p.activation == SF_ACT_JUMPRELU ? (t != t ? __int_as_float(0x7f800000) : fmaxf(t, zc)) : zc;
        } else if (mode == kCsr) {
            t = __int_as_float(0x7f800000);  // +inf: columns past d_sae never fire
        } else if (mode == kTopk) {
            b = __int_as_float(0xff800000);  // -inf: columns past d_sae never enter a top-k list
        }
        sh->bias[buf][j] = b;
        sh->thr[buf][j] = t;
    }
}

// Packs two fp32 values to the 16-bit output type (round to nearest even); returns the bits.
template <typename OT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Dense epilogue of one 32-column chunk: bias, activation, rounding to OT, nonzero count on
// the stored bits, 16-byte stores. FULL: all 32 columns are inside d_sae.
template <typename OT, bool JUMP, bool FULL>
__device__ __forceinline__ void dense_chunk(const TcParams &p, const float *bias, const float *thr,
                                            const uint32_t (&r)[32], int row, int col0, uint64_t pol_out,
                                            int &cnt) {
    float o[32];
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 b4 = *reinterpret_cast<const float4 *>(bias + j);
        float4 t4;
        if (JUMP) t4 = *reinterpret_cast<const float4 *>(thr + j);
        const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
        const float tt[4] = {JUMP ? t4.x : 0.f, JUMP ? t4.y : 0.f, JUMP ? t4.z : 0.f, JUMP ? t4.w : 0.f};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float pre = __uint_as_float(r[j + e]) + bb[e];
            float v = fmaxf(pre, 0.f);
            if (JUMP) v = (pre > tt[e]) ? v : 0.f;
            o[j + e] = (FULL || col0 + j + e < p.N) ? v : 0.f;
        }
    }
    OT *base = reinterpret_cast<OT *>(p.out) + (int64_t)row * p.out_sm;
    if constexpr (sizeof(OT) == 2) {
        uint32_t pk[16];
        uint32_t nz2 = 0;  // per-halfword nonzero counts
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            pk[j] = pack2<OT>(o[2 * j], o[2 * j + 1]);
            nz2 += __vsetne2(pk[j] & 0x7FFF7FFFu, 0u);
        }
        cnt += (int)(nz2 & 0xFFFFu) + (int)(nz2 >> 16);
        if (row < p.M) {
            if (FULL && p.out_vec) {
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                    st_global_v4_hint(base + col0 + 2 * j, make_uint4(pk[j], pk[j + 1], pk[j + 2], pk[j + 3]),
                                      pol_out);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (!FULL && col0 + j >= p.N) break;
                    const uint16_t bits = (j & 1) ? (uint16_t)(pk[j >> 1] >> 16) : (uint16_t)(pk[j >> 1] & 0xFFFFu);
                    reinterpret_cast<uint16_t *>(base)[(int64_t)(col0 + j) * p.out_sn] = bits;
                }
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) cnt += (o[j] != 0.f) ? 1 : 0;
        if (row < p.M) {
            if (FULL && p.out_vec) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    st_global_v4_hint(base + col0 + j,
                                      make_uint4(__float_as_uint(o[j]), __float_as_uint(o[j + 1]),
                                                 __float_as_uint(o[j + 2]), __float_as_uint(o[j + 3])),
                                      pol_out);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (!FULL && col0 + j >= p.N) break;
                    reinterpret_cast<float *>(base)[(int64_t)(col0 + j) * p.out_sn] = o[j];
                }
            }
        }
    }
}

// Per-row top-k state of an epilogue thread. Its list of k packed (value, ~column) keys
// lives in shared memory at topk_lists[s * 128 + et], unordered; `min_key` / `min_slot`
// name its smallest entry once the list is full. Columns that beat the k-th largest seen so
// far (`min_val`, refreshed at each merge) are appended to a per-row candidate buffer
// (topk_buf[i * 128 + et]), and the buffers of a warp's 32 rows are merged into their lists
// together, so one row's insertions never serialise the other 31 rows of the warp.
struct TopkState {
    unsigned long long min_key;  // smallest list key (0 while the list is not full)
    int min_slot;
    int fill;                    // list entries in use (< k while filling)
    int cnt;                     // buffered candidates
    float min_val;               // value part of min_key, -1 while the list is not full
};

__device__ __forceinline__ void topk_reset(TopkState &ts) {
    ts.min_key = 0ull;
    ts.min_slot = 0;
    ts.fill = 0;
    ts.cnt = 0;
    ts.min_val = -1.f;
}

__device__ __forceinline__ float min_value_of(unsigned long long min_key) {
    return __uint_as_float(static_cast<uint32_t>(min_key >> 32));
}

// Smallest key of this thread's full list and its slot: four interleaved compare chains
// over independent shared-memory loads.
__device__ __forceinline__ void topk_rescan(const unsigned long long *lists, int et, int k, TopkState &ts) {
    unsigned long long m[4] = {~0ull, ~0ull, ~0ull, ~0ull};
    int ms[4] = {0, 0, 0, 0};
    int s = 0;
#pragma unroll 2
    for (; s + 4 <= k; s += 4) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const unsigned long long q = lists[(s + c) * 128 + et];
            if (q < m[c]) {
                m[c] = q;
                ms[c] = s + c;
            }
        }
    }
    for (; s < k; ++s) {
        const unsigned long long q = lists[s * 128 + et];
        if (q < m[0]) {
            m[0] = q;
            ms[0] = s;
        }
    }
#pragma unroll
    for (int c = 1; c < 4; ++c) {
        if (m[c] < m[0]) {
            m[0] = m[c];
            ms[0] = ms[c];
        }
    }
    ts.min_key = m[0];
    ts.min_slot = ms[0];
}

// Merges this thread's buffered candidates (in column order) into its list: the first k
// fill the list, each later one replaces the smallest entry when it is larger. Out of line
// and by value, so the state stays in registers on the per-column path.
__device__ __noinline__ TopkState topk_merge_buffer(unsigned long long *lists, const unsigned long long *buf,
                                                    int et, int k, TopkState ts) {
    for (int i = 0; i < ts.cnt; ++i) {
        const unsigned long long key = buf[i * 128 + et];
        if (ts.fill < k) {
            lists[ts.fill * 128 + et] = key;
            if (++ts.fill == k) topk_rescan(lists, et, k, ts);
        } else if (key > ts.min_key) {
            lists[ts.min_slot * 128 + et] = key;
            topk_rescan(lists, et, k, ts);
        }
    }
    ts.cnt = 0;
    ts.min_val = ts.fill < k ? -1.f : min_value_of(ts.min_key);
    return ts;
}

// Top-k epilogue of one 32-column chunk, in groups of kTopkGroup columns: values are
// compared against the k-th largest of the previous merge in fp32 (rounding is monotonic,
// so a value not above it cannot enter) and survivors are buffered as packed keys. After
// each group the warp merges its buffers if any row's buffer could overflow on the next
// group (the host guarantees topk_buf >= kTopkGroup).
constexpr int kTopkGroup = 8;
__device__ __forceinline__ void topk_chunk(const TcParams &p, const float *bias, const uint32_t (&r)[32], int col0,
                                           unsigned long long *topk_lists, int et, TopkState &ts) {
    // pre-activations of the chunk (bias read as float4; -inf past d_sae) and their maximum:
    // once the lists are full, most chunks hold no column above any of the warp's 32 running
    // k-th values, and the whole chunk is skipped on that one test.
    float pre[32];
    float mx = __int_as_float(0xff800000);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 b4 = *reinterpret_cast<const float4 *>(bias + j);
        pre[j + 0] = __uint_as_float(r[j + 0]) + b4.x;
        pre[j + 1] = __uint_as_float(r[j + 1]) + b4.y;
        pre[j + 2] = __uint_as_float(r[j + 2]) + b4.z;
        pre[j + 3] = __uint_as_float(r[j + 3]) + b4.w;
        mx = fmaxf(mx, fmaxf(fmaxf(pre[j], pre[j + 1]), fmaxf(pre[j + 2], pre[j + 3])));
    }
    // relu(pre) > min_val needs pre > min_val when min_val >= 0 (NaN pre stores 0 and never
    // enters then); while a list is filling (min_val = -1) every column below d_sae enters
    const bool need = col0 < p.N && (ts.min_val < 0.f || mx > ts.min_val);
    if (!__any_sync(0xffffffffu, need)) return;
    unsigned long long *buf = topk_lists + p.k * 128;
#pragma unroll
    for (int g = 0; g < 32; g += kTopkGroup) {
        const float min_val = ts.min_val;
#pragma unroll
        for (int j = g; j < g + kTopkGroup; ++j) {
            const int col = col0 + j;
            const float o = fmaxf(pre[j], 0.f);
            if (o > min_val && col < p.N) {
                const float v = round_to(o, p.values_dtype);
                buf[ts.cnt * 128 + et] =
                    (static_cast<unsigned long long>(__float_as_uint(v) & 0x7FFFFFFFu) << 32) |
                    static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(col));
                ++ts.cnt;
            }
        }
        if (__any_sync(0xffffffffu, ts.cnt > p.topk_buf - kTopkGroup))
            ts = topk_merge_buffer(topk_lists, buf, et, p.k, ts);
    }
}

// CSR pass 1 of one 32-column chunk: bit j of the returned mask is set when column col0+j
// stores a nonzero value, i.e. when pre = acc + b_enc exceeds the staged cut (which is +inf
// past d_sae).
__device__ __forceinline__ uint32_t csr_chunk_mask(const float *bias, const float *cut, const uint32_t (&r)[32]) {
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 b4 = *reinterpret_cast<const float4 *>(bias + j);
        const float4 c4 = *reinterpret_cast<const float4 *>(cut + j);
        m |= (__uint_as_float(r[j + 0]) + b4.x > c4.x ? 1u : 0u) << (j + 0);
        m |= (__uint_as_float(r[j + 1]) + b4.y > c4.y ? 1u : 0u) << (j + 1);
        m |= (__uint_as_float(r[j + 2]) + b4.z > c4.z ? 1u : 0u) << (j + 2);
        m |= (__uint_as_float(r[j + 3]) + b4.w > c4.w ? 1u : 0u) << (j + 3);
    }
    return m;
}

// CSR pass 2 of one chunk: writes the (column, value) pairs of the set bits of `m` to the
// staging arrays from `o` on, in column order. A set bit means pre > threshold, so the
// stored value is relu(pre) rounded to OT.
template <typename OT>
__device__ __forceinline__ void csr_chunk_emit(const TcParams &p, const float *bias, const uint32_t (&r)[32],
                                               int col0, uint32_t m, unsigned &o) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (m & (1u << j)) {
            const float v = fmaxf(__uint_as_float(r[j]) + bias[j], 0.f);
            p.stage_idx[o] = col0 + j;
            reinterpret_cast<OT *>(p.stage_val)[o] = from_f32<OT>(v);
            ++o;
        }
    }
}

// CSR epilogue of one tile: pass 1 over all chunks finds each row's nonzeros, one atomicAdd
// per warp reserves staging space for the warp's 32 rows, pass 2 re-reads from TMEM only the
// chunks where some row of the warp has a nonzero and emits them.
template <typename OT, bool PART, typename Release>
__device__ __forceinline__ void csr_tile(const TcParams &p, const TcShared *sh, int row, int n_blk, int buf,
                                         uint32_t taddr, Release release) {
    constexpr int NC = kBN / 32;
    const bool live = row < p.M;
    uint32_t masks[NC];
    int cnt = 0;
    uint32_t ra[32], rb[32];
    const int col_base = n_blk * kBN;
    tmem_ld_32x32b_x32(taddr, ra);
    tmem_ld_wait();
#pragma unroll
    for (int c = 0; c < NC; c += 2) {
        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
        add_partial<PART>(p, row, col_base + c * 32, ra);
        masks[c] = csr_chunk_mask(&sh->bias[buf][c * 32], &sh->thr[buf][c * 32], ra);
        tmem_ld_wait();
        if (c + 2 < NC) tmem_ld_32x32b_x32(taddr + (c + 2) * 32, ra);
        add_partial<PART>(p, row, col_base + (c + 1) * 32, rb);
        masks[c + 1] = csr_chunk_mask(&sh->bias[buf][(c + 1) * 32], &sh->thr[buf][(c + 1) * 32], rb);
        if (c + 2 < NC) tmem_ld_wait();
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        if (!live) masks[c] = 0;
        cnt += __popc(masks[c]);
    }
    // Reserve staging space for the warp's rows with one atomic.
    const int lane = (int)lane_id();
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    unsigned base = 0;
    if (lane == 31 && total > 0) base = atomicAdd(&p.csr_state[0], (unsigned)total);
    base = __shfl_sync(0xffffffffu, base, 31);
    unsigned o = base + (unsigned)(incl - cnt);
    const bool fits = (unsigned long long)base + (unsigned long long)total <= (unsigned long long)p.stage_cap;
    if (lane == 31 && total > 0 && !fits) atomicOr(&p.csr_state[1], 1u);
    if (live) {
        const int64_t cell = (int64_t)row * p.num_n_tiles + n_blk;
        p.tile_cnt[cell] = cnt;
        if (cnt) p.tile_off[cell] = (int)o;
        if (p.row_nnz != nullptr && cnt) atomicAdd(p.row_nnz + row, cnt);
    }
    if (fits) {
#pragma unroll 1
        for (int c = 0; c < NC; ++c) {
            if (__any_sync(0xffffffffu, masks[c] != 0)) {
                uint32_t rr[32];
                tmem_ld_32x32b_x32(taddr + c * 32, rr);
                tmem_ld_wait();
                if (masks[c]) {
                    add_partial<PART>(p, row, col_base + c * 32, rr);
                    csr_chunk_emit<OT>(p, &sh->bias[buf][c * 32], rr, n_blk * kBN + c * 32, masks[c], o);
                }
            }
        }
    }
    release();  // all TMEM reads of this tile have completed
}

// One tile of epilogue for this thread's row: reads the 256 fp32 accumulators of its TMEM
// lane 32 columns at a time, loading chunk c+1 while chunk c is processed; `release` runs
// once all TMEM reads of the tile are complete, so the MMA warp may reuse the buffer.
template <int MODE, typename OT, bool JUMP, bool PART, typename Release>
__device__ __forceinline__ void epilogue_tile_t(const TcParams &p, const TcShared *sh, unsigned long long *topk_lists,
                                                int et, int row, int n_blk, int buf, uint32_t taddr,
                                                uint64_t pol_out, TopkState &ts,
                                                Release release) {
    constexpr int NC = kBN / 32;
    const bool full_tile = (n_blk + 1) * kBN <= p.N;
    int cnt = 0;
    auto process = [&](uint32_t(&r)[32], int c) {
        const int col0 = n_blk * kBN + c * 32;
        const float *bias = &sh->bias[buf][c * 32];
        if constexpr (MODE == kDense) {
            add_partial<PART>(p, row, col0, r);
            if (PART && p.raw)
                raw_chunk(p, r, row, col0);
            else if (full_tile)
                dense_chunk<OT, JUMP, true>(p, bias, &sh->thr[buf][c * 32], r, row, col0, pol_out, cnt);
            else
                dense_chunk<OT, JUMP, false>(p, bias, &sh->thr[buf][c * 32], r, row, col0, pol_out, cnt);
        } else {
            topk_chunk(p, bias, r, col0, topk_lists, et, ts);
        }
    };
    // Two register buffers: the load of the next chunk is in flight while one is processed.
    uint32_t ra[32], rb[32];
    tmem_ld_32x32b_x32(taddr, ra);
    tmem_ld_wait();
#pragma unroll 1
    for (int c = 0; c < NC; c += 2) {
        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
        process(ra, c);
        tmem_ld_wait();
        if (c + 2 < NC)
            tmem_ld_32x32b_x32(taddr + (c + 2) * 32, ra);
        else
            release();  // every TMEM read of this tile has completed
        process(rb, c + 1);
        if (c + 2 < NC) tmem_ld_wait();
    }
    if (MODE == kDense && p.row_nnz != nullptr && row < p.M && cnt != 0) atomicAdd(p.row_nnz + row, cnt);
}

template <int MODE, bool PART, typename Release>
__device__ __forceinline__ void epilogue_tile(const TcParams &p, const TcShared *sh, unsigned long long *topk_lists,
                                              int et, int row, int n_blk, int buf, uint32_t taddr, uint64_t pol_out,
                                              TopkState &ts, Release release) {
    if constexpr (MODE == kCsr) {
        if (p.out_dtype == SF_BF16)
            csr_tile<__nv_bfloat16, PART>(p, sh, row, n_blk, buf, taddr, release);
        else if (p.out_dtype == SF_F16)
            csr_tile<__half, PART>(p, sh, row, n_blk, buf, taddr, release);
        else
            csr_tile<float, PART>(p, sh, row, n_blk, buf, taddr, release);
        return;
    }
    if constexpr (MODE == kTopk) {
        epilogue_tile_t<kTopk, float, false, false>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out, ts, release);
        return;
    }
    const bool jump = p.activation == SF_ACT_JUMPRELU;
    if (p.out_dtype == SF_BF16) {
        if (jump)
            epilogue_tile_t<kDense, __nv_bfloat16, true, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out,
                                                         ts, release);
        else
            epilogue_tile_t<kDense, __nv_bfloat16, false, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out,
                                                          ts, release);
    } else if (p.out_dtype == SF_F16) {
        if (jump)
            epilogue_tile_t<kDense, __half, true, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out, ts, release);
        else
            epilogue_tile_t<kDense, __half, false, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out, ts, release);
    } else {
        if (jump)
            epilogue_tile_t<kDense, float, true, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out, ts, release);
        else
            epilogue_tile_t<kDense, float, false, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out, ts, release);
    }
}

// ------------------------------------------------------------------ fused shift (A converter)
// The 16-bit CTA-pair kernel builds its A tiles itself: four converter warps per CTA read
// 16-byte chunks of x rows from global memory (L2), compute (x - b_dec) in fp32 and round it
// to the MMA dtype (the reference prologue, saeflow/kernels/encode.py:72), and store the
// chunks in the 128-byte-swizzled layout the MMA descriptors expect. This takes the place
// of both the separate shift pass over x (a read and a write of x in HBM) and the TMA load
// of the shifted copy; shared-memory traffic is unchanged (the converters write what the
// TMA wrote).
constexpr int kConvThreads = 128;

// -b_dec[k0 .. k0+8) in fp32 pairs (zeros without a shift or past K).
__device__ __forceinline__ void neg_bdec_chunk(const TcParams &p, int k0, float2 (&nb)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) nb[i] = make_float2(0.f, 0.f);
    if (p.bdec_mode == 0 || k0 >= p.K) return;
    if (p.bdec_mode == 1) {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(p.bdec) + k0));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f;
            if (p.bdec_dtype == SF_BF16) {
                f = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
            } else {
                __half2 h;
                memcpy(&h, &w[i], 4);
                f = __half22float2(h);
            }
            nb[i] = make_float2(-f.x, -f.y);
        }
    } else if (p.bdec_mode == 2) {
        const float4 *b4 = reinterpret_cast<const float4 *>(static_cast<const float *>(p.bdec) + k0);
        const float4 a = __ldg(b4), b = __ldg(b4 + 1);
        nb[0] = make_float2(-a.x, -a.y), nb[1] = make_float2(-a.z, -a.w);
        nb[2] = make_float2(-b.x, -b.y), nb[3] = make_float2(-b.z, -b.w);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            nb[i] = make_float2(-load_as_f32(p.bdec, p.bdec_dtype, (int64_t)(k0 + 2 * i) * p.bdec_stride),
                                -load_as_f32(p.bdec, p.bdec_dtype, (int64_t)(k0 + 2 * i + 1) * p.bdec_stride));
    }
}

// Eight 16-bit elements of x plus -b_dec in fp32, rounded to nearest in the same 16-bit type.
template <int AB_FMT>
__device__ __forceinline__ uint4 shift_chunk(uint4 v, const float2 (&nb)[4]) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (AB_FMT == 1) {
            const float2 f = __fadd2_rn(make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u)),
                                        nb[i]);
            const __nv_bfloat162 r = __float22bfloat162_rn(f);
            memcpy(&w[i], &r, 4);
        } else {
            __half2 h;
            memcpy(&h, &w[i], 4);
            const float2 f = __fadd2_rn(__half22float2(h), nb[i]);
            const __half2 r = __float22half2_rn(f);
            memcpy(&w[i], &r, 4);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int AB_FMT, bool B_MN, int MODE, int STAGES, bool PART>
__global__ void __launch_bounds__(kThreads, 1)
    encode_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const TcParams p) {
    constexpr int ES = (AB_FMT == 2) ? 4 : 2;  // operand element bytes
    constexpr int BK = 128 / ES;               // K elements per stage (one 128 B swizzle row)
    constexpr int UMMA_K = 32 / ES;            // K per tcgen05.mma
    constexpr int KSTEPS = BK / UMMA_K;        // 4
    constexpr int MN_BOX = 128 / ES;           // MN-major B: elements per 128 B chunk
    constexpr int MN_BOX_BYTES = BK * 128;     // one MN chunk: BK rows x 128 B
    constexpr uint32_t IDESC = make_idesc(AB_FMT, B_MN, kBM, kBN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * kTileABytes;
    TcShared *sh = reinterpret_cast<TcShared *>(smem + STAGES * kStageBytes);
    unsigned long long *topk_lists = reinterpret_cast<unsigned long long *>(sh + 1);  // [k][128]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (skip_launch(p)) return;  // before any barrier or TMEM allocation

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&sh->full[s], 1);
            mbar_init(&sh->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sh->tmem_full[b], 1);
            mbar_init(&sh->tmem_empty[b], 128);
        }
        mbar_init(&sh->drain, 1);
        sh->abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(&sh->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = sh->tmem_base;
    volatile int *abort_flag = &sh->abort_flag;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            const uint64_t pol_x = l2_policy_evict_last();
            const uint64_t pol_w = l2_policy_evict_normal();
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0;  // bit s: stage s armed at least once
            uint32_t armed_parity = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                const Unit un = unit_coords(p, u, MODE);
                for (int nt = 0; ok && nt < un.n_count; ++nt) {
                    const int n_blk = un.n_first + nt;
                    for (int kb = 0; kb < p.num_kb; ++kb) {
                        if (!mbar_wait(&sh->empty[stage], phase ^ 1u, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&sh->full[stage], kStageBytes);
                        armed |= 1u << stage;
                        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
                        uint8_t *a_dst = sA + stage * kTileABytes;
                        uint8_t *b_dst = sB + stage * kTileBBytes;
                        int ka, kw;
                        k_coords(p, kb, BK, ka, kw);
                        tma_load_2d(a_dst, &tmA, &sh->full[stage], ka, un.m_blk * kBM, pol_x);
                        if (B_MN) {
#pragma unroll
                            for (int j = 0; j < kBN / MN_BOX; ++j)
                                tma_load_2d(b_dst + j * MN_BOX_BYTES, &tmB, &sh->full[stage],
                                            n_blk * kBN + j * MN_BOX, kw, pol_w);
                        } else {
                            tma_load_2d(b_dst, &tmB, &sh->full[stage], kw, n_blk * kBN, pol_w);
                        }
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (*abort_flag) {
                // Let every copy this thread issued land before shared memory goes away.
                for (int s = 0; s < STAGES; ++s)
                    if (armed & (1u << s)) mbar_wait_drain(&sh->full[s], (armed_parity >> s) & 1u, p.err);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                const Unit un = unit_coords(p, u, MODE);
                for (int nt = 0; ok && nt < un.n_count; ++nt) {
                    if (!mbar_wait(&sh->tmem_empty[acc], acc_phase ^ 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * kAccCols;
                    for (int kb = 0; kb < p.num_kb; ++kb) {
                        if (!mbar_wait(&sh->full[stage], phase, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = smem_u32(sA + stage * kTileABytes);
                        const uint32_t b_addr = smem_u32(sB + stage * kTileBBytes);
#pragma unroll
                        for (int ks = 0; ks < KSTEPS; ++ks) {
                            const uint64_t ad = smem_desc_sw128(a_addr + ks * 32, 16, 1024);
                            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + ks * UMMA_K * 128, MN_BOX_BYTES, 1024)
                                                     : smem_desc_sw128(b_addr + ks * 32, 16, 1024);
                            const uint32_t accum = (kb > 0 || ks > 0) ? 1u : 0u;
                            if (AB_FMT == 2)
                                umma_tf32(d_tmem, ad, bd, IDESC, accum);
                            else
                                umma_f16(d_tmem, ad, bd, IDESC, accum);
                        }
                        umma_commit(&sh->empty[stage]);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    umma_commit(&sh->tmem_full[acc]);
                    if (++acc == 2) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                }
            }
            // Every MMA this thread issued has finished once `drain` completes.
            umma_commit(&sh->drain);
            mbar_wait_drain(&sh->drain, 0, p.err);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int et = threadIdx.x - 64;  // 0..127
        const int quad = warp & 3;        // TMEM lanes [32*quad, 32*quad+32)
        const int row_in_tile = quad * 32 + lane;
        const uint64_t pol_out = l2_policy_evict_first();
        int acc = 0;
        uint32_t acc_phase = 0;
        int tile_iter = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
            const Unit un = unit_coords(p, u, MODE);
            const int row = un.m_blk * kBM + row_in_tile;
            TopkState ts;
            topk_reset(ts);
            if (MODE == kTopk) {
                for (int s = 0; s < p.k; ++s) topk_lists[s * 128 + et] = 0ull;
            }
            for (int nt = 0; nt < un.n_count; ++nt, ++tile_iter) {
                const int n_blk = un.n_first + nt;
                const int buf = tile_iter & 1;
                stage_bias(p, sh, MODE, et, n_blk, buf);
                named_bar_sync(1, 128);
                if (!mbar_wait(&sh->tmem_full[acc], acc_phase, abort_flag, p.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * kAccCols;
                const int acc_now = acc;
                epilogue_tile<MODE, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out, ts, [&] {
                    tc_fence_before();
                    mbar_arrive(&sh->tmem_empty[acc_now]);
                });
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (MODE == kTopk && ok) ts = topk_merge_buffer(topk_lists, topk_lists + p.k * 128, et, p.k, ts);
            if (MODE == kTopk && ok && row < p.M) {
                unsigned long long *dst = p.cand + ((int64_t)row * p.n_chunks + un.chunk) * p.k;
                for (int s = 0; s < p.k; ++s) dst[s] = topk_lists[s * 128 + et];
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// -------------------------------------------------------------------------------------
// CTA-pair kernel (cluster of 2, tcgen05 cta_group::2): 256 x 256 tile per pair.
template <int AB_FMT, bool B_MN, int MODE, int STAGES, bool PART>
__global__ void __launch_bounds__((AB_FMT != 2 && kFusedShift) ? kThreads + kConvThreads : kThreads, 1)
    encode_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const TcParams p) {
    constexpr int ES = (AB_FMT == 2) ? 4 : 2;
    constexpr int BK = 128 / ES;
    constexpr int UMMA_K = 32 / ES;
    constexpr int KSTEPS = BK / UMMA_K;
    constexpr int MN_BOX = 128 / ES;
    constexpr int MN_BOX_BYTES = BK * 128;
    constexpr int HALF_N = kBN / 2;            // columns of W_enc this CTA holds per stage
    constexpr int A_BYTES = 128 * 128;         // 128 rows x 128 B
    constexpr int B_BYTES = HALF_N * 128;      // 128 columns x 128 B
    constexpr bool CONV_A = AB_FMT != 2 && kFusedShift;  // A tiles from the converter warps
    constexpr uint32_t PAIR_TX = CONV_A ? 2u * B_BYTES : 2u * (A_BYTES + B_BYTES);
    constexpr uint32_t IDESC = make_idesc(AB_FMT, B_MN, 256, kBN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    TcShared *sh = reinterpret_cast<TcShared *>(smem + STAGES * (A_BYTES + B_BYTES));
    unsigned long long *topk_lists = reinterpret_cast<unsigned long long *>(sh + 1);  // [k][128]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = (int)cluster_id_x();
    const int npairs = (int)num_clusters_x();
    // Both CTAs of the pair read the same flag, so both leave before any cluster barrier.
    if (skip_launch(p)) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            // leader's: its expect_tx arrive + both CTAs' TMA bytes (+ one arrive per
            // converter warp of both CTAs when the converters build A)
            mbar_init(&sh->full[s], CONV_A ? 1 + 2 * kConvThreads / 32 : 1);
            mbar_init(&sh->empty[s], 1);  // one commit from the leader's MMA thread
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sh->tmem_full[b], 1);
            mbar_init(&sh->tmem_empty[b], 8);  // leader's: one arrive per epilogue warp of both CTAs
        }
        mbar_init(&sh->drain, 1);
        sh->abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(&sh->tmem_base, kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = sh->tmem_base;
    volatile int *abort_flag = &sh->abort_flag;
    const uint32_t peer_abort = map_to_rank(smem_u32(&sh->abort_flag), rank ^ 1u);
    // A wait that runs out (or sees the abort flag) also raises the other CTA's flag.
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_wait(bar, parity, abort_flag, p.err)) return true;
        st_remote_u32(peer_abort, 1u);
        return false;
    };
    // The same with cluster-scope acquire: for phases completed by the peer CTA's converter
    // warps, whose shared-memory writes the MMAs read.
    auto wait_cluster = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_wait_cluster(bar, parity, abort_flag, p.err)) return true;
        st_remote_u32(peer_abort, 1u);
        return false;
    };

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer (both CTAs)
        if (lane == 0) {
            const uint64_t pol_x = l2_policy_evict_last();
            const uint64_t pol_w = l2_policy_evict_normal();
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_parity = 0;
            bool ok = true;
            for (int u = pair; ok && u < p.num_units; u += npairs) {
                const Unit un = unit_coords(p, u, MODE);
                for (int nt = 0; ok && nt < un.n_count; ++nt) {
                    const int n_blk = un.n_first + nt;
                    for (int kb = 0; kb < p.num_kb; ++kb) {
                        if (!wait(&sh->empty[stage], phase ^ 1u)) {
                            ok = false;
                            break;
                        }
                        const uint32_t full_leader = map_to_rank(smem_u32(&sh->full[stage]), 0);
                        if (leader) {
                            mbar_arrive_expect_tx(&sh->full[stage], PAIR_TX);
                            armed |= 1u << stage;
                            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
                        }
                        int ka, kw;
                        k_coords(p, kb, BK, ka, kw);
                        if (!CONV_A)
                            tma_load_2d_pair(sA + stage * A_BYTES, &tmA, full_leader, ka,
                                             un.m_blk * 256 + (int)rank * 128, pol_x);
                        uint8_t *b_dst = sB + stage * B_BYTES;
                        const int n0 = n_blk * kBN + (int)rank * HALF_N;
                        if (B_MN) {
#pragma unroll
                            for (int j = 0; j < HALF_N / MN_BOX; ++j)
                                tma_load_2d_pair(b_dst + j * MN_BOX_BYTES, &tmB, full_leader, n0 + j * MN_BOX,
                                                 kw, pol_w);
                        } else {
                            tma_load_2d_pair(b_dst, &tmB, full_leader, kw, n0, pol_w);
                        }
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (*abort_flag) {
                if (leader) {
                    // Both CTAs' copies of every armed stage complete on these barriers.
                    for (int s = 0; s < STAGES; ++s)
                        if (armed & (1u << s)) mbar_wait_drain(&sh->full[s], (armed_parity >> s) & 1u, p.err);
                } else {
                    // This CTA's copies complete on the leader's barriers: give them time to land.
                    const unsigned long long t0 = global_timer_ns();
                    while (global_timer_ns() - t0 < 2000000ull) __nanosleep(1000);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (leader only)
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int u = pair; ok && u < p.num_units; u += npairs) {
                const Unit un = unit_coords(p, u, MODE);
                for (int nt = 0; ok && nt < un.n_count; ++nt) {
                    if (!wait(&sh->tmem_empty[acc], acc_phase ^ 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + acc * kAccCols;
                    for (int kb = 0; kb < p.num_kb; ++kb) {
                        if (!(CONV_A ? wait_cluster(&sh->full[stage], phase) : wait(&sh->full[stage], phase))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
                        const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                        for (int ks = 0; ks < KSTEPS; ++ks) {
                            const uint64_t ad = smem_desc_sw128(a_addr + ks * 32, 16, 1024);
                            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + ks * UMMA_K * 128, MN_BOX_BYTES, 1024)
                                                     : smem_desc_sw128(b_addr + ks * 32, 16, 1024);
                            const uint32_t accum = (kb > 0 || ks > 0) ? 1u : 0u;
                            if (AB_FMT == 2)
                                umma_tf32_pair(d_tmem, ad, bd, IDESC, accum);
                            else
                                umma_f16_pair(d_tmem, ad, bd, IDESC, accum);
                        }
                        const uint32_t e_off = smem_u32(&sh->empty[stage]);
                        umma_commit_pair(map_to_rank(e_off, 0));
                        umma_commit_pair(map_to_rank(e_off, 1));
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    const uint32_t f_off = smem_u32(&sh->tmem_full[acc]);
                    umma_commit_pair(map_to_rank(f_off, 0));
                    umma_commit_pair(map_to_rank(f_off, 1));
                    if (++acc == 2) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                }
            }
            umma_commit_pair(map_to_rank(smem_u32(&sh->drain), 0));
            mbar_wait_drain(&sh->drain, 0, p.err);
        }
    } else if (CONV_A && warp >= 6) {
        // ---------------------------------------------------------------- A converters (both CTAs)
        // Thread ct owns 16-byte chunk c = ct % 8 of the 128-byte K row of rows
        // ct / 8 + 16 i (i < 8) of this CTA's 128 rows, every stage. Stage j+1's loads are in
        // flight while stage j is converted and stored.
        const int ct = threadIdx.x - kThreads;
        const int c = ct & 7;
        const int r0 = ct >> 3;
        const uint32_t swz = (uint32_t)(((c ^ (r0 & 7)) << 4) + r0 * 128);  // r & 7 == r0 & 7 for every row
        const uint16_t *xa = static_cast<const uint16_t *>(p.xa);
        int u = pair, nt = 0, kb = 0;
        Unit un{};
        bool have = u < p.num_units;
        if (have) un = unit_coords(p, u, MODE);
        auto load = [&](uint4 (&v)[8], float2 (&nb)[4]) {
            const int k0 = kb * 64 + c * 8;
            const int64_t row_base = (int64_t)un.m_blk * 256 + (int)rank * 128 + r0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int64_t row = row_base + 16 * i;
                v[i] = (row < p.M && k0 < p.K)
                           ? __ldg(reinterpret_cast<const uint4 *>(xa + row * p.xa_pitch + k0))
                           : make_uint4(0u, 0u, 0u, 0u);
            }
            neg_bdec_chunk(p, k0, nb);
        };
        auto advance = [&]() {
            if (++kb < p.num_kb) return;
            kb = 0;
            if (++nt < un.n_count) return;
            nt = 0;
            u += npairs;
            have = u < p.num_units;
            if (have) un = unit_coords(p, u, MODE);
        };
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        uint4 va[8], vb[8];
        float2 na[4], nb[4];
        auto put = [&](const uint4 (&v)[8], const float2 (&n)[4]) -> bool {
            if (!wait(&sh->empty[stage], phase ^ 1u)) return false;
            uint8_t *dst = sA + stage * A_BYTES + swz;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                *reinterpret_cast<uint4 *>(dst + i * 16 * 128) = shift_chunk<AB_FMT>(v[i], n);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(map_to_rank(smem_u32(&sh->full[stage]), 0));
            if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
            }
            return true;
        };
        if (have) load(va, na);
        while (ok && have) {
            advance();
            const bool next = have;
            if (next) load(vb, nb);
            ok = put(va, na);
            if (!ok || !next) break;
            advance();
            const bool next2 = have;
            if (next2) load(va, na);
            ok = put(vb, nb);
            if (!next2) break;
        }
    } else if (warp < 6) {
        // ---------------------------------------------------------------- epilogue (both CTAs)
        const int et = threadIdx.x - 64;
        const int quad = warp & 3;
        const int row_in_tile = (int)rank * 128 + quad * 32 + lane;
        const uint64_t pol_out = l2_policy_evict_first();
        int acc = 0;
        uint32_t acc_phase = 0;
        int tile_iter = 0;
        bool ok = true;
        for (int u = pair; ok && u < p.num_units; u += npairs) {
            const Unit un = unit_coords(p, u, MODE);
            const int row = un.m_blk * 256 + row_in_tile;
            TopkState ts;
            topk_reset(ts);
            if (MODE == kTopk) {
                for (int s = 0; s < p.k; ++s) topk_lists[s * 128 + et] = 0ull;
            }
            for (int nt = 0; nt < un.n_count; ++nt, ++tile_iter) {
                const int n_blk = un.n_first + nt;
                const int buf = tile_iter & 1;
                stage_bias(p, sh, MODE, et, n_blk, buf);
                named_bar_sync(1, 128);
                if (!wait(&sh->tmem_full[acc], acc_phase)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * kAccCols;
                const uint32_t empty_leader = map_to_rank(smem_u32(&sh->tmem_empty[acc]), 0);
                epilogue_tile<MODE, PART>(p, sh, topk_lists, et, row, n_blk, buf, taddr, pol_out, ts, [&] {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(empty_leader);
                });
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (MODE == kTopk && ok) ts = topk_merge_buffer(topk_lists, topk_lists + p.k * 128, et, p.k, ts);
            if (MODE == kTopk && ok && row < p.M) {
                unsigned long long *dst = p.cand + ((int64_t)row * p.n_chunks + un.chunk) * p.k;
                for (int s = 0; s < p.k; ++s) dst[s] = topk_lists[s * 128 + et];
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the leader's MMAs no longer read this CTA's shared memory
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// -------------------------------------------------------------------------------------
// Tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry point).
PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

int make_map_2d(CUtensorMap *map, const void *base, int ab_fmt, uint64_t inner, uint64_t outer,
                uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer) {
    auto fn = get_encode_tiled();
    if (!fn) return set_error(SF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const CUtensorMapDataType dt = ab_fmt == 2   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : ab_fmt == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) inner=%llu outer=%llu pitch=%llu", (int)r,
                         (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)row_pitch_bytes);
    return SF_OK;
}

template <int AB_FMT, bool B_MN, int MODE, int STAGES, bool PART>
int launch_single(const CUtensorMap &tmA, const CUtensorMap &tmB, const TcParams &p, size_t extra_smem,
                  cudaStream_t stream) {
    auto kern = encode_tc_kernel<AB_FMT, B_MN, MODE, STAGES, PART>;
    const size_t smem = 1024 + (size_t)STAGES * kStageBytes + sizeof(TcShared) + extra_smem;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(encode_tc)");
    const int grid = std::max(1, std::min(p.num_units, num_sms()));
    kern<<<grid, kThreads, smem, stream>>>(tmA, tmB, p);
    return check_cuda(cudaGetLastError(), "encode_tc launch");
}

template <int AB_FMT, bool B_MN, int MODE, int STAGES, bool PART>
int launch_pair(const CUtensorMap &tmA, const CUtensorMap &tmB, const TcParams &p, size_t extra_smem,
                cudaStream_t stream) {
    auto kern = encode_tc2_kernel<AB_FMT, B_MN, MODE, STAGES, PART>;
    constexpr int threads = (AB_FMT != 2 && kFusedShift) ? kThreads + kConvThreads : kThreads;
    const size_t smem = 1024 + (size_t)STAGES * (kBM * 128 + (kBN / 2) * 128) + sizeof(TcShared) + extra_smem;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(encode_tc2)");
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * std::max(1, num_sms() / 2));
    const int pairs = pair_slots(reinterpret_cast<const void *>(kern), cfg);
    cfg.gridDim = dim3(2 * std::max(1, std::min(p.num_units, pairs)));
    e = cudaLaunchKernelEx(&cfg, kern, tmA, tmB, p);
    if (e != cudaSuccess) return check_cuda(e, "encode_tc2 launch");
    return check_cuda(cudaGetLastError(), "encode_tc2 launch");
}

template <int MODE, int STAGES, bool PAIR>
int dispatch(int ab_fmt, bool b_mn, const CUtensorMap &tmA, const CUtensorMap &tmB, const TcParams &p,
             size_t extra_smem, cudaStream_t s) {
#define SF_LAUNCH(F, MN, PART) \
    (PAIR ? launch_pair<F, MN, MODE, STAGES, PART>(tmA, tmB, p, extra_smem, s) \
          : launch_single<F, MN, MODE, STAGES, PART>(tmA, tmB, p, extra_smem, s))
    if (p.c_in != nullptr || p.raw) {
        // K-range partial sums: the split-precision route only (bf16 operands, MN-major B)
        if constexpr (MODE == kTopk) {
            return set_error(SF_ERR_UNSUPPORTED, "partial sums are not supported by the top-k epilogue");
        } else {
            if (ab_fmt != 1 || !b_mn) return set_error(SF_ERR_UNSUPPORTED, "partial sums need split bf16 operands");
            return SF_LAUNCH(1, true, true);
        }
    }
    if (ab_fmt == 1) return b_mn ? SF_LAUNCH(1, true, false) : SF_LAUNCH(1, false, false);
    if (ab_fmt == 0) return b_mn ? SF_LAUNCH(0, true, false) : SF_LAUNCH(0, false, false);
    return b_mn ? SF_LAUNCH(2, true, false) : SF_LAUNCH(2, false, false);
#undef SF_LAUNCH
}

// Tensor maps: A boxes of 128 rows; B boxes of 256 (single CTA) or 128 (per CTA of a pair)
// columns when K-major, 128 B x BK rows when MN-major.
int build_maps(const GemmOperands &g, bool pair, CUtensorMap *tmA, CUtensorMap *tmB) {
    const int es = g.ab_fmt == 2 ? 4 : 2;
    const uint32_t bk = 128 / es;
    int st = make_map_2d(tmA, g.a, g.ab_fmt, (uint64_t)g.K, (uint64_t)g.M, (uint64_t)g.a_pitch * es, bk, kBM);
    if (st) return st;
    if (g.b_mn_major)  // W[k, n] at b + k*b_pitch + n
        return make_map_2d(tmB, g.b, g.ab_fmt, (uint64_t)g.N, (uint64_t)g.K, (uint64_t)g.b_pitch * es, 128 / es, bk);
    // W[k, n] at b + n*b_pitch + k
    return make_map_2d(tmB, g.b, g.ab_fmt, (uint64_t)g.K, (uint64_t)g.N, (uint64_t)g.b_pitch * es, bk,
                       pair ? kBN / 2 : kBN);
}

void fill_common(TcParams &p, const GemmOperands &g, bool pair, unsigned *err) {
    const int es = g.ab_fmt == 2 ? 4 : 2;
    p.M = (int)g.M;
    p.N = (int)g.N;
    p.K = (int)g.K;
    p.bm = pair ? 256 : kBM;
    p.num_m_tiles = (int)((g.M + p.bm - 1) / p.bm);
    p.num_n_tiles = (int)((g.N + kBN - 1) / kBN);
    p.num_kb = (int)((g.K + (128 / es) - 1) / (128 / es));
    p.seg_kb = g.seg_kb;
    p.seg_a = g.seg_a;
    p.seg_b = g.seg_b;
    p.skip = g.skip;
    if (g.seg_kb > 0) p.num_kb = kEmuPairs * g.seg_kb;
    p.err = err;
    p.xa = g.a;
    p.xa_pitch = g.a_pitch;
    p.bdec = g.bdec;
    p.bdec_dtype = g.bdec_dtype;
    p.bdec_stride = g.bdec_stride;
    p.bdec_mode = g.bdec ? g.bdec_mode : 0;
}

}  // namespace

// Pairs of SMs that can hold one pair-kernel cluster each (cached per kernel).
int pair_slots(const void *kern, const cudaLaunchConfig_t &cfg) {
    static std::mutex mu;
    static const void *keys[64];
    static int vals[64];
    static int n = 0;
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < n; ++i)
        if (keys[i] == kern) return vals[i];
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = std::max(1, num_sms() / 2);
    }
    if (n < 64) {
        keys[n] = kern;
        vals[n] = clusters;
        ++n;
    }
    return clusters;
}

// The CTA-pair kernel needs more than one 128-row tile to pay off.
static bool use_pair(const GemmOperands &g, int variant) {
    if (variant == SF_VARIANT_TCGEN05_SINGLE) return false;
    return g.M > kBM;
}

int encode_tc_dense(const GemmOperands &g, const EpilogueArgs &ep, int variant, cudaStream_t stream) {
    const bool pair = use_pair(g, variant);
    CUtensorMap tmA, tmB;
    int st = build_maps(g, pair, &tmA, &tmB);
    if (st) return st;
    TcParams p{};
    fill_common(p, g, pair, device_error_word());
    // x (A) stays L2-resident when a group of m-tiles fits in kRasterGroupBytes.
    const int es = g.ab_fmt == 2 ? 4 : 2;
    const int64_t a_tile_bytes = (int64_t)p.bm * g.K * es;
    p.group_m = (int)std::max<int64_t>(1, std::min<int64_t>(p.num_m_tiles, kRasterGroupBytes / std::max<int64_t>(1, a_tile_bytes)));
    p.num_units = p.num_m_tiles * p.num_n_tiles;
    p.n_chunks = 1;
    p.tiles_per_chunk = 1;
    p.b_enc = ep.b_enc;
    p.b_enc_dtype = ep.b_enc_dtype;
    p.b_enc_stride = ep.b_enc_stride;
    p.thr = ep.thr;
    p.thr_dtype = ep.thr_dtype;
    p.thr_stride = ep.thr_stride;
    p.activation = ep.activation;
    p.out = ep.out;
    p.out_dtype = ep.out_dtype;
    p.out_sm = ep.out_sm;
    p.out_sn = ep.out_sn;
    p.out_vec = ep.out_vec;
    p.row_nnz = ep.row_nnz;
    p.c_in = ep.c_in;
    p.c_in_pitch = ep.c_in_pitch;
    p.raw = ep.raw;
    if (pair) return dispatch<kDense, 6, true>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, 0, stream);
    return dispatch<kDense, 4, false>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, 0, stream);
}

int encode_tc_csr(const GemmOperands &g, const EpilogueArgs &ep, const CsrArgs &csr, cudaStream_t stream) {
    const bool pair = g.M > kBM;
    CUtensorMap tmA, tmB;
    int st = build_maps(g, pair, &tmA, &tmB);
    if (st) return st;
    TcParams p{};
    fill_common(p, g, pair, device_error_word());
    const int es = g.ab_fmt == 2 ? 4 : 2;
    const int64_t a_tile_bytes = (int64_t)p.bm * g.K * es;
    p.group_m = (int)std::max<int64_t>(1, std::min<int64_t>(p.num_m_tiles, kRasterGroupBytes / std::max<int64_t>(1, a_tile_bytes)));
    p.num_units = p.num_m_tiles * p.num_n_tiles;
    p.n_chunks = 1;
    p.tiles_per_chunk = 1;
    p.b_enc = ep.b_enc;
    p.b_enc_dtype = ep.b_enc_dtype;
    p.b_enc_stride = ep.b_enc_stride;
    p.thr = ep.thr;
    p.thr_dtype = ep.thr_dtype;
    p.thr_stride = ep.thr_stride;
    p.activation = ep.activation;
    p.out_dtype = ep.out_dtype;
    p.row_nnz = ep.row_nnz;
    p.tile_cnt = csr.tile_cnt;
    p.tile_off = csr.tile_off;
    p.stage_idx = csr.stage_idx;
    p.stage_val = csr.stage_val;
    p.csr_state = csr.state;
    p.stage_cap = csr.cap;
    p.c_in = ep.c_in;
    p.c_in_pitch = ep.c_in_pitch;
    if (pair) return dispatch<kCsr, 6, true>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, 0, stream);
    return dispatch<kCsr, 4, false>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, 0, stream);
}

// Column chunks per row for the top-k schedule. Each (m-tile, chunk) unit starts its rows'
// top-k lists empty, and filling them is the epilogue's expensive phase (most columns enter
// while the list is young), so use the FEWEST chunks whose units still fill the available
// CTAs (or CTA pairs) in whole waves to within kTopkWaveEff; failing that, the best-balanced
// count up to 32.
constexpr double kTopkWaveEff = 0.94;
// Smallest per-row candidate buffer (entries) the top-k kernel's operand ring may leave room
// for; a smaller buffer buys operand stages at the price of more frequent merges. 24 gives
// the CTA-pair kernel 5 stages at k=32 (29-entry buffers): at config 4 shapes with 4096
// tokens the tensor pipe went from 60.6% to 68.8% busy (4.16 -> 3.70 ms, ncu); at 32768
// tokens, power-capped, both take the same number of cycles.
#ifndef SF_TOPK_MIN_BUF
#define SF_TOPK_MIN_BUF 24
#endif
#ifndef SF_TOPK_MAX_TPC
#define SF_TOPK_MAX_TPC (1 << 30)
#endif
int topk_chunks(int64_t M, int64_t N) {
    const bool pair = M > kBM;
    const int bm = pair ? 256 : kBM;
    const int m_tiles = (int)((M + bm - 1) / bm);
    const int n_tiles = (int)((N + kBN - 1) / kBN);
    const int slots = pair ? std::max(1, num_sms() / 2) : num_sms();
    const int c_min = std::max(1, (n_tiles + SF_TOPK_MAX_TPC - 1) / SF_TOPK_MAX_TPC);
    int best = c_min;
    double best_eff = -1.0;
    for (int c = c_min; c <= std::min(n_tiles, std::max(32, c_min)); ++c) {
        const int tpc = (n_tiles + c - 1) / c;
        const int chunks = (n_tiles + tpc - 1) / tpc;
        const long units = (long)m_tiles * chunks;
        const long waves = (units + slots - 1) / slots;
        const double eff = (double)units / (double)(waves * slots);
        if (eff >= kTopkWaveEff) return chunks;
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = chunks;
        }
    }
    return best;
}

int encode_tc_topk(const GemmOperands &g, const TopkArgs &tk, cudaStream_t stream) {
    const bool pair = g.M > kBM;  // must match topk_chunks
    CUtensorMap tmA, tmB;
    int st = build_maps(g, pair, &tmA, &tmB);
    if (st) return st;
    TcParams p{};
    fill_common(p, g, pair, device_error_word());
    {
        const int es = g.ab_fmt == 2 ? 4 : 2;
        const int64_t a_tile_bytes = (int64_t)p.bm * g.K * es;
        p.group_m = (int)std::max<int64_t>(
            1, std::min<int64_t>(p.num_m_tiles, kRasterGroupBytes / std::max<int64_t>(1, a_tile_bytes)));
    }
    const int chunks = tk.n_chunks;
    p.tiles_per_chunk = (p.num_n_tiles + chunks - 1) / chunks;
    p.n_chunks = (p.num_n_tiles + p.tiles_per_chunk - 1) / p.tiles_per_chunk;
    if (p.n_chunks != chunks) return set_error(SF_ERR_INVALID, "top-k chunk count %d is not realisable", chunks);
    p.num_units = p.num_m_tiles * p.n_chunks;
    p.b_enc = tk.b_enc;
    p.b_enc_dtype = tk.b_enc_dtype;
    p.b_enc_stride = tk.b_enc_stride;
    p.activation = SF_ACT_RELU;
    p.k = tk.k;
    p.values_dtype = tk.values_dtype;
    p.cand = tk.cand;
    if (tk.k < 1 || tk.k > kTopkMaxK) return set_error(SF_ERR_UNSUPPORTED, "fused top-k supports 1 <= k <= %d", kTopkMaxK);
    // Shared memory per CTA: the operand ring, TcShared, the k-entry lists and a candidate
    // buffer of topk_buf entries per row (1 KB per entry over the 128 rows). The ring keeps
    // the most stages that still leave a buffer of >= 48 entries (up to 64).
    const size_t stage_bytes = pair ? (size_t)(kBM * 128 + (kBN / 2) * 128) : (size_t)kStageBytes;
    const size_t row_entry = 128 * sizeof(unsigned long long);
    auto buffer_for = [&](int stages) -> long {
        const long left = (long)kSmemOptin - 1024 - (long)(stages * stage_bytes) - (long)sizeof(TcShared) -
                          (long)(tk.k * row_entry);
        return std::min<long>(64, left / (long)row_entry);
    };
    int stages = pair ? 6 : 4;
    while (stages > 2 && buffer_for(stages) < SF_TOPK_MIN_BUF) --stages;
    if (buffer_for(stages) < kTopkGroup)
        return set_error(SF_ERR_UNSUPPORTED, "top-k k=%d does not fit in shared memory", tk.k);
    p.topk_buf = (int)buffer_for(stages);
    const size_t extra = (size_t)(tk.k + p.topk_buf) * row_entry;
    if (pair) {
        if (stages == 6) return dispatch<kTopk, 6, true>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
        if (stages == 5) return dispatch<kTopk, 5, true>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
        if (stages == 4) return dispatch<kTopk, 4, true>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
        if (stages == 3) return dispatch<kTopk, 3, true>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
        return dispatch<kTopk, 2, true>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
    }
    if (stages == 4) return dispatch<kTopk, 4, false>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
    if (stages == 3) return dispatch<kTopk, 3, false>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
    return dispatch<kTopk, 2, false>(g.ab_fmt, g.b_mn_major, tmA, tmB, p, extra, stream);
}

}  // namespace sf
