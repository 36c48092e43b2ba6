// Row kernels over the last axis (sm_100a): softmax + top-k, RMSNorm and
// LayerNorm.
//
// The reference computes its row sums left to right in F32
// (src/m3_op_execute_basic.c:150-158, src/m3_op_execute_dense.c:128-140,
// :175-191).  A float sum depends on its order, so these kernels reproduce
// that order exactly: RMSNorm and LayerNorm are then bit-identical to the
// reference and softmax differs only through expf.  An ordered sum is one
// dependent FADD per element, so it must not hold a whole warp per row.
//
// Tile kernels (the main path).  A CTA of 8 warps owns a tile of up to 8
// rows:
//   1. the tile is copied from HBM into shared memory with 16-byte cp.async
//      copies (no registers; several CTAs per SM keep HBM busy while others
//      compute);
//   2. one warp per row does the order-free work (max, NaN, top-k, expf /
//      the residual add);
//   3. lanes of warp 0 run the tile's ordered sums, one row per lane (the
//      padded row pitch keeps those lanes on distinct banks);
//   4. all threads write the outputs with 16-byte stores.
//
// Generic kernels (fallback): one warp per row, any alignment and width.

#include <cuda_runtime.h>

#include <cstdint>

#include "m3c_device.cuh"
#include "m3c_kernels.h"

namespace m3c {
namespace {

constexpr int WARP = 32;

__host__ __device__ __forceinline__ int bytes_of(int dtype)
{
    return (dtype == M3C_F16 || dtype == M3C_BF16) ? 2 : 4;
}

// Element j of a contiguous row of `dtype`, widened to F32.
__device__ __forceinline__ float load_elem(const void *row, int dtype, uint64_t j)
{
    if (bytes_of(dtype) == 2) {
        return widen(dtype, static_cast<const uint16_t *>(row)[j]);
    }
    return as_float(static_cast<const uint32_t *>(row)[j]);
}

__device__ __forceinline__ void store_elem(void *row, int dtype, uint64_t j, float value)
{
    if (bytes_of(dtype) == 2) {
        static_cast<uint16_t *>(row)[j] = static_cast<uint16_t>(narrow(dtype, value));
    } else {
        static_cast<float *>(row)[j] = value;
    }
}

// (value, index) order of the reference's top-k (src/m3_op_execute_sampling.c:7-12).
__device__ __forceinline__ bool precedes(float v, uint32_t i, float w, uint32_t k)
{
    return v > w || (v == w && i < k);
}

__device__ __forceinline__ void warp_best(float &v, uint32_t &i)
{
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, off);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, off);
        if (precedes(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// K passes of warp argmax, each selecting the best element after the previous
// one in the (value desc, index asc) order, reading the row through `at(j)`.
// (best_v, best_i) is this lane's first-pass candidate.
template <typename At>
__device__ void top_k_row(At at, uint64_t width, uint64_t k, float best_v, uint32_t best_i,
                          float *values, int32_t *indices, int lane)
{
    const float neg_inf = -__int_as_float(0x7f800000);
    float last_v = 0.0f;
    uint32_t last_i = 0u;
    for (uint64_t t = 0; t < k; ++t) {
        float v = best_v;
        uint32_t i = best_i;
        if (t > 0) {
            v = neg_inf;
            i = 0xffffffffu;
            for (uint64_t j = lane; j < width; j += WARP) {
                const float x = at(j);
                const uint32_t ji = static_cast<uint32_t>(j);
                if (precedes(last_v, last_i, x, ji) && (i == 0xffffffffu || precedes(x, ji, v, i))) {
                    v = x;
                    i = ji;
                }
            }
        }
        // lanes without a candidate hold index 0xffffffff and lose
        if (i == 0xffffffffu) v = neg_inf;
        warp_best(v, i);
        if (lane == 0) {
            values[t] = v;
            indices[t] = static_cast<int32_t>(i);
        }
        last_v = v;
        last_i = i;
    }
}

// ============================================================ tile kernels

constexpr int TILE_THREADS = 256;
constexpr int TILE_WARPS = TILE_THREADS / WARP;
constexpr int TILE_MAX_ROWS = 8;

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *global_src)
{
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(global_src) : "memory");
}

// Waits for this thread's copies (a hardware wait that always completes).
__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Geometry of one tile: `rows` rows of `width` elements, `nvec` 16-byte
// vectors each.  Raw rows sit `raw_pitch` bytes apart (width * bytes + 16:
// the 16-byte pad puts the rows read by the ordered-sum lanes on different
// banks).  Softmax keeps F32 exponentials `f32_pitch` floats apart, in place
// over the raw rows for F32 input, else in a second area at `f32_offset`.
// The norms keep the scale (and bias) widened to F32 at `param_offset`.  With fewer than 8 rows, `group` warps share a row.
struct Tile {
    int rows;
    int width;
    int nvec;
    int raw_pitch;
    int f32_pitch;
    int f32_offset;
    int param_offset;
    int group;
};

struct RowState {
    float sum[TILE_MAX_ROWS];         // softmax: exponential sum; norms: inverse
    float reciprocal[TILE_MAX_ROWS];  // softmax: RN(1 / sum)
    float mean[TILE_MAX_ROWS];
    int special[TILE_MAX_ROWS];       // softmax: row whose maximum is +-inf
    float part_max[TILE_WARPS];       // per-warp candidates of a row group
    uint32_t part_index[TILE_WARPS];
    int part_nan[TILE_WARPS];
    int skip;
};

// Whether this CTA skips its work because an earlier command of the run
// failed.  Decided once per CTA: another CTA may record a failure at any
// moment, and the barriers need every thread to take the same branch.
__device__ __forceinline__ bool cta_skips(const m3c_status *status, uint32_t skip_before,
                                          int first_of_run, RowState &st)
{
    if (threadIdx.x == 0) {
        st.skip = failed_before(status, skip_before) ? 1 : 0;
        if (!st.skip && first_of_run && blockIdx.x == 0) {
            atomicAdd(const_cast<uint32_t *>(&status->runs_started), 1u);
        }
    }
    __syncthreads();
    return st.skip != 0;
}

// Copy `live` rows of a dense tensor of `nvec` 16-byte vectors per row,
// starting at row `row0`, into shared memory rows `pitch` bytes apart.
__device__ __forceinline__ void tile_copy(unsigned char *dst, const uint4 *src, uint64_t row0,
                                          int live, int nvec, int pitch)
{
    for (int r = 0; r < live; ++r) {
        const uint4 *row = src + (row0 + r) * static_cast<uint64_t>(nvec);
        for (int v = static_cast<int>(threadIdx.x); v < nvec; v += TILE_THREADS) {
            cp_async16(dst + r * pitch + v * 16, row + v);
        }
    }
}

// Widen the 16 / EB elements of 16-byte vector v of a raw row (the
// reference's codecs, NaN payloads included).
template <int EB>
__device__ __forceinline__ void raw_vector(const unsigned char *row, int v, int dtype, float (&x)[16 / EB])
{
    const uint4 q = reinterpret_cast<const uint4 *>(row)[v];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if constexpr (EB == 4) {
#pragma unroll
        for (int t = 0; t < 4; ++t) x[t] = as_float(w[t]);
    } else {
        widen_pairs<4>(dtype, w, x);
    }
}

// Store COUNT (4 or 8) floats converted to `dtype` at element j0 of a 16-byte
// aligned row.
template <int COUNT>
__device__ __forceinline__ void store_vec(void *row, int dtype, uint64_t j0, const float (&v)[COUNT])
{
    if (dtype == M3C_F32) {
        float4 *out = reinterpret_cast<float4 *>(static_cast<float *>(row) + j0);
#pragma unroll
        for (int t = 0; t < COUNT / 4; ++t) {
            __stcs(out + t, make_float4(v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]));
        }
    } else {
        uint32_t h[COUNT / 2];
        narrow_pairs<COUNT / 2>(dtype, v, h);
        uint16_t *base = static_cast<uint16_t *>(row) + j0;
        if constexpr (COUNT == 8) {
            __stcs(reinterpret_cast<uint4 *>(base), make_uint4(h[0], h[1], h[2], h[3]));
        } else {
            __stcs(reinterpret_cast<uint2 *>(base), make_uint2(h[0], h[1]));
        }
    }
}

// Ordered sum of a row of F32 values in shared memory (width % 4 == 0).
__device__ __forceinline__ float ordered_sum_f32(const float *row, int width)
{
    const float4 *v4 = reinterpret_cast<const float4 *>(row);
    float s = 0.0f;
#pragma unroll 8
    for (int j = 0; j < width / 4; ++j) {
        const float4 e = v4[j];
        s = __fadd_rn(s, e.x);
        s = __fadd_rn(s, e.y);
        s = __fadd_rn(s, e.z);
        s = __fadd_rn(s, e.w);
    }
    return s;
}

// Plain widening for the ordered sums: a NaN anywhere makes the sum NaN
// whatever its payload, so the hardware conversion is enough here.
template <int EB>
__device__ __forceinline__ void sum_vector_value(const uint4 &q, int dtype, float (&x)[16 / EB])
{
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if (EB == 4) {
#pragma unroll
        for (int t = 0; t < 4; ++t) x[t] = as_float(w[t]);
    } else if (dtype == M3C_F16) {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            x[t] = __half2float(__ushort_as_half(static_cast<unsigned short>((w[t >> 1] >> ((t & 1) * 16)) & 0xffffu)));
        }
    } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) x[t] = as_float((t & 1) ? (w[t >> 1] & 0xffff0000u) : (w[t >> 1] << 16));
    }
}

template <int EB>
__device__ __forceinline__ void sum_vector(const unsigned char *row, int v, int dtype, float (&x)[16 / EB])
{
    sum_vector_value<EB>(reinterpret_cast<const uint4 *>(row)[v], dtype, x);
}

// Ordered sums over a raw row: KIND 0 sum of x, 1 sum of x*x, 2 sum of
// (x - mean)^2, each product and difference rounded to F32 on its own (the
// statements of src/m3_op_execute_dense.c:128-140 and :175-191).  For F16 the
// square of a value is exact in F32 (11-bit significands, no overflow or
// underflow), so RN(s + RN(x*x)) is one fused multiply-add.
template <int EB, int KIND>
__device__ __forceinline__ float ordered_raw(const unsigned char *row, int nvec, int dtype, float mean)
{
    constexpr int EPV = 16 / EB;
    constexpr int AHEAD = 2;  // vectors loaded while the chain runs over the current ones
    const uint4 *v4 = reinterpret_cast<const uint4 *>(row);
    float s = 0.0f;
    const bool exact_squares = EB == 2 && dtype == M3C_F16;
    uint4 cur[AHEAD];
#pragma unroll
    for (int k = 0; k < AHEAD; ++k) cur[k] = k < nvec ? v4[k] : make_uint4(0u, 0u, 0u, 0u);
    for (int v = 0; v < nvec; v += AHEAD) {
        uint4 next[AHEAD];
#pragma unroll
        for (int k = 0; k < AHEAD; ++k) {
            next[k] = v + AHEAD + k < nvec ? v4[v + AHEAD + k] : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < AHEAD; ++k) {
            if (v + k < nvec) {
                float x[EPV];
                sum_vector_value<EB>(cur[k], dtype, x);
#pragma unroll
                for (int t = 0; t < EPV; ++t) {
                    if (KIND == 0) {
                        s = __fadd_rn(s, x[t]);
                    } else if (KIND == 1) {
                        s = exact_squares ? __fmaf_rn(x[t], x[t], s) : __fadd_rn(s, __fmul_rn(x[t], x[t]));
                    } else {
                        const float c = __fsub_rn(x[t], mean);
                        s = __fadd_rn(s, __fmul_rn(c, c));
                    }
                }
            }
        }
#pragma unroll
        for (int k = 0; k < AHEAD; ++k) cur[k] = next[k];
    }
    return s;
}

// The IEEE quotient out of line, so that the rare operands that need it do
// not put the whole division sequence on every element's path.
__device__ __noinline__ float ieee_div(float a, float b) { return __fdiv_rn(a, b); }

// Softmax and/or TOP_K of up to 8 rows per tile.  Per tile: one cp.async
// copy of the rows; one pass per row (a warp, or a group of warps for wide
// rows) for maximum, first index of the maximum and NaN; the exponentials;
// the reference's left-to-right sums on the lanes of warp 0, one row each;
// then the probabilities, e / sum, with Markstein's refinement of the
// correctly rounded reciprocal.
template <int IN, int OUT, int VPL>
__global__ void __launch_bounds__(TILE_THREADS, 6)
    softmax_tile_kernel(const __grid_constant__ m3c_softmax_params p, Tile g)
{
    constexpr int EB = IN == M3C_F32 ? 4 : 2;
    constexpr int EPV = 16 / EB;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ RowState st;
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (cta_skips(p.status, p.skip_before, p.first_of_run, st)) {
        return;
    }
    const uint4 *in = static_cast<const uint4 *>(p.input);
    float *ebuf = reinterpret_cast<float *>(smem + g.f32_offset);
    const float pos_inf = __int_as_float(0x7f800000);
    const uint32_t first_command = p.softmax_command < p.topk_command ? p.softmax_command : p.topk_command;
    // VPL > 0: the width is a compile-time constant (VPL 16-byte vectors per
    // lane, one warp per row, 8-row tiles), so every loop below has a fixed
    // trip count and every shared-memory address a constant offset
    const int group = VPL > 0 ? 1 : g.group;
    const int nvec = VPL > 0 ? VPL * WARP : g.nvec;
    const int width = nvec * EPV;
    const int raw_pitch = width * EB + 16;
    const int f32_pitch = width + 4;
    const int tile_rows = VPL > 0 ? TILE_WARPS : g.rows;
    const uint64_t tiles = (p.rows + tile_rows - 1) / tile_rows;
    const uint64_t out_pitch = static_cast<uint64_t>(width) * bytes_of(OUT);
    const int r = warp / group;      // this warp's row in the tile
    const int sub = warp % group;    // and its place in the row's group
    const int stride = group * WARP;
    for (uint64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const uint64_t row0 = tile * tile_rows;
        const int live = static_cast<int>(p.rows - row0 < static_cast<uint64_t>(tile_rows) ? p.rows - row0 : tile_rows);
        tile_copy(smem, in, row0, live, nvec, raw_pitch);
        cp_async_wait_all();
        __syncthreads();
        if (p.row_sums != nullptr) {
            // ROW_SUM: the left-to-right F32 sums of the raw rows, one row
            // per lane of warp 0, before the exponentials overwrite them
            if (threadIdx.x < static_cast<unsigned>(live)) {
                p.row_sums[row0 + threadIdx.x] =
                    ordered_raw<EB, 0>(smem + threadIdx.x * raw_pitch, nvec, IN, 0.0f);
            }
            __syncthreads();
        }

        // maximum, its first index and NaN, for the warp's share of its row
        const bool active = r < live;
        const unsigned char *raw = smem + r * raw_pitch;
        float best = -pos_inf;
        uint32_t best_i = 0xffffffffu;
        bool nan = false;
        if (active) {
            for (int v = sub * WARP + lane; v < nvec; v += stride) {
                float x[EPV];
                raw_vector<EB>(raw, v, IN, x);
#pragma unroll
                for (int t = 0; t < EPV; ++t) {
                    const bool greater = x[t] > best;
                    best = greater ? x[t] : best;
                    best_i = greater ? static_cast<uint32_t>(v * EPV + t) : best_i;
                    nan |= x[t] != x[t];
                }
            }
        }
        warp_best(best, best_i);
        nan = __any_sync(0xffffffffu, nan);
        if (group > 1) {
            if (lane == 0) {
                st.part_max[warp] = best;
                st.part_index[warp] = best_i;
                st.part_nan[warp] = nan ? 1 : 0;
            }
            __syncthreads();
            for (int s = 0; s < group; ++s) {
                const int w = r * group + s;
                if (precedes(st.part_max[w], st.part_index[w], best, best_i)) {
                    best = st.part_max[w];
                    best_i = st.part_index[w];
                }
                nan |= st.part_nan[w] != 0;
            }
        }
        // a row of -inf only: the first index (NaN rows fail the command)
        if (best_i == 0xffffffffu) best_i = 0u;
        if (active && nan && sub == 0 && lane == 0 && first_command != 0xffffffffu) {
            record_failure(p.status, first_command);
        }
        if (active && p.top_values != nullptr && sub == 0) {
            const uint64_t row = row0 + r;
            if (p.k == 1) {
                if (lane == 0) {
                    p.top_values[row] = best;
                    p.top_indices[row] = static_cast<int32_t>(best_i);
                }
            } else {
                top_k_row(
                    [&](uint64_t j) {
                        return EB == 4 ? reinterpret_cast<const float *>(raw)[j]
                                       : widen(IN, reinterpret_cast<const uint16_t *>(raw)[j]);
                    },
                    static_cast<uint64_t>(width), p.k, best, best_i, p.top_values + row * p.k,
                    p.top_indices + row * p.k, lane);
            }
        }
        if (p.probs != nullptr) {
            if (p.k > 1 && p.top_values != nullptr) {
                __syncthreads();  // the top-k passes read rows the exponentials overwrite
            }
            float *erow = ebuf + r * f32_pitch;
            if (active && (best == -pos_inf || best == pos_inf)) {
                // src/m3_op_execute_basic.c:165-170: final probabilities now,
                // by the first warp of the row's group
                if (sub == 0) {
                    uint32_t infinities = 0u;
                    for (int v = lane; v < nvec; v += WARP) {
                        float x[EPV];
                        raw_vector<EB>(raw, v, IN, x);
#pragma unroll
                        for (int t = 0; t < EPV; ++t) infinities += x[t] == pos_inf ? 1u : 0u;
                    }
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) {
                        infinities += __shfl_xor_sync(0xffffffffu, infinities, off);
                    }
                    const float share = __fdiv_rn(1.0f, __uint2float_rn(infinities));
                    __syncwarp();
                    for (int v = lane; v < nvec; v += WARP) {
                        float x[EPV];
                        raw_vector<EB>(raw, v, IN, x);
#pragma unroll
                        for (int t = 0; t < EPV; ++t) {
                            erow[v * EPV + t] = (best == pos_inf && x[t] == pos_inf) ? share : 0.0f;
                        }
                    }
                    if (lane == 0) st.special[r] = 1;
                }
            } else if (active) {
                // each lane overwrites only the vector it has just read
                for (int v = sub * WARP + lane; v < nvec; v += stride) {
                    float x[EPV];
                    raw_vector<EB>(raw, v, IN, x);
#pragma unroll
                    for (int t = 0; t < EPV; ++t) erow[v * EPV + t] = expf(__fsub_rn(x[t], best));
                }
                if (sub == 0 && lane == 0) st.special[r] = 0;
            }
            __syncthreads();
            // the reference's left-to-right sums, one row per lane of warp 0
            if (threadIdx.x < static_cast<unsigned>(live) && !st.special[threadIdx.x]) {
                const float sum = ordered_sum_f32(ebuf + threadIdx.x * f32_pitch, width);
                st.sum[threadIdx.x] = sum;
                st.reciprocal[threadIdx.x] = __frcp_rn(sum);
            }
            __syncthreads();
            // probabilities expf(x - max) / sum (src/m3_op_execute_basic.c:171-178)
            unsigned char *out = static_cast<unsigned char *>(p.probs) + row0 * out_pitch;
            const int per_row = width / 4;
            for (int rr = 0; rr < live; ++rr) {
                const float4 *e4 = reinterpret_cast<const float4 *>(ebuf + rr * f32_pitch);
                const bool special = st.special[rr] != 0;
                const float sum = st.sum[rr];
                const float y = st.reciprocal[rr];
                for (int j4 = static_cast<int>(threadIdx.x); j4 < per_row; j4 += TILE_THREADS) {
                    const float4 e = e4[j4];
                    float pr[4] = {e.x, e.y, e.z, e.w};
                    if (!special) {
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            // e in [2^-100, 1] and sum >= 1: Markstein's quotient
                            // is the IEEE one; smaller e stays on the IEEE division
                            pr[t] = pr[t] >= 0x1p-100f ? div_markstein(pr[t], sum, y) : ieee_div(pr[t], sum);
                        }
                    }
                    store_vec<4>(out + rr * out_pitch, OUT, static_cast<uint64_t>(j4) * 4u, pr);
                }
            }
        }
        __syncthreads();
    }
}

// Softmax/TOP_K for the compiled F32 widths, pipelined across tiles.  Two
// shared-memory stages of 8 rows; while warp 0 runs the ordered sums of tile
// i, warps 1-7 write the probabilities of tile i-1 and then prefetch tile
// i+1 into the stage tile i-1 has released, so the sequential sums, the
// stores and the next loads overlap.  Then all warps find max/argmax/NaN and
// the exponentials of tile i+1.
struct PipeState {
    float sum[2][TILE_WARPS];
    float reciprocal[2][TILE_WARPS];
    int special[2][TILE_WARPS];
    int tiny[2][TILE_WARPS];
    int skip;
};

// Copy `live` rows starting at row0 into a stage with threads [first, first + count).
template <int NVEC>
__device__ __forceinline__ void stage_copy(unsigned char *dst, const uint4 *src, uint64_t row0, int live,
                                           int pitch, int thread, int count)
{
    for (int r = 0; r < live; ++r) {
        const uint4 *row = src + (row0 + r) * static_cast<uint64_t>(NVEC);
        for (int v = thread; v < NVEC; v += count) {
            cp_async16(dst + r * pitch + v * 16, row + v);
        }
    }
}

template <int OUT, int VPL>
__global__ void __launch_bounds__(TILE_THREADS, 3)
    softmax_pipe_kernel(const __grid_constant__ m3c_softmax_params p)
{
    constexpr int NVEC = VPL * WARP;          // F32: 4 elements per vector
    constexpr int WIDTH = NVEC * 4;
    constexpr int PITCH = WIDTH * 4 + 16;     // bytes (and 4 * the F32 pitch)
    constexpr int STAGE = TILE_WARPS * PITCH;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ PipeState st;
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (threadIdx.x == 0) {
        st.skip = failed_before(p.status, p.skip_before) ? 1 : 0;
        if (!st.skip && p.first_of_run && blockIdx.x == 0) {
            atomicAdd(const_cast<uint32_t *>(&p.status->runs_started), 1u);
        }
    }
    __syncthreads();
    const uint64_t tiles = (p.rows + TILE_WARPS - 1) / TILE_WARPS;
    if (st.skip || blockIdx.x >= tiles) {
        return;
    }
    const uint4 *in = static_cast<const uint4 *>(p.input);
    const float pos_inf = __int_as_float(0x7f800000);
    const uint32_t first_command = p.softmax_command < p.topk_command ? p.softmax_command : p.topk_command;
    const uint64_t out_pitch = static_cast<uint64_t>(WIDTH) * bytes_of(OUT);
    auto live_rows = [&](uint64_t tile) {
        const uint64_t row0 = tile * TILE_WARPS;
        return static_cast<int>(p.rows - row0 < static_cast<uint64_t>(TILE_WARPS) ? p.rows - row0 : TILE_WARPS);
    };

    // max, first argmax and NaN of row `warp`, then its exponentials in place
    auto row_pass = [&](int stage, uint64_t tile) {
        const int live = live_rows(tile);
        const int r = warp;
        if (r >= live) return;
        float *erow = reinterpret_cast<float *>(smem + stage * STAGE + r * PITCH);
        const float4 *x4 = reinterpret_cast<const float4 *>(erow);
        float best = -pos_inf;
        uint32_t best_i = 0xffffffffu;
        bool nan = false;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int v = lane + j * WARP;
            const float4 q = x4[v];
            const float x[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const bool greater = x[t] > best;
                best = greater ? x[t] : best;
                best_i = greater ? static_cast<uint32_t>(v * 4 + t) : best_i;
                nan |= x[t] != x[t];
            }
        }
        warp_best(best, best_i);
        nan = __any_sync(0xffffffffu, nan);
        if (best_i == 0xffffffffu) best_i = 0u;  // a row of -inf only
        if (nan && lane == 0 && first_command != 0xffffffffu) record_failure(p.status, first_command);
        const uint64_t row = tile * TILE_WARPS + r;
        if (p.top_values != nullptr && lane == 0) {
            p.top_values[row] = best;
            p.top_indices[row] = static_cast<int32_t>(best_i);
        }
        if (p.probs == nullptr) return;
        if (best == -pos_inf || best == pos_inf) {
            // src/m3_op_execute_basic.c:165-170: final probabilities now
            uint32_t infinities = 0u;
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const float4 q = x4[lane + j * WARP];
                infinities += (q.x == pos_inf) + (q.y == pos_inf) + (q.z == pos_inf) + (q.w == pos_inf);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) infinities += __shfl_xor_sync(0xffffffffu, infinities, off);
            const float share = __fdiv_rn(1.0f, __uint2float_rn(infinities));
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const int v = lane + j * WARP;
                const float4 q = x4[v];
                const bool plus = best == pos_inf;
                reinterpret_cast<float4 *>(erow)[v] =
                    make_float4(plus && q.x == pos_inf ? share : 0.0f, plus && q.y == pos_inf ? share : 0.0f,
                                plus && q.z == pos_inf ? share : 0.0f, plus && q.w == pos_inf ? share : 0.0f);
            }
            if (lane == 0) {
                st.special[stage][r] = 1;
                st.tiny[stage][r] = 0;
            }
            return;
        }
        bool tiny = false;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int v = lane + j * WARP;
            const float4 q = x4[v];
            const float4 e = make_float4(expf(__fsub_rn(q.x, best)), expf(__fsub_rn(q.y, best)),
                                         expf(__fsub_rn(q.z, best)), expf(__fsub_rn(q.w, best)));
            tiny |= (e.x < 0x1p-100f) | (e.y < 0x1p-100f) | (e.z < 0x1p-100f) | (e.w < 0x1p-100f);
            reinterpret_cast<float4 *>(erow)[v] = e;
        }
        tiny = __any_sync(0xffffffffu, tiny);
        if (lane == 0) {
            st.special[stage][r] = 0;
            st.tiny[stage][r] = tiny ? 1 : 0;
        }
    };

    // probabilities e / sum (src/m3_op_execute_basic.c:171-178) of a tile,
    // by threads [first, first + count)
    auto store_tile = [&](int stage, uint64_t tile, int thread, int count) {
        const int live = live_rows(tile);
        unsigned char *out = static_cast<unsigned char *>(p.probs) + tile * TILE_WARPS * out_pitch;
        for (int rr = 0; rr < live; ++rr) {
            const float4 *e4 = reinterpret_cast<const float4 *>(smem + stage * STAGE + rr * PITCH);
            unsigned char *orow = out + rr * out_pitch;
            const float sum = st.sum[stage][rr];
            const float y = st.reciprocal[stage][rr];
            const bool special = st.special[stage][rr] != 0;
            const bool tiny = st.tiny[stage][rr] != 0;
            for (int j4 = thread; j4 < NVEC; j4 += count) {
                const float4 e = e4[j4];
                float pr[4] = {e.x, e.y, e.z, e.w};
                if (!special) {
                    if (!tiny) {
                        // e in [2^-100, 1] and sum >= 1: Markstein's quotient
                        // is the IEEE one
#pragma unroll
                        for (int t = 0; t < 4; ++t) pr[t] = div_markstein(pr[t], sum, y);
                    } else {
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            pr[t] = pr[t] >= 0x1p-100f ? div_markstein(pr[t], sum, y) : ieee_div(pr[t], sum);
                        }
                    }
                }
                store_vec<4>(orow, OUT, static_cast<uint64_t>(j4) * 4u, pr);
            }
        }
    };

    uint64_t tile = blockIdx.x;
    int stage = 0;
    stage_copy<NVEC>(smem, in, tile * TILE_WARPS, live_rows(tile), PITCH, threadIdx.x, TILE_THREADS);
    cp_async_wait_all();
    __syncthreads();
    row_pass(stage, tile);
    __syncthreads();
    bool have_previous = false;
    uint64_t previous = 0;
    for (;;) {
        const uint64_t next = tile + gridDim.x;
        const bool has_next = next < tiles;
        if (warp == 0) {
            // the reference's left-to-right sums, one row per lane
            if (p.probs != nullptr && lane < live_rows(tile) && !st.special[stage][lane]) {
                const float sum =
                    ordered_sum_f32(reinterpret_cast<const float *>(smem + stage * STAGE + lane * PITCH), WIDTH);
                st.sum[stage][lane] = sum;
                st.reciprocal[stage][lane] = __frcp_rn(sum);
            }
        } else {
            if (have_previous && p.probs != nullptr) {
                store_tile(stage ^ 1, previous, static_cast<int>(threadIdx.x) - WARP, TILE_THREADS - WARP);
            }
            // every read of the other stage is done before it is refilled
            asm volatile("bar.sync 1, %0;" ::"r"(TILE_THREADS - WARP) : "memory");
            if (has_next) {
                stage_copy<NVEC>(smem + (stage ^ 1) * STAGE, in, next * TILE_WARPS, live_rows(next), PITCH,
                                 static_cast<int>(threadIdx.x) - WARP, TILE_THREADS - WARP);
            }
        }
        cp_async_wait_all();
        __syncthreads();
        have_previous = true;
        previous = tile;
        if (!has_next) break;
        tile = next;
        stage ^= 1;
        row_pass(stage, tile);
        __syncthreads();
    }
    if (p.probs != nullptr) {
        store_tile(stage, previous, static_cast<int>(threadIdx.x), TILE_THREADS);
    }
}

// RMSNorm / LayerNorm with an optional residual-add prologue (RESID: the
// input is round_in(x + b), optionally stored to sum_out).
template <int IN, int OUT, bool RESID, int NVEC>
__global__ void __launch_bounds__(TILE_THREADS)
    norm_tile_kernel(const __grid_constant__ m3c_norm_params p, Tile g)
{
    constexpr int EB = IN == M3C_F32 ? 4 : 2;
    constexpr int EPV = 16 / EB;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ RowState st;
    if (cta_skips(p.status, p.skip_before, p.first_of_run, st)) {
        return;
    }
    const uint4 *xa = static_cast<const uint4 *>(p.x);
    const uint4 *xb = static_cast<const uint4 *>(p.resid_b);
    uint4 *sum_out = static_cast<uint4 *>(p.sum_out);
    float *scale = reinterpret_cast<float *>(smem + g.param_offset);
    float *bias = scale + g.width;
    for (int j = static_cast<int>(threadIdx.x); j < g.width; j += TILE_THREADS) {
        scale[j] = load_elem(p.scale, p.scale_dtype, j);
        if (p.bias != nullptr) bias[j] = load_elem(p.bias, p.bias_dtype, j);
    }
    // NVEC > 0: the row length in 16-byte vectors is a compile-time constant
    // (fixed trip counts, constant shared-memory offsets)
    const int nvec = NVEC > 0 ? NVEC : g.nvec;
    const int width = nvec * EPV;
    const int raw_pitch = width * EB + 16;
    const uint64_t tiles = (p.rows + g.rows - 1) / g.rows;
    const float channels = __int2float_rn(width);
    const uint64_t out_pitch = static_cast<uint64_t>(width) * bytes_of(OUT);
    for (uint64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const uint64_t row0 = tile * g.rows;
        const int live = static_cast<int>(p.rows - row0 < static_cast<uint64_t>(g.rows) ? p.rows - row0 : g.rows);
        tile_copy(smem, xa, row0, live, nvec, raw_pitch);
        cp_async_wait_all();
        __syncthreads();
        if constexpr (RESID) {
            // src/m3_op_execute_basic.c:61-77: one F32 add, stored in the
            // sum's dtype; the stored bits replace x in shared memory
            for (int r = 0; r < live; ++r) {
                uint4 *arow = reinterpret_cast<uint4 *>(smem + r * raw_pitch);
                const uint4 *brow = xb + (row0 + r) * static_cast<uint64_t>(nvec);
                for (int v = static_cast<int>(threadIdx.x); v < nvec; v += TILE_THREADS) {
                    float a[EPV];
                    float b[EPV];
                    // b is read once, straight from HBM (no staging)
                    const uint4 bq = __ldcs(brow + v);
                    raw_vector<EB>(reinterpret_cast<const unsigned char *>(arow), v, IN, a);
                    raw_vector<EB>(reinterpret_cast<const unsigned char *>(&bq), 0, IN, b);
#pragma unroll
                    for (int t = 0; t < EPV; ++t) a[t] = __fadd_rn(a[t], b[t]);
                    uint4 packed;
                    if constexpr (EB == 4) {
                        packed = make_uint4(as_bits(a[0]), as_bits(a[1]), as_bits(a[2]), as_bits(a[3]));
                    } else {
                        uint32_t h[4];
                        narrow_pairs<4>(IN, a, h);
                        packed = make_uint4(h[0], h[1], h[2], h[3]);
                    }
                    arow[v] = packed;
                    if (sum_out != nullptr) {
                        __stcs(sum_out + (row0 + r) * static_cast<uint64_t>(nvec) + v, packed);
                    }
                }
            }
            __syncthreads();
        }
        // ordered sums, one row per lane of warp 0
        if (threadIdx.x < static_cast<unsigned>(live)) {
            const int r = static_cast<int>(threadIdx.x);
            const unsigned char *row = smem + r * raw_pitch;
            if (p.layer_norm) {
                // src/m3_op_execute_dense.c:175-194
                const float mean = __fdiv_rn(ordered_raw<EB, 0>(row, nvec, IN, 0.0f), channels);
                const float centred = ordered_raw<EB, 2>(row, nvec, IN, mean);
                st.mean[r] = mean;
                st.sum[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(centred, channels), p.epsilon)));
            } else {
                // src/m3_op_execute_dense.c:128-141
                const float squares = ordered_raw<EB, 1>(row, nvec, IN, 0.0f);
                st.mean[r] = 0.0f;
                st.sum[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(squares, channels), p.epsilon)));
            }
        }
        __syncthreads();
        // normalised outputs
        unsigned char *out = static_cast<unsigned char *>(p.out) + row0 * out_pitch;
        for (int r = 0; r < live; ++r) {
            const float inverse = st.sum[r];
            const float mean = st.mean[r];
            const unsigned char *row = smem + r * raw_pitch;
            for (int v = static_cast<int>(threadIdx.x); v < nvec; v += TILE_THREADS) {
                float x[EPV];
                float y[EPV];
                raw_vector<EB>(row, v, IN, x);
                if (!p.layer_norm) {
                    // x * inv rounded to the input dtype before scaling,
                    // src/m3_op_execute_dense.c:149-151
#pragma unroll
                    for (int k = 0; k < EPV; ++k) x[k] = __fmul_rn(x[k], inverse);
                    round_values<EPV>(IN, x);
                }
                const float4 *w4 = reinterpret_cast<const float4 *>(scale + v * EPV);
                const float4 *b4 = reinterpret_cast<const float4 *>(bias + v * EPV);
#pragma unroll
                for (int q = 0; q < EPV / 4; ++q) {
                    const float4 w = w4[q];
                    const float ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const int k = 4 * q + t;
                        if (p.layer_norm) {
                            // ((x - mean) * inv) * scale (+ bias), src/m3_op_execute_dense.c:195-213
                            float o = __fmul_rn(__fmul_rn(__fsub_rn(x[k], mean), inverse), ws[t]);
                            if (p.bias != nullptr) {
                                const float4 bb = b4[q];
                                const float bs[4] = {bb.x, bb.y, bb.z, bb.w};
                                o = __fadd_rn(o, bs[t]);
                            }
                            y[k] = o;
                        } else {
                            y[k] = __fmul_rn(x[k], ws[t]);
                        }
                    }
                }
                store_vec<EPV>(out + r * out_pitch, OUT, static_cast<uint64_t>(v) * EPV, y);
            }
        }
        __syncthreads();
    }
}

// ========================================================= generic kernels

// Stage a row into shared memory as F32 (16-byte loads when aligned).
template <typename Visit>
__device__ __forceinline__ void stage_row(const void *row, int dtype, uint64_t width, float *smem,
                                          int lane, Visit visit)
{
    const uintptr_t address = reinterpret_cast<uintptr_t>(row);
    const int eb = bytes_of(dtype);
    const uint64_t per_vec = 16u / static_cast<uint64_t>(eb);
    if ((address & 15u) == 0u && (width % per_vec) == 0u) {
        const uint4 *vec = static_cast<const uint4 *>(row);
        const uint64_t nvec = width / per_vec;
        for (uint64_t v = lane; v < nvec; v += WARP) {
            const uint4 q = vec[v];
            const uint32_t words[4] = {q.x, q.y, q.z, q.w};
            const uint64_t j0 = v * per_vec;
            for (uint64_t t = 0; t < per_vec; ++t) {
                const float x = eb == 4 ? as_float(words[t])
                                        : widen(dtype, (words[t >> 1] >> ((t & 1) * 16)) & 0xffffu);
                if (smem) smem[j0 + t] = x;
                visit(j0 + t, x);
            }
        }
    } else {
        for (uint64_t j = lane; j < width; j += WARP) {
            const float x = load_elem(row, dtype, j);
            if (smem) smem[j] = x;
            visit(j, x);
        }
    }
}

// `smem_row` holds the row as F32 (nullptr: re-read the row from global).
__device__ void softmax_row(const m3c_softmax_params &p, uint64_t row, float *smem_row, int lane)
{
    const uint64_t width = p.width;
    const unsigned char *in_base = static_cast<const unsigned char *>(p.input);
    const void *in_row = in_base + row * width * static_cast<uint64_t>(bytes_of(p.in_dtype));
    const float pos_inf = __int_as_float(0x7f800000);
    float maximum = -pos_inf;
    uint32_t infinities = 0u;
    bool nan = false;
    float best_v = -pos_inf;
    uint32_t best_i = 0xffffffffu;

    stage_row(in_row, p.in_dtype, width, smem_row, lane, [&](uint64_t j, float x) {
        maximum = x > maximum ? x : maximum;
        infinities += x == pos_inf ? 1u : 0u;
        nan |= x != x;
        if (precedes(x, static_cast<uint32_t>(j), best_v, best_i)) {
            best_v = x;
            best_i = static_cast<uint32_t>(j);
        }
    });
    if (p.row_sums != nullptr) {
        // ROW_SUM: the left-to-right F32 sum of the row, on one lane
        __syncwarp();
        if (lane == 0) {
            float s = 0.0f;
            for (uint64_t j = 0; j < width; ++j) {
                s = __fadd_rn(s, smem_row ? smem_row[j] : load_elem(in_row, p.in_dtype, j));
            }
            p.row_sums[row] = s;
        }
        __syncwarp();
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float other = __shfl_xor_sync(0xffffffffu, maximum, off);
        maximum = other > maximum ? other : maximum;
        infinities += __shfl_xor_sync(0xffffffffu, infinities, off);
    }
    if (__any_sync(0xffffffffu, nan) && lane == 0) {
        const uint32_t first = p.softmax_command < p.topk_command ? p.softmax_command : p.topk_command;
        if (first != 0xffffffffu) record_failure(p.status, first);
    }
    __syncwarp();
    if (p.top_values != nullptr) {
        top_k_row(
            [&](uint64_t j) { return smem_row ? smem_row[j] : load_elem(in_row, p.in_dtype, j); },
            width, p.k, best_v, best_i, p.top_values + row * p.k, p.top_indices + row * p.k, lane);
    }
    if (p.probs == nullptr) {
        return;
    }
    unsigned char *out_row = static_cast<unsigned char *>(p.probs) +
                             row * width * static_cast<uint64_t>(bytes_of(p.probs_dtype));
    if (maximum == -pos_inf || maximum == pos_inf) {
        const float share = __fdiv_rn(1.0f, __uint2float_rn(infinities));
        for (uint64_t j = lane; j < width; j += WARP) {
            const float x = smem_row ? smem_row[j] : load_elem(in_row, p.in_dtype, j);
            store_elem(out_row, p.probs_dtype, j, (maximum == pos_inf && x == pos_inf) ? share : 0.0f);
        }
        return;
    }
    float sum = 0.0f;
    if (smem_row != nullptr) {
        for (uint64_t j = lane; j < width; j += WARP) {
            smem_row[j] = expf(__fsub_rn(smem_row[j], maximum));
        }
        __syncwarp();
        if (lane == 0) {
            float s = 0.0f;
            for (uint64_t j = 0; j < width; ++j) s = __fadd_rn(s, smem_row[j]);
            sum = s;
        }
    } else if (lane == 0) {
        float s = 0.0f;
        for (uint64_t j = 0; j < width; ++j) {
            s = __fadd_rn(s, expf(__fsub_rn(load_elem(in_row, p.in_dtype, j), maximum)));
        }
        sum = s;
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (uint64_t j = lane; j < width; j += WARP) {
        const float e = smem_row ? smem_row[j] : expf(__fsub_rn(load_elem(in_row, p.in_dtype, j), maximum));
        store_elem(out_row, p.probs_dtype, j, __fdiv_rn(e, sum));
    }
}

__global__ void softmax_kernel(const __grid_constant__ m3c_softmax_params p, int rows_per_cta,
                               int use_smem)
{
    extern __shared__ float fsmem[];
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (failed_before(p.status, p.skip_before)) {
        return;
    }
    if (p.first_of_run && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    float *row_smem = use_smem ? fsmem + static_cast<uint64_t>(warp) * p.width : nullptr;
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * rows_per_cta + warp; row < p.rows;
         row += static_cast<uint64_t>(gridDim.x) * rows_per_cta) {
        softmax_row(p, row, row_smem, lane);
        __syncwarp();
    }
}

__device__ void norm_row(const m3c_norm_params &p, uint64_t row, float *smem_row, int lane)
{
    const uint64_t width = p.width;
    const uint64_t eb = static_cast<uint64_t>(bytes_of(p.in_dtype));
    const unsigned char *x_row = static_cast<const unsigned char *>(p.x) + row * width * eb;
    unsigned char *out_row = static_cast<unsigned char *>(p.out) +
                             row * width * static_cast<uint64_t>(bytes_of(p.out_dtype));

    if (p.resid_b != nullptr) {
        const unsigned char *b_row = static_cast<const unsigned char *>(p.resid_b) + row * width * eb;
        unsigned char *s_row = p.sum_out ? static_cast<unsigned char *>(p.sum_out) + row * width * eb
                                         : nullptr;
        for (uint64_t j = lane; j < width; j += WARP) {
            const float s = __fadd_rn(load_elem(x_row, p.in_dtype, j), load_elem(b_row, p.in_dtype, j));
            const uint32_t stored = narrow(p.in_dtype, s);
            if (s_row) {
                if (eb == 2) {
                    reinterpret_cast<uint16_t *>(s_row)[j] = static_cast<uint16_t>(stored);
                } else {
                    reinterpret_cast<uint32_t *>(s_row)[j] = stored;
                }
            }
            smem_row[j] = widen(p.in_dtype, stored);
        }
    } else {
        stage_row(x_row, p.in_dtype, width, smem_row, lane, [](uint64_t, float) {});
    }
    __syncwarp();
    float mean = 0.0f;
    float inverse = 0.0f;
    if (lane == 0) {
        const float channels = __ull2float_rn(width);
        if (p.layer_norm) {
            float sum = 0.0f;
            for (uint64_t j = 0; j < width; ++j) sum = __fadd_rn(sum, smem_row[j]);
            mean = __fdiv_rn(sum, channels);
            float centred = 0.0f;
            for (uint64_t j = 0; j < width; ++j) {
                const float c = __fsub_rn(smem_row[j], mean);
                centred = __fadd_rn(centred, __fmul_rn(c, c));
            }
            inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(centred, channels), p.epsilon)));
        } else {
            float squares = 0.0f;
            for (uint64_t j = 0; j < width; ++j) squares = __fadd_rn(squares, __fmul_rn(smem_row[j], smem_row[j]));
            inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(squares, channels), p.epsilon)));
        }
    }
    mean = __shfl_sync(0xffffffffu, mean, 0);
    inverse = __shfl_sync(0xffffffffu, inverse, 0);
    for (uint64_t j = lane; j < width; j += WARP) {
        const float x = smem_row[j];
        const float w = load_elem(p.scale, p.scale_dtype, j);
        float result;
        if (p.layer_norm) {
            result = __fmul_rn(__fmul_rn(__fsub_rn(x, mean), inverse), w);
            if (p.bias != nullptr) result = __fadd_rn(result, load_elem(p.bias, p.bias_dtype, j));
        } else {
            result = __fmul_rn(round_to(p.in_dtype, __fmul_rn(x, inverse)), w);
        }
        store_elem(out_row, p.out_dtype, j, result);
    }
}

__global__ void norm_kernel(const __grid_constant__ m3c_norm_params p, int rows_per_cta)
{
    extern __shared__ float fsmem[];
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (failed_before(p.status, p.skip_before)) {
        return;
    }
    if (p.first_of_run && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    float *row_smem = fsmem + static_cast<uint64_t>(warp) * p.width;
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * rows_per_cta + warp; row < p.rows;
         row += static_cast<uint64_t>(gridDim.x) * rows_per_cta) {
        norm_row(p, row, row_smem, lane);
        __syncwarp();
    }
}

// ================================================================ launchers

int sm_count_current()
{
    static int count = 0;
    if (count == 0) {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        if (count <= 0) count = 148;
    }
    return count;
}

bool aligned16(const void *p)
{
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u;
}

// Tile geometry, or rows = 0 when the tile path does not apply: rows must be
// whole 16-byte vectors, and one tile must fit a 48 KiB shared-memory budget
// (so several CTAs share an SM) or, for very wide rows, one row must fit in
// 200 KiB.  Softmax tiles hold 8, 4, 2 or 1 rows so that the 8 warps split
// evenly over them.
Tile tile_geometry(uint64_t width, int eb, bool softmax, bool residual, bool bias)
{
    Tile g{0, 0, 0, 0, 0, 0, 0, 1};
    const uint64_t per_vec = 16u / static_cast<uint64_t>(eb);
    if (width == 0 || width % per_vec != 0 || width % 4 != 0 || width > 32768) {
        return g;
    }
    g.width = static_cast<int>(width);
    g.nvec = static_cast<int>(width / per_vec);
    g.raw_pitch = static_cast<int>(width) * eb + 16;
    g.f32_pitch = static_cast<int>(width) + 4;
    const size_t budget = 48u * 1024u;
    if (softmax) {
        const size_t row_bytes = static_cast<size_t>(g.raw_pitch) + (eb != 4 ? static_cast<size_t>(g.f32_pitch) * 4u : 0u);
        int rows = TILE_MAX_ROWS;
        while (rows > 1 && static_cast<size_t>(rows) * row_bytes > budget) rows >>= 1;
        if (row_bytes > 200u * 1024u) return g;
        g.rows = rows;
        g.group = TILE_WARPS / rows;
        g.f32_offset = eb != 4 ? rows * g.raw_pitch : 0;
        return g;
    }
    // the residual's second operand is read from HBM in the add pass, not staged
    (void)residual;
    const size_t areas = 1u;
    const size_t row_bytes = static_cast<size_t>(g.raw_pitch) * areas;
    const size_t params = static_cast<size_t>(width) * 4u * (bias ? 2u : 1u);
    int rows = 0;
    if (params + row_bytes <= budget) {
        rows = static_cast<int>((budget - params) / row_bytes);
        if (rows > TILE_MAX_ROWS) rows = TILE_MAX_ROWS;
    } else if (params + row_bytes <= 200u * 1024u) {
        rows = 1;
    }
    g.rows = rows;
    g.param_offset = rows * g.raw_pitch * static_cast<int>(areas);
    return g;
}

size_t tile_smem(const Tile &g, bool softmax, int eb, bool bias)
{
    if (softmax) {
        return static_cast<size_t>(g.rows) *
               (static_cast<size_t>(g.raw_pitch) + (eb != 4 ? static_cast<size_t>(g.f32_pitch) * 4u : 0u));
    }
    return static_cast<size_t>(g.param_offset) + static_cast<size_t>(g.width) * 4u * (bias ? 2u : 1u);
}

template <typename Kernel, typename Params>
int launch_tile(Kernel kernel, const Params &params, const Tile &g, size_t smem, uint64_t rows, void *stream)
{
    if (smem > 48u * 1024u) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, TILE_THREADS, smem) !=
            cudaSuccess ||
        per_sm < 1) {
        per_sm = 1;
    }
    // a persistent grid: every resident CTA strides over the tiles
    const uint64_t tiles = (rows + static_cast<uint64_t>(g.rows) - 1) / static_cast<uint64_t>(g.rows);
    const uint64_t cap = static_cast<uint64_t>(sm_count_current()) * static_cast<uint64_t>(per_sm);
    const unsigned grid = static_cast<unsigned>(tiles == 0 ? 1 : (tiles < cap ? tiles : cap));
    kernel<<<grid, TILE_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(params, g);
    return static_cast<int>(cudaGetLastError());
}

template <typename Kernel>
int launch_pipe(Kernel kernel, const m3c_softmax_params &params, size_t smem, void *stream)
{
    if (smem > 48u * 1024u) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, TILE_THREADS, smem) != cudaSuccess ||
        per_sm < 1) {
        per_sm = 1;
    }
    const uint64_t tiles = (params.rows + TILE_WARPS - 1) / TILE_WARPS;
    const uint64_t cap = static_cast<uint64_t>(sm_count_current()) * static_cast<uint64_t>(per_sm);
    const unsigned grid = static_cast<unsigned>(tiles == 0 ? 1 : (tiles < cap ? tiles : cap));
    kernel<<<grid, TILE_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(params);
    return static_cast<int>(cudaGetLastError());
}

// Tile kernels are compiled per (input, output) dtype pair so that every
// codec folds to straight-line code.
template <int IN, int OUT>
int softmax_tile(const m3c_softmax_params &p, const Tile &g, size_t smem, void *stream)
{
    // widths with a compiled geometry: 8-row tiles in two stages
    if (IN == M3C_F32 && g.rows == TILE_WARPS && g.group == 1 && p.k <= 1 && p.row_sums == nullptr &&
        (g.width == 1024 || g.width == 512)) {
        const size_t stages = 2u * static_cast<size_t>(TILE_WARPS) * static_cast<size_t>(g.raw_pitch);
        if (g.width == 1024) {
            return launch_pipe(softmax_pipe_kernel<OUT, 8>, p, stages, stream);
        }
        return launch_pipe(softmax_pipe_kernel<OUT, 4>, p, stages, stream);
    }
    return launch_tile(softmax_tile_kernel<IN, OUT, 0>, p, g, smem, p.rows, stream);
}

template <int IN>
int softmax_tile_out(const m3c_softmax_params &p, const Tile &g, size_t smem, void *stream)
{
    switch (p.probs == nullptr ? IN : p.probs_dtype) {
    case M3C_F16: return softmax_tile<IN, M3C_F16>(p, g, smem, stream);
    case M3C_BF16: return softmax_tile<IN, M3C_BF16>(p, g, smem, stream);
    default: return softmax_tile<IN, M3C_F32>(p, g, smem, stream);
    }
}

int softmax_tile_dispatch(const m3c_softmax_params &p, const Tile &g, size_t smem, void *stream)
{
    switch (p.in_dtype) {
    case M3C_F16: return softmax_tile_out<M3C_F16>(p, g, smem, stream);
    case M3C_BF16: return softmax_tile_out<M3C_BF16>(p, g, smem, stream);
    default: return softmax_tile_out<M3C_F32>(p, g, smem, stream);
    }
}

template <int IN, int OUT>
int norm_tile(const m3c_norm_params &p, const Tile &g, size_t smem, void *stream)
{
    // 256 vectors per row (F16/BF16 width 2048, F32 width 1024): one vector
    // per thread and row, with a compiled geometry
    if (g.nvec == 256) {
        return p.resid_b != nullptr
                   ? launch_tile(norm_tile_kernel<IN, OUT, true, 256>, p, g, smem, p.rows, stream)
                   : launch_tile(norm_tile_kernel<IN, OUT, false, 256>, p, g, smem, p.rows, stream);
    }
    return p.resid_b != nullptr ? launch_tile(norm_tile_kernel<IN, OUT, true, 0>, p, g, smem, p.rows, stream)
                                : launch_tile(norm_tile_kernel<IN, OUT, false, 0>, p, g, smem, p.rows, stream);
}

template <int IN>
int norm_tile_out(const m3c_norm_params &p, const Tile &g, size_t smem, void *stream)
{
    switch (p.out_dtype) {
    case M3C_F16: return norm_tile<IN, M3C_F16>(p, g, smem, stream);
    case M3C_BF16: return norm_tile<IN, M3C_BF16>(p, g, smem, stream);
    default: return norm_tile<IN, M3C_F32>(p, g, smem, stream);
    }
}

int norm_tile_dispatch(const m3c_norm_params &p, const Tile &g, size_t smem, void *stream)
{
    switch (p.in_dtype) {
    case M3C_F16: return norm_tile_out<M3C_F16>(p, g, smem, stream);
    case M3C_BF16: return norm_tile_out<M3C_BF16>(p, g, smem, stream);
    default: return norm_tile_out<M3C_F32>(p, g, smem, stream);
    }
}

// Rows per CTA and dynamic shared memory of the generic kernels.
void row_shape(uint64_t width, int *rows_per_cta, size_t *smem_bytes, bool *fits)
{
    const size_t row_bytes = static_cast<size_t>(width) * sizeof(float);
    const size_t budget = 96u * 1024u;
    int rows = 4;
    while (rows > 1 && row_bytes * static_cast<size_t>(rows) > budget) rows >>= 1;
    *fits = row_bytes <= 200u * 1024u;
    *rows_per_cta = rows;
    *smem_bytes = *fits ? row_bytes * static_cast<size_t>(rows) : 0u;
}

}  // namespace
}  // namespace m3c

extern "C" int m3c_launch_softmax(const m3c_softmax_params *params, void *stream)
{
    if (params->rows > 0) {
        const int ring = m3c_launch_softmax_ring(params, stream);
        if (ring != -1) return ring;
    }
    const int eb = m3c::bytes_of(params->in_dtype);
    const m3c::Tile g = m3c::tile_geometry(params->width, eb, true, false, false);
    if (g.rows > 0 && params->rows > 0 && m3c::aligned16(params->input) &&
        (params->probs == nullptr || m3c::aligned16(params->probs))) {
        const size_t smem = m3c::tile_smem(g, true, eb, false);
        return m3c::softmax_tile_dispatch(*params, g, smem, stream);
    }
    int rows_per_cta = 4;
    size_t smem = 0;
    bool fits = true;
    m3c::row_shape(params->width, &rows_per_cta, &smem, &fits);
    if (smem > 48u * 1024u) {
        cudaFuncSetAttribute(m3c::softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    }
    const uint64_t needed = (params->rows + rows_per_cta - 1) / rows_per_cta;
    const uint64_t cap = static_cast<uint64_t>(m3c::sm_count_current()) * 32u;
    // at least one CTA: an empty launch still records the start of the run
    const unsigned grid = static_cast<unsigned>(needed == 0 ? 1 : (needed < cap ? needed : cap));
    m3c::softmax_kernel<<<grid, rows_per_cta * m3c::WARP, smem, static_cast<cudaStream_t>(stream)>>>(
        *params, rows_per_cta, fits ? 1 : 0);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int m3c_launch_norm(const m3c_norm_params *params, void *stream)
{
    const int eb = m3c::bytes_of(params->in_dtype);
    const bool resid = params->resid_b != nullptr;
    const bool bias = params->bias != nullptr;
    const m3c::Tile g = m3c::tile_geometry(params->width, eb, false, resid, bias);
    if (g.rows > 0 && params->rows > 0 && m3c::aligned16(params->x) && m3c::aligned16(params->out) &&
        (!resid || m3c::aligned16(params->resid_b)) &&
        (params->sum_out == nullptr || m3c::aligned16(params->sum_out))) {
        const size_t smem = m3c::tile_smem(g, false, eb, bias);
        return m3c::norm_tile_dispatch(*params, g, smem, stream);
    }
    int rows_per_cta = 4;
    size_t smem = 0;
    bool fits = true;
    m3c::row_shape(params->width, &rows_per_cta, &smem, &fits);
    if (!fits) {
        return static_cast<int>(cudaErrorInvalidValue);  // the planner rejects such widths
    }
    if (smem > 48u * 1024u) {
        cudaFuncSetAttribute(m3c::norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    }
    const uint64_t needed = (params->rows + rows_per_cta - 1) / rows_per_cta;
    const uint64_t cap = static_cast<uint64_t>(m3c::sm_count_current()) * 32u;
    const unsigned grid = static_cast<unsigned>(needed == 0 ? 1 : (needed < cap ? needed : cap));
    m3c::norm_kernel<<<grid, rows_per_cta * m3c::WARP, smem, static_cast<cudaStream_t>(stream)>>>(
        *params, rows_per_cta);
    return static_cast<int>(cudaGetLastError());
}
