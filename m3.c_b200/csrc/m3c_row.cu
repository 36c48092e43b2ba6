// Row kernels over the last axis (sm_100a): softmax + top-k, RMSNorm and
// LayerNorm.
//
// Layout: one warp per row.  The warp streams its row from HBM once with
// 16-byte loads into shared memory (widened to F32), computes the
// order-independent row statistics with warp shuffles (maximum, count of
// +inf, NaN, top-k candidates), and then reproduces the reference's
// left-to-right F32 sums with a single lane reading shared memory
// (src/m3_op_execute_basic.c:150-158, src/m3_op_execute_dense.c:128-140,
// :175-191).  A float sum depends on its order; summing in the reference's
// order makes RMSNorm and LayerNorm bit-identical to the reference and limits
// softmax differences to the expf implementation.  The serial lane costs
// width x (FADD latency) per row; other warps of the SM stream their rows
// meanwhile, so the kernels stay HBM-bound.
//
// Rows are contiguous (the session planner only gives these kernels dense
// row-major tensors); widths whose rows do not fit in shared memory fall back
// to re-reading the row from global memory.

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

// Stage a row into shared memory as F32 with 16-byte global loads when the
// row is 16-byte aligned; calls visit(j, v) for every element (in no
// particular order across lanes).
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
            if (eb == 4) {
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float x = as_float(words[t]);
                    if (smem) smem[j0 + t] = x;
                    visit(j0 + t, x);
                }
            } else {
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const uint32_t raw = (words[t >> 1] >> ((t & 1) * 16)) & 0xffffu;
                    const float x = widen(dtype, raw);
                    if (smem) smem[j0 + t] = x;
                    visit(j0 + t, x);
                }
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

// ------------------------------------------------------------------ softmax

// `smem_row` holds the row as F32 (nullptr: re-read the row from global).
__device__ void softmax_row(const m3c_softmax_params &p, uint64_t row, float *smem_row, int lane)
{
    const uint64_t width = p.width;
    const unsigned char *in_base = static_cast<const unsigned char *>(p.input);
    const void *in_row = in_base + row * width * static_cast<uint64_t>(bytes_of(p.in_dtype));
    float maximum = -__int_as_float(0x7f800000);
    uint32_t infinities = 0u;
    bool nan = false;
    float best_v = -__int_as_float(0x7f800000);
    uint32_t best_i = 0xffffffffu;

    // pass 1: maximum, +inf count, NaN, top-1 candidate
    stage_row(in_row, p.in_dtype, width, smem_row, lane, [&](uint64_t j, float x) {
        maximum = x > maximum ? x : maximum;
        infinities += x == __int_as_float(0x7f800000) ? 1u : 0u;
        nan |= x != x;
        if (precedes(x, static_cast<uint32_t>(j), best_v, best_i)) {
            best_v = x;
            best_i = static_cast<uint32_t>(j);
        }
    });
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float other = __shfl_xor_sync(0xffffffffu, maximum, off);
        maximum = other > maximum ? other : maximum;
        infinities += __shfl_xor_sync(0xffffffffu, infinities, off);
    }
    nan = __any_sync(0xffffffffu, nan);
    if (nan && lane == 0) {
        const uint32_t first = p.softmax_command < p.topk_command ? p.softmax_command : p.topk_command;
        record_failure(p.status, first);
    }
    __syncwarp();

    // top-k: K passes, each selecting the best element after the previous
    // one in the (value desc, index asc) order
    if (p.top_values != nullptr) {
        const uint64_t k = p.k;
        float last_v = 0.0f;
        uint32_t last_i = 0u;
        for (uint64_t t = 0; t < k; ++t) {
            float v = best_v;
            uint32_t i = best_i;
            if (t > 0) {
                v = -__int_as_float(0x7f800000);
                i = 0xffffffffu;
                for (uint64_t j = lane; j < width; j += WARP) {
                    const float x = smem_row ? smem_row[j] : load_elem(in_row, p.in_dtype, j);
                    const uint32_t ji = static_cast<uint32_t>(j);
                    if (precedes(last_v, last_i, x, ji) && (i == 0xffffffffu || precedes(x, ji, v, i))) {
                        v = x;
                        i = ji;
                    }
                }
            }
            // lanes without a candidate hold index 0xffffffff and lose
            if (i == 0xffffffffu) v = -__int_as_float(0x7f800000);
            warp_best(v, i);
            if (lane == 0) {
                p.top_values[row * k + t] = v;
                p.top_indices[row * k + t] = static_cast<int32_t>(i);
            }
            last_v = v;
            last_i = i;
        }
    }
    if (p.probs == nullptr) {
        return;
    }
    unsigned char *out_row = static_cast<unsigned char *>(p.probs) +
                             row * width * static_cast<uint64_t>(bytes_of(p.probs_dtype));
    const float pos_inf = __int_as_float(0x7f800000);
    if (maximum == -pos_inf || maximum == pos_inf) {
        // src/m3_op_execute_basic.c:165-170
        const float share = __fdiv_rn(1.0f, __uint2float_rn(infinities));
        for (uint64_t j = lane; j < width; j += WARP) {
            const float x = smem_row ? smem_row[j] : load_elem(in_row, p.in_dtype, j);
            const float prob = (maximum == pos_inf && x == pos_inf) ? share : 0.0f;
            store_elem(out_row, p.probs_dtype, j, prob);
        }
        return;
    }
    // pass 2: e_j = expf(x_j - max), then the reference's sequential sum
    float sum = 0.0f;
    if (smem_row != nullptr) {
        for (uint64_t j = lane; j < width; j += WARP) {
            smem_row[j] = expf(__fsub_rn(smem_row[j], maximum));
        }
        __syncwarp();
        if (lane == 0) {
            float s = 0.0f;
            uint64_t j = 0;
            if ((width & 3u) == 0u) {
                const float4 *e4 = reinterpret_cast<const float4 *>(smem_row);
                for (; j < width; j += 4) {
                    const float4 e = e4[j >> 2];
                    s = __fadd_rn(s, e.x);
                    s = __fadd_rn(s, e.y);
                    s = __fadd_rn(s, e.z);
                    s = __fadd_rn(s, e.w);
                }
            }
            for (; j < width; ++j) s = __fadd_rn(s, smem_row[j]);
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
    // pass 3: probabilities (src/m3_op_execute_basic.c:171-178)
    for (uint64_t j = lane; j < width; j += WARP) {
        const float e = smem_row ? smem_row[j]
                                 : expf(__fsub_rn(load_elem(in_row, p.in_dtype, j), maximum));
        store_elem(out_row, p.probs_dtype, j, __fdiv_rn(e, sum));
    }
}

__global__ void softmax_kernel(const __grid_constant__ m3c_softmax_params p, int rows_per_cta,
                               int use_smem)
{
    extern __shared__ float smem[];
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (run_failed(p.status)) {
        return;
    }
    if (p.first_of_run && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    float *row_smem = use_smem ? smem + static_cast<uint64_t>(warp) * p.width : nullptr;
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * rows_per_cta + warp; row < p.rows;
         row += static_cast<uint64_t>(gridDim.x) * rows_per_cta) {
        softmax_row(p, row, row_smem, lane);
        __syncwarp();
    }
}

// -------------------------------------------------------------------- norms

__device__ void norm_row(const m3c_norm_params &p, uint64_t row, float *smem_row, int lane)
{
    const uint64_t width = p.width;
    const uint64_t eb = static_cast<uint64_t>(bytes_of(p.in_dtype));
    const unsigned char *x_row = static_cast<const unsigned char *>(p.x) + row * width * eb;
    unsigned char *out_row = static_cast<unsigned char *>(p.out) +
                             row * width * static_cast<uint64_t>(bytes_of(p.out_dtype));

    // stage x (or the residual sum a + b rounded to the input dtype)
    if (p.resid_b != nullptr) {
        const unsigned char *b_row = static_cast<const unsigned char *>(p.resid_b) + row * width * eb;
        unsigned char *s_row = p.sum_out ? static_cast<unsigned char *>(p.sum_out) + row * width * eb
                                         : nullptr;
        for (uint64_t j = lane; j < width; j += WARP) {
            // src/m3_op_execute_basic.c:61-77: one F32 add, stored in the
            // sum's dtype, read back widened
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
            // src/m3_op_execute_dense.c:175-194
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
            // src/m3_op_execute_dense.c:128-141
            float squares = 0.0f;
            uint64_t j = 0;
            if ((width & 3u) == 0u) {
                const float4 *v4 = reinterpret_cast<const float4 *>(smem_row);
                for (; j < width; j += 4) {
                    const float4 v = v4[j >> 2];
                    squares = __fadd_rn(squares, __fmul_rn(v.x, v.x));
                    squares = __fadd_rn(squares, __fmul_rn(v.y, v.y));
                    squares = __fadd_rn(squares, __fmul_rn(v.z, v.z));
                    squares = __fadd_rn(squares, __fmul_rn(v.w, v.w));
                }
            }
            for (; j < width; ++j) squares = __fadd_rn(squares, __fmul_rn(smem_row[j], smem_row[j]));
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
            // ((x - mean) * inv) * scale (+ bias), src/m3_op_execute_dense.c:195-213
            result = __fmul_rn(__fmul_rn(__fsub_rn(x, mean), inverse), w);
            if (p.bias != nullptr) {
                result = __fadd_rn(result, load_elem(p.bias, p.bias_dtype, j));
            }
        } else {
            // round to the input dtype before scaling, src/m3_op_execute_dense.c:149-151
            result = __fmul_rn(round_to(p.in_dtype, __fmul_rn(x, inverse)), w);
        }
        store_elem(out_row, p.out_dtype, j, result);
    }
}

__global__ void norm_kernel(const __grid_constant__ m3c_norm_params p, int rows_per_cta)
{
    extern __shared__ float smem[];
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (run_failed(p.status)) {
        return;
    }
    if (p.first_of_run && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    float *row_smem = smem + static_cast<uint64_t>(warp) * p.width;
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * rows_per_cta + warp; row < p.rows;
         row += static_cast<uint64_t>(gridDim.x) * rows_per_cta) {
        norm_row(p, row, row_smem, lane);
        __syncwarp();
    }
}

// ------------------------------------------- register-staged fast paths
//
// For rows that are 16-byte aligned and at most 32 * VPL vectors wide, each
// lane owns VPL 16-byte vectors of the row (vector v = lane + 32 i).  The warp
// issues all of its row's loads at once, and -- before the serial sum of the
// current row -- issues the loads of its next row into the same registers, so
// HBM traffic continues while one lane walks the row in the reference's order.

template <int EB>
struct VecTraits {
    static constexpr int EPV = 16 / EB;  // elements per 16-byte vector
};

template <int EB>
__device__ __forceinline__ void unpack(const uint4 &q, int dtype, float (&x)[16 / EB])
{
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if (EB == 4) {
#pragma unroll
        for (int t = 0; t < 4; ++t) x[t] = as_float(w[t]);
    } else {
#pragma unroll
        for (int t = 0; t < 16 / EB; ++t) x[t] = widen(dtype, (w[t >> 1] >> ((t & 1) * 16)) & 0xffffu);
    }
}

template <int EB>
__device__ __forceinline__ uint4 pack_raw(const uint32_t (&h)[16 / EB])
{
    if (EB == 4) {
        return make_uint4(h[0], h[1], h[2], h[3]);
    }
    return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                      h[6] | (h[7] << 16));
}

template <int VPL>
__device__ __forceinline__ void load_vecs(const uint4 *row, int nvec, int lane, uint4 (&q)[VPL])
{
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int v = lane + WARP * i;
        if (v < nvec) q[i] = __ldcs(row + v);
    }
}

// Store `count` (4 or 8) floats converted to `dtype` at element j0 of a
// 16-byte aligned row.
template <int COUNT>
__device__ __forceinline__ void store_vec(void *row, int dtype, int j0, const float (&v)[COUNT])
{
    if (dtype == M3C_F32) {
        float4 *out = reinterpret_cast<float4 *>(static_cast<float *>(row) + j0);
#pragma unroll
        for (int t = 0; t < COUNT / 4; ++t) {
            __stcs(out + t, make_float4(v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]));
        }
    } else {
        uint32_t h[COUNT];
#pragma unroll
        for (int t = 0; t < COUNT; ++t) h[t] = narrow(dtype, v[t]);
        uint16_t *base = static_cast<uint16_t *>(row) + j0;
        if (COUNT == 8) {
            __stcs(reinterpret_cast<uint4 *>(base),
                   make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                              h[6] | (h[7] << 16)));
        } else {
            __stcs(reinterpret_cast<uint2 *>(base), make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16)));
        }
    }
}

// Lane 0's left-to-right F32 sum of a shared-memory row (width % 4 == 0).
__device__ __forceinline__ float serial_sum(const float *row, int width)
{
    const float4 *v4 = reinterpret_cast<const float4 *>(row);
    float s = 0.0f;
#pragma unroll 16
    for (int j = 0; j < width / 4; ++j) {
        const float4 e = v4[j];
        s = __fadd_rn(s, e.x);
        s = __fadd_rn(s, e.y);
        s = __fadd_rn(s, e.z);
        s = __fadd_rn(s, e.w);
    }
    return s;
}

__device__ __forceinline__ float serial_sum_of_squares(const float *row, int width)
{
    const float4 *v4 = reinterpret_cast<const float4 *>(row);
    float s = 0.0f;
#pragma unroll 16
    for (int j = 0; j < width / 4; ++j) {
        const float4 e = v4[j];
        s = __fadd_rn(s, __fmul_rn(e.x, e.x));
        s = __fadd_rn(s, __fmul_rn(e.y, e.y));
        s = __fadd_rn(s, __fmul_rn(e.z, e.z));
        s = __fadd_rn(s, __fmul_rn(e.w, e.w));
    }
    return s;
}

template <int EB, int VPL>
__global__ void __launch_bounds__(128) softmax_fast_kernel(const __grid_constant__ m3c_softmax_params p)
{
    constexpr int EPV = VecTraits<EB>::EPV;
    extern __shared__ float smem[];
    const int warps = static_cast<int>(blockDim.x) / WARP;
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (run_failed(p.status)) {
        return;
    }
    if (p.first_of_run && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    const int width = static_cast<int>(p.width);
    const int nvec = width / EPV;
    float *srow = smem + static_cast<size_t>(warp) * width;
    const uint4 *in = static_cast<const uint4 *>(p.input);
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * warps;
    const float pos_inf = __int_as_float(0x7f800000);
    const uint32_t first_command = p.softmax_command < p.topk_command ? p.softmax_command : p.topk_command;
    uint64_t row = static_cast<uint64_t>(blockIdx.x) * warps + warp;
    uint4 q[VPL];
    if (row < p.rows) load_vecs<VPL>(in + row * nvec, nvec, lane, q);
    for (; row < p.rows; row += stride) {
        // 1. stage the row as F32 and gather the order-free statistics
        float maximum = -pos_inf;
        uint32_t infinities = 0u;
        bool nan = false;
        float best_v = -pos_inf;
        uint32_t best_i = 0xffffffffu;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int v = lane + WARP * i;
            if (v < nvec) {
                float x[EPV];
                unpack<EB>(q[i], p.in_dtype, x);
                float4 *dst = reinterpret_cast<float4 *>(srow + v * EPV);
#pragma unroll
                for (int t = 0; t < EPV / 4; ++t) dst[t] = make_float4(x[4 * t], x[4 * t + 1], x[4 * t + 2], x[4 * t + 3]);
#pragma unroll
                for (int t = 0; t < EPV; ++t) {
                    const uint32_t j = static_cast<uint32_t>(v * EPV + t);
                    maximum = x[t] > maximum ? x[t] : maximum;
                    infinities += x[t] == pos_inf ? 1u : 0u;
                    nan |= x[t] != x[t];
                    if (x[t] > best_v || (x[t] == best_v && j < best_i)) {
                        best_v = x[t];
                        best_i = j;
                    }
                }
            }
        }
        // 2. prefetch the next row while this one is finished
        const uint64_t next = row + stride;
        if (next < p.rows) load_vecs<VPL>(in + next * nvec, nvec, lane, q);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, maximum, off);
            maximum = other > maximum ? other : maximum;
            infinities += __shfl_xor_sync(0xffffffffu, infinities, off);
        }
        if (__any_sync(0xffffffffu, nan) && lane == 0) {
            record_failure(p.status, first_command);
        }
        __syncwarp();
        // 3. top-k: K passes over the staged row
        if (p.top_values != nullptr) {
            const uint64_t k = p.k;
            float last_v = 0.0f;
            uint32_t last_i = 0u;
            for (uint64_t t = 0; t < k; ++t) {
                float v = best_v;
                uint32_t i = best_i;
                if (t > 0) {
                    v = -pos_inf;
                    i = 0xffffffffu;
                    for (int j = lane; j < width; j += WARP) {
                        const float x = srow[j];
                        const uint32_t ji = static_cast<uint32_t>(j);
                        if (precedes(last_v, last_i, x, ji) && (i == 0xffffffffu || precedes(x, ji, v, i))) {
                            v = x;
                            i = ji;
                        }
                    }
                }
                if (i == 0xffffffffu) v = -pos_inf;
                warp_best(v, i);
                if (lane == 0) {
                    p.top_values[row * k + t] = v;
                    p.top_indices[row * k + t] = static_cast<int32_t>(i);
                }
                last_v = v;
                last_i = i;
            }
        }
        if (p.probs != nullptr) {
            void *out_row = static_cast<unsigned char *>(p.probs) +
                            row * static_cast<uint64_t>(width) * static_cast<uint64_t>(bytes_of(p.probs_dtype));
            if (maximum == -pos_inf || maximum == pos_inf) {
                // src/m3_op_execute_basic.c:165-170
                const float share = __fdiv_rn(1.0f, __uint2float_rn(infinities));
#pragma unroll
                for (int i = 0; i < VPL; ++i) {
                    const int v = lane + WARP * i;
                    if (v < nvec) {
                        float pr[EPV];
#pragma unroll
                        for (int t = 0; t < EPV; ++t) {
                            pr[t] = (maximum == pos_inf && srow[v * EPV + t] == pos_inf) ? share : 0.0f;
                        }
                        store_vec<EPV>(out_row, p.probs_dtype, v * EPV, pr);
                    }
                }
            } else {
                // 4. e = expf(x - max) in place; the reference's ordered sum
#pragma unroll
                for (int i = 0; i < VPL; ++i) {
                    const int v = lane + WARP * i;
                    if (v < nvec) {
                        float4 *e4 = reinterpret_cast<float4 *>(srow + v * EPV);
#pragma unroll
                        for (int t = 0; t < EPV / 4; ++t) {
                            float4 e = e4[t];
                            e.x = expf(__fsub_rn(e.x, maximum));
                            e.y = expf(__fsub_rn(e.y, maximum));
                            e.z = expf(__fsub_rn(e.z, maximum));
                            e.w = expf(__fsub_rn(e.w, maximum));
                            e4[t] = e;
                        }
                    }
                }
                __syncwarp();
                float sum = 0.0f;
                if (lane == 0) sum = serial_sum(srow, width);
                sum = __shfl_sync(0xffffffffu, sum, 0);
                // 5. probabilities (src/m3_op_execute_basic.c:171-178)
#pragma unroll
                for (int i = 0; i < VPL; ++i) {
                    const int v = lane + WARP * i;
                    if (v < nvec) {
                        float pr[EPV];
#pragma unroll
                        for (int t = 0; t < EPV; ++t) pr[t] = __fdiv_rn(srow[v * EPV + t], sum);
                        store_vec<EPV>(out_row, p.probs_dtype, v * EPV, pr);
                    }
                }
            }
        }
        __syncwarp();
    }
}

template <int EB, int VPL, bool RESID>
__global__ void __launch_bounds__(128) norm_fast_kernel(const __grid_constant__ m3c_norm_params p)
{
    constexpr int EPV = VecTraits<EB>::EPV;
    extern __shared__ float smem[];
    const int warps = static_cast<int>(blockDim.x) / WARP;
    const int warp = static_cast<int>(threadIdx.x) / WARP;
    const int lane = static_cast<int>(threadIdx.x) % WARP;
    if (run_failed(p.status)) {
        return;
    }
    if (p.first_of_run && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    const int width = static_cast<int>(p.width);
    const int nvec = width / EPV;
    float *srow = smem + static_cast<size_t>(warp) * width;
    const uint4 *xa = static_cast<const uint4 *>(p.x);
    const uint4 *xb = static_cast<const uint4 *>(p.resid_b);
    uint4 *sum_out = static_cast<uint4 *>(p.sum_out);
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * warps;
    const float channels = __int2float_rn(width);
    uint64_t row = static_cast<uint64_t>(blockIdx.x) * warps + warp;
    uint4 qa[VPL];
    uint4 qb[RESID ? VPL : 1];
    if (row < p.rows) {
        load_vecs<VPL>(xa + row * nvec, nvec, lane, qa);
        if constexpr (RESID) load_vecs<VPL>(xb + row * nvec, nvec, lane, qb);
    }
    for (; row < p.rows; row += stride) {
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int v = lane + WARP * i;
            if (v < nvec) {
                float x[EPV];
                unpack<EB>(qa[i], p.in_dtype, x);
                if constexpr (RESID) {
                    // the residual ADD, stored in the input dtype and read back
                    float b[EPV];
                    uint32_t raw[EPV];
                    unpack<EB>(qb[i], p.in_dtype, b);
#pragma unroll
                    for (int t = 0; t < EPV; ++t) {
                        raw[t] = narrow(p.in_dtype, __fadd_rn(x[t], b[t]));
                        x[t] = widen(p.in_dtype, raw[t]);
                    }
                    if (sum_out != nullptr) __stcs(sum_out + row * nvec + v, pack_raw<EB>(raw));
                }
                float4 *dst = reinterpret_cast<float4 *>(srow + v * EPV);
#pragma unroll
                for (int t = 0; t < EPV / 4; ++t) dst[t] = make_float4(x[4 * t], x[4 * t + 1], x[4 * t + 2], x[4 * t + 3]);
            }
        }
        const uint64_t next = row + stride;
        if (next < p.rows) {
            load_vecs<VPL>(xa + next * nvec, nvec, lane, qa);
            if constexpr (RESID) load_vecs<VPL>(xb + next * nvec, nvec, lane, qb);
        }
        __syncwarp();
        float mean = 0.0f;
        float inverse = 0.0f;
        if (lane == 0) {
            if (p.layer_norm) {
                // src/m3_op_execute_dense.c:175-194
                mean = __fdiv_rn(serial_sum(srow, width), channels);
                float centred = 0.0f;
                for (int j = 0; j < width; ++j) {
                    const float c = __fsub_rn(srow[j], mean);
                    centred = __fadd_rn(centred, __fmul_rn(c, c));
                }
                inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(centred, channels), p.epsilon)));
            } else {
                // src/m3_op_execute_dense.c:128-141
                const float squares = serial_sum_of_squares(srow, width);
                inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(squares, channels), p.epsilon)));
            }
        }
        mean = __shfl_sync(0xffffffffu, mean, 0);
        inverse = __shfl_sync(0xffffffffu, inverse, 0);
        void *out_row = static_cast<unsigned char *>(p.out) +
                        row * static_cast<uint64_t>(width) * static_cast<uint64_t>(bytes_of(p.out_dtype));
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int v = lane + WARP * i;
            if (v < nvec) {
                float r[EPV];
#pragma unroll
                for (int t = 0; t < EPV; ++t) {
                    const int j = v * EPV + t;
                    const float x = srow[j];
                    const float w = load_elem(p.scale, p.scale_dtype, j);
                    if (p.layer_norm) {
                        float y = __fmul_rn(__fmul_rn(__fsub_rn(x, mean), inverse), w);
                        if (p.bias != nullptr) y = __fadd_rn(y, load_elem(p.bias, p.bias_dtype, j));
                        r[t] = y;
                    } else {
                        r[t] = __fmul_rn(round_to(p.in_dtype, __fmul_rn(x, inverse)), w);
                    }
                }
                store_vec<EPV>(out_row, p.out_dtype, v * EPV, r);
            }
        }
        __syncwarp();
    }
}

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

// Rows per CTA and dynamic shared memory for a row of `width` F32 values.
void row_shape(uint64_t width, int *rows_per_cta, size_t *smem_bytes, bool *fits)
{
    const size_t row_bytes = static_cast<size_t>(width) * sizeof(float);
    const size_t budget = 96u * 1024u;  // per CTA; several CTAs share an SM
    int rows = 4;
    while (rows > 1 && row_bytes * static_cast<size_t>(rows) > budget) rows >>= 1;
    *fits = row_bytes <= 200u * 1024u;
    *rows_per_cta = rows;
    *smem_bytes = *fits ? row_bytes * static_cast<size_t>(rows) : 0u;
}

}  // namespace
}  // namespace m3c

namespace m3c {
namespace {

constexpr int FAST_WARPS = 4;

// Smallest VPL in {1,2,4,8,16} that covers `width` elements of `eb` bytes,
// or 0 when the row is too wide for the register-staged path.
int pick_vpl(uint64_t width, int eb)
{
    const uint64_t per_lane = 16u / static_cast<uint64_t>(eb);
    for (int vpl = 1; vpl <= 16; vpl <<= 1) {
        if (width <= static_cast<uint64_t>(WARP) * vpl * per_lane) return vpl;
    }
    return 0;
}

bool aligned16(const void *p)
{
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u;
}

template <typename Kernel, typename Params>
int launch_fast(Kernel kernel, const Params &params, uint64_t rows, uint64_t width, void *stream)
{
    const size_t smem = static_cast<size_t>(FAST_WARPS) * width * sizeof(float);
    if (smem > 48u * 1024u) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, FAST_WARPS * WARP, smem) !=
            cudaSuccess ||
        per_sm < 1) {
        per_sm = 1;
    }
    // persistent grid: every resident CTA strides over rows, so each warp
    // always has its next row in flight
    const uint64_t needed = (rows + FAST_WARPS - 1) / FAST_WARPS;
    const uint64_t cap = static_cast<uint64_t>(sm_count_current()) * static_cast<uint64_t>(per_sm);
    const unsigned grid = static_cast<unsigned>(needed == 0 ? 1 : (needed < cap ? needed : cap));
    kernel<<<grid, FAST_WARPS * WARP, smem, static_cast<cudaStream_t>(stream)>>>(params);
    return static_cast<int>(cudaGetLastError());
}

template <int EB>
int softmax_fast(const m3c_softmax_params &p, int vpl, void *stream)
{
    switch (vpl) {
    case 1: return launch_fast(softmax_fast_kernel<EB, 1>, p, p.rows, p.width, stream);
    case 2: return launch_fast(softmax_fast_kernel<EB, 2>, p, p.rows, p.width, stream);
    case 4: return launch_fast(softmax_fast_kernel<EB, 4>, p, p.rows, p.width, stream);
    case 8: return launch_fast(softmax_fast_kernel<EB, 8>, p, p.rows, p.width, stream);
    default: return launch_fast(softmax_fast_kernel<EB, 16>, p, p.rows, p.width, stream);
    }
}

template <int EB, bool RESID>
int norm_fast(const m3c_norm_params &p, int vpl, void *stream)
{
    switch (vpl) {
    case 1: return launch_fast(norm_fast_kernel<EB, 1, RESID>, p, p.rows, p.width, stream);
    case 2: return launch_fast(norm_fast_kernel<EB, 2, RESID>, p, p.rows, p.width, stream);
    case 4: return launch_fast(norm_fast_kernel<EB, 4, RESID>, p, p.rows, p.width, stream);
    case 8: return launch_fast(norm_fast_kernel<EB, 8, RESID>, p, p.rows, p.width, stream);
    default: return launch_fast(norm_fast_kernel<EB, 16, RESID>, p, p.rows, p.width, stream);
    }
}

}  // namespace
}  // namespace m3c

extern "C" int m3c_launch_softmax(const m3c_softmax_params *params, void *stream)
{
    {
        const int eb = m3c::bytes_of(params->in_dtype);
        const uint64_t per_vec = 16u / static_cast<uint64_t>(eb);
        const int vpl = m3c::pick_vpl(params->width, eb);
        if (vpl != 0 && params->rows != 0 && params->width % per_vec == 0 &&
            m3c::aligned16(params->input) &&
            (params->probs == nullptr || m3c::aligned16(params->probs))) {
            return eb == 4 ? m3c::softmax_fast<4>(*params, vpl, stream)
                           : m3c::softmax_fast<2>(*params, vpl, stream);
        }
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
    {
        const int eb = m3c::bytes_of(params->in_dtype);
        const uint64_t per_vec = 16u / static_cast<uint64_t>(eb);
        const int vpl = m3c::pick_vpl(params->width, eb);
        const bool resid = params->resid_b != nullptr;
        if (vpl != 0 && params->rows != 0 && params->width % per_vec == 0 &&
            m3c::aligned16(params->x) && m3c::aligned16(params->out) &&
            (!resid || m3c::aligned16(params->resid_b)) &&
            (params->sum_out == nullptr || m3c::aligned16(params->sum_out))) {
            if (eb == 4) {
                return resid ? m3c::norm_fast<4, true>(*params, vpl, stream)
                             : m3c::norm_fast<4, false>(*params, vpl, stream);
            }
            return resid ? m3c::norm_fast<2, true>(*params, vpl, stream)
                         : m3c::norm_fast<2, false>(*params, vpl, stream);
        }
    }
    int rows_per_cta = 4;
    size_t smem = 0;
    bool fits = true;
    m3c::row_shape(params->width, &rows_per_cta, &smem, &fits);
    if (!fits) {
        return static_cast<int>(cudaErrorInvalidValue);  // planner rejects such widths
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
