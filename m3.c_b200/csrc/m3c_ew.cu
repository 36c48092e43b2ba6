// Fused element-wise engine (sm_100a).
//
// One launch evaluates a straight-line program of micro-operations over the
// flat index space of one output shape.  Every thread handles VEC = 4
// consecutive elements per step of a grid-stride loop:
//   1. load each operand for the block (a 16-byte or 8-byte vector when the
//      operand runs in output order, one element when the block reads a
//      single broadcast element, per-element strided/broadcast gathers
//      otherwise, or an immediate for folded scalar constants),
//   2. run the ops on 32-bit register words,
//   3. store the outputs (vector stores; outputs are contiguous).
// The program is uniform across the grid, so the op dispatch and the register
// selection are warp-uniform switches over compile-time register indices: the
// register file stays in registers.
//
// Arithmetic follows the reference CPU executors statement by statement with
// F32 rounding per statement (no contraction: the library is compiled with
// --fmad=false and the float statements below use explicit _rn intrinsics):
//   ADD/MUL       src/m3_op_execute_basic.c:61-77
//   GATED_SILU    src/m3_op_execute_basic.c:104-122
//   SNAKE1D       src/m3_op_execute_basic.c:183-215
//   TANH          src/m3_op_execute_basic.c:217-230
//   CAST/COPY     src/m3_op_execute_basic.c:11-59
//   clamp         src/m3_waveform.c:360-380

#include <cuda_runtime.h>

#include <cstdint>

#include "m3c_device.cuh"
#include "m3c_kernels.h"

namespace m3c {
namespace {

constexpr int VEC = 4;
constexpr int THREADS = 256;
constexpr int REGS = M3C_EW_MAX_REGS;

using Word4 = uint32_t[VEC];

struct RegisterFile {
    uint32_t w[REGS][VEC];
};

__device__ __forceinline__ void reg_get(const RegisterFile &rf, int index, uint32_t (&out)[VEC])
{
    switch (index) {
#define M3C_GET(I)                                  \
    case I:                                         \
        _Pragma("unroll") for (int j = 0; j < VEC; ++j) out[j] = rf.w[I][j]; \
        break;
        M3C_GET(0) M3C_GET(1) M3C_GET(2) M3C_GET(3)
        M3C_GET(4) M3C_GET(5) M3C_GET(6) M3C_GET(7)
#undef M3C_GET
    default:
        break;
    }
}

__device__ __forceinline__ void reg_set(RegisterFile &rf, int index, const uint32_t (&in)[VEC])
{
    switch (index) {
#define M3C_SET(I)                                  \
    case I:                                         \
        _Pragma("unroll") for (int j = 0; j < VEC; ++j) rf.w[I][j] = in[j]; \
        break;
        M3C_SET(0) M3C_SET(1) M3C_SET(2) M3C_SET(3)
        M3C_SET(4) M3C_SET(5) M3C_SET(6) M3C_SET(7)
#undef M3C_SET
    default:
        break;
    }
}

__device__ __forceinline__ int dtype_bytes(int dtype)
{
    return (dtype == M3C_F16 || dtype == M3C_BF16) ? 2 : 4;
}

// Byte offset of element f of a strided/broadcast operand.
template <bool WIDE>
__device__ __forceinline__ int64_t operand_offset(const m3c_operand &op, uint64_t f)
{
    int64_t offset = 0;
    if (WIDE) {
        uint64_t q = f;
#pragma unroll
        for (int d = 0; d < M3C_MAX_DIMS; ++d) {
            if (d < op.ndim) {
                const uint64_t next = q / op.size[d];
                offset += static_cast<int64_t>(q - next * op.size[d]) * op.stride[d];
                q = next;
            }
        }
    } else {
        uint32_t q = static_cast<uint32_t>(f);
#pragma unroll
        for (int d = 0; d < M3C_MAX_DIMS; ++d) {
            if (d < op.ndim) {
                const uint32_t next = fastdiv(q, op.fdiv[d]);
                offset += static_cast<int64_t>(q - next * static_cast<uint32_t>(op.size[d])) *
                          op.stride[d];
                q = next;
            }
        }
    }
    return offset;
}

__device__ __forceinline__ uint32_t load_one(const m3c_operand &op, int64_t offset)
{
    const unsigned char *p = static_cast<const unsigned char *>(op.base) + offset;
    if (dtype_bytes(op.dtype) == 2) {
        return *reinterpret_cast<const uint16_t *>(p);
    }
    return *reinterpret_cast<const uint32_t *>(p);
}

// Load the VEC words of a full block starting at flat index f.
template <bool WIDE>
__device__ __forceinline__ void load_block(const m3c_operand &op, uint64_t f, uint32_t (&out)[VEC])
{
    switch (op.vclass) {
    case M3C_V_IMM:
#pragma unroll
        for (int j = 0; j < VEC; ++j) out[j] = op.imm_bits;
        break;
    case M3C_V_CONTIG:
        if (dtype_bytes(op.dtype) == 4) {
            const uint4 v = *reinterpret_cast<const uint4 *>(
                static_cast<const unsigned char *>(op.base) + f * 4u);
            out[0] = v.x;
            out[1] = v.y;
            out[2] = v.z;
            out[3] = v.w;
        } else {
            const uint2 v = *reinterpret_cast<const uint2 *>(
                static_cast<const unsigned char *>(op.base) + f * 2u);
            out[0] = v.x & 0xffffu;
            out[1] = v.x >> 16;
            out[2] = v.y & 0xffffu;
            out[3] = v.y >> 16;
        }
        break;
    case M3C_V_VECTOR: {
        const unsigned char *at = static_cast<const unsigned char *>(op.base) +
                                  operand_offset<WIDE>(op, f);
        if (dtype_bytes(op.dtype) == 4) {
            const uint4 v = *reinterpret_cast<const uint4 *>(at);
            out[0] = v.x;
            out[1] = v.y;
            out[2] = v.z;
            out[3] = v.w;
        } else {
            const uint2 v = *reinterpret_cast<const uint2 *>(at);
            out[0] = v.x & 0xffffu;
            out[1] = v.x >> 16;
            out[2] = v.y & 0xffffu;
            out[3] = v.y >> 16;
        }
        break;
    }
    case M3C_V_UNIFORM: {
        const uint32_t w = load_one(op, operand_offset<WIDE>(op, f));
#pragma unroll
        for (int j = 0; j < VEC; ++j) out[j] = w;
        break;
    }
    default:
#pragma unroll
        for (int j = 0; j < VEC; ++j) out[j] = load_one(op, operand_offset<WIDE>(op, f + j));
        break;
    }
}

// Load the first `valid` words of a partial block (the tail).
template <bool WIDE>
__device__ __forceinline__ void load_partial(const m3c_operand &op, uint64_t f, int valid,
                                             uint32_t (&out)[VEC])
{
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
        out[j] = 0u;
        if (j < valid) {
            out[j] = op.vclass == M3C_V_IMM ? op.imm_bits
                                            : load_one(op, operand_offset<WIDE>(op, f + j));
        }
    }
}

__device__ __forceinline__ float snake(float x, float alpha)
{
    // src/m3_op_execute_basic.c:183-194, epsilon bits 0x3089705f
    const float denominator = __fadd_rn(alpha, 0x1.12e0bep-30f);
    const float inverse = __fdiv_rn(1.0f, denominator);
    const float angle = __fmul_rn(alpha, x);
    const float sine = sinf(angle);
    const float square = __fmul_rn(sine, sine);
    const float scaled = __fmul_rn(inverse, square);
    return __fadd_rn(x, scaled);
}

__device__ __forceinline__ float gated_silu(float gate, float up, int gate_dtype)
{
    // src/m3_op_execute_basic.c:113-117
    const float denominator = __fadd_rn(1.0f, expf(-gate));
    const float activation = round_to(gate_dtype, __fdiv_rn(gate, denominator));
    return __fmul_rn(activation, up);
}

struct Flags {
    uint32_t fail_command;
    uint32_t max_bits;
};

__device__ __forceinline__ void run_op(const m3c_ew_op &op, RegisterFile &rf, int valid,
                                       Flags &flags)
{
    uint32_t a[VEC];
    uint32_t b[VEC];
    uint32_t d[VEC];
    reg_get(rf, op.a, a);
    reg_get(rf, op.b, b);
    const int rdt = op.rdtype;
    switch (op.code) {
    case M3C_OP_ADD:
#pragma unroll
        for (int j = 0; j < VEC; ++j)
            d[j] = as_bits(round_to(rdt, __fadd_rn(as_float(a[j]), as_float(b[j]))));
        break;
    case M3C_OP_MUL:
#pragma unroll
        for (int j = 0; j < VEC; ++j)
            d[j] = as_bits(round_to(rdt, __fmul_rn(as_float(a[j]), as_float(b[j]))));
        break;
    case M3C_OP_GSILU:
#pragma unroll
        for (int j = 0; j < VEC; ++j)
            d[j] = as_bits(round_to(rdt, gated_silu(as_float(a[j]), as_float(b[j]), op.aux)));
        break;
    case M3C_OP_SNAKE:
        if (b[0] == b[1] && b[1] == b[2] && b[2] == b[3]) {
            // one channel per block (the common case): the reciprocal of
            // (alpha + eps) is the same statement for all four elements
            const float alpha = as_float(b[0]);
            const float inverse = __fdiv_rn(1.0f, __fadd_rn(alpha, 0x1.12e0bep-30f));
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                const float x = as_float(a[j]);
                const float sine = sinf(__fmul_rn(alpha, x));
                d[j] = as_bits(__fadd_rn(x, __fmul_rn(inverse, __fmul_rn(sine, sine))));
            }
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) d[j] = as_bits(snake(as_float(a[j]), as_float(b[j])));
        }
        break;
    case M3C_OP_TANH:
#pragma unroll
        for (int j = 0; j < VEC; ++j) d[j] = as_bits(tanhf(as_float(a[j])));
        break;
    case M3C_OP_ROUND:
#pragma unroll
        for (int j = 0; j < VEC; ++j) d[j] = as_bits(round_to(rdt, as_float(a[j])));
        break;
    case M3C_OP_F2I:
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            // src/m3_op_data_preflight.c:17-25 and the C conversion of
            // src/m3_op_execute_basic.c:52 (truncation toward zero)
            const float v = as_float(a[j]);
            const bool ok = v >= -2147483648.0f && v < 2147483648.0f;  // false for NaN
            if (!ok && j < valid) {
                flags.fail_command = min(flags.fail_command, static_cast<uint32_t>(op.command));
            }
            d[j] = ok ? static_cast<uint32_t>(__float2int_rz(v)) : 0u;
        }
        break;
    case M3C_OP_I2F:
#pragma unroll
        for (int j = 0; j < VEC; ++j)
            d[j] = as_bits(round_to(rdt, __int2float_rn(static_cast<int32_t>(a[j]))));
        break;
    case M3C_OP_WIDEN:
#pragma unroll
        for (int j = 0; j < VEC; ++j) d[j] = as_bits(widen(op.aux, a[j]));
        break;
    case M3C_OP_CLAMP:
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            // integer selects: the bits of every in-range value (NaN
            // payloads, signed zeros) pass through unchanged
            const float v = as_float(a[j]);
            uint32_t w = a[j];
            w = v > 1.0f ? 0x3f800000u : w;
            w = v < -1.0f ? 0xbf800000u : w;
            d[j] = w;
        }
        break;
    case M3C_OP_MOV:
#pragma unroll
        for (int j = 0; j < VEC; ++j) d[j] = a[j];
        break;
    case M3C_OP_ABSMAX:
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            if (j < valid) {
                const uint32_t magnitude = a[j] & 0x7fffffffu;
                if (magnitude > 0x7f800000u) {
                    flags.fail_command = min(flags.fail_command, static_cast<uint32_t>(op.command));
                } else {
                    flags.max_bits = max(flags.max_bits, magnitude);
                }
            }
        }
        return;  // no result register
    default:
        return;
    }
    reg_set(rf, op.dst, d);
}

__device__ __forceinline__ void store_block(const m3c_ew_out &out, uint64_t f, const uint32_t (&w)[VEC])
{
    unsigned char *p = static_cast<unsigned char *>(out.base);
    if (out.dtype == M3C_F16 || out.dtype == M3C_BF16) {
        uint32_t h[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) h[j] = out.raw ? (w[j] & 0xffffu) : narrow(out.dtype, as_float(w[j]));
        *reinterpret_cast<uint2 *>(p + f * 2u) = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
    } else {
        *reinterpret_cast<uint4 *>(p + f * 4u) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ void store_partial(const m3c_ew_out &out, uint64_t f, int valid,
                                              const uint32_t (&w)[VEC])
{
    unsigned char *p = static_cast<unsigned char *>(out.base);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
        if (j < valid) {
            if (out.dtype == M3C_F16 || out.dtype == M3C_BF16) {
                const uint32_t h = out.raw ? (w[j] & 0xffffu) : narrow(out.dtype, as_float(w[j]));
                *reinterpret_cast<uint16_t *>(p + (f + j) * 2u) = static_cast<uint16_t>(h);
            } else {
                *reinterpret_cast<uint32_t *>(p + (f + j) * 4u) = w[j];
            }
        }
    }
}

template <bool WIDE>
__device__ __forceinline__ void process(const m3c_ew_params &p, uint64_t f, int valid, Flags &flags)
{
    RegisterFile rf;
#pragma unroll
    for (int i = 0; i < M3C_EW_MAX_OPERANDS && i < REGS; ++i) {
        if (i < p.n_operands) {
            if (valid == VEC) {
                load_block<WIDE>(p.operands[i], f, rf.w[i]);
            } else {
                load_partial<WIDE>(p.operands[i], f, valid, rf.w[i]);
            }
        }
    }
    for (int k = 0; k < p.n_ops; ++k) {
        run_op(p.ops[k], rf, valid, flags);
    }
#pragma unroll
    for (int o = 0; o < M3C_EW_MAX_OUTPUTS; ++o) {
        if (o < p.n_outputs) {
            uint32_t w[VEC];
            reg_get(rf, p.outputs[o].reg, w);
            if (valid == VEC) {
                store_block(p.outputs[o], f, w);
            } else {
                store_partial(p.outputs[o], f, valid, w);
            }
        }
    }
}

template <bool WIDE>
__global__ void __launch_bounds__(THREADS) ew_kernel(const __grid_constant__ m3c_ew_params p)
{
    const bool skip = run_failed(p.status);
    if (p.first_of_run && !skip && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    Flags flags{0xffffffffu, 0u};
    if (!skip) {
        const uint64_t blocks = p.count / VEC;
        const uint64_t stride = static_cast<uint64_t>(gridDim.x) * THREADS;
        for (uint64_t v = static_cast<uint64_t>(blockIdx.x) * THREADS + threadIdx.x; v < blocks;
             v += stride) {
            process<WIDE>(p, v * VEC, VEC, flags);
        }
        const int tail = static_cast<int>(p.count - blocks * VEC);
        if (tail != 0 && blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
            process<WIDE>(p, blocks * VEC, tail, flags);
        }
    }
    if (flags.fail_command != 0xffffffffu) {
        record_failure(p.status, flags.fail_command);
    }
    if (p.reduce == nullptr) {
        return;
    }
    // abs-max: block reduction, one atomic per CTA, last CTA publishes
    __shared__ uint32_t block_max;
    if (threadIdx.x == 0) block_max = 0u;
    __syncthreads();
    const uint32_t warp_max = __reduce_max_sync(0xffffffffu, flags.max_bits);
    if ((threadIdx.x & 31u) == 0u && warp_max != 0u) atomicMax(&block_max, warp_max);
    __syncthreads();
    if (threadIdx.x == 0) {
        if (block_max != 0u) atomicMax(&p.reduce->max_bits, block_max);
        __threadfence();
        const uint32_t finished = atomicAdd(&p.reduce->done_ctas, 1u);
        if (finished == gridDim.x - 1u) {
            __threadfence();
            const uint32_t result = atomicExch(&p.reduce->max_bits, 0u);
            atomicExch(&p.reduce->done_ctas, 0u);
            if (!run_failed(p.status)) {
                *static_cast<uint32_t *>(p.absmax_out) = result;
            }
        }
    }
}

}  // namespace
}  // namespace m3c

extern "C" int m3c_launch_ew(const m3c_ew_params *params, void *stream)
{
    static int sm_count = 0;
    if (sm_count == 0) {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device);
        if (sm_count <= 0) sm_count = 148;
    }
    const uint64_t blocks_needed = (params->count / m3c::VEC + m3c::THREADS - 1) / m3c::THREADS;
    // enough resident CTAs to cover HBM latency, a multiple of the SM count
    const uint64_t cap = static_cast<uint64_t>(sm_count) * 8u;
    uint64_t grid = blocks_needed < cap ? blocks_needed : cap;
    if (grid == 0) grid = 1;  // empty tensors still run the reduction epilogue
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (params->count >= (1ull << 32)) {
        m3c::ew_kernel<true><<<static_cast<unsigned>(grid), m3c::THREADS, 0, s>>>(*params);
    } else {
        m3c::ew_kernel<false><<<static_cast<unsigned>(grid), m3c::THREADS, 0, s>>>(*params);
    }
    return static_cast<int>(cudaGetLastError());
}
