// Fused element-wise engine (sm_100a).
//
// One launch evaluates a straight-line program of micro-operations over the
// flat index space of one output shape.  Every thread handles blocks of
// VEC = 4 consecutive elements in a grid-stride loop:
//   1. load each operand for the block (a 16-byte or 8-byte vector when the
//      operand runs in output order or is a broadcast row vector, one element
//      when the block reads a single broadcast element, per-element strided
//      gathers otherwise, or an immediate for folded scalar constants),
//   2. run the ops on 32-bit register words,
//   3. store the outputs (vector stores; outputs are contiguous).
//
// Two program forms share this code:
//   * fixed programs -- the fusion patterns of the benchmark configurations
//     and the single operators -- are template parameter packs of encoded
//     ops: every opcode, register index and dtype is a compile-time
//     constant, the dispatch folds away, and each thread keeps UNROLL blocks
//     of loads in flight;
//   * any other program runs the same ops from the kernel parameters through
//     warp-uniform switches (the register file stays in registers because
//     every switch arm names a constant register).
// The host picks the fixed instantiation whose ops equal the planned ones.
//
// Arithmetic follows the reference CPU executors statement by statement with
// F32 rounding per statement (explicit _rn intrinsics; the library is also
// compiled with --fmad=false):
//   ADD/MUL       src/m3_op_execute_basic.c:61-77
//   GATED_SILU    src/m3_op_execute_basic.c:104-122
//   SNAKE1D       src/m3_op_execute_basic.c:183-215
//   TANH          src/m3_op_execute_basic.c:217-230
//   CAST/COPY     src/m3_op_execute_basic.c:11-59
//   clamp         src/m3_waveform.c:360-380

#include <cuda_runtime.h>

#include <cstdint>
#include <initializer_list>
#include <type_traits>
#include <utility>

#include "m3c_device.cuh"
#include "m3c_kernels.h"
#include "m3c_bulk.cuh"

namespace m3c {
namespace {

constexpr int VEC = 4;
constexpr int THREADS = 512;
constexpr int REGS = M3C_EW_MAX_REGS;

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

// Byte offset of element f for index spaces of 2^32 elements or more: plain
// 64-bit division, kept out of line (it is large and rare).
__device__ __noinline__ int64_t wide_offset(const m3c_operand &op, uint64_t f)
{
    int64_t offset = 0;
    uint64_t q = f;
    for (int d = 0; d < op.ndim; ++d) {
        const uint64_t next = q / op.size[d];
        offset += static_cast<int64_t>(q - next * op.size[d]) * op.stride[d];
        q = next;
    }
    return offset;
}

// Byte offset of element f of a strided/broadcast operand.
template <bool WIDE>
__device__ __forceinline__ int64_t operand_offset(const m3c_operand &op, uint64_t f)
{
    int64_t offset = 0;
    if (WIDE) {
        offset = wide_offset(op, f);
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

__device__ __forceinline__ void unpack_vector(const unsigned char *at, int dtype, uint32_t (&out)[VEC])
{
    if (dtype_bytes(dtype) == 4) {
        const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(at));
        out[0] = v.x;
        out[1] = v.y;
        out[2] = v.z;
        out[3] = v.w;
    } else {
        const uint2 v = __ldcs(reinterpret_cast<const uint2 *>(at));
        out[0] = v.x & 0xffffu;
        out[1] = v.x >> 16;
        out[2] = v.y & 0xffffu;
        out[3] = v.y >> 16;
    }
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
        unpack_vector(static_cast<const unsigned char *>(op.base) +
                          f * static_cast<uint64_t>(dtype_bytes(op.dtype)),
                      op.dtype, out);
        break;
    case M3C_V_VECTOR: {
        // broadcast rows are re-read by every row of the output: keep them
        // cacheable (plain loads)
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

// ------------------------------------------------ compile-time signatures
//
// A fixed program may also fix how its operands are addressed and how its
// outputs are stored, so that loads and stores compile to straight-line code
// with no class, dtype or register dispatch.  Operand i is described by byte
// i of an operand signature: vclass | dtype << 3 | (ndim - 1) << 5 (ndim only
// for the classes that compute offsets); 0xff leaves the operand to the
// run-time switch.  An output signature holds the output count in bits 0-3
// and, for output o, byte o + 1 = register | dtype << 3 | raw << 5; 0 leaves
// the outputs to run time.

constexpr uint64_t ANY_OPERANDS = ~0ull;

constexpr uint32_t operand_byte(int vclass, int dtype, int ndim)
{
    return static_cast<uint32_t>(vclass) | (static_cast<uint32_t>(dtype) << 3) |
           (static_cast<uint32_t>(vclass == M3C_V_CONTIG || vclass == M3C_V_IMM ? 0 : ndim - 1) << 5);
}

constexpr uint32_t output_byte(int reg, int dtype, int raw)
{
    return static_cast<uint32_t>(reg) | (static_cast<uint32_t>(dtype) << 3) | (static_cast<uint32_t>(raw) << 5);
}

// Byte offset of element f through the first NDIM dimensions (narrow index).
template <int NDIM>
__device__ __forceinline__ int64_t operand_offset_c(const m3c_operand &op, uint32_t f)
{
    int64_t offset = 0;
    uint32_t q = f;
#pragma unroll
    for (int d = 0; d < NDIM; ++d) {
        const uint32_t next = fastdiv(q, op.fdiv[d]);
        offset += static_cast<int64_t>(q - next * static_cast<uint32_t>(op.size[d])) * op.stride[d];
        q = next;
    }
    return offset;
}

template <uint32_t SIG>
__device__ __forceinline__ void load_block_c(const m3c_operand &op, uint64_t f, uint32_t (&out)[VEC])
{
    constexpr int CLS = SIG & 7u;
    constexpr int DT = (SIG >> 3) & 3u;
    constexpr int NDIM = static_cast<int>((SIG >> 5) & 7u) + 1;
    constexpr int EB = DT == M3C_F16 || DT == M3C_BF16 ? 2 : 4;
    const unsigned char *base = static_cast<const unsigned char *>(op.base);
    if constexpr (CLS == M3C_V_IMM) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) out[j] = op.imm_bits;
    } else if constexpr (CLS == M3C_V_CONTIG || CLS == M3C_V_VECTOR) {
        const unsigned char *at = CLS == M3C_V_CONTIG
                                      ? base + f * static_cast<uint64_t>(EB)
                                      : base + operand_offset_c<NDIM>(op, static_cast<uint32_t>(f));
        if constexpr (EB == 4) {
            // broadcast rows are re-read by every output row: keep them
            // cacheable; streamed operands bypass with __ldcs
            const uint4 v = CLS == M3C_V_CONTIG ? __ldcs(reinterpret_cast<const uint4 *>(at))
                                                : *reinterpret_cast<const uint4 *>(at);
            out[0] = v.x;
            out[1] = v.y;
            out[2] = v.z;
            out[3] = v.w;
        } else {
            const uint2 v = CLS == M3C_V_CONTIG ? __ldcs(reinterpret_cast<const uint2 *>(at))
                                                : *reinterpret_cast<const uint2 *>(at);
            out[0] = v.x & 0xffffu;
            out[1] = v.x >> 16;
            out[2] = v.y & 0xffffu;
            out[3] = v.y >> 16;
        }
    } else if constexpr (CLS == M3C_V_UNIFORM) {
        const unsigned char *at = base + operand_offset_c<NDIM>(op, static_cast<uint32_t>(f));
        const uint32_t w = EB == 2 ? *reinterpret_cast<const uint16_t *>(at) : *reinterpret_cast<const uint32_t *>(at);
#pragma unroll
        for (int j = 0; j < VEC; ++j) out[j] = w;
    } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const unsigned char *at = base + operand_offset_c<NDIM>(op, static_cast<uint32_t>(f + j));
            out[j] = EB == 2 ? *reinterpret_cast<const uint16_t *>(at) : *reinterpret_cast<const uint32_t *>(at);
        }
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

// Round four F32 results to `rdtype` (the reference stores each statement in
// its dtype) into register words.
__device__ __forceinline__ void round_words(int rdtype, float (&f)[VEC], uint32_t (&d)[VEC])
{
    round_values<VEC>(rdtype, f);
#pragma unroll
    for (int j = 0; j < VEC; ++j) d[j] = as_bits(f[j]);
}

struct Flags {
    uint32_t fail_command;
    uint32_t max_bits;
    // the snake's 1 / (alpha + eps) for the last alpha this thread saw: a
    // channel spans many blocks, so the division runs once per channel change
    uint32_t snake_alpha = 0u;
    float snake_inverse = 0.0f;
    bool snake_known = false;
    // the word of the program's first broadcast-per-block operand (a
    // channel's alpha) and the element range [lo, hi) it covers: blocks in
    // the range reuse it instead of dividing the index again
    uint32_t uniform_lo = 0u;
    uint32_t uniform_hi = 0u;
    uint32_t uniform_word = 0u;
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
    case M3C_OP_ADD: {
        float f[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) f[j] = __fadd_rn(as_float(a[j]), as_float(b[j]));
        round_words(rdt, f, d);
        break;
    }
    case M3C_OP_MUL: {
        float f[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) f[j] = __fmul_rn(as_float(a[j]), as_float(b[j]));
        round_words(rdt, f, d);
        break;
    }
    case M3C_OP_GSILU: {
        // src/m3_op_execute_basic.c:113-117: the activation g / (1 + e^-g)
        // is stored in the gate's dtype before the product
        float f[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const float gate = as_float(a[j]);
            f[j] = __fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate)));
        }
        round_values<VEC>(op.aux, f);
#pragma unroll
        for (int j = 0; j < VEC; ++j) f[j] = __fmul_rn(f[j], as_float(b[j]));
        round_words(rdt, f, d);
        break;
    }
    case M3C_OP_SNAKE:
        if (b[0] == b[1] && b[1] == b[2] && b[2] == b[3]) {
            // one channel per block (the common case): the reciprocal of
            // (alpha + eps) is the same statement for all four elements
            const float alpha = as_float(b[0]);
            if (!flags.snake_known || b[0] != flags.snake_alpha) {
                flags.snake_known = true;
                flags.snake_alpha = b[0];
                flags.snake_inverse = __fdiv_rn(1.0f, __fadd_rn(alpha, 0x1.12e0bep-30f));
            }
            const float inverse = flags.snake_inverse;
            float angle[VEC];
#pragma unroll
            for (int j = 0; j < VEC; ++j) angle[j] = __fmul_rn(alpha, as_float(a[j]));
            const float largest =
                fmaxf(fmaxf(fabsf(angle[0]), fabsf(angle[1])), fmaxf(fabsf(angle[2]), fabsf(angle[3])));
            if (largest <= SIN_SQUARED_LIMIT) {  // false for NaN
                // the square of the sine straight from sin_squared (a few F32
                // ulps, far inside the activation's 0x1p-19 tolerance), two
                // elements per packed instruction; inverse * sq and x + that
                // stay scalar, separately rounded as the reference's
                // statements are
#pragma unroll
                for (int j = 0; j < VEC; j += 2) {
                    float sq[2];
                    sin_squared2(angle[j], angle[j + 1], sq[0], sq[1]);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        d[j + h] = as_bits(__fadd_rn(as_float(a[j + h]), __fmul_rn(inverse, sq[h])));
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < VEC; ++j) {
                    const float sine = sinf(angle[j]);
                    d[j] = as_bits(__fadd_rn(as_float(a[j]), __fmul_rn(inverse, __fmul_rn(sine, sine))));
                }
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
    case M3C_OP_ROUND: {
        float f[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) f[j] = as_float(a[j]);
        round_words(rdt, f, d);
        break;
    }
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
    case M3C_OP_WIDEN: {
        if (op.aux == M3C_F16 || op.aux == M3C_BF16) {
            const uint32_t pairs[2] = {(a[0] & 0xffffu) | (a[1] << 16), (a[2] & 0xffffu) | (a[3] << 16)};
            float f[VEC];
            widen_pairs<2>(op.aux, pairs, f);
#pragma unroll
            for (int j = 0; j < VEC; ++j) d[j] = as_bits(f[j]);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) d[j] = a[j];
        }
        break;
    }
    case M3C_OP_CLAMP:
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            // Decided on the bit pattern alone, so no float instruction can
            // touch the value: for a non-NaN float, v > 1 exactly when the
            // sign is clear and the magnitude bits exceed those of 1.0 (up to
            // +inf), and v < -1 when the sign is set likewise.  NaN payloads,
            // signed zeros and subnormals pass through unchanged.
            const uint32_t w = a[j];
            const uint32_t magnitude = w & 0x7fffffffu;
            const bool beyond = magnitude > 0x3f800000u && magnitude <= 0x7f800000u;
            d[j] = beyond ? ((w & 0x80000000u) | 0x3f800000u) : w;
        }
        break;
    case M3C_OP_MOV:
#pragma unroll
        for (int j = 0; j < VEC; ++j) d[j] = a[j];
        break;
    case M3C_OP_ABSMAX:
        // the largest magnitude bit pattern; a NaN's pattern exceeds every
        // other, so one test of the running maximum finds NaN inputs (at the
        // end of the kernel: a failed abs-max publishes nothing)
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            flags.max_bits = max(flags.max_bits, j < valid ? (a[j] & 0x7fffffffu) : 0u);
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
        uint32_t h[2];
        if (out.raw) {
            h[0] = (w[0] & 0xffffu) | (w[1] << 16);
            h[1] = (w[2] & 0xffffu) | (w[3] << 16);
        } else {
            const float f[VEC] = {as_float(w[0]), as_float(w[1]), as_float(w[2]), as_float(w[3])};
            narrow_pairs<2>(out.dtype, f, h);
        }
        __stcs(reinterpret_cast<uint2 *>(p + f * 2u), make_uint2(h[0], h[1]));
    } else {
        __stcs(reinterpret_cast<uint4 *>(p + f * 4u), make_uint4(w[0], w[1], w[2], w[3]));
    }
}

template <uint32_t SIG>
__device__ __forceinline__ void store_block_c(const m3c_ew_out &out, uint64_t f, const uint32_t (&w)[VEC])
{
    constexpr int DT = (SIG >> 3) & 3u;
    constexpr bool RAW = ((SIG >> 5) & 1u) != 0u;
    unsigned char *p = static_cast<unsigned char *>(out.base);
    if constexpr (DT == M3C_F16 || DT == M3C_BF16) {
        uint32_t h[2];
        if constexpr (RAW) {
            h[0] = (w[0] & 0xffffu) | (w[1] << 16);
            h[1] = (w[2] & 0xffffu) | (w[3] << 16);
        } else {
            const float f[VEC] = {as_float(w[0]), as_float(w[1]), as_float(w[2]), as_float(w[3])};
            narrow_pairs<2>(DT, f, h);
        }
        __stcs(reinterpret_cast<uint2 *>(p + f * 2u), make_uint2(h[0], h[1]));
    } else {
        __stcs(reinterpret_cast<uint4 *>(p + f * 4u), make_uint4(w[0], w[1], w[2], w[3]));
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

// ----------------------------------------------------------- programs

// Encoded op of a fixed program: code | dst << 8 | a << 16 | b << 24 |
// rdtype << 32 | aux << 40.
constexpr uint64_t op_code(int code, int dst, int a, int b, int rdtype, int aux)
{
    return static_cast<uint64_t>(code) | (static_cast<uint64_t>(dst) << 8) |
           (static_cast<uint64_t>(a) << 16) | (static_cast<uint64_t>(b) << 24) |
           (static_cast<uint64_t>(static_cast<uint8_t>(rdtype)) << 32) |
           (static_cast<uint64_t>(static_cast<uint8_t>(aux)) << 40);
}

__device__ __forceinline__ m3c_ew_op decode(uint64_t e, uint16_t command)
{
    m3c_ew_op op;
    op.code = static_cast<uint8_t>(e & 0xffu);
    op.dst = static_cast<uint8_t>((e >> 8) & 0xffu);
    op.a = static_cast<uint8_t>((e >> 16) & 0xffu);
    op.b = static_cast<uint8_t>((e >> 24) & 0xffu);
    op.rdtype = static_cast<int8_t>((e >> 32) & 0xffu);
    op.aux = static_cast<int8_t>((e >> 40) & 0xffu);
    op.command = command;
    return op;
}

template <int NOPERANDS, uint64_t OPSIG, uint64_t OUTSIG, uint64_t... OPS>
struct Fixed {
    static constexpr bool custom_loop = false;
    static constexpr int unroll = 4;  // blocks per thread and pass, loads all in flight
    // no transcendental op (SNAKE1D's sin^2, TANH, F32 gated SiLU): the
    // program leaves issue slots to spare for a shared-memory pipeline
    __host__ __device__ static constexpr bool light()
    {
        return ((static_cast<int>(OPS & 0xffu) != M3C_OP_SNAKE && static_cast<int>(OPS & 0xffu) != M3C_OP_TANH &&
                 static_cast<int>(OPS & 0xffu) != M3C_OP_GSILU) &&
                ...);
    }
    static constexpr int operands = NOPERANDS;
    static constexpr uint64_t opsig = OPSIG;
    static constexpr uint64_t outsig = OUTSIG;
    __device__ __forceinline__ static void run(const m3c_ew_params &p, RegisterFile &rf, int valid,
                                               Flags &flags)
    {
        int k = 0;
        ((run_op(decode(OPS, p.ops[k].command), rf, valid, flags), ++k), ...);
    }
};

struct Dynamic {
    static constexpr bool custom_loop = false;
    static constexpr int unroll = 1;
    static constexpr int operands = M3C_EW_MAX_OPERANDS;
    static constexpr uint64_t opsig = ANY_OPERANDS;
    static constexpr uint64_t outsig = 0u;
    __device__ __forceinline__ static void run(const m3c_ew_params &p, RegisterFile &rf, int valid,
                                               Flags &flags)
    {
        for (int k = 0; k < p.n_ops; ++k) {
            run_op(p.ops[k], rf, valid, flags);
        }
    }
};

template <bool WIDE, int MAX_OPERANDS>
__device__ __forceinline__ void load_operands(const m3c_ew_params &p, uint64_t f, int valid,
                                              RegisterFile &rf)
{
#pragma unroll
    for (int i = 0; i < MAX_OPERANDS && i < REGS; ++i) {
        if (i < p.n_operands) {
            if (valid == VEC) {
                load_block<WIDE>(p.operands[i], f, rf.w[i]);
            } else {
                load_partial<WIDE>(p.operands[i], f, valid, rf.w[i]);
            }
        }
    }
}

// Which operands a load pass covers: the streamed ones (read once, from
// HBM: their loads go out first for all of a thread's blocks), the cached
// ones (broadcast rows and elements, immediates: loaded just before their
// block runs, so they hold no registers while the streamed loads are in
// flight), or all of them.
enum LoadPass { LOAD_STREAMED, LOAD_CACHED, LOAD_ALL };

// The index of a signature's first operand broadcast per block through at
// least two dimensions (a per-channel scalar), or -1.
__host__ __device__ constexpr int first_uniform(uint64_t opsig, int operands)
{
    for (int i = 0; i < operands && i < 8; ++i) {
        const uint32_t sig = static_cast<uint32_t>((opsig >> (8 * i)) & 0xffu);
        if (sig != 0xffu && (sig & 7u) == M3C_V_UNIFORM && ((sig >> 5) & 7u) >= 1u) return i;
    }
    return -1;
}

// A per-block broadcast operand through the thread's cache: its word holds
// for the whole run of elements that share the index of dimension 1 when
// dimension 0 (innermost) is broadcast (stride 0).
template <uint32_t SIG>
__device__ __forceinline__ void load_uniform_cached(const m3c_operand &op, uint64_t f, uint32_t (&out)[VEC],
                                                    Flags &cache)
{
    const uint32_t g = static_cast<uint32_t>(f);
    if (g - cache.uniform_lo >= cache.uniform_hi - cache.uniform_lo) {
        load_block_c<SIG>(op, f, out);
        cache.uniform_word = out[0];
        if (op.stride[0] == 0) {
            const uint32_t lo = fastdiv(g, op.fdiv[0]) * static_cast<uint32_t>(op.size[0]);
            cache.uniform_lo = lo;
            cache.uniform_hi = lo + static_cast<uint32_t>(op.size[0]);
        } else {
            cache.uniform_lo = cache.uniform_hi = 0u;
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) out[j] = cache.uniform_word;
}

template <class Prog, int I, LoadPass PASS>
__device__ __forceinline__ void load_operand_full(const m3c_ew_params &p, uint64_t f, RegisterFile &rf,
                                                  Flags *cache)
{
    constexpr uint32_t sig = static_cast<uint32_t>((Prog::opsig >> (8 * I)) & 0xffu);
    constexpr bool streamed = sig != 0xffu && (sig & 7u) == M3C_V_CONTIG;
    if constexpr (PASS == LOAD_ALL || (PASS == LOAD_STREAMED) == streamed) {
        if constexpr (sig == 0xffu) {
            load_block<false>(p.operands[I], f, rf.w[I]);
        } else if constexpr (I == first_uniform(Prog::opsig, Prog::operands)) {
            if (cache != nullptr) {
                load_uniform_cached<sig>(p.operands[I], f, rf.w[I], *cache);
            } else {
                load_block_c<sig>(p.operands[I], f, rf.w[I]);
            }
        } else {
            load_block_c<sig>(p.operands[I], f, rf.w[I]);
        }
    }
}

template <class Prog, LoadPass PASS, int... I>
__device__ __forceinline__ void load_full(const m3c_ew_params &p, uint64_t f, RegisterFile &rf, Flags *cache,
                                          std::integer_sequence<int, I...>)
{
    (load_operand_full<Prog, I, PASS>(p, f, rf, cache), ...);
}

// The operands of a full block that a load pass covers: through the
// program's signature when it has one (narrow index only), else the
// run-time dispatch (which loads everything in the first pass).  `cache`
// (the thread's Flags, or null) keeps the first per-block broadcast operand.
template <class Prog, bool WIDE, LoadPass PASS>
__device__ __forceinline__ void load_block_all(const m3c_ew_params &p, uint64_t f, RegisterFile &rf,
                                               Flags *cache = nullptr)
{
    if constexpr (Prog::opsig != ANY_OPERANDS && !WIDE) {
        load_full<Prog, PASS>(p, f, rf, cache, std::make_integer_sequence<int, Prog::operands>{});
    } else if constexpr (PASS != LOAD_CACHED) {
        load_operands<WIDE, Prog::operands>(p, f, VEC, rf);
    }
}

__device__ __forceinline__ void store_outputs(const m3c_ew_params &p, uint64_t f, int valid,
                                              const RegisterFile &rf)
{
#pragma unroll
    for (int o = 0; o < M3C_EW_MAX_OUTPUTS; ++o) {
        if (o < p.n_outputs) {
            uint32_t w[VEC];
            reg_get(rf, p.outputs[o].reg, w);
            if (valid == VEC && !p.outputs[o].scalar_only) {
                store_block(p.outputs[o], f, w);
            } else {
                store_partial(p.outputs[o], f, valid, w);
            }
        }
    }
}

template <class Prog, int O>
__device__ __forceinline__ void store_output_full(const m3c_ew_params &p, uint64_t f, const RegisterFile &rf)
{
    constexpr uint32_t sig = static_cast<uint32_t>((Prog::outsig >> (8 * (O + 1))) & 0xffu);
    constexpr int REG = sig & 7u;
    if (!p.outputs[O].scalar_only) {
        store_block_c<sig>(p.outputs[O], f, rf.w[REG]);
    } else {
        store_partial(p.outputs[O], f, VEC, rf.w[REG]);
    }
}

template <class Prog, int... O>
__device__ __forceinline__ void store_full(const m3c_ew_params &p, uint64_t f, const RegisterFile &rf,
                                           std::integer_sequence<int, O...>)
{
    (store_output_full<Prog, O>(p, f, rf), ...);
}

// All outputs of a full block.
template <class Prog>
__device__ __forceinline__ void store_block_all(const m3c_ew_params &p, uint64_t f, const RegisterFile &rf)
{
    if constexpr (Prog::outsig != 0u) {
        store_full<Prog>(p, f, rf, std::make_integer_sequence<int, static_cast<int>(Prog::outsig & 0xfu)>{});
    } else {
        store_outputs(p, f, VEC, rf);
    }
}

// The grid-stride loop of a program over all blocks, then the tail.
template <class Prog, bool WIDE>
__device__ __forceinline__ void program_loop(const m3c_ew_params &p, Flags &flags)
{
    constexpr int U = Prog::unroll;
    {
        const uint64_t blocks = p.count / VEC;
        const uint64_t threads = static_cast<uint64_t>(gridDim.x) * THREADS;
        for (uint64_t v = static_cast<uint64_t>(blockIdx.x) * THREADS + threadIdx.x; v < blocks;
             v += threads * U) {
            // the streamed loads of the U blocks first, so they are in
            // flight together
            RegisterFile rf[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint64_t b = v + static_cast<uint64_t>(u) * threads;
                if (b < blocks) load_block_all<Prog, WIDE, LOAD_STREAMED>(p, b * VEC, rf[u]);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint64_t b = v + static_cast<uint64_t>(u) * threads;
                if (b < blocks) {
                    load_block_all<Prog, WIDE, LOAD_CACHED>(p, b * VEC, rf[u], &flags);
                    Prog::run(p, rf[u], VEC, flags);
                    store_block_all<Prog>(p, b * VEC, rf[u]);
                }
            }
        }
        const int tail = static_cast<int>(p.count - blocks * VEC);
        if (tail != 0 && blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
            RegisterFile rf;
            load_operands<WIDE, Prog::operands>(p, blocks * VEC, tail, rf);
            Prog::run(p, rf, tail, flags);
            store_outputs(p, blocks * VEC, tail, rf);
        }
    }
}

// Gated SiLU of 16-bit gate and up with a 16-bit result (the benchmark's
// MLP activation), as its own loop over packed words: two 8-byte loads and
// one 8-byte store per four elements.  One test of the raw words finds the
// blocks whose gates and ups are all finite with |gate| <= 80; those take a
// straight path: hardware widening, the approximate exponential and quotient
// (a few F32 ulps, far below the result's half ulp), the activation rounded
// to 16 bits as the reference stores it, the product, and one packed
// narrowing, with no NaN to carry.  Every other block, the tail and outputs
// stored element by element run the table's op-by-op program.
template <int DT, uint64_t OPSIG, uint64_t OUTSIG, uint64_t... OPS>
struct Gsilu16 {
    using Generic = Fixed<2, OPSIG, OUTSIG, OPS...>;
    static_assert(!Generic::custom_loop && Generic::unroll > 0, "the fallback is the table's own program");
    static constexpr bool custom_loop = true;
    static constexpr int unroll = 4;
    static constexpr int operands = Generic::operands;
    static constexpr uint64_t opsig = Generic::opsig;
    static constexpr uint64_t outsig = Generic::outsig;

    __device__ __forceinline__ static void run(const m3c_ew_params &p, RegisterFile &rf, int valid, Flags &flags)
    {
        Generic::run(p, rf, valid, flags);
    }

    __device__ __forceinline__ static void widen2(uint32_t w, float &lo, float &hi)
    {
        if constexpr (DT == M3C_F16) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
            lo = f.x;
            hi = f.y;
        } else {
            lo = as_float(w << 16);
            hi = as_float(w & 0xffff0000u);
        }
    }

    // packed 16-bit product, rounded once
    __device__ __forceinline__ static uint32_t mul2(uint32_t a, uint32_t b)
    {
        if constexpr (DT == M3C_F16) {
            const __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
            return *reinterpret_cast<const uint32_t *>(&r);
        } else {
            const __nv_bfloat162 r =
                __hmul2(*reinterpret_cast<const __nv_bfloat162 *>(&a), *reinterpret_cast<const __nv_bfloat162 *>(&b));
            return *reinterpret_cast<const uint32_t *>(&r);
        }
    }

    __device__ __forceinline__ static uint32_t narrow2(float lo, float hi)
    {
        if constexpr (DT == M3C_F16) {
            const __half2 h = __floats2half2_rn(lo, hi);
            return *reinterpret_cast<const uint32_t *>(&h);
        } else {
            const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
            return *reinterpret_cast<const uint32_t *>(&h);
        }
    }

    // g / (1 + e^-g) for two gates, exp_moderate and div_approx with their
    // F32 statements two lanes per packed instruction (the same bits)
    __device__ __forceinline__ static void silu_pair(float g0, float g1, float &s0, float &s1)
    {
        const uint64_t g = f2_pack(g0, g1);
        const uint64_t d = f2_mul(g, f2_splat(-1.0f));                    // -g, exact
        const uint64_t h = f2_mul(d, f2_splat(0x1.715476p+0f));
        uint64_t c = f2_fma(h, f2_splat(-0x1.62e000p-1f), d);
        c = f2_fma(h, f2_splat(-0x1.0bfbe8p-15f), c);
        float h0, h1, r0, r1;
        f2_unpack(h, h0, h1);
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(h0));
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(h1));
        const uint64_t r = f2_pack(r0, r1);
        const uint64_t den = f2_add(f2_splat(1.0f), f2_fma(r, c, r));  // 1 + e^-g
        float b0, b1, y0, y1;
        f2_unpack(den, b0, b1);
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(b0));
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y1) : "f"(b1));
        const uint64_t y = f2_pack(y0, y1);
        const uint64_t q0 = f2_mul(g, y);
        const uint64_t rem = f2_fma(q0, f2_mul(den, f2_splat(-1.0f)), g);
        f2_unpack(f2_fma(rem, y, q0), s0, s1);
    }

    // four results (two packed words) from four gates and ups
    __device__ __forceinline__ static uint2 block(const m3c_ew_params &p, uint2 gw, uint2 uw, Flags &flags)
    {
        // a half is infinite or NaN when its magnitude reaches the all-ones
        // exponent, i.e. when magnitude + (0x8000 - that) carries into bit 15
        constexpr uint32_t CARRY = DT == M3C_F16 ? 0x04000400u : 0x00800080u;
        const uint32_t special = (((gw.x & 0x7fff7fffu) + CARRY) | ((gw.y & 0x7fff7fffu) + CARRY) |
                                  ((uw.x & 0x7fff7fffu) + CARRY) | ((uw.y & 0x7fff7fffu) + CARRY)) &
                                 0x80008000u;
        float g[VEC];
        float u[VEC];
        widen2(gw.x, g[0], g[1]);
        widen2(gw.y, g[2], g[3]);
        widen2(uw.x, u[0], u[1]);
        widen2(uw.y, u[2], u[3]);
        const float largest = fmaxf(fmaxf(fabsf(g[0]), fabsf(g[1])), fmaxf(fabsf(g[2]), fabsf(g[3])));
        if (special == 0u && largest <= 80.0f) {
            // src/m3_op_execute_basic.c:113-117: the activation is stored in
            // the gate's dtype before the product.  The product of two 16-bit
            // values is exact in F32, so the reference's F32 product rounded
            // to 16 bits is one packed 16-bit multiply (RN of the exact
            // product; no NaN or infinity reaches this path)
            float s[VEC];
#pragma unroll
            for (int j = 0; j < VEC; j += 2) silu_pair(g[j], g[j + 1], s[j], s[j + 1]);
            return make_uint2(mul2(narrow2(s[0], s[1]), uw.x), mul2(narrow2(s[2], s[3]), uw.y));
        }
        RegisterFile rf;
        rf.w[0][0] = gw.x & 0xffffu;
        rf.w[0][1] = gw.x >> 16;
        rf.w[0][2] = gw.y & 0xffffu;
        rf.w[0][3] = gw.y >> 16;
        rf.w[1][0] = uw.x & 0xffffu;
        rf.w[1][1] = uw.x >> 16;
        rf.w[1][2] = uw.y & 0xffffu;
        rf.w[1][3] = uw.y >> 16;
        Generic::run(p, rf, VEC, flags);
        const float f[VEC] = {as_float(rf.w[0][0]), as_float(rf.w[0][1]), as_float(rf.w[0][2]),
                              as_float(rf.w[0][3])};
        uint32_t h[2];
        narrow_pairs<2>(DT, f, h);  // the reference's NaN rules
        return make_uint2(h[0], h[1]);
    }

    __device__ __forceinline__ static void loop(const m3c_ew_params &p, Flags &flags)
    {
        if (p.outputs[0].scalar_only) {
            program_loop<Gsilu16, false>(p, flags);
            return;
        }
        constexpr int U = unroll;
        const uint2 *gate = static_cast<const uint2 *>(p.operands[0].base);
        const uint2 *up = static_cast<const uint2 *>(p.operands[1].base);
        uint2 *out = static_cast<uint2 *>(p.outputs[0].base);
        const uint64_t blocks = p.count / VEC;
        const uint64_t threads = static_cast<uint64_t>(gridDim.x) * THREADS;
        for (uint64_t v = static_cast<uint64_t>(blockIdx.x) * THREADS + threadIdx.x; v < blocks;
             v += threads * U) {
            uint2 gw[U];
            uint2 uw[U];
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const uint64_t b = v + static_cast<uint64_t>(k) * threads;
                if (b < blocks) {
                    gw[k] = __ldcs(gate + b);
                    uw[k] = __ldcs(up + b);
                }
            }
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const uint64_t b = v + static_cast<uint64_t>(k) * threads;
                if (b < blocks) __stcs(out + b, block(p, gw[k], uw[k], flags));
            }
        }
        const int tail = static_cast<int>(p.count - blocks * VEC);
        if (tail != 0 && blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
            RegisterFile rf;
            load_operands<false, operands>(p, blocks * VEC, tail, rf);
            Generic::run(p, rf, tail, flags);
            store_outputs(p, blocks * VEC, tail, rf);
        }
    }
};

// The same gated SiLU fed by 1-D TMA, for contiguous 16-byte-aligned
// operands: two CTAs per SM; in each, warp 0's first lane copies tiles of
// gate and up (TILE elements each, cp.async.bulk with mbarrier completion,
// no tensor map, no multicast) into a ring of STAGES shared-memory stages;
// warps 1-15 take 16 bytes of both per tile (8 elements each), compute them
// with Gsilu16's block, and stream the results to HBM.  2 * STAGES tiles
// (210 KB) are in flight per SM without holding registers, where the
// register-fed loop keeps about 64 KB in flight.
template <int DT, uint64_t OPSIG, uint64_t OUTSIG, uint64_t... OPS>
struct Gsilu16Bulk {
    using Base = Gsilu16<DT, OPSIG, OUTSIG, OPS...>;
    using Generic = typename Base::Generic;
    static constexpr bool custom_loop = true;
    static constexpr bool cta_pipeline = true;  // the CTA's threads wait on one another
    static constexpr int operands = Base::operands;
    static constexpr int CONSUMERS = THREADS - 32;
    static constexpr int TILE = CONSUMERS * 8;       // elements per tile
    static constexpr int TILE_BYTES = TILE * 2;      // per operand
    static constexpr int STAGES = 7;
    static constexpr int SMEM = STAGES * 2 * TILE_BYTES + STAGES * 16;
    static constexpr int CTAS_PER_SM = 2;

    __device__ __forceinline__ static void run(const m3c_ew_params &p, RegisterFile &rf, int valid, Flags &flags)
    {
        Generic::run(p, rf, valid, flags);
    }

    __device__ static void loop(const m3c_ew_params &p, Flags &flags)
    {
        extern __shared__ __align__(16) unsigned char bulk_smem[];
        uint64_t *full = reinterpret_cast<uint64_t *>(bulk_smem + STAGES * 2 * TILE_BYTES);
        uint64_t *empty = full + STAGES;
        const uint16_t *gate = static_cast<const uint16_t *>(p.operands[0].base);
        const uint16_t *up = static_cast<const uint16_t *>(p.operands[1].base);
        uint16_t *out = static_cast<uint16_t *>(p.outputs[0].base);
        const uint32_t command = p.ops[0].command;
        const uint64_t tiles = p.count / TILE;
        const uint64_t first = tiles * blockIdx.x / gridDim.x;
        const int n = static_cast<int>(tiles * (blockIdx.x + 1) / gridDim.x - first);
        const int warp = static_cast<int>(threadIdx.x) / 32;
        const int lane = static_cast<int>(threadIdx.x) % 32;
        if (threadIdx.x == 0) {
            for (int s = 0; s < STAGES; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], CONSUMERS / 32);
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        if (warp == 0) {
            if (lane == 0) {
                int i = 0;
                for (; i < n; ++i) {
                    const int s = i % STAGES;
                    const int use = i / STAGES;
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
                        bulk_timed_out(p.status, command);
                        break;
                    }
                    mbar_expect_tx(&full[s], 2 * TILE_BYTES);
                    const uint64_t e = (first + static_cast<uint64_t>(i)) * TILE;
                    bulk_load(bulk_smem + s * 2 * TILE_BYTES, gate + e, TILE_BYTES, &full[s]);
                    bulk_load(bulk_smem + s * 2 * TILE_BYTES + TILE_BYTES, up + e, TILE_BYTES, &full[s]);
                }
                // every copy issued has landed before the CTA ends
                for (int r = i - STAGES < 0 ? 0 : i - STAGES; r < i; ++r) {
                    (void)mbar_wait(&full[r % STAGES], (r / STAGES) & 1);
                }
            }
        } else {
            // one consumer group takes every tile in order, so a consumer is
            // never a phase ahead of the producer's copies
            const int c = static_cast<int>(threadIdx.x) - 32;
            for (int i = 0; i < n; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
                    bulk_timed_out(p.status, command);
                    break;
                }
                const unsigned char *stage = bulk_smem + s * 2 * TILE_BYTES;
                const uint4 g = reinterpret_cast<const uint4 *>(stage)[c];
                const uint4 u = reinterpret_cast<const uint4 *>(stage + TILE_BYTES)[c];
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                const uint2 lo = Base::block(p, make_uint2(g.x, g.y), make_uint2(u.x, u.y), flags);
                const uint2 hi = Base::block(p, make_uint2(g.z, g.w), make_uint2(u.z, u.w), flags);
                __stcs(reinterpret_cast<uint4 *>(out + (first + static_cast<uint64_t>(i)) * TILE) + c,
                       make_uint4(lo.x, lo.y, hi.x, hi.y));
            }
        }
        if (blockIdx.x != gridDim.x - 1) return;
        // the elements after the last whole tile: the last CTA, from HBM
        const uint2 *g2 = reinterpret_cast<const uint2 *>(gate);
        const uint2 *u2 = reinterpret_cast<const uint2 *>(up);
        uint2 *o2 = reinterpret_cast<uint2 *>(out);
        const uint64_t blocks = p.count / VEC;
        for (uint64_t b = tiles * (TILE / VEC) + threadIdx.x; b < blocks; b += THREADS) {
            __stcs(o2 + b, Base::block(p, __ldcs(g2 + b), __ldcs(u2 + b), flags));
        }
        const int tail = static_cast<int>(p.count - blocks * VEC);
        if (tail != 0 && threadIdx.x == 0) {
            RegisterFile rf;
            load_operands<false, operands>(p, blocks * VEC, tail, rf);
            Generic::run(p, rf, tail, flags);
            store_outputs(p, blocks * VEC, tail, rf);
        }
    }
};

// Any signature program fed by 1-D TMA: its contiguous (streamed) operands
// arrive in shared memory by cp.async.bulk (global -> shared, mbarrier
// completion, no tensor map, no multicast), one tile of TILE elements per
// operand per stage, issued by one thread of warp 0; warps 1-15 each take
// BPT blocks of the tile from shared memory, load the cached operands
// (broadcast rows and elements, immediates) as the register-fed loop does,
// run the program and store from registers.  Two CTAs per SM, up to about
// 200 KB of streamed loads in flight per SM without holding registers.
// (the table also asks programs that keep the register-fed loop for their
// bulk geometry, leaving members of those instantiations unused)
#pragma nv_diag_suppress 177
template <class Prog>
struct BulkFixed {
    static constexpr bool custom_loop = true;
    static constexpr bool cta_pipeline = true;
    static constexpr int operands = Prog::operands;
    static constexpr int CONSUMERS = THREADS - 32;
    static constexpr int BPT = 2;                          // blocks per consumer per tile
    static constexpr int TILE_BLOCKS = CONSUMERS * BPT;
    static constexpr int TILE = TILE_BLOCKS * VEC;         // elements per tile
    static constexpr int CTAS_PER_SM = 2;
    static constexpr int BUDGET = 104 * 1024;              // stage bytes per CTA

    __host__ __device__ static constexpr uint32_t sig_of(int i)
    {
        return static_cast<uint32_t>((Prog::opsig >> (8 * i)) & 0xffu);
    }
    __host__ __device__ static constexpr bool streamed_of(int i)
    {
        return sig_of(i) != 0xffu && (sig_of(i) & 7u) == M3C_V_CONTIG;
    }
    __host__ __device__ static constexpr int eb_of(int i)
    {
        return ((sig_of(i) >> 3) & 3u) == M3C_F16 || ((sig_of(i) >> 3) & 3u) == M3C_BF16 ? 2 : 4;
    }
    // byte offset of operand i's tile in a stage (streamed operands only)
    __host__ __device__ static constexpr int offset_of(int i)
    {
        int o = 0;
        for (int j = 0; j < i; ++j) o += streamed_of(j) ? TILE * eb_of(j) : 0;
        return o;
    }
    static constexpr int STAGE_BYTES = offset_of(Prog::operands);
    __host__ __device__ static constexpr int streamed_count()
    {
        int n = 0;
        for (int j = 0; j < Prog::operands; ++j) n += streamed_of(j) ? 1 : 0;
        return n;
    }
    static constexpr int STREAMED = streamed_count();
    static constexpr int STAGES = STAGE_BYTES == 0 ? 0
                                  : BUDGET / STAGE_BYTES > 8 ? 8
                                  : BUDGET / STAGE_BYTES < 2 ? 2
                                                             : BUDGET / STAGE_BYTES;
    static constexpr int SMEM = STAGES * STAGE_BYTES + STAGES * 16;

    __device__ __forceinline__ static void run(const m3c_ew_params &p, RegisterFile &rf, int valid, Flags &flags)
    {
        Prog::run(p, rf, valid, flags);
    }

    template <int I>
    __device__ __forceinline__ static void issue(const m3c_ew_params &p, unsigned char *stage, uint64_t e,
                                                 uint64_t *bar)
    {
        if constexpr (streamed_of(I)) {
            constexpr int EB = eb_of(I);
            bulk_load(stage + offset_of(I), static_cast<const unsigned char *>(p.operands[I].base) + e * EB,
                      TILE * EB, bar);
        }
    }
    template <int... I>
    __device__ __forceinline__ static void issue_all(const m3c_ew_params &p, unsigned char *stage, uint64_t e,
                                                     uint64_t *bar, std::integer_sequence<int, I...>)
    {
        (issue<I>(p, stage, e, bar), ...);
    }

    template <int I>
    __device__ __forceinline__ static void take(const unsigned char *stage, int blk, RegisterFile &rf)
    {
        if constexpr (streamed_of(I)) {
            if constexpr (eb_of(I) == 4) {
                const uint4 v = reinterpret_cast<const uint4 *>(stage + offset_of(I))[blk];
                rf.w[I][0] = v.x;
                rf.w[I][1] = v.y;
                rf.w[I][2] = v.z;
                rf.w[I][3] = v.w;
            } else {
                const uint2 v = reinterpret_cast<const uint2 *>(stage + offset_of(I))[blk];
                rf.w[I][0] = v.x & 0xffffu;
                rf.w[I][1] = v.x >> 16;
                rf.w[I][2] = v.y & 0xffffu;
                rf.w[I][3] = v.y >> 16;
            }
        }
    }
    template <int... I>
    __device__ __forceinline__ static void take_all(const unsigned char *stage, int blk, RegisterFile &rf,
                                                    std::integer_sequence<int, I...>)
    {
        (take<I>(stage, blk, rf), ...);
    }

    __device__ static void loop(const m3c_ew_params &p, Flags &flags)
    {
        extern __shared__ __align__(16) unsigned char bulk_smem[];
        uint64_t *full = reinterpret_cast<uint64_t *>(bulk_smem + STAGES * STAGE_BYTES);
        uint64_t *empty = full + STAGES;
        constexpr auto ops = std::make_integer_sequence<int, Prog::operands>{};
        const uint32_t command = p.ops[0].command;
        const uint64_t tiles = p.count / TILE;
        const uint64_t first = tiles * blockIdx.x / gridDim.x;
        const int n = static_cast<int>(tiles * (blockIdx.x + 1) / gridDim.x - first);
        const int warp = static_cast<int>(threadIdx.x) / 32;
        const int lane = static_cast<int>(threadIdx.x) % 32;
        if (threadIdx.x == 0) {
            for (int s = 0; s < STAGES; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], CONSUMERS / 32);
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        if (warp == 0) {
            if (lane == 0) {
                int i = 0;
                for (; i < n; ++i) {
                    const int s = i % STAGES;
                    const int use = i / STAGES;
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
                        bulk_timed_out(p.status, command);
                        break;
                    }
                    mbar_expect_tx(&full[s], STAGE_BYTES);
                    issue_all(p, bulk_smem + s * STAGE_BYTES, (first + static_cast<uint64_t>(i)) * TILE, &full[s],
                              ops);
                }
                // every copy issued has landed before the CTA ends
                for (int r = i - STAGES < 0 ? 0 : i - STAGES; r < i; ++r) {
                    (void)mbar_wait(&full[r % STAGES], (r / STAGES) & 1);
                }
            }
        } else {
            // one consumer group takes every tile in order, so a consumer is
            // never a phase ahead of the producer's copies
            const int c = static_cast<int>(threadIdx.x) - 32;
            for (int i = 0; i < n; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
                    bulk_timed_out(p.status, command);
                    break;
                }
                const unsigned char *stage = bulk_smem + s * STAGE_BYTES;
                RegisterFile rf[BPT];
#pragma unroll
                for (int u = 0; u < BPT; ++u) take_all(stage, c + u * CONSUMERS, rf[u], ops);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
                for (int u = 0; u < BPT; ++u) {
                    const uint64_t f =
                        ((first + static_cast<uint64_t>(i)) * TILE_BLOCKS + static_cast<uint64_t>(c + u * CONSUMERS)) *
                        VEC;
                    load_block_all<Prog, false, LOAD_CACHED>(p, f, rf[u]);
                    Prog::run(p, rf[u], VEC, flags);
                    store_block_all<Prog>(p, f, rf[u]);
                }
            }
        }
        if (blockIdx.x != gridDim.x - 1) return;
        // the blocks after the last whole tile, then the partial block: the
        // last CTA, from HBM
        const uint64_t blocks = p.count / VEC;
        for (uint64_t b = tiles * TILE_BLOCKS + threadIdx.x; b < blocks; b += THREADS) {
            RegisterFile rf;
            load_block_all<Prog, false, LOAD_ALL>(p, b * VEC, rf);
            Prog::run(p, rf, VEC, flags);
            store_block_all<Prog>(p, b * VEC, rf);
        }
        const int tail = static_cast<int>(p.count - blocks * VEC);
        if (tail != 0 && threadIdx.x == 0) {
            RegisterFile rf;
            load_operands<false, operands>(p, blocks * VEC, tail, rf);
            Prog::run(p, rf, tail, flags);
            store_outputs(p, blocks * VEC, tail, rf);
        }
    }
};
#pragma nv_diag_default 177

// Programs whose threads wait on one another (a shared-memory pipeline)
// declare cta_pipeline; their CTA decides once whether to skip.
template <class Prog, class = void>
struct UniformSkip {
    static constexpr bool value = false;
};
template <class Prog>
struct UniformSkip<Prog, std::void_t<decltype(Prog::cta_pipeline)>> {
    static constexpr bool value = Prog::cta_pipeline;
};

template <class Prog, bool WIDE>
__global__ void __launch_bounds__(THREADS) ew_kernel(const __grid_constant__ m3c_ew_params p)
{
    bool skip;
    if constexpr (UniformSkip<Prog>::value) {
        // one reading for the whole CTA: its threads meet at barriers
        __shared__ int skip_cta;
        if (threadIdx.x == 0) skip_cta = failed_before(p.status, p.skip_before) ? 1 : 0;
        __syncthreads();
        skip = skip_cta != 0;
    } else {
        skip = failed_before(p.status, p.skip_before);
    }
    if (p.first_of_run && !skip && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    Flags flags{0xffffffffu, 0u};
    if (!skip) {
        if constexpr (Prog::custom_loop) {
            Prog::loop(p, flags);
        } else {
            program_loop<Prog, WIDE>(p, flags);
        }
    }
    if (p.reduce != nullptr && flags.max_bits > 0x7f800000u) {
        flags.fail_command = min(flags.fail_command, p.absmax_command);  // NaN input
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
            if (p.absmax_publish_always || !failed_before(p.status, p.absmax_command + 1u)) {
                *static_cast<uint32_t *>(p.absmax_out) = result;
            }
        }
    }
}

// ------------------------------------------------------ program table
//
// The encodings are what the planner (m3c_plan.c) emits for these graphs.

#define E op_code
#define OPS_MUL_ADD_F32 E(M3C_OP_MUL, 0, 0, 1, 0, 0), E(M3C_OP_ADD, 0, 0, 2, 0, 0)
// the same chain merged by the backend plug-in, which keeps the temporary
#define OPS_MUL_ADD_F32_KEEP E(M3C_OP_MUL, 3, 0, 1, 0, 0), E(M3C_OP_ADD, 4, 3, 2, 0, 0)
#define OPS_CFG_EULER_BF16                                                           \
    E(M3C_OP_MUL, 1, 0, 1, 0, 0), E(M3C_OP_ADD, 1, 2, 1, 0, 0), E(M3C_OP_MUL, 1, 1, 3, 0, 0), \
        E(M3C_OP_ADD, 0, 0, 1, 0, 0), E(M3C_OP_MUL, 0, 0, 4, 0, 0), E(M3C_OP_ADD, 0, 5, 0, 0, 0), \
        E(M3C_OP_ROUND, 1, 0, 0, 2, 0)
#define OPS_GSILU_F32 E(M3C_OP_GSILU, 0, 0, 1, 0, 0)
#define OPS_GSILU_F16 \
    E(M3C_OP_WIDEN, 0, 0, 0, 0, 1), E(M3C_OP_WIDEN, 1, 1, 1, 0, 1), E(M3C_OP_GSILU, 0, 0, 1, 1, 1)
#define OPS_GSILU_BF16 \
    E(M3C_OP_WIDEN, 0, 0, 0, 0, 2), E(M3C_OP_WIDEN, 1, 1, 1, 0, 2), E(M3C_OP_GSILU, 0, 0, 1, 2, 2)
#define OPS_SNAKE_ABSMAX_CLAMP \
    E(M3C_OP_SNAKE, 0, 0, 1, 0, 0), E(M3C_OP_ABSMAX, 0, 0, 0, 0, 0), E(M3C_OP_CLAMP, 0, 0, 0, 0, 0)
#define OPS_SNAKE E(M3C_OP_SNAKE, 0, 0, 1, 0, 0)
#define OPS_TANH E(M3C_OP_TANH, 0, 0, 0, 0, 0)
#define OPS_ADD_F32 E(M3C_OP_ADD, 0, 0, 1, 0, 0)
#define OPS_MUL_F32 E(M3C_OP_MUL, 0, 0, 1, 0, 0)
#define OPS_ADD_F16 \
    E(M3C_OP_WIDEN, 0, 0, 0, 0, 1), E(M3C_OP_WIDEN, 1, 1, 1, 0, 1), E(M3C_OP_ADD, 0, 0, 1, 1, 0)
#define OPS_MUL_F16 \
    E(M3C_OP_WIDEN, 0, 0, 0, 0, 1), E(M3C_OP_WIDEN, 1, 1, 1, 0, 1), E(M3C_OP_MUL, 0, 0, 1, 1, 0)
#define OPS_ADD_BF16 \
    E(M3C_OP_WIDEN, 0, 0, 0, 0, 2), E(M3C_OP_WIDEN, 1, 1, 1, 0, 2), E(M3C_OP_ADD, 0, 0, 1, 2, 0)
#define OPS_MUL_BF16 \
    E(M3C_OP_WIDEN, 0, 0, 0, 0, 2), E(M3C_OP_WIDEN, 1, 1, 1, 0, 2), E(M3C_OP_MUL, 0, 0, 1, 2, 0)
#define OPS_CAST_F32_F16 E(M3C_OP_ROUND, 0, 0, 0, 1, 0)
#define OPS_CAST_F32_BF16 E(M3C_OP_ROUND, 0, 0, 0, 2, 0)
#define OPS_CAST_F16_F32 E(M3C_OP_WIDEN, 0, 0, 0, 0, 1), E(M3C_OP_ROUND, 0, 0, 0, 0, 0)
#define OPS_CAST_BF16_F32 E(M3C_OP_WIDEN, 0, 0, 0, 0, 2), E(M3C_OP_ROUND, 0, 0, 0, 0, 0)
#define OPS_CLAMP E(M3C_OP_CLAMP, 0, 0, 0, 0, 0)
#define OPS_MOV E(M3C_OP_MOV, 0, 0, 0, 0, 0)

constexpr uint64_t operand_sig(std::initializer_list<uint32_t> bytes)
{
    uint64_t sig = 0;
    int i = 0;
    for (uint32_t byte : bytes) sig |= static_cast<uint64_t>(byte) << (8 * i++);
    return sig;
}

constexpr uint64_t output_sig(std::initializer_list<uint32_t> bytes)
{
    uint64_t sig = bytes.size();
    int i = 1;
    for (uint32_t byte : bytes) sig |= static_cast<uint64_t>(byte) << (8 * i++);
    return sig;
}

#define C32 operand_byte(M3C_V_CONTIG, M3C_F32, 1)
#define C16 operand_byte(M3C_V_CONTIG, M3C_F16, 1)
#define CB16 operand_byte(M3C_V_CONTIG, M3C_BF16, 1)
#define I32C operand_byte(M3C_V_IMM, M3C_F32, 1)
#define V32_1 operand_byte(M3C_V_VECTOR, M3C_F32, 1)
#define U32_2 operand_byte(M3C_V_UNIFORM, M3C_F32, 2)
#define OUT(reg, dtype) output_byte(reg, dtype, 0)
#define RAWOUT(reg, dtype) output_byte(reg, dtype, 1)

// X(operand count, operand signature, output signature, ops).  Entries with
// signatures come first: they are the addressing patterns of the benchmark
// graphs and of plain same-shape operators; the signature-free entries
// behind them take any addressing.
#define M3C_PROGRAMS(X)                                                                 \
    X(3, (operand_sig({C32, V32_1, V32_1})), (output_sig({OUT(0, M3C_F32)})), OPS_MUL_ADD_F32) \
    X(3, (operand_sig({C32, V32_1, V32_1})), (output_sig({OUT(3, M3C_F32), OUT(4, M3C_F32)})),   \
      OPS_MUL_ADD_F32_KEEP)                                                             \
    X(6, (operand_sig({C32, I32C, C32, I32C, I32C, C32})),                                \
      (output_sig({OUT(0, M3C_F32), OUT(1, M3C_BF16)})), OPS_CFG_EULER_BF16)             \
    X(2, (operand_sig({C32, C32})), (output_sig({OUT(0, M3C_F32)})), OPS_GSILU_F32)        \
    X(2, (operand_sig({C32, U32_2})), (output_sig({OUT(0, M3C_F32)})), OPS_SNAKE_ABSMAX_CLAMP) \
    X(2, (operand_sig({C32, U32_2})), (output_sig({OUT(0, M3C_F32)})), OPS_SNAKE)          \
    X(1, (operand_sig({C32})), (output_sig({OUT(0, M3C_F32)})), OPS_TANH)                  \
    X(2, (operand_sig({C32, C32})), (output_sig({OUT(0, M3C_F32)})), OPS_ADD_F32)          \
    X(2, (operand_sig({C32, C32})), (output_sig({OUT(0, M3C_F32)})), OPS_MUL_F32)          \
    X(2, (operand_sig({C32, V32_1})), (output_sig({OUT(0, M3C_F32)})), OPS_ADD_F32)        \
    X(2, (operand_sig({C32, V32_1})), (output_sig({OUT(0, M3C_F32)})), OPS_MUL_F32)        \
    X(2, (operand_sig({C32, I32C})), (output_sig({OUT(0, M3C_F32)})), OPS_ADD_F32)         \
    X(2, (operand_sig({C32, I32C})), (output_sig({OUT(0, M3C_F32)})), OPS_MUL_F32)         \
    X(2, (operand_sig({C16, C16})), (output_sig({OUT(0, M3C_F16)})), OPS_ADD_F16)          \
    X(2, (operand_sig({C16, C16})), (output_sig({OUT(0, M3C_F16)})), OPS_MUL_F16)          \
    X(2, (operand_sig({CB16, CB16})), (output_sig({OUT(0, M3C_BF16)})), OPS_ADD_BF16)      \
    X(2, (operand_sig({CB16, CB16})), (output_sig({OUT(0, M3C_BF16)})), OPS_MUL_BF16)      \
    X(1, (operand_sig({C32})), (output_sig({OUT(0, M3C_F16)})), OPS_CAST_F32_F16)          \
    X(1, (operand_sig({C32})), (output_sig({OUT(0, M3C_BF16)})), OPS_CAST_F32_BF16)        \
    X(1, (operand_sig({C16})), (output_sig({OUT(0, M3C_F32)})), OPS_CAST_F16_F32)          \
    X(1, (operand_sig({CB16})), (output_sig({OUT(0, M3C_F32)})), OPS_CAST_BF16_F32)        \
    X(1, (operand_sig({C32})), (output_sig({OUT(0, M3C_F32)})), OPS_CLAMP)                 \
    X(1, (operand_sig({C32})), (output_sig({OUT(0, M3C_F32)})), OPS_MOV)                   \
    X(1, (operand_sig({C16})), (output_sig({RAWOUT(0, M3C_F16)})), OPS_MOV)                \
    X(1, (operand_sig({CB16})), (output_sig({RAWOUT(0, M3C_BF16)})), OPS_MOV)              \
    X(3, ANY_OPERANDS, 0u, OPS_MUL_ADD_F32)                                                          \
    X(6, ANY_OPERANDS, 0u, OPS_CFG_EULER_BF16)                                                       \
    X(2, ANY_OPERANDS, 0u, OPS_GSILU_F32)                                                            \
    X(2, ANY_OPERANDS, 0u, OPS_GSILU_F16)                                                            \
    X(2, ANY_OPERANDS, 0u, OPS_GSILU_BF16)                                                           \
    X(2, ANY_OPERANDS, 0u, OPS_SNAKE_ABSMAX_CLAMP)                                                   \
    X(2, ANY_OPERANDS, 0u, OPS_SNAKE)                                                                \
    X(1, ANY_OPERANDS, 0u, OPS_TANH)                                                                 \
    X(2, ANY_OPERANDS, 0u, OPS_ADD_F32)                                                              \
    X(2, ANY_OPERANDS, 0u, OPS_MUL_F32)                                                              \
    X(2, ANY_OPERANDS, 0u, OPS_ADD_F16)                                                              \
    X(2, ANY_OPERANDS, 0u, OPS_MUL_F16)                                                              \
    X(2, ANY_OPERANDS, 0u, OPS_ADD_BF16)                                                             \
    X(2, ANY_OPERANDS, 0u, OPS_MUL_BF16)                                                             \
    X(1, ANY_OPERANDS, 0u, OPS_CAST_F32_F16)                                                         \
    X(1, ANY_OPERANDS, 0u, OPS_CAST_F32_BF16)                                                        \
    X(1, ANY_OPERANDS, 0u, OPS_CAST_F16_F32)                                                         \
    X(1, ANY_OPERANDS, 0u, OPS_CAST_BF16_F32)                                                        \
    X(1, ANY_OPERANDS, 0u, OPS_CLAMP)                                                                \
    X(1, ANY_OPERANDS, 0u, OPS_MOV)

typedef void (*ew_fn)(m3c_ew_params);

// The TMA-fed kernel of a signature program with a streamed operand, else
// none.
// Measured on the benchmark programs (one B200, L2 flushed): the bulk path
// speeds up light programs with one streamed operand (x * c + b: 16.2 ->
// 14.9 us) and slows the snake (2.27 -> 2.44 ms: its arithmetic needs the
// issue slots the stage handoff takes) and the three-operand CFG chain
// (134 -> 138 us per 30 runs, whose carried runs are mostly L2 hits).
template <class Prog>
ew_fn bulk_kernel_of()
{
    if constexpr (Prog::opsig != ANY_OPERANDS) {
        if constexpr (Prog::light() && BulkFixed<Prog>::STAGE_BYTES != 0 &&
                      BulkFixed<Prog>::STREAMED <= 2) {
            return ew_kernel<BulkFixed<Prog>, false>;
        }
    }
    return nullptr;
}

// Its shared memory, tile and CTAs per SM (0 where it has none).
template <class Prog>
constexpr int bulk_smem_of()
{
    if constexpr (Prog::opsig != ANY_OPERANDS) return BulkFixed<Prog>::SMEM;
    return 0;
}

template <class Prog>
constexpr int bulk_tile_of()
{
    if constexpr (Prog::opsig != ANY_OPERANDS) return BulkFixed<Prog>::TILE;
    return 0;
}

template <class Prog>
constexpr int bulk_ctas_of()
{
    if constexpr (Prog::opsig != ANY_OPERANDS) return BulkFixed<Prog>::CTAS_PER_SM;
    return 0;
}

struct Entry {
    int operands;
    uint64_t opsig;
    uint64_t outsig;
    int count;
    uint64_t ops[M3C_EW_MAX_OPS];
    ew_fn kernel;
    int unroll;  // blocks of VEC elements per thread and pass
    ew_fn bulk;  // the TMA-fed variant (nullptr: none)
    int bulk_smem;
    int bulk_tile;  // elements per TMA tile
    int bulk_ctas;  // resident CTAs per SM
};

constexpr int count_of(std::initializer_list<uint64_t> ops)
{
    return static_cast<int>(ops.size());
}

// Fixed programs cover index spaces below 2^32 elements; larger ones use the
// generic kernel's 64-bit addressing.
#define M3C_ENTRY(NOPERANDS, OPSIG, OUTSIG, OPS)                                                  \
    {NOPERANDS, OPSIG, OUTSIG, count_of({OPS}), {OPS}, ew_kernel<Fixed<NOPERANDS, OPSIG, OUTSIG, OPS>, false>, \
     Fixed<NOPERANDS, OPSIG, OUTSIG, OPS>::unroll, bulk_kernel_of<Fixed<NOPERANDS, OPSIG, OUTSIG, OPS>>(),       \
     bulk_smem_of<Fixed<NOPERANDS, OPSIG, OUTSIG, OPS>>(), bulk_tile_of<Fixed<NOPERANDS, OPSIG, OUTSIG, OPS>>(),     \
     bulk_ctas_of<Fixed<NOPERANDS, OPSIG, OUTSIG, OPS>>()},

// the dedicated 16-bit gated SiLU programs, matched like the table's own
#define M3C_GSILU16_ENTRY(DT, OPSIG, OUTSIG, OPS)                                                  \
    {2, OPSIG, OUTSIG, count_of({OPS}), {OPS}, ew_kernel<Gsilu16<DT, OPSIG, OUTSIG, OPS>, false>,    \
     Gsilu16<DT, OPSIG, OUTSIG, OPS>::unroll, ew_kernel<Gsilu16Bulk<DT, OPSIG, OUTSIG, OPS>, false>,     \
     Gsilu16Bulk<DT, OPSIG, OUTSIG, OPS>::SMEM, Gsilu16Bulk<DT, OPSIG, OUTSIG, OPS>::TILE,                 \
     Gsilu16Bulk<DT, OPSIG, OUTSIG, OPS>::CTAS_PER_SM},

const Entry PROGRAMS[] = {
    M3C_GSILU16_ENTRY(M3C_F16, (operand_sig({C16, C16})), (output_sig({OUT(0, M3C_F16)})), OPS_GSILU_F16)
    M3C_GSILU16_ENTRY(M3C_BF16, (operand_sig({CB16, CB16})), (output_sig({OUT(0, M3C_BF16)})), OPS_GSILU_BF16)
    M3C_PROGRAMS(M3C_ENTRY)};

#undef M3C_GSILU16_ENTRY

#undef M3C_ENTRY
#undef E
#undef C32
#undef C16
#undef CB16
#undef I32C
#undef V32_1
#undef U32_2
#undef OUT
#undef RAWOUT

uint64_t encode_op(const m3c_ew_op &op)
{
    return op_code(op.code, op.dst, op.a, op.b, op.rdtype, op.aux);
}

// Signature byte of a run-time operand; 0xfe (never a table value) where the
// operand's addressing has no signature form.
uint32_t runtime_operand_byte(const m3c_operand &op)
{
    const bool offsets = op.vclass != M3C_V_CONTIG && op.vclass != M3C_V_IMM;
    if (offsets && (op.ndim < 1 || op.ndim > 8)) return 0xfeu;
    if (op.dtype < 0 || op.dtype > 3) return 0xfeu;
    return operand_byte(op.vclass, op.dtype, offsets ? op.ndim : 1);
}

bool signature_matches(const Entry &entry, const m3c_ew_params &p)
{
    if (entry.opsig != ANY_OPERANDS) {
        for (int i = 0; i < p.n_operands; ++i) {
            if (((entry.opsig >> (8 * i)) & 0xffu) != runtime_operand_byte(p.operands[i])) return false;
        }
    }
    if (entry.outsig != 0u) {
        if (static_cast<int>(entry.outsig & 0xfu) != p.n_outputs) return false;
        for (int o = 0; o < p.n_outputs; ++o) {
            const m3c_ew_out &out = p.outputs[o];
            if (out.reg < 0 || out.reg > 7 || out.dtype < 0 || out.dtype > 3) return false;
            if (((entry.outsig >> (8 * (o + 1))) & 0xffu) != output_byte(out.reg, out.dtype, out.raw ? 1 : 0)) {
                return false;
            }
        }
    }
    return true;
}

const Entry *find_program(const m3c_ew_params &p)
{
    for (const Entry &entry : PROGRAMS) {
        if (entry.count != p.n_ops || entry.operands != p.n_operands) continue;
        bool same = true;
        for (int k = 0; k < p.n_ops && same; ++k) same = encode_op(p.ops[k]) == entry.ops[k];
        if (same && signature_matches(entry, p)) return &entry;
    }
    return nullptr;
}

int sm_count()
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

}  // namespace
}  // namespace m3c

extern "C" int m3c_ew_choose(const m3c_ew_params *params, m3c_ew_choice *choice)
{
    const bool wide = params->count >= (1ull << 32);
    const m3c::Entry *entry = wide ? nullptr : m3c::find_program(*params);
    m3c::ew_fn kernel = entry != nullptr
                            ? entry->kernel
                            : (wide ? m3c::ew_kernel<m3c::Dynamic, true> : m3c::ew_kernel<m3c::Dynamic, false>);
    int per_sm = 0;
    const cudaError_t code =
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, m3c::THREADS, 0);
    if (code != cudaSuccess || per_sm < 1) {
        (void)cudaGetLastError();
        per_sm = 1;
    }
    const uint64_t blocks_needed = (params->count / m3c::VEC + m3c::THREADS - 1) / m3c::THREADS;
    uint64_t grid;
    if (params->reduce != nullptr) {
        // a reduction ends with one atomic per CTA: a persistent grid, every
        // resident CTA of every SM and no more
        const uint64_t cap = static_cast<uint64_t>(m3c::sm_count()) * static_cast<uint64_t>(per_sm);
        grid = blocks_needed < cap ? blocks_needed : cap;
    } else {
        // otherwise one pass per thread (`unroll` blocks of VEC elements
        // each): every load of the launch is issued as soon as its CTA is
        // resident and the block scheduler keeps the SMs full to the end
        const uint64_t unroll = entry != nullptr ? static_cast<uint64_t>(entry->unroll) : 2u;
        grid = (blocks_needed + unroll - 1) / unroll;
        if (grid > 0x7fffffffull) grid = 0x7fffffffull;
    }
    if (grid == 0) grid = 1;  // empty tensors still run the reduction epilogue
    choice->kernel = reinterpret_cast<void *>(kernel);
    choice->grid = grid;
    choice->bulk = nullptr;
    choice->bulk_grid = 0;
    choice->bulk_smem = 0;
    choice->reserved = 0;
    if (entry != nullptr && entry->bulk != nullptr) {
        // at least one whole tile per CTA, every resident CTA and no more
        const uint64_t resident = static_cast<uint64_t>(m3c::sm_count()) * static_cast<uint64_t>(entry->bulk_ctas);
        uint64_t tiles = params->count / static_cast<uint64_t>(entry->bulk_tile);
        if (tiles > resident) tiles = resident;
        if (tiles >= 1u && cudaFuncSetAttribute(entry->bulk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                entry->bulk_smem) == cudaSuccess) {
            choice->bulk = reinterpret_cast<void *>(entry->bulk);
            choice->bulk_grid = tiles;
            choice->bulk_smem = static_cast<uint32_t>(entry->bulk_smem);
        } else {
            (void)cudaGetLastError();
        }
    }
    return 0;
}

extern "C" int m3c_launch_ew_chosen(const m3c_ew_choice *choice, const m3c_ew_params *params,
                                    void *stream)
{
    if (choice->bulk != nullptr) {
        // bulk copies of the streamed operands and 16-byte stores need
        // 16-byte-aligned bases
        uintptr_t bits = 0u;
        bool vector_stores = true;
        for (int i = 0; i < params->n_operands && i < M3C_EW_MAX_OPERANDS; ++i) {
            if (params->operands[i].vclass == M3C_V_CONTIG) bits |= reinterpret_cast<uintptr_t>(params->operands[i].base);
        }
        for (int o = 0; o < params->n_outputs && o < M3C_EW_MAX_OUTPUTS; ++o) {
            bits |= reinterpret_cast<uintptr_t>(params->outputs[o].base);
            vector_stores = vector_stores && !params->outputs[o].scalar_only;
        }
        if ((bits & 15u) == 0u && vector_stores) {
            const m3c::ew_fn bulk = reinterpret_cast<m3c::ew_fn>(choice->bulk);
            bulk<<<static_cast<unsigned>(choice->bulk_grid), m3c::THREADS, choice->bulk_smem,
                   static_cast<cudaStream_t>(stream)>>>(*params);
            return static_cast<int>(cudaGetLastError());
        }
    }
    const m3c::ew_fn kernel = reinterpret_cast<m3c::ew_fn>(choice->kernel);
    kernel<<<static_cast<unsigned>(choice->grid), m3c::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        *params);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int m3c_launch_ew(const m3c_ew_params *params, void *stream)
{
    m3c_ew_choice choice;
    m3c_ew_choose(params, &choice);
    return m3c_launch_ew_chosen(&choice, params, stream);
}
