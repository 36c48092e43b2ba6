/* CPU restatement of m3.c's tensor hot path -- TEST INFRASTRUCTURE ONLY.
 * See m3_oracle.h.  Citations are reference file:line (taconotsandwich/m3.c). */

#include "m3_oracle.h"

#include <math.h>
#include <stdbool.h>
#include <string.h>

/* ---------------------------------------------------------------- codecs */

static uint32_t bits_of(float value)
{
    uint32_t bits;
    memcpy(&bits, &value, sizeof(bits));
    return bits;
}

static float float_of(uint32_t bits)
{
    float value;
    memcpy(&value, &bits, sizeof(value));
    return value;
}

/* src/m3_op_numeric.c:27-53: exact widening, subnormals included. */
float m3o_f16_to_f32(uint16_t half)
{
    uint32_t sign = ((uint32_t)half & 0x8000U) << 16;
    uint32_t exponent = ((uint32_t)half >> 10) & 0x1fU;
    uint32_t fraction = (uint32_t)half & 0x3ffU;

    if (exponent == 0U) {
        /* zero or subnormal: fraction * 2^-24 is exact in F32 */
        float magnitude = (float)fraction * 0x1p-24F;
        return float_of(sign | bits_of(magnitude));
    }
    if (exponent == 0x1fU) {
        return float_of(sign | 0x7f800000U | (fraction << 13));
    }
    return float_of(sign | ((exponent + 112U) << 23) | (fraction << 13));
}

/* src/m3_op_numeric.c:55-112: round to nearest even, overflow to infinity,
 * gradual underflow, NaN keeps its top payload bits with the quiet bit set
 * (an all-zero kept payload becomes 1). */
uint16_t m3o_f32_to_f16(float value)
{
    uint32_t bits = bits_of(value);
    uint32_t sign = (bits >> 16) & 0x8000U;
    uint32_t biased = (bits >> 23) & 0xffU;
    uint32_t fraction = bits & 0x7fffffU;
    int exponent = (int)biased - 127;

    if (biased == 0xffU) {
        uint32_t payload;

        if (fraction == 0U) {
            return (uint16_t)(sign | 0x7c00U);
        }
        payload = fraction >> 13;
        return (uint16_t)(sign | 0x7e00U | payload | (payload == 0U));
    }
    if (exponent > 15) {
        return (uint16_t)(sign | 0x7c00U);
    }
    if (exponent >= -14) {
        /* the carry of the rounding increment propagates into the exponent */
        uint32_t half = ((uint32_t)(exponent + 15) << 10) | (fraction >> 13);
        uint32_t rest = fraction & 0x1fffU;

        if (rest > 0x1000U || (rest == 0x1000U && (half & 1U) != 0U)) {
            half += 1U;
        }
        if (half >= 0x7c00U) {
            return (uint16_t)(sign | 0x7c00U);
        }
        return (uint16_t)(sign | half);
    }
    if (exponent >= -25) {
        uint32_t significand = 0x800000U | fraction;
        unsigned shift = (unsigned)(-exponent - 1);
        uint32_t kept = significand >> shift;
        uint32_t rest = significand & ((1U << shift) - 1U);
        uint32_t halfway = 1U << (shift - 1U);

        if (rest > halfway || (rest == halfway && (kept & 1U) != 0U)) {
            kept += 1U;
        }
        return (uint16_t)(sign | kept);
    }
    return (uint16_t)sign;
}

/* src/m3_op_numeric.c:114-117 */
float m3o_bf16_to_f32(uint16_t value)
{
    return float_of((uint32_t)value << 16);
}

/* src/m3_op_numeric.c:119-130: NaN -> upper half with the quiet bit forced;
 * otherwise round to nearest even on the upper half. */
uint16_t m3o_f32_to_bf16(float value)
{
    uint32_t bits = bits_of(value);

    if ((bits & 0x7f800000U) == 0x7f800000U && (bits & 0x7fffffU) != 0U) {
        return (uint16_t)((bits >> 16) | 0x40U);
    }
    return (uint16_t)((bits + 0x7fffU + ((bits >> 16) & 1U)) >> 16);
}

/* src/m3_op_numeric.c:210-222 */
float m3o_round_to_dtype(int32_t dtype, float value)
{
    switch (dtype) {
    case M3O_F32:
        return value;
    case M3O_F16:
        return m3o_f16_to_f32(m3o_f32_to_f16(value));
    case M3O_BF16:
        return m3o_bf16_to_f32(m3o_f32_to_bf16(value));
    default:
        return NAN;
    }
}

/* ---------------------------------------------------------- addressing */

static uint64_t element_count(const m3o_view *view)
{
    uint64_t count = 1U;
    int axis;

    for (axis = 0; axis < view->rank; ++axis) {
        count *= view->shape[axis];
    }
    return count;
}

/* src/m3_op_numeric.c:132-148: row-major unravel of a flat index. */
static uint64_t flat_offset(const m3o_view *view, uint64_t flat)
{
    uint64_t offset = view->byte_offset;
    int axis;

    for (axis = view->rank - 1; axis >= 0; --axis) {
        uint64_t extent = view->shape[axis];

        offset += (flat % extent) * view->byte_strides[axis];
        flat /= extent;
    }
    return offset;
}

/* src/m3_op_numeric.c:150-174: right-aligned broadcast; input axes of size one
 * and missing leading axes do not advance. */
static uint64_t broadcast_offset(const m3o_view *input, const m3o_view *output,
                                 uint64_t flat)
{
    uint64_t offset = input->byte_offset;
    int lead = output->rank - input->rank;
    int axis;

    for (axis = output->rank - 1; axis >= 0; --axis) {
        uint64_t extent = output->shape[axis];
        uint64_t coordinate = flat % extent;
        int input_axis = axis - lead;

        flat /= extent;
        if (input_axis >= 0 && input->shape[input_axis] != 1U) {
            offset += coordinate * input->byte_strides[input_axis];
        }
    }
    return offset;
}

static const uint8_t *cbytes(const m3o_view *view)
{
    return (const uint8_t *)view->base;
}

static uint8_t *wbytes(m3o_view *view)
{
    return (uint8_t *)view->base;
}

static int32_t load_i32(const m3o_view *view, uint64_t offset)
{
    int32_t value;
    memcpy(&value, cbytes(view) + offset, sizeof(value));
    return value;
}

/* src/m3_op_numeric.c:176-199: widen any storage dtype to F32. */
static float load_float(const m3o_view *view, uint64_t offset)
{
    const uint8_t *at = cbytes(view) + offset;
    uint16_t half;
    float value;

    switch (view->dtype) {
    case M3O_F32:
        memcpy(&value, at, sizeof(value));
        return value;
    case M3O_F16:
        memcpy(&half, at, sizeof(half));
        return m3o_f16_to_f32(half);
    case M3O_BF16:
        memcpy(&half, at, sizeof(half));
        return m3o_bf16_to_f32(half);
    default:
        return (float)load_i32(view, offset);
    }
}

/* src/m3_op_numeric.c:224-251: narrow F32 to the storage dtype; I32 truncates. */
static void store_float(m3o_view *view, uint64_t offset, float value)
{
    uint8_t *at = wbytes(view) + offset;
    uint16_t half;
    int32_t integer;

    switch (view->dtype) {
    case M3O_F32:
        memcpy(at, &value, sizeof(value));
        break;
    case M3O_F16:
        half = m3o_f32_to_f16(value);
        memcpy(at, &half, sizeof(half));
        break;
    case M3O_BF16:
        half = m3o_f32_to_bf16(value);
        memcpy(at, &half, sizeof(half));
        break;
    default:
        integer = (int32_t)value;
        memcpy(at, &integer, sizeof(integer));
        break;
    }
}

static void store_i32(m3o_view *view, uint64_t offset, int32_t value)
{
    memcpy(wbytes(view) + offset, &value, sizeof(value));
}

static size_t dtype_bytes(int32_t dtype)
{
    return (dtype == M3O_F16 || dtype == M3O_BF16) ? 2U : 4U;
}

/* ------------------------------------------------------------ preflights */

/* src/m3_op_data_preflight.c:48-64 */
static bool contains_nan(const m3o_view *view)
{
    uint64_t count = element_count(view);
    uint64_t index;

    for (index = 0U; index < count; ++index) {
        if (isnan(load_float(view, flat_offset(view, index)))) {
            return true;
        }
    }
    return false;
}

/* ------------------------------------------------------------- elementwise */

/* src/m3_op_execute_basic.c:11-26 (memmove per element). */
int m3o_copy(const m3o_view *input, m3o_view *output)
{
    uint64_t count = element_count(input);
    size_t size = dtype_bytes(input->dtype);
    uint64_t index;

    for (index = 0U; index < count; ++index) {
        memmove(wbytes(output) + flat_offset(output, index),
                cbytes(input) + flat_offset(input, index), size);
    }
    return M3O_OK;
}

/* src/m3_op_execute_basic.c:28-59 with the float-to-I32 range preflight of
 * src/m3_op_data_preflight.c:8-28 run first (all-or-nothing). */
int m3o_cast(const m3o_view *input, m3o_view *output)
{
    uint64_t count = element_count(input);
    uint64_t index;

    if (input->dtype == output->dtype) {
        return m3o_copy(input, output);
    }
    if (output->dtype == M3O_I32 && input->dtype != M3O_I32) {
        for (index = 0U; index < count; ++index) {
            float value = load_float(input, flat_offset(input, index));

            if (!isfinite(value) || value < -2147483648.0F ||
                value >= 2147483648.0F) {
                return M3O_OUT_OF_RANGE;
            }
        }
    }
    for (index = 0U; index < count; ++index) {
        uint64_t from = flat_offset(input, index);
        uint64_t to = flat_offset(output, index);

        if (input->dtype == M3O_I32) {
            store_float(output, to, (float)load_i32(input, from));
        } else if (output->dtype == M3O_I32) {
            store_i32(output, to, (int32_t)load_float(input, from));
        } else {
            store_float(output, to, load_float(input, from));
        }
    }
    return M3O_OK;
}

/* src/m3_op_execute_basic.c:61-77: one F32 operation per element, rounded once
 * to F32 and once to the output dtype. */
int m3o_binary(int multiply, const m3o_view *left, const m3o_view *right,
               m3o_view *output)
{
    uint64_t count = element_count(output);
    uint64_t index;

    for (index = 0U; index < count; ++index) {
        float a = load_float(left, broadcast_offset(left, output, index));
        float b = load_float(right, broadcast_offset(right, output, index));
        float result = multiply ? a * b : a + b;

        store_float(output, flat_offset(output, index), result);
    }
    return M3O_OK;
}

/* src/m3_op_execute_basic.c:104-122: the activation is rounded to the gate's
 * dtype before the product with the up projection. */
int m3o_gated_silu(const m3o_view *gate, const m3o_view *up, m3o_view *output)
{
    uint64_t count = element_count(output);
    uint64_t index;

    for (index = 0U; index < count; ++index) {
        float g = load_float(gate, flat_offset(gate, index));
        float u = load_float(up, flat_offset(up, index));
        float denominator = 1.0F + expf(-g);
        float activation = m3o_round_to_dtype(gate->dtype, g / denominator);
        float product = activation * u;

        store_float(output, flat_offset(output, index), product);
    }
    return M3O_OK;
}

/* src/m3_op_execute_basic.c:183-194: seven F32 statements, each rounded, no
 * contraction; epsilon has the exact bits 0x3089705f. */
#pragma STDC FP_CONTRACT OFF
static float snake_value(float x, float alpha)
{
    volatile float denominator = alpha + 0x1.12e0bep-30F;
    volatile float inverse = 1.0F / denominator;
    volatile float angle = alpha * x;
    volatile float sine = sinf(angle);
    volatile float square = sine * sine;
    volatile float scaled = inverse * square;
    volatile float result = x + scaled;

    return result;
}
#pragma STDC FP_CONTRACT DEFAULT

/* src/m3_op_execute_basic.c:196-215: alpha [1,C,1] is indexed by the channel
 * (flat / T) % C of the [B,C,T] input. */
int m3o_snake1d(const m3o_view *input, const m3o_view *alpha, m3o_view *output)
{
    uint64_t length = input->shape[2];
    uint64_t channels = input->shape[1];
    uint64_t count = element_count(input);
    uint64_t index;

    for (index = 0U; index < count; ++index) {
        uint64_t channel = (index / length) % channels;
        float x = load_float(input, flat_offset(input, index));
        float a = load_float(alpha, flat_offset(alpha, channel));

        store_float(output, flat_offset(output, index), snake_value(x, a));
    }
    return M3O_OK;
}

/* src/m3_op_execute_basic.c:217-230 */
int m3o_tanh(const m3o_view *input, m3o_view *output)
{
    uint64_t count = element_count(input);
    uint64_t index;

    for (index = 0U; index < count; ++index) {
        float x = load_float(input, flat_offset(input, index));

        store_float(output, flat_offset(output, index), tanhf(x));
    }
    return M3O_OK;
}

/* ---------------------------------------------------------- row reductions */

/* src/m3_op_execute_basic.c:124-180 with the NaN preflight of
 * src/m3_op_data_preflight.c:281-284.  Pass 1: maximum and the count of +inf;
 * pass 2: left-to-right F32 sum of expf(v - max), skipped for an infinite
 * maximum; pass 3: probabilities (all -inf row -> zeros, +inf maximum -> mass
 * split equally among the +inf entries). */
int m3o_softmax(const m3o_view *input, m3o_view *output)
{
    uint64_t count = element_count(input);
    uint64_t width = input->shape[input->rank - 1];
    uint64_t rows = width == 0U ? 0U : count / width;
    uint64_t row;

    if (contains_nan(input)) {
        return M3O_OUT_OF_RANGE;
    }
    for (row = 0U; row < rows; ++row) {
        uint64_t base = row * width;
        float maximum = -INFINITY;
        float sum = 0.0F;
        uint64_t infinities = 0U;
        uint64_t column;

        for (column = 0U; column < width; ++column) {
            float v = load_float(input, flat_offset(input, base + column));

            if (v > maximum) {
                maximum = v;
            }
            infinities += v == INFINITY;
        }
        if (isfinite(maximum)) {
            for (column = 0U; column < width; ++column) {
                float v = load_float(input, flat_offset(input, base + column));

                sum += expf(v - maximum);
            }
        }
        for (column = 0U; column < width; ++column) {
            float v = load_float(input, flat_offset(input, base + column));
            float p;

            if (maximum == -INFINITY) {
                p = 0.0F;
            } else if (maximum == INFINITY) {
                p = v == INFINITY ? 1.0F / (float)infinities : 0.0F;
            } else {
                p = expf(v - maximum) / sum;
            }
            store_float(output, flat_offset(output, base + column), p);
        }
    }
    return M3O_OK;
}

/* src/m3_op_execute_sampling.c:7-12: (value, index) precedes when its value is
 * larger, or equal (so +0 == -0) with a lower index. */
static bool precedes(float value, int32_t index, float other_value,
                     int32_t other_index)
{
    return value > other_value ||
           (value == other_value && index < other_index);
}

/* src/m3_op_execute_sampling.c:42-89 (with the insertion of :14-40) and the
 * NaN preflight of src/m3_op_data_preflight.c:288-291.  K is at most 64 here;
 * the tests use no larger K. */
int m3o_top_k(const m3o_view *logits, m3o_view *values, m3o_view *indices,
              uint64_t k)
{
    uint64_t width = logits->shape[logits->rank - 1];
    uint64_t rows = width == 0U ? 0U : element_count(logits) / width;
    float best_value[64];
    int32_t best_index[64];
    uint64_t row;

    if (k == 0U || k > 64U) {
        return M3O_INVALID_ARGUMENT;
    }
    if (contains_nan(logits)) {
        return M3O_OUT_OF_RANGE;
    }
    for (row = 0U; row < rows; ++row) {
        uint64_t held = 0U;
        uint64_t column;
        uint64_t slot;

        for (column = 0U; column < width; ++column) {
            float v = load_float(logits,
                                 flat_offset(logits, row * width + column));
            int32_t i = (int32_t)column;
            uint64_t position = 0U;

            while (position < held &&
                   !precedes(v, i, best_value[position],
                             best_index[position])) {
                ++position;
            }
            if (position >= k) {
                continue;
            }
            if (held < k) {
                ++held;
            }
            for (slot = held - 1U; slot > position; --slot) {
                best_value[slot] = best_value[slot - 1U];
                best_index[slot] = best_index[slot - 1U];
            }
            best_value[position] = v;
            best_index[position] = i;
        }
        for (slot = 0U; slot < k; ++slot) {
            store_float(values, flat_offset(values, row * k + slot),
                        best_value[slot]);
            store_i32(indices, flat_offset(indices, row * k + slot),
                      best_index[slot]);
        }
    }
    return M3O_OK;
}

/* src/m3_op_execute_dense.c:120-159: sequential F32 sum of squares, then
 * 1/sqrtf(mean + eps); the normalised value is rounded to the input dtype
 * before the product with the scale. */
int m3o_rms_norm(const m3o_view *input, const m3o_view *scale,
                 m3o_view *output, float epsilon)
{
    uint64_t channels = input->shape[input->rank - 1];
    uint64_t rows = channels == 0U ? 0U : element_count(input) / channels;
    uint64_t row;

    for (row = 0U; row < rows; ++row) {
        uint64_t base = row * channels;
        float squares = 0.0F;
        float inverse;
        uint64_t c;

        for (c = 0U; c < channels; ++c) {
            float v = load_float(input, flat_offset(input, base + c));
            float square = v * v;

            squares = squares + square;
        }
        inverse = 1.0F / sqrtf(squares / (float)channels + epsilon);
        for (c = 0U; c < channels; ++c) {
            float v = load_float(input, flat_offset(input, base + c));
            float w = load_float(scale, scale->byte_offset +
                                            c * scale->byte_strides[0]);
            float normalized = m3o_round_to_dtype(input->dtype, v * inverse);

            store_float(output, flat_offset(output, base + c),
                        normalized * w);
        }
    }
    return M3O_OK;
}

/* src/m3_op_execute_dense.c:161-217: sequential mean, sequential sum of
 * centred squares, ((x - mean) * inv) * scale (+ bias), no intermediate
 * rounding to the input dtype. */
int m3o_layer_norm(const m3o_view *input, const m3o_view *scale,
                   const m3o_view *bias, m3o_view *output, float epsilon)
{
    uint64_t channels = input->shape[input->rank - 1];
    uint64_t rows = channels == 0U ? 0U : element_count(input) / channels;
    uint64_t row;

    for (row = 0U; row < rows; ++row) {
        uint64_t base = row * channels;
        float sum = 0.0F;
        float centred_squares = 0.0F;
        float mean;
        float inverse;
        uint64_t c;

        for (c = 0U; c < channels; ++c) {
            sum = sum + load_float(input, flat_offset(input, base + c));
        }
        mean = sum / (float)channels;
        for (c = 0U; c < channels; ++c) {
            float centred =
                load_float(input, flat_offset(input, base + c)) - mean;
            float square = centred * centred;

            centred_squares = centred_squares + square;
        }
        inverse = 1.0F / sqrtf(centred_squares / (float)channels + epsilon);
        for (c = 0U; c < channels; ++c) {
            float v = load_float(input, flat_offset(input, base + c));
            float w = load_float(scale, scale->byte_offset +
                                            c * scale->byte_strides[0]);
            float result = ((v - mean) * inverse) * w;

            if (bias != NULL) {
                result = result + load_float(bias, bias->byte_offset +
                                                       c * bias->byte_strides[0]);
            }
            store_float(output, flat_offset(output, base + c), result);
        }
    }
    return M3O_OK;
}

/* ------------------------------------------------------- extension ops */

/* Global abs-max, an extension operator: the F32 value whose bits are the
 * largest of (bits(x) & 0x7fffffff) over all elements (for non-negative floats
 * the unsigned bit order is the value order, so this is max |x| exactly and
 * independent of evaluation order).  Any NaN fails with OUT_OF_RANGE and leaves
 * the output untouched, mirroring the top-k NaN rule of
 * src/m3_op_data_preflight.c:288-291.  An empty input yields +0. */
int m3o_abs_max(const m3o_view *input, m3o_view *output)
{
    uint64_t count = element_count(input);
    uint32_t largest = 0U;
    uint64_t index;

    for (index = 0U; index < count; ++index) {
        float v = load_float(input, flat_offset(input, index));
        uint32_t magnitude = bits_of(v) & 0x7fffffffU;

        if (magnitude > 0x7f800000U) {
            return M3O_OUT_OF_RANGE;
        }
        if (magnitude > largest) {
            largest = magnitude;
        }
    }
    store_float(output, flat_offset(output, 0U), float_of(largest));
    return M3O_OK;
}

/* Clamp to [-1, 1] as the waveform assembly does it
 * (src/m3_waveform.c:360-380): only values above +1 or below -1 are replaced
 * (by the exact bits of +1.0 / -1.0 in the storage dtype); every other element,
 * NaN payloads, signed zeros and subnormals included, is copied bit for bit.
 * Input and output share one dtype. */
int m3o_clamp_unit(const m3o_view *input, m3o_view *output)
{
    uint64_t count = element_count(input);
    size_t size = dtype_bytes(input->dtype);
    uint64_t index;

    if (input->dtype != output->dtype || input->dtype == M3O_I32) {
        return M3O_INVALID_ARGUMENT;
    }
    for (index = 0U; index < count; ++index) {
        uint64_t from = flat_offset(input, index);
        uint64_t to = flat_offset(output, index);
        float v = load_float(input, from);

        if (v > 1.0F) {
            store_float(output, to, 1.0F);
        } else if (v < -1.0F) {
            store_float(output, to, -1.0F);
        } else {
            memmove(wbytes(output) + to, cbytes(input) + from, size);
        }
    }
    return M3O_OK;
}

/* Row sum, an extension operator: the sum of each row over the last axis,
 * accumulated in F32 from the first column to the last, the order (and the
 * per-addition rounding) of the reference's softmax sum
 * (src/m3_op_execute_basic.c:150-158).  Output: F32, the input's shape with
 * the last axis 1.  A NaN or infinity propagates as IEEE addition makes it;
 * there is no data check.  An empty row sums to +0. */
int m3o_row_sum(const m3o_view *input, m3o_view *output)
{
    uint64_t count = element_count(input);
    uint64_t width = input->rank == 0 ? 1U : input->shape[input->rank - 1];
    uint64_t rows = width == 0U ? element_count(output) : count / width;
    uint64_t row;

    if (output->dtype != M3O_F32 || input->dtype == M3O_I32) {
        return M3O_INVALID_ARGUMENT;
    }
    for (row = 0U; row < rows; ++row) {
        float sum = 0.0F;
        uint64_t column;

        for (column = 0U; column < width; ++column) {
            sum += load_float(input, flat_offset(input, row * width + column));
        }
        store_float(output, flat_offset(output, row), sum);
    }
    return M3O_OK;
}

/* ------------------------------------------------------------------ RNG */

/* The reference's PCG32 stream (src/m3_rng.c:9-39): seeding, then `count`
 * successive 32-bit words.  Benchmark inputs are functions of these words
 * (uniforms: src/m3_rng.c:53-66). */
void m3o_pcg32_fill(uint64_t seed, uint64_t sequence, uint32_t *words,
                    size_t count)
{
    const uint64_t multiplier = UINT64_C(6364136223846793005);
    uint64_t increment = (sequence << 1U) | UINT64_C(1);
    uint64_t state = 0U;
    size_t index;

    state = state * multiplier + increment;
    state += seed;
    state = state * multiplier + increment;
    for (index = 0U; index < count; ++index) {
        uint64_t old = state;
        uint32_t shifted = (uint32_t)(((old >> 18U) ^ old) >> 27U);
        uint32_t rotation = (uint32_t)(old >> 59U);

        state = old * multiplier + increment;
        words[index] = (shifted >> rotation) | (shifted << ((0U - rotation) & 31U));
    }
}

/* ---------------------------------------------------------- flow time grid */

/* src/m3_flow_common.c:159-172 */
float m3o_flow_timestep(uint32_t step, uint32_t step_count)
{
    double sigma;
    volatile float timestep;

    if (step_count == 0U || step >= step_count) {
        return 0.0F;
    }
    sigma = 1.0 - (double)step / (double)step_count;
    timestep = 1.0F - (float)sigma;
    return timestep;
}

/* src/m3_flow_common.c:174-190 */
float m3o_flow_timestep_delta(uint32_t step, uint32_t step_count)
{
    float now;
    float next;
    volatile float delta;

    if (step_count == 0U || step >= step_count) {
        return 0.0F;
    }
    now = m3o_flow_timestep(step, step_count);
    next = step + 1U == step_count ? 1.0F
                                   : m3o_flow_timestep(step + 1U, step_count);
    delta = next - now;
    return delta;
}
