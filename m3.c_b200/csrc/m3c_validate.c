/* Structural validation of commands before any device work.
 *
 * The same checks, order and messages as the reference validators for the
 * operators this provider runs (src/m3_op_validate.c:53-233,
 * src/m3_op_validate_basic.c:5-289, src/m3_op_validate_nn.c:120-164,
 * src/m3_op_validate_sampling.c:13-76), plus the two extension operators.
 * Views are abstracted as (metadata, byte offset, byte strides, storage key)
 * so the graph planner and the backend plug-in share one implementation. */

#include "m3c_internal.h"

#include <math.h>
#include <string.h>

typedef struct {
    size_t begin;
    size_t end;
    bool empty;
} span_t;

static m3_status check_view(const m3c_vview *view, bool output,
                            const char *name, m3_error *error)
{
    if (view == NULL || !view->present || view->metadata == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "%s view is required", name);
    }
    if (view->storage == NULL && view->metadata->element_count != 0U) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "%s view has no storage", name);
    }
    if (output && !m3c_contiguous(view->metadata, view->byte_strides)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "%s output must be contiguous", name);
    }
    return M3_STATUS_OK;
}

/* Byte span [begin, end) touched by a view (src/m3_op_validate.c:79-108). */
static m3_status view_span(const m3c_vview *view, span_t *span,
                           m3_error *error)
{
    size_t end = view->byte_offset;
    uint8_t axis;

    span->begin = view->byte_offset;
    span->end = view->byte_offset;
    span->empty = view->metadata->element_count == 0U;
    if (span->empty) {
        return M3_STATUS_OK;
    }
    for (axis = 0U; axis < view->metadata->rank; ++axis) {
        size_t steps = (size_t)(view->metadata->shape[axis] - 1U);
        size_t stride = view->byte_strides[axis];

        if (steps != 0U && stride > SIZE_MAX / steps) {
            return m3c_error_set(error, M3_STATUS_OVERFLOW,
                                 "tensor storage span overflows");
        }
        if (end > SIZE_MAX - steps * stride) {
            return m3c_error_set(error, M3_STATUS_OVERFLOW,
                                 "tensor storage span overflows");
        }
        end += steps * stride;
    }
    if (end > SIZE_MAX - m3c_dtype_size(view->metadata->dtype)) {
        return m3c_error_set(error, M3_STATUS_OVERFLOW,
                             "tensor storage span end overflows");
    }
    span->end = end + m3c_dtype_size(view->metadata->dtype);
    return M3_STATUS_OK;
}

/* Same storage, offset, element size, shape and strides on non-unit axes
 * (src/m3_op_validate.c:110-129). */
static bool exact_view(const m3c_vview *a, const m3c_vview *b)
{
    uint8_t axis;

    if (a->storage != b->storage || a->byte_offset != b->byte_offset ||
        m3c_dtype_size(a->metadata->dtype) !=
            m3c_dtype_size(b->metadata->dtype) ||
        !m3c_shape_equal(a->metadata, b->metadata)) {
        return false;
    }
    for (axis = 0U; axis < a->metadata->rank; ++axis) {
        if (a->metadata->shape[axis] > 1U &&
            a->byte_strides[axis] != b->byte_strides[axis]) {
            return false;
        }
    }
    return true;
}

static m3_status overlap(const m3c_vview *a, const m3c_vview *b,
                         bool *overlapping, m3_error *error)
{
    span_t sa;
    span_t sb;
    m3_status status;

    *overlapping = false;
    if (a->storage != b->storage) {
        return M3_STATUS_OK;
    }
    status = view_span(a, &sa, error);
    if (status == M3_STATUS_OK) {
        status = view_span(b, &sb, error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    *overlapping = !sa.empty && !sb.empty && sa.begin < sb.end &&
                   sb.begin < sa.end;
    return M3_STATUS_OK;
}

/* Outputs may alias an input only exactly, and only where the operator
 * allows it (src/m3_op_validate.c:156-173). */
static m3_status check_alias(const m3c_vview *output, const m3c_vview *input,
                             bool exact_allowed, const char *name,
                             m3_error *error)
{
    bool overlapping;
    m3_status status = overlap(output, input, &overlapping, error);

    if (status != M3_STATUS_OK || !overlapping) {
        return status;
    }
    if (exact_allowed && exact_view(output, input)) {
        return M3_STATUS_OK;
    }
    return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                         "%s has forbidden partial or in-place overlap", name);
}

static m3_status check_disjoint(const m3c_vview *a, const m3c_vview *b,
                                const char *name, m3_error *error)
{
    bool overlapping;
    m3_status status = overlap(a, b, &overlapping, error);

    if (status != M3_STATUS_OK || !overlapping) {
        return status;
    }
    return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                         "%s outputs overlap", name);
}

/* src/m3_op_validate.c:189-233 */
static m3_status check_broadcast(const m3_tensor_metadata *a,
                                 const m3_tensor_metadata *b,
                                 const m3_tensor_metadata *out,
                                 m3_error *error)
{
    uint8_t rank = a->rank > b->rank ? a->rank : b->rank;
    uint8_t axis;

    if (out->rank != rank) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "broadcast output rank is incorrect");
    }
    for (axis = 0U; axis < rank; ++axis) {
        int ia = (int)axis - (int)(rank - a->rank);
        int ib = (int)axis - (int)(rank - b->rank);
        uint64_t ea = ia < 0 ? 1U : a->shape[ia];
        uint64_t eb = ib < 0 ? 1U : b->shape[ib];
        uint64_t expected;

        if (ea != eb && ea != 1U && eb != 1U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "broadcast dimensions disagree at axis %u",
                                 (unsigned)axis);
        }
        expected = ea == 1U ? eb : ea;
        if (out->shape[axis] != expected) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "broadcast output shape is incorrect");
        }
    }
    return M3_STATUS_OK;
}

static m3_status unary_views(const m3c_vcommand *c, m3_error *error)
{
    m3_status status = check_view(&c->in[0], false, "unary input", error);

    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[0], true, "unary output", error);
    }
    if (status == M3_STATUS_OK &&
        !m3c_shape_equal(c->in[0].metadata, c->out[0].metadata)) {
        status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                               "unary input and output shapes differ");
    }
    return status;
}

/* src/m3_op_validate_basic.c:32-97 */
static m3_status validate_copy_cast(const m3c_vcommand *c, m3_error *error)
{
    m3_status status = unary_views(c, error);
    bool exact;

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (c->kind == M3_OP_COPY) {
        if (c->in[0].metadata->dtype != c->out[0].metadata->dtype) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "copy dtypes differ");
        }
        return check_alias(&c->out[0], &c->in[0], true, "copy", error);
    }
    exact = m3c_dtype_size(c->in[0].metadata->dtype) ==
            m3c_dtype_size(c->out[0].metadata->dtype);
    return check_alias(&c->out[0], &c->in[0], exact, "cast", error);
}

/* src/m3_op_validate_basic.c:66-110 */
static m3_status validate_binary(const m3c_vcommand *c, bool broadcast,
                                 m3_error *error)
{
    const m3_tensor_metadata *l;
    const m3_tensor_metadata *r;
    const m3_tensor_metadata *o;
    m3_status status = check_view(&c->in[0], false, "binary left input",
                                  error);

    if (status == M3_STATUS_OK) {
        status = check_view(&c->in[1], false, "binary right input", error);
    }
    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[0], true, "binary output", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    l = c->in[0].metadata;
    r = c->in[1].metadata;
    o = c->out[0].metadata;
    if (!m3c_dtype_float(l->dtype) || !m3c_dtype_float(r->dtype) ||
        !m3c_dtype_float(o->dtype)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "binary arithmetic requires float tensors");
    }
    if (broadcast) {
        status = check_broadcast(l, r, o, error);
    } else if (!m3c_shape_equal(l, r) || !m3c_shape_equal(l, o)) {
        status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                               "binary tensor shapes differ");
    }
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[0], &c->in[0], m3c_shape_equal(l, o),
                             "binary left input", error);
    }
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[0], &c->in[1], m3c_shape_equal(r, o),
                             "binary right input", error);
    }
    return status;
}

/* src/m3_op_validate_basic.c:161-184 */
static m3_status validate_softmax(const m3c_vcommand *c, m3_error *error)
{
    m3_status status = unary_views(c, error);
    const m3_tensor_metadata *in;

    if (status != M3_STATUS_OK) {
        return status;
    }
    in = c->in[0].metadata;
    if (!m3c_dtype_float(in->dtype)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "softmax input must have a floating-point dtype");
    }
    if (!m3c_dtype_float(c->out[0].metadata->dtype)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "softmax output must have a floating-point dtype");
    }
    if (in->rank == 0U || in->shape[in->rank - 1U] == 0U) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "softmax last axis must be nonempty");
    }
    return check_alias(&c->out[0], &c->in[0], true, "softmax", error);
}

/* src/m3_op_validate_basic.c:186-227 */
static m3_status validate_snake(const m3c_vcommand *c, m3_error *error)
{
    const m3_tensor_metadata *x;
    const m3_tensor_metadata *a;
    const m3_tensor_metadata *o;
    m3_status status = check_view(&c->in[0], false, "Snake1d input", error);

    if (status == M3_STATUS_OK) {
        status = check_view(&c->in[1], false, "Snake1d alpha", error);
    }
    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[0], true, "Snake1d output", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    x = c->in[0].metadata;
    a = c->in[1].metadata;
    o = c->out[0].metadata;
    if (x->dtype != M3_DTYPE_F32 || a->dtype != M3_DTYPE_F32 ||
        o->dtype != M3_DTYPE_F32 || x->rank != 3U || a->rank != 3U ||
        o->rank != 3U) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "Snake1d requires rank-3 F32 tensors");
    }
    if (!m3c_shape_equal(x, o) || a->shape[0] != 1U ||
        a->shape[1] != x->shape[1] || a->shape[2] != 1U) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "Snake1d alpha or output shape is invalid");
    }
    status = check_alias(&c->out[0], &c->in[0], true, "Snake1d input", error);
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[0], &c->in[1], false, "Snake1d alpha",
                             error);
    }
    return status;
}

/* src/m3_op_validate_basic.c:229-247 */
static m3_status validate_tanh(const m3c_vcommand *c, m3_error *error)
{
    m3_status status = unary_views(c, error);

    if (status == M3_STATUS_OK &&
        (c->in[0].metadata->dtype != M3_DTYPE_F32 ||
         c->out[0].metadata->dtype != M3_DTYPE_F32 ||
         c->in[0].metadata->rank == 0U)) {
        status = m3c_error_set(
            error, M3_STATUS_INVALID_ARGUMENT,
            "tanh requires rank-1 through rank-8 F32 tensors");
    }
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[0], &c->in[0], true, "tanh", error);
    }
    return status;
}

static m3_status nn_view(const m3c_vview *view, bool output, const char *name,
                         m3_error *error)
{
    m3_status status = check_view(view, output, name, error);

    if (status == M3_STATUS_OK && !m3c_dtype_float(view->metadata->dtype)) {
        status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                               "%s must have a floating-point dtype", name);
    }
    return status;
}

/* src/m3_op_validate_nn.c:120-164 (scale in[1], optional bias in[2]). */
static m3_status validate_norm(const m3c_vcommand *c, m3_error *error)
{
    const char *name = c->kind == M3_OP_RMS_NORM ? "RMSNorm input"
                                                 : "LayerNorm input";
    const m3c_vview *bias = c->in[2].present ? &c->in[2] : NULL;
    const m3_tensor_metadata *in;
    const m3_tensor_metadata *scale;
    uint64_t channels;
    m3_status status = nn_view(&c->in[0], false, name, error);

    if (status == M3_STATUS_OK) {
        status = nn_view(&c->in[1], false, "norm scale", error);
    }
    if (status == M3_STATUS_OK && bias != NULL) {
        status = nn_view(bias, false, "norm bias", error);
    }
    if (status == M3_STATUS_OK) {
        status = nn_view(&c->out[0], true, "norm output", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    in = c->in[0].metadata;
    scale = c->in[1].metadata;
    if (in->rank == 0U || !m3c_shape_equal(in, c->out[0].metadata) ||
        !isfinite(c->epsilon) || c->epsilon <= 0.0F) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "norm shape or epsilon is invalid");
    }
    channels = in->shape[in->rank - 1U];
    if (channels == 0U || scale->rank != 1U || scale->shape[0] != channels ||
        (bias != NULL && (bias->metadata->rank != 1U ||
                          bias->metadata->shape[0] != channels))) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "norm channel shape is invalid");
    }
    status = check_alias(&c->out[0], &c->in[0], true, name, error);
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[0], &c->in[1], false, "norm scale",
                             error);
    }
    if (status == M3_STATUS_OK && bias != NULL) {
        status = check_alias(&c->out[0], bias, false, "norm bias", error);
    }
    return status;
}

/* src/m3_op_validate_sampling.c:13-76 */
static m3_status validate_top_k(const m3c_vcommand *c, m3_error *error)
{
    const m3_tensor_metadata *logits;
    const m3_tensor_metadata *values;
    const m3_tensor_metadata *indices;
    uint8_t rank;
    uint8_t axis;
    bool shape_ok;
    m3_status status = check_view(&c->in[0], false, "top-k logits", error);

    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[0], true, "top-k values", error);
    }
    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[1], true, "top-k indices", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    logits = c->in[0].metadata;
    values = c->out[0].metadata;
    indices = c->out[1].metadata;
    rank = logits->rank;
    shape_ok = rank != 0U && values->rank == rank && indices->rank == rank;
    for (axis = 0U; shape_ok && axis + 1U < rank; ++axis) {
        shape_ok = values->shape[axis] == logits->shape[axis] &&
                   indices->shape[axis] == logits->shape[axis];
    }
    shape_ok = shape_ok && c->k != 0U && c->k <= logits->shape[rank - 1U] &&
               values->shape[rank - 1U] == c->k &&
               indices->shape[rank - 1U] == c->k;
    if (rank == 0U || !m3c_dtype_float(logits->dtype) ||
        values->dtype != M3_DTYPE_F32 || indices->dtype != M3_DTYPE_I32 ||
        logits->shape[rank - 1U] > (uint64_t)INT32_MAX || !shape_ok) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "top-k dtype, K, or shape is invalid");
    }
    status = check_alias(&c->out[0], &c->in[0], false, "top-k values", error);
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[1], &c->in[0], false, "top-k indices",
                             error);
    }
    if (status == M3_STATUS_OK) {
        status = check_disjoint(&c->out[0], &c->out[1], "top-k", error);
    }
    return status;
}

/* src/m3_op_validate_sampling.c:77-131 */
static m3_status validate_categorical(const m3c_vcommand *c, m3_error *error)
{
    const m3_tensor_metadata *probabilities;
    const m3_tensor_metadata *uniforms;
    const m3_tensor_metadata *output;
    uint8_t rank;
    uint8_t axis;
    bool shape_ok;
    m3_status status = check_view(&c->in[0], false, "categorical probabilities",
                                  error);

    if (status == M3_STATUS_OK) {
        status = check_view(&c->in[1], false, "categorical uniforms", error);
    }
    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[0], true, "categorical output", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    probabilities = c->in[0].metadata;
    uniforms = c->in[1].metadata;
    output = c->out[0].metadata;
    rank = probabilities->rank;
    shape_ok = rank != 0U && probabilities->shape[rank - 1U] != 0U &&
               probabilities->shape[rank - 1U] <= (uint64_t)INT32_MAX &&
               uniforms->rank + 1U == rank && output->rank + 1U == rank &&
               m3c_shape_equal(uniforms, output);
    for (axis = 0U; shape_ok && axis + 1U < rank; ++axis) {
        shape_ok = uniforms->shape[axis] == probabilities->shape[axis];
    }
    if (!m3c_dtype_float(probabilities->dtype) ||
        !m3c_dtype_float(uniforms->dtype) || output->dtype != M3_DTYPE_I32 ||
        !shape_ok) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "categorical dtype or shape is invalid");
    }
    status = check_alias(&c->out[0], &c->in[0], false,
                         "categorical probabilities", error);
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[0], &c->in[1], false,
                             "categorical uniforms", error);
    }
    return status;
}

/* Extension: abs-max of any float tensor into one F32 element. */
static m3_status validate_abs_max(const m3c_vcommand *c, m3_error *error)
{
    m3_status status = check_view(&c->in[0], false, "abs-max input", error);

    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[0], true, "abs-max output", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    if (!m3c_dtype_float(c->in[0].metadata->dtype) ||
        c->out[0].metadata->dtype != M3_DTYPE_F32 ||
        c->out[0].metadata->element_count != 1U) {
        return m3c_error_set(
            error, M3_STATUS_INVALID_ARGUMENT,
            "abs-max requires a float input and one F32 output element");
    }
    return check_alias(&c->out[0], &c->in[0], false, "abs-max", error);
}

/* Extension: row sums of a float tensor into F32 [..., 1]. */
static m3_status validate_row_sum(const m3c_vcommand *c, m3_error *error)
{
    const m3_tensor_metadata *in;
    const m3_tensor_metadata *out;
    bool shape_ok;
    uint8_t axis;
    m3_status status = check_view(&c->in[0], false, "row-sum input", error);

    if (status == M3_STATUS_OK) {
        status = check_view(&c->out[0], true, "row-sum output", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    in = c->in[0].metadata;
    out = c->out[0].metadata;
    shape_ok = in->rank != 0U && out->rank == in->rank &&
               out->shape[in->rank - 1U] == 1U;
    for (axis = 0U; shape_ok && axis + 1U < in->rank; ++axis) {
        shape_ok = out->shape[axis] == in->shape[axis];
    }
    if (!m3c_dtype_float(in->dtype) || out->dtype != M3_DTYPE_F32 || !shape_ok) {
        return m3c_error_set(
            error, M3_STATUS_INVALID_ARGUMENT,
            "row-sum requires a float input and F32 output [..., 1]");
    }
    return check_alias(&c->out[0], &c->in[0], false, "row-sum", error);
}

/* Extension: bit-preserving clamp of F32 to [-1, 1]. */
static m3_status validate_clamp(const m3c_vcommand *c, m3_error *error)
{
    m3_status status = unary_views(c, error);

    if (status == M3_STATUS_OK &&
        (c->in[0].metadata->dtype != M3_DTYPE_F32 ||
         c->out[0].metadata->dtype != M3_DTYPE_F32)) {
        status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                               "clamp requires F32 tensors");
    }
    if (status == M3_STATUS_OK) {
        status = check_alias(&c->out[0], &c->in[0], true, "clamp", error);
    }
    return status;
}

bool m3c_kind_supported(m3_op_kind kind)
{
    switch ((int)kind) {
    case M3_OP_COPY:
    case M3_OP_CAST:
    case M3_OP_ADD:
    case M3_OP_MUL:
    case M3_OP_GATED_SILU:
    case M3_OP_SOFTMAX:
    case M3_OP_TOP_K:
    case M3_OP_CATEGORICAL:
    case M3_OP_RMS_NORM:
    case M3_OP_LAYER_NORM:
    case M3_OP_SNAKE1D:
    case M3_OP_TANH:
    case (int)M3_OP_ABS_MAX:
    case (int)M3_OP_CLAMP_UNIT:
    case (int)M3_OP_ROW_SUM:
        return true;
    default:
        return false;
    }
}

const char *m3c_kind_name(m3_op_kind kind)
{
    switch ((int)kind) {
    case M3_OP_COPY: return "COPY";
    case M3_OP_CAST: return "CAST";
    case M3_OP_ADD: return "ADD";
    case M3_OP_MUL: return "MUL";
    case M3_OP_GATED_SILU: return "GATED_SILU";
    case M3_OP_SOFTMAX: return "SOFTMAX";
    case M3_OP_TOP_K: return "TOP_K";
    case M3_OP_CATEGORICAL: return "CATEGORICAL";
    case M3_OP_RMS_NORM: return "RMS_NORM";
    case M3_OP_LAYER_NORM: return "LAYER_NORM";
    case M3_OP_SNAKE1D: return "SNAKE1D";
    case M3_OP_TANH: return "TANH";
    case (int)M3_OP_ABS_MAX: return "ABS_MAX";
    case (int)M3_OP_CLAMP_UNIT: return "CLAMP_UNIT";
    case (int)M3_OP_ROW_SUM: return "ROW_SUM";
    default: return "UNSUPPORTED";
    }
}

m3_status m3c_validate(const m3c_vcommand *command, m3_error *error)
{
    m3_status status;

    if (command == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "backend and command are required");
    }
    switch ((int)command->kind) {
    case M3_OP_COPY:
    case M3_OP_CAST:
        status = validate_copy_cast(command, error);
        break;
    case M3_OP_ADD:
    case M3_OP_MUL:
        status = validate_binary(command, true, error);
        break;
    case M3_OP_GATED_SILU:
        status = validate_binary(command, false, error);
        break;
    case M3_OP_SOFTMAX:
        status = validate_softmax(command, error);
        break;
    case M3_OP_SNAKE1D:
        status = validate_snake(command, error);
        break;
    case M3_OP_TANH:
        status = validate_tanh(command, error);
        break;
    case M3_OP_RMS_NORM:
    case M3_OP_LAYER_NORM:
        status = validate_norm(command, error);
        break;
    case M3_OP_TOP_K:
        status = validate_top_k(command, error);
        break;
    case M3_OP_CATEGORICAL:
        status = validate_categorical(command, error);
        break;
    case (int)M3_OP_ABS_MAX:
        status = validate_abs_max(command, error);
        break;
    case (int)M3_OP_CLAMP_UNIT:
        status = validate_clamp(command, error);
        break;
    case (int)M3_OP_ROW_SUM:
        status = validate_row_sum(command, error);
        break;
    default:
        status = m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                               "unsupported operation kind %d",
                               (int)command->kind);
        break;
    }
    if (status == M3_STATUS_OK) {
        m3_error_reset(error);
    }
    return status;
}
