/* Status strings, error sinks and tensor metadata for libm3cuda.so.
 * Messages and status spellings follow the reference (src/m3_error.c:7-94,
 * src/m3_tensor.c) so callers see the same diagnostics. */

#include "m3c_internal.h"

#include <stdio.h>
#include <string.h>

const char *m3_version(void)
{
    return M3C_VERSION;
}

/* src/m3_error.c:7-33 */
const char *m3_status_string(m3_status status)
{
    switch (status) {
    case M3_STATUS_OK:
        return "ok";
    case M3_STATUS_INVALID_ARGUMENT:
        return "invalid argument";
    case M3_STATUS_OUT_OF_RANGE:
        return "out of range";
    case M3_STATUS_OVERFLOW:
        return "overflow";
    case M3_STATUS_OUT_OF_MEMORY:
        return "out of memory";
    case M3_STATUS_IO:
        return "I/O error";
    case M3_STATUS_INVALID_FORMAT:
        return "invalid format";
    case M3_STATUS_UNSUPPORTED:
        return "unsupported";
    case M3_STATUS_CANCELLED:
        return "cancelled";
    case M3_STATUS_INTERNAL:
        return "internal error";
    }
    return "unknown status";
}

void m3_error_reset(m3_error *error)
{
    if (error != NULL) {
        error->status = M3_STATUS_OK;
        error->message[0] = '\0';
    }
}

const char *m3_error_message(const m3_error *error)
{
    return error == NULL ? "" : error->message;
}

/* A NULL sink is allowed and only the status is returned
 * (src/m3_error.c:45-86). */
m3_status m3c_error_set(m3_error *error, m3_status status, const char *format,
                        ...)
{
    va_list arguments;
    int written;

    if (error == NULL) {
        return status;
    }
    error->status = status;
    if (status == M3_STATUS_OK) {
        error->message[0] = '\0';
        return status;
    }
    if (format == NULL) {
        (void)snprintf(error->message, sizeof(error->message), "%s",
                       m3_status_string(status));
        return status;
    }
    va_start(arguments, format);
    written = vsnprintf(error->message, sizeof(error->message), format,
                        arguments);
    va_end(arguments);
    if (written < 0) {
        (void)snprintf(error->message, sizeof(error->message), "%s",
                       m3_status_string(status));
    }
    error->message[sizeof(error->message) - 1U] = '\0';
    return status;
}

size_t m3c_dtype_size(m3_dtype dtype)
{
    return (dtype == M3_DTYPE_F16 || dtype == M3_DTYPE_BF16) ? 2U : 4U;
}

bool m3c_dtype_float(m3_dtype dtype)
{
    return dtype == M3_DTYPE_F32 || dtype == M3_DTYPE_F16 ||
           dtype == M3_DTYPE_BF16;
}

/* Same contract and statuses as the reference's m3_tensor_metadata_init
 * (src/m3_tensor.c:39-102): a known dtype, rank <= 8, element and byte counts
 * without overflow. */
m3_status m3c_metadata_init(m3_tensor_metadata *metadata, m3_dtype dtype,
                            uint8_t rank, const uint64_t *shape,
                            m3_error *error)
{
    size_t count = 1U;
    uint8_t axis;

    if (metadata == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "tensor metadata output is null");
    }
    if ((int)dtype < (int)M3_DTYPE_F32 || (int)dtype > (int)M3_DTYPE_I32) {
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "unsupported tensor dtype value %d", (int)dtype);
    }
    if (rank > M3_TENSOR_MAX_RANK) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "tensor rank %u exceeds maximum rank %u",
                             (unsigned)rank, (unsigned)M3_TENSOR_MAX_RANK);
    }
    if (rank != 0U && shape == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "tensor shape is null for rank %u",
                             (unsigned)rank);
    }
    memset(metadata, 0, sizeof(*metadata));
    metadata->dtype = dtype;
    metadata->rank = rank;
    for (axis = 0U; axis < rank; ++axis) {
        uint64_t extent = shape[axis];

        metadata->shape[axis] = extent;
        if (extent != 0U && count > SIZE_MAX / extent) {
            return m3c_error_set(error, M3_STATUS_OVERFLOW,
                                 "tensor element count overflows");
        }
        count *= (size_t)extent;
    }
    if (count > SIZE_MAX / m3c_dtype_size(dtype)) {
        return m3c_error_set(error, M3_STATUS_OVERFLOW,
                             "tensor byte count overflows");
    }
    metadata->element_count = count;
    metadata->byte_count = count * m3c_dtype_size(dtype);
    return M3_STATUS_OK;
}

bool m3c_shape_equal(const m3_tensor_metadata *a, const m3_tensor_metadata *b)
{
    uint8_t axis;

    if (a->rank != b->rank) {
        return false;
    }
    for (axis = 0U; axis < a->rank; ++axis) {
        if (a->shape[axis] != b->shape[axis]) {
            return false;
        }
    }
    return true;
}

/* Contiguity as the reference defines it (src/m3_tensor_runtime.c:222-246):
 * strides of a dense row-major layout, axes of extent one excepted; an empty
 * tensor is contiguous. */
bool m3c_contiguous(const m3_tensor_metadata *metadata,
                    const size_t *byte_strides)
{
    size_t expected = m3c_dtype_size(metadata->dtype);
    int axis;

    if (metadata->element_count == 0U) {
        return true;
    }
    for (axis = (int)metadata->rank - 1; axis >= 0; --axis) {
        if (metadata->shape[axis] > 1U && byte_strides[axis] != expected) {
            return false;
        }
        expected *= (size_t)metadata->shape[axis];
    }
    return true;
}

const char *m3c_categorical_message(uint32_t detail)
{
    switch (detail & 3U) {
    case 1U:
        return "categorical uniform is outside [0,1)";
    case 2U:
        return "categorical probability is invalid";
    default:
        return "categorical row sum is not positive finite";
    }
}
