/* Operand addressing for the element-wise engine: right-aligned broadcast
 * (the reference's m3_op_broadcast_offset, src/m3_op_numeric.c:150-174)
 * resolved once on the host into coalesced (extent, byte stride) pairs over
 * the output's flat index, plus the cheapest vector access class. */

#include "m3c_internal.h"

#include <string.h>

#define VEC 4U

void m3c_fastdiv_init(m3c_fastdiv *fd, uint32_t divisor)
{
    uint32_t shift = 0U;

    if (divisor == 0U) {
        divisor = 1U;   /* never used for division: extents of 0 and 1 are dropped */
    }
    while (shift < 32U && (UINT64_C(1) << shift) < (uint64_t)divisor) {
        ++shift;
    }
    fd->divisor = divisor;
    fd->shift = shift;
    fd->multiplier = (uint32_t)(((UINT64_C(1) << 32) *
                                 ((UINT64_C(1) << shift) - divisor)) /
                                    divisor +
                                1U);
    fd->reserved = 0U;
}

void m3c_operand_setup(m3c_operand *operand, const void *base,
                       const m3_tensor_metadata *metadata, size_t byte_offset,
                       const size_t *byte_strides,
                       const m3_tensor_metadata *out, int32_t load_as)
{
    uint64_t sizes[M3_TENSOR_MAX_RANK];
    int64_t strides[M3_TENSOR_MAX_RANK];
    int ndim = 0;
    int lead = (int)out->rank - (int)metadata->rank;
    size_t element = m3c_dtype_size(metadata->dtype);
    int axis;
    int d;

    memset(operand, 0, sizeof(*operand));
    operand->base = (const unsigned char *)base + byte_offset;
    operand->dtype = (int32_t)metadata->dtype;
    operand->load_as = load_as;
    if (out->element_count == 0U) {
        /* nothing is read: an empty iteration space */
        operand->vclass = M3C_V_UNIFORM;
        return;
    }
    /* innermost first; drop unit extents; merge axes that step evenly */
    for (axis = (int)out->rank - 1; axis >= 0; --axis) {
        uint64_t extent = out->shape[axis];
        int in_axis = axis - lead;
        int64_t stride = 0;

        if (extent == 1U) {
            continue;
        }
        if (in_axis >= 0 && metadata->shape[in_axis] != 1U) {
            stride = (int64_t)byte_strides[in_axis];
        }
        if (ndim > 0 &&
            strides[ndim - 1] * (int64_t)sizes[ndim - 1] == stride) {
            sizes[ndim - 1] *= extent;
            continue;
        }
        if (ndim > 0 && strides[ndim - 1] == 0 && stride == 0) {
            sizes[ndim - 1] *= extent;
            continue;
        }
        sizes[ndim] = extent;
        strides[ndim] = stride;
        ++ndim;
    }
    /* outer axes that do not move add nothing to any offset */
    while (ndim > 1 && strides[ndim - 1] == 0) {
        --ndim;
    }
    operand->ndim = ndim;
    for (d = 0; d < ndim; ++d) {
        operand->size[d] = sizes[d];
        operand->stride[d] = strides[d];
        m3c_fastdiv_init(&operand->fdiv[d],
                         sizes[d] > UINT32_MAX ? UINT32_MAX : (uint32_t)sizes[d]);
    }
    if (ndim == 0) {
        /* every output element reads the first element */
        operand->vclass = M3C_V_UNIFORM;
        return;
    }
    if (ndim == 1 && strides[0] == (int64_t)element &&
        sizes[0] == (uint64_t)out->element_count &&
        ((uintptr_t)operand->base % (VEC * element)) == 0U) {
        operand->vclass = M3C_V_CONTIG;
        return;
    }
    if (strides[0] == 0 && sizes[0] % VEC == 0U) {
        /* a block of VEC consecutive outputs shares one input element */
        operand->vclass = M3C_V_UNIFORM;
        return;
    }
    if (strides[0] == (int64_t)element && sizes[0] % VEC == 0U &&
        ((uintptr_t)operand->base % (VEC * element)) == 0U) {
        bool aligned = true;

        for (d = 1; d < ndim; ++d) {
            aligned = aligned && strides[d] % (int64_t)(VEC * element) == 0;
        }
        if (aligned) {
            /* a block is VEC adjacent input elements (e.g. a broadcast row
             * vector): one vector load at the block's offset */
            operand->vclass = M3C_V_VECTOR;
            return;
        }
    }
    operand->vclass = M3C_V_GATHER;
}
