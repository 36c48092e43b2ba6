/* The backend plug-in of the reference (m3_backend_vtable,
 * src/m3_backend_internal.h:9-17) backed by the CUDA kernels.
 *
 * The reference's scheduler hands this backend whole command lists
 * (src/m3_backend.c:113-154 validates them first).  Commands run in order on
 * one stream.  Consecutive commands merge into one launch where that cannot
 * change a result (fuse_ew, fuse_rows below): every output is still written,
 * since no liveness information reaches a backend, but a value a fused
 * command wrote is not read back.  Views may be strided: element-wise
 * operands are addressed through their strides directly; row operators gather
 * a non-contiguous input into the backend's reusable gather buffer first.
 * Data-checked operators
 * (SOFTMAX/TOP_K NaN, float-to-I32 CAST range) run a scan kernel before the
 * computing kernel; the computing kernel skips its writes when the scan (or
 * any earlier command) failed, so a failing list leaves the failing command's
 * outputs and everything after it untouched, as in the reference.
 * `execute` returns after the stream is idle (the reference's Metal backend
 * likewise waits for completion, src/m3_backend_metal.m:211-212). */

#include "m3c_internal.h"

#include <cuda_runtime_api.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int device;
    void *(*storage_data)(m3_storage *storage);
    bool managed;
    cudaStream_t stream;
    m3c_status *status;
    m3c_status *status_host;
    m3c_reduce_scratch *reduce;
    /* dense copies of strided row-operator inputs: one buffer, grown on
     * demand and reused (commands run in stream order, so each command's
     * copy is consumed before the next command overwrites it) */
    void *gather;
    size_t gather_bytes;
    /* kernels launched by the last execute */
    unsigned launches;
    /* the stream created with the context; `stream` may be a caller's */
    cudaStream_t own_stream;
} cuda_backend;

static const m3c_status clean = {UINT32_MAX, 0U, 0U, UINT32_MAX};

static m3_status fail_cuda(m3_error *error, cudaError_t code, const char *what)
{
    (void)cudaGetLastError();
    return m3c_error_set(error,
                         code == cudaErrorMemoryAllocation
                             ? M3_STATUS_OUT_OF_MEMORY
                             : M3_STATUS_INTERNAL,
                         "%s: %s", what, cudaGetErrorString(code));
}

bool m3_cuda_backend_supports_kind(m3_op_kind kind)
{
    return m3c_kind_supported(kind);
}

m3_status m3_cuda_backend_context_create(
    const m3_cuda_backend_options *options, void **context, m3_error *error)
{
    cuda_backend *b;
    cudaError_t code;
    int devices = 0;

    if (context == NULL || options == NULL || options->storage_data == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "backend options and storage accessor are required");
    }
    *context = NULL;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
        (void)cudaGetLastError();
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "no CUDA device is available");
    }
    b = calloc(1U, sizeof(*b));
    if (b == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate CUDA backend context");
    }
    b->device = options->device < 0 ? 0 : options->device;
    b->storage_data = options->storage_data;
    b->managed = options->managed_memory;
    code = cudaSetDevice(b->device);
    if (code == cudaSuccess) {
        code = cudaStreamCreateWithFlags(&b->own_stream, cudaStreamNonBlocking);
        b->stream = b->own_stream;
    }
    if (code == cudaSuccess) {
        code = cudaMalloc((void **)&b->status, sizeof(m3c_status));
    }
    if (code == cudaSuccess) {
        code = cudaMalloc((void **)&b->reduce, sizeof(m3c_reduce_scratch));
    }
    if (code == cudaSuccess) {
        code = cudaMallocHost((void **)&b->status_host, sizeof(m3c_status));
    }
    if (code == cudaSuccess) {
        code = cudaMemset(b->reduce, 0, sizeof(m3c_reduce_scratch));
    }
    if (code == cudaSuccess) {
        code = cudaMemcpy(b->status, &clean, sizeof(clean),
                          cudaMemcpyHostToDevice);
    }
    if (code != cudaSuccess) {
        m3_cuda_backend_destroy_context(b);
        return fail_cuda(error, code, "cannot create CUDA backend");
    }
    *context = b;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

void m3_cuda_backend_destroy_context(void *context)
{
    cuda_backend *b = context;

    if (b == NULL) {
        return;
    }
    (void)cudaSetDevice(b->device);
    if (b->stream != NULL) {
        (void)cudaStreamSynchronize(b->stream);
    }
    if (b->own_stream != NULL) {
        (void)cudaStreamSynchronize(b->own_stream);
        (void)cudaStreamDestroy(b->own_stream);
    }
    (void)cudaFree(b->status);
    (void)cudaFree(b->reduce);
    (void)cudaFree(b->gather);
    (void)cudaFreeHost(b->status_host);
    (void)cudaGetLastError();
    free(b);
}

m3_status m3_cuda_backend_allocate(void *context, size_t byte_count,
                                   size_t alignment, void **handle,
                                   void **data, m3_error *error)
{
    cuda_backend *b = context;
    cudaError_t code;
    void *memory = NULL;

    *handle = NULL;
    *data = NULL;
    if (byte_count == 0U) {
        return M3_STATUS_OK;
    }
    if (alignment > M3C_ARENA_ALIGNMENT) {
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "CUDA storage alignment above 256 bytes");
    }
    (void)cudaSetDevice(b->device);
    code = b->managed ? cudaMallocManaged(&memory, byte_count,
                                          cudaMemAttachGlobal)
                      : cudaMalloc(&memory, byte_count);
    if (code != cudaSuccess) {
        return fail_cuda(error, code, "cannot allocate CUDA storage");
    }
    *handle = memory;
    *data = memory;
    return M3_STATUS_OK;
}

void m3_cuda_backend_free_storage(void *context, void *handle, void *data)
{
    cuda_backend *b = context;

    (void)data;
    if (handle != NULL) {
        (void)cudaSetDevice(b->device);
        (void)cudaFree(handle);
        (void)cudaGetLastError();
    }
}

m3_status m3_cuda_backend_write(void *context, void *data, size_t byte_offset,
                                const void *source, size_t byte_count,
                                m3_error *error)
{
    cuda_backend *b = context;
    cudaError_t code;

    if (byte_count == 0U) {
        return M3_STATUS_OK;
    }
    (void)cudaSetDevice(b->device);
    code = cudaMemcpyAsync((unsigned char *)data + byte_offset, source,
                           byte_count, cudaMemcpyHostToDevice, b->stream);
    if (code == cudaSuccess) {
        code = cudaStreamSynchronize(b->stream);
    }
    return code == cudaSuccess ? M3_STATUS_OK
                               : fail_cuda(error, code, "storage write failed");
}

m3_status m3_cuda_backend_read(void *context, const void *data,
                               size_t byte_offset, void *destination,
                               size_t byte_count, m3_error *error)
{
    cuda_backend *b = context;
    cudaError_t code;

    if (byte_count == 0U) {
        return M3_STATUS_OK;
    }
    (void)cudaSetDevice(b->device);
    code = cudaMemcpyAsync(destination, (const unsigned char *)data + byte_offset,
                           byte_count, cudaMemcpyDeviceToHost, b->stream);
    if (code == cudaSuccess) {
        code = cudaStreamSynchronize(b->stream);
    }
    return code == cudaSuccess ? M3_STATUS_OK
                               : fail_cuda(error, code, "storage read failed");
}

/* ------------------------------------------------------------ execution */

static unsigned char *view_base(const cuda_backend *b, const m3_tensor_view *v)
{
    return (unsigned char *)b->storage_data(v->storage);
}

static void vview_of(const m3_tensor_view *view, m3c_vview *out)
{
    memset(out, 0, sizeof(*out));
    if (view == NULL) {
        return;
    }
    out->metadata = &view->metadata;
    out->byte_offset = view->byte_offset;
    out->byte_strides = view->byte_strides;
    out->storage = view->storage;
    out->present = true;
}

/* The reference command, in the validator's positional form. */
static void to_vcommand(const m3_command *c, m3c_vcommand *v)
{
    memset(v, 0, sizeof(*v));
    v->kind = c->kind;
    switch ((int)c->kind) {
    case M3_OP_ADD:
    case M3_OP_MUL:
    case M3_OP_GATED_SILU:
        vview_of(c->descriptor.add.left, &v->in[0]);
        vview_of(c->descriptor.add.right, &v->in[1]);
        vview_of(c->descriptor.add.output, &v->out[0]);
        break;
    case M3_OP_RMS_NORM:
        vview_of(c->descriptor.rms_norm.input, &v->in[0]);
        vview_of(c->descriptor.rms_norm.scale, &v->in[1]);
        vview_of(c->descriptor.rms_norm.output, &v->out[0]);
        v->epsilon = c->descriptor.rms_norm.epsilon;
        break;
    case M3_OP_LAYER_NORM:
        vview_of(c->descriptor.layer_norm.input, &v->in[0]);
        vview_of(c->descriptor.layer_norm.scale, &v->in[1]);
        vview_of(c->descriptor.layer_norm.bias, &v->in[2]);
        vview_of(c->descriptor.layer_norm.output, &v->out[0]);
        v->epsilon = c->descriptor.layer_norm.epsilon;
        break;
    case M3_OP_TOP_K:
        vview_of(c->descriptor.top_k.logits, &v->in[0]);
        vview_of(c->descriptor.top_k.values, &v->out[0]);
        vview_of(c->descriptor.top_k.indices, &v->out[1]);
        v->k = c->descriptor.top_k.k;
        break;
    case M3_OP_CATEGORICAL:
        vview_of(c->descriptor.categorical.probabilities, &v->in[0]);
        vview_of(c->descriptor.categorical.uniforms, &v->in[1]);
        vview_of(c->descriptor.categorical.output, &v->out[0]);
        break;
    case M3_OP_SNAKE1D:
        vview_of(c->descriptor.snake1d.input, &v->in[0]);
        vview_of(c->descriptor.snake1d.alpha, &v->in[1]);
        vview_of(c->descriptor.snake1d.output, &v->out[0]);
        break;
    default: /* unary shapes: COPY, CAST, SOFTMAX, TANH, extensions */
        vview_of(c->descriptor.copy.input, &v->in[0]);
        vview_of(c->descriptor.copy.output, &v->out[0]);
        break;
    }
}

/* One element-wise op over views (single-op program). */
static int launch_unary_ew(cuda_backend *b, uint32_t command, uint8_t code,
                           const m3_tensor_view *a, const m3_tensor_view *x,
                           const m3_tensor_view *out, int aux,
                           const m3_tensor_metadata *space)
{
    m3c_ew_params p;
    int reg = 0;

    memset(&p, 0, sizeof(p));
    p.count = space->element_count;
    p.status = b->status;
    /* a range-checked cast runs after its scan: skip when the scan failed */
    p.skip_before = code == M3C_OP_F2I ? command + 1U : command;
    p.first_of_run = 0;
    p.n_operands = 0;
    if (a != NULL) {
        m3c_operand_setup(&p.operands[p.n_operands++], view_base(b, a),
                          &a->metadata, a->byte_offset, a->byte_strides, space,
                          a->metadata.dtype == M3_DTYPE_I32 ? M3C_LOAD_INT
                                                            : M3C_LOAD_RAW);
    }
    if (x != NULL) {
        m3c_operand_setup(&p.operands[p.n_operands++], view_base(b, x),
                          &x->metadata, x->byte_offset, x->byte_strides, space,
                          x->metadata.dtype == M3_DTYPE_I32 ? M3C_LOAD_INT
                                                            : M3C_LOAD_RAW);
    }
    /* widen 16-bit operands explicitly (registers 0, 1 -> 2, 3) */
    {
        int k;
        int regs[2] = {0, 1};

        for (k = 0; k < p.n_operands; ++k) {
            const m3_tensor_view *v = k == 0 ? a : x;
            bool raw_copy = code == M3C_OP_MOV;

            if (!raw_copy && (v->metadata.dtype == M3_DTYPE_F16 ||
                              v->metadata.dtype == M3_DTYPE_BF16)) {
                m3c_ew_op *op = &p.ops[p.n_ops++];

                op->code = M3C_OP_WIDEN;
                op->dst = (uint8_t)(2 + k);
                op->a = (uint8_t)k;
                op->b = (uint8_t)k;
                op->rdtype = M3C_F32;
                op->aux = (int8_t)v->metadata.dtype;
                op->command = (uint16_t)command;
                regs[k] = 2 + k;
            }
        }
        {
            m3c_ew_op *op = &p.ops[p.n_ops++];

            op->code = code;
            op->a = (uint8_t)regs[0];
            op->b = (uint8_t)(p.n_operands > 1 ? regs[1] : regs[0]);
            op->dst = code == M3C_OP_ABSMAX ? op->a : 4U;
            op->rdtype = out != NULL ? (int8_t)out->metadata.dtype : M3C_F32;
            op->aux = (int8_t)aux;
            op->command = (uint16_t)command;
            reg = 4;
        }
    }
    if (code == M3C_OP_ABSMAX) {
        p.reduce = b->reduce;
        p.absmax_out = view_base(b, out) + out->byte_offset;
        p.absmax_command = command;
    } else {
        size_t vector_bytes = 4U * m3c_dtype_size(out->metadata.dtype);

        p.n_outputs = 1;
        p.outputs[0].base = view_base(b, out) + out->byte_offset;
        p.outputs[0].dtype = (int32_t)out->metadata.dtype;
        p.outputs[0].reg = (int16_t)reg;
        p.outputs[0].scalar_only =
            ((uintptr_t)p.outputs[0].base % vector_bytes) != 0U ? 1U : 0U;
        p.outputs[0].raw = (code == M3C_OP_MOV &&
                            m3c_dtype_size(out->metadata.dtype) == 2U)
                               ? 1
                               : 0;
    }
    ++b->launches;
    return m3c_launch_ew(&p, b->stream);
}

/* Row operators need a dense row-major input: gather strided views into the
 * backend's gather buffer. */
static int dense_input(cuda_backend *b, const m3_tensor_view *view,
                       uint32_t command,
                       const void **data, void **temporary)
{
    m3_tensor_view dense;
    size_t stride = m3c_dtype_size(view->metadata.dtype);
    int axis;
    int result;

    *temporary = NULL;
    if (m3c_contiguous(&view->metadata, view->byte_strides)) {
        *data = view_base(b, view) + view->byte_offset;
        return 0;
    }
    if (view->metadata.byte_count > b->gather_bytes) {
        /* grow: earlier commands of this list may still read the old
         * buffer, so wait for them before releasing it */
        cudaError_t code = cudaStreamSynchronize(b->stream);

        if (code == cudaSuccess) {
            (void)cudaFree(b->gather);
            b->gather = NULL;
            b->gather_bytes = 0U;
            code = cudaMalloc(&b->gather, view->metadata.byte_count);
        }
        if (code != cudaSuccess) {
            b->gather = NULL;
            return (int)code;
        }
        b->gather_bytes = view->metadata.byte_count;
    }
    *temporary = b->gather;
    dense = *view;
    dense.byte_offset = 0U;
    for (axis = (int)dense.metadata.rank - 1; axis >= 0; --axis) {
        dense.byte_strides[axis] = stride;
        stride *= (size_t)dense.metadata.shape[axis];
    }
    {
        m3c_ew_params p;

        memset(&p, 0, sizeof(p));
        p.count = view->metadata.element_count;
        p.status = b->status;
        p.skip_before = command;
        p.n_operands = 1;
        m3c_operand_setup(&p.operands[0], view_base(b, view), &view->metadata,
                          view->byte_offset, view->byte_strides,
                          &view->metadata, M3C_LOAD_RAW);
        p.n_ops = 1;
        p.ops[0].code = M3C_OP_MOV;
        p.ops[0].dst = 1;
        p.n_outputs = 1;
        p.outputs[0].base = *temporary;
        p.outputs[0].dtype = (int32_t)view->metadata.dtype;
        p.outputs[0].reg = 1;
        p.outputs[0].raw = 1;
        ++b->launches;
        result = m3c_launch_ew(&p, b->stream);
    }
    *data = *temporary;
    return result;
}

/* The NaN check of a SOFTMAX / TOP_K input (dense rows), recorded against
 * `command`, visiting the rows in the reverse of the order the row pass
 * `p` reads them, so that its first reads hit L2. */
static int scan_rows(cuda_backend *b, const m3c_softmax_params *p, uint32_t command)
{
    ++b->launches;
    return m3c_launch_row_scan(p->input, p->in_dtype, p->rows, p->width,
                               m3c_softmax_row_ranges(p), 0, command, b->status,
                               b->stream);
}

static int run_command(cuda_backend *b, const m3_command *c, uint32_t index,
                       void **temporary)
{
    const m3_tensor_metadata *space;
    int code = 0;

    switch ((int)c->kind) {
    case M3_OP_COPY:
        space = &c->descriptor.copy.output->metadata;
        return launch_unary_ew(b, index, M3C_OP_MOV, c->descriptor.copy.input,
                               NULL, c->descriptor.copy.output, 0, space);
    case M3_OP_CAST: {
        const m3_tensor_view *in = c->descriptor.cast.input;
        const m3_tensor_view *out = c->descriptor.cast.output;

        space = &out->metadata;
        if (in->metadata.dtype == out->metadata.dtype) {
            return launch_unary_ew(b, index, M3C_OP_MOV, in, NULL, out, 0,
                                   space);
        }
        if (in->metadata.dtype == M3_DTYPE_I32) {
            return launch_unary_ew(b, index, M3C_OP_I2F, in, NULL, out, 0,
                                   space);
        }
        if (out->metadata.dtype == M3_DTYPE_I32) {
            const void *data;
            code = dense_input(b, in, index, &data, temporary);
            if (code == 0) {
                ++b->launches;
                code = m3c_launch_scan(data, (int32_t)in->metadata.dtype,
                                       in->metadata.element_count, 1, index,
                                       b->status, b->stream);
            }
            if (code == 0) {
                code = launch_unary_ew(b, index, M3C_OP_F2I, in, NULL, out, 0,
                                       space);
            }
            return code;
        }
        return launch_unary_ew(b, index, M3C_OP_ROUND, in, NULL, out, 0,
                               space);
    }
    case M3_OP_ADD:
    case M3_OP_MUL:
    case M3_OP_GATED_SILU: {
        const m3_op_binary *op = &c->descriptor.add;
        uint8_t opcode = c->kind == M3_OP_ADD   ? M3C_OP_ADD
                         : c->kind == M3_OP_MUL ? M3C_OP_MUL
                                                : M3C_OP_GSILU;

        return launch_unary_ew(b, index, opcode, op->left, op->right,
                               op->output, (int)op->left->metadata.dtype,
                               &op->output->metadata);
    }
    case M3_OP_SNAKE1D:
        return launch_unary_ew(b, index, M3C_OP_SNAKE,
                               c->descriptor.snake1d.input,
                               c->descriptor.snake1d.alpha,
                               c->descriptor.snake1d.output, 0,
                               &c->descriptor.snake1d.output->metadata);
    case M3_OP_TANH:
        return launch_unary_ew(b, index, M3C_OP_TANH, c->descriptor.tanh.input,
                               NULL, c->descriptor.tanh.output, 0,
                               &c->descriptor.tanh.output->metadata);
    case (int)M3_OP_CLAMP_UNIT:
        return launch_unary_ew(b, index, M3C_OP_CLAMP, c->descriptor.copy.input,
                               NULL, c->descriptor.copy.output, 0,
                               &c->descriptor.copy.output->metadata);
    case (int)M3_OP_ABS_MAX:
        return launch_unary_ew(b, index, M3C_OP_ABSMAX, c->descriptor.copy.input,
                               NULL, c->descriptor.copy.output, 0,
                               &c->descriptor.copy.input->metadata);
    case M3_OP_SOFTMAX:
    case M3_OP_TOP_K: {
        const m3_tensor_view *in = c->kind == M3_OP_SOFTMAX
                                       ? c->descriptor.softmax.input
                                       : c->descriptor.top_k.logits;
        m3c_softmax_params p;
        const void *data;

        code = dense_input(b, in, index, &data, temporary);
        if (code != 0) {
            return code;
        }
        memset(&p, 0, sizeof(p));
        p.input = data;
        p.in_dtype = (int32_t)in->metadata.dtype;
        p.width = in->metadata.shape[in->metadata.rank - 1U];
        p.rows = p.width ? in->metadata.element_count / p.width : 0U;
        p.status = b->status;
        p.softmax_command = UINT32_MAX;
        p.skip_before = index + 1U;     /* after the NaN scan of this command */
        p.topk_command = UINT32_MAX;
        if (c->kind == M3_OP_SOFTMAX) {
            p.probs = view_base(b, c->descriptor.softmax.output) +
                      c->descriptor.softmax.output->byte_offset;
            p.probs_dtype = (int32_t)c->descriptor.softmax.output->metadata.dtype;
            p.softmax_command = index;
        } else {
            p.top_values = (float *)(view_base(b, c->descriptor.top_k.values) +
                                     c->descriptor.top_k.values->byte_offset);
            p.top_indices =
                (int32_t *)(view_base(b, c->descriptor.top_k.indices) +
                            c->descriptor.top_k.indices->byte_offset);
            p.k = c->descriptor.top_k.k;
            p.topk_command = index;
        }
        code = scan_rows(b, &p, index);
        if (code != 0) {
            return code;
        }
        ++b->launches;
        return m3c_launch_softmax(&p, b->stream);
    }
    case (int)M3_OP_ROW_SUM: {
        const m3_tensor_view *in = c->descriptor.copy.input;
        m3c_softmax_params p;
        const void *data;

        code = dense_input(b, in, index, &data, temporary);
        if (code != 0) {
            return code;
        }
        memset(&p, 0, sizeof(p));
        p.input = data;
        p.in_dtype = (int32_t)in->metadata.dtype;
        p.width = in->metadata.shape[in->metadata.rank - 1U];
        p.rows = p.width ? in->metadata.element_count / p.width : 0U;
        p.status = b->status;
        p.softmax_command = UINT32_MAX;
        p.topk_command = UINT32_MAX;
        p.skip_before = index;
        p.row_sums = (float *)(view_base(b, c->descriptor.copy.output) +
                               c->descriptor.copy.output->byte_offset);
        p.rowsum_command = index;
        if (p.width == 0U) {
            /* empty rows sum to +0 */
            return (int)cudaMemsetAsync(p.row_sums, 0,
                                        c->descriptor.copy.output->metadata.byte_count,
                                        b->stream);
        }
        ++b->launches;
        return m3c_launch_softmax(&p, b->stream);
    }
    case M3_OP_CATEGORICAL: {
        const m3_tensor_view *probabilities = c->descriptor.categorical.probabilities;
        const m3_tensor_view *uniforms = c->descriptor.categorical.uniforms;
        m3c_categorical_params p;
        const void *data;

        if (!m3c_contiguous(&uniforms->metadata, uniforms->byte_strides)) {
            return -1;  /* strided uniforms are not supported */
        }
        code = dense_input(b, probabilities, index, &data, temporary);
        if (code != 0) {
            return code;
        }
        memset(&p, 0, sizeof(p));
        p.probabilities = data;
        p.probabilities_dtype = (int32_t)probabilities->metadata.dtype;
        p.uniforms = view_base(b, uniforms) + uniforms->byte_offset;
        p.uniforms_dtype = (int32_t)uniforms->metadata.dtype;
        p.output = (int32_t *)(view_base(b, c->descriptor.categorical.output) +
                               c->descriptor.categorical.output->byte_offset);
        p.width = probabilities->metadata.shape[probabilities->metadata.rank - 1U];
        p.rows = p.width ? probabilities->metadata.element_count / p.width : 0U;
        p.status = b->status;
        p.command = index;
        /* the checks of every row first, then the draws, which run only
         * when no row failed: a failing command writes nothing */
        p.skip_before = index;
        p.check_only = 1;
        b->launches += 2U;
        code = m3c_launch_categorical(&p, b->stream);
        if (code == 0) {
            p.skip_before = index + 1U;
            p.check_only = 0;
            code = m3c_launch_categorical(&p, b->stream);
        }
        return code;
    }
    case M3_OP_RMS_NORM:
    case M3_OP_LAYER_NORM: {
        bool layer = c->kind == M3_OP_LAYER_NORM;
        const m3_tensor_view *in = layer ? c->descriptor.layer_norm.input
                                         : c->descriptor.rms_norm.input;
        const m3_tensor_view *scale = layer ? c->descriptor.layer_norm.scale
                                            : c->descriptor.rms_norm.scale;
        const m3_tensor_view *bias = layer ? c->descriptor.layer_norm.bias : NULL;
        const m3_tensor_view *out = layer ? c->descriptor.layer_norm.output
                                          : c->descriptor.rms_norm.output;
        m3c_norm_params p;
        const void *data;

        if ((scale->metadata.element_count > 1U &&
             scale->byte_strides[0] != m3c_dtype_size(scale->metadata.dtype)) ||
            (bias != NULL && bias->metadata.element_count > 1U &&
             bias->byte_strides[0] != m3c_dtype_size(bias->metadata.dtype))) {
            return -1;  /* strided norm vectors are not supported */
        }
        code = dense_input(b, in, index, &data, temporary);
        if (code != 0) {
            return code;
        }
        memset(&p, 0, sizeof(p));
        p.x = data;
        p.in_dtype = (int32_t)in->metadata.dtype;
        p.scale = view_base(b, scale) + scale->byte_offset;
        p.scale_dtype = (int32_t)scale->metadata.dtype;
        if (bias != NULL) {
            p.bias = view_base(b, bias) + bias->byte_offset;
            p.bias_dtype = (int32_t)bias->metadata.dtype;
        }
        p.layer_norm = layer ? 1 : 0;
        p.out = view_base(b, out) + out->byte_offset;
        p.out_dtype = (int32_t)out->metadata.dtype;
        p.width = in->metadata.shape[in->metadata.rank - 1U];
        p.rows = p.width ? in->metadata.element_count / p.width : 0U;
        p.skip_before = index;
        p.epsilon = layer ? c->descriptor.layer_norm.epsilon
                          : c->descriptor.rms_norm.epsilon;
        p.status = b->status;
        ++b->launches;
        return m3c_launch_norm(&p, b->stream);
    }
    default:
        return -1;
    }
}

/* ------------------------------------------------------- fused launches */

static bool same_view(const m3_tensor_view *x, const m3_tensor_view *y)
{
    uint8_t d;

    if (x->storage != y->storage || x->byte_offset != y->byte_offset ||
        x->metadata.dtype != y->metadata.dtype ||
        x->metadata.rank != y->metadata.rank) {
        return false;
    }
    for (d = 0U; d < x->metadata.rank; ++d) {
        if (x->metadata.shape[d] != y->metadata.shape[d] ||
            (x->metadata.shape[d] > 1U &&
             x->byte_strides[d] != y->byte_strides[d])) {
            return false;
        }
    }
    return true;
}

static bool same_shape(const m3_tensor_metadata *x, const m3_tensor_metadata *y)
{
    uint8_t d;

    if (x->rank != y->rank) {
        return false;
    }
    for (d = 0U; d < x->rank; ++d) {
        if (x->shape[d] != y->shape[d]) {
            return false;
        }
    }
    return true;
}

/* Do the byte ranges two views can touch intersect? */
static bool views_overlap(const cuda_backend *b, const m3_tensor_view *x,
                          const m3_tensor_view *y)
{
    const m3_tensor_view *v[2] = {x, y};
    uintptr_t lo[2];
    uintptr_t hi[2];
    int k;

    for (k = 0; k < 2; ++k) {
        size_t extent = m3c_dtype_size(v[k]->metadata.dtype);
        uint8_t d;

        lo[k] = (uintptr_t)view_base(b, v[k]) + v[k]->byte_offset;
        if (v[k]->metadata.element_count == 0U) {
            hi[k] = lo[k];
            continue;
        }
        for (d = 0U; d < v[k]->metadata.rank; ++d) {
            extent += (size_t)(v[k]->metadata.shape[d] - 1U) * v[k]->byte_strides[d];
        }
        hi[k] = lo[k] + extent;
    }
    return lo[0] < hi[1] && lo[1] < hi[0];
}

/* An element-wise command without a data check, as one micro-op. */
typedef struct {
    uint8_t code;
    int n_in;
    const m3_tensor_view *in[2];
    const m3_tensor_view *out;
    int aux;
} ew_step;

static bool ew_step_of(const m3_command *c, ew_step *step)
{
    memset(step, 0, sizeof(*step));
    switch ((int)c->kind) {
    case M3_OP_COPY:
        step->code = M3C_OP_MOV;
        step->in[0] = c->descriptor.copy.input;
        step->out = c->descriptor.copy.output;
        break;
    case M3_OP_CAST: {
        const m3_tensor_view *in = c->descriptor.cast.input;
        const m3_tensor_view *out = c->descriptor.cast.output;

        if (out->metadata.dtype == M3_DTYPE_I32 &&
            in->metadata.dtype != M3_DTYPE_I32) {
            return false;  /* range-checked: runs on its own */
        }
        step->code = in->metadata.dtype == out->metadata.dtype ? M3C_OP_MOV
                     : in->metadata.dtype == M3_DTYPE_I32      ? M3C_OP_I2F
                                                               : M3C_OP_ROUND;
        step->in[0] = in;
        step->out = out;
        break;
    }
    case M3_OP_ADD:
    case M3_OP_MUL:
    case M3_OP_GATED_SILU:
        step->code = c->kind == M3_OP_ADD   ? M3C_OP_ADD
                     : c->kind == M3_OP_MUL ? M3C_OP_MUL
                                            : M3C_OP_GSILU;
        step->in[0] = c->descriptor.add.left;
        step->in[1] = c->descriptor.add.right;
        step->out = c->descriptor.add.output;
        step->aux = (int)c->descriptor.add.left->metadata.dtype;
        break;
    case M3_OP_SNAKE1D:
        step->code = M3C_OP_SNAKE;
        step->in[0] = c->descriptor.snake1d.input;
        step->in[1] = c->descriptor.snake1d.alpha;
        step->out = c->descriptor.snake1d.output;
        break;
    case M3_OP_TANH:
        step->code = M3C_OP_TANH;
        step->in[0] = c->descriptor.tanh.input;
        step->out = c->descriptor.tanh.output;
        break;
    case (int)M3_OP_CLAMP_UNIT:
        step->code = M3C_OP_CLAMP;
        step->in[0] = c->descriptor.copy.input;
        step->out = c->descriptor.copy.output;
        break;
    default:
        return false;
    }
    step->n_in = step->in[1] != NULL ? 2 : 1;
    return true;
}

static bool is_16bit(const m3_tensor_view *v)
{
    return v->metadata.dtype == M3_DTYPE_F16 || v->metadata.dtype == M3_DTYPE_BF16;
}

/* Merge commands [first, first + *count) of the list into one element-wise
 * launch (*count >= 2 on success; 0: nothing merged).  A command joins when
 * it has no data check, its output has the group's shape, and it cannot race
 * with the group:
 *   - an input that is exactly an earlier member's output view is taken from
 *     that member's register, which holds the value rounded to its stored
 *     dtype (what the reference reloads); an input that only partly overlaps
 *     a member's output ends the group;
 *   - its output, where it overlaps a member's memory input or output (or its
 *     own memory input), is exactly that view and contiguous, so each element
 *     is read and written by the thread that owns its index, in command
 *     order.
 * Copies move raw words: a copy reads memory only, and only F32 copies feed
 * later members. */
static int fuse_ew(cuda_backend *b, const m3_command *commands, size_t first,
                   size_t available, size_t *count)
{
    enum { MAXSTEPS = 8 };
    ew_step steps[MAXSTEPS];
    const m3_tensor_view *loaded[M3C_EW_MAX_OPERANDS];
    int source[MAXSTEPS][2];   /* >= 0: operand index; < 0: -(member + 1) */
    int reg_of_step[MAXSTEPS];
    int reg_of_operand[M3C_EW_MAX_OPERANDS];
    int n_loaded = 0;
    int n_widen = 0;           /* registers reserved for widened operands */
    size_t n = 0U;
    size_t k;
    int next_reg;
    int n_out;
    m3c_ew_params p;

    *count = 0U;
    while (n < MAXSTEPS && first + n < available) {
        ew_step st;
        int in_src[2] = {0, 0};
        int new_loads = 0;
        int new_widen = 0;
        bool ok = true;
        int i;
        size_t m;

        if (!ew_step_of(&commands[first + n], &st) ||
            (n > 0U && !same_shape(&st.out->metadata, &steps[0].out->metadata))) {
            break;
        }
        for (i = 0; i < st.n_in && ok; ++i) {
            int found = INT32_MIN;

            /* the latest member that wrote exactly this view */
            for (m = n; m-- > 0U;) {
                if (same_view(st.in[i], steps[m].out)) {
                    found = -(int)m - 1;
                    break;
                }
            }
            if (found != INT32_MIN) {
                const ew_step *w = &steps[-found - 1];

                if (st.code == M3C_OP_MOV ||
                    (w->code == M3C_OP_MOV && w->out->metadata.dtype != M3_DTYPE_F32)) {
                    ok = false;
                }
                in_src[i] = found;
                continue;
            }
            for (m = 0U; m < n; ++m) {
                if (views_overlap(b, st.in[i], steps[m].out)) {
                    ok = false;  /* part of a member's output */
                }
            }
            for (m = 0U; m < (size_t)n_loaded && found == INT32_MIN; ++m) {
                if (same_view(st.in[i], loaded[m])) {
                    found = (int)m;
                }
            }
            if (found == INT32_MIN && i == 1 && in_src[0] >= n_loaded &&
                same_view(st.in[1], st.in[0])) {
                found = in_src[0];  /* both inputs one new operand */
            }
            if (found == INT32_MIN) {
                if (n_loaded + new_loads >= M3C_EW_MAX_OPERANDS) {
                    ok = false;
                    break;
                }
                found = n_loaded + new_loads++;
                if (is_16bit(st.in[i])) {
                    ++new_widen;
                }
            }
            in_src[i] = found;
        }
        if (ok) {
            const m3_tensor_view *out = st.out;
            bool dense = m3c_contiguous(&out->metadata, out->byte_strides);

            for (m = 0U; m < (size_t)n_loaded && ok; ++m) {
                if (views_overlap(b, out, loaded[m]) && !(dense && same_view(out, loaded[m]))) {
                    ok = false;
                }
            }
            for (i = 0; i < st.n_in && ok; ++i) {
                if (in_src[i] >= n_loaded && views_overlap(b, out, st.in[i]) &&
                    !(dense && same_view(out, st.in[i]))) {
                    ok = false;
                }
            }
            for (m = 0U; m < n && ok; ++m) {
                if (views_overlap(b, out, steps[m].out) && !(dense && same_view(out, steps[m].out))) {
                    ok = false;
                }
            }
        }
        if (!ok || n_loaded + new_loads + n_widen + new_widen + (int)n + 1 > M3C_EW_MAX_REGS ||
            n_widen + new_widen + (int)n + 1 > M3C_EW_MAX_OPS) {
            break;
        }
        for (i = 0; i < st.n_in; ++i) {
            if (in_src[i] >= n_loaded) {
                loaded[n_loaded] = st.in[i];
                in_src[i] = n_loaded++;
            }
        }
        n_widen += new_widen;
        source[n][0] = in_src[0];
        source[n][1] = st.n_in == 2 ? in_src[1] : in_src[0];
        steps[n++] = st;
    }
    if (n < 2U) {
        return 0;
    }
    /* registers: the loaded operands, their widened copies, one per member */
    memset(&p, 0, sizeof(p));
    p.count = steps[0].out->metadata.element_count;
    p.status = b->status;
    p.skip_before = (uint32_t)first;
    p.n_operands = n_loaded;
    next_reg = n_loaded;
    for (k = 0U; k < (size_t)n_loaded; ++k) {
        const m3_tensor_view *v = loaded[k];
        bool read_as_float = false;
        size_t s;
        int i;

        for (s = 0U; s < n; ++s) {
            for (i = 0; i < steps[s].n_in; ++i) {
                if (source[s][i] == (int)k && steps[s].code != M3C_OP_MOV) {
                    read_as_float = true;
                }
            }
        }
        m3c_operand_setup(&p.operands[k], view_base(b, v), &v->metadata, v->byte_offset,
                          v->byte_strides, &steps[0].out->metadata,
                          v->metadata.dtype == M3_DTYPE_I32 ? M3C_LOAD_INT : M3C_LOAD_RAW);
        reg_of_operand[k] = (int)k;
        if (read_as_float && is_16bit(v)) {
            m3c_ew_op *op = &p.ops[p.n_ops++];

            op->code = M3C_OP_WIDEN;
            op->dst = (uint8_t)next_reg;
            op->a = (uint8_t)k;
            op->b = (uint8_t)k;
            op->rdtype = M3C_F32;
            op->aux = (int8_t)v->metadata.dtype;
            op->command = (uint16_t)first;
            reg_of_operand[k] = next_reg++;
        }
    }
    for (k = 0U; k < n; ++k) {
        m3c_ew_op *op = &p.ops[p.n_ops++];
        int r[2];
        int i;

        for (i = 0; i < 2; ++i) {
            int src = source[k][i];

            if (src < 0) {
                r[i] = reg_of_step[-src - 1];
            } else {
                r[i] = steps[k].code == M3C_OP_MOV ? src : reg_of_operand[src];
            }
        }
        op->code = steps[k].code;
        op->a = (uint8_t)r[0];
        op->b = (uint8_t)r[1];
        op->dst = (uint8_t)next_reg;
        op->rdtype = (int8_t)steps[k].out->metadata.dtype;
        op->aux = (int8_t)steps[k].aux;
        op->command = (uint16_t)(first + k);
        reg_of_step[k] = next_reg++;
    }
    /* every output view is stored once, from its last writer in the group */
    n_out = 0;
    for (k = 0U; k < n; ++k) {
        const m3_tensor_view *out = steps[k].out;
        size_t vector_bytes = 4U * m3c_dtype_size(out->metadata.dtype);
        bool overwritten = false;
        size_t later;
        m3c_ew_out *o;

        for (later = k + 1U; later < n; ++later) {
            if (same_view(out, steps[later].out)) {
                overwritten = true;
            }
        }
        if (overwritten) {
            continue;
        }
        if (n_out == M3C_EW_MAX_OUTPUTS) {
            return 0;  /* nothing launched: the commands run one by one */
        }
        o = &p.outputs[n_out++];
        o->base = view_base(b, out) + out->byte_offset;
        o->dtype = (int32_t)out->metadata.dtype;
        o->reg = (int16_t)reg_of_step[k];
        o->scalar_only = ((uintptr_t)o->base % vector_bytes) != 0U ? 1U : 0U;
        o->raw = (steps[k].code == M3C_OP_MOV && m3c_dtype_size(out->metadata.dtype) == 2U) ? 1 : 0;
    }
    p.n_outputs = n_out;
    *count = n;
    ++b->launches;
    return m3c_launch_ew(&p, b->stream);
}

/* Merge SOFTMAX / TOP_K / ROW_SUM commands [first, first + *count) over one
 * input view into one NaN scan and one row pass (*count >= 2 on success).
 * The data-checked commands (SOFTMAX, TOP_K) come first: a ROW_SUM ahead of
 * a failing check would have been written by the reference, so it runs on
 * its own.  No member's output may overlap the input or another member's
 * output. */
static int fuse_rows(cuda_backend *b, const m3_command *commands, size_t first,
                     size_t available, size_t *count, void **temporary)
{
    const m3_tensor_view *in = NULL;
    const m3_tensor_view *outs[6];
    int n_outs = 0;
    size_t n = 0U;
    size_t softmax = SIZE_MAX;
    size_t topk = SIZE_MAX;
    size_t rowsum = SIZE_MAX;
    m3c_softmax_params p;
    const void *data;
    int code;

    *count = 0U;
    while (first + n < available) {
        const m3_command *c = &commands[first + n];
        const m3_tensor_view *cin;
        const m3_tensor_view *cout[2] = {NULL, NULL};
        bool ok = true;
        int i;

        if (c->kind == M3_OP_SOFTMAX && softmax == SIZE_MAX && rowsum == SIZE_MAX) {
            cin = c->descriptor.softmax.input;
            cout[0] = c->descriptor.softmax.output;
        } else if (c->kind == M3_OP_TOP_K && topk == SIZE_MAX && rowsum == SIZE_MAX) {
            cin = c->descriptor.top_k.logits;
            cout[0] = c->descriptor.top_k.values;
            cout[1] = c->descriptor.top_k.indices;
        } else if ((int)c->kind == (int)M3_OP_ROW_SUM && rowsum == SIZE_MAX && n > 0U) {
            cin = c->descriptor.copy.input;
            cout[0] = c->descriptor.copy.output;
        } else {
            break;
        }
        if (in != NULL && !same_view(cin, in)) {
            break;
        }
        for (i = 0; i < 2 && cout[i] != NULL && ok; ++i) {
            int j;

            if (views_overlap(b, cout[i], cin)) {
                ok = false;
            }
            for (j = 0; j < n_outs; ++j) {
                if (views_overlap(b, cout[i], outs[j])) {
                    ok = false;
                }
            }
        }
        if (!ok) {
            break;
        }
        in = cin;
        for (i = 0; i < 2 && cout[i] != NULL; ++i) {
            outs[n_outs++] = cout[i];
        }
        if (c->kind == M3_OP_SOFTMAX) {
            softmax = first + n;
        } else if (c->kind == M3_OP_TOP_K) {
            topk = first + n;
        } else {
            rowsum = first + n;
        }
        ++n;
    }
    if (n < 2U || in->metadata.shape[in->metadata.rank - 1U] == 0U) {
        return 0;
    }
    code = dense_input(b, in, (uint32_t)first, &data, temporary);
    if (code != 0) {
        return code;
    }
    memset(&p, 0, sizeof(p));
    p.input = data;
    p.in_dtype = (int32_t)in->metadata.dtype;
    p.width = in->metadata.shape[in->metadata.rank - 1U];
    p.rows = in->metadata.element_count / p.width;
    p.status = b->status;
    p.skip_before = (uint32_t)first + 1U;
    p.softmax_command = UINT32_MAX;
    p.topk_command = UINT32_MAX;
    p.rowsum_command = UINT32_MAX;
    if (softmax != SIZE_MAX) {
        const m3_tensor_view *out = commands[softmax].descriptor.softmax.output;

        p.probs = view_base(b, out) + out->byte_offset;
        p.probs_dtype = (int32_t)out->metadata.dtype;
        p.softmax_command = (uint32_t)softmax;
    }
    if (topk != SIZE_MAX) {
        const m3_op_top_k *t = &commands[topk].descriptor.top_k;

        p.top_values = (float *)(view_base(b, t->values) + t->values->byte_offset);
        p.top_indices = (int32_t *)(view_base(b, t->indices) + t->indices->byte_offset);
        p.k = t->k;
        p.topk_command = (uint32_t)topk;
    }
    if (rowsum != SIZE_MAX) {
        const m3_tensor_view *out = commands[rowsum].descriptor.copy.output;

        p.row_sums = (float *)(view_base(b, out) + out->byte_offset);
        p.rowsum_command = (uint32_t)rowsum;
    }
    /* the NaN check, reported against the group's first (checked) command */
    code = scan_rows(b, &p, (uint32_t)first);
    if (code != 0) {
        return code;
    }
    *count = n;
    ++b->launches;
    return m3c_launch_softmax(&p, b->stream);
}

static const char *check_message(m3_op_kind kind, uint32_t detail)
{
    switch ((int)kind) {
    case M3_OP_CATEGORICAL:
        return m3c_categorical_message(detail);
    case M3_OP_SOFTMAX:
        return "softmax input contains NaN";
    case M3_OP_TOP_K:
        return "top-k logits contain NaN";
    case M3_OP_CAST:
        return "float-to-I32 cast value is invalid";
    default:
        return "abs-max input contains NaN";
    }
}

m3_status m3_cuda_backend_execute(void *context, const m3_command *commands,
                                  size_t command_count,
                                  m3_scratch_arena *scratch, m3_error *error)
{
    cuda_backend *b = context;
    void **temporaries;
    size_t i;
    m3_status status = M3_STATUS_OK;
    cudaError_t code;

    (void)scratch;
    if (b == NULL || (command_count != 0U && commands == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "backend and commands are required");
    }
    for (i = 0U; i < command_count; ++i) {
        m3c_vcommand v;

        to_vcommand(&commands[i], &v);
        status = m3c_validate(&v, error);
        if (status != M3_STATUS_OK) {
            return status;
        }
    }
    temporaries = calloc(command_count ? command_count : 1U, sizeof(void *));
    if (temporaries == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate execution state");
    }
    (void)cudaSetDevice(b->device);
    b->launches = 0U;
    for (i = 0U; i < command_count;) {
        size_t merged = 0U;
        size_t failing = i;
        int result = fuse_ew(b, commands, i, command_count, &merged);

        if (result == 0 && merged == 0U) {
            result = fuse_rows(b, commands, i, command_count, &merged,
                               &temporaries[i]);
        }
        if (result == 0 && merged == 0U) {
            result = run_command(b, &commands[i], (uint32_t)i, &temporaries[i]);
            merged = 1U;
        }
        i += merged;
        if (result != 0) {
            i = failing;
            status = m3c_error_set(
                error, result < 0 ? M3_STATUS_UNSUPPORTED : M3_STATUS_INTERNAL,
                "CUDA execution of %s failed: %s",
                m3c_kind_name(commands[i].kind),
                result < 0 ? "unsupported view layout"
                           : m3c_cuda_error_string(result));
            break;
        }
    }
    free(temporaries);
    code = cudaMemcpyAsync(b->status_host, b->status, sizeof(m3c_status),
                           cudaMemcpyDeviceToHost, b->stream);
    if (code == cudaSuccess) {
        code = cudaStreamSynchronize(b->stream);
    }
    if (code != cudaSuccess) {
        return fail_cuda(error, code, "CUDA execution failed");
    }
    if (b->status_host->fail_command != UINT32_MAX) {
        uint32_t failing = b->status_host->fail_command;

        code = cudaMemcpy(b->status, &clean, sizeof(clean),
                          cudaMemcpyHostToDevice);
        if (code != cudaSuccess) {
            return fail_cuda(error, code, "cannot reset backend status");
        }
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE, "%s",
                             check_message(commands[failing].kind,
                                           b->status_host->detail));
    }
    if (status == M3_STATUS_OK) {
        m3_error_reset(error);
    }
    return status;
}

unsigned m3_cuda_backend_launch_count(const void *context)
{
    const cuda_backend *b = context;

    return b == NULL ? 0U : b->launches;
}

m3_status m3_cuda_backend_set_stream(void *context, void *stream, m3_error *error)
{
    cuda_backend *b = context;
    cudaError_t code;

    if (b == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "backend context is required");
    }
    (void)cudaSetDevice(b->device);
    /* work already queued on the old stream finishes first */
    code = cudaStreamSynchronize(b->stream);
    if (code != cudaSuccess) {
        return fail_cuda(error, code, "cannot switch the backend stream");
    }
    b->stream = stream != NULL ? (cudaStream_t)stream : b->own_stream;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

void *m3_cuda_storage_is_address(m3_storage *storage)
{
    return (void *)storage;
}
