/* Sharding layer: one fixed graph split across the GPUs of a box, one
 * process (and one session, one device arena) per GPU.
 *
 * Partition.  The split axis is an axis of the "primary" value, the first
 * graph input of largest rank (a constant if the graph has no input of that
 * rank).  Every other value is right-aligned against the primary's shape, as
 * broadcasting aligns operands: at the aligned position a value either has
 * the primary's extent (it is split: this rank keeps the slab
 * [begin, begin + extent) of that axis), or extent 1, or no such axis (it is
 * replicated).  Any other extent there makes the axis unusable.  Row
 * operators reduce their input's last axis, which must therefore not be the
 * split axis; their per-row outputs keep the input's rank and split with it.
 * ABS_MAX reduces everything: its one-element output is replicated and
 * combined across ranks after each run (m3c_session.c), so it may not feed
 * another node.  CATEGORICAL drops an axis of its input, which right
 * alignment cannot place, and is not sharded.
 *
 * Slabs are balanced: in whole blocks of 4 elements when the extent is a
 * multiple of 4 and at least 4 per rank (so vectorised kernels keep full
 * blocks), else in single elements; the first ranks take one unit more.
 *
 * Each rank's session is an ordinary session of the LOCAL graph (the same
 * nodes over the slab shapes, constants sliced), so planning, fusion and
 * kernels are those of a single GPU; the sharded parts are the partition,
 * the slab I/O and the per-run agreement of the ranks. */

#include "m3c_internal.h"

#include <cuda_runtime_api.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

void m3_cuda_shard_options_init(m3_cuda_shard_options *options)
{
    if (options != NULL) {
        options->rank = 0;
        options->count = 1;
        options->axis = M3_CUDA_SHARD_AXIS_AUTO;
        options->id = NULL;
        options->timeout_seconds = 120.0;
    }
}

bool m3c_shard_collective(const m3c_shard *shard)
{
    return shard != NULL && shard->comm != NULL &&
           (shard->reduction_count > 0 || shard->checks);
}

void m3c_shard_free(m3c_shard *shard)
{
    if (shard != NULL) {
        free(shard->slabs);
        free(shard);
    }
}

static bool row_reducing(m3_op_kind kind)
{
    switch ((int)kind) {
    case M3_OP_SOFTMAX:
    case M3_OP_TOP_K:
    case M3_OP_RMS_NORM:
    case M3_OP_LAYER_NORM:
    case (int)M3_OP_ROW_SUM:
        return true;
    default:
        return false;
    }
}

static bool data_checked(const m3_graph *graph, const m3_graph_node_desc *node)
{
    switch ((int)node->kind) {
    case M3_OP_SOFTMAX:
    case M3_OP_TOP_K:
    case (int)M3_OP_ABS_MAX:
    case M3_OP_CATEGORICAL:
        return true;
    case M3_OP_CAST:
        return node->outputs[0] < graph->value_count &&
               graph->values[node->outputs[0]].metadata.dtype == M3_DTYPE_I32 &&
               node->inputs[0] < graph->value_count &&
               graph->values[node->inputs[0]].metadata.dtype != M3_DTYPE_I32;
    default:
        return false;
    }
}

/* The primary value: first INPUT of largest rank, else first CONSTANT of
 * largest rank (SIZE_MAX: none). */
static size_t primary_value(const m3_graph *graph)
{
    size_t best = SIZE_MAX;
    size_t v;
    int pass;

    for (pass = 0; pass < 2 && best == SIZE_MAX; ++pass) {
        m3_graph_value_role role = pass == 0 ? M3_GRAPH_INPUT : M3_GRAPH_CONSTANT;

        for (v = 0U; v < graph->value_count; ++v) {
            if (graph->values[v].description.role == role &&
                (best == SIZE_MAX ||
                 graph->values[v].metadata.rank > graph->values[best].metadata.rank)) {
                best = v;
            }
        }
    }
    return best;
}

/* Position of the split axis in value v (right-aligned), or -1. */
static int aligned_axis(const m3_tensor_metadata *value, int primary_rank,
                        int axis)
{
    int position = axis - (primary_rank - (int)value->rank);

    return position >= 0 && position < (int)value->rank ? position : -1;
}

/* Whether `axis` can split `graph`; on failure, why (into `why`). */
static bool axis_allowed(const m3_graph *graph, size_t primary, int axis,
                         int count, char *why, size_t why_size)
{
    const m3_tensor_metadata *p = &graph->values[primary].metadata;
    uint64_t extent = p->shape[axis];
    size_t v;
    size_t n;

    if (extent < (uint64_t)count) {
        snprintf(why, why_size, "axis %d has extent %llu, fewer than %d shards",
                 axis, (unsigned long long)extent, count);
        return false;
    }
    for (v = 0U; v < graph->value_count; ++v) {
        const m3_tensor_metadata *m = &graph->values[v].metadata;
        int position = aligned_axis(m, (int)p->rank, axis);

        if (position >= 0 && m->shape[position] != extent &&
            m->shape[position] != 1U) {
            snprintf(why, why_size,
                     "value %zu has extent %llu on the split axis (neither %llu nor 1)",
                     v, (unsigned long long)m->shape[position],
                     (unsigned long long)extent);
            return false;
        }
    }
    for (n = 0U; n < graph->node_count; ++n) {
        const m3_graph_node_desc *node = &graph->nodes[n];

        if (node->kind == M3_OP_CATEGORICAL) {
            snprintf(why, why_size, "CATEGORICAL (node %zu) cannot be sharded", n);
            return false;
        }
        if (row_reducing(node->kind) && node->inputs[0] < graph->value_count) {
            const m3_tensor_metadata *in = &graph->values[node->inputs[0]].metadata;
            int position = aligned_axis(in, (int)p->rank, axis);

            if (position >= 0 && position == (int)in->rank - 1 &&
                in->shape[position] == extent && extent != 1U) {
                snprintf(why, why_size,
                         "node %zu reduces the split axis (its rows' last axis)", n);
                return false;
            }
        }
    }
    return true;
}

static void slab_range(uint64_t extent, int rank, int count, uint64_t *begin,
                       uint64_t *length)
{
    uint64_t unit = (extent % 4U == 0U && extent >= 4U * (uint64_t)count) ? 4U : 1U;
    uint64_t units = extent / unit;
    uint64_t per = units / (uint64_t)count;
    uint64_t extra = units % (uint64_t)count;
    uint64_t r = (uint64_t)rank;

    *begin = (r * per + (r < extra ? r : extra)) * unit;
    *length = (per + (r < extra ? 1U : 0U)) * unit;
}

/* Slabs of every value for `options`; chooses the axis when asked. */
static m3_status partition(const m3_graph *graph,
                           const m3_cuda_shard_options *options,
                           m3_cuda_shard_slab *slabs, int *axis_out,
                           m3_error *error)
{
    size_t primary;
    const m3_tensor_metadata *p;
    int axis = options->axis;
    char why[160] = "";
    size_t v;

    if (options->count < 1 || options->rank < 0 ||
        options->rank >= options->count) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "shard rank %d of %d is invalid", options->rank,
                             options->count);
    }
    primary = primary_value(graph);
    if (primary == SIZE_MAX || graph->values[primary].metadata.rank == 0U) {
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "a sharded graph needs an input of rank >= 1");
    }
    p = &graph->values[primary].metadata;
    if (axis == M3_CUDA_SHARD_AXIS_AUTO) {
        int candidate;

        axis = -1;
        for (candidate = 0; candidate < (int)p->rank && axis < 0; ++candidate) {
            if (axis_allowed(graph, primary, candidate, options->count, why,
                             sizeof(why))) {
                axis = candidate;
            }
        }
        if (axis < 0) {
            return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                                 "no axis of the graph can be split %d ways",
                                 options->count);
        }
    } else if (axis < 0 || axis >= (int)p->rank) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "shard axis %d is outside rank %u", axis,
                             (unsigned)p->rank);
    } else if (!axis_allowed(graph, primary, axis, options->count, why,
                             sizeof(why))) {
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "cannot split axis %d: %s", axis, why);
    }
    for (v = 0U; v < graph->value_count; ++v) {
        const m3_tensor_metadata *m = &graph->values[v].metadata;
        m3_cuda_shard_slab *slab = &slabs[v];
        int position = aligned_axis(m, (int)p->rank, axis);
        uint64_t shape[M3_TENSOR_MAX_RANK];
        m3_status status;

        memset(slab, 0, sizeof(*slab));
        slab->global = *m;
        slab->local = *m;
        if (position < 0 || m->shape[position] != p->shape[axis] ||
            p->shape[axis] == 1U) {
            continue;   /* replicated */
        }
        slab->split = true;
        slab->axis = (uint8_t)position;
        slab_range(m->shape[position], options->rank, options->count,
                   &slab->begin, &slab->extent);
        memcpy(shape, m->shape, sizeof(shape));
        shape[position] = slab->extent;
        status = m3c_metadata_init(&slab->local, m->dtype, m->rank, shape, error);
        if (status != M3_STATUS_OK) {
            return status;
        }
    }
    for (v = 0U; v < graph->node_count; ++v) {
        const m3_graph_node_desc *node = &graph->nodes[v];
        size_t u;

        if (node->kind != M3_OP_ABS_MAX) {
            continue;
        }
        for (u = 0U; u < graph->node_count; ++u) {
            int k;

            for (k = 0; k < (int)M3_GRAPH_NODE_INPUT_CAPACITY; ++k) {
                if (graph->nodes[u].inputs[k] == node->outputs[0]) {
                    return m3c_error_set(
                        error, M3_STATUS_UNSUPPORTED,
                        "a sharded graph's ABS_MAX result (node %zu) cannot "
                        "feed another node", v);
                }
            }
        }
    }
    if (axis_out != NULL) {
        *axis_out = axis;
    }
    return M3_STATUS_OK;
}

m3_status m3_cuda_shard_plan(const m3_graph *graph,
                             const m3_cuda_shard_options *shard,
                             m3_graph_value_id value, m3_cuda_shard_slab *slab,
                             int *axis_out, m3_error *error)
{
    m3_cuda_shard_slab *slabs;
    m3_status status;

    if (graph == NULL || shard == NULL || slab == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "graph, shard options and slab output are required");
    }
    if ((size_t)value >= graph->value_count) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "shard plan value is out of range");
    }
    slabs = calloc(graph->value_count, sizeof(*slabs));
    if (slabs == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate shard plan");
    }
    status = partition(graph, shard, slabs, axis_out, error);
    if (status == M3_STATUS_OK) {
        *slab = slabs[value];
        m3_error_reset(error);
    }
    free(slabs);
    return status;
}

/* Copy the slab of a dense tensor laid out as `global` (outer x extent x
 * inner elements) out of / into a dense tensor of the slab's shape. */
static void slab_geometry(const m3_cuda_shard_slab *slab, size_t *outer,
                          size_t *row_bytes, size_t *pitch, size_t *offset)
{
    size_t element = m3c_dtype_size(slab->global.dtype);
    size_t inner = 1U;
    size_t before = 1U;
    uint8_t a;

    for (a = 0U; a < slab->global.rank; ++a) {
        if (a < slab->axis) {
            before *= (size_t)slab->global.shape[a];
        } else if (a > slab->axis) {
            inner *= (size_t)slab->global.shape[a];
        }
    }
    *outer = before;
    *row_bytes = (size_t)slab->extent * inner * element;
    *pitch = (size_t)slab->global.shape[slab->axis] * inner * element;
    *offset = (size_t)slab->begin * inner * element;
}

/* The local graph: the global graph's nodes over slab shapes, constants
 * sliced where split. */
static m3_status local_graph(const m3_graph *graph,
                             const m3_cuda_shard_slab *slabs,
                             m3_graph **local, m3_error *error)
{
    m3_graph *g = NULL;
    m3_status status = m3_graph_create(&g, error);
    size_t v;

    for (v = 0U; status == M3_STATUS_OK && v < graph->value_count; ++v) {
        const m3c_graph_value *src = &graph->values[v];
        m3_graph_value_desc d = src->description;
        m3_graph_value_id id;

        memcpy(d.shape, slabs[v].local.shape, sizeof(d.shape));
        status = m3_graph_add_value(g, &d, &id, error);
        if (status == M3_STATUS_OK && src->constant_set) {
            if (!slabs[v].split) {
                status = m3_graph_set_constant(g, id, src->constant_data,
                                               src->constant_size, error);
            } else {
                size_t outer, row, pitch, offset, r;
                unsigned char *part;

                slab_geometry(&slabs[v], &outer, &row, &pitch, &offset);
                part = malloc(outer * row != 0U ? outer * row : 1U);
                if (part == NULL) {
                    status = m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                           "cannot slice a constant");
                    break;
                }
                for (r = 0U; r < outer; ++r) {
                    memcpy(part + r * row,
                           (const unsigned char *)src->constant_data + r * pitch + offset,
                           row);
                }
                status = m3_graph_set_constant(g, id, part, outer * row, error);
                free(part);
            }
        }
    }
    for (v = 0U; status == M3_STATUS_OK && v < graph->node_count; ++v) {
        status = m3_graph_add_node(g, &graph->nodes[v], error);
    }
    if (status != M3_STATUS_OK) {
        m3_graph_free(g);
        return status;
    }
    *local = g;
    return M3_STATUS_OK;
}

m3_status m3_cuda_shard_session_create(m3_session **session,
                                       const m3_graph *graph,
                                       const m3_session_options *options,
                                       const m3_cuda_session_options *cuda,
                                       const m3_cuda_shard_options *shard,
                                       m3_error *error)
{
    m3c_shard *sh;
    m3_graph *local = NULL;
    m3_status status;
    size_t n;

    if (session == NULL || *session != NULL || graph == NULL || shard == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session output must be empty; graph and shard "
                             "options are required");
    }
    sh = calloc(1U, sizeof(*sh));
    if (sh != NULL) {
        sh->slabs = calloc(graph->value_count ? graph->value_count : 1U,
                           sizeof(*sh->slabs));
    }
    if (sh == NULL || sh->slabs == NULL) {
        m3c_shard_free(sh);
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate shard state");
    }
    sh->rank = shard->rank;
    sh->count = shard->count;
    sh->value_count = graph->value_count;
    sh->timeout_seconds = shard->timeout_seconds > 0.0 ? shard->timeout_seconds : 120.0;
    status = partition(graph, shard, sh->slabs, &sh->axis, error);
    for (n = 0U; status == M3_STATUS_OK && n < graph->node_count; ++n) {
        const m3_graph_node_desc *node = &graph->nodes[n];

        sh->checks = sh->checks || data_checked(graph, node);
        if (node->kind == M3_OP_ABS_MAX) {
            if (sh->reduction_count == M3C_SHARD_MAX_REDUCTIONS) {
                status = m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                                       "a sharded graph holds at most %d ABS_MAX nodes",
                                       M3C_SHARD_MAX_REDUCTIONS);
                break;
            }
            sh->reductions[sh->reduction_count] = node->outputs[0];
            sh->reduction_commands[sh->reduction_count] = (uint32_t)n;
            ++sh->reduction_count;
        }
    }
    if (status == M3_STATUS_OK) {
        status = local_graph(graph, sh->slabs, &local, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_cuda_session_create(session, local, options, cuda, error);
        m3_graph_free(local);
    }
    if (status != M3_STATUS_OK) {
        m3c_shard_free(sh);
        return status;
    }
    if (shard->id != NULL && shard->count > 1 &&
        (sh->reduction_count > 0 || sh->checks)) {
        cudaError_t code = cudaSetDevice(m3_cuda_session_device(*session));

        if (code == cudaSuccess) {
            code = cudaMalloc((void **)&sh->staging,
                              (M3C_SHARD_MAX_REDUCTIONS + 1U) * sizeof(uint32_t));
        }
        if (code != cudaSuccess) {
            (void)cudaGetLastError();
            status = m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                   "cannot allocate shard staging: %s",
                                   cudaGetErrorString(code));
        } else {
            status = m3c_comm_create(shard->id, shard->rank, shard->count,
                                     sh->timeout_seconds, &sh->comm, error);
        }
        if (status != M3_STATUS_OK) {
            (void)cudaFree(sh->staging);
            m3c_shard_free(sh);
            m3_session_free(*session);
            *session = NULL;
            return status;
        }
    }
    m3c_session_attach_shard(*session, sh);
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_shard_get_slab(const m3_session *session,
                                 m3_graph_value_id value,
                                 m3_cuda_shard_slab *slab, m3_error *error)
{
    const m3c_shard *sh;

    if (session == NULL || slab == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session and slab output are required");
    }
    if ((size_t)value >= m3c_session_value_count(session)) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "value is out of range");
    }
    sh = m3c_session_shard(session);
    if (sh != NULL) {
        *slab = sh->slabs[value];
    } else {
        /* an unsharded session is one shard holding everything */
        memset(slab, 0, sizeof(*slab));
        slab->global = *m3c_session_metadata(session, value);
        slab->local = slab->global;
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

static m3_status slab_copy(m3_session *session, m3_graph_value_id value,
                           void *global, size_t global_bytes,
                           bool device_memory, bool to_session,
                           m3_graph_value_role role, m3_error *error)
{
    m3_cuda_shard_slab slab;
    void *local = NULL;
    size_t local_bytes = 0U;
    cudaStream_t stream;
    cudaError_t code;
    m3_status status = m3_cuda_shard_get_slab(session, value, &slab, error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (m3c_session_role(session, value) != role) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "shard %s value has the wrong role",
                             to_session ? "input write" : "output read");
    }
    if (global_bytes != slab.global.byte_count ||
        (global_bytes != 0U && global == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "shard %s size does not match the global tensor",
                             to_session ? "input write" : "output read");
    }
    if (slab.local.byte_count == 0U) {
        m3_error_reset(error);
        return M3_STATUS_OK;
    }
    /* settles pending runs and selects the session's device */
    status = m3_cuda_session_value_device_pointer(session, value, &local,
                                                  &local_bytes, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    (void)cudaSetDevice(m3_cuda_session_device(session));
    stream = (cudaStream_t)m3_cuda_session_stream(session);
    if (!slab.split) {
        enum cudaMemcpyKind kind = device_memory ? cudaMemcpyDeviceToDevice
                                   : to_session  ? cudaMemcpyHostToDevice
                                                 : cudaMemcpyDeviceToHost;

        code = to_session ? cudaMemcpyAsync(local, global, local_bytes, kind, stream)
                          : cudaMemcpyAsync(global, local, local_bytes, kind, stream);
    } else {
        size_t outer, row, pitch, offset;
        enum cudaMemcpyKind kind = device_memory ? cudaMemcpyDeviceToDevice
                                   : to_session  ? cudaMemcpyHostToDevice
                                                 : cudaMemcpyDeviceToHost;

        slab_geometry(&slab, &outer, &row, &pitch, &offset);
        code = to_session
                   ? cudaMemcpy2DAsync(local, row, (const unsigned char *)global + offset,
                                       pitch, row, outer, kind, stream)
                   : cudaMemcpy2DAsync((unsigned char *)global + offset, pitch, local,
                                       row, row, outer, kind, stream);
    }
    if (code == cudaSuccess) {
        code = cudaStreamSynchronize(stream);
    }
    if (code != cudaSuccess) {
        (void)cudaGetLastError();
        return m3c_error_set(error, M3_STATUS_INTERNAL, "shard copy failed: %s",
                             cudaGetErrorString(code));
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_shard_write_input(m3_session *session,
                                    m3_graph_value_id value,
                                    const void *global_data,
                                    size_t global_byte_count,
                                    bool device_memory, m3_error *error)
{
    return slab_copy(session, value, (void *)global_data, global_byte_count,
                     device_memory, true, M3_GRAPH_INPUT, error);
}

m3_status m3_cuda_shard_read_output(const m3_session *session,
                                    m3_graph_value_id value,
                                    void *global_data,
                                    size_t global_byte_count,
                                    bool device_memory, m3_error *error)
{
    return slab_copy((m3_session *)session, value, global_data,
                     global_byte_count, device_memory, false, M3_GRAPH_OUTPUT,
                     error);
}
