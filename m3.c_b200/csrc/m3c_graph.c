/* Graph builder and shape inference of the m3.h graph API.
 *
 * Same contracts as the reference: descriptors are copied, constants are
 * copied at m3_graph_set_constant, topology is only checked at session
 * creation (reference src/m3_graph.c:27-341, src/m3_graph_infer.c:41-296).
 * Shape inference covers the operators this provider executes (and the
 * extensions); the reference's other kinds (contractions, attention, RoPE,
 * embedding, convolutions, resize) are M3_STATUS_UNSUPPORTED here, as they
 * would be at placement. */

#include "m3c_internal.h"

#include <stdlib.h>
#include <string.h>

void m3_graph_value_desc_init(m3_graph_value_desc *description,
                              m3_graph_value_role role, m3_dtype dtype,
                              uint8_t rank, const uint64_t *shape)
{
    uint8_t axis;

    if (description == NULL) {
        return;
    }
    memset(description, 0, sizeof(*description));
    description->role = role;
    description->dtype = dtype;
    description->rank = rank;
    for (axis = 0U; shape != NULL && axis < rank && axis < M3_TENSOR_MAX_RANK;
         ++axis) {
        description->shape[axis] = shape[axis];
    }
}

void m3_graph_node_desc_init(m3_graph_node_desc *description, m3_op_kind kind)
{
    size_t slot;

    if (description == NULL) {
        return;
    }
    memset(description, 0, sizeof(*description));
    description->kind = kind;
    for (slot = 0U; slot < M3_GRAPH_NODE_INPUT_CAPACITY; ++slot) {
        description->inputs[slot] = M3_GRAPH_VALUE_NONE;
    }
    for (slot = 0U; slot < M3_GRAPH_NODE_OUTPUT_CAPACITY; ++slot) {
        description->outputs[slot] = M3_GRAPH_VALUE_NONE;
    }
}

/* Defaults enable every provider, as in the reference
 * (src/m3_graph.c:65-72). */
void m3_session_options_init(m3_session_options *options)
{
    if (options != NULL) {
        options->allow_neural_engine = true;
        options->allow_metal = true;
        options->allow_cpu = true;
    }
}

m3_status m3_graph_create(m3_graph **graph, m3_error *error)
{
    m3_graph *created;

    if (graph == NULL || *graph != NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "graph output must be empty");
    }
    created = calloc(1U, sizeof(*created));
    if (created == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate graph");
    }
    *graph = created;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

void m3_graph_free(m3_graph *graph)
{
    size_t index;

    if (graph == NULL) {
        return;
    }
    for (index = 0U; index < graph->value_count; ++index) {
        free(graph->values[index].constant_data);
    }
    free(graph->values);
    free(graph->nodes);
    free(graph);
}

static bool grow(void **items, size_t *capacity, size_t item_size)
{
    size_t wanted = *capacity == 0U ? 8U : *capacity * 2U;
    void *moved;

    if (wanted < *capacity || wanted > SIZE_MAX / item_size) {
        return false;
    }
    moved = realloc(*items, wanted * item_size);
    if (moved == NULL) {
        return false;
    }
    *items = moved;
    *capacity = wanted;
    return true;
}

m3_status m3_graph_add_value(m3_graph *graph,
                             const m3_graph_value_desc *description,
                             m3_graph_value_id *value, m3_error *error)
{
    m3c_graph_value added;
    m3_status status;

    if (graph == NULL || description == NULL || value == NULL) {
        return m3c_error_set(
            error, M3_STATUS_INVALID_ARGUMENT,
            "graph, value description, and output are required");
    }
    if ((int)description->role < (int)M3_GRAPH_INPUT ||
        (int)description->role > (int)M3_GRAPH_OUTPUT) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "graph value role is invalid");
    }
    if (graph->value_count >= (size_t)M3_GRAPH_VALUE_NONE) {
        return m3c_error_set(error, M3_STATUS_OVERFLOW,
                             "graph value identifiers are exhausted");
    }
    memset(&added, 0, sizeof(added));
    status = m3c_metadata_init(&added.metadata, description->dtype,
                               description->rank, description->shape, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    added.description = *description;
    if (graph->value_count == graph->value_capacity &&
        !grow((void **)&graph->values, &graph->value_capacity,
              sizeof(*graph->values))) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot grow graph values");
    }
    graph->values[graph->value_count] = added;
    *value = (m3_graph_value_id)graph->value_count;
    ++graph->value_count;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_graph_set_constant(m3_graph *graph, m3_graph_value_id value,
                                const void *data, size_t byte_count,
                                m3_error *error)
{
    m3c_graph_value *target;
    void *copy = NULL;

    if (graph == NULL || (size_t)value >= graph->value_count) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "constant graph value is out of range");
    }
    target = &graph->values[value];
    if (target->description.role != M3_GRAPH_CONSTANT ||
        byte_count != target->metadata.byte_count ||
        (byte_count != 0U && data == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "constant data does not match its graph value");
    }
    if (byte_count != 0U) {
        copy = malloc(byte_count);
        if (copy == NULL) {
            return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                 "cannot copy graph constant");
        }
        memcpy(copy, data, byte_count);
    }
    free(target->constant_data);
    target->constant_data = copy;
    target->constant_size = byte_count;
    target->constant_set = true;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_graph_add_node(m3_graph *graph,
                            const m3_graph_node_desc *description,
                            m3_error *error)
{
    if (graph == NULL || description == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "graph and node description are required");
    }
    if (graph->node_count == graph->node_capacity &&
        !grow((void **)&graph->nodes, &graph->node_capacity,
              sizeof(*graph->nodes))) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot grow graph nodes");
    }
    graph->nodes[graph->node_count] = *description;
    ++graph->node_count;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

/* ------------------------------------------------------ shape inference */

static m3_status inferred_input(const m3_graph *graph, m3_graph_value_id id,
                                const m3_tensor_metadata **metadata,
                                m3_error *error)
{
    *metadata = NULL;
    if (id == M3_GRAPH_VALUE_NONE || (size_t)id >= graph->value_count) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "inferred graph input is absent or out of range");
    }
    *metadata = &graph->values[id].metadata;
    return M3_STATUS_OK;
}

static void copy_shape(m3_graph_value_desc *out, const m3_tensor_metadata *in)
{
    out->rank = in->rank;
    memcpy(out->shape, in->shape, sizeof(out->shape));
}

/* Right-aligned broadcast (src/m3_graph_infer.c:41-63). */
static m3_status infer_broadcast(const m3_tensor_metadata *a,
                                 const m3_tensor_metadata *b,
                                 m3_graph_value_desc *out, m3_error *error)
{
    uint8_t rank = a->rank > b->rank ? a->rank : b->rank;
    uint8_t axis;

    out->rank = rank;
    for (axis = 0U; axis < rank; ++axis) {
        int ia = (int)axis - (int)(rank - a->rank);
        int ib = (int)axis - (int)(rank - b->rank);
        uint64_t ea = ia < 0 ? 1U : a->shape[ia];
        uint64_t eb = ib < 0 ? 1U : b->shape[ib];

        if (ea != eb && ea != 1U && eb != 1U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "inferred broadcast dimensions disagree");
        }
        out->shape[axis] = ea == 1U ? eb : ea;
    }
    return M3_STATUS_OK;
}

/* Output length of the 1-D convolutions (src/m3_graph_infer.c:65-131). */
static m3_status infer_shape(const m3_graph *graph,
                             const m3_graph_node_desc *node,
                             size_t output_index, m3_graph_value_desc *out,
                             m3_error *error)
{
    const m3_tensor_metadata *first = NULL;
    const m3_tensor_metadata *second = NULL;
    m3_status status = inferred_input(graph, node->inputs[0], &first, error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (output_index != 0U && node->kind != M3_OP_TOP_K) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "operation has no requested inferred output");
    }
    switch ((int)node->kind) {
    case M3_OP_COPY:
    case M3_OP_CAST:
    case M3_OP_RMS_NORM:
    case M3_OP_LAYER_NORM:
    case M3_OP_SOFTMAX:
    case M3_OP_SNAKE1D:
    case M3_OP_TANH:
    case M3_OP_GATED_SILU:
    case (int)M3_OP_CLAMP_UNIT:
        copy_shape(out, first);
        if (node->kind == M3_OP_COPY) {
            out->dtype = first->dtype;
        } else if (node->kind == M3_OP_SNAKE1D || node->kind == M3_OP_TANH ||
                   node->kind == M3_OP_CLAMP_UNIT) {
            out->dtype = M3_DTYPE_F32;
        }
        return M3_STATUS_OK;
    case (int)M3_OP_ABS_MAX:
        out->rank = 1U;
        out->shape[0] = 1U;
        out->dtype = M3_DTYPE_F32;
        return M3_STATUS_OK;
    case (int)M3_OP_ROW_SUM:
        if (first->rank == 0U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "cannot infer row-sum shape");
        }
        copy_shape(out, first);
        out->shape[first->rank - 1U] = 1U;
        out->dtype = M3_DTYPE_F32;
        return M3_STATUS_OK;
    case M3_OP_ADD:
    case M3_OP_MUL:
        status = inferred_input(graph, node->inputs[1], &second, error);
        return status != M3_STATUS_OK
                   ? status
                   : infer_broadcast(first, second, out, error);
    case M3_OP_TOP_K:
        if (first->rank == 0U || output_index > 1U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "cannot infer top-k shape");
        }
        copy_shape(out, first);
        out->shape[first->rank - 1U] = node->parameters.top_k.k;
        out->dtype = output_index == 0U ? M3_DTYPE_F32 : M3_DTYPE_I32;
        return M3_STATUS_OK;
    case M3_OP_CATEGORICAL:
        if (first->rank == 0U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "cannot infer categorical shape");
        }
        copy_shape(out, first);
        out->rank = (uint8_t)(first->rank - 1U);
        out->dtype = M3_DTYPE_I32;
        return M3_STATUS_OK;
    default:
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "cannot infer unsupported operation kind %d",
                             (int)node->kind);
    }
}

m3_status m3_graph_add_inferred_value(
    m3_graph *graph, const m3_graph_node_desc *node, size_t output_index,
    m3_graph_value_role role, m3_dtype dtype, m3_graph_value_id *value,
    m3_error *error)
{
    m3_graph_value_desc inferred;
    m3_status status;

    if (graph == NULL || node == NULL || value == NULL ||
        (role != M3_GRAPH_TEMPORARY && role != M3_GRAPH_OUTPUT)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "inferred graph value request is invalid");
    }
    memset(&inferred, 0, sizeof(inferred));
    inferred.role = role;
    inferred.dtype = dtype;
    status = infer_shape(graph, node, output_index, &inferred, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    return m3_graph_add_value(graph, &inferred, value, error);
}
