/* Host-side session compiler: topology, liveness slots, binding, validation,
 * placement and the fusion pass.  Needs no GPU (m3_cuda_graph_plan runs it on
 * any host).
 *
 * Topology and the liveness planner follow the reference exactly
 * (src/m3_graph_compile.c:18-324), so m3_session_get_plan_info reports the
 * same slot count and bytes as the reference for the same graph.
 *
 * Fusion.  Consecutive element-wise nodes over one iteration shape become one
 * launch; their intermediates stay in registers when nothing outside the
 * group reads them.  A residual ADD feeding RMSNorm/LayerNorm becomes the
 * norm kernel's prologue; SOFTMAX, TOP_K and ROW_SUM of one input share one
 * row kernel.
 *
 * Atomic commit.  Operators with all-or-nothing data checks (SOFTMAX and
 * TOP_K reject NaN, CAST to I32 rejects out-of-range values, ABS_MAX rejects
 * NaN; reference src/m3_op_data_preflight.c) must leave their outputs
 * untouched on failure, yet the check and the computation share one pass over
 * HBM.  Such a command and every later command of its launch write the
 * *shadow* buffer of their output slot; at the end of a clean run the slot
 * flips to the shadow buffer (a pointer swap, no copy).  A failing run
 * commits only the flips of commands before the failing one, exactly the
 * state the reference leaves after a failing command. */

#include "m3c_internal.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define NO_VALUE UINT32_MAX

/* --------------------------------------------------------------- schema */

typedef struct {
    size_t inputs;
    size_t outputs;
    uint32_t optional;
} schema_t;

/* Input/output positions per operator (src/m3_graph_compile.c:18-66). */
static m3_status regular_schema(m3_op_kind kind, schema_t *schema,
                                m3_error *error)
{
    memset(schema, 0, sizeof(*schema));
    schema->outputs = 1U;
    switch ((int)kind) {
    case M3_OP_COPY:
    case M3_OP_CAST:
    case M3_OP_SOFTMAX:
    case M3_OP_NEAREST_RESIZE1D:
    case M3_OP_TANH:
    case (int)M3_OP_ABS_MAX:
    case (int)M3_OP_CLAMP_UNIT:
    case (int)M3_OP_ROW_SUM:
        schema->inputs = 1U;
        return M3_STATUS_OK;
    case M3_OP_ADD:
    case M3_OP_MUL:
    case M3_OP_EMBEDDING:
    case M3_OP_MATMUL:
    case M3_OP_RMS_NORM:
    case M3_OP_GATED_SILU:
    case M3_OP_CATEGORICAL:
    case M3_OP_SNAKE1D:
        schema->inputs = 2U;
        return M3_STATUS_OK;
    case M3_OP_LINEAR:
    case M3_OP_LAYER_NORM:
    case M3_OP_CONV1D:
    case M3_OP_CONV_TRANSPOSE1D:
        schema->inputs = 3U;
        schema->optional = 1U << 2U;
        return M3_STATUS_OK;
    case M3_OP_ROPE:
        schema->inputs = 3U;
        return M3_STATUS_OK;
    case M3_OP_ATTENTION:
        schema->inputs = 4U;
        schema->optional = 1U << 3U;
        return M3_STATUS_OK;
    case M3_OP_TOP_K:
        schema->inputs = 1U;
        schema->outputs = 2U;
        return M3_STATUS_OK;
    default:
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "unsupported graph operation kind %d",
                             (int)kind);
    }
}

static m3_status check_id(const m3_graph *graph, m3_graph_value_id id,
                          bool optional, const char *what, m3_error *error)
{
    if (id == M3_GRAPH_VALUE_NONE) {
        return optional ? M3_STATUS_OK
                        : m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                        "required graph node %s is absent",
                                        what);
    }
    if ((size_t)id >= graph->value_count) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "graph node %s is out of range", what);
    }
    return M3_STATUS_OK;
}

static m3_status node_ids(const m3_graph *graph,
                          const m3_graph_node_desc *node, schema_t *schema,
                          m3_error *error)
{
    size_t slot;
    m3_status status = regular_schema(node->kind, schema, error);

    for (slot = 0U; status == M3_STATUS_OK &&
                    slot < M3_GRAPH_NODE_INPUT_CAPACITY; ++slot) {
        bool used = slot < schema->inputs;

        if (!used && node->inputs[slot] != M3_GRAPH_VALUE_NONE) {
            status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                   "graph node has an extra input");
        } else if (used) {
            status = check_id(graph, node->inputs[slot],
                              (schema->optional & (1U << slot)) != 0U,
                              "input", error);
        }
    }
    for (slot = 0U; status == M3_STATUS_OK &&
                    slot < M3_GRAPH_NODE_OUTPUT_CAPACITY; ++slot) {
        bool used = slot < schema->outputs;

        if (!used && node->outputs[slot] != M3_GRAPH_VALUE_NONE) {
            status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                   "graph node has an extra output");
        } else if (used) {
            status = check_id(graph, node->outputs[slot], false, "output",
                              error);
        }
    }
    return status;
}

/* Read-before-produce, single producer, no writes of inputs or constants,
 * every temporary/output produced; records producers and last uses
 * (src/m3_graph_compile.c:122-245). */
static m3_status topology(const m3_graph *graph, size_t *producers,
                          size_t *last_uses, m3_error *error)
{
    bool *available = calloc(graph->value_count ? graph->value_count : 1U,
                             sizeof(*available));
    m3_status status = M3_STATUS_OK;
    size_t v;
    size_t n;

    if (available == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate graph topology state");
    }
    for (v = 0U; v < graph->value_count; ++v) {
        m3_graph_value_role role = graph->values[v].description.role;

        producers[v] = SIZE_MAX;
        last_uses[v] = 0U;
        available[v] = role == M3_GRAPH_INPUT || role == M3_GRAPH_CONSTANT;
        if (role == M3_GRAPH_CONSTANT && !graph->values[v].constant_set) {
            status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                   "graph constant has no data");
            break;
        }
    }
    for (n = 0U; status == M3_STATUS_OK && n < graph->node_count; ++n) {
        const m3_graph_node_desc *node = &graph->nodes[n];
        schema_t schema;
        size_t slot;

        status = node_ids(graph, node, &schema, error);
        for (slot = 0U; status == M3_STATUS_OK && slot < schema.inputs;
             ++slot) {
            m3_graph_value_id in = node->inputs[slot];

            if (in == M3_GRAPH_VALUE_NONE) {
                continue;
            }
            if (!available[in]) {
                status = m3c_error_set(
                    error, M3_STATUS_INVALID_ARGUMENT,
                    "graph node reads a value before it is produced");
            } else {
                last_uses[in] = n;
            }
        }
        for (slot = 0U; status == M3_STATUS_OK && slot < schema.outputs;
             ++slot) {
            m3_graph_value_id out = node->outputs[slot];
            m3_graph_value_role role = graph->values[out].description.role;
            size_t other;

            if (role != M3_GRAPH_TEMPORARY && role != M3_GRAPH_OUTPUT) {
                status = m3c_error_set(
                    error, M3_STATUS_INVALID_ARGUMENT,
                    "graph node writes an input or constant value");
            } else if (producers[out] != SIZE_MAX) {
                status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                       "graph value has multiple producers");
            }
            for (other = 0U; status == M3_STATUS_OK && other < slot;
                 ++other) {
                if (node->outputs[other] == out) {
                    status = m3c_error_set(
                        error, M3_STATUS_INVALID_ARGUMENT,
                        "graph node repeats an output value");
                }
            }
            if (status == M3_STATUS_OK) {
                producers[out] = n;
                last_uses[out] = n;
                available[out] = true;
            }
        }
    }
    for (v = 0U; status == M3_STATUS_OK && v < graph->value_count; ++v) {
        m3_graph_value_role role = graph->values[v].description.role;

        if ((role == M3_GRAPH_TEMPORARY || role == M3_GRAPH_OUTPUT) &&
            producers[v] == SIZE_MAX) {
            status = m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                   "graph value has no producer");
        }
    }
    free(available);
    return status;
}

/* Greedy best-fit slot reuse (src/m3_graph_compile.c:247-324): inputs,
 * constants and outputs own a slot each; a temporary takes the smallest slot
 * whose last use is before its producer and that is large enough, else a new
 * slot. */
static m3_status plan_slots(const m3_graph *graph, m3c_plan *plan,
                            m3_error *error)
{
    size_t count = graph->value_count;
    size_t *slot_last_use = calloc(count ? count : 1U, sizeof(size_t));
    size_t v;
    size_t n;

    if (slot_last_use == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate liveness slots");
    }
    plan->slot_count = 0U;
    for (v = 0U; v < count; ++v) {
        plan->value_slot[v] = M3C_NO_SLOT;
        if (graph->values[v].description.role != M3_GRAPH_TEMPORARY) {
            size_t s = plan->slot_count++;

            plan->slot_bytes[s] = graph->values[v].metadata.byte_count;
            plan->value_slot[v] = s;
            slot_last_use[s] = SIZE_MAX;
        }
    }
    for (n = 0U; n < graph->node_count; ++n) {
        for (v = 0U; v < count; ++v) {
            size_t bytes = graph->values[v].metadata.byte_count;
            size_t best = SIZE_MAX;
            size_t s;

            if (graph->values[v].description.role != M3_GRAPH_TEMPORARY ||
                plan->producers[v] != n) {
                continue;
            }
            for (s = 0U; s < plan->slot_count; ++s) {
                if (slot_last_use[s] < n && plan->slot_bytes[s] >= bytes &&
                    (best == SIZE_MAX ||
                     plan->slot_bytes[s] < plan->slot_bytes[best])) {
                    best = s;
                }
            }
            if (best == SIZE_MAX) {
                best = plan->slot_count++;
                plan->slot_bytes[best] = bytes;
            }
            plan->value_slot[v] = best;
            slot_last_use[best] = plan->last_uses[v];
        }
    }
    free(slot_last_use);
    plan->allocated_bytes = 0U;
    for (v = 0U; v < plan->slot_count; ++v) {
        if (plan->slot_bytes[v] > SIZE_MAX - plan->allocated_bytes) {
            return m3c_error_set(error, M3_STATUS_OVERFLOW,
                                 "graph allocation total overflows");
        }
        plan->allocated_bytes += plan->slot_bytes[v];
    }
    return M3_STATUS_OK;
}

/* ------------------------------------------------- binding + validation */

static size_t canonical_strides[M3_TENSOR_MAX_RANK];

static void value_view(const m3_graph *graph, const m3c_plan *plan,
                       m3_graph_value_id id, size_t *strides, m3c_vview *view)
{
    const m3_tensor_metadata *meta;
    size_t stride;
    int axis;

    memset(view, 0, sizeof(*view));
    if (id == M3_GRAPH_VALUE_NONE) {
        return;
    }
    meta = &graph->values[id].metadata;
    stride = m3c_dtype_size(meta->dtype);
    for (axis = (int)meta->rank - 1; axis >= 0; --axis) {
        strides[axis] = stride;
        stride *= (size_t)meta->shape[axis];
    }
    view->metadata = meta;
    view->byte_offset = 0U;
    view->byte_strides = strides;
    /* one storage per slot: the key is the slot number + 1 */
    view->storage = (const void *)(uintptr_t)(plan->value_slot[id] + 1U);
    view->present = true;
}

static m3_status validate_node(const m3_graph *graph, const m3c_plan *plan,
                               const m3_graph_node_desc *node,
                               m3_error *error)
{
    size_t strides[5][M3_TENSOR_MAX_RANK];
    m3c_vcommand command;
    int i;

    memset(&command, 0, sizeof(command));
    command.kind = node->kind;
    for (i = 0; i < 3; ++i) {
        value_view(graph, plan, node->inputs[i], strides[i], &command.in[i]);
    }
    for (i = 0; i < 2; ++i) {
        value_view(graph, plan, node->outputs[i], strides[3 + i],
                   &command.out[i]);
    }
    command.epsilon = node->parameters.norm.epsilon;
    command.k = node->parameters.top_k.k;
    return m3c_validate(&command, error);
}

/* ------------------------------------------------------- fusion planner */

static bool is_elementwise(m3_op_kind kind)
{
    switch ((int)kind) {
    case M3_OP_COPY:
    case M3_OP_CAST:
    case M3_OP_ADD:
    case M3_OP_MUL:
    case M3_OP_GATED_SILU:
    case M3_OP_SNAKE1D:
    case M3_OP_TANH:
    case (int)M3_OP_CLAMP_UNIT:
    case (int)M3_OP_ABS_MAX:
        return true;
    default:
        return false;
    }
}

static bool has_data_check(const m3_graph *graph,
                           const m3_graph_node_desc *node)
{
    switch ((int)node->kind) {
    case M3_OP_SOFTMAX:
    case M3_OP_TOP_K:
    case M3_OP_CATEGORICAL:
    case (int)M3_OP_ABS_MAX:
        return true;
    case M3_OP_CAST:
        return graph->values[node->outputs[0]].metadata.dtype ==
                   M3_DTYPE_I32 &&
               graph->values[node->inputs[0]].metadata.dtype != M3_DTYPE_I32;
    default:
        return false;
    }
}

/* Element-wise group under construction, in virtual registers (SSA): vreg
 * numbers < n_operands are loaded operands, the rest are op results. */
#define VMAX 64

typedef struct {
    size_t first_node;
    size_t last_node;
    uint32_t shape_value;
    int n_operands;
    uint32_t operand_value[M3C_EW_MAX_OPERANDS];
    int32_t operand_load[M3C_EW_MAX_OPERANDS];
    uint32_t operand_imm[M3C_EW_MAX_OPERANDS];
    bool operand_is_imm[M3C_EW_MAX_OPERANDS];
    int n_ops;
    m3c_ew_op ops[M3C_EW_MAX_OPS];      /* dst/a/b are vregs */
    int n_vregs;
    uint32_t vreg_value[VMAX];          /* value held (NO_VALUE: internal) */
    bool vreg_is_raw[VMAX];             /* holds raw storage bits */
    int value_vreg_count;
    bool has_absmax;
    uint32_t absmax_value;              /* output value of ABS_MAX */
    uint32_t absmax_command;
    bool has_check;
    size_t first_check_node;
} ew_group;

typedef struct {
    const m3_graph *graph;
    m3c_plan *plan;
    uint8_t *side;            /* per slot: parity relative to run start */
    size_t launch_capacity;
    size_t flip_capacity;
} planner;

static const m3_tensor_metadata *meta_of(const planner *p, uint32_t v)
{
    return &p->graph->values[v].metadata;
}

static m3_status push_launch(planner *p, const m3c_launch *launch,
                             m3_error *error)
{
    m3c_plan *plan = p->plan;

    if (plan->launch_count == p->launch_capacity) {
        size_t wanted = p->launch_capacity ? p->launch_capacity * 2U : 8U;
        m3c_launch *moved = realloc(plan->launches, wanted * sizeof(*moved));

        if (moved == NULL) {
            return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                 "cannot grow the launch plan");
        }
        plan->launches = moved;
        p->launch_capacity = wanted;
    }
    plan->launches[plan->launch_count++] = *launch;
    return M3_STATUS_OK;
}

static m3_status push_flip(planner *p, size_t slot, uint32_t command,
                           m3_error *error)
{
    m3c_plan *plan = p->plan;

    if (plan->flip_count == p->flip_capacity) {
        size_t wanted = p->flip_capacity ? p->flip_capacity * 2U : 8U;
        size_t *slots = realloc(plan->flip_slot, wanted * sizeof(*slots));
        uint32_t *commands;

        if (slots == NULL) {
            return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                 "cannot grow the commit plan");
        }
        plan->flip_slot = slots;
        commands = realloc(plan->flip_command, wanted * sizeof(*commands));
        if (commands == NULL) {
            return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                 "cannot grow the commit plan");
        }
        plan->flip_command = commands;
        p->flip_capacity = wanted;
    }
    plan->flip_slot[plan->flip_count] = slot;
    plan->flip_command[plan->flip_count] = command;
    ++plan->flip_count;
    return M3_STATUS_OK;
}

/* Reference to a value read at this point of the run. */
static m3c_ref read_ref(const planner *p, uint32_t value)
{
    m3c_ref ref;

    ref.value = value;
    ref.shadow = p->side[p->plan->value_slot[value]] != 0U;
    return ref;
}

/* Reference for a write by `command`; a checked write goes to the other
 * buffer of the slot and flips the slot's parity (committed at run end). */
static m3_status write_ref(planner *p, uint32_t value, bool checked,
                           uint32_t command, m3c_ref *ref, m3_error *error)
{
    size_t slot = p->plan->value_slot[value];

    ref->value = value;
    if (!checked) {
        ref->shadow = p->side[slot] != 0U;
        return M3_STATUS_OK;
    }
    p->side[slot] ^= 1U;
    ref->shadow = p->side[slot] != 0U;
    p->plan->slot_shadowed[slot] = true;
    return push_flip(p, slot, command, error);
}

/* Scalar constants are folded into immediates: their bytes are known when
 * the session is compiled. */
static bool scalar_constant(const planner *p, uint32_t value, uint32_t *bits)
{
    const m3c_graph_value *gv = &p->graph->values[value];
    uint16_t half;

    if (gv->description.role != M3_GRAPH_CONSTANT ||
        gv->metadata.element_count != 1U || gv->constant_data == NULL) {
        return false;
    }
    switch (gv->metadata.dtype) {
    case M3_DTYPE_F32:
    case M3_DTYPE_I32:
        memcpy(bits, gv->constant_data, 4U);
        return true;
    case M3_DTYPE_F16:
    case M3_DTYPE_BF16:
        memcpy(&half, gv->constant_data, 2U);
        *bits = half;       /* raw; widened by an explicit op */
        return true;
    }
    return false;
}

static int find_vreg(const ew_group *g, uint32_t value)
{
    int r;

    for (r = g->n_vregs - 1; r >= 0; --r) {
        if (g->vreg_value[r] == value) {
            return r;
        }
    }
    return -1;
}

/* Operand vreg for reading `value` as a float (or raw / int). */
static int operand_vreg(const planner *p, ew_group *g, uint32_t value,
                        int32_t load_as, bool *ok)
{
    const m3_tensor_metadata *meta = meta_of(p, value);
    int existing = find_vreg(g, value);
    uint32_t imm = 0U;
    bool is_imm;
    int vreg;
    int i;

    if (existing >= 0) {
        return existing;
    }
    /* operands precede every op vreg: they are loaded at program start */
    for (i = 0; i < g->n_operands; ++i) {
        if (g->operand_value[i] == value && g->operand_load[i] == load_as) {
            return i;
        }
    }
    if (g->n_operands >= M3C_EW_MAX_OPERANDS || g->n_ops > 0) {
        /* new operands after ops were emitted would renumber vregs; the
         * caller pre-registers operands before emitting a node's ops */
        *ok = false;
        return -1;
    }
    is_imm = scalar_constant(p, value, &imm);
    vreg = g->n_operands++;
    g->operand_value[vreg] = value;
    g->operand_load[vreg] = load_as;
    g->operand_is_imm[vreg] = is_imm;
    g->operand_imm[vreg] = imm;
    (void)meta;
    return vreg;
}

/* ------------------------------------------------------------------------ */
/* Element-wise groups are built per node in two phases: first every memory
 * operand of the node is registered (they must precede op vregs), then the
 * node's ops are appended.  Because operands must all be known before the
 * first op, a group is assembled from a list of nodes and re-derived from
 * scratch whenever a node is appended. */

typedef struct {
    size_t nodes[M3C_EW_MAX_OPS];
    size_t count;
} node_list;

static bool produced_in(const planner *p, const node_list *list,
                        uint32_t value)
{
    size_t producer = p->plan->producers[value];
    size_t i;

    if (producer == SIZE_MAX) {
        return false;
    }
    for (i = 0U; i < list->count; ++i) {
        if (list->nodes[i] == producer) {
            return true;
        }
    }
    return false;
}

/* The iteration value of an element-wise node: its output, or for ABS_MAX
 * its input. */
static uint32_t iteration_value(const m3_graph_node_desc *node)
{
    return node->kind == M3_OP_ABS_MAX ? node->inputs[0] : node->outputs[0];
}

static int new_vreg(ew_group *g, uint32_t value, bool raw)
{
    int r = g->n_vregs;

    if (r >= VMAX) {
        return -1;
    }
    g->vreg_value[r] = value;
    g->vreg_is_raw[r] = raw;
    ++g->n_vregs;
    return r;
}

static bool emit(ew_group *g, uint8_t code, int dst, int a, int b,
                 m3_dtype rdtype, int aux, size_t command)
{
    m3c_ew_op *op;

    if (g->n_ops >= M3C_EW_MAX_OPS || dst < 0 || a < 0 || b < 0) {
        return false;
    }
    op = &g->ops[g->n_ops++];
    op->code = code;
    op->dst = (uint8_t)dst;
    op->a = (uint8_t)a;
    op->b = (uint8_t)b;
    op->rdtype = (int8_t)rdtype;
    op->aux = (int8_t)aux;
    op->command = (uint16_t)command;
    return true;
}

/* A float view of vreg r holding `value`: widens raw 16-bit words. */
static int as_float(const planner *p, ew_group *g, int r, uint32_t value,
                    size_t command)
{
    m3_dtype dtype = meta_of(p, value)->dtype;
    int w;

    if (r < 0 || !g->vreg_is_raw[r] ||
        (dtype != M3_DTYPE_F16 && dtype != M3_DTYPE_BF16)) {
        return r;
    }
    w = new_vreg(g, NO_VALUE, false);
    if (!emit(g, M3C_OP_WIDEN, w, r, r, M3_DTYPE_F32, (int)dtype, command)) {
        return -1;
    }
    return w;
}

/* External values are loaded as raw storage bits (F32 bits are the value;
 * 16-bit words are widened by an explicit op where a float is needed, and
 * stored unchanged by exact copies), I32 as integers. */
static int32_t load_mode_for(const planner *p, uint32_t value)
{
    return meta_of(p, value)->dtype == M3_DTYPE_I32 ? M3C_LOAD_INT
                                                    : M3C_LOAD_RAW;
}

/* Re-derive the whole group program for `list`.  Returns false when the list
 * does not fit the kernel limits. */
static bool derive_group(const planner *p, const node_list *list,
                         ew_group *g)
{
    size_t i;
    bool ok = true;

    memset(g, 0, sizeof(*g));
    g->first_node = list->nodes[0];
    g->last_node = list->nodes[list->count - 1U];
    g->shape_value = iteration_value(&p->graph->nodes[list->nodes[0]]);
    g->first_check_node = SIZE_MAX;
    /* phase 1: operands (values produced outside the list) */
    for (i = 0U; i < list->count && ok; ++i) {
        const m3_graph_node_desc *node = &p->graph->nodes[list->nodes[i]];
        schema_t schema;
        size_t s;

        (void)regular_schema(node->kind, &schema, NULL);
        for (s = 0U; s < schema.inputs && ok; ++s) {
            uint32_t in = node->inputs[s];

            if (in == M3_GRAPH_VALUE_NONE || produced_in(p, list, in)) {
                continue;
            }
            (void)operand_vreg(p, g, in, load_mode_for(p, in), &ok);
        }
    }
    if (!ok) {
        return false;
    }
    g->n_vregs = g->n_operands;
    for (i = 0U; i < (size_t)g->n_operands; ++i) {
        g->vreg_value[i] = g->operand_value[i];
        /* every memory operand is loaded raw (or int) and widened on use;
         * F32 raw bits are already the float value */
        g->vreg_is_raw[i] = g->operand_load[i] == M3C_LOAD_RAW &&
                            meta_of(p, g->operand_value[i])->dtype !=
                                M3_DTYPE_F32;
    }
    /* phase 2: ops */
    for (i = 0U; i < list->count && ok; ++i) {
        size_t n = list->nodes[i];
        const m3_graph_node_desc *node = &p->graph->nodes[n];
        uint32_t out = node->outputs[0];
        m3_dtype odt = meta_of(p, out)->dtype;
        int a = -1;
        int b = -1;
        int d;

        if (has_data_check(p->graph, node) && g->first_check_node == SIZE_MAX) {
            g->first_check_node = n;
            g->has_check = true;
        }
        a = find_vreg(g, node->inputs[0]);
        if (node->inputs[1] != M3_GRAPH_VALUE_NONE &&
            node->kind != M3_OP_ABS_MAX) {
            b = find_vreg(g, node->inputs[1]);
        }
        switch ((int)node->kind) {
        case M3_OP_COPY:
            d = new_vreg(g, out, g->vreg_is_raw[a]);
            ok = emit(g, M3C_OP_MOV, d, a, a, odt, 0, n);
            break;
        case M3_OP_CAST: {
            m3_dtype idt = meta_of(p, node->inputs[0])->dtype;

            if (idt == odt) {
                d = new_vreg(g, out, g->vreg_is_raw[a]);
                ok = emit(g, M3C_OP_MOV, d, a, a, odt, 0, n);
            } else if (idt == M3_DTYPE_I32) {
                d = new_vreg(g, out, false);
                ok = emit(g, M3C_OP_I2F, d, a, a, odt, 0, n);
            } else if (odt == M3_DTYPE_I32) {
                a = as_float(p, g, a, node->inputs[0], n);
                d = new_vreg(g, out, false);
                ok = emit(g, M3C_OP_F2I, d, a, a, odt, 0, n);
            } else {
                a = as_float(p, g, a, node->inputs[0], n);
                d = new_vreg(g, out, false);
                ok = emit(g, M3C_OP_ROUND, d, a, a, odt, 0, n);
            }
            break;
        }
        case M3_OP_ADD:
        case M3_OP_MUL:
            a = as_float(p, g, a, node->inputs[0], n);
            b = as_float(p, g, b, node->inputs[1], n);
            d = new_vreg(g, out, false);
            ok = emit(g, node->kind == M3_OP_ADD ? M3C_OP_ADD : M3C_OP_MUL, d,
                      a, b, odt, 0, n);
            break;
        case M3_OP_GATED_SILU:
            a = as_float(p, g, a, node->inputs[0], n);
            b = as_float(p, g, b, node->inputs[1], n);
            d = new_vreg(g, out, false);
            ok = emit(g, M3C_OP_GSILU, d, a, b, odt,
                      (int)meta_of(p, node->inputs[0])->dtype, n);
            break;
        case M3_OP_SNAKE1D:
            d = new_vreg(g, out, false);
            ok = emit(g, M3C_OP_SNAKE, d, a, b, odt, 0, n);
            break;
        case M3_OP_TANH:
            d = new_vreg(g, out, false);
            ok = emit(g, M3C_OP_TANH, d, a, a, odt, 0, n);
            break;
        case (int)M3_OP_CLAMP_UNIT:
            d = new_vreg(g, out, false);
            ok = emit(g, M3C_OP_CLAMP, d, a, a, odt, 0, n);
            break;
        case (int)M3_OP_ABS_MAX:
            if (g->has_absmax) {
                ok = false;
                break;
            }
            a = as_float(p, g, a, node->inputs[0], n);
            ok = emit(g, M3C_OP_ABSMAX, a, a, a, M3_DTYPE_F32, 0, n);
            g->has_absmax = true;
            g->absmax_value = out;
            g->absmax_command = (uint32_t)n;
            break;
        default:
            ok = false;
            break;
        }
        if (a < 0 || (node->inputs[1] != M3_GRAPH_VALUE_NONE && b < 0 &&
                      node->kind != M3_OP_ABS_MAX && node->kind != M3_OP_COPY &&
                      node->kind != M3_OP_CAST && node->kind != M3_OP_TANH)) {
            ok = false;
        }
    }
    return ok;
}

/* Physical register allocation by liveness; outputs live to the end.
 * Returns false when more than M3C_EW_MAX_REGS words are live at once. */
static bool allocate_registers(const planner *p, const ew_group *g,
                               const bool *stored, m3c_launch *launch)
{
    int last_use[VMAX];
    int phys[VMAX];
    int owner[M3C_EW_MAX_REGS];
    int r;
    int k;

    (void)p;
    for (r = 0; r < g->n_vregs; ++r) {
        last_use[r] = -1;
        phys[r] = -1;
    }
    for (k = 0; k < g->n_ops; ++k) {
        last_use[g->ops[k].a] = k;
        last_use[g->ops[k].b] = k;
    }
    for (r = 0; r < g->n_vregs; ++r) {
        if (stored[r]) {
            last_use[r] = g->n_ops;     /* stored after the last op */
        }
    }
    for (k = 0; k < M3C_EW_MAX_REGS; ++k) {
        owner[k] = -1;
    }
    /* operands: loaded at start */
    for (r = 0; r < g->n_operands; ++r) {
        for (k = 0; k < M3C_EW_MAX_REGS && owner[k] >= 0; ++k) {
        }
        if (k == M3C_EW_MAX_REGS) {
            return false;
        }
        owner[k] = r;
        phys[r] = k;
    }
    for (k = 0; k < g->n_ops; ++k) {
        const m3c_ew_op *op = &g->ops[k];
        int dst = op->dst;
        int q;

        /* free registers whose value dies at this op (inputs may be
         * overwritten by the result: the kernel reads before it writes) */
        for (q = 0; q < M3C_EW_MAX_REGS; ++q) {
            if (owner[q] >= 0 && last_use[owner[q]] <= k &&
                owner[q] != dst) {
                owner[q] = -1;
            }
        }
        if (op->code == M3C_OP_ABSMAX) {
            continue;       /* no result */
        }
        if (phys[dst] >= 0) {
            continue;
        }
        for (q = 0; q < M3C_EW_MAX_REGS && owner[q] >= 0; ++q) {
        }
        if (q == M3C_EW_MAX_REGS) {
            return false;
        }
        owner[q] = dst;
        phys[dst] = q;
    }
    for (k = 0; k < g->n_ops; ++k) {
        m3c_ew_op op = g->ops[k];

        op.a = (uint8_t)phys[op.a];
        op.b = (uint8_t)phys[op.b];
        op.dst = op.code == M3C_OP_ABSMAX ? op.a : (uint8_t)phys[op.dst];
        launch->ops[k] = op;
    }
    launch->n_ops = g->n_ops;
    for (r = 0; r < g->n_vregs; ++r) {
        if (stored[r]) {
            int o = launch->n_outputs;

            if (o >= M3C_EW_MAX_OUTPUTS) {
                return false;
            }
            launch->output_regs[o] = phys[r];
            launch->output_raw[o] = g->vreg_is_raw[r];
            launch->outputs[o].value = g->vreg_value[r];
            launch->n_outputs = o + 1;
        }
    }
    return true;
}

/* Would writing the group's stored outputs clobber an operand another
 * thread still reads?  Liveness lets a slot be reused once its previous
 * value's last reader ran, which inside one fused kernel is not ordered. */
static bool slot_hazard(const planner *p, const ew_group *g,
                        const bool *stored)
{
    const m3_tensor_metadata *space = meta_of(p, g->shape_value);
    int r;
    int i;

    for (r = g->n_operands; r < g->n_vregs; ++r) {
        uint32_t v = g->vreg_value[r];

        if (!stored[r] || v == NO_VALUE) {
            continue;
        }
        for (i = 0; i < g->n_operands; ++i) {
            uint32_t u = g->operand_value[i];
            const m3_tensor_metadata *mu = meta_of(p, u);
            const m3_tensor_metadata *mv = meta_of(p, v);

            if (g->operand_is_imm[i] ||
                p->plan->value_slot[u] != p->plan->value_slot[v]) {
                continue;
            }
            if (!(m3c_shape_equal(mu, space) && m3c_shape_equal(mv, space) &&
                  m3c_dtype_size(mu->dtype) == m3c_dtype_size(mv->dtype))) {
                return true;
            }
        }
    }
    return false;
}

static void mark_stored(const planner *p, const ew_group *g, bool *stored)
{
    int r;

    for (r = 0; r < g->n_vregs; ++r) {
        uint32_t v = g->vreg_value[r];

        stored[r] = false;
        if (r < g->n_operands || v == NO_VALUE) {
            continue;
        }
        /* the last vreg holding v (a value has exactly one producer) */
        if (find_vreg(g, v) != r) {
            continue;
        }
        stored[r] = p->graph->values[v].description.role == M3_GRAPH_OUTPUT ||
                    p->plan->last_uses[v] > g->last_node;
    }
}

/* Try to build a launch for the node list; false when it does not fit. */
static bool build_ew(const planner *p, const node_list *list,
                     m3c_launch *launch, ew_group *g)
{
    bool stored[VMAX];
    int i;

    if (!derive_group(p, list, g)) {
        return false;
    }
    mark_stored(p, g, stored);
    if (slot_hazard(p, g, stored)) {
        return false;
    }
    memset(launch, 0, sizeof(*launch));
    launch->kind = M3C_LAUNCH_EW;
    launch->first_node = g->first_node;
    launch->node_count = list->count;
    launch->shape_value = g->shape_value;
    launch->n_operands = g->n_operands;
    for (i = 0; i < g->n_operands; ++i) {
        launch->operands[i].ref.value =
            g->operand_is_imm[i] ? NO_VALUE : g->operand_value[i];
        launch->operands[i].load_as = g->operand_load[i];
        launch->operands[i].imm_bits = g->operand_imm[i];
    }
    if (!allocate_registers(p, g, stored, launch)) {
        return false;
    }
    launch->has_absmax = g->has_absmax;
    launch->absmax_command = g->absmax_command;
    launch->absmax_out.value = g->has_absmax ? g->absmax_value : NO_VALUE;
    return true;
}

/* Can `node` join the open group of `list`? */
static bool compatible(const planner *p, const node_list *list,
                       const m3_graph_node_desc *node)
{
    const m3_graph_node_desc *head = &p->graph->nodes[list->nodes[0]];

    if (list->count >= M3C_EW_MAX_OPS) {
        return false;
    }
    return m3c_shape_equal(meta_of(p, iteration_value(head)),
                           meta_of(p, iteration_value(node)));
}

/* Assign sides (shadow or not) to an element-wise launch's memory accesses
 * in run order, and record the commit flips. */
static m3_status finish_ew(planner *p, const ew_group *g, m3c_launch *launch,
                           m3_error *error)
{
    int i;
    m3_status status = M3_STATUS_OK;

    for (i = 0; i < launch->n_operands; ++i) {
        if (launch->operands[i].ref.value != NO_VALUE) {
            launch->operands[i].ref = read_ref(p, launch->operands[i].ref.value);
        }
    }
    for (i = 0; i < launch->n_outputs && status == M3_STATUS_OK; ++i) {
        uint32_t v = launch->outputs[i].value;
        size_t producer = p->plan->producers[v];
        bool checked = g->has_check && producer >= g->first_check_node;

        status = write_ref(p, v, checked, (uint32_t)producer,
                           &launch->outputs[i], error);
    }
    if (status == M3_STATUS_OK && launch->has_absmax) {
        status = write_ref(p, launch->absmax_out.value, true,
                           launch->absmax_command, &launch->absmax_out, error);
    }
    if (status == M3_STATUS_OK) {
        int k;
        int off = 0;

        off += snprintf(launch->text, sizeof(launch->text), "ew[");
        for (k = 0; k < (int)launch->node_count && off < 80; ++k) {
            off += snprintf(launch->text + off, sizeof(launch->text) - off,
                            "%s%s", k ? "," : "",
                            m3c_kind_name(
                                p->graph->nodes[launch->first_node + k].kind));
        }
        (void)snprintf(launch->text + off, sizeof(launch->text) - off,
                       "] stores=%d", launch->n_outputs + launch->has_absmax);
    }
    return status;
}

static m3_status flush_ew(planner *p, node_list *list, m3_error *error)
{
    m3c_launch launch;
    ew_group g;
    m3_status status;

    if (list->count == 0U) {
        return M3_STATUS_OK;
    }
    if (!build_ew(p, list, &launch, &g)) {
        return m3c_error_set(error, M3_STATUS_INTERNAL,
                             "element-wise launch does not fit");
    }
    status = finish_ew(p, &g, &launch, error);
    if (status == M3_STATUS_OK) {
        status = push_launch(p, &launch, error);
        if (list->count > 1U) {
            p->plan->fused_node_count += list->count;
        }
    }
    list->count = 0U;
    return status;
}

static bool row_pass_kind(m3_op_kind kind)
{
    return kind == M3_OP_SOFTMAX || kind == M3_OP_TOP_K ||
           kind == M3_OP_ROW_SUM;
}

static int row_pass_bit(m3_op_kind kind)
{
    return kind == M3_OP_SOFTMAX ? 0 : kind == M3_OP_TOP_K ? 1 : 2;
}

/* Row launch for SOFTMAX, TOP_K and/or ROW_SUM reading one input (one row
 * pass).  With a data-checked sibling every output is shadowed under its own
 * command, so a NaN failure commits exactly the outputs of the commands
 * before the failing one. */
static m3_status plan_softmax(planner *p, size_t n, size_t count,
                              m3_error *error)
{
    m3c_launch launch;
    size_t i;
    bool checked = false;
    char parts[3][12] = {"", "", ""};
    int named = 0;
    m3_status status = M3_STATUS_OK;

    memset(&launch, 0, sizeof(launch));
    launch.kind = M3C_LAUNCH_SOFTMAX;
    launch.first_node = n;
    launch.node_count = count;
    launch.row_in = read_ref(p, p->graph->nodes[n].inputs[0]);
    launch.row_out.value = NO_VALUE;
    launch.row_out2.value = NO_VALUE;
    launch.row_out3.value = NO_VALUE;
    launch.row_out4.value = NO_VALUE;
    launch.row_in_b.value = NO_VALUE;
    launch.row_sum_out.value = NO_VALUE;
    launch.norm_scale.value = NO_VALUE;
    launch.norm_bias.value = NO_VALUE;
    launch.command_a = UINT32_MAX;
    launch.command_b = UINT32_MAX;
    launch.command_c = UINT32_MAX;
    for (i = 0U; i < count; ++i) {
        checked = checked || p->graph->nodes[n + i].kind != M3_OP_ROW_SUM;
    }
    for (i = 0U; i < count && status == M3_STATUS_OK; ++i) {
        const m3_graph_node_desc *node = &p->graph->nodes[n + i];

        if (node->kind == M3_OP_SOFTMAX) {
            launch.command_a = (uint32_t)(n + i);
            status = write_ref(p, node->outputs[0], true, (uint32_t)(n + i),
                               &launch.row_out, error);
            (void)snprintf(parts[named++], sizeof(parts[0]), "SOFTMAX");
        } else if (node->kind == M3_OP_ROW_SUM) {
            launch.command_c = (uint32_t)(n + i);
            status = write_ref(p, node->outputs[0], checked, (uint32_t)(n + i),
                               &launch.row_out4, error);
            (void)snprintf(parts[named++], sizeof(parts[0]), "ROW_SUM");
        } else {
            launch.command_b = (uint32_t)(n + i);
            launch.k = node->parameters.top_k.k;
            status = write_ref(p, node->outputs[0], true, (uint32_t)(n + i),
                               &launch.row_out2, error);
            if (status == M3_STATUS_OK) {
                status = write_ref(p, node->outputs[1], true,
                                   (uint32_t)(n + i), &launch.row_out3, error);
            }
            (void)snprintf(parts[named++], sizeof(parts[0]), "TOP_K");
        }
    }
    (void)snprintf(launch.text, sizeof(launch.text), "row[%s%s%s%s%s]", parts[0],
                   named > 1 ? "+" : "", parts[1], named > 2 ? "+" : "", parts[2]);
    if (status == M3_STATUS_OK) {
        status = push_launch(p, &launch, error);
        if (count > 1U) {
            p->plan->fused_node_count += count;
        }
    }
    return status;
}

/* Row launch for categorical sampling; its output is checked (written to
 * the shadow buffer and committed only when the run is clean). */
static m3_status plan_categorical(planner *p, size_t n, m3_error *error)
{
    const m3_graph_node_desc *node = &p->graph->nodes[n];
    m3c_launch launch;
    m3_status status;

    memset(&launch, 0, sizeof(launch));
    launch.kind = M3C_LAUNCH_CATEGORICAL;
    launch.first_node = n;
    launch.node_count = 1U;
    launch.row_in = read_ref(p, node->inputs[0]);
    launch.row_in_b = read_ref(p, node->inputs[1]);
    launch.row_sum_out.value = NO_VALUE;
    launch.row_out2.value = NO_VALUE;
    launch.row_out3.value = NO_VALUE;
    launch.norm_scale.value = NO_VALUE;
    launch.norm_bias.value = NO_VALUE;
    launch.command_a = (uint32_t)n;
    launch.command_b = UINT32_MAX;
    status = write_ref(p, node->outputs[0], true, (uint32_t)n, &launch.row_out,
                       error);
    (void)snprintf(launch.text, sizeof(launch.text), "row[CATEGORICAL]");
    if (status == M3_STATUS_OK) {
        status = push_launch(p, &launch, error);
    }
    return status;
}

/* Row launch for a norm; `residual` is the index of an ADD node whose output
 * is the norm input and that runs as the kernel's prologue (or SIZE_MAX). */
static m3_status plan_norm(planner *p, size_t n, size_t residual,
                           m3_error *error)
{
    const m3_graph_node_desc *node = &p->graph->nodes[n];
    m3c_launch launch;
    m3_status status = M3_STATUS_OK;

    memset(&launch, 0, sizeof(launch));
    launch.kind = M3C_LAUNCH_NORM;
    launch.first_node = residual != SIZE_MAX ? residual : n;
    launch.node_count = residual != SIZE_MAX ? 2U : 1U;
    launch.layer_norm = node->kind == M3_OP_LAYER_NORM;
    launch.epsilon = node->parameters.norm.epsilon;
    launch.row_in_b.value = NO_VALUE;
    launch.row_sum_out.value = NO_VALUE;
    launch.row_out2.value = NO_VALUE;
    launch.row_out3.value = NO_VALUE;
    launch.command_a = (uint32_t)n;
    launch.command_b = UINT32_MAX;
    if (residual != SIZE_MAX) {
        const m3_graph_node_desc *add = &p->graph->nodes[residual];

        launch.row_in = read_ref(p, add->inputs[0]);
        launch.row_in_b = read_ref(p, add->inputs[1]);
    } else {
        launch.row_in = read_ref(p, node->inputs[0]);
    }
    launch.norm_scale = read_ref(p, node->inputs[1]);
    launch.norm_bias.value = NO_VALUE;
    if (launch.layer_norm && node->inputs[2] != M3_GRAPH_VALUE_NONE) {
        launch.norm_bias = read_ref(p, node->inputs[2]);
    }
    if (residual != SIZE_MAX) {
        uint32_t sum = p->graph->nodes[residual].outputs[0];

        if (p->graph->values[sum].description.role == M3_GRAPH_OUTPUT ||
            p->plan->last_uses[sum] > n) {
            status = write_ref(p, sum, false, (uint32_t)residual,
                               &launch.row_sum_out, error);
        }
        p->plan->fused_node_count += 2U;
    }
    if (status == M3_STATUS_OK) {
        status = write_ref(p, node->outputs[0], false, (uint32_t)n,
                           &launch.row_out, error);
    }
    (void)snprintf(launch.text, sizeof(launch.text), "row[%s%s]",
                   residual != SIZE_MAX ? "ADD+" : "",
                   launch.layer_norm ? "LAYER_NORM" : "RMS_NORM");
    return status == M3_STATUS_OK ? push_launch(p, &launch, error) : status;
}

/* An ADD that can run as a norm prologue: same shape and dtype for both
 * operands and the sum, the sum not read by another node of the list. */
static bool residual_prologue(const planner *p, const node_list *open,
                              size_t norm_node)
{
    const m3_graph_node_desc *norm = &p->graph->nodes[norm_node];
    const m3_graph_node_desc *add;
    const m3_tensor_metadata *s;
    const m3_tensor_metadata *a;
    const m3_tensor_metadata *b;
    size_t producer;

    if (open->count != 1U) {
        return false;
    }
    producer = p->plan->producers[norm->inputs[0]];
    if (producer != open->nodes[0] || producer + 1U != norm_node) {
        return false;
    }
    add = &p->graph->nodes[producer];
    if (add->kind != M3_OP_ADD) {
        return false;
    }
    s = meta_of(p, add->outputs[0]);
    a = meta_of(p, add->inputs[0]);
    b = meta_of(p, add->inputs[1]);
    if (!m3c_shape_equal(a, s) || !m3c_shape_equal(b, s) ||
        a->dtype != s->dtype || b->dtype != s->dtype) {
        return false;
    }
    /* the kernel writes the sum and the norm output while other rows still
     * read the operands: liveness may have given an operand's slot to one
     * of them, which only the unfused order makes safe */
    {
        size_t sa = p->plan->value_slot[add->inputs[0]];
        size_t sb = p->plan->value_slot[add->inputs[1]];
        size_t ss = p->plan->value_slot[add->outputs[0]];
        size_t so = p->plan->value_slot[norm->outputs[0]];

        if (sa == ss || sb == ss || sa == so || sb == so) {
            return false;
        }
    }
    return true;
}

static m3_status fuse(planner *p, bool fuse_enabled, m3_error *error)
{
    const m3_graph *graph = p->graph;
    node_list open;
    size_t n = 0U;
    m3_status status = M3_STATUS_OK;

    open.count = 0U;
    while (n < graph->node_count && status == M3_STATUS_OK) {
        const m3_graph_node_desc *node = &graph->nodes[n];

        if (is_elementwise(node->kind)) {
            if (open.count > 0U && fuse_enabled && compatible(p, &open, node)) {
                node_list trial = open;
                m3c_launch scratch;
                ew_group g;

                trial.nodes[trial.count++] = n;
                if (build_ew(p, &trial, &scratch, &g)) {
                    open = trial;
                    ++n;
                    continue;
                }
            }
            status = flush_ew(p, &open, error);
            open.nodes[0] = n;
            open.count = 1U;
            if (status == M3_STATUS_OK) {
                m3c_launch scratch;
                ew_group g;

                if (!build_ew(p, &open, &scratch, &g)) {
                    status = m3c_error_set(
                        error, M3_STATUS_INTERNAL,
                        "operation %s does not fit the element-wise kernel",
                        m3c_kind_name(node->kind));
                }
            }
            ++n;
            continue;
        }
        if (node->kind == M3_OP_RMS_NORM || node->kind == M3_OP_LAYER_NORM) {
            if (fuse_enabled && residual_prologue(p, &open, n)) {
                size_t add = open.nodes[0];

                open.count = 0U;
                status = plan_norm(p, n, add, error);
            } else {
                status = flush_ew(p, &open, error);
                if (status == M3_STATUS_OK) {
                    status = plan_norm(p, n, SIZE_MAX, error);
                }
            }
            ++n;
            continue;
        }
        status = flush_ew(p, &open, error);
        if (status != M3_STATUS_OK) {
            break;
        }
        if (node->kind == M3_OP_CATEGORICAL) {
            status = plan_categorical(p, n, error);
            ++n;
            continue;
        }
        if (row_pass_kind(node->kind)) {
            /* siblings: consecutive SOFTMAX / TOP_K / ROW_SUM nodes of
             * distinct kinds reading the same input share one row pass */
            size_t count = 1U;
            unsigned seen = 1U << row_pass_bit(node->kind);

            while (fuse_enabled && count < 3U && n + count < graph->node_count) {
                const m3_graph_node_desc *next = &graph->nodes[n + count];

                if (!row_pass_kind(next->kind) ||
                    (seen & (1U << row_pass_bit(next->kind))) != 0U ||
                    next->inputs[0] != node->inputs[0]) {
                    break;
                }
                seen |= 1U << row_pass_bit(next->kind);
                ++count;
            }
            status = plan_softmax(p, n, count, error);
            n += count;
            continue;
        }
        status = m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                               "no enabled provider supports the command list");
    }
    if (status == M3_STATUS_OK) {
        status = flush_ew(p, &open, error);
    }
    return status;
}

/* ----------------------------------------------------------------- entry */

void m3c_plan_free(m3c_plan *plan)
{
    if (plan == NULL) {
        return;
    }
    free(plan->value_slot);
    free(plan->slot_bytes);
    free(plan->producers);
    free(plan->last_uses);
    free(plan->slot_shadowed);
    free(plan->slot_needed);
    free(plan->launches);
    free(plan->flip_slot);
    free(plan->flip_command);
    memset(plan, 0, sizeof(*plan));
}

static size_t align_up(size_t value)
{
    return (value + M3C_ARENA_ALIGNMENT - 1U) &
           ~(size_t)(M3C_ARENA_ALIGNMENT - 1U);
}

static void mark_ref(m3c_plan *plan, m3c_ref ref)
{
    if (ref.value != UINT32_MAX && ref.value < plan->value_count) {
        plan->slot_needed[plan->value_slot[ref.value]] = true;
    }
}

/* Slots that need memory: every slot holding an input, output or constant
 * (the host writes or reads them) and every slot a launch reads or stores.
 * A temporary that lives only in the registers of a fused launch needs
 * none. */
static m3_status mark_needed_slots(const m3_graph *graph, m3c_plan *plan,
                                   m3_error *error)
{
    size_t v;
    size_t l;
    int k;

    plan->slot_needed = calloc(plan->slot_count ? plan->slot_count : 1U, sizeof(bool));
    if (plan->slot_needed == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate slot plan");
    }
    for (v = 0U; v < plan->value_count; ++v) {
        if (graph->values[v].description.role != M3_GRAPH_TEMPORARY) {
            plan->slot_needed[plan->value_slot[v]] = true;
        }
    }
    for (l = 0U; l < plan->launch_count; ++l) {
        const m3c_launch *launch = &plan->launches[l];

        if (launch->kind == M3C_LAUNCH_EW) {
            for (k = 0; k < launch->n_operands; ++k) {
                mark_ref(plan, launch->operands[k].ref);
            }
            for (k = 0; k < launch->n_outputs; ++k) {
                mark_ref(plan, launch->outputs[k]);
            }
            if (launch->has_absmax) {
                mark_ref(plan, launch->absmax_out);
            }
            continue;
        }
        mark_ref(plan, launch->row_in);
        mark_ref(plan, launch->row_out);
        if (launch->kind == M3C_LAUNCH_CATEGORICAL) {
            mark_ref(plan, launch->row_in_b);
        } else if (launch->kind == M3C_LAUNCH_SOFTMAX) {
            mark_ref(plan, launch->row_out2);
            mark_ref(plan, launch->row_out3);
            mark_ref(plan, launch->row_out4);
        } else {
            mark_ref(plan, launch->row_in_b);
            mark_ref(plan, launch->row_sum_out);
            mark_ref(plan, launch->norm_scale);
            mark_ref(plan, launch->norm_bias);
        }
    }
    return M3_STATUS_OK;
}

m3_status m3c_plan_build(const m3_graph *graph, bool fuse_enabled,
                         m3c_plan *plan, m3_error *error)
{
    planner p;
    size_t count;
    size_t n;
    size_t s;
    m3_status status;

    memset(plan, 0, sizeof(*plan));
    if (graph == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "graph is required");
    }
    count = graph->value_count ? graph->value_count : 1U;
    plan->value_count = graph->value_count;
    plan->node_count = graph->node_count;
    plan->value_slot = calloc(count, sizeof(size_t));
    plan->slot_bytes = calloc(count, sizeof(size_t));
    plan->producers = calloc(count, sizeof(size_t));
    plan->last_uses = calloc(count, sizeof(size_t));
    plan->slot_shadowed = calloc(count, sizeof(bool));
    if (plan->value_slot == NULL || plan->slot_bytes == NULL ||
        plan->producers == NULL || plan->last_uses == NULL ||
        plan->slot_shadowed == NULL) {
        m3c_plan_free(plan);
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate session plan arrays");
    }
    status = topology(graph, plan->producers, plan->last_uses, error);
    if (status == M3_STATUS_OK) {
        status = plan_slots(graph, plan, error);
    }
    for (n = 0U; status == M3_STATUS_OK && n < graph->node_count; ++n) {
        if (!m3c_kind_supported(graph->nodes[n].kind)) {
            status = m3c_error_set(
                error, M3_STATUS_UNSUPPORTED,
                "no enabled provider supports the command list");
            break;
        }
        status = validate_node(graph, plan, &graph->nodes[n], error);
    }
    if (status == M3_STATUS_OK) {
        memset(&p, 0, sizeof(p));
        p.graph = graph;
        p.plan = plan;
        p.side = calloc(count, 1U);
        if (p.side == NULL) {
            status = m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                   "cannot allocate commit state");
        } else {
            status = fuse(&p, fuse_enabled, error);
            free(p.side);
        }
    }
    if (status != M3_STATUS_OK) {
        m3c_plan_free(plan);
        return status;
    }
    status = mark_needed_slots(graph, plan, error);
    if (status != M3_STATUS_OK) {
        m3c_plan_free(plan);
        return status;
    }
    plan->arena_bytes = 0U;
    plan->shadow_bytes = 0U;
    for (s = 0U; s < plan->slot_count; ++s) {
        if (!plan->slot_needed[s]) {
            continue;
        }
        plan->arena_bytes += align_up(plan->slot_bytes[s]);
        if (plan->slot_shadowed[s]) {
            plan->shadow_bytes += align_up(plan->slot_bytes[s]);
        }
    }
    plan->arena_bytes += plan->shadow_bytes;
    (void)canonical_strides;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

void m3c_plan_describe(const m3c_plan *plan, char *text, size_t capacity)
{
    size_t off = 0U;
    size_t i;

    if (text == NULL || capacity == 0U) {
        return;
    }
    text[0] = '\0';
    for (i = 0U; i < plan->launch_count && off + 1U < capacity; ++i) {
        int written = snprintf(text + off, capacity - off, "%s%s",
                               i ? "; " : "", plan->launches[i].text);

        if (written < 0) {
            break;
        }
        off += (size_t)written;
    }
}
