/* Sessions of the m3.h API on one CUDA device.
 *
 * Compile (m3_session_create): the host planner (m3c_plan.c) produces the
 * reference's liveness slots and the fused launch list; the session then
 * allocates ONE device arena holding every slot (256-byte aligned offsets)
 * plus a shadow buffer for each slot written by a data-checked command, and
 * uploads the constants.
 *
 * Run (m3_session_run = run_async + synchronize): each launch's parameters
 * are resolved from the current slot buffers and the kernels are enqueued on
 * the session's stream.  Kernels skip their work once an earlier command of
 * the run has failed a data check (the device status word), so a failing run
 * stops exactly where the reference stops.  On the host, every slot written
 * to its shadow side flips after the run; when a synchronise finds a failure,
 * the flips are replayed from the last synchronised state, keeping only those
 * of commands before the failing one (reference semantics: outputs of the
 * failing command and of everything after it are unchanged).
 *
 * I/O: m3_session_write_input / read_output copy host <-> device through the
 * stream and return after the copy, like the reference's memcpy-based
 * storage I/O (src/m3_graph_session.c:58-98). */

#include "m3c_internal.h"

#include <cuda_runtime_api.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef enum { EVENT_RUN = 0, EVENT_SWAP } event_kind;

typedef struct {
    event_kind kind;
    size_t slot_a;
    size_t slot_b;
} session_event;

/* Launches of one run that may execute at the same time: up to
 * 1 + M3C_SIDE_STREAMS per wave. */
#define M3C_SIDE_STREAMS 3

/* A captured sequence of `runs` runs with slots swap_a/swap_b exchanged
 * between consecutive runs (SIZE_MAX: none), valid for the buffer assignment
 * it was captured from (kernel parameters hold buffer addresses). */
#define M3C_RUN_GRAPHS 8

typedef struct {
    size_t runs;
    size_t swap_a;
    size_t swap_b;
    unsigned char **start_buffer[2];
    uint8_t *start_current;
    cudaGraphExec_t exec;
} run_graph;

/* Pipelined host submissions (m3_cuda_session_submit_host_async): uploads
 * on one stream and downloads on another, through two staging areas used in
 * turn, so one submission's upload overlaps the previous one's download. */
typedef struct {
    cudaStream_t upload;
    cudaStream_t download;
    unsigned char *stage_in[2];
    unsigned char *stage_out[2];
    size_t in_bytes;
    size_t out_bytes;
    cudaEvent_t uploaded[2];   /* staging input filled */
    cudaEvent_t consumed[2];   /* staging input copied into the session */
    cudaEvent_t produced[2];   /* staging output filled */
    cudaEvent_t drained[2];    /* staging output copied to the host */
    unsigned turn;
    bool ready;
} host_pipe;

struct m3_session {
    m3c_plan plan;
    m3_graph_value_desc *descriptions;
    m3_tensor_metadata *metadata;
    m3_op_kind *node_kinds;
    m3_cuda_session_options cuda;
    int device;
    cudaStream_t stream;
    bool own_stream;
    unsigned char *arena;
    /* per slot: the two buffers and which one is current */
    unsigned char **buffer[2];
    uint8_t *current;
    /* state at the last synchronise, for replay after a failure */
    unsigned char **sync_buffer[2];
    uint8_t *sync_current;
    session_event *events;
    size_t event_count;
    size_t event_capacity;
    size_t pending_runs;
    m3c_status *status_device;
    m3c_status *status_host;         /* pinned */
    m3c_reduce_scratch *reduce;      /* one per launch */
    m3c_ew_params *ew_templates;     /* one per launch (EW launches only) */
    m3c_ew_choice *ew_choices;       /* kernel and grid of each EW launch */
    /* a failure found by an implicit synchronise, reported by the next
     * explicit one */
    m3_status sticky_status;
    m3_error sticky_error;
    /* captured run sequences, replayed as one graph launch each */
    run_graph graphs[M3C_RUN_GRAPHS];
    size_t graph_count;
    size_t graph_next;
    /* host submissions: copy streams, double-buffered staging, events */
    host_pipe pipe;
    /* this rank's share of a sharded session (NULL: not sharded) */
    m3c_shard *shard;
    /* concurrent launches: wave_join[i] is true when launch i runs beside
     * the launches before it in its wave (independent slots, no data check
     * before it in the run); side streams and fork/join events */
    bool *wave_join;
    cudaStream_t side[M3C_SIDE_STREAMS];
    cudaEvent_t fork_event;
    cudaEvent_t join_event[M3C_SIDE_STREAMS];
};

static const m3c_status clean_status = {UINT32_MAX, 0U, 0U, UINT32_MAX};

/* ------------------------------------------------------------ helpers */

static m3_status cuda_failure(m3_error *error, cudaError_t code,
                              const char *what)
{
    m3_status status = code == cudaErrorMemoryAllocation
                           ? M3_STATUS_OUT_OF_MEMORY
                           : M3_STATUS_INTERNAL;

    (void)cudaGetLastError();
    return m3c_error_set(error, status, "%s: %s", what,
                         cudaGetErrorString(code));
}

static m3_status use_device(const m3_session *session, m3_error *error)
{
    int current = -1;
    cudaError_t code = cudaGetDevice(&current);

    if (code == cudaSuccess && current != session->device) {
        code = cudaSetDevice(session->device);
    }
    return code == cudaSuccess ? M3_STATUS_OK
                               : cuda_failure(error, code, "cannot select device");
}

void m3_cuda_session_options_init(m3_cuda_session_options *options)
{
    if (options != NULL) {
        options->device = M3_CUDA_DEVICE_CURRENT;
        options->stream = NULL;
        options->fuse = true;
        options->cuda_graphs = true;
    }
}

static unsigned char *value_pointer(const m3_session *s, uint32_t value,
                                    bool shadow)
{
    size_t slot = s->plan.value_slot[value];
    int side = (int)(s->current[slot] ^ (shadow ? 1U : 0U));

    return s->buffer[side][slot];
}

static unsigned char *ref_pointer(const m3_session *s, m3c_ref ref)
{
    return ref.value == UINT32_MAX ? NULL
                                   : value_pointer(s, ref.value, ref.shadow);
}

/* ---------------------------------------------------------- lifecycle */

static void drop_graph(run_graph *g)
{
    if (g->exec != NULL) {
        (void)cudaGraphExecDestroy(g->exec);
    }
    free(g->start_buffer[0]);
    free(g->start_buffer[1]);
    free(g->start_current);
    memset(g, 0, sizeof(*g));
}

static void drop_pipe(host_pipe *p)
{
    int k;

    if (p->upload != NULL) {
        (void)cudaStreamSynchronize(p->upload);
        (void)cudaStreamDestroy(p->upload);
    }
    if (p->download != NULL) {
        (void)cudaStreamSynchronize(p->download);
        (void)cudaStreamDestroy(p->download);
    }
    for (k = 0; k < 2; ++k) {
        (void)cudaFree(p->stage_in[k]);
        (void)cudaFree(p->stage_out[k]);
        if (p->uploaded[k] != NULL) (void)cudaEventDestroy(p->uploaded[k]);
        if (p->consumed[k] != NULL) (void)cudaEventDestroy(p->consumed[k]);
        if (p->produced[k] != NULL) (void)cudaEventDestroy(p->produced[k]);
        if (p->drained[k] != NULL) (void)cudaEventDestroy(p->drained[k]);
    }
    memset(p, 0, sizeof(*p));
}

void m3_session_free(m3_session *session)
{
    if (session == NULL) {
        return;
    }
    if (session->stream != NULL || session->arena != NULL) {
        int current = -1;

        if (cudaGetDevice(&current) == cudaSuccess &&
            current != session->device) {
            (void)cudaSetDevice(session->device);
        }
        if (session->stream != NULL) {
            (void)cudaStreamSynchronize(session->stream);
        }
    }
    for (size_t g = 0; g < session->graph_count; ++g) {
        drop_graph(&session->graphs[g]);
    }
    drop_pipe(&session->pipe);
    if (session->shard != NULL) {
        /* the stream is idle: no collective of this communicator is pending */
        m3c_comm_destroy(session->shard->comm);
        session->shard->comm = NULL;
        (void)cudaFree(session->shard->staging);
        session->shard->staging = NULL;
        m3c_shard_free(session->shard);
        session->shard = NULL;
    }
    if (session->arena != NULL) {
        (void)cudaFree(session->arena);
    }
    if (session->status_device != NULL) {
        (void)cudaFree(session->status_device);
    }
    if (session->reduce != NULL) {
        (void)cudaFree(session->reduce);
    }
    if (session->status_host != NULL) {
        (void)cudaFreeHost(session->status_host);
    }
    for (int k = 0; k < M3C_SIDE_STREAMS; ++k) {
        if (session->side[k] != NULL) {
            (void)cudaStreamSynchronize(session->side[k]);
            (void)cudaStreamDestroy(session->side[k]);
        }
        if (session->join_event[k] != NULL) {
            (void)cudaEventDestroy(session->join_event[k]);
        }
    }
    if (session->fork_event != NULL) {
        (void)cudaEventDestroy(session->fork_event);
    }
    free(session->wave_join);
    if (session->own_stream && session->stream != NULL) {
        (void)cudaStreamDestroy(session->stream);
    }
    (void)cudaGetLastError();
    free(session->buffer[0]);
    free(session->buffer[1]);
    free(session->sync_buffer[0]);
    free(session->sync_buffer[1]);
    free(session->current);
    free(session->sync_current);
    free(session->events);
    free(session->ew_templates);
    free(session->ew_choices);
    free(session->descriptions);
    free(session->metadata);
    free(session->node_kinds);
    m3c_plan_free(&session->plan);
    free(session);
}

static size_t align_up(size_t value)
{
    return (value + M3C_ARENA_ALIGNMENT - 1U) &
           ~(size_t)(M3C_ARENA_ALIGNMENT - 1U);
}

/* Element-wise launch templates: operand addressing is fixed at compile
 * time; only base pointers change between runs. */
static void build_templates(m3_session *s)
{
    size_t i;

    for (i = 0U; i < s->plan.launch_count; ++i) {
        const m3c_launch *l = &s->plan.launches[i];
        m3c_ew_params *t = &s->ew_templates[i];
        const m3_tensor_metadata *space;
        int k;

        memset(t, 0, sizeof(*t));
        if (l->kind != M3C_LAUNCH_EW) {
            continue;
        }
        space = &s->metadata[l->shape_value];
        t->count = space->element_count;
        t->n_operands = l->n_operands;
        t->n_ops = l->n_ops;
        t->n_outputs = l->n_outputs;
        for (k = 0; k < l->n_operands; ++k) {
            const m3c_ew_operand_plan *o = &l->operands[k];

            if (o->ref.value == UINT32_MAX) {
                t->operands[k].vclass = M3C_V_IMM;
                t->operands[k].imm_bits = o->imm_bits;
                t->operands[k].load_as = o->load_as;
            } else {
                const m3_tensor_metadata *m = &s->metadata[o->ref.value];
                size_t strides[M3_TENSOR_MAX_RANK];
                size_t stride = m3c_dtype_size(m->dtype);
                int axis;

                for (axis = (int)m->rank - 1; axis >= 0; --axis) {
                    strides[axis] = stride;
                    stride *= (size_t)m->shape[axis];
                }
                /* buffers are arena-aligned, so buffer 0 stands for both */
                m3c_operand_setup(&t->operands[k],
                                  s->buffer[0][s->plan.value_slot[o->ref.value]],
                                  m, 0U, strides, space, o->load_as);
            }
        }
        memcpy(t->ops, l->ops, sizeof(t->ops));
        for (k = 0; k < l->n_outputs; ++k) {
            t->outputs[k].dtype = (int32_t)s->metadata[l->outputs[k].value].dtype;
            t->outputs[k].reg = (int16_t)l->output_regs[k];
            t->outputs[k].raw = l->output_raw[k] ? 1 : 0;
        }
        t->absmax_command = l->absmax_command;
        {
            /* the choice depends on whether the launch reduces */
            m3c_ew_params probe = *t;

            probe.reduce = l->has_absmax ? &s->reduce[i] : NULL;
            (void)m3c_ew_choose(&probe, &s->ew_choices[i]);
        }
    }
}

/* Slots a launch reads or writes (both buffers of a slot count as one). */
static size_t launch_slots(const m3c_plan *plan, const m3c_launch *l,
                           size_t *slots, size_t capacity)
{
    m3c_ref refs[M3C_EW_MAX_OPERANDS + M3C_EW_MAX_OUTPUTS + 12];
    size_t n = 0U;
    size_t count = 0U;
    size_t i;
    int k;

    if (l->kind == M3C_LAUNCH_EW) {
        for (k = 0; k < l->n_operands; ++k) refs[n++] = l->operands[k].ref;
        for (k = 0; k < l->n_outputs; ++k) refs[n++] = l->outputs[k];
        if (l->has_absmax) refs[n++] = l->absmax_out;
    } else {
        refs[n++] = l->row_in;
        refs[n++] = l->row_in_b;
        refs[n++] = l->row_sum_out;
        refs[n++] = l->row_out;
        refs[n++] = l->row_out2;
        refs[n++] = l->row_out3;
        refs[n++] = l->row_out4;
        refs[n++] = l->norm_scale;
        refs[n++] = l->norm_bias;
    }
    for (i = 0U; i < n && count < capacity; ++i) {
        if (refs[i].value != UINT32_MAX) {
            slots[count++] = plan->value_slot[refs[i].value];
        }
    }
    return count;
}

/* Waves of launches that may run at the same time: only in a plan without
 * data checks (no launch can fail, so no later launch must wait for an
 * earlier one's verdict), a launch joins the wave before it when it shares
 * no slot with any launch of that wave. */
static m3_status plan_waves(m3_session *s, m3_error *error)
{
    size_t n = s->plan.launch_count;
    size_t wave_start = 0U;
    size_t i;
    size_t widest = 0U;
    enum { CAP = 32 };

    if (n < 2U || s->plan.flip_count != 0U) {
        return M3_STATUS_OK;
    }
    s->wave_join = calloc(n, sizeof(bool));
    if (s->wave_join == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate the launch waves");
    }
    for (i = 1U; i < n; ++i) {
        size_t mine[CAP];
        size_t mine_count = launch_slots(&s->plan, &s->plan.launches[i], mine, CAP);
        bool independent = i - wave_start <= M3C_SIDE_STREAMS;
        size_t j;

        for (j = wave_start; j < i && independent; ++j) {
            size_t theirs[CAP];
            size_t theirs_count = launch_slots(&s->plan, &s->plan.launches[j], theirs, CAP);
            size_t a;
            size_t b;

            for (a = 0U; a < mine_count && independent; ++a) {
                for (b = 0U; b < theirs_count; ++b) {
                    if (mine[a] == theirs[b]) {
                        independent = false;
                        break;
                    }
                }
            }
        }
        if (independent) {
            s->wave_join[i] = true;
            if (i - wave_start > widest) {
                widest = i - wave_start;
            }
        } else {
            wave_start = i;
        }
    }
    if (widest == 0U) {
        free(s->wave_join);
        s->wave_join = NULL;
        return M3_STATUS_OK;
    }
    {
        cudaError_t code = cudaEventCreateWithFlags(&s->fork_event,
                                                    cudaEventDisableTiming);

        for (i = 0U; code == cudaSuccess && i < widest; ++i) {
            code = cudaStreamCreateWithFlags(&s->side[i], cudaStreamNonBlocking);
            if (code == cudaSuccess) {
                code = cudaEventCreateWithFlags(&s->join_event[i],
                                                cudaEventDisableTiming);
            }
        }
        if (code != cudaSuccess) {
            return cuda_failure(error, code, "cannot create side streams");
        }
    }
    return M3_STATUS_OK;
}

m3_status m3_cuda_session_create(m3_session **session_output,
                                  const m3_graph *graph,
                                  const m3_session_options *options,
                                  const m3_cuda_session_options *cuda,
                                  m3_error *error)
{
    m3_session_options selected;
    m3_session *s;
    size_t slot;
    size_t offset;
    size_t count;
    cudaError_t code;
    m3_status status;
    int devices = 0;

    if (session_output == NULL || *session_output != NULL || graph == NULL) {
        return m3c_error_set(
            error, M3_STATUS_INVALID_ARGUMENT,
            "session output must be empty and graph is required");
    }
    m3_session_options_init(&selected);
    if (options != NULL) {
        selected = *options;
    }
    if (!selected.allow_neural_engine && !selected.allow_metal &&
        !selected.allow_cpu) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session has no enabled provider");
    }
    s = calloc(1U, sizeof(*s));
    if (s == NULL) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate session");
    }
    m3_cuda_session_options_init(&s->cuda);
    if (cuda != NULL) {
        s->cuda = *cuda;
    }
    s->device = -1;
    status = m3c_plan_build(graph, s->cuda.fuse, &s->plan, error);
    if (status != M3_STATUS_OK) {
        free(s);
        return status;
    }
    if (!selected.allow_metal && !selected.allow_neural_engine &&
        graph->node_count != 0U) {
        m3_session_free(s);
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "no enabled provider supports the command list");
    }
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
        (void)cudaGetLastError();
        m3_session_free(s);
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED,
                             "no CUDA device is available");
    }
    if (s->cuda.device == M3_CUDA_DEVICE_CURRENT) {
        code = cudaGetDevice(&s->device);
    } else {
        s->device = s->cuda.device;
        code = cudaSetDevice(s->device);
    }
    if (code != cudaSuccess) {
        m3_session_free(s);
        return cuda_failure(error, code, "cannot select device");
    }
    count = graph->value_count ? graph->value_count : 1U;
    s->descriptions = calloc(count, sizeof(*s->descriptions));
    s->metadata = calloc(count, sizeof(*s->metadata));
    s->buffer[0] = calloc(count, sizeof(unsigned char *));
    s->buffer[1] = calloc(count, sizeof(unsigned char *));
    s->sync_buffer[0] = calloc(count, sizeof(unsigned char *));
    s->sync_buffer[1] = calloc(count, sizeof(unsigned char *));
    s->current = calloc(count, 1U);
    s->sync_current = calloc(count, 1U);
    s->ew_templates = calloc(s->plan.launch_count ? s->plan.launch_count : 1U,
                             sizeof(*s->ew_templates));
    s->ew_choices = calloc(s->plan.launch_count ? s->plan.launch_count : 1U,
                           sizeof(*s->ew_choices));
    s->node_kinds = calloc(graph->node_count ? graph->node_count : 1U,
                           sizeof(*s->node_kinds));
    if (s->node_kinds != NULL) {
        for (slot = 0U; slot < graph->node_count; ++slot) {
            s->node_kinds[slot] = graph->nodes[slot].kind;
        }
    }
    if (s->descriptions == NULL || s->metadata == NULL ||
        s->node_kinds == NULL ||
        s->buffer[0] == NULL || s->buffer[1] == NULL ||
        s->sync_buffer[0] == NULL || s->sync_buffer[1] == NULL ||
        s->current == NULL || s->sync_current == NULL ||
        s->ew_templates == NULL || s->ew_choices == NULL) {
        m3_session_free(s);
        return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                             "cannot allocate session plan arrays");
    }
    for (slot = 0U; slot < graph->value_count; ++slot) {
        s->descriptions[slot] = graph->values[slot].description;
        s->metadata[slot] = graph->values[slot].metadata;
    }
    if (s->cuda.stream != NULL) {
        s->stream = (cudaStream_t)s->cuda.stream;
    } else {
        code = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
        if (code != cudaSuccess) {
            m3_session_free(s);
            return cuda_failure(error, code, "cannot create stream");
        }
        s->own_stream = true;
    }
    /* one arena: every slot, then the shadow buffers */
    code = cudaMalloc((void **)&s->arena,
                      s->plan.arena_bytes ? s->plan.arena_bytes
                                          : M3C_ARENA_ALIGNMENT);
    if (code != cudaSuccess) {
        s->arena = NULL;
        m3_session_free(s);
        return cuda_failure(error, code, "cannot allocate the device arena");
    }
    offset = 0U;
    for (slot = 0U; slot < s->plan.slot_count; ++slot) {
        if (!s->plan.slot_needed[slot]) {
            s->buffer[0][slot] = NULL;   /* lives in registers only */
            continue;
        }
        s->buffer[0][slot] = s->arena + offset;
        offset += align_up(s->plan.slot_bytes[slot]);
    }
    for (slot = 0U; slot < s->plan.slot_count; ++slot) {
        if (s->plan.slot_shadowed[slot] && s->plan.slot_needed[slot]) {
            s->buffer[1][slot] = s->arena + offset;
            offset += align_up(s->plan.slot_bytes[slot]);
        } else {
            s->buffer[1][slot] = s->buffer[0][slot];
        }
    }
    code = cudaMalloc((void **)&s->status_device, sizeof(m3c_status));
    if (code == cudaSuccess) {
        code = cudaMalloc((void **)&s->reduce,
                          (s->plan.launch_count ? s->plan.launch_count : 1U) *
                              sizeof(m3c_reduce_scratch));
    }
    if (code == cudaSuccess) {
        code = cudaMallocHost((void **)&s->status_host, sizeof(m3c_status));
    }
    if (code == cudaSuccess) {
        code = cudaMemcpy(s->status_device, &clean_status,
                          sizeof(clean_status), cudaMemcpyHostToDevice);
    }
    if (code == cudaSuccess) {
        code = cudaMemset(s->reduce, 0,
                          (s->plan.launch_count ? s->plan.launch_count : 1U) *
                              sizeof(m3c_reduce_scratch));
    }
    for (slot = 0U; code == cudaSuccess && slot < graph->value_count; ++slot) {
        const m3c_graph_value *v = &graph->values[slot];

        if (v->description.role == M3_GRAPH_CONSTANT && v->constant_size) {
            code = cudaMemcpy(s->buffer[0][s->plan.value_slot[slot]],
                              v->constant_data, v->constant_size,
                              cudaMemcpyHostToDevice);
        }
    }
    if (code != cudaSuccess) {
        m3_session_free(s);
        return cuda_failure(error, code, "cannot initialise session memory");
    }
    build_templates(s);
    status = plan_waves(s, error);
    if (status != M3_STATUS_OK) {
        m3_session_free(s);
        return status;
    }
    memcpy(s->sync_buffer[0], s->buffer[0], count * sizeof(unsigned char *));
    memcpy(s->sync_buffer[1], s->buffer[1], count * sizeof(unsigned char *));
    s->sticky_status = M3_STATUS_OK;
    *session_output = s;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_session_create(m3_session **session, const m3_graph *graph,
                             const m3_session_options *options,
                             m3_error *error)
{
    return m3_cuda_session_create(session, graph, options, NULL, error);
}

/* ---------------------------------------------------------------- runs */

static m3_status push_event(m3_session *s, event_kind kind, size_t a,
                            size_t b, m3_error *error)
{
    if (s->event_count == s->event_capacity) {
        size_t wanted = s->event_capacity ? s->event_capacity * 2U : 16U;
        session_event *moved = realloc(s->events, wanted * sizeof(*moved));

        if (moved == NULL) {
            return m3c_error_set(error, M3_STATUS_OUT_OF_MEMORY,
                                 "cannot record session event");
        }
        s->events = moved;
        s->event_capacity = wanted;
    }
    s->events[s->event_count].kind = kind;
    s->events[s->event_count].slot_a = a;
    s->events[s->event_count].slot_b = b;
    ++s->event_count;
    return M3_STATUS_OK;
}

static int launch_one(m3_session *s, size_t index, bool first, cudaStream_t stream)
{
    const m3c_launch *l = &s->plan.launches[index];

    if (l->kind == M3C_LAUNCH_EW) {
        m3c_ew_params p = s->ew_templates[index];
        int k;

        for (k = 0; k < l->n_operands; ++k) {
            if (l->operands[k].ref.value != UINT32_MAX) {
                p.operands[k].base = ref_pointer(s, l->operands[k].ref);
            }
        }
        for (k = 0; k < l->n_outputs; ++k) {
            p.outputs[k].base = ref_pointer(s, l->outputs[k]);
        }
        p.first_of_run = first ? 1 : 0;
        p.status = s->status_device;
        p.skip_before = (uint32_t)l->first_node;
        if (l->has_absmax) {
            p.reduce = &s->reduce[index];
            p.absmax_out = ref_pointer(s, l->absmax_out);
            p.absmax_publish_always = m3c_shard_collective(s->shard) ? 1 : 0;
        }
        return m3c_launch_ew_chosen(&s->ew_choices[index], &p, stream);
    }
    if (l->kind == M3C_LAUNCH_CATEGORICAL) {
        const m3_tensor_metadata *in = &s->metadata[l->row_in.value];
        m3c_categorical_params p;

        memset(&p, 0, sizeof(p));
        p.probabilities = ref_pointer(s, l->row_in);
        p.probabilities_dtype = (int32_t)in->dtype;
        p.uniforms = ref_pointer(s, l->row_in_b);
        p.uniforms_dtype = (int32_t)s->metadata[l->row_in_b.value].dtype;
        p.output = (int32_t *)ref_pointer(s, l->row_out);
        p.width = in->shape[in->rank - 1U];
        p.rows = p.width ? in->element_count / p.width : 0U;
        p.status = s->status_device;
        p.command = l->command_a;
        p.skip_before = (uint32_t)l->first_node;
        p.first_of_run = first ? 1 : 0;
        return m3c_launch_categorical(&p, stream);
    }
    if (l->kind == M3C_LAUNCH_SOFTMAX) {
        const m3_tensor_metadata *in = &s->metadata[l->row_in.value];
        m3c_softmax_params p;

        memset(&p, 0, sizeof(p));
        p.input = ref_pointer(s, l->row_in);
        p.in_dtype = (int32_t)in->dtype;
        p.first_of_run = first ? 1 : 0;
        p.width = in->shape[in->rank - 1U];
        p.rows = p.width ? in->element_count / p.width : 0U;
        p.status = s->status_device;
        p.skip_before = (uint32_t)l->first_node;
        p.softmax_command = l->command_a;
        p.topk_command = l->command_b;
        if (l->row_out.value != UINT32_MAX) {
            p.probs = ref_pointer(s, l->row_out);
            p.probs_dtype = (int32_t)s->metadata[l->row_out.value].dtype;
        }
        if (l->row_out2.value != UINT32_MAX) {
            p.top_values = (float *)ref_pointer(s, l->row_out2);
            p.top_indices = (int32_t *)ref_pointer(s, l->row_out3);
            p.k = l->k;
        }
        p.rowsum_command = l->command_c;
        if (l->row_out4.value != UINT32_MAX) {
            p.row_sums = (float *)ref_pointer(s, l->row_out4);
            if (p.width == 0U) {
                /* rows of no element sum to +0 */
                cudaError_t code = cudaMemsetAsync(
                    p.row_sums, 0, s->metadata[l->row_out4.value].byte_count,
                    stream);

                if (code != cudaSuccess) {
                    return (int)code;
                }
            }
        }
        return m3c_launch_softmax(&p, stream);
    }
    {
        const m3_tensor_metadata *in = &s->metadata[l->row_in.value];
        m3c_norm_params p;

        memset(&p, 0, sizeof(p));
        p.x = ref_pointer(s, l->row_in);
        p.resid_b = ref_pointer(s, l->row_in_b);
        p.sum_out = ref_pointer(s, l->row_sum_out);
        p.in_dtype = (int32_t)in->dtype;
        p.first_of_run = first ? 1 : 0;
        p.scale = ref_pointer(s, l->norm_scale);
        p.scale_dtype = (int32_t)s->metadata[l->norm_scale.value].dtype;
        p.bias = ref_pointer(s, l->norm_bias);
        p.bias_dtype = l->norm_bias.value == UINT32_MAX
                           ? 0
                           : (int32_t)s->metadata[l->norm_bias.value].dtype;
        p.layer_norm = l->layer_norm ? 1 : 0;
        p.out = ref_pointer(s, l->row_out);
        p.out_dtype = (int32_t)s->metadata[l->row_out.value].dtype;
        p.width = in->shape[in->rank - 1U];
        p.rows = p.width ? in->element_count / p.width : 0U;
        p.epsilon = l->epsilon;
        p.status = s->status_device;
        p.skip_before = (uint32_t)l->first_node;
        return m3c_launch_norm(&p, stream);
    }
}

static void apply_swap(m3_session *s, size_t a, size_t b)
{
    unsigned char *held = s->buffer[s->current[a]][a];

    s->buffer[s->current[a]][a] = s->buffer[s->current[b]][b];
    s->buffer[s->current[b]][b] = held;
}

/* Host bookkeeping of one enqueued run: its event and the shadow flips a
 * clean run commits (a failure found at synchronise is replayed). */
static m3_status account_run(m3_session *s, m3_error *error)
{
    size_t i;
    m3_status status = push_event(s, EVENT_RUN, 0U, 0U, error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    for (i = 0U; i < s->plan.flip_count; ++i) {
        s->current[s->plan.flip_slot[i]] ^= 1U;
    }
    ++s->pending_runs;
    return M3_STATUS_OK;
}

static m3_status account_swap(m3_session *s, size_t a, size_t b,
                              m3_error *error)
{
    m3_status status = push_event(s, EVENT_SWAP, a, b, error);

    if (status == M3_STATUS_OK) {
        apply_swap(s, a, b);
    }
    return status;
}

/* The launches of one run with the buffer assignment as it stands.  A wave
 * of independent launches forks onto the side streams and joins back (under
 * stream capture this records parallel branches of the run's graph). */
static int launch_run(m3_session *s)
{
    size_t i = 0U;

    while (i < s->plan.launch_count) {
        size_t end = i + 1U;
        size_t k;
        cudaError_t code;

        while (s->wave_join != NULL && end < s->plan.launch_count &&
               s->wave_join[end]) {
            ++end;
        }
        if (end == i + 1U) {
            int result = launch_one(s, i, i == 0U, s->stream);

            if (result != 0) {
                return result;
            }
            i = end;
            continue;
        }
        code = cudaEventRecord(s->fork_event, s->stream);
        for (k = i + 1U; code == cudaSuccess && k < end; ++k) {
            code = cudaStreamWaitEvent(s->side[k - i - 1U], s->fork_event, 0);
        }
        if (code != cudaSuccess) {
            return (int)code;
        }
        for (k = i; k < end; ++k) {
            int result = launch_one(s, k, k == 0U,
                                    k == i ? s->stream : s->side[k - i - 1U]);

            if (result != 0) {
                return result;
            }
        }
        for (k = i + 1U; code == cudaSuccess && k < end; ++k) {
            code = cudaEventRecord(s->join_event[k - i - 1U], s->side[k - i - 1U]);
            if (code == cudaSuccess) {
                code = cudaStreamWaitEvent(s->stream, s->join_event[k - i - 1U], 0);
            }
        }
        if (code != cudaSuccess) {
            return (int)code;
        }
        i = end;
    }
    return 0;
}

static bool graph_matches(const m3_session *s, const run_graph *g,
                          size_t runs, size_t a, size_t b)
{
    size_t slots = s->plan.slot_count;

    return g->exec != NULL && g->runs == runs && g->swap_a == a &&
           g->swap_b == b &&
           memcmp(g->start_current, s->current, slots) == 0 &&
           memcmp(g->start_buffer[0], s->buffer[0],
                  slots * sizeof(unsigned char *)) == 0 &&
           memcmp(g->start_buffer[1], s->buffer[1],
                  slots * sizeof(unsigned char *)) == 0;
}

/* Record the launches of `runs` runs (slots a/b exchanged between them) into
 * a CUDA graph by stream capture, leaving the host state as it was.  NULL
 * when capture is not possible on this stream; the caller then launches
 * directly. */
static cudaGraphExec_t capture_runs(m3_session *s, size_t runs, size_t a,
                                    size_t b)
{
    size_t slots = s->plan.slot_count ? s->plan.slot_count : 1U;
    run_graph entry;
    cudaGraph_t graph = NULL;
    cudaGraphExec_t exec = NULL;
    cudaError_t code;
    int launched = 0;
    size_t r;
    size_t i;

    memset(&entry, 0, sizeof(entry));
    entry.start_buffer[0] = malloc(slots * sizeof(unsigned char *));
    entry.start_buffer[1] = malloc(slots * sizeof(unsigned char *));
    entry.start_current = malloc(slots);
    if (entry.start_buffer[0] == NULL || entry.start_buffer[1] == NULL ||
        entry.start_current == NULL) {
        drop_graph(&entry);
        return NULL;
    }
    memcpy(entry.start_buffer[0], s->buffer[0], slots * sizeof(unsigned char *));
    memcpy(entry.start_buffer[1], s->buffer[1], slots * sizeof(unsigned char *));
    memcpy(entry.start_current, s->current, slots);
    code = cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeRelaxed);
    if (code != cudaSuccess) {
        (void)cudaGetLastError();
        drop_graph(&entry);
        return NULL;
    }
    for (r = 0U; r < runs && launched == 0; ++r) {
        if (r > 0U && s->plan.flip_count != 0U) {
            launched = m3c_launch_run_gate(s->status_device, s->stream);
        }
        if (launched == 0) {
            launched = launch_run(s);
        }
        for (i = 0U; i < s->plan.flip_count; ++i) {
            s->current[s->plan.flip_slot[i]] ^= 1U;
        }
        if (r + 1U < runs && a != SIZE_MAX) {
            apply_swap(s, a, b);
        }
    }
    code = cudaStreamEndCapture(s->stream, &graph);
    /* back to the state the runs start from */
    memcpy(s->buffer[0], entry.start_buffer[0], slots * sizeof(unsigned char *));
    memcpy(s->buffer[1], entry.start_buffer[1], slots * sizeof(unsigned char *));
    memcpy(s->current, entry.start_current, slots);
    if (code == cudaSuccess && launched == 0) {
        code = cudaGraphInstantiate(&exec, graph, 0ULL);
    }
    if (graph != NULL) {
        (void)cudaGraphDestroy(graph);
    }
    (void)cudaGetLastError();
    if (code != cudaSuccess || launched != 0 || exec == NULL) {
        drop_graph(&entry);
        return NULL;
    }
    entry.runs = runs;
    entry.swap_a = a;
    entry.swap_b = b;
    entry.exec = exec;
    if (s->graph_count < M3C_RUN_GRAPHS) {
        s->graphs[s->graph_count++] = entry;
    } else {
        drop_graph(&s->graphs[s->graph_next]);
        s->graphs[s->graph_next] = entry;
        s->graph_next = (s->graph_next + 1U) % M3C_RUN_GRAPHS;
    }
    return exec;
}

/* The ranks of a sharded session agree after each run: the global
 * reductions' bit patterns and the first failing command, packed into one
 * staging area, all-reduced (MAX) on the session's stream, unpacked. */
static m3_status shard_collect(m3_session *s, m3_error *error)
{
    m3c_shard *sh = s->shard;
    m3c_shard_words w;
    int code;
    int i;
    m3_status status;

    memset(&w, 0, sizeof(w));
    w.count = sh->reduction_count;
    for (i = 0; i < sh->reduction_count; ++i) {
        w.values[i] = (uint32_t *)value_pointer(s, sh->reductions[i], false);
        w.commands[i] = sh->reduction_commands[i];
    }
    w.status = s->status_device;
    w.staging = sh->staging;
    code = m3c_launch_shard_pack(&w, s->stream);
    if (code != 0) {
        return m3c_error_set(error, M3_STATUS_INTERNAL, "shard pack failed: %s",
                             m3c_cuda_error_string(code));
    }
    status = m3c_comm_max_u32(sh->comm, sh->staging,
                              (size_t)sh->reduction_count + 1U, s->stream,
                              sh->timeout_seconds, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    code = m3c_launch_shard_unpack(&w, s->stream);
    if (code != 0) {
        return m3c_error_set(error, M3_STATUS_INTERNAL,
                             "shard unpack failed: %s",
                             m3c_cuda_error_string(code));
    }
    return M3_STATUS_OK;
}

/* Enqueue `runs` runs, exchanging slots a and b between consecutive runs
 * (SIZE_MAX: no exchange).  With cuda_graphs the whole sequence is one graph
 * launch, captured on first use for each starting buffer assignment and kept
 * (up to M3C_RUN_GRAPHS sequences); without it, or on a stream that cannot
 * be captured (the legacy default stream, or one the caller is capturing
 * already), the kernels are launched one by one. */
static m3_status enqueue_runs(m3_session *s, size_t runs, size_t a, size_t b,
                              m3_error *error)
{
    bool graphed = false;
    m3_status status;
    size_t r;

    if (runs == 0U) {
        m3_error_reset(error);
        return M3_STATUS_OK;
    }
    if (s->plan.launch_count == 0U) {
        /* nothing runs; only the exchanges take effect */
        for (r = 0U; r + 1U < runs && a != SIZE_MAX; ++r) {
            status = account_swap(s, a, b, error);
            if (status != M3_STATUS_OK) {
                return status;
            }
        }
        m3_error_reset(error);
        return M3_STATUS_OK;
    }
    status = use_device(s, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    if (s->plan.flip_count != 0U && s->pending_runs != 0U) {
        /* an earlier run of this batch may have failed: halt this one then */
        int code = m3c_launch_run_gate(s->status_device, s->stream);

        if (code != 0) {
            return m3c_error_set(error, M3_STATUS_INTERNAL,
                                 "kernel launch failed: %s",
                                 m3c_cuda_error_string(code));
        }
    }
    if (s->cuda.cuda_graphs && !m3c_shard_collective(s->shard)) {
        enum cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;

        if (cudaStreamIsCapturing(s->stream, &capturing) == cudaSuccess &&
            capturing == cudaStreamCaptureStatusNone) {
            cudaGraphExec_t exec = NULL;
            size_t g;

            for (g = 0U; g < s->graph_count && exec == NULL; ++g) {
                if (graph_matches(s, &s->graphs[g], runs, a, b)) {
                    exec = s->graphs[g].exec;
                }
            }
            if (exec == NULL) {
                exec = capture_runs(s, runs, a, b);
            }
            if (exec != NULL) {
                cudaError_t code = cudaGraphLaunch(exec, s->stream);

                if (code != cudaSuccess) {
                    return cuda_failure(error, code, "graph launch failed");
                }
                graphed = true;
            }
        }
        (void)cudaGetLastError();
    }
    for (r = 0U; r < runs; ++r) {
        if (!graphed) {
            int code = r > 0U && s->plan.flip_count != 0U
                           ? m3c_launch_run_gate(s->status_device, s->stream)
                           : 0;

            if (code == 0) {
                code = launch_run(s);
            }

            if (code != 0) {
                return m3c_error_set(error, M3_STATUS_INTERNAL,
                                     "kernel launch failed: %s",
                                     m3c_cuda_error_string(code));
            }
        }
        /* assume success; a failure found at synchronise is replayed */
        status = account_run(s, error);
        if (status == M3_STATUS_OK && m3c_shard_collective(s->shard)) {
            status = shard_collect(s, error);
        }
        if (status == M3_STATUS_OK && r + 1U < runs && a != SIZE_MAX) {
            status = account_swap(s, a, b, error);
        }
        if (status != M3_STATUS_OK) {
            return status;
        }
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_session_run_async(m3_session *s, m3_error *error)
{
    if (s == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session is null");
    }
    return enqueue_runs(s, 1U, SIZE_MAX, SIZE_MAX, error);
}


/* The reference's data-check messages (src/m3_op_data_preflight.c:23,
 * :283-291). */
static const char *failure_message(const m3_session *s, uint32_t command,
                                   uint32_t detail)
{
    if (command >= s->plan.node_count) {
        return "data check failed";
    }
    switch ((int)s->node_kinds[command]) {
    case M3_OP_CATEGORICAL:
        return m3c_categorical_message(detail);
    case M3_OP_SOFTMAX:
        return "softmax input contains NaN";
    case M3_OP_TOP_K:
        return "top-k logits contain NaN";
    case M3_OP_CAST:
        return "float-to-I32 cast value is invalid";
    case (int)M3_OP_ABS_MAX:
        return "abs-max input contains NaN";
    default:
        return "data check failed";
    }
}

/* Wait for everything enqueued; returns the first data-check failure. */
static m3_status settle(m3_session *s, m3_error *error)
{
    cudaError_t code;
    m3c_status seen;
    size_t count = s->plan.value_count ? s->plan.value_count : 1U;
    m3_status status = M3_STATUS_OK;

    code = cudaMemcpyAsync(s->status_host, s->status_device, sizeof(m3c_status),
                           cudaMemcpyDeviceToHost, s->stream);
    if (code == cudaSuccess) {
        code = cudaStreamSynchronize(s->stream);
    }
    if (code == cudaSuccess && s->pipe.ready) {
        /* host submissions: their downloads finish after the runs */
        code = cudaStreamSynchronize(s->pipe.upload);
        if (code == cudaSuccess) {
            code = cudaStreamSynchronize(s->pipe.download);
        }
    }
    if (code != cudaSuccess) {
        return cuda_failure(error, code, "device execution failed");
    }
    seen = *s->status_host;
    if (seen.fail_command != UINT32_MAX) {
        size_t started = seen.runs_started & ~(uint32_t)M3C_RUN_HALTED;
        size_t failing_run = started ? started - 1U : 0U;
        size_t run = 0U;
        size_t e;
        size_t f;

        /* replay from the last synchronised state */
        memcpy(s->buffer[0], s->sync_buffer[0], count * sizeof(unsigned char *));
        memcpy(s->buffer[1], s->sync_buffer[1], count * sizeof(unsigned char *));
        memcpy(s->current, s->sync_current, count);
        for (e = 0U; e < s->event_count; ++e) {
            if (s->events[e].kind == EVENT_SWAP) {
                apply_swap(s, s->events[e].slot_a, s->events[e].slot_b);
                continue;
            }
            for (f = 0U; f < s->plan.flip_count; ++f) {
                if (run < failing_run ||
                    (run == failing_run &&
                     s->plan.flip_command[f] < seen.fail_command)) {
                    s->current[s->plan.flip_slot[f]] ^= 1U;
                }
            }
            ++run;
        }
        status = m3c_error_set(error, M3_STATUS_OUT_OF_RANGE, "%s",
                               failure_message(s, seen.fail_command,
                                               seen.detail));
        code = cudaMemcpyAsync(s->status_device, &clean_status,
                               sizeof(clean_status), cudaMemcpyHostToDevice,
                               s->stream);
        if (code == cudaSuccess) {
            code = cudaStreamSynchronize(s->stream);
        }
        if (code != cudaSuccess) {
            return cuda_failure(error, code, "cannot reset session status");
        }
    } else if (seen.runs_started != 0U) {
        static const uint32_t zero = 0U;

        code = cudaMemcpyAsync(&s->status_device->runs_started, &zero,
                               sizeof(zero), cudaMemcpyHostToDevice, s->stream);
        if (code == cudaSuccess) {
            code = cudaStreamSynchronize(s->stream);
        }
        if (code != cudaSuccess) {
            return cuda_failure(error, code, "cannot reset session status");
        }
    }
    memcpy(s->sync_buffer[0], s->buffer[0], count * sizeof(unsigned char *));
    memcpy(s->sync_buffer[1], s->buffer[1], count * sizeof(unsigned char *));
    memcpy(s->sync_current, s->current, count);
    s->event_count = 0U;
    s->pending_runs = 0U;
    return status;
}

m3_status m3_cuda_session_synchronize(m3_session *s, m3_error *error)
{
    m3_status status;

    if (s == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session is null");
    }
    status = use_device(s, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    status = settle(s, error);
    if (status == M3_STATUS_OK && s->sticky_status != M3_STATUS_OK) {
        status = s->sticky_status;
        if (error != NULL) {
            *error = s->sticky_error;
        }
    }
    s->sticky_status = M3_STATUS_OK;
    if (status == M3_STATUS_OK) {
        m3_error_reset(error);
    }
    return status;
}

m3_status m3_session_run(m3_session *s, m3_error *error)
{
    m3_status status = m3_cuda_session_run_async(s, error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    return m3_cuda_session_synchronize(s, error);
}

/* Pending runs must finish before the host touches slot memory; a failure
 * found here is kept for the next explicit synchronise. */
static m3_status settle_quietly(m3_session *s, m3_error *error)
{
    m3_error local;
    m3_status status;

    if (s->pending_runs == 0U && s->event_count == 0U) {
        return M3_STATUS_OK;
    }
    status = settle(s, &local);
    if (status == M3_STATUS_OUT_OF_RANGE) {
        if (s->sticky_status == M3_STATUS_OK) {
            s->sticky_status = status;
            s->sticky_error = local;
        }
        return M3_STATUS_OK;
    }
    if (status != M3_STATUS_OK && error != NULL) {
        *error = local;
    }
    return status;
}

/* ----------------------------------------------------------------- I/O */

static m3_status value_check(const m3_session *s, m3_graph_value_id value,
                             m3_graph_value_role expected,
                             const char *operation, m3_error *error)
{
    if (s == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "%s session is null", operation);
    }
    if ((size_t)value >= s->plan.value_count) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "%s value is out of range", operation);
    }
    if (s->descriptions[value].role != expected) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "%s value has the wrong role", operation);
    }
    return M3_STATUS_OK;
}

static m3_status copy_value(m3_session *s, m3_graph_value_id value,
                            const void *source, void *destination,
                            size_t byte_count, enum cudaMemcpyKind kind,
                            m3_error *error)
{
    cudaError_t code;
    m3_status status = use_device(s, error);

    if (status == M3_STATUS_OK) {
        status = settle_quietly(s, error);
    }
    if (status != M3_STATUS_OK || byte_count == 0U) {
        if (status == M3_STATUS_OK) {
            m3_error_reset(error);
        }
        return status;
    }
    if (source == NULL) {
        source = value_pointer(s, value, false);
    } else {
        destination = value_pointer(s, value, false);
    }
    code = cudaMemcpyAsync(destination, source, byte_count, kind, s->stream);
    if (code == cudaSuccess) {
        code = cudaStreamSynchronize(s->stream);
    }
    if (code != cudaSuccess) {
        return cuda_failure(error, code, "session copy failed");
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_session_write_input(m3_session *s, m3_graph_value_id value,
                                  const void *data, size_t byte_count,
                                  m3_error *error)
{
    m3_status status = value_check(s, value, M3_GRAPH_INPUT, "input write",
                                   error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (byte_count != s->metadata[value].byte_count ||
        (byte_count != 0U && data == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "input write size does not match tensor");
    }
    return copy_value(s, value, data, NULL, byte_count, cudaMemcpyHostToDevice,
                      error);
}

m3_status m3_session_read_output(const m3_session *session,
                                  m3_graph_value_id value, void *data,
                                  size_t byte_count, m3_error *error)
{
    m3_session *s = (m3_session *)session;
    m3_status status = value_check(s, value, M3_GRAPH_OUTPUT, "output read",
                                   error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (byte_count != s->metadata[value].byte_count ||
        (byte_count != 0U && data == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "output read size does not match tensor");
    }
    return copy_value(s, value, NULL, data, byte_count, cudaMemcpyDeviceToHost,
                      error);
}

m3_status m3_cuda_session_write_input_device(m3_session *s,
                                             m3_graph_value_id value,
                                             const void *device_source,
                                             size_t byte_count,
                                             m3_error *error)
{
    m3_status status = value_check(s, value, M3_GRAPH_INPUT, "input write",
                                   error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (byte_count != s->metadata[value].byte_count ||
        (byte_count != 0U && device_source == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "input write size does not match tensor");
    }
    return copy_value(s, value, device_source, NULL, byte_count,
                      cudaMemcpyDeviceToDevice, error);
}

m3_status m3_cuda_session_read_output_device(const m3_session *session,
                                             m3_graph_value_id value,
                                             void *device_destination,
                                             size_t byte_count,
                                             m3_error *error)
{
    m3_session *s = (m3_session *)session;
    m3_status status = value_check(s, value, M3_GRAPH_OUTPUT, "output read",
                                   error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (byte_count != s->metadata[value].byte_count ||
        (byte_count != 0U && device_destination == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "output read size does not match tensor");
    }
    return copy_value(s, value, NULL, device_destination, byte_count,
                      cudaMemcpyDeviceToDevice, error);
}

m3_status m3_cuda_session_read_output_device_async(
    m3_session *s, m3_graph_value_id value, void *device_destination,
    size_t byte_count, m3_error *error)
{
    cudaError_t code;
    m3_status status = value_check(s, value, M3_GRAPH_OUTPUT, "output read",
                                   error);

    if (status != M3_STATUS_OK) {
        return status;
    }
    if (byte_count != s->metadata[value].byte_count ||
        (byte_count != 0U && device_destination == NULL)) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "output read size does not match tensor");
    }
    status = use_device(s, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    if (byte_count != 0U) {
        /* the buffer the value occupies once the pending runs succeed */
        code = cudaMemcpyAsync(device_destination, value_pointer(s, value, false),
                               byte_count, cudaMemcpyDeviceToDevice, s->stream);
        if (code != cudaSuccess) {
            return cuda_failure(error, code, "session copy failed");
        }
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_session_value_device_pointer(const m3_session *session,
                                               m3_graph_value_id value,
                                               void **device_pointer,
                                               size_t *byte_count,
                                               m3_error *error)
{
    m3_session *s = (m3_session *)session;
    m3_status status;

    if (s == NULL || device_pointer == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session and pointer output are required");
    }
    if ((size_t)value >= s->plan.value_count) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "value is out of range");
    }
    if (!s->plan.slot_needed[s->plan.value_slot[value]]) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "value has no device storage: it lives only in "
                             "the registers of a fused launch");
    }
    status = settle_quietly(s, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    *device_pointer = value_pointer(s, value, false);
    if (byte_count != NULL) {
        *byte_count = s->metadata[value].byte_count;
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_session_swap_values(m3_session *s, m3_graph_value_id input,
                                      m3_graph_value_id output,
                                      m3_error *error)
{
    m3_status status = value_check(s, input, M3_GRAPH_INPUT, "swap input",
                                   error);
    size_t a;
    size_t b;

    if (status == M3_STATUS_OK) {
        status = value_check(s, output, M3_GRAPH_OUTPUT, "swap output", error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    if (s->metadata[input].byte_count != s->metadata[output].byte_count) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "swapped values differ in size");
    }
    a = s->plan.value_slot[input];
    b = s->plan.value_slot[output];
    status = push_event(s, EVENT_SWAP, a, b, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    apply_swap(s, a, b);
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_session_run_steps_async(m3_session *s, size_t count,
                                          m3_graph_value_id input,
                                          m3_graph_value_id output,
                                          m3_error *error)
{
    size_t a = SIZE_MAX;
    size_t b = SIZE_MAX;

    if (s == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session is null");
    }
    if (input != M3_GRAPH_VALUE_NONE || output != M3_GRAPH_VALUE_NONE) {
        m3_status status = value_check(s, input, M3_GRAPH_INPUT,
                                       "carried input", error);

        if (status == M3_STATUS_OK) {
            status = value_check(s, output, M3_GRAPH_OUTPUT, "carried output",
                                 error);
        }
        if (status != M3_STATUS_OK) {
            return status;
        }
        if (s->metadata[input].byte_count != s->metadata[output].byte_count) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "carried values differ in size");
        }
        a = s->plan.value_slot[input];
        b = s->plan.value_slot[output];
    }
    return enqueue_runs(s, count, a, b, error);
}

/* Copy streams, events and staging areas of at least the given sizes. */
static m3_status pipe_ready(m3_session *s, size_t in_bytes, size_t out_bytes,
                            m3_error *error)
{
    host_pipe *p = &s->pipe;
    cudaError_t code = cudaSuccess;
    int k;

    if (p->ready && in_bytes <= p->in_bytes && out_bytes <= p->out_bytes) {
        return M3_STATUS_OK;
    }
    if (p->ready) {
        /* grow: earlier submissions may still use the old areas */
        code = cudaStreamSynchronize(s->stream);
        if (code == cudaSuccess) code = cudaStreamSynchronize(p->upload);
        if (code == cudaSuccess) code = cudaStreamSynchronize(p->download);
        for (k = 0; k < 2; ++k) {
            (void)cudaFree(p->stage_in[k]);
            (void)cudaFree(p->stage_out[k]);
            p->stage_in[k] = NULL;
            p->stage_out[k] = NULL;
        }
    } else {
        code = cudaStreamCreateWithFlags(&p->upload, cudaStreamNonBlocking);
        if (code == cudaSuccess) {
            code = cudaStreamCreateWithFlags(&p->download, cudaStreamNonBlocking);
        }
        for (k = 0; k < 2 && code == cudaSuccess; ++k) {
            code = cudaEventCreateWithFlags(&p->uploaded[k], cudaEventDisableTiming);
            if (code == cudaSuccess) code = cudaEventCreateWithFlags(&p->consumed[k], cudaEventDisableTiming);
            if (code == cudaSuccess) code = cudaEventCreateWithFlags(&p->produced[k], cudaEventDisableTiming);
            if (code == cudaSuccess) code = cudaEventCreateWithFlags(&p->drained[k], cudaEventDisableTiming);
        }
    }
    for (k = 0; k < 2 && code == cudaSuccess; ++k) {
        code = cudaMalloc((void **)&p->stage_in[k], in_bytes ? in_bytes : 1U);
        if (code == cudaSuccess) {
            code = cudaMalloc((void **)&p->stage_out[k], out_bytes ? out_bytes : 1U);
        }
    }
    if (code != cudaSuccess) {
        drop_pipe(p);
        return cuda_failure(error, code, "cannot set up host submissions");
    }
    p->in_bytes = in_bytes;
    p->out_bytes = out_bytes;
    p->ready = true;
    return M3_STATUS_OK;
}

m3_status m3_cuda_session_submit_host_async(
    m3_session *s, size_t input_count, const m3_graph_value_id *inputs,
    const void *const *input_data, size_t output_count,
    const m3_graph_value_id *outputs, void *const *output_data,
    m3_error *error)
{
    host_pipe *p;
    size_t in_bytes = 0U;
    size_t out_bytes = 0U;
    size_t offset;
    size_t k;
    unsigned t;
    cudaError_t code = cudaSuccess;
    m3_status status;

    if (s == NULL || (input_count != 0U && (inputs == NULL || input_data == NULL)) ||
        (output_count != 0U && (outputs == NULL || output_data == NULL))) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session, values and host buffers are required");
    }
    for (k = 0U; k < input_count; ++k) {
        status = value_check(s, inputs[k], M3_GRAPH_INPUT, "submitted input", error);
        if (status != M3_STATUS_OK) {
            return status;
        }
        if (input_data[k] == NULL && s->metadata[inputs[k]].byte_count != 0U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "submitted input %zu has no host buffer", k);
        }
        in_bytes += (s->metadata[inputs[k]].byte_count + 255U) & ~(size_t)255U;
    }
    for (k = 0U; k < output_count; ++k) {
        status = value_check(s, outputs[k], M3_GRAPH_OUTPUT, "submitted output", error);
        if (status != M3_STATUS_OK) {
            return status;
        }
        if (output_data[k] == NULL && s->metadata[outputs[k]].byte_count != 0U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "submitted output %zu has no host buffer", k);
        }
        out_bytes += (s->metadata[outputs[k]].byte_count + 255U) & ~(size_t)255U;
    }
    status = use_device(s, error);
    if (status == M3_STATUS_OK) {
        status = pipe_ready(s, in_bytes, out_bytes, error);
    }
    if (status != M3_STATUS_OK) {
        return status;
    }
    p = &s->pipe;
    t = p->turn;
    /* upload into this turn's staging area once its last reader is done */
    code = cudaStreamWaitEvent(p->upload, p->consumed[t], 0);
    for (k = 0U, offset = 0U; k < input_count && code == cudaSuccess; ++k) {
        size_t bytes = s->metadata[inputs[k]].byte_count;

        if (bytes != 0U) {
            code = cudaMemcpyAsync(p->stage_in[t] + offset, input_data[k], bytes,
                                   cudaMemcpyHostToDevice, p->upload);
        }
        offset += (bytes + 255U) & ~(size_t)255U;
    }
    if (code == cudaSuccess) code = cudaEventRecord(p->uploaded[t], p->upload);
    /* on the session stream: staging -> inputs, the run, outputs -> staging */
    if (code == cudaSuccess) code = cudaStreamWaitEvent(s->stream, p->uploaded[t], 0);
    for (k = 0U, offset = 0U; k < input_count && code == cudaSuccess; ++k) {
        size_t bytes = s->metadata[inputs[k]].byte_count;

        if (bytes != 0U) {
            code = cudaMemcpyAsync(value_pointer(s, inputs[k], false), p->stage_in[t] + offset,
                                   bytes, cudaMemcpyDeviceToDevice, s->stream);
        }
        offset += (bytes + 255U) & ~(size_t)255U;
    }
    if (code == cudaSuccess) code = cudaEventRecord(p->consumed[t], s->stream);
    if (code != cudaSuccess) {
        return cuda_failure(error, code, "host submission upload failed");
    }
    status = enqueue_runs(s, 1U, SIZE_MAX, SIZE_MAX, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    code = cudaStreamWaitEvent(s->stream, p->drained[t], 0);
    for (k = 0U, offset = 0U; k < output_count && code == cudaSuccess; ++k) {
        size_t bytes = s->metadata[outputs[k]].byte_count;

        if (bytes != 0U) {
            /* the buffer the output occupies once this run succeeds */
            code = cudaMemcpyAsync(p->stage_out[t] + offset, value_pointer(s, outputs[k], false),
                                   bytes, cudaMemcpyDeviceToDevice, s->stream);
        }
        offset += (bytes + 255U) & ~(size_t)255U;
    }
    if (code == cudaSuccess) code = cudaEventRecord(p->produced[t], s->stream);
    /* download once produced */
    if (code == cudaSuccess) code = cudaStreamWaitEvent(p->download, p->produced[t], 0);
    for (k = 0U, offset = 0U; k < output_count && code == cudaSuccess; ++k) {
        size_t bytes = s->metadata[outputs[k]].byte_count;

        if (bytes != 0U) {
            code = cudaMemcpyAsync(output_data[k], p->stage_out[t] + offset, bytes,
                                   cudaMemcpyDeviceToHost, p->download);
        }
        offset += (bytes + 255U) & ~(size_t)255U;
    }
    if (code == cudaSuccess) code = cudaEventRecord(p->drained[t], p->download);
    if (code != cudaSuccess) {
        return cuda_failure(error, code, "host submission download failed");
    }
    p->turn = t ^ 1U;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

void *m3_cuda_session_stream(const m3_session *s)
{
    return s == NULL ? NULL : (void *)s->stream;
}

int m3_cuda_session_device(const m3_session *s)
{
    return s == NULL ? -1 : s->device;
}

/* ------------------------------------------------------------ plan info */

m3_status m3_session_get_plan_info(const m3_session *s,
                                    m3_session_plan_info *info,
                                    m3_error *error)
{
    if (s == NULL || info == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session and plan info output are required");
    }
    info->value_count = s->plan.value_count;
    info->node_count = s->plan.node_count;
    info->storage_slot_count = s->plan.slot_count;
    info->allocated_bytes = s->plan.allocated_bytes;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_session_get_node_provider(const m3_session *s, size_t node_index,
                                        m3_provider_kind *provider,
                                        m3_error *error)
{
    if (s == NULL || provider == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session and provider output are required");
    }
    if (node_index >= s->plan.node_count) {
        return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE,
                             "session node index is out of range");
    }
    *provider = M3_PROVIDER_CUDA;
    m3_error_reset(error);
    return M3_STATUS_OK;
}

static void fill_report(const m3c_plan *plan, m3_cuda_plan_report *report,
                        char *text, size_t capacity)
{
    if (report != NULL) {
        report->launch_count = plan->launch_count;
        report->fused_node_count = plan->fused_node_count;
        report->shadow_bytes = plan->shadow_bytes;
        report->arena_bytes = plan->arena_bytes;
    }
    m3c_plan_describe(plan, text, capacity);
}

m3_status m3_cuda_session_get_plan_report(const m3_session *s,
                                          m3_cuda_plan_report *report,
                                          char *text, size_t text_capacity,
                                          m3_error *error)
{
    if (s == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "session is required");
    }
    fill_report(&s->plan, report, text, text_capacity);
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_graph_plan(const m3_graph *graph,
                             const m3_cuda_session_options *cuda,
                             m3_session_plan_info *info,
                             m3_cuda_plan_report *report, char *text,
                             size_t text_capacity, m3_error *error)
{
    m3_cuda_session_options options;
    m3c_plan plan;
    m3_status status;

    m3_cuda_session_options_init(&options);
    if (cuda != NULL) {
        options = *cuda;
    }
    status = m3c_plan_build(graph, options.fuse, &plan, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    if (info != NULL) {
        info->value_count = plan.value_count;
        info->node_count = plan.node_count;
        info->storage_slot_count = plan.slot_count;
        info->allocated_bytes = plan.allocated_bytes;
    }
    fill_report(&plan, report, text, text_capacity);
    m3c_plan_free(&plan);
    m3_error_reset(error);
    return M3_STATUS_OK;
}

/* ------------------------------------------------- sharding internals */

void m3c_session_attach_shard(m3_session *session, m3c_shard *shard)
{
    session->shard = shard;
}

const m3c_shard *m3c_session_shard(const m3_session *session)
{
    return session->shard;
}

const m3_tensor_metadata *m3c_session_metadata(const m3_session *session,
                                               m3_graph_value_id value)
{
    return &session->metadata[value];
}

m3_graph_value_role m3c_session_role(const m3_session *session,
                                     m3_graph_value_id value)
{
    return session->descriptions[value].role;
}

size_t m3c_session_value_count(const m3_session *session)
{
    return session->plan.value_count;
}
