/* m3_cuda.h -- the C ABI of libm3cuda.so, a B200 (sm_100a) CUDA provider for
 * m3.c's tensor hot path: element-wise, broadcast, cast, activation and
 * row-reduction operators.
 *
 * Three layers are exported, all plain C, plain pointers and sizes:
 *
 *  1. The graph/session API of the reference's include/m3.h:197-259, same
 *     names, same argument meaning, same status codes and same failure
 *     atomicity.  A program written against m3.h that builds graphs from the
 *     operators below links against this library unchanged; its regular nodes
 *     run on the GPU, planned into liveness slots of one device arena and
 *     fused into few kernels.
 *
 *  2. The reference's backend plug-in interface (m3_backend_vtable,
 *     reference src/m3_backend_internal.h:9-17) as free functions with the
 *     exact vtable signatures, so the reference's own provider scheduler
 *     (src/m3_provider.c) can register this library as one more provider.
 *
 *  3. CUDA-only extensions: device and stream selection, asynchronous runs,
 *     device pointers of session values, a host-only planner for tests, and
 *     the seeded input generators of the reference's m3_rng.
 *
 * ABI compatibility.  The reference types that cross this boundary are
 * restated below with identical layout.  Each block is guarded by the
 * reference header's own include guard, so a translation unit that already
 * included the reference headers uses their definitions; include this header
 * after the reference headers when both are used.
 *
 * Operators executed on the GPU: COPY, CAST, ADD, MUL, GATED_SILU, SOFTMAX,
 * TOP_K, CATEGORICAL, RMS_NORM, LAYER_NORM, SNAKE1D, TANH, and the extensions
 * M3_OP_ABS_MAX and M3_OP_CLAMP_UNIT.  Other m3.h kinds (contractions,
 * attention, convolutions, embedding, RoPE) are rejected with
 * M3_STATUS_UNSUPPORTED at session creation; there is no CPU fallback inside
 * this library.
 *
 * Threading: as in the reference (include/m3.h:270-273) a session is neither
 * reentrant nor thread-safe; distinct sessions are independent. */

#ifndef M3_CUDA_H
#define M3_CUDA_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * Reference ABI (include/m3.h)
 * ------------------------------------------------------------------------ */
#ifndef M3_H
#define M3_TENSOR_MAX_RANK 8U
#define M3_GRAPH_NODE_INPUT_CAPACITY 5U
#define M3_GRAPH_NODE_OUTPUT_CAPACITY 2U
#define M3_GRAPH_VALUE_NONE UINT32_MAX

/* include/m3.h:20-31 */
typedef enum {
    M3_STATUS_OK = 0,
    M3_STATUS_INVALID_ARGUMENT = 1,
    M3_STATUS_OUT_OF_RANGE = 2,
    M3_STATUS_OVERFLOW = 3,
    M3_STATUS_OUT_OF_MEMORY = 4,
    M3_STATUS_IO = 5,
    M3_STATUS_INVALID_FORMAT = 6,
    M3_STATUS_UNSUPPORTED = 7,
    M3_STATUS_CANCELLED = 8,
    M3_STATUS_INTERNAL = 9
} m3_status;

#define M3_ERROR_MESSAGE_CAPACITY 256U

/* include/m3.h:35-38 */
typedef struct {
    m3_status status;
    char message[M3_ERROR_MESSAGE_CAPACITY];
} m3_error;

/* include/m3.h:45-50 */
typedef enum {
    M3_DTYPE_F32 = 0,
    M3_DTYPE_F16,
    M3_DTYPE_BF16,
    M3_DTYPE_I32
} m3_dtype;

/* include/m3.h:52-73 */
typedef enum {
    M3_OP_COPY = 0,
    M3_OP_CAST,
    M3_OP_ADD,
    M3_OP_MUL,
    M3_OP_EMBEDDING,
    M3_OP_MATMUL,
    M3_OP_LINEAR,
    M3_OP_RMS_NORM,
    M3_OP_LAYER_NORM,
    M3_OP_ROPE,
    M3_OP_ATTENTION,
    M3_OP_GATED_SILU,
    M3_OP_SOFTMAX,
    M3_OP_TOP_K,
    M3_OP_CATEGORICAL,
    M3_OP_CONV1D,
    M3_OP_CONV_TRANSPOSE1D,
    M3_OP_NEAREST_RESIZE1D,
    M3_OP_SNAKE1D,
    M3_OP_TANH
} m3_op_kind;

/* include/m3.h:75-78 */
typedef enum {
    M3_ROPE_HALF_SPLIT = 0,
    M3_ROPE_INTERLEAVED
} m3_rope_mode;

/* include/m3.h:80-84 */
typedef enum {
    M3_PROVIDER_NEURAL_ENGINE = 0,
    M3_PROVIDER_METAL,
    M3_PROVIDER_CPU
} m3_provider_kind;

/* include/m3.h:86-91 */
typedef enum {
    M3_GRAPH_INPUT = 0,
    M3_GRAPH_CONSTANT,
    M3_GRAPH_TEMPORARY,
    M3_GRAPH_OUTPUT
} m3_graph_value_role;

typedef uint32_t m3_graph_value_id;

/* include/m3.h:95-100 */
typedef struct {
    m3_dtype dtype;
    uint8_t rank;
    uint64_t shape[M3_TENSOR_MAX_RANK];
    m3_graph_value_role role;
} m3_graph_value_desc;

/* include/m3.h:102-135 */
typedef struct {
    m3_op_kind kind;
    m3_graph_value_id inputs[M3_GRAPH_NODE_INPUT_CAPACITY];
    m3_graph_value_id outputs[M3_GRAPH_NODE_OUTPUT_CAPACITY];
    union {
        struct {
            float epsilon;
        } norm;
        struct {
            uint64_t position_offset;
            uint32_t rotary_dimension;
            m3_rope_mode mode;
        } rope;
        struct {
            float scale;
            int64_t causal_offset;
            bool causal;
        } attention;
        struct {
            uint64_t k;
        } top_k;
        struct {
            uint64_t groups;
            uint64_t stride;
            uint64_t dilation;
            uint64_t pad_left;
            uint64_t pad_right;
            uint64_t output_padding;
        } convolution;
        struct {
            uint64_t output_length;
        } resize;
    } parameters;
} m3_graph_node_desc;

/* include/m3.h:147-151 */
typedef struct {
    bool allow_neural_engine;
    bool allow_metal;
    bool allow_cpu;
} m3_session_options;

/* include/m3.h:153-158 */
typedef struct {
    size_t value_count;
    size_t node_count;
    size_t storage_slot_count;
    size_t allocated_bytes;
} m3_session_plan_info;

typedef struct m3_graph m3_graph;
typedef struct m3_session m3_session;

/* include/m3.h:197-259 (the graph/session subset; Music3 and Core ML
 * partitions are not part of this library). */
const char *m3_version(void);
const char *m3_status_string(m3_status status);
void m3_error_reset(m3_error *error);
const char *m3_error_message(const m3_error *error);
void m3_graph_value_desc_init(m3_graph_value_desc *description,
                              m3_graph_value_role role, m3_dtype dtype,
                              uint8_t rank, const uint64_t *shape);
void m3_graph_node_desc_init(m3_graph_node_desc *description,
                             m3_op_kind kind);
void m3_session_options_init(m3_session_options *options);
m3_status m3_graph_create(m3_graph **graph, m3_error *error);
void m3_graph_free(m3_graph *graph);
m3_status m3_graph_add_value(m3_graph *graph,
                             const m3_graph_value_desc *description,
                             m3_graph_value_id *value, m3_error *error);
m3_status m3_graph_set_constant(m3_graph *graph, m3_graph_value_id value,
                                const void *data, size_t byte_count,
                                m3_error *error);
m3_status m3_graph_add_inferred_value(
    m3_graph *graph, const m3_graph_node_desc *node, size_t output_index,
    m3_graph_value_role role, m3_dtype dtype, m3_graph_value_id *value,
    m3_error *error);
m3_status m3_graph_add_node(m3_graph *graph,
                            const m3_graph_node_desc *description,
                            m3_error *error);
m3_status m3_session_create(m3_session **session, const m3_graph *graph,
                             const m3_session_options *options,
                             m3_error *error);
void m3_session_free(m3_session *session);
m3_status m3_session_write_input(m3_session *session, m3_graph_value_id value,
                                  const void *data, size_t byte_count,
                                  m3_error *error);
m3_status m3_session_read_output(const m3_session *session,
                                  m3_graph_value_id value, void *data,
                                  size_t byte_count, m3_error *error);
m3_status m3_session_run(m3_session *session, m3_error *error);
m3_status m3_session_get_plan_info(const m3_session *session,
                                    m3_session_plan_info *info,
                                    m3_error *error);
m3_status m3_session_get_node_provider(const m3_session *session,
                                        size_t node_index,
                                        m3_provider_kind *provider,
                                        m3_error *error);
#endif /* M3_H */

/* ------------------------------------------------------------------------
 * Reference ABI (src/m3_tensor.h, src/m3_scratch.h, src/m3_op.h)
 * ------------------------------------------------------------------------ */
#ifndef M3_TENSOR_H
/* src/m3_tensor.h:12-18 */
typedef struct {
    m3_dtype dtype;
    uint8_t rank;
    uint64_t shape[M3_TENSOR_MAX_RANK];
    size_t element_count;
    size_t byte_count;
} m3_tensor_metadata;

/* Opaque storage of the host library (src/m3_backend.c:9-16). */
typedef struct m3_storage m3_storage;

/* src/m3_tensor.h:22-27 */
typedef struct {
    m3_tensor_metadata metadata;
    size_t byte_offset;
    size_t byte_strides[M3_TENSOR_MAX_RANK];
    m3_storage *storage;
} m3_tensor_view;
#endif /* M3_TENSOR_H */

#ifndef M3_SCRATCH_H
/* src/m3_scratch.h:11-15 */
typedef struct {
    uint8_t *data;
    size_t capacity;
    size_t offset;
} m3_scratch_arena;
#endif /* M3_SCRATCH_H */

#ifndef M3_OP_H
/* src/m3_op.h:14-148 */
typedef struct {
    const m3_tensor_view *input;
    m3_tensor_view *output;
} m3_op_unary;

typedef struct {
    const m3_tensor_view *left;
    const m3_tensor_view *right;
    m3_tensor_view *output;
} m3_op_binary;

typedef struct {
    const m3_tensor_view *ids;
    const m3_tensor_view *table;
    m3_tensor_view *output;
} m3_op_embedding;

typedef struct {
    const m3_tensor_view *left;
    const m3_tensor_view *right;
    m3_tensor_view *output;
} m3_op_matmul;

typedef struct {
    const m3_tensor_view *input;
    const m3_tensor_view *weight;
    const m3_tensor_view *bias;
    m3_tensor_view *output;
} m3_op_linear;

typedef struct {
    const m3_tensor_view *input;
    const m3_tensor_view *scale;
    m3_tensor_view *output;
    float epsilon;
} m3_op_rms_norm;

typedef struct {
    const m3_tensor_view *input;
    const m3_tensor_view *scale;
    const m3_tensor_view *bias;
    m3_tensor_view *output;
    float epsilon;
} m3_op_layer_norm;

typedef struct {
    const m3_tensor_view *input;
    const m3_tensor_view *cosines;
    const m3_tensor_view *sines;
    m3_tensor_view *output;
    uint64_t position_offset;
    uint32_t rotary_dimension;
    m3_rope_mode mode;
} m3_op_rope;

typedef struct {
    const m3_tensor_view *query;
    const m3_tensor_view *key;
    const m3_tensor_view *value;
    const m3_tensor_view *mask;
    m3_tensor_view *output;
    float scale;
    int64_t causal_offset;
    bool causal;
} m3_op_attention;

typedef struct {
    const m3_tensor_view *logits;
    m3_tensor_view *values;
    m3_tensor_view *indices;
    uint64_t k;
} m3_op_top_k;

typedef struct {
    const m3_tensor_view *probabilities;
    const m3_tensor_view *uniforms;
    m3_tensor_view *output;
} m3_op_categorical;

typedef struct {
    const m3_tensor_view *input;
    const m3_tensor_view *weight;
    const m3_tensor_view *bias;
    m3_tensor_view *output;
    uint64_t groups;
    uint64_t stride;
    uint64_t dilation;
    uint64_t pad_left;
    uint64_t pad_right;
} m3_op_conv1d;

typedef struct {
    const m3_tensor_view *input;
    const m3_tensor_view *weight;
    const m3_tensor_view *bias;
    m3_tensor_view *output;
    uint64_t groups;
    uint64_t stride;
    uint64_t dilation;
    uint64_t pad_left;
    uint64_t pad_right;
    uint64_t output_padding;
} m3_op_conv_transpose1d;

typedef struct {
    const m3_tensor_view *input;
    const m3_tensor_view *alpha;
    m3_tensor_view *output;
} m3_op_snake1d;

typedef struct {
    m3_op_kind kind;
    union {
        m3_op_unary copy;
        m3_op_unary cast;
        m3_op_binary add;
        m3_op_binary mul;
        m3_op_embedding embedding;
        m3_op_matmul matmul;
        m3_op_linear linear;
        m3_op_rms_norm rms_norm;
        m3_op_layer_norm layer_norm;
        m3_op_rope rope;
        m3_op_attention attention;
        m3_op_binary gated_silu;
        m3_op_unary softmax;
        m3_op_top_k top_k;
        m3_op_categorical categorical;
        m3_op_conv1d conv1d;
        m3_op_conv_transpose1d conv_transpose1d;
        m3_op_unary nearest_resize1d;
        m3_op_snake1d snake1d;
        m3_op_unary tanh;
    } descriptor;
} m3_command;
#endif /* M3_OP_H */

/* ------------------------------------------------------------------------
 * CUDA provider extensions
 * ------------------------------------------------------------------------ */

/* Provider reported by m3_session_get_node_provider for GPU-placed nodes.
 * Appended after the reference's last value (include/m3.h:80-84). */
#define M3_PROVIDER_CUDA ((m3_provider_kind)3)

/* Extension operators (no reference counterpart).  Both are unary: graph
 * nodes use inputs[0] / outputs[0]; commands use descriptor.copy.
 *
 * M3_OP_ABS_MAX: output is one F32 element holding max |x| over the whole
 *   input (any float dtype), computed on bit patterns so the result is exact
 *   and order-free; an empty input gives +0.  Any NaN fails the operator with
 *   M3_STATUS_OUT_OF_RANGE and leaves the output untouched (the reference's
 *   top-k NaN rule, src/m3_op_data_preflight.c:288-291).
 * M3_OP_CLAMP_UNIT: same shape and dtype; values above +1 become +1, values
 *   below -1 become -1, everything else (NaN payloads, signed zeros,
 *   subnormals) is copied bit for bit (the waveform clamp of the reference,
 *   src/m3_waveform.c:360-380). */
#define M3_OP_ABS_MAX ((m3_op_kind)64)
#define M3_OP_CLAMP_UNIT ((m3_op_kind)65)

/* M3_OP_ROW_SUM (extension, unary like the two above): the sum of each row
 * over the last axis, output F32 with the input's shape and the last axis 1
 * (input F32, F16 or BF16).  The additions run left to right in F32, each
 * rounded on its own: the order of the reference's softmax sum
 * (src/m3_op_execute_basic.c:150-158), so results are bit-exact against a
 * sequential F32 loop.  No data check: a NaN or infinity propagates as IEEE
 * addition makes it.  A SOFTMAX, TOP_K or ROW_SUM of the same input in one
 * graph shares one row pass. */
#define M3_OP_ROW_SUM ((m3_op_kind)66)

#define M3_CUDA_DEVICE_CURRENT (-1)

typedef struct {
    int device;            /* CUDA ordinal, or M3_CUDA_DEVICE_CURRENT */
    void *stream;          /* cudaStream_t to run on; NULL: the session owns
                              a non-blocking stream */
    bool fuse;             /* fuse element-wise chains and row prologues
                              (default true) */
    bool cuda_graphs;      /* enqueue each run (or each run sequence of
                              m3_cuda_session_run_steps_async) as one CUDA
                              graph launch, captured on first use for each
                              buffer assignment and kept (default true);
                              falls back to single launches on a stream that
                              cannot be captured */
} m3_cuda_session_options;

void m3_cuda_session_options_init(m3_cuda_session_options *options);

/* m3_session_create with explicit CUDA options.  m3_session_create itself
 * uses the defaults.  The accelerator is permitted when options->allow_metal
 * or options->allow_neural_engine is set (the reference's GPU switches); a
 * CPU-only request is M3_STATUS_UNSUPPORTED because this library holds no CPU
 * provider. */
m3_status m3_cuda_session_create(m3_session **session, const m3_graph *graph,
                                  const m3_session_options *options,
                                  const m3_cuda_session_options *cuda,
                                  m3_error *error);

/* Enqueue one run without waiting.  Failures of data checks (NaN, range) are
 * recorded on the device; later runs enqueued before the next synchronise
 * become no-ops after a failure, exactly as a failing m3_session_run stops.
 * m3_cuda_session_synchronize waits and returns the first failure since the
 * previous synchronise, with the reference's message. */
m3_status m3_cuda_session_run_async(m3_session *session, m3_error *error);

/* Enqueue `count` runs, exchanging the buffers of `input` and `output` (as
 * m3_cuda_session_swap_values) between consecutive runs, so each run reads
 * the previous run's output: the state of an iterative solver, e.g. the
 * flow-matching Euler loop x <- x + dt * v that the reference's flow solver
 * runs as repeated m3_session_run calls (src/m3_flow_solver_math.c:36-135).
 * No exchange follows the last run.  Pass M3_GRAPH_VALUE_NONE for both to
 * repeat runs without carrying state.  With cuda_graphs the whole sequence
 * is one graph launch.  Failure semantics are those of `count` calls of
 * m3_cuda_session_run_async. */
m3_status m3_cuda_session_run_steps_async(m3_session *session, size_t count,
                                          m3_graph_value_id input,
                                          m3_graph_value_id output,
                                          m3_error *error);

/* One run fed from and drained to host memory, enqueued without waiting.
 * The inputs are uploaded on a copy stream of the session into one of two
 * device staging areas and copied into their values on the session's stream
 * ahead of the run; after the run the outputs are copied to the other side
 * of the staging and downloaded on a second copy stream.  Consecutive
 * submissions alternate staging areas, so one submission's upload overlaps
 * the previous one's download (PCIe carries both directions at once) and the
 * runs themselves.  Host buffers should be pinned (cudaHostAlloc) for the
 * copies to be asynchronous; they must stay valid and untouched until the
 * next m3_cuda_session_synchronize, which waits for the downloads too.  If a
 * run fails (reported by that synchronise), the host outputs of its
 * submission and of later ones are unspecified; the values in the session
 * keep the reference's failure semantics.  The staging areas (twice the
 * submitted bytes) are allocated on first use and grown when needed. */
m3_status m3_cuda_session_submit_host_async(
    m3_session *session, size_t input_count, const m3_graph_value_id *inputs,
    const void *const *input_data, size_t output_count,
    const m3_graph_value_id *outputs, void *const *output_data,
    m3_error *error);
m3_status m3_cuda_session_synchronize(m3_session *session, m3_error *error);

/* Device address and byte size of a value's current storage (valid until the
 * next run, write or swap).  For zero-copy interoperation, e.g. handing an
 * output to a collective.  A temporary that a fused launch keeps in registers
 * has no storage (M3_STATUS_INVALID_ARGUMENT): the arena holds only the
 * slots that launches store or read and those of inputs, outputs and
 * constants, while m3_session_get_plan_info still reports the reference's
 * liveness plan. */
m3_status m3_cuda_session_value_device_pointer(const m3_session *session,
                                               m3_graph_value_id value,
                                               void **device_pointer,
                                               size_t *byte_count,
                                               m3_error *error);

/* Device-to-device input write / output read (no host staging).  The copy
 * runs on the session's stream after the runs enqueued there and the call
 * returns once it is complete.  Work on other streams is not waited for: a
 * source written on another stream (including the legacy default stream,
 * which a session-owned non-blocking stream does not wait on) must be
 * complete, or be ordered before the call with an event, by the caller. */
m3_status m3_cuda_session_write_input_device(m3_session *session,
                                             m3_graph_value_id value,
                                             const void *device_source,
                                             size_t byte_count,
                                             m3_error *error);
m3_status m3_cuda_session_read_output_device(const m3_session *session,
                                             m3_graph_value_id value,
                                             void *device_destination,
                                             size_t byte_count,
                                             m3_error *error);

/* As m3_cuda_session_read_output_device, but enqueued on the session's
 * stream without waiting: the copy reads the output as it stands after the
 * runs already enqueued, assuming they succeed.  If one of them fails (as
 * the next m3_cuda_session_synchronize reports), the copied bytes are
 * unspecified.  For pipelines that hand an output to another stream-ordered
 * consumer, such as a collective, without a host round trip. */
m3_status m3_cuda_session_read_output_device_async(
    m3_session *session, m3_graph_value_id value, void *device_destination,
    size_t byte_count, m3_error *error);

/* Exchange the storage of an INPUT and an OUTPUT value of equal byte size, in
 * O(1) and without copying: the next run reads as input what the last run
 * wrote as output.  Carries a solver state between runs (the flow solver's
 * x' -> x, reference src/m3_flow_solver_math.c:102-135). */
m3_status m3_cuda_session_swap_values(m3_session *session,
                                      m3_graph_value_id input,
                                      m3_graph_value_id output,
                                      m3_error *error);

/* The session's stream (cudaStream_t) and device ordinal. */
void *m3_cuda_session_stream(const m3_session *session);
int m3_cuda_session_device(const m3_session *session);

/* Execution plan summary: kernel launches per run and a one-line description
 * of each launch group ("ew[MUL,ADD] out=1", "row[SOFTMAX+TOP_K] ..."). */
typedef struct {
    size_t launch_count;
    size_t fused_node_count;     /* nodes that share a launch with another */
    size_t shadow_bytes;         /* extra arena bytes for atomic commit */
    size_t arena_bytes;          /* total device arena bytes */
} m3_cuda_plan_report;

m3_status m3_cuda_session_get_plan_report(const m3_session *session,
                                          m3_cuda_plan_report *report,
                                          char *text, size_t text_capacity,
                                          m3_error *error);

/* The same compile steps as session creation (topology, liveness slots,
 * binding, validation, placement, fusion) without touching a GPU: for tests
 * and capacity planning on hosts without a device. */
m3_status m3_cuda_graph_plan(const m3_graph *graph,
                             const m3_cuda_session_options *cuda,
                             m3_session_plan_info *info,
                             m3_cuda_plan_report *report, char *text,
                             size_t text_capacity, m3_error *error);

/* ------------------------------------------------------------------------
 * Sharding: one fixed graph split across the GPUs of a box
 * ------------------------------------------------------------------------
 * One process per GPU.  Every rank creates a shard session from the same
 * GLOBAL graph (global shapes and constants); the library cuts each value
 * along one split axis and keeps only this rank's slab in its own device
 * arena.  The split axis is counted in the shape of the graph's first input
 * of largest rank; other values are right-aligned against that shape.  A
 * value whose extent on that axis equals the global extent is split (slabs
 * are contiguous ranges, balanced, in whole blocks of 4 elements when the
 * extent allows); a value of extent 1 there, or without that axis, is
 * replicated (broadcast constants such as a snake alpha [1,C,1] split along
 * time, a norm scale, scalars).  Row operators (SOFTMAX, TOP_K, ROW_SUM,
 * RMS_NORM, LAYER_NORM, CATEGORICAL) need the split axis to differ from
 * their input's last axis.  M3_OP_ABS_MAX is a global reduction: every rank
 * reduces its slab, then one NCCL all-reduce (MAX over the unsigned bit
 * patterns, exact and order-free) on the session's stream gives every rank
 * the global result; its output may not feed another node.  When the graph
 * has a data check (NaN, F32-to-I32 range, categorical checks) the first
 * failing command is agreed on by the same all-reduce, so a failure on any
 * rank fails the run on every rank and leaves every rank's outputs as the
 * reference leaves them.  Element-wise and row operators exchange nothing.
 *
 * m3_session_write_input / read_output on a shard session move this rank's
 * slab (the local shape); m3_cuda_shard_write_input / read_output move it
 * out of / into a buffer laid out as the whole global tensor. */
#define M3_CUDA_SHARD_AXIS_AUTO (-1)

/* The identity of one communicator (NCCL's unique id). */
typedef struct {
    unsigned char bytes[128];
} m3_cuda_shard_id;

typedef struct {
    int rank;                    /* this process's shard, 0 <= rank < count */
    int count;                   /* number of shards (GPUs) */
    int axis;                    /* split axis, or M3_CUDA_SHARD_AXIS_AUTO:
                                    the outermost axis that every value
                                    allows and whose extent is at least
                                    `count` */
    const m3_cuda_shard_id *id;  /* communicator shared by all ranks, used
                                    when the graph has a global reduction or
                                    a data check (one id per communicator:
                                    each such session needs a fresh id);
                                    NULL: no collective (count 1, or a caller
                                    that combines global reductions itself) */
    double timeout_seconds;      /* bound on communicator set-up and each
                                    collective enqueue (default 120) */
} m3_cuda_shard_options;

void m3_cuda_shard_options_init(m3_cuda_shard_options *options);

/* A new communicator id (rank 0 calls this and hands the bytes to the other
 * ranks by its own means: MPI, a store, torch.distributed).  Loads NCCL
 * (libnccl.so.2) on first use; M3_STATUS_UNSUPPORTED when it is absent. */
m3_status m3_cuda_shard_id_create(m3_cuda_shard_id *id, m3_error *error);

/* Where one value's slab lies in the global tensor. */
typedef struct {
    bool split;                  /* false: replicated on every rank */
    uint8_t axis;                /* the value's own split axis (if split) */
    uint64_t begin;              /* this rank's first index on that axis */
    uint64_t extent;             /* this rank's extent on that axis */
    m3_tensor_metadata global;   /* the value in the global graph */
    m3_tensor_metadata local;    /* this rank's part */
} m3_cuda_shard_slab;

/* Host-only partition of `graph` for `shard` (no GPU, no communicator):
 * the slab of `value` and, through `axis_out`, the split axis chosen. */
m3_status m3_cuda_shard_plan(const m3_graph *graph,
                             const m3_cuda_shard_options *shard,
                             m3_graph_value_id value, m3_cuda_shard_slab *slab,
                             int *axis_out, m3_error *error);

/* This rank's session of the global graph: the local graph is planned,
 * fused and allocated as any session on `cuda->device`; with shard->id set
 * and count > 1 the ranks then join one communicator (every rank must call
 * this; the call returns once all have joined, or fails after the
 * timeout). */
m3_status m3_cuda_shard_session_create(m3_session **session,
                                       const m3_graph *graph,
                                       const m3_session_options *options,
                                       const m3_cuda_session_options *cuda,
                                       const m3_cuda_shard_options *shard,
                                       m3_error *error);

m3_status m3_cuda_shard_get_slab(const m3_session *session,
                                 m3_graph_value_id value,
                                 m3_cuda_shard_slab *slab, m3_error *error);

/* This rank's slab of an INPUT out of `global_data`, a buffer laid out as
 * the whole global tensor (global_byte_count bytes, host memory, or device
 * memory of any device when `device_memory`): one strided copy on the
 * session's stream, complete when the call returns.  A replicated input
 * takes the whole buffer. */
m3_status m3_cuda_shard_write_input(m3_session *session,
                                    m3_graph_value_id value,
                                    const void *global_data,
                                    size_t global_byte_count,
                                    bool device_memory, m3_error *error);

/* This rank's slab of an OUTPUT into its place in `global_data` (the rest of
 * the buffer is not touched); a replicated output is written whole. */
m3_status m3_cuda_shard_read_output(const m3_session *session,
                                    m3_graph_value_id value,
                                    void *global_data,
                                    size_t global_byte_count,
                                    bool device_memory, m3_error *error);

/* ------------------------------------------------------------------------
 * Backend plug-in (reference src/m3_backend_internal.h:9-17)
 * ------------------------------------------------------------------------
 * Free functions with the exact signatures of m3_backend_vtable's members,
 * to be registered with the reference's m3_backend_create_internal
 * (src/m3_backend.c:80-111).  The context is created here; the host library
 * supplies its storage accessor so views can be resolved to device
 * addresses. */
typedef struct {
    int device;                                    /* CUDA ordinal */
    /* The host library's m3_storage_data (reference src/m3_backend.h:52). */
    void *(*storage_data)(m3_storage *storage);
    /* true: storages are cudaMallocManaged, so the reference's memcpy-based
     * m3_storage_write/read (src/m3_backend.c:319-366) work unchanged and
     * the backend reports unified memory; false: device memory, and the
     * host library must route writes/reads to m3_cuda_backend_write/read. */
    bool managed_memory;
} m3_cuda_backend_options;

m3_status m3_cuda_backend_context_create(
    const m3_cuda_backend_options *options, void **context, m3_error *error);
/* vtable.destroy_context */
void m3_cuda_backend_destroy_context(void *context);
/* vtable.allocate: 256-byte aligned device (or managed) memory. */
m3_status m3_cuda_backend_allocate(void *context, size_t byte_count,
                                   size_t alignment, void **handle,
                                   void **data, m3_error *error);
/* vtable.free_storage */
void m3_cuda_backend_free_storage(void *context, void *handle, void *data);
/* vtable.execute: runs the commands in order on the GPU and returns after the
 * stream has finished, with the reference's all-or-nothing data checks. */
m3_status m3_cuda_backend_execute(void *context, const m3_command *commands,
                                  size_t command_count,
                                  m3_scratch_arena *scratch, m3_error *error);
/* The write/read hooks a non-unified backend needs (host <-> device). */
m3_status m3_cuda_backend_write(void *context, void *data, size_t byte_offset,
                                const void *source, size_t byte_count,
                                m3_error *error);
m3_status m3_cuda_backend_read(void *context, const void *data,
                               size_t byte_offset, void *destination,
                               size_t byte_count, m3_error *error);
/* Placement table for m3_provider_select_regular (src/m3_provider.c:7-33). */
bool m3_cuda_backend_supports_kind(m3_op_kind kind);
/* Kernels the last m3_cuda_backend_execute on this context launched (no
 * reference counterpart: a measurement hook).  Consecutive element-wise
 * commands over one output shape, and SOFTMAX / TOP_K / ROW_SUM commands over
 * one input view, share a launch where that cannot change a result. */
unsigned m3_cuda_backend_launch_count(const void *context);
/* Run this context's executes on a caller's cudaStream_t (NULL: the stream
 * the context created), e.g. one shared with a framework or timed with
 * events; no reference counterpart.  Waits for work already queued on the
 * previous stream.  execute still returns after the stream is idle. */
m3_status m3_cuda_backend_set_stream(void *context, void *stream, m3_error *error);
/* A storage accessor for hosts whose storage handles are the device
 * addresses themselves (pass it as m3_cuda_backend_options.storage_data);
 * no reference counterpart: the reference's own accessor is
 * m3_storage_data. */
void *m3_cuda_storage_is_address(m3_storage *storage);

/* ------------------------------------------------------------------------
 * Seeded synthetic inputs (reference src/m3_rng.c:9-110)
 * ------------------------------------------------------------------------
 * PCG32 seeded as m3_rng_seed(seed, sequence).  Host fills produce exactly the
 * reference's sequence; device fills produce the same sequence by jumping the
 * generator ahead per element block (bit-identical for uniforms; normals use
 * the GPU's double-precision log/sin/cos and agree to within 1 ulp of F32). */
m3_status m3_cuda_fill_uniform_host(uint64_t seed, uint64_t sequence,
                                    float low, float high, float *values,
                                    size_t count, m3_error *error);
m3_status m3_cuda_fill_normal_host(uint64_t seed, uint64_t sequence,
                                   float mean, float deviation, float *values,
                                   size_t count, m3_error *error);
m3_status m3_cuda_fill_uniform_device(uint64_t seed, uint64_t sequence,
                                      float low, float high,
                                      float *device_values, size_t count,
                                      void *stream, m3_error *error);
m3_status m3_cuda_fill_normal_device(uint64_t seed, uint64_t sequence,
                                     float mean, float deviation,
                                     float *device_values, size_t count,
                                     void *stream, m3_error *error);

/* Number of CUDA devices visible (0 without a driver or GPU). */
int m3_cuda_device_count(void);

/* Diagnostics: the kernels narrow F32 to F16/BF16 with the hardware
 * round-to-nearest-even conversions and apply the reference's NaN payload
 * rules (src/m3_op_numeric.c:55-130) in software.  This runs every F32 bit
 * pattern (and every F16 pattern for widening) through both that path and an
 * integer restatement of the reference encoders on `device` and reports the
 * number of disagreements (0 expected). */
m3_status m3_cuda_codec_self_test(int device, uint64_t *mismatches,
                                  m3_error *error);

/* Diagnostics: softmax divides by the row sum with an FMA refinement of the
 * correctly rounded reciprocal (Markstein, IBM J. Res. Develop. 34(1), 1990)
 * instead of the IEEE division sequence.  This draws `samples` quotients
 * e / s with e in [2^-100, 1] and s in [1, 2^24] (the softmax domain) and
 * reports how many differ from the IEEE division (0 expected). */
m3_status m3_cuda_division_self_test(int device, uint64_t samples,
                                     uint64_t *mismatches, m3_error *error);

/* Diagnostics: gated SiLU with F16 or BF16 results evaluates e^-g with the
 * PTX base-2 approximation after a Cody-Waite reduction (for |g| <= 80;
 * other gates, and F32 results, take the IEEE path), since a few F32 ulps
 * are far below the half-ulp of the 16-bit result.  This runs every F32
 * argument in [-87, 87] on `device` against the correctly rounded e^d and
 * reports the largest distance in ulps (`max_ulp`) and `violations`, the
 * count of wrong special values (e^0 must be exactly 1). */
m3_status m3_cuda_exp_self_test(int device, uint32_t *max_ulp,
                                uint64_t *violations, m3_error *error);

/* Diagnostics: SNAKE1D evaluates sin^2(alpha x) with its own reduction and
 * series for |alpha x| <= 8192 (other arguments take sinf), within the
 * activation's 0x1p-19 tolerance.  This runs every F32 argument in
 * [-8192, 8192] on `device` against sin(t)^2 in double precision and reports
 * the largest absolute error and the largest distance in ulps where
 * sin(t)^2 >= 2^-10. */
m3_status m3_cuda_sin_squared_self_test(int device, float *max_abs_error,
                                        uint32_t *max_ulp, m3_error *error);

/* Diagnostics: the snake's sin^2 runs two arguments per packed F32x2
 * instruction; this compares that evaluation with the scalar one, bit for
 * bit, on every F32 argument in [-8192, 8192] and reports the number of
 * differing results (0 expected). */
m3_status m3_cuda_sin_squared_packed_self_test(int device, uint64_t *mismatches,
                                               m3_error *error);

/* ------------------------------------------------------------------------
 * Abs-max without allocation.  No counterpart in the reference: m3.c has no
 * device memory to manage, so it has no allocation-free variant either.
 *
 * Who needs it: the session and the backend plug-in both allocate device
 * memory for their reduction scratch (cudaMalloc at creation).  Some callers
 * cannot do that at the point where they want a peak level: a real-time audio
 * render thread must not call cudaMalloc or cudaFree, whose latency has no
 * bound (they take driver locks, and cudaFree waits for the whole device to go
 * idle); and a caller that has already divided the device's memory among its
 * own pools has none left to hand out.  This entry point needs no memory
 * beyond what the caller passes in: its scratch is a fixed array compiled
 * into this library's device code.
 *
 * m3_cuda_abs_max_static computes M3_OP_ABS_MAX of each of `tensor_count`
 * dense tensors of `dtype` (F32, F16 or BF16) that live on `device`:
 * maxima[i] (device memory, 4-byte aligned, F32) receives max |x| over the
 * element_counts[i] elements at inputs[i], exactly as a graph or backend
 * ABS_MAX command would compute it (the same kernel and program); an empty
 * tensor gives +0.  A tensor holding a NaN leaves its maxima[i] untouched; the
 * others are still written, and the call returns M3_STATUS_OUT_OF_RANGE
 * naming the first such tensor.  The work runs on `stream` (a cudaStream_t;
 * NULL is the legacy default stream) and the call waits for that stream to
 * finish before it returns.
 *
 * Limit: at most M3_CUDA_ABS_MAX_STATIC_MAX_TENSORS tensors per call (the
 * scratch holds one reduction slot and one status word set per tensor,
 * 24 bytes each, 1.5 KiB in all); more returns M3_STATUS_INVALID_ARGUMENT
 * before any device work.  Each call zeroes the reduction slots it uses and
 * resets their status words before its kernels start.
 *
 * The scratch is one array per device, shared by every caller in the process:
 * two calls on the same device whose work overlaps in time (from two host
 * threads, or on two streams) race on it and return wrong maxima.  Callers
 * must serialise calls per device.
 *
 * The first call on each device looks the scratch up with
 * cudaGetSymbolAddress, with `device` made current; that lookup can load this
 * library's device code.  Make the first call for each device before any
 * stream capture begins.  The calling thread's current device is restored
 * before return. */
#define M3_CUDA_ABS_MAX_STATIC_MAX_TENSORS 64U

m3_status m3_cuda_abs_max_static(int device, void *stream, m3_dtype dtype,
                                 const void *const *inputs,
                                 const uint64_t *element_counts,
                                 size_t tensor_count, float *maxima,
                                 m3_error *error);

#ifdef __cplusplus
}
#endif

#endif /* M3_CUDA_H */
