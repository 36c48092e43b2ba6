/* Internal host-side declarations of libm3cuda.so (C11). */

#ifndef M3C_INTERNAL_H
#define M3C_INTERNAL_H

#include "m3_cuda.h"
#include "m3c_kernels.h"

#include <stdarg.h>
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#define M3C_VERSION "0.1.0-cuda"
#define M3C_ARENA_ALIGNMENT 256U
#define M3C_NO_SLOT SIZE_MAX

/* ------------------------------------------------------------ errors */

m3_status m3c_error_set(m3_error *error, m3_status status, const char *format,
                        ...);
/* The reference's preflight message for a failed categorical check, from the
 * status detail word (row * 4 + reason; src/m3_op_data_preflight.c:246-265). */
const char *m3c_categorical_message(uint32_t detail);

/* ------------------------------------------------------------- tensors */

size_t m3c_dtype_size(m3_dtype dtype);
bool m3c_dtype_float(m3_dtype dtype);
m3_status m3c_metadata_init(m3_tensor_metadata *metadata, m3_dtype dtype,
                            uint8_t rank, const uint64_t *shape,
                            m3_error *error);
bool m3c_shape_equal(const m3_tensor_metadata *a, const m3_tensor_metadata *b);

/* --------------------------------------------------------------- graph */

/* Mirrors the reference's graph state (src/m3_graph_internal.h:10-48). */
typedef struct {
    m3_graph_value_desc description;
    m3_tensor_metadata metadata;
    void *constant_data;
    size_t constant_size;
    bool constant_set;
} m3c_graph_value;

struct m3_graph {
    m3c_graph_value *values;
    size_t value_count;
    size_t value_capacity;
    m3_graph_node_desc *nodes;
    size_t node_count;
    size_t node_capacity;
};

/* --------------------------------------------------- validation (views) */

/* A view as the validators see it: metadata, byte offset and strides within
 * a storage, identified by an opaque storage key (same key = same storage). */
typedef struct {
    const m3_tensor_metadata *metadata;
    size_t byte_offset;
    const size_t *byte_strides;
    const void *storage;
    bool present;
} m3c_vview;

/* One operator with its views, in reference positions. */
typedef struct {
    m3_op_kind kind;
    m3c_vview in[3];
    m3c_vview out[2];
    float epsilon;
    uint64_t k;
} m3c_vcommand;

m3_status m3c_validate(const m3c_vcommand *command, m3_error *error);
bool m3c_kind_supported(m3_op_kind kind);
const char *m3c_kind_name(m3_op_kind kind);

/* ---------------------------------------------------------------- plan */

typedef enum {
    M3C_LAUNCH_EW = 0,
    M3C_LAUNCH_SOFTMAX,     /* softmax, top-k and/or row sums of the same rows */
    M3C_LAUNCH_NORM,        /* RMSNorm / LayerNorm, optional residual add */
    M3C_LAUNCH_CATEGORICAL  /* categorical sampling: row_in probabilities,
                               row_in_b uniforms, row_out indices */
} m3c_launch_kind;

/* A reference to a value's device bytes at run time: slot + byte offset, and
 * whether the access goes to the slot's shadow buffer (outputs committed
 * atomically at the end of the run). */
typedef struct {
    uint32_t value;     /* graph value id, UINT32_MAX: none */
    bool shadow;        /* write/read the pending (shadow) side */
} m3c_ref;

typedef struct {
    m3c_ref ref;        /* memory operand; value == UINT32_MAX: immediate */
    int32_t load_as;
    uint32_t imm_bits;
} m3c_ew_operand_plan;

typedef struct {
    m3c_launch_kind kind;
    size_t first_node;
    size_t node_count;
    /* element-wise */
    uint32_t shape_value;          /* value whose shape is the iteration space */
    int n_operands;
    m3c_ew_operand_plan operands[M3C_EW_MAX_OPERANDS];
    int n_ops;
    m3c_ew_op ops[M3C_EW_MAX_OPS];
    int n_outputs;
    m3c_ref outputs[M3C_EW_MAX_OUTPUTS];
    int output_regs[M3C_EW_MAX_OUTPUTS];
    bool output_raw[M3C_EW_MAX_OUTPUTS];
    bool has_absmax;
    m3c_ref absmax_out;
    uint32_t absmax_command;
    /* row kernels */
    m3c_ref row_in;
    m3c_ref row_in_b;              /* residual second operand, or none */
    m3c_ref row_sum_out;           /* residual sum output, or none */
    m3c_ref row_out;               /* softmax probs / norm output */
    m3c_ref row_out2;              /* top-k values */
    m3c_ref row_out3;              /* top-k indices */
    m3c_ref row_out4;              /* row sums */
    m3c_ref norm_scale;
    m3c_ref norm_bias;
    bool layer_norm;
    float epsilon;
    uint64_t k;
    uint32_t command_a;            /* softmax command */
    uint32_t command_b;            /* top-k command */
    uint32_t command_c;            /* row-sum command */
    char text[96];
} m3c_launch;

typedef struct {
    /* liveness plan, identical to the reference planner */
    size_t value_count;
    size_t node_count;
    size_t slot_count;
    size_t *value_slot;            /* value -> slot */
    size_t *slot_bytes;            /* slot -> bytes */
    size_t allocated_bytes;        /* sum of slot bytes (reference plan) */
    size_t *producers;
    size_t *last_uses;
    bool *slot_shadowed;           /* slot needs a second (shadow) buffer */
    bool *slot_needed;             /* slot is stored or read by some launch or
                                      holds an input, output or constant;
                                      temporaries fused into registers get no
                                      memory */
    /* launches */
    m3c_launch *launches;
    size_t launch_count;
    size_t fused_node_count;
    size_t shadow_bytes;
    size_t arena_bytes;
    /* flips: (slot, command) pairs committed at the end of a clean run */
    size_t *flip_slot;
    uint32_t *flip_command;
    size_t flip_count;
} m3c_plan;

m3_status m3c_plan_build(const m3_graph *graph, bool fuse, m3c_plan *plan,
                         m3_error *error);
void m3c_plan_free(m3c_plan *plan);
void m3c_plan_describe(const m3c_plan *plan, char *text, size_t capacity);

/* --------------------------------------------------- operand addressing */

/* Fill `operand` to read `metadata` at byte_offset/byte_strides (bytes) from
 * `base`, broadcast right-aligned against the output shape `out`. */
void m3c_operand_setup(m3c_operand *operand, const void *base,
                       const m3_tensor_metadata *metadata, size_t byte_offset,
                       const size_t *byte_strides,
                       const m3_tensor_metadata *out, int32_t load_as);
void m3c_fastdiv_init(m3c_fastdiv *fd, uint32_t divisor);
bool m3c_contiguous(const m3_tensor_metadata *metadata,
                    const size_t *byte_strides);

/* ------------------------------------------------ kernel launch ABI (.cu) */

int m3c_launch_ew(const m3c_ew_params *params, void *stream);
int m3c_launch_softmax(const m3c_softmax_params *params, void *stream);
int m3c_launch_norm(const m3c_norm_params *params, void *stream);
/* mode 0: NaN check; mode 1: float-to-I32 range check (contiguous data) */
int m3c_launch_scan(const void *data, int32_t dtype, uint64_t count, int mode,
                    uint32_t command, m3c_status *status, void *stream);
/* The same checks over `rows` rows of `width` elements, one warp per row,
 * visiting the rows in the reverse of the order a row kernel reading
 * `ranges` contiguous row ranges side by side consumes them (so they are
 * still in L2 when it does); falls back to m3c_launch_scan for rows that are
 * not whole 16-byte vectors. */
int m3c_launch_row_scan(const void *data, int32_t dtype, uint64_t rows, uint64_t width,
                        uint32_t ranges, int mode, uint32_t command, m3c_status *status,
                        void *stream);
int m3c_launch_rng_uniform(uint64_t seed, uint64_t sequence, float low,
                           float high, float *out, uint64_t count,
                           void *stream);
int m3c_launch_rng_normal(uint64_t seed, uint64_t sequence, float mean,
                          float deviation, float *out, uint64_t count,
                          void *stream);
const char *m3c_cuda_error_string(int code);

/* ------------------------------------------------------------ sharding */

/* One rank's share of a sharded session (m3c_shard.c). */
typedef struct {
    int rank;
    int count;
    int axis;                      /* split axis in the primary value's shape */
    size_t value_count;
    m3_cuda_shard_slab *slabs;     /* per value */
    void *comm;                    /* NCCL communicator, or NULL */
    double timeout_seconds;
    int reduction_count;           /* ABS_MAX outputs, all-reduced per run */
    uint32_t reductions[M3C_SHARD_MAX_REDUCTIONS];
    uint32_t reduction_commands[M3C_SHARD_MAX_REDUCTIONS];
    bool checks;                   /* the graph has a data-checked command */
    uint32_t *staging;             /* device words: reductions, then status */
} m3c_shard;

/* The collective step after each run is needed (a communicator and
 * something to agree on). */
bool m3c_shard_collective(const m3c_shard *shard);
void m3c_shard_free(m3c_shard *shard);

/* NCCL (m3c_nccl.c), loaded at run time. */
m3_status m3c_comm_create(const m3_cuda_shard_id *id, int rank, int count,
                          double limit_seconds, void **comm, m3_error *error);
void m3c_comm_destroy(void *comm);
m3_status m3c_comm_max_u32(void *comm, uint32_t *words, size_t count,
                           void *stream, double limit_seconds,
                           m3_error *error);

/* Session internals the sharding layer needs (m3c_session.c). */
void m3c_session_attach_shard(m3_session *session, m3c_shard *shard);
const m3c_shard *m3c_session_shard(const m3_session *session);
const m3_tensor_metadata *m3c_session_metadata(const m3_session *session,
                                               m3_graph_value_id value);
m3_graph_value_role m3c_session_role(const m3_session *session,
                                     m3_graph_value_id value);
size_t m3c_session_value_count(const m3_session *session);

/* Halts the runs after a failed one in a batch (m3c_util.cu). */
int m3c_launch_run_gate(m3c_status *status, void *stream);

/* Pack / unpack around the per-run all-reduce (m3c_util.cu). */
int m3c_launch_shard_pack(const m3c_shard_words *words, void *stream);
int m3c_launch_shard_unpack(const m3c_shard_words *words, void *stream);

/* -------------------------------------------------------------- rng */

typedef struct {
    uint64_t state;
    uint64_t increment;
} m3c_pcg32;

void m3c_pcg32_seed(m3c_pcg32 *rng, uint64_t seed, uint64_t sequence);
uint32_t m3c_pcg32_next(m3c_pcg32 *rng);

#endif
