/* Kernel parameter blocks shared by the C11 host planner and the sm_100a
 * kernels.  Plain C structs of fixed size, passed by value as kernel
 * parameters, so a launch needs no device-side descriptor memory. */

#ifndef M3C_KERNELS_H
#define M3C_KERNELS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage dtypes: the reference numbering (include/m3.h:45-50). */
#define M3C_F32 0
#define M3C_F16 1
#define M3C_BF16 2
#define M3C_I32 3

#define M3C_MAX_DIMS 8

/* 32-bit division by an invariant divisor d > 0 as a multiply-high and a
 * shift (Granlund and Montgomery, "Division by invariant integers using
 * multiplication", PLDI 1994): q = (umulhi(n, m) + n) >> s for n < 2^32,
 * with s = ceil(log2 d) and m = floor(2^32 * (2^s - d) / d) + 1. */
typedef struct {
    uint32_t divisor;
    uint32_t multiplier;
    uint32_t shift;
    uint32_t reserved;
} m3c_fastdiv;

/* How an element-wise operand is addressed for a block of VEC consecutive
 * output elements. */
enum {
    M3C_V_CONTIG = 0,   /* same order as the output: one vector load */
    M3C_V_UNIFORM = 1,  /* the whole block reads one element */
    M3C_V_GATHER = 2,   /* general strided/broadcast: per-element offsets */
    M3C_V_IMM = 3,      /* folded scalar constant */
    M3C_V_VECTOR = 4    /* adjacent input elements at a strided offset */
};

/* How a loaded element becomes a 32-bit register word. */
enum {
    M3C_LOAD_FLOAT = 0, /* widen F16/BF16/F32 to F32 */
    M3C_LOAD_INT = 1,   /* I32 bits */
    M3C_LOAD_RAW = 2    /* the raw storage bits (16 or 32), for exact copies */
};

/* A strided, broadcast operand addressed by the flat output index f: with the
 * output dimensions coalesced for this operand, innermost first,
 *   offset(f) = sum_d ((f / prod_{e<d} size_e) % size_d) * stride_d
 * in bytes (stride 0 on broadcast dimensions). */
typedef struct {
    const void *base;
    int32_t dtype;
    int32_t load_as;
    int32_t vclass;
    int32_t ndim;
    uint32_t imm_bits;
    uint32_t reserved;
    uint64_t size[M3C_MAX_DIMS];
    int64_t stride[M3C_MAX_DIMS];
    m3c_fastdiv fdiv[M3C_MAX_DIMS];
} m3c_operand;

/* Element-wise micro-operations on 32-bit register words.  Every float result
 * is rounded to F32 and then to `rdtype` (the dtype the reference stores it
 * in), which reproduces the reference's store-then-reload between commands. */
enum {
    M3C_OP_ADD = 0,     /* dst = a + b */
    M3C_OP_MUL,         /* dst = a * b */
    M3C_OP_GSILU,       /* dst = round_aux(a / (1 + expf(-a))) * b */
    M3C_OP_SNAKE,       /* dst = snake1d(x = a, alpha = b) */
    M3C_OP_TANH,        /* dst = tanhf(a) */
    M3C_OP_ROUND,       /* dst = round_rdtype(a): float-to-float cast */
    M3C_OP_F2I,         /* dst = (int32)trunc(a), range-checked */
    M3C_OP_I2F,         /* dst = round_rdtype((float)(int32)a) */
    M3C_OP_WIDEN,       /* dst = widen raw 16-bit word of dtype aux */
    M3C_OP_CLAMP,       /* dst = bits-preserving clamp of F32 a to [-1,1] */
    M3C_OP_MOV,         /* dst = a (raw word) */
    M3C_OP_ABSMAX       /* reduce |a| (bits) into the group's max word */
};

typedef struct {
    uint8_t code;
    uint8_t dst;
    uint8_t a;
    uint8_t b;
    int8_t rdtype;      /* dtype the result is rounded to */
    int8_t aux;         /* GSILU: gate dtype; WIDEN: source dtype */
    uint16_t command;   /* reference command (node) index, for failures */
} m3c_ew_op;

typedef struct {
    void *base;
    int32_t dtype;
    int16_t reg;
    uint8_t raw;         /* register holds raw storage bits (exact copies) */
    uint8_t scalar_only; /* base not aligned for vector stores */
} m3c_ew_out;

#define M3C_EW_MAX_OPERANDS 8
#define M3C_EW_MAX_OPS 16
#define M3C_EW_MAX_OUTPUTS 4
#define M3C_EW_MAX_REGS 8

/* Device status of a session: the first failing command and its code, and the
 * number of runs that started clean since the last synchronise.  A launch
 * skips its work when a command before its `skip_before` bound has failed
 * (an earlier command of the run), but not for failures of its own
 * commands, so unchecked commands of a fused launch always complete. */
/* runs_started's top bit: a run of the batch failed and the run gate that
 * precedes the next run halted everything after it (every launch skips). */
#define M3C_RUN_HALTED 0x80000000u

typedef struct {
    uint32_t fail_command;  /* UINT32_MAX when clean */
    uint32_t fail_code;
    uint32_t runs_started;  /* runs started clean; M3C_RUN_HALTED bit */
    uint32_t detail;        /* categorical: smallest row * 4 + reason that
                               failed (UINT32_MAX when clean) */
} m3c_status;

/* Reduction scratch of one launch: the running abs-max bit pattern and the
 * count of finished CTAs (the last CTA publishes and resets both). */
typedef struct {
    uint32_t max_bits;
    uint32_t done_ctas;
} m3c_reduce_scratch;

typedef struct {
    uint64_t count;                 /* output elements */
    int32_t n_operands;
    int32_t n_ops;
    int32_t n_outputs;
    int32_t first_of_run;           /* count this run in status->runs_started */
    m3c_status *status;
    /* abs-max reduction (n_ops contains one M3C_OP_ABSMAX) */
    m3c_reduce_scratch *reduce;
    void *absmax_out;               /* one F32 element */
    uint32_t absmax_command;
    uint32_t skip_before;           /* skip when a command < this failed */
    int32_t absmax_publish_always;  /* shard of a sharded session: publish the
                                       slab's maximum even when it is a NaN
                                       pattern (the all-reduce after the run
                                       turns it into the failure of every
                                       rank) */
    int32_t reserved;
    m3c_operand operands[M3C_EW_MAX_OPERANDS];
    m3c_ew_op ops[M3C_EW_MAX_OPS];
    m3c_ew_out outputs[M3C_EW_MAX_OUTPUTS];
} m3c_ew_params;

/* Row kernels over the last axis of a contiguous [rows, width] tensor. */
typedef struct {
    const void *input;          /* [rows, width] */
    int32_t in_dtype;
    int32_t first_of_run;
    uint64_t rows;
    uint64_t width;
    m3c_status *status;
    /* softmax output (NULL: none) */
    void *probs;
    int32_t probs_dtype;
    uint32_t softmax_command;
    /* top-k outputs (NULL: none) */
    float *top_values;          /* [rows, k] F32 */
    int32_t *top_indices;       /* [rows, k] I32 */
    uint64_t k;
    uint32_t topk_command;
    uint32_t skip_before;       /* skip when a command < this failed */
    /* row sums (NULL: none): F32 [rows], left to right in F32 */
    float *row_sums;
    uint32_t rowsum_command;
    uint32_t reserved;
} m3c_softmax_params;

typedef struct {
    /* input = x, or x = round_in(resid_a + resid_b) when resid_b != NULL */
    const void *x;
    const void *resid_b;
    void *sum_out;              /* write x (the residual sum) here if non-NULL */
    int32_t in_dtype;
    int32_t first_of_run;
    const void *scale;          /* [width] */
    int32_t scale_dtype;
    int32_t out_dtype;
    const void *bias;           /* [width] or NULL (LayerNorm only) */
    int32_t bias_dtype;
    int32_t layer_norm;         /* 0: RMSNorm, 1: LayerNorm */
    void *out;
    uint64_t rows;
    uint64_t width;
    float epsilon;
    uint32_t skip_before;       /* skip when a command < this failed */
    m3c_status *status;
} m3c_norm_params;

/* Categorical sampling (reference src/m3_op_execute_sampling.c:90-137 with
 * the checks of src/m3_op_data_preflight.c:231-268): one index per row. */
typedef struct {
    const void *probabilities;  /* dense [rows, width] */
    int32_t probabilities_dtype;
    const void *uniforms;       /* dense [rows] */
    int32_t uniforms_dtype;
    int32_t *output;            /* [rows] I32 */
    uint64_t rows;
    uint64_t width;
    m3c_status *status;
    uint32_t command;
    uint32_t skip_before;
    int32_t first_of_run;
    int32_t check_only;         /* 1: record failures, write nothing */
} m3c_categorical_params;

int m3c_launch_categorical(const m3c_categorical_params *params, void *stream);

/* The warp-specialised SOFTMAX/TOP_K(k <= 1)/ROW_SUM pipeline for F32 rows of
 * 512 or 1024 elements (m3c_ring.cu); -1 when it does not apply. */
int m3c_launch_softmax_ring(const m3c_softmax_params *params, void *stream);

/* The number of contiguous row ranges the row pass for `params` reads side
 * by side (1: ascending order). */
uint32_t m3c_softmax_row_ranges(const m3c_softmax_params *params);

/* The words a sharded session's ranks agree on after each run: the bit
 * patterns of its global reductions (ABS_MAX outputs) and the complement of
 * the first failing command, all combined by one MAX all-reduce. */
#define M3C_SHARD_MAX_REDUCTIONS 8

typedef struct {
    uint32_t *values[M3C_SHARD_MAX_REDUCTIONS];   /* F32 reduction outputs */
    uint32_t commands[M3C_SHARD_MAX_REDUCTIONS];
    int32_t count;
    int32_t reserved;
    m3c_status *status;
    uint32_t *staging;                            /* count + 1 words */
} m3c_shard_words;

/* The kernel and grid m3c_launch_ew would use, chosen once (sessions keep it
 * per launch so repeated runs skip the program search), and the launch with
 * that choice. */
typedef struct {
    void *kernel;
    uint64_t grid;
    /* a TMA-fed variant (NULL: none), taken when the launch's pointers are
     * 16-byte aligned */
    void *bulk;
    uint64_t bulk_grid;
    uint32_t bulk_smem;
    uint32_t reserved;
} m3c_ew_choice;
int m3c_ew_choose(const m3c_ew_params *params, m3c_ew_choice *choice);
int m3c_launch_ew_chosen(const m3c_ew_choice *choice, const m3c_ew_params *params,
                         void *stream);

#ifdef __cplusplus
}
#endif

#endif
