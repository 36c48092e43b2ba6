/* CPU restatement of m3.c's tensor hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker for the CUDA provider in this repository.  It is
 * never linked into, loaded by, or called from the product library; only the
 * tests, the smoke check and the benchmark's CPU-baseline leg use it.
 *
 * Every function restates one reference algorithm, cited by file:line of the
 * reference project (taconotsandwich/m3.c), with the same statement order and
 * the same per-statement F32 rounding, so its outputs are bit-identical to the
 * reference CPU provider for the same inputs (pinned by tests against the
 * reference's own known-answer values and against the reference library
 * compiled from source into oracle/_ref).
 *
 * Views follow the reference's m3_tensor_view (src/m3_tensor.h:12-27): a dtype,
 * a rank <= 8, a shape, byte strides, a byte offset and a base pointer. */

#ifndef M3_ORACLE_H
#define M3_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define M3O_MAX_RANK 8

/* Same numbering as the reference include/m3.h:20-31 and :45-50. */
enum { M3O_OK = 0, M3O_INVALID_ARGUMENT = 1, M3O_OUT_OF_RANGE = 2 };
enum { M3O_F32 = 0, M3O_F16 = 1, M3O_BF16 = 2, M3O_I32 = 3 };

typedef struct {
    int32_t dtype;
    int32_t rank;
    uint64_t shape[M3O_MAX_RANK];
    uint64_t byte_strides[M3O_MAX_RANK];
    uint64_t byte_offset;
    void *base;
} m3o_view;

/* Scalar codecs (reference src/m3_op_numeric.c:27-130). */
float m3o_f16_to_f32(uint16_t half);
uint16_t m3o_f32_to_f16(float value);
float m3o_bf16_to_f32(uint16_t value);
uint16_t m3o_f32_to_bf16(float value);
float m3o_round_to_dtype(int32_t dtype, float value);

/* Element-wise operators.  Inputs may be strided; outputs are written through
 * their own strides (the reference requires contiguous outputs). */
int m3o_copy(const m3o_view *input, m3o_view *output);
int m3o_cast(const m3o_view *input, m3o_view *output);
int m3o_binary(int multiply, const m3o_view *left, const m3o_view *right,
               m3o_view *output);
int m3o_gated_silu(const m3o_view *gate, const m3o_view *up,
                   m3o_view *output);
int m3o_snake1d(const m3o_view *input, const m3o_view *alpha,
                m3o_view *output);
int m3o_tanh(const m3o_view *input, m3o_view *output);

/* Row reductions over the last axis. */
int m3o_softmax(const m3o_view *input, m3o_view *output);
int m3o_top_k(const m3o_view *logits, m3o_view *values, m3o_view *indices,
              uint64_t k);
int m3o_rms_norm(const m3o_view *input, const m3o_view *scale,
                 m3o_view *output, float epsilon);
int m3o_layer_norm(const m3o_view *input, const m3o_view *scale,
                   const m3o_view *bias, m3o_view *output, float epsilon);

/* Extension operators of the CUDA provider (no reference operator exists). */
int m3o_abs_max(const m3o_view *input, m3o_view *output);
int m3o_clamp_unit(const m3o_view *input, m3o_view *output);
int m3o_row_sum(const m3o_view *input, m3o_view *output);

/* The reference RNG's 32-bit word stream (src/m3_rng.c:9-39). */
void m3o_pcg32_fill(uint64_t seed, uint64_t sequence, uint32_t *words,
                    size_t count);

/* Flow-matching time grid (reference src/m3_flow_common.c:159-190). */
float m3o_flow_timestep(uint32_t step, uint32_t step_count);
float m3o_flow_timestep_delta(uint32_t step, uint32_t step_count);

#endif
