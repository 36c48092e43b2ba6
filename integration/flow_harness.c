/* Test harness (test infrastructure, built only into the patched reference
 * library under _ref/): runs the reference's own flow-solver arithmetic --
 * m3_flow_guided_velocity, m3_flow_euler_step and m3_flow_blend_overlap
 * (src/m3_flow_solver_math.c:36-205) -- on a backend of the caller's choice.
 * Those functions build their MUL/ADD commands on views of a velocity
 * tensor and of flow workspace slots and hand them to
 * m3_command_executor_execute (src/m3_command_executor.c:55-92), which
 * selects the provider; on the CUDA backend every command reaches
 * m3_cuda_backend_execute.  The harness only sets up the minimal flow run
 * those functions read (config, workspace storages, executor). */

#include "m3_flow_internal.h"
#include "m3_provider.h"

#include <string.h>

static m3_status storage_for(m3_backend *backend, size_t bytes,
                             m3_storage **storage, m3_error *error)
{
    return m3_storage_allocate(backend, bytes, 64U, storage, error);
}

/* velocity [2, length, channels] (conditional, then unconditional rows),
 * latent [1, length, channels]; noise_prompt and previous_latent
 * [1, overlap, channels].  Outputs: guided velocity and the latent after
 * the Euler step and the overlap blend.  `cuda` selects the CUDA backend
 * (else the host backend).  Returns the provider of the executor's command
 * lists through `provider` (M3_PROVIDER_*). */
m3_status m3h_flow_solver_math(int cuda, uint64_t length, uint32_t channels,
                               float guidance, float delta, uint64_t overlap,
                               float timestep, const float *velocity,
                               const float *latent, const float *noise_prompt,
                               const float *previous_latent,
                               float *guided_out, float *latent_out,
                               int *provider, m3_error *error)
{
    m3_flow_config config;
    m3_flow_run run;
    m3_storage *slots[M3_FLOW_WORKSPACE_COUNT];
    m3_storage *velocity_storage = NULL;
    m3_storage *latent_storage = NULL;
    m3_backend *backend = NULL;
    m3_tensor_view velocity_view;
    m3_tensor_view latent_view;
    const uint64_t velocity_shape[] = {2U, length, channels};
    const uint64_t latent_shape[] = {1U, length, channels};
    size_t plane = (size_t)length * channels * sizeof(float);
    size_t carry = (size_t)overlap * channels * sizeof(float);
    m3_provider_kind chosen = M3_PROVIDER_CPU;
    m3_command probe;
    m3_status status;
    size_t i;

    memset(slots, 0, sizeof(slots));
    status = cuda ? m3_backend_create_cuda(&backend, error)
                  : m3_backend_create_host(&backend, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    m3_flow_config_init(&config);
    config.latent_channels = channels;
    config.guidance_scale = guidance;
    config.carry_length = (uint32_t)overlap;
    memset(&run, 0, sizeof(run));
    run.backend = backend;
    run.config = &config;
    run.maximum_length = length;
    m3_runtime_workspace_init(&run.workspace);
    run.workspace.backend = backend;
    run.workspace.storages = slots;
    run.workspace.count = M3_FLOW_WORKSPACE_COUNT;
    m3_command_executor_init(&run.executor, backend);

    status = storage_for(backend, plane, &slots[M3_FLOW_WS_SCALAR], error);
    if (status == M3_STATUS_OK) {
        status = storage_for(backend, plane, &slots[M3_FLOW_WS_ARITHMETIC], error);
    }
    if (status == M3_STATUS_OK) {
        status = storage_for(backend, carry, &slots[M3_FLOW_WS_NOISE_PROMPT], error);
    }
    if (status == M3_STATUS_OK) {
        status = storage_for(backend, carry, &slots[M3_FLOW_WS_PREVIOUS_LATENT], error);
    }
    if (status == M3_STATUS_OK) {
        status = storage_for(backend, 2U * plane, &velocity_storage, error);
    }
    if (status == M3_STATUS_OK) {
        status = storage_for(backend, plane, &latent_storage, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_storage_write(velocity_storage, 0U, velocity, 2U * plane, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_storage_write(latent_storage, 0U, latent, plane, error);
    }
    if (status == M3_STATUS_OK && carry != 0U) {
        status = m3_storage_write(slots[M3_FLOW_WS_NOISE_PROMPT], 0U, noise_prompt,
                                  carry, error);
    }
    if (status == M3_STATUS_OK && carry != 0U) {
        status = m3_storage_write(slots[M3_FLOW_WS_PREVIOUS_LATENT], 0U,
                                  previous_latent, carry, error);
    }
    if (status == M3_STATUS_OK) {
        m3_tensor_view_init(&velocity_view);
        status = m3_tensor_view_contiguous(&velocity_view, velocity_storage,
                                           M3_DTYPE_F32, 3U, velocity_shape, 0U,
                                           error);
    }
    if (status == M3_STATUS_OK) {
        m3_tensor_view_init(&latent_view);
        status = m3_tensor_view_contiguous(&latent_view, latent_storage,
                                           M3_DTYPE_F32, 3U, latent_shape, 0U,
                                           error);
    }
    if (status == M3_STATUS_OK) {
        /* where the executor places a MUL of two latent-shaped views */
        memset(&probe, 0, sizeof(probe));
        probe.kind = M3_OP_MUL;
        probe.descriptor.mul.left = &latent_view;
        probe.descriptor.mul.right = &latent_view;
        probe.descriptor.mul.output = &latent_view;
        status = m3_provider_select_regular(backend, true, true, &probe, 1U,
                                            &chosen, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_flow_guided_velocity(&run, &velocity_view, length, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_storage_read(velocity_view.storage, velocity_view.byte_offset,
                                 guided_out, plane, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_flow_euler_step(&run, &latent_view, &velocity_view, length,
                                    delta, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_flow_blend_overlap(&run, &latent_view, length, overlap,
                                       timestep, error);
    }
    if (status == M3_STATUS_OK) {
        status = m3_storage_read(latent_storage, 0U, latent_out, plane, error);
    }
    if (provider != NULL) {
        *provider = (int)chosen;
    }
    m3_command_executor_dispose(&run.executor);
    for (i = 0U; i < M3_FLOW_WORKSPACE_COUNT; ++i) {
        m3_storage_free(slots[i]);
    }
    m3_storage_free(velocity_storage);
    m3_storage_free(latent_storage);
    m3_backend_free(backend);
    return status;
}

/* The flow workspace unit also sizes the condition encoder's workspace
 * (src/m3_condition_validate.c), which the solver arithmetic never reaches;
 * these two entry points stand in for that unit so the harness links
 * without the condition encoder. */
m3_status m3_condition_output_length(uint64_t frames, uint32_t numerator,
                                     uint32_t denominator, uint64_t *length,
                                     m3_error *error)
{
    (void)frames;
    (void)numerator;
    (void)denominator;
    (void)length;
    return m3_error_set(error, M3_STATUS_UNSUPPORTED,
                        "condition encoder is not part of this build");
}

void m3_condition_workspace_specs(const m3_condition_config *config,
                                  uint64_t frames, uint64_t output_length,
                                  m3_runtime_tensor_spec *specs)
{
    (void)config;
    (void)frames;
    (void)output_length;
    (void)specs;
}
