/* Test infrastructure only (oracle build).
 *
 * The reference's provider scheduler links against two Apple-only providers:
 * m3_backend_create_metal (reference src/m3_provider.c:51, defined in
 * src/m3_backend_metal.m) and the Core ML partition entry points (reference
 * src/m3_graph_internal.h:89-96, defined in src/m3_coreml.m).  Neither exists
 * on Linux.  These stubs report them as unsupported, which is exactly what the
 * reference's own tests expect on a machine without the device: sessions then
 * place every regular node on the CPU provider. */

#include "m3_backend.h"
#include "m3_graph_internal.h"

m3_status m3_backend_create_metal(m3_backend **backend, m3_error *error)
{
    if (backend != NULL) {
        *backend = NULL;
    }
    return m3_error_set(error, M3_STATUS_UNSUPPORTED,
                        "Metal is not available on this host");
}

m3_status m3_coreml_partition_create(
    const m3_graph_coreml *description, const m3_tensor_view *views,
    size_t value_count, m3_coreml_partition **partition, m3_error *error)
{
    (void)description;
    (void)views;
    (void)value_count;
    if (partition != NULL) {
        *partition = NULL;
    }
    return m3_error_set(error, M3_STATUS_UNSUPPORTED,
                        "Core ML is not available on this host");
}

void m3_coreml_partition_free(m3_coreml_partition *partition)
{
    (void)partition;
}

m3_status m3_coreml_partition_execute(
    m3_coreml_partition *partition, m3_tensor_view *views,
    size_t value_count, m3_error *error)
{
    (void)partition;
    (void)views;
    (void)value_count;
    return m3_error_set(error, M3_STATUS_UNSUPPORTED,
                        "Core ML is not available on this host");
}
