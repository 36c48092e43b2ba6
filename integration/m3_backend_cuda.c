/* The file a maintainer adds to the reference tree (src/m3_backend_cuda.c)
 * to register libm3cuda.so as one more provider of the reference's backend
 * layer, next to the host and Metal backends (src/m3_backend_host.c,
 * src/m3_backend_metal.m).  cuda_provider.patch adds the rest: the
 * M3_BACKEND_CUDA kind and these two declarations (src/m3_backend.h), the
 * optional storage I/O hooks of the vtable (src/m3_backend_internal.h) that
 * m3_storage_write/read call for storage the host cannot address
 * (src/m3_backend.c), and the CUDA branches of backend creation, placement
 * and execution (src/m3_provider.c).
 *
 * Storage modes.  Managed (the default): storages are cudaMallocManaged,
 * info.unified_memory is true, and every host touch the reference makes on a
 * storage (memcpy in m3_storage_write/read, the flow solver's scalar fills,
 * waveform assembly) works unchanged; command lists the GPU does not
 * implement may still fall back to the CPU provider.  Device: storages are
 * cudaMalloc, info.unified_memory is false, storage I/O goes through the
 * vtable hooks, and a command list must run on the GPU entirely. */

#include "m3_backend_internal.h"
#include "m3_cuda.h"

#include <stdint.h>
#include <stdio.h>
#include <string.h>

static int cuda_device = 0;
static bool cuda_managed = true;

void m3_backend_cuda_configure(int device, bool managed_memory)
{
    cuda_device = device < 0 ? 0 : device;
    cuda_managed = managed_memory;
}

static const m3_backend_vtable cuda_vtable = {
    .destroy_context = m3_cuda_backend_destroy_context,
    .allocate = m3_cuda_backend_allocate,
    .free_storage = m3_cuda_backend_free_storage,
    .execute = m3_cuda_backend_execute,
    .write = m3_cuda_backend_write,
    .read = m3_cuda_backend_read,
};

m3_status m3_backend_create_cuda(m3_backend **backend, m3_error *error)
{
    m3_cuda_backend_options options;
    m3_backend_info info;
    void *context = NULL;
    m3_status status;

    if (backend == NULL) {
        return m3_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                            "CUDA backend output is null");
    }
    *backend = NULL;
    memset(&options, 0, sizeof(options));
    options.device = cuda_device;
    options.storage_data = m3_storage_data;
    options.managed_memory = cuda_managed;
    /* M3_STATUS_UNSUPPORTED without a device: the caller tries the next
     * provider, as it does when Metal is absent */
    status = m3_cuda_backend_context_create(&options, &context, error);
    if (status != M3_STATUS_OK) {
        return status;
    }
    memset(&info, 0, sizeof(info));
    (void)snprintf(info.name, sizeof(info.name), "CUDA %s storage, device %d",
                   cuda_managed ? "managed" : "device", cuda_device);
    info.kind = M3_BACKEND_CUDA;
    info.unified_memory = cuda_managed;
    info.recommended_working_set_bytes = 0U;
    info.maximum_storage_bytes = UINT64_MAX;
    status = m3_backend_create_internal(&cuda_vtable, context, &info, backend,
                                        error);
    if (status != M3_STATUS_OK) {
        m3_cuda_backend_destroy_context(context);
    }
    return status;
}
