// m3_cuda_abs_max_static: ABS_MAX over a batch of device tensors with no
// allocation of any kind.  The reduction scratch and the status words that the
// element-wise kernel needs live in a fixed array of this library's device
// code instead of in cudaMalloc'd memory; the kernel and its ABS_MAX program
// are the ones the session and the backend plug-in launch.
//
// Callers that cannot allocate: a real-time audio render thread (cudaMalloc
// and cudaFree take driver locks, and cudaFree waits for the device to go
// idle, so neither has a latency bound), and a caller that has already split
// all device memory among its own pools.

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>

extern "C" {
#include "m3c_internal.h"
}

namespace {

constexpr size_t kSlots = M3_CUDA_ABS_MAX_STATIC_MAX_TENSORS;
constexpr size_t kStatusWords = sizeof(m3c_status) / sizeof(uint32_t);
constexpr size_t kReduceWords = sizeof(m3c_reduce_scratch) / sizeof(uint32_t);
constexpr int kMaxDevices = 64;

static_assert(sizeof(m3c_status) == 16, "status is four 32-bit words");
static_assert(sizeof(m3c_reduce_scratch) == 8, "reduction slot is two 32-bit words");

// Slot i's status words sit at word kStatusWords * i, its reduction words
// (running max, finished-CTA count) at kStatusWords * kSlots + kReduceWords * i:
// 1536 bytes per device.  Zero-filled when the module loads; every call resets
// the slots it uses before its kernels run.
static __device__ __align__(256) uint32_t abs_max_scratch[(kStatusWords + kReduceWords) * kSlots];

// Device address of abs_max_scratch per device, looked up on first use.
std::atomic<uint32_t *> scratch_by_device[kMaxDevices];

m3_status fail(m3_error *error, cudaError_t code, const char *what)
{
    (void)cudaGetLastError();
    return m3c_error_set(error, M3_STATUS_INTERNAL, "%s: %s", what, cudaGetErrorString(code));
}

// The scratch address on `device`, which the caller has made current.
cudaError_t scratch_on(int device, uint32_t **words)
{
    uint32_t *known = scratch_by_device[device].load(std::memory_order_acquire);
    if (known == nullptr) {
        void *address = nullptr;
        const cudaError_t code = cudaGetSymbolAddress(&address, abs_max_scratch);
        if (code != cudaSuccess) {
            return code;
        }
        known = static_cast<uint32_t *>(address);
        scratch_by_device[device].store(known, std::memory_order_release);
    }
    *words = known;
    return cudaSuccess;
}

// The ABS_MAX launch of one dense tensor, built the way the backend plug-in
// builds a single ABS_MAX command: widen 16-bit input to F32 in register 2,
// then fold |x| into the reduction; command index 0.
int launch_one(const void *input, m3_dtype dtype, uint64_t count, float *result, m3c_status *status,
               m3c_reduce_scratch *reduce, cudaStream_t stream)
{
    m3_tensor_metadata metadata;
    m3_error ignored;
    if (m3c_metadata_init(&metadata, dtype, 1U, &count, &ignored) != M3_STATUS_OK) {
        return static_cast<int>(cudaErrorInvalidValue);
    }
    const size_t stride = m3c_dtype_size(dtype);
    m3c_ew_params p;
    std::memset(&p, 0, sizeof(p));
    p.count = count;
    p.status = status;
    p.skip_before = 0U;
    p.first_of_run = 0;
    p.n_operands = 1;
    m3c_operand_setup(&p.operands[0], input, &metadata, 0U, &stride, &metadata, M3C_LOAD_RAW);
    int reg = 0;
    if (dtype == M3_DTYPE_F16 || dtype == M3_DTYPE_BF16) {
        m3c_ew_op *op = &p.ops[p.n_ops++];
        op->code = M3C_OP_WIDEN;
        op->dst = 2U;
        op->a = 0U;
        op->b = 0U;
        op->rdtype = M3C_F32;
        op->aux = static_cast<int8_t>(dtype);
        op->command = 0U;
        reg = 2;
    }
    m3c_ew_op *op = &p.ops[p.n_ops++];
    op->code = M3C_OP_ABSMAX;
    op->a = static_cast<uint8_t>(reg);
    op->b = static_cast<uint8_t>(reg);
    op->dst = static_cast<uint8_t>(reg);
    op->rdtype = M3C_F32;
    op->aux = 0;
    op->command = 0U;
    p.reduce = reduce;
    p.absmax_out = result;
    p.absmax_command = 0U;
    return m3c_launch_ew(&p, stream);
}

}  // namespace

extern "C" m3_status m3_cuda_abs_max_static(int device, void *stream, m3_dtype dtype,
                                            const void *const *inputs, const uint64_t *element_counts,
                                            size_t tensor_count, float *maxima, m3_error *error)
{
    if (tensor_count > kSlots) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "abs-max batch of %zu tensors exceeds the static scratch limit of %zu "
                             "tensors per call",
                             tensor_count, kSlots);
    }
    if (tensor_count == 0U) {
        m3_error_reset(error);
        return M3_STATUS_OK;
    }
    if (inputs == nullptr || element_counts == nullptr || maxima == nullptr) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "abs-max inputs, element counts and maxima are required");
    }
    if (dtype != M3_DTYPE_F32 && dtype != M3_DTYPE_F16 && dtype != M3_DTYPE_BF16) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "abs-max input must be F32, F16 or BF16");
    }
    if ((reinterpret_cast<uintptr_t>(maxima) & 3U) != 0U) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT, "abs-max maxima must be 4-byte aligned");
    }
    const size_t element = m3c_dtype_size(dtype);
    for (size_t i = 0; i < tensor_count; ++i) {
        if (element_counts[i] != 0U && inputs[i] == nullptr) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT, "abs-max input %zu is null", i);
        }
        if ((reinterpret_cast<uintptr_t>(inputs[i]) % element) != 0U) {
            return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                                 "abs-max input %zu is not aligned to its element size", i);
        }
        if (element_counts[i] > UINT64_MAX / element) {
            return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE, "abs-max input %zu is too large", i);
        }
    }
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices == 0) {
        (void)cudaGetLastError();
        return m3c_error_set(error, M3_STATUS_UNSUPPORTED, "no CUDA device is available");
    }
    if (device < 0 || device >= devices || device >= kMaxDevices) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT, "CUDA device %d is not available", device);
    }
    int previous = 0;
    cudaError_t code = cudaGetDevice(&previous);
    if (code != cudaSuccess) {
        return fail(error, code, "cannot read the current CUDA device");
    }
    code = cudaSetDevice(device);
    if (code != cudaSuccess) {
        return fail(error, code, "cannot select the CUDA device");
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t *words = nullptr;
    code = scratch_on(device, &words);
    if (code != cudaSuccess) {
        (void)cudaSetDevice(previous);
        return fail(error, code, "cannot locate the static abs-max scratch");
    }
    m3c_status *status = reinterpret_cast<m3c_status *>(words);
    m3c_reduce_scratch *reduce = reinterpret_cast<m3c_reduce_scratch *>(words + kStatusWords * kSlots);

    // status words to "no failure" (all ones) with no run counted yet (the
    // run counter word zero: its top bit would halt the kernel), reduction
    // slots to zero
    code = cudaMemsetAsync(status, 0xff, tensor_count * sizeof(m3c_status), s);
    if (code == cudaSuccess) {
        code = cudaMemset2DAsync(&status[0].runs_started, sizeof(m3c_status), 0, sizeof(uint32_t),
                                 tensor_count, s);
    }
    if (code == cudaSuccess) {
        code = cudaMemsetAsync(reduce, 0, tensor_count * sizeof(m3c_reduce_scratch), s);
    }
    int launch = 0;
    size_t i = 0;
    for (; code == cudaSuccess && launch == 0 && i < tensor_count; ++i) {
        launch = launch_one(inputs[i], dtype, element_counts[i], maxima + i, &status[i], &reduce[i], s);
    }
    m3c_status seen[kSlots];
    if (code == cudaSuccess) {
        code = cudaMemcpyAsync(seen, status, tensor_count * sizeof(m3c_status), cudaMemcpyDeviceToHost, s);
    }
    const cudaError_t waited = cudaStreamSynchronize(s);
    (void)cudaSetDevice(previous);
    if (code != cudaSuccess) {
        return fail(error, code, "abs-max scratch reset or status read failed");
    }
    if (launch != 0) {
        (void)cudaGetLastError();
        return m3c_error_set(error, M3_STATUS_INTERNAL, "abs-max launch for input %zu failed: %s", i - 1U,
                             m3c_cuda_error_string(launch));
    }
    if (waited != cudaSuccess) {
        return fail(error, waited, "abs-max execution failed");
    }
    for (size_t t = 0; t < tensor_count; ++t) {
        if (seen[t].fail_command != UINT32_MAX) {
            return m3c_error_set(error, M3_STATUS_OUT_OF_RANGE, "abs-max input %zu contains NaN", t);
        }
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}
