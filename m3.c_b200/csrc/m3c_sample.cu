// Categorical sampling (sm_100a): one index per row drawn from that row's
// probabilities with one uniform number, exactly as the reference's CPU
// executor picks it (src/m3_op_execute_sampling.c:90-137): the row sum and
// the last positive index in one left-to-right F32 pass, the target
// uniform * sum, then the first index whose left-to-right cumulative sum
// exceeds the target (the last positive index when rounding leaves none).
//
// The data checks of the reference's preflight
// (src/m3_op_data_preflight.c:231-268) run in the same pass: a uniform
// outside [0, 1), a negative or non-finite probability, or a row sum that is
// not positive and finite fails the command.  The status word keeps the
// smallest failing row * 4 + reason, so the host reports the check the
// reference's row-ordered preflight would have reported first.
//
// Both passes are inherently sequential per row (the sums are order
// dependent), so a thread owns a row; rows are independent.

#include <cuda_runtime.h>

#include <cstdint>

#include "m3c_device.cuh"
#include "m3c_kernels.h"

namespace m3c {
namespace {

constexpr int SAMPLE_THREADS = 256;

__device__ __forceinline__ float load_float(const void *base, int dtype, uint64_t i)
{
    if (dtype == M3C_F16 || dtype == M3C_BF16) {
        return widen(dtype, static_cast<const uint16_t *>(base)[i]);
    }
    return static_cast<const float *>(base)[i];
}

__global__ void __launch_bounds__(SAMPLE_THREADS)
    categorical_kernel(const __grid_constant__ m3c_categorical_params p)
{
    if (failed_before(p.status, p.skip_before)) {
        return;
    }
    if (p.first_of_run && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(&p.status->runs_started, 1u);
    }
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t row = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; row < p.rows;
         row += stride) {
        const float uniform = load_float(p.uniforms, p.uniforms_dtype, row);
        const uint64_t base = row * p.width;
        uint32_t reason = 0u;
        float sum = 0.0f;
        uint64_t last_positive = 0u;
        if (!(isfinite(uniform) && uniform >= 0.0f && uniform < 1.0f)) {
            reason = 1u;  // "categorical uniform is outside [0,1)"
        } else {
            for (uint64_t j = 0; j < p.width; ++j) {
                const float probability = load_float(p.probabilities, p.probabilities_dtype, base + j);
                if (!isfinite(probability) || probability < 0.0f) {
                    reason = 2u;  // "categorical probability is invalid"
                    break;
                }
                sum = __fadd_rn(sum, probability);
                if (probability > 0.0f) {
                    last_positive = j;
                }
            }
            if (reason == 0u && !(isfinite(sum) && sum > 0.0f)) {
                reason = 3u;  // "categorical row sum is not positive finite"
            }
        }
        if (reason != 0u) {
            const uint64_t key = (row < 0x3fffffffull ? row : 0x3fffffffull) * 4u + reason;
            atomicMin(&p.status->detail, static_cast<uint32_t>(key));
            record_failure(p.status, p.command);
            continue;
        }
        if (p.check_only) {
            continue;
        }
        const float target = __fmul_rn(uniform, sum);
        uint64_t selected = last_positive;
        float cumulative = 0.0f;
        for (uint64_t j = 0; j < p.width; ++j) {
            cumulative = __fadd_rn(cumulative, load_float(p.probabilities, p.probabilities_dtype, base + j));
            if (target < cumulative) {
                selected = j;
                break;
            }
        }
        p.output[row] = static_cast<int32_t>(selected);
    }
}

}  // namespace
}  // namespace m3c

extern "C" int m3c_launch_categorical(const m3c_categorical_params *params, void *stream)
{
    int device = 0;
    int sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    }
    const uint64_t needed = (params->rows + m3c::SAMPLE_THREADS - 1) / m3c::SAMPLE_THREADS;
    const uint64_t cap = static_cast<uint64_t>(sms) * 8u;
    // at least one CTA: an empty launch still records the start of the run
    const unsigned grid = static_cast<unsigned>(needed == 0 ? 1 : (needed < cap ? needed : cap));
    m3c::categorical_kernel<<<grid, m3c::SAMPLE_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(*params);
    return static_cast<int>(cudaGetLastError());
}
