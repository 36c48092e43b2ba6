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
// dependent), so a thread owns a row; rows are independent.  Rows of whole
// 128-byte chunks up to 8 KiB go through categorical_group_kernel (coalesced
// staging, one warp per 32 rows); other shapes read global memory directly.

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

// ------------------------------------------------------- warp row groups
//
// For rows of whole 128-byte chunks (up to 8 KiB), one warp owns 32
// consecutive rows and walks them chunk by chunk: the warp copies the 32
// rows' next chunk into shared memory with coalesced 16-byte cp.async copies
// (double-buffered, so one chunk lands while the previous is summed), and
// lane r runs row r's first pass over it, recording the running sum at the
// end of every chunk.  The second pass repeats the same additions from zero,
// so its cumulative sum at a chunk boundary is that recorded sum: the first
// chunk whose end sum exceeds the target holds the selected index, and only
// that chunk is read again.  Arithmetic, order and checks are those of
// categorical_kernel.

constexpr int GROUP_WARPS = 4;                       // warps per CTA
constexpr int CHUNK_BYTES = 128;                     // per row and step
constexpr int CHUNK_PITCH = CHUNK_BYTES + 16;        // padded shared-memory row
constexpr int MAX_CHUNKS = 64;                       // rows up to 8 KiB

__device__ __forceinline__ void copy16(void *smem_dst, const void *global_src)
{
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(global_src) : "memory");
}

template <int EB>
__device__ __forceinline__ void widen_vector(const uint4 &q, int dtype, float (&x)[16 / EB])
{
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if constexpr (EB == 4) {
#pragma unroll
        for (int t = 0; t < 4; ++t) x[t] = __uint_as_float(w[t]);
    } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) x[t] = widen(dtype, (w[t >> 1] >> ((t & 1) * 16)) & 0xffffu);
    }
}

template <int EB>
__global__ void __launch_bounds__(GROUP_WARPS * 32)
    categorical_group_kernel(const __grid_constant__ m3c_categorical_params p, int chunks)
{
    constexpr int EPV = 16 / EB;                         // elements per 16-byte vector
    constexpr int VPC = CHUNK_BYTES / 16;                // vectors per chunk
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int skip;
    if (threadIdx.x == 0) {
        skip = failed_before(p.status, p.skip_before) ? 1 : 0;
        if (!skip && p.first_of_run && blockIdx.x == 0) atomicAdd(&p.status->runs_started, 1u);
    }
    __syncthreads();
    if (skip) return;
    const int warp = static_cast<int>(threadIdx.x) / 32;
    const int lane = static_cast<int>(threadIdx.x) % 32;
    const uint64_t row0 = (static_cast<uint64_t>(blockIdx.x) * GROUP_WARPS + warp) * 32u;
    if (row0 >= p.rows) return;
    const int live = static_cast<int>(p.rows - row0 < 32u ? p.rows - row0 : 32u);
    // this warp's two chunk buffers and its recorded chunk-end sums
    unsigned char *buffer = smem + warp * (2 * 32 * CHUNK_PITCH + 32 * MAX_CHUNKS * 4);
    float *ends = reinterpret_cast<float *>(buffer + 2 * 32 * CHUNK_PITCH) + lane * MAX_CHUNKS;
    const unsigned char *rows = static_cast<const unsigned char *>(p.probabilities) +
                                row0 * static_cast<uint64_t>(chunks) * CHUNK_BYTES;
    const uint64_t row_bytes = static_cast<uint64_t>(chunks) * CHUNK_BYTES;
    // the warp's copies of chunk c: 32 rows x 8 vectors, 8 per lane
    auto copy_chunk = [&](int c) {
        unsigned char *dst = buffer + (c & 1) * 32 * CHUNK_PITCH;
#pragma unroll
        for (int k = 0; k < 32 * VPC / 32; ++k) {
            const int piece = lane + 32 * k;
            const int r = piece / VPC;
            const int v = piece % VPC;
            if (r < live) copy16(dst + r * CHUNK_PITCH + v * 16, rows + r * row_bytes + c * CHUNK_BYTES + v * 16);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const uint64_t row = row0 + lane;
    const bool mine = lane < live;
    const float uniform = mine ? load_float(p.uniforms, p.uniforms_dtype, row) : 0.0f;
    uint32_t reason = 0u;
    if (mine && !(isfinite(uniform) && uniform >= 0.0f && uniform < 1.0f)) {
        reason = 1u;  // "categorical uniform is outside [0,1)"
    }
    float sum = 0.0f;
    uint64_t last_positive = 0u;
    copy_chunk(0);
    for (int c = 0; c < chunks; ++c) {
        if (c + 1 < chunks) {
            copy_chunk(c + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncwarp();
        if (mine && reason == 0u) {
            const uint4 *v4 = reinterpret_cast<const uint4 *>(buffer + (c & 1) * 32 * CHUNK_PITCH + lane * CHUNK_PITCH);
            uint4 next = v4[0];
#pragma unroll
            for (int v = 0; v < VPC; ++v) {
                const uint4 cur = next;
                if (v + 1 < VPC) next = v4[v + 1];
                float x[EPV];
                widen_vector<EB>(cur, p.probabilities_dtype, x);
#pragma unroll
                for (int t = 0; t < EPV; ++t) {
                    if (reason == 0u) {
                        if (!isfinite(x[t]) || x[t] < 0.0f) {
                            reason = 2u;  // "categorical probability is invalid"
                        } else {
                            sum = __fadd_rn(sum, x[t]);
                            if (x[t] > 0.0f) {
                                last_positive = static_cast<uint64_t>(c) * (CHUNK_BYTES / EB) + v * EPV + t;
                            }
                        }
                    }
                }
            }
            ends[c] = sum;
        }
        __syncwarp();  // the buffer is refilled two chunks on
    }
    if (!mine) return;
    if (reason == 0u && !(isfinite(sum) && sum > 0.0f)) {
        reason = 3u;  // "categorical row sum is not positive finite"
    }
    if (reason != 0u) {
        const uint64_t key = (row < 0x3fffffffull ? row : 0x3fffffffull) * 4u + reason;
        atomicMin(&p.status->detail, static_cast<uint32_t>(key));
        record_failure(p.status, p.command);
        return;
    }
    if (p.check_only) return;
    const float target = __fmul_rn(uniform, sum);
    int chunk = -1;
    for (int c = 0; c < chunks && chunk < 0; ++c) {
        if (target < ends[c]) chunk = c;
    }
    uint64_t selected = last_positive;
    if (chunk >= 0) {
        float cumulative = chunk == 0 ? 0.0f : ends[chunk - 1];
        const uint4 *v4 = reinterpret_cast<const uint4 *>(rows + lane * row_bytes + chunk * CHUNK_BYTES);
        bool found = false;
        for (int v = 0; v < VPC && !found; ++v) {
            float x[EPV];
            widen_vector<EB>(v4[v], p.probabilities_dtype, x);
#pragma unroll
            for (int t = 0; t < EPV; ++t) {
                if (!found) {
                    cumulative = __fadd_rn(cumulative, x[t]);
                    if (target < cumulative) {
                        selected = static_cast<uint64_t>(chunk) * (CHUNK_BYTES / EB) + v * EPV + t;
                        found = true;
                    }
                }
            }
        }
    }
    p.output[row] = static_cast<int32_t>(selected);
}

}  // namespace
}  // namespace m3c

extern "C" int m3c_launch_categorical(const m3c_categorical_params *params, void *stream)
{
    const int eb = params->probabilities_dtype == M3C_F16 || params->probabilities_dtype == M3C_BF16 ? 2 : 4;
    const uint64_t row_bytes = params->width * static_cast<uint64_t>(eb);
    if (params->rows != 0 && row_bytes != 0 && row_bytes % m3c::CHUNK_BYTES == 0 &&
        row_bytes / m3c::CHUNK_BYTES <= static_cast<uint64_t>(m3c::MAX_CHUNKS) &&
        reinterpret_cast<uintptr_t>(params->probabilities) % 16u == 0u) {
        const int chunks = static_cast<int>(row_bytes / m3c::CHUNK_BYTES);
        const size_t per_warp = 2u * 32u * m3c::CHUNK_PITCH + 32u * m3c::MAX_CHUNKS * 4u;
        const size_t smem = per_warp * m3c::GROUP_WARPS;
        void (*kernel)(m3c_categorical_params, int) =
            eb == 4 ? m3c::categorical_group_kernel<4> : m3c::categorical_group_kernel<2>;
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        const uint64_t warps = (params->rows + 31u) / 32u;
        const unsigned grid = static_cast<unsigned>((warps + m3c::GROUP_WARPS - 1) / m3c::GROUP_WARPS);
        kernel<<<grid, m3c::GROUP_WARPS * 32, smem, static_cast<cudaStream_t>(stream)>>>(*params, chunks);
        return static_cast<int>(cudaGetLastError());
    }
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
