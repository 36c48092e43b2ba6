// Utility kernels: seeded input generation and the standalone data scans used
// by the backend plug-in path (where outputs cannot be double-buffered).

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <cstdio>

#include "m3_cuda.h"
#include "m3c_device.cuh"
#include "m3c_kernels.h"

namespace m3c {
namespace {

constexpr uint64_t PCG_MULTIPLIER = 6364136223846793005ull;

struct Pcg {
    uint64_t state;
    uint64_t increment;
};

// PCG32 XSH-RR output of the reference (src/m3_rng.c:9-20).
__device__ __forceinline__ uint32_t pcg_next(Pcg &rng)
{
    const uint64_t old = rng.state;
    rng.state = old * PCG_MULTIPLIER + rng.increment;
    const uint32_t shifted = static_cast<uint32_t>(((old >> 18u) ^ old) >> 27u);
    const uint32_t rotation = static_cast<uint32_t>(old >> 59u);
    return (shifted >> rotation) | (shifted << ((0u - rotation) & 31u));
}

// Seeding of src/m3_rng.c:22-39.
__device__ __forceinline__ Pcg pcg_seed(uint64_t seed, uint64_t sequence)
{
    Pcg rng{0u, (sequence << 1u) | 1u};
    (void)pcg_next(rng);
    rng.state += seed;
    (void)pcg_next(rng);
    return rng;
}

// Advance an LCG by `delta` steps in O(log delta) (F. Brown, "Random number
// generation with arbitrary strides", Trans. Am. Nucl. Soc. 71, 1994).
__device__ __forceinline__ void pcg_advance(Pcg &rng, uint64_t delta)
{
    uint64_t acc_mult = 1u;
    uint64_t acc_plus = 0u;
    uint64_t cur_mult = PCG_MULTIPLIER;
    uint64_t cur_plus = rng.increment;
    while (delta > 0u) {
        if (delta & 1u) {
            acc_mult *= cur_mult;
            acc_plus = acc_plus * cur_mult + cur_plus;
        }
        cur_plus = (cur_mult + 1u) * cur_plus;
        cur_mult *= cur_mult;
        delta >>= 1u;
    }
    rng.state = acc_mult * rng.state + acc_plus;
}

constexpr uint64_t CHUNK = 1024;  // values per thread

__global__ void uniform_kernel(uint64_t seed, uint64_t sequence, float low, float high, float *out,
                               uint64_t count)
{
    const uint64_t first = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * CHUNK;
    if (first >= count) return;
    Pcg rng = pcg_seed(seed, sequence);
    pcg_advance(rng, first);
    const float span = __fsub_rn(high, low);
    const uint64_t end = first + CHUNK < count ? first + CHUNK : count;
    for (uint64_t i = first; i < end; ++i) {
        // src/m3_rng.c:53-66, then scaled: low + (high - low) * u
        const float u = __fmul_rn(__uint2float_rn(pcg_next(rng) >> 8u), 0x1p-24f);
        out[i] = __fadd_rn(low, __fmul_rn(span, u));
    }
}

__global__ void normal_kernel(uint64_t seed, uint64_t sequence, float mean, float deviation,
                              float *out, uint64_t count)
{
    // values come in pairs from two draws; CHUNK is even so pairs never split
    const uint64_t first = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * CHUNK;
    if (first >= count) return;
    Pcg rng = pcg_seed(seed, sequence);
    pcg_advance(rng, first);
    const uint64_t end = first + CHUNK < count ? first + CHUNK : count;
    for (uint64_t i = first; i < end; i += 2) {
        // Box-Muller in double, src/m3_rng.c:68-110
        const double radius_u = (static_cast<double>(pcg_next(rng)) + 0.5) * 0x1p-32;
        const double angle_u = static_cast<double>(pcg_next(rng)) * 0x1p-32;
        const double radius = sqrt(-2.0 * log(radius_u));
        const double angle = 6.283185307179586476925286766559 * angle_u;
        const float z0 = static_cast<float>(radius * cos(angle));
        const float z1 = static_cast<float>(radius * sin(angle));
        out[i] = __fadd_rn(mean, __fmul_rn(deviation, z0));
        if (i + 1 < end) out[i + 1] = __fadd_rn(mean, __fmul_rn(deviation, z1));
    }
}

// Whole-tensor data check for one command: NaN (mode 0) or a value that is
// not a valid float-to-I32 cast source (mode 1).  Contiguous input.
__global__ void scan_kernel(const void *data, int dtype, uint64_t count, int mode, uint32_t command,
                            m3c_status *status)
{
    bool bad = false;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += stride) {
        float v;
        if (dtype == M3C_F16 || dtype == M3C_BF16) {
            v = widen(dtype, static_cast<const uint16_t *>(data)[i]);
        } else {
            v = as_float(static_cast<const uint32_t *>(data)[i]);
        }
        bad |= mode == 0 ? (v != v) : !(v >= -2147483648.0f && v < 2147483648.0f);
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31u) == 0u) {
        record_failure(status, command);
    }
}

// The data checks of a row operator's input, one warp per row, 16-byte loads.
// Rows are visited in the reverse of the order in which the row kernel that
// follows reads them (it reads `ranges` contiguous row ranges side by side,
// from their starts), so the rows it reads first are the ones still in L2.
__device__ __forceinline__ bool vector_fails(const uint4 &q, int dtype, int mode)
{
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if (mode == 0) {
        if (dtype == M3C_F32) {
            bool nan = false;
#pragma unroll
            for (int t = 0; t < 4; ++t) nan |= (w[t] & 0x7fffffffu) > 0x7f800000u;
            return nan;
        }
        // a 16-bit magnitude m is a NaN when m + (0x3ff or 0x7f) carries
        // into bit 15
        const uint32_t add = dtype == M3C_F16 ? 0x03ff03ffu : 0x007f007fu;
        uint32_t acc = 0u;
#pragma unroll
        for (int t = 0; t < 4; ++t) acc |= (w[t] & 0x7fff7fffu) + add;
        return (acc & 0x80008000u) != 0u;
    }
    bool bad = false;
    if (dtype == M3C_F32) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float v = as_float(w[t]);
            bad |= !(v >= -2147483648.0f && v < 2147483648.0f);
        }
    } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const float v = widen(dtype, (w[t >> 1] >> ((t & 1) * 16)) & 0xffffu);
            bad |= !(v >= -2147483648.0f && v < 2147483648.0f);
        }
    }
    return bad;
}

__global__ void row_scan_kernel(const uint4 *data, int dtype, uint64_t rows, uint32_t nvec, uint32_t ranges,
                                int mode, uint32_t command, m3c_status *status)
{
    const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x / 32);
    const uint64_t first = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = static_cast<int>(threadIdx.x % 32);
    const uint64_t longest = (rows + ranges - 1) / ranges;
    const uint64_t visits = longest * ranges;
    bool bad = false;
    for (uint64_t j = first; j < visits; j += warps) {
        const uint64_t offset = longest - 1 - j / ranges;   // within a range, last first
        const uint64_t range = j % ranges;
        const uint64_t begin = rows * range / ranges;
        const uint64_t end = rows * (range + 1) / ranges;
        const uint64_t row = begin + offset;
        if (row >= end) continue;
        const uint4 *r = data + row * nvec;
        for (uint32_t v = static_cast<uint32_t>(lane); v < nvec; v += 4u * 32u) {
            uint4 q[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t e = v + static_cast<uint32_t>(k) * 32u;
                q[k] = e < nvec ? __ldcg(r + e) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) bad |= vector_fails(q[k], dtype, mode);
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) {
        record_failure(status, command);
    }
}

// Exhaustive agreement of the hardware-assisted codecs with the integer
// restatement of the reference's encoders: every F32 bit pattern through
// both F16 and BF16 narrowing, every F16 pattern through widening; and the
// vector codecs on eight-value vectors built around every F32 pattern (so
// both their NaN-free fast path and their NaN path are exercised).
__global__ void codec_check_kernel(unsigned long long *mismatches)
{
    unsigned long long local = 0;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (1ull << 32);
         i += stride) {
        const float v = as_float(static_cast<uint32_t>(i));
        local += f32_to_f16_fast(v) != f32_to_f16(v) ? 1u : 0u;
        local += f32_to_bf16_fast(v) != f32_to_bf16(v) ? 1u : 0u;
        local += as_bits(round_to(M3C_F16, v)) != as_bits(f16_to_f32(f32_to_f16(v))) ? 1u : 0u;
        local += as_bits(round_to(M3C_BF16, v)) != as_bits(bf16_to_f32(f32_to_bf16(v))) ? 1u : 0u;
        if (i < 65536u) {
            local += as_bits(f16_to_f32_fast(static_cast<uint32_t>(i))) !=
                             as_bits(f16_to_f32(static_cast<uint32_t>(i)))
                         ? 1u
                         : 0u;
        }
        {
            // vector codecs: eight values around this pattern (a NaN in any
            // lane sends the whole vector to the exact path)
            const uint32_t b = static_cast<uint32_t>(i);
            const uint32_t h = b * 2654435761u;
            float x[8] = {v, as_float(b ^ 0x80000000u), as_float(b + 1u), as_float(h),
                          as_float(h ^ 0x00400000u), as_float(b >> 3), as_float(~b), as_float(b << 7)};
            uint32_t w16[4];
            uint32_t wb[4];
            narrow_pairs<4>(M3C_F16, x, w16);
            narrow_pairs<4>(M3C_BF16, x, wb);
            float r16[8];
            float rb[8];
            for (int t = 0; t < 8; ++t) {
                r16[t] = x[t];
                rb[t] = x[t];
            }
            round_values<8>(M3C_F16, r16);
            round_values<8>(M3C_BF16, rb);
            for (int t = 0; t < 8; ++t) {
                const uint32_t e16 = (w16[t >> 1] >> ((t & 1) * 16)) & 0xffffu;
                const uint32_t eb = (wb[t >> 1] >> ((t & 1) * 16)) & 0xffffu;
                local += e16 != f32_to_f16(x[t]) ? 1u : 0u;
                local += eb != f32_to_bf16(x[t]) ? 1u : 0u;
                local += as_bits(r16[t]) != as_bits(f16_to_f32(f32_to_f16(x[t]))) ? 1u : 0u;
                local += as_bits(rb[t]) != as_bits(bf16_to_f32(f32_to_bf16(x[t]))) ? 1u : 0u;
            }
            const uint32_t pw[4] = {b, h, b ^ 0x7c007c00u, ~h};
            float wide16[8];
            float wideb[8];
            widen_pairs<4>(M3C_F16, pw, wide16);
            widen_pairs<4>(M3C_BF16, pw, wideb);
            for (int t = 0; t < 8; ++t) {
                const uint32_t e = (pw[t >> 1] >> ((t & 1) * 16)) & 0xffffu;
                local += as_bits(wide16[t]) != as_bits(f16_to_f32(e)) ? 1u : 0u;
                local += as_bits(wideb[t]) != as_bits(bf16_to_f32(e)) ? 1u : 0u;
            }
        }
    }
    if (local != 0) atomicAdd(mismatches, local);
}

// Markstein quotients against __fdiv_rn on the softmax domain: numerators
// e in [2^-100, 1] (exponentials of non-positive arguments), denominators
// s in [1, 2^24] (a sum whose largest term is 1).  Pairs come from a
// splitmix64 stream; every exponent of both ranges is covered.
__global__ void division_check_kernel(uint64_t samples, unsigned long long *mismatches)
{
    unsigned long long local = 0;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < samples;
         i += stride) {
        uint64_t z = (i + 1) * 0x9e3779b97f4a7c15ull;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        z ^= z >> 31;
        const uint32_t lo = static_cast<uint32_t>(z);
        const uint32_t hi = static_cast<uint32_t>(z >> 32);
        // e: exponent in [-100, -1] or exactly 1.0; s: exponent in [0, 23]
        const uint32_t e_exp = 127u - 100u + (lo >> 23) % 100u;
        float e = as_float((e_exp << 23) | (lo & 0x7fffffu));
        if ((lo & 0xffffu) == 0u) e = 1.0f;
        const uint32_t s_exp = 127u + (hi >> 23) % 24u;
        const float s = as_float((s_exp << 23) | (hi & 0x7fffffu));
        const float y = __frcp_rn(s);
        local += as_bits(div_markstein(e, s, y)) != as_bits(__fdiv_rn(e, s)) ? 1u : 0u;
    }
    if (local != 0) atomicAdd(mismatches, local);
}

// exp_moderate against the correctly rounded e^d (the double-precision exp
// rounded to F32) for every F32 argument d in [-87, 87]: the largest distance
// in ulps, and the count of wrong special values (e^+-0 must be exactly 1).
__global__ void exp_check_kernel(unsigned int *worst, unsigned long long *violations)
{
    constexpr uint32_t last = 0x42ae0000u;  // |87.0|
    unsigned int local = 0u;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i <= last; i += stride) {
#pragma unroll
        for (int sign = 0; sign < 2; ++sign) {
            const float d = as_float((sign ? 0x80000000u : 0u) | i);
            const float got = exp_moderate(d);
            const float want = __double2float_rn(exp(static_cast<double>(d)));
            const int32_t distance = static_cast<int32_t>(as_bits(got)) - static_cast<int32_t>(as_bits(want));
            const unsigned int ulps = static_cast<unsigned int>(distance < 0 ? -distance : distance);
            local = ulps > local ? ulps : local;
        }
    }
    atomicMax(worst, local);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const bool ok = exp_moderate(0.0f) == 1.0f && exp_moderate(-0.0f) == 1.0f;
        if (!ok) atomicAdd(violations, 1ull);
    }
}

// sin_squared against sin(t)^2 in double precision for every F32 argument t
// in [-8192, 8192]: the largest absolute error (as F32 bits of a
// non-negative float, so integer maxima order them) and the largest distance
// in ulps of RN(sin(t)^2) where that is at least 2^-10.
__global__ void sin_squared_check_kernel(unsigned int *worst_abs_bits, unsigned int *worst_ulps)
{
    constexpr uint32_t last = 0x46000000u;  // |8192.0|
    unsigned int abs_bits = 0u;
    unsigned int ulps = 0u;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i <= last; i += stride) {
#pragma unroll
        for (int sign = 0; sign < 2; ++sign) {
            const float t = as_float((sign ? 0x80000000u : 0u) | i);
            const float got = sin_squared(t);
            const double sine = sin(static_cast<double>(t));
            const double exact = sine * sine;
            const float error = __double2float_ru(fabs(static_cast<double>(got) - exact));
            abs_bits = max(abs_bits, as_bits(error));
            const float want = __double2float_rn(exact);
            if (want >= 0x1p-10f) {
                const int32_t d = static_cast<int32_t>(as_bits(got)) - static_cast<int32_t>(as_bits(want));
                ulps = max(ulps, static_cast<unsigned int>(d < 0 ? -d : d));
            }
        }
    }
    atomicMax(worst_abs_bits, abs_bits);
    atomicMax(worst_ulps, ulps);
}

// sin_squared2 against sin_squared, bit for bit, on every F32 argument in
// [-8192, 8192] (each argument once in each lane).
__global__ void sin_squared_packed_check_kernel(unsigned long long *mismatches)
{
    constexpr uint32_t last = 0x46000000u;  // |8192.0|
    unsigned long long bad = 0ull;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i <= last; i += stride) {
        const float t = as_float(i);
        const float u = as_float(0x80000000u | (last - i));
        float p0, p1, q0, q1;
        sin_squared2(t, u, p0, p1);
        sin_squared2(u, t, q0, q1);
        const uint32_t want_t = as_bits(sin_squared(t));
        const uint32_t want_u = as_bits(sin_squared(u));
        bad += (as_bits(p0) != want_t) + (as_bits(p1) != want_u) + (as_bits(q0) != want_u) +
               (as_bits(q1) != want_t);
    }
    if (bad != 0ull) atomicAdd(mismatches, bad);
}

}  // namespace
}  // namespace m3c

extern "C" m3_status m3_cuda_division_self_test(int device, uint64_t samples, uint64_t *mismatches,
                                                m3_error *error)
{
    unsigned long long *counter = nullptr;
    unsigned long long host = 0;
    cudaError_t code = cudaSetDevice(device);
    if (code == cudaSuccess) code = cudaMalloc(&counter, sizeof(*counter));
    if (code == cudaSuccess) code = cudaMemset(counter, 0, sizeof(*counter));
    if (code == cudaSuccess) {
        m3c::division_check_kernel<<<148 * 16, 256>>>(samples, counter);
        code = cudaGetLastError();
    }
    if (code == cudaSuccess) code = cudaMemcpy(&host, counter, sizeof(host), cudaMemcpyDeviceToHost);
    if (counter != nullptr) cudaFree(counter);
    if (code != cudaSuccess) {
        if (error != nullptr) {
            error->status = M3_STATUS_INTERNAL;
            snprintf(error->message, sizeof(error->message), "division self-test failed: %s",
                     cudaGetErrorString(code));
        }
        return M3_STATUS_INTERNAL;
    }
    if (mismatches != nullptr) *mismatches = host;
    if (error != nullptr) {
        error->status = M3_STATUS_OK;
        error->message[0] = '\0';
    }
    return M3_STATUS_OK;
}

extern "C" m3_status m3_cuda_exp_self_test(int device, uint32_t *max_ulp, uint64_t *violations, m3_error *error)
{
    struct Result {
        unsigned int worst;
        unsigned int pad;
        unsigned long long violations;
    };
    Result *result = nullptr;
    Result host = {};
    cudaError_t code = cudaSetDevice(device);
    if (code == cudaSuccess) code = cudaMalloc(&result, sizeof(*result));
    if (code == cudaSuccess) code = cudaMemset(result, 0, sizeof(*result));
    if (code == cudaSuccess) {
        m3c::exp_check_kernel<<<148 * 16, 256>>>(&result->worst, &result->violations);
        code = cudaGetLastError();
    }
    if (code == cudaSuccess) code = cudaMemcpy(&host, result, sizeof(host), cudaMemcpyDeviceToHost);
    if (result != nullptr) cudaFree(result);
    if (code != cudaSuccess) {
        if (error != nullptr) {
            error->status = M3_STATUS_INTERNAL;
            snprintf(error->message, sizeof(error->message), "exp self-test failed: %s", cudaGetErrorString(code));
        }
        return M3_STATUS_INTERNAL;
    }
    if (max_ulp != nullptr) *max_ulp = host.worst;
    if (violations != nullptr) *violations = host.violations;
    if (error != nullptr) {
        error->status = M3_STATUS_OK;
        error->message[0] = '\0';
    }
    return M3_STATUS_OK;
}

extern "C" m3_status m3_cuda_sin_squared_self_test(int device, float *max_abs_error, uint32_t *max_ulp,
                                                   m3_error *error)
{
    unsigned int *result = nullptr;
    unsigned int host[2] = {0u, 0u};
    cudaError_t code = cudaSetDevice(device);
    if (code == cudaSuccess) code = cudaMalloc(&result, sizeof(host));
    if (code == cudaSuccess) code = cudaMemset(result, 0, sizeof(host));
    if (code == cudaSuccess) {
        m3c::sin_squared_check_kernel<<<148 * 16, 256>>>(result, result + 1);
        code = cudaGetLastError();
    }
    if (code == cudaSuccess) code = cudaMemcpy(host, result, sizeof(host), cudaMemcpyDeviceToHost);
    if (result != nullptr) cudaFree(result);
    if (code != cudaSuccess) {
        if (error != nullptr) {
            error->status = M3_STATUS_INTERNAL;
            snprintf(error->message, sizeof(error->message), "sin^2 self-test failed: %s",
                     cudaGetErrorString(code));
        }
        return M3_STATUS_INTERNAL;
    }
    if (max_abs_error != nullptr) memcpy(max_abs_error, &host[0], sizeof(float));
    if (max_ulp != nullptr) *max_ulp = host[1];
    if (error != nullptr) {
        error->status = M3_STATUS_OK;
        error->message[0] = '\0';
    }
    return M3_STATUS_OK;
}

extern "C" m3_status m3_cuda_codec_self_test(int device, uint64_t *mismatches, m3_error *error)
{
    unsigned long long *counter = nullptr;
    unsigned long long host = 0;
    cudaError_t code = cudaSetDevice(device);
    if (code == cudaSuccess) code = cudaMalloc(&counter, sizeof(*counter));
    if (code == cudaSuccess) code = cudaMemset(counter, 0, sizeof(*counter));
    if (code == cudaSuccess) {
        m3c::codec_check_kernel<<<148 * 16, 256>>>(counter);
        code = cudaGetLastError();
    }
    if (code == cudaSuccess) code = cudaMemcpy(&host, counter, sizeof(host), cudaMemcpyDeviceToHost);
    if (counter != nullptr) cudaFree(counter);
    if (code != cudaSuccess) {
        if (error != nullptr) {
            error->status = M3_STATUS_INTERNAL;
            snprintf(error->message, sizeof(error->message), "codec self-test failed: %s",
                     cudaGetErrorString(code));
        }
        return M3_STATUS_INTERNAL;
    }
    if (mismatches != nullptr) *mismatches = host;
    if (error != nullptr) {
        error->status = M3_STATUS_OK;
        error->message[0] = '\0';
    }
    return M3_STATUS_OK;
}

extern "C" int m3c_launch_rng_uniform(uint64_t seed, uint64_t sequence, float low, float high,
                                      float *out, uint64_t count, void *stream)
{
    if (count == 0) return 0;
    const uint64_t threads = (count + m3c::CHUNK - 1) / m3c::CHUNK;
    const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
    m3c::uniform_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(seed, sequence, low,
                                                                               high, out, count);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int m3c_launch_rng_normal(uint64_t seed, uint64_t sequence, float mean, float deviation,
                                     float *out, uint64_t count, void *stream)
{
    if (count == 0) return 0;
    const uint64_t threads = (count + m3c::CHUNK - 1) / m3c::CHUNK;
    const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
    m3c::normal_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(seed, sequence, mean,
                                                                              deviation, out, count);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int m3c_launch_scan(const void *data, int32_t dtype, uint64_t count, int mode,
                               uint32_t command, m3c_status *status, void *stream);

extern "C" int m3c_launch_row_scan(const void *data, int32_t dtype, uint64_t rows, uint64_t width,
                                   uint32_t ranges, int mode, uint32_t command, m3c_status *status,
                                   void *stream)
{
    const uint64_t eb = dtype == M3C_F32 || dtype == M3C_I32 ? 4u : 2u;
    if (rows == 0 || width == 0) return 0;
    if ((width * eb) % 16u != 0u || (reinterpret_cast<uintptr_t>(data) & 15u) != 0u || ranges == 0 ||
        width * eb / 16u > 0xffffffffull) {
        return m3c_launch_scan(data, dtype, rows * width, mode, command, status, stream);
    }
    const uint64_t blocks = (rows + 7u) / 8u;
    const unsigned grid = static_cast<unsigned>(blocks < 148u * 8u ? blocks : 148u * 8u);
    m3c::row_scan_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4 *>(data), dtype, rows, static_cast<uint32_t>(width * eb / 16u),
        ranges < rows ? ranges : static_cast<uint32_t>(rows), mode, command, status);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int m3c_launch_scan(const void *data, int32_t dtype, uint64_t count, int mode,
                               uint32_t command, m3c_status *status, void *stream)
{
    if (count == 0) return 0;
    uint64_t grid = (count + 255) / 256;
    if (grid > 148u * 16u) grid = 148u * 16u;
    m3c::scan_kernel<<<static_cast<unsigned>(grid), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        data, dtype, count, mode, command, status);
    return static_cast<int>(cudaGetLastError());
}

namespace m3c {
namespace {

// staging = [reduction bits..., ~first failing command]: a MAX over ranks of
// each word is the largest bit pattern (|x| of non-NaN F32 values orders like
// the value; a NaN pattern beats every number) and the smallest failing
// command.
__global__ void shard_pack_kernel(m3c_shard_words w)
{
    const int i = static_cast<int>(threadIdx.x);
    if (i < w.count) {
        w.staging[i] = *reinterpret_cast<volatile uint32_t *>(w.values[i]);
    } else if (i == w.count) {
        w.staging[i] = ~*reinterpret_cast<volatile uint32_t *>(&w.status->fail_command);
    }
}

__global__ void shard_unpack_kernel(m3c_shard_words w)
{
    const int i = static_cast<int>(threadIdx.x);
    if (i < w.count) {
        const uint32_t bits = w.staging[i];
        *w.values[i] = bits;
        if (bits > 0x7f800000u) record_failure(w.status, w.commands[i]);  // a NaN on some rank
    } else if (i == w.count) {
        const uint32_t first = ~w.staging[i];
        if (first != 0xffffffffu) record_failure(w.status, first);
    }
}

}  // namespace
}  // namespace m3c

namespace m3c {
namespace {

// Between two runs of one batch (no synchronise between them): once a run
// has failed, every later run is halted, as the reference stops at the
// failing m3_session_run.
__global__ void run_gate_kernel(m3c_status *status)
{
    if (*reinterpret_cast<volatile uint32_t *>(&status->fail_command) != 0xffffffffu) {
        atomicOr(&status->runs_started, M3C_RUN_HALTED);
    }
}

}  // namespace
}  // namespace m3c

extern "C" int m3c_launch_run_gate(m3c_status *status, void *stream)
{
    m3c::run_gate_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(status);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int m3c_launch_shard_pack(const m3c_shard_words *words, void *stream)
{
    m3c::shard_pack_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*words);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int m3c_launch_shard_unpack(const m3c_shard_words *words, void *stream)
{
    m3c::shard_unpack_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*words);
    return static_cast<int>(cudaGetLastError());
}

extern "C" const char *m3c_cuda_error_string(int code)
{
    return cudaGetErrorString(static_cast<cudaError_t>(code));
}

extern "C" m3_status m3_cuda_sin_squared_packed_self_test(int device, uint64_t *mismatches, m3_error *error)
{
    unsigned long long *counter = nullptr;
    unsigned long long host = 0;
    cudaError_t code = cudaSetDevice(device);
    if (code == cudaSuccess) code = cudaMalloc(&counter, sizeof(*counter));
    if (code == cudaSuccess) code = cudaMemset(counter, 0, sizeof(*counter));
    if (code == cudaSuccess) {
        m3c::sin_squared_packed_check_kernel<<<148 * 16, 256>>>(counter);
        code = cudaGetLastError();
    }
    if (code == cudaSuccess) code = cudaMemcpy(&host, counter, sizeof(host), cudaMemcpyDeviceToHost);
    if (counter != nullptr) cudaFree(counter);
    if (code != cudaSuccess) {
        if (error != nullptr) {
            error->status = M3_STATUS_INTERNAL;
            snprintf(error->message, sizeof(error->message), "packed sin^2 self-test failed: %s",
                     cudaGetErrorString(code));
        }
        return M3_STATUS_INTERNAL;
    }
    if (mismatches != nullptr) *mismatches = host;
    if (error != nullptr) {
        error->status = M3_STATUS_OK;
        error->message[0] = '\0';
    }
    return M3_STATUS_OK;
}
