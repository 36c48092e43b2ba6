/* Seeded synthetic inputs: the reference's PCG32 generator and Box-Muller
 * normal fill (src/m3_rng.c:9-110), restated so benchmark and test inputs are
 * reproducible bit for bit on any host.  The device fills (m3c_util.cu) jump
 * the same generator ahead per block of values. */

#include "m3c_internal.h"

#include <cuda_runtime_api.h>
#include <math.h>

#define PCG_MULTIPLIER UINT64_C(6364136223846793005)

/* src/m3_rng.c:9-20 */
uint32_t m3c_pcg32_next(m3c_pcg32 *rng)
{
    uint64_t old = rng->state;
    uint32_t shifted;
    uint32_t rotation;

    rng->state = old * PCG_MULTIPLIER + rng->increment;
    shifted = (uint32_t)(((old >> 18U) ^ old) >> 27U);
    rotation = (uint32_t)(old >> 59U);
    return (shifted >> rotation) | (shifted << ((0U - rotation) & 31U));
}

/* src/m3_rng.c:22-39 */
void m3c_pcg32_seed(m3c_pcg32 *rng, uint64_t seed, uint64_t sequence)
{
    rng->state = 0U;
    rng->increment = (sequence << 1U) | UINT64_C(1);
    (void)m3c_pcg32_next(rng);
    rng->state += seed;
    (void)m3c_pcg32_next(rng);
}

m3_status m3_cuda_fill_uniform_host(uint64_t seed, uint64_t sequence,
                                    float low, float high, float *values,
                                    size_t count, m3_error *error)
{
    m3c_pcg32 rng;
    float span = high - low;
    size_t i;

    if (count != 0U && values == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "uniform fill output is null");
    }
    m3c_pcg32_seed(&rng, seed, sequence);
    for (i = 0U; i < count; ++i) {
        /* src/m3_rng.c:62-63: 24 random bits scaled to [0, 1) */
        float u = (float)(m3c_pcg32_next(&rng) >> 8U) * 0x1.0p-24F;
        float scaled = span * u;

        values[i] = low + scaled;
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_fill_normal_host(uint64_t seed, uint64_t sequence,
                                   float mean, float deviation, float *values,
                                   size_t count, m3_error *error)
{
    static const double two_pi = 6.283185307179586476925286766559;
    m3c_pcg32 rng;
    size_t i = 0U;

    if (count != 0U && values == NULL) {
        return m3c_error_set(error, M3_STATUS_INVALID_ARGUMENT,
                             "normal fill output is null");
    }
    m3c_pcg32_seed(&rng, seed, sequence);
    while (i < count) {
        /* src/m3_rng.c:87-105 */
        double radius_u = ((double)m3c_pcg32_next(&rng) + 0.5) * 0x1.0p-32;
        double angle_u = (double)m3c_pcg32_next(&rng) * 0x1.0p-32;
        double radius = sqrt(-2.0 * log(radius_u));
        double angle = two_pi * angle_u;
        float first = (float)(radius * cos(angle));
        float second = (float)(radius * sin(angle));
        float scaled = deviation * first;

        values[i++] = mean + scaled;
        if (i < count) {
            scaled = deviation * second;
            values[i++] = mean + scaled;
        }
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_fill_uniform_device(uint64_t seed, uint64_t sequence,
                                      float low, float high,
                                      float *device_values, size_t count,
                                      void *stream, m3_error *error)
{
    int code = m3c_launch_rng_uniform(seed, sequence, low, high,
                                      device_values, count, stream);

    if (code != 0) {
        return m3c_error_set(error, M3_STATUS_INTERNAL,
                             "uniform fill kernel failed: %s",
                             m3c_cuda_error_string(code));
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

m3_status m3_cuda_fill_normal_device(uint64_t seed, uint64_t sequence,
                                     float mean, float deviation,
                                     float *device_values, size_t count,
                                     void *stream, m3_error *error)
{
    int code = m3c_launch_rng_normal(seed, sequence, mean, deviation,
                                     device_values, count, stream);

    if (code != 0) {
        return m3c_error_set(error, M3_STATUS_INTERNAL,
                             "normal fill kernel failed: %s",
                             m3c_cuda_error_string(code));
    }
    m3_error_reset(error);
    return M3_STATUS_OK;
}

int m3_cuda_device_count(void)
{
    int count = 0;

    if (cudaGetDeviceCount(&count) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return count;
}
