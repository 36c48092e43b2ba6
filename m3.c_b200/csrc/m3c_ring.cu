// Softmax / TOP_K (k <= 1) / ROW_SUM over F32 rows of 512 or 1024 elements:
// a persistent, warp-specialised row pipeline (sm_100a).
//
// The reference sums each row left to right in F32
// (src/m3_op_execute_basic.c:150-158).  Reproducing that order makes every
// row sum one chain of dependent additions (1024 here); a sum of another
// order differs from the reference's by up to 4.3e-6 relative on the C2
// benchmark rows, over the 1e-6 bar, so the chain stays.  A chain is cheap in
// issue slots when one lane runs one row (a warp instruction then advances 32
// rows) but long in latency, and the warp scheduler starves it next to warps
// with independent work.  So the CTA is split by role, and the chain gets a
// scheduler of its own:
//
//   warp 0 (sub-partition 0)  the chain warp.  Its first 24 lanes sum 24
//                             rows at a time, in four groups of 6 lanes that
//                             start their rows a quarter of a row apart: the
//                             CTA's local row i is summed by lane i % 24, and
//                             at the start of every quarter one group
//                             publishes the sums of the rows it finished and
//                             takes up the next 6.  A lane's loads run 8
//                             vectors ahead of its additions; the 16-byte row
//                             padding puts the lanes of a load phase on
//                             distinct bank groups.  A row holds its slot
//                             from its copy until its probabilities are
//                             written, so the rows in the chain and the
//                             copies in flight share the ring: 24 rows (of
//                             16, 20, 24, 28 and 32 measured) balance the
//                             chain's speed against the depth of the copies;
//   warp 5 (sub-partition 1)  the producer: one thread issues a 1-D TMA bulk
//                             copy (cp.async.bulk, global -> shared, mbarrier
//                             completion, no tensor map, no multicast) per
//                             row as soon as the row's slot is free;
//   warps 4, 8, 12            idle (they leave sub-partition 0 to the chain);
//   the other 11 warps of sub-partitions 1-3, the row warps: row warp w owns
//                             rows i = w (mod 11); for each it computes max /
//                             first argmax / NaN in one pass, writes the
//                             top-1 outputs and the exponentials in place, and
//                             33 rows later (once the chain is done with that
//                             row) the probabilities e / sum with Markstein's
//                             quotient, streamed to HBM.
//
// Row i lives in ring slot i % SLOTS (55 slots of 4 KiB + 16, nearly all of
// the 227 KiB of shared memory).  Per slot, two mbarriers carry the row
// between the producer and the row warps -- full (TMA landed), empty
// (written out; the producer may reuse the slot) -- and two sequence words
// (the slot's use count, published after a block fence) between the row
// warps and the chain: expd (exponentials ready), summed (the chain is
// done).  Every wait is bounded: a wait past its deadline records an
// internal failure in the status word and the thread leaves its loop.  Each row
// depends only on rows with smaller indices, so the waits form no cycle and
// the bound is never reached by a correct run.

#include <cuda_runtime.h>

#include <cstdint>

#include "m3c_device.cuh"
#include "m3c_kernels.h"
#include "m3c_bulk.cuh"

namespace m3c {
namespace {

constexpr int RING_THREADS = 512;
constexpr int CHAIN_WARP = 0;
constexpr int PRODUCER_WARP = 5;        // sub-partition 1: none shares the chain's
constexpr int CHAIN_LANES = 24;         // rows the chain warp sums at once
constexpr int GROUPS = 4;               // chain lane groups, a quarter row apart
constexpr int PREFETCH = 8;             // 16-byte loads a chain lane runs ahead
constexpr int ROW_WARPS = 11;           // the other warps of sub-partitions 1-3

template <int WIDTH>
struct RingGeometry {
    static constexpr int BYTES = WIDTH * 4;
    static constexpr int PITCH = BYTES + 16;
    static constexpr int VPL = WIDTH / 128;            // 16-byte vectors per lane
    // a chain lane's row in GROUPS periods of PV 16-byte vectors each
    static constexpr int PV = WIDTH / 4 / GROUPS;
    static_assert(PV % PREFETCH == 0, "whole prefetch windows per period");
    static constexpr int SLOTS = WIDTH == 1024 ? 55 : 96;
    static constexpr int LAG = 33;                     // exp(i) ... out(i - LAG)
    // per slot: full, empty barriers; the published sum; the exponentials'
    // sequence word; flags, issued
    static constexpr int ROWS_BYTES = SLOTS * PITCH;
    static constexpr int SMEM = ROWS_BYTES + SLOTS * (2 * 8 + 8 + 4 + 1 + 1);
    static_assert(LAG % 11 == 0 && LAG > CHAIN_LANES, "a row warp's out lag: its own rows, after the chain");
};

// Poll a published (use, value) word until its use is `want`.
__device__ __forceinline__ bool poll_sum(volatile unsigned long long *word, unsigned want,
                                         unsigned long long *value)
{
    uint64_t deadline = 0;
    for (uint32_t spin = 0;; ++spin) {
        const unsigned long long seen = *word;
        if (static_cast<unsigned>(seen) == want) {
            *value = seen;
            return true;
        }
        __nanosleep(32);
        if ((spin & 255u) == 0u) {
            const uint64_t t = now_ns();
            if (deadline == 0) {
                deadline = t + BULK_WAIT_NS;
            } else if (t > deadline) {
                return false;
            }
        }
    }
}

// NaN-propagating maximum (PTX max.NaN).
__device__ __forceinline__ float max_nan(float a, float b)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}


__device__ __noinline__ float ring_ieee_div(float a, float b) { return __fdiv_rn(a, b); }

constexpr int FLAG_SPECIAL = 1;   // row maximum is +-inf: probabilities final
constexpr int FLAG_TINY = 2;      // some e < 2^-100: IEEE division needed

template <int OUT, int WIDTH>
__global__ void __launch_bounds__(RING_THREADS, 1)
    softmax_ring_kernel(const __grid_constant__ m3c_softmax_params p)
{
    using Geo = RingGeometry<WIDTH>;
    constexpr int SLOTS = Geo::SLOTS;
    constexpr int PITCH = Geo::PITCH;
    constexpr int VPL = Geo::VPL;
    constexpr int PV = Geo::PV;
    constexpr int LAG = Geo::LAG;
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char *rows_area = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Geo::ROWS_BYTES);
    uint64_t *empty = full + SLOTS;
    // the uses of a slot whose exponentials / sum are ready (plain words:
    // the chain warp polls and publishes one row every 32 steps, too often
    // for mbarrier round trips)
    // (use, sum bits): one 64-bit store publishes a row's sum with its use
    // count, so the reader needs no fence for the sum itself
    volatile unsigned long long *summed = reinterpret_cast<volatile unsigned long long *>(empty + SLOTS);
    volatile int *expd_seq = reinterpret_cast<volatile int *>(summed + SLOTS);
    unsigned char *slot_flags = reinterpret_cast<unsigned char *>(const_cast<int *>(expd_seq + SLOTS));
    unsigned char *slot_issued = slot_flags + SLOTS;
    __shared__ int skip;

    const int warp = static_cast<int>(threadIdx.x) / 32;
    const int lane = static_cast<int>(threadIdx.x) % 32;
    const float pos_inf = __int_as_float(0x7f800000);
    uint32_t first_command = p.softmax_command < p.topk_command ? p.softmax_command : p.topk_command;
    if (p.rowsum_command < first_command) first_command = p.rowsum_command;
    const uint32_t check_command = p.softmax_command < p.topk_command ? p.softmax_command : p.topk_command;

    // this CTA's rows: a balanced contiguous range
    const uint64_t row_begin = p.rows * blockIdx.x / gridDim.x;
    const uint64_t row_end = p.rows * (blockIdx.x + 1) / gridDim.x;
    const int local_rows = static_cast<int>(row_end - row_begin);

    if (threadIdx.x == 0) {
        skip = failed_before(p.status, p.skip_before) ? 1 : 0;
        if (!skip && p.first_of_run && blockIdx.x == 0) {
            atomicAdd(&p.status->runs_started, 1u);
        }
        for (int s = 0; s < SLOTS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 32);
            expd_seq[s] = 0;
            summed[s] = 0ull;
            slot_issued[s] = 0;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (skip || local_rows <= 0) {
        return;
    }
    const float4 *in = static_cast<const float4 *>(p.input);

    if (warp == PRODUCER_WARP) {
        if (lane != 0) return;
        bool ok = true;
        for (int i = 0; i < local_rows; ++i) {
            const int s = i % SLOTS;
            const int use = i / SLOTS;
            if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
                bulk_timed_out(p.status, first_command);
                ok = false;
                break;
            }
            mbar_expect_tx(&full[s], Geo::BYTES);
            bulk_load(rows_area + s * PITCH, in + (row_begin + i) * (WIDTH / 4), Geo::BYTES, &full[s]);
            // bit 0: a copy was issued; bit 1: the parity of its phase
            slot_issued[s] = static_cast<unsigned char>(1u | ((use & 1) << 1));
        }
        if (!ok) {
            // let every copy this thread issued land before the CTA ends
            for (int s = 0; s < SLOTS; ++s) {
                if (slot_issued[s] & 1u) (void)mbar_wait(&full[s], (slot_issued[s] >> 1) & 1u);
            }
        }
        return;
    }

    if (warp == CHAIN_WARP) {
        // Lane l < CHAIN_LANES sums rows l, l + CHAIN_LANES, ...  Its group
        // g = l / (CHAIN_LANES / GROUPS) starts its n-th row in period
        // n * GROUPS + g and spends GROUPS periods on it, so at the start of
        // every period one group publishes the rows it finished and takes
        // up the next ones: rows enter and leave the chain a few at a time.
        constexpr int PER_GROUP = CHAIN_LANES / GROUPS;
        const bool summing = p.probs != nullptr || p.row_sums != nullptr;
        const int group = lane < CHAIN_LANES ? lane / PER_GROUP : GROUPS;
        float sum = 0.0f;
        int cur = -1;        // the row this lane sums, -1: none
        int slot = 0;
        int part = 0;        // the period of the row this lane is in
        const int per_lane = (local_rows + CHAIN_LANES - 1) / CHAIN_LANES;
        const int periods = (per_lane + 1) * GROUPS;
        for (int q = 0; q < periods; ++q) {
            bool failed = false;
            if (group < GROUPS && q >= group && (q - group) % GROUPS == 0) {
                if (cur >= 0) {
                    // the row is complete: publish its sum (ROW_SUM alone:
                    // straight to its output)
                    if (p.row_sums != nullptr && p.probs == nullptr) {
                        p.row_sums[row_begin + cur] = sum;
                    }
                    summed[slot] = (static_cast<unsigned long long>(__float_as_uint(sum)) << 32) |
                                   static_cast<unsigned>(cur / SLOTS + 1);
                }
                const int next = (q - group) / GROUPS * CHAIN_LANES + lane;
                cur = next < local_rows ? next : -1;
                sum = 0.0f;
                part = 0;
                if (cur >= 0) {
                    slot = cur % SLOTS;
                    failed = !poll_acquire(&expd_seq[slot], cur / SLOTS + 1);
                }
            }
            if (__any_sync(0xffffffffu, failed)) {
                if (failed) bulk_timed_out(p.status, first_command);
                break;
            }
            if (cur >= 0 && summing) {
                // the reference's left-to-right F32 sum over a quarter of
                // the row (of e, or of x for ROW_SUM without SOFTMAX); the
                // loads run PREFETCH vectors ahead of the additions
                const float4 *v4 = reinterpret_cast<const float4 *>(rows_area + slot * PITCH) + part * PV;
                float4 a[PREFETCH];
#pragma unroll
                for (int j = 0; j < PREFETCH; ++j) a[j] = v4[j];
#pragma unroll
                for (int j = 0; j < PV; ++j) {
                    const float4 v = a[j % PREFETCH];
                    if (j + PREFETCH < PV) a[j % PREFETCH] = v4[j + PREFETCH];
                    sum = __fadd_rn(sum, v.x);
                    sum = __fadd_rn(sum, v.y);
                    sum = __fadd_rn(sum, v.z);
                    sum = __fadd_rn(sum, v.w);
                }
                ++part;
            }
        }
        return;
    }
    if ((warp & 3) == 0) {
        return;  // warps 4, 8 and 12: sub-partition 0 belongs to the chain
    }

    // row warps: index 0..10 over sub-partitions 1-3 (warp 5 is the producer)
    const int rw = warp - 1 - warp / 4 - (warp > PRODUCER_WARP ? 1 : 0);
    const uint64_t out_pitch = static_cast<uint64_t>(WIDTH) * (OUT == M3C_F32 ? 4u : 2u);

    // max / first argmax / NaN, top-1, exponentials in place
    auto exp_row = [&](int i) -> bool {
        const int s = i % SLOTS;
        if (!mbar_wait(&full[s], (i / SLOTS) & 1)) {
            bulk_timed_out(p.status, first_command);
            return false;
        }
        float4 *row4 = reinterpret_cast<float4 *>(rows_area + s * PITCH);
        float4 q[VPL];
#pragma unroll
        for (int k = 0; k < VPL; ++k) q[k] = row4[lane + 32 * k];
        float m = -pos_inf;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            m = max_nan(m, max_nan(max_nan(q[k].x, q[k].y), max_nan(q[k].z, q[k].w)));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, off));
        const bool nan = m != m;
        const uint64_t row = row_begin + static_cast<uint64_t>(i);
        if (nan && lane == 0 && check_command != 0xffffffffu) {
            record_failure(p.status, check_command);
        }
        if (p.top_values != nullptr) {
            // first index holding a value equal to the maximum (+0 == -0,
            // src/m3_op_execute_sampling.c:7-12), and its value
            uint32_t best = 0xffffffffu;
#pragma unroll
            for (int k = VPL - 1; k >= 0; --k) {
                const uint32_t base = static_cast<uint32_t>(lane + 32 * k) * 4u;
                best = q[k].w == m ? base + 3u : best;
                best = q[k].z == m ? base + 2u : best;
                best = q[k].y == m ? base + 1u : best;
                best = q[k].x == m ? base : best;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, off));
            if (best == 0xffffffffu) best = 0u;  // NaN row (the command fails)
            if (lane == 0) {
                p.top_values[row] = reinterpret_cast<const float *>(row4)[best];
                p.top_indices[row] = static_cast<int32_t>(best);
            }
        }
        if (p.probs != nullptr) {
            int flags = 0;
            if (m == pos_inf || m == -pos_inf) {
                // src/m3_op_execute_basic.c:165-170
                uint32_t infinities = 0u;
#pragma unroll
                for (int k = 0; k < VPL; ++k) {
                    infinities += (q[k].x == pos_inf) + (q[k].y == pos_inf) + (q[k].z == pos_inf) +
                                  (q[k].w == pos_inf);
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    infinities += __shfl_xor_sync(0xffffffffu, infinities, off);
                }
                const float share = __fdiv_rn(1.0f, __uint2float_rn(infinities));
                const bool plus = m == pos_inf;
                __syncwarp();
#pragma unroll
                for (int k = 0; k < VPL; ++k) {
                    row4[lane + 32 * k] =
                        make_float4(plus && q[k].x == pos_inf ? share : 0.0f, plus && q[k].y == pos_inf ? share : 0.0f,
                                    plus && q[k].z == pos_inf ? share : 0.0f, plus && q[k].w == pos_inf ? share : 0.0f);
                }
                flags = FLAG_SPECIAL;
            } else {
                bool tiny = false;
                __syncwarp();   // the top-1 value was read from the row
#pragma unroll
                for (int k = 0; k < VPL; ++k) {
                    const float4 e = make_float4(expf(__fsub_rn(q[k].x, m)), expf(__fsub_rn(q[k].y, m)),
                                                 expf(__fsub_rn(q[k].z, m)), expf(__fsub_rn(q[k].w, m)));
                    tiny |= fminf(fminf(e.x, e.y), fminf(e.z, e.w)) < 0x1p-100f;
                    row4[lane + 32 * k] = e;
                }
                flags = __any_sync(0xffffffffu, tiny) ? FLAG_TINY : 0;
            }
            if (lane == 0) slot_flags[s] = static_cast<unsigned char>(flags);
        }
        __syncwarp();
        if (lane == 0) {
            asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(const_cast<int *>(&expd_seq[s]))),
                         "r"(i / SLOTS + 1)
                         : "memory");
        }
        return true;
    };

    // probabilities e / sum once the chain is done with the row; frees the slot
    auto out_row = [&](int j) -> bool {
        const int s = j % SLOTS;
        unsigned long long published = 0ull;
        if (!poll_sum(&summed[s], j / SLOTS + 1, &published)) {
            bulk_timed_out(p.status, first_command);
            return false;
        }
        if (p.probs != nullptr) {
            const float4 *e4 = reinterpret_cast<const float4 *>(rows_area + s * PITCH);
            const int flags = slot_flags[s];
            const float sum = __uint_as_float(static_cast<uint32_t>(published >> 32));
            const float y = __frcp_rn(sum);
            unsigned char *orow = static_cast<unsigned char *>(p.probs) +
                                  (row_begin + static_cast<uint64_t>(j)) * out_pitch;
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const int v = lane + 32 * k;
                const float4 e = e4[v];
                float pr[4] = {e.x, e.y, e.z, e.w};
                if ((flags & FLAG_SPECIAL) == 0) {
                    if ((flags & FLAG_TINY) == 0) {
                        // e in [2^-100, 1] and sum >= 1: Markstein's quotient
                        // is the IEEE one
#pragma unroll
                        for (int t = 0; t < 4; ++t) pr[t] = div_markstein(pr[t], sum, y);
                    } else {
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            pr[t] = pr[t] >= 0x1p-100f ? div_markstein(pr[t], sum, y) : ring_ieee_div(pr[t], sum);
                        }
                    }
                }
                if (OUT == M3C_F32) {
                    __stcs(reinterpret_cast<float4 *>(orow) + v, make_float4(pr[0], pr[1], pr[2], pr[3]));
                } else {
                    uint32_t h[2];
                    narrow_pairs<2>(OUT, pr, h);
                    __stcs(reinterpret_cast<uint2 *>(orow) + v, make_uint2(h[0], h[1]));
                }
            }
        }
        // the slot's reads (and the exponentials' generic-proxy writes) are
        // ordered before the next bulk copy into it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&empty[s]);
        return true;
    };

    for (int i = rw;; i += ROW_WARPS) {
        const int j = i - LAG;
        if (j >= local_rows) break;
        if (i < local_rows && !exp_row(i)) return;
        if (j >= 0 && !out_row(j)) return;
    }
}

template <int OUT, int WIDTH>
int launch_ring(const m3c_softmax_params &p, void *stream)
{
    using Geo = RingGeometry<WIDTH>;
    auto kernel = softmax_ring_kernel<OUT, WIDTH>;
    static int sm_count = 0;
    if (sm_count == 0) {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device);
        if (sm_count <= 0) sm_count = 148;
    }
    cudaError_t code = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo::SMEM);
    if (code != cudaSuccess) return static_cast<int>(code);
    // one CTA per SM; fewer when a CTA would get less than a chain's rows
    uint64_t grid = (p.rows + CHAIN_LANES - 1) / CHAIN_LANES;
    if (grid > static_cast<uint64_t>(sm_count)) grid = static_cast<uint64_t>(sm_count);
    if (grid == 0) grid = 1;
    kernel<<<static_cast<unsigned>(grid), RING_THREADS, Geo::SMEM, static_cast<cudaStream_t>(stream)>>>(p);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace
}  // namespace m3c

// F32 rows of 512 or 1024 elements, k <= 1, not both probabilities and row
// sums (the chain warp sums e for SOFTMAX, x for ROW_SUM alone); -1 when the
// pipeline does not apply.
static bool ring_applies(const m3c_softmax_params *p)
{
    return p->in_dtype == M3C_F32 && p->k <= 1 && (p->probs == nullptr || p->row_sums == nullptr) &&
           (p->width == 1024 || p->width == 512) && (reinterpret_cast<uintptr_t>(p->input) & 15u) == 0u &&
           (p->probs == nullptr || (reinterpret_cast<uintptr_t>(p->probs) & 15u) == 0u);
}

// The contiguous row ranges the row pass for `p` reads side by side: the
// pipeline's CTAs (one range each), else 1 (the tile kernels take tiles in
// ascending order).
extern "C" uint32_t m3c_softmax_row_ranges(const m3c_softmax_params *p)
{
    if (!ring_applies(p) || p->rows == 0) return 1u;
    int device = 0;
    int sms = 0;
    cudaGetDevice(&device);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) {
        (void)cudaGetLastError();
        sms = 148;
    }
    const uint64_t grid = (p->rows + m3c::CHAIN_LANES - 1) / m3c::CHAIN_LANES;
    return static_cast<uint32_t>(grid < static_cast<uint64_t>(sms) ? grid : static_cast<uint64_t>(sms));
}

extern "C" int m3c_launch_softmax_ring(const m3c_softmax_params *p, void *stream)
{
    if (!ring_applies(p)) {
        return -1;
    }
    const int out = p->probs == nullptr ? M3C_F32 : p->probs_dtype;
    if (p->width == 1024) {
        switch (out) {
        case M3C_F16: return m3c::launch_ring<M3C_F16, 1024>(*p, stream);
        case M3C_BF16: return m3c::launch_ring<M3C_BF16, 1024>(*p, stream);
        default: return m3c::launch_ring<M3C_F32, 1024>(*p, stream);
        }
    }
    switch (out) {
    case M3C_F16: return m3c::launch_ring<M3C_F16, 512>(*p, stream);
    case M3C_BF16: return m3c::launch_ring<M3C_BF16, 512>(*p, stream);
    default: return m3c::launch_ring<M3C_F32, 512>(*p, stream);
    }
}
