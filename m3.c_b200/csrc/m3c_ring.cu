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
//   warp 0 (sub-partition 0)  the chain warp.  Its lanes are staggered: the
//                             CTA's local row i is summed by lane i % 32 over
//                             chunks i .. i+31 of 32 elements each, so at
//                             every chunk boundary exactly one lane finishes a
//                             row (publishes its sum) and starts the next.
//                             Rows enter and leave the chain one at a time;
//                             the 16-byte row padding keeps the 8 lanes of
//                             each quarter-warp load phase on distinct bank
//                             groups;
//   warp 4 (sub-partition 0)  the producer: one thread issues a 1-D TMA bulk
//                             copy (cp.async.bulk, global -> shared, mbarrier
//                             completion, no tensor map, no multicast) per
//                             row as soon as the row's slot is free;
//   warps 8, 12               idle (they leave sub-partition 0 to the chain);
//   the 12 warps of sub-partitions 1-3, the row warps: row warp w owns rows
//                             i = w (mod 12); for each it computes max /
//                             first argmax / NaN in one pass, writes the
//                             top-1 outputs and the exponentials in place, and
//                             36 rows later (once the chain is done with that
//                             row) the probabilities e / sum with Markstein's
//                             quotient, streamed to HBM.
//
// Row i lives in ring slot i % SLOTS (55 slots of 4 KiB + 16, nearly all of
// the 227 KiB of shared memory).  Four mbarriers per slot carry the row
// through its life: full (TMA landed), expd (exponentials ready), summed
// (the chain is done), empty (written out; the producer may reuse the slot).
// Every wait is bounded: a wait past its deadline records an internal
// failure in the status word and the thread leaves its loop.  Each row
// depends only on rows with smaller indices, so the waits form no cycle and
// the bound is never reached by a correct run.

#include <cuda_runtime.h>

#include <cstdint>

#include "m3c_device.cuh"
#include "m3c_kernels.h"

namespace m3c {
namespace {

constexpr int RING_THREADS = 512;
constexpr int CHAIN_WARP = 0;
constexpr int PRODUCER_WARP = 4;
constexpr int ROW_WARPS = 12;           // the warps of sub-partitions 1-3
constexpr uint64_t WAIT_NS = 2000000000ull;   // 2 s per wait, then give up
constexpr uint32_t INTERNAL_CODE = 9u;  // M3_STATUS_INTERNAL

template <int WIDTH>
struct RingGeometry {
    static constexpr int BYTES = WIDTH * 4;
    static constexpr int PITCH = BYTES + 16;
    static constexpr int VPL = WIDTH / 128;            // 16-byte vectors per lane
    static constexpr int CHUNKS = 32;                  // chain chunks per row (one per lane)
    static constexpr int VPC = WIDTH / 128;            // 16-byte vectors per chunk
    static constexpr int SLOTS = WIDTH == 1024 ? 55 : 96;
    static constexpr int LAG = 36;                     // exp(i) ... out(i - LAG)
    // per slot: full, expd, summed, empty barriers; sum, reciprocal; flags,
    // issued
    static constexpr int ROWS_BYTES = SLOTS * PITCH;
    static constexpr int SMEM = ROWS_BYTES + SLOTS * (4 * 8 + 4 + 4 + 1 + 1);
    static_assert(LAG % 12 == 0 && LAG >= 32, "a row warp's out lag: its own rows, after the chain");
};

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("{\n\t.reg .b64 state;\n\tmbarrier.arrive.shared::cta.b64 state, [%0];\n\t}" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 state;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 state, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t now_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for the phase of `parity` to complete; false after WAIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity)
{
    const uint32_t addr = smem_addr(bar);
    uint64_t deadline = 0;
    for (uint32_t spin = 0;; ++spin) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((spin & 255u) == 0u) {
            const uint64_t t = now_ns();
            if (deadline == 0) {
                deadline = t + WAIT_NS;
            } else if (t > deadline) {
                return false;
            }
        }
    }
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// NaN-propagating maximum (PTX max.NaN).
__device__ __forceinline__ float max_nan(float a, float b)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ void timed_out(m3c_status *status, uint32_t command)
{
    atomicMin(&status->fail_command, command);
    atomicExch(&status->fail_code, INTERNAL_CODE);
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
    constexpr int CHUNKS = Geo::CHUNKS;
    constexpr int VPC = Geo::VPC;
    constexpr int LAG = Geo::LAG;
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char *rows_area = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Geo::ROWS_BYTES);
    uint64_t *expd = full + SLOTS;
    uint64_t *summed = expd + SLOTS;
    uint64_t *empty = summed + SLOTS;
    float *slot_sum = reinterpret_cast<float *>(empty + SLOTS);
    float *slot_rcp = slot_sum + SLOTS;
    unsigned char *slot_flags = reinterpret_cast<unsigned char *>(slot_rcp + SLOTS);
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
            mbar_init(&expd[s], 32);
            mbar_init(&summed[s], 1);
            mbar_init(&empty[s], 32);
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
                timed_out(p.status, first_command);
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
        // lane l sums rows l, l + 32, ...; row i over chunks i .. i + 31, a
        // 32nd of the row each
        const bool summing = p.probs != nullptr || p.row_sums != nullptr;
        float sum = 0.0f;
        int cur = -1;        // the row this lane sums, -1: none
        int slot = 0;
        bool failed = false;
        for (int k = 0; k < local_rows + CHUNKS && !failed; ++k) {
            if (lane == (k % 32)) {
                if (cur >= 0) {
                    // the row is complete: publish its sum
                    if (p.probs != nullptr) {
                        slot_sum[slot] = sum;
                        slot_rcp[slot] = __frcp_rn(sum);
                    } else if (p.row_sums != nullptr) {
                        p.row_sums[row_begin + cur] = sum;
                    }
                    mbar_arrive(&summed[slot]);
                }
                cur = k < local_rows ? k : -1;
                sum = 0.0f;
                if (cur >= 0) {
                    slot = cur % SLOTS;
                    if (!mbar_wait(&expd[slot], (cur / SLOTS) & 1)) {
                        timed_out(p.status, first_command);
                        failed = true;
                    }
                }
            }
            failed = __any_sync(0xffffffffu, failed);
            if (cur >= 0 && summing) {
                // the reference's left-to-right F32 sum, 32 elements of the
                // row (of e, or of x for ROW_SUM without SOFTMAX)
                const float4 *v4 =
                    reinterpret_cast<const float4 *>(rows_area + slot * PITCH) + (k - cur) * VPC;
                float4 a[VPC];
#pragma unroll
                for (int j = 0; j < VPC; ++j) a[j] = v4[j];
#pragma unroll
                for (int j = 0; j < VPC; ++j) {
                    sum = __fadd_rn(sum, a[j].x);
                    sum = __fadd_rn(sum, a[j].y);
                    sum = __fadd_rn(sum, a[j].z);
                    sum = __fadd_rn(sum, a[j].w);
                }
            }
        }
        return;
    }
    if ((warp & 3) == 0) {
        return;  // warps 8 and 12: sub-partition 0 belongs to the chain
    }

    // row warps: index 0..11 over sub-partitions 1-3
    const int rw = warp - 1 - warp / 4;
    const uint64_t out_pitch = static_cast<uint64_t>(WIDTH) * (OUT == M3C_F32 ? 4u : 2u);

    // max / first argmax / NaN, top-1, exponentials in place
    auto exp_row = [&](int i) -> bool {
        const int s = i % SLOTS;
        if (!mbar_wait(&full[s], (i / SLOTS) & 1)) {
            timed_out(p.status, first_command);
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
        mbar_arrive(&expd[s]);
        return true;
    };

    // probabilities e / sum once the chain is done with the row; frees the slot
    auto out_row = [&](int j) -> bool {
        const int s = j % SLOTS;
        if (!mbar_wait(&summed[s], (j / SLOTS) & 1)) {
            timed_out(p.status, first_command);
            return false;
        }
        if (p.probs != nullptr) {
            const float4 *e4 = reinterpret_cast<const float4 *>(rows_area + s * PITCH);
            const int flags = slot_flags[s];
            const float sum = slot_sum[s];
            const float y = slot_rcp[s];
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
    uint64_t grid = (p.rows + 31) / 32;
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
extern "C" int m3c_launch_softmax_ring(const m3c_softmax_params *p, void *stream)
{
    if (p->in_dtype != M3C_F32 || p->k > 1 || (p->probs != nullptr && p->row_sums != nullptr) ||
        (p->width != 1024 && p->width != 512) ||
        (reinterpret_cast<uintptr_t>(p->input) & 15u) != 0u ||
        (p->probs != nullptr && (reinterpret_cast<uintptr_t>(p->probs) & 15u) != 0u)) {
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
