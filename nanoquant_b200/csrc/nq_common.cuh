// Shared device helpers for the sm_100a NanoQuant kernels: bounded mbarrier waits,
// 1-D bulk (TMA engine) copies, a bounded grid barrier, warp-level tensor-core MMA,
// and host-side error bookkeeping for the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/nq_b200.h"

namespace nq {

// Every device-side spin gives up after this long and records NQ_ERR_DEVICE_TIMEOUT.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

// Workspace control block (first 256 bytes of a GEMV/GEMM workspace).
struct Ctrl {
    unsigned long long arrivals;  // grid-barrier arrivals, monotonic (never reset)
    int status;                   // first device-side error (nq_status), 0 if none
    unsigned int pad[61];
};
static_assert(sizeof(Ctrl) == 256, "control block is 256 bytes");

// ------------------------------------------------------------------ host errors
void set_error(const char *fmt, ...);
int fail(int status, const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);

// Whether launches use programmatic dependent launch (env NQ_PDL=0 turns it off).
bool pdl_enabled();

struct DeviceInfo {
    int sms = 0;
    int max_smem_optin = 0;
    int coop = 0;
    int cc_major = 0, cc_minor = 0;
};
const DeviceInfo &device_info(int dev);

// ------------------------------------------------------------------ device helpers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_status(int *status, int code) {
    if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Programmatic dependent launch: let the next kernel on the stream be scheduled once every
// CTA of this one has started (it then waits in pdl_wait until this grid has completed and its
// memory is visible), and wait for the previous kernel the same way.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of an mbarrier; gives up after kWaitTimeoutNs and records
// NQ_ERR_DEVICE_TIMEOUT.  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(a, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            record_status(status, NQ_ERR_DEVICE_TIMEOUT);
            return false;
        }
    }
}

// 1-D bulk copy global -> this CTA's shared memory, completion signalled on `bar`
// as transaction bytes.  dst, src and bytes must be multiples of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Issue a bulk copy of `bytes` (multiple of 16) in pieces of at most 64 KiB.
__device__ __forceinline__ void bulk_g2s_pieces(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    uint32_t done = 0;
    while (done < bytes) {
        uint32_t n = bytes - done;
        if (n > 65536u) n = 65536u;
        bulk_g2s(static_cast<char *>(dst) + done, static_cast<const char *>(src) + done, n, bar);
        done += n;
    }
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long atom_add_release_gpu_u64(unsigned long long *p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}

__device__ __forceinline__ void red_add_release_gpu_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Grid barriers for a cooperative launch (all CTAs co-resident).  Arrivals increment a
// monotonic 64-bit counter that starts at 0 with the workspace; every launch adds exactly
// nblocks per barrier, so nothing is ever reset.  Thread 0 of each CTA reads the counter
// once, before its first arrival (grid_barrier_base): all earlier launches' barriers are
// complete and this launch's first one is not, so the count rounded down to a multiple of
// nblocks is where this launch started.  Barrier k (1-based) then waits for base + k * nblocks;
// arrivals are fire-and-forget reductions, so the last arrival costs one trip to L2.
// Bounded: gives up after kWaitTimeoutNs, records NQ_ERR_DEVICE_TIMEOUT, returns false.
__device__ __forceinline__ unsigned long long grid_barrier_base(Ctrl *ctrl, unsigned int nblocks) {
    return (ld_acquire_gpu_u64(&ctrl->arrivals) / nblocks) * nblocks;
}

__device__ __forceinline__ bool grid_barrier(Ctrl *ctrl, unsigned long long target) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        __threadfence();
        red_add_release_gpu_u64(&ctrl->arrivals, 1ull);
        // plain spin (one L2 poll per round trip): the wait is short and every CTA is resident
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu_u64(&ctrl->arrivals) < target) {
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                record_status(&ctrl->status, NQ_ERR_DEVICE_TIMEOUT);
                ok = 0;
                break;
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// D(16x8, f32) += A(16x16) * B(16x8), A row-major / B column-major fragments.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T>
struct Elem;
template <>
struct Elem<__half> {
    static constexpr int kDtype = NQ_DTYPE_F16;
    __device__ static __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
        mma_f16_16816(d, a0, a1, a2, a3, b0, b1);
    }
    __device__ static __forceinline__ float to_f(__half v) { return __half2float(v); }
    // Output conversion with the reference's clamp (cuda_utils.cuh:80-86).
    __device__ static __forceinline__ __half out(float v) {
        return __float2half_rn(fminf(fmaxf(v, -64504.0f), 64504.0f));
    }
    __device__ static __forceinline__ __half rn(float v) { return __float2half_rn(v); }
};
template <>
struct Elem<__nv_bfloat16> {
    static constexpr int kDtype = NQ_DTYPE_BF16;
    __device__ static __forceinline__ void mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
        mma_bf16_16816(d, a0, a1, a2, a3, b0, b1);
    }
    __device__ static __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    // Output conversion with the reference's clamp (cuda_utils.cuh:87-90).
    __device__ static __forceinline__ __nv_bfloat16 out(float v) {
        return __float2bfloat16_rn(fminf(fmaxf(v, -3.3895313892515355e+38f), 3.3895313892515355e+38f));
    }
    __device__ static __forceinline__ __nv_bfloat16 rn(float v) { return __float2bfloat16_rn(v); }
};

// Sign mask of a 16-bit pair: bits 15 and 31 of `w` select the signs of the low and
// high element (HALF2 bit order puts the pair (2p, 2p+1) of a 16-column half-word at
// bits (15-p, 31-p), so `w << p` lines both up).
constexpr uint32_t kPairSign = 0x80008000u;

__device__ __forceinline__ uint32_t lop_sign(uint32_t shifted_bits, uint32_t value_pair) {
    return (shifted_bits & kPairSign) ^ value_pair;
}

}  // namespace nq
