// One-shot all-reduce of a small vector across the GPUs of one node, over peer memory (sm_100a).
//
// Tensor-parallel decode sums the row-parallel layers' partial outputs (o, down) once per
// attention / MLP block; at batch 1 that is a few kilobytes, so the collective is pure latency.
// Each rank owns a region (the layout below) that every other rank has mapped through CUDA IPC.
// A call with n elements runs kArBlocks CTAs; CTA c owns slice c of the vector and
//   1. stores its slice of x into every rank's receive buffer (NVLink stores to peer memory),
//   2. raises its flag for slice c on every rank (a release store of the call's epoch),
//   3. waits, bounded, until every rank's flag for slice c has reached the epoch (acquire),
//   4. sums the world slices in rank order in float32 and writes out (identical bits on every
//      rank, so the replicated residual streams stay identical).
// Epochs are per-CTA counters in the local region, advanced by every call, so the same launch
// replayed from a CUDA graph stays in step on all ranks as long as every rank makes the same
// sequence of calls.  Receive buffers alternate by epoch parity: a rank can be at most one call
// ahead of another (it needs the other's flag for call k + 1 before it can start call k + 2,
// and that flag is raised only after the other finished reading call k).
#include <cstring>

#include "../../include/nq_decoder.h"
#include "nq_common.cuh"

namespace nq {
namespace ar {

constexpr int kArBlocks = 16;    // CTAs (slices) per call
constexpr int kArThreads = 256;
constexpr int kArMaxWorld = 8;

// Region layout (bytes): [Ctrl 256][epochs kArBlocks x u32, padded to 256]
// [flags kArMaxWorld x kArBlocks x u32][data 2 parities x world x max_elems x 2 B]
constexpr size_t kOffEpochs = sizeof(Ctrl);
constexpr size_t kOffFlags = kOffEpochs + 256;
constexpr size_t kOffData = kOffFlags + (size_t)kArMaxWorld * kArBlocks * 4;
static_assert(kOffData % 256 == 0, "data starts 256-byte aligned");

inline size_t region_bytes(int world, int64_t max_elems) {
    return kOffData + 2 * (size_t)world * (size_t)max_elems * 2;
}

struct ArParams {
    const void *x;
    void *out;
    unsigned char *region[kArMaxWorld];  // every rank's region as mapped in this process
    int64_t n, max_elems;
    int rank, world;
};

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <typename T>
__device__ __forceinline__ void add8(float (&acc)[8], const uint4 &v) {
    const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += Elem<T>::to_f(e[i]);
}

template <typename T>
__global__ void __launch_bounds__(kArThreads) allreduce_kernel(const __grid_constant__ ArParams p) {
    __shared__ unsigned e_s;
    const int c = blockIdx.x, tid = threadIdx.x;
    unsigned char *mine = p.region[p.rank];
    Ctrl *ctrl = reinterpret_cast<Ctrl *>(mine);
    const int64_t pieces = p.n / 8;  // 16-byte pieces (the host requires n % 8 == 0)
    const int64_t per = (pieces + kArBlocks - 1) / kArBlocks;
    const int64_t q0 = (int64_t)c * per, q1 = q0 + per < pieces ? q0 + per : pieces;
    if (tid == 0) {
        unsigned *ep = reinterpret_cast<unsigned *>(mine + kOffEpochs) + c;
        e_s = *ep + 1u;
        *ep = e_s;
    }
    __syncthreads();
    const unsigned e = e_s;
    const size_t plane = (size_t)p.max_elems * 2;  // bytes of one source's buffer
    const size_t par_off = kOffData + (size_t)(e & 1u) * p.world * plane;
    // 1. my slice into every rank's receive buffer for source p.rank
    const uint4 *x4 = static_cast<const uint4 *>(p.x);
    for (int r = 0; r < p.world; ++r) {
        uint4 *dst = reinterpret_cast<uint4 *>(p.region[r] + par_off + (size_t)p.rank * plane);
        for (int64_t q = q0 + tid; q < q1; q += kArThreads) dst[q] = x4[q];
    }
    __threadfence_system();
    __syncthreads();
    // 2. flag slice c on every rank; 3. wait for every source's flag here
    if (tid < p.world) {
        st_release_sys(reinterpret_cast<unsigned *>(p.region[tid] + kOffFlags) + p.rank * kArBlocks + c, e);
        const unsigned *f = reinterpret_cast<const unsigned *>(mine + kOffFlags) + tid * kArBlocks + c;
        if (ld_acquire_sys(f) < e) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_sys(f) < e) {
                if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                    record_status(&ctrl->status, NQ_ERR_DEVICE_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
    // 4. sum the sources in rank order (L2 reads: peers wrote this memory over NVLink)
    uint4 *o4 = static_cast<uint4 *>(p.out);
    for (int64_t q = q0 + tid; q < q1; q += kArThreads) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < p.world; ++s)
            add8<T>(acc, __ldcg(reinterpret_cast<const uint4 *>(mine + par_off + (size_t)s * plane) + q));
        uint4 r;
        T *re = reinterpret_cast<T *>(&r);
#pragma unroll
        for (int i = 0; i < 8; ++i) re[i] = Elem<T>::rn(acc[i]);
        o4[q] = r;
    }
}

}  // namespace ar
}  // namespace nq

using namespace nq;

extern "C" {

NQ_API size_t nq_allreduce_region_bytes(int world, int64_t max_elems) {
    if (world < 1 || world > ar::kArMaxWorld || max_elems <= 0) return 0;
    return ar::region_bytes(world, max_elems);
}

NQ_API int nq_allreduce_region_alloc(int world, int64_t max_elems, void **region_out) {
    const size_t bytes = nq_allreduce_region_bytes(world, max_elems);
    if (!bytes || !region_out) return fail(NQ_ERR_INVALID_ARGUMENT, "allreduce region: world %d, max_elems %lld", world,
                                            (long long)max_elems);
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);  // its own allocation: an IPC handle maps whole allocations
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(allreduce region)");
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "cudaMemset(allreduce region)");
    }
    *region_out = p;
    return NQ_OK;
}

NQ_API int nq_allreduce_region_free(void *region) {
    if (!region) return NQ_OK;
    const cudaError_t e = cudaFree(region);
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "cudaFree(allreduce region)");
}

NQ_API int nq_ipc_handle(const void *region, void *handle_out) {
    if (!region || !handle_out) return fail(NQ_ERR_INVALID_ARGUMENT, "nq_ipc_handle: null pointer");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(region));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle_out, &h, sizeof(h));
    return NQ_OK;
}

NQ_API int nq_ipc_open(const void *handle, void **region_out) {
    if (!handle || !region_out) return fail(NQ_ERR_INVALID_ARGUMENT, "nq_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(region_out, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    return NQ_OK;
}

NQ_API int nq_ipc_close(void *region) {
    if (!region) return NQ_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(region);
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

NQ_API int nq_allreduce(int dtype, const void *x, void *out, int64_t n, int rank, int world,
                        void *const *regions, int64_t max_elems, void *stream) {
    if (dtype != NQ_DTYPE_F16 && dtype != NQ_DTYPE_BF16) return fail(NQ_ERR_UNSUPPORTED, "allreduce dtype");
    if (world < 1 || world > ar::kArMaxWorld || rank < 0 || rank >= world)
        return fail(NQ_ERR_INVALID_ARGUMENT, "allreduce: rank %d of world %d (at most %d)", rank, world,
                    ar::kArMaxWorld);
    if (!x || !out || !regions || n <= 0 || n % 8 || n > max_elems)
        return fail(NQ_ERR_INVALID_ARGUMENT, "allreduce: n %lld must be a positive multiple of 8 <= %lld",
                    (long long)n, (long long)max_elems);
    if (((uintptr_t)x | (uintptr_t)out) & 15) return fail(NQ_ERR_INVALID_ARGUMENT, "allreduce: x, out 16B aligned");
    ar::ArParams p{};
    p.x = x;
    p.out = out;
    p.n = n;
    p.max_elems = max_elems;
    p.rank = rank;
    p.world = world;
    for (int r = 0; r < world; ++r) {
        if (!regions[r] || ((uintptr_t)regions[r] & 255))
            return fail(NQ_ERR_INVALID_ARGUMENT, "allreduce: region %d missing or not 256-byte aligned", r);
        p.region[r] = static_cast<unsigned char *>(regions[r]);
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == NQ_DTYPE_F16)
        ar::allreduce_kernel<__half><<<ar::kArBlocks, ar::kArThreads, 0, s>>>(p);
    else
        ar::allreduce_kernel<__nv_bfloat16><<<ar::kArBlocks, ar::kArThreads, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "allreduce launch");
}

}  // extern "C"
