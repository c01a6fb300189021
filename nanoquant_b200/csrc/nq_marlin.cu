// The reference's Marlin sign layout on the GPU (sm_100a): packing, unpacking and conversion to
// the HALF2 planes that this build's GEMM / GEMV read.
//
// The reference packs the factors of its prefill-GEMM kernel type with pack_binary_marlin
// (src/nanoquant/kernel/utils.py:186-214): for a weight [n_out, k_red] (output rows, reduction
// columns) element (o, r), with
//     o = ((tile_out * 4 + o16) * 2 + o8) * 8 + o1,   r = ((tile_red * 2 + r8) * 4 + r2) * 2 + r1,
// is stored in the int32 word [tile_red][tile_out * 32 + o1 * 4 + r2] at bit
//     15 - (2 * o8 + r8) + 16 * r1 - 4 * o16,
// set for -1 (utils.py:191-205: its reshape / permute and exponent table).  Words form
// [k_red / 16, n_out / 2]; n_out % 64 == 0 and k_red % 16 == 0.
//
// marlin_to_half2 lets torch.ops.binary_kernels.marlin_* run this build's tensor-core GEMM on
// Marlin-packed weights: one thread per HALF2 word gathers its 32 bits from the (at most 8)
// Marlin words that hold them.
#include "nq_common.cuh"

namespace nq {
namespace marlin {

constexpr int kThreads = 256;

__device__ __forceinline__ void position(int o, int r, int n_out, int &row, int &col, int &bit) {
    (void)n_out;
    const int tile_out = o >> 6, o16 = (o & 63) >> 4, o8 = (o & 15) >> 3, o1 = o & 7;
    const int tile_red = r >> 4, r8 = (r & 15) >> 3, r2 = (r & 7) >> 1, r1 = r & 1;
    row = tile_red;
    col = tile_out * 32 + o1 * 4 + r2;
    bit = 15 - (2 * o8 + r8) + 16 * r1 - 4 * o16;
}

// One thread per Marlin word: gathers its 32 signs (8 output rows x 4 reduction columns).
__global__ void __launch_bounds__(kThreads) pack_kernel(const int8_t *__restrict__ signs, int n_out, int k_red,
                                                        uint32_t *__restrict__ words, int *__restrict__ invalid) {
    const int64_t half_n = n_out / 2;
    const int64_t id = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (id >= (int64_t)(k_red / 16) * half_n) return;
    const int tile_red = (int)(id / half_n), col = (int)(id % half_n);
    const int tile_out = col >> 5, o1 = (col & 31) >> 2, r2 = col & 3;
    uint32_t w = 0;
    int bad = 0;
#pragma unroll
    for (int o16 = 0; o16 < 4; ++o16)
#pragma unroll
        for (int o8 = 0; o8 < 2; ++o8) {
            const int o = tile_out * 64 + o16 * 16 + o8 * 8 + o1;
            const int8_t *row = signs + (size_t)o * k_red + tile_red * 16 + r2 * 2;
#pragma unroll
            for (int r8 = 0; r8 < 2; ++r8)
#pragma unroll
                for (int r1 = 0; r1 < 2; ++r1) {
                    const int8_t s = row[r8 * 8 + r1];
                    bad += (s != 1 && s != -1);
                    if (s < 0) w |= 1u << (15 - (2 * o8 + r8) + 16 * r1 - 4 * o16);
                }
        }
    words[id] = w;
    if (bad && invalid) atomicAdd(invalid, bad);
}

__global__ void __launch_bounds__(kThreads) unpack_kernel(const uint32_t *__restrict__ words, int n_out, int k_red,
                                                          int8_t *__restrict__ signs) {
    const int64_t id = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (id >= (int64_t)n_out * k_red) return;
    const int o = (int)(id / k_red), r = (int)(id % k_red);
    int row, col, bit;
    position(o, r, n_out, row, col, bit);
    const uint32_t w = words[(size_t)row * (n_out / 2) + col];
    signs[id] = ((w >> bit) & 1u) ? int8_t(-1) : int8_t(1);
}

// HALF2 word (o, q) holds columns r = 32 q + j, j < 32, at bit 15 - j/2 + 16 (j % 2); columns at
// or beyond k_red are +1 (bit clear).
__global__ void __launch_bounds__(kThreads) to_half2_kernel(const uint32_t *__restrict__ words, int n_out, int k_red,
                                                            uint32_t *__restrict__ planes) {
    const int wq = (k_red + 31) / 32;
    const int64_t id = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (id >= (int64_t)n_out * wq) return;
    const int o = (int)(id / wq), q = (int)(id % wq);
    const int tile_out = o >> 6, o16 = (o & 63) >> 4, o8 = (o & 15) >> 3, o1 = o & 7;
    const size_t ld = (size_t)n_out / 2;
    uint32_t out = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // the two 16-column tiles of this word
        const int tile_red = 2 * q + h;
        if (tile_red * 16 >= k_red) break;
        const uint32_t *wr = words + (size_t)tile_red * ld + tile_out * 32 + o1 * 4;
        uint32_t m[4];
#pragma unroll
        for (int r2 = 0; r2 < 4; ++r2) m[r2] = __ldg(wr + r2);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
            const int r8 = jj >> 3, r2 = (jj & 7) >> 1, r1 = jj & 1;
            const uint32_t b = (m[r2] >> (15 - (2 * o8 + r8) + 16 * r1 - 4 * o16)) & 1u;
            const int j = 16 * h + jj;
            out |= b << (15 - j / 2 + 16 * (j & 1));
        }
    }
    planes[id] = out;
}

static int check_shape(int64_t n_out, int64_t k_red) {
    if (n_out <= 0 || k_red <= 0) return fail(NQ_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (n_out % 64 || k_red % 16)
        return fail(NQ_ERR_UNSUPPORTED, "the Marlin layout needs n_out %% 64 == 0 and k_red %% 16 == 0 (got %lld x %lld)",
                    (long long)n_out, (long long)k_red);
    if (n_out > (1 << 24) || k_red > (1 << 24) || n_out * k_red > (int64_t)1 << 40)
        return fail(NQ_ERR_UNSUPPORTED, "sizes beyond the supported range");
    return NQ_OK;
}

static unsigned blocks_for(int64_t n) { return (unsigned)((n + kThreads - 1) / kThreads); }

}  // namespace marlin
}  // namespace nq

extern "C" {

int nq_pack_marlin(const int8_t *signs, int64_t n_out, int64_t k_red, int32_t *words, int32_t *invalid_count,
                   void *stream) {
    using namespace nq::marlin;
    int st = check_shape(n_out, k_red);
    if (st) return st;
    if (!signs || !words) return nq::fail(NQ_ERR_INVALID_ARGUMENT, "null tensor pointer");
    const int64_t n = (k_red / 16) * (n_out / 2);
    pack_kernel<<<blocks_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        signs, (int)n_out, (int)k_red, reinterpret_cast<uint32_t *>(words), invalid_count);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : nq::cuda_fail(e, "marlin pack launch");
}

int nq_unpack_marlin(const int32_t *words, int64_t n_out, int64_t k_red, int8_t *signs, void *stream) {
    using namespace nq::marlin;
    int st = check_shape(n_out, k_red);
    if (st) return st;
    if (!signs || !words) return nq::fail(NQ_ERR_INVALID_ARGUMENT, "null tensor pointer");
    unpack_kernel<<<blocks_for(n_out * k_red), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint32_t *>(words), (int)n_out, (int)k_red, signs);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : nq::cuda_fail(e, "marlin unpack launch");
}

int nq_marlin_to_half2(const int32_t *words, int64_t n_out, int64_t k_red, int32_t *planes, void *stream) {
    using namespace nq::marlin;
    int st = check_shape(n_out, k_red);
    if (st) return st;
    if (!planes || !words) return nq::fail(NQ_ERR_INVALID_ARGUMENT, "null tensor pointer");
    to_half2_kernel<<<blocks_for(n_out * ((k_red + 31) / 32)), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint32_t *>(words), (int)n_out, (int)k_red, reinterpret_cast<uint32_t *>(planes));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : nq::cuda_fail(e, "marlin to half2 launch");
}

}  // extern "C"
