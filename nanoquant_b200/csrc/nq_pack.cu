// Sign-plane packing kernels (sm_100a).
//
// pack   : int8 +-1 [rows, cols] -> int32 [rows, ceil(cols/32)]  (reference pack_binary_gemv,
//          src/nanoquant/kernel/utils.py:51-113: +1 -> 0, -1 -> 1, +1 padding)
// unpack : the inverse (reference unpack_binary_gemv, utils.py:116-183)
// repack : bit-order conversion between LSB_FIRST and HALF2 planes
//
// One thread owns one 32-bit word.  Consecutive threads own consecutive words of a
// row, so a warp reads 1 KiB of contiguous int8 signs (two 16-byte loads per thread
// when aligned) and writes 128 contiguous bytes of packed words.  These kernels are
// pure HBM streaming (1 byte in per 1/8 byte out); grids are sized as a multiple of
// the SM count and grid-stride over the words.
#include "nq_common.cuh"

namespace nq {

// Bit position of column j (0..31) of a word.
__host__ __device__ __forceinline__ int bit_pos(int j, int order) {
    return order == NQ_BITS_LSB_FIRST ? j : 15 - (j >> 1) + ((j & 1) << 4);
}

// Sign bit (bit 7) of each byte of v gathered into 4 bits; flags bytes other than 0x01/0xFF.
__device__ __forceinline__ uint32_t gather4(uint32_t v, int &bad) {
    const uint32_t m = (v >> 7) & 0x01010101u;  // 1 where the byte is negative
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t b = (v >> (8 * i)) & 0xFFu;
        bad += (b != 0x01u && b != 0xFFu);
    }
    // m has byte i's flag at bit 8i; the product places it at bit 24+i (the other partial
    // products land below bit 24 on distinct bits or above bit 31, so nothing carries).
    return ((m * 0x01020408u) >> 24) & 0xFu;
}

template <int ORDER>
__device__ __forceinline__ uint32_t place_lsb_word(uint32_t lsb) {
    if (ORDER == NQ_BITS_LSB_FIRST) return lsb;
    uint32_t out = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) out |= ((lsb >> j) & 1u) << (15 - (j >> 1) + ((j & 1) << 4));
    return out;
}

template <int ORDER>
__global__ void __launch_bounds__(256) pack_kernel(const int8_t *__restrict__ signs, int64_t rows, int64_t cols,
                                                   uint32_t *__restrict__ packed, int *invalid_count) {
    const int64_t words = (cols + 31) >> 5;
    const int64_t total = rows * words;
    int bad = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / words, w = i - r * words;
        const int64_t c0 = w * 32;
        const int8_t *src = signs + r * cols + c0;
        uint32_t lsb = 0;
        if (c0 + 32 <= cols && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
            const uint4 a = __ldg(reinterpret_cast<const uint4 *>(src));
            const uint4 b = __ldg(reinterpret_cast<const uint4 *>(src) + 1);
            const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int q = 0; q < 8; ++q) lsb |= gather4(v[q], bad) << (4 * q);
        } else {
            const int n = (int)((cols - c0) < 32 ? (cols - c0) : 32);
            for (int j = 0; j < n; ++j) {
                const int8_t s = src[j];
                bad += (s != 1 && s != -1);
                lsb |= (uint32_t)(s < 0) << j;
            }
        }
        packed[i] = place_lsb_word<ORDER>(lsb);
    }
    if (invalid_count) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, off);
        if ((threadIdx.x & 31) == 0 && bad) atomicAdd(invalid_count, bad);
    }
}

template <int ORDER>
__global__ void __launch_bounds__(256) unpack_kernel(const uint32_t *__restrict__ packed, int64_t rows, int64_t cols,
                                                     int8_t *__restrict__ signs) {
    const int64_t words = (cols + 31) >> 5;
    const int64_t total = rows * words;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / words, w = i - r * words;
        const int64_t c0 = w * 32;
        const uint32_t word = __ldg(packed + i);
        int8_t *dst = signs + r * cols + c0;
        if (c0 + 32 <= cols && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            uint32_t v[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                uint32_t o = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int j = 4 * q + b;
                    const uint32_t bit = (word >> bit_pos(j, ORDER)) & 1u;
                    o |= (bit ? 0xFFu : 0x01u) << (8 * b);
                }
                v[q] = o;
            }
            reinterpret_cast<uint4 *>(dst)[0] = make_uint4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<uint4 *>(dst)[1] = make_uint4(v[4], v[5], v[6], v[7]);
        } else {
            const int n = (int)((cols - c0) < 32 ? (cols - c0) : 32);
            for (int j = 0; j < n; ++j) dst[j] = ((word >> bit_pos(j, ORDER)) & 1u) ? int8_t(-1) : int8_t(1);
        }
    }
}

__global__ void __launch_bounds__(256) repack_kernel(const uint32_t *__restrict__ src, int64_t rows, int64_t cols,
                                                     int src_order, int dst_order, uint32_t *__restrict__ dst) {
    const int64_t words = (cols + 31) >> 5;
    const int64_t total = rows * words;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = i % words;
        const int64_t c0 = w * 32;
        const int n = (int)((cols - c0) < 32 ? (cols - c0) : 32);
        const uint32_t in = __ldg(src + i);
        uint32_t out = 0;
        for (int j = 0; j < n; ++j) out |= ((in >> bit_pos(j, src_order)) & 1u) << bit_pos(j, dst_order);
        dst[i] = out;
    }
}

static int grid_for(int64_t work) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_info(dev).sms > 0 ? device_info(dev).sms : 148;
    int64_t blocks = (work + 255) / 256;
    const int64_t cap = (int64_t)sms * 8;  // 8 resident 256-thread CTAs per SM
    if (blocks > cap) blocks = cap;
    return (int)(blocks < 1 ? 1 : blocks);
}

static int check_plane_args(const void *a, const void *b, int64_t rows, int64_t cols, int order) {
    if (!a || !b) return fail(NQ_ERR_INVALID_ARGUMENT, "null pointer");
    if (rows <= 0 || cols <= 0) return fail(NQ_ERR_INVALID_ARGUMENT, "rows and cols must be positive (got %lld x %lld)",
                                            (long long)rows, (long long)cols);
    if (order != NQ_BITS_LSB_FIRST && order != NQ_BITS_HALF2)
        return fail(NQ_ERR_INVALID_ARGUMENT, "unsupported bit order %d (0 = lsb_first, 1 = half2)", order);
    return NQ_OK;
}

}  // namespace nq

extern "C" {

int nq_pack_signs(const int8_t *signs, int64_t rows, int64_t cols, int bit_order, int32_t *packed,
                  int32_t *invalid_count, void *stream) {
    using namespace nq;
    int st = check_plane_args(signs, packed, rows, cols, bit_order);
    if (st) return st;
    if (reinterpret_cast<uintptr_t>(packed) & 3) return fail(NQ_ERR_INVALID_ARGUMENT, "packed must be 4-byte aligned");
    const int64_t words = rows * ((cols + 31) / 32);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = grid_for(words);
    if (bit_order == NQ_BITS_LSB_FIRST)
        pack_kernel<NQ_BITS_LSB_FIRST><<<grid, 256, 0, s>>>(signs, rows, cols, reinterpret_cast<uint32_t *>(packed),
                                                            invalid_count);
    else
        pack_kernel<NQ_BITS_HALF2><<<grid, 256, 0, s>>>(signs, rows, cols, reinterpret_cast<uint32_t *>(packed),
                                                        invalid_count);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "pack_kernel launch");
}

int nq_unpack_signs(const int32_t *packed, int64_t rows, int64_t cols, int bit_order, int8_t *signs, void *stream) {
    using namespace nq;
    int st = check_plane_args(packed, signs, rows, cols, bit_order);
    if (st) return st;
    if (reinterpret_cast<uintptr_t>(packed) & 3) return fail(NQ_ERR_INVALID_ARGUMENT, "packed must be 4-byte aligned");
    const int64_t words = rows * ((cols + 31) / 32);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = grid_for(words);
    const uint32_t *p = reinterpret_cast<const uint32_t *>(packed);
    if (bit_order == NQ_BITS_LSB_FIRST)
        unpack_kernel<NQ_BITS_LSB_FIRST><<<grid, 256, 0, s>>>(p, rows, cols, signs);
    else
        unpack_kernel<NQ_BITS_HALF2><<<grid, 256, 0, s>>>(p, rows, cols, signs);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "unpack_kernel launch");
}

int nq_repack_signs(const int32_t *src, int64_t rows, int64_t cols, int src_order, int dst_order, int32_t *dst,
                    void *stream) {
    using namespace nq;
    int st = check_plane_args(src, dst, rows, cols, src_order);
    if (st) return st;
    if (dst_order != NQ_BITS_LSB_FIRST && dst_order != NQ_BITS_HALF2)
        return fail(NQ_ERR_INVALID_ARGUMENT, "unsupported destination bit order %d", dst_order);
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 3)
        return fail(NQ_ERR_INVALID_ARGUMENT, "planes must be 4-byte aligned");
    const int64_t words = rows * ((cols + 31) / 32);
    repack_kernel<<<grid_for(words), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint32_t *>(src), rows, cols, src_order, dst_order, reinterpret_cast<uint32_t *>(dst));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "repack_kernel launch");
}

}  // extern "C"
