// Kernels around the quantized linears in a Llama-architecture decoder (sm_100a):
// fused residual-add + RMSNorm, rotary embedding + KV-cache write, split-KV decode
// attention with a combine pass, and SiLU(gate) * up.  They exist so that a decode
// step is a short, CUDA-graph-capturable sequence of launches; every kernel reads
// positions / sequence lengths from device memory, never from the host.
//
// Numerics follow the HF Llama modules the reference harness runs
// (src/nanoquant/kernel/test_decode.py loads transformers' LlamaForCausalLM): the
// residual sum is rounded to the model dtype, RMSNorm computes in float32 and rounds
// once before the weight multiply, attention accumulates in float32.
#include <cfloat>

#include "../../include/nq_decoder.h"
#include "nq_common.cuh"

namespace nq {
namespace dec {

template <typename T>
__device__ __forceinline__ float tof(T v);
template <>
__device__ __forceinline__ float tof(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float tof(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T fromf(float v);
template <>
__device__ __forceinline__ __half fromf(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 fromf(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float block_sum(float v, float *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += sh[i];
    return s;
}

// ------------------------------------------------------------------ RMSNorm
// h = x (+ residual), rounded to T; residual_out = h; out = weight * T(h * rsqrt(mean(h^2) + eps)).
// One CTA per row; each thread keeps its 8-element chunks in registers between the two
// passes, and all its loads are issued before any is used.
constexpr int kNormThreads = 256;
constexpr int kNormChunks = 4;  // hidden <= 256 * 8 * 4 = 8192 on the vector path

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_vec_kernel(const T *__restrict__ x, const T *__restrict__ res_in,
                                                                   T *__restrict__ res_out, const T *__restrict__ w,
                                                                   T *__restrict__ out, int hidden, float eps) {
    __shared__ float sh[32];
    const size_t row = blockIdx.x;
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * hidden);
    const uint4 *rr = res_in ? reinterpret_cast<const uint4 *>(res_in + row * hidden) : nullptr;
    const uint4 *wr = reinterpret_cast<const uint4 *>(w);
    const int n8 = hidden / 8;
    uint4 xv[kNormChunks], rv[kNormChunks], wv[kNormChunks];
#pragma unroll
    for (int c = 0; c < kNormChunks; ++c) {
        const int i = threadIdx.x + c * kNormThreads;
        if (i < n8) {
            xv[c] = __ldg(xr + i);
            wv[c] = __ldg(wr + i);
            if (rr) rv[c] = __ldg(rr + i);
        }
    }
    float ss = 0.f;
    float h[kNormChunks][8];
#pragma unroll
    for (int c = 0; c < kNormChunks; ++c) {
        const int i = threadIdx.x + c * kNormThreads;
        if (i >= n8) continue;
        const T *xe = reinterpret_cast<const T *>(&xv[c]);
        const T *re = reinterpret_cast<const T *>(&rv[c]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float v = tof(xe[j]);
            if (rr) v = tof(fromf<T>(v + tof(re[j])));
            h[c][j] = v;
            ss += v * v;
        }
    }
    const float inv = rsqrtf(block_sum(ss, sh) / (float)hidden + eps);
#pragma unroll
    for (int c = 0; c < kNormChunks; ++c) {
        const int i = threadIdx.x + c * kNormThreads;
        if (i >= n8) continue;
        const T *we = reinterpret_cast<const T *>(&wv[c]);
        uint4 o, hr;
        T *oe = reinterpret_cast<T *>(&o);
        T *he = reinterpret_cast<T *>(&hr);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            he[j] = fromf<T>(h[c][j]);
            oe[j] = fromf<T>(tof(we[j]) * tof(fromf<T>(h[c][j] * inv)));
        }
        reinterpret_cast<uint4 *>(out + row * hidden)[i] = o;
        if (res_out) reinterpret_cast<uint4 *>(res_out + row * hidden)[i] = rr ? hr : xv[c];
    }
}

// Scalar fallback for rows that are not 16-byte aligned or longer than the vector path.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T *__restrict__ x, const T *__restrict__ res_in,
                                                      T *__restrict__ res_out, const T *__restrict__ w,
                                                      T *__restrict__ out, int hidden, float eps) {
    __shared__ float sh[32];
    const size_t row = blockIdx.x;
    x += row * hidden;
    out += row * hidden;
    if (res_in) res_in += row * hidden;
    if (res_out) res_out += row * hidden;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float h = tof(x[i]);
        if (res_in) h = tof(fromf<T>(h + tof(res_in[i])));
        ss += h * h;
    }
    const float inv = rsqrtf(block_sum(ss, sh) / (float)hidden + eps);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float h = tof(x[i]);
        if (res_in) {
            const T hs = fromf<T>(h + tof(res_in[i]));
            h = tof(hs);
            if (res_out) res_out[i] = hs;
        } else if (res_out) {
            res_out[i] = x[i];
        }
        out[i] = fromf<T>(tof(w[i]) * tof(fromf<T>(h * inv)));
    }
}

// ------------------------------------------------------------------ rotary + cache write
// q [n, hq, D], k [n, hkv, D] rotated in place (pairs (i, i + D/2), angle = pos * theta^(-2i/D));
// k, v written to cache[batch][kv head][pos][D].
template <typename T>
__global__ void rope_cache_kernel(T *__restrict__ q, T *__restrict__ k, const T *__restrict__ v,
                                  const int *__restrict__ pos, const int *__restrict__ batch_of, T *__restrict__ kc,
                                  T *__restrict__ vc, int hq, int hkv, int D, int max_seq, float log2_theta) {
    const int tok = blockIdx.y, head = blockIdx.x, i = threadIdx.x;  // i < D/2
    const int p = pos[tok];
    const int half = D / 2;
    const float inv_freq = exp2f(-(2.f * i / (float)D) * log2_theta);
    float sn, cs;
    sincosf((float)p * inv_freq, &sn, &cs);
    const float c = tof(fromf<T>(cs)), s = tof(fromf<T>(sn));
    T *row = head < hq ? q + ((size_t)tok * hq + head) * D : k + ((size_t)tok * hkv + (head - hq)) * D;
    const float a = tof(row[i]), b = tof(row[i + half]);
    const T ra = fromf<T>(a * c - b * s), rb = fromf<T>(b * c + a * s);
    row[i] = ra;
    row[i + half] = rb;
    if (head >= hq && p >= 0 && p < max_seq) {
        const int kh = head - hq;
        const int bb = batch_of ? batch_of[tok] : tok;
        const size_t off = (((size_t)bb * hkv + kh) * max_seq + p) * D;
        kc[off + i] = ra;
        kc[off + i + half] = rb;
        const T *vr = v + ((size_t)tok * hkv + kh) * D;
        vc[off + i] = vr[i];
        vc[off + i + half] = vr[i + half];
    }
}

// ------------------------------------------------------------------ decode attention
// One CTA = (position chunk, kv head, batch row); it serves all `grp` query heads of
// the kv head.  Scores: thread-per-position over the chunk; P.V: thread-per-dimension.
constexpr int kChunk = 256;
constexpr int kAttnThreads = 128;

template <typename T, int D, int GRP>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const T *__restrict__ q, const T *__restrict__ kc,
                                                                  const T *__restrict__ vc,
                                                                  const int *__restrict__ seq_len, float *__restrict__ part,
                                                                  int hkv, int max_seq, int nsplit, float scale) {
    __shared__ float qs[GRP][D];
    __shared__ float sc[GRP][kChunk];
    __shared__ float red[GRP][kAttnThreads / 32];
    __shared__ float osm[(kAttnThreads / 32) * GRP * D];  // per-warp partial P.V sums
    const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const int hq = hkv * GRP;
    const int L = seq_len[b];
    const int p0 = split * kChunk, p1 = min(p0 + kChunk, L);
    float *po = part + (((size_t)b * hq + (size_t)kh * GRP) * nsplit + split) * (D + 2);
    if (p0 >= p1) {  // empty chunk
        for (int g = 0; g < GRP; ++g)
            if (threadIdx.x == 0) {
                float *pg = po + (size_t)g * nsplit * (D + 2);
                pg[D] = -FLT_MAX;
                pg[D + 1] = 0.f;
            }
        return;
    }
    for (int i = threadIdx.x; i < GRP * D; i += kAttnThreads) {
        const int g = i / D, d = i - g * D;
        qs[g][d] = tof(q[((size_t)b * hq + kh * GRP + g) * D + d]) * scale;
    }
    __syncthreads();
    const T *kb = kc + (((size_t)b * hkv + kh) * max_seq) * D;
    const T *vb = vc + (((size_t)b * hkv + kh) * max_seq) * D;
    for (int pp = threadIdx.x; pp < kChunk; pp += kAttnThreads) {
        const int p = p0 + pp;
        float acc[GRP];
#pragma unroll
        for (int g = 0; g < GRP; ++g) acc[g] = 0.f;
        if (p < p1) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(kb + (size_t)p * D);
#pragma unroll 4
            for (int c = 0; c < D / 8; ++c) {
                const uint4 u = __ldg(kr + c);
                const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float kv = tof(e[j]);
#pragma unroll
                    for (int g = 0; g < GRP; ++g) acc[g] += kv * qs[g][8 * c + j];
                }
            }
        }
#pragma unroll
        for (int g = 0; g < GRP; ++g) sc[g][pp] = (p < p1) ? acc[g] : -FLT_MAX;
    }
    __syncthreads();
    // per head: max and sum of exp over the chunk
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    float m[GRP];
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        float v = -FLT_MAX;
        for (int pp = threadIdx.x; pp < kChunk; pp += kAttnThreads) v = fmaxf(v, sc[g][pp]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (l == 0) red[g][w] = v;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        float v = red[g][0];
        for (int i = 1; i < kAttnThreads / 32; ++i) v = fmaxf(v, red[g][i]);
        m[g] = v;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        float s = 0.f;
        for (int pp = threadIdx.x; pp < kChunk; pp += kAttnThreads) {
            const float e = (p0 + pp < p1) ? expf(sc[g][pp] - m[g]) : 0.f;
            sc[g][pp] = e;
            s += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (l == 0) red[g][w] = s;
    }
    __syncthreads();
    // P.V: warp w takes positions p0 + w, p0 + w + 4, ...; lane l holds dimensions 4l..4l+3
    // (8-byte coalesced loads), then the four warps' partial sums meet in shared memory.
    static_assert(D == 128 && kAttnThreads == 128, "P.V layout assumes 4 warps x 32 lanes x 4 dims");
    float o[GRP][4];
#pragma unroll
    for (int g = 0; g < GRP; ++g) o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
#pragma unroll 4
    for (int p = p0 + w; p < p1; p += kAttnThreads / 32) {
        const uint2 u = __ldg(reinterpret_cast<const uint2 *>(vb + (size_t)p * D) + l);
        const T *e = reinterpret_cast<const T *>(&u);
        const float v0 = tof(e[0]), v1 = tof(e[1]), v2 = tof(e[2]), v3 = tof(e[3]);
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            const float pw = sc[g][p - p0];
            o[g][0] += pw * v0;
            o[g][1] += pw * v1;
            o[g][2] += pw * v2;
            o[g][3] += pw * v3;
        }
    }
#pragma unroll
    for (int g = 0; g < GRP; ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i) osm[(w * GRP + g) * D + 4 * l + i] = o[g][i];
    __syncthreads();
    for (int i = threadIdx.x; i < GRP * D; i += kAttnThreads) {
        const int g = i / D, d = i - g * D;
        float acc = 0.f;
#pragma unroll
        for (int ww = 0; ww < kAttnThreads / 32; ++ww) acc += osm[(ww * GRP + g) * D + d];
        po[(size_t)g * nsplit * (D + 2) + d] = acc;
    }
    if (threadIdx.x == 0) {
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            float s = 0.f;
            for (int i = 0; i < kAttnThreads / 32; ++i) s += red[g][i];
            float *pg = po + (size_t)g * nsplit * (D + 2);
            pg[D] = m[g];
            pg[D + 1] = s;
        }
    }
}

template <typename T, int D>
__global__ void __launch_bounds__(D) attn_combine_kernel(const float *__restrict__ part, T *__restrict__ out, int hq,
                                                         int nsplit) {
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const float *ph = part + ((size_t)b * hq + h) * nsplit * (D + 2);
    float M = -FLT_MAX;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ph[(size_t)s * (D + 2) + D]);
    float num = 0.f, den = 0.f;
    for (int s = 0; s < nsplit; ++s) {
        const float *ps = ph + (size_t)s * (D + 2);
        const float l = ps[D + 1];
        if (l <= 0.f) continue;
        const float wgt = expf(ps[D] - M);
        num += wgt * ps[d];
        den += wgt * l;
    }
    out[((size_t)b * hq + h) * D + d] = fromf<T>(den > 0.f ? num / den : 0.f);
}

// ------------------------------------------------------------------ SwiGLU
template <typename T>
__global__ void silu_mul_kernel(const T *__restrict__ gate, const T *__restrict__ up, T *__restrict__ out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float g = tof(gate[i]);
        const T s = fromf<T>(g / (1.f + expf(-g)));
        out[i] = fromf<T>(tof(s) * tof(up[i]));
    }
}

static int sm_count() {
    int dev = 0;
    cudaGetDevice(&dev);
    return device_info(dev).sms > 0 ? device_info(dev).sms : 148;
}

}  // namespace dec
}  // namespace nq

extern "C" {

int nq_rmsnorm(int dtype, const void *x, const void *residual_in, void *residual_out, const void *weight, void *out,
               int64_t rows, int64_t hidden, float eps, void *stream) {
    using namespace nq;
    if (!x || !weight || !out || rows <= 0 || hidden <= 0) return fail(NQ_ERR_INVALID_ARGUMENT, "bad rmsnorm args");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec = hidden % 8 == 0 && hidden <= 8 * dec::kNormThreads * dec::kNormChunks &&
                     (((uintptr_t)x | (uintptr_t)residual_in | (uintptr_t)residual_out | (uintptr_t)weight |
                       (uintptr_t)out) & 15) == 0;
    if (vec && dtype == NQ_DTYPE_F16)
        dec::rmsnorm_vec_kernel<__half><<<(unsigned)rows, dec::kNormThreads, 0, s>>>(
            (const __half *)x, (const __half *)residual_in, (__half *)residual_out, (const __half *)weight,
            (__half *)out, (int)hidden, eps);
    else if (vec && dtype == NQ_DTYPE_BF16)
        dec::rmsnorm_vec_kernel<__nv_bfloat16><<<(unsigned)rows, dec::kNormThreads, 0, s>>>(
            (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)residual_in, (__nv_bfloat16 *)residual_out,
            (const __nv_bfloat16 *)weight, (__nv_bfloat16 *)out, (int)hidden, eps);
    else if (dtype == NQ_DTYPE_F16)
        dec::rmsnorm_kernel<__half><<<(unsigned)rows, 256, 0, s>>>(
            (const __half *)x, (const __half *)residual_in, (__half *)residual_out, (const __half *)weight,
            (__half *)out, (int)hidden, eps);
    else if (dtype == NQ_DTYPE_BF16)
        dec::rmsnorm_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, s>>>(
            (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)residual_in, (__nv_bfloat16 *)residual_out,
            (const __nv_bfloat16 *)weight, (__nv_bfloat16 *)out, (int)hidden, eps);
    else
        return fail(NQ_ERR_UNSUPPORTED, "dtype");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "rmsnorm launch");
}

int nq_rope_cache(int dtype, void *q, void *k, const void *v, const int32_t *positions, const int32_t *batch_of,
                  void *k_cache, void *v_cache, int64_t n_tokens, int64_t hq, int64_t hkv, int64_t head_dim,
                  int64_t max_seq, float theta, void *stream) {
    using namespace nq;
    if (!q || !k || !v || !positions || !k_cache || !v_cache || n_tokens <= 0 || hq <= 0 || hkv <= 0)
        return fail(NQ_ERR_INVALID_ARGUMENT, "bad rope_cache args");
    if (head_dim % 2 || head_dim > 1024) return fail(NQ_ERR_UNSUPPORTED, "head_dim must be even and <= 1024");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    dim3 grid((unsigned)(hq + hkv), (unsigned)n_tokens);
    const float l2t = log2f(theta);
    if (dtype == NQ_DTYPE_F16)
        dec::rope_cache_kernel<__half><<<grid, (unsigned)(head_dim / 2), 0, s>>>(
            (__half *)q, (__half *)k, (const __half *)v, positions, batch_of, (__half *)k_cache, (__half *)v_cache,
            (int)hq, (int)hkv, (int)head_dim, (int)max_seq, l2t);
    else if (dtype == NQ_DTYPE_BF16)
        dec::rope_cache_kernel<__nv_bfloat16><<<grid, (unsigned)(head_dim / 2), 0, s>>>(
            (__nv_bfloat16 *)q, (__nv_bfloat16 *)k, (const __nv_bfloat16 *)v, positions, batch_of,
            (__nv_bfloat16 *)k_cache, (__nv_bfloat16 *)v_cache, (int)hq, (int)hkv, (int)head_dim, (int)max_seq, l2t);
    else
        return fail(NQ_ERR_UNSUPPORTED, "dtype");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "rope_cache launch");
}

size_t nq_decode_attention_workspace_bytes(int64_t batch, int64_t hq, int64_t head_dim, int64_t max_seq) {
    const int64_t nsplit = (max_seq + nq::dec::kChunk - 1) / nq::dec::kChunk;
    return (size_t)batch * hq * nsplit * (head_dim + 2) * sizeof(float);
}

int nq_decode_attention(int dtype, const void *q, const void *k_cache, const void *v_cache, const int32_t *seq_len,
                        void *out, int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim, int64_t max_seq,
                        void *workspace, size_t workspace_bytes, void *stream) {
    using namespace nq;
    using namespace nq::dec;
    if (!q || !k_cache || !v_cache || !seq_len || !out || batch <= 0 || hq <= 0 || hkv <= 0 || max_seq <= 0)
        return fail(NQ_ERR_INVALID_ARGUMENT, "bad decode_attention args");
    if (head_dim != 128) return fail(NQ_ERR_UNSUPPORTED, "decode attention supports head_dim 128");
    if (hq % hkv) return fail(NQ_ERR_INVALID_ARGUMENT, "query heads must be a multiple of kv heads");
    const int grp = (int)(hq / hkv);
    const size_t need = nq_decode_attention_workspace_bytes(batch, hq, head_dim, max_seq);
    if (!workspace || workspace_bytes < need) return fail(NQ_ERR_WORKSPACE, "attention workspace needs %zu bytes", need);
    if (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15) return fail(NQ_ERR_INVALID_ARGUMENT, "caches must be 16B aligned");
    const int nsplit = (int)((max_seq + kChunk - 1) / kChunk);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    dim3 grid((unsigned)nsplit, (unsigned)hkv, (unsigned)batch);
    const float scale = 1.0f / sqrtf((float)head_dim);
    float *part = static_cast<float *>(workspace);
#define NQ_ATTN(TT, G)                                                                                        \
    attn_split_kernel<TT, 128, G><<<grid, kAttnThreads, 0, s>>>((const TT *)q, (const TT *)k_cache,           \
                                                                 (const TT *)v_cache, seq_len, part, (int)hkv, \
                                                                 (int)max_seq, nsplit, scale)
#define NQ_ATTN_DT(TT)                                     \
    switch (grp) {                                         \
        case 1: NQ_ATTN(TT, 1); break;                     \
        case 2: NQ_ATTN(TT, 2); break;                     \
        case 4: NQ_ATTN(TT, 4); break;                     \
        case 8: NQ_ATTN(TT, 8); break;                     \
        default: return fail(NQ_ERR_UNSUPPORTED, "GQA group %d not in {1,2,4,8}", grp); \
    }
    if (dtype == NQ_DTYPE_F16) {
        NQ_ATTN_DT(__half)
        attn_combine_kernel<__half, 128><<<dim3((unsigned)hq, (unsigned)batch), 128, 0, s>>>(part, (__half *)out,
                                                                                          (int)hq, nsplit);
    } else if (dtype == NQ_DTYPE_BF16) {
        NQ_ATTN_DT(__nv_bfloat16)
        attn_combine_kernel<__nv_bfloat16, 128><<<dim3((unsigned)hq, (unsigned)batch), 128, 0, s>>>(
            part, (__nv_bfloat16 *)out, (int)hq, nsplit);
    } else {
        return fail(NQ_ERR_UNSUPPORTED, "dtype");
    }
#undef NQ_ATTN_DT
#undef NQ_ATTN
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "decode attention launch");
}

int nq_silu_mul(int dtype, const void *gate, const void *up, void *out, int64_t n, void *stream) {
    using namespace nq;
    if (!gate || !up || !out || n <= 0) return fail(NQ_ERR_INVALID_ARGUMENT, "bad silu_mul args");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = (int64_t)dec::sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (dtype == NQ_DTYPE_F16)
        dec::silu_mul_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>((const __half *)gate, (const __half *)up,
                                                                      (__half *)out, (size_t)n);
    else if (dtype == NQ_DTYPE_BF16)
        dec::silu_mul_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(
            (const __nv_bfloat16 *)gate, (const __nv_bfloat16 *)up, (__nv_bfloat16 *)out, (size_t)n);
    else
        return fail(NQ_ERR_UNSUPPORTED, "dtype");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "silu_mul launch");
}

}  // extern "C"
