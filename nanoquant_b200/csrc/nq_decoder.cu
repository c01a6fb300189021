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
#include <algorithm>
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
    pdl_launch_dependents();
    pdl_wait();
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
// k, v written to cache[batch][kv head][pos][D].  One CTA per token: thread (i, g) computes the
// angle of pair i once and rotates that pair in heads g, g + G, ... (G = blockDim.x / (D/2)).
template <typename T>
__global__ void rope_cache_kernel(T *__restrict__ q, T *__restrict__ k, const T *__restrict__ v,
                                  const int *__restrict__ pos, const int *__restrict__ batch_of, T *__restrict__ kc,
                                  T *__restrict__ vc, int hq, int hkv, int D, int max_seq, float log2_theta) {
    const int half = D / 2;
    const int tok = blockIdx.x, i = threadIdx.x % half, g0 = threadIdx.x / half, G = blockDim.x / half;
    const int p = pos[tok];
    const float inv_freq = exp2f(-(2.f * i / (float)D) * log2_theta);
    float sn, cs;
    sincosf((float)p * inv_freq, &sn, &cs);
    const float c = tof(fromf<T>(cs)), s = tof(fromf<T>(sn));
    const int bb = batch_of ? batch_of[tok] : tok;
    for (int head = g0; head < hq + hkv; head += G) {
        T *row = head < hq ? q + ((size_t)tok * hq + head) * D : k + ((size_t)tok * hkv + (head - hq)) * D;
        const float a = tof(row[i]), b = tof(row[i + half]);
        const T ra = fromf<T>(a * c - b * s), rb = fromf<T>(b * c + a * s);
        row[i] = ra;
        row[i + half] = rb;
        if (head >= hq && p >= 0 && p < max_seq) {
            const int kh = head - hq;
            const size_t off = (((size_t)bb * hkv + kh) * max_seq + p) * D;
            kc[off + i] = ra;
            kc[off + i + half] = rb;
            const T *vr = v + ((size_t)tok * hkv + kh) * D;
            vc[off + i] = vr[i];
            vc[off + i + half] = vr[i + half];
        }
    }
}

// ------------------------------------------------------------------ decode attention
// One CTA = (chunk of positions, kv head, batch row); it serves the `GRP` query heads of the
// kv head.  A chunk is `nsub` sub-blocks of kSub positions; each sub-block's K and V rows are
// contiguous in the cache, so one thread brings them into a two-stage shared-memory ring with
// two bulk copies and every byte of the chunk is in flight at once.  Softmax is online over the
// sub-blocks.  The chunk's partial (unnormalised output, max, sum of exponentials) goes to the
// workspace; the CTA that finishes last for its (batch row, kv head) -- found with an atomic
// counter that it resets afterwards -- combines the partials and writes the output, so there
// is no second launch.  A head whose sequence fits one chunk writes its output directly.
//
// ROPE = true fuses the rotary embedding and the cache write of the new position (the work of
// rope_cache_kernel, same arithmetic and roundings): every CTA rotates q itself, and the CTA
// whose chunk holds position pos[b] rotates k, writes k and v to the caches, and patches its
// shared-memory copy of that row.  The sequence length is then pos[b] + 1.
constexpr int kSub = 64;           // positions per sub-block (one ring stage)
constexpr int kAttnThreads = 256;  // 8 warps
constexpr int kMaxChunks = 64;     // chunk length grows with max_seq to keep at most this many
constexpr int kHeadDim = 128;
constexpr int kAttnMaxStages = 12;  // copy ring depth limit (sub-blocks of K or V in flight)
constexpr int kAttnCtasPerSm = 4;   // chunks per head are sized for about this many CTAs per SM
constexpr size_t kAttnScoreBytes = 48 * 1024;  // per-chunk score buffer limit (GRP x chunk x 4 B)
constexpr int kClusterChunks = 8;  // chunks of one head combined through distributed shared memory

struct AttnParams {
    const void *q;      // [batch, hq, D]; already rotated unless ROPE
    const void *k_new;  // ROPE: [batch, hkv, D] (not rotated yet)
    const void *v_new;  // ROPE: [batch, hkv, D]
    const int *pos;     // ROPE: position of the new row per batch row
    const int *seq_len; // !ROPE: attended positions per batch row
    void *kc, *vc;      // [batch][hkv][max_seq][D]
    void *out;          // [batch, hq, D]
    Ctrl *ctrl;         // status
    unsigned *count;    // [batch][hkv] arrival counters, zero between launches
    float *part;        // [batch][hq][nchunk][D + 2]
    int hkv, max_seq, nchunk, nsub, nst;
    int cl;             // chunks of a head combined in a cluster (nchunk <= kClusterChunks)
    int ncl;            // cluster size (a power of two >= nchunk) when cl
    int qsplit;         // CTAs sharing one kv head's chunk, each with GRP of its hq / hkv query heads
    float scale, log2_theta;
};

template <typename T>
__device__ __forceinline__ float2 f2_of(uint32_t w);
template <>
__device__ __forceinline__ float2 f2_of<__half>(uint32_t w) {
    return __half22float2(*reinterpret_cast<__half2 *>(&w));
}
template <>
__device__ __forceinline__ float2 f2_of<__nv_bfloat16>(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162 *>(&w));
}

__host__ __device__ constexpr size_t attn_stage_bytes() { return (size_t)kSub * kHeadDim * 2u; }  // K or V, 2-byte types

// Cluster helpers (the chunks of one head combine their partials through distributed shared
// memory; every CTA of a cluster is resident at once, and all reach the cluster barrier).
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store v at the address of `local` in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ void st_cluster_f32(float *local, uint32_t rank, float v) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
// Shared-memory bytes of rank 0's receive buffer for the cluster's partials.
template <int GRP>
__host__ __device__ constexpr size_t attn_recv_bytes() { return (size_t)kClusterChunks * GRP * (kHeadDim + 2) * 4u; }

// CL: the chunks of a head form one cluster (gridDim.x CTAs) and rank 0 combines their partials
// from distributed shared memory; otherwise partials go to the workspace and the CTA that
// finishes last for its head (atomic counter, reset after) combines them.
template <typename T, int GRP, bool ROPE, bool CL>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnParams p) {
    constexpr int D = kHeadDim;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kAttnMaxStages];
    __shared__ float mrow[GRP], lrow[GRP];
    __shared__ float red[kAttnThreads / 32];
    __shared__ int last;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int chunk = blockIdx.x, b = blockIdx.z;
    const int kh = blockIdx.y / p.qsplit, qsub = blockIdx.y - kh * p.qsplit;  // kv head, query-head subgroup
    const int hq = p.hkv * GRP * p.qsplit;
    const int qh0 = (kh * p.qsplit + qsub) * GRP;  // this CTA's first query head
    pdl_launch_dependents();
    // Programmatic dependent launch: the RoPE variant (one decode step) reads the positions and
    // issues its cache copies before waiting for the previous kernel -- the positions change
    // only between steps and the rows before positions[b] were written by earlier steps; the
    // plain variant waits first.
    if (!ROPE) pdl_wait();
    const int pos = ROPE ? p.pos[b] : 0;
    int L = ROPE ? pos + 1 : p.seq_len[b];
    L = min(L, p.max_seq);
    // Chunks of whole 64-position blocks sized from this row's actual length: the CTAs along x
    // share the row's blocks evenly, so none idles while L is below the capacity (the score
    // buffer holds p.nsub blocks, and ceil(blocks / CTAs) never exceeds it), and every block of
    // a chunk starts on a 64-row (16 KB) boundary of the cache.
    const int nch = (int)gridDim.x;
    const int spc = max(1, ((L + kSub - 1) / kSub + nch - 1) / nch);
    const int clen = spc * kSub;
    const int c0 = chunk * clen;
    const int c1 = max(c0, min(c0 + clen, L));
    const bool active = c1 > c0;
    T *out = static_cast<T *>(p.out) + ((size_t)b * hq + (size_t)qh0) * D;
    if (!CL) {
        if (L <= 0) {  // nothing to attend to: zeros, written once
            if (ROPE) pdl_wait();
            if (chunk == 0)
                for (int i = tid; i < GRP * D; i += kAttnThreads) out[i] = fromf<T>(0.f);
            return;
        }
        if (!active) return;  // beyond the sequence: no partial, not counted
    }
    // (in a cluster every CTA stays to the end; one past the sequence contributes nothing)
    const int nact = L > 0 ? (L + clen - 1) / clen : 0;
    const int npos = c1 - c0;                               // positions of this chunk
    const int nsb = active ? (npos + kSub - 1) / kSub : 0;  // 64-position sub-blocks
    const int nst = p.nst;                                  // ring stages of one sub-block of K or V
    const size_t head_row0 = ((size_t)b * p.hkv + kh) * (size_t)p.max_seq;
    const T *kg = static_cast<const T *>(p.kc) + head_row0 * D;
    const T *vg = static_cast<const T *>(p.vc) + head_row0 * D;
    T *qsm = reinterpret_cast<T *>(smem + nst * attn_stage_bytes());
    float *sc = reinterpret_cast<float *>(qsm + GRP * D);  // [GRP][clen]: scores, then P

    // Copy items 0 .. 2 nsb - 1: the chunk's K sub-blocks, then its V sub-blocks.
    auto issue = [&](int it) {  // thread 0
        const bool isv = it >= nsb;
        const int sb = isv ? it - nsb : it;
        const int r0 = c0 + sb * kSub, nr = min(kSub, c1 - r0);
        const int st = it % nst;
        const uint32_t bytes = (uint32_t)nr * D * (uint32_t)sizeof(T);
        mbar_arrive_expect_tx(&bars[st], bytes);
        bulk_g2s(smem + st * attn_stage_bytes(), (isv ? vg : kg) + (size_t)r0 * D, bytes, &bars[st]);
    };
    if (tid == 0) {
        for (int i = 0; i < kAttnMaxStages; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
        for (int it = 0; it < nst && it < 2 * nsb; ++it) issue(it);
    }
    if (tid < GRP) {  // an empty chunk's partial: no mass (a cluster combine weights it 0)
        mrow[tid] = -INFINITY;
        lrow[tid] = 0.f;
    }
    if (ROPE) pdl_wait();  // q, k and v of this step come from the previous kernel
    // q (rotated here when ROPE) into shared memory; the owner of the new row rotates k too.
    const bool owner = ROPE && L > 0 && pos >= 0 && pos < p.max_seq && (L - 1) / clen == chunk;
    T knew_a = fromf<T>(0.f), knew_b = knew_a, vnew_a = knew_a, vnew_b = knew_a;
    const T *qg = static_cast<const T *>(p.q) + ((size_t)b * hq + (size_t)qh0) * D;
    if (ROPE) {
        if (tid < D / 2) {
            const int j = tid;
            const float inv_freq = exp2f(-(2.f * j / (float)D) * p.log2_theta);
            float sn, cs;
            sincosf((float)pos * inv_freq, &sn, &cs);
            const float c = tof(fromf<T>(cs)), s = tof(fromf<T>(sn));
#pragma unroll
            for (int g = 0; g < GRP; ++g) {
                const float a = tof(qg[g * D + j]), bb = tof(qg[g * D + j + D / 2]);
                qsm[g * D + j] = fromf<T>(a * c - bb * s);
                qsm[g * D + j + D / 2] = fromf<T>(bb * c + a * s);
            }
            if (owner) {
                const size_t kv = ((size_t)b * p.hkv + kh) * D;
                const T *kn = static_cast<const T *>(p.k_new) + kv;
                const T *vn = static_cast<const T *>(p.v_new) + kv;
                const float a = tof(kn[j]), bb = tof(kn[j + D / 2]);
                knew_a = fromf<T>(a * c - bb * s);
                knew_b = fromf<T>(bb * c + a * s);
                vnew_a = vn[j];
                vnew_b = vn[j + D / 2];
                if (qsub == 0) {  // one writer per kv head; every subgroup patches its own copy
                    T *kd = static_cast<T *>(p.kc) + (head_row0 + pos) * D;
                    T *vd = static_cast<T *>(p.vc) + (head_row0 + pos) * D;
                    kd[j] = knew_a;
                    kd[j + D / 2] = knew_b;
                    vd[j] = vnew_a;
                    vd[j + D / 2] = vnew_b;
                }
            }
        }
    } else {
        for (int i = tid; i < GRP * D; i += kAttnThreads) qsm[i] = qg[i];
    }
    __syncthreads();

    const int rnew = owner ? (L - 1) - c0 : -1;  // chunk row of the new position
    // ---- phase 1: scores of every position of the chunk (four threads per position, 16-byte
    // chunks in a rotated order so a warp's reads spread over all banks, two accumulators)
    const int pp = tid >> 2, qd = tid & 3;
    for (int it = 0; it < nsb; ++it) {
        const int nv = min(kSub, npos - it * kSub);
        T *ks = reinterpret_cast<T *>(smem + (it % nst) * attn_stage_bytes());
        mbar_wait(&bars[it % nst], (uint32_t)(it / nst) & 1u, &p.ctrl->status);
        if (rnew >= it * kSub && rnew < it * kSub + kSub) {  // the new key row, as written to the cache
            if (tid < D / 2) {
                ks[(rnew - it * kSub) * D + tid] = knew_a;
                ks[(rnew - it * kSub) * D + tid + D / 2] = knew_b;
            }
            __syncthreads();
        }
        float acc[GRP][2];
#pragma unroll
        for (int g = 0; g < GRP; ++g) acc[g][0] = acc[g][1] = 0.f;
        if (pp < nv) {
            const T *kr = ks + pp * D + qd * 32;
            const T *qr = qsm + qd * 32;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int c8 = 8 * ((cc + pp) & 3);
                const uint4 kv = *reinterpret_cast<const uint4 *>(kr + c8);
                const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                for (int g = 0; g < GRP; ++g) {
                    const uint4 qv = *reinterpret_cast<const uint4 *>(qr + g * D + c8);
                    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 kf = f2_of<T>(kw[e]), qf = f2_of<T>(qw[e]);
                        acc[g][e & 1] = fmaf(kf.x, qf.x, acc[g][e & 1]);
                        acc[g][e & 1] = fmaf(kf.y, qf.y, acc[g][e & 1]);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            float a = acc[g][0] + acc[g][1];
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            a += __shfl_xor_sync(0xffffffffu, a, 2);
            if (qd == 0 && pp < nv) sc[g * clen + it * kSub + pp] = a * p.scale;
        }
        __syncthreads();  // the stage is free again
        if (tid == 0 && it + nst < 2 * nsb) {
            fence_proxy_async_smem();
            issue(it + nst);
        }
    }
    // ---- phase 2: one softmax per head over the whole chunk: P = e^(s - m), l = sum P.  The
    // heads run side by side, kAttnThreads / 32 / GRP warps each, so a GQA group costs three
    // block barriers in all rather than four per head.
    {
        constexpr int kWph = kAttnThreads / 32 / GRP;  // warps per head
        const int g = w / kWph, wi = w - g * kWph;
        const int tl = wi * 32 + lane;
        float mx = -INFINITY;
        for (int i = tl; i < npos; i += kWph * 32) mx = fmaxf(mx, sc[g * clen + i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        if (lane == 0) red[w] = mx;
        __syncthreads();
        float m = red[g * kWph];
#pragma unroll
        for (int j = 1; j < kWph; ++j) m = fmaxf(m, red[g * kWph + j]);
        float sm = 0.f;
        for (int i = tl; i < npos; i += kWph * 32) {
            const float e = expf(sc[g * clen + i] - m);
            sc[g * clen + i] = e;
            sm += e;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
        __syncthreads();  // every warp has read the maxima before red is reused
        if (lane == 0) red[w] = sm;
        __syncthreads();
        if (wi == 0 && lane == 0 && npos > 0) {  // an empty chunk keeps m = -inf, l = 0
            float l = 0.f;
#pragma unroll
            for (int j = 0; j < kWph; ++j) l += red[g * kWph + j];
            mrow[g] = m;
            lrow[g] = l;
        }
        __syncthreads();
    }
    // ---- phase 3: P.V over the V sub-blocks (half2 of V per thread, four position groups)
    const int dp = tid & 63, pg = tid >> 6;
    float o[GRP][2];
#pragma unroll
    for (int g = 0; g < GRP; ++g) o[g][0] = o[g][1] = 0.f;
    for (int it = nsb; it < 2 * nsb; ++it) {
        const int sb = it - nsb;
        const int nv = min(kSub, npos - sb * kSub);
        T *vs = reinterpret_cast<T *>(smem + (it % nst) * attn_stage_bytes());
        mbar_wait(&bars[it % nst], (uint32_t)(it / nst) & 1u, &p.ctrl->status);
        if (rnew >= sb * kSub && rnew < sb * kSub + kSub) {  // the new value row
            if (tid < D / 2) {
                vs[(rnew - sb * kSub) * D + tid] = vnew_a;
                vs[(rnew - sb * kSub) * D + tid + D / 2] = vnew_b;
            }
            __syncthreads();
        }
        const uint32_t *vw = reinterpret_cast<const uint32_t *>(vs) + dp;
        const float *pb = sc + sb * kSub;
#pragma unroll 4
        for (int q2 = pg; q2 < nv; q2 += 4) {
            const float2 v = f2_of<T>(vw[q2 * (D / 2)]);
#pragma unroll
            for (int g = 0; g < GRP; ++g) {
                const float pw = pb[g * clen + q2];
                o[g][0] = fmaf(pw, v.x, o[g][0]);
                o[g][1] = fmaf(pw, v.y, o[g][1]);
            }
        }
        __syncthreads();  // the stage is free again
        if (tid == 0 && it + nst < 2 * nsb) {
            fence_proxy_async_smem();
            issue(it + nst);
        }
    }
    // the four position groups meet in shared memory (stage 0 is free: no copy in flight)
    float *osm = reinterpret_cast<float *>(smem);  // [3][GRP][D]
    if (pg > 0)
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            osm[((pg - 1) * GRP + g) * D + 2 * dp] = o[g][0];
            osm[((pg - 1) * GRP + g) * D + 2 * dp + 1] = o[g][1];
        }
    __syncthreads();
    if (pg == 0)
#pragma unroll
        for (int g = 0; g < GRP; ++g)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                o[g][0] += osm[(q * GRP + g) * D + 2 * dp];
                o[g][1] += osm[(q * GRP + g) * D + 2 * dp + 1];
            }
    if (CL) {
        // every chunk stores its partial (unnormalised o, max, sum) straight into rank 0's
        // receive buffer [gridDim.x][GRP][D + 2]; one cluster barrier (release / acquire)
        // publishes them, and rank 0 combines from its own shared memory
        float *recv = reinterpret_cast<float *>(smem + nst * attn_stage_bytes() + GRP * D * sizeof(T) +
                                                (size_t)GRP * p.nsub * kSub * sizeof(float));
        const uint32_t me = cluster_rank();
        if (pg == 0)
#pragma unroll
            for (int g = 0; g < GRP; ++g) {
                float *dst = recv + ((size_t)me * GRP + g) * (D + 2);
                st_cluster_f32(dst + 2 * dp, 0, o[g][0]);
                st_cluster_f32(dst + 2 * dp + 1, 0, o[g][1]);
                if (dp == 0) {
                    st_cluster_f32(dst + D, 0, mrow[g]);
                    st_cluster_f32(dst + D + 1, 0, lrow[g]);
                }
            }
        cluster_sync_all();
        if (me == 0 && tid < D) {
            for (int g = 0; g < GRP; ++g) {
                float M = -INFINITY;
#pragma unroll
                for (int c = 0; c < (int)gridDim.x; ++c) M = fmaxf(M, recv[(c * GRP + g) * (D + 2) + D]);
                float num = 0.f, den = 0.f;
#pragma unroll
                for (int c = 0; c < (int)gridDim.x; ++c) {
                    const float *pc = recv + (c * GRP + g) * (D + 2);
                    const float lc = pc[D + 1], mc = pc[D];
                    const float wc = lc > 0.f ? expf(mc - M) : 0.f;
                    den = fmaf(wc, lc, den);
                    num = fmaf(wc, pc[tid], num);
                }
                out[g * D + tid] = fromf<T>(den > 0.f ? num / den : 0.f);
            }
        }
        return;
    }
    float *pbase = p.part + ((size_t)b * hq + (size_t)qh0) * p.nchunk * (D + 2);
    if (nact == 1) {  // the whole sequence was this chunk
        if (pg == 0)
#pragma unroll
            for (int g = 0; g < GRP; ++g) {
                const float inv = 1.f / lrow[g];
                out[g * D + 2 * dp] = fromf<T>(o[g][0] * inv);
                out[g * D + 2 * dp + 1] = fromf<T>(o[g][1] * inv);
            }
        return;
    }
    if (pg == 0)
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            float *pc = pbase + ((size_t)g * p.nchunk + chunk) * (D + 2);
            *reinterpret_cast<float2 *>(pc + 2 * dp) = make_float2(o[g][0], o[g][1]);
            if (dp == 0) *reinterpret_cast<float2 *>(pc + D) = make_float2(mrow[g], lrow[g]);
        }
    __threadfence();
    __syncthreads();
    unsigned *cnt = p.count + (size_t)b * p.hkv * p.qsplit + blockIdx.y;
    if (tid == 0) last = atomicAdd(cnt, 1u) == (unsigned)(nact - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // combine: out = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c  (nact <= kMaxChunks = 64).
    // One warp per head forms the chunk weights (lanes hold chunks lane and lane + 32); then every
    // thread takes output values (head, dim) and sums the chunks' partials with independent loads,
    // so the heads of a GQA group are combined at once rather than one after another.
    float *cw = reinterpret_cast<float *>(smem);  // [GRP][kMaxChunks] weights (the copy ring is idle)
    float *cden = cw + GRP * kMaxChunks;          // [GRP] sum_c e^(m_c - M) l_c
    for (int g = w; g < GRP; g += kAttnThreads / 32) {
        const float *pg_ = pbase + (size_t)g * p.nchunk * (D + 2);
        float mc[2], lc[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int ci = lane + 32 * j;
            mc[j] = -INFINITY;
            lc[j] = 0.f;
            if (ci < nact) {
                const float2 ml = __ldcg(reinterpret_cast<const float2 *>(pg_ + (size_t)ci * (D + 2) + D));
                mc[j] = ml.x;
                lc[j] = ml.y;
            }
        }
        float mx = fmaxf(mc[0], mc[1]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float den = 0.f;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float wc = lane + 32 * j < nact ? expf(mc[j] - mx) : 0.f;
            cw[g * kMaxChunks + lane + 32 * j] = wc;
            den = fmaf(wc, lc[j], den);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
        if (lane == 0) cden[g] = den;
    }
    __syncthreads();
    for (int i = tid; i < GRP * D; i += kAttnThreads) {
        const int g = i / D, d = i - g * D;
        const float *src = pbase + (size_t)g * p.nchunk * (D + 2) + d;
        const float *wg = cw + g * kMaxChunks;
        // 16 loads in flight per round trip (the weights of chunks >= nact are 0)
        float num = 0.f;
        for (int c0 = 0; c0 < nact; c0 += 16) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = c0 + j < nact ? __ldcg(src + (size_t)(c0 + j) * (D + 2)) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) num = fmaf(wg[c0 + j], v[j], num);
        }
        out[g * D + d] = fromf<T>(num / cden[g]);
    }
    if (tid == 0) *cnt = 0u;
}

// Chunking for a cache of max_seq positions: nsub sub-blocks per chunk, nchunk chunks.
struct AttnChunks {
    int nsub, nchunk;
};
// The most chunks a cache of max_seq positions is ever split into (sizes the workspace).
inline AttnChunks attn_chunks(int64_t max_seq) {
    const int64_t n64 = (max_seq + kSub - 1) / kSub;
    const int64_t nsub = (n64 + kMaxChunks - 1) / kMaxChunks;
    return {(int)nsub, (int)((n64 + nsub - 1) / nsub)};
}
// The chunking of a launch: about two CTAs per SM over (batch rows x kv heads), so every CTA
// streams several sub-blocks through its copy ring; never more chunks than attn_chunks().
// The chunk's scores stay in shared memory, so a chunk is at most kAttnScoreBytes / (grp x 4 B)
// positions; nsub = 0 when max_seq needs longer chunks than that (more than kMaxChunks).
inline AttnChunks attn_chunks_for(int64_t max_seq, int64_t heads_x_batch, int sms, int grp) {
    const int64_t n64 = (max_seq + kSub - 1) / kSub;
    const int64_t target = std::max<int64_t>(1, (kAttnCtasPerSm * (int64_t)sms) / std::max<int64_t>(1, heads_x_batch));
    const int64_t nsub_cap = (int64_t)(kAttnScoreBytes / ((size_t)grp * kSub * sizeof(float)));
    const int64_t nsub_min = attn_chunks(max_seq).nsub;
    if (nsub_min > nsub_cap) return {0, 0};
    const int64_t nsub = std::min(nsub_cap, std::max<int64_t>(nsub_min, (n64 + target - 1) / target));
    return {(int)nsub, (int)((n64 + nsub - 1) / nsub)};
}
inline size_t attn_count_bytes(int64_t batch, int64_t hq) { return ((size_t)batch * hq * 4 + 255) & ~(size_t)255; }

// ------------------------------------------------------------------ SwiGLU
template <typename T>
__global__ void silu_mul_kernel(const T *__restrict__ gate, const T *__restrict__ up, T *__restrict__ out, size_t n) {
    auto one = [&](size_t i) {
        const float g = tof(gate[i]);
        const T s = fromf<T>(g / (1.f + expf(-g)));
        out[i] = fromf<T>(tof(s) * tof(up[i]));
    };
    const size_t stride = (size_t)gridDim.x * blockDim.x, t0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    const bool vec = ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) |
                       reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    size_t done = 0;
    if (vec) {  // eight values per 16-byte access, the same arithmetic per value
        const size_t n8 = n / 8;
        for (size_t c = t0; c < n8; c += stride) {
            const uint4 gv = reinterpret_cast<const uint4 *>(gate)[c], uv = reinterpret_cast<const uint4 *>(up)[c];
            const T *ge = reinterpret_cast<const T *>(&gv), *ue = reinterpret_cast<const T *>(&uv);
            uint4 ov;
            T *oe = reinterpret_cast<T *>(&ov);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float g = tof(ge[j]);
                const T s = fromf<T>(g / (1.f + expf(-g)));
                oe[j] = fromf<T>(tof(s) * tof(ue[j]));
            }
            reinterpret_cast<uint4 *>(out)[c] = ov;
        }
        done = n8 * 8;
    }
    for (size_t i = done + t0; i < n; i += stride) one(i);
}

template <typename T, int GRP, bool ROPE>
cudaError_t launch_attn(const AttnParams &p, int batch, cudaStream_t s) {
    // the ring (>= 2 stages) also holds the final position-group reduction (< 16 KB) once the
    // chunk is done; a cluster launch adds rank 0's receive buffer for the chunks' partials
    const size_t smem = p.nst * attn_stage_bytes() + GRP * kHeadDim * sizeof(T) +
                        (size_t)GRP * p.nsub * kSub * sizeof(float) + (p.cl ? attn_recv_bytes<GRP>() : 0);
    auto fn = p.cl ? attn_decode_kernel<T, GRP, ROPE, true> : attn_decode_kernel<T, GRP, ROPE, false>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.cl ? (unsigned)p.ncl : (unsigned)p.nchunk, (unsigned)(p.hkv * p.qsplit), (unsigned)batch);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (p.cl) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)p.ncl;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

template <bool ROPE>
cudaError_t dispatch_attn(int dtype, int grp, const AttnParams &p, int batch, cudaStream_t s) {
#define NQ_ATTN_GRP(TT)                                          \
    switch (grp) {                                               \
        case 1: return launch_attn<TT, 1, ROPE>(p, batch, s);    \
        case 2: return launch_attn<TT, 2, ROPE>(p, batch, s);    \
        case 4: return launch_attn<TT, 4, ROPE>(p, batch, s);    \
        default: return launch_attn<TT, 8, ROPE>(p, batch, s);   \
    }
    if (dtype == NQ_DTYPE_F16) {
        NQ_ATTN_GRP(__half)
    }
    NQ_ATTN_GRP(__nv_bfloat16)
#undef NQ_ATTN_GRP
}

// Host checks shared by both attention entry points; fills the workspace pointers of p.
static int sm_count();

int attn_prepare(int dtype, int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim, int64_t max_seq,
                 void *workspace, size_t workspace_bytes, AttnParams &p) {
    if (batch <= 0 || hq <= 0 || hkv <= 0 || max_seq <= 0 || max_seq > INT32_MAX)
        return fail(NQ_ERR_INVALID_ARGUMENT, "bad decode_attention sizes");
    if (dtype != NQ_DTYPE_F16 && dtype != NQ_DTYPE_BF16) return fail(NQ_ERR_UNSUPPORTED, "dtype");
    if (head_dim != kHeadDim) return fail(NQ_ERR_UNSUPPORTED, "decode attention supports head_dim 128");
    if (hq % hkv) return fail(NQ_ERR_INVALID_ARGUMENT, "query heads must be a multiple of kv heads");
    const int64_t grp = hq / hkv;
    if (grp != 1 && grp != 2 && grp != 4 && grp != 8)
        return fail(NQ_ERR_UNSUPPORTED, "GQA group %lld not in {1,2,4,8}", (long long)grp);
    if (batch > 65535 || hkv > 65535) return fail(NQ_ERR_UNSUPPORTED, "batch and kv heads must be <= 65535");
    const size_t need = nq_decode_attention_workspace_bytes(batch, hq, head_dim, max_seq);
    if (!workspace || workspace_bytes < need) return fail(NQ_ERR_WORKSPACE, "attention workspace needs %zu bytes", need);
    if (((uintptr_t)workspace) & 255) return fail(NQ_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
    if ((((uintptr_t)p.kc) | ((uintptr_t)p.vc)) & 15) return fail(NQ_ERR_INVALID_ARGUMENT, "caches must be 16B aligned");
    const AttnChunks ch = attn_chunks_for(max_seq, batch * hkv, sm_count(), (int)grp);
    if (ch.nsub == 0)
        return fail(NQ_ERR_UNSUPPORTED, "max_seq %lld needs chunks longer than the %zu-byte score buffer allows",
                    (long long)max_seq, kAttnScoreBytes);
    unsigned char *ws = static_cast<unsigned char *>(workspace);
    p.ctrl = reinterpret_cast<Ctrl *>(ws);
    p.count = reinterpret_cast<unsigned *>(ws + sizeof(Ctrl));
    p.part = reinterpret_cast<float *>(ws + sizeof(Ctrl) + attn_count_bytes(batch, hq));
    p.hkv = (int)hkv;
    p.max_seq = (int)max_seq;
    p.nchunk = ch.nchunk;
    p.nsub = ch.nsub;
    p.cl = ch.nchunk <= kClusterChunks ? 1 : 0;
    p.ncl = 1;
    while (p.ncl < ch.nchunk) p.ncl *= 2;
    // GQA: the query heads of a kv head are split over up to `grp` CTAs per chunk (each reads the
    // chunk's K / V; the second and later reads hit L2) until the grid reaches about four CTAs per
    // SM (70B, L = 2048: 18.6 -> 13.3 us per layer at TP1 against a limit of one CTA per SM)
    int64_t ctas = (int64_t)(p.cl ? p.ncl : ch.nchunk) * hkv * batch;
    p.qsplit = 1;
    while (p.qsplit < grp && ctas * p.qsplit * 2 <= 4 * (int64_t)sm_count()) p.qsplit *= 2;
    ctas *= p.qsplit;
    const int64_t gcta = grp / p.qsplit;  // query heads per CTA
    // ring depth: every sub-block of the chunk in flight if shared memory allows, keeping room
    // for two or four CTAs per SM when the grid needs that many (7B, L = 2048: 12.7 -> 12.3 us
    // with the chunking sized for four CTAs per SM instead of two; L = 4096: 19.2 -> 17.4 us)
    const size_t budget = ctas > 2 * (int64_t)sm_count() ? 54 * 1024 : ctas > sm_count() ? 110 * 1024 : 200 * 1024;
    const size_t fixed = (size_t)gcta * kHeadDim * 2 + (size_t)gcta * ch.nsub * kSub * sizeof(float) +
                         (p.cl ? (size_t)kClusterChunks * gcta * (kHeadDim + 2) * 4 : 0);
    int nst = (int)std::min<int64_t>(kAttnMaxStages, 2 * (int64_t)ch.nsub);
    while (nst > 2 && fixed + (size_t)nst * attn_stage_bytes() > budget) --nst;
    p.nst = nst;
    p.scale = 1.0f / sqrtf((float)head_dim);
    return NQ_OK;
}

// 1-D launch with programmatic dependent launch allowed (the kernel calls pdl_wait itself).
template <typename... KArgs, typename... Args>
void launch_pdl(void (*fn)(KArgs...), unsigned grid, unsigned block, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, fn, static_cast<KArgs>(args)...);
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
        dec::launch_pdl(dec::rmsnorm_vec_kernel<__half>, (unsigned)rows, dec::kNormThreads, s, (const __half *)x,
                        (const __half *)residual_in, (__half *)residual_out, (const __half *)weight, (__half *)out,
                        (int)hidden, eps);
    else if (vec && dtype == NQ_DTYPE_BF16)
        dec::launch_pdl(dec::rmsnorm_vec_kernel<__nv_bfloat16>, (unsigned)rows, dec::kNormThreads, s,
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
    if (n_tokens > INT32_MAX) return fail(NQ_ERR_UNSUPPORTED, "too many tokens");
    // one CTA per token; as many head groups as fit 256 threads (at least one)
    const unsigned block = (unsigned)(head_dim / 2) * (unsigned)std::max<int64_t>(1, 256 / (head_dim / 2));
    const unsigned grid = (unsigned)n_tokens;
    const float l2t = log2f(theta);
    if (dtype == NQ_DTYPE_F16)
        dec::rope_cache_kernel<__half><<<grid, block, 0, s>>>(
            (__half *)q, (__half *)k, (const __half *)v, positions, batch_of, (__half *)k_cache, (__half *)v_cache,
            (int)hq, (int)hkv, (int)head_dim, (int)max_seq, l2t);
    else if (dtype == NQ_DTYPE_BF16)
        dec::rope_cache_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(
            (__nv_bfloat16 *)q, (__nv_bfloat16 *)k, (const __nv_bfloat16 *)v, positions, batch_of,
            (__nv_bfloat16 *)k_cache, (__nv_bfloat16 *)v_cache, (int)hq, (int)hkv, (int)head_dim, (int)max_seq, l2t);
    else
        return fail(NQ_ERR_UNSUPPORTED, "dtype");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "rope_cache launch");
}

size_t nq_decode_attention_workspace_bytes(int64_t batch, int64_t hq, int64_t head_dim, int64_t max_seq) {
    if (batch <= 0 || hq <= 0 || head_dim <= 0 || max_seq <= 0) return 0;
    const nq::dec::AttnChunks ch = nq::dec::attn_chunks(max_seq);
    return sizeof(nq::Ctrl) + nq::dec::attn_count_bytes(batch, hq) +
           (size_t)batch * hq * ch.nchunk * (head_dim + 2) * sizeof(float);
}

int nq_decode_attention(int dtype, const void *q, const void *k_cache, const void *v_cache, const int32_t *seq_len,
                        void *out, int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim, int64_t max_seq,
                        void *workspace, size_t workspace_bytes, void *stream) {
    using namespace nq;
    using namespace nq::dec;
    if (!q || !k_cache || !v_cache || !seq_len || !out) return fail(NQ_ERR_INVALID_ARGUMENT, "bad decode_attention args");
    AttnParams p{};
    p.q = q;
    p.seq_len = seq_len;
    p.kc = const_cast<void *>(k_cache);
    p.vc = const_cast<void *>(v_cache);
    p.out = out;
    const int st = attn_prepare(dtype, batch, hq, hkv, head_dim, max_seq, workspace, workspace_bytes, p);
    if (st != NQ_OK) return st;
    const cudaError_t e =
        dispatch_attn<false>(dtype, (int)(hq / hkv) / p.qsplit, p, (int)batch, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "decode attention launch");
}

int nq_decode_attention_rope(int dtype, const void *q, const void *k, const void *v, const int32_t *positions,
                             void *k_cache, void *v_cache, void *out, int64_t batch, int64_t hq, int64_t hkv,
                             int64_t head_dim, int64_t max_seq, float theta, void *workspace, size_t workspace_bytes,
                             void *stream) {
    using namespace nq;
    using namespace nq::dec;
    if (!q || !k || !v || !positions || !k_cache || !v_cache || !out)
        return fail(NQ_ERR_INVALID_ARGUMENT, "bad decode_attention_rope args");
    if (!(theta > 0.f)) return fail(NQ_ERR_INVALID_ARGUMENT, "theta must be positive");
    AttnParams p{};
    p.q = q;
    p.k_new = k;
    p.v_new = v;
    p.pos = positions;
    p.kc = k_cache;
    p.vc = v_cache;
    p.out = out;
    p.log2_theta = log2f(theta);
    const int st = attn_prepare(dtype, batch, hq, hkv, head_dim, max_seq, workspace, workspace_bytes, p);
    if (st != NQ_OK) return st;
    const cudaError_t e =
        dispatch_attn<true>(dtype, (int)(hq / hkv) / p.qsplit, p, (int)batch, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "decode attention (rope) launch");
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
