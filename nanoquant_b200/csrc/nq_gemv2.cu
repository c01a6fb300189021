// Decode GEMV for batch <= 2 as two lean kernels chained by programmatic dependent launch (sm_100a).
//
// Computes exactly what the fused single-launch GEMV (nq_gemv.cu) computes for a group of up to
// three NanoQuant layers sharing one input:
//   t[b, k] = smid[k] * sum_n sign(V[k, n]) * s2[n] * x'[b, n]       (stage 1 kernel)
//   y[b, m] = clamp(s1[m] * sum_k sign(U[m, k]) * t[b, k])           (stage 2 kernel)
// replacing the reference's two launches (src/nanoquant/kernel/cuda/gemv_kernel.cu:43-301, dispatched
// at :308-429), with x' formed in the stage-1 prologue (RMSNorm with the residual add, x*up,
// SiLU(x)*up) and SiLU applied in the stage-2 epilogue where asked.
//
// Why two kernels and not one with a grid barrier: each launch's CTAs use at most ~113 KB of shared
// memory and 256 threads, so two CTAs fit one SM.  Under programmatic dependent launch the next
// kernel's CTAs then become resident while the current kernel runs and issue their weight copies
// (V or U slabs, scales) before griddepcontrol.wait: the weight stream of every stage overlaps the
// previous stage's compute, and the only serial cost per stage is the dependency itself
// (griddepcontrol.wait returns when the previous grid has completed and flushed).
//
// Stage 1 work is split into units of (16-row tile, K chunk): each tile's 64-column K blocks are
// cut into `nsplit` chunks and the units are spread evenly over the grid, so no CTA idles when a
// layer has fewer tiles than SMs.  Each unit's float32 partial goes to its own slot
// tpart[chunk][b][k] of the workspace; stage 2 sums the nsplit slots in order (deterministic, no
// atomics), multiplies by smid and splits t into bf16 hi + lo (two B columns per batch row).
// Both stages use mma.sync.m16n8k16 with A fragments built in registers from the HALF2 sign words
// (stage 1: A = +-s2 exact in the input dtype, B = x'; stage 2: A = +-1, B = t hi/lo), float32
// accumulation, K blocks of each CTA split evenly over its 8 warps, partials summed in warp order.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "nq_common.cuh"

namespace nq {
namespace gemv2 {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxMembers = 3;
constexpr int kMaxBatch = 2;
constexpr int kMaxSplit = 8;
constexpr int kMaxSegs = 16;  // units (stage 1) / tiles (stage 2) one warp's K range may touch

enum XMode : int { kPlain = NQ_CHAIN_X_PLAIN, kNorm = NQ_CHAIN_X_RMSNORM, kSiluMul = NQ_CHAIN_X_SILU_MUL, kMul = NQ_CHAIN_X_MUL };

struct M1 {
    const void *s2;          // [in]
    const uint32_t *vbits;   // [rank, wv] HALF2
    float *tpart;            // [nsplit][batch][ldt]
    int rank, tiles, tstart; // tstart: first global tile of this member
    int ldt;                 // slot row stride: rank rounded up to 64
};

struct P1 {
    const void *x, *x2, *nw;
    void *res_out;
    float eps;
    int xmode;
    int batch, in_f, wv, kb, in_pad;
    int nm, nsplit, kbc, units;
    int *status;
    uint32_t off_s2, off_x, off_v, off_red;
    int segs;
    M1 m[kMaxMembers];
};

struct M2 {
    const void *smid;        // [rank] or null
    const uint32_t *ubits;   // [out, wu] HALF2
    const void *s1;          // [out]
    void *y;                 // [batch, out]
    const float *tpart;      // [nsplit][batch][ldt]
    int rank, out_f, wu, kb2, tiles, tstart;
    int ldt;                 // slot row stride: rank rounded up to 64 (= kb2 * 64)
};

struct P2 {
    int batch, nm, nsplit, tiles, act;
    int *status;
    uint32_t off_u, off_s1, off_t, off_red;
    int kpad;                // largest member's K padding (multiple of 64)
    int segs;
    M2 m[kMaxMembers];
};

__device__ __forceinline__ int member_of(const int *tstart, int nm, int tile) {
    int l = 0;
    while (l + 1 < nm && tile >= tstart[l + 1]) ++l;
    return l;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
    const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = Elem<T>::to_f(e[j]);
}

__device__ __forceinline__ float block_sum(float v, float *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += sh[i];
    return s;
}

// ------------------------------------------------------------------ stage 1
// Work split: CTA c owns units [U c / G, U (c+1) / G) (unit u = global tile u / nsplit, chunk
// u % nsplit).  Its units cover the contiguous global tiles [gt0, gt1], whose V rows are copied
// (whole rows, one bulk copy per member) into shared memory before griddepcontrol.wait.
template <typename T>
__global__ void __launch_bounds__(kThreads, 2) stage1_kernel(const __grid_constant__ P1 p) {
    using E = Elem<T>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ float sred[kWarps];
    __shared__ int wfirst[kWarps], wlast[kWarps];
    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int u0 = (int)((long long)p.units * c / G), u1 = (int)((long long)p.units * (c + 1) / G);
    const int gt0 = u0 / p.nsplit, gt1 = (u1 - 1) / p.nsplit;  // u1 > u0: the host sizes G <= units
    int tstart[kMaxMembers];
#pragma unroll
    for (int l = 0; l < kMaxMembers; ++l) tstart[l] = l < p.nm ? p.m[l].tstart : 0x7fffffff;

    T *s2s = reinterpret_cast<T *>(smem + p.off_s2);        // [nm][in_pad]
    T *xs = reinterpret_cast<T *>(smem + p.off_x);          // [batch][in_pad]
    uint32_t *vs = reinterpret_cast<uint32_t *>(smem + p.off_v);  // [tiles gt0..gt1][16][wv]
    float *red = reinterpret_cast<float *>(smem + p.off_red);     // [warp][segs][16][2]

    // ---- weight copies (independent of the previous kernel): V rows of the covered tiles, s2
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        uint32_t bytes = 0;
        for (int l = 0; l < p.nm; ++l) {
            const M1 &mb = p.m[l];
            const int a = max(gt0, mb.tstart), b = min(gt1 + 1, mb.tstart + mb.tiles);
            if (a >= b) continue;
            const int r0 = 16 * (a - mb.tstart), r1 = min(16 * (b - mb.tstart), mb.rank);
            bytes += (uint32_t)(r1 - r0) * (uint32_t)p.wv * 4u + (uint32_t)p.in_f * 2u;
        }
        mbar_arrive_expect_tx(&bar, bytes);
        for (int l = 0; l < p.nm; ++l) {
            const M1 &mb = p.m[l];
            const int a = max(gt0, mb.tstart), b = min(gt1 + 1, mb.tstart + mb.tiles);
            if (a >= b) continue;
            const int r0 = 16 * (a - mb.tstart), r1 = min(16 * (b - mb.tstart), mb.rank);
            bulk_g2s_pieces(vs + (size_t)16 * (a - gt0) * p.wv, mb.vbits + (size_t)r0 * p.wv,
                            (uint32_t)(r1 - r0) * (uint32_t)p.wv * 4u, &bar);
            bulk_g2s_pieces(s2s + (size_t)l * p.in_pad, mb.s2, (uint32_t)p.in_f * 2u, &bar);
        }
    }
    // (in_features % 128 == 0 on this path, so x' and s2 need no K padding: in_pad == in_f)

    pdl_wait();  // the previous kernel has completed: x and the transform inputs are visible

    // ---- x' into shared memory (the same roundings as nq_rmsnorm / nq_silu_mul)
    const int n8 = p.in_f / 8;
    for (int b = 0; b < p.batch; ++b) {
        const uint4 *xg = reinterpret_cast<const uint4 *>(static_cast<const T *>(p.x) + (size_t)b * p.in_f);
        const uint4 *x2g = p.x2 ? reinterpret_cast<const uint4 *>(static_cast<const T *>(p.x2) + (size_t)b * p.in_f)
                                : nullptr;
        uint4 *xr = reinterpret_cast<uint4 *>(xs + (size_t)b * p.in_pad);
        if (p.xmode == kNorm) {
            uint4 *ro = (c == 0 && p.res_out)
                            ? reinterpret_cast<uint4 *>(static_cast<T *>(p.res_out) + (size_t)b * p.in_f)
                            : nullptr;
            float ss = 0.f;
            for (int ch = tid; ch < n8; ch += kThreads) {
                uint4 hv = __ldcg(xg + ch);
                float h[8];
                unpack8<T>(hv, h);
                if (x2g) {
                    float r[8];
                    unpack8<T>(__ldcg(x2g + ch), r);
                    T o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        o[e] = E::rn(h[e] + r[e]);
                        h[e] = E::to_f(o[e]);
                    }
                    hv = *reinterpret_cast<const uint4 *>(o);
                }
                xr[ch] = hv;
                if (ro) ro[ch] = hv;
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += h[e] * h[e];
            }
            const float inv = rsqrtf(block_sum(ss, sred) / (float)p.in_f + p.eps);
            const uint4 *wg = reinterpret_cast<const uint4 *>(p.nw);
            for (int ch = tid; ch < n8; ch += kThreads) {
                float h[8], w[8];
                unpack8<T>(xr[ch], h);
                unpack8<T>(__ldg(wg + ch), w);
                T o[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = E::rn(w[e] * E::to_f(E::rn(h[e] * inv)));
                xr[ch] = *reinterpret_cast<const uint4 *>(o);
            }
            __syncthreads();  // sred is reused by the next batch row
        } else if (p.xmode == kPlain) {
            for (int ch = tid; ch < n8; ch += kThreads) xr[ch] = __ldcg(xg + ch);
        } else {
            const bool silu = p.xmode == kSiluMul;
            for (int ch = tid; ch < n8; ch += kThreads) {
                float a[8], u[8];
                unpack8<T>(__ldcg(xg + ch), a);
                unpack8<T>(__ldcg(x2g + ch), u);
                T o[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float sg = silu ? E::to_f(E::rn(a[e] / (1.f + expf(-a[e])))) : a[e];
                    o[e] = E::rn(sg * u[e]);
                }
                xr[ch] = *reinterpret_cast<const uint4 *>(o);
            }
        }
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, p.status);

    // ---- units x K blocks of this CTA over the 8 warps (virtual blocks: kbc per unit)
    const int g = lane >> 2, t = lane & 3, sh0 = 8 * (t & 1);
    const int nu = u1 - u0, V = nu * p.kbc;
    const int v0 = V * warp / kWarps, v1 = V * (warp + 1) / kWarps;
    const int i0 = v0 / p.kbc;
    if (lane == 0) {
        wfirst[warp] = v0 < v1 ? i0 : 0;
        wlast[warp] = v0 < v1 ? (v1 - 1) / p.kbc + 1 : 0;
    }
    const bool xrow = g < p.batch;
    for (int i = i0; v0 < v1 && i * p.kbc < v1; ++i) {
        const int u = u0 + i, gt = u / p.nsplit, chunk = u % p.nsplit;
        const int l = member_of(tstart, p.nm, gt);
        const int ka = chunk * p.kbc + max(v0 - i * p.kbc, 0);
        const int kz = min(chunk * p.kbc + min(v1 - i * p.kbc, p.kbc), p.kb);
        const uint32_t *rowA = vs + (size_t)(16 * (gt - gt0) + g) * p.wv;
        const uint32_t *rowB = rowA + (size_t)8 * p.wv;
        const uint32_t *sw = reinterpret_cast<const uint32_t *>(s2s + (size_t)l * p.in_pad);
        const uint32_t *xw = reinterpret_cast<const uint32_t *>(xs + (size_t)(xrow ? g : 0) * p.in_pad);
        float acc[4][4] = {};
#pragma unroll 2
        for (int kb = ka; kb < kz; ++kb) {
            const int wi = 2 * kb + (t >> 1);
            const uint32_t wA = ok ? rowA[wi] << sh0 : 0u, wB = ok ? rowB[wi] << sh0 : 0u;
            const int kc2 = (64 * kb + 16 * t) / 2;
            const uint4 sa = *reinterpret_cast<const uint4 *>(sw + kc2), sb = *reinterpret_cast<const uint4 *>(sw + kc2 + 4);
            uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
            if (xrow) {
                xa = *reinterpret_cast<const uint4 *>(xw + kc2);
                xb = *reinterpret_cast<const uint4 *>(xw + kc2 + 4);
            }
            const uint32_t sp[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
            const uint32_t xp[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t a0 = lop_sign(wA << (2 * j), sp[2 * j]);
                const uint32_t a1 = lop_sign(wB << (2 * j), sp[2 * j]);
                const uint32_t a2 = lop_sign(wA << (2 * j + 1), sp[2 * j + 1]);
                const uint32_t a3 = lop_sign(wB << (2 * j + 1), sp[2 * j + 1]);
                E::mma(acc[j], a0, a1, a2, a3, xp[2 * j], xp[2 * j + 1]);
            }
        }
        if (t == 0) {  // D columns 0 / 1 = batch rows 0 / 1
            float *r = red + ((size_t)warp * p.segs + (i - i0)) * 32;
            r[g * 2] = (acc[0][0] + acc[1][0]) + (acc[2][0] + acc[3][0]);
            r[g * 2 + 1] = (acc[0][1] + acc[1][1]) + (acc[2][1] + acc[3][1]);
            r[(g + 8) * 2] = (acc[0][2] + acc[1][2]) + (acc[2][2] + acc[3][2]);
            r[(g + 8) * 2 + 1] = (acc[0][3] + acc[1][3]) + (acc[2][3] + acc[3][3]);
        }
    }
    __syncthreads();

    // ---- sum the warps' partials per unit (warp order) and store the unit's slot
    for (int idx = tid; idx < nu * 16 * p.batch; idx += kThreads) {
        const int i = idx / (16 * p.batch), rem = idx % (16 * p.batch), row = rem >> (p.batch - 1), b = rem & (p.batch - 1);
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w)
            if (i >= wfirst[w] && i < wlast[w]) s += red[((size_t)w * p.segs + (i - wfirst[w])) * 32 + row * 2 + b];
        const int u = u0 + i, gt = u / p.nsplit, chunk = u % p.nsplit;
        const int l = member_of(tstart, p.nm, gt);
        const M1 &mb = p.m[l];
        const int k = 16 * (gt - mb.tstart) + row;
        if (k < mb.rank) mb.tpart[((size_t)chunk * p.batch + b) * mb.ldt + k] = s;
    }
}

// ------------------------------------------------------------------ stage 2
// CTA c owns tiles [T c / G, T (c+1) / G) of the members' concatenated output tiles; their U
// rows and s1 slices are copied before griddepcontrol.wait.  After it, t of every member the
// CTA touches is assembled from the stage-1 slots into bf16 hi / lo columns in shared memory.
template <typename T>
__global__ void __launch_bounds__(kThreads, 2) stage2_kernel(const __grid_constant__ P2 p) {
    using E = Elem<T>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int wfirst[kWarps], wlast[kWarps];
    __shared__ uint32_t uoffs[kMaxMembers];
    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int t0 = (int)((long long)p.tiles * c / G), t1 = (int)((long long)p.tiles * (c + 1) / G);
    int tstart[kMaxMembers];
#pragma unroll
    for (int l = 0; l < kMaxMembers; ++l) tstart[l] = l < p.nm ? p.m[l].tstart : 0x7fffffff;
    uint32_t *us = reinterpret_cast<uint32_t *>(smem + p.off_u);
    T *s1s = reinterpret_cast<T *>(smem + p.off_s1);                       // [16 * tiles]
    __nv_bfloat16 *ts = reinterpret_cast<__nv_bfloat16 *>(smem + p.off_t); // [member][4][kpad]
    float *red = reinterpret_cast<float *>(smem + p.off_red);             // [warp][segs][16][2]

    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        uint32_t bytes = 0, off = 0;
        for (int l = 0; l < p.nm; ++l) {
            const M2 &mb = p.m[l];
            const int a = max(t0, mb.tstart), b = min(t1, mb.tstart + mb.tiles);
            uoffs[l] = off;
            if (a >= b) continue;
            bytes += (uint32_t)(16 * (b - a)) * (uint32_t)mb.wu * 4u + (uint32_t)(16 * (b - a)) * 2u;
            off += ((uint32_t)(16 * (b - a)) * (uint32_t)mb.wu + 3u) & ~3u;
        }
        mbar_arrive_expect_tx(&bar, bytes);
        for (int l = 0; l < p.nm; ++l) {
            const M2 &mb = p.m[l];
            const int a = max(t0, mb.tstart), b = min(t1, mb.tstart + mb.tiles);
            if (a >= b) continue;
            const int r0 = 16 * (a - mb.tstart);
            bulk_g2s_pieces(us + uoffs[l], mb.ubits + (size_t)r0 * mb.wu, (uint32_t)(16 * (b - a)) * (uint32_t)mb.wu * 4u,
                            &bar);
            bulk_g2s_pieces(s1s + 16 * (a - t0), static_cast<const T *>(mb.s1) + r0, (uint32_t)(16 * (b - a)) * 2u, &bar);
        }
    }
    __syncthreads();

    pdl_wait();  // stage 1 has completed: its slots are visible

    // ---- t of the touched members: sum of the nsplit slots, * smid, bf16 hi / lo columns
    const int lf = member_of(tstart, p.nm, t0), ll = member_of(tstart, p.nm, t1 - 1);
    for (int l = lf; l <= ll; ++l) {
        const M2 &mb = p.m[l];
        __nv_bfloat16 *tl = ts + (size_t)(l - lf) * 4 * p.kpad;
        const int kp = mb.kb2 * 64;
        for (int idx = tid; idx < p.batch * (kp / 4); idx += kThreads) {
            const int b = idx / (kp / 4), k = 4 * (idx % (kp / 4));
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (k < mb.rank) {
                for (int s = 0; s < p.nsplit; ++s) {
                    const float4 q = __ldcg(reinterpret_cast<const float4 *>(mb.tpart + ((size_t)s * p.batch + b) * mb.ldt + k));
                    v[0] += q.x; v[1] += q.y; v[2] += q.z; v[3] += q.w;
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (k + e >= mb.rank) v[e] = 0.f;
                    else if (mb.smid) v[e] *= E::to_f(static_cast<const T *>(mb.smid)[k + e]);
                }
            }
            __nv_bfloat16 hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                hi[e] = __float2bfloat16_rn(v[e]);
                lo[e] = __float2bfloat16_rn(v[e] - __bfloat162float(hi[e]));
            }
            *reinterpret_cast<uint2 *>(tl + (size_t)(2 * b) * p.kpad + k) = *reinterpret_cast<const uint2 *>(hi);
            *reinterpret_cast<uint2 *>(tl + (size_t)(2 * b + 1) * p.kpad + k) = *reinterpret_cast<const uint2 *>(lo);
        }
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, p.status);

    // ---- tiles x K blocks over the warps; K blocks counted with the largest member's kb2
    const int g = lane >> 2, t = lane & 3, sh0 = 8 * (t & 1);
    const int KB = p.kpad / 64;
    const int nt = t1 - t0, V = nt * KB;
    const int v0 = V * warp / kWarps, v1 = V * (warp + 1) / kWarps;
    const int i0 = v0 / KB;
    if (lane == 0) {
        wfirst[warp] = v0 < v1 ? i0 : 0;
        wlast[warp] = v0 < v1 ? (v1 - 1) / KB + 1 : 0;
    }
    const bool bcol = g < 2 * p.batch;  // B columns: (hi, lo) of batch row 0, then of row 1
    for (int i = i0; v0 < v1 && i * KB < v1; ++i) {
        const int tile = t0 + i;
        const int l = member_of(tstart, p.nm, tile);
        const M2 &mb = p.m[l];
        const int ka = max(v0 - i * KB, 0), kz = min(min(v1 - i * KB, KB), mb.kb2);
        const uint32_t *rowA = us + uoffs[l] + (size_t)(16 * (tile - max(t0, mb.tstart)) + g) * mb.wu;
        const uint32_t *rowB = rowA + (size_t)8 * mb.wu;
        const uint32_t *tw = reinterpret_cast<const uint32_t *>(ts + ((size_t)(l - lf) * 4 + (bcol ? g : 0)) * p.kpad);
        float acc[4][4] = {};
#pragma unroll 2
        for (int kb = ka; kb < kz; ++kb) {
            const int wi = 2 * kb + (t >> 1);
            const uint32_t wA = (ok && wi < mb.wu) ? rowA[wi] << sh0 : 0u;
            const uint32_t wB = (ok && wi < mb.wu) ? rowB[wi] << sh0 : 0u;
            const int kc2 = (64 * kb + 16 * t) / 2;
            uint4 ta = make_uint4(0u, 0u, 0u, 0u), tb = ta;
            if (bcol) {
                ta = *reinterpret_cast<const uint4 *>(tw + kc2);
                tb = *reinterpret_cast<const uint4 *>(tw + kc2 + 4);
            }
            const uint32_t bp[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                constexpr uint32_t kOne = 0x3F803F80u;  // bf16 (1.0, 1.0)
                const uint32_t a0 = lop_sign(wA << (2 * j), kOne);
                const uint32_t a1 = lop_sign(wB << (2 * j), kOne);
                const uint32_t a2 = lop_sign(wA << (2 * j + 1), kOne);
                const uint32_t a3 = lop_sign(wB << (2 * j + 1), kOne);
                mma_bf16_16816(acc[j], a0, a1, a2, a3, bp[2 * j], bp[2 * j + 1]);
            }
        }
        if (t < p.batch) {  // D columns 2t, 2t+1 = (hi, lo) of batch row t
            float *r = red + ((size_t)warp * p.segs + (i - i0)) * 32;
            r[g * 2 + t] = ((acc[0][0] + acc[1][0]) + (acc[2][0] + acc[3][0])) +
                           ((acc[0][1] + acc[1][1]) + (acc[2][1] + acc[3][1]));
            r[(g + 8) * 2 + t] = ((acc[0][2] + acc[1][2]) + (acc[2][2] + acc[3][2])) +
                                 ((acc[0][3] + acc[1][3]) + (acc[2][3] + acc[3][3]));
        }
    }
    __syncthreads();

    // ---- epilogue: sum warps in order, * s1, round (fp16 clamp), SiLU where asked, store
    for (int idx = tid; idx < nt * 16 * p.batch; idx += kThreads) {
        const int i = idx / (16 * p.batch), rem = idx % (16 * p.batch), b = rem / 16, row = rem % 16;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w)
            if (i >= wfirst[w] && i < wlast[w]) s += red[((size_t)w * p.segs + (i - wfirst[w])) * 32 + row * 2 + b];
        const int tile = t0 + i;
        const int l = member_of(tstart, p.nm, tile);
        const M2 &mb = p.m[l];
        const int m = 16 * (tile - mb.tstart) + row;
        if (m < mb.out_f) {
            T out = E::out(s * E::to_f(s1s[16 * i + row]));
            if ((p.act >> l) & 1) {  // SiLU on the rounded output, rounded again (the SwiGLU gate)
                const float gv = E::to_f(out);
                out = E::rn(gv / (1.f + expf(-gv)));
            }
            static_cast<T *>(mb.y)[(size_t)b * mb.out_f + m] = out;
        }
    }
}

// ------------------------------------------------------------------ host planning
static inline uint32_t a128(size_t v) { return (uint32_t)((v + 127) & ~size_t(127)); }

struct Plan2 {
    P1 p1{};
    P2 p2{};
    int g1 = 0, g2 = 0;
    size_t smem1 = 0, smem2 = 0;
};

// Largest per-CTA / per-warp extents of a contiguous split of `n` items (each `k` virtual K
// blocks) over `G` CTAs and kWarps warps: items per CTA and segments per warp.
static void split_extents(long long n, int G, int k, int &max_items, int &max_segs) {
    max_items = 0;
    max_segs = 1;
    for (int c = 0; c < G; ++c) {
        const int a = (int)(n * c / G), b = (int)(n * (c + 1) / G);
        max_items = std::max(max_items, b - a);
        const int V = (b - a) * k;
        for (int w = 0; w < kWarps; ++w) {
            const int v0 = V * w / kWarps, v1 = V * (w + 1) / kWarps;
            if (v0 < v1) max_segs = std::max(max_segs, (v1 - 1) / k - v0 / k + 1);
        }
    }
}

// Per-CTA shared-memory cap that still lets two CTAs share an SM.
static size_t smem_cap(int dev) {
    const DeviceInfo &di = device_info(dev);
    (void)di;
    return (size_t)113 * 1024 - 1024;
}

}  // namespace gemv2
}  // namespace nq

// Entry used by nq_gemv.cu's group dispatch.  Returns NQ_OK after launching, NQ_ERR_UNSUPPORTED
// (with nothing launched and no error message set) when the group does not fit this path.
int nq_gemv2_try(int dtype, const void *x, int64_t batch, int64_t in_features, int n, const nq_gemv_layer *layers,
                 int xmode, const void *x2, const void *nw, void *res_out, float eps, int act, void *workspace,
                 size_t workspace_bytes, void *stream) {
    using namespace nq;
    using namespace nq::gemv2;
    static const bool enabled = [] {
        const char *e = std::getenv("NQ_GEMV2");
        return !(e && e[0] == '0');
    }();
    if (!enabled || batch < 1 || batch > kMaxBatch || n < 1 || n > kMaxMembers) return NQ_ERR_UNSUPPORTED;
    if (in_features % 128 || in_features > 32768) return NQ_ERR_UNSUPPORTED;
    uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(x2) | reinterpret_cast<uintptr_t>(nw) |
                   reinterpret_cast<uintptr_t>(res_out) | reinterpret_cast<uintptr_t>(workspace);
    for (int l = 0; l < n; ++l) {
        const nq_gemv_layer &L = layers[l];
        al |= reinterpret_cast<uintptr_t>(L.scale_pre) | reinterpret_cast<uintptr_t>(L.scale_post);
        if (L.out_features % 16 || L.rank < 1) return NQ_ERR_UNSUPPORTED;
    }
    if (al & 15) return NQ_ERR_UNSUPPORTED;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NQ_ERR_UNSUPPORTED;
    const DeviceInfo &di = device_info(dev);
    const int G = di.sms;
    const size_t cap = smem_cap(dev);

    Plan2 pl;
    P1 &a = pl.p1;
    P2 &b = pl.p2;
    a.x = x;
    a.x2 = x2;
    a.nw = nw;
    a.res_out = res_out;
    a.eps = eps;
    a.xmode = xmode;
    a.batch = (int)batch;
    a.in_f = (int)in_features;
    a.wv = a.in_f / 32;
    a.kb = a.wv / 2;
    a.in_pad = a.kb * 64;
    a.nm = n;
    a.status = &static_cast<Ctrl *>(workspace)->status;
    b.batch = (int)batch;
    b.nm = n;
    b.act = act;
    b.status = a.status;
    int tiles1 = 0, tiles2 = 0, max_kb2 = 1;
    for (int l = 0; l < n; ++l) {
        const nq_gemv_layer &L = layers[l];
        a.m[l].s2 = L.scale_pre;
        a.m[l].vbits = reinterpret_cast<const uint32_t *>(L.v_bits);
        a.m[l].rank = (int)L.rank;
        a.m[l].tiles = (int)((L.rank + 15) / 16);
        a.m[l].tstart = tiles1;
        tiles1 += a.m[l].tiles;
        M2 &m2 = b.m[l];
        m2.smid = L.scale_mid;
        m2.ubits = reinterpret_cast<const uint32_t *>(L.u_bits);
        m2.s1 = L.scale_post;
        m2.y = L.y;
        m2.rank = (int)L.rank;
        m2.out_f = (int)L.out_features;
        m2.wu = (int)((L.rank + 31) / 32);
        m2.kb2 = (m2.wu + 1) / 2;
        m2.tiles = m2.out_f / 16;
        m2.tstart = tiles2;
        tiles2 += m2.tiles;
        max_kb2 = std::max(max_kb2, m2.kb2);
    }
    // choose nsplit: the smallest largest per-CTA stage-1 work (units x K blocks per unit)
    int best_s = 1;
    long long best_w = -1;
    for (int s = 1; s <= kMaxSplit && s <= a.kb; ++s) {
        if (s * (int)batch > 8) break;  // slots must fit the member's workspace region
        const long long U = (long long)tiles1 * s;
        const int kbc = (a.kb + s - 1) / s;
        const long long w = ((U + G - 1) / G) * kbc;
        if (best_w < 0 || w < best_w) {
            best_w = w;
            best_s = s;
        }
    }
    a.nsplit = b.nsplit = best_s;
    a.kbc = (a.kb + best_s - 1) / best_s;
    a.units = tiles1 * best_s;
    pl.g1 = std::min(G, a.units);
    int max_units = 0, segs1 = 0;
    split_extents(a.units, pl.g1, a.kbc, max_units, segs1);
    if (segs1 > kMaxSegs) return NQ_ERR_UNSUPPORTED;
    a.segs = segs1;
    const int max_tiles_cov = (max_units - 1) / best_s + 2;  // global tiles a CTA's units cover
    // t slots [nsplit][batch][ldt] float per member, inside the member's region of the workspace
    // (nq_gemv_group_workspace_bytes gives each member 32 * round_up(rank, 64) bytes)
    char *wsp = static_cast<char *>(workspace) + sizeof(Ctrl);
    size_t need = sizeof(Ctrl);
    for (int l = 0; l < n; ++l) {
        const int ldt = ((int)layers[l].rank + 63) / 64 * 64;
        a.m[l].ldt = b.m[l].ldt = ldt;
        const size_t region = (size_t)32 * (size_t)ldt;
        const size_t slots = (size_t)best_s * (size_t)batch * (size_t)ldt * 4;
        if (slots > region) return NQ_ERR_UNSUPPORTED;
        a.m[l].tpart = reinterpret_cast<float *>(wsp);
        b.m[l].tpart = a.m[l].tpart;
        wsp += region;
        need += region;
    }
    if (workspace_bytes < need) return NQ_ERR_UNSUPPORTED;
    // stage-1 shared memory
    size_t off = 0;
    a.off_s2 = (uint32_t)off;
    off = a128(off + (size_t)n * a.in_pad * 2);
    a.off_x = (uint32_t)off;
    off = a128(off + (size_t)batch * a.in_pad * 2);
    a.off_v = (uint32_t)off;
    off = a128(off + (size_t)max_tiles_cov * 16 * a.wv * 4);
    a.off_red = (uint32_t)off;
    off = a128(off + (size_t)kWarps * segs1 * 32 * 4);
    pl.smem1 = off;
    // stage 2
    b.tiles = tiles2;
    b.kpad = max_kb2 * 64;
    pl.g2 = std::min(G, tiles2);
    int max_t2 = 0, segs2 = 0;
    split_extents(tiles2, pl.g2, max_kb2, max_t2, segs2);
    if (segs2 > kMaxSegs) return NQ_ERR_UNSUPPORTED;
    b.segs = segs2;
    int max_wu = 1;
    for (int l = 0; l < n; ++l) max_wu = std::max(max_wu, b.m[l].wu);
    off = 0;
    b.off_u = (uint32_t)off;
    off = a128(off + ((size_t)16 * max_t2 * max_wu + 4 * n) * 4);
    b.off_s1 = (uint32_t)off;
    off = a128(off + (size_t)16 * max_t2 * 2);
    b.off_t = (uint32_t)off;
    // members one CTA touches: at most all of them
    off = a128(off + (size_t)std::min(n, max_t2 + 1) * 4 * b.kpad * 2);
    b.off_red = (uint32_t)off;
    off = a128(off + (size_t)kWarps * segs2 * 32 * 4);
    pl.smem2 = off;
    if (pl.smem1 > cap || pl.smem2 > cap) return NQ_ERR_UNSUPPORTED;

    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    if (dev < 0 || dev >= 64) return NQ_ERR_UNSUPPORTED;
    std::call_once(once[dev], [&] {
        cudaError_t e = cudaSuccess;
        for (auto f : {(const void *)stage1_kernel<__half>, (const void *)stage1_kernel<__nv_bfloat16>,
                       (const void *)stage2_kernel<__half>, (const void *)stage2_kernel<__nv_bfloat16>})
            if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cap);
        attr_err[dev] = e;
    });
    if (attr_err[dev] != cudaSuccess) return cuda_fail(attr_err[dev], "cudaFuncSetAttribute(gemv2)");

    cudaLaunchAttribute attr[1];
    int na = 0;
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        na = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = na;
    cfg.gridDim = dim3(pl.g1);
    cfg.dynamicSmemBytes = pl.smem1;
    cudaError_t e = dtype == NQ_DTYPE_F16 ? cudaLaunchKernelEx(&cfg, stage1_kernel<__half>, a)
                                          : cudaLaunchKernelEx(&cfg, stage1_kernel<__nv_bfloat16>, a);
    if (e != cudaSuccess) return cuda_fail(e, "gemv2 stage-1 launch");
    cfg.gridDim = dim3(pl.g2);
    cfg.dynamicSmemBytes = pl.smem2;
    e = dtype == NQ_DTYPE_F16 ? cudaLaunchKernelEx(&cfg, stage2_kernel<__half>, b)
                              : cudaLaunchKernelEx(&cfg, stage2_kernel<__nv_bfloat16>, b);
    if (e != cudaSuccess) return cuda_fail(e, "gemv2 stage-2 launch");
    return NQ_OK;
}
