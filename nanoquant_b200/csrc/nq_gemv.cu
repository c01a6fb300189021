// Fused NanoQuant decode GEMV for sm_100a (one launch per <= 8 rows of x).
//
// Computes, for b < batch (<= 8):
//   t[b, k] = smid[k] * sum_n sign(V[k, n]) * s2[n] * x[b, n]          (stage 1, k < rank)
//   y[b, m] = clamp(s1[m] * sum_k sign(U[m, k]) * t[b, k])             (stage 2, m < out)
// replacing the reference's two launches with a half-precision interm round trip
// (src/nanoquant/kernel/cuda/gemv_kernel.cu:43-301, dispatched at :308-429).
//
// Design (one CTA per SM, cooperative launch):
//  * At kernel start one thread issues 1-D bulk copies (TMA engine, no multicast) of
//    this CTA's contiguous slab of V rows AND of U rows into shared memory, so every
//    weight byte the CTA will ever need is in flight at once; U streams in while
//    stage 1 computes and while the grid waits at the barrier.
//  * s2 and x are staged in shared memory by plain coalesced loads (zero-padded to a
//    multiple of 64 columns).
//  * Both stages are tensor-core matrix-vector products with mma.sync.m16n8k16 and
//    float32 accumulation: the A fragment (16 weight rows x 16 columns) is built in
//    registers straight from the HALF2 sign words -- the bit pair of columns
//    (2p, 2p+1) sits at bits (15-p, 31-p), so `(w << p) & 0x80008000` is the sign mask
//    of one bf16/fp16 pair -- and the B fragment is the activation column(s).
//    Stage 1 folds s2 into A (A = +-s2[n], exact in the input dtype; B = x, exact),
//    so the products are exact and only the float32 accumulation rounds.
//    Stage 2 uses A = +-1.0 (bf16) and B = t split into bf16 hi + lo halves (two
//    B columns per batch row), which keeps ~16 mantissa bits of the float32 t.
//  * Each warp owns a contiguous range of 64-column K blocks of every 16-row tile;
//    the 8 warps' partial 16x8 tiles are reduced through shared memory.
//  * t[b, :] goes to the (L2-resident) workspace; one bounded grid barrier separates
//    the stages.  The barrier resets itself, so the workspace stays reusable.
// Layers too large for the per-CTA shared-memory budget run the same kernel as two
// ordinary launches (stage 1 then stage 2), each over the fewest whole waves of CTAs whose
// slabs fit in shared memory.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "nq_common.cuh"

namespace nq {
namespace gemv {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxBatch = 8;
constexpr int kStaticSmemReserve = 1024;  // static __shared__ of the kernel (grid barrier flag)
constexpr int kFoldMaxBatch = 2;         // batch rows for which stage 1 folds s2 into the B operand

enum Mode : int { kStage1 = 1, kStage2 = 2, kFused = 3 };

// Tensor-parallel exchange fused into the GEMVs (nq_gemv_group_tp).  A PUSH launch (the
// row-parallel o / down projection) stores its rounded output rows into every rank's receive
// buffer over NVLink; the next PULL launch (q/k/v or gate/up, whose RMSNorm prologue needs the
// summed vector) sums the ranks' buffers in rank order (float32, rounded once: the same bits on
// every rank) in place of reading x.  The messages are a few kilobytes, so the protocol is built
// for latency: every 8-byte store carries two values and the exchange's epoch as a flag
// ({2 x 16-bit values, u32 epoch}, single-copy atomic), so the producer needs no fence and no
// separate signal, and the consumer polls the words it sums until their flags show the epoch.
// Region of each rank (mapped by every other rank over CUDA IPC), bytes:
//   [Ctrl 256][push epochs kTpMaxCtas x u32][pull epochs kTpMaxCtas x u32][reserved]
//   [data 2 parities x world x max_elems / 2 words of 8 B]
// Epochs are per-CTA counters advanced by every launch of their kind (push / pull), so graph
// replays stay in step on all ranks as long as every rank makes the same sequence of calls,
// pushes and pulls alternating.  Receive buffers alternate by epoch parity: a rank runs at most one
// exchange ahead of another (its next push needs its own pull, which needs every rank's push),
// so a buffer is rewritten only after every rank has read it, and a flag equals the epoch only
// once that exchange's word has landed.
constexpr int kTpMaxWorld = 8;
constexpr int kTpMaxCtas = 256;
enum TpMode : int { kTpPull = NQ_TP_PULL, kTpPush = NQ_TP_PUSH };
constexpr size_t kTpOffPush = sizeof(Ctrl);
constexpr size_t kTpOffPull = kTpOffPush + 4 * kTpMaxCtas;
constexpr size_t kTpOffFlags = kTpOffPull + 4 * kTpMaxCtas;
constexpr size_t kTpOffData = kTpOffFlags + 4 * (size_t)kTpMaxWorld * kTpMaxCtas;
static_assert(kTpOffData % 256 == 0, "exchange data starts 256-byte aligned");

struct TpX {
    unsigned char *region[kTpMaxWorld];  // every rank's region as mapped in this process
    int rank, world, mode, gprod;        // gprod: CTAs of the PUSH launches (one flag each)
    long long max_elems;                 // values per source buffer
};

// One receive buffer of rank `dst`: source `src`'s words for exchange e (max_elems / 2 words).
__device__ __forceinline__ uint2 *tp_words(const TpX &tp, int dst, unsigned e, int src) {
    const size_t plane = (size_t)tp.max_elems * 4;
    return reinterpret_cast<uint2 *>(tp.region[dst] + kTpOffData + ((size_t)(e & 1u) * tp.world + src) * plane);
}
__device__ __forceinline__ void tp_st_word(uint2 *p, uint32_t vals, unsigned e) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(vals), "r"(e) : "memory");
}
__device__ __forceinline__ uint4 tp_ld_words(const uint2 *p) {  // two 8-byte words
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// 8 values (4 words) of source src for exchange e, polled (bounded) until every word carries e.
// Returns false (and records NQ_ERR_DEVICE_TIMEOUT) when the source did not come within the limit.
__device__ __forceinline__ bool tp_read8(const TpX &tp, unsigned e, int src, int64_t word0, uint32_t (&v)[4],
                                         int *status) {
    const uint2 *w = tp_words(tp, tp.rank, e, src) + word0;
    uint4 a = tp_ld_words(w), b = tp_ld_words(w + 2);
    if (a.y != e || a.w != e || b.y != e || b.w != e) {
        const uint64_t t0 = globaltimer_ns();
        while (a.y != e || a.w != e || b.y != e || b.w != e) {
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                record_status(status, NQ_ERR_DEVICE_TIMEOUT);
                return false;
            }
            a = tp_ld_words(w);
            b = tp_ld_words(w + 2);
        }
    }
    v[0] = a.x;
    v[1] = a.z;
    v[2] = b.x;
    v[3] = b.z;
    return true;
}

// Phase timeline of the fused kernel, compiled only into debug builds (-DNQ_GEMV_TRACE):
// thread 0 of every CTA keeps globaltimer stamps at the phase boundaries in registers and
// stores them at the end into the launch's slot of g_trace (slot = launches seen so far,
// read after griddepcontrol.wait, advanced by CTA 0 after the grid barrier).
// nq_debug_gemv_trace copies the stamps out.  Release builds compile none of this.
#ifdef NQ_GEMV_TRACE
constexpr int kTraceLaunches = 512, kTraceCtas = 160, kTraceStamps = 12;
__device__ unsigned long long g_trace[kTraceLaunches][kTraceCtas][kTraceStamps];
__device__ unsigned int g_trace_launch;
#define NQ_STAMP(i) do { if (threadIdx.x == 0) tr_[i] = globaltimer_ns(); } while (0)
#else
#define NQ_STAMP(i) do { } while (0)
#endif

__device__ __forceinline__ void tile_range(int tiles, int c, int G, int &b, int &e) {
    if ((long long)tiles * G < (1LL << 31)) {  // every launch of the decode shapes
        b = (tiles * c) / G;
        e = (tiles * (c + 1)) / G;
    } else {  // split launches of very tall layers (tiles <= 2^16, grid up to the tile count)
        b = (int)(((long long)tiles * c) / G);
        e = (int)(((long long)tiles * (c + 1)) / G);
    }
}

// Copy `n` 16-bit values into a zero-padded shared row of `npad` values (unaligned inputs).
template <typename T>
__device__ __forceinline__ void stage_row(T *dst, const T *src, int n, int npad) {
    const bool vec = ((reinterpret_cast<uintptr_t>(src) & 15) == 0);
    for (int c8 = threadIdx.x; c8 < npad / 8; c8 += kThreads) {
        const int c = c8 * 8;
        uint4 v;
        if (vec && c + 8 <= n) {
            v = __ldg(reinterpret_cast<const uint4 *>(src + c));
        } else {
            uint16_t h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                h[j] = (c + j < n) ? reinterpret_cast<const uint16_t *>(src)[c + j] : uint16_t(0);
            v = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                           h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
        }
        reinterpret_cast<uint4 *>(dst + c)[0] = v;
    }
}

// 16 consecutive 16-bit values from a global row with bounds checks (zero beyond n).
template <typename T>
__device__ __forceinline__ void load16_global(const T *row, int c, int n, uint32_t (&v)[8]) {
    if (c + 16 <= n && (reinterpret_cast<uintptr_t>(row + c) & 15) == 0) {
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(row + c));
        const uint4 b = __ldg(reinterpret_cast<const uint4 *>(row + c) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint16_t *r = reinterpret_cast<const uint16_t *>(row);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t lo = (c + 2 * j < n) ? r[c + 2 * j] : 0u;
            const uint32_t hi = (c + 2 * j + 1 < n) ? r[c + 2 * j + 1] : 0u;
            v[j] = lo | (hi << 16);
        }
    }
}

__device__ __forceinline__ void load16_smem(const void *p, uint32_t (&v)[8]) {
    const uint4 a = reinterpret_cast<const uint4 *>(p)[0];
    const uint4 b = reinterpret_cast<const uint4 *>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Bytes the TMA engine delivers for rows [r0, r1) of a plane with `w` words per row:
// every row when copied row by row, else the 16-byte-multiple prefix of the slab.
__device__ __forceinline__ uint32_t slab_bulk_bytes(int r0, int r1, int w, bool by_rows) {
    const uint32_t words = (r1 > r0) ? (uint32_t)(r1 - r0) * (uint32_t)w : 0u;
    return by_rows ? words * 4u : (words * 4u) & ~15u;
}

// Rows [r0, r1) of a plane -> smem.  By rows (w % 4 == 0): one bulk copy per row into a
// padded stride `ws`, issued by the lanes of warp `issuer`.  Otherwise the slab keeps
// stride w: the 16-byte-multiple prefix goes through the TMA engine (leader thread), the
// remaining <16 bytes by plain loads (the caller syncs afterwards).
__device__ __forceinline__ void copy_slab(uint32_t *dst, const uint32_t *plane, int r0, int r1, int w, int ws,
                                          bool by_rows, uint64_t *bar, int issuer) {
    const uint32_t *src = plane + (size_t)r0 * w;
    if (by_rows) {
        if ((int)(threadIdx.x >> 5) == issuer)
            for (int r = (int)(threadIdx.x & 31); r < r1 - r0; r += 32)
                bulk_g2s(dst + (size_t)r * ws, src + (size_t)r * w, (uint32_t)w * 4u, bar);
        return;
    }
    const uint32_t words = (r1 > r0) ? (uint32_t)(r1 - r0) * (uint32_t)w : 0u;
    const uint32_t bulk = (words * 4u) & ~15u;
    if ((int)threadIdx.x == issuer * 32 && bulk) bulk_g2s_pieces(dst, src, bulk, bar);
    for (uint32_t i = bulk / 4 + threadIdx.x; i < words; i += kThreads) dst[i] = __ldg(src + i);
}

// A slab of rows [r0, r1) (w words each) copied contiguously: the 16-byte-multiple prefix
// through the copy engine (one thread) and the rest by plain loads (all threads).
__device__ __forceinline__ void slab_bulk(uint32_t *dst, const uint32_t *plane, int r0, int r1, int w, uint64_t *bar) {
    const uint32_t words = (r1 > r0) ? (uint32_t)(r1 - r0) * (uint32_t)w : 0u;
    const uint32_t bulk = (words * 4u) & ~15u;
    if (bulk) bulk_g2s_pieces(dst, plane + (size_t)r0 * w, bulk, bar);
}
__device__ __forceinline__ void slab_tail(uint32_t *dst, const uint32_t *plane, int r0, int r1, int w) {
    const uint32_t words = (r1 > r0) ? (uint32_t)(r1 - r0) * (uint32_t)w : 0u;
    const uint32_t bulk = (words * 4u) & ~15u;
    const uint32_t *src = plane + (size_t)r0 * w;
    for (uint32_t i = bulk / 4 + threadIdx.x; i < words; i += kThreads) dst[i] = __ldg(src + i);
}

// Zero the padding columns [n, npad) of a staged 16-bit row.
template <typename T>
__device__ __forceinline__ void zero_tail(T *dst, int n, int npad) {
    uint16_t *d = reinterpret_cast<uint16_t *>(dst);
    for (int c = n + threadIdx.x; c < npad; c += kThreads) d[c] = 0;
}

// Work split inside a CTA: its tiles x K blocks form U = tiles * KB units (tile-major); warp w
// takes the contiguous units [U w / W, U (w+1) / W), which cover at most S consecutive tiles
// (S from seg_bound), and writes one partial 16x8 tile per covered tile to `red` slot
// w * S + (tile - first tile of w).  Every warp gets the same amount of K work whatever the
// tile count, and each tile's partials are summed in warp order, so results are deterministic.
__host__ __device__ __forceinline__ void warp_units(int U, int w, int &u0, int &u1) {
    u0 = (U * w) / kWarps;
    u1 = (U * (w + 1)) / kWarps;
}
// Upper bound on the tiles one warp's range covers, for at most `tiles` tiles of KB units.
__host__ __device__ __forceinline__ int seg_bound(int tiles, int KB) {
    if (tiles <= 0 || KB <= 0) return 1;
    const int n = (tiles * KB + kWarps - 1) / kWarps;
    const int s = (n + KB - 1) / KB + 1;
    return s < tiles ? s : tiles;
}
// Per-CTA table of the current stage's warp ranges, written by lane 0 of every warp before
// its partials: first and one-past-last tile covered (first = last when the range is empty).
// The reduction reads it instead of recomputing ranges (runtime integer divisions).
struct WarpTab {
    int lt0[kWarps], lt1[kWarps];
};
__device__ __forceinline__ void record_range(WarpTab *wt, int warp, int u0, int u1, int KB) {
    if ((threadIdx.x & 31) == 0) {
        wt->lt0[warp] = u0 < u1 ? u0 / KB : 0;
        wt->lt1[warp] = u0 < u1 ? (u1 - 1) / KB + 1 : 0;
    }
}
// Sum over warps, in warp order, of tile lt's partial at float offset `off` of each slot.
__device__ __forceinline__ float sum_partials(const float *red, const WarpTab *wt, int S, int lt, int off, bool pair) {
    // branch-free so that all the loads are in flight together; uncovered slots read slot 0
    float v[kWarps];
    bool in[kWarps];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        const int a = wt->lt0[w];
        in[w] = lt >= a && lt < wt->lt1[w];
        const float *r = red + (in[w] ? (w * S + (lt - a)) * 256 + off : off);
        v[w] = pair ? r[0] + r[1] : r[0];
    }
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += in[w] ? v[w] : 0.f;
    return s;
}

__device__ __forceinline__ void store_partial(float *r, const float (&acc)[4], int g, int t) {
    r[g * 8 + 2 * t] = acc[0];
    r[g * 8 + 2 * t + 1] = acc[1];
    r[(g + 8) * 8 + 2 * t] = acc[2];
    r[(g + 8) * 8 + 2 * t + 1] = acc[3];
}

// 8 bf16 pairs (16 values along k) of one B column in global memory (L2-resident);
// zeros when the column belongs to a batch row that does not exist.
__device__ __forceinline__ void load_t_pairs(const __nv_bfloat16 *p, bool valid, uint32_t (&v)[8]) {
    uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
    if (valid) {
        a = __ldcg(reinterpret_cast<const uint4 *>(p));
        b = __ldcg(reinterpret_cast<const uint4 *>(p) + 1);
    }
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// bf16 (hi, lo) pairs of two floats: hi = bf16(v), lo = bf16(v - hi)
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat16 ha = __float2bfloat16_rn(a), hb = __float2bfloat16_rn(b);
    const __nv_bfloat16 la = __float2bfloat16_rn(a - __bfloat162float(ha));
    const __nv_bfloat16 lb = __float2bfloat16_rn(b - __bfloat162float(hb));
    hi = (uint32_t)__bfloat16_as_ushort(ha) | ((uint32_t)__bfloat16_as_ushort(hb) << 16);
    lo = (uint32_t)__bfloat16_as_ushort(la) | ((uint32_t)__bfloat16_as_ushort(lb) << 16);
}

// A fragment of a +-1 (bf16) tile: rows g / g+8 words already shifted by 8*(t&1).
__device__ __forceinline__ void sign_frag(uint32_t wA, uint32_t wB, int j, uint32_t (&a)[4]) {
    constexpr uint32_t kOne = 0x3F803F80u;  // bf16 (1.0, 1.0)
    a[0] = lop_sign(wA << (2 * j), kOne);
    a[1] = lop_sign(wB << (2 * j), kOne);
    a[2] = lop_sign(wA << (2 * j + 1), kOne);
    a[3] = lop_sign(wB << (2 * j + 1), kOne);
}

constexpr int kMaxGroup = 3;  // layers sharing one input x in a single launch (q/k/v, gate/up)
enum ChainXMode : int {
    kChainPlain = NQ_CHAIN_X_PLAIN,
    kChainNorm = NQ_CHAIN_X_RMSNORM,
    kChainSiluMul = NQ_CHAIN_X_SILU_MUL,
    kChainMul = NQ_CHAIN_X_MUL
};

// One NanoQuant layer of a launch group.
struct Member {
    const void *s2;            // scale_pre [in]
    const uint32_t *vbits;     // V planes [rank, wv]
    const void *smid;          // scale_mid [rank] or null
    const uint32_t *ubits;     // U planes [out, wu]
    const void *s1;            // scale_post [out]
    void *y;                   // [batch, out]
    __nv_bfloat16 *tb;         // stage-2 B operand [16 columns][ldi]: (hi, lo) of t for 8 batch rows
    int rank, out_f, wu, kb2, ldi;
    int tiles1, tiles2;        // 16-row tiles of this layer in stage 1 / stage 2
    int t1_start, t2_start;    // its first tile in the group's concatenated tile lists
    int u_rows, wus;           // U slab copied row by row (wu % 4 == 0) and its smem row stride
};

struct Params {
    const void *x;             // [batch, in], shared by every member
    Ctrl *ctrl;
    int batch, in_f, wv, kb1, nm;
    Member m[kMaxGroup];
    int tiles1, tiles2;        // totals over members
    int wvs, v_rows;           // V slab smem stride (words) and row-by-row copy flag (wv % 4 == 0)
    int mode, x_in_smem, fold;
    int kbu2;                  // stage-2 K blocks per tile in the work split: the largest member's kb2
    int seg1, seg2;            // red slots per warp (seg_bound) in stage 1 / stage 2
    // input transform of the single-group kernel (fold mode, x staged in shared memory):
    int xmode;                 // ChainXMode; the input every member reads is x' (not x)
    const void *x2;            // RMSNORM: added to x first (may be null); MUL / SILU_MUL: second factor
    const void *nw;            // RMSNORM weight
    void *res_out;             // RMSNORM: receives x (+ x2), written by the CTA owning stage-1 tile 0
    float eps;
    int act;                   // bit l: SiLU on member l's output
    uint32_t off_red, off_s2, off_x, off_xs2, off_v, off_u, off_s1, off_x2, off_nw;
};

__device__ __forceinline__ int member_of1(const Params &p, int tile) {
    int l = 0;
    while (l + 1 < p.nm && tile >= p.m[l + 1].t1_start) ++l;
    return l;
}
__device__ __forceinline__ int member_of2(const Params &p, int tile) {
    int l = 0;
    while (l + 1 < p.nm && tile >= p.m[l + 1].t2_start) ++l;
    return l;
}

// Whether a CTA's stage-1 tile range [t1b, t1e) holds any tile of member mb.
__device__ __forceinline__ bool owns1(const Member &mb, int t1b, int t1e) {
    return max(t1b, mb.t1_start) < min(t1e, mb.t1_start + mb.tiles1);
}

// The part of a CTA's stage-2 tile range [t2b, t2e) that belongs to member l:
// tiles [a, b) (global indices); a >= b when there is none.
__device__ __forceinline__ void seg_tiles(const Member &mb, int t2b, int t2e, int &a, int &b) {
    a = max(t2b, mb.t2_start);
    b = min(t2e, mb.t2_start + mb.tiles2);
}

__device__ __forceinline__ float block_sum_512(float v, float *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();  // sh may still be read by a previous call
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += sh[i];
    return s;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
    const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = Elem<T>::to_f(e[j]);
}

// ------------------------------------------------------------------ stage bodies
// Stage 1: this CTA's tiles [t1b, t1e) split over the warps by K-block units (warp_units),
// partial 16x8 tiles into `red`.
// FOLD: 1 compiles only the folded-operand path, -1 decides at run time (p.fold).
template <typename T, int FOLD = -1>
__device__ __forceinline__ void stage1_items(const Params &p, const uint32_t *vch, const T *s2s, const T *xs,
                                            const __nv_bfloat16 *xs2, float *red, int t1b, int t1e, bool ok,
                                            WarpTab *wt) {
    const bool fold = FOLD >= 0 ? FOLD != 0 : p.fold != 0;
    using E = Elem<T>;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int sh0 = 8 * (t & 1);
    const int in_pad = p.kb1 * 64;
    const int nxc = 2 * p.batch;
    const T *xg = static_cast<const T *>(p.x) + (size_t)g * p.in_f;
    const uint32_t *xsw = reinterpret_cast<const uint32_t *>(xs + (size_t)g * in_pad);
    const bool xrow = g < p.batch, fcol = g < nxc;
    const int ntiles = t1e - t1b, KB = p.kb1, S = p.seg1;
    int u0, u1;
    warp_units(ntiles * KB, warp, u0, u1);
    const int lt0 = u0 / KB;
    record_range(wt, warp, u0, u1, KB);
    for (int lt = lt0; u0 < u1 && lt * KB < u1; ++lt) {
        const int kbeg = max(u0 - lt * KB, 0), kend = min(u1 - lt * KB, KB);
        const int tile = t1b + lt;
        const int l = member_of1(p, tile);
        const int row0 = 16 * (tile - p.m[l].t1_start), rank = p.m[l].rank;
        const bool vA = ok && (row0 + g < rank), vB = ok && (row0 + g + 8 < rank);
        const uint32_t *rowA = vch + (size_t)(lt * 16 + g) * p.wvs;
        const uint32_t *rowB = rowA + (size_t)8 * p.wvs;
        float acc[4][4] = {};
        if (fold) {
            const __nv_bfloat16 *xcol = xs2 + ((size_t)l * nxc + g) * in_pad;
#pragma unroll 2
            for (int kb = kbeg; kb < kend; ++kb) {
                const int wi = 2 * kb + (t >> 1);
                const uint32_t wA = (vA && wi < p.wv) ? rowA[wi] << sh0 : 0u;
                const uint32_t wB = (vB && wi < p.wv) ? rowB[wi] << sh0 : 0u;
                const int kc = 64 * kb + 16 * t;
                uint32_t bp[8];
                if (fcol) {
                    load16_smem(xcol + kc, bp);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) bp[j] = 0u;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t a[4];
                    sign_frag(wA, wB, j, a);
                    mma_bf16_16816(acc[j], a[0], a[1], a[2], a[3], bp[2 * j], bp[2 * j + 1]);
                }
            }
        } else {
            const uint32_t *sw = reinterpret_cast<const uint32_t *>(s2s + (size_t)l * in_pad);
#pragma unroll 2
            for (int kb = kbeg; kb < kend; ++kb) {
                const int wi = 2 * kb + (t >> 1);
                const uint32_t wA = (vA && wi < p.wv) ? rowA[wi] << sh0 : 0u;
                const uint32_t wB = (vB && wi < p.wv) ? rowB[wi] << sh0 : 0u;
                const int kc = 64 * kb + 16 * t;
                uint32_t sp[8], xp[8];
                load16_smem(sw + kc / 2, sp);
                if (!xrow) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) xp[j] = 0u;
                } else if (p.x_in_smem) {
                    load16_smem(xsw + kc / 2, xp);
                } else {
                    load16_global<T>(xg, kc, p.in_f, xp);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t a0 = lop_sign(wA << (2 * j), sp[2 * j]);
                    const uint32_t a1 = lop_sign(wB << (2 * j), sp[2 * j]);
                    const uint32_t a2 = lop_sign(wA << (2 * j + 1), sp[2 * j + 1]);
                    const uint32_t a3 = lop_sign(wB << (2 * j + 1), sp[2 * j + 1]);
                    E::mma(acc[j], a0, a1, a2, a3, xp[2 * j], xp[2 * j + 1]);
                }
            }
        }
        float sum[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sum[i] = (acc[0][i] + acc[1][i]) + (acc[2][i] + acc[3][i]);
        store_partial(red + (warp * S + (lt - lt0)) * 256, sum, g, t);
    }
}

// Stage 1, second half: sum the warps' partials, apply scale_mid, store t as bf16 (hi, lo) into
// each member's stage-2 operand, and zero its K padding (the CTA owning the member's last tile).
template <typename T, int FOLD = -1>
__device__ __forceinline__ void stage1_finish(const Params &p, const float *red, int t1b, int t1e, const WarpTab *wt) {
    using E = Elem<T>;
    const bool fold = FOLD >= 0 ? FOLD != 0 : p.fold != 0;
    const int tid = threadIdx.x;
    const int ntiles = t1e - t1b;
    for (int i = tid; i < ntiles * 16 * p.batch; i += kThreads) {
        const int lt = i / (16 * p.batch), rem = i - lt * 16 * p.batch;
        const int b = rem >> 4, row = rem & 15;
        const float s0 = fold ? sum_partials(red, wt, p.seg1, lt, row * 8 + 2 * b, true)
                                : sum_partials(red, wt, p.seg1, lt, row * 8 + b, false);
        float s = s0;
        const int tile = t1b + lt;
        const int l = member_of1(p, tile);
        const Member &mb = p.m[l];
        const int k = 16 * (tile - mb.t1_start) + row;
        if (k < mb.rank) {
            if (mb.smid) s *= E::to_f(static_cast<const T *>(mb.smid)[k]);
            const __nv_bfloat16 hi = __float2bfloat16_rn(s);
            const int col = (b >> 2) * 8 + 2 * (b & 3);
            mb.tb[(size_t)col * mb.ldi + k] = hi;
            mb.tb[(size_t)(col + 1) * mb.ldi + k] = __float2bfloat16_rn(s - __bfloat162float(hi));
        }
    }
    // the CTA owning a member's last stage-1 tile zeroes that member's K padding [rank, ldi)
    for (int l = 0; l < p.nm; ++l) {
        const Member &mb = p.m[l];
        const int last = mb.t1_start + mb.tiles1 - 1;
        const int padw = mb.ldi - mb.rank;
        if (last >= t1b && last < t1e && padw > 0)
            for (int i = tid; i < 16 * padw; i += kThreads) {
                const int col = i / padw;
                mb.tb[(size_t)col * mb.ldi + mb.rank + (i - col * padw)] = __float2bfloat16_rn(0.f);
            }
    }
}

// Stage 2: this CTA's tiles [t2b, t2e) of U against t, split like stage 1; partials into `red`.
// NT = 8-column B tiles: (hi, lo) of 4 batch rows each, so 1 for batch <= 4; the members' t
// columns are read from global memory (L2), where stage 1 left them.
template <typename T, int NT>
__device__ __forceinline__ void stage2_items(const Params &p, const uint32_t *uch, float *red, int t2b, int t2e,
                                             bool ok, WarpTab *wt) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int sh0 = 8 * (t & 1);
    constexpr int nt = NT;
    // units: KB = the largest member's K blocks per tile; a smaller member's tiles end early
    const int ntiles = t2e - t2b, KB = p.kbu2, S = p.seg2;
    int u0, u1;
    warp_units(ntiles * KB, warp, u0, u1);
    const int lt0 = u0 / KB;
    record_range(wt, warp, u0, u1, KB);
    // B column g of n-tile q is the hi (g even) or lo (g odd) part of batch row 4q + g/2,
    // stored ready-made by stage 1 as bf16 pairs along k
    const int b0 = g >> 1, b1 = 4 + (g >> 1);
    const bool v0 = b0 < p.batch, v1 = nt == 2 && b1 < p.batch;
    constexpr int kChunkKb = 4;  // K blocks whose B fragments are fetched together
    for (int lt = lt0; u0 < u1 && lt * KB < u1; ++lt) {
        const int tile = t2b + lt;
        const int l = member_of2(p, tile);
        const Member &mb = p.m[l];
        const int kbeg = max(u0 - lt * KB, 0), kend = min(min(u1 - lt * KB, KB), mb.kb2);
        // this tile's rows in the smem U region: after the earlier members' segments
        uint32_t uoff = 0;
        for (int q = 0; q < l; ++q) {
            int a, b;
            seg_tiles(p.m[q], t2b, t2e, a, b);
            if (a < b) uoff = ((uoff + (uint32_t)(16 * (b - a)) * (uint32_t)p.m[q].wus) + 3u) & ~3u;
        }
        int a0, b0s;
        seg_tiles(mb, t2b, t2e, a0, b0s);
        const int row0 = 16 * (tile - mb.t2_start);
        const bool vA = ok && (row0 + g < mb.out_f), vB = ok && (row0 + g + 8 < mb.out_f);
        const uint32_t *rowA = uch + uoff + (size_t)(16 * (tile - a0) + g) * mb.wus;
        const uint32_t *rowB = rowA + (size_t)8 * mb.wus;
        const __nv_bfloat16 *trow0 = mb.tb + (size_t)g * mb.ldi;
        const __nv_bfloat16 *trow1 = mb.tb + (size_t)(8 + g) * mb.ldi;
        float acc0[4][4] = {}, acc1[NT][4][4] = {};
        for (int kb0 = kbeg; kb0 < kend; kb0 += kChunkKb) {
            uint32_t bp0[kChunkKb][8], bp1[NT][kChunkKb][8];
#pragma unroll
            for (int q = 0; q < kChunkKb; ++q) {
                const int kc = 64 * (kb0 + q) + 16 * t;
                const bool in = kb0 + q < kend;
                load_t_pairs(trow0 + kc, in && v0, bp0[q]);
                if (NT == 2) load_t_pairs(trow1 + kc, in && v1, bp1[NT - 1][q]);
            }
#pragma unroll
            for (int q = 0; q < kChunkKb; ++q) {
                const int kb = kb0 + q;
                if (kb >= kend) break;
                const int wi = 2 * kb + (t >> 1);
                const uint32_t wA = (vA && wi < mb.wu) ? rowA[wi] << sh0 : 0u;
                const uint32_t wB = (vB && wi < mb.wu) ? rowB[wi] << sh0 : 0u;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t a[4];
                    sign_frag(wA, wB, j, a);
                    mma_bf16_16816(acc0[j], a[0], a[1], a[2], a[3], bp0[q][2 * j], bp0[q][2 * j + 1]);
                    if (NT == 2)
                        mma_bf16_16816(acc1[NT - 1][j], a[0], a[1], a[2], a[3], bp1[NT - 1][q][2 * j],
                                       bp1[NT - 1][q][2 * j + 1]);
                }
            }
        }
        float s0[4], s1v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            s0[i] = (acc0[0][i] + acc0[1][i]) + (acc0[2][i] + acc0[3][i]);
            s1v[i] = (acc1[NT - 1][0][i] + acc1[NT - 1][1][i]) + (acc1[NT - 1][2][i] + acc1[NT - 1][3][i]);
        }
        store_partial(red + (warp * S + (lt - lt0)) * 256, s0, g, t);
        if (NT == 2) store_partial(red + (warp * S + (lt - lt0)) * 256 + 128, s1v, g, t);
    }
}

// Stage 2, second half: reduce, scale by s1, round, and store y (optionally y = y + res).
template <typename T>
__device__ __forceinline__ void stage2_finish(const Params &p, const float *red, const T *s1s, int t2b, int t2e,
                                              const void *res, int act, const WarpTab *wt, const TpX *push = nullptr,
                                              unsigned push_e = 0, T *stage = nullptr) {
    using E = Elem<T>;
    const int tid = threadIdx.x;
    const int ntiles = t2e - t2b;
    for (int i = tid; i < ntiles * 16 * p.batch; i += kThreads) {
        const int lt = i / (16 * p.batch), rem = i - lt * 16 * p.batch;
        const int b = rem >> 4, row = rem & 15;
        const int half = (b >> 2) * 128, col = 2 * (b & 3);
        const float s = sum_partials(red, wt, p.seg2, lt, half + row * 8 + col, true);
        const int tile = t2b + lt;
        const int l = member_of2(p, tile);
        const Member &mb = p.m[l];
        const int m = 16 * (tile - mb.t2_start) + row;
        if (m < mb.out_f) {
            const float v = s * E::to_f(s1s[16 * lt + row]);
            const size_t o = (size_t)b * mb.out_f + m;
            T out = E::out(v);
            if ((act >> l) & 1) {  // SiLU on the rounded output, rounded again (the SwiGLU gate)
                const float g = E::to_f(out);
                out = E::rn(g / (1.f + expf(-g)));
            }
            if (res) {  // residual add on the rounded output; res may alias y (same element, same thread)
                const unsigned short rb = __ldcg(reinterpret_cast<const unsigned short *>(res) + o);
                out = E::rn(E::to_f(out) + E::to_f(*reinterpret_cast<const T *>(&rb)));
            }
            static_cast<T *>(mb.y)[o] = out;
            if (push) stage[i] = out;  // staged for the flagged pair stores below
        }
    }
    if (push) {  // every rank's receive buffer for this source: one flagged word per row pair
        __syncthreads();
        const int n = ntiles * 16 * p.batch;
        for (int i = 2 * tid; i < n; i += 2 * kThreads) {
            const int lt = i / (16 * p.batch), rem = i - lt * 16 * p.batch;
            const int b = rem >> 4, row = rem & 15;  // row is even: pairs never straddle a tile
            const int tile = t2b + lt;
            const Member &mb = p.m[member_of2(p, tile)];
            const int m = 16 * (tile - mb.t2_start) + row;
            if (m >= mb.out_f) continue;
            const uint32_t vals = (uint32_t)*reinterpret_cast<const uint16_t *>(&stage[i]) |
                                  ((uint32_t)*reinterpret_cast<const uint16_t *>(&stage[i + 1]) << 16);
            const int64_t word = ((int64_t)b * mb.out_f + m) >> 1;
            for (int d = 0; d < push->world; ++d) tp_st_word(tp_words(*push, d, push_e, push->rank) + word, vals, push_e);
        }
    }
}

// x' in place in shared memory (x rows, x2 rows and the norm weight staged by the prologue):
// RMSNORM: h = dtype(x + x2) (x alone without x2), res_out = h (by `owner`),
// x' = dtype(w * dtype(h * rsqrt(mean(h^2) + eps))); MUL: x' = dtype(x * x2);
// SILU_MUL: x' = dtype(dtype(silu(x)) * x2).  The same roundings as the separate kernels.
template <typename T, bool SILU = true>
__device__ __forceinline__ void x_transform(const Params &p, T *xs, const T *x2s, const T *nws, int in_pad, bool owner,
                                            float *sred) {
    using E = Elem<T>;
    const int n8 = p.in_f / 8;
    for (int b = 0; b < p.batch; ++b) {
        uint4 *xr = reinterpret_cast<uint4 *>(xs + (size_t)b * in_pad);
        const uint4 *x2r = reinterpret_cast<const uint4 *>(x2s + (size_t)b * in_pad);
        if (p.xmode == kChainNorm) {
            uint4 *ro = owner && p.res_out
                            ? reinterpret_cast<uint4 *>(static_cast<T *>(p.res_out) + (size_t)b * p.in_f)
                            : nullptr;
            float ss = 0.f;
#pragma unroll 1
            for (int ch = threadIdx.x; ch < n8; ch += kThreads) {
                float h[8];
                unpack8<T>(xr[ch], h);
                if (p.x2) {
                    float r[8];
                    unpack8<T>(x2r[ch], r);
                    T o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        o[e] = E::rn(h[e] + r[e]);
                        h[e] = E::to_f(o[e]);
                    }
                    xr[ch] = *reinterpret_cast<const uint4 *>(o);
                }
                if (ro) ro[ch] = xr[ch];
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += h[e] * h[e];
            }
            const float inv = rsqrtf(block_sum_512(ss, sred) / (float)p.in_f + p.eps);
            const uint4 *wr = reinterpret_cast<const uint4 *>(nws);
#pragma unroll 1
            for (int ch = threadIdx.x; ch < n8; ch += kThreads) {
                float h[8], w[8];
                unpack8<T>(xr[ch], h);
                unpack8<T>(wr[ch], w);
                T o[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = E::rn(w[e] * E::to_f(E::rn(h[e] * inv)));
                xr[ch] = *reinterpret_cast<const uint4 *>(o);
            }
        } else {
            const bool silu = SILU && p.xmode == kChainSiluMul;
#pragma unroll 1
            for (int ch = threadIdx.x; ch < n8; ch += kThreads) {
                float a[8], u[8];
                unpack8<T>(xr[ch], a);
                unpack8<T>(x2r[ch], u);
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
}

// DECODE = true: the instantiation for fused launches with x staged and folded (batch <= 2,
// the decode case) -- only that path is compiled, which keeps its code small enough for the
// instruction cache; DECODE = false decides every variant at run time.
template <typename T, bool DECODE, bool TP>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const Params p, const TpX tp) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float sred[kWarps];
    __shared__ WarpTab wtab;
    __shared__ unsigned s_tp_epoch;
    using E = Elem<T>;
    const bool x_in_smem = DECODE || p.x_in_smem;
    const bool fold = DECODE || p.fold;
    const int tid = threadIdx.x;
    const int G = gridDim.x, c = blockIdx.x;
    const bool do1 = DECODE || (p.mode & kStage1) != 0, do2 = DECODE || (p.mode & kStage2) != 0;
    unsigned long long bar_base = 0;  // thread 0 only; read after pdl_wait
#ifdef NQ_GEMV_TRACE
    unsigned long long tr_[kTraceStamps] = {};
    unsigned int tr_slot = 0;
#endif
    NQ_STAMP(0);
    pdl_launch_dependents();
    // First touches of the parameter block miss the parameter cache; lane 0 of eight warps
    // reads one field each from different parts of it so that those misses overlap (the
    // prologue would otherwise take them one after another).
    if ((tid & 31) == 0 && tid < 8 * 32) {
        const int w = tid >> 5;
        const Member &mw = p.m[w < 3 ? w : w - 3];
        const uintptr_t v = w < 3 ? reinterpret_cast<uintptr_t>(mw.s2) ^ (uintptr_t)mw.t2_start
                                  : w < 6 ? (uintptr_t)mw.wus ^ reinterpret_cast<uintptr_t>(mw.tb)
                                          : w == 6 ? reinterpret_cast<uintptr_t>(p.x) ^ (uintptr_t)p.nm
                                                   : (uintptr_t)p.off_s1 ^ (uintptr_t)p.xmode;
        if (v == 1) sred[w] = 0.f;  // never true in practice; keeps the loads
    }

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    float *red = reinterpret_cast<float *>(smem + p.off_red);
    T *s2s = reinterpret_cast<T *>(smem + p.off_s2);              // [nm][in_pad]
    T *xs = reinterpret_cast<T *>(smem + p.off_x);                // [batch][in_pad]
    __nv_bfloat16 *xs2 = reinterpret_cast<__nv_bfloat16 *>(smem + p.off_xs2);  // [nm][2*batch][in_pad]
    uint32_t *vch = reinterpret_cast<uint32_t *>(smem + p.off_v); // [16 * tiles][wvs]
    uint32_t *uch = reinterpret_cast<uint32_t *>(smem + p.off_u); // per-member segments
    T *s1s = reinterpret_cast<T *>(smem + p.off_s1);              // [16 * tiles]

    int t1b = 0, t1e = 0, t2b = 0, t2e = 0;
    if (do1) tile_range(p.tiles1, c, G, t1b, t1e);
    if (do2) tile_range(p.tiles2, c, G, t2b, t2e);
    const bool has1 = t1e > t1b, has2 = t2e > t2b;
    const int in_pad = p.kb1 * 64;

    // Copies are issued by separate warps so that their issue latencies (several hundred cycles
    // each: the copy engine accepts a request only after translating its source) overlap.
    // Barrier 0 (V side): warp 0 the s2 rows, warp 1 x and the transform inputs, warp 2 the V
    // slabs.  Barrier 1 (U side): warp 3 the U slabs, warp 4 the s1 slices.  Each issuing warp
    // arrives once with the bytes it put in flight (zero when it has none), so a barrier
    // completes only after every issuer declared its bytes and all of them landed.  Bytes the
    // copy engine cannot take (unaligned rows, sub-16-byte tails) are loaded by all threads.
    constexpr int kIssuers0 = 3, kIssuers1 = 2;
    if (tid == 0) {
        mbar_init(&bars[0], kIssuers0);
        mbar_init(&bars[1], kIssuers1);
        fence_mbar_init();
    }
    __syncthreads();
    bool vec_rows = true;  // DECODE: the host checked the alignment
    if (!DECODE) {
        vec_rows = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 && (p.in_f % 8) == 0;
        _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm) vec_rows = vec_rows && (reinterpret_cast<uintptr_t>(p.m[l].s2) & 15) == 0;
    }
    const int warp_id = tid >> 5;
    // Weight-side copies first: they do not depend on the previous kernel, so under programmatic
    // dependent launch they overlap its tail.  Everything that reads the previous kernel's
    // output (x and the transform inputs, the barrier counter) comes after pdl_wait.
    if (has1) {
        if ((tid & 31) == 0 && (warp_id == 0 || warp_id == 2)) {
            uint32_t bytes = 0;
            if (warp_id == 0) {  // s2 of the members whose stage-1 tiles this CTA owns
                if (vec_rows)
                    _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm && owns1(p.m[l], t1b, t1e))
                        bytes += (uint32_t)p.in_f * 2u;
                mbar_arrive_expect_tx(&bars[0], bytes);
                if (vec_rows)
                    _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm && owns1(p.m[l], t1b, t1e))
                        bulk_g2s_pieces(s2s + (size_t)l * in_pad, p.m[l].s2, (uint32_t)p.in_f * 2u, &bars[0]);
            } else {
                _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm) {
                    const Member &mb = p.m[l];
                    const int a = max(t1b, mb.t1_start), b = min(t1e, mb.t1_start + mb.tiles1);
                    if (a < b)
                        bytes += slab_bulk_bytes(16 * (a - mb.t1_start), min(16 * (b - mb.t1_start), mb.rank), p.wv, false);
                }
                mbar_arrive_expect_tx(&bars[0], bytes);
                _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm) {
                    const Member &mb = p.m[l];
                    const int a = max(t1b, mb.t1_start), b = min(t1e, mb.t1_start + mb.tiles1);
                    if (a < b)
                        slab_bulk(vch + (size_t)16 * (a - t1b) * p.wvs, mb.vbits, 16 * (a - mb.t1_start),
                                  min(16 * (b - mb.t1_start), mb.rank), p.wv, &bars[0]);
                }
            }
        }
        // what the copy engine does not carry: slab tails (none in DECODE launches: the host
        // checked that every slab is a multiple of 16 bytes), zero padding, unaligned rows
        if (!DECODE) _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm) {
            const Member &mb = p.m[l];
            const int a = max(t1b, mb.t1_start), b = min(t1e, mb.t1_start + mb.tiles1);
            if (a < b)
                slab_tail(vch + (size_t)16 * (a - t1b) * p.wvs, mb.vbits, 16 * (a - mb.t1_start),
                          min(16 * (b - mb.t1_start), mb.rank), p.wv);
        }
        if (!DECODE) _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm && owns1(p.m[l], t1b, t1e)) {
            if (vec_rows) {
                zero_tail<T>(s2s + (size_t)l * in_pad, p.in_f, in_pad);
            } else {
                stage_row<T>(s2s + (size_t)l * in_pad, static_cast<const T *>(p.m[l].s2), p.in_f, in_pad);
            }
        }
    }
    if (has2) {
        // U slabs and s1 slices, one segment per member; segment k of the smem U region starts
        // after the previous segments' rows (each rounded up to 4 words)
        if ((tid & 31) == 0 && (warp_id == kIssuers0 || warp_id == kIssuers0 + 1)) {
            const bool u_side = warp_id == kIssuers0;
            uint32_t bytes = 0;
            _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm) {
                const Member &mb = p.m[l];
                int a, b;
                seg_tiles(mb, t2b, t2e, a, b);
                if (a >= b) continue;
                const int r0 = 16 * (a - mb.t2_start), r1 = min(16 * (b - mb.t2_start), mb.out_f);
                if (u_side) {
                    bytes += slab_bulk_bytes(r0, r1, mb.wu, false);
                } else {
                    const T *s1src = static_cast<const T *>(mb.s1) + r0;
                    if ((reinterpret_cast<uintptr_t>(s1src) & 15) == 0) bytes += ((uint32_t)(r1 - r0) * 2u) & ~15u;
                }
            }
            mbar_arrive_expect_tx(&bars[1], bytes);
            uint32_t uoff = 0;  // words
            _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm) {
                const Member &mb = p.m[l];
                int a, b;
                seg_tiles(mb, t2b, t2e, a, b);
                if (a >= b) continue;
                const int r0 = 16 * (a - mb.t2_start), r1 = min(16 * (b - mb.t2_start), mb.out_f);
                if (u_side) {
                    slab_bulk(uch + uoff, mb.ubits, r0, r1, mb.wu, &bars[1]);
                } else {
                    const T *s1src = static_cast<const T *>(mb.s1) + r0;
                    const uint32_t s1_bulk =
                        (reinterpret_cast<uintptr_t>(s1src) & 15) == 0 ? ((uint32_t)(r1 - r0) * 2u) & ~15u : 0u;
                    if (s1_bulk) bulk_g2s(s1s + 16 * (a - t2b), s1src, s1_bulk, &bars[1]);
                }
                uoff += (uint32_t)(16 * (b - a)) * (uint32_t)mb.wus;
                uoff = (uoff + 3u) & ~3u;
            }
        }
        uint32_t uoff = 0;  // words
        if (!DECODE) _Pragma("unroll 1") for (int l = 0; l < kMaxGroup; ++l) if (l < p.nm) {
            const Member &mb = p.m[l];
            int a, b;
            seg_tiles(mb, t2b, t2e, a, b);
            if (a >= b) continue;
            const int r0 = 16 * (a - mb.t2_start), r1 = min(16 * (b - mb.t2_start), mb.out_f);
            slab_tail(uch + uoff, mb.ubits, r0, r1, mb.wu);
            uoff += (uint32_t)(16 * (b - a)) * (uint32_t)mb.wus;
            uoff = (uoff + 3u) & ~3u;  // keep every segment 16-byte aligned
            const T *s1src = static_cast<const T *>(mb.s1) + r0;
            T *s1dst = s1s + 16 * (a - t2b);
            const uint32_t s1_bulk =
                (reinterpret_cast<uintptr_t>(s1src) & 15) == 0 ? ((uint32_t)(r1 - r0) * 2u) & ~15u : 0u;
            for (int i = (int)(s1_bulk / 2) + tid; i < r1 - r0; i += kThreads) s1dst[i] = s1src[i];
        }
    }
    __syncthreads();
    NQ_STAMP(1);

    pdl_wait();  // the previous kernel on the stream has completed; its outputs are visible
    NQ_STAMP(2);
    if (TP && tp.mode && tid == 0) {  // this launch's exchange epoch (after pdl_wait: earlier launches are done)
        unsigned *ep = reinterpret_cast<unsigned *>(tp.region[tp.rank] +
                                                    ((tp.mode & kTpPush) ? kTpOffPush : kTpOffPull)) + c;
        s_tp_epoch = *ep + 1u;
        *ep = s_tp_epoch;
    }
    const bool pull = TP && (tp.mode & kTpPull) != 0;
#ifdef NQ_GEMV_TRACE
    if (tid == 0) tr_slot = *reinterpret_cast<volatile unsigned int *>(&g_trace_launch);
#endif
    if (tid == 0 && (DECODE || p.mode == kFused)) bar_base = grid_barrier_base(p.ctrl, (unsigned)G);
    if (has1) {
        if (tid == 32) {  // warp 1: x and the transform inputs
            uint32_t bytes = 0;
            // transform inputs: the host guarantees vec_rows and x in shared memory for them
            // (a PULL launch forms x from the ranks' receive buffers instead)
            if (vec_rows && x_in_smem && !pull) bytes += (uint32_t)p.in_f * 2u * (uint32_t)p.batch;
            if (p.x2) bytes += (uint32_t)p.in_f * 2u * (uint32_t)p.batch;
            if (p.xmode == kChainNorm) bytes += (uint32_t)p.in_f * 2u;
            mbar_arrive_expect_tx(&bars[0], bytes);
            if (vec_rows && x_in_smem && !pull) {
                if (DECODE || in_pad == p.in_f)  // DECODE: in_f is a multiple of 64 (no padding)
                    bulk_g2s_pieces(xs, p.x, (uint32_t)p.batch * (uint32_t)p.in_f * 2u, &bars[0]);
                else
                    for (int b = 0; b < p.batch; ++b)
                        bulk_g2s_pieces(xs + (size_t)b * in_pad, static_cast<const T *>(p.x) + (size_t)b * p.in_f,
                                        (uint32_t)p.in_f * 2u, &bars[0]);
            }
            if (p.x2 && (DECODE || in_pad == p.in_f))
                bulk_g2s_pieces(smem + p.off_x2, p.x2, (uint32_t)p.batch * (uint32_t)p.in_f * 2u, &bars[0]);
            else if (p.x2)
                for (int b = 0; b < p.batch; ++b)
                    bulk_g2s_pieces(smem + p.off_x2 + (size_t)b * in_pad * 2,
                                    static_cast<const T *>(p.x2) + (size_t)b * p.in_f, (uint32_t)p.in_f * 2u,
                                    &bars[0]);
            if (p.xmode == kChainNorm) bulk_g2s_pieces(smem + p.off_nw, p.nw, (uint32_t)p.in_f * 2u, &bars[0]);
        }
        if (!DECODE && x_in_smem)
            for (int b = 0; b < p.batch; ++b) {
                if (vec_rows)
                    zero_tail<T>(xs + (size_t)b * in_pad, p.in_f, in_pad);
                else
                    stage_row<T>(xs + (size_t)b * in_pad, static_cast<const T *>(p.x) + (size_t)b * p.in_f, p.in_f,
                                 in_pad);
            }
    }
    __syncthreads();

    bool ok = true;
    // ------------------------------------------------------------------ stage 1
    if (has1) {
        ok = mbar_wait(&bars[0], 0, &p.ctrl->status);
        if (pull) {  // x = sum over ranks (rank order) of their pushed partials, rounded once
            __syncthreads();  // s_tp_epoch
            const unsigned e = s_tp_epoch;
            const int n8 = p.in_f / 8;
            for (int i = tid; i < p.batch * n8; i += kThreads) {
                const int b = i / n8, ch = i - b * n8;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                for (int src = 0; src < tp.world; ++src) {
                    uint32_t w4[4];
                    if (!tp_read8(tp, e, src, (int64_t)i * 4, w4, &p.ctrl->status)) ok = false;
                    float v[8];
                    unpack8<T>(make_uint4(w4[0], w4[1], w4[2], w4[3]), v);
#pragma unroll
                    for (int q = 0; q < 8; ++q) acc[q] += v[q];
                }
                T o[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) o[q] = E::rn(acc[q]);
                reinterpret_cast<uint4 *>(xs + (size_t)b * in_pad)[ch] = *reinterpret_cast<const uint4 *>(o);
            }
            __syncthreads();
        }
        NQ_STAMP(3);
        const int nxc = 2 * p.batch;  // folded B columns per member: hi / lo of x*s2 per batch row
        if (p.xmode != kChainPlain) {
            x_transform<T, !DECODE>(p, xs, reinterpret_cast<const T *>(smem + p.off_x2), reinterpret_cast<const T *>(smem + p.off_nw),
                           in_pad, t1b == 0, sred);
            __syncthreads();
        }
        NQ_STAMP(4);
        if (fold) {
            // xs2[l][col][k] = bf16 hi (col even) / lo (col odd) of x[col/2][k] * s2_l[k]
            // (members and batch rows outside, 8-value chunks inside: no runtime divisions)
            const int chunks = in_pad / 8;
#pragma unroll 1
            for (int l = 0; l < kMaxGroup; ++l)
                if (l < p.nm && owns1(p.m[l], t1b, t1e))
                    for (int b = 0; b < p.batch; ++b)
                        for (int c8 = tid; c8 < chunks; c8 += kThreads) {
                            const int k = 8 * c8;
                            const uint4 xv = *reinterpret_cast<const uint4 *>(xs + (size_t)b * in_pad + k);
                            const uint4 sv = *reinterpret_cast<const uint4 *>(s2s + (size_t)l * in_pad + k);
                            const T *xe = reinterpret_cast<const T *>(&xv);
                            const T *se = reinterpret_cast<const T *>(&sv);
                            uint32_t hi[4], lo[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                split_pair(E::to_f(xe[2 * j]) * E::to_f(se[2 * j]),
                                           E::to_f(xe[2 * j + 1]) * E::to_f(se[2 * j + 1]), hi[j], lo[j]);
                            __nv_bfloat16 *dst = xs2 + ((size_t)l * nxc + 2 * b) * in_pad + k;
                            *reinterpret_cast<uint4 *>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                            *reinterpret_cast<uint4 *>(dst + in_pad) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        }
            __syncthreads();
        }
        NQ_STAMP(5);
        stage1_items<T, DECODE ? 1 : -1>(p, vch, s2s, xs, xs2, red, t1b, t1e, ok, &wtab);
        __syncthreads();
        NQ_STAMP(6);
        stage1_finish<T, DECODE ? 1 : -1>(p, red, t1b, t1e, &wtab);
    }
    NQ_STAMP(7);

    if (DECODE || p.mode == kFused) {
        if (!grid_barrier(p.ctrl, bar_base + (unsigned)G)) ok = false;
    } else if (has1 && do2) {
        __syncthreads();
    }
    NQ_STAMP(8);

    // ------------------------------------------------------------------ stage 2
    if (has2) {
        if (!mbar_wait(&bars[1], 0, &p.ctrl->status)) ok = false;
        NQ_STAMP(9);
        if (DECODE || p.batch <= 4)
            stage2_items<T, 1>(p, uch, red, t2b, t2e, ok, &wtab);
        else
            stage2_items<T, 2>(p, uch, red, t2b, t2e, ok, &wtab);
        __syncthreads();
        NQ_STAMP(10);
        // a PUSH stages its rows in the x region (stage 1 is over; the host checked its size)
        stage2_finish<T>(p, red, s1s, t2b, t2e, nullptr, p.act, &wtab, (TP && (tp.mode & kTpPush)) ? &tp : nullptr,
                         s_tp_epoch, xs);
    }
    NQ_STAMP(11);
#ifdef NQ_GEMV_TRACE
    if (tid == 0 && tr_slot < kTraceLaunches && c < kTraceCtas) {
        for (int i = 0; i < kTraceStamps; ++i) g_trace[tr_slot][c][i] = tr_[i];
        if (c == 0) atomicAdd(&g_trace_launch, 1u);
    }
#endif
}

struct Plan {
    int mode = kFused;
    int grid = 0, grid1 = 0, grid2 = 0;
    size_t smem = 0, smem1 = 0, smem2 = 0;
    Params prm{};
    Params prm1{}, prm2{};
};

static inline uint32_t align128(size_t v) { return (uint32_t)((v + 127) & ~size_t(127)); }

// Shared-memory row stride (words) for a plane with w words per row copied row by row:
// a multiple of 4 words (16-byte aligned rows) that is an odd multiple of 4, so rows
// g = 0..7 of an MMA tile start in 8 different 4-bank groups and the per-k sign-word
// loads are conflict free.
static inline int padded_stride(int w) {
    int s = (w + 3) & ~3;
    if (((s / 4) & 1) == 0) s += 4;
    return s;
}

// Shared-memory layout for a launch whose CTAs own at most `tiles1`/`tiles2` tiles.
// `push_rows`: a stage-2-only launch that PUSHes its rows gets a staging region for them
// (a launch with stage 1 stages them in its x region).
static size_t layout(Params &p, int tiles1, int tiles2, bool stage1, bool stage2, bool x_in_smem, bool fold,
                     bool push_rows = false) {
    size_t off = 128;  // mbarriers
    p.kbu2 = 1;
    for (int l = 0; l < p.nm; ++l) p.kbu2 = std::max(p.kbu2, p.m[l].kb2);
    p.seg1 = seg_bound(tiles1, p.kb1);
    p.seg2 = seg_bound(tiles2, p.kbu2);
    const int slots = kWarps * std::max(stage1 ? p.seg1 : 1, stage2 ? p.seg2 : 1);
    p.off_red = (uint32_t)off;
    off = align128(off + (size_t)slots * 256 * sizeof(float));
    const size_t in_pad = (size_t)p.kb1 * 64;
    // Every slab goes in one contiguous bulk copy: the copy engine takes row copies one at a
    // time (a 32-row slab costs ~1.5 us to issue), which outweighs the bank conflicts that an
    // unpadded stride (a multiple of 32 words) gives the sign-word loads.
    p.v_rows = 0;
    p.wvs = p.v_rows ? padded_stride(p.wv) : p.wv;
    int max_wus = 0;
    for (int l = 0; l < p.nm; ++l) {
        p.m[l].u_rows = 0;
        p.m[l].wus = p.m[l].u_rows ? padded_stride(p.m[l].wu) : p.m[l].wu;
        max_wus = std::max(max_wus, p.m[l].wus);
    }
    p.off_s2 = p.off_x = p.off_xs2 = p.off_v = (uint32_t)off;
    p.fold = 0;
    if (stage1) {
        off = align128(off + (size_t)p.nm * in_pad * 2);
        p.off_x = (uint32_t)off;
        if (x_in_smem) off = align128(off + (size_t)p.batch * in_pad * 2);
        p.off_x2 = (uint32_t)off;  // transform inputs, staged next to x
        if (x_in_smem && p.x2) off = align128(off + (size_t)p.batch * in_pad * 2);
        p.off_nw = (uint32_t)off;
        if (x_in_smem && p.xmode == kChainNorm) off = align128(off + (size_t)in_pad * 2);
        p.off_xs2 = (uint32_t)off;
        if (fold && x_in_smem) {
            p.fold = 1;
            off = align128(off + (size_t)p.nm * 2 * p.batch * in_pad * 2);
        }
        p.off_v = (uint32_t)off;
        off = align128(off + (size_t)16 * tiles1 * p.wvs * 4 + 16);
    }
    if (stage2 && !stage1 && push_rows) {
        p.off_x = (uint32_t)off;
        off = align128(off + (size_t)16 * tiles2 * p.batch * 2 + 16);
    }
    p.off_u = (uint32_t)off;
    p.off_s1 = (uint32_t)off;
    if (stage2) {
        // segments of different members are rounded up to 4 words each
        off = align128(off + ((size_t)16 * tiles2 * max_wus + 4 * (size_t)p.nm) * 4 + 16);
        p.off_s1 = (uint32_t)off;
        off = align128(off + (size_t)16 * tiles2 * 2 + 16);
    }
    p.x_in_smem = x_in_smem ? 1 : 0;
    return off;
}

// NQ_GEMV_SPLIT_GRID=tiles gives the two-launch plan one 16-row tile per CTA (its earlier
// form, kept for A/B timing); unset, the split launches run in whole waves (make_plan).
static bool split_one_tile() {
    static const bool v = [] {
        const char *e = std::getenv("NQ_GEMV_SPLIT_GRID");
        return e != nullptr && std::strcmp(e, "tiles") == 0;
    }();
    return v;
}

// `push_rows`: the stage-2 launch of a split plan PUSHes its rows (tensor-parallel exchange).
static int make_plan(int dev, const Params &base, Plan &plan, bool push_rows = false) {
    const DeviceInfo &di = device_info(dev);
    const size_t cap = (size_t)di.max_smem_optin - kStaticSmemReserve;
    const int G = di.sms;
    const Params &p = base;
    // fused: one CTA per SM, tiles spread evenly; prefer x staged and the folded operand
    const int tpc1 = (p.tiles1 + G - 1) / G, tpc2 = (p.tiles2 + G - 1) / G;
    const int variants[3][2] = {{1, 1}, {1, 0}, {0, 0}};  // (x in smem, fold)
    for (const auto &v : variants) {
        if (v[1] && p.batch > kFoldMaxBatch) continue;
        if (p.xmode != kChainPlain && !v[0]) continue;  // a transformed input lives in shared memory
        Params q = p;
        q.mode = kFused;
        const size_t need = layout(q, tpc1, tpc2, true, true, v[0] != 0, v[1] != 0);
        if (need <= cap && di.coop) {
            plan.mode = kFused;
            plan.grid = G;
            plan.smem = need;
            plan.prm = q;
            return NQ_OK;
        }
    }
    // Two ordinary launches (stage 1, then stage 2).  Each spreads its tiles over the fewest
    // whole waves of CTAs (multiples of the SM count; the kernel holds one CTA per SM) whose
    // slabs fit in shared memory: a CTA copies all its tiles' weights at once, so a large layer
    // streams its planes in one wave rather than in tiles / SMs waves of one 16-row tile per
    // CTA, and the per-CTA prologue (x staging, input transform, fold) runs once per CTA, not
    // once per tile.  Stage 1 takes the first variant that fits at the smallest grid.
    const bool one_tile = split_one_tile();
    Params q1{}, q2 = p;
    size_t n1 = 0, n2 = 0;
    int g1 = 0, g2 = 0;
    for (int g = one_tile ? p.tiles1 : std::min(G, p.tiles1); g1 == 0; g = std::min(g + G, p.tiles1)) {
        const int tpc = (p.tiles1 + g - 1) / g;
        for (const auto &v : variants) {
            if (v[1] && p.batch > kFoldMaxBatch) continue;
            if (p.xmode != kChainPlain && !v[0]) continue;
            Params q = p;
            q.mode = kStage1;
            const size_t n = layout(q, tpc, 0, true, false, v[0] != 0, v[1] != 0);
            if (n <= cap) {
                q1 = q;
                n1 = n;
                g1 = g;
                break;
            }
        }
        if (g1 == 0 && g >= p.tiles1) break;
    }
    q2.mode = kStage2;
    for (int g = one_tile ? p.tiles2 : std::min(G, p.tiles2); g2 == 0; g = std::min(g + G, p.tiles2)) {
        const size_t n = layout(q2, 0, (p.tiles2 + g - 1) / g, false, true, false, false, push_rows);
        if (n <= cap) {
            n2 = n;
            g2 = g;
        } else if (g >= p.tiles2) {
            break;
        }
    }
    if (g1 == 0 || g2 == 0)
        return fail(NQ_ERR_UNSUPPORTED, "layer group too large for the shared-memory budget (in=%d)", p.in_f);
    plan.mode = kStage1 | kStage2 | 4;  // marker: split
    plan.grid1 = g1;
    plan.grid2 = g2;
    plan.smem1 = n1;
    plan.smem2 = n2;
    plan.prm1 = q1;
    plan.prm2 = q2;
    return NQ_OK;
}

template <typename T>
static int launch(const Plan &plan, cudaStream_t stream, const TpX &tp) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        const int cap = device_info(dev).max_smem_optin - kStaticSmemReserve;
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<T, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemv_kernel<T, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemv_kernel<T, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemv_kernel<T, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
        attr_set[dev] = true;
    }
    // programmatic dependent launch: the kernel waits for its predecessor itself (pdl_wait)
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    if (plan.mode == kFused) {
        // the DECODE instantiation: x staged and folded, batch <= 4, 16-byte aligned rows of x
        // and s2 that need no K padding (in_f a multiple of 64), no SiLU*up input transform
        const Params &q = plan.prm;
        bool vec = (reinterpret_cast<uintptr_t>(q.x) & 15) == 0 && (q.in_f % 8) == 0;
        for (int l = 0; l < q.nm; ++l) vec = vec && (reinterpret_cast<uintptr_t>(q.m[l].s2) & 15) == 0;
        // and every V / U slab and s1 slice a whole number of 16-byte pieces (no tail loads)
        for (int l = 0; l < q.nm; ++l) {
            const Member &mb = q.m[l];
            vec = vec && (q.wv % 4 == 0 || mb.rank % 4 == 0) && (mb.wu % 4 == 0 || mb.out_f % 4 == 0) &&
                  mb.out_f % 8 == 0 && (reinterpret_cast<uintptr_t>(mb.s1) & 15) == 0;
        }
        const bool decode = q.fold && q.x_in_smem && q.batch <= 4 && vec && q.xmode != kChainSiluMul && q.in_f % 64 == 0;
        attr[na].id = cudaLaunchAttributeCooperative;
        attr[na].val.cooperative = 1;
        cfg.numAttrs = na + 1;
        cfg.gridDim = dim3(plan.grid);
        cfg.dynamicSmemBytes = plan.smem;
        // the exchange code is compiled only into the TP instantiations (single-GPU code stays small)
        cudaError_t e = tp.mode ? (decode ? cudaLaunchKernelEx(&cfg, gemv_kernel<T, true, true>, plan.prm, tp)
                                          : cudaLaunchKernelEx(&cfg, gemv_kernel<T, false, true>, plan.prm, tp))
                                : (decode ? cudaLaunchKernelEx(&cfg, gemv_kernel<T, true, false>, plan.prm, tp)
                                          : cudaLaunchKernelEx(&cfg, gemv_kernel<T, false, false>, plan.prm, tp));
        return e == cudaSuccess ? NQ_OK : cuda_fail(e, "gemv fused launch");
    }
    // split: a PULL exchanges in the stage-1 launch (it forms x), a PUSH in the stage-2 launch
    // (it stores y); group_impl checked that launch's grid
    const TpX none{};
    TpX pull = none, push = none;
    if (tp.mode & kTpPull) pull = tp, pull.mode = kTpPull;
    if (tp.mode & kTpPush) push = tp, push.mode = kTpPush;
    cfg.numAttrs = na;
    cfg.gridDim = dim3(plan.grid1);
    cfg.dynamicSmemBytes = plan.smem1;
    cudaError_t e = pull.mode ? cudaLaunchKernelEx(&cfg, gemv_kernel<T, false, true>, plan.prm1, pull)
                              : cudaLaunchKernelEx(&cfg, gemv_kernel<T, false, false>, plan.prm1, none);
    if (e != cudaSuccess) return cuda_fail(e, "gemv stage-1 launch");
    cfg.gridDim = dim3(plan.grid2);
    cfg.dynamicSmemBytes = plan.smem2;
    e = push.mode ? cudaLaunchKernelEx(&cfg, gemv_kernel<T, false, true>, plan.prm2, push)
                  : cudaLaunchKernelEx(&cfg, gemv_kernel<T, false, false>, plan.prm2, none);
    return e == cudaSuccess ? NQ_OK : cuda_fail(e, "gemv stage-2 launch");
}

static inline size_t tb_bytes(int64_t rank) { return (size_t)16 * (size_t)((rank + 63) / 64) * 64 * 2; }

// The input of a launch group: x, or x' formed from x (and x2, norm_weight) as nq_gemv_input says.
struct GroupInput {
    const void *x = nullptr;
    int xmode = kChainPlain;
    const void *x2 = nullptr, *nw = nullptr;
    void *res_out = nullptr;
    float eps = 0.f;
    int act = 0;
};

static int group_impl(int dtype, const GroupInput &in, int64_t batch, int64_t in_features, int n,
                      const nq_gemv_layer *layers, void *workspace, size_t workspace_bytes, void *stream,
                      const TpX *tpx = nullptr, bool plan_only = false) {
    const TpX tp = tpx ? *tpx : TpX{};
    const void *x = in.x;
    if (n >= 1 && n <= kMaxGroup) {
        if (in.act & ~((1 << n) - 1)) return fail(NQ_ERR_INVALID_ARGUMENT, "act bit beyond the %d layers", n);
        if (in.xmode != kChainPlain) {
            if (in.xmode != kChainNorm && in.xmode != kChainMul && in.xmode != kChainSiluMul)
                return fail(NQ_ERR_INVALID_ARGUMENT, "unknown x_mode %d", in.xmode);
            if (batch > kMaxBatch)
                return fail(NQ_ERR_UNSUPPORTED, "a transformed input supports batch <= %d (got %lld)", kMaxBatch,
                            (long long)batch);
            if (in_features % 8) return fail(NQ_ERR_UNSUPPORTED, "a transformed input needs in_features %% 8 == 0");
            if (in.xmode != kChainNorm && !in.x2) return fail(NQ_ERR_INVALID_ARGUMENT, "x_mode needs x2");
            if (in.xmode == kChainNorm && !in.nw) return fail(NQ_ERR_INVALID_ARGUMENT, "RMSNORM needs norm_weight");
            uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(in.x2) |
                           reinterpret_cast<uintptr_t>(in.nw) | reinterpret_cast<uintptr_t>(in.res_out);
            for (int l = 0; l < n && layers; ++l) al |= reinterpret_cast<uintptr_t>(layers[l].scale_pre);
            if (al & 15)
                return fail(NQ_ERR_INVALID_ARGUMENT, "x, x2, norm_weight, residual_out and scale_pre must be 16-byte aligned");
        }
    }
    if (dtype != NQ_DTYPE_F16 && dtype != NQ_DTYPE_BF16)
        return fail(NQ_ERR_UNSUPPORTED, "dtype must be NQ_DTYPE_F16 or NQ_DTYPE_BF16 (got %d)", dtype);
    if (n < 1 || n > kMaxGroup) return fail(NQ_ERR_INVALID_ARGUMENT, "a group holds 1..%d layers (got %d)", kMaxGroup, n);
    if (!x || !layers) return fail(NQ_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (batch <= 0 || in_features <= 0)
        return fail(NQ_ERR_INVALID_ARGUMENT, "sizes must be positive (batch=%lld in=%lld)", (long long)batch,
                    (long long)in_features);
    if (in_features > (1 << 24)) return fail(NQ_ERR_UNSUPPORTED, "in_features beyond the supported range");
    if (reinterpret_cast<uintptr_t>(x) & 1) return fail(NQ_ERR_INVALID_ARGUMENT, "x must be 2-byte aligned");
    int64_t tiles1 = 0, tiles2 = 0;
    size_t need = sizeof(Ctrl);
    for (int l = 0; l < n; ++l) {
        const nq_gemv_layer &L = layers[l];
        if (!L.scale_pre || !L.v_bits || !L.u_bits || !L.scale_post || !L.y)
            return fail(NQ_ERR_INVALID_ARGUMENT, "null tensor pointer in layer %d", l);
        if (L.rank <= 0 || L.out_features <= 0)
            return fail(NQ_ERR_INVALID_ARGUMENT, "layer %d: sizes must be positive (rank=%lld out=%lld)", l,
                        (long long)L.rank, (long long)L.out_features);
        if (L.rank > (1 << 20) || L.out_features > (1 << 24))
            return fail(NQ_ERR_UNSUPPORTED, "layer %d: sizes beyond the supported range", l);
        const uintptr_t a2 = reinterpret_cast<uintptr_t>(L.scale_pre) | reinterpret_cast<uintptr_t>(L.scale_post) |
                             reinterpret_cast<uintptr_t>(L.y) | reinterpret_cast<uintptr_t>(L.scale_mid);
        if (a2 & 1) return fail(NQ_ERR_INVALID_ARGUMENT, "layer %d: 16-bit tensors must be 2-byte aligned", l);
        if ((reinterpret_cast<uintptr_t>(L.v_bits) | reinterpret_cast<uintptr_t>(L.u_bits)) & 15)
            return fail(NQ_ERR_INVALID_ARGUMENT, "layer %d: sign planes must be 16-byte aligned", l);
        tiles1 += (L.rank + 15) / 16;
        tiles2 += (L.out_features + 15) / 16;
        need += tb_bytes(L.rank);
    }
    if (tiles1 > 65536 || tiles2 > 65536) return fail(NQ_ERR_UNSUPPORTED, "layer group too large");
    if (!workspace || workspace_bytes < need)
        return fail(NQ_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(NQ_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    const DeviceInfo &di = device_info(dev);
    if (di.cc_major != 10)
        return fail(NQ_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", dev, di.cc_major,
                    di.cc_minor);

    Params base{};
    base.ctrl = static_cast<Ctrl *>(workspace);
    base.in_f = (int)in_features;
    base.wv = (int)((in_features + 31) / 32);
    base.kb1 = (base.wv + 1) / 2;
    base.nm = n;
    char *tbp = static_cast<char *>(workspace) + sizeof(Ctrl);
    int t1 = 0, t2 = 0;
    for (int l = 0; l < n; ++l) {
        const nq_gemv_layer &L = layers[l];
        Member &mb = base.m[l];
        mb.s2 = L.scale_pre;
        mb.vbits = reinterpret_cast<const uint32_t *>(L.v_bits);
        mb.smid = L.scale_mid;
        mb.ubits = reinterpret_cast<const uint32_t *>(L.u_bits);
        mb.s1 = L.scale_post;
        mb.rank = (int)L.rank;
        mb.out_f = (int)L.out_features;
        mb.wu = (int)((L.rank + 31) / 32);
        mb.kb2 = (mb.wu + 1) / 2;
        mb.ldi = mb.kb2 * 64;
        mb.tiles1 = (int)((L.rank + 15) / 16);
        mb.tiles2 = (int)((L.out_features + 15) / 16);
        mb.t1_start = t1;
        mb.t2_start = t2;
        t1 += mb.tiles1;
        t2 += mb.tiles2;
        mb.tb = reinterpret_cast<__nv_bfloat16 *>(tbp);
        tbp += tb_bytes(L.rank);
    }
    base.tiles1 = t1;
    base.tiles2 = t2;
    base.xmode = in.xmode;
    base.x2 = in.x2;
    base.nw = in.nw;
    base.res_out = in.res_out;
    base.eps = in.eps;
    base.act = in.act;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int64_t b0 = 0; b0 < batch; b0 += kMaxBatch) {
        Params p = base;
        p.batch = (int)((batch - b0) < kMaxBatch ? (batch - b0) : kMaxBatch);
        p.x = static_cast<const char *>(x) + (size_t)b0 * in_features * 2;
        for (int l = 0; l < n; ++l)
            p.m[l].y = static_cast<char *>(layers[l].y) + (size_t)b0 * layers[l].out_features * 2;
        Plan plan;
        int st = make_plan(dev, p, plan, (tp.mode & kTpPush) != 0);
        if (st) return st;
        if (tp.mode) {
            if (batch > kMaxBatch) return fail(NQ_ERR_UNSUPPORTED, "the exchange supports batch <= %d", kMaxBatch);
            // The launch that forms x (PULL: stage 1) and the one that stores y (PUSH: stage 2) run
            // one CTA per SM: every launch of a kind advances the epoch counter of each CTA index.
            // A split plan exchanges in its stage-1 (PULL) or stage-2 (PUSH) launch, not both.
            const bool fused = plan.mode == kFused;
            const int gpull = fused ? plan.grid : plan.grid1, gpush = fused ? plan.grid : plan.grid2;
            const bool xs_ok = fused ? plan.prm.x_in_smem != 0 : plan.prm1.x_in_smem != 0;
            if (((tp.mode & kTpPull) && (gpull != tp.gprod || !xs_ok)) || ((tp.mode & kTpPush) && gpush != tp.gprod) ||
                (!fused && tp.mode == (kTpPull | kTpPush)))
                return fail(NQ_ERR_UNSUPPORTED, "the exchange needs its GEMV launches on %d CTAs", tp.gprod);
            if ((tp.mode & kTpPull) && (p.in_f % 8 || (long long)p.batch * p.in_f > tp.max_elems))
                return fail(NQ_ERR_UNSUPPORTED, "pull: batch * in_features must fit the exchange buffers");
            if ((tp.mode & kTpPush) && (n != 1 || (long long)p.batch * p.m[0].out_f > tp.max_elems ||
                                         p.m[0].out_f % 8 != 0))
                return fail(NQ_ERR_UNSUPPORTED, "push: one layer, out_features % 8 == 0, batch * out within the buffers");
            if ((tp.mode & kTpPush) && fused &&
                (!plan.prm.x_in_smem || (size_t)plan.prm.kb1 * 64 < (size_t)16 * ((p.tiles2 + plan.grid - 1) / plan.grid)))
                return fail(NQ_ERR_UNSUPPORTED, "push: the rows of a CTA must fit its staged-x region");
        }
        if (plan_only) continue;
        st = (dtype == NQ_DTYPE_F16) ? launch<__half>(plan, s, tp) : launch<__nv_bfloat16>(plan, s, tp);
        if (st) return st;
    }
    return NQ_OK;
}

// Standalone PULL (the final norm after the last row-parallel layer): one CTA sums the ranks'
// buffers into `out` and advances every GEMV CTA's pull epoch, keeping them in step.
template <typename T>
__global__ void __launch_bounds__(512) tp_pull_kernel(const TpX tp, int64_t n, T *out) {
    __shared__ unsigned se;
    Ctrl *ctrl = reinterpret_cast<Ctrl *>(tp.region[tp.rank]);
    if ((int)threadIdx.x < tp.gprod) {
        unsigned *ep = reinterpret_cast<unsigned *>(tp.region[tp.rank] + kTpOffPull) + threadIdx.x;
        const unsigned v = *ep + 1u;
        *ep = v;
        if (threadIdx.x == 0) se = v;
    }
    __syncthreads();
    const unsigned e = se;
    for (int64_t i = threadIdx.x; i < n / 8; i += blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int src = 0; src < tp.world; ++src) {
            uint32_t w4[4];
            tp_read8(tp, e, src, i * 4, w4, &ctrl->status);
            float v[8];
            unpack8<T>(make_uint4(w4[0], w4[1], w4[2], w4[3]), v);
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[q] += v[q];
        }
        T o[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = Elem<T>::rn(acc[q]);
        reinterpret_cast<uint4 *>(out)[i] = *reinterpret_cast<const uint4 *>(o);
    }
}

// `need_regions` false: the descriptor of a plan-only check (NQ_TP_CHECK), regions not read.
static int make_tpx(const nq_tp_exchange *x, int mode, TpX &tp, bool need_regions = true) {
    if (!x) return fail(NQ_ERR_INVALID_ARGUMENT, "null exchange descriptor");
    if (x->world < 1 || x->world > kTpMaxWorld || x->rank < 0 || x->rank >= x->world)
        return fail(NQ_ERR_INVALID_ARGUMENT, "exchange: rank %d of world %d (at most %d)", x->rank, x->world, kTpMaxWorld);
    if (x->max_elems <= 0 || x->max_elems % 8)
        return fail(NQ_ERR_INVALID_ARGUMENT, "exchange: max_elems must be a positive multiple of 8");
    tp = TpX{};
    for (int r = 0; r < x->world && need_regions; ++r) {
        if (!x->regions[r] || (reinterpret_cast<uintptr_t>(x->regions[r]) & 255))
            return fail(NQ_ERR_INVALID_ARGUMENT, "exchange: region %d missing or not 256-byte aligned", r);
        tp.region[r] = static_cast<unsigned char *>(x->regions[r]);
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    tp.rank = x->rank;
    tp.world = x->world;
    tp.mode = mode;
    tp.gprod = device_info(dev).sms;  // the single-launch GEMV runs one CTA per SM
    tp.max_elems = x->max_elems;
    if (tp.gprod > kTpMaxCtas) return fail(NQ_ERR_UNSUPPORTED, "exchange: more than %d SMs", kTpMaxCtas);
    return NQ_OK;
}

}  // namespace gemv
}  // namespace nq

extern "C" {

size_t nq_tp_region_bytes(int world, int64_t max_elems) {
    if (world < 1 || world > nq::gemv::kTpMaxWorld || max_elems <= 0) return 0;
    return nq::gemv::kTpOffData + 2 * (size_t)world * (size_t)max_elems * 4;  // 8-byte words per value pair
}

int nq_tp_region_alloc(int world, int64_t max_elems, void **region_out) {
    const size_t bytes = nq_tp_region_bytes(world, max_elems);
    if (!bytes || !region_out)
        return nq::fail(NQ_ERR_INVALID_ARGUMENT, "exchange region: world %d, max_elems %lld", world, (long long)max_elems);
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);  // its own allocation: an IPC handle maps whole allocations
    if (e != cudaSuccess) return nq::cuda_fail(e, "cudaMalloc(exchange region)");
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return nq::cuda_fail(e, "cudaMemset(exchange region)");
    }
    *region_out = p;
    return NQ_OK;
}

int nq_gemv_group_tp(int dtype, const nq_gemv_input *input, int64_t batch, int64_t in_features, int n_layers,
                     const nq_gemv_layer *layers, int act, const nq_tp_exchange *tp, int tp_mode, void *workspace,
                     size_t workspace_bytes, void *stream) {
    using namespace nq::gemv;
    if (!input) return nq::fail(NQ_ERR_INVALID_ARGUMENT, "null input descriptor");
    if (tp_mode & ~(kTpPull | kTpPush | NQ_TP_CHECK))
        return nq::fail(NQ_ERR_INVALID_ARGUMENT, "unknown exchange mode %d", tp_mode);
    const bool check = (tp_mode & NQ_TP_CHECK) != 0;
    tp_mode &= kTpPull | kTpPush;
    if ((tp_mode & kTpPull) && input->x_mode != NQ_CHAIN_X_RMSNORM)
        return nq::fail(NQ_ERR_UNSUPPORTED, "a PULL launch forms its input with RMSNORM");
    TpX tpx{};
    if (tp_mode) {
        const int st = make_tpx(tp, tp_mode, tpx, !check);
        if (st) return st;
    }
    GroupInput in;
    in.x = input->x;
    in.xmode = input->x_mode;
    in.x2 = input->x2;
    in.nw = input->norm_weight;
    in.res_out = input->residual_out;
    in.eps = input->eps;
    in.act = act;
    return group_impl(dtype, in, batch, in_features, n_layers, layers, workspace, workspace_bytes, stream,
                      tp_mode ? &tpx : nullptr, check);
}

int nq_tp_pull(int dtype, const nq_tp_exchange *tp, int64_t n, void *out, void *stream) {
    using namespace nq::gemv;
    if (dtype != NQ_DTYPE_F16 && dtype != NQ_DTYPE_BF16) return nq::fail(NQ_ERR_UNSUPPORTED, "exchange dtype");
    TpX tpx{};
    int st = make_tpx(tp, kTpPull, tpx);
    if (st) return st;
    if (!out || n <= 0 || n % 8 || n > tpx.max_elems || (reinterpret_cast<uintptr_t>(out) & 15))
        return nq::fail(NQ_ERR_INVALID_ARGUMENT, "pull: n must be a multiple of 8 <= max_elems, out 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == NQ_DTYPE_F16)
        tp_pull_kernel<__half><<<1, 512, 0, s>>>(tpx, n, static_cast<__half *>(out));
    else
        tp_pull_kernel<__nv_bfloat16><<<1, 512, 0, s>>>(tpx, n, static_cast<__nv_bfloat16 *>(out));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NQ_OK : nq::cuda_fail(e, "exchange pull launch");
}

size_t nq_gemv_workspace_bytes(int64_t batch, int64_t rank) {
    (void)batch;  // batches above 8 reuse the same 8-row operand buffer, launch after launch
    if (rank <= 0) return 0;
    return sizeof(nq::Ctrl) + nq::gemv::tb_bytes(rank);
}

size_t nq_gemv_group_workspace_bytes(int n_layers, const int64_t *ranks) {
    if (n_layers < 1 || !ranks) return 0;
    size_t need = sizeof(nq::Ctrl);
    for (int l = 0; l < n_layers; ++l) {
        if (ranks[l] <= 0) return 0;
        need += nq::gemv::tb_bytes(ranks[l]);
    }
    return need;
}

int nq_gemv_group(int dtype, const void *x, int64_t batch, int64_t in_features, int n_layers,
                  const nq_gemv_layer *layers, void *workspace, size_t workspace_bytes, void *stream) {
    nq::gemv::GroupInput in;
    in.x = x;
    return nq::gemv::group_impl(dtype, in, batch, in_features, n_layers, layers, workspace, workspace_bytes, stream);
}

int nq_gemv_group_ex(int dtype, const nq_gemv_input *input, int64_t batch, int64_t in_features, int n_layers,
                     const nq_gemv_layer *layers, int act, void *workspace, size_t workspace_bytes, void *stream) {
    if (!input) return nq::fail(NQ_ERR_INVALID_ARGUMENT, "null input descriptor");
    nq::gemv::GroupInput in;
    in.x = input->x;
    in.xmode = input->x_mode;
    in.x2 = input->x2;
    in.nw = input->norm_weight;
    in.res_out = input->residual_out;
    in.eps = input->eps;
    in.act = act;
    return nq::gemv::group_impl(dtype, in, batch, in_features, n_layers, layers, workspace, workspace_bytes, stream);
}

int nq_gemv(int dtype, const void *x, int64_t batch, int64_t in_features, const void *scale_pre,
            const int32_t *v_bits, int64_t rank, const void *scale_mid, const int32_t *u_bits, int64_t out_features,
            const void *scale_post, void *y, void *workspace, size_t workspace_bytes, void *stream) {
    nq_gemv_layer L;
    L.scale_pre = scale_pre;
    L.v_bits = v_bits;
    L.rank = rank;
    L.scale_mid = scale_mid;
    L.u_bits = u_bits;
    L.out_features = out_features;
    L.scale_post = scale_post;
    L.y = y;
    nq::gemv::GroupInput in;
    in.x = x;
    return nq::gemv::group_impl(dtype, in, batch, in_features, 1, &L, workspace, workspace_bytes, stream);
}

}  // extern "C"

// ------------------------------------------------------------------ allocation-free entry point
// Some callers cannot allocate device memory: a plugin or custom-op interface that hands the
// kernel only its input and output buffers (no allocator, no workspace), or a serving process
// that fixes its device memory at start-up and must not call cudaMalloc afterwards (it can
// synchronise the whole device).  nq_gemv_static serves them with scratch that lives in this
// library's own device image: a file-scope static array, resident on every GPU that loads the
// library until the process exits.
namespace nq {
namespace gemv {

constexpr int kStaticMaxRank = NQ_GEMV_STATIC_MAX_RANK;
// control block + stage-2 operand [16 columns][round_up(rank, 64)] bf16 at the largest rank
constexpr size_t kStaticScratchBytes = sizeof(Ctrl) + (size_t)2 * kMaxBatch * kStaticMaxRank * 2;
static_assert(kStaticMaxRank % 64 == 0, "the scratch holds whole 64-column K blocks");

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device.  In host code the array's name
// is only a host-side stand-in, so the address comes from cudaGetSymbolAddress, once per
// device, with that device current.  The cached address belongs to the device's primary
// context: after cudaDeviceReset the library's module is loaded anew and the entry point
// must not be used again in that process.
static int static_scratch(void **out) {
    static std::mutex mu;
    static void *addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(NQ_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static GEMV scratch)");
        addr[dev] = p;
    }
    *out = addr[dev];
    return NQ_OK;
}

}  // namespace gemv
}  // namespace nq

extern "C" {

int nq_gemv_static(int dtype, const void *x, int64_t batch, int64_t in_features, const void *scale_pre,
                   const int32_t *v_bits, int64_t rank, const void *scale_mid, const int32_t *u_bits,
                   int64_t out_features, const void *scale_post, void *y, void *stream) {
    using namespace nq;
    using namespace nq::gemv;
    if (rank > kStaticMaxRank)
        return fail(NQ_ERR_UNSUPPORTED, "nq_gemv_static supports rank <= %d (got %lld); use nq_gemv with a workspace",
                    kStaticMaxRank, (long long)rank);
    if (rank <= 0) return fail(NQ_ERR_INVALID_ARGUMENT, "rank must be positive");
    void *scratch = nullptr;
    int st = static_scratch(&scratch);
    if (st) return st;
    // The grid-barrier counter and the status word start from zero on every call; the
    // stage-2 operand needs no clearing (each launch writes what it reads).
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(Ctrl), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(static GEMV control block)");
    return nq_gemv(dtype, x, batch, in_features, scale_pre, v_bits, rank, scale_mid, u_bits, out_features, scale_post,
                   y, scratch, kStaticScratchBytes, stream);
}

int nq_gemv_static_status(void *stream, int *status_out) {
    using namespace nq;
    using namespace nq::gemv;
    if (!status_out) return fail(NQ_ERR_INVALID_ARGUMENT, "null status_out");
    void *scratch = nullptr;
    int st = static_scratch(&scratch);
    if (st) return st;
    return nq_workspace_status(scratch, kStaticScratchBytes, stream, status_out);
}

}  // extern "C"

#ifdef NQ_GEMV_TRACE
// Debug builds only: copy the phase stamps of up to `max_launches` fused launches
// ([launch][kTraceCtas][kTraceStamps] u64, host memory) and return how many were recorded;
// `reset` != 0 then clears the launch counter.
extern "C" NQ_API int nq_debug_gemv_trace(unsigned long long *host, int max_launches, int reset) {
    using namespace nq::gemv;
    unsigned int n = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    if (cudaMemcpyFromSymbol(&n, g_trace_launch, sizeof(n)) != cudaSuccess) return -1;
    const int m = (int)std::min<unsigned int>(n, (unsigned)std::min(max_launches, kTraceLaunches));
    if (m > 0 && cudaMemcpyFromSymbol(host, g_trace, (size_t)m * kTraceCtas * kTraceStamps * 8) != cudaSuccess) return -1;
    if (reset) {
        const unsigned int z = 0;
        if (cudaMemcpyToSymbol(g_trace_launch, &z, sizeof(z)) != cudaSuccess) return -1;
    }
    return (int)n;
}
#endif
