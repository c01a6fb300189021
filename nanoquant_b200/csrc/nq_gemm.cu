// NanoQuant prefill GEMM on 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// A layer y = s1 * (U (smid * (V (s2 * x)))) over M tokens is two contractions:
//   stage 1:  T[M, r]   = (X[M, in] . B1^T) * smid,  B1[n, k] = sign(V[n, k]) * s2[k]
//   stage 2:  Y[M, out] = (T[M, r]  . B2^T) * s1,    B2[n, k] = sign(U[n, k])
// replacing the reference's two Marlin mma.sync GEMMs (src/nanoquant/kernel/cuda/gemm.cpp:112-122,
// gemm_kernel.cu:278-932).  T stays in the workspace (L2-resident) between the stages; in
// precise mode it is kept as a bf16 hi/lo pair and stage 2 issues two MMAs per K step into
// the same TMEM accumulator (T_hi . B2^T + T_lo . B2^T), which keeps ~16 mantissa bits of
// the float32 T; otherwise T is rounded once to bf16 like the reference's intermediate.
//
// One CTA computes one 128 x 128 output tile; 6 warps with fixed roles:
//   warp 0     TMA producer: the activation tile (128 rows x 64 K, SWIZZLE_128B) and, in
//              stage 1, the 64-entry s2 slice (1-D tensor map, zero-filled past `in`);
//   warp 1     TMEM allocator and the single MMA-issuing thread (tcgen05.mma kind::f16,
//              M=128 N=128 K=16, fp32 accumulator in TMEM), tcgen05.commit frees stages;
//   warps 2-5  weight expanders: each thread owns one weight row of the tile and turns its
//              two HALF2 sign words per K step into 64 exact +-s2 (stage 1) or +-1 (stage 2)
//              values written straight into the UMMA SWIZZLE_128B K-major layout; the same
//              warps then drain TMEM (tcgen05.ld 32x32b) in the epilogue.
// Stages rotate through a 4-deep shared-memory ring guarded by mbarriers; every wait is
// bounded (globaltimer) and an abort flag stops the pipeline if one gives up.  No TMA
// multicast is used.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "nq_common.cuh"

namespace nq {
namespace gemm {

constexpr int BM = 128, BN = 128, BK = 64;

// Weight expanders (and epilogue warps) per CTA: 16 for 256-column tiles, 8 for 128-column
// tiles (one 32-column word of a row per thread either way); plus the TMA producer and the MMA
// issuer.
__host__ __device__ constexpr int exp_warps(int bn) { return bn == 256 ? 16 : 8; }
__host__ __device__ constexpr int cta_threads(int bn) { return 64 + 32 * exp_warps(bn); }
constexpr int kTileBytes = 128 * 128;  // 128 rows x 128 bytes (64 16-bit values)

struct Params {
    const uint32_t *bits;  // sign plane [N, W], HALF2 order
    int W;                 // words per plane row
    int M, N, K;           // output rows (tokens), output columns, contraction length
    int nk;                // number of BK steps
    const void *col_scale; // per-output-column scale (smid or s1) or null; element type TScale
    void *out_hi;          // stage 1: T (or T_hi) bf16 [M, ldo]; stage 2: y [M, ldo]
    void *out_lo;          // stage 1 precise: T_lo bf16 [M, ldo]
    int ldo;
    int *status;
    // split-K (small M, too few output tiles to fill the GPU): CTA z of the grid's third
    // dimension runs K steps [z * kbs, min((z + 1) * kbs, nk)) and, when `partial` is set,
    // stores its raw float32 accumulator tile in partial[z][M][ldp]; splitk_finalize sums the
    // slots in order and applies the column scale and the output format.
    int kbs;
    float *partial;
    int ldp;
};

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_1d(void *dst, const CUtensorMap *map, uint64_t *bar, int x) {
    asm volatile(
        "cp.async.bulk.tensor.1d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, SWIZZLE_128B, rows of 128 bytes,
// 8-row groups 1024 bytes apart (SBO), version 1 (sm_100), LBO unused (encoded 1).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;             // leading byte offset (16 B, ignored for SW128 K-major)
    d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset
    d |= (uint64_t)1u << 46;             // descriptor version for tcgen05
    d |= (uint64_t)2u << 61;             // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, K-major A and B, M = 128.
template <typename TA>
__host__ __device__ constexpr uint32_t f16_idesc(int n) {
    return (1u << 4)                                              // D format f32
           | ((std::is_same<TA, __nv_bfloat16>::value ? 1u : 0u) << 7)  // A format
           | ((std::is_same<TA, __nv_bfloat16>::value ? 1u : 0u) << 10) // B format
           | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// Shared-memory layout (offsets from a 1024-byte aligned base).  Stage i holds the
// activation tile(s) (128 rows x 128 bytes each) and the expanded weight tile (kBN rows x 128
// bytes), so every operand buffer is 1024-byte aligned as SWIZZLE_128B requires; the s2 slices
// follow.  Four stages when they fit in 200 KB, else three.
template <bool kTwoA, bool kS2, int kBN>
struct Layout {
    static constexpr uint32_t kStageBytes = (kTwoA ? 2 : 1) * kTileBytes + kBN * 128;
    static constexpr int kStg = kStageBytes * 4 <= 200 * 1024 ? 4 : 3;
    __host__ __device__ static constexpr uint32_t a_hi(int s) { return s * kStageBytes; }
    __host__ __device__ static constexpr uint32_t a_lo(int s) { return s * kStageBytes + (kTwoA ? kTileBytes : 0); }
    __host__ __device__ static constexpr uint32_t b(int s) { return s * kStageBytes + (kTwoA ? 2 : 1) * kTileBytes; }
    __host__ __device__ static constexpr uint32_t s2(int s) { return kStg * kStageBytes + 128 * s; }
    static constexpr uint32_t kBars = kStg * kStageBytes + (kS2 ? 128 * kStg : 0);
    static constexpr uint32_t kTmemSlot = kBars + (3 * kStg + 1) * 8;
    static constexpr uint32_t kAbort = kTmemSlot + 4;
    static constexpr uint32_t kTotal = (kAbort + 4 + 127) & ~127u;
};

// TA: MMA operand type (stage 1: the layer dtype; stage 2: bf16 in precise mode, the layer dtype
// otherwise).  TOut: the layer dtype, the type of the column scale (smid / s1) and of what the
// epilogue stores unless kStoreT.  kS2: fold the s2 slice into the weight operand (stage 1, and
// the single-stage GEMM).  kTwoA: two activation tiles (T_hi, T_lo) per K step (stage 2, precise).
// kStoreT: the epilogue stores T as bf16 (hi, and lo when kHiLo) -- stage 1 of precise mode; else
// it stores TOut (stage 1 of fast mode: T in the layer dtype; stage 2; the single-stage GEMM).
// kBN: output columns per CTA (128 or 256; the MMA is M=128 N=kBN K=16, each expander thread
// owns kBN / 128 weight rows).  A 256-wide tile reads the activation tile once per two weight
// row blocks, which lowers the shared-memory traffic per MMA.
template <typename TA, typename TOut, bool kS2, bool kTwoA, bool kHiLo, bool kStoreT, int kBN>
__global__ void __launch_bounds__(cta_threads(kBN), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                const __grid_constant__ CUtensorMap map_s2, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte align the working area (the launch reserves the slack)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using L = Layout<kTwoA, kS2, kBN>;
    constexpr int kStages = L::kStg;
    constexpr int kExpWarps = exp_warps(kBN);
    uint64_t *full_a = reinterpret_cast<uint64_t *>(smem + L::kBars);
    uint64_t *full_b = full_a + kStages;
    uint64_t *empty = full_b + kStages;
    uint64_t *accum = empty + kStages;
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(smem + L::kTmemSlot);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::kAbort);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * BM;
    const int kb_begin = blockIdx.z * p.kbs;
    const int nk = min(p.nk - kb_begin, p.kbs);  // this CTA's K steps (>= 1, the host checks)

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full_a[i], 1);
            mbar_init(&full_b[i], kExpWarps);
            mbar_init(&empty[i], 1);
        }
        mbar_init(accum, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(const_cast<uint32_t *>(tmem_slot), kBN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (*abort_flag) return false;
        if (!mbar_wait(bar, parity, p.status)) {
            *abort_flag = 1;
            return false;
        }
        return true;
    };

    if (warp == 0) {
        // ---------------------------------------------------------- TMA producer
        if (lane == 0) {
            const uint32_t bytes = kTileBytes * (kTwoA ? 2 : 1) + (kS2 ? 128 : 0);
            int issued_until = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages;
                const int kx = (kb_begin + kb) * BK;
                if (kb >= kStages && !wait(&empty[s], ((kb / kStages) - 1) & 1)) break;
                mbar_arrive_expect_tx(&full_a[s], bytes);
                tma_load_2d(smem + L::a_hi(s), &map_a, &full_a[s], kx, m0);
                if (kTwoA) tma_load_2d(smem + L::a_lo(s), &map_a2, &full_a[s], kx, m0);
                if (kS2) tma_load_1d(smem + L::s2(s), &map_s2, &full_a[s], kx);
                issued_until = kb + 1;
            }
            // on abort, let copies already in flight land before the CTA exits
            if (*abort_flag)
                for (int kb = (issued_until > kStages ? issued_until - kStages : 0); kb < issued_until; ++kb)
                    mbar_wait(&full_a[kb % kStages], (kb / kStages) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = f16_idesc<TA>(kBN);
            const uint32_t sbase = smem_u32(smem);
            uint32_t acc = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages;
                const uint32_t par = (kb / kStages) & 1;
                if (!wait(&full_a[s], par) || !wait(&full_b[s], par)) break;
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < BK / 16; ++j) {
                    const uint64_t bd = sw128_desc(sbase + L::b(s) + 32u * j);
                    umma_f16(tmem, sw128_desc(sbase + L::a_hi(s) + 32u * j), bd, idesc, acc);
                    acc = 1;
                    if (kTwoA) umma_f16(tmem, sw128_desc(sbase + L::a_lo(s) + 32u * j), bd, idesc, 1u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accum);
        }
    } else {
        // ---------------------------------------------------------- weight expanders
        // 32 * kExpWarps threads over the tile's kBN rows x 2 sign words per K step: kTpr threads
        // per row, each expanding kWords of the row's words (kBN 256: one row, both words;
        // kBN 128: half a row, one word)
        constexpr int kExp = 32 * kExpWarps;
        constexpr int kTpr = kExp / kBN;
        constexpr int kWords = 2 / kTpr;
        static_assert(kTpr * kBN == kExp && kWords * kTpr == 2, "expander split");
        const int ex = threadIdx.x - 64;
        const int e = ex % kBN, h0 = (ex / kBN) * kWords;  // row in the tile, first word of the two
        const int n = n0 + e;
        const bool row_ok = n < p.N;
        // this CTA's K range starts at word 2 * kb_begin of each row (two words per K step)
        const int wl = p.W - 2 * kb_begin;
        const uint32_t *row = p.bits + (size_t)(row_ok ? n : 0) * p.W + 2 * kb_begin + h0;
        const int wl_h = wl - h0;
        // words for the next steps are fetched ahead (a register queue as deep as the ring)
        uint32_t q[kWords][kStages];
#pragma unroll
        for (int j = 0; j < kWords; ++j)
#pragma unroll
            for (int i = 0; i < kStages; ++i) {
                const int w = 2 * i + j;
                q[j][i] = (row_ok && i < nk && w < wl_h) ? __ldg(row + w) : 0u;
            }
        uint8_t *const brow_base = smem;
        for (int kb0 = 0; kb0 < nk; kb0 += kStages) {
#pragma unroll
            for (int i = 0; i < kStages; ++i) {
                const int kb = kb0 + i;
                if (kb < nk) {
                    const int s = i;  // kb % kStages == i because kb0 is a multiple of kStages
                    // slot s is free once this step's activation tile is in flight-complete:
                    // the producer only re-arms full_a[s] after empty[s] fired
                    const bool ok = wait(&full_a[s], (kb / kStages) & 1);
                    const uint32_t *s2w = reinterpret_cast<const uint32_t *>(smem + L::s2(s));
                    const int nxt = kb + kStages;
                    uint8_t *brow = brow_base + L::b(s) + e * 128;
#pragma unroll
                    for (int j = 0; j < kWords; ++j) {
                        const uint32_t w = q[j][i];
                        const int wn = 2 * nxt + j;
                        q[j][i] = (row_ok && nxt < nk && wn < wl_h) ? __ldg(row + wn) : 0u;
                        const int h = h0 + j;  // word of the K step: columns 32 h .. 32 h + 31
#pragma unroll
                        for (int qc = 0; qc < 4; ++qc) {
                            uint32_t v[4], sv[4] = {0u, 0u, 0u, 0u};
                            if (kS2) {  // the four s2 pairs of this chunk in one 16-byte (broadcast) load
                                const uint4 s4 = reinterpret_cast<const uint4 *>(s2w)[4 * h + qc];
                                sv[0] = s4.x, sv[1] = s4.y, sv[2] = s4.z, sv[3] = s4.w;
                            }
#pragma unroll
                            for (int pp = 0; pp < 4; ++pp) {
                                const int P = 4 * qc + pp;  // pair index inside the word
                                const uint32_t val =
                                    kS2 ? sv[pp] : (std::is_same<TA, __nv_bfloat16>::value ? 0x3F803F80u : 0x3C003C00u);
                                v[pp] = row_ok && ok ? lop_sign(w << P, val) : 0u;
                            }
                            const int chunk = 4 * h + qc;
                            *reinterpret_cast<uint4 *>(brow + ((chunk ^ (e & 7)) << 4)) =
                                make_uint4(v[0], v[1], v[2], v[3]);
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full_b[s]);
                }
            }
        }
        // ---------------------------------------------------------- epilogue
        const bool ok = wait(accum, 0);
        tc_fence_after();
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int m = m0 + quarter * 32 + lane;
        const TOut *sc = static_cast<const TOut *>(p.col_scale);
        // kExpWarps / 4 warps share a lane quarter: each drains its own share of the columns
        constexpr int kColParts = kExpWarps / 4, kColsPer = kBN / kColParts;
        const int cpart = (warp - 2) / 4;
        for (int c = cpart * kColsPer; c < (cpart + 1) * kColsPer; c += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c, r);
            if (!ok || m >= p.M || n0 + c >= p.N) continue;
            if (p.partial) {  // split-K: the raw accumulator row segment, scaled and converted later
                float *dst = p.partial + ((size_t)blockIdx.z * p.M + m) * p.ldp + n0 + c;
                const int nc = min(32, p.N - (n0 + c));
                if (nc == 32) {
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        reinterpret_cast<uint4 *>(dst)[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
                } else {  // unrolled with a predicate: constant indices keep r in registers
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < nc) dst[j] = __uint_as_float(r[j]);
                }
                continue;
            }
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                v[j] = __uint_as_float(r[j]);
                if (sc) {
                    const int col = n0 + c + j;
                    v[j] *= (col < p.N) ? Elem<TOut>::to_f(sc[col]) : 0.f;
                }
            }
            const int ncols = min(32, p.N - (n0 + c));
            if (kStoreT) {
                // stage 1: T (bf16) and optionally T_lo
                __nv_bfloat16 *hi = static_cast<__nv_bfloat16 *>(p.out_hi) + (size_t)m * p.ldo + n0 + c;
                __nv_bfloat16 *lo = static_cast<__nv_bfloat16 *>(p.out_lo) + (size_t)m * p.ldo + n0 + c;
                uint32_t ph[16], pl[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * j]), h1 = __float2bfloat16_rn(v[2 * j + 1]);
                    ph[j] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
                    if (kHiLo) {
                        const __nv_bfloat16 l0 = __float2bfloat16_rn(v[2 * j] - __bfloat162float(h0));
                        const __nv_bfloat16 l1 = __float2bfloat16_rn(v[2 * j + 1] - __bfloat162float(h1));
                        pl[j] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
                    }
                }
                if (ncols == 32 && (reinterpret_cast<uintptr_t>(hi) & 15) == 0) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        reinterpret_cast<uint4 *>(hi)[q] = make_uint4(ph[4 * q], ph[4 * q + 1], ph[4 * q + 2], ph[4 * q + 3]);
                        if (kHiLo)
                            reinterpret_cast<uint4 *>(lo)[q] = make_uint4(pl[4 * q], pl[4 * q + 1], pl[4 * q + 2], pl[4 * q + 3]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (j >= ncols) continue;
                        hi[j] = __ushort_as_bfloat16((uint16_t)(ph[j >> 1] >> (16 * (j & 1))));
                        if (kHiLo) lo[j] = __ushort_as_bfloat16((uint16_t)(pl[j >> 1] >> (16 * (j & 1))));
                    }
                }
            } else {
                TOut *o = static_cast<TOut *>(p.out_hi) + (size_t)m * p.ldo + n0 + c;
                uint32_t po[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const TOut a = Elem<TOut>::out(v[2 * j]), b = Elem<TOut>::out(v[2 * j + 1]);
                    po[j] = (uint32_t)(*reinterpret_cast<const uint16_t *>(&a)) |
                            ((uint32_t)(*reinterpret_cast<const uint16_t *>(&b)) << 16);
                }
                if (ncols == 32 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        reinterpret_cast<uint4 *>(o)[q] = make_uint4(po[4 * q], po[4 * q + 1], po[4 * q + 2], po[4 * q + 3]);
                } else {
                    uint16_t *o16 = reinterpret_cast<uint16_t *>(o);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < ncols) o16[j] = (uint16_t)(po[j >> 1] >> (16 * (j & 1)));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kBN);
    }
}

// Split-K epilogue: out[m][n] = format(scale[n] * sum_z partial[z][m][n]), the slots summed in
// order (deterministic).  Four columns per thread; formats as gemm_kernel's epilogue.
template <typename TOut, bool kStoreT, bool kHiLo>
__global__ void __launch_bounds__(256) splitk_finalize(const float *__restrict__ part, int splits, int M, int N,
                                                       int ldp, const TOut *__restrict__ scale, void *out_hi,
                                                       void *out_lo, int ldo) {
    const int q = (N + 3) >> 2;
    const int64_t total = (int64_t)M * q;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / q), n = (int)(i % q) * 4;
        const float *src = part + (size_t)m * ldp + n;
        float4 acc = *reinterpret_cast<const float4 *>(src);
        for (int z = 1; z < splits; ++z) {
            const float4 v = *reinterpret_cast<const float4 *>(src + (size_t)z * M * ldp);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const float a[4] = {acc.x, acc.y, acc.z, acc.w};
        for (int j = 0; j < 4 && n + j < N; ++j) {
            const float v = scale ? a[j] * Elem<TOut>::to_f(scale[n + j]) : a[j];
            const size_t o = (size_t)m * ldo + n + j;
            if (kStoreT) {
                const __nv_bfloat16 h = __float2bfloat16_rn(v);
                static_cast<__nv_bfloat16 *>(out_hi)[o] = h;
                if (kHiLo) static_cast<__nv_bfloat16 *>(out_lo)[o] = __float2bfloat16_rn(v - __bfloat162float(h));
            } else {
                static_cast<TOut *>(out_hi)[o] = Elem<TOut>::out(v);
            }
        }
    }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D map over a row-major [rows, cols] 16-bit matrix with leading dimension ld (elements),
// box 64 x 128, SWIZZLE_128B, out-of-range elements read as zero.
static int make_map_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int64_t rows, int64_t cols,
                       int64_t ld) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(NQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {BK, BM};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NQ_ERR_CUDA, "cuTensorMapEncodeTiled(2d) failed (%d)", (int)r);
    return NQ_OK;
}

static int make_map_1d(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int64_t n) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(NQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[1] = {(cuuint64_t)n};
    cuuint64_t strides[1] = {0};
    cuuint32_t box[1] = {BK};
    cuuint32_t estr[1] = {1};
    CUresult r = fn(map, dt, 1, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NQ_ERR_CUDA, "cuTensorMapEncodeTiled(1d) failed (%d)", (int)r);
    return NQ_OK;
}

// Most CTAs a split-K launch may use; the workspace reserves kMaxSplitCtas * BM * BN float32
// partial values (the tiles x splits of one launch never exceed it).
constexpr int kMaxSplitCtas = 160;
constexpr int64_t kSplitMaxM = 1024;  // split-K only for M up to this many rows
constexpr int kMinStepsPerSplit = 4;

// K splits for a launch of `tiles` output tiles and nk K steps on `sms` SMs: enough CTAs for
// about one wave when the tiles alone leave more than half of the SMs idle.
static int choose_splits(int64_t m, int tiles, int nk, int sms) {
    const int cap = std::min(sms, kMaxSplitCtas);
    if (m > kSplitMaxM || tiles * 2 > cap) return 1;
    int splits = std::min(cap / tiles, nk / kMinStepsPerSplit);
    return splits < 2 ? 1 : splits;
}

template <typename TA, typename TOut, bool kS2, bool kTwoA, bool kHiLo, bool kStoreT, int kBN>
static int launch_stage(const CUtensorMap &a, const CUtensorMap &a2, const CUtensorMap &s2, const Params &p_in,
                        cudaStream_t stream, float *partial = nullptr, int splits = 1) {
    Params p = p_in;
    p.kbs = (p.nk + splits - 1) / splits;
    splits = (p.nk + p.kbs - 1) / p.kbs;  // no empty split
    p.partial = splits > 1 ? partial : nullptr;
    p.ldp = (p.N + 3) & ~3;
    auto kern = gemm_kernel<TA, TOut, kS2, kTwoA, kHiLo, kStoreT, kBN>;
    const size_t smem = Layout<kTwoA, kS2, kBN>::kTotal + 1024;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
        attr_set[dev] = true;
    }
    dim3 grid((p.N + kBN - 1) / kBN, (p.M + BM - 1) / BM, p.partial ? splits : 1);
    kern<<<grid, cta_threads(kBN), smem, stream>>>(a, a2, s2, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
    if (p.partial) {
        const int64_t work = (int64_t)p.M * ((p.N + 3) / 4);
        const int blocks = (int)std::min<int64_t>((work + 255) / 256, 4 * 148);
        splitk_finalize<TOut, kStoreT, kHiLo><<<blocks, 256, 0, stream>>>(
            p.partial, splits, p.M, p.N, p.ldp, static_cast<const TOut *>(p.col_scale), p.out_hi, p.out_lo, p.ldo);
        e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "gemm split-K finalize launch");
    }
    return NQ_OK;
}

// 256-wide tiles when they alone give most SMs a CTA (or NQ_GEMM_TILE_N=128 / 256 forces a
// width); otherwise 128-wide tiles, split along K when M is small.
static int tile_width(int64_t m, int64_t n, int sms) {
    static const int forced = [] {
        const char *v = getenv("NQ_GEMM_TILE_N");
        return v ? atoi(v) : 0;
    }();
    if (forced == 128 || forced == 256) return forced;
    const int64_t t256 = (m + BM - 1) / BM * ((n + 255) / 256);
    return t256 * 4 >= (int64_t)sms * 3 ? 256 : 128;
}

template <typename TA, typename TOut, bool kS2, bool kTwoA, bool kHiLo, bool kStoreT>
static int launch_tiled(int64_t m, int sms, const CUtensorMap &a, const CUtensorMap &a2, const CUtensorMap &s2,
                        const Params &p, cudaStream_t stream, float *partial) {
    if (tile_width(m, p.N, sms) == 256)
        return launch_stage<TA, TOut, kS2, kTwoA, kHiLo, kStoreT, 256>(a, a2, s2, p, stream);
    const int splits = partial ? choose_splits(m, (int)((m + BM - 1) / BM * ((p.N + 127) / 128)), p.nk, sms) : 1;
    return launch_stage<TA, TOut, kS2, kTwoA, kHiLo, kStoreT, 128>(a, a2, s2, p, stream, partial, splits);
}

static inline size_t t_ld(int64_t rank) { return (size_t)((rank + 7) / 8 * 8); }

}  // namespace gemm
}  // namespace nq

extern "C" {

size_t nq_gemm_workspace_bytes(int64_t m, int64_t rank) {
    using namespace nq::gemm;
    if (m <= 0 || rank <= 0) return 0;
    const size_t plane = (size_t)m * t_ld(rank) * 2;
    const size_t planeal = (plane + 255) & ~size_t(255);
    // split-K partial slots for small M (both stages use them in turn)
    const size_t part = m <= kSplitMaxM ? (size_t)kMaxSplitCtas * BM * BN * sizeof(float) : 0;
    return sizeof(nq::Ctrl) + 2 * planeal + part;
}

int nq_gemm(int dtype, const void *x, int64_t m, int64_t in_features, const void *scale_pre, const int32_t *v_bits,
            int64_t rank, const void *scale_mid, const int32_t *u_bits, int64_t out_features, const void *scale_post,
            int precise, void *y, void *workspace, size_t workspace_bytes, void *stream) {
    using namespace nq;
    using namespace nq::gemm;
    if (dtype != NQ_DTYPE_F16 && dtype != NQ_DTYPE_BF16)
        return fail(NQ_ERR_UNSUPPORTED, "dtype must be NQ_DTYPE_F16 or NQ_DTYPE_BF16 (got %d)", dtype);
    if (!x || !scale_pre || !v_bits || !u_bits || !scale_post || !y)
        return fail(NQ_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (m <= 0 || in_features <= 0 || rank <= 0 || out_features <= 0)
        return fail(NQ_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (in_features % 8 != 0) return fail(NQ_ERR_UNSUPPORTED, "in_features must be a multiple of 8 for the GEMM");
    if (m > (1 << 24) || in_features > (1 << 24) || rank > (1 << 20) || out_features > (1 << 24))
        return fail(NQ_ERR_UNSUPPORTED, "sizes beyond the supported range");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(scale_pre)) &
        15)
        return fail(NQ_ERR_INVALID_ARGUMENT, "x, y and scale_pre must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(scale_post) | reinterpret_cast<uintptr_t>(scale_mid)) & 1)
        return fail(NQ_ERR_INVALID_ARGUMENT, "scales must be 2-byte aligned");
    if ((reinterpret_cast<uintptr_t>(v_bits) | reinterpret_cast<uintptr_t>(u_bits)) & 3)
        return fail(NQ_ERR_INVALID_ARGUMENT, "sign planes must be 4-byte aligned");
    const size_t need = nq_gemm_workspace_bytes(m, rank);
    if (!workspace || workspace_bytes < need)
        return fail(NQ_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(NQ_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
    if (device_info(dev).cc_major != 10) return fail(NQ_ERR_UNSUPPORTED, "this build targets sm_100a");

    const size_t ldt = t_ld(rank);
    const size_t plane = (size_t)m * ldt * 2;
    const size_t planeal = (plane + 255) & ~size_t(255);
    Ctrl *ctrl = static_cast<Ctrl *>(workspace);
    void *t_hi = static_cast<char *>(workspace) + sizeof(Ctrl);
    void *t_lo = static_cast<char *>(t_hi) + planeal;
    float *partial = m <= kSplitMaxM ? reinterpret_cast<float *>(static_cast<char *>(t_lo) + planeal) : nullptr;
    const CUtensorMapDataType in_dt =
        dtype == NQ_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap mx, ms2, mth, mtl;
    int st = make_map_2d(&mx, x, in_dt, m, in_features, in_features);
    if (!st) st = make_map_1d(&ms2, scale_pre, in_dt, in_features);
    // precise: T as bf16 hi / lo planes; fast: T in the layer dtype (one plane)
    if (!st) st = make_map_2d(&mth, t_hi, precise ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : in_dt, m, rank, (int64_t)ldt);
    if (!st) st = make_map_2d(&mtl, t_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, m, rank, (int64_t)ldt);
    if (st) return st;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Params p1{};
    p1.bits = reinterpret_cast<const uint32_t *>(v_bits);
    p1.W = (int)((in_features + 31) / 32);
    p1.M = (int)m;
    p1.N = (int)rank;
    p1.K = (int)in_features;
    p1.nk = (int)((in_features + BK - 1) / BK);
    p1.col_scale = scale_mid;
    p1.out_hi = t_hi;
    p1.out_lo = t_lo;
    p1.ldo = (int)ldt;
    p1.status = &ctrl->status;
    Params p2{};
    p2.bits = reinterpret_cast<const uint32_t *>(u_bits);
    p2.W = (int)((rank + 31) / 32);
    p2.M = (int)m;
    p2.N = (int)out_features;
    p2.K = (int)rank;
    p2.nk = (int)((rank + BK - 1) / BK);
    p2.col_scale = scale_post;
    p2.out_hi = y;
    p2.out_lo = nullptr;
    p2.ldo = (int)out_features;
    p2.status = &ctrl->status;

    const int sms = device_info(dev).sms;
    using H = __half;
    using B = __nv_bfloat16;
    if (dtype == NQ_DTYPE_F16) {
        st = precise ? launch_tiled<H, H, true, false, true, true>(m, sms, mx, mx, ms2, p1, s, partial)
                     : launch_tiled<H, H, true, false, false, false>(m, sms, mx, mx, ms2, p1, s, partial);
        if (st) return st;
        st = precise ? launch_tiled<B, H, false, true, false, false>(m, sms, mth, mtl, ms2, p2, s, partial)
                     : launch_tiled<H, H, false, false, false, false>(m, sms, mth, mth, ms2, p2, s, partial);
    } else {
        st = precise ? launch_tiled<B, B, true, false, true, true>(m, sms, mx, mx, ms2, p1, s, partial)
                     : launch_tiled<B, B, true, false, false, false>(m, sms, mx, mx, ms2, p1, s, partial);
        if (st) return st;
        st = precise ? launch_tiled<B, B, false, true, false, false>(m, sms, mth, mtl, ms2, p2, s, partial)
                     : launch_tiled<B, B, false, false, false, false>(m, sms, mth, mth, ms2, p2, s, partial);
    }
    return st;
}

size_t nq_gemm_onebit_workspace_bytes(void) { return sizeof(nq::Ctrl); }

int nq_gemm_onebit(int dtype, const void *x, int64_t m, int64_t k, const void *scale_in, const int32_t *w_bits,
                   int64_t n, const void *scale_out, void *y, void *workspace, size_t workspace_bytes, void *stream) {
    using namespace nq;
    using namespace nq::gemm;
    if (dtype != NQ_DTYPE_F16 && dtype != NQ_DTYPE_BF16)
        return fail(NQ_ERR_UNSUPPORTED, "dtype must be NQ_DTYPE_F16 or NQ_DTYPE_BF16 (got %d)", dtype);
    if (!x || !scale_in || !w_bits || !y) return fail(NQ_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (m <= 0 || k <= 0 || n <= 0) return fail(NQ_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (k % 8 != 0) return fail(NQ_ERR_UNSUPPORTED, "k must be a multiple of 8 for the GEMM");
    if (m > (1 << 24) || k > (1 << 24) || n > (1 << 24)) return fail(NQ_ERR_UNSUPPORTED, "sizes beyond the supported range");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(scale_in)) & 15)
        return fail(NQ_ERR_INVALID_ARGUMENT, "x, y and scale_in must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(scale_out) & 1) return fail(NQ_ERR_INVALID_ARGUMENT, "scale_out must be 2-byte aligned");
    if (reinterpret_cast<uintptr_t>(w_bits) & 3) return fail(NQ_ERR_INVALID_ARGUMENT, "sign planes must be 4-byte aligned");
    if (!workspace || workspace_bytes < sizeof(Ctrl))
        return fail(NQ_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", sizeof(Ctrl), workspace_bytes);
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return cuda_fail(ce, "cudaGetDevice");
    if (device_info(dev).cc_major != 10) return fail(NQ_ERR_UNSUPPORTED, "this build targets sm_100a");
    const CUtensorMapDataType in_dt =
        dtype == NQ_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap mx, ms;
    int st = make_map_2d(&mx, x, in_dt, m, k, k);
    if (!st) st = make_map_1d(&ms, scale_in, in_dt, k);
    if (st) return st;
    Params p{};
    p.bits = reinterpret_cast<const uint32_t *>(w_bits);
    p.W = (int)((k + 31) / 32);
    p.M = (int)m;
    p.N = (int)n;
    p.K = (int)k;
    p.nk = (int)((k + BK - 1) / BK);
    p.col_scale = scale_out;
    p.out_hi = y;
    p.out_lo = nullptr;
    p.ldo = (int)n;
    p.status = &static_cast<Ctrl *>(workspace)->status;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return dtype == NQ_DTYPE_F16 ? launch_stage<__half, __half, true, false, false, false, 128>(mx, mx, ms, p, s)
                                 : launch_stage<__nv_bfloat16, __nv_bfloat16, true, false, false, false, 128>(mx, mx, ms, p, s);
}

}  // extern "C"
