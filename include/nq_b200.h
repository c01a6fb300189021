/*
 * nq_b200.h -- C ABI of the B200 (sm_100a) NanoQuant quantized-linear kernels.
 *
 * A NanoQuant layer stores W ~= diag(s1) . U . V^T . diag(s2) with U (out x r) and
 * V^T (r x in) in {-1,+1}, kept as bit-packed int32 sign planes, and computes
 *     y = s1 * (U (smid * (V (s2 * x))))          (smid optional, length r)
 * Naming follows the reference module (src/nanoquant/modules/linear.py:74-114):
 *     scale_pre = s2 [in], scale_post = s1 [out], scale_mid [r],
 *     V planes [r, ceil(in/32)], U planes [out, ceil(r/32)].
 *
 * Conventions shared by every entry point:
 *   - all pointers are device pointers unless stated; nothing here allocates;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     work is enqueued asynchronously, no entry point synchronises;
 *   - the caller selects the device (cudaSetDevice) before calling;
 *   - return value is an nq_status; on failure nq_last_error_message() gives a
 *     human-readable reason (thread-local) and nothing was enqueued;
 *   - errors detected on the device (a bounded wait that gave up, a pack input that
 *     was not +-1) are recorded in a status word inside the caller's workspace or
 *     counter and read back with nq_workspace_status().
 */
#ifndef NQ_B200_H_
#define NQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NQ_API __attribute__((visibility("default")))
#else
#define NQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    NQ_OK = 0,
    NQ_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, misaligned pointer */
    NQ_ERR_UNSUPPORTED = 2,      /* well-formed but unsupported (dtype, bit order, shape) */
    NQ_ERR_WORKSPACE = 3,        /* workspace missing or smaller than the query says */
    NQ_ERR_CUDA = 4,             /* the CUDA runtime refused the launch */
    NQ_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait gave up (status word) */
    NQ_ERR_NOT_SIGNS = 6         /* a pack input held values other than +-1 */
} nq_status;

typedef enum { NQ_DTYPE_F16 = 0, NQ_DTYPE_BF16 = 1 } nq_dtype;

/* Bit order inside each 32-bit word (src/nanoquant/kernel/utils.py:98-106):
 * LSB_FIRST: column j of a 32-column chunk -> bit j (checkpoint format);
 * HALF2:     column j -> bit 15 - j/2 + 16*(j%2) (the decode-kernel format). */
typedef enum { NQ_BITS_LSB_FIRST = 0, NQ_BITS_HALF2 = 1 } nq_bit_order;

NQ_API int nq_abi_version(void);
NQ_API const char *nq_status_string(int status);
NQ_API const char *nq_last_error_message(void);

/* ---------------------------------------------------------------------------------
 * Sign packing.
 * nq_pack_signs replaces pack_binary_gemv (src/nanoquant/kernel/utils.py:51-113):
 * int8 +-1 [rows, cols] -> int32 [rows, ceil(cols/32)], +1 -> bit 0, -1 -> bit 1,
 * columns padded with +1.  If `invalid_count` (device int32, may be NULL) is given,
 * the number of inputs that are not exactly +-1 is atomically ADDED to it (the caller
 * zeroes it); those entries are packed by their sign.
 * nq_unpack_signs replaces unpack_binary_gemv (utils.py:116-183); padding bits ignored.
 * nq_repack_signs has no single reference counterpart: it converts planes between bit
 * orders on the device (the reference does unpack -> dense -> pack for this,
 * src/nanoquant/modules/linear.py:205-206 after load_utils.py:392), clearing padding bits.
 * ------------------------------------------------------------------------------- */
NQ_API int nq_pack_signs(const int8_t *signs, int64_t rows, int64_t cols, int bit_order,
                  int32_t *packed, int32_t *invalid_count, void *stream);
NQ_API int nq_unpack_signs(const int32_t *packed, int64_t rows, int64_t cols, int bit_order,
                    int8_t *signs, void *stream);
NQ_API int nq_repack_signs(const int32_t *src, int64_t rows, int64_t cols, int src_order,
                    int dst_order, int32_t *dst, void *stream);

/* ---------------------------------------------------------------------------------
 * Decode GEMV: replaces nanoquant_dyn_forward (src/nanoquant/kernel/cuda/gemv_kernel.cu:308-429,
 * op schema src/nanoquant/kernel/pybind.cpp:85-90), fused into ONE launch per 8 rows of x.
 *   x [batch, in], scale_pre [in], scale_mid [rank] or NULL, scale_post [out], y [batch, out]
 *   all of `dtype`; v_bits [rank, ceil(in/32)] and u_bits [out, ceil(rank/32)] in HALF2 order.
 * Accumulation is float32; fp16 outputs are clamped to +-64504 like the reference
 * (src/nanoquant/kernel/cuda/cuda_utils.cuh:80-90).
 * The workspace (>= nq_gemv_workspace_bytes) must be zero-filled once before its
 * first use (nq_workspace_reset); every successful call leaves it reusable.  Calls
 * that share one workspace must be ordered on one stream.
 * ------------------------------------------------------------------------------- */
NQ_API size_t nq_gemv_workspace_bytes(int64_t batch, int64_t rank);
NQ_API int nq_gemv(int dtype, const void *x, int64_t batch, int64_t in_features,
            const void *scale_pre, const int32_t *v_bits, int64_t rank,
            const void *scale_mid, const int32_t *u_bits, int64_t out_features,
            const void *scale_post, void *y, void *workspace, size_t workspace_bytes,
            void *stream);

/* ---------------------------------------------------------------------------------
 * Grouped decode GEMV: up to 3 NanoQuant layers that read the same x (the q/k/v or
 * gate/up projections of a decoder block) in ONE launch; layer l behaves exactly like
 * nq_gemv on its own arguments.  No single reference counterpart: the reference calls
 * nanoquant_dyn_forward once per layer (src/nanoquant/modules/linear.py:155-164).
 * Workspace: nq_gemv_group_workspace_bytes(n_layers, ranks); same rules as nq_gemv.
 * ------------------------------------------------------------------------------- */
typedef struct {
    const void *scale_pre;     /* [in] */
    const int32_t *v_bits;     /* [rank, ceil(in/32)], HALF2 */
    int64_t rank;
    const void *scale_mid;     /* [rank] or NULL */
    const int32_t *u_bits;     /* [out, ceil(rank/32)], HALF2 */
    int64_t out_features;
    const void *scale_post;    /* [out] */
    void *y;                   /* [batch, out] */
} nq_gemv_layer;
NQ_API size_t nq_gemv_group_workspace_bytes(int n_layers, const int64_t *ranks);
NQ_API int nq_gemv_group(int dtype, const void *x, int64_t batch, int64_t in_features, int n_layers,
                         const nq_gemv_layer *layers, void *workspace, size_t workspace_bytes,
                         void *stream);

/* ---------------------------------------------------------------------------------
 * Grouped decode GEMV whose input is formed in the kernel's prologue from its neighbours'
 * outputs -- the decoder's RMSNorm (with the residual add) before q/k/v and gate/up, and
 * SiLU(gate) * up before down -- and whose `act` bit l puts layer l's output through SiLU
 * (the SwiGLU gate, stored as dtype(silu(dtype(y)))).  No reference counterpart: the reference
 * runs these neighbours as HF modules between its nanoquant_dyn_forward calls
 * (src/nanoquant/kernel/test_decode.py).  The layers see x' where, with x_mode
 *   NQ_CHAIN_X_PLAIN     x' = x
 *   NQ_CHAIN_X_RMSNORM   h = dtype(x + x2) (h = x when x2 is NULL); residual_out = h when given;
 *                        x' = dtype(norm_weight * dtype(h * rsqrt(mean(h^2) + eps)))
 *   NQ_CHAIN_X_SILU_MUL  x' = dtype(dtype(silu(x)) * x2)
 *   NQ_CHAIN_X_MUL       x' = dtype(x * x2)
 * (the roundings of nq_rmsnorm and nq_silu_mul; the mean's summation order differs).
 * Transformed inputs need batch <= 8, in_features % 8 == 0 and 16-byte aligned x, x2,
 * norm_weight, residual_out and scale_pre.  Workspace as nq_gemv_group.
 * ------------------------------------------------------------------------------- */
enum { NQ_CHAIN_X_PLAIN = 0, NQ_CHAIN_X_RMSNORM = 1, NQ_CHAIN_X_SILU_MUL = 2, NQ_CHAIN_X_MUL = 3 };
typedef struct {
    int x_mode;                /* NQ_CHAIN_X_* */
    float eps;                 /* NQ_CHAIN_X_RMSNORM */
    const void *x;             /* [batch, in] */
    const void *x2;            /* residual [batch, in] (RMSNORM, may be NULL) or second factor */
    const void *norm_weight;   /* [in] (RMSNORM) */
    void *residual_out;        /* [batch, in] (RMSNORM, may be NULL) */
} nq_gemv_input;
NQ_API int nq_gemv_group_ex(int dtype, const nq_gemv_input *input, int64_t batch,
                            int64_t in_features, int n_layers, const nq_gemv_layer *layers, int act,
                            void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------------------
 * Tensor-parallel exchange fused into the decode GEMVs.  No reference counterpart: the reference
 * is single-GPU.  The decoder's per-block sum of the row-parallel layers' partial outputs (o and
 * down) runs inside the GEMVs themselves, over peer memory (one process per GPU, CUDA IPC):
 *   NQ_TP_PUSH  (one layer) the output rows, rounded to dtype, are also stored into every rank's
 *               receive buffer (NVLink stores), two values per 8-byte word together with the
 *               exchange's epoch as a flag, so no fence or separate signal is needed;
 *   NQ_TP_PULL  (x_mode NQ_CHAIN_X_RMSNORM) x is not read: the launch polls (bounded, 2 s) the
 *               ranks' words until their flags show the epoch and uses x = dtype(sum over ranks, in
 *               rank order, of their pushed rows), float32 accumulation -- the same bits on every rank.
 * Every rank allocates a zeroed region with nq_tp_region_alloc (nq_tp_region_bytes; free it with
 * nq_allreduce_region_free), exports it with nq_ipc_handle and maps the others with nq_ipc_open
 * (include/nq_decoder.h); `regions` lists every rank's region as mapped in the calling process.
 * Every rank must make the same sequence of calls, PUSH and PULL alternating (nq_tp_pull counts
 * as a PULL); batch <= 8; the launch that exchanges must run one CTA per SM: the single
 * cooperative launch, or for a layer group too large for it the stage-1 launch of its two (a
 * PULL) or the stage-2 launch (a PUSH), not both in one call; a timed-out wait records
 * NQ_ERR_DEVICE_TIMEOUT in the region's status word (nq_workspace_status).
 * NQ_TP_CHECK added to tp_mode plans the call without launching it (and without reading the
 * regions, which may be NULL): NQ_OK when the exchange can run at these shapes, otherwise the
 * error the launch would return (for instance a two-launch GEMV whose exchanging launch needs
 * more CTAs than SMs), so a caller can fall back to a separate all-reduce before it starts.
 * ------------------------------------------------------------------------------- */
#define NQ_TP_PULL 1
#define NQ_TP_PUSH 2
#define NQ_TP_CHECK 4
typedef struct {
    void *regions[8];          /* every rank's region as mapped in this process (own at `rank`) */
    int rank;
    int world;                 /* <= 8 */
    int64_t max_elems;         /* values per source buffer (>= batch * hidden), multiple of 8 */
} nq_tp_exchange;
NQ_API size_t nq_tp_region_bytes(int world, int64_t max_elems);
NQ_API int nq_tp_region_alloc(int world, int64_t max_elems, void **region_out);
NQ_API int nq_gemv_group_tp(int dtype, const nq_gemv_input *input, int64_t batch, int64_t in_features,
                            int n_layers, const nq_gemv_layer *layers, int act,
                            const nq_tp_exchange *tp, int tp_mode, void *workspace,
                            size_t workspace_bytes, void *stream);
/* A PULL on its own: out [n] = the summed vector (the final norm's input after the last layer). */
NQ_API int nq_tp_pull(int dtype, const nq_tp_exchange *tp, int64_t n, void *out, void *stream);

/* ---------------------------------------------------------------------------------
 * Allocation-free decode GEMV.  No counterpart in the reference: its kernels allocate their
 * intermediate with the torch caching allocator on every call (gemv_kernel.cu:345-346).
 * For callers that cannot allocate device memory -- a plugin or custom-op interface that
 * receives only input and output buffers, or a process that fixes its device memory at
 * start-up and must not call cudaMalloc later -- this runs nq_gemv with scratch held in a
 * static device array of this library (NQ_GEMV_STATIC_MAX_RANK caps the rank; about 128 KiB,
 * resident on every GPU that loads the library until the process exits).  Arguments and
 * results are those of nq_gemv, minus the workspace.
 *   - It calls no cudaMalloc / cudaFree and no allocating library routine.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress);
 *     make that first call before any stream capture.
 *   - Every call clears the scratch's control block (barrier counter, status word) on
 *     `stream`, then launches; all calls share the one array, so calls that may overlap on
 *     the GPU (different streams without ordering) race and must be serialised by the caller.
 *   - rank > NQ_GEMV_STATIC_MAX_RANK returns NQ_ERR_UNSUPPORTED without launching.
 * ------------------------------------------------------------------------------- */
#define NQ_GEMV_STATIC_MAX_RANK 4096
NQ_API int nq_gemv_static(int dtype, const void *x, int64_t batch, int64_t in_features,
                          const void *scale_pre, const int32_t *v_bits, int64_t rank,
                          const void *scale_mid, const int32_t *u_bits, int64_t out_features,
                          const void *scale_post, void *y, void *stream);
/* Device-side status of the last nq_gemv_static call on the current device: synchronises
 * `stream`, then reads the static scratch's status word (NQ_OK, or NQ_ERR_DEVICE_TIMEOUT when
 * a bounded wait inside the kernel gave up and y is not valid).  The next nq_gemv_static call
 * clears the word, so read it before that call.  Neither function may be used after a
 * cudaDeviceReset in the same process (the cached scratch address would be stale). */
NQ_API int nq_gemv_static_status(void *stream, int *status_out);

/* ---------------------------------------------------------------------------------
 * Prefill GEMM: replaces marlin_nanoquant_cuda (src/nanoquant/kernel/cuda/gemm.cpp:112-122,
 * schema src/nanoquant/kernel/pybind.cpp:99-104) on the same HALF2 planes the GEMV uses.
 * tcgen05 tensor-core contraction in two stages, T = (x*s2) V^T * smid then y = (T U^T) * s1.
 * `precise` = 1 keeps T as a bf16 hi/lo pair (float32-grade intermediate); 0 rounds T once to
 * the layer dtype, as the reference's fp16/bf16 intermediate `imm` (gemm.cpp:119), and runs one
 * MMA per K step in stage 2 instead of two.
 * Requires in_features % 8 == 0 and 16-byte aligned x / y.
 * ------------------------------------------------------------------------------- */
NQ_API size_t nq_gemm_workspace_bytes(int64_t m, int64_t rank);
NQ_API int nq_gemm(int dtype, const void *x, int64_t m, int64_t in_features, const void *scale_pre,
            const int32_t *v_bits, int64_t rank, const void *scale_mid, const int32_t *u_bits,
            int64_t out_features, const void *scale_post, int precise, void *y, void *workspace,
            size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------------------
 * Single-stage GEMM y = ((x * scale_in) W^T) * scale_out with W [n, k] in +-1 (HALF2 planes
 * [n, ceil(k/32)]): replaces marlin_onebit_cuda (src/nanoquant/kernel/cuda/gemm.cpp:58-93,
 * schema pybind.cpp:93-98) on this build's planes.  scale_in [k] must be given (pass ones for
 * none); scale_out [n] may be NULL.  Requires k % 8 == 0 and 16-byte aligned x, y, scale_in.
 * The workspace holds only the status word (nq_gemm_onebit_workspace_bytes()).
 * ------------------------------------------------------------------------------- */
NQ_API size_t nq_gemm_onebit_workspace_bytes(void);
NQ_API int nq_gemm_onebit(int dtype, const void *x, int64_t m, int64_t k, const void *scale_in,
                          const int32_t *w_bits, int64_t n, const void *scale_out, void *y,
                          void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------------------
 * The reference's Marlin sign layout (its prefill-GEMM kernel type's packing).
 * nq_pack_marlin replaces the sign packing of pack_binary_marlin (src/nanoquant/kernel/
 * utils.py:186-206): int8 +-1 weight [n_out, k_red] -> int32 words [k_red/16, n_out/2], element
 * (o, r) at word [r/16][(o/64)*32 + (o%8)*4 + (r%8)/2], bit 15 - (2*((o%16)/8) + (r%16)/8)
 * + 16*(r%2) - 4*((o%64)/16), set for -1; needs n_out % 64 == 0 and k_red % 16 == 0.
 * `invalid_count` as in nq_pack_signs.  nq_unpack_marlin is its inverse (no reference
 * counterpart).  nq_marlin_to_half2 converts Marlin words to HALF2 planes [n_out, ceil(k_red/32)]
 * on the device (no reference counterpart: it lets the marlin_* ops run this build's GEMM).
 * ------------------------------------------------------------------------------- */
NQ_API int nq_pack_marlin(const int8_t *signs, int64_t n_out, int64_t k_red, int32_t *words,
                          int32_t *invalid_count, void *stream);
NQ_API int nq_unpack_marlin(const int32_t *words, int64_t n_out, int64_t k_red, int8_t *signs,
                            void *stream);
NQ_API int nq_marlin_to_half2(const int32_t *words, int64_t n_out, int64_t k_red, int32_t *planes,
                              void *stream);

/* ---------------------------------------------------------------------------------
 * Workspace status word (no reference counterpart: the reference kernels have no
 * device-side error reporting).
 * nq_workspace_reset zero-fills a workspace (enqueued on `stream`).
 * nq_workspace_status synchronises `stream`, then reads the status word: NQ_OK or the
 * first device-side error (NQ_ERR_DEVICE_TIMEOUT); the word is left as it was.
 * ------------------------------------------------------------------------------- */
NQ_API int nq_workspace_reset(void *workspace, size_t workspace_bytes, void *stream);
NQ_API int nq_workspace_status(const void *workspace, size_t workspace_bytes, void *stream,
                        int *status_out);

#ifdef __cplusplus
}
#endif
#endif /* NQ_B200_H_ */
