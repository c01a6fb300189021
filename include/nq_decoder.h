/*
 * nq_decoder.h -- C ABI of the kernels that sit around the quantized linears in a
 * Llama-architecture decoder step (no reference counterpart as kernels: the reference
 * runs these parts as stock HF / PyTorch modules, src/nanoquant/kernel/test_decode.py).
 * Conventions are those of nq_b200.h: device pointers, void* cudaStream_t, nq_status.
 */
#ifndef NQ_DECODER_H_
#define NQ_DECODER_H_

#include "nq_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* h = x (+ residual_in) rounded to dtype; residual_out = h (may be NULL);
 * out = weight * dtype(h * rsqrt(mean(h^2) + eps)).  x, out: [rows, hidden]. */
NQ_API int nq_rmsnorm(int dtype, const void *x, const void *residual_in, void *residual_out,
                      const void *weight, void *out, int64_t rows, int64_t hidden, float eps,
                      void *stream);

/* Rotary embedding (rotate-half pairs (i, i + head_dim/2), angle pos * theta^(-2i/head_dim))
 * applied in place to q [n_tokens, hq, head_dim] and k [n_tokens, hkv, head_dim]; the rotated
 * k and the untouched v [n_tokens, hkv, head_dim] are written to the caches
 * [batch][hkv][max_seq][head_dim] at row batch_of[t] (t itself when NULL), position positions[t]. */
NQ_API int nq_rope_cache(int dtype, void *q, void *k, const void *v, const int32_t *positions,
                         const int32_t *batch_of, void *k_cache, void *v_cache, int64_t n_tokens,
                         int64_t hq, int64_t hkv, int64_t head_dim, int64_t max_seq, float theta,
                         void *stream);

/* Single-query attention over the first seq_len[b] cache positions (device int32 [batch]):
 * out [batch, hq, head_dim].  One launch: positions are split into chunks (a multiple of 64
 * positions, at most 64 chunks per head) whose partial results the last chunk to finish
 * combines.  head_dim 128, hq / hkv in {1, 2, 4, 8}, caches 16-byte aligned.  A capacity
 * max_seq that is a multiple of 64 positions keeps every 64-row block of a head 16 KB aligned;
 * other capacities work but were measured up to 1.9x slower on B200 (L = 2048: 12.9 us per
 * launch at max_seq 2112, 24.1 us at 2197, same chunking).
 * Workspace: nq_decode_attention_workspace_bytes() bytes, 256-byte aligned, zeroed before its
 * first use; every call leaves it zeroed again (arrival counters) except for a device-side
 * error, which nq_workspace_status() reads.  One call at a time per workspace. */
NQ_API size_t nq_decode_attention_workspace_bytes(int64_t batch, int64_t hq, int64_t head_dim,
                                                  int64_t max_seq);
NQ_API int nq_decode_attention(int dtype, const void *q, const void *k_cache, const void *v_cache,
                               const int32_t *seq_len, void *out, int64_t batch, int64_t hq,
                               int64_t hkv, int64_t head_dim, int64_t max_seq, void *workspace,
                               size_t workspace_bytes, void *stream);

/* nq_rope_cache followed by nq_decode_attention for one new token per batch row, in one
 * launch: q [batch, hq, head_dim] and k [batch, hkv, head_dim] are the projections before the
 * rotary embedding (left unmodified), v [batch, hkv, head_dim]; the rotated k and v are written
 * to the caches at positions[b] and attention runs over positions 0 .. positions[b].  Rotated
 * values and cache contents are bit-identical to nq_rope_cache's.  Workspace as above. */
NQ_API int nq_decode_attention_rope(int dtype, const void *q, const void *k, const void *v,
                                    const int32_t *positions, void *k_cache, void *v_cache,
                                    void *out, int64_t batch, int64_t hq, int64_t hkv,
                                    int64_t head_dim, int64_t max_seq, float theta,
                                    void *workspace, size_t workspace_bytes, void *stream);

/* One-shot all-reduce (sum) of a small vector over the GPUs of one node, through peer memory:
 * the tensor-parallel decoder's per-block sum of the row-parallel layers' partial outputs, which
 * the reference harness leaves to torch.distributed / NCCL (it has no kernel of its own).
 * One process per GPU.  Every rank allocates a region with nq_allreduce_region_alloc (zeroed;
 * nq_allreduce_region_bytes says how large), exports it with nq_ipc_handle (64 bytes), and maps
 * the other ranks' regions with nq_ipc_open, all before the first call; `regions` lists every
 * rank's region as mapped in the calling process (its own at index `rank`).  A call sums x over
 * the ranks into out (may alias x), n a multiple of 8 and <= max_elems, float32 accumulation in
 * rank order (every rank gets the same bits).  Every rank must make the same sequence of calls;
 * each call's CTAs wait (bounded, 2 s) for the other ranks and record NQ_ERR_DEVICE_TIMEOUT in
 * the region's status word (nq_workspace_status) when one does not come. */
NQ_API size_t nq_allreduce_region_bytes(int world, int64_t max_elems);
NQ_API int nq_allreduce_region_alloc(int world, int64_t max_elems, void **region_out);
NQ_API int nq_allreduce_region_free(void *region);
NQ_API int nq_ipc_handle(const void *region, void *handle_out);
NQ_API int nq_ipc_open(const void *handle, void **region_out);
NQ_API int nq_ipc_close(void *region);
NQ_API int nq_allreduce(int dtype, const void *x, void *out, int64_t n, int rank, int world,
                        void *const *regions, int64_t max_elems, void *stream);

/* out = dtype(silu(gate)) * up, elementwise over n values. */
NQ_API int nq_silu_mul(int dtype, const void *gate, const void *up, void *out, int64_t n,
                       void *stream);

#ifdef __cplusplus
}
#endif
#endif /* NQ_DECODER_H_ */
