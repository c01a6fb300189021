// Prefill GEMM entry points (tcgen05 implementation lands in this file).
#include "nq_common.cuh"

extern "C" {

size_t nq_gemm_workspace_bytes(int64_t m, int64_t rank) {
    if (m <= 0 || rank <= 0) return 0;
    return sizeof(nq::Ctrl);
}

int nq_gemm(int, const void *, int64_t, int64_t, const void *, const int32_t *, int64_t, const void *,
            const int32_t *, int64_t, const void *, int, void *, void *, size_t, void *) {
    return nq::fail(NQ_ERR_UNSUPPORTED, "nq_gemm is not available in this build");
}

}  // extern "C"
