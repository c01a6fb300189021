// C ABI bookkeeping: status strings, thread-local error messages, per-device
// properties and the workspace status word.
#include <cstdlib>
#include <mutex>

#include "nq_common.cuh"

namespace nq {

static thread_local char g_last_error[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int fail(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return NQ_ERR_CUDA;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("NQ_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

const DeviceInfo &device_info(int dev) {
    static std::mutex mu;
    static DeviceInfo infos[64];
    static bool ready[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!ready[dev]) {
        DeviceInfo &d = infos[dev];
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaDeviceGetAttribute(&d.coop, cudaDevAttrCooperativeLaunch, dev);
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
        ready[dev] = true;
    }
    return infos[dev];
}

}  // namespace nq

extern "C" {

int nq_abi_version(void) { return 1; }

const char *nq_status_string(int status) {
    switch (status) {
        case NQ_OK: return "ok";
        case NQ_ERR_INVALID_ARGUMENT: return "invalid argument";
        case NQ_ERR_UNSUPPORTED: return "unsupported";
        case NQ_ERR_WORKSPACE: return "workspace too small";
        case NQ_ERR_CUDA: return "CUDA error";
        case NQ_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case NQ_ERR_NOT_SIGNS: return "input values are not +-1";
        default: return "unknown status";
    }
}

const char *nq_last_error_message(void) { return nq::g_last_error; }

int nq_workspace_reset(void *workspace, size_t workspace_bytes, void *stream) {
    if (!workspace || workspace_bytes < sizeof(nq::Ctrl))
        return nq::fail(NQ_ERR_WORKSPACE, "workspace must be at least %zu bytes", sizeof(nq::Ctrl));
    cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? NQ_OK : nq::cuda_fail(e, "cudaMemsetAsync(workspace)");
}

int nq_workspace_status(const void *workspace, size_t workspace_bytes, void *stream, int *status_out) {
    if (!workspace || workspace_bytes < sizeof(nq::Ctrl) || !status_out)
        return nq::fail(NQ_ERR_INVALID_ARGUMENT, "workspace and status_out are required");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return nq::cuda_fail(e, "cudaStreamSynchronize");
    int v = 0;
    e = cudaMemcpy(&v, &static_cast<const nq::Ctrl *>(workspace)->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return nq::cuda_fail(e, "cudaMemcpy(status)");
    *status_out = v;
    return NQ_OK;
}

}  // extern "C"
