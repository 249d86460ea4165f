// Runtime plumbing of the C ABI: status strings, the CUDA error of the last call
// and the per-device status word.
#include "ima_common.cuh"

static thread_local int g_last_cuda_error = 0;

int ima_note_cuda(cudaError_t e) {
    if (e == cudaSuccess) return IMA_OK;
    g_last_cuda_error = (int)e;
    return IMA_ERR_CUDA;
}

extern "C" {

int ima_abi_version(void) { return 1; }

const char* ima_status_string(int status) {
    switch (status) {
        case IMA_OK: return "ok";
        case IMA_ERR_INVALID_ARGUMENT: return "invalid argument";
        case IMA_ERR_UNSUPPORTED: return "unsupported parameter";
        case IMA_ERR_CUDA: return "CUDA error";
        case IMA_ERR_TIMEOUT: return "device wait timed out";
        case IMA_ERR_DEVICE_BOUNDS: return "device index out of bounds";
        case IMA_ERR_OVERFLOW: return "operand outside the exact range of the digit scheme";
        default: return "unknown status";
    }
}

int ima_last_cuda_error(void) { return g_last_cuda_error; }

}  // extern "C"

// Issue-rate probe for the integer ALU roofline: every thread runs 8 independent
// LOP3/IADD3 chains, so the kernel is bound by integer instruction issue alone.
__global__ void __launch_bounds__(256) int32_issue_probe_kernel(int64_t iters, uint32_t seed, uint32_t* sink) {
    uint32_t a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = seed + threadIdx.x * 8 + j;
    for (int64_t i = 0; i < iters; ++i) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            a[j] = (a[j] ^ a[(j + 1) & 7]) + a[(j + 3) & 7];
        }
    }
    uint32_t r = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) r ^= a[j];
    if (r == 0x12345678u) sink[threadIdx.x] = r;   // practically never; keeps the chains alive
}

extern "C" {

int ima_int32_issue_probe(int64_t iters, int blocks, uint32_t* sink, void* stream) {
    if (iters <= 0 || blocks <= 0 || !sink) return IMA_ERR_INVALID_ARGUMENT;
    int32_issue_probe_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(iters, 0x9E3779B9u, sink);
    return IMA_LAUNCH_STATUS();
}

int ima_struct_sizes(int64_t* out, int n) {
    if (!out || n < 3) return IMA_ERR_INVALID_ARGUMENT;
    out[0] = (int64_t)sizeof(ima_quantize_problem);
    out[1] = (int64_t)sizeof(ima_gemm_problem);
    out[2] = (int64_t)sizeof(ima_freivalds_rows_problem);
    return IMA_OK;
}

int ima_device_status(int device, int* code, int* where, int* detail, int clear) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return ima_note_cuda(cudaGetLastError());
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return ima_note_cuda(cudaGetLastError());
    ImaDeviceStatus st;
    int rc = ima_note_cuda(cudaMemcpyFromSymbol(&st, g_ima_status, sizeof(st)));
    if (rc == IMA_OK && clear) {
        ImaDeviceStatus zero = {0, 0, 0, 0};
        rc = ima_note_cuda(cudaMemcpyToSymbol(g_ima_status, &zero, sizeof(zero)));
    }
    if (prev != device) cudaSetDevice(prev);
    if (rc != IMA_OK) return rc;
    if (code) *code = st.code;
    if (where) *where = st.where;
    if (detail) *detail = st.detail;
    return IMA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Multi-GPU plumbing for collectives on the copy engines: device buffers shared between
// the processes of one node through CUDA IPC, and asynchronous copies into a peer's
// buffer (peer-to-peer over NVLink, no kernel).  No reference counterpart.
// ---------------------------------------------------------------------------
extern "C" {

int ima_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int ima_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
    if (bytes <= 0 || !ptr || !handle) return IMA_ERR_INVALID_ARGUMENT;
    *ptr = nullptr;
    int rc = ima_note_cuda(cudaMalloc(ptr, (size_t)bytes));
    if (rc != IMA_OK) return rc;
    rc = ima_note_cuda(cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), *ptr));
    if (rc != IMA_OK) {
        cudaFree(*ptr);
        *ptr = nullptr;
    }
    return rc;
}

int ima_ipc_free(void* ptr) { return ptr ? ima_note_cuda(cudaFree(ptr)) : IMA_OK; }

int ima_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return IMA_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return ima_note_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int ima_ipc_close(void* ptr) { return ptr ? ima_note_cuda(cudaIpcCloseMemHandle(ptr)) : IMA_OK; }

int ima_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
    if (bytes < 0 || (bytes > 0 && (!dst || !src))) return IMA_ERR_INVALID_ARGUMENT;
    if (bytes == 0) return IMA_OK;
    return ima_note_cuda(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, (cudaStream_t)stream));
}

}  // extern "C"
