// Runtime plumbing of the C ABI: status strings, the CUDA error of the last call
// and the per-device status word.
#include <algorithm>
#include <cstring>
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
namespace {

// Many copies in one launch on a few SMs: the copies form one list of 512-byte units (a warp
// moves one unit per step, 16 bytes per lane, so every warp access is 512 contiguous bytes:
// full-width NVLink writes when the destination is another GPU's memory), dealt to the warps
// of the grid in turn, four units in flight per warp.
struct CopyBatch {
    ima_copy_desc d[IMA_COPY_MAX];
    int64_t unit_start[IMA_COPY_MAX + 1];   // first unit of each copy; unit_start[n] = total
    int32_t n;
};

IMA_DEVINL int copy_of_unit(const CopyBatch& b, int64_t u) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (b.unit_start[mid] <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__global__ void __launch_bounds__(512) copy_many_kernel(const __grid_constant__ CopyBatch b) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t total = b.unit_start[b.n];
    constexpr int U = 4;
    for (int64_t u0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u0 < total; u0 += U * warps) {
        uint4 v[U];
        unsigned char* dst[U];
        int64_t left[U];
#pragma unroll
        for (int i = 0; i < U; ++i) {
            const int64_t u = u0 + i * warps;
            left[i] = 0;
            dst[i] = nullptr;
            if (u < total) {
                const int c = copy_of_unit(b, u);
                const int64_t off = (u - b.unit_start[c]) * 512 + lane * 16;
                left[i] = b.d[c].bytes - off;
                const unsigned char* src = reinterpret_cast<const unsigned char*>(b.d[c].src) + off;
                dst[i] = reinterpret_cast<unsigned char*>(b.d[c].dst) + off;
                if (left[i] >= 16) {
                    v[i] = __ldg(reinterpret_cast<const uint4*>(src));
                } else if (left[i] > 0) {
                    uint32_t w[4] = {0, 0, 0, 0};
                    for (int e = 0; e < left[i]; ++e) w[e >> 2] |= (uint32_t)src[e] << (8 * (e & 3));
                    v[i] = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < U; ++i) {
            if (left[i] >= 16) {
                *reinterpret_cast<uint4*>(dst[i]) = v[i];
            } else if (left[i] > 0) {
                const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
                for (int e = 0; e < left[i]; ++e) dst[i][e] = (unsigned char)(w[e >> 2] >> (8 * (e & 3)));
            }
        }
    }
    // stores into other GPUs' memory are visible there once the launch is complete
    __threadfence_system();
}

}  // namespace

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

int ima_copy_many(const ima_copy_desc* copies, int count, int ctas, void* stream) {
    if (count < 0 || count > IMA_COPY_MAX || ctas < 1 || (count > 0 && !copies)) return IMA_ERR_INVALID_ARGUMENT;
    CopyBatch b;
    memset(&b, 0, sizeof(b));
    int64_t units = 0;
    for (int i = 0; i < count; ++i) {
        const ima_copy_desc& c = copies[i];
        if (c.bytes < 0 || (c.bytes > 0 && (!c.dst || !c.src))) return IMA_ERR_INVALID_ARGUMENT;
        // the unit loads and stores are 16 bytes wide
        if ((reinterpret_cast<uintptr_t>(c.dst) | reinterpret_cast<uintptr_t>(c.src)) & 15)
            return IMA_ERR_INVALID_ARGUMENT;
        b.d[i] = c;
        b.unit_start[i] = units;
        units += (c.bytes + 511) / 512;
    }
    b.n = count;
    b.unit_start[count] = units;
    if (units == 0) return IMA_OK;
    const int64_t warps_needed = (units + 3) / 4;
    const int grid = (int)std::min<int64_t>(ctas, (warps_needed + 15) / 16);
    copy_many_kernel<<<grid, 512, 0, (cudaStream_t)stream>>>(b);
    return IMA_LAUNCH_STATUS();
}

}  // extern "C"
