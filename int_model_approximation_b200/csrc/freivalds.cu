// Freivalds check of a claimed int64 product C = A B: accept row m iff
//     sum_k A[m,k] * (sum_n B[k,n] r[n]) == sum_n C[m,n] r[n]      (mod 2^64).
// ref: tests/test_real_integer_gemms.py:67-93 (the reference checks with Python
// integers; a correct product satisfies the identity over Z, hence mod 2^64, and a
// single corrupted entry C[m,n] + d is rejected whenever d * r[n] != 0 mod 2^64).
//
// Two bandwidth-bound GEMV passes:
//   weight pass  t = B r          (reads B once: N*K codes).  B and r are fixed per
//                linear, so a caller that checks many products of the same weight
//                computes t once (ima_freivalds_weight_vector) and reuses it.
//   row pass     per row m: A[m,:] . t  vs  C[m,:] . r  (reads A and C once: M*K + 8*M*N
//                bytes); one warp per row, many products per launch.
// All arithmetic is uint64 (wrapping), identical to the CPU oracle.
#include "ima_common.cuh"

namespace {

constexpr int FV_THREADS = 256;
constexpr int FV_WCOLS = 16;    // weight pass: 16 consecutive k per thread (one 16-byte load per row)
constexpr int FV_WROWS = 32;    // weight pass: rows n summed per thread before the atomic

// Weight pass for fp8 weights w [N,K]: t[k] += sum_{n in chunk} code(w[n,k]) * r[n].
__global__ void __launch_bounds__(FV_THREADS) fv_weight_fp8_kernel(const uint8_t* __restrict__ w, int64_t ldw,
                                                                  const int64_t* __restrict__ r, int64_t N, int64_t K,
                                                                  unsigned long long* __restrict__ t) {
    const int64_t k_groups = (K + FV_WCOLS - 1) / FV_WCOLS;
    const int64_t idx = (int64_t)blockIdx.x * FV_THREADS + threadIdx.x;
    const int64_t kg = idx % k_groups;
    const int64_t n0 = (idx / k_groups) * FV_WROWS;
    if (n0 >= N) return;
    const int64_t k0 = kg * FV_WCOLS;
    uint64_t acc[FV_WCOLS];
#pragma unroll
    for (int j = 0; j < FV_WCOLS; ++j) acc[j] = 0;
    const int64_t n1 = n0 + FV_WROWS < N ? n0 + FV_WROWS : N;
    const bool vec = (k0 + FV_WCOLS <= K) && ((ldw & 15) == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
    for (int64_t n = n0; n < n1; ++n) {
        const uint64_t rn = (uint64_t)__ldg(r + n);
        uint32_t wd[4];
        if (vec) {
            uint4 v = __ldg(reinterpret_cast<const uint4*>(w + n * ldw + k0));
            wd[0] = v.x; wd[1] = v.y; wd[2] = v.z; wd[3] = v.w;
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t word = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    int64_t k = k0 + q * 4 + b;
                    if (k < K) word |= (uint32_t)w[n * ldw + k] << (8 * b);
                }
                wd[q] = word;
            }
        }
#pragma unroll
        for (int j = 0; j < FV_WCOLS; ++j)
            acc[j] += (uint64_t)(int64_t)ima_e4m3_codebook((wd[j >> 2] >> (8 * (j & 3))) & 0xFFu) * rn;
    }
#pragma unroll
    for (int j = 0; j < FV_WCOLS; ++j)
        if (k0 + j < K) atomicAdd(t + k0 + j, (unsigned long long)acc[j]);
}

// Weight pass for int32 b [K,N] (row-major, the reference's weight_t): one warp per row k.
__global__ void __launch_bounds__(FV_THREADS) fv_weight_i32_kernel(const int32_t* __restrict__ b, int64_t ldb,
                                                                  const int64_t* __restrict__ r, int64_t N, int64_t K,
                                                                  unsigned long long* __restrict__ t) {
    int64_t k = (int64_t)blockIdx.x * (FV_THREADS / 32) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (k >= K) return;
    uint64_t acc = 0;
    for (int64_t n = lane; n < N; n += 32) acc += (uint64_t)(int64_t)b[k * ldb + n] * (uint64_t)r[n];
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) t[k] = acc;
}

}  // namespace

// One product of a row-pass batch.
struct FvRowProblem {
    const void* a;           // activations: fp8 codes (a_kind 0) or int32 (a_kind 1), [M, K] row stride lda
    const unsigned long long* t;   // [K] = B r
    const int64_t* c;        // [M, N] row stride ldc
    const int64_t* r;        // [N]
    int32_t* mismatch;       // device counter
    int64_t lda, ldc, M, N, K;
    int64_t row_start;       // first global row of this product in the batch
    int32_t a_kind, pad;
};

constexpr int FV_MAXP = 192;
struct FvRowBatch {
    FvRowProblem p[FV_MAXP];
    int32_t n;
    int64_t total_rows;
};

namespace {

// Row pass, aligned fp8 path (every product of the launch has K a multiple of 4, N even,
// 4-byte aligned code rows, 16-byte aligned C rows, t and r): one warp per (product, row).
// The pass is bound by how many loads each warp keeps in flight (rows are short: 896 to
// 4864 codes, 128 to 4864 int64 outputs), so each lane reads FV_UA 4-byte code words (with
// t as two 16-byte pairs per word) and then FV_UC 16-byte pairs of C and r before using any
// of them.  Measured on the 168 c1 products in one launch: 274 us against 319 us with one
// load in flight per lane.
constexpr int FV_UA = 4;   // 4-byte code words in flight per lane
constexpr int FV_UC = 4;   // 16-byte C pairs in flight per lane

IMA_DEVINL uint64_t fv_code_word_dot(uint32_t w, ulonglong2 ta, ulonglong2 tb) {
    return (uint64_t)(int64_t)ima_e4m3_codebook(w & 0xFFu) * ta.x +
           (uint64_t)(int64_t)ima_e4m3_codebook((w >> 8) & 0xFFu) * ta.y +
           (uint64_t)(int64_t)ima_e4m3_codebook((w >> 16) & 0xFFu) * tb.x +
           (uint64_t)(int64_t)ima_e4m3_codebook(w >> 24) * tb.y;
}

__global__ void __launch_bounds__(FV_THREADS) fv_rows_aligned_kernel(const __grid_constant__ FvRowBatch batch) {
    const int lane = threadIdx.x & 31;
    const int64_t warps_total = (int64_t)gridDim.x * (FV_THREADS / 32);
    for (int64_t g = (int64_t)blockIdx.x * (FV_THREADS / 32) + (threadIdx.x >> 5); g < batch.total_rows;
         g += warps_total) {
        int lo = 0, hi = batch.n - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (batch.p[mid].row_start <= g) lo = mid; else hi = mid - 1;
        }
        const FvRowProblem& P = batch.p[lo];
        const int64_t m = g - P.row_start;
        uint64_t acc = 0;   // lane share of A[m,:] . t - C[m,:] . r
        const uint32_t* a4 = reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(P.a) + m * P.lda);
        const ulonglong2* t2 = reinterpret_cast<const ulonglong2*>(P.t);
        const int64_t k4 = P.K / 4;
        int64_t i = lane;
        for (; i + 32 * (FV_UA - 1) < k4; i += 32 * FV_UA) {
            uint32_t wd[FV_UA];
            ulonglong2 ta[FV_UA], tb[FV_UA];
#pragma unroll
            for (int u = 0; u < FV_UA; ++u) wd[u] = __ldcs(a4 + i + 32 * u);
#pragma unroll
            for (int u = 0; u < FV_UA; ++u) {
                ta[u] = __ldg(t2 + 2 * (i + 32 * u));
                tb[u] = __ldg(t2 + 2 * (i + 32 * u) + 1);
            }
#pragma unroll
            for (int u = 0; u < FV_UA; ++u) acc += fv_code_word_dot(wd[u], ta[u], tb[u]);
        }
        for (; i < k4; i += 32) acc += fv_code_word_dot(__ldcs(a4 + i), __ldg(t2 + 2 * i), __ldg(t2 + 2 * i + 1));

        const longlong2* c2 = reinterpret_cast<const longlong2*>(P.c + m * P.ldc);
        const longlong2* r2 = reinterpret_cast<const longlong2*>(P.r);
        const int64_t n2 = P.N / 2;
        i = lane;
        for (; i + 32 * (FV_UC - 1) < n2; i += 32 * FV_UC) {
            longlong2 cv[FV_UC], rv[FV_UC];
#pragma unroll
            for (int u = 0; u < FV_UC; ++u) cv[u] = __ldcs(c2 + i + 32 * u);   // read once: stream
#pragma unroll
            for (int u = 0; u < FV_UC; ++u) rv[u] = __ldg(r2 + i + 32 * u);
#pragma unroll
            for (int u = 0; u < FV_UC; ++u)
                acc -= (uint64_t)cv[u].x * (uint64_t)rv[u].x + (uint64_t)cv[u].y * (uint64_t)rv[u].y;
        }
        for (; i < n2; i += 32) {
            const longlong2 cv = __ldcs(c2 + i), rv = __ldg(r2 + i);
            acc -= (uint64_t)cv.x * (uint64_t)rv.x + (uint64_t)cv.y * (uint64_t)rv.y;
        }
        // the row passes iff the lane shares sum to 0 (mod 2^64)
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (lane == 0 && acc != 0) atomicAdd(P.mismatch, 1);
    }
}

// Row pass, general path (int32 activations, unaligned rows or vectors): one warp per
// (product, row), one load in flight per lane.
__global__ void __launch_bounds__(FV_THREADS) fv_rows_kernel(const __grid_constant__ FvRowBatch batch) {
    const int lane = threadIdx.x & 31;
    const int64_t warps_total = (int64_t)gridDim.x * (FV_THREADS / 32);
    for (int64_t g = (int64_t)blockIdx.x * (FV_THREADS / 32) + (threadIdx.x >> 5); g < batch.total_rows;
         g += warps_total) {
        int lo = 0, hi = batch.n - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (batch.p[mid].row_start <= g) lo = mid; else hi = mid - 1;
        }
        const FvRowProblem& P = batch.p[lo];
        const int64_t m = g - P.row_start;
        uint64_t lhs = 0, rhs = 0;
        if (P.a_kind == 0) {
            const uint8_t* arow = reinterpret_cast<const uint8_t*>(P.a) + m * P.lda;
            const bool vec = ((reinterpret_cast<uintptr_t>(arow) & 3) == 0);
            if (vec) {
                const int64_t k4 = P.K / 4;
                for (int64_t i = lane; i < k4; i += 32) {
                    uint32_t wd = __ldg(reinterpret_cast<const uint32_t*>(arow) + i);
#pragma unroll
                    for (int b = 0; b < 4; ++b)
                        lhs += (uint64_t)(int64_t)ima_e4m3_codebook((wd >> (8 * b)) & 0xFFu) * (uint64_t)P.t[4 * i + b];
                }
                for (int64_t k = 4 * k4 + lane; k < P.K; k += 32)
                    lhs += (uint64_t)(int64_t)ima_e4m3_codebook(arow[k]) * (uint64_t)P.t[k];
            } else {
                for (int64_t k = lane; k < P.K; k += 32)
                    lhs += (uint64_t)(int64_t)ima_e4m3_codebook(arow[k]) * (uint64_t)P.t[k];
            }
        } else {
            const int32_t* arow = reinterpret_cast<const int32_t*>(P.a) + m * P.lda;
            for (int64_t k = lane; k < P.K; k += 32) lhs += (uint64_t)(int64_t)arow[k] * (uint64_t)P.t[k];
        }
        const int64_t* crow = P.c + m * P.ldc;
        const bool cvec = ((reinterpret_cast<uintptr_t>(crow) & 15) == 0) && ((reinterpret_cast<uintptr_t>(P.r) & 15) == 0);
        if (cvec) {
            const int64_t n2 = P.N / 2;
            for (int64_t i = lane; i < n2; i += 32) {
                longlong2 cv = __ldcs(reinterpret_cast<const longlong2*>(crow) + i);   // read once: stream
                longlong2 rv = __ldg(reinterpret_cast<const longlong2*>(P.r) + i);
                rhs += (uint64_t)cv.x * (uint64_t)rv.x + (uint64_t)cv.y * (uint64_t)rv.y;
            }
            if (lane == 0 && (P.N & 1)) rhs += (uint64_t)crow[P.N - 1] * (uint64_t)P.r[P.N - 1];
        } else {
            for (int64_t n = lane; n < P.N; n += 32) rhs += (uint64_t)crow[n] * (uint64_t)P.r[n];
        }
        uint64_t d = lhs - rhs;   // the row passes iff the lane partial differences sum to 0 (mod 2^64)
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
        if (lane == 0 && d != 0) atomicAdd(P.mismatch, 1);
    }
}

int launch_rows(const FvRowBatch& b, cudaStream_t s) {
    if (b.total_rows == 0) return IMA_OK;
    int64_t blocks = (b.total_rows + (FV_THREADS / 32) - 1) / (FV_THREADS / 32);
    if (blocks > 148 * 64) blocks = 148 * 64;
    bool aligned = true;
    for (int i = 0; i < b.n && aligned; ++i) {
        const FvRowProblem& P = b.p[i];
        aligned = P.a_kind == 0 && (P.K & 3) == 0 && (P.N & 1) == 0 &&
                  (reinterpret_cast<uintptr_t>(P.a) & 3) == 0 && (P.lda & 3) == 0 &&
                  (reinterpret_cast<uintptr_t>(P.t) & 15) == 0 && (reinterpret_cast<uintptr_t>(P.c) & 15) == 0 &&
                  (P.ldc & 1) == 0 && (reinterpret_cast<uintptr_t>(P.r) & 15) == 0;
    }
    if (aligned)
        fv_rows_aligned_kernel<<<(unsigned)blocks, FV_THREADS, 0, s>>>(b);
    else
        fv_rows_kernel<<<(unsigned)blocks, FV_THREADS, 0, s>>>(b);
    return IMA_LAUNCH_STATUS();
}

int weight_vector_fp8(const uint8_t* w, int64_t ldw, const int64_t* r, int64_t N, int64_t K,
                      unsigned long long* t, cudaStream_t s) {
    int rc = ima_note_cuda(cudaMemsetAsync(t, 0, (size_t)(K > 0 ? K : 1) * 8, s));
    if (rc != IMA_OK || K == 0 || N == 0) return rc;
    int64_t units = ((K + FV_WCOLS - 1) / FV_WCOLS) * ((N + FV_WROWS - 1) / FV_WROWS);
    fv_weight_fp8_kernel<<<(unsigned)((units + FV_THREADS - 1) / FV_THREADS), FV_THREADS, 0, s>>>(w, ldw, r, N, K, t);
    return IMA_LAUNCH_STATUS();
}

}  // namespace

extern "C" {

int64_t ima_freivalds_workspace_bytes(int64_t K) { return (K > 0 ? K : 1) * 8; }

int ima_freivalds_weight_vector(const uint8_t* w_fp8, int64_t ldw, const int64_t* r, int64_t N, int64_t K,
                                int64_t* t, void* stream) {
    if (!w_fp8 || !r || !t || N < 0 || K < 0 || ldw < K) return IMA_ERR_INVALID_ARGUMENT;
    return weight_vector_fp8(w_fp8, ldw, r, N, K, reinterpret_cast<unsigned long long*>(t), (cudaStream_t)stream);
}

int ima_freivalds_rows_grouped(const ima_freivalds_rows_problem* problems, int count, void* stream) {
    if (count < 0 || (count > 0 && !problems)) return IMA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < count; ++i) {
        const ima_freivalds_rows_problem& q = problems[i];
        if (!q.a || !q.t || !q.c || !q.r || !q.mismatch_rows) return IMA_ERR_INVALID_ARGUMENT;
        if (q.M < 0 || q.N < 0 || q.K < 0 || q.lda < q.K || q.ldc < q.N) return IMA_ERR_INVALID_ARGUMENT;
        if (q.a_kind != IMA_FREIVALDS_A_FP8 && q.a_kind != IMA_FREIVALDS_A_INT32) return IMA_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    FvRowBatch b;
    memset(&b, 0, sizeof(b));
    for (int i = 0; i < count; ++i) {
        const ima_freivalds_rows_problem& q = problems[i];
        FvRowProblem& P = b.p[b.n];
        P.a = q.a; P.t = reinterpret_cast<const unsigned long long*>(q.t); P.c = q.c; P.r = q.r;
        P.mismatch = q.mismatch_rows; P.lda = q.lda; P.ldc = q.ldc; P.M = q.M; P.N = q.N; P.K = q.K;
        P.a_kind = q.a_kind; P.row_start = b.total_rows;
        b.total_rows += q.M;
        if (++b.n == FV_MAXP) {
            int rc = launch_rows(b, s);
            if (rc != IMA_OK) return rc;
            memset(&b, 0, sizeof(b));
        }
    }
    return b.n ? launch_rows(b, s) : IMA_OK;
}

int ima_freivalds_fp8(const uint8_t* x_fp8, int64_t ldx, const uint8_t* w_fp8, int64_t ldw, const int64_t* c,
                      int64_t ldc, const int64_t* r, int64_t M, int64_t N, int64_t K, void* workspace,
                      int32_t* mismatch_rows, void* stream) {
    if (!x_fp8 || !w_fp8 || !c || !r || !workspace || !mismatch_rows) return IMA_ERR_INVALID_ARGUMENT;
    if (M < 0 || N < 0 || K < 0 || ldx < K || ldw < K || ldc < N) return IMA_ERR_INVALID_ARGUMENT;
    if (M == 0) return IMA_OK;
    int rc = ima_freivalds_weight_vector(w_fp8, ldw, r, N, K, reinterpret_cast<int64_t*>(workspace), stream);
    if (rc != IMA_OK) return rc;
    ima_freivalds_rows_problem q = {x_fp8, ldx, reinterpret_cast<const int64_t*>(workspace), c, ldc, r,
                                    M, N, K, IMA_FREIVALDS_A_FP8, mismatch_rows};
    return ima_freivalds_rows_grouped(&q, 1, stream);
}

int ima_freivalds_i32(const int32_t* a, int64_t lda, const int32_t* b, int64_t ldb, const int64_t* c, int64_t ldc,
                      const int64_t* r, int64_t M, int64_t N, int64_t K, void* workspace, int32_t* mismatch_rows,
                      void* stream) {
    if (!a || !b || !c || !r || !workspace || !mismatch_rows) return IMA_ERR_INVALID_ARGUMENT;
    if (M < 0 || N < 0 || K < 0 || lda < K || ldb < N || ldc < N) return IMA_ERR_INVALID_ARGUMENT;
    if (M == 0) return IMA_OK;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* t = reinterpret_cast<unsigned long long*>(workspace);
    if (K > 0) {
        unsigned g1 = (unsigned)((K + FV_THREADS / 32 - 1) / (FV_THREADS / 32));
        fv_weight_i32_kernel<<<g1, FV_THREADS, 0, s>>>(b, ldb, r, N, K, t);
        int rc = IMA_LAUNCH_STATUS();
        if (rc != IMA_OK) return rc;
    }
    ima_freivalds_rows_problem q = {a, lda, reinterpret_cast<const int64_t*>(workspace), c, ldc, r,
                                    M, N, K, IMA_FREIVALDS_A_INT32, mismatch_rows};
    return ima_freivalds_rows_grouped(&q, 1, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of the codebook Freivalds check.
//
// Some callers cannot allocate device memory for the check's scratch vector: a verifier
// embedded in a process whose device memory is already reserved by another allocator
// (a framework's caching allocator can hold nearly all of it, so a cudaMalloc from here
// could fail or fragment that pool), or a latency-sensitive verification path that must
// not pay for cudaMalloc/cudaFree, which can synchronise the device.  For them the scratch
// t = codebook(W)^T r lives in a fixed array in this library's device image instead.
//
// The array is a host-side stand-in in host code, so its device address is looked up once
// per device with that device current (cudaGetSymbolAddress) and passed to the kernels.
// Every GPU that loads the library holds the array (IMA_FREIVALDS_NOALLOC_MAX_K * 8 bytes)
// until the process exits.  All calls on a device share it and it keeps the last call's
// contents; the weight pass clears it at the start of each call.  Calls whose work
// overlaps on the GPU (different streams, or several host threads) race on the array.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned long long g_fv_noalloc_scratch[IMA_FREIVALDS_NOALLOC_MAX_K];

namespace {

constexpr int FV_NOALLOC_MAX_DEVICES = 64;
std::mutex g_fv_noalloc_mutex;
unsigned long long* g_fv_noalloc_ptr[FV_NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on the current device (looked up on first use);
// *dev_out receives that device.
int fv_noalloc_scratch(unsigned long long** out, int* dev_out) {
    int dev = -1;
    int rc = ima_note_cuda(cudaGetDevice(&dev));
    if (rc != IMA_OK) return rc;
    if (dev < 0 || dev >= FV_NOALLOC_MAX_DEVICES) return IMA_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_fv_noalloc_mutex);
    if (!g_fv_noalloc_ptr[dev]) {
        void* p = nullptr;
        rc = ima_note_cuda(cudaGetSymbolAddress(&p, g_fv_noalloc_scratch));
        if (rc != IMA_OK) return rc;
        if (!p) return IMA_ERR_CUDA;
        g_fv_noalloc_ptr[dev] = reinterpret_cast<unsigned long long*>(p);
    }
    *out = g_fv_noalloc_ptr[dev];
    *dev_out = dev;
    return IMA_OK;
}

// The scratch array used is the current device's copy, so the stream and every operand
// must belong to that device: a stream of another GPU would run the kernels there against
// this GPU's array, and a host or other-GPU pointer would reach a kernel.  Checked before
// any launch; a mismatch is IMA_ERR_INVALID_ARGUMENT.
int fv_noalloc_same_device(int dev, cudaStream_t s, const void* const* ptrs, int n) {
    int sdev = -1;
    if (cudaStreamGetDevice(s, &sdev) != cudaSuccess) {
        cudaGetLastError();
        return IMA_ERR_INVALID_ARGUMENT;
    }
    if (sdev != dev) return IMA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < n; ++i) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, ptrs[i]) != cudaSuccess) {
            cudaGetLastError();
            return IMA_ERR_INVALID_ARGUMENT;
        }
        if (a.type == cudaMemoryTypeManaged) continue;
        if (a.type != cudaMemoryTypeDevice || a.device != dev) return IMA_ERR_INVALID_ARGUMENT;
    }
    return IMA_OK;
}

}  // namespace

extern "C" int ima_freivalds_fp8_noalloc(const uint8_t* x_fp8, int64_t ldx, const uint8_t* w_fp8, int64_t ldw,
                                         const int64_t* c, int64_t ldc, const int64_t* r, int64_t M, int64_t N,
                                         int64_t K, int32_t* mismatch_rows, void* stream) {
    if (!x_fp8 || !w_fp8 || !c || !r || !mismatch_rows) return IMA_ERR_INVALID_ARGUMENT;
    if (M < 0 || N < 0 || K < 0 || ldx < K || ldw < K || ldc < N) return IMA_ERR_INVALID_ARGUMENT;
    if (K > IMA_FREIVALDS_NOALLOC_MAX_K) return IMA_ERR_UNSUPPORTED;   // the fixed scratch holds K <= max
    unsigned long long* scratch = nullptr;
    int dev = -1;
    int rc = fv_noalloc_scratch(&scratch, &dev);
    if (rc != IMA_OK) return rc;
    const void* operands[5] = {x_fp8, w_fp8, c, r, mismatch_rows};
    rc = fv_noalloc_same_device(dev, (cudaStream_t)stream, operands, 5);
    if (rc != IMA_OK) return rc;
    return ima_freivalds_fp8(x_fp8, ldx, w_fp8, ldw, c, ldc, r, M, N, K, scratch, mismatch_rows, stream);
}
