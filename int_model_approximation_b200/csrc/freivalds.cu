// Freivalds check of a claimed int64 product C = A B: accept row m iff
//     sum_k A[m,k] * (sum_n B[k,n] r[n]) == sum_n C[m,n] r[n]      (mod 2^64).
// ref: tests/test_real_integer_gemms.py:67-93 (the reference checks with Python
// integers; a correct product satisfies the identity over Z, hence mod 2^64, and a
// single corrupted entry C[m,n] + d is rejected whenever d * r[n] != 0 mod 2^64).
//
// Two bandwidth-bound GEMV passes:
//   pass 1  t = B r          (reads B once: N*K codes)
//   pass 2  per row m: A[m,:] . t  vs  C[m,:] . r   (reads A and C once: M*K + 8*M*N bytes)
// All arithmetic is uint64 (wrapping), identical to the CPU oracle.
#include "ima_common.cuh"

namespace {

constexpr int FV_THREADS = 256;
constexpr int FV_COLS_PER_THREAD = 16;   // fp8 pass 1: one 16-byte load per row per thread
constexpr int FV_ROWS_PER_BLOCK = 64;    // fp8 pass 1: rows (n) summed by one block before the atomic

// Pass 1 for fp8 weights w [N,K]: t[k] += sum_{n in block rows} code(w[n,k]) * r[n].
__global__ void __launch_bounds__(FV_THREADS) fv_br_fp8_kernel(const uint8_t* __restrict__ w, int64_t ldw,
                                                              const int64_t* __restrict__ r, int64_t N, int64_t K,
                                                              unsigned long long* __restrict__ t) {
    int64_t k0 = ((int64_t)blockIdx.x * FV_THREADS + threadIdx.x) * FV_COLS_PER_THREAD;
    int64_t n0 = (int64_t)blockIdx.y * FV_ROWS_PER_BLOCK;
    if (k0 >= K) return;
    uint64_t acc[FV_COLS_PER_THREAD];
#pragma unroll
    for (int j = 0; j < FV_COLS_PER_THREAD; ++j) acc[j] = 0;
    int64_t n1 = n0 + FV_ROWS_PER_BLOCK < N ? n0 + FV_ROWS_PER_BLOCK : N;
    bool vec = (k0 + FV_COLS_PER_THREAD <= K) && ((ldw & 15) == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
    for (int64_t n = n0; n < n1; ++n) {
        uint64_t rn = (uint64_t)r[n];
        uint8_t b[FV_COLS_PER_THREAD];
        if (vec) {
            uint4 v = __ldg(reinterpret_cast<const uint4*>(w + n * ldw + k0));
            memcpy(b, &v, 16);
        } else {
#pragma unroll
            for (int j = 0; j < FV_COLS_PER_THREAD; ++j) b[j] = (k0 + j < K) ? w[n * ldw + k0 + j] : 0;
        }
#pragma unroll
        for (int j = 0; j < FV_COLS_PER_THREAD; ++j) acc[j] += (uint64_t)(int64_t)ima_e4m3_codebook(b[j]) * rn;
    }
#pragma unroll
    for (int j = 0; j < FV_COLS_PER_THREAD; ++j)
        if (k0 + j < K) atomicAdd(t + k0 + j, (unsigned long long)acc[j]);
}

// Pass 1 for int32 b [K,N] (row-major, the reference's weight_t): one warp per row k.
__global__ void __launch_bounds__(FV_THREADS) fv_br_i32_kernel(const int32_t* __restrict__ b, int64_t ldb,
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

IMA_DEVINL uint64_t block_sum_u64(uint64_t v, uint64_t* s_red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) s_red[warp] = v;
    __syncthreads();
    uint64_t s = 0;
    if (threadIdx.x == 0)
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += s_red[i];
    __syncthreads();
    return s;   // valid in thread 0 only
}

// Pass 2: one block per row m.  A is fp8 codes (kind 0) or int32 (kind 1).
template <int KIND>
__global__ void __launch_bounds__(FV_THREADS) fv_rows_kernel(const void* __restrict__ a, int64_t lda,
                                                            const unsigned long long* __restrict__ t,
                                                            const int64_t* __restrict__ c, int64_t ldc,
                                                            const int64_t* __restrict__ r, int64_t M, int64_t N,
                                                            int64_t K, int32_t* __restrict__ mismatch_rows) {
    __shared__ uint64_t s_red[FV_THREADS / 32];
    for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
        uint64_t lhs = 0, rhs = 0;
        for (int64_t k = threadIdx.x; k < K; k += FV_THREADS) {
            int64_t av;
            if (KIND == 0) av = ima_e4m3_codebook(reinterpret_cast<const uint8_t*>(a)[m * lda + k]);
            else av = reinterpret_cast<const int32_t*>(a)[m * lda + k];
            lhs += (uint64_t)av * (uint64_t)t[k];
        }
        const int64_t* crow = c + m * ldc;
        bool vec = ((reinterpret_cast<uintptr_t>(crow) & 15) == 0) && ((reinterpret_cast<uintptr_t>(r) & 15) == 0);
        if (vec) {
            int64_t n2 = N / 2;
            for (int64_t i = threadIdx.x; i < n2; i += FV_THREADS) {
                longlong2 cv = __ldcs(reinterpret_cast<const longlong2*>(crow) + i);   // streamed: read once
                longlong2 rv = __ldg(reinterpret_cast<const longlong2*>(r) + i);
                rhs += (uint64_t)cv.x * (uint64_t)rv.x + (uint64_t)cv.y * (uint64_t)rv.y;
            }
            if (threadIdx.x == 0 && (N & 1)) rhs += (uint64_t)crow[N - 1] * (uint64_t)r[N - 1];
        } else {
            for (int64_t n = threadIdx.x; n < N; n += FV_THREADS) rhs += (uint64_t)crow[n] * (uint64_t)r[n];
        }
        uint64_t d = block_sum_u64(lhs - rhs, s_red);
        if (threadIdx.x == 0 && d != 0) atomicAdd(mismatch_rows, 1);
    }
}

inline unsigned rows_grid(int64_t M) { return (unsigned)(M < 148 * 16 ? M : 148 * 16); }

}  // namespace

extern "C" {

int64_t ima_freivalds_workspace_bytes(int64_t K) { return (K > 0 ? K : 1) * 8; }

int ima_freivalds_fp8(const uint8_t* x_fp8, int64_t ldx, const uint8_t* w_fp8, int64_t ldw, const int64_t* c,
                      int64_t ldc, const int64_t* r, int64_t M, int64_t N, int64_t K, void* workspace,
                      int32_t* mismatch_rows, void* stream) {
    if (!x_fp8 || !w_fp8 || !c || !r || !workspace || !mismatch_rows) return IMA_ERR_INVALID_ARGUMENT;
    if (M < 0 || N < 0 || K < 0 || ldx < K || ldw < K || ldc < N) return IMA_ERR_INVALID_ARGUMENT;
    if (M == 0) return IMA_OK;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* t = reinterpret_cast<unsigned long long*>(workspace);
    int rc = ima_note_cuda(cudaMemsetAsync(t, 0, (size_t)(K > 0 ? K : 1) * 8, s));
    if (rc != IMA_OK) return rc;
    if (K > 0 && N > 0) {
        dim3 g1((unsigned)((K + FV_THREADS * FV_COLS_PER_THREAD - 1) / (FV_THREADS * FV_COLS_PER_THREAD)),
                (unsigned)((N + FV_ROWS_PER_BLOCK - 1) / FV_ROWS_PER_BLOCK));
        if (g1.y > 65535u) return IMA_ERR_UNSUPPORTED;
        fv_br_fp8_kernel<<<g1, FV_THREADS, 0, s>>>(w_fp8, ldw, r, N, K, t);
        rc = IMA_LAUNCH_STATUS();
        if (rc != IMA_OK) return rc;
    }
    fv_rows_kernel<0><<<rows_grid(M), FV_THREADS, 0, s>>>(x_fp8, ldx, t, c, ldc, r, M, N, K, mismatch_rows);
    return IMA_LAUNCH_STATUS();
}

int ima_freivalds_i32(const int32_t* a, int64_t lda, const int32_t* b, int64_t ldb, const int64_t* c, int64_t ldc,
                      const int64_t* r, int64_t M, int64_t N, int64_t K, void* workspace, int32_t* mismatch_rows,
                      void* stream) {
    if (!a || !b || !c || !r || !workspace || !mismatch_rows) return IMA_ERR_INVALID_ARGUMENT;
    if (M < 0 || N < 0 || K < 0 || lda < K || ldb < N || ldc < N) return IMA_ERR_INVALID_ARGUMENT;
    if (M == 0) return IMA_OK;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* t = reinterpret_cast<unsigned long long*>(workspace);
    int rc = ima_note_cuda(cudaMemsetAsync(t, 0, (size_t)(K > 0 ? K : 1) * 8, s));
    if (rc != IMA_OK) return rc;
    if (K > 0) {
        unsigned g1 = (unsigned)((K + FV_THREADS / 32 - 1) / (FV_THREADS / 32));
        fv_br_i32_kernel<<<g1, FV_THREADS, 0, s>>>(b, ldb, r, N, K, t);
        rc = IMA_LAUNCH_STATUS();
        if (rc != IMA_OK) return rc;
    }
    fv_rows_kernel<1><<<rows_grid(M), FV_THREADS, 0, s>>>(a, lda, t, c, ldc, r, M, N, K, mismatch_rows);
    return IMA_LAUNCH_STATUS();
}

}  // extern "C"
