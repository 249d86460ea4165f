// Per-token FP8 quantiser and the digit planes consumed by the tensor-core GEMM.
//
// ref: __main__.py:148-163 (_per_token_fp8, _fp8_e4m3_to_int32, _per_token_fp8_int32).
//   scale = max(amax_k |x[m,k]| / 448, 1e-12)     fp32, IEEE division
//   q     = e4m3_rne(float(x) / scale)           fp32, IEEE division, torch's e4m3fn cast
//   code  = round(q * 512)                       exact integer, |code| <= 229376
//
// Digit planes.  The GEMM multiplies int8 operands, so each integer operand value v
// is written in balanced base-128 digits.  Scheme KARATSUBA3 (|v| <= 1,064,960, which
// covers every codebook value): v = d0 + 2^7 d1 + 2^14 d2 and the six planes
//     P0 = d0, P1 = d1, P2 = d2, P3 = d0 + d1, P4 = d1 + d2, P5 = d0 + d2
// all fit int8 (d0, d1 in [-64, 63]); the GEMM forms the six plane products and
// recombines them Karatsuba-style.  Scheme DIGITS5 (any int32): five digits
// v = sum_i 2^(7 i) d_i and the 25 digit products are grouped by shift.
#include "ima_common.cuh"

namespace {

IMA_DEVINL float load_as_f32(const void* x, int dtype, int64_t idx) {
    if (dtype == IMA_DTYPE_BF16) return ima_bf16_to_f32(reinterpret_cast<const uint16_t*>(x)[idx]);
    if (dtype == IMA_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(x)[idx]);
    return reinterpret_cast<const float*>(x)[idx];
}

// Six Karatsuba planes of a codebook value (int8 each, packed little-endian per plane).
IMA_DEVINL void karatsuba_planes(int32_t v, int32_t p[6]) {
    int32_t d0, d1, d2;
    ima_digits3(v, d0, d1, d2);
    p[0] = d0; p[1] = d1; p[2] = d2; p[3] = d0 + d1; p[4] = d1 + d2; p[5] = d0 + d2;
}

IMA_DEVINL void digits5(int32_t v, int32_t d[5]) {
    int64_t w = v;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int32_t di = (int32_t)(((w + 64) & 127) - 64);
        d[i] = di;
        w = (w - di) >> 7;
    }
    d[4] = (int32_t)w;  // |w| <= 8 for any int32
}

}  // namespace

// One quantisation problem of a batch (a kernel parameter; no device-side descriptor memory).
struct QuantProblem {
    const void* x;
    int64_t ldx;
    int64_t M, K;
    uint8_t* q;
    int64_t ldq;
    float* scale;
    float* code_scale;
    int32_t* codebook;
    int64_t ldc;
    int8_t* planes;
    int64_t ldp;
    int64_t row_start;
    int32_t dtype, pad;
};

constexpr int QZ_MAXP = 192;
struct QuantBatch {
    QuantProblem p[QZ_MAXP];
    int32_t n;
    int64_t total_rows;
};

namespace {

// One CTA per (problem, row), grid-stride over all rows of the batch.  Pass 1:
// NaN-propagating amax.  Pass 2: quantise four consecutive columns per thread-iteration
// so each plane store is one 32-bit word.
__global__ void __launch_bounds__(256) quantize_rows_kernel(const __grid_constant__ QuantBatch batch) {
    __shared__ float s_red[32];
    __shared__ int s_nan[32];
    for (int64_t g = blockIdx.x; g < batch.total_rows; g += gridDim.x) {
        int lo = 0, hi = batch.n - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (batch.p[mid].row_start <= g) lo = mid; else hi = mid - 1;
        }
        const QuantProblem& P = batch.p[lo];
        const int64_t m = g - P.row_start;
        const void* x = P.x;
        const int dtype = P.dtype;
        const int64_t M = P.M, K = P.K, ldx = P.ldx, ldq = P.ldq, ldc = P.ldc, ldp = P.ldp;
        uint8_t* q = P.q;
        float* scale_out = P.scale;
        float* code_scale = P.code_scale;
        int32_t* codebook = P.codebook;
        int8_t* planes = P.planes;
        float amax = 0.0f;
        int has_nan = 0;
        for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
            float v = fabsf(load_as_f32(x, dtype, m * ldx + k));
            if (v != v) has_nan = 1;
            else amax = fmaxf(amax, v);
        }
        for (int o = 16; o > 0; o >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
            has_nan |= __shfl_xor_sync(0xFFFFFFFFu, has_nan, o);
        }
        int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        if (lane == 0) { s_red[warp] = amax; s_nan[warp] = has_nan; }
        __syncthreads();
        if (warp == 0) {
            int nw = blockDim.x >> 5;
            amax = lane < nw ? s_red[lane] : 0.0f;
            has_nan = lane < nw ? s_nan[lane] : 0;
            for (int o = 16; o > 0; o >>= 1) {
                amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
                has_nan |= __shfl_xor_sync(0xFFFFFFFFu, has_nan, o);
            }
            if (lane == 0) { s_red[0] = amax; s_nan[0] = has_nan; }
        }
        __syncthreads();
        float s = s_nan[0] ? __int_as_float(0x7FC00000) : s_red[0];
        s = __fdiv_rn(s, 448.0f);
        s = (s < 1e-12f) ? 1e-12f : s;   // clamp_min keeps NaN
        if (threadIdx.x == 0) {
            scale_out[m] = s;
            if (code_scale) code_scale[m] = __fdiv_rn(s, 512.0f);
        }
        int64_t kq = planes ? ldp : K;   // planes are zero-filled up to ldp
        for (int64_t k0 = (int64_t)threadIdx.x * 4; k0 < kq; k0 += (int64_t)blockDim.x * 4) {
            uint32_t word[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                int64_t k = k0 + j;
                if (k >= K) break;
                float f = __fdiv_rn(load_as_f32(x, dtype, m * ldx + k), s);
                uint8_t b = ima_f32_to_e4m3(f);
                q[m * ldq + k] = b;
                int32_t v = ima_e4m3_codebook(b);
                if (codebook) codebook[m * ldc + k] = v;
                if (planes) {
                    int32_t p[6];
                    karatsuba_planes(v, p);
#pragma unroll
                    for (int i = 0; i < 6; ++i) word[i] |= ((uint32_t)p[i] & 0xFFu) << (8 * j);
                }
            }
            if (planes) {
#pragma unroll
                for (int i = 0; i < 6; ++i)
                    *reinterpret_cast<uint32_t*>(planes + ((int64_t)i * M + m) * ldp + k0) = word[i];
            }
        }
        __syncthreads();
    }
}

// Planes of an e4m3 matrix (weights): one thread per 4 consecutive columns.
__global__ void planes_from_fp8_kernel(const uint8_t* __restrict__ src, int64_t rows, int64_t K, int64_t ld,
                                       int8_t* __restrict__ planes, int64_t ldp, int32_t* __restrict__ codebook_t) {
    int64_t words = ldp / 4;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * words) return;
    int64_t r = idx / words, k0 = (idx % words) * 4;
    uint32_t word[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        int64_t k = k0 + j;
        if (k >= K) break;
        int32_t v = ima_e4m3_codebook(src[r * ld + k]);
        if (codebook_t) codebook_t[k * rows + r] = v;
        int32_t p[6];
        karatsuba_planes(v, p);
#pragma unroll
        for (int i = 0; i < 6; ++i) word[i] |= ((uint32_t)p[i] & 0xFFu) << (8 * j);
    }
#pragma unroll
    for (int i = 0; i < 6; ++i) *reinterpret_cast<uint32_t*>(planes + ((int64_t)i * rows + r) * ldp + k0) = word[i];
}

// Planes of a strided int32 matrix.
__global__ void planes_from_int32_kernel(const int32_t* __restrict__ src, int64_t rows, int64_t K,
                                         int64_t stride_row, int64_t stride_k, int scheme,
                                         int8_t* __restrict__ planes, int64_t ldp) {
    int64_t words = ldp / 4;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * words) return;
    int64_t r = idx / words, k0 = (idx % words) * 4;
    uint32_t word[6] = {0, 0, 0, 0, 0, 0};
    int np = scheme == IMA_SCHEME_KARATSUBA3 ? 6 : 5;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        int64_t k = k0 + j;
        if (k >= K) break;
        int32_t v = src[r * stride_row + k * stride_k];
        int32_t p[6] = {0, 0, 0, 0, 0, 0};
        if (scheme == IMA_SCHEME_KARATSUBA3) {
            if (v > 1064960 || v < -1064960) ima_record_error(IMA_ERR_OVERFLOW, IMA_WHERE_PLANES, 0);
            karatsuba_planes(v, p);
        } else {
            digits5(v, p);
        }
#pragma unroll
        for (int i = 0; i < 6; ++i) word[i] |= ((uint32_t)p[i] & 0xFFu) << (8 * j);
    }
    for (int i = 0; i < np; ++i) *reinterpret_cast<uint32_t*>(planes + ((int64_t)i * rows + r) * ldp + k0) = word[i];
}

__global__ void int32_maxabs_kernel(const int32_t* __restrict__ src, int64_t rows, int64_t cols, int64_t sr,
                                    int64_t sc, unsigned long long* __restrict__ out) {
    unsigned long long mx = 0;
    int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i / cols, c = i % cols;
        int64_t v = src[r * sr + c * sc];
        unsigned long long a = (unsigned long long)(v < 0 ? -v : v);
        mx = a > mx ? a : mx;
    }
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
        mx = t > mx ? t : mx;
    }
    if ((threadIdx.x & 31) == 0 && mx) atomicMax(out, mx);
}

__global__ void codebook_from_fp8_kernel(const uint8_t* __restrict__ src, int64_t rows, int64_t K, int64_t ld,
                                         int32_t* __restrict__ dst, int64_t ldd) {
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * K) return;
    int64_t r = idx / K, k = idx % K;
    dst[r * ldd + k] = ima_e4m3_codebook(src[r * ld + k]);
}

inline unsigned grid_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

extern "C" {

int ima_scheme_planes(int scheme) {
    return scheme == IMA_SCHEME_KARATSUBA3 ? 6 : (scheme == IMA_SCHEME_DIGITS5 ? 5 : 0);
}

static int check_quant_problem(const ima_quantize_problem& q) {
    if (!q.x || !q.q_fp8 || !q.scale || q.M < 0 || q.K < 0 || q.ldx < q.K || q.ldq < q.K) return IMA_ERR_INVALID_ARGUMENT;
    if (q.x_dtype != IMA_DTYPE_F32 && q.x_dtype != IMA_DTYPE_BF16 && q.x_dtype != IMA_DTYPE_F16)
        return IMA_ERR_INVALID_ARGUMENT;
    if (q.codebook && q.ldc < q.K) return IMA_ERR_INVALID_ARGUMENT;
    if (q.planes && (q.ldp < q.K || q.ldp % 16 != 0 || (reinterpret_cast<uintptr_t>(q.planes) & 15)))
        return IMA_ERR_INVALID_ARGUMENT;
    return IMA_OK;
}

static int launch_quant(const QuantBatch& b, cudaStream_t s) {
    if (b.total_rows == 0) return IMA_OK;
    int64_t grid = b.total_rows < 148 * 64 ? b.total_rows : 148 * 64;
    quantize_rows_kernel<<<(unsigned)grid, 256, 0, s>>>(b);
    return IMA_LAUNCH_STATUS();
}

int ima_quantize_grouped(const ima_quantize_problem* problems, int count, void* stream) {
    if (count < 0 || (count > 0 && !problems)) return IMA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < count; ++i) {
        int rc = check_quant_problem(problems[i]);
        if (rc != IMA_OK) return rc;
    }
    QuantBatch b;
    memset(&b, 0, sizeof(b));
    for (int i = 0; i < count; ++i) {
        const ima_quantize_problem& q = problems[i];
        QuantProblem& P = b.p[b.n];
        P.x = q.x; P.ldx = q.ldx; P.M = q.M; P.K = q.K; P.q = q.q_fp8; P.ldq = q.ldq; P.scale = q.scale;
        P.code_scale = q.code_scale; P.codebook = q.codebook; P.ldc = q.ldc; P.planes = q.planes; P.ldp = q.ldp;
        P.dtype = q.x_dtype; P.row_start = b.total_rows;
        b.total_rows += q.M;
        if (++b.n == QZ_MAXP) {
            int rc = launch_quant(b, (cudaStream_t)stream);
            if (rc != IMA_OK) return rc;
            memset(&b, 0, sizeof(b));
        }
    }
    return b.n ? launch_quant(b, (cudaStream_t)stream) : IMA_OK;
}

int ima_quantize_per_token(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, uint8_t* q_fp8,
                           int64_t ldq, float* scale, int32_t* codebook, int64_t ldc, float* code_scale,
                           int8_t* planes, int64_t ldp, void* stream) {
    ima_quantize_problem q = {x, x_dtype, M, K, ldx, q_fp8, ldq, scale, codebook, ldc, code_scale, planes, ldp};
    return ima_quantize_grouped(&q, 1, stream);
}

int ima_codebook_from_fp8(const uint8_t* src, int64_t rows, int64_t K, int64_t ld, int32_t* dst, int64_t ldd,
                          void* stream) {
    if (!src || !dst || rows < 0 || K < 0 || ld < K || ldd < K) return IMA_ERR_INVALID_ARGUMENT;
    int64_t n = rows * K;
    if (n == 0) return IMA_OK;
    codebook_from_fp8_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(src, rows, K, ld, dst, ldd);
    return IMA_LAUNCH_STATUS();
}

int ima_planes_from_fp8(const uint8_t* src, int64_t rows, int64_t K, int64_t ld, int8_t* planes, int64_t ldp,
                        int32_t* codebook_t, void* stream) {
    if (!src || !planes || rows < 0 || K < 0 || ld < K || ldp < K || ldp % 16 != 0) return IMA_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(planes) & 15)) return IMA_ERR_INVALID_ARGUMENT;
    int64_t n = rows * (ldp / 4);
    if (n == 0) return IMA_OK;
    planes_from_fp8_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(src, rows, K, ld, planes, ldp,
                                                                               codebook_t);
    return IMA_LAUNCH_STATUS();
}

int ima_planes_from_int32(const int32_t* src, int64_t rows, int64_t K, int64_t stride_row, int64_t stride_k,
                          int scheme, int8_t* planes, int64_t ldp, void* stream) {
    if (!src || !planes || rows < 0 || K < 0 || ldp < K || ldp % 16 != 0) return IMA_ERR_INVALID_ARGUMENT;
    if (scheme != IMA_SCHEME_KARATSUBA3 && scheme != IMA_SCHEME_DIGITS5) return IMA_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(planes) & 15)) return IMA_ERR_INVALID_ARGUMENT;
    int64_t n = rows * (ldp / 4);
    if (n == 0) return IMA_OK;
    planes_from_int32_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(src, rows, K, stride_row, stride_k,
                                                                                 scheme, planes, ldp);
    return IMA_LAUNCH_STATUS();
}

int ima_int32_maxabs(const int32_t* src, int64_t rows, int64_t cols, int64_t stride_row, int64_t stride_col,
                     int64_t* out_maxabs, void* stream) {
    if (!src || !out_maxabs || rows < 0 || cols < 0) return IMA_ERR_INVALID_ARGUMENT;
    int64_t n = rows * cols;
    if (n == 0) return IMA_OK;
    unsigned grid = grid_for(n, 256);
    if (grid > 4096) grid = 4096;
    int32_maxabs_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(src, rows, cols, stride_row, stride_col,
                                                                reinterpret_cast<unsigned long long*>(out_maxabs));
    return IMA_LAUNCH_STATUS();
}

}  // extern "C"
