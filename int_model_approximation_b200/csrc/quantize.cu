// Per-token FP8 quantiser and the digit planes consumed by the tensor-core GEMM.
//
// ref: __main__.py:148-163 (_per_token_fp8, _fp8_e4m3_to_int32, _per_token_fp8_int32).
//   scale = max(amax_k |x[m,k]| * RN(1/448), 1e-12)   fp32 (see qz_row_scale)
//   q     = e4m3_rne(float(x) / scale)           fp32, IEEE division, torch's e4m3fn cast
//   code  = round(q * 512)                       exact integer, |code| <= 229376
//
// Digit planes.  The GEMM multiplies int8 operands, so each integer operand value v
// is written in balanced base-128 digits v = sum_i 2^(7 i) d_i, one int8 plane per digit.
// Scheme DIGITS3 (|v| <= 1,064,960, which covers every codebook value): three planes
// d0, d1 in [-64, 63], d2.  Scheme DIGITS5 (any int32): five planes.
#include "ima_common.cuh"
#include "hawkeye_layout.cuh"

namespace {

IMA_DEVINL float load_as_f32(const void* x, int dtype, int64_t idx) {
    if (dtype == IMA_DTYPE_BF16) return ima_bf16_to_f32(reinterpret_cast<const uint16_t*>(x)[idx]);
    if (dtype == IMA_DTYPE_F16) return __half2float(reinterpret_cast<const __half*>(x)[idx]);
    return reinterpret_cast<const float*>(x)[idx];
}

// The three digit planes of a codebook value.
IMA_DEVINL void digits3_planes(int32_t v, int32_t p[3]) { ima_digits3(v, p[0], p[1], p[2]); }

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

// Eight consecutive elements of a row as fp32 (zeros beyond K); one or two 16-byte
// loads when the row and the chunk are 16-byte aligned.
IMA_DEVINL void load8(const void* row, int dtype, int64_t k0, int64_t K, bool vec, float v[8]) {
    if (vec && k0 + 8 <= K) {
        if (dtype == IMA_DTYPE_F32) {
            const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(row) + k0);
            float4 a = __ldg(p), b = __ldg(p + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
            uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(row) + k0));
            uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint16_t lo = (uint16_t)(w[j] & 0xFFFFu), hi = (uint16_t)(w[j] >> 16);
                if (dtype == IMA_DTYPE_BF16) {
                    v[2 * j] = ima_bf16_to_f32(lo);
                    v[2 * j + 1] = ima_bf16_to_f32(hi);
                } else {
                    v[2 * j] = __half2float(__ushort_as_half(lo));
                    v[2 * j + 1] = __half2float(__ushort_as_half(hi));
                }
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (k0 + j < K) ? load_as_f32(row, dtype, k0 + j) : 0.0f;
}

// ---------------------------------------------------------------------------
// Fast per-element path for rows whose scale s is finite.
//
// Division.  Markstein's correction (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
// with y = RN(1/s) and q0 = RN(x y), the residual r = x - s q0 is exact and
// RN(q0 + r y) is the correctly rounded quotient RN(x / s).  It is used for bf16 and
// fp16 inputs, whose every (row scale, element) pair ima_quant_fast_selftest checks
// against IEEE division; fp32 inputs keep __fdiv_rn.
//
// e4m3.  The hardware cvt.rn.satfinite.e4m3x2.f32 rounds to nearest even like
// torch's cast; the two differ only for |f| >= 464 (torch gives NaN, satfinite
// clamps) and NaN signs.  With a finite scale |x / s| <= 448.0002, and
// ima_quant_fast_selftest checks the two casts on every fp32 value with |f| < 464.
// Rows with a NaN or infinite scale take the exact reference-shaped path instead.
// ---------------------------------------------------------------------------
// Row scale.  The reference computes `amax / FP8_E4M3_MAX` with the Python float 448.0 on
// CUDA tensors, and torch's CUDA division kernel evaluates a tensor divided by a host scalar
// as the tensor times the scalar's fp32 reciprocal: scale = RN(amax * RN(1/448)), then
// clamp_min(1e-12), which keeps NaN.  (IEEE division amax / 448 gives a different fp32
// value for about a third of the bf16 amax values; torch on the CPU divides.)
constexpr float kQzInv448 = 0x1.24924ap-9f;   // RN(1 / 448) in fp32

IMA_DEVINL float qz_row_scale(float amax) {
    const float s = __fmul_rn(amax, kQzInv448);
    return (s < 1e-12f) ? 1e-12f : s;
}

// (computed on |x| with x's sign restored, so that -0 / s stays -0)
IMA_DEVINL float qz_div(float x, float s, float y) {
    const float ax = fabsf(x);
    const float q0 = __fmul_rn(ax, y);
    const float r = __fmaf_rn(-q0, s, ax);
    const float q = __fmaf_rn(r, y, q0);
    return __uint_as_float(__float_as_uint(q) | (__float_as_uint(x) & 0x80000000u));
}

IMA_DEVINL uint32_t qz_cvt_e4m3x2(float lo, float hi) {
    uint16_t d;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(hi), "f"(lo));
    return d;   // lo in bits 0..7, hi in bits 8..15
}

// round(e4m3 * 512) of a non-NaN e4m3 byte
IMA_DEVINL int32_t qz_codebook(uint32_t b) {
    const uint32_t e = (b >> 3) & 15u, m = b & 7u;
    const int32_t v = (int32_t)((e ? (m | 8u) : m) << (e ? e - 1u : 0u));
    const int32_t sg = -(int32_t)((b >> 7) & 1u);
    return (v ^ sg) - sg;
}

// NaN-propagating max of packed |bf16| / |f16| pairs
IMA_DEVINL uint32_t qz_absmax2(uint32_t acc, uint32_t w, bool bf16) {
    uint32_t a = w & 0x7FFF7FFFu, d;
    if (bf16) asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(acc), "r"(a));
    else asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(d) : "r"(acc), "r"(a));
    return d;
}

IMA_DEVINL float qz_half_to_f32(uint32_t h, bool bf16) {
    return bf16 ? __uint_as_float(h << 16) : __half2float(__ushort_as_half((unsigned short)h));
}

// Eight consecutive 16-bit elements of a row as raw bits (zeros beyond K): one 16-byte
// load when the row is 16-byte aligned and the chunk is whole.
IMA_DEVINL uint4 qz_load_half8(const uint16_t* row, int64_t k0, int64_t K, bool vec) {
    if (vec && k0 + 8 <= K) return __ldg(reinterpret_cast<const uint4*>(row + k0));
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (k0 + j < K) w[j >> 1] |= (uint32_t)__ldg(row + k0 + j) << (16 * (j & 1));
    return make_uint4(w[0], w[1], w[2], w[3]);
}

IMA_DEVINL void qz_unpack_half8(uint4 u, bool bf16, float v[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (bf16) {
            v[2 * j] = __uint_as_float(w[j] << 16);
            v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        } else {
            v[2 * j] = __half2float(__ushort_as_half((unsigned short)(w[j] & 0xFFFFu)));
            v[2 * j + 1] = __half2float(__ushort_as_half((unsigned short)(w[j] >> 16)));
        }
    }
}

// Output pointers of one row, hoisted out of the batch descriptor.
struct QzRow {
    uint8_t* q;          // e4m3 codes
    int32_t* cb;         // codebook values (optional)
    int8_t* pl;          // plane 0 of the row (optional); plane i at pl + i * pstride
    int64_t pstride;
    int64_t K;
    bool qvec;           // q row 8-byte aligned
};

// e4m3 codes of eight columns by the fast path (finite scale, half-precision input).
IMA_DEVINL uint2 qz_codes_fast(const float v[8], float s, float y) {
    float qv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) qv[j] = qz_div(v[j], s, y);
    return make_uint2(qz_cvt_e4m3x2(qv[0], qv[1]) | (qz_cvt_e4m3x2(qv[2], qv[3]) << 16),
                      qz_cvt_e4m3x2(qv[4], qv[5]) | (qz_cvt_e4m3x2(qv[6], qv[7]) << 16));
}

// e4m3 codes of eight columns with IEEE division: fp32 inputs (hardware cast when the
// scale is finite) and rows with a NaN or infinite scale (torch-shaped software cast).
// Columns at or beyond `valid` give code 0.
IMA_DEVINL uint2 qz_codes_ieee(const float v[8], float s, bool finite, int64_t valid) {
    uint32_t qw[2] = {0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float q = __fdiv_rn(v[j], s);
        uint32_t b = finite ? (qz_cvt_e4m3x2(q, 0.0f) & 0xFFu) : ima_f32_to_e4m3(q);
        if (j >= valid) b = 0;
        qw[j >> 2] |= b << (8 * (j & 3));
    }
    return make_uint2(qw[0], qw[1]);
}

// Store the codes of columns k0..k0+7, their codebook values and their digit planes.
// lut[b] packs the three digit bytes of the codebook value of e4m3 byte b; code[b] is
// that value (NaN codes give 0, as in ima_e4m3_codebook).  Columns >= K hold code 0
// (digits 0), which the planes carry up to their zero-filled width.
IMA_DEVINL void qz_emit(const QzRow& R, int64_t k0, uint2 qv, const uint32_t* lut, const int32_t* code) {
    const uint32_t qw[2] = {qv.x, qv.y};
    if (k0 < R.K) {
        if (R.qvec && k0 + 8 <= R.K) {
            *reinterpret_cast<uint2*>(R.q + k0) = qv;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (k0 + j < R.K) R.q[k0 + j] = (uint8_t)(qw[j >> 2] >> (8 * (j & 3)));
        }
        if (R.cb) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (k0 + j < R.K) R.cb[k0 + j] = code[__byte_perm(qw[j >> 2], 0, 0x4440 | (j & 3))];
        }
    }
    if (R.pl) {
        uint32_t L[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) L[j] = lut[__byte_perm(qw[j >> 2], 0, 0x4440 | (j & 3))];
#pragma unroll
        for (int i = 0; i < 3; ++i) {
            const uint32_t sel = (uint32_t)i | ((uint32_t)(4 + i) << 4);   // byte i of x, byte i of y
            const uint32_t w0 = __byte_perm(__byte_perm(L[0], L[1], sel), __byte_perm(L[2], L[3], sel), 0x5410);
            const uint32_t w1 = __byte_perm(__byte_perm(L[4], L[5], sel), __byte_perm(L[6], L[7], sel), 0x5410);
            *reinterpret_cast<uint2*>(R.pl + i * R.pstride + k0) = make_uint2(w0, w1);
        }
    }
}

// One warp per (problem, row), grid-stride over all rows of the batch.  Pass 1: the
// NaN-propagating amax, with four 16-byte loads in flight per lane (packed pairs for
// bf16/fp16); a row of at most 1024 half-precision elements stays in registers for
// pass 2, longer rows are re-read from L2.  Pass 2 quantises eight consecutive columns
// per lane and chunk, so the code store is 8 bytes and each plane store one 8-byte word.
__global__ void __launch_bounds__(256, 3) quantize_rows_kernel(const __grid_constant__ QuantBatch batch) {
    __shared__ uint32_t s_lut[256];
    __shared__ int32_t s_code[256];
    {
        const uint32_t b = threadIdx.x;   // blockDim.x == 256
        const int32_t c = ima_e4m3_codebook(b);
        const int32_t u = c + 8256;       // digits of u are (d0 + 64, d1 + 64, d2)
        s_code[b] = c;
        s_lut[b] = ((uint32_t)((u & 127) - 64) & 0xFFu) | (((uint32_t)(((u >> 7) & 127) - 64) & 0xFFu) << 8) |
                   (((uint32_t)(u >> 14) & 0xFFu) << 16);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warps_total = (int64_t)gridDim.x * 8;
    for (int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); g < batch.total_rows; g += warps_total) {
        int lo = 0, hi = batch.n - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (batch.p[mid].row_start <= g) lo = mid; else hi = mid - 1;
        }
        const QuantProblem& P = batch.p[lo];
        const int64_t m = g - P.row_start;
        const int dtype = P.dtype;
        const int64_t K = P.K;
        const bool half = dtype != IMA_DTYPE_F32, bf16 = dtype == IMA_DTYPE_BF16;
        const unsigned char* row = reinterpret_cast<const unsigned char*>(P.x) + m * P.ldx * (half ? 2 : 4);
        const uint16_t* hrow = reinterpret_cast<const uint16_t*>(row);
        const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
        const bool qvec = ((reinterpret_cast<uintptr_t>(P.q + m * P.ldq) & 7) == 0);
        const bool resident = half && K <= 1024;

        // ---- pass 1: amax ----
        float amax = 0.0f;
        int has_nan = 0;
        uint4 keep[4];
        if (half) {
            uint32_t mx2 = 0;
            for (int64_t base = (int64_t)lane * 8; base < K; base += 1024) {
                uint4 u[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) u[t] = qz_load_half8(hrow, base + t * 256, K, vec);
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    mx2 = qz_absmax2(mx2, u[t].x, bf16);
                    mx2 = qz_absmax2(mx2, u[t].y, bf16);
                    mx2 = qz_absmax2(mx2, u[t].z, bf16);
                    mx2 = qz_absmax2(mx2, u[t].w, bf16);
                    keep[t] = u[t];
                }
            }
            const float a0 = qz_half_to_f32(mx2 & 0xFFFFu, bf16), a1 = qz_half_to_f32(mx2 >> 16, bf16);
            has_nan = (a0 != a0) || (a1 != a1);
            amax = fmaxf(a0, a1);
        } else {
            for (int64_t k0 = (int64_t)lane * 8; k0 < K; k0 += 256) {
                float v[8];
                load8(row, dtype, k0, K, vec, v);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float a = fabsf(v[j]);
                    if (a != a) has_nan = 1;
                    else amax = fmaxf(amax, a);
                }
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
            has_nan |= __shfl_xor_sync(0xFFFFFFFFu, has_nan, o);
        }
        const float s = qz_row_scale(has_nan ? __int_as_float(0x7FC00000) : amax);
        if (lane == 0) {
            P.scale[m] = s;
            if (P.code_scale) P.code_scale[m] = __fdiv_rn(s, 512.0f);
        }
        const bool finite = fabsf(s) <= 3.402823466e38f;   // false for NaN and inf
        const bool markstein = finite && half;
        const float y = __frcp_rn(s);

        // ---- pass 2: codes, codebook values, digit planes (planes zero-filled to ldp) ----
        QzRow R;
        R.q = P.q + m * P.ldq;
        R.cb = P.codebook ? P.codebook + m * P.ldc : nullptr;
        R.pl = P.planes ? P.planes + m * P.ldp : nullptr;
        R.pstride = P.M * P.ldp;
        R.K = K;
        R.qvec = qvec;
        const int64_t kq = P.planes ? P.ldp : K;
        if (markstein) {   // finite scale, half-precision input: the fast path
            for (int64_t base = (int64_t)lane * 8; base < kq; base += 1024) {
                uint4 u[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) u[t] = resident ? keep[t] : qz_load_half8(hrow, base + t * 256, K, vec);
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int64_t k0 = base + t * 256;
                    if (k0 >= kq) break;
                    float v[8];
                    qz_unpack_half8(u[t], bf16, v);
                    qz_emit(R, k0, qz_codes_fast(v, s, y), s_lut, s_code);
                }
            }
        } else {           // fp32 input, or a NaN / infinite scale: IEEE division per element
#pragma unroll 1
            for (int64_t k0 = (int64_t)lane * 8; k0 < kq; k0 += 256) {
                float v[8];
                load8(row, dtype, k0, K, vec, v);
                qz_emit(R, k0, qz_codes_ieee(v, s, finite, K - k0), s_lut, s_code);
            }
        }
    }
}

// Per-token quantisation fused with the Hawkeye operand staging (ima_hawkeye_quantize_prepare):
// the row scale and the e4m3 codes exactly as quantize_rows_kernel computes them (the same
// amax, scale, division and cast functions), written straight into the [k][row] records the
// replay reads (the blocks of hawkeye_layout.cuh: per k the record {|s| 2^e as fp32 bits, sign
// mask}, per group the exponent powers and the sign word), and optionally the codes.
// A block covers 32 rows.  Phase 1: 8 warps x 4 rows, the NaN-propagating amax and the scale.
// Phase 2: thread (row = lane, warp) takes groups warp, warp + 8, ...: 32 elements -> 32 codes
// -> records; for each k the 32 rows of a thread block form one contiguous 256-byte store.
constexpr int HQ_GROUP = HK_GROUP;

__global__ void __launch_bounds__(256) hawkeye_quant_stage_kernel(const void* __restrict__ x, int dtype, int64_t M,
                                                                  int64_t K, int64_t ldx, float* __restrict__ scale,
                                                                  uint8_t* __restrict__ q, int64_t ldq, int64_t pitch,
                                                                  int64_t groups, unsigned char* __restrict__ op) {
    __shared__ float s_s[32], s_y[32];
    __shared__ int s_mode[32];   // 1: fast path (finite scale, half input); 2: IEEE, finite scale; 0: IEEE, NaN/inf
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = (int64_t)blockIdx.x * 32;
    const bool half = dtype != IMA_DTYPE_F32, bf16 = dtype == IMA_DTYPE_BF16;
    const int esz = half ? 2 : 4;
    // ---- phase 1: row scales ----
    for (int i = 0; i < 4; ++i) {
        const int rl = warp * 4 + i;
        const int64_t m = r0 + rl;
        float amax = 0.0f;
        int has_nan = 0;
        if (m < M) {
            const unsigned char* row = reinterpret_cast<const unsigned char*>(x) + m * ldx * esz;
            const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
            if (half) {
                uint32_t mx2 = 0;
                const uint16_t* hrow = reinterpret_cast<const uint16_t*>(row);
                for (int64_t k0 = (int64_t)lane * 8; k0 < K; k0 += 256) {
                    const uint4 u = qz_load_half8(hrow, k0, K, vec);
                    mx2 = qz_absmax2(mx2, u.x, bf16);
                    mx2 = qz_absmax2(mx2, u.y, bf16);
                    mx2 = qz_absmax2(mx2, u.z, bf16);
                    mx2 = qz_absmax2(mx2, u.w, bf16);
                }
                const float a0 = qz_half_to_f32(mx2 & 0xFFFFu, bf16), a1 = qz_half_to_f32(mx2 >> 16, bf16);
                has_nan = (a0 != a0) || (a1 != a1);
                amax = fmaxf(a0, a1);
            } else {
                for (int64_t k0 = (int64_t)lane * 8; k0 < K; k0 += 256) {
                    float v[8];
                    load8(row, dtype, k0, K, vec, v);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float a = fabsf(v[j]);
                        if (a != a) has_nan = 1;
                        else amax = fmaxf(amax, a);
                    }
                }
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
            has_nan |= __shfl_xor_sync(0xFFFFFFFFu, has_nan, o);
        }
        if (lane == 0) {
            const float sc = qz_row_scale(has_nan ? __int_as_float(0x7FC00000) : amax);
            const bool finite = fabsf(sc) <= 3.402823466e38f;
            s_s[rl] = sc;
            s_y[rl] = __frcp_rn(sc);
            s_mode[rl] = (finite && half) ? 1 : (finite ? 2 : 0);
            if (m < M) scale[m] = sc;
        }
    }
    __syncthreads();
    // ---- phase 2: codes and staged records ----
    const int64_t m = r0 + lane;
    const bool live = m < M;
    const float sc = s_s[lane], y = s_y[lane];
    const int mode = s_mode[lane];
    const unsigned char* row = reinterpret_cast<const unsigned char*>(x) + (live ? m : 0) * ldx * esz;
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
    for (int64_t g = warp; g < groups; g += 8) {
        uint32_t codes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (live) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int64_t k0 = g * HQ_GROUP + c * 8;
                if (k0 >= K) break;
                float v[8];
                uint2 qv;
                if (mode == 1) {
                    qz_unpack_half8(qz_load_half8(reinterpret_cast<const uint16_t*>(row), k0, K, vec), bf16, v);
                    qv = qz_codes_fast(v, sc, y);   // columns beyond K load as +0: code 0
                } else {
                    load8(row, dtype, k0, K, vec, v);
                    qv = qz_codes_ieee(v, sc, mode == 2, K - k0);
                }
                codes[2 * c] = qv.x;
                codes[2 * c + 1] = qv.y;
            }
            if (q) {
                uint8_t* qrow = q + m * ldq + g * HQ_GROUP;
                const int64_t valid = K - g * HQ_GROUP;
                if (valid >= HQ_GROUP && (reinterpret_cast<uintptr_t>(qrow) & 15) == 0) {
                    reinterpret_cast<uint4*>(qrow)[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
                    reinterpret_cast<uint4*>(qrow)[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
                } else {
                    for (int j = 0; j < HQ_GROUP && j < valid; ++j) qrow[j] = (uint8_t)(codes[j >> 2] >> (8 * (j & 3)));
                }
            }
        }
        // the replay's operand records, element by element as ima_hawkeye_prepare writes them
        uint32_t signs = 0, pw[16];
        uint2 rec[HQ_GROUP];
#pragma unroll
        for (int j = 0; j < HQ_GROUP; ++j) {
            const int64_t k = g * HQ_GROUP + j;
            const bool valid = live && k < K;
            const uint32_t b = valid ? (codes[j >> 2] >> (8 * (j & 3))) & 0xFFu : 0u;
            const uint32_t e_bits = (b >> 3) & 15u, mant = b & 7u;
            const uint32_t sig = e_bits ? (mant | 8u) : mant;
            const int e = e_bits ? (int)e_bits : 1;
            const float mag = valid ? (float)sig * (float)(1u << e) : 0.0f;
            const uint32_t mask = (valid && (b & 0x80u)) ? 0xFFFFFFFFu : 0u;
            signs |= (mask & 1u) << j;
            rec[j] = make_uint2(__float_as_uint(mag), mask);
            const uint32_t p = hk_pow_bits(valid && sig != 0, e);
            if (j & 1) pw[j >> 1] |= p << 16;
            else pw[j >> 1] = p;
        }
        hk_store_row(op, g, m, pitch, rec, pw, signs);
    }
}

// Self-test of the fast path (no reference counterpart; run by the GPU tests).
//   kind 0: every fp32 value |f| < 464: hardware cvt vs ima_f32_to_e4m3
//   kind 1 / 2: every positive finite bf16 (1) / fp16 (2) amax and every element x of
//     that type with |x| <= amax (the pairs a row can hold): the e4m3 code of the fast
//     quotient vs ima_f32_to_e4m3(__fdiv_rn(x, s)), with the kernel's own scale formula
//   kind 3 / 4: the same pairs, the fp32 quotient itself vs __fdiv_rn wherever the
//     theorem's no-underflow condition holds: a normal quotient and |x| >= 2^-100, so
//     that the residual x - s q0 (about |x| 2^-24) is a normal number.  Below that the
//     quotients are many binades under the e4m3 range, where kinds 1 / 2 cover them.
__global__ void quant_fast_selftest_kernel(int kind, unsigned long long* __restrict__ mismatches) {
    unsigned long long bad = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    if (kind == 0) {
        for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32); i += stride) {
            const float f = __uint_as_float((uint32_t)i);
            if (!(fabsf(f) < 464.0f)) continue;
            const uint32_t hw = qz_cvt_e4m3x2(f, 0.0f) & 0xFFu;
            if (hw != ima_f32_to_e4m3(f)) ++bad;
        }
    } else {
        const bool bf16 = kind == 1 || kind == 3, codes = kind <= 2;
        for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 31); i += stride) {
            const uint32_t ha = (uint32_t)(i >> 16) & 0x7FFFu, hx = (uint32_t)i & 0xFFFFu;
            const float amax = qz_half_to_f32(ha, bf16), x = qz_half_to_f32(hx, bf16);
            if (!(amax > 0.0f) || !(amax <= 3.402823466e38f) || !(fabsf(x) <= amax)) continue;
            const float s = qz_row_scale(amax);
            const float y = __frcp_rn(s);
            const float fast = qz_div(x, s, y), ieee = __fdiv_rn(x, s);
            if (codes) {
                if ((qz_cvt_e4m3x2(fast, 0.0f) & 0xFFu) != ima_f32_to_e4m3(ieee)) ++bad;
            } else if (fabsf(x) >= 0x1p-100f && fabsf(ieee) >= 1.17549435e-38f &&
                       __float_as_uint(fast) != __float_as_uint(ieee)) {
                ++bad;
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xFFFFFFFFu, bad, o);
    if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

// Planes of an e4m3 matrix (weights): one thread per 4 consecutive columns.
__global__ void planes_from_fp8_kernel(const uint8_t* __restrict__ src, int64_t rows, int64_t K, int64_t ld,
                                       int8_t* __restrict__ planes, int64_t ldp, int32_t* __restrict__ codebook_t) {
    int64_t words = ldp / 4;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * words) return;
    int64_t r = idx / words, k0 = (idx % words) * 4;
    uint32_t word[3] = {0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        int64_t k = k0 + j;
        if (k >= K) break;
        int32_t v = ima_e4m3_codebook(src[r * ld + k]);
        if (codebook_t) codebook_t[k * rows + r] = v;
        int32_t p[3];
        digits3_planes(v, p);
#pragma unroll
        for (int i = 0; i < 3; ++i) word[i] |= ((uint32_t)p[i] & 0xFFu) << (8 * j);
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) *reinterpret_cast<uint32_t*>(planes + ((int64_t)i * rows + r) * ldp + k0) = word[i];
}

// Planes of a strided int32 matrix.
__global__ void planes_from_int32_kernel(const int32_t* __restrict__ src, int64_t rows, int64_t K,
                                         int64_t stride_row, int64_t stride_k, int scheme,
                                         int8_t* __restrict__ planes, int64_t ldp) {
    int64_t words = ldp / 4;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * words) return;
    int64_t r = idx / words, k0 = (idx % words) * 4;
    uint32_t word[5] = {0, 0, 0, 0, 0};
    int np = scheme == IMA_SCHEME_DIGITS3 ? 3 : 5;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        int64_t k = k0 + j;
        if (k >= K) break;
        int32_t v = src[r * stride_row + k * stride_k];
        int32_t p[5] = {0, 0, 0, 0, 0};
        if (scheme == IMA_SCHEME_DIGITS3) {
            if (v > 1064960 || v < -1064960) ima_record_error(IMA_ERR_OVERFLOW, IMA_WHERE_PLANES, 0);
            digits3_planes(v, p);
        } else {
            digits5(v, p);
        }
#pragma unroll
        for (int i = 0; i < 5; ++i) word[i] |= ((uint32_t)p[i] & 0xFFu) << (8 * j);
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

int ima_quant_fast_selftest(int kind, unsigned long long* mismatches, void* stream) {
    if (kind < 0 || kind > 4 || !mismatches) return IMA_ERR_INVALID_ARGUMENT;
    quant_fast_selftest_kernel<<<148 * 16, 256, 0, (cudaStream_t)stream>>>(kind, mismatches);
    return IMA_LAUNCH_STATUS();
}

int ima_scheme_planes(int scheme) {
    return scheme == IMA_SCHEME_DIGITS3 ? 3 : (scheme == IMA_SCHEME_DIGITS5 ? 5 : 0);
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
    int64_t grid = (b.total_rows + 7) / 8;   // one warp per row, 8 warps per block
    if (grid > 148 * 32) grid = 148 * 32;
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

int ima_hawkeye_quantize_prepare(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, float* scale,
                                 uint8_t* q_fp8, int64_t ldq, void* operand, void* stream) {
    if (!x || !scale || !operand || M < 0 || K < 0 || ldx < K) return IMA_ERR_INVALID_ARGUMENT;
    if (x_dtype != IMA_DTYPE_F32 && x_dtype != IMA_DTYPE_BF16 && x_dtype != IMA_DTYPE_F16) return IMA_ERR_INVALID_ARGUMENT;
    if (q_fp8 && ldq < K) return IMA_ERR_INVALID_ARGUMENT;
    const int64_t pitch = ima_hawkeye_operand_pitch(M), groups = (K + HQ_GROUP - 1) / HQ_GROUP;
    if (pitch == 0 || groups == 0) return IMA_OK;
    if (pitch / 32 > INT32_MAX) return IMA_ERR_UNSUPPORTED;
    hawkeye_quant_stage_kernel<<<(unsigned)(pitch / 32), 256, 0, (cudaStream_t)stream>>>(
        x, x_dtype, M, K, ldx, scale, q_fp8, ldq, pitch, groups, reinterpret_cast<unsigned char*>(operand));
    return IMA_LAUNCH_STATUS();
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
    if (scheme != IMA_SCHEME_DIGITS3 && scheme != IMA_SCHEME_DIGITS5) return IMA_ERR_UNSUPPORTED;
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
