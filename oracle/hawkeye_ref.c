/*
 * CPU oracle (test infrastructure only; never part of the product path).
 *
 * Scalar C restatement of int-model-approximation's student-linear arithmetic,
 * used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg to
 * check the CUDA kernels.  Every function follows the reference literally, with
 * int64 arithmetic and the reference's own clamps, rather than the algebraic
 * shortcuts the CUDA kernels take:
 *
 *   oracle_hawkeye          hawkeye.py:127-219 (_hawkeye_fp8_sum_kernel) with the
 *                           helpers hawkeye.py:27-123 and their int64 twins in
 *                           hawkeye_freivalds.py:39-144; returns the fp32 value
 *                           (gfloat * x_scale) * w_scale, before the bf16 store.
 *   oracle_int_gemm         __main__.py:188-225 (_int32_raw_matmul_kernel):
 *                           int32 x int32 -> int64, row-major a [M,K], b [K,N].
 *   oracle_int_gemm_nk      the same product with b given as [N,K] (the weight's
 *                           own layout, i.e. weight_t transposed).
 *
 * Paths are relative to the reference project's src/int_model_approximation/.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define FP32_SIGNIFICAND_WIDTH 24
#define FP32_MIN_NONZERO_EXPONENT (-126)

/* hawkeye.py:27-37 / hawkeye_freivalds.py:39-48 */
static inline void decode_e4m3(uint8_t raw, int64_t *exp_eff, int64_t *signed_sig, int *nonzero) {
    int64_t sign = (raw >> 7) & 1;
    int64_t exp_bits = (raw >> 3) & 15;
    int64_t mant = raw & 7;
    int64_t sig_abs = exp_bits != 0 ? (mant | 8) : mant;
    *exp_eff = exp_bits != 0 ? exp_bits : 1;
    *signed_sig = sign ? -sig_abs : sig_abs;
    *nonzero = sig_abs != 0;
}

static inline int64_t i64abs(int64_t x) { return x < 0 ? -x : x; }

/* torch.bitwise_right_shift on int64 saturates shifts >= 64 to the sign fill */
static inline int64_t shr64(int64_t x, int64_t s) {
    if (s >= 63) return x < 0 ? -1 : 0;
    return x >> s;
}
static inline int64_t shl64(int64_t x, int64_t s) {
    if (s >= 64) return 0;
    return (int64_t)((uint64_t)x << s);
}

/* hawkeye_freivalds.py:60-63 (the Triton twin hawkeye.py:48-52 also clamps to 62) */
static inline int64_t shift_right_towards_zero(int64_t x, int64_t shift) {
    if (shift < 0) shift = 0;
    if (shift > 62) shift = 62;
    int64_t mag = i64abs(x) >> shift;
    return x < 0 ? -mag : mag;
}

/* hawkeye_freivalds.py:66-70 */
static inline int64_t scale_to_internal(int64_t x, int internal_width) {
    int shift = internal_width - 7;
    if (shift >= 0) return shl64(x, shift);
    return shift_right_towards_zero(x, -shift);
}

/* hawkeye_freivalds.py:73-76 */
static inline int64_t accumulator_base(int64_t acc_sig, int internal_width) {
    if (internal_width < FP32_SIGNIFICAND_WIDTH) return acc_sig >> (FP32_SIGNIFICAND_WIDTH - internal_width);
    return shl64(acc_sig, internal_width - FP32_SIGNIFICAND_WIDTH);
}

/* hawkeye_freivalds.py:79-117 */
static inline void normalize_total(int64_t total, int64_t max_exp, int internal_width, int zero_exponent,
                                   int *out_sign, int64_t *out_exp, int64_t *out_sig) {
    int sign = total < 0;
    int64_t magnitude = i64abs(total);
    int nonzero = magnitude != 0;
    int64_t width = 0;
    for (int bit = 0; bit < 63; ++bit)
        if (magnitude >= ((int64_t)1 << bit)) width = bit + 1;
    int64_t exp = max_exp + width - internal_width;
    int64_t right = width - internal_width; if (right < 0) right = 0;
    int64_t left = internal_width - width; if (left < 0) left = 0;
    int64_t sig = width > internal_width ? shr64(magnitude, right) : shl64(magnitude, left);
    int64_t sub = FP32_MIN_NONZERO_EXPONENT - exp; if (sub < 0) sub = 0;
    if (exp < FP32_MIN_NONZERO_EXPONENT) sig = shr64(sig, sub);
    if (exp < FP32_MIN_NONZERO_EXPONENT) exp = FP32_MIN_NONZERO_EXPONENT;
    if (internal_width < FP32_SIGNIFICAND_WIDTH) sig = shl64(sig, FP32_SIGNIFICAND_WIDTH - internal_width);
    else sig = shr64(sig, internal_width - FP32_SIGNIFICAND_WIDTH);
    if (!(nonzero && sig != 0)) sig = 0;
    *out_sig = sig;
    *out_exp = sig != 0 ? exp : zero_exponent;
    *out_sign = sig != 0 ? sign : 0;
}

/* hawkeye_freivalds.py:120-144 */
static inline float gfloat_to_float32(int sign, int64_t exponent, int64_t significand) {
    int64_t exponent_bits = exponent + 127;
    int leading_bit_missing = (significand & 0x800000) == 0;
    if (leading_bit_missing && significand != 0) exponent_bits -= 1;
    if (exponent_bits < 0) exponent_bits = 0;
    if (exponent_bits > 254) exponent_bits = 254;
    int64_t mantissa = significand & 0x7FFFFF;
    int64_t bits = ((int64_t)sign << 31) | (exponent_bits << 23) | mantissa;
    if (significand == 0) bits = 0;
    uint32_t b32 = (uint32_t)(int32_t)bits;
    float f;
    memcpy(&f, &b32, 4);
    return f;
}

typedef struct { int8_t exp_eff; int8_t signed_sig; uint8_t nonzero; } decoded_t;

static decoded_t *decode_all(const uint8_t *raw, size_t n) {
    decoded_t *d = (decoded_t *)malloc(sizeof(decoded_t) * (n ? n : 1));
    for (size_t i = 0; i < n; ++i) {
        int64_t e, s;
        int nz;
        decode_e4m3(raw[i], &e, &s, &nz);
        d[i].exp_eff = (int8_t)e;
        d[i].signed_sig = (int8_t)s;
        d[i].nonzero = (uint8_t)nz;
    }
    return d;
}

/*
 * Direct Hawkeye replay of one output element (hawkeye.py:142-214 for a single
 * (m, n)): a and b are the decoded K-vectors of row m of x and row n of w.
 * Returns the fp32 gfloat before scaling.
 */
static float hawkeye_one(const decoded_t *a, const decoded_t *b, int K, int products_per_group,
                         int internal_width, int zero_exponent) {
    int acc_sign = 0;
    int64_t acc_exp = zero_exponent, acc_sig = 0;
    for (int k0 = 0; k0 < K; k0 += products_per_group) {
        int k1 = k0 + products_per_group < K ? k0 + products_per_group : K;
        int64_t acc_exp_eff = acc_sig != 0 ? acc_exp : zero_exponent;
        int64_t max_exp = acc_exp_eff;
        for (int k = k0; k < k1; ++k) {
            if (!(a[k].nonzero && b[k].nonzero)) continue;
            int64_t pe = (int64_t)a[k].exp_eff + b[k].exp_eff - 14;
            if (pe > max_exp) max_exp = pe;
        }
        int64_t contribution = 0;
        for (int k = k0; k < k1; ++k) {
            if (!(a[k].nonzero && b[k].nonzero)) continue;
            int64_t pe = (int64_t)a[k].exp_eff + b[k].exp_eff - 14;
            int64_t scaled = scale_to_internal((int64_t)a[k].signed_sig * b[k].signed_sig, internal_width);
            contribution += shift_right_towards_zero(scaled, max_exp - pe);
        }
        int64_t acc_base = accumulator_base(acc_sig, internal_width);
        int64_t sh = max_exp - acc_exp_eff;
        if (sh < 0) sh = 0;
        if (sh > 62) sh = 62;
        int64_t aligned = acc_base >> sh;
        if (acc_sign) aligned = -aligned;
        normalize_total(aligned + contribution, max_exp, internal_width, zero_exponent, &acc_sign, &acc_exp,
                        &acc_sig);
    }
    return gfloat_to_float32(acc_sign, acc_exp, acc_sig);
}

/*
 * Direct Hawkeye replay (hawkeye.py:127-219).
 * x: [M,K] e4m3 bytes, w: [N,K] e4m3 bytes, x_scale [M], w_scale [N];
 * rows: optional list of n_rows output rows to compute (NULL = all M rows);
 * out: [n_rows or M, N] fp32 = (gfloat * x_scale[m]) * w_scale[n] (hawkeye.py:211-214).
 */
void oracle_hawkeye(const uint8_t *x, const float *x_scale, const uint8_t *w, const float *w_scale, int M,
                    int N, int K, int products_per_group, int internal_width, int zero_exponent,
                    const int64_t *rows, int n_rows, float *out) {
    if (!rows) n_rows = M;
    decoded_t *wd = decode_all(w, (size_t)N * K);
    for (int i = 0; i < n_rows; ++i) {
        int m = rows ? (int)rows[i] : i;
        decoded_t *ad = decode_all(x + (size_t)m * K, (size_t)K);
        for (int n = 0; n < N; ++n) {
            float g = hawkeye_one(ad, wd + (size_t)n * K, K, products_per_group, internal_width, zero_exponent);
            volatile float t = g * x_scale[m];
            out[(size_t)i * N + n] = t * w_scale[n];
        }
        free(ad);
    }
    free(wd);
}

/* __main__.py:188-225: C[m,n] = sum_k a[m,k] * b[k,n] in int64 (wrapping like the GPU). */
void oracle_int_gemm(const int32_t *a, const int32_t *b, int M, int N, int K, int64_t *c) {
    for (int m = 0; m < M; ++m) {
        uint64_t *row = (uint64_t *)(c + (size_t)m * N);
        for (int n = 0; n < N; ++n) row[n] = 0;
        for (int k = 0; k < K; ++k) {
            uint64_t av = (uint64_t)(int64_t)a[(size_t)m * K + k];
            const int32_t *brow = b + (size_t)k * N;
            for (int n = 0; n < N; ++n) row[n] += av * (uint64_t)(int64_t)brow[n];
        }
    }
}

/* Same product with the second operand stored [N,K]. */
void oracle_int_gemm_nk(const int32_t *a, const int32_t *bnk, int M, int N, int K, int64_t *c) {
    for (int m = 0; m < M; ++m) {
        const int32_t *arow = a + (size_t)m * K;
        for (int n = 0; n < N; ++n) {
            const int32_t *brow = bnk + (size_t)n * K;
            uint64_t s = 0;
            for (int k = 0; k < K; ++k) s += (uint64_t)(int64_t)arow[k] * (uint64_t)(int64_t)brow[k];
            c[(size_t)m * N + n] = (int64_t)s;
        }
    }
}

/* hawkeye_freivalds.py:120-144 over arrays (for the gfloat known-answer checks). */
void oracle_gfloat_to_float32(const int32_t *sign, const int64_t *exponent, const int64_t *significand, int n,
                              float *out) {
    for (int i = 0; i < n; ++i) out[i] = gfloat_to_float32(sign[i], exponent[i], significand[i]);
}
