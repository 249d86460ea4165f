/*
 * ima_b200.h -- C ABI of the B200-native student-linear hot path of
 * int-model-approximation (codebook exact int GEMM, direct Hawkeye replay,
 * Hawkeye class-count products, Freivalds check).
 *
 * Conventions
 *   - Plain device pointers, 64-bit sizes and leading dimensions in ELEMENTS,
 *     and a cudaStream_t passed as void*.  No framework types.
 *   - Every entry point returns an int status (IMA_OK == 0).  Argument checks
 *     happen before any launch; kernels never trap: a device-side failure (a
 *     bounded wait that ran out, an index outside a tensor) is recorded in a
 *     per-device status word read by ima_device_status().
 *   - Launches are asynchronous on the given stream; no entry point
 *     synchronises unless its comment says so.
 *   - "ref:" cites the reference interface each entry point replaces, as
 *     path:line inside the reference package src/int_model_approximation/.
 */
#ifndef IMA_B200_H
#define IMA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------- */
#define IMA_OK 0
#define IMA_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, bad leading dim */
#define IMA_ERR_UNSUPPORTED 2      /* parameter value the B200 kernels do not implement */
#define IMA_ERR_CUDA 3             /* a CUDA runtime call or launch failed */
#define IMA_ERR_TIMEOUT 4          /* device: a bounded wait ran out */
#define IMA_ERR_DEVICE_BOUNDS 5    /* device: an index fell outside a tensor */
#define IMA_ERR_OVERFLOW 6         /* operand magnitude outside the exact range of the scheme */

/* element types for untyped buffers */
#define IMA_DTYPE_F32 0
#define IMA_DTYPE_BF16 1
#define IMA_DTYPE_F16 2

/* ---- runtime -------------------------------------------------------------- */
int ima_abi_version(void);                 /* bumped on any signature change */
const char* ima_status_string(int status); /* static string, never NULL */
int ima_last_cuda_error(void);             /* cudaError_t of the last failing CUDA call (this thread) */
/* sizeof of the batch descriptor structs below, in declaration order (quantize, gemm,
 * freivalds rows), so that foreign-language bindings can check their layouts. */
int ima_struct_sizes(int64_t* out, int n);
/* Diagnostic for the integer-ALU roofline: `blocks` x 256 threads each run `iters`
 * iterations of 8 interleaved 2-instruction integer chains (XOR + ADD), i.e.
 * blocks * 256 * iters * 16 integer instructions; time it with events on `stream`. */
int ima_int32_issue_probe(int64_t iters, int blocks, uint32_t* sink, void* stream);
/* Self-test of the quantiser's fast path (no reference counterpart).  Adds to
 * *mismatches (device memory, zeroed by the caller) the number of disagreements:
 * kind 0 - the hardware e4m3 cast vs the torch-shaped software cast on every fp32
 * value with |f| < 464; kind 1 / 2 - for every positive finite bf16 / fp16 amax
 * (s = max(amax * RN(1/448), 1e-12)) and every bf16 / fp16 element x with |x| <= amax, the e4m3
 * code of the corrected-reciprocal quotient vs the code of the IEEE quotient x / s;
 * kind 3 / 4 - the same pairs, the fp32 quotients themselves wherever x / s is a normal
 * number and |x| >= 2^-100 (no underflow in the correction step).  A correct build
 * reports 0 for every kind. */
int ima_quant_fast_selftest(int kind, unsigned long long* mismatches, void* stream);

/* Reads (synchronously: waits for the device) and optionally clears the device status
 * word of `device`.  code == IMA_OK when no kernel recorded a failure. */
int ima_device_status(int device, int* code, int* where, int* detail, int clear);

/* ---- multi-GPU plumbing (no reference counterpart) -----------------------------
 * Collectives on the copy engines: a process allocates a device buffer it shares with
 * the other processes of the node (ima_ipc_alloc returns the pointer and an opaque handle
 * of ima_ipc_handle_bytes() bytes to send to them), a peer maps it with ima_ipc_open, and
 * ima_copy_async copies into it (peer to peer over NVLink, no kernel: it uses no SM).
 * ima_ipc_close unmaps a peer's buffer, ima_ipc_free releases one's own. */
int ima_ipc_handle_bytes(void);
int ima_ipc_alloc(int64_t bytes, void** ptr, void* handle);
int ima_ipc_free(void* ptr);
int ima_ipc_open(const void* handle, void** ptr);
int ima_ipc_close(void* ptr);
int ima_copy_async(void* dst, const void* src, int64_t bytes, void* stream);
/* Up to IMA_COPY_MAX copies in one kernel launch on at most `ctas` thread blocks (512
 * threads each): the SM-driven counterpart of ima_copy_async for a multi-GPU caller that
 * keeps a few SMs free of its persistent GEMM (ima_set_gemm_sm_limit) and gathers through
 * them.  Every warp store is 512 contiguous bytes.  dst and src of every copy must be
 * 16-byte aligned (IMA_ERR_INVALID_ARGUMENT otherwise); the copies must not overlap. */
#define IMA_COPY_MAX 128
typedef struct ima_copy_desc {
    void* dst;
    const void* src;
    int64_t bytes;
} ima_copy_desc;
int ima_copy_many(const ima_copy_desc* copies, int count, int ctas, void* stream);

/* ---- A1/A2: per-token FP8 quantiser -----------------------------------------
 * ref: __main__.py:148-154 _per_token_fp8, :157-158 _fp8_e4m3_to_int32,
 *      :161-163 _per_token_fp8_int32.
 * x [M,K] (dtype IMA_DTYPE_*, row stride ldx) ->
 *   q_fp8 [M,K] e4m3 bytes (row stride ldq),
 *   scale [M] fp32 = max(amax_row|x| * RN(1/448), 1e-12): the reference's amax / 448.0 as
 *     torch evaluates it on CUDA tensors (multiplication by the fp32 reciprocal),
 *   codebook [M,K] int32 = round(q * 512) (optional, row stride ldc),
 *   code_scale [M] fp32 = scale / 512 (optional),
 *   planes [3][M][ldp] int8: the three balanced base-128 digit planes of the codebook
 *   values (scheme IMA_SCHEME_DIGITS3) used by ima_int_gemm (optional; ldp >= K,
 *   multiple of 16; columns K..ldp-1 are written as zero). */
int ima_quantize_per_token(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, uint8_t* q_fp8,
                           int64_t ldq, float* scale, int32_t* codebook, int64_t ldc, float* code_scale,
                           int8_t* planes, int64_t ldp, void* stream);

/* The same quantiser for many independent activation matrices in one launch (e.g. every
 * linear of a model); fields mean what the arguments of ima_quantize_per_token mean. */
typedef struct ima_quantize_problem {
    const void* x;
    int32_t x_dtype;
    int64_t M, K, ldx;
    uint8_t* q_fp8;
    int64_t ldq;
    float* scale;
    int32_t* codebook;
    int64_t ldc;
    float* code_scale;
    int8_t* planes;
    int64_t ldp;
} ima_quantize_problem;
int ima_quantize_grouped(const ima_quantize_problem* problems, int count, void* stream);

/* Exact codebook values round(fp8 * 512) of an e4m3 matrix [rows,K] into int32 [rows,K]
 * (row stride ldd).  ref: __main__.py:157-158 _fp8_e4m3_to_int32.  NaN codes give 0,
 * like CUDA's float->int32 conversion of NaN in the reference expression. */
int ima_codebook_from_fp8(const uint8_t* src, int64_t rows, int64_t K, int64_t ld, int32_t* dst, int64_t ldd,
                          void* stream);

/* DIGITS3 planes of the codebook values of a matrix of e4m3 bytes ([rows,K], row stride ld), e.g. the
 * weight of a CodebookLinear (ref: __main__.py:429-432, done once per linear).
 * codebook_t [K,rows] int32 (optional) receives the transposed codebook the reference
 * keeps as `weight_t`. */
int ima_planes_from_fp8(const uint8_t* src, int64_t rows, int64_t K, int64_t ld, int8_t* planes, int64_t ldp,
                        int32_t* codebook_t, void* stream);

/* Digit planes of an int32 matrix given by element strides (stride_row, stride_k), so that
 * both the activation layout [M,K] and the reference's weight_t layout [K,N] can be
 * expanded.  Digits are balanced base-128 (v = sum_i 2^(7 i) d_i); scheme
 * IMA_SCHEME_DIGITS3 (3 planes, |v| <= 1064960, every codebook value) or
 * IMA_SCHEME_DIGITS5 (5 planes, any int32).  Values outside the scheme's range set the
 * device status to IMA_ERR_OVERFLOW. */
#define IMA_SCHEME_DIGITS3 3
#define IMA_SCHEME_DIGITS5 5
int ima_planes_from_int32(const int32_t* src, int64_t rows, int64_t K, int64_t stride_row, int64_t stride_k,
                          int scheme, int8_t* planes, int64_t ldp, void* stream);
int ima_scheme_planes(int scheme); /* number of planes a scheme uses (3 or 5) */

/* Largest |v| over an int32 matrix (device reduction into *out_maxabs, a device int64
 * the caller zeroes).  Used to choose the digit scheme of _int32_matmul. */
int ima_int32_maxabs(const int32_t* src, int64_t rows, int64_t cols, int64_t stride_row, int64_t stride_col,
                     int64_t* out_maxabs, void* stream);

/* ---- A3: exact int32 x int32 -> int64 GEMM on tcgen05 kind::i8 tensor cores ----
 * ref: __main__.py:188-253 _int32_raw_matmul (c only) and :256-333 _int32_matmul
 *      (y = (fp32_rn(C) * x_scale[m]) * w_scale[n]).
 * a_planes: [P][M][lda] int8, b_planes: [P][N][ldb] int8 (both K-major), P =
 * ima_scheme_planes(scheme).  Outputs (each optional, at least one):
 *   c [M,N] int64 (row stride ldc), exact modulo 2^64 like the reference's int64
 *   accumulator;
 *   y [M,N] of y_dtype (row stride ldy) = (fp32_rn(C) * x_scale[m]) * w_scale[n]
 *   (+ bias[n] in fp32 when bias != NULL), rounded once to y_dtype.
 * x_scale / w_scale may be NULL only when y == NULL. */
int ima_int_gemm(const int8_t* a_planes, int64_t lda, const int8_t* b_planes, int64_t ldb, int64_t M, int64_t N,
                 int64_t K, int scheme, int64_t* c, int64_t ldc, const float* x_scale, const float* w_scale,
                 const float* bias, void* y, int y_dtype, int64_t ldy, void* stream);

/* Many independent products in as few launches as possible (one per 64 problems): every
 * linear of a model in one call.  Fields mean what the arguments of ima_int_gemm mean;
 * all problems use the same digit scheme. */
typedef struct ima_gemm_problem {
    const int8_t* a_planes;
    int64_t lda;
    const int8_t* b_planes;
    int64_t ldb;
    int64_t M, N, K;
    int64_t* c;
    int64_t ldc;
    const float* x_scale;
    const float* w_scale;
    const float* bias;
    void* y;
    int32_t y_dtype;
    int64_t ldy;
} ima_gemm_problem;
int ima_int_gemm_grouped(const ima_gemm_problem* problems, int count, int scheme, void* stream);
/* The same GEMMs, with each problem's y written to up to 8 further destinations besides
 * problems[i].y, all with y's layout (row stride ldy, dtype y_dtype): copies[i].y[d], NULL
 * entries skipped.  For a multi-GPU caller these are the other GPUs' gathered-output
 * buffers (peer memory opened through CUDA IPC, or local memory): the epilogue stores each
 * output chunk to every destination, so the gather of the outputs rides on the GEMM itself
 * (plain stores over NVLink, no copy engines, no collective launch) and is complete when
 * the launch is.  copies == NULL is ima_int_gemm_grouped.  A problem without y must have no
 * copies (IMA_ERR_INVALID_ARGUMENT).  No reference counterpart: the reference runs on one
 * GPU (__main__.py:115-126). */
#define IMA_GEMM_MAX_Y_COPIES 8
typedef struct ima_gemm_y_copies {
    void* y[IMA_GEMM_MAX_Y_COPIES];
} ima_gemm_y_copies;
int ima_int_gemm_grouped_copies(const ima_gemm_problem* problems, const ima_gemm_y_copies* copies, int count,
                                int scheme, void* stream);
/* Process-wide cap on the number of persistent GEMM CTAs (one per SM); 0 (the default)
 * uses every SM.  A multi-GPU caller leaves a few SMs to the collectives it overlaps with
 * the GEMM (a persistent CTA never yields its SM, so a collective kernel queued behind a
 * full-machine GEMM launch would otherwise wait for it).  No reference counterpart. */
int ima_set_gemm_sm_limit(int sms);
/* Test knob of the failure-detection path (no reference counterpart): while stall_ns > 0,
 * every later GEMM launch makes its MMA thread first wait, for stall_ns nanoseconds (at most
 * 2 s), on an mbarrier that nothing arrives on.  The wait runs out: the kernel records
 * IMA_ERR_TIMEOUT (where 3, detail -2) in the device status word, every role of each CTA
 * stops, the loads and tensor-core work already in flight complete before the CTA frees
 * its tensor memory, and the launch returns without writing outputs.  0 (the default)
 * switches it off.  Process-wide, like ima_set_gemm_sm_limit. */
int ima_set_gemm_wait_test(int64_t stall_ns);

/* ---- A4: direct Hawkeye replay ---------------------------------------------
 * ref: hawkeye.py:222-275 hawkeye_fp8_sum (kernel hawkeye.py:127-219).
 * Each operand (activations and weights alike) is first staged once with
 * ima_hawkeye_prepare into a buffer of ima_hawkeye_operand_bytes(rows, K) bytes.
 * Replay supports products_per_group == 32, internal_width == 14,
 * zero_exponent == -139 (IMA_ERR_UNSUPPORTED otherwise).
 * out_bf16 [M,N] (bf16 bits) and/or out_f32 [M,N]: (gfloat * x_scale[m]) * w_scale[n]. */
int64_t ima_hawkeye_operand_pitch(int64_t rows);
int64_t ima_hawkeye_operand_bytes(int64_t rows, int64_t K);
int ima_hawkeye_prepare(const uint8_t* fp8, int64_t rows, int64_t K, int64_t ld, void* operand, void* stream);
int ima_hawkeye_replay(const void* x_operand, const void* w_operand, const float* x_scale, const float* w_scale,
                       int64_t M, int64_t N, int64_t K, int products_per_group, int internal_width,
                       int zero_exponent, uint16_t* out_bf16, int64_t ld_bf16, float* out_f32, int64_t ld_f32,
                       void* stream);
/* Activation side of one Hawkeye linear in one launch: per-token quantisation
 * (ref: __main__.py:148-154 _fp8_per_token, the same bits as ima_quantize_per_token)
 * fused with the staging of ima_hawkeye_prepare (ref: hawkeye.py:222-275 reads the
 * quantised rows).  x [M, K] (row stride ldx elements, x_dtype IMA_DTYPE_*) ->
 * scale[M] (fp32), the staged operand (ima_hawkeye_operand_bytes(M, K) bytes,
 * identical to ima_hawkeye_prepare of the codes) and, when q_fp8 is not NULL, the
 * e4m3 codes [M, K] (row stride ldq). */
int ima_hawkeye_quantize_prepare(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, float* scale,
                                 uint8_t* q_fp8, int64_t ldq, void* operand, void* stream);

/* ---- A6: Freivalds check A (B r) == (A B) r, wrapping int64 ------------------
 * ref: tests/test_real_integer_gemms.py:67-93 (_exact_matvec /
 *      _assert_freivalds_verifies_int_product; the reference has no production API).
 * Adds to *mismatch_rows (device int32, the caller zeroes it) the number of rows m with
 * sum_k A[m,k] (sum_n B[k,n] r[n]) != sum_n C[m,n] r[n] (mod 2^64).
 * workspace: device buffer of ima_freivalds_workspace_bytes(K) bytes. */
int64_t ima_freivalds_workspace_bytes(int64_t K);

/* The weight half of the check, t = codebook(w)^T r (t [K] int64, wrapping), with
 * w_fp8 [N,K].  It depends only on the weight and the vector, so a verifier that
 * checks every forward of a linear computes it once and reuses it. */
int ima_freivalds_weight_vector(const uint8_t* w_fp8, int64_t ldw, const int64_t* r, int64_t N, int64_t K,
                                int64_t* t, void* stream);

/* The row half for many products in one launch: for each problem, adds to
 * *mismatch_rows the rows m with A[m,:] . t != C[m,:] . r (mod 2^64).  A is e4m3 codes
 * (a_kind IMA_FREIVALDS_A_FP8, checked through their codebook values) or int32.  Up to
 * 192 problems go into one launch (more are split).  A launch whose problems are all fp8
 * with K a multiple of 4, N even, 4-byte aligned code rows and 16-byte aligned C rows, t
 * and r takes the faster unrolled path; any other launch the general one (same result). */
#define IMA_FREIVALDS_A_FP8 0
#define IMA_FREIVALDS_A_INT32 1
typedef struct ima_freivalds_rows_problem {
    const void* a;
    int64_t lda;
    const int64_t* t;
    const int64_t* c;
    int64_t ldc;
    const int64_t* r;
    int64_t M, N, K;
    int32_t a_kind;
    int32_t* mismatch_rows;
} ima_freivalds_rows_problem;
int ima_freivalds_rows_grouped(const ima_freivalds_rows_problem* problems, int count, void* stream);
/* A = codebook(x_fp8) [M,K], B = codebook(w_fp8)^T with w_fp8 [N,K] (CodebookLinear's operands) */
int ima_freivalds_fp8(const uint8_t* x_fp8, int64_t ldx, const uint8_t* w_fp8, int64_t ldw, const int64_t* c,
                      int64_t ldc, const int64_t* r, int64_t M, int64_t N, int64_t K, void* workspace,
                      int32_t* mismatch_rows, void* stream);
/* Same check as ima_freivalds_fp8 for callers that cannot allocate device memory (a
 * verifier inside a process whose device memory is reserved by another allocator, or a
 * latency-sensitive path that must not pay for cudaMalloc/cudaFree): no workspace
 * argument, no allocation.  No counterpart in the reference.  The scratch vector lives in
 * a fixed device array of IMA_FREIVALDS_NOALLOC_MAX_K int64 (512 KiB) that every GPU
 * loading the library holds until exit; K above that maximum returns IMA_ERR_UNSUPPORTED.
 * The first call on a device looks the array's address up with that device current.  The
 * call uses the current device's array, so `stream` and every pointer argument must belong
 * to the current device: a stream of another GPU, or a host or other-GPU pointer, returns
 * IMA_ERR_INVALID_ARGUMENT before any launch.  All calls on a device share the array (each
 * call clears it first), so calls whose work overlaps on the GPU race; the caller still
 * zeroes *mismatch_rows. */
#define IMA_FREIVALDS_NOALLOC_MAX_K 65536
int ima_freivalds_fp8_noalloc(const uint8_t* x_fp8, int64_t ldx, const uint8_t* w_fp8, int64_t ldw,
                              const int64_t* c, int64_t ldc, const int64_t* r, int64_t M, int64_t N, int64_t K,
                              int32_t* mismatch_rows, void* stream);
/* A int32 [M,K] (row stride lda), B int32 [K,N] (row stride ldb; the reference's weight_t) */
int ima_freivalds_i32(const int32_t* a, int64_t lda, const int32_t* b, int64_t ldb, const int64_t* c, int64_t ldc,
                      const int64_t* r, int64_t M, int64_t N, int64_t K, void* workspace, int32_t* mismatch_rows,
                      void* stream);

/* ---- A5: Hawkeye class counts -----------------------------------------------
 * ref: hawkeye_freivalds.py:51-57 _class_ids; the per-pack class sets the reference
 * builds with torch.unique (hawkeye_freivalds.py:906-907, :1097-1098).
 * masks [packs][16] uint32 (packs = ceil(K / pack_width)): bit c of pack p is set iff
 * class id c occurs in columns [p*pack_width, (p+1)*pack_width) of any row. */
int ima_class_presence(const uint8_t* fp8, int64_t rows, int64_t K, int64_t ld, int64_t pack_width, uint32_t* masks,
                       void* stream);

/* The class-count engine.  ref: hawkeye_freivalds.py:1017-1246 exact_hawkeye_fp8_sum with
 * its count products (:147-213, :593-704) and replays (:329-412 K5, :464-545 K6, :707-790 K7).
 * Per group of 32 k, the counts count[a, b, m, n] of every (activation class a, weight class b)
 * pair are formed on the tensor cores (one-hot int8 operands, int32 tensor memory): for each
 * token row the (at most 32) classes present in the group against those of each weight row,
 * i.e. every row and column of the reference's count product that can be nonzero.  The
 * Hawkeye accumulator is replayed from the counts in the same kernel (output bit-identical to
 * ima_hawkeye_replay), and every count tile is checked with a Freivalds fingerprint before it
 * is discarded.
 * Operands (activations and weights) are staged once each with ima_class_count_prepare into
 * a buffer of ima_class_count_operand_bytes(rows, K) bytes (16-byte aligned).  A staged weight
 * [N, K] is expanded once more with ima_class_count_weight_tiles into
 * ima_class_count_weight_tiles_bytes(N, K) bytes: per 8 weight rows and pair of groups its
 * one-hot slot rows, class magnitudes and the fingerprint weights, drawn from `seed`.
 * Outputs: out_bf16 and/or out_f32 [M,N] = (gfloat * x_scale[m]) * w_scale[n];
 * *mismatch_rows (device int32, zeroed by the caller) += slot rows whose count tile failed
 * the fingerprint (0 for a correct run).
 * tiles_out (optional, ima_class_count_tile_entries(M, N, K) int32) receives every count tile
 * as the tensor cores formed it: tile (strip, group pair gp, tile t, group h) at index
 * ((strip * ceil(G/2) + gp) * 8 + t) * 2 + h of [128 rows][256 cols], strip = sm + sn *
 * ceil(M/4) covering tokens 4 sm .. 4 sm + 3 and weight rows 64 sn + 8 t .. + 7; row = 32 *
 * token + activation slot, col = 32 * weight row + weight slot, value = count times the sign
 * of the weight class (slots: ima_class_count_prepare's class order).  tiles_in (optional,
 * same layout) replays and checks the given counts instead of the tensor-memory ones. */
int64_t ima_class_count_operand_bytes(int64_t rows, int64_t K);
int ima_class_count_prepare(const uint8_t* fp8, int64_t rows, int64_t K, int64_t ld, void* operand, void* stream);
int64_t ima_class_count_weight_tiles_bytes(int64_t N, int64_t K);
int ima_class_count_weight_tiles(const void* w_operand, int64_t N, int64_t K, uint64_t seed, void* tiles,
                                 void* stream);
int64_t ima_class_count_tile_entries(int64_t M, int64_t N, int64_t K);
int ima_class_count_replay(const void* x_operand, const void* w_operand, const void* w_tiles, const float* x_scale,
                           const float* w_scale, int64_t M, int64_t N, int64_t K, uint16_t* out_bf16, int64_t ld_bf16,
                           float* out_f32, int64_t ld_f32, int32_t* mismatch_rows, int32_t* tiles_out,
                           const int32_t* tiles_in, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IMA_B200_H */
