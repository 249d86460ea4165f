// Exact int32 x int32 -> int64 GEMM on tcgen05 kind::i8 tensor cores.
//
// ref: __main__.py:188-225 (_int32_raw_matmul_kernel) and :256-298 (_int32_matmul_kernel):
//   C[m,n] = sum_k a[m,k] * b[k,n]  (int64),   y = (fp32_rn(C) * x_scale[m]) * w_scale[n].
//
// Operands arrive as int8 digit planes (quantize.cu).  Per 128 x BN output tile the
// kernel accumulates one int32 product per "accumulator" in tensor memory and
// recombines them into int64 in the epilogue:
//   KARATSUBA3: six plane products P_p = A_p B_p^T (p = 0..5, planes d0, d1, d2,
//     d0+d1, d1+d2, d0+d2), C = P0 (1-2^7-2^14) + P1 (2^14-2^7-2^21) + P2 (2^28-2^21-2^14)
//     + P3 2^7 + P4 2^21 + P5 2^14.  Each |P_p| <= K * 2^14, exact in int32 for K < 2^17.
//   DIGITS5: 25 digit products grouped by shift s = i + j into 9 accumulators,
//     C = sum_s 2^(7 s) acc_s.  Each |acc_s| <= 5 * 2^12 * K, exact for K <= 100000.
// C is formed modulo 2^64, i.e. exactly the reference's wrapping int64 accumulator.
//
// CTA organisation (one persistent CTA per SM, 6 warps):
//   warp 0  TMA producer: per stage one A-plane tile [128 x 128 B] and one B-plane tile
//           [BN x 128 B], both 128-byte swizzled (no cluster multicast anywhere);
//   warp 1  TMEM allocator and single-thread MMA issuer (4 MMAs of K = 32 per stage);
//   warps 2-5 epilogue: tcgen05.ld of the accumulators (warp w reads TMEM lanes
//           32 (w % 4) .. + 31, i.e. one output row per thread), int64 recombine,
//           fused rescale, global stores.
// Every mbarrier wait is bounded (IMA_WAIT_LIMIT_NS); a timeout records
// IMA_ERR_TIMEOUT in the device status word and the CTA drains and exits.
#include <cudaTypedefs.h>
#include "sm100_primitives.cuh"

namespace {

constexpr int GM_BM = 128;
constexpr int GM_BK = 128;                 // bytes of K per stage (one 128-byte swizzle row)
constexpr int GM_THREADS = 192;
constexpr uint32_t GM_TMEM_COLS = 512;

template <int SCHEME>
struct Scheme;

template <>
struct Scheme<IMA_SCHEME_KARATSUBA3> {
    static constexpr int BN = 64;
    static constexpr int STAGES = 8;
    static constexpr int NACC = 6;
    static constexpr int PRODUCTS = 6;     // stages per K tile
    static constexpr int CHUNK = 16;       // epilogue columns per tcgen05.ld
    IMA_DEVINL static void product(int p, int& a, int& b, int& acc) { a = p; b = p; acc = p; }
    IMA_DEVINL static int64_t weight(int acc) {
        switch (acc) {
            case 0: return 1 - (1ll << 7) - (1ll << 14);
            case 1: return (1ll << 14) - (1ll << 7) - (1ll << 21);
            case 2: return (1ll << 28) - (1ll << 21) - (1ll << 14);
            case 3: return 1ll << 7;
            case 4: return 1ll << 21;
            default: return 1ll << 14;
        }
    }
};

template <>
struct Scheme<IMA_SCHEME_DIGITS5> {
    static constexpr int BN = 32;
    static constexpr int STAGES = 8;
    static constexpr int NACC = 9;
    static constexpr int PRODUCTS = 25;
    static constexpr int CHUNK = 8;
    IMA_DEVINL static void product(int p, int& a, int& b, int& acc) { a = p / 5; b = p % 5; acc = a + b; }
    IMA_DEVINL static int64_t weight(int acc) { return 1ll << (7 * acc); }
};

template <int SCHEME>
struct GemmSmem {
    static constexpr int BN = Scheme<SCHEME>::BN;
    static constexpr int STAGES = Scheme<SCHEME>::STAGES;
    static constexpr int A_BYTES = GM_BM * GM_BK;
    static constexpr int B_BYTES = BN * GM_BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TILES_BYTES = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFFSET = TILES_BYTES;   // full[S], empty[S], tmem_full, tmem_empty
    static constexpr int TOTAL = TILES_BYTES + (2 * STAGES + 2) * 8 + 16;
    static constexpr int ALLOC = TOTAL + 1024;        // slack to align the base to 1024 B
};

struct GemmParams {
    int64_t M, N, K;
    int64_t* c;
    int64_t ldc;
    const float* x_scale;
    const float* w_scale;
    const float* bias;
    void* y;
    int y_dtype;
    int64_t ldy;
};

template <int SCHEME>
__global__ void __launch_bounds__(GM_THREADS, 1)
int_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const GemmParams prm) {
    using S = Scheme<SCHEME>;
    using L = GemmSmem<SCHEME>;
    constexpr int BN = S::BN;
    extern __shared__ unsigned char gm_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gm_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
    uint64_t* empty = full + L::STAGES;
    uint64_t* tmem_full = empty + L::STAGES;
    uint64_t* tmem_empty = tmem_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m_tiles = (prm.M + GM_BM - 1) / GM_BM;
    const int64_t n_tiles = (prm.N + BN - 1) / BN;
    const int64_t num_tiles = m_tiles * n_tiles;
    const int k_tiles = (int)((prm.K + GM_BK - 1) / GM_BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tmem_full, 1);
        mbar_init(tmem_empty, 128);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, GM_TMEM_COLS);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
        uint32_t stage = 0, phase = 0;
        for (int64_t t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
            const int32_t m0 = (int32_t)((t % m_tiles) * GM_BM);
            const int32_t n0 = (int32_t)((t / m_tiles) * BN);
            for (int kt = 0; kt < k_tiles && !*abort_flag; ++kt) {
                for (int p = 0; p < S::PRODUCTS; ++p) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, IMA_WHERE_GEMM_PRODUCER, (int)stage)) {
                        *abort_flag = 1;
                        break;
                    }
                    int pa, pb, acc;
                    S::product(p, pa, pb, acc);
                    unsigned char* sa = smem + stage * L::STAGE_BYTES;
                    unsigned char* sb = sa + L::A_BYTES;
                    mbar_arrive_expect_tx(&full[stage], (uint32_t)L::STAGE_BYTES);
                    tma_load_3d(sa, &map_a, &full[stage], kt * GM_BK, m0, pa);
                    tma_load_3d(sb, &map_b, &full[stage], kt * GM_BK, n0, pb);
                    if (++stage == (uint32_t)L::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = idesc_i8(GM_BM, BN);
        uint32_t stage = 0, phase = 0, tphase = 0;
        for (int64_t t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
            // wait until the epilogue drained the accumulators of the previous tile
            if (!mbar_wait_bounded(tmem_empty, tphase ^ 1u, IMA_WHERE_GEMM_MMA, -1)) { *abort_flag = 1; break; }
            tphase ^= 1u;
            tc_fence_after();
            uint32_t started = 0;   // bit per accumulator: first MMA of this tile issued
            for (int kt = 0; kt < k_tiles && !*abort_flag; ++kt) {
                for (int p = 0; p < S::PRODUCTS; ++p) {
                    if (!mbar_wait_bounded(&full[stage], phase, IMA_WHERE_GEMM_MMA, (int)stage)) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    int pa, pb, acc;
                    S::product(p, pa, pb, acc);
                    uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
                    uint32_t sb = sa + L::A_BYTES;
                    uint32_t d = tmem_base + (uint32_t)(acc * BN);
#pragma unroll
                    for (int ks = 0; ks < GM_BK / 32; ++ks) {
                        uint32_t accumulate = (started >> acc) & 1u;
                        mma_i8(d, umma_desc_sw128_kmajor(sa + ks * 32), umma_desc_sw128_kmajor(sb + ks * 32), idesc,
                               accumulate);
                        started |= 1u << acc;
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == (uint32_t)L::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            mma_commit(tmem_full);
        }
    } else if (warp >= 2) {
        // ---------------- epilogue ----------------
        const int q = warp & 3;                // TMEM lane quadrant of this warp
        const int row_in_tile = q * 32 + lane;
        uint32_t tphase = 0;
        for (int64_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            bool ok = mbar_wait_bounded(tmem_full, tphase, IMA_WHERE_GEMM_EPILOGUE, -1);
            __syncwarp();   // tcgen05.ld below is warp-collective
            if (!__all_sync(0xFFFFFFFFu, ok)) { *abort_flag = 1; break; }
            tphase ^= 1u;
            tc_fence_after();
            const int64_t m = (t % m_tiles) * GM_BM + row_in_tile;
            const int64_t n0 = (t / m_tiles) * BN;
            const bool row_ok = m < prm.M;
            const float xs = (row_ok && prm.y) ? prm.x_scale[m] : 0.0f;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += S::CHUNK) {
                uint64_t cval[S::CHUNK];
#pragma unroll
                for (int j = 0; j < S::CHUNK; ++j) cval[j] = 0;
                if (k_tiles > 0) {
#pragma unroll
                    for (int a = 0; a < S::NACC; ++a) {
                        uint32_t r[S::CHUNK];
                        uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN + c0);
                        if constexpr (S::CHUNK == 16) tmem_ld16(taddr, r); else tmem_ld8(taddr, r);
                        tmem_wait_ld();
                        const uint64_t w = (uint64_t)S::weight(a);
#pragma unroll
                        for (int j = 0; j < S::CHUNK; ++j) cval[j] += w * (uint64_t)(int64_t)(int32_t)r[j];
                    }
                }
                if (row_ok) {
#pragma unroll
                    for (int j = 0; j < S::CHUNK; ++j) {
                        const int64_t n = n0 + c0 + j;
                        if (n >= prm.N) break;
                        const int64_t cv = (int64_t)cval[j];
                        if (prm.c) prm.c[m * prm.ldc + n] = cv;
                        if (prm.y) {
                            float yv = __fmul_rn(__fmul_rn(__ll2float_rn(cv), xs), prm.w_scale[n]);
                            if (prm.bias) yv = __fadd_rn(yv, prm.bias[n]);
                            if (prm.y_dtype == IMA_DTYPE_F32)
                                reinterpret_cast<float*>(prm.y)[m * prm.ldy + n] = yv;
                            else if (prm.y_dtype == IMA_DTYPE_BF16)
                                reinterpret_cast<__nv_bfloat16*>(prm.y)[m * prm.ldy + n] = __float2bfloat16_rn(yv);
                            else
                                reinterpret_cast<__half*>(prm.y)[m * prm.ldy + n] = __float2half_rn(yv);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(tmem_empty);
        }
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, GM_TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 3-D map over planes [P][rows][ld] int8 with a {128 B, box_rows, 1} box, 128-byte swizzle.
int make_plane_map(CUtensorMap* map, const int8_t* base, int64_t ld, int64_t rows, int planes, int box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return IMA_ERR_CUDA;
    cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)ld, (cuuint64_t)(ld * rows)};
    cuuint32_t box[3] = {(cuuint32_t)GM_BK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? IMA_OK : IMA_ERR_INVALID_ARGUMENT;
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int SCHEME>
int launch_int_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t ldb, const GemmParams& prm,
                    cudaStream_t stream) {
    using L = GemmSmem<SCHEME>;
    constexpr int P = SCHEME == IMA_SCHEME_KARATSUBA3 ? 6 : 5;
    CUtensorMap ma, mb;
    int rc = make_plane_map(&ma, a, lda, prm.M, P, GM_BM);
    if (rc != IMA_OK) return rc;
    rc = make_plane_map(&mb, b, ldb, prm.N, P, L::BN);
    if (rc != IMA_OK) return rc;
    auto kern = int_gemm_kernel<SCHEME>;
    rc = ima_note_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
    if (rc != IMA_OK) return rc;
    int64_t tiles = ((prm.M + GM_BM - 1) / GM_BM) * ((prm.N + L::BN - 1) / L::BN);
    int grid = (int)(tiles < num_sms() ? tiles : num_sms());
    kern<<<grid, GM_THREADS, L::ALLOC, stream>>>(ma, mb, prm);
    return IMA_LAUNCH_STATUS();
}

}  // namespace

extern "C" int ima_int_gemm(const int8_t* a_planes, int64_t lda, const int8_t* b_planes, int64_t ldb, int64_t M,
                            int64_t N, int64_t K, int scheme, int64_t* c, int64_t ldc, const float* x_scale,
                            const float* w_scale, const float* bias, void* y, int y_dtype, int64_t ldy,
                            void* stream) {
    if (!a_planes || !b_planes || M < 0 || N < 0 || K < 0) return IMA_ERR_INVALID_ARGUMENT;
    if (!c && !y) return IMA_ERR_INVALID_ARGUMENT;
    if (c && ldc < N) return IMA_ERR_INVALID_ARGUMENT;
    if (y && (!x_scale || !w_scale || ldy < N)) return IMA_ERR_INVALID_ARGUMENT;
    if (y && y_dtype != IMA_DTYPE_F32 && y_dtype != IMA_DTYPE_BF16 && y_dtype != IMA_DTYPE_F16)
        return IMA_ERR_INVALID_ARGUMENT;
    if (lda < K || ldb < K || lda % 16 || ldb % 16) return IMA_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(a_planes) & 15) || (reinterpret_cast<uintptr_t>(b_planes) & 15))
        return IMA_ERR_INVALID_ARGUMENT;
    if (M == 0 || N == 0) return IMA_OK;
    if (M > INT32_MAX || N > INT32_MAX || lda > INT32_MAX || ldb > INT32_MAX) return IMA_ERR_UNSUPPORTED;
    GemmParams prm{M, N, K, c, ldc, x_scale, w_scale, bias, y, y_dtype, ldy};
    if (scheme == IMA_SCHEME_KARATSUBA3) {
        if (K >= (1 << 17)) return IMA_ERR_UNSUPPORTED;
        return launch_int_gemm<IMA_SCHEME_KARATSUBA3>(a_planes, lda, b_planes, ldb, prm, (cudaStream_t)stream);
    }
    if (scheme == IMA_SCHEME_DIGITS5) {
        if (K > 100000) return IMA_ERR_UNSUPPORTED;
        return launch_int_gemm<IMA_SCHEME_DIGITS5>(a_planes, lda, b_planes, ldb, prm, (cudaStream_t)stream);
    }
    return IMA_ERR_UNSUPPORTED;
}
