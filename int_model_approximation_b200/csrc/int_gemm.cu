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
// One launch processes a batch of up to GM_MAXP independent problems (e.g. every linear
// of a model): the problem descriptors and their TMA tensor maps travel in the kernel
// parameters, tiles of all problems form one persistent work list (problems ordered by
// K, largest first), and each CTA walks it with stride gridDim.x.
//
// CTA organisation (one persistent CTA per SM, 6 warps):
//   warp 0  TMA producer: per stage one A-plane tile [128 x 128 B] and one B-plane tile
//           [BN x 128 B], both 128-byte swizzled (no cluster multicast anywhere);
//   warp 1  TMEM allocator and single-thread MMA issuer (4 MMAs of K = 32 per stage);
//   warps 2-5 epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (one output row per
//           thread), recombines int64, applies the fused rescale, stages 32 x 16 chunks in
//           shared memory (128-byte swizzled for the int64 tile) and writes them with TMA
//           stores.  The accumulators are released to the MMA warp as soon as the last
//           chunk is read, so the stores of tile t overlap the MMAs of tile t + 1.
// Every mbarrier wait is bounded (IMA_WAIT_LIMIT_NS); a timeout records
// IMA_ERR_TIMEOUT in the device status word and the CTA drains and exits.
#include <cudaTypedefs.h>
#include <algorithm>
#include <vector>
#include "sm100_primitives.cuh"

namespace {

constexpr int GM_BM = 128;
constexpr int GM_BK = 128;                 // bytes of K per stage (one 128-byte swizzle row)
constexpr int GM_THREADS = 192;
constexpr uint32_t GM_TMEM_COLS = 512;
constexpr int GM_MAXP = 80;                // problems per launch (kernel-parameter budget)
constexpr int GM_EPI_WARPS = 4;

template <int SCHEME>
struct Scheme;

template <>
struct Scheme<IMA_SCHEME_KARATSUBA3> {
    static constexpr int BN = 64;
    static constexpr int STAGES = 8;
    static constexpr int NACC = 6;
    static constexpr int PRODUCTS = 6;     // stages per K tile
    static constexpr int CHUNK = 16;       // epilogue columns per tcgen05.ld
    static constexpr bool TMA_STORE = true;
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
    static constexpr bool TMA_STORE = false;
    IMA_DEVINL static void product(int p, int& a, int& b, int& acc) { a = p / 5; b = p % 5; acc = a + b; }
    IMA_DEVINL static int64_t weight(int acc) { return 1ll << (7 * acc); }
};

template <int SCHEME>
struct GemmSmem {
    using S = Scheme<SCHEME>;
    static constexpr int BN = S::BN;
    static constexpr int STAGES = S::STAGES;
    static constexpr int A_BYTES = GM_BM * GM_BK;
    static constexpr int B_BYTES = BN * GM_BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TILES_BYTES = STAGES * STAGE_BYTES;
    // epilogue staging: per epilogue warp, two buffers of [32 rows x CHUNK] int64 (SW128) and y
    static constexpr int CST_BYTES = S::TMA_STORE ? 32 * S::CHUNK * 8 : 0;   // 4 KB
    static constexpr int YST_BYTES = S::TMA_STORE ? 32 * S::CHUNK * 4 : 0;   // room for fp32 y
    static constexpr int CST_OFFSET = TILES_BYTES;
    static constexpr int YST_OFFSET = CST_OFFSET + GM_EPI_WARPS * CST_BYTES;
    static constexpr int SCALE_OFFSET = YST_OFFSET + GM_EPI_WARPS * YST_BYTES;   // ws, bias: [warp][2][BN]
    static constexpr int BAR_OFFSET = SCALE_OFFSET + 2 * GM_EPI_WARPS * 2 * BN * 4;
    static constexpr int TOTAL = BAR_OFFSET + (2 * STAGES + 2) * 8 + 16;
    static constexpr int ALLOC = TOTAL + 1024;        // slack to align the base to 1024 B
};

struct GemmProblemDev {
    int64_t* c;
    void* y;
    const float* xs;
    const float* ws;
    const float* bias;
    int64_t ldc, ldy;
    int32_t M, N, K, y_dtype;
    int32_t m_tiles, k_tiles, tma_store, pad;
};

struct __align__(64) GemmBatch {
    CUtensorMap maps[GM_MAXP][2];   // A planes, B planes
    GemmProblemDev p[GM_MAXP];
    int32_t tile_start[GM_MAXP + 1];
    int32_t n;
};

IMA_DEVINL int find_problem(const GemmBatch& b, int64_t t) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (b.tile_start[mid] <= t) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <int SCHEME>
__global__ void __launch_bounds__(GM_THREADS, 1) int_gemm_kernel(const __grid_constant__ GemmBatch batch) {
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
    float* s_ws = reinterpret_cast<float*>(smem + L::SCALE_OFFSET);   // [warp][2][BN]
    float* s_bias = s_ws + GM_EPI_WARPS * 2 * BN;                     // [warp][2][BN]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t num_tiles = batch.tile_start[batch.n];

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tmem_full, 1);
        mbar_init(tmem_empty, GM_EPI_WARPS * 32);
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
        uint32_t stage = 0, phase = 0;
        for (int64_t t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
            const int pi = find_problem(batch, t);
            const GemmProblemDev& P = batch.p[pi];
            const int64_t lt = t - batch.tile_start[pi];
            const int32_t m0 = (int32_t)((lt % P.m_tiles) * GM_BM);
            const int32_t n0 = (int32_t)((lt / P.m_tiles) * BN);
            const CUtensorMap* ma = &batch.maps[pi][0];
            const CUtensorMap* mb = &batch.maps[pi][1];
            for (int kt = 0; kt < P.k_tiles && !*abort_flag; ++kt) {
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
                    tma_load_3d(sa, ma, &full[stage], kt * GM_BK, m0, pa);
                    tma_load_3d(sb, mb, &full[stage], kt * GM_BK, n0, pb);
                    if (++stage == (uint32_t)L::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = idesc_i8(GM_BM, BN);
        uint32_t stage = 0, phase = 0, tphase = 0;
        for (int64_t t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
            const GemmProblemDev& P = batch.p[find_problem(batch, t)];
            // wait until the epilogue drained the accumulators of the previous tile
            if (!mbar_wait_bounded(tmem_empty, tphase ^ 1u, IMA_WHERE_GEMM_MMA, -1)) { *abort_flag = 1; break; }
            tphase ^= 1u;
            tc_fence_after();
            uint32_t started = 0;   // bit per accumulator: first MMA of this tile issued
            for (int kt = 0; kt < P.k_tiles && !*abort_flag; ++kt) {
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
        const int ew = warp - 2;               // epilogue warp index 0..3
        const int q = warp & 3;                // TMEM lane quadrant of this warp
        uint32_t tphase = 0, tile_ctr = 0;
        for (int64_t t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tile_ctr) {
            const int pi = find_problem(batch, t);
            const GemmProblemDev& P = batch.p[pi];
            const int64_t lt = t - batch.tile_start[pi];
            const int32_t m0 = (int32_t)((lt % P.m_tiles) * GM_BM);
            const int32_t n0 = (int32_t)((lt / P.m_tiles) * BN);
            // per-warp copy of this tile's column scales and bias (no cross-warp barrier needed)
            float* ws_t = s_ws + (ew * 2 + (tile_ctr & 1)) * BN;
            float* bias_t = s_bias + (ew * 2 + (tile_ctr & 1)) * BN;
            for (int i = lane; i < BN; i += 32) {
                const int64_t n = n0 + i;
                ws_t[i] = (P.y && n < P.N) ? P.ws[n] : 0.0f;
                bias_t[i] = (P.bias && n < P.N) ? P.bias[n] : 0.0f;
            }
            __syncwarp();
            bool ok = mbar_wait_bounded(tmem_full, tphase, IMA_WHERE_GEMM_EPILOGUE, -1);
            __syncwarp();   // tcgen05.ld below is warp-collective
            if (!__all_sync(0xFFFFFFFFu, ok)) { *abort_flag = 1; break; }
            tphase ^= 1u;
            tc_fence_after();
            const int64_t m = (int64_t)m0 + q * 32 + lane;
            const bool row_ok = m < P.M;
            const float xs = (row_ok && P.y) ? P.xs[m] : 0.0f;
            const bool tma = S::TMA_STORE && P.tma_store;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += S::CHUNK) {
                uint64_t cval[S::CHUNK];
#pragma unroll
                for (int j = 0; j < S::CHUNK; ++j) cval[j] = 0;
                if (P.k_tiles > 0) {
                    uint32_t r[S::NACC][S::CHUNK];
#pragma unroll
                    for (int a = 0; a < S::NACC; ++a) {
                        uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN + c0);
                        if constexpr (S::CHUNK == 16) tmem_ld16(taddr, r[a]); else tmem_ld8(taddr, r[a]);
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int a = 0; a < S::NACC; ++a) {
                        const uint64_t w = (uint64_t)S::weight(a);
#pragma unroll
                        for (int j = 0; j < S::CHUNK; ++j) cval[j] += w * (uint64_t)(int64_t)(int32_t)r[a][j];
                    }
                }
                if (c0 + S::CHUNK >= BN) {
                    // every accumulator of this tile has been read: hand TMEM back to the MMA warp
                    tc_fence_before();
                    mbar_arrive(tmem_empty);
                }
                float yv[S::CHUNK];
#pragma unroll
                for (int j = 0; j < S::CHUNK; ++j) {
                    float v = __fmul_rn(__fmul_rn(__ll2float_rn((int64_t)cval[j]), xs), ws_t[c0 + j]);
                    yv[j] = P.bias ? __fadd_rn(v, bias_t[c0 + j]) : v;
                }
                if constexpr (S::TMA_STORE) {
                    if (tma) {
                        unsigned char* cst = smem + L::CST_OFFSET + ew * L::CST_BYTES;
                        unsigned char* yst = smem + L::YST_OFFSET + ew * L::YST_BYTES;
                        __syncwarp();   // the previous chunk's copy-out has finished reading the staging
                        if (P.c) {
                            // row `lane` = 128 bytes = 8 chunks of 16 B, chunk j stored at slot j ^ (lane % 8)
#pragma unroll
                            for (int j = 0; j < S::CHUNK / 2; ++j) {
                                uint4 v;
                                v.x = (uint32_t)cval[2 * j];
                                v.y = (uint32_t)(cval[2 * j] >> 32);
                                v.z = (uint32_t)cval[2 * j + 1];
                                v.w = (uint32_t)(cval[2 * j + 1] >> 32);
                                *reinterpret_cast<uint4*>(cst + lane * 128 + ((j ^ (lane & 7)) << 4)) = v;
                            }
                        }
                        if (P.y) {
                            if (P.y_dtype == IMA_DTYPE_F32) {
#pragma unroll
                                for (int j = 0; j < S::CHUNK / 4; ++j)
                                    *reinterpret_cast<float4*>(yst + lane * (S::CHUNK * 4) + j * 16) =
                                        make_float4(yv[4 * j], yv[4 * j + 1], yv[4 * j + 2], yv[4 * j + 3]);
                            } else {
                                uint32_t h[S::CHUNK / 2];
#pragma unroll
                                for (int j = 0; j < S::CHUNK / 2; ++j) {
                                    if (P.y_dtype == IMA_DTYPE_BF16) {
                                        __nv_bfloat162 b2 = __floats2bfloat162_rn(yv[2 * j], yv[2 * j + 1]);
                                        h[j] = *reinterpret_cast<uint32_t*>(&b2);
                                    } else {
                                        __half2 f2 = __floats2half2_rn(yv[2 * j], yv[2 * j + 1]);
                                        h[j] = *reinterpret_cast<uint32_t*>(&f2);
                                    }
                                }
#pragma unroll
                                for (int j = 0; j < S::CHUNK / 8; ++j)
                                    *reinterpret_cast<uint4*>(yst + lane * (S::CHUNK * 2) + j * 16) =
                                        make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
                            }
                        }
                        __syncwarp();
                        // copy-out: each instruction writes 4 rows x 128 B of C (lanes 8r..8r+7
                        // read row r's 16-byte slots back through the swizzle) and 16 or 8 rows of y
                        const int64_t rbase = (int64_t)m0 + q * 32;
                        const int64_t cbase = (int64_t)n0 + c0;
                        if (P.c) {
#pragma unroll
                            for (int it = 0; it < 8; ++it) {
                                const int r = it * 4 + (lane >> 3), j = lane & 7;
                                const int64_t gm = rbase + r, gn = cbase + 2 * j;
                                const uint4 v = *reinterpret_cast<const uint4*>(cst + r * 128 + ((j ^ (r & 7)) << 4));
                                if (gm < P.M) {
                                    int64_t* dst = P.c + gm * P.ldc + gn;
                                    if (gn + 1 < P.N) {
                                        *reinterpret_cast<uint4*>(dst) = v;
                                    } else if (gn < P.N) {
                                        dst[0] = (int64_t)(((uint64_t)v.y << 32) | v.x);
                                    }
                                }
                            }
                        }
                        if (P.y) {
                            const int esize = P.y_dtype == IMA_DTYPE_F32 ? 4 : 2;
                            const int row_bytes = S::CHUNK * esize;            // 32 or 64
                            const int lanes_per_row = row_bytes / 16;           // 2 or 4
                            const int rows_per_it = 32 / lanes_per_row;         // 16 or 8
                            for (int it = 0; it < 32 / rows_per_it; ++it) {
                                const int r = it * rows_per_it + lane / lanes_per_row;
                                const int part = lane % lanes_per_row;
                                const int64_t gm = rbase + r;
                                const int64_t gn = cbase + part * (16 / esize);
                                const uint4 v = *reinterpret_cast<const uint4*>(yst + r * row_bytes + part * 16);
                                if (gm < P.M && gn < P.N) {
                                    unsigned char* dst = reinterpret_cast<unsigned char*>(P.y) + (gm * P.ldy + gn) * esize;
                                    if (gn + 16 / esize <= P.N) {
                                        *reinterpret_cast<uint4*>(dst) = v;
                                    } else if (esize == 4) {
                                        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                                        for (int e = 0; e < 4; ++e)
                                            if (gn + e < P.N) reinterpret_cast<uint32_t*>(dst)[e] = w4[e];
                                    } else {
                                        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                                        for (int e = 0; e < 8; ++e)
                                            if (gn + e < P.N)
                                                reinterpret_cast<uint16_t*>(dst)[e] = (uint16_t)(w4[e >> 1] >> (16 * (e & 1)));
                                    }
                                }
                            }
                        }
                        continue;
                    }
                }
                if (row_ok) {
#pragma unroll
                    for (int j = 0; j < S::CHUNK; ++j) {
                        const int64_t n = n0 + c0 + j;
                        if (n >= P.N) break;
                        if (P.c) P.c[m * P.ldc + n] = (int64_t)cval[j];
                        if (P.y) {
                            if (P.y_dtype == IMA_DTYPE_F32)
                                reinterpret_cast<float*>(P.y)[m * P.ldy + n] = yv[j];
                            else if (P.y_dtype == IMA_DTYPE_BF16)
                                reinterpret_cast<__nv_bfloat16*>(P.y)[m * P.ldy + n] = __float2bfloat16_rn(yv[j]);
                            else
                                reinterpret_cast<__half*>(P.y)[m * P.ldy + n] = __float2half_rn(yv[j]);
                        }
                    }
                }
            }
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

int check_problem(const ima_gemm_problem& q, int scheme) {
    if (!q.a_planes || !q.b_planes || q.M < 0 || q.N < 0 || q.K < 0) return IMA_ERR_INVALID_ARGUMENT;
    if (!q.c && !q.y) return IMA_ERR_INVALID_ARGUMENT;
    if (q.c && q.ldc < q.N) return IMA_ERR_INVALID_ARGUMENT;
    if (q.y && (!q.x_scale || !q.w_scale || q.ldy < q.N)) return IMA_ERR_INVALID_ARGUMENT;
    if (q.y && q.y_dtype != IMA_DTYPE_F32 && q.y_dtype != IMA_DTYPE_BF16 && q.y_dtype != IMA_DTYPE_F16)
        return IMA_ERR_INVALID_ARGUMENT;
    if (q.lda < q.K || q.ldb < q.K || q.lda % 16 || q.ldb % 16) return IMA_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(q.a_planes) & 15) || (reinterpret_cast<uintptr_t>(q.b_planes) & 15))
        return IMA_ERR_INVALID_ARGUMENT;
    if (q.M > INT32_MAX / 2 || q.N > INT32_MAX / 2 || q.lda > INT32_MAX || q.ldb > INT32_MAX) return IMA_ERR_UNSUPPORTED;
    if (scheme == IMA_SCHEME_KARATSUBA3 && q.K >= (1 << 17)) return IMA_ERR_UNSUPPORTED;
    if (scheme == IMA_SCHEME_DIGITS5 && q.K > 100000) return IMA_ERR_UNSUPPORTED;
    return IMA_OK;
}

template <int SCHEME>
int launch_batch(GemmBatch& b, cudaStream_t stream) {
    using L = GemmSmem<SCHEME>;
    auto kern = int_gemm_kernel<SCHEME>;
    int rc = ima_note_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
    if (rc != IMA_OK) return rc;
    int64_t tiles = b.tile_start[b.n];
    if (tiles == 0) return IMA_OK;
    int grid = (int)(tiles < num_sms() ? tiles : num_sms());
    kern<<<grid, GM_THREADS, L::ALLOC, stream>>>(b);
    return IMA_LAUNCH_STATUS();
}

template <int SCHEME>
int run_grouped(const ima_gemm_problem* problems, int count, cudaStream_t stream) {
    using L = GemmSmem<SCHEME>;
    constexpr int P = SCHEME == IMA_SCHEME_KARATSUBA3 ? 6 : 5;
    // largest K first: the most expensive tiles start first on the persistent grid
    std::vector<int> order;
    for (int i = 0; i < count; ++i)
        if (problems[i].M > 0 && problems[i].N > 0) order.push_back(i);
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return problems[a].K > problems[b].K; });
    static thread_local GemmBatch b;   // host staging of the kernel parameters (copied at launch)
    // deal the K-sorted problems round-robin into as few launches as the parameter budget
    // allows, so every launch gets a similar mix of expensive and cheap tiles
    const size_t nb = (order.size() + GM_MAXP - 1) / GM_MAXP;
    for (size_t batch = 0; batch < nb; ++batch) {
        memset(&b, 0, sizeof(b));
        int32_t tiles = 0;
        for (size_t i = batch; i < order.size(); i += nb) {
            const ima_gemm_problem& q = problems[order[i]];
            const int k = b.n;
            GemmProblemDev& D = b.p[k];
            int rc = make_plane_map(&b.maps[k][0], q.a_planes, q.lda, q.M, P, GM_BM);
            if (rc != IMA_OK) return rc;
            rc = make_plane_map(&b.maps[k][1], q.b_planes, q.ldb, q.N, P, L::BN);
            if (rc != IMA_OK) return rc;
            D.c = q.c; D.y = q.y; D.xs = q.x_scale; D.ws = q.w_scale; D.bias = q.bias;
            D.ldc = q.ldc; D.ldy = q.ldy;
            D.M = (int32_t)q.M; D.N = (int32_t)q.N; D.K = (int32_t)q.K; D.y_dtype = q.y_dtype;
            D.m_tiles = (int32_t)((q.M + GM_BM - 1) / GM_BM);
            D.k_tiles = (int32_t)((q.K + GM_BK - 1) / GM_BK);
            // staged 16-byte copy-out needs 16-byte aligned rows; otherwise element stores
            const int yes = q.y_dtype == IMA_DTYPE_F32 ? 4 : 2;
            bool vec = Scheme<SCHEME>::TMA_STORE;
            if (q.c) vec = vec && !(reinterpret_cast<uintptr_t>(q.c) & 15) && !((q.ldc * 8) & 15);
            if (q.y) vec = vec && !(reinterpret_cast<uintptr_t>(q.y) & 15) && !((q.ldy * yes) & 15);
            D.tma_store = vec ? 1 : 0;
            b.tile_start[k] = tiles;
            tiles += D.m_tiles * (int32_t)((q.N + L::BN - 1) / L::BN);
            b.n = k + 1;
        }
        b.tile_start[b.n] = tiles;
        int rc = launch_batch<SCHEME>(b, stream);
        if (rc != IMA_OK) return rc;
    }
    return IMA_OK;
}

}  // namespace

extern "C" int ima_int_gemm_grouped(const ima_gemm_problem* problems, int count, int scheme, void* stream) {
    if (count < 0 || (count > 0 && !problems)) return IMA_ERR_INVALID_ARGUMENT;
    if (scheme != IMA_SCHEME_KARATSUBA3 && scheme != IMA_SCHEME_DIGITS5) return IMA_ERR_UNSUPPORTED;
    for (int i = 0; i < count; ++i) {
        int rc = check_problem(problems[i], scheme);
        if (rc != IMA_OK) return rc;
    }
    if (scheme == IMA_SCHEME_KARATSUBA3)
        return run_grouped<IMA_SCHEME_KARATSUBA3>(problems, count, (cudaStream_t)stream);
    return run_grouped<IMA_SCHEME_DIGITS5>(problems, count, (cudaStream_t)stream);
}

extern "C" int ima_int_gemm(const int8_t* a_planes, int64_t lda, const int8_t* b_planes, int64_t ldb, int64_t M,
                            int64_t N, int64_t K, int scheme, int64_t* c, int64_t ldc, const float* x_scale,
                            const float* w_scale, const float* bias, void* y, int y_dtype, int64_t ldy,
                            void* stream) {
    ima_gemm_problem q = {a_planes, lda, b_planes, ldb, M, N, K, c, ldc, x_scale, w_scale, bias, y, y_dtype, ldy};
    return ima_int_gemm_grouped(&q, 1, scheme, stream);
}
