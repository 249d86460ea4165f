// Exact int32 x int32 -> int64 GEMM on tcgen05 kind::i8 tensor cores.
//
// ref: __main__.py:188-225 (_int32_raw_matmul_kernel) and :256-298 (_int32_matmul_kernel):
//   C[m,n] = sum_k a[m,k] * b[k,n]  (int64),   y = (fp32_rn(C) * x_scale[m]) * w_scale[n].
//
// Operands arrive as int8 digit planes (quantize.cu): v = sum_i 2^(7 i) d_i with balanced
// base-128 digits.  With NP digits per operand the product is
//   C = sum_s 2^(7 s) c_s,     c_s = sum_{i + j = s} A_i B_j^T      (s = 0 .. 2 NP - 2),
// i.e. NP^2 int8 digit products grouped by shift into 2 NP - 1 int32 accumulators in tensor
// memory, recombined into int64 in the epilogue.  DIGITS3 (NP = 3, |v| <= 1,064,960, every
// codebook value): 9 products, 5 accumulators, |c_s| <= 3 * 2^12 * K, exact for K < 174,762.
// DIGITS5 (NP = 5, any int32): 25 products, 9 accumulators, exact for K <= 100,000.
// C is formed modulo 2^64, i.e. exactly the reference's wrapping int64 accumulator.
//
// Data movement.  A stage holds one 64-byte K-slice of all NP A planes (128 rows each) and
// all NP B planes (BN rows each, stacked), 64-byte swizzled; each operand byte crosses
// L2 -> SM once per tile.
//
// MMA fan-out.  The accumulators c_0 .. c_{2NP-2} sit side by side in tensor memory, BN
// columns each, so A_i times the stacked B planes [B_0; ..; B_{NP-1}] (one MMA of
// N = NP * BN <= 256) lands A_i B_j^T in accumulator i + j for every j at once: NP MMAs per
// 32-byte K step instead of NP^2, and each A plane is read from shared memory once.  The
// MMA of i = 0 in the first K step of a tile overwrites accumulators 0 .. NP-1; the others
// accumulate, so accumulators NP .. 2NP-2 must start at zero: the epilogue warps zero them
// with tcgen05.st after draining a tile (and once at kernel start).
//
// One launch processes a batch of up to GM_MAXP independent problems (e.g. every linear
// of a model): the problem descriptors and their TMA tensor maps travel in the kernel
// parameters, tiles of all problems form one persistent work list, and each CTA walks it
// with stride gridDim.x.
//
// CTA organisation (one persistent CTA per SM, 10 warps):
//   warp 0    TMA producer (no cluster multicast anywhere);
//   warp 1    TMEM allocator and single-thread MMA issuer (2 x NP^2 MMAs of K = 32 per stage);
//   warps 2-9 epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (one output row per
//             thread) and half of the tile's columns, recombines them into int64 registers and
//             hands the accumulators back to the MMA warp at once; it then applies the fused
//             rescale, stages 32 x CHUNK chunks in swizzled shared memory and copies them out
//             with coalesced 16-byte stores while the next tile's MMAs run.
// Every mbarrier wait is bounded (IMA_WAIT_LIMIT_NS); a timeout records
// IMA_ERR_TIMEOUT in the device status word and the CTA drains and exits.
#include <cudaTypedefs.h>
#include <algorithm>
#include <vector>
#include "sm100_primitives.cuh"

namespace {

constexpr int GM_BM = 128;
constexpr int GM_KT = 64;                  // bytes of K per stage (one 64-byte swizzle row)
constexpr int GM_EPI_WARPS = 8;            // two per TMEM lane quadrant
constexpr int GM_THREADS = 64 + GM_EPI_WARPS * 32;
constexpr uint32_t GM_TMEM_COLS = 512;
constexpr int GM_MAXP = 64;                // problems per launch (kernel-parameter budget)
constexpr int GM_MAXD = 8;                 // extra destinations of y per problem (ima_int_gemm_grouped_copies)

template <int SCHEME>
struct Scheme;

template <>
struct Scheme<IMA_SCHEME_DIGITS3> {
    static constexpr int NP = 3;
    static constexpr int BN = 80;          // NP * BN = 240 <= 256 (one MMA per A plane)
    static constexpr int STAGES = 4;
    static constexpr int CHUNK = 8;        // epilogue columns per tcgen05.ld
};

template <>
struct Scheme<IMA_SCHEME_DIGITS5> {
    static constexpr int NP = 5;
    static constexpr int BN = 48;
    static constexpr int STAGES = 3;
    static constexpr int CHUNK = 8;
};

template <int SCHEME>
struct GemmCfg {
    using S = Scheme<SCHEME>;
    static constexpr int NP = S::NP;
    static constexpr int NACC = 2 * NP - 1;
    static constexpr int BN = S::BN;
    static constexpr int STAGES = S::STAGES;
    static constexpr int CHUNK = S::CHUNK;
    static constexpr int SLOTS = CHUNK / 2;                 // 16-byte slots per staged int64 row
    static constexpr int HALF = BN / 2;                     // columns per epilogue warp
    static_assert(HALF % CHUNK == 0, "columns per epilogue warp must be whole chunks");
    static_assert(NACC * BN <= (int)GM_TMEM_COLS, "accumulators exceed tensor memory");
    static_assert(NP * BN <= 256 && (NP * BN) % 16 == 0, "stacked B planes must form one MMA of N <= 256");
    static_assert((BN * GM_KT) % 512 == 0, "each stacked B plane must start on a 64-byte swizzle atom");
    static constexpr int A_PLANE = GM_BM * GM_KT;           // 8 KB
    static constexpr int B_PLANE = BN * GM_KT;
    static constexpr int STAGE_BYTES = NP * (A_PLANE + B_PLANE);
    static constexpr int TILES_BYTES = STAGES * STAGE_BYTES;
    static constexpr int CST_BYTES = 32 * CHUNK * 8;        // one staged int64 chunk per warp
    static constexpr int YST_BYTES = 32 * CHUNK * 4;        // room for fp32 y
    static constexpr int CST_OFFSET = TILES_BYTES;
    static constexpr int YST_OFFSET = CST_OFFSET + GM_EPI_WARPS * CST_BYTES;
    static constexpr int SCALE_OFFSET = YST_OFFSET + GM_EPI_WARPS * YST_BYTES;   // ws, bias: [warp][2][HALF]
    static constexpr int BAR_OFFSET = SCALE_OFFSET + 2 * GM_EPI_WARPS * 2 * HALF * 4;
    static constexpr int TOTAL = BAR_OFFSET + (2 * STAGES + 4) * 8 + 16;
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
    int32_t m_tiles, k_tiles, vec_out, ncopy;   // ncopy: extra destinations of y (batch.ycopy)
    int32_t N_tile, group_m;                    // column tile width (BN); row tiles per group
};

struct __align__(64) GemmBatch {
    CUtensorMap maps[GM_MAXP][2];   // A planes, B planes
    GemmProblemDev p[GM_MAXP];
    void* ycopy[GM_MAXP][GM_MAXD];  // further copies of each problem's y (same layout, ldy)
    int32_t tile_start[GM_MAXP + 1];
    int32_t n;
    int32_t has_copies;             // some problem writes copies of y
    uint64_t stall_ns;              // test knob (ima_set_gemm_wait_test); 0 in normal use
};

static_assert(sizeof(GemmBatch) <= 32764, "kernel parameters of one grouped GEMM launch");
static_assert(GM_MAXD == IMA_GEMM_MAX_Y_COPIES, "copies per problem");

// Tile lt of a problem -> (row tile, column tile).  Row tiles are taken in groups of
// P.group_m and, within a group, the column tiles in order with the group's row tiles
// fastest: the tiles in flight at once (one per CTA, consecutive tile numbers) share both
// the activation and the weight k-slices they stream, and the group's activation planes stay
// in L2 while its column tiles pass, so the weight planes are read once per group.  (Row
// tiles fastest over the whole problem would have every column tile stream all the
// activation planes from DRAM again once they exceed L2.)
IMA_DEVINL void tile_coords(const GemmProblemDev& P, int64_t lt, int32_t& mt, int32_t& nt) {
    const int32_t n_tiles = (P.N + (P.N_tile - 1)) / P.N_tile;
    const int64_t per_group = (int64_t)P.group_m * n_tiles;
    const int32_t group = (int32_t)(lt / per_group);
    const int32_t within = (int32_t)(lt - (int64_t)group * per_group);
    const int32_t gm = min(P.group_m, P.m_tiles - group * P.group_m);
    mt = group * P.group_m + within % gm;
    nt = within / gm;
}

IMA_DEVINL int find_problem(const GemmBatch& b, int64_t t) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (b.tile_start[mid] <= t) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA with the
// 64-byte swizzle: rows of 64 bytes, 8-row core-matrix groups 512 bytes apart.
IMA_DEVINL uint64_t umma_desc_sw64_kmajor(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);          // start address
    d |= (uint64_t)1u << 16;                               // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(512u >> 4) << 32;                      // stride byte offset: 8 rows * 64 B
    d |= (uint64_t)1u << 46;                               // descriptor version (sm_100)
    d |= (uint64_t)4u << 61;                               // layout: SWIZZLE_64B
    return d;
}

template <int SCHEME>
__global__ void __launch_bounds__(GM_THREADS, 1) int_gemm_kernel(const __grid_constant__ GemmBatch batch) {
    using L = GemmCfg<SCHEME>;
    constexpr int NP = L::NP, NACC = L::NACC, BN = L::BN, CHUNK = L::CHUNK, HALF = L::HALF;
    extern __shared__ unsigned char gm_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gm_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
    uint64_t* empty = full + L::STAGES;
    uint64_t* tmem_full = empty + L::STAGES;
    uint64_t* tmem_empty = tmem_full + 1;
    uint64_t* mma_drained = tmem_empty + 1;   // the MMA thread's final commit
    uint64_t* never = mma_drained + 1;        // nothing arrives on it (the test stall waits here)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(never + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* s_ws = reinterpret_cast<float*>(smem + L::SCALE_OFFSET);   // [warp][2][HALF]
    float* s_bias = s_ws + GM_EPI_WARPS * 2 * HALF;                   // [warp][2][HALF]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t num_tiles = batch.tile_start[batch.n];

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tmem_full, 1);
        mbar_init(tmem_empty, GM_EPI_WARPS * 32);
        mbar_init(mma_drained, 1);
        mbar_init(never, 1);
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
        uint64_t issued = 0;   // stages filled so far (drained below whatever happens)
        for (int64_t t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
            const int pi = find_problem(batch, t);
            const GemmProblemDev& P = batch.p[pi];
            const int64_t lt = t - batch.tile_start[pi];
            int32_t mt, nt;
            tile_coords(P, lt, mt, nt);
            const int32_t m0 = mt * GM_BM;
            const int32_t n0 = nt * BN;
            const CUtensorMap* ma = &batch.maps[pi][0];
            const CUtensorMap* mb = &batch.maps[pi][1];
            for (int kt = 0; kt < P.k_tiles; ++kt) {
                if (!mbar_wait_or_abort(&empty[stage], phase ^ 1u, abort_flag, IMA_WAIT_LIMIT_NS,
                                        IMA_WHERE_GEMM_PRODUCER, (int)stage))
                    break;
                ++issued;
                unsigned char* sbase = smem + stage * L::STAGE_BYTES;
                mbar_arrive_expect_tx(&full[stage], (uint32_t)L::STAGE_BYTES);
#pragma unroll
                for (int i = 0; i < NP; ++i) {
                    tma_load_3d(sbase + i * L::A_PLANE, ma, &full[stage], kt * GM_KT, m0, i);
                    tma_load_3d(sbase + NP * L::A_PLANE + i * L::B_PLANE, mb, &full[stage], kt * GM_KT, n0, i);
                }
                if (++stage == (uint32_t)L::STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        // Drain: after an abort the MMA thread may not have consumed the last stages, so
        // wait (bounded) until every TMA load issued into shared memory has landed before
        // the CTA can exit.  Stage s received the fills of rounds 0 .. R_s - 1; the last one
        // completes the phase of parity (R_s - 1) & 1 of full[s].
        for (int s = 0; s < L::STAGES; ++s) {
            const uint64_t rounds = issued / L::STAGES + ((uint64_t)s < issued % L::STAGES ? 1u : 0u);
            if (rounds > 0)
                mbar_wait_bounded(&full[s], (uint32_t)((rounds - 1) & 1u), IMA_WHERE_GEMM_PRODUCER, 100 + s);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = idesc_i8(GM_BM, NP * BN);
        uint32_t stage = 0, phase = 0, tphase = 0;
        if (batch.stall_ns) {
            // test knob: a wait that nothing ends runs out, records IMA_ERR_TIMEOUT and
            // sets the abort flag; every role then drains and the kernel returns
            mbar_wait_or_abort(never, 0u, abort_flag, batch.stall_ns, IMA_WHERE_GEMM_MMA, -2);
        }
        for (int64_t t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
            const GemmProblemDev& P = batch.p[find_problem(batch, t)];
            // wait until the epilogue drained the previous tile and zeroed accumulators
            // NP .. NACC-1 (for the first tile: zeroed them at kernel start)
            if (!mbar_wait_or_abort(tmem_empty, tphase, abort_flag, IMA_WAIT_LIMIT_NS, IMA_WHERE_GEMM_MMA, -1)) break;
            tphase ^= 1u;
            tc_fence_after();
            bool fed = true;
            for (int kt = 0; kt < P.k_tiles; ++kt) {
                if (!mbar_wait_or_abort(&full[stage], phase, abort_flag, IMA_WAIT_LIMIT_NS, IMA_WHERE_GEMM_MMA,
                                        (int)stage)) {
                    fed = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + stage * L::STAGE_BYTES);
                const uint32_t sb = sa + NP * L::A_PLANE;
#pragma unroll
                for (int ks = 0; ks < GM_KT / 32; ++ks) {
#pragma unroll
                    for (int i = 0; i < NP; ++i) {
                        // accumulators i .. i+NP-1 += A_i [B_0; ..; B_{NP-1}]^T
                        const bool first = kt == 0 && ks == 0 && i == 0;
                        mma_i8(tmem_base + (uint32_t)(i * BN), umma_desc_sw64_kmajor(sa + i * L::A_PLANE + ks * 32),
                               umma_desc_sw64_kmajor(sb + ks * 32), idesc, first ? 0u : 1u);
                    }
                }
                mma_commit(&empty[stage]);
                if (++stage == (uint32_t)L::STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!fed) break;
            mma_commit(tmem_full);
        }
        // Drain: every MMA this thread issued completes before the CTA frees tensor memory
        // (a commit with nothing outstanding arrives at once).
        mma_commit(mma_drained);
        mbar_wait_bounded(mma_drained, 0u, IMA_WHERE_GEMM_MMA, -3);
    } else if (warp >= 2) {
        // ---------------- epilogue ----------------
        const int ew = warp - 2;               // epilogue warp index 0..7
        const int q = warp & 3;                // TMEM lane quadrant of this warp
        const int h = ew >> 2;                 // column half of the tile
        uint32_t tphase = 0, tile_ctr = 0;
        // zero this warp's share of accumulators NP .. NACC-1, then hand TMEM to the MMA warp
        auto zero_upper_and_release = [&]() {
            const uint32_t zero[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int a = NP; a < NACC; ++a)
#pragma unroll
                for (int c0 = 0; c0 < HALF; c0 += 8)
                    tmem_st8(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN + h * HALF + c0), zero);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(tmem_empty);
        };
        zero_upper_and_release();
        for (int64_t t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tile_ctr) {
            const int pi = find_problem(batch, t);
            const GemmProblemDev& P = batch.p[pi];
            const int64_t lt = t - batch.tile_start[pi];
            int32_t mt, nt;
            tile_coords(P, lt, mt, nt);
            const int32_t m0 = mt * GM_BM;
            const int32_t n0 = nt * BN + h * HALF;
            // per-warp copy of this warp's column scales and bias (no cross-warp barrier needed)
            float* ws_t = s_ws + (ew * 2 + (tile_ctr & 1)) * HALF;
            float* bias_t = s_bias + (ew * 2 + (tile_ctr & 1)) * HALF;
            for (int i = lane; i < HALF; i += 32) {
                const int64_t n = n0 + i;
                ws_t[i] = (P.y && n < P.N) ? P.ws[n] : 0.0f;
                bias_t[i] = (P.bias && n < P.N) ? P.bias[n] : 0.0f;
            }
            __syncwarp();
            bool ok = mbar_wait_or_abort(tmem_full, tphase, abort_flag, IMA_WAIT_LIMIT_NS, IMA_WHERE_GEMM_EPILOGUE, -1);
            __syncwarp();   // tcgen05.ld below is warp-collective
            if (!__all_sync(0xFFFFFFFFu, ok)) { *abort_flag = 1; break; }
            tphase ^= 1u;
            tc_fence_after();
            const int64_t m = (int64_t)m0 + q * 32 + lane;
            const bool row_ok = m < P.M;
            const float xs = (row_ok && P.y) ? P.xs[m] : 0.0f;
            // Drain: every accumulator column of this warp into int64 registers, then hand
            // TMEM back at once, so that the conversion and copy-out below overlap the MMAs
            // of the next tile.
            uint64_t call[HALF];
#pragma unroll
            for (int j = 0; j < HALF; ++j) call[j] = 0;
            if (P.k_tiles > 0) {
#pragma unroll
                for (int c0 = 0; c0 < HALF; c0 += CHUNK) {
                    uint32_t r[NACC][CHUNK];
#pragma unroll
                    for (int a = 0; a < NACC; ++a) {
                        const uint32_t taddr =
                            tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN + h * HALF + c0);
                        if constexpr (CHUNK == 16) tmem_ld16(taddr, r[a]); else tmem_ld8(taddr, r[a]);
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int a = 0; a < NACC; ++a) {
#pragma unroll
                        for (int j = 0; j < CHUNK; ++j)
                            call[c0 + j] += (uint64_t)(int64_t)(int32_t)r[a][j] << (7 * a);
                    }
                }
            }
            zero_upper_and_release();
#pragma unroll
            for (int c0 = 0; c0 < HALF; c0 += CHUNK) {
                const uint64_t* cval = call + c0;
                float yv[CHUNK];
#pragma unroll
                for (int j = 0; j < CHUNK; ++j) {
                    float v = __fmul_rn(__fmul_rn(__ll2float_rn((int64_t)cval[j]), xs), ws_t[c0 + j]);
                    yv[j] = P.bias ? __fadd_rn(v, bias_t[c0 + j]) : v;
                }
                if (P.vec_out) {
                    unsigned char* cst = smem + L::CST_OFFSET + ew * L::CST_BYTES;
                    unsigned char* yst = smem + L::YST_OFFSET + ew * L::YST_BYTES;
                    constexpr int SLOTS = L::SLOTS;
                    __syncwarp();   // the previous chunk's copy-out has finished reading the staging
                    if (P.c) {
                        // row `lane` = SLOTS 16-byte slots; slot j stored at j ^ (lane % SLOTS)
#pragma unroll
                        for (int j = 0; j < SLOTS; ++j) {
                            uint4 v;
                            v.x = (uint32_t)cval[2 * j];
                            v.y = (uint32_t)(cval[2 * j] >> 32);
                            v.z = (uint32_t)cval[2 * j + 1];
                            v.w = (uint32_t)(cval[2 * j + 1] >> 32);
                            *reinterpret_cast<uint4*>(cst + lane * (SLOTS * 16) + ((j ^ (lane % SLOTS)) << 4)) = v;
                        }
                    }
                    if (P.y) {
                        if (P.y_dtype == IMA_DTYPE_F32) {
#pragma unroll
                            for (int j = 0; j < CHUNK / 4; ++j)
                                *reinterpret_cast<float4*>(yst + lane * (CHUNK * 4) + j * 16) =
                                    make_float4(yv[4 * j], yv[4 * j + 1], yv[4 * j + 2], yv[4 * j + 3]);
                        } else {
                            uint32_t hw[CHUNK / 2];
#pragma unroll
                            for (int j = 0; j < CHUNK / 2; ++j) {
                                if (P.y_dtype == IMA_DTYPE_BF16) {
                                    __nv_bfloat162 b2 = __floats2bfloat162_rn(yv[2 * j], yv[2 * j + 1]);
                                    hw[j] = *reinterpret_cast<uint32_t*>(&b2);
                                } else {
                                    __half2 f2 = __floats2half2_rn(yv[2 * j], yv[2 * j + 1]);
                                    hw[j] = *reinterpret_cast<uint32_t*>(&f2);
                                }
                            }
#pragma unroll
                            for (int j = 0; j < CHUNK / 8; ++j)
                                *reinterpret_cast<uint4*>(yst + lane * (CHUNK * 2) + j * 16) =
                                    make_uint4(hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]);
                        }
                    }
                    __syncwarp();
                    // copy-out: each instruction writes 32 / SLOTS rows of C (lanes read their
                    // row's 16-byte slots back through the swizzle) and 16 or 8 rows of y
                    const int64_t rbase = (int64_t)m0 + q * 32;
                    const int64_t cbase = (int64_t)n0 + c0;
                    if (P.c) {
#pragma unroll
                        for (int it = 0; it < SLOTS; ++it) {
                            const int r = it * (32 / SLOTS) + lane / SLOTS, j = lane % SLOTS;
                            const int64_t gm = rbase + r, gn = cbase + 2 * j;
                            const uint4 v =
                                *reinterpret_cast<const uint4*>(cst + r * (SLOTS * 16) + ((j ^ (r % SLOTS)) << 4));
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
                        const int row_bytes = CHUNK * esize;
                        const int lanes_per_row = row_bytes / 16;
                        const int rows_per_it = 32 / lanes_per_row;
                        for (int it = 0; it < 32 / rows_per_it; ++it) {
                            const int r = it * rows_per_it + lane / lanes_per_row;
                            const int part = lane % lanes_per_row;
                            const int64_t gm = rbase + r;
                            const int64_t gn = cbase + part * (16 / esize);
                            const uint4 v = *reinterpret_cast<const uint4*>(yst + r * row_bytes + part * 16);
                            if (gm < P.M && gn < P.N) {
                                const int64_t off = (gm * P.ldy + gn) * esize;
                                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
                                // y, then each further copy of it (another GPU's gathered
                                // buffer: plain stores over NVLink), starting at a different
                                // copy in each CTA so that the CTAs spread over the destinations
                                for (int d = -1; d < P.ncopy; ++d) {
                                    const int dc = d < 0 ? 0 : (int)((d + blockIdx.x) % (uint32_t)P.ncopy);
                                    unsigned char* dst =
                                        reinterpret_cast<unsigned char*>(d < 0 ? P.y : batch.ycopy[pi][dc]) + off;
                                    if (gn + 16 / esize <= P.N) {
                                        *reinterpret_cast<uint4*>(dst) = v;
                                    } else if (esize == 4) {
#pragma unroll
                                        for (int e = 0; e < 4; ++e)
                                            if (gn + e < P.N) reinterpret_cast<uint32_t*>(dst)[e] = w4[e];
                                    } else {
#pragma unroll
                                        for (int e = 0; e < 8; ++e)
                                            if (gn + e < P.N)
                                                reinterpret_cast<uint16_t*>(dst)[e] =
                                                    (uint16_t)(w4[e >> 1] >> (16 * (e & 1)));
                                    }
                                }
                            }
                        }
                    }
                } else if (row_ok) {
#pragma unroll
                    for (int j = 0; j < CHUNK; ++j) {
                        const int64_t n = n0 + c0 + j;
                        if (n >= P.N) break;
                        if (P.c) P.c[m * P.ldc + n] = (int64_t)cval[j];
                        if (P.y) {
                            for (int d = -1; d < P.ncopy; ++d) {
                                void* yd = d < 0 ? P.y : batch.ycopy[pi][d];
                                if (P.y_dtype == IMA_DTYPE_F32)
                                    reinterpret_cast<float*>(yd)[m * P.ldy + n] = yv[j];
                                else if (P.y_dtype == IMA_DTYPE_BF16)
                                    reinterpret_cast<__nv_bfloat16*>(yd)[m * P.ldy + n] = __float2bfloat16_rn(yv[j]);
                                else
                                    reinterpret_cast<__half*>(yd)[m * P.ldy + n] = __float2half_rn(yv[j]);
                            }
                        }
                    }
                }
            }
        }
    }
    // copies of y written into other GPUs' memory are visible there once the launch is complete
    if (batch.has_copies) __threadfence_system();
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

// 3-D map over planes [P][rows][ld] int8 with a {64 B, box_rows, 1} box, 64-byte swizzle.
int make_plane_map(CUtensorMap* map, const int8_t* base, int64_t ld, int64_t rows, int planes, int box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return IMA_ERR_CUDA;
    cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)ld, (cuuint64_t)(ld * rows)};
    cuuint32_t box[3] = {(cuuint32_t)GM_KT, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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

// Upper bound on the persistent GEMM grid (0: every SM); see ima_set_gemm_sm_limit.
int g_gemm_sm_limit = 0;
// Test knob of ima_set_gemm_wait_test: length of the stall wait (0: off).
uint64_t g_gemm_stall_ns = 0;

int gemm_grid_limit() {
    const int n = num_sms();
    return (g_gemm_sm_limit > 0 && g_gemm_sm_limit < n) ? g_gemm_sm_limit : n;
}

// Row tiles per tile group: as many as keep the group's activation planes (GM_BM rows x K
// bytes x NP planes) within GM_GROUP_BYTES of L2, a power of two in [2, 32].
constexpr int64_t GM_GROUP_BYTES = 64ll << 20;
int32_t gemm_group_m(int64_t K, int np) {
    const int64_t per_tile = (int64_t)GM_BM * std::max<int64_t>(K, 1) * np;
    int32_t g = 2;
    while (g < 32 && (int64_t)(2 * g) * per_tile <= GM_GROUP_BYTES) g *= 2;
    return g;
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
    if (scheme == IMA_SCHEME_DIGITS3 && q.K > 174000) return IMA_ERR_UNSUPPORTED;
    if (scheme == IMA_SCHEME_DIGITS5 && q.K > 100000) return IMA_ERR_UNSUPPORTED;
    return IMA_OK;
}

template <int SCHEME>
int launch_batch(GemmBatch& b, cudaStream_t stream) {
    using L = GemmCfg<SCHEME>;
    auto kern = int_gemm_kernel<SCHEME>;
    int rc = ima_note_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
    if (rc != IMA_OK) return rc;
    int64_t tiles = b.tile_start[b.n];
    if (tiles == 0) return IMA_OK;
    const int limit = gemm_grid_limit();
    int grid = (int)(tiles < limit ? tiles : limit);
    kern<<<grid, GM_THREADS, L::ALLOC, stream>>>(b);
    return IMA_LAUNCH_STATUS();
}

template <int SCHEME>
int run_grouped(const ima_gemm_problem* problems, const ima_gemm_y_copies* copies, int count, cudaStream_t stream) {
    using L = GemmCfg<SCHEME>;
    struct Item { int idx; int64_t cost; };
    std::vector<Item> items;
    for (int i = 0; i < count; ++i) {
        const ima_gemm_problem& q = problems[i];
        if (q.M <= 0 || q.N <= 0) continue;
        const int64_t tiles = ((q.M + GM_BM - 1) / GM_BM) * ((q.N + L::BN - 1) / L::BN);
        items.push_back({i, tiles * ((q.K + GM_KT - 1) / GM_KT + 4)});
    }
    // largest cost first; greedy assignment to the launch with the least work keeps launches balanced
    std::stable_sort(items.begin(), items.end(), [](const Item& a, const Item& b) { return a.cost > b.cost; });
    const size_t nb = (items.size() + GM_MAXP - 1) / GM_MAXP;
    std::vector<std::vector<int>> groups(nb);
    std::vector<int64_t> load(nb, 0);
    for (const Item& it : items) {
        size_t best = 0;
        for (size_t g = 1; g < nb; ++g)
            if (groups[best].size() >= (size_t)GM_MAXP || (groups[g].size() < (size_t)GM_MAXP && load[g] < load[best]))
                best = g;
        groups[best].push_back(it.idx);
        load[best] += it.cost;
    }
    static thread_local GemmBatch b;   // host staging of the kernel parameters (copied at launch)
    for (size_t g = 0; g < nb; ++g) {
        memset(&b, 0, sizeof(b));
        int32_t tiles = 0;
        for (int idx : groups[g]) {
            const ima_gemm_problem& q = problems[idx];
            const int k = b.n;
            GemmProblemDev& D = b.p[k];
            int rc = make_plane_map(&b.maps[k][0], q.a_planes, q.lda, q.M, L::NP, GM_BM);
            if (rc != IMA_OK) return rc;
            rc = make_plane_map(&b.maps[k][1], q.b_planes, q.ldb, q.N, L::NP, L::BN);
            if (rc != IMA_OK) return rc;
            D.c = q.c; D.y = q.y; D.xs = q.x_scale; D.ws = q.w_scale; D.bias = q.bias;
            D.ldc = q.ldc; D.ldy = q.ldy;
            D.M = (int32_t)q.M; D.N = (int32_t)q.N; D.K = (int32_t)q.K; D.y_dtype = q.y_dtype;
            D.m_tiles = (int32_t)((q.M + GM_BM - 1) / GM_BM);
            D.N_tile = L::BN;
            D.group_m = gemm_group_m(q.K, L::NP);
            D.k_tiles = (int32_t)((q.K + GM_KT - 1) / GM_KT);
            // staged 16-byte copy-out needs 16-byte aligned rows; otherwise element stores
            const int yes = q.y_dtype == IMA_DTYPE_F32 ? 4 : 2;
            bool vec = true;
            if (q.c) vec = vec && !(reinterpret_cast<uintptr_t>(q.c) & 15) && !((q.ldc * 8) & 15);
            if (q.y) vec = vec && !(reinterpret_cast<uintptr_t>(q.y) & 15) && !((q.ldy * yes) & 15);
            D.ncopy = 0;
            if (copies && q.y) {
                for (int d = 0; d < GM_MAXD; ++d) {
                    void* yc = copies[idx].y[d];
                    if (!yc) continue;
                    vec = vec && !(reinterpret_cast<uintptr_t>(yc) & 15);
                    b.ycopy[k][D.ncopy++] = yc;
                }
                if (D.ncopy) b.has_copies = 1;
            }
            D.vec_out = vec ? 1 : 0;
            b.tile_start[k] = tiles;
            tiles += D.m_tiles * (int32_t)((q.N + L::BN - 1) / L::BN);
            b.n = k + 1;
        }
        b.tile_start[b.n] = tiles;
        b.stall_ns = g_gemm_stall_ns;
        int rc = launch_batch<SCHEME>(b, stream);
        if (rc != IMA_OK) return rc;
    }
    return IMA_OK;
}

}  // namespace

extern "C" int ima_set_gemm_wait_test(int64_t stall_ns) {
    if (stall_ns < 0 || stall_ns > (int64_t)IMA_WAIT_LIMIT_NS) return IMA_ERR_INVALID_ARGUMENT;
    g_gemm_stall_ns = (uint64_t)stall_ns;
    return IMA_OK;
}

extern "C" int ima_set_gemm_sm_limit(int sms) {
    if (sms < 0) return IMA_ERR_INVALID_ARGUMENT;
    g_gemm_sm_limit = sms;
    return IMA_OK;
}

extern "C" int ima_int_gemm_grouped_copies(const ima_gemm_problem* problems, const ima_gemm_y_copies* copies,
                                           int count, int scheme, void* stream) {
    if (count < 0 || (count > 0 && !problems)) return IMA_ERR_INVALID_ARGUMENT;
    if (scheme != IMA_SCHEME_DIGITS3 && scheme != IMA_SCHEME_DIGITS5) return IMA_ERR_UNSUPPORTED;
    for (int i = 0; i < count; ++i) {
        int rc = check_problem(problems[i], scheme);
        if (rc != IMA_OK) return rc;
        if (copies && !problems[i].y) {
            for (int d = 0; d < GM_MAXD; ++d)
                if (copies[i].y[d]) return IMA_ERR_INVALID_ARGUMENT;   // copies of a y that is not written
        }
    }
    if (scheme == IMA_SCHEME_DIGITS3)
        return run_grouped<IMA_SCHEME_DIGITS3>(problems, copies, count, (cudaStream_t)stream);
    return run_grouped<IMA_SCHEME_DIGITS5>(problems, copies, count, (cudaStream_t)stream);
}

extern "C" int ima_int_gemm_grouped(const ima_gemm_problem* problems, int count, int scheme, void* stream) {
    return ima_int_gemm_grouped_copies(problems, nullptr, count, scheme, stream);
}

extern "C" int ima_int_gemm(const int8_t* a_planes, int64_t lda, const int8_t* b_planes, int64_t ldb, int64_t M,
                            int64_t N, int64_t K, int scheme, int64_t* c, int64_t ldc, const float* x_scale,
                            const float* w_scale, const float* bias, void* y, int y_dtype, int64_t ldy,
                            void* stream) {
    ima_gemm_problem q = {a_planes, lda, b_planes, ldb, M, N, K, c, ldc, x_scale, w_scale, bias, y, y_dtype, ldy};
    return ima_int_gemm_grouped(&q, 1, scheme, stream);
}
