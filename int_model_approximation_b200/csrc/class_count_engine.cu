// Class-count engine: the Freivalds-checkable count products of the hawkeye-class-counts
// student formed on tcgen05 tensor cores and replayed, in the same kernel, into the Hawkeye
// accumulator.
//
// ref: hawkeye_freivalds.py:1017-1246 (exact_hawkeye_fp8_sum), :860-1014 (packed groups),
// :147-213 and :593-704 (the count products), :329-412 (K5, count product and replay in one
// kernel: the model of this engine), :464-545 / :707-790 (K6/K7, the replay from counts).
// Per group of 32 k the reference forms
//     count[a, b, m, n] = #{k in the group : class(x[m,k]) = a, class(w[n,k]) = b}
// as integer products A_flat @ B_flat (A_flat[(a, m), k] = [class(x[m,k]) = a], B_flat the
// class indicators of the weights, optionally packed in base-64 lanes) and replays
//     T = aligned(acc) + sum_{a,b} count[a,b,m,n] * trunc0((s_a s_b << 7) >> (maxe - e_a - e_b + 14)),
// then normalises T to the 14-bit accumulator, group after group.
//
// Which products are formed.  Row (a, m) of A_flat is zero unless class a occurs in token m's
// group, and a group has 32 k, so a token row has at most 32 classes per group (likewise each
// weight row).  The engine forms exactly the rows and columns that can be nonzero: token row m
// contributes 32 "slot" rows (its classes in first-occurrence order, unused slots all-zero),
// weight row n 32 slot columns.  One tcgen05.mma of M = 128 (4 tokens x 32 slots), N = 256 (8
// weight rows x 32 slots), K = 32 (one group) puts the count of every (a, b) class pair of 32
// outputs into tensor memory.  Every nonzero lane of every product the reference forms is
// such a count; the entries left out are zero by construction.  The weight one-hot carries the
// class's sign (+1 / -1, int8), so a TMEM entry is the count times the weight class's sign.
//
// Fused replay.  An epilogue thread owns one slot row (token m, class a) and walks the 32
// slot columns of a weight row n: with fa = |s_a| 2^e_a, fb = |s_b| 2^e_b and S = maxe + 7,
//     bits(fma_rz(fa, fb, M_S)) = bits(M_S) + floor(fa fb / 2^S),    M_S = 1.5 * 2^(23+S)
// (the product stays in the binade whose ulp is 2^S), so the thread accumulates
// part = sum_b c_ab * bits(fma_rz(fa, fb, M_S)) with one FFMA.RZ and one IMAD per count.  The
// 32 slot rows of a token are the 32 lanes of one warp: one REDUX adds sgn_a * part over them,
// and the bits(M_S) offsets come out as bits(M_S) * (npos - nneg), the signed number of
// present products of the output, known from the operands' masks.  The accumulator update is
// then the direct replay's (hawkeye.cu), bit for bit.
//
// Freivalds fingerprint of every count tile.  Before a tile's counts are discarded, each
// thread forms sum_col c[row, col] r[col] over the columns it read and compares it with
// (A (B^T r))[row] over the same columns, computed from the operands, r = (r1 + 2^16 r2) with r1, r2 seeded per tile in [1, 15]: a product the
// tensor cores got wrong fails the check (any single wrong count always; several wrong counts
// cancel in both 16-bit halves with probability about 1/225).  Failed rows are counted in a
// device word the caller reads.
//
// Modes for tests and offload: `tiles_out` receives every count tile as the tensor cores
// formed it; `tiles_in` makes the epilogue replay (and check) counts supplied by the caller
// instead of the tensor-memory ones.
//
// CTA (one per SM, persistent over "strips" of 4 tokens x 64 weight rows, all groups):
//   warp 0     TMEM allocation (512 columns: two 256-column count tiles) and MMA issue
//   warp 1     loader: bulk copies of each unit's operands (the weight tile record of
//              ima_class_count_weight_tiles -- one-hot weight slot rows in the 64-byte swizzle,
//              class magnitudes, fingerprint weights -- and the tokens' and weight rows' staged
//              records) into one of four unit buffers, up to four units ahead
//   warps 2-3  builders: the one-hot token slot rows per group pair, and each output's
//              present-exponent maximum and signed present count per unit
//   warps 4-19 epilogue: warp (q = warp % 4, part) reads TMEM lanes 32q.. (token q of the
//              strip) and the count columns of 2 of the 8 weight rows of a tile; lane j < 16
//              keeps the accumulator of one output (tile j / 2)
// Every mbarrier wait is bounded and abort-aware; the MMA thread drains its work before the
// CTA frees tensor memory.
#include "sm100_primitives.cuh"

namespace {

constexpr int CE_GROUP = 32;
constexpr int CE_TM = 4;                       // token rows per MMA tile: 4 x 32 slot rows = M 128
constexpr int CE_TN = 8;                       // weight rows per MMA tile: 8 x 32 slot rows = N 256
constexpr int CE_TN_CONST = CE_TN;
constexpr int CE_MAX_TILES = 8;                // MMA tiles per strip
constexpr int CE_STRIP_N = CE_TN * CE_MAX_TILES;
constexpr int CE_PITCH = 64;                   // staged rows are padded to a multiple of this
constexpr int CE_BUILD_WARPS = 2;
constexpr int CE_EPI_WARPS = 16;                // four per TMEM lane quadrant
constexpr int CE_PARTS = CE_EPI_WARPS / 4;      // column parts of a tile, one per warp of a quadrant
constexpr int CE_NLW = CE_TN_CONST / CE_PARTS;  // weight rows per epilogue warp and tile
constexpr int CE_BUILDERS = 32 * CE_BUILD_WARPS;
constexpr int CE_FIRST_EPI_WARP = 2 + CE_BUILD_WARPS;   // warp 0 MMA, warp 1 loader, then builders
constexpr int CE_THREADS = 32 * (CE_FIRST_EPI_WARP + CE_EPI_WARPS);
constexpr uint32_t CE_TMEM_COLS = 512;
constexpr int CE_ABSENT_EXP = -8192;
constexpr uint32_t CE_NO_SLOT = 0xFFu;
constexpr int CE_WHERE = 6;                    // where-tag of this kernel's bounded waits
constexpr int CE_UNITS = 4;                    // unit buffers in shared memory (the loader runs ahead)

// Weight tile record (ima_class_count_weight_tiles), one per (8 weight rows, group pair),
// copied into shared memory unchanged by one bulk copy:
constexpr int CE_R_B = 0;                      // one-hot weight slot rows [256][64 B], 64-byte swizzle
constexpr int CE_R_FB = 256 * 64;              // f32 [2 h][256]: |s| 2^e of each slot column's class
constexpr int CE_R_RR = CE_R_FB + 2 * 256 * 4; // u32 [2][256]: fingerprint weights r1 + 2^16 r2
constexpr int CE_R_BR = CE_R_RR + 2 * 256 * 4; // s8 [2 h][CE_PARTS][2 vec][32 k]: B^T r per column part
constexpr int CE_RECORD = CE_R_BR + 2 * CE_PARTS * 2 * 32;
// unit buffer in shared memory: the weight record, then the per-unit staging and tables
constexpr int CE_U_EXB = CE_RECORD;                    // u32 [2 h][8][16] exponent pairs of the 8 weight rows
constexpr int CE_U_PSB = CE_U_EXB + 2 * CE_TN * 64;    // uint4 [2][8] masks
constexpr int CE_U_SLA = CE_U_PSB + 2 * CE_TN * 16;    // u8 [2][4][32] token slots
constexpr int CE_U_CTA = CE_U_SLA + 2 * CE_TM * 32;    // u8 [2][4][32] token class codes
constexpr int CE_U_EXA = CE_U_CTA + 2 * CE_TM * 32;    // u32 [2][4][16]
constexpr int CE_U_PSA = CE_U_EXA + 2 * CE_TM * 64;    // uint4 [2][4]
constexpr int CE_U_PE = CE_U_PSA + 2 * CE_TM * 16;     // i32 [2 h][32 outputs]: largest present exponent sum
constexpr int CE_U_PN = CE_U_PE + 2 * 32 * 4;          // i32 [2][32]: signed present-product count
constexpr int CE_U_END = CE_U_PN + 2 * 32 * 4;
constexpr int CE_UNIT_BYTES = ((CE_U_END + 1023) / 1024) * 1024;   // 24576: each B tile 1024-aligned
constexpr int CE_STAGED_BYTES = CE_U_PE - CE_RECORD;                // bytes of the per-unit bulk copies
constexpr int CE_A_BYTES = 128 * 64;                   // one-hot token slot rows, both groups
constexpr int CE_OFF_U = 0;
constexpr int CE_OFF_A = CE_OFF_U + CE_UNITS * CE_UNIT_BYTES;      // [2]
constexpr int CE_OFF_FA = CE_OFF_A + 2 * CE_A_BYTES;               // f32 [2 buf][2 h][128]
constexpr int CE_OFF_BAR = CE_OFF_FA + 2 * 2 * 128 * 4;
// barriers: s_full[U], b_full[U], b_empty[U], a_full[2], a_empty[2], t_full[2], t_empty[2], drained
constexpr int CE_NBAR = 3 * CE_UNITS + 9;
constexpr int CE_TOTAL = CE_OFF_BAR + CE_NBAR * 8 + 16;
constexpr int CE_ALLOC = CE_TOTAL + 1024;
static_assert(CE_RECORD % 16 == 0 && CE_U_EXB % 16 == 0 && CE_U_PSA % 16 == 0, "bulk copies need 16-byte alignment");

struct CeOperand {
    uint8_t* sl;
    uint8_t* ct;
    uint32_t* ex;
    uint4* ps;
    int64_t pitch, groups;
};

__host__ __device__ inline int64_t ce_pitch(int64_t rows) { return ((rows + CE_PITCH - 1) / CE_PITCH) * CE_PITCH; }
__host__ __device__ inline int64_t ce_groups(int64_t K) { return (K + CE_GROUP - 1) / CE_GROUP; }

__host__ __device__ inline CeOperand ce_operand(const void* base, int64_t rows, int64_t K) {
    CeOperand op;
    op.pitch = ce_pitch(rows);
    op.groups = ce_groups(K);
    const int64_t recs = op.pitch * op.groups;
    uint8_t* p = const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(base));
    op.sl = p;
    op.ct = p + recs * 32;
    op.ex = reinterpret_cast<uint32_t*>(p + recs * 64);
    op.ps = reinterpret_cast<uint4*>(p + recs * 128);
    return op;
}

// One warp per (row, group): lane = k.  Classes are identified by their e4m3 code (a code
// with a nonzero significand determines its class (e - 1) * 31 + (s + 15) and back).
__global__ void __launch_bounds__(256) ce_prepare_kernel(const uint8_t* __restrict__ src, int64_t rows, int64_t K,
                                                         int64_t ld, CeOperand op) {
    const unsigned FULL = 0xFFFFFFFFu;
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int64_t g = blockIdx.y;
    if (r >= op.pitch) return;                        // whole warps only
    const int64_t k = g * CE_GROUP + lane;
    const uint32_t b = (r < rows && k < K) ? (uint32_t)src[r * ld + k] : 0u;
    const uint32_t eb = (b >> 3) & 15u, mant = b & 7u;
    const uint32_t sig = eb ? (mant | 8u) : mant;
    const bool present = sig != 0;
    const unsigned peers = __match_any_sync(FULL, present ? b : (0x100u + (unsigned)lane));
    const int leader = __ffs(peers) - 1;
    const bool is_leader = present && leader == lane;
    const unsigned leaders = __ballot_sync(FULL, is_leader);
    const unsigned nslots = __popc(leaders);
    const unsigned own_slot = __popc(leaders & ((1u << lane) - 1u));   // meaningful on leaders
    const unsigned slot = __shfl_sync(FULL, own_slot, leader);
    const unsigned slot_sign = __reduce_or_sync(FULL, (is_leader && (b & 0x80u)) ? (1u << own_slot) : 0u);
    const int64_t rec = g * op.pitch + r;
    op.sl[rec * 32 + lane] = present ? (uint8_t)slot : (uint8_t)CE_NO_SLOT;
    if (is_leader) op.ct[rec * 32 + own_slot] = (uint8_t)b;
    if ((unsigned)lane >= nslots) op.ct[rec * 32 + lane] = 0;
    const int e = present ? (eb ? (int)eb : 1) : CE_ABSENT_EXP;
    const int e_next = __shfl_down_sync(FULL, e, 1);
    if ((lane & 1) == 0) op.ex[rec * 16 + (lane >> 1)] = ((uint32_t)e & 0xFFFFu) | ((uint32_t)e_next << 16);
    const unsigned pres = __ballot_sync(FULL, present);
    const unsigned sgn = __ballot_sync(FULL, present && (b & 0x80u));
    if (lane == 0) op.ps[rec] = make_uint4(pres, sgn, slot_sign, nslots);
}

// |s| 2^e of an e4m3 code as an exact fp32 value (0 for a zero code).
IMA_DEVINL float ce_magnitude(uint32_t code) {
    const uint32_t eb = (code >> 3) & 15u, mant = code & 7u;
    const uint32_t sig = eb ? (mant | 8u) : mant;
    return (float)(sig << (eb ? eb : 1u));
}

// Seeded fingerprint weights r1, r2 in [1, 15] of count column `col` of a tile, packed r1 + 2^16 r2.
IMA_DEVINL uint32_t ce_fingerprint_weight(uint64_t seed, uint64_t tile, uint32_t col) {
    uint32_t h = (uint32_t)seed ^ (uint32_t)(seed >> 32) ^ (uint32_t)(tile * 0x9E3779B97F4A7C15ull >> 32) ^
                 (col * 0x85EBCA6Bu);
    h ^= h >> 15;
    h *= 0x2C1B3C6Du;
    h ^= h >> 12;
    h *= 0x297A2D39u;
    h ^= h >> 15;
    return (1u + (h & 0xFFFFu) % 15u) | ((1u + (h >> 16) % 15u) << 16);
}

// One 16-byte chunk (16 k) of a one-hot slot row: byte = `one` where slot byte == s, else 0.
IMA_DEVINL uint4 ce_onehot_chunk(uint4 slots, uint32_t s, uint32_t one) {
    const uint32_t pat = s * 0x01010101u;
    uint32_t w[4] = {slots.x ^ pat, slots.y ^ pat, slots.z ^ pat, slots.w ^ pat};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        // exact per-byte zero test: 0x80 in the bytes that are zero, no carries between bytes
        const uint32_t z = ~(((w[j] & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | w[j] | 0x7F7F7F7Fu);
        w[j] = (z >> 7) * one;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Byte offset of (row, 16-byte chunk c) in a K-major tile of 64-byte rows with the 64-byte
// swizzle (the layout a TMA SWIZZLE_64B load writes and umma_desc_sw64_kmajor describes).
IMA_DEVINL uint32_t ce_sw64(uint32_t row, uint32_t c) { return row * 64u + ((c ^ ((row >> 1) & 3u)) << 4); }
// Weight tile records: for each 8 weight rows `nt` and group pair `gp`, the one-hot weight
// slot rows (carrying the class sign) in the layout the MMA reads, the slot columns' class
// magnitudes, the fingerprint weights and B^T r.  They depend on the weight alone, so they
// are built once per weight (one block per record).
__global__ void __launch_bounds__(256) ce_weight_tiles_kernel(CeOperand B, int64_t GP, uint64_t seed,
                                                            unsigned char* __restrict__ out) {
    const int64_t nt = blockIdx.x, gp = blockIdx.y;
    unsigned char* rec = out + (nt * GP + gp) * (int64_t)CE_RECORD;
    const int64_t n0 = nt * CE_TN, G = B.groups;
    for (int i = threadIdx.x; i < 256 * 4; i += blockDim.x) {
        const uint32_t row = (uint32_t)(i >> 2), c = (uint32_t)(i & 3);
        const uint32_t h = c >> 1, nl = row >> 5, s = row & 31u;
        const int64_t g = 2 * gp + h;
        uint4 sl = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
        uint32_t one = 1u;
        if (g < G) {
            const int64_t r = g * B.pitch + n0 + nl;
            sl = *reinterpret_cast<const uint4*>(B.sl + r * 32 + (c & 1u) * 16);
            one = ((B.ps[r].z >> s) & 1u) ? 0xFFu : 1u;
        }
        *reinterpret_cast<uint4*>(rec + CE_R_B + ce_sw64(row, c)) = ce_onehot_chunk(sl, s, one);
    }
    float* FB = reinterpret_cast<float*>(rec + CE_R_FB);
    uint32_t* RR = reinterpret_cast<uint32_t*>(rec + CE_R_RR);
    const uint64_t tile = (uint64_t)(nt * GP + gp);
    for (int i = threadIdx.x; i < 2 * 256; i += blockDim.x) {
        const int h = i >> 8, col = i & 255;
        const int64_t g = 2 * gp + h;
        const uint32_t code = g < G ? B.ct[(g * B.pitch + n0 + (col >> 5)) * 32 + (col & 31)] : 0u;
        FB[i] = ce_magnitude(code);
        RR[i] = ce_fingerprint_weight(seed, tile * 2 + h, (uint32_t)col);
    }
    int8_t* BR = reinterpret_cast<int8_t*>(rec + CE_R_BR);
    for (int i = threadIdx.x; i < 2 * CE_PARTS * 32; i += blockDim.x) {
        const int h = i / (CE_PARTS * 32), part = (i >> 5) % CE_PARTS, k = i & 31;
        const int64_t g = 2 * gp + h;
        int s1 = 0, s2 = 0;
        if (g < G) {
            for (int nl = part * CE_NLW; nl < part * CE_NLW + CE_NLW; ++nl) {
                const int64_t r = g * B.pitch + n0 + nl;
                const uint32_t slot = B.sl[r * 32 + k];
                if (slot == CE_NO_SLOT) continue;
                const uint32_t rr = ce_fingerprint_weight(seed, tile * 2 + h, (uint32_t)(nl * 32 + slot));
                const bool neg = (B.ps[r].z >> slot) & 1u;
                s1 += neg ? -(int)(rr & 0xFFFFu) : (int)(rr & 0xFFFFu);
                s2 += neg ? -(int)(rr >> 16) : (int)(rr >> 16);
            }
        }
        BR[((h * CE_PARTS + part) * 2 + 0) * 32 + k] = (int8_t)s1;
        BR[((h * CE_PARTS + part) * 2 + 1) * 32 + k] = (int8_t)s2;
    }
}

struct CeParams {
    CeOperand a, b;
    const unsigned char* w_tiles;
    const float* xs;
    const float* ws;
    int64_t M, N, groups, strips_m, strips_n;
    __nv_bfloat16* out_bf16;
    int64_t ld_bf16;
    float* out_f32;
    int64_t ld_f32;
    int32_t* mismatch;
    int32_t* tiles_out;
    const int32_t* tiles_in;
};

// mbarrier try_wait that may suspend the thread (up to 20 us, or until the phase completes)
// instead of spinning, so waiting warps leave their issue slots to the warps that work.
IMA_DEVINL bool ce_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}

// Bounded, abort-aware wait (as mbar_wait_or_abort) built on the suspending try_wait.
IMA_DEVINL bool ce_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t limit_ns, int detail) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = ima_globaltimer();
    while (!ce_try_wait_sleep(bar, parity)) {
        if (*abort) return false;
        if (ima_globaltimer() - t0 > limit_ns) {
            ima_record_error(IMA_ERR_TIMEOUT, CE_WHERE, detail);
            *abort = 1;
            return false;
        }
    }
    return true;
}

// Position of a CTA's work: strip `sid` (stride gridDim.x), group pair `gp`, tile `t` of the strip.
struct CeCursor {
    int64_t sid, gp;
    int t, tiles;
    bool valid;
};

IMA_DEVINL int ce_strip_tiles(const CeParams& P, int64_t sid) {
    const int64_t n0 = (sid / P.strips_m) * CE_STRIP_N;
    return (int)min((int64_t)CE_MAX_TILES, (P.N - n0 + CE_TN - 1) / CE_TN);
}

IMA_DEVINL CeCursor ce_cursor_first(const CeParams& P, int64_t strips) {
    CeCursor c;
    c.sid = blockIdx.x;
    c.gp = 0;
    c.t = 0;
    c.valid = c.sid < strips;
    c.tiles = c.valid ? ce_strip_tiles(P, c.sid) : 0;
    return c;
}

IMA_DEVINL void ce_cursor_next(CeCursor& c, const CeParams& P, int64_t strips, int64_t GP) {
    if (++c.t < c.tiles) return;
    c.t = 0;
    if (++c.gp < GP) return;
    c.gp = 0;
    c.sid += gridDim.x;
    c.valid = c.sid < strips;
    c.tiles = c.valid ? ce_strip_tiles(P, c.sid) : 0;
}

// 1-D bulk copy global -> shared, completion counted on an mbarrier (no multicast).
IMA_DEVINL void ce_bulk_copy(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Stage the unit at `c` into a unit buffer: the weight tile record, and for both groups of the
// pair the 8 weight rows' exponent pairs and masks and the 4 tokens' slots, codes, exponent
// pairs and masks (all 16-byte aligned).
IMA_DEVINL void ce_stage_unit(const CeParams& P, const CeCursor& c, int64_t GP, unsigned char* dst, uint64_t* bar) {
    const int64_t m0 = (c.sid % P.strips_m) * CE_TM;
    const int64_t ntile = (c.sid / P.strips_m) * CE_MAX_TILES + c.t;
    const int64_t nt = ntile * CE_TN;
    const int live = (2 * c.gp + 1 < P.groups) ? 2 : 1;
    mbar_arrive_expect_tx(bar, (uint32_t)(CE_RECORD + live * (CE_STAGED_BYTES / 2)));
    ce_bulk_copy(dst, P.w_tiles + (ntile * GP + c.gp) * (int64_t)CE_RECORD, CE_RECORD, bar);
    for (int h = 0; h < live; ++h) {
        const int64_t g = 2 * c.gp + h;
        const int64_t rb = g * P.b.pitch + nt, ra = g * P.a.pitch + m0;
        ce_bulk_copy(dst + CE_U_EXB + h * CE_TN * 64, P.b.ex + rb * 16, CE_TN * 64, bar);
        ce_bulk_copy(dst + CE_U_PSB + h * CE_TN * 16, P.b.ps + rb, CE_TN * 16, bar);
        ce_bulk_copy(dst + CE_U_SLA + h * CE_TM * 32, P.a.sl + ra * 32, CE_TM * 32, bar);
        ce_bulk_copy(dst + CE_U_CTA + h * CE_TM * 32, P.a.ct + ra * 32, CE_TM * 32, bar);
        ce_bulk_copy(dst + CE_U_EXA + h * CE_TM * 64, P.a.ex + ra * 16, CE_TM * 64, bar);
        ce_bulk_copy(dst + CE_U_PSA + h * CE_TM * 16, P.a.ps + ra, CE_TM * 16, bar);
    }
}
static_assert(CE_STAGED_BYTES == 2 * (CE_TN * 64 + CE_TN * 16 + CE_TM * 32 * 2 + CE_TM * 64 + CE_TM * 16),
              "the per-unit copies fill the staging area exactly");

// tcgen05.wait::ld that also names the 16 registers the last tcgen05.ld wrote, so that the
// compiler cannot schedule a use of them before the wait.
IMA_DEVINL void ce_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// 16 supplied counts of one tile row (tiles_in layout, include/ima_b200.h).
IMA_DEVINL void ce_load_supplied(const int32_t* tiles, int64_t tile_id, int row, int col0, uint32_t (&c)[16]) {
    const int4* src = reinterpret_cast<const int4*>(tiles + (tile_id * 128 + row) * 256 + col0);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        const int4 x = src[v];
        c[4 * v] = (uint32_t)x.x;
        c[4 * v + 1] = (uint32_t)x.y;
        c[4 * v + 2] = (uint32_t)x.z;
        c[4 * v + 3] = (uint32_t)x.w;
    }
}

// MODE: CE_TENSOR_COUNTS (normal), CE_DUMP_TILES (also write every count tile to tiles_out),
// CE_SUPPLIED_TILES (replay and check the counts in tiles_in instead of the tensor-memory ones).
enum { CE_TENSOR_COUNTS = 0, CE_DUMP_TILES = 1, CE_SUPPLIED_TILES = 2 };

template <int MODE>
__global__ void __launch_bounds__(CE_THREADS, 1) class_count_replay_kernel(const __grid_constant__ CeParams P) {
    extern __shared__ __align__(1024) unsigned char ce_raw[];
    // align to 1024 bytes by pointer arithmetic on the shared array itself, so that every
    // access below stays a shared-memory access (not a generic one)
    unsigned char* smem = ce_raw + ((1024u - (smem_u32(ce_raw) & 1023u)) & 1023u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CE_OFF_BAR);
    uint64_t* s_full = bars;                        // [U] loader's copies landed (expect_tx)
    uint64_t* b_full = bars + CE_UNITS;             // [U] builders' per-unit tables ready
    uint64_t* b_empty = bars + 2 * CE_UNITS;        // [U] MMA commit + epilogue warps: unit buffer free
    uint64_t* a_full = bars + 3 * CE_UNITS;         // [2] one-hot token rows built
    uint64_t* a_empty = a_full + 2;                 // [2] MMA commit + epilogue warps
    uint64_t* t_full = a_full + 4;                  // [2] count tile in tensor memory
    uint64_t* t_empty = a_full + 6;                 // [2] epilogue warps read it
    uint64_t* drained = a_full + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + CE_NBAR);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t G = P.groups;
    const int64_t GP = (G + 1) / 2;
    const int64_t strips = P.strips_m * P.strips_n;

    if (threadIdx.x == 0) {
        for (int i = 0; i < CE_UNITS; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&b_full[i], CE_BUILDERS);
            mbar_init(&b_empty[i], 1 + CE_EPI_WARPS);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&a_full[i], CE_BUILDERS);
            mbar_init(&a_empty[i], 1 + CE_EPI_WARPS);
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], CE_EPI_WARPS);
        }
        mbar_init(drained, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, CE_TMEM_COLS);
        tmem_relinquish();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint64_t LIMIT = IMA_WAIT_LIMIT_NS;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = idesc_i8(128, 256);
            uint64_t a_cnt = 0, u = 0;
            bool ok = true;
            for (int64_t sid = blockIdx.x; sid < strips && ok; sid += gridDim.x) {
                const int tiles = ce_strip_tiles(P, sid);
                for (int64_t gp = 0; gp < GP && ok; ++gp) {
                    const uint32_t abuf = (uint32_t)(a_cnt & 1u), aph = (uint32_t)((a_cnt >> 1) & 1u);
                    ++a_cnt;
                    ok = ce_wait(&a_full[abuf], aph, abort_flag, LIMIT, 1);
                    for (int t = 0; t < tiles && ok; ++t) {
                        const uint32_t slot = (uint32_t)(u % CE_UNITS), sph = (uint32_t)((u / CE_UNITS) & 1u);
                        const uint32_t tph = (uint32_t)(u & 1u);   // each tensor-memory tile is used once per unit
                        ++u;
                        ok = ce_wait(&s_full[slot], sph, abort_flag, LIMIT, 2);
                        for (int h = 0; h < 2 && ok; ++h) {
                            ok = ce_wait(&t_empty[h], tph ^ 1u, abort_flag, LIMIT, 3);
                            if (!ok) break;
                            tc_fence_after();
                            const uint32_t sa = smem_u32(smem + CE_OFF_A + abuf * CE_A_BYTES) + h * 32;
                            const uint32_t sb = smem_u32(smem + CE_OFF_U + slot * CE_UNIT_BYTES + CE_R_B) + h * 32;
                            mma_i8(tmem_base + (uint32_t)(h * 256), umma_desc_sw64_kmajor(sa), umma_desc_sw64_kmajor(sb),
                                   idesc, 0u);
                            mma_commit(&t_full[h]);
                        }
                        if (ok) mma_commit(&b_empty[slot]);
                    }
                    if (ok) mma_commit(&a_empty[abuf]);
                }
            }
            // every MMA issued completes before tensor memory is freed
            mma_commit(drained);
            mbar_wait_bounded(drained, 0u, CE_WHERE, 9);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- loader: bulk copies of each unit's operands, up to CE_UNITS ahead ----
            CeCursor c = ce_cursor_first(P, strips);
            uint64_t v = 0;
            bool ok = true;
            while (c.valid && ok) {
                const uint32_t slot = (uint32_t)(v % CE_UNITS), ph = (uint32_t)((v / CE_UNITS) & 1u);
                ok = ce_wait(&b_empty[slot], ph ^ 1u, abort_flag, LIMIT, 10);
                if (!ok) break;
                ce_stage_unit(P, c, GP, smem + CE_OFF_U + slot * CE_UNIT_BYTES, &s_full[slot]);
                ++v;
                ce_cursor_next(c, P, strips, GP);
            }
            // every bulk copy issued has landed before the CTA can exit
            for (uint64_t s = 0; s < CE_UNITS; ++s) {
                if (v > s) {
                    const uint64_t last = v - 1 - ((v - 1 - s) % CE_UNITS);   // last unit staged into slot s
                    mbar_wait_bounded(&s_full[s], (uint32_t)((last / CE_UNITS) & 1u), CE_WHERE, 12);
                }
            }
            if (!ok) *abort_flag = 1;
        }
    } else if (warp < CE_FIRST_EPI_WARP) {
        // ---------------- builders: one-hot token rows per group pair, per-output tables ----
        const int tb = threadIdx.x - 64;
        float* FA = reinterpret_cast<float*>(smem + CE_OFF_FA);
        CeCursor c = ce_cursor_first(P, strips);
        uint64_t u = 0, a_cnt = 0;
        bool ok = true;
        while (c.valid && ok) {
            const uint32_t slot = (uint32_t)(u % CE_UNITS), sph = (uint32_t)((u / CE_UNITS) & 1u);
            ok = ce_wait(&s_full[slot], sph, abort_flag, LIMIT, 11);
            if (!ok) break;
            unsigned char* U = smem + CE_OFF_U + slot * CE_UNIT_BYTES;
            const int64_t gp = c.gp;
            if (c.t == 0) {
                const uint32_t abuf = (uint32_t)(a_cnt & 1u), aph = (uint32_t)((a_cnt >> 1) & 1u);
                ++a_cnt;
                ok = ce_wait(&a_empty[abuf], aph ^ 1u, abort_flag, LIMIT, 4);
                if (!ok) break;
                const uint8_t* SLA = U + CE_U_SLA;
                const uint8_t* CTA = U + CE_U_CTA;
                unsigned char* As = smem + CE_OFF_A + abuf * CE_A_BYTES;
                for (int i = tb; i < 2 * 128; i += CE_BUILDERS) {
                    const int h = i >> 7, row = i & 127;
                    const uint32_t code = 2 * gp + h < G ? CTA[(h * CE_TM + (row >> 5)) * 32 + (row & 31)] : 0u;
                    const float mag = ce_magnitude(code);
                    FA[(abuf * 2 + h) * 128 + row] = (code & 0x80u) ? -mag : mag;
                }
                for (int i = tb; i < 128 * 4; i += CE_BUILDERS) {
                    const uint32_t row = (uint32_t)(i >> 2), cc = (uint32_t)(i & 3);   // 8 rows x 4 chunks per warp store
                    const uint32_t h = cc >> 1;
                    uint4 sl = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
                    if (2 * gp + h < G)
                        sl = *reinterpret_cast<const uint4*>(SLA + (h * CE_TM + (row >> 5)) * 32 + (cc & 1u) * 16);
                    *reinterpret_cast<uint4*>(As + ce_sw64(row, cc)) = ce_onehot_chunk(sl, row & 31u, 1u);
                }
                fence_proxy_async_smem();
                mbar_arrive(&a_full[abuf]);
            }
            // each output's largest present exponent sum and signed present count
            const uint32_t* EXA = reinterpret_cast<const uint32_t*>(U + CE_U_EXA);
            const uint32_t* EXB = reinterpret_cast<const uint32_t*>(U + CE_U_EXB);
            const uint4* PSA = reinterpret_cast<const uint4*>(U + CE_U_PSA);
            const uint4* PSB = reinterpret_cast<const uint4*>(U + CE_U_PSB);
            int32_t* PE = reinterpret_cast<int32_t*>(U + CE_U_PE);
            int32_t* PN = reinterpret_cast<int32_t*>(U + CE_U_PN);
            for (int i = tb; i < 2 * 32; i += CE_BUILDERS) {
                const int h = i >> 5, o = i & 31, ml = o >> 3, nl = o & 7;
                int pe = -16384, pn = 0;
                if (2 * gp + h < G) {
                    const uint32_t* ea = EXA + (h * CE_TM + ml) * 16;
                    const uint32_t* eb = EXB + (h * CE_TN + nl) * 16;
                    uint32_t e2 = 0xC000C000u;
#pragma unroll
                    for (int j = 0; j < 16; ++j) e2 = __viaddmax_s16x2(ea[j], eb[j], e2);
                    pe = max((int)(int16_t)(e2 & 0xFFFFu), (int)(int16_t)(e2 >> 16));
                    const uint4 pa = PSA[h * CE_TM + ml], pb = PSB[h * CE_TN + nl];
                    const uint32_t both = pa.x & pb.x;
                    pn = __popc(both) - 2 * __popc(both & (pa.y ^ pb.y));
                }
                PE[i] = pe;
                PN[i] = pn;
            }
            mbar_arrive(&b_full[slot]);
            ++u;
            ce_cursor_next(c, P, strips, GP);
        }
        if (!ok) *abort_flag = 1;
    } else {
        // ---------------- epilogue: replay from the counts ----------------
        const int q = warp & 3;                      // token of the strip = TMEM lane quadrant
        const int part = (warp - CE_FIRST_EPI_WARP) >> 2;   // weight rows part*NLW .. of each tile
        const unsigned FULL = 0xFFFFFFFFu;
        const float* FA = reinterpret_cast<const float*>(smem + CE_OFF_FA);
        const int row = q * 32 + lane;               // this thread's slot row of the MMA tile
        uint64_t a_cnt = 0, u_cnt = 0;
        bool ok = true;
        for (int64_t sid = blockIdx.x; sid < strips && ok; sid += gridDim.x) {
            const int64_t m0 = (sid % P.strips_m) * CE_TM;
            const int64_t n0 = (sid / P.strips_m) * CE_STRIP_N;
            const int tiles = (int)min((int64_t)CE_MAX_TILES, (P.N - n0 + CE_TN - 1) / CE_TN);
            float acc = 0.0f;   // lane j < 8 NLW: output (m0 + q, n0 + 8 (j / NLW) + NLW part + j % NLW)
            for (int64_t gp = 0; gp < GP && ok; ++gp) {
                const uint32_t abuf = a_cnt & 1u, aph = (a_cnt >> 1) & 1u;
                ++a_cnt;
                ok = ce_wait(&a_full[abuf], aph, abort_flag, LIMIT, 6);
                if (!__all_sync(FULL, ok)) { ok = false; break; }
                for (int t = 0; t < tiles && ok; ++t) {
                    const uint32_t slot = (uint32_t)(u_cnt % CE_UNITS), sph = (uint32_t)((u_cnt / CE_UNITS) & 1u);
                    const uint32_t tph = (uint32_t)(u_cnt & 1u);
                    ++u_cnt;
                    ok = ce_wait(&b_full[slot], sph, abort_flag, LIMIT, 7);
                    ok = ok && ce_wait(&s_full[slot], sph, abort_flag, LIMIT, 7);   // the record's bytes are visible
                    if (!__all_sync(FULL, ok)) { ok = false; break; }
                    const unsigned char* U = smem + CE_OFF_U + slot * CE_UNIT_BYTES;
                    for (int h = 0; h < 2; ++h) {
                        const int64_t g = 2 * gp + h;
                        ok = ce_wait(&t_full[h], tph, abort_flag, LIMIT, 8);
                        __syncwarp();
                        if (!__all_sync(FULL, ok)) { ok = false; break; }
                        tc_fence_after();
                        // M_S of this warp's NLW outputs of the tile (owner lanes NLW t ..)
                        const int own_i = lane % CE_NLW;
                        const int own_o = q * 8 + CE_NLW * part + own_i;
                        const float* FB = reinterpret_cast<const float*>(U + CE_R_FB) + h * 256;
                        const uint32_t* RR = reinterpret_cast<const uint32_t*>(U + CE_R_RR) + h * 256;
                        const int8_t* BR = reinterpret_cast<const int8_t*>(U + CE_R_BR) + h * CE_PARTS * 64;
                        const int32_t* PE = reinterpret_cast<const int32_t*>(U + CE_U_PE) + h * 32;
                        const int32_t* PN = reinterpret_cast<const int32_t*>(U + CE_U_PN) + h * 32;
                        const int pe = PE[own_o];
                        const int acc_e14 = (int)((__float_as_uint(acc) << 1) >> 24) - 133;
                        const uint32_t ms_own = (uint32_t)max(pe, acc_e14) * (1u << 23) + ((143u << 23) | 0x400000u);
                        uint32_t ms[CE_NLW];
#pragma unroll
                        for (int i = 0; i < CE_NLW; ++i) ms[i] = __shfl_sync(FULL, ms_own, t * CE_NLW + i);
                        const float fa = FA[(abuf * 2 + h) * 128 + row];
                        const float fa_abs = fabsf(fa);
                        uint32_t psum[CE_NLW], fp = 0;
#pragma unroll
                        for (int i = 0; i < CE_NLW; ++i) psum[i] = 0u;
                        const int64_t tile_id = (((sid * GP + gp) * CE_MAX_TILES + t) * 2 + h);
                        // 2 NLW chunks of 16 count columns (weight row NLW part + (chunk >> 1), slots
                        // 16 (chunk & 1) ..): the tensor-memory load of chunk j + 1 is in flight
                        // while chunk j is replayed
                        constexpr int CHUNKS = 2 * CE_NLW, PCOLS = 256 / CE_PARTS;
                        const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 256 + part * PCOLS);
                        uint32_t ca[16], cb[16];
                        if constexpr (MODE == CE_SUPPLIED_TILES) {
                            ce_load_supplied(P.tiles_in, tile_id, row, part * PCOLS, ca);
                        } else {
                            tmem_ld16(trow, ca);
                            ce_wait_ld(ca);
                        }
#pragma unroll
                        for (int chunk = 0; chunk < CHUNKS; ++chunk) {
                            uint32_t (&cur)[16] = (chunk & 1) ? cb : ca;
                            uint32_t (&nxt)[16] = (chunk & 1) ? ca : cb;
                            if (chunk < CHUNKS - 1) {
                                if constexpr (MODE == CE_SUPPLIED_TILES)
                                    ce_load_supplied(P.tiles_in, tile_id, row, part * PCOLS + (chunk + 1) * 16, nxt);
                                else
                                    tmem_ld16(trow + (uint32_t)((chunk + 1) * 16), nxt);
                            }
                            const int col0 = part * PCOLS + chunk * 16;
                            if constexpr (MODE == CE_DUMP_TILES) {
                                int4* dst = reinterpret_cast<int4*>(P.tiles_out + (tile_id * 128 + row) * 256 + col0);
#pragma unroll
                                for (int v = 0; v < 4; ++v)
                                    dst[v] = make_int4((int)cur[4 * v], (int)cur[4 * v + 1], (int)cur[4 * v + 2],
                                                       (int)cur[4 * v + 3]);
                            }
                            const float msf = __uint_as_float(ms[chunk >> 1]);
                            const float4* fb4 = reinterpret_cast<const float4*>(FB + col0);
                            const uint4* rr4 = reinterpret_cast<const uint4*>(RR + col0);
                            uint32_t acc_c = 0;
#pragma unroll
                            for (int v = 0; v < 4; ++v) {
                                const float4 fb = fb4[v];
                                const uint4 rr = rr4[v];
                                acc_c += cur[4 * v] * __float_as_uint(__fmaf_rz(fa_abs, fb.x, msf));
                                acc_c += cur[4 * v + 1] * __float_as_uint(__fmaf_rz(fa_abs, fb.y, msf));
                                acc_c += cur[4 * v + 2] * __float_as_uint(__fmaf_rz(fa_abs, fb.z, msf));
                                acc_c += cur[4 * v + 3] * __float_as_uint(__fmaf_rz(fa_abs, fb.w, msf));
                                fp += cur[4 * v] * rr.x + cur[4 * v + 1] * rr.y + cur[4 * v + 2] * rr.z +
                                      cur[4 * v + 3] * rr.w;
                            }
                            psum[chunk >> 1] += acc_c;
                            if constexpr (MODE != CE_SUPPLIED_TILES) {
                                if (chunk < CHUNKS - 1) ce_wait_ld(nxt);
                            }
                        }
                        // the counts are in registers: hand the tensor-memory tile back
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&t_empty[h]);
                        if (g >= G) continue;                 // padding group of an odd group count
                        // fingerprint: this row of the tile against (A (B^T r))[row]
                        {
                            const unsigned char* As = smem + CE_OFF_A + abuf * CE_A_BYTES;
                            const uint4 a0 = *reinterpret_cast<const uint4*>(As + ce_sw64((uint32_t)row, 2 * h));
                            const uint4 a1 = *reinterpret_cast<const uint4*>(As + ce_sw64((uint32_t)row, 2 * h + 1));
                            const uint4* br1 = reinterpret_cast<const uint4*>(BR + (part * 2 + 0) * 32);
                            const uint4* br2 = reinterpret_cast<const uint4*>(BR + (part * 2 + 1) * 32);
                            const uint4 x0 = br1[0], x1 = br1[1], y0 = br2[0], y1 = br2[1];
                            int e1 = 0, e2 = 0;
                            e1 = __dp4a((int)a0.x, (int)x0.x, e1); e1 = __dp4a((int)a0.y, (int)x0.y, e1);
                            e1 = __dp4a((int)a0.z, (int)x0.z, e1); e1 = __dp4a((int)a0.w, (int)x0.w, e1);
                            e1 = __dp4a((int)a1.x, (int)x1.x, e1); e1 = __dp4a((int)a1.y, (int)x1.y, e1);
                            e1 = __dp4a((int)a1.z, (int)x1.z, e1); e1 = __dp4a((int)a1.w, (int)x1.w, e1);
                            e2 = __dp4a((int)a0.x, (int)y0.x, e2); e2 = __dp4a((int)a0.y, (int)y0.y, e2);
                            e2 = __dp4a((int)a0.z, (int)y0.z, e2); e2 = __dp4a((int)a0.w, (int)y0.w, e2);
                            e2 = __dp4a((int)a1.x, (int)y1.x, e2); e2 = __dp4a((int)a1.y, (int)y1.y, e2);
                            e2 = __dp4a((int)a1.z, (int)y1.z, e2); e2 = __dp4a((int)a1.w, (int)y1.w, e2);
                            const uint32_t expect = (uint32_t)e1 + ((uint32_t)e2 << 16);
                            if (fp != expect) atomicAdd(P.mismatch, 1);
                        }
                        // sum sgn_a * psum over the 32 slot rows of the token: one REDUX per weight row
                        const uint32_t neg = fa < 0.0f ? 0xFFFFFFFFu : 0u;
                        uint32_t total = 0;
#pragma unroll
                        for (int i = 0; i < CE_NLW; ++i) {
                            const uint32_t tot = __reduce_add_sync(FULL, (psum[i] ^ neg) - neg);
                            if (own_i == i) total = tot;
                        }
                        if (lane / CE_NLW == t) {
                            const uint32_t m = ms_own;
                            const int pn = PN[own_o];
                            const uint32_t amask = (uint32_t)((int32_t)__float_as_uint(acc) >> 31);
                            const uint32_t av = __float_as_uint(__fmaf_rz(fabsf(acc), 1.0f, __uint_as_float(m))) - m;
                            const uint32_t T = ((av ^ amask) - amask) + total - m * (uint32_t)pn;
                            int32_t f = (int32_t)(m - ((23u << 23) + 0x400000u));   // (S + 127) << 23
                            f = max(f, 0);
                            const float v = __fmul_rn((float)(int32_t)T, __int_as_float(f));
                            acc = __uint_as_float(__float_as_uint(v) & 0xFFFFFC00u);
                        }
                    }
                    if (!ok) break;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&b_empty[slot]);
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_empty[abuf]);
            }
            if (!ok) break;
            // outputs of the strip: gfloat = acc * 2^-20, y = (gfloat * xs) * ws
            const int64_t m = m0 + q;
            const int64_t n = n0 + 8 * (lane / CE_NLW) + CE_NLW * part + (lane % CE_NLW);
            if (lane / CE_NLW < tiles && m < P.M && n < P.N) {
                const float gf = __fmul_rn(acc, 9.5367431640625e-07f);
                const float y = __fmul_rn(__fmul_rn(gf, P.xs[m]), P.ws[n]);
                if (P.out_bf16) P.out_bf16[m * P.ld_bf16 + n] = __float2bfloat16_rn(y);
                if (P.out_f32) P.out_f32[m * P.ld_f32 + n] = y;
            }
        }
        if (!ok) *abort_flag = 1;
    }
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, CE_TMEM_COLS);
    }
}

}  // namespace

extern "C" {

int64_t ima_class_count_operand_bytes(int64_t rows, int64_t K) {
    if (rows < 0 || K < 0) return 0;
    return ce_pitch(rows) * ce_groups(K) * 144;
}

int ima_class_count_prepare(const uint8_t* fp8, int64_t rows, int64_t K, int64_t ld, void* operand, void* stream) {
    if (!fp8 || !operand || rows < 0 || K < 0 || ld < K) return IMA_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(operand) & 15) return IMA_ERR_INVALID_ARGUMENT;
    const int64_t pitch = ce_pitch(rows), groups = ce_groups(K);
    if (pitch == 0 || groups == 0) return IMA_OK;
    if (groups > 65535) return IMA_ERR_UNSUPPORTED;
    CeOperand op = ce_operand(operand, rows, K);
    dim3 grid((unsigned)(pitch / 8), (unsigned)groups);
    ce_prepare_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(fp8, rows, K, ld, op);
    return IMA_LAUNCH_STATUS();
}

int64_t ima_class_count_weight_tiles_bytes(int64_t N, int64_t K) {
    if (N <= 0 || K <= 0) return 0;
    return ((N + CE_TN - 1) / CE_TN) * ((ce_groups(K) + 1) / 2) * (int64_t)CE_RECORD;
}

int ima_class_count_weight_tiles(const void* w_operand, int64_t N, int64_t K, uint64_t seed, void* tiles,
                                 void* stream) {
    if (!w_operand || !tiles || N < 0 || K < 0) return IMA_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(w_operand) & 15) || (reinterpret_cast<uintptr_t>(tiles) & 15))
        return IMA_ERR_INVALID_ARGUMENT;
    if (N == 0 || K == 0) return IMA_OK;
    const int64_t ntiles = (N + CE_TN - 1) / CE_TN, gp = (ce_groups(K) + 1) / 2;
    if (gp > 65535) return IMA_ERR_UNSUPPORTED;
    ce_weight_tiles_kernel<<<dim3((unsigned)ntiles, (unsigned)gp), 256, 0, (cudaStream_t)stream>>>(
        ce_operand(w_operand, N, K), gp, seed, reinterpret_cast<unsigned char*>(tiles));
    return IMA_LAUNCH_STATUS();
}

int64_t ima_class_count_tile_entries(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const int64_t strips = ((M + CE_TM - 1) / CE_TM) * ((N + CE_STRIP_N - 1) / CE_STRIP_N);
    const int64_t gp = (ce_groups(K) + 1) / 2;
    return strips * gp * CE_MAX_TILES * 2 * 128 * 256;
}

int ima_class_count_replay(const void* x_operand, const void* w_operand, const void* w_tiles, const float* x_scale,
                           const float* w_scale, int64_t M, int64_t N, int64_t K, uint16_t* out_bf16, int64_t ld_bf16,
                           float* out_f32, int64_t ld_f32, int32_t* mismatch_rows, int32_t* tiles_out,
                           const int32_t* tiles_in, void* stream) {
    if (!x_operand || !w_operand || !w_tiles || !x_scale || !w_scale || !mismatch_rows || M < 0 || N < 0 || K < 0)
        return IMA_ERR_INVALID_ARGUMENT;
    if (!out_bf16 && !out_f32) return IMA_ERR_INVALID_ARGUMENT;
    if ((out_bf16 && ld_bf16 < N) || (out_f32 && ld_f32 < N)) return IMA_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(x_operand) & 15) || (reinterpret_cast<uintptr_t>(w_operand) & 15) ||
        (reinterpret_cast<uintptr_t>(w_tiles) & 15) || (reinterpret_cast<uintptr_t>(tiles_out) & 15) ||
        (reinterpret_cast<uintptr_t>(tiles_in) & 15))
        return IMA_ERR_INVALID_ARGUMENT;
    if (tiles_out && tiles_in) return IMA_ERR_INVALID_ARGUMENT;
    if (M == 0 || N == 0) return IMA_OK;
    CeParams p;
    p.a = ce_operand(x_operand, M, K);
    p.b = ce_operand(w_operand, N, K);
    p.w_tiles = reinterpret_cast<const unsigned char*>(w_tiles);
    p.xs = x_scale;
    p.ws = w_scale;
    p.M = M;
    p.N = N;
    p.groups = ce_groups(K);
    p.strips_m = (M + CE_TM - 1) / CE_TM;
    p.strips_n = (N + CE_STRIP_N - 1) / CE_STRIP_N;
    p.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
    p.ld_bf16 = ld_bf16;
    p.out_f32 = out_f32;
    p.ld_f32 = ld_f32;
    p.mismatch = mismatch_rows;
    p.tiles_out = tiles_out;
    p.tiles_in = tiles_in;
    auto kern = tiles_in ? class_count_replay_kernel<CE_SUPPLIED_TILES>
                         : tiles_out ? class_count_replay_kernel<CE_DUMP_TILES> : class_count_replay_kernel<CE_TENSOR_COUNTS>;
    int rc = ima_note_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, CE_ALLOC));
    if (rc != IMA_OK) return rc;
    if (K == 0) {
        // no products: every output is the zero accumulator
        if (out_bf16) rc = ima_note_cuda(cudaMemset2DAsync(out_bf16, ld_bf16 * 2, 0, N * 2, M, (cudaStream_t)stream));
        if (rc == IMA_OK && out_f32)
            rc = ima_note_cuda(cudaMemset2DAsync(out_f32, ld_f32 * 4, 0, N * 4, M, (cudaStream_t)stream));
        return rc;
    }
    const int64_t strips = p.strips_m * p.strips_n;
    const int grid = (int)(strips < num_sms() ? strips : num_sms());
    kern<<<grid, CE_THREADS, CE_ALLOC, (cudaStream_t)stream>>>(p);
    return IMA_LAUNCH_STATUS();
}

}  // extern "C"
