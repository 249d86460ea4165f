// Hawkeye class-count bookkeeping.
//
// ref: hawkeye_freivalds.py:51-57 (_class_ids): an e4m3 element with effective
// exponent e and signed significand s belongs to class (e - 1) * 31 + (s + 15);
// zeros have no class.  Ids lie in [0, 465); 252 of them are reachable by
// non-NaN codes.
//
// ima_class_presence marks, for every pack of `pack_width` consecutive k, which
// classes occur anywhere in the operand (the reference computes the same set with
// torch.unique per pack, hawkeye_freivalds.py:906-907 / :1097-1098, one host sync
// each; here one kernel covers all packs and the host reads the bitmasks once).
#include "ima_common.cuh"

namespace {

constexpr int CC_CLASS_WORDS = 16;   // 512-bit presence mask per pack

IMA_DEVINL int class_id(uint32_t b) {
    uint32_t eb = (b >> 3) & 15u, mant = b & 7u;
    int sig = (int)(eb ? (mant | 8u) : mant);
    if (sig == 0) return -1;
    int e = eb ? (int)eb : 1;
    int s = (b & 0x80u) ? -sig : sig;
    return (e - 1) * 31 + (s + 15);
}

// grid: (row blocks, packs); each block ORs its rows' classes of one pack into smem,
// then merges into the global mask with atomicOr.
__global__ void __launch_bounds__(256) class_presence_kernel(const uint8_t* __restrict__ src, int64_t rows,
                                                             int64_t K, int64_t ld, int64_t pack_width,
                                                             uint32_t* __restrict__ masks) {
    __shared__ uint32_t s_mask[CC_CLASS_WORDS];
    if (threadIdx.x < CC_CLASS_WORDS) s_mask[threadIdx.x] = 0;
    __syncthreads();
    const int64_t pack = blockIdx.y;
    const int64_t k0 = pack * pack_width;
    const int64_t k1 = k0 + pack_width < K ? k0 + pack_width : K;
    const int64_t width = k1 - k0;
    const int64_t rows_per_block = 64;
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
    const int64_t r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
    for (int64_t i = threadIdx.x; i < (r1 - r0) * width; i += blockDim.x) {
        int64_t r = r0 + i / width, k = k0 + i % width;
        int c = class_id(src[r * ld + k]);
        if (c >= 0) atomicOr(&s_mask[c >> 5], 1u << (c & 31));
    }
    __syncthreads();
    if (threadIdx.x < CC_CLASS_WORDS) {
        uint32_t v = s_mask[threadIdx.x];
        if (v) atomicOr(&masks[pack * CC_CLASS_WORDS + threadIdx.x], v);
    }
}

}  // namespace

extern "C" {

int ima_class_presence(const uint8_t* fp8, int64_t rows, int64_t K, int64_t ld, int64_t pack_width, uint32_t* masks,
                       void* stream) {
    if (!fp8 || !masks || rows < 0 || K < 0 || ld < K || pack_width <= 0) return IMA_ERR_INVALID_ARGUMENT;
    int64_t packs = (K + pack_width - 1) / pack_width;
    if (packs == 0) return IMA_OK;
    cudaStream_t s = (cudaStream_t)stream;
    int rc = ima_note_cuda(cudaMemsetAsync(masks, 0, (size_t)packs * CC_CLASS_WORDS * 4, s));
    if (rc != IMA_OK || rows == 0) return rc;
    if (packs > 65535) return IMA_ERR_UNSUPPORTED;
    dim3 grid((unsigned)((rows + 63) / 64), (unsigned)packs);
    class_presence_kernel<<<grid, 256, 0, s>>>(fp8, rows, K, ld, pack_width, masks);
    return IMA_LAUNCH_STATUS();
}

}  // extern "C"
