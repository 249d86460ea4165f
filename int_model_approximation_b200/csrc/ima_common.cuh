// Shared device/host helpers for the B200 student-linear kernels.
//
// Everything here is sm_100a-only: the library is compiled with
// -gencode arch=compute_100a,code=sm_100a and nothing else.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>
#include <mutex>

#include "../../include/ima_b200.h"

#define IMA_DEVINL __device__ __forceinline__

// ---------------------------------------------------------------------------
// Device-side error word.  Kernels never trap: on a bad state (a bounded wait
// that ran out, an index outside the tensor) they record a code in a per-device
// status word and return.  The host reads it with ima_device_status().
// ---------------------------------------------------------------------------
struct ImaDeviceStatus {
    int code;    // first IMA_ERR_* recorded since the last reset
    int where;   // kernel-specific location tag
    int detail;  // kernel-specific detail (e.g. a stage index)
    int pad;
};

// One status word per device.  The library is built as a single translation unit
// (ima_b200.cu includes every kernel file), so this definition is unique.
__device__ ImaDeviceStatus g_ima_status;

IMA_DEVINL void ima_record_error(int code, int where, int detail) {
    if (atomicCAS(&g_ima_status.code, 0, code) == 0) {
        g_ima_status.where = where;
        g_ima_status.detail = detail;
    }
}

// Where-tags for ima_record_error.
enum ImaWhere {
    IMA_WHERE_PLANES = 1,
    IMA_WHERE_GEMM_PRODUCER = 2,
    IMA_WHERE_GEMM_MMA = 3,
    IMA_WHERE_GEMM_EPILOGUE = 4,
    IMA_WHERE_CLASS_COUNTS = 5,
};

// Host-side helper: record the CUDA error of the last call for ima_last_cuda_error().
int ima_note_cuda(cudaError_t e);
#define IMA_LAUNCH_STATUS() ima_note_cuda(cudaGetLastError())

// Nanosecond wall clock of the GPU (used to bound every spin-wait).
IMA_DEVINL uint64_t ima_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Upper bound for any spin-wait inside a kernel (2 s): far above any legal
// wait, far below anything that would look like a hung GPU.
#define IMA_WAIT_LIMIT_NS 2000000000ull

// ---------------------------------------------------------------------------
// fp32 -> e4m3fn with round-to-nearest-even, matching torch's
// Tensor.to(torch.float8_e4m3fn): magnitudes >= 480 (and inf/NaN) become the
// NaN code 0x7F, the sign bit is kept.  Written from the IEEE definitions.
// ---------------------------------------------------------------------------
IMA_DEVINL uint8_t ima_f32_to_e4m3(float f) {
    uint32_t bits = __float_as_uint(f);
    uint32_t sign = (bits >> 24) & 0x80u;
    uint32_t a = bits & 0x7FFFFFFFu;
    uint32_t code;
    if (a >= 0x43F00000u) {            // |f| >= 480, inf or NaN
        code = 0x7Fu;
    } else if (a < 0x3C800000u) {      // |f| < 2^-6: e4m3 subnormal grid 2^-9
        float v = __uint_as_float(a) * 512.0f;   // exact power-of-two scaling
        code = __float2uint_rn(v);               // RNE onto 0..8 (8 = smallest normal)
    } else {
        uint32_t e = (a >> 23) - 120u;           // rebias 127 -> 7
        uint32_t m = a & 0x7FFFFFu;
        uint32_t q = (e << 3) | (m >> 20);
        uint32_t rem = m & 0xFFFFFu;
        if (rem > 0x80000u || (rem == 0x80000u && (q & 1u))) q += 1u;
        code = q;                                // a carry may reach 0x7F (NaN) like torch
    }
    return (uint8_t)(code | sign);
}

// Exact codebook value round(fp8 * 512) of an e4m3 byte: sign * sig * 2^(max(E,1)-1).
// The NaN codes (0x7F / 0xFF) map to 0, which is what CUDA's float->int32
// conversion of NaN gives for the reference's (x.float() * 512).round().to(int32).
IMA_DEVINL int32_t ima_e4m3_codebook(uint32_t b) {
    uint32_t e = (b >> 3) & 15u, m = b & 7u;
    if (e == 15u && m == 7u) return 0;
    int32_t sig = (int32_t)(e ? (m | 8u) : m);
    int32_t v = sig << ((e ? e : 1u) - 1u);
    return (b & 0x80u) ? -v : v;
}

// Balanced base-128 digits of a codebook value |v| <= 1,064,960: v = d0 + 128 d1 + 16384 d2,
// d0, d1 in [-64, 63].
IMA_DEVINL void ima_digits3(int32_t v, int32_t& d0, int32_t& d1, int32_t& d2) {
    d0 = ((v + 64) & 127) - 64;
    int32_t v1 = (v - d0) >> 7;
    d1 = ((v1 + 64) & 127) - 64;
    d2 = (v1 - d1) >> 7;
}

IMA_DEVINL float ima_bf16_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
