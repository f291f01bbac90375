#pragma once

// 16-bit tensor-core operands (tcgen05 kind::f16): weights and activations
// are stored as raw 16-bit words in one of two formats, fp16 or bf16, chosen
// per model and carried beside the pointers as a flag (the GEMM turns it into
// the MMA instruction descriptor's A/B format; both operands of one MMA must
// share it). fp16 keeps 11 significant bits against bf16's 8 at the same 2
// bytes per element, so float32 packs run their fast path in fp16; bfloat16
// packs keep their own bf16 values.
//
// Activations are two-term: x = hi + lo with hi = r(x), lo = r(x - hi), r
// rounding to nearest even in the chosen format.

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace opworks::detail {

__device__ __forceinline__ uint16_t to16(float x, bool f16) {
    return f16 ? __half_as_ushort(__float2half_rn(x)) : __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float from16(uint16_t v, bool f16) {
    return f16 ? __half2float(__ushort_as_half(v)) : __bfloat162float(__ushort_as_bfloat16(v));
}
// (a, b) rounded to the format and packed, a in the low half (the element
// order of two consecutive columns in memory)
__device__ __forceinline__ uint32_t pack16x2(float a, float b, bool f16) {
    if (f16) {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    }
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ float2 unpack16x2(uint32_t v, bool f16) {
    if (f16)
        return __half22float2(*reinterpret_cast<const __half2 *>(&v));
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&v));
}

} // namespace opworks::detail
