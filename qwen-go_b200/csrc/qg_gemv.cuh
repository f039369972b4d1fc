// Weight decoding shared by the CUDA-core expert kernels (qg_gemv.cu) and the
// decode kernels (qg_decode.cu): 16-byte chunks of float32, raw bf16, int8
// or packed int4 weights to float32 (quantLinear.dequantize without the
// scale, model/moe.go:134-157; bf16f32, model/model.go:113-115), the
// lane-interleaved staging of activation rows, and silu.
#pragma once
#include "qg_common.cuh"

namespace qg {

// Elements carried by one 16-byte weight chunk.
template <int BITS>
struct Chunk {
    static constexpr int V = BITS == 32 ? 4 : BITS == 16 ? 8 : (BITS == 8 ? 16 : 32);
};

// int8 x4 -> float x4 exactly: bias to unsigned, splice under 2^23, subtract.
__device__ __forceinline__ void i8x4(uint32_t w, float *f) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.f;
    f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.f;
    f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.f;
    f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.f;
}

// 4 packed bytes = 8 int4 codes -> float x8 (code - 8), element order
// hi(b0), lo(b0), hi(b1), lo(b1), ...
__device__ __forceinline__ void i4x8(uint32_t w, float *f) {
    const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;
    const uint32_t lo = w & 0x0F0F0F0Fu;
    f[0] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540)) - 8388616.f;
    f[1] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540)) - 8388616.f;
    f[2] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7541)) - 8388616.f;
    f[3] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7541)) - 8388616.f;
    f[4] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7542)) - 8388616.f;
    f[5] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7542)) - 8388616.f;
    f[6] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7543)) - 8388616.f;
    f[7] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7543)) - 8388616.f;
}

template <int BITS>
__device__ __forceinline__ void decode_chunk(uint4 raw, float *v) {
    if constexpr (BITS == 32) {
        v[0] = __uint_as_float(raw.x);
        v[1] = __uint_as_float(raw.y);
        v[2] = __uint_as_float(raw.z);
        v[3] = __uint_as_float(raw.w);
    } else if constexpr (BITS == 16) {
        // bf16f32 (model/model.go:113-115): the bits as the high half of a float32
        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[2 * i] = __uint_as_float(w4[i] << 16);
            v[2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
        }
    } else if constexpr (BITS == 8) {
        i8x4(raw.x, v);
        i8x4(raw.y, v + 4);
        i8x4(raw.z, v + 8);
        i8x4(raw.w, v + 12);
    } else {
        i4x8(raw.x, v);
        i4x8(raw.y, v + 8);
        i4x8(raw.z, v + 16);
        i4x8(raw.w, v + 24);
    }
}

// Floats a staged row of K inputs occupies: whole rounds of 32 chunks.
__host__ __device__ __forceinline__ int kpad_for(int K, int V) {
    return ((K / V + 31) / 32) * 32 * V;
}

// Position (in floats) of element (chunk c, offset j) of a staged row, so
// that lane (c % 32) reading float4 j/4 of iteration c/32 is conflict-free.
template <int V>
__device__ __forceinline__ int stage_pos(int c, int j) {
    return (((c >> 5) * (V / 4) + (j >> 2)) * 32 + (c & 31)) * 4 + (j & 3);
}

__device__ __forceinline__ float silu_ref(float g) {
    // g / (1 + float32(exp(-float64(g))))   (model/tensors.go:93)
    return __fdiv_rn(g, __fadd_rn(1.f, (float)exp(-(double)g)));
}

}  // namespace qg
