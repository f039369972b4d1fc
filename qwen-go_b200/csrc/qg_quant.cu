// QuantLinear helpers on the GPU: quantizeInt8/Int4 (bit-exact with
// model/moe.go:165-217), dequantize (model/moe.go:134-157, kernel K6),
// f32 -> fp16 scale conversion and the synthetic-input generator.
#include "qg_common.cuh"

namespace qg {

// One thread per (row, group of 32).  Division and rounding follow the Go
// code: s = amax/127 (or /7) in float32, floored at 1e-8; code =
// clamp(round_half_away(w/s)) with an IEEE float32 quotient.
__global__ void k_quantize(int bits, int O, int I, const float *__restrict__ w,
                           uint8_t *__restrict__ q, float *__restrict__ s32,
                           __half *__restrict__ s16) {
    const int ng = I / QG_GROUP;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)O * ng) return;
    const int64_t o = gid / ng;
    const int b = (int)(gid - o * ng);
    const float *src = w + o * I + (int64_t)b * QG_GROUP;
    float vals[QG_GROUP];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < QG_GROUP; j += 4) {
        float4 v = *reinterpret_cast<const float4 *>(src + j);
        vals[j] = v.x;
        vals[j + 1] = v.y;
        vals[j + 2] = v.z;
        vals[j + 3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < QG_GROUP; j++) {
        float a = fabsf(vals[j]);
        if (a > amax) amax = a;
    }
    const float qmax = bits == 8 ? 127.f : 7.f;
    float s = __fdiv_rn(amax, qmax);
    if (s < 1e-8f) s = 1e-8f;
    if (s32) s32[gid] = s;
    if (s16) s16[gid] = __float2half_rn(s);
    if (bits == 8) {
        uint32_t packed[QG_GROUP / 4];
#pragma unroll
        for (int j = 0; j < QG_GROUP / 4; j++) packed[j] = 0;
#pragma unroll
        for (int j = 0; j < QG_GROUP; j++) {
            float v = roundf(__fdiv_rn(vals[j], s));
            v = fminf(fmaxf(v, -127.f), 127.f);
            uint32_t byte = (uint32_t)(uint8_t)(int8_t)(int)v;
            packed[j / 4] |= byte << (8 * (j % 4));
        }
        uint4 *dst = reinterpret_cast<uint4 *>(q + o * I + (int64_t)b * QG_GROUP);
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    } else {
        uint32_t packed[QG_GROUP / 8];
#pragma unroll
        for (int j = 0; j < QG_GROUP / 8; j++) packed[j] = 0;
#pragma unroll
        for (int j = 0; j < QG_GROUP; j++) {
            float v = roundf(__fdiv_rn(vals[j], s));
            v = fminf(fmaxf(v, -7.f), 7.f) + 8.f;
            uint32_t nib = (uint32_t)(int)v & 0xFu;
            // byte j/2: even j -> high nibble, odd j -> low nibble
            const int byte = j / 2;
            const int shift = 8 * (byte % 4) + ((j % 2 == 0) ? 4 : 0);
            packed[byte / 4] |= nib << shift;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(q + o * (I / 2) + (int64_t)b * (QG_GROUP / 2));
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
}

int launch_quantize(int bits, int O, int I, const float *w, uint8_t *q, float *s32, __half *s16,
                    cudaStream_t s) {
    const int64_t n = (int64_t)O * (I / QG_GROUP);
    if (n == 0) return QGMOE_OK;
    const int threads = 128;
    const int64_t blocks = (n + threads - 1) / threads;
    k_quantize<<<(unsigned)blocks, threads, 0, s>>>(bits, O, I, w, q, s32, s16);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

// w[o, c] = code * scale[o, c/32] as float32 (model/moe.go:134-157).
__global__ void k_dequantize(int bits, int O, int I, const uint8_t *__restrict__ q,
                             const __half *__restrict__ s, const float *__restrict__ w32,
                             float *__restrict__ w) {
    const int64_t n = (int64_t)O * I;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (bits == 32) {
            w[i] = w32[i];
            continue;
        }
        const int64_t o = i / I;
        const int c = (int)(i - o * I);
        const float sc = __half2float(s[o * (I / QG_GROUP) + c / QG_GROUP]);
        float v;
        if (bits == 8) {
            v = (float)(int8_t)q[i];
        } else {
            const uint8_t b = q[o * (I / 2) + c / 2];
            v = (float)((c % 2 == 0) ? (b >> 4) : (b & 0xF)) - 8.f;
        }
        w[i] = __fmul_rn(v, sc);
    }
}

int launch_dequantize(int bits, int O, int I, const uint8_t *q, const __half *s, const float *w32,
                      float *w, cudaStream_t st) {
    const int64_t n = (int64_t)O * I;
    if (n == 0) return QGMOE_OK;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    k_dequantize<<<(unsigned)blocks, 256, 0, st>>>(bits, O, I, q, s, w32, w);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

// Router rows as float32 [E, H] from a bf16 (bits 16) or quantLinear (8 / 4)
// mlp.gate, exactly the values the reference multiplies by: bf16f32
// (model/model.go:113-115), or dequantize (model/moe.go:134-157):
// float32(code) * scale rounded to nearest, with fp16 scales widened (exact)
// and f32 scales used as given -- cmd/qwen-quant writes f32 scales and the
// loader keeps them (model/load.go:553-563).
__global__ void k_router_rows(int bits, int E, int H, const uint8_t *__restrict__ q,
                              const void *__restrict__ scale, int scale_f32,
                              float *__restrict__ w) {
    const int64_t n = (int64_t)E * H;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (bits == 16) {
            const uint32_t u = reinterpret_cast<const uint16_t *>(q)[i];
            w[i] = __uint_as_float(u << 16);
            continue;
        }
        const int64_t o = i / H;
        const int c = (int)(i - o * H);
        const int64_t si = o * (H / QG_GROUP) + c / QG_GROUP;
        const float sc = scale_f32 ? reinterpret_cast<const float *>(scale)[si]
                                   : __half2float(reinterpret_cast<const __half *>(scale)[si]);
        float v;
        if (bits == 8) {
            v = (float)(int8_t)q[i];
        } else {
            const uint8_t b = q[o * (H / 2) + c / 2];
            v = (float)((c % 2 == 0) ? (b >> 4) : (b & 0xF)) - 8.f;
        }
        w[i] = __fmul_rn(v, sc);
    }
}

int launch_router_rows(int bits, int E, int H, const uint8_t *q, const void *scale, int scale_f32,
                       float *w, cudaStream_t s) {
    const int64_t n = (int64_t)E * H;
    if (n == 0) return QGMOE_OK;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    k_router_rows<<<(unsigned)blocks, 256, 0, s>>>(bits, E, H, q, scale, scale_f32, w);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

__global__ void k_f32_to_f16(const float *__restrict__ in, __half *__restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(in[i]);
}

int launch_f32_to_f16(const float *in, __half *out, int64_t n, cudaStream_t s) {
    if (n == 0) return QGMOE_OK;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    k_f32_to_f16<<<(unsigned)blocks, 256, 0, s>>>(in, out, n);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

// Counter-based normal generator: splitmix64 finaliser keyed by
// (seed, stream), Box-Muller on the pair (2i, 2i+1) of uniforms in (0, 1].
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double uniform01(uint64_t key, uint64_t ctr) {
    uint64_t r = mix64(key ^ mix64(ctr));
    return ((double)(r >> 11) + 1.0) * (1.0 / 9007199254740992.0);
}

__global__ void k_randn(uint64_t key, uint64_t offset, int64_t n, float stdv, float *out) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
         j += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t i = offset + (uint64_t)j;
        const uint64_t pair = i >> 1;
        const double u1 = uniform01(key, 2 * pair);
        const double u2 = uniform01(key, 2 * pair + 1);
        const double r = sqrt(-2.0 * log(u1));
        const double z = (i & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
        out[j] = (float)(z * (double)stdv);
    }
}

static uint64_t host_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

int launch_randn(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, float stdv,
                 float *out, cudaStream_t s) {
    if (n == 0) return QGMOE_OK;
    const uint64_t key = host_mix64(host_mix64(seed) + stream * 0xD1B54A32D192ED03ULL);
    int64_t blocks = (n + 255) / 256;
    if (blocks > 65535LL * 8) blocks = 65535LL * 8;
    k_randn<<<(unsigned)blocks, 256, 0, s>>>(key, offset, n, stdv, out);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

}  // namespace qg
