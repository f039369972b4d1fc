// Per-token routing shared by the router kernels (qg_route.cu) and the
// decode kernels (qg_decode.cu): softmax exactly as model/tensors.go:106-121
// and the top-k of model/moe.go:44-63, one warp per token.
#pragma once
#include "qg_common.cuh"

namespace qg {

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

// Larger prob, then lower index: the order a stable descending insertion
// sort produces.
__device__ __forceinline__ void better(float &v, int &i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

// float32(exp(float64(v - mx))), the softmax numerator (model/tensors.go:116).
__device__ __forceinline__ float sm_num(float v, float mx) {
    return (float)exp((double)__fsub_rn(v, mx));
}

// Warp-wide best (larger value, then lower expert index) over the lane's
// values v[j] (expert lane + 32 j) whose bit is set in `usable`.
template <int NJ>
__device__ __forceinline__ void warp_best(const float (&v)[NJ], unsigned usable, int lane,
                                          float &bv, int &bi) {
    bv = -INFINITY;
    bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < NJ; j++)
        if ((usable >> j) & 1u) better(bv, bi, v[j], lane + 32 * j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(FULL, bv, o);
        const int i2 = __shfl_xor_sync(FULL, bi, o);
        better(bv, bi, v2, i2);
    }
}

// One token's routing from its float32 logits lrow[0..E) (every logit the
// reference's own value): max by `x > mx` (fmaxf skips NaN as `x > mx` does,
// a NaN in lrow[0] stays), numerators float32(exp(float64(v - mx))), their
// float32 sum in index order, probabilities numerator / sum -- the
// reference's softmax bit for bit -- then TOPK (probability descending, ties
// to the lower index: the insertion sort over all experts) or the literal
// PREFIX bound (only experts 0..k-1 ordered), and w = p / (wSum + 1e-9) with
// wSum summed in rank order (model/moe.go:53-63).  A NaN anywhere makes
// every probability NaN; no comparison then succeeds and the selection is
// 0..k-1, as in the reference.  Lane l owns experts l, l+32, ... (NJ =
// ceil(E/32) rounded up to a power of two).  Writes the selected experts in
// rank order to sel[0..k) (shared memory of this warp) and returns, in lane
// r < k, the rank-r weight.
template <int NJ>
__device__ __forceinline__ float route_token(const float *__restrict__ lrow, int E, int k, int mode,
                                             int lane, int *sel) {
    unsigned valid = 0;
    float v[NJ];
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int e = lane + 32 * j;
        if (e < E) valid |= 1u << j;
        v[j] = e < E ? lrow[e] : -INFINITY;
    }
    // mx = v[0]; for x in v[1:]: if x > mx { mx = x }: fmaxf skips NaN
    // as `x > mx` does, and a NaN in v[0] stays
    const float v0 = __shfl_sync(FULL, v[0], 0);
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < NJ; j++)
        if ((valid >> j) & 1u) m = fmaxf(m, v[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, o));
    const float mx = isnan(v0) ? v0 : m;
    float p[NJ];
#pragma unroll
    for (int j = 0; j < NJ; j++) p[j] = ((valid >> j) & 1u) ? sm_num(v[j], mx) : 0.f;
    // float32 sum in index order (every lane forms the same sum)
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; j++)
#pragma unroll
        for (int l = 0; l < 32; l++) {
            const float u = __shfl_sync(FULL, p[j], l);
            if (l + 32 * j < E) sum = __fadd_rn(sum, u);
        }
#pragma unroll
    for (int j = 0; j < NJ; j++) p[j] = ((valid >> j) & 1u) ? __fdiv_rn(p[j], sum) : -1.f;
    float selp = 0.f;  // lane r < k: probability of the rank-r expert
    if (isnan(sum)) {
        // every probability NaN: no comparison succeeds, the order stays 0..k-1
        const float pr = __shfl_sync(FULL, p[0], lane < k ? lane : 0);
        if (lane < k) {
            sel[lane] = lane;
            selp = pr;
        }
    } else if (mode == QGMOE_ROUTER_TOPK) {
        // rank r: the largest remaining probability, ties to the lower
        // expert -- one warp max over the probabilities' bits (p >= 0, so
        // the bits order like the values), then one warp min over the
        // experts that hold it
        unsigned usable = valid;
        for (int r = 0; r < k; r++) {
            unsigned lkey = 0u;
            int lj = -1;
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if ((usable >> j) & 1u) {
                    const unsigned key = __float_as_uint(p[j]) | 0x80000000u;
                    if (lj < 0 || key > lkey) lkey = key, lj = j;  // equal: lower j kept
                }
            const unsigned top = __reduce_max_sync(FULL, lj >= 0 ? lkey : 0u);
            const unsigned bi = __reduce_min_sync(
                FULL, (lj >= 0 && lkey == top) ? (unsigned)(lane + 32 * lj) : 0xFFFFFFFFu);
            if ((int)(bi & 31u) == lane) usable &= ~(1u << (bi >> 5));
            if (lane == r) selp = __uint_as_float(top & 0x7FFFFFFFu);
            if (lane == 0) sel[r] = (int)bi;
        }
    } else {
        // PREFIX: the literal moe.go:49 bound orders only experts 0..k-1
        // (k <= 32, so expert q < k is p[0] of lane q): insertion sort
        const float pq = p[0];
        float pk[QG_MAX_TOPK];
#pragma unroll
        for (int q = 0; q < QG_MAX_TOPK; q++) pk[q] = __shfl_sync(FULL, pq, q);
        if (lane == 0) {
            int ik[QG_MAX_TOPK];
            for (int q = 0; q < k; q++) ik[q] = q;
            for (int a2 = 1; a2 < k && a2 < E; a2++)
                for (int b2 = a2; b2 > 0 && pk[ik[b2]] > pk[ik[b2 - 1]]; b2--) {
                    const int ti = ik[b2];
                    ik[b2] = ik[b2 - 1];
                    ik[b2 - 1] = ti;
                }
            for (int q = 0; q < k; q++) sel[q] = ik[q];
        }
        __syncwarp();
        const int myexp = lane < k ? sel[lane] : 0;
        const float got = __shfl_sync(FULL, pq, myexp);
        if (lane < k) selp = got;
    }
    __syncwarp();
    // wSum over ranks in rank order, then w = p / (wSum + 1e-9)
    float wsum = 0.f;
    for (int r = 0; r < k; r++) wsum = __fadd_rn(wsum, __shfl_sync(FULL, selp, r));
    const float den = __fadd_rn(wsum, 1e-9f);
    return __fdiv_rn(selp, den);
}

}  // namespace qg
