// Grouped expert products on CUDA cores (kernels K3/K4/K5 for decode-sized
// token counts) and the weighted combine (K4 epilogue).
//
// Reference arithmetic: gate_up matvec (model/moe.go:64-69), SwiGLU
// g/(1+exp(-g)) * u (model/moe.go:70-76, model/tensors.go:91-95), down
// matvec (model/moe.go:77-81), out += w*d in rank order (model/moe.go:82-85),
// shared expert down(silu(gate x) * up x) gated by sigmoid (model/moe.go:
// 86-97, model/model.go:350-358).  Quantised weights are dequantised in
// registers as they stream in: int8 code * fp16 group scale, or int4 nibble
// (hi nibble = even element, stored +8) * scale (model/moe.go:134-157).
//
// Work decomposition: a persistent grid walks (active group, 32-row block)
// items.  A group is one routed expert with its tokens, or the shared expert
// with all T tokens.  Each CTA stages up to NT input rows of the group in
// shared memory (in a lane-interleaved order so every warp read is a
// conflict-free 512-byte LDS.128 sweep), then each warp streams whole weight
// rows with 128-bit loads (16 B per lane), FMAs them against the NT staged
// rows and reduces with warp shuffles.
#include "qg_common.cuh"
#include "qg_gemv.cuh"

namespace qg {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int GEMV_ROWS = 8;   // output rows per work item (1 per warp)
constexpr int GEMV_UNR = 4;    // 16-byte chunks per lane loaded ahead
constexpr int GEMV_NT = 4;     // tokens staged per pass

// Dot products of NR weight rows (gate and up for GATEUP) against the staged
// rows: acc[r][t] += row_r . x_t.  Each lane takes chunks lane, lane+32, ...;
// the loads of up to GEMV_UNR chunks of every row are issued before any is
// used, so a row pair of a few KB costs one memory round trip, not one per
// chunk and row.
template <int BITS, int NR>
__device__ __forceinline__ void rows_dot(const uint8_t *const (&row_bytes)[NR],
                                         const __half *const (&row_scales)[NR], int nchunks,
                                         const float *xs, int kpad, int nt, int lane,
                                         float (&acc)[NR][GEMV_NT]) {
    constexpr int V = Chunk<BITS>::V;
    for (int c0 = lane; c0 < nchunks; c0 += 32 * GEMV_UNR) {
        uint4 raw[NR][GEMV_UNR];
        float sc[NR][GEMV_UNR];
#pragma unroll
        for (int u = 0; u < GEMV_UNR; u++) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < NR; r++) {
                sc[r][u] = 1.f;
                if (c < nchunks) {
                    raw[r][u] = __ldcs(reinterpret_cast<const uint4 *>(row_bytes[r]) + c);  // evict-first
                    if constexpr (BITS <= 8) sc[r][u] = __half2float(row_scales[r][(c * V) / QG_GROUP]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < GEMV_UNR; u++) {
            const int c = c0 + 32 * u;
            if (c >= nchunks) break;
#pragma unroll
            for (int r = 0; r < NR; r++) {
                float v[V];
                decode_chunk<BITS>(raw[r][u], v);
#pragma unroll
                for (int t = 0; t < GEMV_NT; t++) {
                    if (t < nt) {
                        const float *xt = xs + t * kpad;
                        float part = 0.f;
#pragma unroll
                        for (int j4 = 0; j4 < V / 4; j4++) {
                            const float4 xv =
                                *reinterpret_cast<const float4 *>(xt + stage_pos<V>(c, j4 * 4));
                            part = fmaf(v[j4 * 4 + 0], xv.x, part);
                            part = fmaf(v[j4 * 4 + 1], xv.y, part);
                            part = fmaf(v[j4 * 4 + 2], xv.z, part);
                            part = fmaf(v[j4 * 4 + 3], xv.w, part);
                        }
                        acc[r][t] = fmaf(part, sc[r][u], acc[r][t]);
                    }
                }
            }
        }
    }
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int BITS, bool GATEUP>
__global__ void __launch_bounds__(GEMV_THREADS)
k_expert_gemv(ExpertArgs a) {
    pdl_enter();
    extern __shared__ __align__(16) float xs[];
    constexpr int V = Chunk<BITS>::V;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const int n_act = a.n_act ? *a.n_act : 1;
    const int n_routed = n_act - a.has_shared;
    const int out_rows_r = GATEUP ? a.routed.rows / 2 : a.routed.rows;
    const int out_rows_s = a.has_shared ? (GATEUP ? a.shared.rows / 2 : a.shared.rows) : 0;
    const int nrb_r = (out_rows_r + GEMV_ROWS - 1) / GEMV_ROWS;
    const int nrb_s = (out_rows_s + GEMV_ROWS - 1) / GEMV_ROWS;
    const int n_items = n_routed * nrb_r + (a.has_shared ? nrb_s : 0);

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        int ai, rb;
        if (item < n_routed * nrb_r) {
            ai = item / nrb_r;
            rb = item % nrb_r;
        } else {
            ai = n_routed;
            rb = item - n_routed * nrb_r;
        }
        const int g = a.act_group ? a.act_group[ai] : a.n_experts;
        const bool is_shared = (g == a.n_experts);
        if (g < 0 || g > a.n_experts || (is_shared && !a.has_shared)) {
            if (tid == 0) atomicOr(a.err, QG_FLAG_BAD_GROUP);
            continue;
        }
        const WeightSet &ws = is_shared ? a.shared : a.routed;
        const int eidx = is_shared ? 0 : g;
        const int K = ws.K;
        const int out_rows = GATEUP ? ws.rows / 2 : ws.rows;
        const int nchunks = K / V;
        const int kpad = ((nchunks + 31) / 32) * 32 * V;
        const size_t row_bytes = BITS == 32   ? (size_t)K * 4
                                 : BITS == 16 ? (size_t)K * 2
                                 : BITS == 8  ? (size_t)K
                                              : (size_t)K / 2;
        const uint8_t *wbase = BITS == 32 ? reinterpret_cast<const uint8_t *>(ws.w32) : ws.q;
        wbase += (size_t)eidx * ws.rows * row_bytes;
        const __half *sbase = ws.s ? ws.s + (size_t)eidx * ws.rows * (K / QG_GROUP) : nullptr;
        const int slot0 = a.act_begin ? a.act_begin[ai] : 0;
        const int ntok = a.act_n ? a.act_n[ai] : a.single_n;
        const int r0 = rb * GEMV_ROWS;

        for (int tc = 0; tc < ntok; tc += GEMV_NT) {
            const int nt = min(GEMV_NT, ntok - tc);
            __syncthreads();  // previous pass done with xs
            for (int i = tid; i < nt * K; i += GEMV_THREADS) {
                const int t = i / K, kk = i - t * K;
                const int slot = slot0 + tc + t;
                const float *src = GATEUP ? a.in + (size_t)a.slot_token[slot] * a.in_stride
                                          : a.in + (size_t)slot * a.in_stride;
                xs[t * kpad + stage_pos<V>(kk / V, kk % V)] = src[kk];
            }
            __syncthreads();
            for (int rr = warp; rr < GEMV_ROWS; rr += GEMV_WARPS) {
                const int r = r0 + rr;
                if (r >= out_rows) break;
                if constexpr (GATEUP) {
                    const int ru = r + out_rows;  // up rows follow the gate rows
                    const uint8_t *const rows[2] = {wbase + (size_t)r * row_bytes,
                                                    wbase + (size_t)ru * row_bytes};
                    const __half *const scs[2] = {
                        sbase ? sbase + (size_t)r * (K / QG_GROUP) : nullptr,
                        sbase ? sbase + (size_t)ru * (K / QG_GROUP) : nullptr};
                    float acc[2][GEMV_NT] = {};
                    rows_dot<BITS, 2>(rows, scs, nchunks, xs, kpad, nt, lane, acc);
#pragma unroll
                    for (int t = 0; t < GEMV_NT; t++) {
                        const float gsum = warp_allsum(acc[0][t]);
                        const float usum = warp_allsum(acc[1][t]);
                        if (lane == t && t < nt)
                            a.out[(size_t)(slot0 + tc + t) * a.out_stride + r] =
                                __fmul_rn(silu_ref(gsum), usum);
                    }
                } else {
                    const uint8_t *const rows[1] = {wbase + (size_t)r * row_bytes};
                    const __half *const scs[1] = {
                        sbase ? sbase + (size_t)r * (K / QG_GROUP) : nullptr};
                    float acc[1][GEMV_NT] = {};
                    rows_dot<BITS, 1>(rows, scs, nchunks, xs, kpad, nt, lane, acc);
#pragma unroll
                    for (int t = 0; t < GEMV_NT; t++) {
                        const float s = warp_allsum(acc[0][t]);
                        if (lane == t && t < nt)
                            a.out[(size_t)(slot0 + tc + t) * a.out_stride + r] = s;
                    }
                }
            }
        }
        __syncthreads();
    }
}

template <int BITS, bool GATEUP>
static int launch_t(const ExpertArgs &a, int max_items, cudaStream_t s) {
    constexpr int V = Chunk<BITS>::V;
    int kmax = a.routed.K;
    if (a.has_shared && a.shared.K > kmax) kmax = a.shared.K;
    const int kpad = ((kmax / V + 31) / 32) * 32 * V;
    const size_t smem = sizeof(float) * (size_t)GEMV_NT * kpad;
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_done[64] = {false};
    if (dev < 64 && !attr_done[dev]) {
        QG_CUDA(cudaFuncSetAttribute(k_expert_gemv<BITS, GATEUP>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_done[dev] = true;
    }
    int per_sm = 0;
    QG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_expert_gemv<BITS, GATEUP>,
                                                          GEMV_THREADS, smem));
    if (per_sm < 1) per_sm = 1;
    int grid = num_sms(dev) * per_sm;
    if (max_items < grid) grid = max_items;
    if (grid < 1) grid = 1;
    QG_CUDA(launch_pdl(k_expert_gemv<BITS, GATEUP>, dim3(grid), dim3(GEMV_THREADS), smem, s, 1, a));
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_expert(bool gateup, const ExpertArgs &a, int max_items_groups, cudaStream_t s) {
    // max work items: groups x row blocks (upper bound, the kernel reads the
    // true count from the device).
    const int rows = gateup ? a.routed.rows / 2 : a.routed.rows;
    const int rs = a.has_shared ? (gateup ? a.shared.rows / 2 : a.shared.rows) : 0;
    const int mr = rows > rs ? rows : rs;
    const int nrb = (mr + GEMV_ROWS - 1) / GEMV_ROWS;
    const int max_items = max_items_groups * nrb;
    const int bits = a.routed.bits;
    if (gateup) {
        if (bits == 32) return launch_t<32, true>(a, max_items, s);
        if (bits == 16) return launch_t<16, true>(a, max_items, s);
        if (bits == 8) return launch_t<8, true>(a, max_items, s);
        if (bits == 4) return launch_t<4, true>(a, max_items, s);
    } else {
        if (bits == 32) return launch_t<32, false>(a, max_items, s);
        if (bits == 16) return launch_t<16, false>(a, max_items, s);
        if (bits == 8) return launch_t<8, false>(a, max_items, s);
        if (bits == 4) return launch_t<4, false>(a, max_items, s);
    }
    return set_error(QGMOE_ERR_INVALID_ARG, "bits must be 32, 16, 8 or 4 (got %d)", bits);
}

// out[t, j] = sum_r w[t,r] * d[slot(t,r), j]  (+ sg[t] * ds[T*k + t, j]),
// accumulated from zero in rank order with separately rounded products, as
// `out[j] += w * d[j]` in model/moe.go:82-85 and :94-96.  Routed rows d and
// shared-expert rows ds are f32 (CUDA-core path) or fp16 (tensor-core path);
// they differ when the shared expert's format keeps it off the tensor cores.
__device__ __forceinline__ float4 load4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 load4(const __half *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

template <typename D, typename DS>
__global__ void k_combine(const D *__restrict__ d, const DS *__restrict__ ds, int H, int T, int k,
                          const int32_t *__restrict__ pair_slot,
                          const float *__restrict__ topk_w, const float *__restrict__ shared_w,
                          int has_shared, float *__restrict__ out) {
    pdl_enter();
    const int t = blockIdx.y;
    const int j4 = blockIdx.x * blockDim.x + threadIdx.x;
    if (j4 * 4 >= H) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < k; r++) {
        const int slot = pair_slot[(size_t)t * k + r];
        const float w = topk_w[(size_t)t * k + r];
        const float4 v = load4(d + (size_t)slot * H + 4 * j4);
        acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
    }
    if (has_shared) {
        const float w = shared_w[t];
        const float4 v = load4(ds + (size_t)(T * k + t) * H + 4 * j4);
        acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
    }
    reinterpret_cast<float4 *>(out + (size_t)t * H)[j4] = acc;
}

template <typename D, typename DS>
static int launch_combine_t(const D *d, const DS *ds, int H, int T, int k,
                            const int32_t *pair_slot, const float *topk_w, const float *shared_w,
                            int has_shared, float *out, cudaStream_t s) {
    const int threads = 128;
    dim3 grid((H / 4 + threads - 1) / threads, T);
    QG_CUDA(launch_pdl(k_combine<D, DS>, grid, dim3(threads), 0, s, 1, d, ds, H, T, k, pair_slot,
                       topk_w, shared_w, has_shared, out));
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_combine(const float *d, int H, int T, int k, const int32_t *pair_slot,
                   const float *topk_w, const float *shared_w, int has_shared, float *out,
                   cudaStream_t s) {
    return launch_combine_t(d, d, H, T, k, pair_slot, topk_w, shared_w, has_shared, out, s);
}

int launch_combine_f16(const __half *d, int H, int T, int k, const int32_t *pair_slot,
                       const float *topk_w, const float *shared_w, int has_shared, float *out,
                       cudaStream_t s) {
    return launch_combine_t(d, d, H, T, k, pair_slot, topk_w, shared_w, has_shared, out, s);
}

int launch_combine_mixed(const __half *d, const float *ds, int H, int T, int k,
                         const int32_t *pair_slot, const float *topk_w, const float *shared_w,
                         float *out, cudaStream_t s) {
    return launch_combine_t(d, ds, H, T, k, pair_slot, topk_w, shared_w, 1, out, s);
}

}  // namespace qg
