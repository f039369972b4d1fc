// The MoE forward of a decode-sized batch (T <= FD_MAX_T tokens) in four
// kernels instead of seven: k_logits_rows (qg_route.cu, the router logits in
// the reference's serial order), then
//   k_dec_route (one CTA, a warp per token): route_token -- the reference's
//     softmax, top-k and renormalised weights (model/moe.go:41-63) -- the
//     routing outputs, and the batch's distinct experts with their tokens and
//     (token, rank) pairs, for the two expert kernels;
//   k_dec_gateup: gate/up row pairs of the selected experts and of the shared
//     expert, h = silu(x.Wg) * (x.Wu) (model/moe.go:64-76, model/model.go:
//     350-358) for every (token, rank);
//   k_dec_down: stages every h row in shared memory and, per output row j,
//     forms the down products of all (token, rank) pairs and of the shared
//     expert, then combines them in rank order, out[t][j] = sum_r w * d
//     (+ sigmoid gate * shared), model/moe.go:77-97 -- no separate combine.
// Each expert's gate/up rows are read once per batch however many tokens chose
// it.  The row arithmetic (16-byte chunks dequantised in registers, per-lane
// FMA over chunks lane, lane+32, ..., a warp reduction) is the CUDA-core
// GEMV's (qg_gemv.cu), so the two paths give identical results; the combine
// rounds like k_combine.  The expert kernels are instantiated for the batch's
// token count rounded up to 1, 2, 4 or 8 (MT) to keep their code small.
#include "qg_common.cuh"
#include "qg_gemv.cuh"
#include "qg_router.cuh"

namespace qg {

constexpr int FD_THREADS = 256, FD_WARPS = FD_THREADS / 32;
constexpr int FD_UNR = 4;   // 16-byte chunks per lane loaded ahead
constexpr int FD_PAIRS = 4; // (token, rank) pairs whose down rows load together

// ---- routing -----------------------------------------------------------------
template <int NJ>
__global__ void __launch_bounds__(32 * FD_MAX_T)
k_dec_route(DecodeArgs a) {
    __shared__ DecRoute R;
    const int tid = threadIdx.x, lane = tid & 31, t = tid >> 5;
    pdl_enter();
    if (t < a.T) {
        const float wr = route_token<NJ>(a.logits + (size_t)t * a.Ep, a.E, a.k, a.mode, lane,
                                         R.sel[t]);
        if (lane < a.k) {
            R.w[t][lane] = wr;
            a.topk_idx[(size_t)t * a.k + lane] = R.sel[t][lane];
            a.topk_w[(size_t)t * a.k + lane] = wr;
        }
        if (a.has_shared && lane == 0) {
            // sigmoid1 (model/tensors.go:97) of the shared-gate logit
            const float g = a.logits[(size_t)t * a.Ep + a.E];
            R.sg[t] = __fdiv_rn(1.f, __fadd_rn(1.f, (float)exp(-(double)g)));
            a.shared_w[t] = R.sg[t];
        }
    }
    __syncthreads();
    if (tid == 0) {
        int nd = 0;
        for (int tt = 0; tt < a.T; tt++)
            for (int r = 0; r < a.k; r++) {
                int e = R.sel[tt][r];
                if (e < 0 || e >= a.E) {
                    atomicOr(a.err, QG_FLAG_BAD_EXPERT);
                    e = 0;  // keeps every index in range; the flag reports the fault
                }
                int d = 0;
                while (d < nd && R.dexp[d] != e) d++;
                if (d == nd) {
                    R.dexp[nd] = e;
                    R.dmask[nd] = 0;
                    nd++;
                }
                R.dmask[d] |= 1u << tt;
                R.drank[d][tt] = (signed char)r;
            }
        R.nd = nd;
        int np = 0;  // pairs grouped by expert: a run of pairs shares its rows in L1
        for (int d = 0; d < nd; d++)
            for (int tt = 0; tt < a.T; tt++)
                if ((R.dmask[d] >> tt) & 1u) {
                    R.pexp[np] = R.dexp[d];
                    R.prow[np] = tt * a.k + R.drank[d][tt];
                    np++;
                }
        R.np = np;
    }
    __syncthreads();
    const int *src = reinterpret_cast<const int *>(&R);
    int *dst = reinterpret_cast<int *>(a.route);
    for (int i = tid; i < (int)(sizeof(DecRoute) / sizeof(int)); i += blockDim.x) dst[i] = src[i];
}

__device__ __forceinline__ void load_route(const DecRoute *g, DecRoute &R) {
    const int *src = reinterpret_cast<const int *>(g);
    int *dst = reinterpret_cast<int *>(&R);
    for (int i = threadIdx.x; i < (int)(sizeof(DecRoute) / sizeof(int)); i += FD_THREADS)
        dst[i] = src[i];
}

// ---- row dot products ------------------------------------------------------------
// NR weight rows: row r dots with the staged rows x_t = xs[r] + t * kpad of
// the tokens t < MT in mask[r]: acc[r][t] = row_r . x_t, reduced over the
// warp.  Per lane the chunks lane, lane+32, ... are accumulated in order (FMA
// over a chunk's V elements, then FMA with the chunk's group scale), exactly
// as the CUDA-core GEMV does.
template <int BITS, int NR, int MT>
__device__ __forceinline__ void dec_dot(const uint8_t *const (&rows)[NR],
                                        const __half *const (&scales)[NR], int nchunks,
                                        const float *const (&xs)[NR], int kpad,
                                        const unsigned (&mask)[NR], int lane,
                                        float (&acc)[NR][MT]) {
    constexpr int V = Chunk<BITS>::V;
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
        for (int t = 0; t < MT; t++) acc[r][t] = 0.f;
    for (int c0 = lane; c0 < nchunks; c0 += 32 * FD_UNR) {
        uint4 raw[NR][FD_UNR];
        float sc[NR][FD_UNR];
#pragma unroll
        for (int u = 0; u < FD_UNR; u++) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < NR; r++) {
                sc[r][u] = 1.f;
                if (c < nchunks && mask[r]) {
                    raw[r][u] = __ldcs(reinterpret_cast<const uint4 *>(rows[r]) + c);
                    if constexpr (BITS <= 8) sc[r][u] = __half2float(scales[r][(c * V) / QG_GROUP]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < FD_UNR; u++) {
            const int c = c0 + 32 * u;
            if (c >= nchunks) break;
#pragma unroll
            for (int r = 0; r < NR; r++) {
                if (!mask[r]) continue;
                float v[V];
                decode_chunk<BITS>(raw[r][u], v);
#pragma unroll
                for (int t = 0; t < MT; t++) {
                    if (!((mask[r] >> t) & 1u)) continue;
                    const float *xt = xs[r] + t * kpad;
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
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
        for (int t = 0; t < MT; t++)
            if ((mask[r] >> t) & 1u)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
                    acc[r][t] += __shfl_xor_sync(FULL, acc[r][t], o);
}

// count rows of K floats (row i at src + i * stride) into the staged layout
// the chunk reader expects (row i at dst + i * kpad).
template <int V>
__device__ void dec_stage(const float *__restrict__ src, int count, int K, size_t stride,
                          float *dst, int kpad) {
    for (int i = threadIdx.x; i < count * K; i += FD_THREADS) {
        const int row = i / K, kk = i - row * K;
        dst[row * kpad + stage_pos<V>(kk / V, kk % V)] = src[(size_t)row * stride + kk];
    }
}

template <int BITS>
__device__ __forceinline__ size_t row_bytes(int K) {
    return BITS == 32 ? (size_t)K * 4 : BITS == 16 ? (size_t)K * 2 : BITS == 8 ? (size_t)K
                                                                               : (size_t)K / 2;
}

// ---- gate_up + SwiGLU ----------------------------------------------------------------
template <int BITS, int MT>
__global__ void __launch_bounds__(FD_THREADS)
k_dec_gateup(DecodeArgs a) {
    constexpr int V = Chunk<BITS>::V;
    extern __shared__ __align__(16) float fd_smem[];
    __shared__ DecRoute R;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kpad = kpad_for(a.H, V);
    float *xs = fd_smem;  // [T][kpad]
    pdl_enter();
    dec_stage<V>(a.x, a.T, a.H, a.H, xs, kpad);
    load_route(a.route, R);
    __syncthreads();
    const int I = a.I, nrb = (I + FD_WARPS - 1) / FD_WARPS;
    const int n_routed = R.nd * nrb;
    const int n_items = n_routed + (a.has_shared ? (a.Is + FD_WARPS - 1) / FD_WARPS : 0);
    const size_t rb = row_bytes<BITS>(a.H);
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
        const bool shared = it >= n_routed;
        const WeightSet &ws = shared ? a.sgu : a.gu;
        const int out_rows = shared ? a.Is : I;
        const int row = (shared ? it - n_routed : it % nrb) * FD_WARPS + warp;
        if (row >= out_rows) continue;  // whole warp
        const int d = shared ? 0 : it / nrb;
        const int e = shared ? 0 : R.dexp[d];
        const unsigned m = shared ? (1u << a.T) - 1u : R.dmask[d];
        const uint8_t *wb = BITS == 32 ? reinterpret_cast<const uint8_t *>(ws.w32) : ws.q;
        const size_t g_row = (size_t)e * ws.rows + row, u_row = g_row + out_rows;
        const uint8_t *const rows[2] = {wb + g_row * rb, wb + u_row * rb};
        const __half *const scs[2] = {ws.s ? ws.s + g_row * (a.H / QG_GROUP) : nullptr,
                                      ws.s ? ws.s + u_row * (a.H / QG_GROUP) : nullptr};
        const float *const xr[2] = {xs, xs};
        const unsigned mk[2] = {m, m};
        float acc[2][MT];
        dec_dot<BITS, 2, MT>(rows, scs, a.H / V, xr, kpad, mk, lane, acc);
        if (lane == 0)
#pragma unroll
            for (int t = 0; t < MT; t++) {
                if (!((m >> t) & 1u)) continue;
                const size_t hr = shared ? (size_t)a.T * a.k + t
                                         : (size_t)t * a.k + (size_t)R.drank[d][t];
                a.h[hr * a.hmax + row] = __fmul_rn(silu_ref(acc[0][t]), acc[1][t]);
            }
    }
}

// ---- down + combine ---------------------------------------------------------------------
template <int BITS, int MT>
__global__ void __launch_bounds__(FD_THREADS)
k_dec_down(DecodeArgs a) {
    constexpr int V = Chunk<BITS>::V;
    extern __shared__ __align__(16) float fd_smem[];
    __shared__ DecRoute R;
    __shared__ float dv[FD_WARPS][FD_MAX_T * QG_MAX_TOPK + FD_MAX_T];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int T = a.T, k = a.k;
    const int kpi = kpad_for(a.I, V), kps = a.has_shared ? kpad_for(a.Is, V) : 0;
    float *hs = fd_smem;                            // [T*k][kpi] routed pairs
    float *hsh = hs + (size_t)T * k * kpi;          // [T][kps]  shared expert
    pdl_enter();
    dec_stage<V>(a.h, T * k, a.I, a.hmax, hs, kpi);
    if (a.has_shared) dec_stage<V>(a.h + (size_t)T * k * a.hmax, T, a.Is, a.hmax, hsh, kps);
    load_route(a.route, R);
    __syncthreads();
    const size_t rbi = row_bytes<BITS>(a.I), rbs = row_bytes<BITS>(a.Is);
    const int nrb = (a.H + FD_WARPS - 1) / FD_WARPS;
    const uint8_t *wb = BITS == 32 ? reinterpret_cast<const uint8_t *>(a.dn.w32) : a.dn.q;
    float *my = dv[warp];
    for (int rb = blockIdx.x; rb < nrb; rb += gridDim.x) {
        const int j = rb * FD_WARPS + warp;
        if (j >= a.H) continue;  // whole warp
        // the (token, rank) pairs, FD_PAIRS down rows in flight at a time
        for (int p0 = 0; p0 < R.np; p0 += FD_PAIRS) {
            const uint8_t *rows[FD_PAIRS];
            const __half *scs[FD_PAIRS];
            const float *xr[FD_PAIRS];
            unsigned mk[FD_PAIRS];
#pragma unroll
            for (int i = 0; i < FD_PAIRS; i++) {
                const int p = p0 + i < R.np ? p0 + i : p0;
                const size_t row = (size_t)R.pexp[p] * a.dn.rows + j;
                rows[i] = wb + row * rbi;
                scs[i] = a.dn.s ? a.dn.s + row * (a.I / QG_GROUP) : nullptr;
                xr[i] = hs + (size_t)R.prow[p] * kpi;
                mk[i] = p0 + i < R.np ? 1u : 0u;
            }
            float acc[FD_PAIRS][1];
            dec_dot<BITS, FD_PAIRS, 1>(rows, scs, a.I / V, xr, 0, mk, lane, acc);
            if (lane == 0)
#pragma unroll
                for (int i = 0; i < FD_PAIRS; i++)
                    if (mk[i]) my[R.prow[p0 + i]] = acc[i][0];
        }
        if (a.has_shared) {
            const uint8_t *sb = BITS == 32 ? reinterpret_cast<const uint8_t *>(a.sdn.w32) : a.sdn.q;
            const uint8_t *const rows[1] = {sb + (size_t)j * rbs};
            const __half *const scs[1] = {a.sdn.s ? a.sdn.s + (size_t)j * (a.Is / QG_GROUP)
                                                  : nullptr};
            const float *const xr[1] = {hsh};
            const unsigned mk[1] = {(1u << T) - 1u};
            float acc[1][MT];
            dec_dot<BITS, 1, MT>(rows, scs, a.Is / V, xr, kps, mk, lane, acc);
            if (lane == 0)
#pragma unroll
                for (int t = 0; t < MT; t++)
                    if (t < T) my[T * k + t] = acc[0][t];
        }
        __syncwarp();
        // out[t][j] = sum over ranks in order of w * d, then + sg * shared
        // (the rounding of k_combine and model/moe.go:82-85, 94-96)
        if (lane < T) {
            float o = 0.f;
            for (int r = 0; r < k; r++) o = __fadd_rn(o, __fmul_rn(R.w[lane][r], my[lane * k + r]));
            if (a.has_shared) o = __fadd_rn(o, __fmul_rn(R.sg[lane], my[T * k + lane]));
            a.out[(size_t)lane * a.H + j] = o;
        }
        __syncwarp();
    }
}

// ---- launches -------------------------------------------------------------------------------
static int chunk_elems(int bits) { return bits == 32 ? 4 : bits == 16 ? 8 : bits == 8 ? 16 : 32; }

size_t dec_smem_gateup(int bits, int T, int H) {
    return sizeof(float) * (size_t)T * kpad_for(H, chunk_elems(bits));
}

size_t dec_smem_down(int bits, int T, int k, int I, int Is) {
    const int V = chunk_elems(bits);
    return sizeof(float) * ((size_t)T * k * kpad_for(I, V) + (Is ? (size_t)T * kpad_for(Is, V) : 0));
}

static int launch_route_t(const DecodeArgs &a, cudaStream_t s) {
    const int nj = (a.E + 31) / 32;
    using K = void (*)(DecodeArgs);
    const K kern = nj <= 1 ? k_dec_route<1> : nj <= 2 ? k_dec_route<2> : nj <= 4 ? k_dec_route<4>
                 : nj <= 8 ? k_dec_route<8> : nj <= 16 ? k_dec_route<16> : k_dec_route<32>;
    QG_CUDA(launch_pdl(kern, dim3(1), dim3(32 * FD_MAX_T), 0, s, 1, a));
    return QGMOE_OK;
}

template <int BITS, int MT>
static int launch_dec_t(const DecodeArgs &a, bool gateup, int dev, cudaStream_t s) {
    static bool attr[64] = {false};
    if (dev < 64 && !attr[dev]) {
        QG_CUDA(cudaFuncSetAttribute(k_dec_gateup<BITS, MT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, FD_SMEM_MAX));
        QG_CUDA(cudaFuncSetAttribute(k_dec_down<BITS, MT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, FD_SMEM_MAX));
        attr[dev] = true;
    }
    const int sms = num_sms(dev);
    int per_sm = 0;
    if (gateup) {
        const size_t sm = dec_smem_gateup(BITS, a.T, a.H);
        QG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_dec_gateup<BITS, MT>,
                                                              FD_THREADS, sm));
        QG_CUDA(launch_pdl(k_dec_gateup<BITS, MT>, dim3(sms * (per_sm > 0 ? per_sm : 1)),
                           dim3(FD_THREADS), sm, s, 1, a));
    } else {
        const size_t sm = dec_smem_down(BITS, a.T, a.k, a.I, a.has_shared ? a.Is : 0);
        QG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_dec_down<BITS, MT>,
                                                              FD_THREADS, sm));
        int g = sms * (per_sm > 0 ? per_sm : 1);
        const int nrb = (a.H + FD_WARPS - 1) / FD_WARPS;
        if (g > nrb) g = nrb;
        QG_CUDA(launch_pdl(k_dec_down<BITS, MT>, dim3(g), dim3(FD_THREADS), sm, s, 1, a));
    }
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

template <int BITS>
static int launch_dec_b(const DecodeArgs &a, bool gateup, int dev, cudaStream_t s) {
    if (a.T <= 1) return launch_dec_t<BITS, 1>(a, gateup, dev, s);
    if (a.T <= 2) return launch_dec_t<BITS, 2>(a, gateup, dev, s);
    if (a.T <= 4) return launch_dec_t<BITS, 4>(a, gateup, dev, s);
    return launch_dec_t<BITS, 8>(a, gateup, dev, s);
}

int launch_decode(int bits, const DecodeArgs &a, int stage, cudaStream_t s) {
    if (a.T < 1 || a.T > FD_MAX_T)
        return set_error(QGMOE_ERR_INVALID_ARG, "decode path: T=%d outside 1..%d", a.T, FD_MAX_T);
    if (stage == 0) return launch_route_t(a, s);
    int dev = 0;
    cudaGetDevice(&dev);
    const bool gateup = stage == 1;
    switch (bits) {
        case 32: return launch_dec_b<32>(a, gateup, dev, s);
        case 16: return launch_dec_b<16>(a, gateup, dev, s);
        case 8: return launch_dec_b<8>(a, gateup, dev, s);
        case 4: return launch_dec_b<4>(a, gateup, dev, s);
    }
    return set_error(QGMOE_ERR_INVALID_ARG, "decode path: bits %d", bits);
}

}  // namespace qg
