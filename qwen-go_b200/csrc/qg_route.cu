// Router + dispatch (kernels K1 and K2).
//
// Launches: k_logits, k_topk, k_scatter (+ k_gather_f16 for the tensor path).
// 1. k_logits: logits = x . router^T (proj(x,1,&m.gate,...), model/moe.go:42)
//    as a split-K tiled f32 GEMM on CUDA cores: a CTA owns 32 tokens x 128
//    router rows x one K slice, writes its partial sums.  The shared-expert
//    gate vector rides along as router row E (model/moe.go:87-93).  Split-K
//    keeps decode-sized batches (T = 1..64) spread over the SMs while the
//    1 MiB router matrix is read about once.
// 2. k_topk: one warp per token adds the partials in a fixed order, then
//    softmax (model/tensors.go:106-121: max-subtract, exp in float64 rounded
//    to float32, divide by the sum), top-k (model/moe.go:44-52, TOPK or the
//    literal PREFIX bound), w = p / (wSum + 1e-9) (model/moe.go:53-63) and
//    sigmoid of the shared gate.  Each CTA writes its expert histogram; the
//    last CTA (atomic ticket) scans the totals into expert offsets, the list
//    of active experts and the tensor-core tile prefix, and re-zeroes the
//    counters and the ticket so the next call (or a graph replay) starts clean.
// 3. k_scatter: each CTA ranks its own (token, rank) pairs per expert in pair
//    order (warp match + per-warp counts) and adds the histograms of the CTAs
//    before it, so slots are expert-sorted and deterministic without a serial
//    pass.  For the tensor-core path k_gather_f16 then writes each slot's fp16
//    activation row.
#include "qg_common.cuh"

namespace qg {

constexpr int LG_TOK = 64;   // tokens per logits tile (8 per warp)
constexpr int LG_ROWS = 128; // router rows per logits tile (4 per lane)
constexpr int LG_KC = 32;    // K chunk staged in shared memory
constexpr int TK_TOK = 32;   // tokens per top-k / scatter CTA
constexpr int RT_THREADS = 1024;  // top-k and scatter CTAs: one warp per token
constexpr int RT_WARPS = RT_THREADS / 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
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

int route_splits(int T, int H, int Ep, int sms) {
    const int tt = (T + LG_TOK - 1) / LG_TOK;
    const int te = (Ep + LG_ROWS - 1) / LG_ROWS;
    int s = (2 * sms) / (tt * te);
    const int smax = H / LG_KC < 32 ? H / LG_KC : 32;
    if (s > smax) s = smax;
    if (s < 1) s = 1;
    return s;
}

// ---- 1. logits ------------------------------------------------------------------
// CTA tile: 64 tokens x 128 router rows x one K slice.  Warp w owns tokens
// 8w..8w+7, lane l owns rows 4l..4l+3: per K step two broadcast float4 reads
// of x and one float4 read of the router feed 32 FMAs.  The next K chunk is
// fetched into registers while the current one is consumed.
__global__ void __launch_bounds__(256)
k_logits(const float *__restrict__ x, int T, int H, int E, int Ep, const float *__restrict__ router,
         const float *__restrict__ shared_gate, int ksplit, float *__restrict__ part) {
    __shared__ __align__(16) float xs[LG_KC][LG_TOK + 4];
    __shared__ __align__(16) float ws[LG_KC][LG_ROWS + 4];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * LG_TOK, r0 = blockIdx.y * LG_ROWS, s = blockIdx.z;
    const int kc = ((H / LG_KC + ksplit - 1) / ksplit) * LG_KC;
    const int k0 = s * kc, k1 = min(H, k0 + kc);
    float acc[8][4] = {};
    const int lrow = tid >> 3, k4 = (tid & 7) * 4;  // loader: row / token, float4 column
    const float *xrow[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int t = t0 + lrow + 32 * j;
        xrow[j] = t < T ? x + (size_t)t * H : nullptr;
    }
    const float *wrow[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int r = r0 + lrow + 32 * j;
        wrow[j] = r < Ep ? (r < E ? router + (size_t)r * H : shared_gate) : nullptr;
    }
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 xn[2], wn[4];
    auto fetch = [&](int kb) {
#pragma unroll
        for (int j = 0; j < 2; j++)
            xn[j] = xrow[j] ? *reinterpret_cast<const float4 *>(xrow[j] + kb + k4) : zero;
#pragma unroll
        for (int j = 0; j < 4; j++)
            wn[j] = wrow[j] ? __ldg(reinterpret_cast<const float4 *>(wrow[j] + kb + k4)) : zero;
    };
    if (k0 < k1) fetch(k0);
    for (int kb = k0; kb < k1; kb += LG_KC) {
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int t = lrow + 32 * j;
            xs[k4][t] = xn[j].x;
            xs[k4 + 1][t] = xn[j].y;
            xs[k4 + 2][t] = xn[j].z;
            xs[k4 + 3][t] = xn[j].w;
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int row = lrow + 32 * j;
            ws[k4][row] = wn[j].x;
            ws[k4 + 1][row] = wn[j].y;
            ws[k4 + 2][row] = wn[j].z;
            ws[k4 + 3][row] = wn[j].w;
        }
        __syncthreads();
        if (kb + LG_KC < k1) fetch(kb + LG_KC);
#pragma unroll 4
        for (int kk = 0; kk < LG_KC; kk++) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&xs[kk][8 * warp]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&xs[kk][8 * warp + 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&ws[kk][4 * lane]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int t = t0 + 8 * warp + i;
        if (t >= T) continue;
        const int r = r0 + 4 * lane;
        float *dst = part + ((size_t)s * T + t) * Ep + r;
        if (r + 3 < Ep && (Ep & 3) == 0) {
            *reinterpret_cast<float4 *>(dst) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (r + j < Ep) dst[j] = acc[i][j];
        }
    }
}

// Sum of the split-K partials of one logit, in a fixed order; four
// independent accumulators keep the loads in flight together.
__device__ __forceinline__ float sum_splits(const float *__restrict__ part, int ksplit,
                                            size_t stride, size_t off) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int s = 0;
    for (; s + 4 <= ksplit; s += 4) {
        a0 += part[off + s * stride];
        a1 += part[off + (s + 1) * stride];
        a2 += part[off + (s + 2) * stride];
        a3 += part[off + (s + 3) * stride];
    }
    for (; s < ksplit; s++) a0 += part[off + s * stride];
    return (a0 + a1) + (a2 + a3);
}

// ---- 2. softmax + top-k + histograms --------------------------------------------
// A warp holds one token's probabilities in registers: lane l owns experts
// l, l+32, ..., l+32*(NJ-1) (NJ = ceil(E/32) rounded up to a power of two).
template <int NJ>
__global__ void __launch_bounds__(RT_THREADS)
k_topk(const float *__restrict__ part, int ksplit, int T, int E, int Ep, int k, int mode,
       int has_shared, RouteState st, int *err) {
    extern __shared__ int hist_s[];  // [E]
    __shared__ int s_idx[RT_WARPS][QG_MAX_TOPK];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += RT_THREADS) hist_s[e] = 0;
    __syncthreads();

    for (int i = 0; i < TK_TOK / RT_WARPS; i++) {
        const int t = blockIdx.x * TK_TOK + warp * (TK_TOK / RT_WARPS) + i;
        if (t >= T) break;
        float v[NJ];
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            v[j] = e < E ? sum_splits(part, ksplit, (size_t)T * Ep, (size_t)t * Ep + e) : -INFINITY;
        }
        float mx = v[0];
#pragma unroll
        for (int j = 1; j < NJ; j++) mx = fmaxf(mx, v[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            if (lane + 32 * j < E) {
                v[j] = (float)exp((double)(v[j] - mx));
                sum += v[j];
            } else {
                v[j] = -1.f;  // never selected
            }
        }
        sum = warp_sum(sum);
#pragma unroll
        for (int j = 0; j < NJ; j++)
            if (lane + 32 * j < E) v[j] = v[j] / sum;
        int *sel = s_idx[warp];
        float selp = 0.f;  // lane r < k: probability of the rank-r expert
        if (mode == QGMOE_ROUTER_TOPK) {
            unsigned used = 0;
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if (lane + 32 * j >= E) used |= 1u << j;  // padding lanes never win
            for (int r = 0; r < k; r++) {
                float bv = -2.f;
                int bi = 0x7fffffff;
#pragma unroll
                for (int j = 0; j < NJ; j++)
                    if (!((used >> j) & 1u)) better(bv, bi, v[j], lane + 32 * j);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
                    better(bv, bi, v2, i2);
                }
                if ((bi & 31) == lane) used |= 1u << (bi >> 5);
                if (lane == r) selp = bv;
                if (lane == 0) sel[r] = bi;
            }
        } else {
            // PREFIX: the literal moe.go:49 bound orders only experts 0..k-1
            // (k <= 32, so expert q < k is v[0] of lane q).
            const float pq = v[0];
            float pk[QG_MAX_TOPK];
            int ik[QG_MAX_TOPK];
            for (int q = 0; q < k; q++) {
                pk[q] = __shfl_sync(0xffffffffu, pq, q);
                ik[q] = q;
            }
            if (lane == 0) {
                for (int a2 = 1; a2 < k && a2 < E; a2++)
                    for (int b2 = a2; b2 > 0 && pk[b2] > pk[b2 - 1]; b2--) {
                        const float tp = pk[b2];
                        pk[b2] = pk[b2 - 1];
                        pk[b2 - 1] = tp;
                        const int ti = ik[b2];
                        ik[b2] = ik[b2 - 1];
                        ik[b2 - 1] = ti;
                    }
                for (int q = 0; q < k; q++) sel[q] = ik[q];
            }
            __syncwarp();
            // probability of rank `lane`: the owner of expert sel[lane] is lane sel[lane]
            const int myexp = lane < k ? sel[lane] : 0;
            const float got = __shfl_sync(0xffffffffu, pq, myexp);
            if (lane < k) selp = got;
        }
        __syncwarp();
        // wSum over ranks in rank order, then w = p / (wSum + 1e-9)
        float wsum = 0.f;
        for (int r = 0; r < k; r++) wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, selp, r));
        const float den = __fadd_rn(wsum, 1e-9f);
        if (lane < k) {
            const int e = sel[lane];
            st.topk_idx[(size_t)t * k + lane] = e;
            st.topk_w[(size_t)t * k + lane] = __fdiv_rn(selp, den);
            if (e >= 0 && e < E)
                atomicAdd(&hist_s[dispatch_key(e, E, st.ep_world)], 1);
            else
                atomicOr(err, QG_FLAG_BAD_EXPERT);
        }
        if (has_shared && lane == 0) {
            const float g = sum_splits(part, ksplit, (size_t)T * Ep, (size_t)t * Ep + E);
            st.shared_w[t] = 1.f / (1.f + (float)exp(-(double)g));
        }
        __syncwarp();
    }
    __syncthreads();
    for (int e = tid; e < E; e += RT_THREADS) {
        const int c = hist_s[e];
        st.hist[(size_t)blockIdx.x * E + e] = c;
        if (c) atomicAdd(&st.counts[e], c);
    }

    // ---- last CTA: expert offsets, active list, tile prefix ------------------
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(st.done_ctr, 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    int *cnt = hist_s;
    for (int e = tid; e < E; e += RT_THREADS) {
        cnt[e] = __ldcg(st.counts + e);
        st.counts[e] = 0;
    }
    __syncthreads();
    if (warp == 0) {
        const int per = (E + 31) / 32;
        const int lo = lane * per, hi = min(E, lo + per);
        int run = 0, nz = 0;
        for (int e = lo; e < hi; e++) {
            run += cnt[e];
            nz += cnt[e] > 0;
        }
        int incl = run, nzi = nz;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            const int w = __shfl_up_sync(0xffffffffu, nzi, o);
            if (lane >= o) {
                incl += v;
                nzi += w;
            }
        }
        int base = incl - run, a = nzi - nz;
        for (int e = lo; e < hi; e++) {
            st.expert_off[e] = base;
            if (cnt[e] > 0) {
                st.act_group[a] = e;
                st.act_begin[a] = base;
                st.act_n[a] = cnt[e];
                a++;
            }
            base += cnt[e];
        }
        int total_act = __shfl_sync(0xffffffffu, nzi, 31);
        if (lane == 0) {
            const int tt = st.tile_tokens > 0 ? st.tile_tokens : 256;
            int tiles = 0, ai = 0;
            for (int e = 0; e < E; e++)
                if (cnt[e] > 0) {
                    st.tile_prefix[ai++] = tiles;
                    tiles += (cnt[e] + tt - 1) / tt;
                }
            st.tile_prefix[ai] = tiles;
            if (st.n_act_routed) *st.n_act_routed = ai;
            if (has_shared && st.shared_act) {
                st.shared_act[0] = 0;
                st.shared_act[1] = T * k;
                st.shared_act[2] = T;
                st.shared_act[3] = 1;
                st.shared_act[4] = 0;
                st.shared_act[5] = (T + tt - 1) / tt;
            }
            if (has_shared) {
                st.act_group[total_act] = E;
                st.act_begin[total_act] = T * k;
                st.act_n[total_act] = T;
                total_act++;
            }
            *st.n_act = total_act;
            *st.done_ctr = 0;
        }
    }
}

// ---- 3. scatter (+ fp16 gather) ---------------------------------------------------
__global__ void __launch_bounds__(RT_THREADS)
k_scatter(int T, int E, int k, int has_shared, RouteState st, int *err) {
    extern __shared__ int sm[];
    int *cur = sm;            // [E] next slot per expert for this CTA
    int *wcnt = sm + E;       // [RT_WARPS][E]
    __shared__ int partial[RT_THREADS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = blockIdx.x;
    // Slots of this CTA's pairs start after the earlier CTAs' pairs of the
    // same expert: sum histogram rows 0..c-1, split over nparts threads per
    // expert with independent accumulators so the loads overlap.
    const int nparts = E >= RT_THREADS ? 1 : RT_THREADS / E;
    for (int e0 = 0; e0 < E; e0 += RT_THREADS) {
        const int stride = E >= RT_THREADS ? RT_THREADS : E;
        const int e = e0 + tid % stride, part = tid / stride;
        int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
        if (e < E && part < nparts) {
            const int per = (c + nparts - 1) / nparts;
            const int lo = part * per, hi = min(c, lo + per);
            int cc = lo;
            for (; cc + 4 <= hi; cc += 4) {
                acc0 += st.hist[(size_t)cc * E + e];
                acc1 += st.hist[(size_t)(cc + 1) * E + e];
                acc2 += st.hist[(size_t)(cc + 2) * E + e];
                acc3 += st.hist[(size_t)(cc + 3) * E + e];
            }
            for (; cc < hi; cc++) acc0 += st.hist[(size_t)cc * E + e];
        }
        partial[tid] = acc0 + acc1 + acc2 + acc3;
        __syncthreads();
        if (tid < stride && e0 + tid < E) {
            const int ee = e0 + tid;
            int base = st.expert_off[ee];
            for (int pp = 0; pp < nparts; pp++) base += partial[pp * stride + tid];
            cur[ee] = base;
        }
        __syncthreads();
    }
    const int p0 = c * TK_TOK * k;
    const int p1 = min(T * k, p0 + TK_TOK * k);
    const unsigned lt = (1u << lane) - 1u;
    for (int base = p0; base < p1; base += RT_THREADS) {
        for (int i = tid; i < RT_WARPS * E; i += RT_THREADS) wcnt[i] = 0;
        __syncthreads();
        const int pi = base + tid;
        int e = -1;
        if (pi < p1) {
            e = st.topk_idx[pi];
            if (e < 0 || e >= E) {
                atomicOr(err, QG_FLAG_BAD_EXPERT);
                e = -1;
            } else {
                e = dispatch_key(e, E, st.ep_world);
            }
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & lt);
        if (e >= 0 && rank == 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int slot = cur[e] + rank;
            for (int w = 0; w < warp; w++) slot += wcnt[w * E + e];
            if (slot < 0 || slot >= T * k) {
                atomicOr(err, QG_FLAG_BAD_SLOT);
            } else {
                st.pair_slot[pi] = slot;
                st.slot_token[slot] = pi / k;
            }
        }
        __syncthreads();
        for (int ee = tid; ee < E; ee += RT_THREADS) {
            int add = 0;
            for (int w = 0; w < RT_WARPS; w++) add += wcnt[w * E + ee];
            cur[ee] += add;
        }
        __syncthreads();
    }
    if (has_shared)
        for (int t = c * TK_TOK + tid; t < min(T, (c + 1) * TK_TOK); t += RT_THREADS)
            st.slot_token[T * k + t] = t;
}

int launch_route(const float *x, int T, int H, int E, int k, int mode, const float *router,
                 const float *shared_gate, int has_shared, RouteState st, __half *xp, int *err,
                 cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int Ep = E + (has_shared ? 1 : 0);
    const int ks = route_splits(T, H, Ep, num_sms(dev));
    dim3 g1((T + LG_TOK - 1) / LG_TOK, (Ep + LG_ROWS - 1) / LG_ROWS, ks);
    k_logits<<<g1, 256, 0, s>>>(x, T, H, E, Ep, router, shared_gate, ks, st.logits);
    QG_CUDA(cudaGetLastError());
    const int nc = (T + TK_TOK - 1) / TK_TOK;
    const size_t sm2 = sizeof(int) * (size_t)E;
    const size_t sm3 = sizeof(int) * (size_t)(RT_WARPS + 1) * E;
    static bool attr[64] = {false};
    if (dev < 64 && !attr[dev]) {
        QG_CUDA(cudaFuncSetAttribute(k_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        attr[dev] = true;
    }
    const int nj = (E + 31) / 32;
    if (nj <= 1)
        k_topk<1><<<nc, RT_THREADS, sm2, s>>>(st.logits, ks, T, E, Ep, k, mode, has_shared, st, err);
    else if (nj <= 2)
        k_topk<2><<<nc, RT_THREADS, sm2, s>>>(st.logits, ks, T, E, Ep, k, mode, has_shared, st, err);
    else if (nj <= 4)
        k_topk<4><<<nc, RT_THREADS, sm2, s>>>(st.logits, ks, T, E, Ep, k, mode, has_shared, st, err);
    else if (nj <= 8)
        k_topk<8><<<nc, RT_THREADS, sm2, s>>>(st.logits, ks, T, E, Ep, k, mode, has_shared, st, err);
    else if (nj <= 16)
        k_topk<16><<<nc, RT_THREADS, sm2, s>>>(st.logits, ks, T, E, Ep, k, mode, has_shared, st, err);
    else
        k_topk<32><<<nc, RT_THREADS, sm2, s>>>(st.logits, ks, T, E, Ep, k, mode, has_shared, st, err);
    QG_CUDA(cudaGetLastError());
    k_scatter<<<nc, RT_THREADS, sm3, s>>>(T, E, k, has_shared, st, err);
    QG_CUDA(cudaGetLastError());
    if (xp) return launch_gather_f16(x, st.slot_token, T * k + (has_shared ? T : 0), H, xp, s);
    return QGMOE_OK;
}

}  // namespace qg
