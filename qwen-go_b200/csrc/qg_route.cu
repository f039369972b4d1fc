// Router + dispatch (kernels K1 and K2).
//
// One CTA per token computes the router logits (proj(x,1,&m.gate,...),
// model/moe.go:42), the softmax (model/tensors.go:106-121: max-subtract, exp
// evaluated in float64 and rounded to float32, divide by the sum), the top-k
// selection (model/moe.go:44-52, PREFIX or TOPK mode), the renormalised
// weights w = p / (wSum + 1e-9) (model/moe.go:53-63) and the shared-expert
// gate sigmoid(sharedGate . x) (model/moe.go:87-93).  The last CTA to finish
// (atomic ticket) builds the per-expert token lists in one pass: exclusive
// scan of the expert histogram, a stable scatter of the (token, rank) pairs
// into expert-sorted slots, and the compact list of active experts.  It
// re-zeroes the histogram and the ticket so the next call (or a CUDA-graph
// replay) starts clean.
#include <cstdio>

#include "qg_common.cuh"

namespace qg {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Picks the better of two (prob, index) candidates: larger prob, then lower
// index -- the order a stable descending insertion sort produces.
__device__ __forceinline__ void better(float &v, int &i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

__global__ void __launch_bounds__(QG_ROUTE_THREADS)
k_route(const float *__restrict__ x, int T, int H, int E, int k, int mode,
        const float *__restrict__ router, const float *__restrict__ shared_gate,
        int has_shared, RouteState st, int *err) {
    extern __shared__ float smem[];
    float *xs = smem;              // [H]
    float *p = smem + H;           // [E + 1] logits -> probabilities
    __shared__ int s_idx[QG_MAX_TOPK];
    __shared__ int s_last;

    const int t = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = QG_ROUTE_THREADS / 32;

    const float4 *xg = reinterpret_cast<const float4 *>(x + (size_t)t * H);
    for (int i = tid; i < H / 4; i += QG_ROUTE_THREADS)
        reinterpret_cast<float4 *>(xs)[i] = xg[i];
    __syncthreads();

    // logits: one warp per router row; the shared gate vector is row E.
    const int nrows = E + (has_shared ? 1 : 0);
    for (int e = warp; e < nrows; e += nwarps) {
        const float4 *wr = reinterpret_cast<const float4 *>(e < E ? router + (size_t)e * H
                                                                  : shared_gate);
        float acc = 0.f;
        for (int i = lane; i < H / 4; i += 32) {
            float4 w = __ldg(wr + i);
            float4 xv = reinterpret_cast<const float4 *>(xs)[i];
            acc = fmaf(xv.x, w.x, acc);
            acc = fmaf(xv.y, w.y, acc);
            acc = fmaf(xv.z, w.z, acc);
            acc = fmaf(xv.w, w.w, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) p[e] = acc;
    }
    __syncthreads();

    if (warp == 0) {
        // softmax over E (tensors.go:106-121)
        float mx = -INFINITY;
        for (int e = lane; e < E; e += 32) mx = fmaxf(mx, p[e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        for (int e = lane; e < E; e += 32) {
            float v = (float)exp((double)(p[e] - mx));
            p[e] = v;
            sum += v;
        }
        sum = warp_sum(sum);
        for (int e = lane; e < E; e += 32) p[e] = p[e] / sum;
        __syncwarp();

        if (mode == QGMOE_ROUTER_TOPK) {
            // k rounds of warp arg-max; winners are knocked out by index.
            for (int r = 0; r < k; r++) {
                float bv = -1.f;
                int bi = 0x7fffffff;
                for (int e = lane; e < E; e += 32) {
                    bool used = false;
                    for (int q = 0; q < r; q++) used |= (s_idx[q] == e);
                    if (!used) better(bv, bi, p[e], e);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
                    int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
                    better(bv, bi, v2, i2);
                }
                if (lane == 0) s_idx[r] = bi;
                __syncwarp();
            }
        } else {
            // PREFIX: the literal moe.go:49 bound orders only experts 0..k-1.
            if (lane == 0) {
                for (int i = 0; i < k; i++) s_idx[i] = i;
                for (int i = 1; i < k && i < E; i++)
                    for (int j = i; j > 0 && p[s_idx[j]] > p[s_idx[j - 1]]; j--) {
                        int tmp = s_idx[j];
                        s_idx[j] = s_idx[j - 1];
                        s_idx[j - 1] = tmp;
                    }
            }
            __syncwarp();
        }
        if (lane == 0) {
            float wsum = 0.f;
            for (int r = 0; r < k; r++) wsum = __fadd_rn(wsum, p[s_idx[r]]);
            const float den = __fadd_rn(wsum, 1e-9f);
            for (int r = 0; r < k; r++) {
                int e = s_idx[r];
                st.topk_idx[(size_t)t * k + r] = e;
                st.topk_w[(size_t)t * k + r] = __fdiv_rn(p[e], den);
            }
            if (has_shared) {
                float g = p[E];  // raw logit row E was not touched by softmax
                st.shared_w[t] = 1.f / (1.f + (float)exp(-(double)g));
            }
        }
        __syncwarp();
        if (lane < k) {
            int e = s_idx[lane];
            if (e >= 0 && e < E)
                atomicAdd(&st.counts[e], 1);
            else
                atomicOr(err, QG_FLAG_BAD_EXPERT);
        }
    }

    // ---- last CTA: dispatch --------------------------------------------
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(st.done_ctr, 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // Reuse dynamic smem: cnt[E], off[E], cur[E], wcnt[nwarps][E].
    int *cnt = reinterpret_cast<int *>(smem);
    int *cur = cnt + E;
    int *wcnt = cur + E;
    for (int e = tid; e < E; e += QG_ROUTE_THREADS) {
        cnt[e] = __ldcg(st.counts + e);
        st.counts[e] = 0;  // ready for the next call
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scan (serial per lane chunk, then warp scan of totals)
        const int per = (E + 31) / 32;
        int lo = lane * per, hi = min(E, lo + per);
        int run = 0;
        for (int e = lo; e < hi; e++) run += cnt[e];
        int incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int base = incl - run;
        for (int e = lo; e < hi; e++) {
            cur[e] = base;
            base += cnt[e];
        }
        // compact list of active experts, ascending id
        int nz = 0;
        for (int e = lo; e < hi; e++) nz += cnt[e] > 0;
        int nzi = nz;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, nzi, o);
            if (lane >= o) nzi += v;
        }
        int a = nzi - nz;
        for (int e = lo; e < hi; e++)
            if (cnt[e] > 0) {
                st.act_group[a] = e;
                st.act_begin[a] = cur[e];
                st.act_n[a] = cnt[e];
                a++;
            }
        int total_act = __shfl_sync(0xffffffffu, nzi, 31);
        if (lane == 0) {
            // 128-token tiles per routed group, for the tensor-core kernels
            int tiles = 0, ai = 0;
            for (int e = 0; e < E; e++)
                if (cnt[e] > 0) {
                    st.tile_prefix[ai++] = tiles;
                    tiles += (cnt[e] + 127) / 128;
                }
            st.tile_prefix[ai] = tiles;
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
    __syncthreads();

    // stable scatter of pairs (t, r) in pair order
    const int npairs = T * k;
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int base = 0; base < npairs; base += QG_ROUTE_THREADS) {
        for (int i = tid; i < nwarps * E; i += QG_ROUTE_THREADS) wcnt[i] = 0;
        __syncthreads();
        const int pi = base + tid;
        int e = -1;
        if (pi < npairs) {
            e = __ldcg(st.topk_idx + pi);
            if (e < 0 || e >= E) {
                atomicOr(err, QG_FLAG_BAD_EXPERT);
                e = -1;
            }
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & lt_mask);
        if (e >= 0 && rank == 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int slot = cur[e] + rank;
            for (int w = 0; w < warp; w++) slot += wcnt[w * E + e];
            if (slot < 0 || slot >= npairs) {
                atomicOr(err, QG_FLAG_BAD_SLOT);
            } else {
                st.pair_slot[pi] = slot;
                st.slot_token[slot] = pi / k;
            }
        }
        __syncthreads();
        for (int ee = tid; ee < E; ee += QG_ROUTE_THREADS) {
            int add = 0;
            for (int w = 0; w < nwarps; w++) add += wcnt[w * E + ee];
            cur[ee] += add;
        }
        __syncthreads();
    }
    if (has_shared)
        for (int i = tid; i < T; i += QG_ROUTE_THREADS) st.slot_token[npairs + i] = i;
}

int launch_route(const float *x, int T, int H, int E, int k, int mode, const float *router,
                 const float *shared_gate, int has_shared, RouteState st, int *err,
                 cudaStream_t s) {
    const int nwarps = QG_ROUTE_THREADS / 32;
    size_t route_bytes = sizeof(float) * ((size_t)H + E + 1);
    size_t disp_bytes = sizeof(int) * ((size_t)2 * E + (size_t)nwarps * E);
    size_t smem = route_bytes > disp_bytes ? route_bytes : disp_bytes;
    static bool attr_set = false;
    if (!attr_set) {
        QG_CUDA(cudaFuncSetAttribute(k_route, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024));
        attr_set = true;
    }
    k_route<<<T, QG_ROUTE_THREADS, smem, s>>>(x, T, H, E, k, mode, router, shared_gate,
                                              has_shared, st, err);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

}  // namespace qg
