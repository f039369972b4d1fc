// Router + dispatch (kernels K1 and K2).
//
// Launches: k_logits, k_topk, k_scatter (fused into k_topk for <= 32 tokens)
// (+ k_gather_f16 for the tensor path).
// 1. k_logits: logits = x . router^T (proj(x,1,&m.gate,...), model/moe.go:42)
//    as a split-K tiled f32 GEMM on CUDA cores: a CTA owns 64 tokens x 128
//    router rows (32 x 32 for 9-64 tokens, 8 x 32 for up to 8) x one K
//    slice.  The shared-expert gate vector rides along as
//    router row E (model/moe.go:87-93).  Split-K keeps decode-sized batches
//    (T = 1..64) spread over the SMs while the 1 MiB router matrix is read
//    about once; the K slices of one tile form a thread-block cluster and add
//    their partial tiles through distributed shared memory in rank order
//    (deterministic), so only final logits reach global memory.
// 2. k_topk: one warp per token reads its logits, then softmax (model/tensors.go:106-121: max-subtract, exp in float64 rounded
//    to float32, divide by the sum), top-k (model/moe.go:44-52, TOPK or the
//    literal PREFIX bound), w = p / (wSum + 1e-9) (model/moe.go:53-63) and
//    sigmoid of the shared gate.  Each CTA writes its expert histogram; the
//    last CTA (atomic ticket) scans the totals into expert offsets, the list
//    of active experts and the tensor-core tile prefix, and re-zeroes the
//    counters and the ticket so the next call (or a graph replay) starts clean.
// 3. k_scatter: each CTA ranks its own (token, rank) pairs per expert in pair
//    order (warp match + per-warp counts) and adds the histograms of the CTAs
//    before it, so slots are expert-sorted and deterministic without a serial
//    pass.  With one token chunk (<= 32 tokens) the single top-k CTA does this
//    itself once the offsets are known, one launch fewer.  For the tensor-core path k_gather_f16 then writes each slot's fp16
//    activation row.
#include "qg_common.cuh"
#include "qg_sm100.cuh"

namespace qg {
using sm100::cluster_ctarank;
using sm100::cluster_sync;
using sm100::ld_cluster_f32;
using sm100::mapa_shared;
using sm100::smem_u32;

constexpr int LG_KC = 32;    // K chunk staged in shared memory
constexpr int LG_MAX_SPLIT = 16; // K slices per tile = cluster size (16: non-portable opt-in)
constexpr int LG_SMALL_T = 8;    // up to this many tokens: 8 x 32 tiles,
constexpr int LG_MID_T = 64;     // up to this many: 32 x 32, else 64 x 128
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

// logits tile tier: 0 = 64 x 128, 1 = 8 x 32, 2 = 32 x 32
static int lg_tier(int T) { return T <= LG_SMALL_T ? 1 : T <= LG_MID_T ? 2 : 0; }

int route_splits(int T, int H, int Ep, int sms) {
    static const int tts[3] = {64, 8, 32}, rrs[3] = {128, 32, 32};
    const int TT = tts[lg_tier(T)], RR = rrs[lg_tier(T)];
    const int tiles = ((T + TT - 1) / TT) * ((Ep + RR - 1) / RR);
    int s = 1;  // a power of two: the cluster size
    while (s < LG_MAX_SPLIT && 2 * s * tiles <= sms && 2 * s * LG_KC <= H) s *= 2;
    return s;
}

// ---- 1. logits ------------------------------------------------------------------
// CTA tile: TT tokens x RR router rows x one K slice (TT x RR = 64 x 128 for
// prefill batches, 8 x 32 or 32 x 32 for decode batches, so that a handful
// of tokens still spreads over many CTAs).  Warp w owns tokens w*TT/8 ..., lane l owns
// rows l*RR/32 ...: per K step the warp's x values and the lane's router
// values come from shared memory and feed (TT/8) x (RR/32) FMAs.  The next K
// chunk is fetched into registers while the current one is consumed.  With
// KS > 1 the KS slices of a tile are one cluster: each CTA parks its partial
// tile in its shared memory, and CTA c then sums elements
// [c*TT*RR/KS, (c+1)*TT*RR/KS) of the tile over the ranks 0..KS-1 in order.
template <int TT, int RR>
struct LgTile {
    static constexpr int TPW = TT / 8;   // tokens per warp
    static constexpr int RPL = RR / 32;  // rows per lane
    static constexpr int STAGE_FLOATS = LG_KC * (TT + 4) + LG_KC * (RR + 4);
    static constexpr int SMEM =
        4 * (STAGE_FLOATS > TT * RR ? STAGE_FLOATS : TT * RR);
};

template <int TT, int RR, int KS>
__global__ void __launch_bounds__(256)
k_logits(const float *__restrict__ x, int T, int H, int E, int Ep, const float *__restrict__ router,
         const float *__restrict__ shared_gate, float *__restrict__ logits) {
    using Tl = LgTile<TT, RR>;
    constexpr int TPW = Tl::TPW, RPL = Tl::RPL;
    constexpr int XV = TT * LG_KC / 4;   // float4 loads of x per K chunk
    constexpr int WV = RR * LG_KC / 4;   // float4 loads of router rows per K chunk
    constexpr int XPT = (XV + 255) / 256, WPT = WV / 256;
    static_assert(WV % 256 == 0, "router chunk must split evenly over the CTA");
    pdl_enter();
    extern __shared__ __align__(16) float lg_smem[];
    float (*xs)[TT + 4] = reinterpret_cast<float (*)[TT + 4]>(lg_smem);
    float (*ws)[RR + 4] = reinterpret_cast<float (*)[RR + 4]>(lg_smem + LG_KC * (TT + 4));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * TT, r0 = blockIdx.y * RR, s = blockIdx.z;
    const int kc = ((H / LG_KC + KS - 1) / KS) * LG_KC;
    const int k0 = s * kc, k1 = min(H, k0 + kc);
    float acc[TPW][RPL] = {};
    // loaders: float4 i of a chunk covers item i / 8 (token or row), column (i % 8) * 4
    const float *xrow[XPT];
    int xi[XPT];
#pragma unroll
    for (int j = 0; j < XPT; j++) {
        xi[j] = tid + 256 * j;
        const int t = t0 + xi[j] / 8;
        xrow[j] = (xi[j] < XV && t < T) ? x + (size_t)t * H : nullptr;
    }
    const float *wrow[WPT];
#pragma unroll
    for (int j = 0; j < WPT; j++) {
        const int r = r0 + (tid + 256 * j) / 8;
        wrow[j] = r < Ep ? (r < E ? router + (size_t)r * H : shared_gate) : nullptr;
    }
    const int c4 = (tid % 8) * 4;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 xn[XPT], wn[WPT];
    auto fetch = [&](int kb) {
#pragma unroll
        for (int j = 0; j < XPT; j++)
            xn[j] = xrow[j] ? *reinterpret_cast<const float4 *>(xrow[j] + kb + c4) : zero;
#pragma unroll
        for (int j = 0; j < WPT; j++)
            wn[j] = wrow[j] ? __ldg(reinterpret_cast<const float4 *>(wrow[j] + kb + c4)) : zero;
    };
    if (k0 < k1) fetch(k0);
    for (int kb = k0; kb < k1; kb += LG_KC) {
#pragma unroll
        for (int j = 0; j < XPT; j++)
            if (xi[j] < XV) {
                const int t = xi[j] / 8;
                xs[c4][t] = xn[j].x;
                xs[c4 + 1][t] = xn[j].y;
                xs[c4 + 2][t] = xn[j].z;
                xs[c4 + 3][t] = xn[j].w;
            }
#pragma unroll
        for (int j = 0; j < WPT; j++) {
            const int row = (tid + 256 * j) / 8;
            ws[c4][row] = wn[j].x;
            ws[c4 + 1][row] = wn[j].y;
            ws[c4 + 2][row] = wn[j].z;
            ws[c4 + 3][row] = wn[j].w;
        }
        __syncthreads();
        if (kb + LG_KC < k1) fetch(kb + LG_KC);
#pragma unroll 4
        for (int kk = 0; kk < LG_KC; kk++) {
            float av[TPW], bv[RPL];
            if constexpr (TPW % 4 == 0) {
#pragma unroll
                for (int i = 0; i < TPW; i += 4) {
                    const float4 v = *reinterpret_cast<const float4 *>(&xs[kk][TPW * warp + i]);
                    av[i] = v.x, av[i + 1] = v.y, av[i + 2] = v.z, av[i + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < TPW; i++) av[i] = xs[kk][TPW * warp + i];
            }
            if constexpr (RPL % 4 == 0) {
#pragma unroll
                for (int j = 0; j < RPL; j += 4) {
                    const float4 v = *reinterpret_cast<const float4 *>(&ws[kk][RPL * lane + j]);
                    bv[j] = v.x, bv[j + 1] = v.y, bv[j + 2] = v.z, bv[j + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < RPL; j++) bv[j] = ws[kk][RPL * lane + j];
            }
#pragma unroll
            for (int i = 0; i < TPW; i++)
#pragma unroll
                for (int j = 0; j < RPL; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
    if constexpr (KS == 1) {
#pragma unroll
        for (int i = 0; i < TPW; i++) {
            const int t = t0 + TPW * warp + i;
            if (t >= T) continue;
#pragma unroll
            for (int j = 0; j < RPL; j++) {
                const int r = r0 + RPL * lane + j;
                if (r < Ep) logits[(size_t)t * Ep + r] = acc[i][j];
            }
        }
    } else {
        // partial tile [TT tokens][RR rows] over the staging buffers (the K
        // loop ended with a barrier)
        float *red = lg_smem;
#pragma unroll
        for (int i = 0; i < TPW; i++)
#pragma unroll
            for (int j = 0; j < RPL; j++) red[(TPW * warp + i) * RR + RPL * lane + j] = acc[i][j];
        cluster_sync();
        constexpr int EPC = TT * RR / KS;  // tile elements reduced by this CTA
        const int c = (int)cluster_ctarank();
        for (int idx = c * EPC + tid; idx < (c + 1) * EPC; idx += 256) {
            const uint32_t off = smem_u32(red + idx);
            float v[KS];
#pragma unroll
            for (int q = 0; q < KS; q++) v[q] = ld_cluster_f32(mapa_shared(off, q));
            float sum = v[0];
#pragma unroll
            for (int q = 1; q < KS; q++) sum += v[q];
            const int t = t0 + idx / RR, row = r0 + idx % RR;
            if (t < T && row < Ep) logits[(size_t)t * Ep + row] = sum;
        }
        cluster_sync();  // no CTA leaves while others still read its tile
    }
}

// ---- 2. softmax + top-k + histograms --------------------------------------------
// A warp holds one token's probabilities in registers: lane l owns experts
// l, l+32, ..., l+32*(NJ-1) (NJ = ceil(E/32) rounded up to a power of two).
__device__ __forceinline__ void scatter_chunk(int c, int T, int E, int k, int has_shared,
                                              const RouteState &st, int *err, int *sm,
                                              int *partial);

// FUSED (T <= TK_TOK, one CTA): the scatter of the single token chunk
// follows in the same CTA once the expert offsets are known.
template <int NJ, bool FUSED>
__global__ void __launch_bounds__(RT_THREADS)
k_topk(const float *__restrict__ logits, int T, int E, int Ep, int k, int mode,
       int has_shared, RouteState st, int *err) {
    pdl_enter();
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
            v[j] = e < E ? logits[(size_t)t * Ep + e] : -INFINITY;
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
                atomicAdd(&hist_s[dispatch_key(e, E, st.ep_world, st.ep_slot)], 1);
            else
                atomicOr(err, QG_FLAG_BAD_EXPERT);
        }
        if (has_shared && lane == 0) {
            const float g = logits[(size_t)t * Ep + E];
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
        // one warp-wide exclusive scan of (pairs, active experts, tiles) over
        // contiguous per-lane expert ranges; every lane then writes its own
        // experts' offsets, active-list entries and tile prefixes
        const int tt = st.tile_tokens > 0 ? st.tile_tokens : 256;  // a power of two
        const int tsh = __ffs(tt) - 1;
        const int per = (E + 31) / 32;
        const int lo = min(E, lane * per), hi = min(E, lo + per);
        int run = 0, nz = 0, tl = 0;
        for (int e = lo; e < hi; e++) {
            const int c = cnt[e];
            run += c;
            nz += c > 0;
            tl += (c + tt - 1) >> tsh;
        }
        int incl = run, nzi = nz, tli = tl;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            const int w = __shfl_up_sync(0xffffffffu, nzi, o);
            const int x = __shfl_up_sync(0xffffffffu, tli, o);
            if (lane >= o) {
                incl += v;
                nzi += w;
                tli += x;
            }
        }
        int base = incl - run, a = nzi - nz, tb = tli - tl;
        for (int e = lo; e < hi; e++) {
            const int c = cnt[e];
            st.expert_off[e] = base;
            if (c > 0) {
                st.act_group[a] = e;
                st.act_begin[a] = base;
                st.act_n[a] = c;
                st.tile_prefix[a] = tb;
                tb += (c + tt - 1) >> tsh;
                a++;
            }
            base += c;
        }
        const int routed_act = __shfl_sync(0xffffffffu, nzi, 31);
        if (lane == 31) {
            st.tile_prefix[routed_act] = tli;
            if (st.n_act_routed) *st.n_act_routed = routed_act;
            int total_act = routed_act;
            if (has_shared && st.shared_act) {
                st.shared_act[0] = 0;
                st.shared_act[1] = T * k;
                st.shared_act[2] = T;
                st.shared_act[3] = 1;
                st.shared_act[4] = 0;
                st.shared_act[5] = (T + tt - 1) >> tsh;
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
    if constexpr (FUSED) {
        __shared__ int partial[RT_THREADS];
        __syncthreads();  // expert offsets and top-k pairs written by this CTA
        scatter_chunk(0, T, E, k, has_shared, st, err, hist_s, partial);
    }
}

// ---- 3. scatter ---------------------------------------------------------------------
// Slots of token chunk c (TK_TOK tokens, one CTA of RT_THREADS threads); sm
// holds (RT_WARPS + 1) * E ints.
__device__ __forceinline__ void scatter_chunk(int c, int T, int E, int k, int has_shared,
                                              const RouteState &st, int *err, int *sm,
                                              int *partial) {
    int *cur = sm;            // [E] next slot per expert for this CTA
    int *wcnt = sm + E;       // [RT_WARPS][E]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
                e = dispatch_key(e, E, st.ep_world, st.ep_slot);
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

__global__ void __launch_bounds__(RT_THREADS)
k_scatter(int T, int E, int k, int has_shared, RouteState st, int *err) {
    pdl_enter();
    extern __shared__ int sm[];
    __shared__ int partial[RT_THREADS];
    scatter_chunk(blockIdx.x, T, E, k, has_shared, st, err, sm, partial);
}

// CUDA-core logits: the split-K tiled f32 GEMM above.
static int launch_logits(const float *x, int T, int H, int E, int Ep, const float *router,
                         const float *shared_gate, float *logits, int dev, cudaStream_t s) {
    const int ks = route_splits(T, H, Ep, num_sms(dev));
    const int tier = lg_tier(T);
    using LgKern = void (*)(const float *, int, int, int, int, const float *, const float *, float *);
    static const LgKern kerns[3][5] = {
        {k_logits<64, 128, 1>, k_logits<64, 128, 2>, k_logits<64, 128, 4>, k_logits<64, 128, 8>,
         k_logits<64, 128, 16>},
        {k_logits<8, 32, 1>, k_logits<8, 32, 2>, k_logits<8, 32, 4>, k_logits<8, 32, 8>,
         k_logits<8, 32, 16>},
        {k_logits<32, 32, 1>, k_logits<32, 32, 2>, k_logits<32, 32, 4>, k_logits<32, 32, 8>,
         k_logits<32, 32, 16>}};
    static const int tts[3] = {64, 8, 32}, rrs[3] = {128, 32, 32};
    static const int smems[3] = {LgTile<64, 128>::SMEM, LgTile<8, 32>::SMEM, LgTile<32, 32>::SMEM};
    const int ki = ks == 1 ? 0 : ks == 2 ? 1 : ks == 4 ? 2 : ks == 8 ? 3 : 4;
    const LgKern kern = kerns[tier][ki];
    static bool wide[64] = {false};  // 16-CTA clusters need the non-portable opt-in
    if (dev < 64 && !wide[dev]) {
        for (int i = 0; i < 3; i++)
            QG_CUDA(cudaFuncSetAttribute(kerns[i][4], cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        wide[dev] = true;
    }
    const int TT = tts[tier], RR = rrs[tier];
    QG_CUDA(launch_pdl(kern, dim3((T + TT - 1) / TT, (Ep + RR - 1) / RR, ks), dim3(256),
                       smems[tier], s, ks, x, T, H, E, Ep, router, shared_gate, logits));
    return QGMOE_OK;
}

int launch_route(const float *x, int T, int H, int E, int k, int mode, const float *router,
                 const float *shared_gate, int has_shared, RouteState st, __half *xp, int *err,
                 cudaStream_t s, const RouterTC *tc) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int Ep = E + (has_shared ? 1 : 0);
    const bool on_tc = tc && T >= RTC_MIN_T && T <= tc->cap && Ep <= tc->rows_pad;
    if (on_tc) {
        int rc = launch_logits_tc(*tc, x, T, H, Ep, st.logits, err, s);
        if (rc) return rc;
    } else {
        int rc = launch_logits(x, T, H, E, Ep, router, shared_gate, st.logits, dev, s);
        if (rc) return rc;
    }
    const int nc = (T + TK_TOK - 1) / TK_TOK;
    const size_t sm2 = sizeof(int) * (size_t)E;
    const size_t sm3 = sizeof(int) * (size_t)(RT_WARPS + 1) * E;
    static bool attr[64] = {false}, attr_f[64] = {false};
    if (dev < 64 && !attr[dev]) {
        QG_CUDA(cudaFuncSetAttribute(k_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        attr[dev] = true;
    }
    const int nj = (E + 31) / 32;
    using TkKern = void (*)(const float *, int, int, int, int, int, int, RouteState, int *);
    static const TkKern tk[2][6] = {
        {k_topk<1, false>, k_topk<2, false>, k_topk<4, false>, k_topk<8, false>,
         k_topk<16, false>, k_topk<32, false>},
        {k_topk<1, true>, k_topk<2, true>, k_topk<4, true>, k_topk<8, true>, k_topk<16, true>,
         k_topk<32, true>}};
    const int ji = nj <= 1 ? 0 : nj <= 2 ? 1 : nj <= 4 ? 2 : nj <= 8 ? 3 : nj <= 16 ? 4 : 5;
    const bool fused = nc == 1;  // one token chunk: top-k and scatter in one CTA
    if (fused && dev < 64 && !attr_f[dev]) {
        for (int i = 0; i < 6; i++)
            QG_CUDA(cudaFuncSetAttribute(tk[1][i], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         160 * 1024));
        attr_f[dev] = true;
    }
    QG_CUDA(launch_pdl(tk[fused][ji], dim3(nc), dim3(RT_THREADS), fused ? sm3 : sm2, s, 1,
                       (const float *)st.logits, T, E, Ep, k, mode, has_shared, st, err));
    QG_CUDA(cudaGetLastError());
    if (!fused) {
        QG_CUDA(launch_pdl(k_scatter, dim3(nc), dim3(RT_THREADS), sm3, s, 1, T, E, k, has_shared,
                           st, err));
        QG_CUDA(cudaGetLastError());
    }
    if (xp) {
        const int nslots = T * k + (has_shared ? T : 0);
        // after the tensor-core logits the fp16 rows exist already (xh = fp16(x))
        return on_tc ? launch_gather_h16(tc->xh, st.slot_token, nslots, H, xp, s)
                     : launch_gather_f16(x, st.slot_token, nslots, H, xp, s);
    }
    return QGMOE_OK;
}

}  // namespace qg
