// The MoE forward of a decode-sized batch (T <= FD_MAX_T tokens) as ONE
// persistent kernel: one CTA per SM, phases separated by grid barriers whose
// waits all give up after about a second (QG_FLAG_TIMEOUT).
//
// The router logits must be the reference's serial float32 sums
// (model/tensors.go:77-89 via model/moe.go:42): H dependent adds per
// (token, router row), a few microseconds that no parallelism shortens.  So
// they run on their own warp in each CTA (the "chain" warp: CTA b owns
// router rows b, b + G, ..., one chain per lane) while the other warps do
// everything else speculatively:
//   1. approximate logits (the same products, summed in parallel) of the
//      CTA's router rows -> grid barrier;
//   2. every CTA: the approximate top-k of each token (the candidates) and
//      the batch's distinct candidate experts;
//   3. gate_up + SwiGLU of the candidates and the shared expert
//      (model/moe.go:64-76, model/model.go:350-358) -> grid barrier (f32 /
//      bf16 experts) or, on the tensor path, per-task counters: a down task
//      starts once its own gate_up tiles are done;
//   4. down rows of every (token, candidate) pair -> grid barrier;
//   5. wait for the exact routing, which the chain warps publish once every
//      chain has finished: the reference's softmax, top-k and weights
//      (model/moe.go:41-63) per token; pairs the candidates missed (a near
//      tie the approximate sums ordered differently, or a NaN) get their
//      own gate_up and down phases here;
//   6. combine: out[t] = sum over ranks in order of w * d (+ sigmoid gate *
//      shared), model/moe.go:77-97, rounded like k_combine.
// Expert weights stream through a ring of a.ns stages in shared memory, fed
// by 1-D bulk copies (cp.async.bulk + mbarriers).
//
// Expert products.  int8 / int4 experts run on the tensor cores with
// mma.sync m16n8k16 (fp16 operands, f32 accumulation) over the tensor
// path's packed weight tiles (128 rows x 64 codes, codes chunk-major so that
// a tile's rows sit side by side in shared memory): one bulk copy brings
// several k blocks of a tile, each of 8 warps owns 16 rows of it for the
// tile's whole K, and the batch's tokens are the 8 columns of B, so one
// dequantisation of a weight serves every token.  A group's two MMAs are
// scaled by its fp16 group scale in f32 -- the arithmetic of the prefill
// tensor-core path (activations and h in fp16; a finite value beyond fp16
// range raises QG_FLAG_RANGE).  bf16 / f32 experts keep the CUDA-core
// GEMV's arithmetic (fz_dot, row-major rows copied one by one), bit for bit.
#include <algorithm>

#include "qg_common.cuh"
#include "qg_gemv.cuh"
#include "qg_router.cuh"
#include "qg_sm100.cuh"

namespace qg {

constexpr int FZ_THREADS = 384;
constexpr int FZ_WORKERS = FZ_THREADS / 32 - 1;  // warp FZ_WORKERS runs the logit chains
constexpr int FZ_WT = FZ_WORKERS * 32;
constexpr int FZ_NSMAX = 6;                      // weight ring stages at most
constexpr int FZ_RMAX = 64;                      // output rows per item (CUDA-core path)
constexpr int FZ_MW = 8;                         // tensor-core path: warps, 16 tile rows each
constexpr int FZ_PROD = FZ_MW;                   // tensor-core path: the producer warp
constexpr int FZ_MAXD = FD_MAX_T * QG_MAX_TOPK;  // distinct experts of a batch
constexpr int FZ_B4 = 8;                         // float4 per chain block
constexpr long long FZ_WAIT = 2000000000LL;      // ~1 s of cycles, then a wait gives up
constexpr int FZ_SMEM_MAX = 200 * 1024;          // dynamic shared memory of the plan
constexpr int FZ_STAGE_MAX = 36 * 1024;
constexpr int FZ_PAD = 16;                       // bytes after each staged row

// A phase's expert tasks: task d is expert dexp[d] for the tokens in
// dmask[d]; its h / d row for token t is slot base + t * k + rank[d][t].
struct FzList {
    int n, base;
    int dexp[FZ_MAXD];
    unsigned dmask[FZ_MAXD];
    signed char rank[FZ_MAXD][FD_MAX_T];
};

struct FzShared {
    uint64_t full[FZ_NSMAX], empty[FZ_NSMAX];
    uint64_t wbar, hbar, xbar;             // router rows; staged h rows; token rows
    FzList A, B;                           // speculative tasks; tasks after exact routing
    int cand[FD_MAX_T][QG_MAX_TOPK];       // approximate selection (-1: none)
    int sel[FD_MAX_T][QG_MAX_TOPK];        // exact selection
    float w[FD_MAX_T][QG_MAX_TOPK];        // exact weights
    float sg[FD_MAX_T];
    int slot[FD_MAX_T][QG_MAX_TOPK];       // d row of (token, exact rank)
    float part[FZ_WORKERS][2 * FD_MAX_T];  // approximate-logit partial sums
    int rsel[QG_MAX_TOPK];
    unsigned long long base;               // barrier arrivals before this launch
    int nbar;                              // grid barriers passed (thread 0)
    int cand_ready;                        // S.cand is final
};

__device__ __forceinline__ void wsync() {
    asm volatile("bar.sync 1, %0;" ::"r"(FZ_WT) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acq(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_rel(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Generic-proxy writes (other CTAs' h rows, acquired through a barrier)
// ordered before this thread's bulk copies read them.
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async;" ::: "memory");
}

__device__ __forceinline__ void fz_timeout(const DecodeArgs &a) { atomicOr(a.err, QG_FLAG_TIMEOUT); }

// All worker threads of every CTA.  The arrival counter only grows, by G
// per barrier: a launch's n-th barrier completes when it reaches base +
// n G, where base (a multiple of G) is the count when the launch began.
// Arrivals are fire-and-forget releases; thread 0 polls with acquires.  The
// CTA barrier orders the other workers' writes before thread 0's release
// (release is cumulative) and after its acquire, so no separate fences.
__device__ void fz_grid_sync(const DecodeArgs &a, FzShared &S) {
    wsync();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(a.bar) : "memory");
        const unsigned long long target = S.base + (unsigned long long)(++S.nbar) * gridDim.x;
        if (ld_acq(a.bar) < target) {
            const long long budget = a.wait > 0 ? a.wait : FZ_WAIT;
            const long long t0 = clock64();
            while (ld_acq(a.bar) < target) {
                if (clock64() - t0 > budget) {
                    fz_timeout(a);
                    break;
                }
            }
        }
    }
    wsync();
}

__device__ __forceinline__ bool fz_wait_flag(const DecodeArgs &a, const unsigned long long *f,
                                             unsigned long long v) {
    if (ld_acq(f) >= v) return true;
    const long long budget = a.wait > 0 ? a.wait : FZ_WAIT;
    const long long t0 = clock64();
    while (ld_acq(f) < v) {
        if (clock64() - t0 > budget) {
            fz_timeout(a);
            return false;
        }
        __nanosleep(32);
    }
    return true;
}

// Bounded wait until *p >= v (acquire).
__device__ __forceinline__ bool fz_wait_u32(const DecodeArgs &a, const unsigned *p, unsigned v) {
    auto ld = [&]() {
        unsigned r;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
        return r;
    };
    if (ld() >= v) return true;
    const long long budget = a.wait > 0 ? a.wait : FZ_WAIT;
    const long long t0 = clock64();
    while (ld() < v) {
        if (clock64() - t0 > budget) return false;
        __nanosleep(32);
    }
    return true;
}

// ---- CUDA-core products (f32 / bf16 experts) ---------------------------------------
// NR weight rows in shared memory dotted with the staged rows of the tokens
// in `mask` (token t at xs + t * xstride): per lane the chunks lane,
// lane+32, ... in order (FMA over a chunk's V elements, then FMA with the
// unit scale), then a warp reduction -- the CUDA-core GEMV's arithmetic.
template <int BITS, int NR, int MT>
__device__ __forceinline__ void fz_dot(const uint8_t *const (&rows)[NR], int nchunks,
                                       const float *xs, int xstride, unsigned mask, int lane,
                                       float (&acc)[NR][MT]) {
    constexpr int V = Chunk<BITS>::V;
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
        for (int t = 0; t < MT; t++) acc[r][t] = 0.f;
    for (int c = lane; c < nchunks; c += 32) {
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const uint4 raw = reinterpret_cast<const uint4 *>(rows[r])[c];
            float v[V];
            decode_chunk<BITS>(raw, v);
#pragma unroll
            for (int t = 0; t < MT; t++) {
                if (!((mask >> t) & 1u)) continue;
                const float *xt = xs + t * xstride;
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
                acc[r][t] = fmaf(part, 1.f, acc[r][t]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
        for (int t = 0; t < MT; t++)
            if ((mask >> t) & 1u)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[r][t] += __shfl_xor_sync(FULL, acc[r][t], o);
}

// ---- tensor-core products (int8 / int4 experts) -------------------------------------
// The packed tile (k_repack, qg_umma.cu): codes chunk-major [chunk c of 16
// codes][128 rows][CB bytes] -- int8 biased (q + 128), int4 words holding
// elements 2j at bits 4j.. and 2j+1 at bits 16+4j.. -- then each row's two
// fp16 group scales.
template <int BITS>
struct PTile {
    static constexpr int CB = BITS == 8 ? 16 : 8;
    static constexpr int CODE = 128 * 64 * BITS / 8;
    static constexpr int BYTES = CODE + 128 * 4;
};

__device__ __forceinline__ void msync() {
    asm volatile("bar.sync 2, %0;" ::"r"(FZ_MW * 32) : "memory");
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Eight consecutive codes of one tile row -> four fp16 pairs {0,1} {2,3}
// {4,5} {6,7}, exact (code - 8, or the unbiased int8 code).
template <int BITS>
__device__ __forceinline__ void tc_word(const unsigned char *p, uint32_t (&c)[4]) {
    if constexpr (BITS == 4) {
        const __half2 b1032 = u2h(0x64086408u), r16 = u2h(0x2C002C00u), m72 = u2h(0xD480D480u);
        const uint32_t w = *reinterpret_cast<const uint32_t *>(p), w8 = w >> 8;
        c[0] = h2u(__hsub2(u2h((w & 0x000F000Fu) | 0x64006400u), b1032));
        c[1] = h2u(__hfma2(u2h((w & 0x00F000F0u) | 0x64006400u), r16, m72));
        c[2] = h2u(__hsub2(u2h((w8 & 0x000F000Fu) | 0x64006400u), b1032));
        c[3] = h2u(__hfma2(u2h((w8 & 0x00F000F0u) | 0x64006400u), r16, m72));
    } else {
        const __half2 b1152 = u2h(0x64806480u);
        const uint2 u = *reinterpret_cast<const uint2 *>(p);
        c[0] = h2u(__hsub2(u2h(__byte_perm(u.x, 0x64646464u, 0x4140)), b1152));
        c[1] = h2u(__hsub2(u2h(__byte_perm(u.x, 0x64646464u, 0x4342)), b1152));
        c[2] = h2u(__hsub2(u2h(__byte_perm(u.y, 0x64646464u, 0x4140)), b1152));
        c[3] = h2u(__hsub2(u2h(__byte_perm(u.y, 0x64646464u, 0x4342)), b1152));
    }
}

// One 32-wide scale group (chunks 2 grp, 2 grp + 1) of tile rows r0 and
// r0 + 8 against B (this thread's token row, fp16, at xb = the k block's 64
// elements): thread (g, q) takes codes base .. base+7, base = 16 (q / 2) +
// 8 (q % 2) of the group, as k slots 2q, 2q+1, 2q+8, 2q+9 of the group's two
// MMAs (codes base+0..3, then base+4..7); B holds the same elements.
template <int BITS>
__device__ __forceinline__ void tc_group(const unsigned char *tile, const unsigned char *xb,
                                         int grp, int r0, int q, float (&d)[4]) {
    using P = PTile<BITS>;
    const unsigned char *ra = tile + ((grp * 2 + (q >> 1)) * 128 + r0) * P::CB + (q & 1) * (P::CB / 2);
    uint32_t ca[4], cb[4];
    tc_word<BITS>(ra, ca);
    tc_word<BITS>(ra + 8 * P::CB, cb);
    const uint4 b = *reinterpret_cast<const uint4 *>(xb + (grp * 32 + (q >> 1) * 16 + (q & 1) * 8) * 2);
    d[0] = d[1] = d[2] = d[3] = 0.f;
    mma16816(d, ca[0], cb[0], ca[1], cb[1], b.x, b.y);
    mma16816(d, ca[2], cb[2], ca[3], cb[3], b.z, b.w);
}

// One 64-code k block: its two groups, each scaled by the rows' group scale
// in f32 into acc (C rows g / g + 8, columns 2q, 2q+1).
template <int BITS>
__device__ __forceinline__ void tc_kblock(const unsigned char *tile, const unsigned char *xb,
                                          int r0, int q, float (&acc)[4]) {
    using P = PTile<BITS>;
    const float2 s0 = __half22float2(u2h(*reinterpret_cast<const uint32_t *>(tile + P::CODE + r0 * 4)));
    const float2 s1 =
        __half22float2(u2h(*reinterpret_cast<const uint32_t *>(tile + P::CODE + (r0 + 8) * 4)));
#pragma unroll
    for (int grp = 0; grp < 2; grp++) {
        float d[4];
        tc_group<BITS>(tile, xb, grp, r0, q, d);
        const float sa = grp ? s0.y : s0.x, sb = grp ? s1.y : s1.x;
        acc[0] = fmaf(d[0], sa, acc[0]);
        acc[1] = fmaf(d[1], sa, acc[1]);
        acc[2] = fmaf(d[2], sb, acc[2]);
        acc[3] = fmaf(d[3], sb, acc[3]);
    }
}

// One streaming phase on the tensor cores.  Units are (task, 128-row tile):
// a gate_up tile holds 64 gate rows and the matching 64 up rows, a down tile
// 128 output rows; each CTA takes a contiguous range of units, and the
// producer warp streams their k blocks, kbi per item, one bulk copy each.
// Warp m accumulates tile rows 16m .. 16m+15 over the tile's whole K; at a
// gate_up tile's end the up warps hand their sums to the gate warps, which
// form h = silu(g) * u (fp16) for the tile's 64 rows.
template <int BITS, bool GATEUP>
__device__ void fz_phase_tc(const DecodeArgs &a, FzShared &S, const FzList &L, bool with_shared,
                            unsigned char *smem, int &qi, int &qc, int &hph, int &nx,
                            unsigned *tdone) {
    using P = PTile<BITS>;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, b = blockIdx.x, T = a.T, k = a.k;
    const int rt_r = GATEUP ? a.I / 64 : a.H / 128, rt_s = GATEUP ? a.Is / 64 : a.H / 128;
    const int KB_r = (GATEUP ? a.H : a.I) / 64, KB_s = (GATEUP ? a.H : a.Is) / 64;
    const int kbi_r = GATEUP ? a.kbi_gu : a.kbi_dn, kbi_s = GATEUP ? a.kbi_gu : a.kbi_sdn;
    const int ni_r = KB_r / kbi_r, ni_s = with_shared ? KB_s / kbi_s : 1;
    const int nu_r = L.n * rt_r, nu = nu_r + (with_shared ? rt_s : 0);
    const int u0 = (int)((long long)nu * b / G), u1 = (int)((long long)nu * (b + 1) / G);
    if (u0 >= u1) return;
    const int cr = max(0, min(u1, nu_r) - u0);  // routed units of the range, then shared ones
    const int nitems = cr * ni_r + (u1 - u0 - cr) * ni_s;
    const unsigned all = (1u << T) - 1u;
    struct It {
        int d, rt, it, ni, kbi, KB, e;
        unsigned mask;
        bool shared;
    };
    auto item = [&](int j) {
        It x;
        x.shared = j >= cr * ni_r;
        if (!x.shared) {
            const int u = u0 + j / ni_r;
            x.it = j % ni_r, x.ni = ni_r, x.kbi = kbi_r, x.KB = KB_r;
            x.d = u / rt_r, x.rt = u - x.d * rt_r, x.e = L.dexp[x.d], x.mask = L.dmask[x.d];
        } else {
            const int jj = j - cr * ni_r;
            const int u = max(u0, nu_r) + jj / ni_s;
            x.it = jj % ni_s, x.ni = ni_s, x.kbi = kbi_s, x.KB = KB_s;
            x.d = L.n, x.rt = u - nu_r, x.e = 0, x.mask = all;
        }
        return x;
    };
    auto slot = [&](int d, int t) {
        return d < L.n ? L.base + t * k + L.rank[d][t] : T * k + t;
    };
    if (warp == FZ_PROD) {
        if (lane == 0)
            for (int j = 0; j < nitems; j++) {
                const It x = item(j);
                const int q = qi++, s = q % a.ns;
                if (q >= a.ns && !sm100::mbar_wait(&S.empty[s], ((q / a.ns) + 1) & 1, 0, FZ_WAIT))
                    fz_timeout(a);
                const uint8_t *pq = x.shared ? (GATEUP ? a.sgu_pq : a.sdn_pq)
                                             : (GATEUP ? a.gu_pq : a.dn_pq);
                const size_t tile0 =
                    ((size_t)x.e * (x.shared ? rt_s : rt_r) + x.rt) * x.KB + (size_t)x.it * x.kbi;
                const uint32_t bytes = (uint32_t)(x.kbi * P::BYTES);
                sm100::mbar_arrive_expect_tx(&S.full[s], bytes);
                sm100::bulk_load(smem + a.off_ring + s * a.stage_bytes, pq + tile0 * P::BYTES,
                                 bytes, &S.full[s]);
            }
        __syncwarp();
        return;
    }
    if (warp >= FZ_MW) return;
    const int g = lane >> 2, qq = lane & 3, m = warp;
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    int hd = -1;  // task whose h rows are staged (down)
    for (int j = 0; j < nitems; j++) {
        const It x = item(j);
        if (!GATEUP && x.it == 0 && x.d != hd) {
            msync();  // every warp is past the previous task's items
            hd = x.d;
            const int K = x.shared ? a.Is : a.I;
            if (tid == 0) {
                // every gate_up tile of the task has written its h rows
                if (!fz_wait_u32(a, tdone + x.d, (unsigned)(x.shared ? a.Is / 64 : a.I / 64)))
                    fz_timeout(a);
                fence_proxy_async();
                sm100::mbar_arrive_expect_tx(&S.hbar, (uint32_t)(__popc(x.mask) * K * 2));
                for (int t = 0; t < T; t++)
                    if ((x.mask >> t) & 1u)
                        sm100::bulk_load(smem + a.off_hs + t * a.h16tok,
                                         a.hbuf + (size_t)slot(x.d, t) * a.hrow, K * 2, &S.hbar);
            }
            if (!sm100::mbar_wait(&S.hbar, hph & 1, 0, FZ_WAIT) && lane == 0) fz_timeout(a);
            hph++;
        }
        const int q = qc++, s = q % a.ns;
        if (!sm100::mbar_wait(&S.full[s], (q / a.ns) & 1, 0, FZ_WAIT) && lane == 0) fz_timeout(a);
        const unsigned char *st = smem + a.off_ring + s * a.stage_bytes;
        const unsigned char *xrow =
            GATEUP ? smem + a.off_x16 + g * a.x16tok : smem + a.off_hs + g * a.h16tok;
        // even and odd k blocks into separate sums: two independent chains
        const unsigned char *xk = xrow + (size_t)x.it * x.kbi * 128;
        int kk = 0;
        for (; kk + 1 < x.kbi; kk += 2) {
            tc_kblock<BITS>(st + kk * P::BYTES, xk + kk * 128, 16 * m + g, qq, acc);
            tc_kblock<BITS>(st + (kk + 1) * P::BYTES, xk + (kk + 1) * 128, 16 * m + g, qq, acc2);
        }
        if (kk < x.kbi) tc_kblock<BITS>(st + kk * P::BYTES, xk + kk * 128, 16 * m + g, qq, acc);
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&S.empty[s]);
        if (x.it != x.ni - 1) continue;
        // the unit's rows are complete; C rows g / g + 8, columns (tokens) 2q, 2q+1
#pragma unroll
        for (int i = 0; i < 4; i++) acc[i] += acc2[i], acc2[i] = 0.f;
        if constexpr (GATEUP) {
            float4 *xch = reinterpret_cast<float4 *>(smem + a.off_xch) + (nx & 1) * 4 * 32;
            if (m >= 4) xch[(m - 4) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            msync();
            nx++;
            if (m < 4) {
                const float4 u4 = xch[m * 32 + lane];
                const float up[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int t = 2 * qq + h;
                    if (t >= T || !((x.mask >> t) & 1u)) continue;
                    __half *hrow = reinterpret_cast<__half *>(a.hbuf + (size_t)slot(x.d, t) * a.hrow);
#pragma unroll
                    for (int hf = 0; hf < 2; hf++) {
                        const float hv = __fmul_rn(silu_ref(acc[2 * hf + h]), up[2 * hf + h]);
                        const __half hh = __float2half_rn(hv);
                        if (isinf(__half2float(hh)) && isfinite(hv)) atomicOr(a.err, QG_FLAG_RANGE);
                        hrow[x.rt * 64 + 16 * m + g + 8 * hf] = hh;
                    }
                }
            }
            // the tile's h rows are out: count it for its task (the down
            // phase stages a task's h rows once all its tiles are counted)
            msync();
            if (tid == 0)
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(tdone + x.d) : "memory");
        } else {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int t = 2 * qq + h;
                if (t >= T || !((x.mask >> t) & 1u)) continue;
                float *drow = a.dbuf + (size_t)slot(x.d, t) * a.H + x.rt * 128 + 16 * m + g;
                drow[0] = acc[h];
                drow[8] = acc[2 + h];
            }
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
}

template <int BITS>
__device__ __forceinline__ int fz_row_bytes(int K) {
    return BITS == 32 ? K * 4 : BITS == 16 ? K * 2 : BITS == 8 ? K : K / 2;
}

// Rows per item of the CUDA-core phase.
struct FzGeom {
    int R;
    __device__ FzGeom(int stage, int nblk, int rbp) { R = min(FZ_RMAX, stage / (nblk * rbp)); }
};

// One streaming phase on CUDA cores (f32 / bf16 experts): GATEUP computes h
// rows of the list's tasks (and of the shared expert), else down rows.  The
// phase's items (task, block of R output rows) are split into one
// contiguous range per CTA; warp 0 keeps a.ns - 1 items of weight rows in
// flight ahead of the workers, one bulk copy per row into rows padded by
// FZ_PAD bytes.  qi / qc count the ring's items issued (warp 0) and consumed
// (every worker) over the whole kernel, hph the h-staging rounds.
template <int BITS, int MT, bool GATEUP>
__device__ void fz_phase(const DecodeArgs &a, FzShared &S, const FzList &L, bool with_shared,
                         unsigned char *smem, int &qi, int &qc, int &hph) {
    constexpr int V = Chunk<BITS>::V;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, b = blockIdx.x, T = a.T, k = a.k;
    const int nblk = GATEUP ? 2 : 1;
    const int rows_r = GATEUP ? a.I : a.H, rows_s = GATEUP ? a.Is : a.H;
    const int K_r = GATEUP ? a.H : a.I, K_s = GATEUP ? a.H : a.Is;
    const int rb_r = fz_row_bytes<BITS>(K_r), rb_s = fz_row_bytes<BITS>(K_s);
    const int rbp_r = rb_r + FZ_PAD, rbp_s = rb_s + FZ_PAD;
    const FzGeom gr(a.stage_bytes, nblk, rbp_r);
    const FzGeom gs = with_shared ? FzGeom(a.stage_bytes, nblk, rbp_s) : gr;
    const int nb_r = (rows_r + gr.R - 1) / gr.R;
    const int nb_s = with_shared ? (rows_s + gs.R - 1) / gs.R : 0;
    const int n_routed = L.n * nb_r;
    const long long N = (long long)n_routed + nb_s;
    const int i0 = (int)(N * b / G), i1 = (int)(N * (b + 1) / G), cnt = i1 - i0;
    if (cnt <= 0) return;
    const WeightSet &wr = GATEUP ? a.gu : a.dn;
    const WeightSet &wsh = GATEUP ? a.sgu : a.sdn;
    const unsigned all = (1u << T) - 1u;

    struct Item {
        int d, o0, n, R, rb, rbp, K, out_rows, e;
        unsigned mask;
        const WeightSet *ws;
    };
    auto item = [&](int i) {
        Item it;
        const bool routed = i < n_routed;
        it.d = routed ? i / nb_r : L.n;
        const int blk = routed ? i - it.d * nb_r : i - n_routed;
        it.R = routed ? gr.R : gs.R;
        it.rb = routed ? rb_r : rb_s, it.rbp = routed ? rbp_r : rbp_s;
        it.K = routed ? K_r : K_s, it.out_rows = routed ? rows_r : rows_s;
        it.e = routed ? L.dexp[it.d] : 0, it.mask = routed ? L.dmask[it.d] : all;
        it.ws = routed ? &wr : &wsh;
        it.o0 = blk * it.R;
        it.n = min(it.R, it.out_rows - it.o0);
        return it;
    };
    auto slot = [&](int d, int t) {
        return d < L.n ? L.base + t * k + L.rank[d][t] : T * k + t;
    };
    // warp 0: one bulk copy per weight row of item i
    auto issue = [&](int i) {
        const int q = qi++, s = q % a.ns;
        if (q >= a.ns && !sm100::mbar_wait(&S.empty[s], ((q / a.ns) + 1) & 1, 0, FZ_WAIT) &&
            lane == 0)
            fz_timeout(a);
        const Item it = item(i);
        unsigned char *st = smem + a.off_ring + s * a.stage_bytes;
        if (lane == 0) sm100::mbar_arrive_expect_tx(&S.full[s], (uint32_t)(nblk * it.n * it.rb));
        __syncwarp();
        const uint8_t *wb =
            BITS == 32 ? reinterpret_cast<const uint8_t *>(it.ws->w32) : it.ws->q;
        for (int c = lane; c < nblk * it.n; c += 32) {
            const int bk = c / it.n, r = c - bk * it.n;
            const size_t srow = (size_t)it.e * it.ws->rows + (bk ? it.out_rows : 0) + it.o0 + r;
            sm100::bulk_load(st + (bk * it.R + r) * it.rbp, wb + srow * it.rb, it.rb, &S.full[s]);
        }
    };

    const int last_task = item(i1 - 1).d;
    int win0 = 0, win1 = -1;  // tasks whose h rows are staged (down)
    if (warp == 0)
        for (int p = 0; p < a.ns - 1 && p < cnt; p++) issue(i0 + p);
    for (int j = 0; j < cnt; j++) {
        const Item it = item(i0 + j);
        if (!GATEUP && it.d >= win1) {
            // stage the h rows of the next window of tasks (every worker
            // is past the previous window's items)
            wsync();
            win0 = it.d;
            win1 = min(it.d + a.hwin, last_task + 1);
            if (tid == 0) {
                fence_proxy_async();
                uint32_t bytes = 0;
                for (int d = win0; d < win1; d++) {
                    const int K = d < L.n ? K_r : K_s;
                    const unsigned m = d < L.n ? L.dmask[d] : all;
                    bytes += (uint32_t)__popc(m) * kpad_for(K, V) * 4;
                }
                sm100::mbar_arrive_expect_tx(&S.hbar, bytes);
                for (int d = win0; d < win1; d++) {
                    const int K = d < L.n ? K_r : K_s;
                    const unsigned m = d < L.n ? L.dmask[d] : all;
                    for (int t = 0; t < T; t++)
                        if ((m >> t) & 1u)
                            sm100::bulk_load(
                                smem + a.off_hs + ((d - win0) * T + t) * a.hsstride * 4,
                                a.hbuf + (size_t)slot(d, t) * a.hrow, kpad_for(K, V) * 4, &S.hbar);
                }
            }
            if (!sm100::mbar_wait(&S.hbar, hph & 1, 0, FZ_WAIT) && lane == 0) fz_timeout(a);
            hph++;
        }
        if (warp == 0 && j + a.ns - 1 < cnt) issue(i0 + j + a.ns - 1);
        const int q = qc++, s = q % a.ns;
        if (!sm100::mbar_wait(&S.full[s], (q / a.ns) & 1, 0, FZ_WAIT) && lane == 0) fz_timeout(a);
        const unsigned char *st = smem + a.off_ring + s * a.stage_bytes;
        const float *xs = reinterpret_cast<const float *>(smem + a.off_xs);
        for (int o = warp; o < it.n; o += FZ_WORKERS) {
            if constexpr (GATEUP) {
                const uint8_t *const rows[2] = {st + o * it.rbp, st + (it.R + o) * it.rbp};
                float acc[2][MT];
                fz_dot<BITS, 2, MT>(rows, it.K / V, xs, a.xstride, it.mask, lane, acc);
                if (lane == 0) {
                    const int orow = it.o0 + o;
                    const int pos = stage_pos<V>(orow / V, orow % V);
#pragma unroll
                    for (int t = 0; t < MT; t++)
                        if ((it.mask >> t) & 1u)
                            reinterpret_cast<float *>(a.hbuf + (size_t)slot(it.d, t) * a.hrow)[pos] =
                                __fmul_rn(silu_ref(acc[0][t]), acc[1][t]);
                }
            } else {
                const uint8_t *const rows[1] = {st + o * it.rbp};
                float acc[1][MT];
                fz_dot<BITS, 1, MT>(rows, it.K / V,
                                    reinterpret_cast<const float *>(smem + a.off_hs) +
                                        (it.d - win0) * T * a.hsstride,
                                    a.hsstride, it.mask, lane, acc);
                if (lane == 0)
#pragma unroll
                    for (int t = 0; t < MT; t++)
                        if ((it.mask >> t) & 1u)
                            a.dbuf[(size_t)slot(it.d, t) * a.H + it.o0 + o] = acc[0][t];
            }
        }
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&S.empty[s]);
    }
}

// Warp 0: the experts whose bit is set in tok[0..E), in index order, into L.
__device__ void fz_compact(const unsigned *tok, int E, FzList &L, int base) {
    const int lane = threadIdx.x & 31;
    int n = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const unsigned m = e < E ? tok[e] : 0u;
        const unsigned bal = __ballot_sync(FULL, m != 0u);
        if (m) {
            const int idx = n + __popc(bal & ((1u << lane) - 1u));
            L.dexp[idx] = e;
            L.dmask[idx] = m;
        }
        n += __popc(bal);
    }
    if (lane == 0) {
        L.n = n;
        L.base = base;
    }
}

// Approximate top-k of token t (warp): larger logit first, then the lower
// index; experts whose logits are NaN are never chosen (-1).  A candidate
// set only has to be close -- the exact routing computes what it missed --
// so each logit becomes one 32-bit key, its order-preserving bits with the
// low byte replaced by 255 - expert (E <= 256), and each rank is one
// warp-wide max reduction; logits within 2^-15 of each other order by index.
template <int NJ>
__device__ void fz_topk(const DecodeArgs &a, int t, int lane, int *cand) {
    unsigned key[NJ];
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int e = lane + 32 * j;
        const float v = e < a.E ? __ldcg(a.approx + (size_t)t * a.Ep + e) : __int_as_float(0x7fffffff);
        const unsigned u = __float_as_uint(v);
        const unsigned mono = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        key[j] = (e < a.E && !isnan(v)) ? ((mono & ~0xFFu) | (unsigned)(255 - e)) : 0u;
    }
    for (int r = 0; r < a.k; r++) {
        unsigned best = 0u;
#pragma unroll
        for (int j = 0; j < NJ; j++) best = max(best, key[j]);
        best = __reduce_max_sync(FULL, best);
        const int bi = best ? 255 - (int)(best & 0xFFu) : -1;
        if (bi >= 0 && (bi & 31) == lane) {
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if (j == (bi >> 5)) key[j] = 0u;
        }
        if (lane == 0) cand[r] = bi;
    }
    __syncwarp();
}

__device__ float fz_route(const float *lrow, int E, int k, int mode, int lane, int *sel) {
    const int nj = (E + 31) / 32;
    if (nj <= 1) return route_token<1>(lrow, E, k, mode, lane, sel);
    if (nj <= 2) return route_token<2>(lrow, E, k, mode, lane, sel);
    if (nj <= 4) return route_token<4>(lrow, E, k, mode, lane, sel);
    return route_token<8>(lrow, E, k, mode, lane, sel);
}

// float4 m of token t's float32 row: staged (CUDA-core path) or plain.
template <int BITS>
__device__ __forceinline__ float4 x4(const float *xs, int xstride, int t, int m) {
    constexpr int V = Chunk<BITS>::V;
    const int kk = 4 * m;
    const int pos = BITS <= 8 ? kk : stage_pos<V>(kk / V, kk % V);
    return *reinterpret_cast<const float4 *>(xs + t * xstride + pos);
}

// The chain warp of CTA b: serial logits of router rows b + q * G (q < nr)
// for every token, then, once every chain of the batch is done, the exact
// routing of tokens t = b, b + n_chain, ...
template <int BITS>
__device__ void fz_chains(const DecodeArgs &a, FzShared &S, unsigned char *smem, int nr) {
    const int lane = threadIdx.x & 31, G = gridDim.x, b = blockIdx.x, T = a.T, H = a.H;
    const int n_chain = min(a.Ep, G);
    const bool act = lane < nr * T;
    const int q = act ? lane / T : 0, t = act ? lane % T : 0;
    const float4 *wp = reinterpret_cast<const float4 *>(smem + (size_t)q * (H + 4) * 4);
    const float *xs = reinterpret_cast<const float *>(smem + a.off_xs);
    if (!sm100::mbar_wait(&S.wbar, 0, 0, FZ_WAIT)) {
        if (lane == 0) fz_timeout(a);
        return;
    }
    // products of a block of FZ_B4 float4 first, the next block's loads
    // issued, then the block's dependent adds: the chain is the critical path
    float acc = 0.f;
    const int n4 = H / 4, nfull = n4 / FZ_B4;
    float4 ca[FZ_B4], cb[FZ_B4];
#pragma unroll
    for (int j = 0; j < FZ_B4; j++) ca[j] = x4<BITS>(xs, a.xstride, t, j), cb[j] = wp[j];
    for (int blk = 0; blk < nfull; blk++) {
        float p[4 * FZ_B4];
#pragma unroll
        for (int j = 0; j < FZ_B4; j++) {
            p[4 * j] = __fmul_rn(ca[j].x, cb[j].x);
            p[4 * j + 1] = __fmul_rn(ca[j].y, cb[j].y);
            p[4 * j + 2] = __fmul_rn(ca[j].z, cb[j].z);
            p[4 * j + 3] = __fmul_rn(ca[j].w, cb[j].w);
        }
        const int nxt = blk + 1 < nfull ? blk + 1 : blk;
#pragma unroll
        for (int j = 0; j < FZ_B4; j++)
            ca[j] = x4<BITS>(xs, a.xstride, t, nxt * FZ_B4 + j), cb[j] = wp[nxt * FZ_B4 + j];
#pragma unroll
        for (int j = 0; j < 4 * FZ_B4; j++) acc = __fadd_rn(acc, p[j]);
    }
    for (int m = nfull * FZ_B4; m < n4; m++) {
        const float4 xv = x4<BITS>(xs, a.xstride, t, m), wv = wp[m];
        acc = __fadd_rn(acc, __fmul_rn(xv.x, wv.x));
        acc = __fadd_rn(acc, __fmul_rn(xv.y, wv.y));
        acc = __fadd_rn(acc, __fmul_rn(xv.z, wv.z));
        acc = __fadd_rn(acc, __fmul_rn(xv.w, wv.w));
    }
    if (act) a.logits[(size_t)t * a.Ep + b + q * G] = acc;
    __syncwarp();
    // publish "this CTA's logits are written" under this launch's epoch
    // (base / G: unique per launch, larger than any earlier launch's)
    const unsigned long long want = S.base / G + 1;
    if (lane == 0) {
        __threadfence();
        st_rel(&a.flags[b], want);
    }
    __syncwarp();
    float *lrow = reinterpret_cast<float *>(smem + a.off_lrow);
    for (int tt = b; tt < T; tt += n_chain) {
        for (int i = lane; i < n_chain; i += 32) fz_wait_flag(a, &a.flags[i], want);
        __syncwarp();
        for (int e = lane; e < a.Ep; e += 32) lrow[e] = __ldcg(a.logits + (size_t)tt * a.Ep + e);
        __syncwarp();
        const float wr = fz_route(lrow, a.E, a.k, a.mode, lane, S.rsel);
        // where each (token, rank) pair's down row will be: the speculative
        // pair's if the expert was a candidate, else a row computed after
        // routing (this CTA's candidates equal every CTA's)
        if (lane == 0) {
            const long long t0 = clock64();
            while (!*reinterpret_cast<volatile int *>(&S.cand_ready)) {
                if (clock64() - t0 > FZ_WAIT) {
                    fz_timeout(a);
                    break;
                }
                __nanosleep(64);
            }
        }
        __syncwarp();
        bool missed = false;
        if (lane < a.k) {
            int e = S.rsel[lane];
            if (e < 0 || e >= a.E) {
                atomicOr(a.err, QG_FLAG_BAD_EXPERT);
                e = 0;  // keeps every index in range; the flag reports the fault
            }
            int c = -1;
            for (int i = 0; i < a.k; i++)
                if (reinterpret_cast<volatile int *>(S.cand[tt])[i] == e) c = i;
            missed = c < 0;
            a.route->sel[tt][lane] = e;
            a.route->w[tt][lane] = wr;
            a.route->slot[tt][lane] = missed ? T * a.k + T + tt * a.k + lane : tt * a.k + c;
            a.topk_idx[(size_t)tt * a.k + lane] = e;
            a.topk_w[(size_t)tt * a.k + lane] = wr;
        }
        const unsigned anymiss = __ballot_sync(FULL, missed);
        if (lane == 0) a.route->miss[tt] = anymiss != 0u;
        if (a.has_shared && lane == 0) {
            // sigmoid1 (model/tensors.go:97) of the shared-gate logit
            const float g = lrow[a.E];
            const float sg = __fdiv_rn(1.f, __fadd_rn(1.f, (float)exp(-(double)g)));
            a.route->sg[tt] = sg;
            a.shared_w[tt] = sg;
        }
        __syncwarp();
        if (lane == 0) {
            __threadfence();
            st_rel(&a.flags[G + tt], want);
        }
        __syncwarp();
    }
}

template <int BITS, int MT>
__global__ void __launch_bounds__(FZ_THREADS, 1) k_decode(const __grid_constant__ DecodeArgs a) {
    constexpr bool TC = BITS <= 8;
    constexpr int V = Chunk<BITS>::V;
    extern __shared__ __align__(16) unsigned char fz_smem[];
    __shared__ FzShared S;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, b = blockIdx.x, T = a.T, k = a.k, H = a.H;
    const int nr = b < a.Ep ? min(a.nrc, (a.Ep - b + G - 1) / G) : 0;
    unsigned *tok = reinterpret_cast<unsigned *>(fz_smem + a.off_tok);
    float *xs = reinterpret_cast<float *>(fz_smem + a.off_xs);
    if (tid == 0) {
        for (int i = 0; i < a.ns; i++) {
            sm100::mbar_init(&S.full[i], 1);
            sm100::mbar_init(&S.empty[i], TC ? FZ_MW : FZ_WORKERS);
        }
        sm100::mbar_init(&S.wbar, 1);
        sm100::mbar_init(&S.hbar, 1);
        sm100::mbar_init(&S.xbar, 1);
        sm100::fence_mbar_init();
        S.nbar = 0;
        S.cand_ready = 0;
    }
    __syncthreads();
    // router rows: static weights, fetched while the previous kernel ends
    if (tid == 0 && nr > 0) {
        sm100::mbar_arrive_expect_tx(&S.wbar, (uint32_t)(nr * H * 4));
        for (int q = 0; q < nr; q++) {
            const int r = b + q * G;
            sm100::bulk_load(fz_smem + (size_t)q * (H + 4) * 4,
                             r < a.E ? a.router + (size_t)r * H : a.shared_gate, H * 4, &S.wbar);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    if (tid == 0) {
        // earlier launches are complete, and this launch's first barrier
        // cannot complete before this CTA arrives: the count lies in
        // [base, base + G)
        const unsigned long long v = ld_acq(a.bar);
        S.base = v - v % (unsigned long long)G;
    }
    bool range = false;
    if (TC && !(reinterpret_cast<uintptr_t>(a.x) & 15)) {
        // token rows by bulk copies (one memory round trip), then fp16 rows
        // converted from shared memory
        if (tid == 0) {
            sm100::mbar_arrive_expect_tx(&S.xbar, (uint32_t)(T * H * 4));
            for (int t = 0; t < T; t++)
                sm100::bulk_load(xs + t * a.xstride, a.x + (size_t)t * H, H * 4, &S.xbar);
        }
        if (!sm100::mbar_wait(&S.xbar, 0, 0, FZ_WAIT) && lane == 0) fz_timeout(a);
        const int h4 = H / 4;
        for (int i = tid; i < T * h4; i += FZ_THREADS) {
            const int t = i / h4, k4 = i - t * h4;
            const float4 v = *reinterpret_cast<const float4 *>(xs + t * a.xstride + 4 * k4);
            const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
            const float2 lf = __half22float2(lo), hf = __half22float2(hi);
            range |= (isinf(lf.x) && isfinite(v.x)) || (isinf(lf.y) && isfinite(v.y)) ||
                     (isinf(hf.x) && isfinite(v.z)) || (isinf(hf.y) && isfinite(v.w));
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t *>(&lo);
            u.y = *reinterpret_cast<const uint32_t *>(&hi);
            *reinterpret_cast<uint2 *>(fz_smem + a.off_x16 + t * a.x16tok + 8 * k4) = u;
        }
    } else {
        for (int i = tid; i < T * H; i += FZ_THREADS) {
            const int t = i / H, kk = i - t * H;
            const float v = a.x[i];
            xs[t * a.xstride + (TC ? kk : stage_pos<V>(kk / V, kk % V))] = v;
            if constexpr (TC) {  // fp16 B rows; absent tokens' columns are never read back
                const __half hv = __float2half_rn(v);
                range |= isinf(__half2float(hv)) && isfinite(v);
                reinterpret_cast<__half *>(fz_smem + a.off_x16 + t * a.x16tok)[kk] = hv;
            }
        }
    }
    if (range) atomicOr(a.err, QG_FLAG_RANGE);
    for (int e = tid; e < a.E; e += FZ_THREADS) tok[e] = 0u;
    // this launch's task counters start at zero; the first grid barrier
    // orders the clearing before any tile is counted
    if (b == 0)
        for (int i = tid; i < 2 * (FZ_MAXD + 1); i += FZ_THREADS) a.tdone[i] = 0u;
    __syncthreads();
    if (warp == FZ_WORKERS) {
        if (nr > 0) fz_chains<BITS>(a, S, fz_smem, nr);
        return;
    }

    // ---- 1. approximate logits of this CTA's router rows ----
    const bool spec_topk = a.speculate && a.mode == QGMOE_ROUTER_TOPK;
    if (spec_topk && nr > 0) {
        if (!sm100::mbar_wait(&S.wbar, 0, 0, FZ_WAIT) && lane == 0) fz_timeout(a);
        const int nl = nr * T;  // (row, token) pairs, pair q T + t
        float acc[2][FD_MAX_T];
#pragma unroll
        for (int q = 0; q < 2; q++)
#pragma unroll
            for (int t = 0; t < FD_MAX_T; t++) acc[q][t] = 0.f;
        for (int p = tid; p < H / 4; p += FZ_WT) {
#pragma unroll
            for (int q = 0; q < 2; q++) {
                if (q >= nr) break;
                const float4 wv =
                    *reinterpret_cast<const float4 *>(fz_smem + ((size_t)q * (H + 4) + 4 * p) * 4);
#pragma unroll
                for (int t = 0; t < FD_MAX_T; t++) {
                    if (t >= T) break;
                    const float4 xv = x4<BITS>(xs, a.xstride, t, p);
                    acc[q][t] = fmaf(wv.x, xv.x,
                                     fmaf(wv.y, xv.y, fmaf(wv.z, xv.z, fmaf(wv.w, xv.w, acc[q][t]))));
                }
            }
        }
#pragma unroll
        for (int q = 0; q < 2; q++) {
            if (q >= nr) break;
#pragma unroll
            for (int t = 0; t < FD_MAX_T; t++) {
                if (t >= T) break;
                float v = acc[q][t];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
                if (lane == 0) S.part[warp][q * T + t] = v;
            }
        }
        wsync();
        if (tid < nl) {
            const int q = tid / T, t = tid - q * T;
            float v = 0.f;
            for (int w = 0; w < FZ_WORKERS; w++) v += S.part[w][tid];
            a.approx[(size_t)t * a.Ep + b + q * G] = v;
        }
    }
    fz_grid_sync(a, S);
    const unsigned long long epoch = S.base / G;

    // ---- 2. candidates: approximate top-k per token, distinct experts ----
    if (warp < T) {
        int *cand = S.cand[warp];
        if (spec_topk) {
            const int nj = (a.E + 31) / 32;
            if (nj <= 1) fz_topk<1>(a, warp, lane, cand);
            else if (nj <= 2) fz_topk<2>(a, warp, lane, cand);
            else if (nj <= 4) fz_topk<4>(a, warp, lane, cand);
            else fz_topk<8>(a, warp, lane, cand);
        } else if (lane < k) {
            // PREFIX (model/moe.go:49) only ever selects experts 0..k-1
            cand[lane] = a.speculate && lane < a.E ? lane : -1;
        }
        __syncwarp();
        if (lane < k && cand[lane] >= 0) atomicOr(&tok[cand[lane]], 1u << warp);
    }
    wsync();
    if (tid == 0) {
        __threadfence_block();
        *reinterpret_cast<volatile int *>(&S.cand_ready) = 1;
    }
    if (warp == 0) fz_compact(tok, a.E, S.A, 0);
    wsync();
    for (int i = tid; i < S.A.n * T; i += FZ_WT) {
        const int d = i / T, t = i - d * T;
        if ((S.A.dmask[d] >> t) & 1u)
            for (int r = 0; r < k; r++)
                if (S.cand[t][r] == S.A.dexp[d]) {
                    S.A.rank[d][t] = (signed char)r;
                    break;
                }
    }
    wsync();

    // ---- 3, 4. gate_up and down of the candidates and the shared expert ----
    int qi = 0, qc = 0, hph = 0, nx = 0;
    // Tensor cores: no grid barrier between gate_up and down -- a down task
    // waits only for its own gate_up tiles (counted in a.tdone, one counter
    // set per list), so CTAs done with gate_up early start their down work.
    auto phases = [&](const FzList &L, bool with_shared, unsigned *tdone) {
        if constexpr (TC) {
            fz_phase_tc<BITS, true>(a, S, L, with_shared, fz_smem, qi, qc, hph, nx, tdone);
            fz_phase_tc<BITS, false>(a, S, L, with_shared, fz_smem, qi, qc, hph, nx, tdone);
        } else {
            fz_phase<BITS, MT, true>(a, S, L, with_shared, fz_smem, qi, qc, hph);
            fz_grid_sync(a, S);
            fz_phase<BITS, MT, false>(a, S, L, with_shared, fz_smem, qi, qc, hph);
        }
        fz_grid_sync(a, S);
    };
    phases(S.A, a.has_shared, a.tdone);

    // ---- 5. exact routing; pairs the candidates missed ----
    if (warp == 0) {
        if (lane < T) fz_wait_flag(a, &a.flags[G + lane], epoch + 1);
        __syncwarp();
    }
    wsync();
    // (values of a wait that ran out may be stale: indices stay in range)
    for (int i = tid; i < T * k; i += FZ_WT) {
        const int t = i / k, r = i - t * k;
        const int e = __ldcg(&a.route->sel[t][r]), sl = __ldcg(&a.route->slot[t][r]);
        S.sel[t][r] = e >= 0 && e < a.E ? e : 0;
        S.w[t][r] = __ldcg(&a.route->w[t][r]);
        S.slot[t][r] = sl >= 0 && sl < dec_slots(k) ? sl : 0;
    }
    if (a.has_shared && tid < T) S.sg[tid] = __ldcg(&a.route->sg[tid]);
    // S.sel / S.w / S.slot / S.sg are read by other threads below (the
    // missed pairs' list, the combine): every write lands first
    wsync();
    bool anymiss = false;  // the T loads in flight together
#pragma unroll
    for (int t = 0; t < FD_MAX_T; t++)
        if (t < T) anymiss |= __ldcg(&a.route->miss[t]) != 0;
    const int base_b = T * k + T;
    if (anymiss) {
        // rare: experts the approximate top-k missed, by expert
        for (int e = tid; e < a.E; e += FZ_WT) tok[e] = 0u;
        wsync();
        for (int i = tid; i < T * k; i += FZ_WT) {
            const int t = i / k, r = i - t * k;
            if (S.slot[t][r] >= base_b) atomicOr(&tok[S.sel[t][r]], 1u << t);
        }
        wsync();
        if (warp == 0) fz_compact(tok, a.E, S.B, base_b);
        wsync();
        for (int i = tid; i < S.B.n * T; i += FZ_WT) {
            const int d = i / T, t = i - d * T;
            if ((S.B.dmask[d] >> t) & 1u)
                for (int r = 0; r < k; r++)
                    if (S.sel[t][r] == S.B.dexp[d]) {
                        S.B.rank[d][t] = (signed char)r;
                        break;
                    }
        }
        wsync();
        phases(S.B, false, a.tdone + FZ_MAXD + 1);
    }

    // ---- 6. combine, output columns split over the CTAs ----
    const int j0 = (int)((long long)H * b / G), j1 = (int)((long long)H * (b + 1) / G);
    const int ncol = j1 - j0;
    for (int i = tid; i < T * ncol; i += FZ_WT) {
        const int t = i / ncol, j = j0 + (i - t * ncol);
        float o = 0.f;
        for (int r = 0; r < k; r++)
            o = __fadd_rn(o, __fmul_rn(S.w[t][r], __ldcg(a.dbuf + (size_t)S.slot[t][r] * H + j)));
        if (a.has_shared)
            o = __fadd_rn(o, __fmul_rn(S.sg[t], __ldcg(a.dbuf + (size_t)(T * k + t) * H + j)));
        a.out[(size_t)t * H + j] = o;
    }
}

// ---- host side ------------------------------------------------------------------
static int chunk_elems(int bits) { return bits == 32 ? 4 : bits == 16 ? 8 : bits == 8 ? 16 : 32; }
static int row_bytes_host(int bits, int K) {
    return bits == 32 ? K * 4 : bits == 16 ? K * 2 : bits == 8 ? K : K / 2;
}
static int up16(int v) { return (v + 15) & ~15; }

int decode_hrow_bytes(int bits, int I, int Is) {
    const int kmax = std::max(I, Is);
    return bits <= 8 ? up16(kmax * 2) : (kpad_for(kmax, chunk_elems(bits)) + 4) * 4;
}

// k blocks per streamed item: the largest divisor of KB whose tiles fit a stage
static int kbi_for(int KB, int tile, int stage) {
    int best = 0;
    for (int d = 1; d <= KB; d++)
        if (KB % d == 0 && d * tile <= stage) best = d;
    return best;
}

bool decode_plan(DecodeArgs &a, int bits, int sms) {
    if (a.T < 1 || a.T > FD_MAX_T || a.E > FD_MAX_E || a.k < 1 || a.k > QG_MAX_TOPK || a.k > a.E)
        return false;
    const bool tc = bits <= 8;
    // tensor cores: the packed tiles (128 rows x 64 codes); CUDA cores: bulk
    // copies of whole rows, multiples of 16 bytes
    const int kq = tc ? 128 : 32;
    if (a.H % kq || a.I % kq || (a.has_shared && a.Is % kq)) return false;
    if (tc && !(a.gu_pq && a.dn_pq && (!a.has_shared || (a.sgu_pq && a.sdn_pq)))) return false;
    a.nrc = (a.Ep + sms - 1) / sms;
    if (a.nrc > 2 || a.nrc * a.T > 32) return false;
    const int V = chunk_elems(bits);
    const int kmax = std::max(a.I, a.has_shared ? a.Is : 0);
    a.hrow = decode_hrow_bytes(bits, a.I, a.has_shared ? a.Is : 0);
    a.xstride = tc ? a.H + 4 : kpad_for(a.H, V) + 4;
    a.x16tok = tc ? a.H * 2 + 32 : 0;
    a.h16tok = tc ? kmax * 2 + 32 : 0;
    a.hsstride = tc ? 0 : kpad_for(kmax, V) + 4;
    const int wrows = a.nrc * (a.H + 4) * 4;
    const int xs = a.T * a.xstride * 4;
    const int x16 = FD_MAX_T * a.x16tok;
    const int xch = tc ? 2 * 4 * 32 * 16 : 0;
    const int lrow = up16(a.Ep * 4), tok = up16(a.E * 4);
    const int hs_one = tc ? FD_MAX_T * a.h16tok : a.T * a.hsstride * 4;
    const int fixed = wrows + xs + x16 + xch + lrow + tok;
    const int avail = FZ_SMEM_MAX - fixed - hs_one;
    if (tc) {
        const int tile = bits == 8 ? 128 * 64 + 512 : 128 * 32 + 512;
        int stage = std::min(FZ_STAGE_MAX, avail / 3);
        a.kbi_gu = kbi_for(a.H / 64, tile, stage);
        a.kbi_dn = kbi_for(a.I / 64, tile, stage);
        a.kbi_sdn = a.has_shared ? kbi_for(a.Is / 64, tile, stage) : 1;
        if (!a.kbi_gu || !a.kbi_dn || !a.kbi_sdn) return false;
        stage = tile * std::max(a.kbi_gu, std::max(a.kbi_dn, a.kbi_sdn));
        a.stage_bytes = stage;
        a.ns = std::min(FZ_NSMAX, avail / stage);
        a.hwin = 1;
    } else {
        auto rowp = [&](int K) { return row_bytes_host(bits, K) + FZ_PAD; };
        const int need = std::max(2 * rowp(a.H), std::max(rowp(a.I), a.has_shared ? rowp(a.Is) : 0));
        if (avail < 2 * up16(need)) return false;
        a.stage_bytes = std::max(std::min(FZ_STAGE_MAX, avail / 3) & ~15, up16(need));
        a.ns = std::min(FZ_NSMAX, avail / a.stage_bytes);
        a.hwin = std::max(1, std::min(4, (avail + hs_one - a.ns * a.stage_bytes) / hs_one));
    }
    if (a.ns < 2) return false;
    a.off_xs = wrows;
    a.off_x16 = a.off_xs + xs;
    a.off_xch = a.off_x16 + x16;
    a.off_lrow = a.off_xch + xch;
    a.off_tok = a.off_lrow + lrow;
    a.off_ring = a.off_tok + tok;
    a.off_hs = a.off_ring + a.ns * a.stage_bytes;
    a.smem = a.off_hs + a.hwin * hs_one;
    return a.smem <= FZ_SMEM_MAX;
}

template <int BITS, int MT>
static int launch_decode_t(const DecodeArgs &a, cudaStream_t s) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr[dev]) {
        QG_CUDA(cudaFuncSetAttribute(k_decode<BITS, MT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, FZ_SMEM_MAX));
        int per_sm = 0;
        QG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode<BITS, MT>,
                                                              FZ_THREADS, FZ_SMEM_MAX));
        if (per_sm < 1) return set_error(QGMOE_ERR_CUDA, "decode kernel does not fit one SM");
        if (dev < 64) attr[dev] = true;
    }
    QG_CUDA(launch_pdl(k_decode<BITS, MT>, dim3(num_sms(dev)), dim3(FZ_THREADS), a.smem, s, 1, a));
    return QGMOE_OK;
}

// The tensor-core path serves every batch size with one kernel (the tokens
// are the MMA's 8 columns); the CUDA-core path is instantiated per token count.
template <int BITS>
static int launch_decode_b(const DecodeArgs &a, cudaStream_t s) {
    if constexpr (BITS <= 8) {
        return launch_decode_t<BITS, 1>(a, s);
    } else {
        if (a.T <= 1) return launch_decode_t<BITS, 1>(a, s);
        if (a.T <= 2) return launch_decode_t<BITS, 2>(a, s);
        if (a.T <= 4) return launch_decode_t<BITS, 4>(a, s);
        return launch_decode_t<BITS, 8>(a, s);
    }
}

int launch_decode(int bits, const DecodeArgs &a, cudaStream_t s) {
    if (a.T < 1 || a.T > FD_MAX_T)
        return set_error(QGMOE_ERR_INVALID_ARG, "decode path: T=%d outside 1..%d", a.T, FD_MAX_T);
    switch (bits) {
        case 32: return launch_decode_b<32>(a, s);
        case 16: return launch_decode_b<16>(a, s);
        case 8: return launch_decode_b<8>(a, s);
        case 4: return launch_decode_b<4>(a, s);
    }
    return set_error(QGMOE_ERR_INVALID_ARG, "decode path: bits %d", bits);
}

}  // namespace qg
