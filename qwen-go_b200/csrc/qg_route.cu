// Router + dispatch (kernels K1 and K2).
//
// Launches: k_logits, k_topk, k_scatter (fused into k_topk for <= 32 tokens)
// (+ k_gather_h16 for the tensor path).
// 1. k_logits: logits = x . router^T (proj(x,1,&m.gate,...),
//    model/moe.go:42) in the reference's own order: each logit is a serial
//    float32 sum in index order of separately rounded products (matmulVec,
//    model/tensors.go:77-89; Go on amd64 does not contract a*b+c into FMA),
//    so every logit equals the reference's bit for bit.  A serial sum cannot
//    be split along K, so the parallelism is over (token, row) pairs: each
//    thread carries TPT x RPT independent chains (register tiling, the
//    chains hide the add latency), token and router tiles are staged in
//    shared memory K-major, and __fmul_rn / __fadd_rn keep the compiler from
//    fusing.  The shared-expert gate vector rides along as router row E
//    (model/moe.go:87-93).  For the tensor path the CTAs of the first row
//    tile also write fp16(x) (a finite value beyond fp16 range raises
//    QG_FLAG_RANGE).
// 2. k_topk: one warp per token: softmax exactly as model/tensors.go:106-121
//    (max by `x > mx`, exp in float64 rounded to float32, float32 sum in
//    index order, divide), so the probabilities are the reference's bit for
//    bit; then top-k (model/moe.go:44-52: TOPK = the insertion sort over all
//    experts, i.e. probability descending with ties to the lower index;
//    PREFIX = its literal bound over experts 0..k-1), w = p / (wSum + 1e-9)
//    (model/moe.go:53-63) and the sigmoid of the shared gate.  NaN behaves
//    as in the reference: `x > mx` and `p[j] > p[j-1]` are false on NaN, so
//    a NaN or infinite activation makes every probability of its token NaN
//    and its selection experts 0..k-1.  Each CTA writes its expert
//    histogram; the last CTA (atomic ticket) scans the totals into expert
//    offsets, the list of active experts and the tensor-core tile prefix,
//    and re-zeroes the counters and the ticket so the next call (or a graph
//    replay) starts clean.
// 3. k_scatter: each CTA ranks its own (token, rank) pairs per expert in pair
//    order (warp match + per-warp counts) and adds the histograms of the CTAs
//    before it, so slots are expert-sorted and deterministic without a serial
//    pass.  With one token chunk (<= 32 tokens) the single top-k CTA does this
//    itself once the offsets are known, one launch fewer.  For the tensor-core
//    path k_gather_h16 then copies each slot's fp16 activation row.
#include "qg_common.cuh"
#include "qg_router.cuh"
#include "qg_sm100.cuh"

namespace qg {

constexpr int LG_KC = 32;                // K chunk staged in shared memory
constexpr int TK_TOK = QG_TOPK_TOK;      // tokens per top-k / scatter CTA
constexpr int RT_THREADS = 1024;         // top-k and scatter CTAs: one warp per token
constexpr int RT_WARPS = RT_THREADS / 32;

// ---- 1. logits ------------------------------------------------------------------
// CTA tile: TT = TPT*TTH tokens x RR = RPT*RTH router rows; thread (ty, tx)
// owns tokens ty*TPT.. and rows tx*RPT...  Per 32-wide K chunk the tiles are
// fetched into registers (the next chunk while the current one is consumed),
// then stored K-major into shared memory so that a thread reads its TPT
// activations and RPT router values of step kk with one vector load each.
// For every kk in order: chain(t, r) = fl(chain + fl(x[t][kk] * w[r][kk])).
template <int TPT, int RPT, int TTH, int RTH>
struct LgCfg {
    static constexpr int THREADS = TTH * RTH, TT = TPT * TTH, RR = RPT * RTH;
    static constexpr int XV = TT * LG_KC / 4, WV = RR * LG_KC / 4;  // float4 per chunk
    static constexpr int XPT = (XV + THREADS - 1) / THREADS, WPT = (WV + THREADS - 1) / THREADS;
};

// Two float32 additions per instruction (sm_100 packed f32x2), each rounded
// to nearest exactly as a scalar __fadd_rn.  The products stay scalar
// __fmul_rn: a packed multiply feeding a packed add is contracted into a
// packed FMA by the compiler even with explicit .rn (measured on B200: 3658
// of 4096 serial sums differed from separately rounded ones), while a
// scalar product feeding the packed add is not (0 of 4096).
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

template <int N>
__device__ __forceinline__ void lds_vec(const float *p, float (&v)[N]) {
    if constexpr (N == 4) {
        const float4 a = *reinterpret_cast<const float4 *>(p);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
    } else if constexpr (N == 2) {
        const float2 a = *reinterpret_cast<const float2 *>(p);
        v[0] = a.x, v[1] = a.y;
    } else {
#pragma unroll
        for (int i = 0; i < N; i++) v[i] = p[i];
    }
}

template <int TPT, int RPT, int TTH, int RTH>
__global__ void __launch_bounds__(TTH *RTH)
k_logits(const float *__restrict__ x, int T, int H, int E, int Ep,
         const float *__restrict__ router, const float *__restrict__ shared_gate,
         float *__restrict__ logits, __half *__restrict__ xh, int *err) {
    using C = LgCfg<TPT, RPT, TTH, RTH>;
    constexpr int TT = C::TT, RR = C::RR, NTH = C::THREADS;
    __shared__ __align__(16) float xs[LG_KC][TT + 4];
    __shared__ __align__(16) float ws[LG_KC][RR + 4];
    pdl_enter();
    const int tid = threadIdx.x, tx = tid % RTH, ty = tid / RTH;
    const int t0 = blockIdx.x * TT, r0 = blockIdx.y * RR;
    const bool write_h = xh && blockIdx.y == 0;
    // loaders: float4 i of a chunk covers item i % TT (token) or i % RR (row)
    // and columns 4 (i / TT) .. + 3, so a warp stores one K column of 32
    // consecutive tokens or rows: conflict-free transposed stores
    const float *xrow[C::XPT];
    const float *wrow[C::WPT];
    int xc[C::XPT], wc[C::WPT];
#pragma unroll
    for (int j = 0; j < C::XPT; j++) {
        const int i = tid + NTH * j, t = t0 + i % TT;
        xc[j] = (i / TT) * 4;
        xrow[j] = (i < C::XV && t < T) ? x + (size_t)t * H : nullptr;
    }
#pragma unroll
    for (int j = 0; j < C::WPT; j++) {
        const int i = tid + NTH * j, r = r0 + i % RR;
        wc[j] = (i / RR) * 4;
        wrow[j] = (i < C::WV && r < Ep) ? (r < E ? router + (size_t)r * H : shared_gate) : nullptr;
    }
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 xn[C::XPT], wn[C::WPT];
    auto fetch = [&](int kb) {
#pragma unroll
        for (int j = 0; j < C::XPT; j++)
            xn[j] = xrow[j] ? __ldg(reinterpret_cast<const float4 *>(xrow[j] + kb + xc[j])) : zero;
#pragma unroll
        for (int j = 0; j < C::WPT; j++)
            wn[j] = wrow[j] ? __ldg(reinterpret_cast<const float4 *>(wrow[j] + kb + wc[j])) : zero;
    };
    static_assert(RPT % 2 == 0, "rows per thread are paired for the packed adds");
    float2 acc[TPT][RPT / 2];
#pragma unroll
    for (int i = 0; i < TPT; i++)
#pragma unroll
        for (int j = 0; j < RPT / 2; j++) acc[i][j] = make_float2(0.f, 0.f);
    bool range = false;
    fetch(0);
    for (int kb = 0; kb < H; kb += LG_KC) {
#pragma unroll
        for (int j = 0; j < C::XPT; j++) {
            const int i = tid + NTH * j;
            if (i < C::XV) {
                const int t = i % TT, c4 = xc[j];
                xs[c4][t] = xn[j].x;
                xs[c4 + 1][t] = xn[j].y;
                xs[c4 + 2][t] = xn[j].z;
                xs[c4 + 3][t] = xn[j].w;
                if (write_h && xrow[j]) {
                    const __half2 a = __floats2half2_rn(xn[j].x, xn[j].y);
                    const __half2 b = __floats2half2_rn(xn[j].z, xn[j].w);
                    const float2 af = __half22float2(a), bf = __half22float2(b);
                    range |= (isfinite(xn[j].x) && isinf(af.x)) ||
                             (isfinite(xn[j].y) && isinf(af.y)) ||
                             (isfinite(xn[j].z) && isinf(bf.x)) ||
                             (isfinite(xn[j].w) && isinf(bf.y));
                    uint2 u;
                    u.x = *reinterpret_cast<const uint32_t *>(&a);
                    u.y = *reinterpret_cast<const uint32_t *>(&b);
                    *reinterpret_cast<uint2 *>(xh + (size_t)(t0 + t) * H + kb + c4) = u;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < C::WPT; j++) {
            const int i = tid + NTH * j;
            if (i < C::WV) {
                const int row = i % RR, c4 = wc[j];
                ws[c4][row] = wn[j].x;
                ws[c4 + 1][row] = wn[j].y;
                ws[c4 + 2][row] = wn[j].z;
                ws[c4 + 3][row] = wn[j].w;
            }
        }
        __syncthreads();
        if (kb + LG_KC < H) fetch(kb + LG_KC);
        // the operands of step kk + 2 are loaded while step kk's chains advance
        float a0[TPT], b0[RPT], a1[TPT], b1[RPT];
        lds_vec<TPT>(&xs[0][ty * TPT], a0);
        lds_vec<RPT>(&ws[0][tx * RPT], b0);
        lds_vec<TPT>(&xs[1][ty * TPT], a1);
        lds_vec<RPT>(&ws[1][tx * RPT], b1);
#pragma unroll
        for (int kk = 0; kk < LG_KC; kk++) {
            float a2[TPT], b2[RPT];
            if (kk + 2 < LG_KC) {
                lds_vec<TPT>(&xs[kk + 2][ty * TPT], a2);
                lds_vec<RPT>(&ws[kk + 2][tx * RPT], b2);
            }
#pragma unroll
            for (int i = 0; i < TPT; i++)
#pragma unroll
                for (int j = 0; j < RPT / 2; j++)
                    acc[i][j] = add2_rn(acc[i][j], make_float2(__fmul_rn(a0[i], b0[2 * j]),
                                                               __fmul_rn(a0[i], b0[2 * j + 1])));
#pragma unroll
            for (int i = 0; i < TPT; i++) a0[i] = a1[i], a1[i] = a2[i];
#pragma unroll
            for (int j = 0; j < RPT; j++) b0[j] = b1[j], b1[j] = b2[j];
        }
        __syncthreads();
    }
    if (range) atomicOr(err, QG_FLAG_RANGE);
#pragma unroll
    for (int i = 0; i < TPT; i++) {
        const int t = t0 + ty * TPT + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < RPT; j++) {
            const int r = r0 + tx * RPT + j;
            if (r < Ep) logits[(size_t)t * Ep + r] = (j & 1) ? acc[i][j / 2].y : acc[i][j / 2].x;
        }
    }
}

// ---- 1b. logits of decode-sized batches ----------------------------------------------
// A serial chain is H dependent adds long, so at a few tokens the tiled
// kernel above spends its time waiting for each 32-wide K chunk.  Here a CTA
// owns LR_RR router rows and TT tokens and holds their WHOLE rows in shared
// memory: one thread issues 1-D bulk copies of every row in LR_SEG K
// segments (one mbarrier each) -- the router rows before waiting for the
// previous kernel, since they do not depend on it -- and each thread runs one
// chain (row tid % LR_RR, token tid / LR_RR) segment by segment as the
// segments land.  Rows are padded by 4 floats so the 8 rows (and 4 tokens)
// a warp reads at one k fall in distinct banks.
constexpr int LR_RR = 8, LR_SEG = 4, LR_B4 = 8;
constexpr long long LR_WAIT_CYCLES = 2000000000LL;  // ~1 s: a lost copy cannot hang the GPU
constexpr size_t LR_SMEM_MAX = 220 * 1024;           // of the 227 KB a CTA may opt into

__host__ __device__ constexpr size_t lr_smem_bytes(int TT, int H) {
    return sizeof(float) * (size_t)(LR_RR + TT) * (H + 4) + sizeof(uint64_t) * 2 * LR_SEG;
}

template <int TT>
__global__ void __launch_bounds__(LR_RR *TT)
k_logits_rows(const float *__restrict__ x, int T, int H, int E, int Ep,
              const float *__restrict__ router, const float *__restrict__ shared_gate,
              float *__restrict__ logits, __half *__restrict__ xh, int *err) {
    extern __shared__ __align__(16) float lr_smem[];
    const int HP = H + 4, L = H / LR_SEG;
    float *ws = lr_smem;                                          // [LR_RR][HP]
    float *xs = ws + LR_RR * HP;                                  // [TT][HP]
    uint64_t *bar = reinterpret_cast<uint64_t *>(xs + TT * HP);   // w segments, x segments
    const int tid = threadIdx.x;
    const int r0 = blockIdx.x * LR_RR, t0 = blockIdx.y * TT;
    const int nr = min(LR_RR, Ep - r0), nt = min(TT, T - t0);
    if (tid == 0) {
        for (int i = 0; i < 2 * LR_SEG; i++) sm100::mbar_init(&bar[i], 1);
        sm100::fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)  // router rows (weights): before the wait for the previous kernel
        for (int s = 0; s < LR_SEG; s++) {
            sm100::mbar_arrive_expect_tx(&bar[s], (uint32_t)(nr * L * 4));
            for (int r = 0; r < nr; r++) {
                const float *src = (r0 + r < E ? router + (size_t)(r0 + r) * H : shared_gate);
                sm100::bulk_load(ws + r * HP + s * L, src + s * L, L * 4, &bar[s]);
            }
        }
    pdl_launch_dependents();
    pdl_wait();
    if (tid == 0)
        for (int s = 0; s < LR_SEG; s++) {
            sm100::mbar_arrive_expect_tx(&bar[LR_SEG + s], (uint32_t)(nt * L * 4));
            for (int t = 0; t < nt; t++)
                sm100::bulk_load(xs + t * HP + s * L, x + (size_t)(t0 + t) * H + s * L, L * 4,
                                 &bar[LR_SEG + s]);
        }
    const int r = tid % LR_RR, t = tid / LR_RR;
    float acc = 0.f;
    bool ok = true;
    for (int s = 0; s < LR_SEG && ok; s++) {
        ok = sm100::mbar_wait(&bar[s], 0, 0, LR_WAIT_CYCLES) &&
             sm100::mbar_wait(&bar[LR_SEG + s], 0, 0, LR_WAIT_CYCLES);
        if (!ok) break;
        const float4 *wp = reinterpret_cast<const float4 *>(ws + r * HP + s * L);
        const float4 *xp = reinterpret_cast<const float4 *>(xs + t * HP + s * L);
        // the add chain is the critical path (5 cycles per dependent add on
        // B200): operands come in register blocks of LR_B4 float4 each; a
        // block's products are formed first (independent of the chain), the
        // next block's shared-memory loads are issued, then the block's
        // dependent adds run from registers
        const int L4 = L / 4, nfull = L4 / LR_B4;  // float4 per segment, full blocks
        if (nfull > 0) {
            float4 ca[LR_B4], cb[LR_B4];
#pragma unroll
            for (int j = 0; j < LR_B4; j++) ca[j] = xp[j], cb[j] = wp[j];
            for (int blk = 0; blk < nfull; blk++) {
                float p[4 * LR_B4];
#pragma unroll
                for (int j = 0; j < LR_B4; j++) {
                    p[4 * j] = __fmul_rn(ca[j].x, cb[j].x);
                    p[4 * j + 1] = __fmul_rn(ca[j].y, cb[j].y);
                    p[4 * j + 2] = __fmul_rn(ca[j].z, cb[j].z);
                    p[4 * j + 3] = __fmul_rn(ca[j].w, cb[j].w);
                }
                const int nxt = blk + 1 < nfull ? blk + 1 : blk;
#pragma unroll
                for (int j = 0; j < LR_B4; j++)
                    ca[j] = xp[nxt * LR_B4 + j], cb[j] = wp[nxt * LR_B4 + j];
#pragma unroll
                for (int j = 0; j < 4 * LR_B4; j++) acc = __fadd_rn(acc, p[j]);
            }
        }
        for (int c = nfull * LR_B4; c < L4; c++) {  // the segment's remainder
            const float4 a = xp[c], b = wp[c];
            acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
            acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
            acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
            acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
        }
    }
    if (!ok) {
        atomicOr(err, QG_FLAG_TIMEOUT);
        // this CTA's copies must land before its shared memory goes away
        if (tid == 0)
            for (int i = 0; i < 2 * LR_SEG; i++) sm100::mbar_wait(&bar[i], 0, 0, LR_WAIT_CYCLES);
        return;
    }
    if (r < nr && t < nt) logits[(size_t)(t0 + t) * Ep + r0 + r] = acc;
    if (xh && blockIdx.x == 0) {  // fp16 rows of this token tile for the tensor path
        bool range = false;
        const int q4 = H / 4;
        for (int i = tid; i < nt * q4; i += LR_RR * TT) {
            const int tt = i / q4, c = i - tt * q4;
            const float4 v = *reinterpret_cast<const float4 *>(xs + tt * HP + 4 * c);
            const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
            const float2 af = __half22float2(a), bf = __half22float2(b);
            range |= (isfinite(v.x) && isinf(af.x)) || (isfinite(v.y) && isinf(af.y)) ||
                     (isfinite(v.z) && isinf(bf.x)) || (isfinite(v.w) && isinf(bf.y));
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t *>(&a);
            u.y = *reinterpret_cast<const uint32_t *>(&b);
            *reinterpret_cast<uint2 *>(xh + (size_t)(t0 + tt) * H + 4 * c) = u;
        }
        if (range) atomicOr(err, QG_FLAG_RANGE);
    }
}

// ---- 1c. logits of prefill batches: TMA-fed, about one CTA per SM ------------------
// The serial chains leave no K parallelism, so the limit is the FP32 pipe (a
// separately rounded product and sum per step, 2048 steps per chain at
// H = 2048) fed from shared memory.  k_logits runs 256 CTAs of 4 warps with a
// 4 x 4 register tile: 108 SMs get two CTAs and 40 get one.  Here a CTA owns
// TT = 4 TPT tokens x RR = 64 RPT router rows, and TPT is picked per batch so
// the grid is about one CTA per SM (4096 tokens x 128 rows: 147 CTAs of 28
// tokens).  Eight consumer warps, two per scheduler so one's dependent adds
// hide behind the other's: warp w takes tokens (w % 4) TPT .. + TPT - 1 (the
// same for all its lanes: broadcast loads) and lane l rows
// l + 32 (RPT (w / 4) + j), j < RPT.  Router rows and token rows arrive in
// 32-wide K chunks by TMA (128B swizzle) into an LT_S-stage ring that a
// producer warp keeps full.  Every product and sum is rounded separately in
// index order as in k_logits, so the logits are the reference's bit for bit.
// In row tile 0 a converter warp also writes the fp16 activation rows of the
// tensor path from the staged token chunks (kept off the consumer warps,
// whose pace sets the ring's).
constexpr int LT_G = 4;               // token groups per CTA
constexpr int LT_W = 2 * LT_G;        // consumer warps: token group x row half
constexpr int LT_S = 4;               // ring stages
constexpr int LT_THREADS = (LT_W + 2) * 32;  // + producer warp + converter warp

template <int TPT, int RPT>
struct LtCfg {
    static constexpr int TT = LT_G * TPT, RR = 64 * RPT;
    static constexpr int W_BYTES = RR * 128;                        // multiple of 1024
    static constexpr int X_BYTES = (TT * 128 + 1023) / 1024 * 1024;
    static constexpr int STAGE = W_BYTES + X_BYTES;
    static constexpr int TX = (RR + TT) * 128;                      // bytes per stage
    static constexpr int SMEM = LT_S * STAGE + 1024 + 2 * LT_S * 8;
};

// Shared address of line r of a 1024-byte aligned tile written by TMA with
// the 128B swizzle, pre-swizzled: 16-byte chunk c of the line is at
// lt_line(tile, r) ^ (c << 4).
__device__ __forceinline__ uint32_t lt_line(uint32_t tile, int r) {
    return tile + r * 128 + ((r & 7) << 4);
}

__device__ __forceinline__ float lt_el(const float4 &v, int e) {
    return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
}

template <int TPT, int RPT>
__global__ void __launch_bounds__(LT_THREADS, 1)
k_logits_tma(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
             int T, int H, int Ep, float *__restrict__ logits, __half *__restrict__ xh,
             int *err) {
    using C = LtCfg<TPT, RPT>;
    extern __shared__ __align__(1024) uint8_t lt_raw[];
    // offset, not integer casts, so the compiler keeps shared-memory accesses
    uint8_t *base = lt_raw + ((1024u - (sm100::smem_u32(lt_raw) & 1023u)) & 1023u);
    const uint32_t sbase = sm100::smem_u32(base);
    uint64_t *full = reinterpret_cast<uint64_t *>(base + LT_S * C::STAGE);
    uint64_t *empty = full + LT_S;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * C::TT, r0 = blockIdx.y * C::RR, nk = H / 32;
    const bool do_h = xh && blockIdx.y == 0;
    if (tid == 0) {
        for (int s = 0; s < LT_S; s++) {
            sm100::mbar_init(&full[s], 1);
            sm100::mbar_init(&empty[s], LT_W + (do_h ? 1 : 0));
        }
        sm100::fence_mbar_init();
    }
    __syncthreads();
    pdl_enter();
    if (warp == LT_W + 1) {
        // converter: lane = (token of a group of 4, 16-byte chunk); fp16 rows
        // out as 8-byte stores
        if (!do_h) return;
        bool range = false;
        const int sub = lane >> 3, q = lane & 7;
        for (int c = 0; c < nk; c++) {
            const int s = c % LT_S;
            if (!sm100::mbar_wait(&full[s], (c / LT_S) & 1, 0, LR_WAIT_CYCLES)) {
                atomicOr(err, QG_FLAG_TIMEOUT);
                break;
            }
            const uint32_t X = sbase + s * C::STAGE + C::W_BYTES;
#pragma unroll
            for (int i = 0; i < TPT; i++) {
                const int ti = 4 * i + sub, t = t0 + ti;
                const float4 v = sm100::ld_shared_f4(lt_line(X, ti) ^ (q << 4));
                const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
                const float2 af = __half22float2(a), bf = __half22float2(b);
                range |= (isfinite(v.x) && isinf(af.x)) || (isfinite(v.y) && isinf(af.y)) ||
                         (isfinite(v.z) && isinf(bf.x)) || (isfinite(v.w) && isinf(bf.y));
                if (t < T) {
                    uint2 u;
                    u.x = *reinterpret_cast<const uint32_t *>(&a);
                    u.y = *reinterpret_cast<const uint32_t *>(&b);
                    *reinterpret_cast<uint2 *>(xh + (size_t)t * H + c * 32 + q * 4) = u;
                }
            }
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&empty[s]);
        }
        if (range) atomicOr(err, QG_FLAG_RANGE);
        return;
    }
    if (warp == LT_W) {
        // producer: chunk c into stage c % LT_S once the consumers freed it
        if (lane == 0) {
            sm100::prefetch_tmap(&tm_x);
            sm100::prefetch_tmap(&tm_w);
            int last = -1;
            for (int c = 0; c < nk; c++) {
                const int s = c % LT_S;
                if (c >= LT_S &&
                    !sm100::mbar_wait(&empty[s], ((c / LT_S) + 1) & 1, 0, LR_WAIT_CYCLES)) {
                    atomicOr(err, QG_FLAG_TIMEOUT);
                    break;
                }
                uint8_t *st = base + s * C::STAGE;
                sm100::mbar_arrive_expect_tx(&full[s], C::TX);
                sm100::tma_load_2d(st, &tm_w, c * 32, r0, &full[s]);
                sm100::tma_load_2d(st + C::W_BYTES, &tm_x, c * 32, t0, &full[s]);
                last = c;
            }
            // the CTA's shared memory must outlive every copy issued into it
            if (last >= 0)
                sm100::mbar_wait(&full[last % LT_S], (last / LT_S) & 1, 0, LR_WAIT_CYCLES);
        }
        return;
    }
    const int g = warp % LT_G, half = warp / LT_G;
    const int tq = g * TPT;                // first token of this warp in the tile
    const int rq = 32 * RPT * half;        // first row block of this warp
    constexpr int NP = RPT / 2;  // row pairs (packed adds), plus one single row if RPT is odd
    float2 acc[TPT][NP > 0 ? NP : 1];
    float acc1[TPT];
#pragma unroll
    for (int i = 0; i < TPT; i++) {
#pragma unroll
        for (int j = 0; j < NP; j++) acc[i][j] = make_float2(0.f, 0.f);
        acc1[i] = 0.f;
    }
    for (int c = 0; c < nk; c++) {
        const int s = c % LT_S;
        if (!sm100::mbar_wait(&full[s], (c / LT_S) & 1, 0, LR_WAIT_CYCLES)) {
            atomicOr(err, QG_FLAG_TIMEOUT);
            break;
        }
        const uint32_t W = sbase + s * C::STAGE, X = W + C::W_BYTES;
        // rows rq + lane + 32 j share the swizzle phase lane & 7
        const uint32_t wl = lt_line(W, rq + lane);
        // operands of 4 K steps; the next group's loads are issued before
        // the current group's products
        float4 xa[2][TPT], wa[2][RPT];
        auto load = [&](int q4, float4 (&xd)[TPT], float4 (&wd)[RPT]) {
#pragma unroll
            for (int i = 0; i < TPT; i++) xd[i] = sm100::ld_shared_f4(lt_line(X, tq + i) ^ (q4 << 4));
#pragma unroll
            for (int j = 0; j < RPT; j++) wd[j] = sm100::ld_shared_f4((wl + j * 4096) ^ (q4 << 4));
        };
        load(0, xa[0], wa[0]);
#pragma unroll
        for (int q4 = 0; q4 < 8; q4++) {
            if (q4 < 7) load(q4 + 1, xa[(q4 + 1) & 1], wa[(q4 + 1) & 1]);
            const float4 (&xc)[TPT] = xa[q4 & 1];
            const float4 (&wc)[RPT] = wa[q4 & 1];
#pragma unroll
            for (int e = 0; e < 4; e++) {
#pragma unroll
                for (int i = 0; i < TPT; i++) {
                    const float xv = lt_el(xc[i], e);
#pragma unroll
                    for (int j = 0; j < NP; j++)
                        acc[i][j] = add2_rn(acc[i][j], make_float2(__fmul_rn(xv, lt_el(wc[2 * j], e)),
                                                                   __fmul_rn(xv, lt_el(wc[2 * j + 1], e))));
                    if constexpr (RPT % 2 == 1)
                        acc1[i] = __fadd_rn(acc1[i], __fmul_rn(xv, lt_el(wc[RPT - 1], e)));
                }
            }
        }
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int i = 0; i < TPT; i++) {
        const int t = t0 + tq + i;
        if (t >= T) continue;
        float *row = logits + (size_t)t * Ep;
#pragma unroll
        for (int j = 0; j < NP; j++) {
            const int r = r0 + rq + lane + 64 * j;
            if (r < Ep) row[r] = acc[i][j].x;
            if (r + 32 < Ep) row[r + 32] = acc[i][j].y;
        }
        if constexpr (RPT % 2 == 1) {
            const int r = r0 + rq + lane + 32 * (RPT - 1);
            if (r < Ep) row[r] = acc1[i];
        }
    }
}

template <int TT>
static int launch_logits_rows(const float *x, int T, int H, int E, int Ep, const float *router,
                              const float *shared_gate, float *logits, __half *xh, int *err,
                              int dev, cudaStream_t s) {
    static bool attr[64] = {false};
    const size_t smem = lr_smem_bytes(TT, H);
    if (dev < 64 && !attr[dev]) {
        QG_CUDA(cudaFuncSetAttribute(k_logits_rows<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)LR_SMEM_MAX));
        attr[dev] = true;
    }
    QG_CUDA(launch_pdl(k_logits_rows<TT>, dim3((Ep + LR_RR - 1) / LR_RR, (T + TT - 1) / TT),
                       dim3(LR_RR * TT), smem, s, 1, x, T, H, E, Ep, router, shared_gate, logits,
                       xh, err));
    return QGMOE_OK;
}

// Tile shapes by batch size: the chains are long (H steps each), so small
// batches hold whole rows in shared memory (k_logits_rows) and large batches
// keep enough chains per thread to keep the FP32 pipes busy.
template <int TPT, int RPT, int TTH, int RTH>
static int launch_logits_t(const float *x, int T, int H, int E, int Ep, const float *router,
                           const float *shared_gate, float *logits, __half *xh, int *err,
                           cudaStream_t s) {
    using C = LgCfg<TPT, RPT, TTH, RTH>;
    QG_CUDA(launch_pdl(k_logits<TPT, RPT, TTH, RTH>,
                       dim3((T + C::TT - 1) / C::TT, (Ep + C::RR - 1) / C::RR), dim3(C::THREADS),
                       0, s, 1, x, T, H, E, Ep, router, shared_gate, logits, xh, err));
    return QGMOE_OK;
}

template <int TPT, int RPT>
static int launch_logits_tma_t(const CUtensorMap &mx, const CUtensorMap &mw, int T, int H, int Ep,
                               float *logits, __half *xh, int *err, int dev, cudaStream_t s) {
    using C = LtCfg<TPT, RPT>;
    static bool attr[64] = {false};
    if (dev >= 64 || !attr[dev]) {
        QG_CUDA(cudaFuncSetAttribute(k_logits_tma<TPT, RPT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        if (dev < 64) attr[dev] = true;
    }
    QG_CUDA(launch_pdl(k_logits_tma<TPT, RPT>, dim3((T + C::TT - 1) / C::TT, (Ep + C::RR - 1) / C::RR),
                       dim3(LT_THREADS), C::SMEM, s, 1, mx, mw, T, H, Ep, logits, xh, err));
    return QGMOE_OK;
}

using LtLaunch = int (*)(const CUtensorMap &, const CUtensorMap &, int, int, int, float *, __half *,
                         int *, int, cudaStream_t);
template <int RPT>
static LtLaunch lt_pick(int tpt) {
    static const LtLaunch f[8] = {launch_logits_tma_t<1, RPT>, launch_logits_tma_t<2, RPT>,
                                  launch_logits_tma_t<3, RPT>, launch_logits_tma_t<4, RPT>,
                                  launch_logits_tma_t<5, RPT>, launch_logits_tma_t<6, RPT>,
                                  launch_logits_tma_t<7, RPT>, launch_logits_tma_t<8, RPT>};
    return f[tpt - 1];
}

// k_logits_tma when its layout applies (router rows and the shared gate row
// contiguous, x and the router 16-byte aligned); returns 1 when it does not,
// so the caller takes k_logits.  Router rows per CTA: 64 RPT (RPT = 1..4,
// the smallest that holds Ep, row tiles of 256 beyond); tokens per CTA:
// 4 TPT, the smallest TPT <= 8 that covers the batch in one wave.
static int launch_logits_tma(const float *x, int T, int H, int E, int Ep, const float *router,
                             const float *shared_gate, float *logits, __half *xh, int *err,
                             int dev, cudaStream_t s) {
    if (Ep > E && shared_gate != router + (size_t)E * H) return 1;
    const int RPT = Ep <= 64 ? 1 : Ep <= 128 ? 2 : Ep <= 192 ? 3 : 4;
    const int RT = (Ep + 64 * RPT - 1) / (64 * RPT);
    const int per = LT_G * num_sms(dev);  // token groups of one wave
    int tpt = (int)(((int64_t)T * RT + per - 1) / per);
    tpt = tpt < 1 ? 1 : tpt > 8 ? 8 : tpt;
    CUtensorMap mx, mw;
    if (!encode_f32_map(&mx, x, T, H, LT_G * tpt) || !encode_f32_map(&mw, router, Ep, H, 64 * RPT))
        return 1;
    const LtLaunch f = RPT == 1 ? lt_pick<1>(tpt) : RPT == 2 ? lt_pick<2>(tpt)
                     : RPT == 3 ? lt_pick<3>(tpt) : lt_pick<4>(tpt);
    return f(mx, mw, T, H, Ep, logits, xh, err, dev, s);
}

static int launch_logits(const float *x, int T, int H, int E, int Ep, const float *router,
                         const float *shared_gate, float *logits, __half *xh, int *err, int dev,
                         cudaStream_t s) {
    // up to 64 tokens: 8-token tiles, so the chains spread over more SMs
    // (64 tokens x 128 rows: 128 CTAs) -- each chain's serial adds, not the
    // copies, set the time
    if (T <= 64 && lr_smem_bytes(8, H) <= LR_SMEM_MAX)
        return launch_logits_rows<8>(x, T, H, E, Ep, router, shared_gate, logits, xh, err, dev, s);
    if (T <= 64 && lr_smem_bytes(16, H) <= LR_SMEM_MAX)
        return launch_logits_rows<16>(x, T, H, E, Ep, router, shared_gate, logits, xh, err, dev, s);
    const int rc = launch_logits_tma(x, T, H, E, Ep, router, shared_gate, logits, xh, err, dev, s);
    if (rc != 1) return rc;
    // 32 tokens x 64 rows, 16 chains per thread (8 f32x2 pairs)
    return launch_logits_t<4, 4, 8, 16>(x, T, H, E, Ep, router, shared_gate, logits, xh, err, s);
}

// ---- 2. softmax + top-k + histograms --------------------------------------------
__device__ __forceinline__ void scatter_chunk(int c, int T, int E, int k, int has_shared,
                                              const RouteState &st, int *err, int *sm,
                                              int *partial);

// One warp per token: lane l owns experts l, l+32, ..., l+32*(NJ-1) (NJ =
// ceil(E/32) rounded up to a power of two).  FUSED (T <= TK_TOK, one CTA):
// the scatter of the single token chunk follows in the same CTA once the
// expert offsets are known.
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
        int *sel = s_idx[warp];
        const float wr = route_token<NJ>(logits + (size_t)t * Ep, E, k, mode, lane, sel);
        if (lane < k) {
            const int e = sel[lane];
            st.topk_idx[(size_t)t * k + lane] = e;
            st.topk_w[(size_t)t * k + lane] = wr;
            if (e >= 0 && e < E)
                atomicAdd(&hist_s[dispatch_key(e, E, st.ep_world, st.ep_slot)], 1);
            else
                atomicOr(err, QG_FLAG_BAD_EXPERT);
        }
        if (has_shared && lane == 0) {
            // sigmoid1 (model/tensors.go:97) of the shared-gate logit
            const float g = logits[(size_t)t * Ep + E];
            st.shared_w[t] = __fdiv_rn(1.f, __fadd_rn(1.f, (float)exp(-(double)g)));
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


// xp[s, :] = xh[slot_token[s], :] (fp16 rows, 16-byte copies).
__global__ void k_gather_h16(const __half *__restrict__ xh, const int32_t *__restrict__ slot_token,
                             int nslots, int H, __half *__restrict__ xp) {
    pdl_enter();
    const int wg = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int s = wg; s < nslots; s += nw) {
        const uint4 *src = reinterpret_cast<const uint4 *>(xh + (size_t)slot_token[s] * H);
        uint4 *dst = reinterpret_cast<uint4 *>(xp + (size_t)s * H);
        for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
    }
}

static int launch_gather_h16(const __half *xh, const int32_t *slot_token, int nslots, int H,
                             __half *xp, int dev, cudaStream_t s) {
    if (nslots <= 0) return QGMOE_OK;
    int blocks = (nslots + 7) / 8;
    const int cap = num_sms(dev) * 8;
    if (blocks > cap) blocks = cap;
    QG_CUDA(launch_pdl(k_gather_h16, dim3(blocks), dim3(256), 0, s, 1, xh, slot_token, nslots, H,
                       xp));
    return QGMOE_OK;
}

int launch_route(const float *x, int T, int H, int E, int k, int mode, const float *router,
                 const float *shared_gate, int has_shared, RouteState st, __half *xh, __half *xp,
                 int *err, cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int Ep = E + (has_shared ? 1 : 0);
    int rc = launch_logits(x, T, H, E, Ep, router, shared_gate, st.logits, xp ? xh : nullptr, err,
                           dev, s);
    if (rc) return rc;
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
        return launch_gather_h16(xh, st.slot_token, nslots, H, xp, dev, s);
    }
    return QGMOE_OK;
}

}  // namespace qg
