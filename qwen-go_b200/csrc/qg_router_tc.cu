// Router logits on the 5th-generation tensor cores, for prefill-sized
// batches (logits = x . router^T, proj(x,1,&m.gate,...) in model/moe.go:42;
// the shared-expert gate vector rides along as router row E,
// model/moe.go:87-93).
//
// The logits decide the routing, so they need f32 accuracy, not fp16: each
// operand is split into an fp16 head and an fp16 tail (a = ah + al, al =
// fp16(a - ah), together about 22 significant bits) and
//   logits = xh.Wh + xh.Wl + xl.Wh       (the xl.Wl term is below 2^-22)
// with the products accumulated in f32 in TMEM.  The router rows are split
// once at create time; x is split per call (k_split_x), and its head xh is
// also the fp16 activation row the expert GEMMs gather, so the gather then
// copies fp16 rows instead of converting f32 ones.
//
// k_logits_tc: CTA tile = 128 router rows x 256 tokens x one K slice; the
// KS slices of a tile form a cluster and add their partial tiles through
// distributed shared memory in rank order (deterministic), as the CUDA-core
// kernel does.  Warp 0 lane 0 issues the TMA loads (four 64-wide tiles per
// stage: Wh, Wl, xh, xl, SWIZZLE_128B) into a 2-stage ring, warp 1 lane 0
// issues three tcgen05.mma (M=128, N=256, K=16) per 16-wide K step, warps
// 2-5 drain the TMEM accumulator.  Inputs beyond fp16 range (|x| > 65504)
// raise QG_FLAG_RANGE instead of silently routing on infinities.
#include "qg_common.cuh"
#include "qg_sm100.cuh"

namespace qg {
using namespace sm100;

constexpr int RTC_M = 128, RTC_N = 256, RTC_BK = 64, RTC_STAGES = 2;
constexpr int RTC_A = RTC_M * RTC_BK * 2;               // 16 KB fp16 tile
constexpr int RTC_B = RTC_N * RTC_BK * 2;               // 32 KB fp16 tile
constexpr int RTC_STAGE = 2 * RTC_A + 2 * RTC_B;        // Wh, Wl, xh, xl
constexpr int RTC_RED = RTC_N * RTC_M * 4;              // partial tile, f32
constexpr int RTC_BODY = RTC_STAGES * RTC_STAGE > RTC_RED ? RTC_STAGES * RTC_STAGE : RTC_RED;
constexpr int RTC_SMEM = RTC_BODY + 1024 + 128;         // + alignment + barriers
constexpr int RTC_THREADS = 6 * 32;                     // producer, MMA, 4 epilogue warps
constexpr long long RTC_WAIT_CYCLES = 4000000000LL;     // ~2 s

// a (f32) -> head, tail (fp16); flags a finite value whose head overflows.
__device__ __forceinline__ void split2(float a, __half &h, __half &l, bool &bad) {
    h = __float2half_rn(a);
    const float hf = __half2float(h);
    bad |= isfinite(a) && !isfinite(hf);
    l = __float2half_rn(a - hf);
}

// Router rows (and the shared-gate row) -> [rows_pad, H] heads and tails,
// padding rows zero.
__global__ void k_split_rows(const float *__restrict__ router, const float *__restrict__ gate,
                             int E, int Ep, int H, int rows_pad, __half *__restrict__ wh,
                             __half *__restrict__ wl, int *err) {
    const int64_t n = (int64_t)rows_pad * H;
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / H), c = (int)(i - (int64_t)r * H);
        const float v = r < E ? router[(size_t)r * H + c] : (r < Ep ? gate[c] : 0.f);
        __half h, l;
        split2(v, h, l, bad);
        wh[i] = h;
        wl[i] = l;
    }
    if (bad) atomicOr(err, QG_FLAG_RANGE);
}

// x [T, H] -> xh, xl (fp16), four elements per thread step.
__global__ void k_split_x(const float *__restrict__ x, int64_t n4, __half *__restrict__ xh,
                          __half *__restrict__ xl, int *err) {
    pdl_enter();
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        __half h0, h1, h2, h3, l0, l1, l2, l3;
        split2(v.x, h0, l0, bad);
        split2(v.y, h1, l1, bad);
        split2(v.z, h2, l2, bad);
        split2(v.w, h3, l3, bad);
        reinterpret_cast<__half2 *>(xh)[2 * i] = __halves2half2(h0, h1);
        reinterpret_cast<__half2 *>(xh)[2 * i + 1] = __halves2half2(h2, h3);
        reinterpret_cast<__half2 *>(xl)[2 * i] = __halves2half2(l0, l1);
        reinterpret_cast<__half2 *>(xl)[2 * i + 1] = __halves2half2(l2, l3);
    }
    if (bad) atomicOr(err, QG_FLAG_RANGE);
}

template <int KS>
__global__ void __launch_bounds__(RTC_THREADS, 1)
k_logits_tc(const __grid_constant__ CUtensorMap mwh, const __grid_constant__ CUtensorMap mwl,
            const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl,
            int T, int Ep, int KB, float *__restrict__ logits, int *err) {
    pdl_enter();
    extern __shared__ uint8_t rtc_smem[];
    uint8_t *base = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(rtc_smem) + 1023) & ~uintptr_t(1023));
    const uint32_t base_u32 = smem_u32(base);
    uint64_t *full = reinterpret_cast<uint64_t *>(base + RTC_BODY);   // [2]
    uint64_t *empty = full + RTC_STAGES;                              // [2]
    uint64_t *acc_full = empty + RTC_STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    const uint32_t abort_addr = smem_u32(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * RTC_N, r0 = blockIdx.y * RTC_M;
    const int kbs = KB / KS, kb0 = blockIdx.z * kbs;  // this CTA's K blocks

    if (tid == 0) {
        for (int s = 0; s < RTC_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        st_volatile_shared(abort_addr, 0);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, RTC_N);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto fail = [&]() {
        if (!ld_volatile_shared(abort_addr)) {
            st_volatile_shared(abort_addr, 1);
            atomicOr(err, QG_FLAG_TIMEOUT);
        }
    };

    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            prefetch_tmap(&mwh);
            prefetch_tmap(&mxh);
            int last = -1;
            for (int i = 0; i < kbs; i++) {
                const int s = i % RTC_STAGES;
                if (!mbar_wait(&empty[s], ((i / RTC_STAGES) & 1) ^ 1, abort_addr, RTC_WAIT_CYCLES)) {
                    fail();
                    break;
                }
                uint8_t *st = base + s * RTC_STAGE;
                const int kx = (kb0 + i) * RTC_BK;
                mbar_arrive_expect_tx(&full[s], RTC_STAGE);
                tma_load_2d(st, &mwh, kx, r0, &full[s]);
                tma_load_2d(st + RTC_A, &mwl, kx, r0, &full[s]);
                tma_load_2d(st + 2 * RTC_A, &mxh, kx, t0, &full[s]);
                tma_load_2d(st + 2 * RTC_A + RTC_B, &mxl, kx, t0, &full[s]);
                last = i;
            }
            if (last >= 0)  // our own copies land before shared memory is reused or freed
                mbar_wait(&full[last % RTC_STAGES], (last / RTC_STAGES) & 1, 0, RTC_WAIT_CYCLES);
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(RTC_M, RTC_N);
            bool ok = true;
            for (int i = 0; i < kbs; i++) {
                const int s = i % RTC_STAGES;
                if (!mbar_wait(&full[s], (i / RTC_STAGES) & 1, abort_addr, RTC_WAIT_CYCLES)) {
                    fail();
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = base_u32 + s * RTC_STAGE;
                const uint64_t ah = desc_k_sw128(st), al = desc_k_sw128(st + RTC_A);
                const uint64_t bh = desc_k_sw128(st + 2 * RTC_A);
                const uint64_t bl = desc_k_sw128(st + 2 * RTC_A + RTC_B);
                umma_ss_k64(tmem, ah, bh, idesc, i != 0);  // heads
                umma_ss_k64(tmem, ah, bl, idesc, 1);       // Wh . xl
                umma_ss_k64(tmem, al, bh, idesc, 1);       // Wl . xh
                umma_commit(&empty[s]);
            }
            umma_commit(acc_full);  // every MMA issued above has completed when this arrives
            if (!ok) mbar_wait(acc_full, 0, 0, RTC_WAIT_CYCLES);
        }
    } else {
        // ---- epilogue: TMEM -> [token][row] partial tile over the stage buffers ----
        const bool got = mbar_wait(acc_full, 0, abort_addr, RTC_WAIT_CYCLES);
        if (!got) fail();
        tc_fence_after();
        const int q = warp & 3, row = q * 32 + lane;
        float *red = reinterpret_cast<float *>(base);
        for (int c0 = 0; c0 < RTC_N; c0 += 32) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c0, v);
#pragma unroll
            for (int j = 0; j < 32; j++) red[(c0 + j) * RTC_M + row] = v[j];
        }
    }
    tc_fence_before();
    __syncthreads();
    // ---- partial tiles added over the cluster, tokens split over its CTAs ----
    const bool ok = !ld_volatile_shared(abort_addr);
    if constexpr (KS > 1) cluster_sync();
    const float *red = reinterpret_cast<const float *>(base);
    constexpr int TPC = RTC_N / KS;
    const int c = KS > 1 ? (int)cluster_ctarank() : 0;
    for (int idx = tid; idx < TPC * RTC_M; idx += RTC_THREADS) {
        const int tl = c * TPC + idx / RTC_M, r = idx % RTC_M;
        const int t = t0 + tl, row = r0 + r;
        float sum;
        if constexpr (KS > 1) {
            const uint32_t off = smem_u32(red + tl * RTC_M + r);
            float v[KS];
#pragma unroll
            for (int j = 0; j < KS; j++) v[j] = ld_cluster_f32(mapa_shared(off, j));
            sum = v[0];
#pragma unroll
            for (int j = 1; j < KS; j++) sum += v[j];
        } else {
            sum = red[tl * RTC_M + r];
        }
        if (ok && t < T && row < Ep) logits[(size_t)t * Ep + row] = sum;
    }
    if constexpr (KS > 1) cluster_sync();  // no CTA leaves while others read its tile
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, RTC_N);
    }
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

int launch_split_rows(const float *router, const float *shared_gate, int E, int Ep, int H,
                      int rows_pad, __half *wh, __half *wl, int *err, cudaStream_t s) {
    k_split_rows<<<256, 256, 0, s>>>(router, shared_gate, E, Ep, H, rows_pad, wh, wl, err);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_logits_tc(const RouterTC &tc, const float *x, int T, int H, int Ep, float *logits,
                     int *err, cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = num_sms(dev);
    const int64_t n4 = (int64_t)T * H / 4;
    int blocks = (int)((n4 + 255) / 256);
    if (blocks > sms * 8) blocks = sms * 8;
    QG_CUDA(launch_pdl(k_split_x, dim3(blocks), dim3(256), 0, s, 1, x, n4, tc.xh, tc.xl, err));
    // K split: a power of two <= 8 dividing the K blocks, about one wave of CTAs
    const int KB = H / RTC_BK;
    const int tiles = ((T + RTC_N - 1) / RTC_N) * (tc.rows_pad / RTC_M);
    int ks = 1;
    while (ks < 8 && 2 * ks * tiles <= sms && KB % (2 * ks) == 0 && KB / (2 * ks) >= 2) ks *= 2;
    using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const CUtensorMap, int, int, int, float *, int *);
    const Kern kern = ks == 1 ? k_logits_tc<1> : ks == 2 ? k_logits_tc<2>
                    : ks == 4 ? k_logits_tc<4> : k_logits_tc<8>;
    static bool attr[64] = {false};
    if (dev < 64 && !attr[dev]) {
        const Kern all[4] = {k_logits_tc<1>, k_logits_tc<2>, k_logits_tc<4>, k_logits_tc<8>};
        for (Kern k : all)
            QG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, RTC_SMEM));
        attr[dev] = true;
    }
    QG_CUDA(launch_pdl(kern, dim3((T + RTC_N - 1) / RTC_N, tc.rows_pad / RTC_M, ks),
                       dim3(RTC_THREADS), RTC_SMEM, s, ks, tc.map_wh, tc.map_wl, tc.map_xh,
                       tc.map_xl, T, Ep, KB, logits, err));
    return QGMOE_OK;
}

int launch_gather_h16(const __half *xh, const int32_t *slot_token, int nslots, int H, __half *xp,
                      cudaStream_t s) {
    if (nslots <= 0) return QGMOE_OK;
    int dev = 0;
    cudaGetDevice(&dev);
    int blocks = (nslots + 7) / 8;
    const int cap = num_sms(dev) * 8;
    if (blocks > cap) blocks = cap;
    QG_CUDA(launch_pdl(k_gather_h16, dim3(blocks), dim3(256), 0, s, 1, xh, slot_token, nslots, H,
                       xp));
    return QGMOE_OK;
}

}  // namespace qg
