// Grouped expert GEMMs on the 5th-generation tensor cores (kernels K3'/K4',
// prefill-sized token counts; also used for decode batches when forced).
//
// Swap-AB formulation per work unit (expert e, 128-row weight tile, <=NT
// token tile):
//   D[rows, tokens] = W[rows, K] * X[tokens, K]^T      (tcgen05.mma kind::f16)
// A = expert weights, dequantised from int8/int4 group-32 codes with fp16
//     scales (model/moe.go:134-157) by converter warps; the raw codes and
//     scales arrive through a deep ring of bulk TMA copies.  Two variants:
//       k_umma    (NT = 256, prefill): A goes to shared memory in the
//                 128B-swizzled UMMA layout;
//       k_umma_ts (NT = 64 / 16, decode): A goes straight to TMEM with
//                 tcgen05.st and the MMA reads it from there, which halves
//                 the shared-memory traffic per weight byte -- the limit for
//                 weight-streaming batches;
// B = the expert's token rows in fp16, brought in by tiled TMA (SWIZZLE_128B);
// D = fp32 accumulators in TMEM, double-buffered (2 x NT columns): a
//     dedicated epilogue warpgroup drains one buffer (tcgen05.ld) while the
//     next unit accumulates into the other.
//
// GEMM1 (SWIGLU): a weight tile holds 64 gate rows [r, r+64) in TMEM lanes
// 0-63 and the matching up rows [I + r, I + r + 64) (model/moe.go:70-71) in
// lanes 64-127, so one 128-row dequantised tile feeds a 256-token MMA and the
// epilogue pairs gate and up through a small shared-memory exchange to write
// h = silu(gate) * up (model/moe.go:72-76) in fp16 for GEMM2.
// GEMM2 (STORE): D = W_down * h^T (model/moe.go:77-81), written as fp16 d
// rows for the rank-ordered combine.
//
// The kernel is persistent (one CTA per SM, static stride over work units)
// and warp-specialised: converters, epilogue, code producer, MMA issuer and
// activation producer each run their own loop over the same unit sequence,
// coupled only by mbarriers.  Every mbarrier wait is bounded (clock64 budget);
// on timeout the CTA raises QG_FLAG_TIMEOUT, drains its own TMA loads and
// UMMAs, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <cstdio>

#include "qg_common.cuh"
#include "qg_sm100.cuh"

namespace qg {
using namespace sm100;

// Warp roles of the persistent CTA (one per SM).
constexpr int UM_CONV_WARPS = 8;   // warps 0-7: dequantise codes into swizzled fp16 A tiles
constexpr int UM_EPI_WARP0 = 8;    // warps 8-11: epilogue (TMEM lanes 0-127, one warp each)
constexpr int UM_CODE_WARP = 12;   // bulk TMA of raw codes + scales
constexpr int UM_MMA_WARP = 13;    // TMEM alloc + UMMA issue
constexpr int UM_ACT_WARP = 14;    // tiled TMA of the activation (B) tiles
constexpr int UM_THREADS = 15 * 32;
constexpr int UM_CONV = UM_CONV_WARPS * 32;
constexpr int UM_M = 128;          // weight rows per tile (= TMEM lanes)
// Max tokens per tile NT (= TMEM columns per accumulator buffer) is a template
// parameter: 256 for prefill batches, 64 or 16 for decode batches (smaller
// activation stages leave room for deeper rings).
constexpr int UM_BK = 64;          // K elements per stage (one 128-byte fp16 row)
constexpr int UM_XS = UM_M + 4;    // epilogue staging row stride (floats, 16 B aligned)
constexpr int UM_EC = 16;          // token columns per epilogue chunk
constexpr int UM_MAX_UNITS = 64;   // work units per CTA decoded once into shared memory
constexpr long long UM_WAIT_CYCLES = 4000000000LL;  // ~2 s at 1.9 GHz

// Raw tile of one k block (128 rows x 64 codes), the unit of the packed
// weight layout in HBM and of the code ring in shared memory: four 16-code
// chunks per row, stored chunk-major ([chunk][row][CB bytes]) so that
// consecutive rows are consecutive in shared memory, then the rows' two fp16
// group scales.  A tile's k blocks follow each other, so several k blocks
// travel as one bulk copy (copies of 4 KB reach only about half the HBM
// bandwidth that 8 KB and larger copies do).
template <int BITS>
struct RawTile {
    static constexpr int CB = BITS == 8 ? 16 : 8;            // bytes of one 16-code chunk
    static constexpr int CODE = UM_M * UM_BK * BITS / 8;     // 8 KB int8, 4 KB int4
    static constexpr int BYTES = CODE + UM_M * 4;
};

template <int BITS, int NT>
struct UmCfg {
    static constexpr int STAGES = 3;
    static constexpr int RAW_STAGES = BITS == 8 ? 6 : 8;
    static constexpr int A_BYTES = UM_M * UM_BK * 2;            // 16 KB fp16
    static constexpr int B_BYTES = NT * UM_BK * 2;              // 32 KB fp16
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RAW_CODE = RawTile<BITS>::CODE;
    static constexpr int RAW_BYTES = RawTile<BITS>::BYTES;
    static constexpr int ACC_COLS = NT;
    static constexpr int TMEM_COLS = 2 * ACC_COLS;
    static constexpr int XCH_BYTES = UM_EC * UM_XS * 4;
    static constexpr int UNIT_BYTES = UM_MAX_UNITS * 16;
    static constexpr int BAR_BYTES = 8 * (3 * STAGES + 2 * RAW_STAGES + 5) + 16;
    static constexpr int SMEM =
        STAGES * STAGE_BYTES + RAW_STAGES * RAW_BYTES + XCH_BYTES + UNIT_BYTES + BAR_BYTES + 1024;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(STAGE_BYTES % 1024 == 0, "UMMA tiles must stay 1024-byte aligned");
};

// Decode-tile variant (A in TMEM): warp roles.  Converter warp w writes K
// chunk w >> 2 (16 codes = 8 TMEM columns) of TMEM lane quarter w & 3.
constexpr int TS_CONV_WARPS = 16;  // warps 0-15
constexpr int TS_EPI_WARP0 = 16;   // warps 16-19 (lane quarter = warp & 3)
constexpr int TS_CODE_WARP = 20;
constexpr int TS_MMA_WARP = 21;
constexpr int TS_ACT_WARP = 22;
constexpr int TS_THREADS = 23 * 32;
constexpr int TS_KS = 4;           // k blocks per pipeline stage
constexpr int TS_S = 3;            // stages: A 4 x 32 TMEM columns, B 4 activation tiles

template <int BITS, int NT>
struct TsCfg {
    static constexpr int B_BYTES = NT * UM_BK * 2;                    // one tile: 8 / 2 KB fp16
    static constexpr int STAGE_B = TS_KS * B_BYTES;
    static constexpr int RAW_CODE = RawTile<BITS>::CODE;
    static constexpr int RAW_BYTES = RawTile<BITS>::BYTES;
    static constexpr int RAW_SLOT = TS_KS * RAW_BYTES;                // one stage of codes
    static constexpr int S = NT == 128 ? 2 : TS_S;                   // stages (TMEM budget)
    static constexpr int R = NT == 128 ? (BITS == 8 ? 2 : 4)
                           : NT == 64  ? (BITS == 8 ? 3 : 6)
                                       : (BITS == 8 ? 5 : 9);
    static constexpr int A_COL0 = 2 * NT;                             // after the accumulators
    static constexpr int TMEM_COLS = 512;
    static constexpr int XCH_BYTES = UM_EC * UM_XS * 4;
    static constexpr int UNIT_BYTES = UM_MAX_UNITS * 16;
    static constexpr int BAR_BYTES = 8 * (3 * S + 2 * R + 5) + 16;
    static constexpr int SMEM =
        S * STAGE_B + R * RAW_SLOT + XCH_BYTES + UNIT_BYTES + BAR_BYTES + 1024;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(B_BYTES % 1024 == 0, "UMMA tiles must stay 1024-byte aligned");
    static_assert(A_COL0 + S * TS_KS * 32 <= TMEM_COLS, "TMEM budget");
};

// int8 x4 stored biased (q + 128, repacked at create time) -> two fp16x2
// (q * s): exact codes, then one correctly rounded product.
__device__ __forceinline__ void cvt_i8x4(uint32_t u, __half2 s2, uint32_t &o0, uint32_t &o1) {
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    uint32_t p0 = __byte_perm(u, 0x64646464u, 0x4140);
    uint32_t p1 = __byte_perm(u, 0x64646464u, 0x4342);
    __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p0), bias), s2);
    __half2 h1 = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p1), bias), s2);
    o0 = *reinterpret_cast<uint32_t *>(&h0);
    o1 = *reinterpret_cast<uint32_t *>(&h1);
}

// int4 word in the repacked nibble order (element 2j in bits [4j, 4j+4),
// element 2j+1 in bits [16+4j, 20+4j)) -> four fp16x2 ((code - 8) * s), pairs
// j = 0..3.  Pairs 1 and 3 are taken in place (mask 0x00F0: 1024 + 16 code)
// and scaled back by an exact fma, so the word needs one shift and four masks:
// integer ops slow the tensor pipe of the same SM far more than fp16x2 ops.
__device__ __forceinline__ void cvt_i4_word(uint32_t w, __half2 s2, uint32_t *o) {
    const __half2 b1032 = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
    const __half2 r16 = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));  // 1/16
    const __half2 m72 = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));  // -72
    const uint32_t w8 = w >> 8;
    uint32_t p0 = (w & 0x000F000Fu) | 0x64006400u;   // 1024 + code
    uint32_t p1 = (w & 0x00F000F0u) | 0x64006400u;   // 1024 + 16 code
    uint32_t p2 = (w8 & 0x000F000Fu) | 0x64006400u;
    uint32_t p3 = (w8 & 0x00F000F0u) | 0x64006400u;
    __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p0), b1032), s2);
    __half2 h1 = __hmul2(__hfma2(*reinterpret_cast<__half2 *>(&p1), r16, m72), s2);
    __half2 h2 = __hmul2(__hsub2(*reinterpret_cast<__half2 *>(&p2), b1032), s2);
    __half2 h3 = __hmul2(__hfma2(*reinterpret_cast<__half2 *>(&p3), r16, m72), s2);
    o[0] = *reinterpret_cast<uint32_t *>(&h0);
    o[1] = *reinterpret_cast<uint32_t *>(&h1);
    o[2] = *reinterpret_cast<uint32_t *>(&h2);
    o[3] = *reinterpret_cast<uint32_t *>(&h3);
}

// One 16-code chunk of a raw tile (at shared address `code`) -> eight fp16x2
// words (K pairs 0-1, 2-3, ..., 14-15), scaled by the group scale `s2`.
template <int BITS>
__device__ __forceinline__ void cvt_chunk(uint32_t code, __half2 s2, uint32_t (&o)[8]) {
    if constexpr (BITS == 8) {
        const uint4 q = ld_shared_v4(code);
        cvt_i8x4(q.x, s2, o[0], o[1]);
        cvt_i8x4(q.y, s2, o[2], o[3]);
        cvt_i8x4(q.z, s2, o[4], o[5]);
        cvt_i8x4(q.w, s2, o[6], o[7]);
    } else {
        const uint2 q = ld_shared_v2(code);
        cvt_i4_word(q.x, s2, o);
        cvt_i4_word(q.y, s2, o + 4);
    }
}

// Group scale of tile row `row` for K chunk `q` (chunks 0-1: group 0, 2-3: group 1).
__device__ __forceinline__ __half2 chunk_scale(uint32_t scales, int row, int q) {
    uint32_t w = ld_shared_u32(scales + row * 4);
    const __half2 sc = *reinterpret_cast<__half2 *>(&w);
    return q >= 2 ? __high2half2(sc) : __low2half2(sc);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Named barrier for the 4 epilogue warps only.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Same barrier, returning the OR of every participant's predicate, so the
// four warps take one uniform decision.
__device__ __forceinline__ bool epi_bar_or(bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, 1, 128, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p)
        : "memory");
    return r != 0;
}

struct UmmaArgs {
    const uint8_t *wq;    // packed tiles [E][RT][KB] x RawTile<BITS>::BYTES
    int RT, KB;
    const int32_t *act_group, *act_begin, *act_n, *n_act, *tile_prefix;
    __half *out;          // SWIGLU: h [slots, out_stride]; STORE: d [slots, out_stride]
    int out_stride;
    const int32_t *out_map;  // STORE: output row of each slot (null = the slot itself)
    uint8_t *const *out_peers;  // STORE over peers: out_map = rank << 24 | row
    size_t out_peer_off;
    float *out32;         // STORE: f32 rows [slots, out_stride] instead of fp16 (QuantLinear)
    int *err;
};

// Decodes work unit u = (token tile, row tile) of the routed groups.
struct Unit {
    int e, rt, slot0, nval, N;
};
template <int NT>
__device__ __forceinline__ Unit decode_unit(const UmmaArgs &a, int n_act, int u) {
    Unit w;
    const int ti = u / a.RT;
    w.rt = u - ti * a.RT;
    int lo = 0, hi = n_act - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.tile_prefix[mid] <= ti) lo = mid; else hi = mid - 1;
    }
    w.e = a.act_group[lo];
    const int tt = ti - a.tile_prefix[lo];
    w.slot0 = a.act_begin[lo] + tt * NT;
    w.nval = min(NT, a.act_n[lo] - tt * NT);
    w.N = (w.nval + 15) & ~15;
    return w;
}

// Drains one accumulator buffer (this warp's TMEM lane quarter, token
// columns from lane_addr) into h rows (SwiGLU) or d rows.  Per chunk of 16
// token columns: every thread copies its TMEM lane (tile row) into a
// [token][row] staging buffer; then each thread takes one token and 8
// (SwiGLU) or 16 (store) consecutive rows and writes them as 16-byte vectors,
// so each token row of h / d goes out in coalesced 128-256 byte runs.  The
// four epilogue warps call it together (named barrier 1).
template <bool SWIGLU>
__device__ __forceinline__ void epi_unit(const UmmaArgs &a, const Unit &w, uint32_t lane_addr,
                                         uint32_t xch_u32, int L, int ej, int er) {
    for (int c0 = 0; c0 < w.N; c0 += UM_EC) {
        float v[16];
        tmem_ld16(lane_addr + c0, v);
#pragma unroll
        for (int j = 0; j < UM_EC; j++) st_shared_f32(xch_u32 + (j * UM_XS + L) * 4, v[j]);
        epi_bar();
        const int t = c0 + ej;
        if (t < w.nval) {
            const uint32_t rowp = xch_u32 + (ej * UM_XS + er) * 4;
            if constexpr (SWIGLU) {
                const float4 g0 = ld_shared_f4(rowp), g1 = ld_shared_f4(rowp + 16);
                const float4 u0 = ld_shared_f4(rowp + 256), u1 = ld_shared_f4(rowp + 272);
                const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
                const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                uint32_t o[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float h0 = __fdividef(gv[2 * q], 1.f + __expf(-gv[2 * q])) * uv[2 * q];
                    const float h1 =
                        __fdividef(gv[2 * q + 1], 1.f + __expf(-gv[2 * q + 1])) * uv[2 * q + 1];
                    __half2 hh = __floats2half2_rn(h0, h1);
                    o[q] = *reinterpret_cast<uint32_t *>(&hh);
                }
                __half *dst = a.out + (size_t)(w.slot0 + t) * a.out_stride + w.rt * 64 + er;
                *reinterpret_cast<uint4 *>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
            } else if (a.out32) {  // f32 rows (QuantLinear): 16 rows as four 16-byte stores
                float4 *dst = reinterpret_cast<float4 *>(
                    a.out32 + (size_t)(w.slot0 + t) * a.out_stride + w.rt * UM_M + er);
#pragma unroll
                for (int q = 0; q < 4; q++) dst[q] = ld_shared_f4(rowp + 16 * q);
            } else {
                uint32_t o[8];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float4 f = ld_shared_f4(rowp + 16 * q);
                    __half2 a2 = __floats2half2_rn(f.x, f.y), b2 = __floats2half2_rn(f.z, f.w);
                    o[2 * q] = *reinterpret_cast<uint32_t *>(&a2);
                    o[2 * q + 1] = *reinterpret_cast<uint32_t *>(&b2);
                }
                __half *dst;
                if (a.out_peers) {  // expert parallelism: straight into the source rank
                    const int code = a.out_map[w.slot0 + t];
                    dst = reinterpret_cast<__half *>(a.out_peers[code >> 24] + a.out_peer_off) +
                          (size_t)(code & 0xFFFFFF) * a.out_stride + w.rt * UM_M + er;
                } else {
                    const int orow = a.out_map ? a.out_map[w.slot0 + t] : w.slot0 + t;
                    dst = a.out + (size_t)orow * a.out_stride + w.rt * UM_M + er;
                }
                reinterpret_cast<uint4 *>(dst)[0] = make_uint4(o[0], o[1], o[2], o[3]);
                reinterpret_cast<uint4 *>(dst)[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
        }
        epi_bar();
    }
}

template <int BITS, bool SWIGLU, int NT>
__global__ void __launch_bounds__(UM_THREADS, 1)
k_umma(const __grid_constant__ CUtensorMap tmap_b, const UmmaArgs a) {
    pdl_enter();
    using Cfg = UmCfg<BITS, NT>;
    constexpr int S = Cfg::STAGES;
    constexpr int R = Cfg::RAW_STAGES;
    extern __shared__ uint8_t smem_raw[];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_act = *a.n_act;
    const int n_units = a.tile_prefix[n_act] * a.RT;
    if ((int)blockIdx.x >= n_units) return;

    uint8_t *base = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base_u32 = smem_u32(base);
    uint8_t *raw = base + S * Cfg::STAGE_BYTES;
    const uint32_t raw_u32 = base_u32 + S * Cfg::STAGE_BYTES;
    const uint32_t xch_u32 = raw_u32 + R * Cfg::RAW_BYTES;  // [UM_EC tokens][UM_XS] f32
    const uint32_t utab_u32 = xch_u32 + Cfg::XCH_BYTES;      // this CTA's decoded units
    uint64_t *fullA = reinterpret_cast<uint64_t *>(raw + R * Cfg::RAW_BYTES + Cfg::XCH_BYTES +
                                                   Cfg::UNIT_BYTES);
    uint64_t *fullB = fullA + S;
    uint64_t *empty = fullB + S;
    uint64_t *rawFull = empty + S;
    uint64_t *rawEmpty = rawFull + R;
    uint64_t *accFull = rawEmpty + R;   // [2]
    uint64_t *accEmpty = accFull + 2;   // [2]
    uint64_t *drain = accEmpty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    const uint32_t abort_addr = smem_u32(tmem_slot + 1);

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&fullA[s], UM_CONV_WARPS);
            mbar_init(&fullB[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < R; r++) {
            mbar_init(&rawFull[r], 1);
            mbar_init(&rawEmpty[r], UM_CONV_WARPS);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accFull[b], 1);
            mbar_init(&accEmpty[b], 4);
        }
        mbar_init(drain, 1);
        st_volatile_shared(abort_addr, 0);
        fence_mbar_init();
    }
    if (warp == UM_MMA_WARP) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    // Decode this CTA's units once (one binary search per unit, in parallel),
    // so no role walks the active-expert tables in global memory per unit.
    const int n_mine = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const bool utab = n_mine <= UM_MAX_UNITS;
    if (utab)
        for (int i = tid; i < n_mine; i += UM_THREADS) {
            const Unit w = decode_unit<NT>(a, n_act, blockIdx.x + i * gridDim.x);
            st_shared_v4(utab_u32 + i * 16, w.e, w.rt, w.slot0, w.nval);
        }
    auto unit_at = [&](int i, int u) -> Unit {
        if (!utab) return decode_unit<NT>(a, n_act, u);
        const uint4 v = ld_shared_v4(utab_u32 + i * 16);
        return Unit{(int)v.x, (int)v.y, (int)v.z, (int)v.w, ((int)v.w + 15) & ~15};
    };
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&]() {
        if (!ld_volatile_shared(abort_addr)) {
            st_volatile_shared(abort_addr, 1);
            atomicOr(a.err, QG_FLAG_TIMEOUT);
        }
    };

    if (warp < UM_CONV_WARPS) {
        // ============ converters: raw ring -> fp16 swizzled A tiles ==========
        // Thread i of 256 converts chunks i and i + 256 (chunk c = (q, row) with
        // q = c / 128): 16 codes -> two 16-byte fp16 runs of the row's 128-byte
        // swizzled line.  Its shared-memory offsets are fixed.
        constexpr int PER_THREAD = 4 * UM_M / UM_CONV;
        constexpr int CB = RawTile<BITS>::CB;
        uint32_t code_off[PER_THREAD], st_off[PER_THREAD][2];
        int row_of[PER_THREAD], q_of[PER_THREAD];
#pragma unroll
        for (int j = 0; j < PER_THREAD; j++) {
            const int i = tid + UM_CONV * j;
            const int q = i / UM_M, row = i % UM_M;
            row_of[j] = row;
            q_of[j] = q;
            code_off[j] = i * CB;
            st_off[j][0] = row * 128 + (((2 * q) ^ (row & 7)) << 4);
            st_off[j][1] = row * 128 + (((2 * q + 1) ^ (row & 7)) << 4);
        }
        int g = 0;  // running k-block counter across this CTA's units
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            for (int kb = 0; kb < a.KB; kb++, g++) {
                const int r = g % R, s = g % S;
                if (!mbar_wait(&rawFull[r], (g / R) & 1, abort_addr, UM_WAIT_CYCLES) ||
                    !mbar_wait(&empty[s], ((g / S) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                    fail();
                    ok = false;
                    break;
                }
                const uint32_t rs = raw_u32 + r * Cfg::RAW_BYTES;
                const uint32_t A = base_u32 + s * Cfg::STAGE_BYTES;
#pragma unroll
                for (int j = 0; j < PER_THREAD; j++) {
                    uint32_t o[8];
                    cvt_chunk<BITS>(rs + code_off[j],
                                    chunk_scale(rs + Cfg::RAW_CODE, row_of[j], q_of[j]), o);
                    st_shared_v4(A + st_off[j][0], o[0], o[1], o[2], o[3]);
                    st_shared_v4(A + st_off[j][1], o[4], o[5], o[6], o[7]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&fullA[s]);
                    mbar_arrive(&rawEmpty[r]);
                }
            }
        }
    } else if (warp < UM_EPI_WARP0 + 4) {
        // ============ epilogue: TMEM -> SwiGLU / store ============================
        const int ew = warp - UM_EPI_WARP0;  // TMEM lane quarter
        const int L = ew * 32 + lane;        // TMEM lane = tile row
        const int et = tid - UM_EPI_WARP0 * 32;  // 0..127
        const int ej = et >> 3;                  // token column within the chunk
        const int er = (et & 7) * (SWIGLU ? 8 : 16);  // first row handled
        int lt = 0;
        for (int u = blockIdx.x; u < n_units; u += gridDim.x, lt++) {
            const int buf = lt & 1;
            bool bad = !mbar_wait(&accFull[buf], (lt >> 1) & 1, abort_addr, UM_WAIT_CYCLES);
            // the four warps meet at named barriers below, so they must agree
            // on stopping; the OR-barrier makes that decision uniform
            bad = epi_bar_or(bad || ld_volatile_shared(abort_addr));
            if (bad) {
                fail();
                break;
            }
            tc_fence_after();
            const Unit w = unit_at(lt, u);
            const uint32_t lane_addr = tmem + buf * Cfg::ACC_COLS + ((uint32_t)(ew * 32) << 16);
            epi_unit<SWIGLU>(a, w, lane_addr, xch_u32, L, ej, er);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accEmpty[buf]);
        }
    } else if (warp == UM_CODE_WARP) {
        // ============ code/scale producer (bulk TMA) ==============================
        if (lane == 0) {
            int g = 0, last = -1;
            bool ok = true;
            for (int u = blockIdx.x, i = 0; u < n_units && ok; u += gridDim.x, i++) {
                const Unit w = unit_at(i, u);
                const uint8_t *tile =
                    a.wq + (size_t)(w.e * a.RT + w.rt) * a.KB * Cfg::RAW_BYTES;
                for (int kb = 0; kb < a.KB; kb++, g++) {
                    const int r = g % R;
                    if (!mbar_wait(&rawEmpty[r], ((g / R) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                        fail();
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&rawFull[r], Cfg::RAW_BYTES);
                    bulk_load(raw + r * Cfg::RAW_BYTES, tile + (size_t)kb * Cfg::RAW_BYTES,
                              Cfg::RAW_BYTES, &rawFull[r]);
                    last = g;
                }
            }
            if (!ok && last >= 0)  // let our own last copy land before smem goes away
                mbar_wait(&rawFull[last % R], (last / R) & 1, 0, UM_WAIT_CYCLES);
        }
    } else if (warp == UM_ACT_WARP) {
        // ============ activation producer (tiled TMA) =============================
        if (lane == 0) {
            prefetch_tmap(&tmap_b);
            int g = 0, last = -1;
            bool ok = true;
            for (int u = blockIdx.x, i = 0; u < n_units && ok; u += gridDim.x, i++) {
                const Unit w = unit_at(i, u);
                for (int kb = 0; kb < a.KB; kb++, g++) {
                    const int s = g % S;
                    if (!mbar_wait(&empty[s], ((g / S) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                        fail();
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&fullB[s], Cfg::B_BYTES);
                    tma_load_2d(base + s * Cfg::STAGE_BYTES + Cfg::A_BYTES, &tmap_b, kb * UM_BK,
                                w.slot0, &fullB[s]);
                    last = g;
                }
            }
            if (!ok && last >= 0)
                mbar_wait(&fullB[last % S], (last / S) & 1, 0, UM_WAIT_CYCLES);
        }
    } else {
        // ============ MMA issuer =====================================================
        if (lane == 0) {
            int g = 0, lt = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, lt++) {
                const Unit w = unit_at(lt, u);
                const uint32_t idesc = idesc_f16_f32(UM_M, w.N);
                const int buf = lt & 1;
                if (!mbar_wait(&accEmpty[buf], ((lt >> 1) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                    fail();
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + buf * Cfg::ACC_COLS;
                for (int kb = 0; kb < a.KB; kb++, g++) {
                    const int s = g % S;
                    const uint32_t par = (g / S) & 1;
                    if (!mbar_wait(&fullB[s], par, abort_addr, UM_WAIT_CYCLES) ||
                        !mbar_wait(&fullA[s], par, abort_addr, UM_WAIT_CYCLES)) {
                        fail();
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t asm_ = base_u32 + s * Cfg::STAGE_BYTES;
                    umma_ss_k64(acc, desc_k_sw128(asm_), desc_k_sw128(asm_ + Cfg::A_BYTES), idesc,
                                kb != 0);
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&accFull[buf]);
            }
            if (!ok) {
                umma_commit(drain);  // our own UMMAs finish before TMEM is released
                mbar_wait(drain, 0, 0, UM_WAIT_CYCLES);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == UM_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

// ---- decode tiles: A operand in TMEM ---------------------------------------------
// Same unit sequence and roles as k_umma, with the dequantised weight tile
// written to TMEM (tcgen05.st.32x32b: thread = tile row = TMEM lane, 16 K
// codes -> 8 columns of fp16 pairs) instead of shared memory.  A pipeline
// stage covers four k blocks (A: 128 TMEM columns, B: four activation
// tiles), so the MMA issuer waits once, issues 16 MMAs and commits once per
// stage, and each converter thread loads and converts four independent
// chunks before storing them: at N <= 64 the per-stage barrier and latency
// chains, not the MMAs, would otherwise pace the weight stream.
// TMEM columns: [0, NT) and [NT, 2NT) accumulators, then 3 A stages of 128.
// Barriers: fullA[s] completes when the 16 converter warps have stored A,
// fullB[s] when both activation tiles have landed, empty[s] when the stage's
// MMAs have completed (one tcgen05.commit frees A and B together).
template <int BITS, bool SWIGLU, int NT>
__global__ void __launch_bounds__(TS_THREADS, 1)
k_umma_ts(const __grid_constant__ CUtensorMap tmap_b, const UmmaArgs a) {
    pdl_launch_dependents();
    using Cfg = TsCfg<BITS, NT>;
    constexpr int S = Cfg::S, R = Cfg::R;
    constexpr int CB = RawTile<BITS>::CB;
    extern __shared__ uint8_t smem_raw[];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KP = (a.KB + TS_KS - 1) / TS_KS;  // stages per unit (the last may be partial)

    uint8_t *base = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base_u32 = smem_u32(base);                 // activation stages
    uint8_t *raw = base + S * Cfg::STAGE_B;
    const uint32_t raw_u32 = base_u32 + S * Cfg::STAGE_B;
    const uint32_t xch_u32 = raw_u32 + R * Cfg::RAW_SLOT;
    const uint32_t utab_u32 = xch_u32 + Cfg::XCH_BYTES;
    uint64_t *fullA = reinterpret_cast<uint64_t *>(raw + R * Cfg::RAW_SLOT + Cfg::XCH_BYTES +
                                                   Cfg::UNIT_BYTES);
    uint64_t *fullB = fullA + S;
    uint64_t *empty = fullB + S;
    uint64_t *rawFull = empty + S;
    uint64_t *rawEmpty = rawFull + R;
    uint64_t *accFull = rawEmpty + R;   // [2]
    uint64_t *accEmpty = accFull + 2;   // [2]
    uint64_t *drain = accEmpty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    const uint32_t abort_addr = smem_u32(tmem_slot + 1);

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&fullA[s], TS_CONV_WARPS / 2);  // the stage's converter group
            mbar_init(&fullB[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < R; r++) {
            mbar_init(&rawFull[r], 1);
            mbar_init(&rawEmpty[r], TS_CONV_WARPS / 2);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accFull[b], 1);
            mbar_init(&accEmpty[b], 4);
        }
        mbar_init(drain, 1);
        st_volatile_shared(abort_addr, 0);
        fence_mbar_init();
    }
    if (warp == TS_MMA_WARP) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    // everything above reads no global memory; the routing tables below come
    // from the previous kernels
    pdl_wait();
    const int n_act = *a.n_act;
    const int n_units = a.tile_prefix[n_act] * a.RT;
    if ((int)blockIdx.x >= n_units) {  // no work: give the TMEM back and leave
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (warp == TS_MMA_WARP) tmem_dealloc(*tmem_slot, Cfg::TMEM_COLS);
        return;
    }
    const int n_mine = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const bool utab = n_mine <= UM_MAX_UNITS;
    if (utab)
        for (int i = tid; i < n_mine; i += TS_THREADS) {
            const Unit w = decode_unit<NT>(a, n_act, blockIdx.x + i * gridDim.x);
            st_shared_v4(utab_u32 + i * 16, w.e, w.rt, w.slot0, w.nval);
        }
    // this CTA's i-th unit (units b, b + grid, b + 2 grid, ...)
    auto unit_at = [&](int i) -> Unit {
        if (!utab) return decode_unit<NT>(a, n_act, blockIdx.x + i * gridDim.x);
        const uint4 v = ld_shared_v4(utab_u32 + i * 16);
        return Unit{(int)v.x, (int)v.y, (int)v.z, (int)v.w, ((int)v.w + 15) & ~15};
    };
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&]() {
        if (!ld_volatile_shared(abort_addr)) {
            st_volatile_shared(abort_addr, 1);
            atomicOr(a.err, QG_FLAG_TIMEOUT);
        }
    };

    if (warp < TS_CONV_WARPS) {
        // ============ converters: raw ring -> fp16 A tiles in TMEM ===========
        // Two groups of 8 warps take alternate stages, so one group converts
        // stage s+1 while the other's stores for stage s drain.  In a group,
        // warp w covers TMEM lane quarter w & 3 and K chunks 2c, 2c+1
        // (c = (w >> 2) & 1) of every k block of the stage.
        const int grp = warp >> 3;
        const int qd = warp & 3, c2 = ((warp >> 2) & 1) * 2;
        const int row = qd * 32 + lane;
        const uint32_t ta = tmem + ((uint32_t)(qd * 32) << 16) + Cfg::A_COL0;
        int gs = 0;
        bool ok = true;
        for (int i = 0; i < n_mine && ok; i++) {
            for (int kp = 0; kp < KP; kp++, gs++) {
                if ((gs & 1) != grp) continue;
                const int s = gs % S;
                const int nk = min(TS_KS, a.KB - kp * TS_KS);
                if (!mbar_wait(&empty[s], ((gs / S) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                    fail();
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int r = gs % R;  // one raw slot per stage
                if (!mbar_wait(&rawFull[r], (gs / R) & 1, abort_addr, UM_WAIT_CYCLES)) {
                    fail();
                    ok = false;
                    break;
                }
                // per half of the stage: the two chunks of two k blocks,
                // converted as independent chains, then stored to TMEM
#pragma unroll
                for (int hh = 0; hh < TS_KS; hh += 2) {
                    uint32_t o[4][8];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int h = hh + (j >> 1), q = c2 + (j & 1);
                        if (h < nk) {
                            const uint32_t rs = raw_u32 + r * Cfg::RAW_SLOT + h * Cfg::RAW_BYTES;
                            cvt_chunk<BITS>(rs + (uint32_t)(q * UM_M + row) * CB,
                                            chunk_scale(rs + Cfg::RAW_CODE, row, q), o[j]);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int h = hh + (j >> 1), q = c2 + (j & 1);
                        if (h < nk) tmem_st8(ta + s * (TS_KS * 32) + h * 32 + q * 8, o[j]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&rawEmpty[r]);  // codes consumed by the stores
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&fullA[s]);
            }
        }
    } else if (warp < TS_EPI_WARP0 + 4) {
        // ============ epilogue: TMEM -> SwiGLU / store ============================
        const int ew = warp & 3;                 // TMEM lane quarter
        const int L = ew * 32 + lane;            // TMEM lane = tile row
        const int et = tid - TS_EPI_WARP0 * 32;  // 0..127
        const int ej = et >> 3;
        const int er = (et & 7) * (SWIGLU ? 8 : 16);
        for (int lt = 0; lt < n_mine; lt++) {
            const int buf = lt & 1;
            bool bad = !mbar_wait(&accFull[buf], (lt >> 1) & 1, abort_addr, UM_WAIT_CYCLES);
            bad = epi_bar_or(bad || ld_volatile_shared(abort_addr));
            if (bad) {
                fail();
                break;
            }
            tc_fence_after();
            const Unit w = unit_at(lt);
            const uint32_t lane_addr = tmem + buf * NT + ((uint32_t)(ew * 32) << 16);
            epi_unit<SWIGLU>(a, w, lane_addr, xch_u32, L, ej, er);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accEmpty[buf]);
        }
    } else if (warp == TS_CODE_WARP) {
        // ============ code/scale producer (bulk TMA) ==============================
        if (lane == 0) {
            int g = 0, last = -1;
            bool ok = true;
            for (int i = 0; i < n_mine && ok; i++) {
                const Unit w = unit_at(i);
                const uint8_t *tile =
                    a.wq + (size_t)(w.e * a.RT + w.rt) * a.KB * Cfg::RAW_BYTES;
                for (int kp = 0; kp < KP; kp++, g++) {
                    const int r = g % R;
                    const int nk = min(TS_KS, a.KB - kp * TS_KS);
                    if (!mbar_wait(&rawEmpty[r], ((g / R) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                        fail();
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&rawFull[r], nk * Cfg::RAW_BYTES);
                    bulk_load(raw + r * Cfg::RAW_SLOT, tile + (size_t)kp * Cfg::RAW_SLOT,
                              nk * Cfg::RAW_BYTES, &rawFull[r]);
                    last = g;
                }
            }
            if (!ok && last >= 0)
                mbar_wait(&rawFull[last % R], (last / R) & 1, 0, UM_WAIT_CYCLES);
        }
    } else if (warp == TS_ACT_WARP) {
        // ============ activation producer (tiled TMA, two tiles per stage) =========
        if (lane == 0) {
            prefetch_tmap(&tmap_b);
            int gs = 0, last = -1;
            bool ok = true;
            for (int i = 0; i < n_mine && ok; i++) {
                const Unit w = unit_at(i);
                for (int kp = 0; kp < KP; kp++, gs++) {
                    const int s = gs % S;
                    const int nk = min(TS_KS, a.KB - kp * TS_KS);
                    if (!mbar_wait(&empty[s], ((gs / S) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                        fail();
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&fullB[s], nk * Cfg::B_BYTES);
                    uint8_t *dst = base + s * Cfg::STAGE_B;
                    for (int h = 0; h < nk; h++)
                        tma_load_2d(dst + h * Cfg::B_BYTES, &tmap_b, (kp * TS_KS + h) * UM_BK,
                                    w.slot0, &fullB[s]);
                    last = gs;
                }
            }
            if (!ok && last >= 0)  // let our own last copies land before smem goes away
                mbar_wait(&fullB[last % S], (last / S) & 1, 0, UM_WAIT_CYCLES);
        }
    } else {
        // ============ MMA issuer =====================================================
        if (lane == 0) {
            int gs = 0;
            bool ok = true;
            for (int lt = 0; lt < n_mine && ok; lt++) {
                const Unit w = unit_at(lt);
                const uint32_t idesc = idesc_f16_f32(UM_M, w.N);
                const int buf = lt & 1;
                if (!mbar_wait(&accEmpty[buf], ((lt >> 1) & 1) ^ 1, abort_addr, UM_WAIT_CYCLES)) {
                    fail();
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + buf * NT;
                for (int kp = 0; kp < KP; kp++, gs++) {
                    const int s = gs % S;
                    if (!mbar_wait(&fullB[s], (gs / S) & 1, abort_addr, UM_WAIT_CYCLES) ||
                        !mbar_wait(&fullA[s], (gs / S) & 1, abort_addr, UM_WAIT_CYCLES)) {
                        fail();
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int nk = min(TS_KS, a.KB - kp * TS_KS);
                    const uint32_t at = tmem + Cfg::A_COL0 + s * (TS_KS * 32);
                    const uint64_t bd = desc_k_sw128(base_u32 + s * Cfg::STAGE_B);
                    umma_ts_k64(acc, at, bd, idesc, kp != 0);
#pragma unroll
                    for (int h = 1; h < TS_KS; h++)
                        if (h < nk)
                            umma_ts_k64(acc, at + h * 32, bd + ((h * Cfg::B_BYTES) >> 4), idesc, 1);
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&accFull[buf]);
            }
            if (!ok) {
                umma_commit(drain);
                mbar_wait(drain, 0, 0, UM_WAIT_CYCLES);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == TS_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

// ---- QuantLinear on the tensor cores: fp16 rows + one-group tables ----------
__global__ void k_ql_prep(const float *__restrict__ x, int64_t n4, __half *__restrict__ xp, int T,
                          int nt, int32_t *__restrict__ tab, int *err) {
    pdl_enter();
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        tab[0] = 0;                  // act_group: the one weight matrix
        tab[1] = 0;                  // act_begin: slot of token 0
        tab[2] = T;                  // act_n
        tab[3] = 1;                  // n_act
        tab[4] = 0;                  // tile_prefix[0]
        tab[5] = (T + nt - 1) / nt;  // tile_prefix[1]
    }
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
        const float2 fa = __half22float2(a), fb = __half22float2(b);
        bad |= (isfinite(v.x) && !isfinite(fa.x)) || (isfinite(v.y) && !isfinite(fa.y)) ||
               (isfinite(v.z) && !isfinite(fb.x)) || (isfinite(v.w) && !isfinite(fb.y));
        reinterpret_cast<__half2 *>(xp)[2 * i] = a;
        reinterpret_cast<__half2 *>(xp)[2 * i + 1] = b;
    }
    if (bad) atomicOr(err, QG_FLAG_RANGE);
}

int launch_ql_prep(const float *x, int T, int K, int nt, __half *xp, int32_t *tab, int *err,
                   cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t n4 = (int64_t)T * K / 4;
    int64_t blocks = (n4 + 255) / 256;
    const int64_t cap = (int64_t)num_sms(dev) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    QG_CUDA(launch_pdl(k_ql_prep, dim3((unsigned)blocks), dim3(256), 0, s, 1, x, n4, xp, T, nt,
                       tab, err));
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

// ---- expert parallelism: regroup received rows by local expert ------------
// Received rows arrive source-rank-major (each source's rows sorted by local
// expert).  Segment i = (source, local expert) starts at seg_recv_off[i] in
// the received buffer and at seg_grp_off[i] in the expert-major buffer.  One
// warp per row: find its segment, copy the 2H-byte row, record the mapping
// back (GEMM2 writes its output rows in received order through it).
__global__ void k_ep_regroup(const __half *__restrict__ recv, int R, int H,
                             const int32_t *__restrict__ seg_recv_off,
                             const int32_t *__restrict__ seg_grp_off, int nseg,
                             __half *__restrict__ grouped, int32_t *__restrict__ grp2recv) {
    const int wg = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int r = wg; r < R; r += nw) {
        int lo = 0, hi = nseg - 1;  // last segment with seg_recv_off <= r
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (seg_recv_off[mid] <= r) lo = mid; else hi = mid - 1;
        }
        const int g = seg_grp_off[lo] + (r - seg_recv_off[lo]);
        if (lane == 0) grp2recv[g] = r;
        const uint4 *src = reinterpret_cast<const uint4 *>(recv + (size_t)r * H);
        uint4 *dst = reinterpret_cast<uint4 *>(grouped + (size_t)g * H);
        for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
    }
}

int launch_ep_regroup(const __half *recv, int R, int H, const int32_t *seg_recv_off,
                      const int32_t *seg_grp_off, int nseg, __half *grouped, int32_t *grp2recv,
                      cudaStream_t s) {
    if (R <= 0) return QGMOE_OK;
    int dev = 0;
    cudaGetDevice(&dev);
    int blocks = (R + 7) / 8;
    const int cap = num_sms(dev) * 8;
    if (blocks > cap) blocks = cap;
    k_ep_regroup<<<blocks, 256, 0, s>>>(recv, R, H, seg_recv_off, seg_grp_off, nseg, grouped,
                                        grp2recv);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

// ---- weight repack into UMMA tiles --------------------------------------
// One thread per (e, rt, kb, row).  Tile row `row` comes from source row
//   interleave (SWIGLU): row < 64 -> rt*64 + row (gate),
//                        row >= 64 -> up_offset + rt*64 + row - 64 (up);
//   plain (STORE):       rt*128 + row.
// Output: one RawTile block per (e, rt, kb), codes chunk-major then the
// rows' two group scales.  int8 codes are stored biased (q + 128) for the
// converter's byte splice; int4 words are reordered so element 2j sits in
// bits [4j, 4j+4) and element 2j+1 in bits [16+4j, 20+4j): one shift+mask
// per fp16 pair.
__global__ void k_repack(const uint8_t *__restrict__ q, const __half *__restrict__ sc, int bits,
                         int E, int rows_per_e, int K, int RT, int interleave, int up_offset,
                         uint8_t *__restrict__ qo) {
    const int KB = K / UM_BK;
    const int64_t n = (int64_t)E * RT * KB * UM_M;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int row = (int)(i % UM_M);
    int64_t rest = i / UM_M;
    const int kb = (int)(rest % KB);
    rest /= KB;
    const int rt = (int)(rest % RT);
    const int e = (int)(rest / RT);
    int64_t srow;
    if (interleave)
        srow = (int64_t)e * rows_per_e + (row < 64 ? rt * 64 + row : up_offset + rt * 64 + row - 64);
    else
        srow = (int64_t)e * rows_per_e + rt * UM_M + row;
    const int row_bytes = bits == 8 ? K : K / 2;
    const int blk_bytes = bits == 8 ? UM_BK : UM_BK / 2;
    const int code_bytes = UM_M * blk_bytes;
    const int cb = blk_bytes / 4;  // bytes of one 16-code chunk
    const uint8_t *s = q + srow * row_bytes + (int64_t)kb * blk_bytes;
    const int64_t tile = ((int64_t)e * RT + rt) * KB + kb;
    uint8_t *d = qo + tile * (code_bytes + UM_M * 4);
    for (int c = 0; c < 4; c++) {
        uint8_t *dc = d + ((int64_t)c * UM_M + row) * cb;  // [chunk][row][cb]
        const uint8_t *sc4 = s + c * cb;
        if (bits == 8) {
            uint4 v = *reinterpret_cast<const uint4 *>(sc4);
            v.x ^= 0x80808080u;
            v.y ^= 0x80808080u;
            v.z ^= 0x80808080u;
            v.w ^= 0x80808080u;
            *reinterpret_cast<uint4 *>(dc) = v;
        } else {
            for (int w = 0; w < 2; w++) {
                const uint32_t src = *reinterpret_cast<const uint32_t *>(sc4 + 4 * w);
                uint32_t out = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t byte = (src >> (8 * j)) & 0xFFu;
                    out |= (byte >> 4) << (4 * j);          // element 2j
                    out |= (byte & 0xFu) << (16 + 4 * j);   // element 2j+1
                }
                *reinterpret_cast<uint32_t *>(dc + 4 * w) = out;
            }
        }
    }
    const __half *ss = sc + srow * (K / QG_GROUP) + kb * 2;
    reinterpret_cast<__half2 *>(d + code_bytes)[row] = __halves2half2(ss[0], ss[1]);
}

// ---- host side --------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D fp16 [rows, cols] tensor with row pitch `ld` elements, box 64 cols x
// box_rows rows, 128B swizzle.
int encode_act_map(void *map_out, const __half *ptr, int rows, int cols, int ld, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(QGMOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16 || cols > ld)
        return set_error(QGMOE_ERR_INVALID_ARG, "activation buffer not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {UM_BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(reinterpret_cast<CUtensorMap *>(map_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<__half *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(QGMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QGMOE_OK;
}

// 2-D float32 [rows, cols] row-major tensor (row pitch = cols), box 32 cols
// (one 128-byte line) x box_rows rows, 128B swizzle, zero fill beyond the
// edges.  Returns false (and leaves the error state alone) when the driver
// entry point is missing or the layout does not suit TMA, so the caller can
// take a path without tensor maps.
bool encode_f32_map(void *map_out, const float *ptr, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || cols % 32 || rows <= 0 ||
        box_rows <= 0 || box_rows > 256)
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(reinterpret_cast<CUtensorMap *>(map_out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
              const_cast<float *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t packed_bytes(int bits, int E, int rows_per_e, int K) {
    // rows_per_e / 128 row tiles x K / 64 k blocks per expert
    const size_t tiles = (size_t)E * (rows_per_e / UM_M) * (K / UM_BK);
    return tiles * (size_t)(bits == 8 ? RawTile<8>::BYTES : RawTile<4>::BYTES);
}

int launch_repack(const uint8_t *q, const __half *sc, int bits, int E, int rows_per_e, int K,
                  int RT, int interleave, int up_offset, uint8_t *qo, cudaStream_t s) {
    const int64_t n = (int64_t)E * RT * (K / UM_BK) * UM_M;
    if (n == 0) return QGMOE_OK;
    k_repack<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(q, sc, bits, E, rows_per_e, K, RT,
                                                          interleave, up_offset, qo);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

template <int BITS, bool SWIGLU, int NT>
static int launch_umma_t(const void *tmap, const UmmaArgs &a, int grid, cudaStream_t s) {
    // NT = 256: A in shared memory; NT = 64 / 16: A in TMEM.
    int smem, threads;
    void (*kern)(const CUtensorMap, const UmmaArgs);
    if constexpr (NT != 256) {
        smem = TsCfg<BITS, NT>::SMEM;
        threads = TS_THREADS;
        kern = k_umma_ts<BITS, SWIGLU, NT>;
    } else {
        smem = UmCfg<BITS, NT>::SMEM;
        threads = UM_THREADS;
        kern = k_umma<BITS, SWIGLU, NT>;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    static bool done[64] = {false};
    if (dev < 64 && !done[dev]) {
        QG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        done[dev] = true;
    }
    int g = num_sms(dev);
    if (grid < g) g = grid;
    QG_CUDA(launch_pdl(kern, dim3(g), dim3(threads), smem, s, 1,
                       *reinterpret_cast<const CUtensorMap *>(tmap), a));
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_umma(int bits, bool swiglu, const void *tmap, const UmmaLaunch &l, cudaStream_t s) {
    UmmaArgs a{};
    a.wq = l.wq;
    a.RT = l.RT;
    a.KB = l.KB;
    a.act_group = l.act_group;
    a.act_begin = l.act_begin;
    a.act_n = l.act_n;
    a.n_act = l.n_act;
    a.tile_prefix = l.tile_prefix;
    a.out = l.out;
    a.out_stride = l.out_stride;
    a.out_map = l.out_map;
    a.out_peers = l.out_peers;
    a.out_peer_off = l.out_peer_off;
    a.out32 = l.out32;
    a.err = l.err;
    if (l.grid <= 0) return QGMOE_OK;
    const int nt = l.tile_tokens == 128 || l.tile_tokens == 64 || l.tile_tokens == 16
                       ? l.tile_tokens : 256;
#define QG_UMMA_CASE(B, SW)                                                        \
    if (bits == B && swiglu == SW)                                                 \
        return nt == 256   ? launch_umma_t<B, SW, 256>(tmap, a, l.grid, s)         \
               : nt == 128 ? launch_umma_t<B, SW, 128>(tmap, a, l.grid, s)         \
               : nt == 64  ? launch_umma_t<B, SW, 64>(tmap, a, l.grid, s)          \
                           : launch_umma_t<B, SW, 16>(tmap, a, l.grid, s);
    QG_UMMA_CASE(8, true)
    QG_UMMA_CASE(8, false)
    QG_UMMA_CASE(4, true)
    QG_UMMA_CASE(4, false)
#undef QG_UMMA_CASE
    return set_error(QGMOE_ERR_UNSUPPORTED, "tensor path needs int8/int4 weights");
}

}  // namespace qg
