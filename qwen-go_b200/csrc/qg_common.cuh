// Shared definitions for the qgmoe CUDA library (sm_100a only).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qgmoe.h"

#define QG_GROUP 32        // quantGroup, model/moe.go:124
#define QG_MAX_TOPK 32     // router keeps the k winners in one warp
#define QG_MAX_EXPERTS 1024
#define QG_ROUTE_THREADS 256

namespace qg {

// Tokens per top-k / scatter CTA of the router (one warp per token): the
// router's per-CTA expert histograms have ceil(T / QG_TOPK_TOK) rows.
constexpr int QG_TOPK_TOK = 32;

// Records a failure detail for qgmoe_last_error() and returns `code`.
int set_error(int code, const char *fmt, ...);

#define QG_CUDA(call)                                                                 \
    do {                                                                              \
        cudaError_t e_ = (call);                                                      \
        if (e_ != cudaSuccess)                                                        \
            return ::qg::set_error(QGMOE_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__, \
                                   #call, cudaGetErrorString(e_));                    \
    } while (0)

// Programmatic dependent launch.  The forward's kernels are launched with
// launch_pdl: the next kernel of the stream may be scheduled while this one
// is still running, and each kernel opens with pdl_enter(), which lets its
// own successor be scheduled and then waits until every earlier kernel of
// the stream has completed and its writes are visible.  Nothing is read or
// written before that wait, so the only effect is that launch latency and
// CTA start-up overlap the previous kernel's tail.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// The two halves of pdl_enter, for kernels with set-up that touches no
// global memory an earlier kernel writes (barriers, TMEM allocation): that
// set-up runs between them, under the previous kernel's tail.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, int cluster_z, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    int n = 1;
    if (cluster_z > 1) {
        at[1].id = cudaLaunchAttributeClusterDimension;
        at[1].val.clusterDim.x = 1;
        at[1].val.clusterDim.y = 1;
        at[1].val.clusterDim.z = cluster_z;
        n = 2;
    }
    cfg.attrs = at;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Device-side error word bits (an int in device memory, read back by the host).
enum : int {
    QG_FLAG_BAD_EXPERT = 1,   // router produced an expert id out of [0, E)
    QG_FLAG_BAD_SLOT = 2,     // dispatch slot out of range
    QG_FLAG_BAD_GROUP = 4,    // expert kernel saw an active group out of range
    QG_FLAG_TIMEOUT = 8,      // a bounded mbarrier wait in the tensor-core kernel ran out
    QG_FLAG_RANGE = 16,       // a finite activation beyond fp16 range reached the tensor-core path
};

// One stacked weight family (e.g. all experts' gate_up) in device memory.
// bits 32: w32 [G*rows, K]; bits 8: q [G*rows, K] int8; bits 4: q [G*rows, K/2].
// Scales: [G*rows, K/32] fp16.
struct WeightSet {
    int bits;
    int rows;  // output rows per group (expert)
    int K;     // input features
    const float *w32;
    const uint8_t *q;
    const __half *s;
};

// Per-call routing state produced by the router/dispatch kernel.
struct RouteState {
    int32_t *topk_idx;   // [T*k]
    float *topk_w;       // [T*k]
    float *shared_w;     // [T]   sigmoid(sharedGate . x)
    int32_t *counts;     // [E]   zero between calls
    int32_t *done_ctr;   // [1]   zero between calls
    int32_t *pair_slot;  // [T*k] slot of pair (t, r)
    int32_t *slot_token; // [T*k + T] token of each slot (shared slots appended)
    int32_t *act_group;  // [E+1] active groups, ascending expert id, shared last
    int32_t *act_begin;  // [E+1] first slot of the group
    int32_t *act_n;      // [E+1] tokens in the group
    int32_t *n_act;      // [1]
    int32_t *tile_prefix;  // [E+2] tile_tokens-token tiles before each routed group, total last
    int32_t *n_act_routed; // [1] routed groups in the active list (the shared one excluded)
    int32_t *shared_act;   // [6] the shared expert as a one-group list: group 0, first
                           //     slot T*k, T tokens, count 1, tile prefix {0, tiles}
    int tile_tokens;       // tile granularity of tile_prefix (256 or 64; 0 = 256)
    float *logits;         // [splits][T][E+1] split-K partial router logits
    int32_t *hist;         // [ceil(T/32)][E] expert histogram of each top-k CTA
    int32_t *expert_off;   // [E] first slot of each dispatch key
    // Expert parallelism over ep_world ranks (1 = off): slots are sorted by
    // the dispatch key = owner rank * (E / W) + local index of the expert,
    // i.e. by destination rank, then local expert.  ep_slot [E] (device)
    // holds the key of each expert; null = round-robin (expert e on rank
    // e % W, local index e / W).
    int ep_world;
    const int32_t *ep_slot;
};

__device__ __forceinline__ int dispatch_key(int e, int E, int W, const int32_t *slot) {
    if (slot) return slot[e];
    return W > 1 ? (e % W) * (E / W) + e / W : e;
}

// Expert-parallel exchange over NVLink peer memory (qg_peer.cu): every
// rank's exchange region, mapped into this process, and its layout.
constexpr int PX_CNT = 0, PX_DATA = 1, PX_BACK = 2;  // flag kinds
constexpr int PX_FLAG_BLOCK = 256;                   // bytes per flag kind (W <= 32)
constexpr int PX_MAX_WORLD = 32;
struct PxArgs {
    uint8_t *const *bases;  // device array [W]: every rank's region as mapped here
    int W, me, G, H, k, T;
    int64_t recv_cap;       // rows of a region's recv buffer
    size_t off_epoch, off_ticket, off_inbox, off_recv, off_back;
    long long wait;         // clock cycles a wait on a peer's flag may take (<= 0: default)
};
struct PxTables {  // this rank's grouped-row tables (device)
    int32_t *act_group, *act_begin, *act_n, *n_act, *tile_prefix, *out_map, *n_rows;
};
int launch_px_counts(const PxArgs &a, const int32_t *expert_off, int *err, cudaStream_t s);
int launch_px_send(const PxArgs &a, const float *x, const int32_t *expert_off,
                   const int32_t *slot_token, int *err, cudaStream_t s);
int launch_px_tables(const PxArgs &a, int tile_tokens, const PxTables &t, int *err,
                     cudaStream_t s);
int launch_px_signal(const PxArgs &a, cudaStream_t s);
int launch_px_wait(const PxArgs &a, int *err, cudaStream_t s);

// One launch of the tensor-core grouped GEMM (qg_umma.cu).
struct UmmaLaunch {
    const uint8_t *wq;          // packed tiles: per (expert, row tile, k block) the codes
                                // then the rows' fp16 scales, contiguous
    int RT, KB;                 // row tiles per expert, 64-wide K blocks
    const int32_t *act_group, *act_begin, *act_n, *n_act, *tile_prefix;
    __half *out;                // GEMM1: h [slots, I]; GEMM2: d [slots, H] (fp16)
    int out_stride;
    const int32_t *out_map;     // GEMM2 only: output row of each slot (null = same slot)
    // GEMM2 only, expert parallelism over peer memory: out_map holds
    // (rank << 24 | row) and row goes to out_peers[rank] + out_peer_off
    uint8_t *const *out_peers;
    size_t out_peer_off;
    float *out32;               // GEMM2 only: f32 output rows instead of fp16 (QuantLinear)
    int *err;
    int grid;                   // upper bound of work units
    int tile_tokens;            // max tokens per work unit: 256 (prefill) or 64 (decode)
};

// Arguments of the grouped expert kernels.
struct ExpertArgs {
    WeightSet routed;     // gate_up (GATEUP) or down (DOWN) of the routed experts
    WeightSet shared;     // same for the shared expert (group id == n_experts)
    int n_experts;
    int has_shared;
    // Active-group list from the dispatch kernel.  When n_act is null the
    // kernel runs one group: the `shared` weight set over single_n rows
    // starting at slot 0 (the plain QuantLinear forward).
    const int32_t *act_group, *act_begin, *act_n, *n_act;
    int single_n;
    const int32_t *slot_token;  // GATEUP: input row of a slot; DOWN: unused
    const float *in;            // GATEUP: x [T, H]; DOWN: h [slots, in_stride]
    int in_stride;
    float *out;                 // GATEUP: h [slots, out_stride]; DOWN: d [slots, out_stride]
    int out_stride;
    int *err;
};

// The decode forward (qg_decode.cu): batches of up to FD_MAX_T tokens in one
// persistent kernel, one CTA per SM.
constexpr int FD_MAX_T = 8;
constexpr int FD_MAX_E = 256;  // experts the decode kernel routes (ceil(E/32) <= 8)
// The batch's exact routing, published by the kernel's routing warps.
struct DecRoute {
    int sel[FD_MAX_T][QG_MAX_TOPK];   // experts in rank order
    float w[FD_MAX_T][QG_MAX_TOPK];   // their renormalised weights
    float sg[FD_MAX_T];               // shared-expert gate
    int slot[FD_MAX_T][QG_MAX_TOPK];  // the down row holding (token, rank)
    int miss[FD_MAX_T];               // a selected expert was not a candidate
};
struct DecodeArgs {
    const float *x;                   // [T, H]
    int T, H, E, Ep, k, mode, has_shared, I, Is;
    const float *router;              // [E, H] float32 router rows
    const float *shared_gate;         // [H] or null
    WeightSet gu, dn, sgu, sdn;       // routed and shared expert weights (one format)
    // int8/int4: the tensor path's packed 128-row x 64-code tiles of the same
    // weights (qg_umma.cu k_repack), streamed instead of the row-major codes
    const uint8_t *gu_pq, *dn_pq, *sgu_pq, *sdn_pq;
    int kbi_gu, kbi_dn, kbi_sdn;      // 64-code k blocks per streamed item
    unsigned *tdone;                  // [2][FD_MAX_T * QG_MAX_TOPK + 1] gate_up tiles done per task
    float *approx;                    // [T, Ep] approximate logits (speculation)
    float *logits;                    // [T, Ep] logits in the reference's serial order
    unsigned char *hbuf;              // h rows, [dec_slots(k), hrow bytes]
    int hrow;
    float *dbuf;                      // down rows, [dec_slots(k), H]
    float *out;                       // [T, H]
    int32_t *topk_idx;                // [T, k] routing outputs
    float *topk_w, *shared_w;
    DecRoute *route;
    unsigned long long *bar;          // grid barrier arrivals (never reset)
    unsigned long long *flags;        // [gridDim.x] logits-done, then [FD_MAX_T] routed
    int *err;
    long long wait;                   // cycles a wait on other CTAs may take (<= 0: default)
    int speculate;                    // stream the approximate top-k's experts early
    // shared-memory plan (bytes from the start of dynamic shared memory)
    int nrc;                          // router rows per CTA
    int xstride;                      // float32 token rows (floats)
    int x16tok, h16tok;               // fp16 operand rows per token (bytes, tensor-core path)
    int ns;                           // weight ring stages
    int hsstride;                     // staged float32 h rows (floats, CUDA-core path)
    int hwin;                         // down-phase tasks whose h rows are staged at once
    int stage_bytes;                  // one weight ring stage
    int off_xs, off_x16, off_hs, off_ring, off_xch, off_tok, off_lrow;
    int smem;                         // total dynamic bytes
};
// h / d rows of the decode buffers: pairs of the speculative phase, the
// shared expert's tokens, pairs computed after exact routing.
__host__ __device__ inline int dec_slots(int k) { return 2 * FD_MAX_T * k + FD_MAX_T; }
// Fills a's shared-memory plan for T tokens on a device with `sms` SMs;
// false when the batch does not fit the decode kernel.
bool decode_plan(DecodeArgs &a, int bits, int sms);
// Bytes of one h row of the decode buffers for a layer's widest expert.
int decode_hrow_bytes(int bits, int I, int Is);
int launch_decode(int bits, const DecodeArgs &a, cudaStream_t s);

// Launch helpers implemented in the .cu files.
// The router: logits in the reference's serial order, exact softmax, top-k
// and weights, dispatch.  x, router and shared_gate are float32 device
// arrays.  With xp set (the tensor path), xh [T, H] receives fp16(x) (a
// finite value beyond fp16 range raises QG_FLAG_RANGE) and xp [slots, H] the
// fp16 row of every slot.
int launch_route(const float *x, int T, int H, int E, int k, int mode, const float *router,
                 const float *shared_gate, int has_shared, RouteState st, __half *xh, __half *xp,
                 int *err, cudaStream_t s);

int launch_expert(bool gateup, const ExpertArgs &a, int max_items, cudaStream_t s);
// d rows are f32 (CUDA-core path) or fp16 (tensor-core path).
int launch_combine_f16(const __half *d, int H, int T, int k, const int32_t *pair_slot,
                       const float *topk_w, const float *shared_w, int has_shared, float *out,
                       cudaStream_t s);
// Routed rows fp16 (tensor path), shared-expert rows f32 (its CUDA-core GEMV).
int launch_combine_mixed(const __half *d, const float *ds, int H, int T, int k,
                         const int32_t *pair_slot, const float *topk_w, const float *shared_w,
                         float *out, cudaStream_t s);
int launch_combine(const float *d, int H, int T, int k, const int32_t *pair_slot,
                   const float *topk_w, const float *shared_w, int has_shared, float *out,
                   cudaStream_t s);
int launch_quantize(int bits, int O, int I, const float *w, uint8_t *q, float *s32,
                    __half *s16, cudaStream_t s);
int launch_dequantize(int bits, int O, int I, const uint8_t *q, const __half *scale,
                      const float *w32, float *w, cudaStream_t s);
// The router as float32 rows from bf16 bits (16) or codes + scales (8 / 4;
// scale_f32: float scales, else fp16), as the reference forms them.
int launch_router_rows(int bits, int E, int H, const uint8_t *q, const void *scale, int scale_f32,
                       float *w, cudaStream_t s);
int launch_f32_to_f16(const float *in, __half *out, int64_t n, cudaStream_t s);
int launch_randn(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, float stdv,
                 float *out, cudaStream_t s);
int num_sms(int device);
int encode_act_map(void *map_out, const __half *ptr, int rows, int cols, int ld, int box_rows);
bool encode_f32_map(void *map_out, const float *ptr, int rows, int cols, int box_rows);
int launch_repack(const uint8_t *q, const __half *sc, int bits, int E, int rows_per_e, int K,
                  int RT, int interleave, int up_offset, uint8_t *qo, cudaStream_t s);
// Bytes of the packed tensor-core copy of a weight set (codes + scales).
size_t packed_bytes(int bits, int E, int rows_per_e, int K);
int launch_umma(int bits, bool swiglu, const void *tmap, const UmmaLaunch &l, cudaStream_t s);
// QuantLinear on the tensor cores: x [T, K] f32 -> fp16 rows xp (a finite
// value beyond fp16 range raises QG_FLAG_RANGE) and the one-group work
// tables tab = {group 0, first slot 0, T slots, 1 group, tile prefix 0,
// ceil(T / nt)}.
int launch_ql_prep(const float *x, int T, int K, int nt, __half *xp, int32_t *tab, int *err,
                   cudaStream_t s);
// Expert parallelism: copies received rows into local-expert-major order.
int launch_ep_regroup(const __half *recv, int R, int H, const int32_t *seg_recv_off,
                      const int32_t *seg_grp_off, int nseg, __half *grouped, int32_t *grp2recv,
                      cudaStream_t s);

}  // namespace qg
