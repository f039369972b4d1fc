/*
 * qgmoe.h -- C ABI of the B200 (sm_100a) Mixture-of-Experts layer and
 * group-32 QuantLinear matmuls for qwen-go.
 *
 * Plain C: pointers, sizes and integer status codes only.  Every entry point
 * returns 0 (QGMOE_OK) or a negative QGMOE_ERR_* code; none aborts or exits.
 * qgmoe_strerror() and qgmoe_last_error() give the text.
 *
 * Seams of the reference this library replaces (jackkey143084/qwen-go):
 *   mixer.forward(x []float32) []float32        model/model.go:373-375, called
 *                                               per token at model/model.go:512
 *   moeMLP{...} / moeMLP.forward                model/moe.go:10-25, 41-99
 *   quantLinear{...} / .forward / .dequantize   model/moe.go:126-162
 *   quantizeInt8 / quantizeInt4                 model/moe.go:165-217, 233-239
 *   proj(x, T, l, q, out) over a quantLinear     model/model.go:196-205
 *
 * Threading: a handle is not re-entrant; callers serialise calls on one
 * handle (the Go shim holds a mutex).  Each call sets its CUDA device first,
 * so the calling OS thread may change between calls (cgo).
 */
#ifndef QGMOE_H
#define QGMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define QGMOE_OK 0
#define QGMOE_ERR_INVALID_ARG (-1) /* bad shape, null pointer, unsupported combo */
#define QGMOE_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define QGMOE_ERR_NCCL (-3)        /* reserved for the expert-parallel path */
#define QGMOE_ERR_TIMEOUT (-4)     /* a bounded device wait ran out */
#define QGMOE_ERR_DEVICE_FLAG (-5) /* a kernel's bounds check fired (see last_error) */
#define QGMOE_ERR_UNSUPPORTED (-6) /* valid request this build does not implement */
#define QGMOE_ERR_NO_DEVICE (-7)   /* no CUDA device / not an sm_100 device */

/* ---- enums ------------------------------------------------------------ */
/* Router selection.  TOPK: the documented semantics (softmax then the k
 * largest probabilities, descending, ties to the lower expert index) -- the
 * insertion sort of model/moe.go:49-53 run over all experts.  PREFIX: the
 * literal loop bound of model/moe.go:49 (`i < m.topK`), which orders only
 * experts 0..k-1. */
#define QGMOE_ROUTER_TOPK 0
#define QGMOE_ROUTER_PREFIX 1

/* dtype of the host/device scale arrays handed to create(); the library
 * always stores fp16 scales on the device (RNE rounding from f32). */
#define QGMOE_SCALE_F16 0 /* uint16_t IEEE half bits */
#define QGMOE_SCALE_F32 1 /* float, as quantizeInt8/Int4 emit (moe.go:164) */

/* ---- MoE layer -------------------------------------------------------- */
typedef struct qgmoe qgmoe_t;

/* Weights of one moeMLP (model/moe.go:10-25).  Layouts are the reference's:
 * rows are (out, in), row-major.  A weight group's format is one of
 *   32  float32 rows (gateUpW / downW, linear.w);
 *   16  raw bf16 rows (gateUpRaw / downRaw, linear.raw; model/moe.go:14-15,
 *       102-113, model/model.go:167-176): the *_q pointers hold the bf16 bit
 *       patterns, 2 bytes per element, no scales;
 *   8/4 quantLinear codes (int8 [O, I] two's-complement bytes, or int4
 *       packed [O, I/2] with element 2c in the high nibble of byte c and
 *       element 2c+1 in the low nibble, each stored as code + 8,
 *       model/moe.go:190-217) plus group-32 scales [O, I/32] (scale_dtype).
 * bits is the routed experts' format; shared_bits the shared expert's (0 =
 * same as bits) and router_bits the router's (0 or 32 = float32 `router`).
 * The reference mixes them: a quantised router (routerQuant, model/moe.go:16,
 * installed by model/load.go:651-652) and quantised shared-expert linears
 * beside bf16 or f32 routed experts -- what cmd/qwen-quant writes for an MoE
 * model, which quantises only the shared-expert projections
 * (cmd/qwen-quant/main.go:61-65).  The router is turned into float32 rows at
 * create time exactly as the reference's dequantize / bf16f32 do
 * (model/moe.go:134-157, model/model.go:113-115; f32 scales used as given,
 * the product rounded to nearest), so routing stays bit-exact.  Expert and
 * shared-expert scales are stored as fp16 on the device (f32 scales rounded
 * to nearest even).  sharedGate stays float32.
 * All pointers are either host pointers (weights_on_device = 0) or device
 * pointers on `device` (1); create() copies them, the caller keeps
 * ownership of its buffers. */
typedef struct qgmoe_desc {
    int32_t n_embed;      /* H   moeMLP.nEmbed */
    int32_t n_experts;    /* E   moeMLP.nExperts */
    int32_t top_k;        /* k   moeMLP.topK (1..32, <= E) */
    int32_t n_moe_mlp;    /* I   moeMLP.nMoeMlp */
    int32_t n_shared_mlp; /* Is  shared expert width, 0 = none */
    int32_t bits;         /* routed experts: 32, 16, 8 or 4 */
    int32_t router_mode;  /* QGMOE_ROUTER_* */
    int32_t scale_dtype;  /* QGMOE_SCALE_* for the *_scale arrays */
    int32_t weights_on_device;
    int32_t device;       /* CUDA ordinal that owns the handle */
    const float *router;        /* [E, H]   mlp.gate.weight (router_bits 0 / 32) */
    const float *shared_gate;   /* [H]      mlp.shared_expert_gate.weight (Is > 0) */
    /* format 32 */
    const float *gate_up;       /* [E, 2I, H] mlp.experts.gate_up_proj (gate rows 0..I-1) */
    const float *down;          /* [E, H, I]  mlp.experts.down_proj */
    const float *shared_gate_proj; /* [Is, H] */
    const float *shared_up_proj;   /* [Is, H] */
    const float *shared_down_proj; /* [H, Is] */
    /* formats 16 / 8 / 4: bf16 bits, or codes and scales of the same
     * tensors quantised row-wise */
    const uint8_t *gate_up_q;
    const void *gate_up_scale;
    const uint8_t *down_q;
    const void *down_scale;
    const uint8_t *shared_gate_q;
    const void *shared_gate_scale;
    const uint8_t *shared_up_q;
    const void *shared_up_scale;
    const uint8_t *shared_down_q;
    const void *shared_down_scale;
    /* Expert parallelism (0 or 1 = off).  With ep_world = W > 1 each rank
     * owns E/W experts; the expert stacks above then hold only this rank's
     * experts, in local order, while the router stays [E, H].  Forward then
     * goes through the qgmoe_ep_* calls below. */
    int32_t ep_world;
    int32_t ep_rank;
    /* Placement (host array [E], may be NULL): ep_slot[e] = owner rank *
     * (E/W) + local index of expert e, a permutation of 0..E-1 identical on
     * every rank (e.g. balanced by measured expert load).  NULL = round-robin:
     * expert e on rank e % W, local index e / W. */
    const int32_t *ep_slot;
    /* Per-group formats (see above).  router_q: bf16 bits [E, H] (16) or
     * codes (8 / 4) of mlp.gate, router_scale its group-32 scales. */
    int32_t router_bits;
    const void *router_q;
    const void *router_scale;
    int32_t shared_bits;
} qgmoe_desc;

/* Uploads the weights (device copies owned by the handle). */
int qgmoe_create(const qgmoe_desc *desc, qgmoe_t **out);
int qgmoe_destroy(qgmoe_t *h);

/* moeMLP.forward over T independent tokens (T = 1 is mixer.forward; T > 1
 * is the batched form decodeLayers hands over).  HOST pointers; blocking.
 * x [T, H] f32 -> out [T, H] f32.  sel_idx [T, k] int32 and sel_w [T, k]
 * f32 (the selected experts in routing order and their renormalised
 * weights, model/moe.go:53-63) are optional (NULL to skip). */
int qgmoe_forward(qgmoe_t *h, const float *x, int32_t T, float *out, int32_t *sel_idx,
                  float *sel_w);

/* Same on DEVICE pointers, enqueued on `stream` (a cudaStream_t; NULL = the
 * handle's own stream).  Returns after enqueueing; device-side bounds flags
 * are reported by qgmoe_sync(). */
int qgmoe_forward_device(qgmoe_t *h, const float *x, int32_t T, float *out, int32_t *sel_idx,
                         float *sel_w, void *stream);

/* ---- expert-parallel forward --------------------------------------------
 * One process (handle) per GPU; the host moves rows between ranks, e.g. with
 * NCCL all-to-all.  No reference counterpart: qwen-go is one process with no
 * multi-GPU code; the per-token math is still moeMLP.forward's.
 *   1. qgmoe_ep_dispatch: route this rank's T tokens over all E experts and
 *      write the fp16 activation rows of its T*k (token, rank) pairs to
 *      send_rows [T*k, H], sorted by owner rank, then local expert.
 *   2. qgmoe_ep_send_counts: blocking; counts [W][E/W] of those rows.
 *   3. host: exchange counts, then rows (rank r gets its block of each peer).
 *   4. qgmoe_ep_experts: this rank's experts on the R received rows
 *      (recv_rows [R, H] fp16, source-rank-major, each source's rows sorted
 *      by local expert; recv_counts [W][E/W] host array) -> out_rows [R, H]
 *      fp16 in the same order (SwiGLU expert outputs, model/moe.go:64-81).
 *   5. host: send out_rows back (the reverse exchange).
 *   6. qgmoe_ep_combine: back_rows [T*k, H] fp16 in send order -> out [T, H]
 *      f32, the rank-ordered weighted sum of model/moe.go:82-85; sel_idx /
 *      sel_w optional as in qgmoe_forward.
 * All pointers except recv_counts / counts are DEVICE pointers; calls are
 * enqueued on `stream` (NULL = the handle's stream). */
int qgmoe_ep_dispatch(qgmoe_t *h, const float *x, int32_t T, void *send_rows, void *stream);
int qgmoe_ep_send_counts(qgmoe_t *h, int32_t *counts, void *stream);
int qgmoe_ep_experts(qgmoe_t *h, const void *recv_rows, int32_t R, const int32_t *recv_counts,
                     void *out_rows, void *stream);
int qgmoe_ep_combine(qgmoe_t *h, const void *back_rows, int32_t T, float *out, int32_t *sel_idx,
                     float *sel_w, void *stream);

/* ---- expert-parallel forward over NVLink peer memory ----------------------
 * The same expert-parallel layer with the row exchange done by the library's
 * own kernels through CUDA IPC mappings of every rank's exchange region: no
 * host synchronisation and no collective library in the data path (rows are
 * stored straight into their owner's grouped buffer; the down GEMM stores its
 * outputs straight into the source rank's buffer).  No reference counterpart
 * (qwen-go has no multi-GPU code).  Setup, collective over the W ranks:
 *   1. qgmoe_ep_px_setup: allocate this rank's region for up to max_tokens
 *      tokens per rank and forward; writes its IPC handle
 *      (QGMOE_IPC_HANDLE_BYTES bytes) to ipc_handle;
 *   2. the host gathers all W handles in rank order (e.g. all_gather);
 *   3. qgmoe_ep_px_connect: map the peers' regions.
 * Then every rank calls qgmoe_ep_px_forward once per step (each with its own
 * T <= max_tokens, T = 0 allowed): x [T, H] f32 -> out [T, H] f32, DEVICE
 * pointers, enqueued on `stream`.  Ranks wait for each other on the GPU
 * (bounded waits, ~2 s; a timeout is reported by qgmoe_sync).  Every rank
 * must take the same number of steps; destroy handles only after all ranks
 * finished their last step. */
#define QGMOE_IPC_HANDLE_BYTES 64
int qgmoe_ep_px_setup(qgmoe_t *h, int32_t max_tokens, void *ipc_handle);
int qgmoe_ep_px_connect(qgmoe_t *h, const void *ipc_handles);
int qgmoe_ep_px_forward(qgmoe_t *h, const float *x, int32_t T, float *out, void *stream);

/* Waits for `stream` (NULL = the handle's stream) and reports any
 * device-side bounds flag raised since the last check. */
int qgmoe_sync(qgmoe_t *h, void *stream);

/* Number of kernel launches the last forward enqueued (instrumentation). */
int qgmoe_last_launch_count(const qgmoe_t *h);

/* Expert-product path.  AUTO runs decode-sized batches (up to 8 tokens,
 * routed and shared experts in one format, at most 256 experts, the batch
 * within the kernel's shared memory) on the decode kernel: one persistent
 * launch over every SM (it expects the device to itself; a grid barrier
 * that waits about a second raises QGMOE_ERR_DEVICE_FLAG, flag 8).  Larger
 * batches run on the tcgen05 tensor-core grouped GEMMs whenever the layer
 * allows them (int8/int4 routed experts; H and I multiples of 128), except
 * for the smallest batches of a layer with a shared expert (T*k < 16), and
 * on the CUDA-core streaming GEMV otherwise.  CUDA_CORE / TENSOR force one
 * of the general paths (TENSOR returns QGMOE_ERR_UNSUPPORTED when the layer
 * does not allow it). */
/* CUDA graphs (default on): the second forward with the same T, x, out and
 * stream is captured into a graph and later identical calls replay it, which
 * removes the per-launch host cost of decode-sized calls.  Disabled while
 * stage timing is on.  enable = 0 turns graphs off and drops cached ones. */
int qgmoe_set_graphs(qgmoe_t *h, int32_t enable);

#define QGMOE_PATH_AUTO 0
#define QGMOE_PATH_CUDA_CORE 1
#define QGMOE_PATH_TENSOR 2
int qgmoe_set_path(qgmoe_t *h, int32_t mode);

/* Decode kernel speculation (default on): while the router logits are
 * summed in the reference's serial order, the experts of an approximate
 * top-k are streamed already; experts the exact routing picks that the
 * approximation missed are computed afterwards.  Results are identical
 * either way; enable = 0 computes every expert after the exact routing. */
int qgmoe_set_decode_speculation(qgmoe_t *h, int32_t enable);

/* How long a device-side wait on another CTA or another rank (the decode
 * kernel's grid barriers and routing flags, the expert-parallel exchange's
 * peer flags) spins before it gives up, in microseconds of SM clock; 0
 * restores the defaults (about 1 s, 2 s for peers).  A wait that gives up
 * raises device flag 8: the next qgmoe_sync / blocking forward returns
 * QGMOE_ERR_TIMEOUT and the outputs of that call are not valid; the handle
 * stays usable.  Waits on a CTA's own copies keep their defaults. */
int qgmoe_set_wait_limit(qgmoe_t *h, int64_t microseconds);

/* Per-stage device timing (instrumentation for benchmarks): when enabled,
 * every forward records CUDA events on its stream between consecutive
 * stages, without host syncs.  read_timing waits for those forwards, writes
 * up to n per-stage durations in milliseconds SUMMED over the forwards since
 * the previous read to ms, their count to *n_forwards, and returns the stage
 * count (or a negative status); stage_name gives stage i's name ("route",
 * "gate_up", ...). */
int qgmoe_set_timing(qgmoe_t *h, int32_t enable);
int qgmoe_read_timing(qgmoe_t *h, float *ms, int32_t n, int32_t *n_forwards);
const char *qgmoe_stage_name(const qgmoe_t *h, int32_t i);

/* ---- allocation-free router ---------------------------------------------
 * No counterpart in the reference: qwen-go runs on the CPU with Go's heap.
 * For callers that cannot call cudaMalloc -- a host runtime that owns every
 * device allocation itself, a stream-capture region in which allocation is
 * not permitted, or a serving loop whose memory budget is fixed at start-up
 * -- this runs the router step (logits, softmax, top-k and renormalised
 * weights: the kernels and the exact routing of qgmoe_forward's router) with
 * all of its scratch in one static device array of
 * QGMOE_ROUTE_STATIC_SCRATCH bytes, which every GPU that loads this library
 * holds until the process exits.  x [T, H] f32, router [E, H] f32 and the
 * outputs sel_idx / sel_w [T, k] are DEVICE pointers on the calling thread's
 * current device (x and router 16-byte aligned); the work is enqueued on
 * `stream` (a cudaStream_t, NULL = legacy default stream) and the call
 * returns.  flags (optional, a DEVICE int32) receives the call's device
 * error word once the work has run: 0, or 1 (an expert id out of range) / 2
 * (a dispatch slot out of range), which only a corrupted call can raise;
 * NaN or infinite activations are not errors -- they route as the reference
 * does (experts 0..k-1 with NaN weights).  A size whose scratch would not
 * fit the array is rejected with QGMOE_ERR_INVALID_ARG.  The first call on a
 * device loads the library's device code there; make that first call before
 * any stream capture.  All calls on a device share the array and it keeps
 * the previous call's contents (the counters are cleared by each call):
 * calls that overlap on the GPU race, so order them on one stream. */
#define QGMOE_ROUTE_STATIC_SCRATCH (8 << 20)
int qgmoe_route_static(const float *x, const float *router, int32_t T, int32_t H, int32_t E,
                       int32_t k, int32_t mode, int32_t *sel_idx, float *sel_w, int32_t *flags,
                       void *stream);

/* ---- on-disk quantised MoE layers --------------------------------------
 * The reference's quantised checkpoint convention (quant.json + safetensors
 * with <name>.qweight / <name>.scale, model/load.go:478-582) extended to the
 * stacked expert tensors its loader cannot read (model/load.go:419-449 only
 * takes them as f32/bf16), so a quantised layer goes from the file to the
 * device without an intermediate host copy.  Tensor names, with a caller
 * prefix such as "model.layers.3.mlp." (the reference's mlp.* names,
 * model/load.go:415-456):
 *   gate.weight                          F32 (or BF16) [E, H] router
 *   experts.gate_up_proj.qweight         I8/U8 [E, 2I, H]     int8 codes, or
 *                                        U8 [E, 2I, H/2]      int4 pairs
 *   experts.gate_up_proj.scale           F16/F32 [E, 2I, H/32]
 *   experts.down_proj.qweight / .scale   [E, H, I] or [E, H, I/2] / [E, H, I/32]
 *   shared_expert.gate_proj, .up_proj, .down_proj (.qweight / .scale; all
 *   three or none), [Is, H], [Is, H], [H, Is] as above
 *   shared_expert_gate.weight            F32 [1, H] or [H]    (with the shared expert)
 * int8 vs int4 follows from the code and scale shapes; every tensor must
 * have the same scale dtype.  Raw (unquantised) layers, as the reference
 * reads bf16 checkpoints: <base>.weight instead of .qweight / .scale, BF16
 * (bits 16) or F32 (bits 32) [E, 2I, H] / [E, H, I] / [Is, H] ...; then a
 * BF16 router or shared-expert gate is widened into a float32 copy the file
 * handle owns.  One format per layer.  Safetensors layout: u64
 * little-endian header size, JSON header {name: {dtype, shape,
 * data_offsets}}, data. */
typedef struct qgmoe_file qgmoe_file_t;
#define QGMOE_DT_F32 0
#define QGMOE_DT_F16 1
#define QGMOE_DT_BF16 2
#define QGMOE_DT_I8 3
#define QGMOE_DT_U8 4
#define QGMOE_DT_I32 5
#define QGMOE_DT_OTHER 6
/* Maps a safetensors file read-only and parses its header (host only; no
 * CUDA call). */
int qgmoe_file_open(const char *path, qgmoe_file_t **out);
int qgmoe_file_close(qgmoe_file_t *f);
/* One tensor: dtype (QGMOE_DT_*), rank (<= 8) and shape, its bytes inside
 * the mapping.  Any out pointer may be NULL.  INVALID_ARG if absent. */
int qgmoe_file_tensor(const qgmoe_file_t *f, const char *name, int32_t *dtype, int32_t *rank,
                      int64_t *shape, const void **data, int64_t *nbytes);
/* Fills desc for the layer at `prefix`: shapes, bits and scale dtype from
 * the tensors, host pointers into the mapping (weights_on_device = 0, no
 * expert parallelism); top_k, router_mode and device from the caller.  The
 * mapping must stay open until qgmoe_create has returned. */
int qgmoe_file_layer_desc(const qgmoe_file_t *f, const char *prefix, int32_t top_k,
                          int32_t router_mode, int32_t device, qgmoe_desc *desc);

/* ---- QuantLinear -------------------------------------------------------- */
typedef struct qgql qgql_t;

/* quantLinear{bits, outFeatures, inFeatures, qweight, scale}
 * (model/moe.go:126-132).  bits 8 or 4, or 32 for a plain f32 linear
 * (then q holds float32 rows and scale is ignored).  in_features % 32 == 0. */
int qgql_create(int32_t bits, int32_t out_features, int32_t in_features, const void *q,
                const void *scale, int32_t scale_dtype, int32_t weights_on_device,
                int32_t device, qgql_t **out);
int qgql_destroy(qgql_t *h);

/* proj(x, T, nil, q, out) / quantLinear.forward: y[T, out] = x[T, in] W^T
 * with the dequantisation fused into the weight load.  HOST pointers;
 * blocking; reports device error flags like qgql_sync.
 * Paths (qgql_set_path): AUTO and CUDA_CORE run the CUDA-core GEMV (f32
 * arithmetic, the reference's dequantise-then-dot within f32 rounding).
 * TENSOR (opt-in; int8 / int4 weights with out % 128 == 0 and in % 64 == 0,
 * 16-byte aligned x and y, else the GEMV) runs on the tensor cores: x
 * rounded to fp16, fp16 dequantised weights, f32 accumulation and f32 y, so
 * each output is within about 2^-10 * sum_k |w_k x_k| of the f32 result,
 * which for unit-scale activations over rows of 1024+ can exceed the 1e-3
 * element-wise bar of the GEMV path.  A finite activation beyond fp16 range
 * on the tensor path raises QGMOE_ERR_DEVICE_FLAG instead of producing
 * infinities.  The tensor path keeps per-handle workspace: calls of one
 * handle must not overlap on the GPU (order them on one stream). */
int qgql_forward(qgql_t *h, const float *x, int32_t T, float *y);
/* Same on DEVICE pointers, enqueued on `stream` (NULL = handle stream). */
int qgql_forward_device(qgql_t *h, const float *x, int32_t T, float *y, void *stream);
/* QGMOE_PATH_AUTO / _CUDA_CORE / _TENSOR (UNSUPPORTED when the shape or
 * bits exclude the tensor path). */
int qgql_set_path(qgql_t *h, int32_t mode);
/* Waits for `stream` (NULL = handle stream) and returns
 * QGMOE_ERR_DEVICE_FLAG (clearing the flag) if a kernel raised one. */
int qgql_sync(qgql_t *h, void *stream);
/* quantLinear.dequantize (model/moe.go:134-157) into w_dev [out, in] f32. */
int qgql_dequantize_device(qgql_t *h, float *w_dev, void *stream);

/* quantizeInt8 / quantizeInt4 (model/moe.go:165-217) on the GPU, bit-exact:
 * w_dev [out, in] f32 -> q_dev (int8 [out,in] or int4 [out,in/2] bytes),
 * scale_f32_dev [out, in/32] (optional) and scale_f16_dev (optional, RNE). */
int qgql_quantize_device(int32_t bits, int32_t out_features, int32_t in_features,
                         const float *w_dev, uint8_t *q_dev, float *scale_f32_dev,
                         uint16_t *scale_f16_dev, void *stream);

/* ---- utilities -------------------------------------------------------------- */
/* Fills dev[0..n) with stdv * N(0,1) from the counter-based generator
 * (splitmix64 + Box-Muller) keyed by (seed, stream), values offset..offset+n. */
int qg_randn_device(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, float stdv,
                    float *dev, void *cuda_stream);

const char *qgmoe_strerror(int status);
/* Detail of the last failure on this thread (e.g. the CUDA error string). */
const char *qgmoe_last_error(void);
/* 1 when built for and running on an sm_100 device, else 0. */
int qgmoe_device_ok(int32_t device);

#ifdef __cplusplus
}
#endif
#endif /* QGMOE_H */
