// qgmoe_route_static: the router top-k (K1) for callers that cannot allocate.
//
// Some hosts of this library may not call cudaMalloc at all: a runtime that
// owns every device allocation itself (an arena or pool handed out by the
// embedding program), a CUDA-graph capture region in which allocation is not
// permitted, or a real-time serving loop whose memory budget is fixed at
// start-up.  qgmoe_route_static gives them the router step with no
// allocation: its scratch (logits, per-CTA histograms,
// counters and dispatch lists) lives in one file-scope __device__ array of
// QGMOE_ROUTE_STATIC_SCRATCH bytes.  The caller passes the activations, the
// router weights, the two output arrays and, optionally, a device word that
// receives the call's error flags.
//
// The array's device address is looked up with cudaGetSymbolAddress on every
// call (cheap once the module is loaded), so there is no cached address that
// two host threads could race on or that a cudaDeviceReset could leave
// stale.  The first call on a device loads the module; make it before any
// stream capture.
//
// Sharing rules: every call on a device uses the same array, and it keeps
// the previous call's contents.  The counters that must start at zero are
// cleared on the call's stream at the start of each call.  Two calls whose
// work overlaps on the GPU (different streams, no ordering between them)
// race on the array and give undefined results; order them on one stream.
#include "qg_common.cuh"

namespace qg {

static __device__ __align__(256) unsigned char g_route_scratch[QGMOE_ROUTE_STATIC_SCRATCH];

static size_t al256(size_t b) { return (b + 255) & ~size_t(255); }

// Bytes of scratch a route of T tokens needs, laid out in 256-byte aligned
// pieces in the order qgmoe_route_static carves them.
static size_t route_scratch_bytes(int T, int E, int k) {
    const size_t chunks = (size_t)(T + QG_TOPK_TOK - 1) / QG_TOPK_TOK;
    size_t n = 0;
    n += al256(sizeof(float) * (size_t)T * E);           // logits
    n += al256(sizeof(int32_t) * chunks * E);            // per-CTA histograms
    n += al256(sizeof(int32_t) * E);                     // counts (zeroed per call)
    n += al256(sizeof(int32_t) * 2);                     // ticket + error word (zeroed)
    n += al256(sizeof(int32_t) * (size_t)T * k) * 2;     // pair_slot, slot_token
    n += al256(sizeof(int32_t) * (E + 1)) * 3;           // active list
    n += al256(sizeof(int32_t) * 1);                     // n_act
    n += al256(sizeof(int32_t) * (E + 2));               // tile prefix
    n += al256(sizeof(int32_t) * E);                     // expert offsets
    n += al256(sizeof(float) * T);                       // shared-gate slot (unused)
    return n;
}

}  // namespace qg

using namespace qg;

extern "C" int qgmoe_route_static(const float *x, const float *router, int32_t T, int32_t H,
                                  int32_t E, int32_t k, int32_t mode, int32_t *sel_idx,
                                  float *sel_w, int32_t *flags, void *stream) {
    if (T < 0 || H <= 0 || H % QG_GROUP || E <= 0 || E > QG_MAX_EXPERTS || k <= 0 ||
        k > QG_MAX_TOPK || k > E)
        return set_error(QGMOE_ERR_INVALID_ARG,
                         "bad shape T=%d H=%d E=%d k=%d (H multiple of 32, 1<=k<=min(E,32))", T,
                         H, E, k);
    if (mode != QGMOE_ROUTER_TOPK && mode != QGMOE_ROUTER_PREFIX)
        return set_error(QGMOE_ERR_INVALID_ARG, "bad router_mode %d", mode);
    if (T == 0) return QGMOE_OK;
    if (!x || !router || !sel_idx || !sel_w)
        return set_error(QGMOE_ERR_INVALID_ARG, "null pointer argument");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router)) & 15)
        return set_error(QGMOE_ERR_INVALID_ARG, "x and router must be 16-byte aligned");
    const size_t need = route_scratch_bytes(T, E, k);
    if (need > QGMOE_ROUTE_STATIC_SCRATCH)
        return set_error(QGMOE_ERR_INVALID_ARG,
                         "route of T=%d tokens over E=%d experts needs %zu bytes of scratch; "
                         "the static scratch holds %d (use fewer tokens per call)",
                         T, E, need, (int)QGMOE_ROUTE_STATIC_SCRATCH);
    void *sym = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&sym, g_route_scratch);
    if (e != cudaSuccess)
        return set_error(QGMOE_ERR_CUDA, "cudaGetSymbolAddress(route scratch): %s",
                         cudaGetErrorString(e));
    unsigned char *base = static_cast<unsigned char *>(sym);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        void *p = base + off;
        off += al256(bytes);
        return p;
    };
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    RouteState st{};
    st.topk_idx = sel_idx;  // outputs go straight to the caller's arrays
    st.topk_w = sel_w;
    st.logits = static_cast<float *>(take(sizeof(float) * (size_t)T * E));
    st.hist = static_cast<int32_t *>(
        take(sizeof(int32_t) * (size_t)((T + QG_TOPK_TOK - 1) / QG_TOPK_TOK) * E));
    st.counts = static_cast<int32_t *>(take(sizeof(int32_t) * E));
    int32_t *words = static_cast<int32_t *>(take(sizeof(int32_t) * 2));
    st.done_ctr = words;
    int *err = flags ? flags : words + 1;
    st.pair_slot = static_cast<int32_t *>(take(sizeof(int32_t) * (size_t)T * k));
    st.slot_token = static_cast<int32_t *>(take(sizeof(int32_t) * (size_t)T * k));
    st.act_group = static_cast<int32_t *>(take(sizeof(int32_t) * (E + 1)));
    st.act_begin = static_cast<int32_t *>(take(sizeof(int32_t) * (E + 1)));
    st.act_n = static_cast<int32_t *>(take(sizeof(int32_t) * (E + 1)));
    st.n_act = static_cast<int32_t *>(take(sizeof(int32_t)));
    st.tile_prefix = static_cast<int32_t *>(take(sizeof(int32_t) * (E + 2)));
    st.expert_off = static_cast<int32_t *>(take(sizeof(int32_t) * E));
    st.shared_w = static_cast<float *>(take(sizeof(float) * T));
    // The array keeps the previous call's contents: the histogram counters,
    // the last-CTA ticket and the error word must start at zero.
    QG_CUDA(cudaMemsetAsync(st.counts, 0, sizeof(int32_t) * E, s));
    QG_CUDA(cudaMemsetAsync(words, 0, sizeof(int32_t) * 2, s));
    if (flags) QG_CUDA(cudaMemsetAsync(flags, 0, sizeof(int32_t), s));
    return launch_route(x, T, H, E, k, mode, router, nullptr, 0, st, nullptr, nullptr, err, s);
}
