// Expert parallelism without host round trips: the row exchange of the
// expert-parallel forward goes through NVLink peer memory (CUDA IPC
// mappings of every rank's exchange region) instead of NCCL all-to-all.
//
// Per rank, one exchange region (identical layout on every rank):
//   flags   cnt[W], data[W], back[W]  (u64 epochs, written by the peers)
//   epoch   this rank's forward counter (local)
//   ticket  last-CTA counter of k_px_send (local)
//   inbox   [W src][W dst][G] int32: every rank's count matrix (broadcast)
//   recv    [W*cap][H] fp16: rows received for this rank's experts, grouped
//           by local expert; within an expert the sources follow each other
//           starting at this rank (me, me+1, ..., me-1 mod W), so that the
//           owners' down GEMMs, which walk their experts' rows in this
//           order, start by returning rows to different sources
//   back    [cap][H] fp16: expert outputs of this rank's own rows, returned
//           by their owners in this rank's send order
// One forward (rank me, epoch e):
//   k_px_counts  my count matrix c[d][g] (rows I send to rank d for its local
//                expert g) into every rank's inbox, then cnt[me] = e there;
//   k_px_send    wait for every cnt flag; from the W count matrices compute
//                where each of my rows lands in its owner's grouped buffer
//                and store it there (fp16, converted from x on the fly); the
//                warps are split evenly over the destinations, rotated by
//                rank, so every destination receives from every source at
//                once instead of all sources sending to one rank at a time;
//                the last CTA sets data[me] = e on every rank;
//   k_px_tables  wait for every data flag; build this rank's active-expert
//                list, tile prefix and, per received row, the (source rank,
//                send position) its output goes back to;
//   GEMMs        gate_up on the grouped rows, down with an epilogue that
//                stores each output row straight into its source's back
//                buffer over NVLink;
//   k_px_signal  back[me] = e on every rank;
//   k_px_wait    wait for every back flag; then the usual rank-ordered
//                combine reads the back buffer in send order.
// Ordering: every writer fences (system scope) before a barrier, and one
// thread publishes with st.release.sys; readers poll with ld.acquire.sys.
// Every wait is bounded (clock64 budget); a timeout raises
// QG_FLAG_TIMEOUT in the rank's error word and the kernel skips its work.
// Region reuse is safe across forwards: a rank can only write epoch e+1
// data into a peer after that peer finished epoch e (each forward ends with
// a wait on every rank's back flag, issued after its own reads).
#include "qg_common.cuh"

namespace qg {

constexpr long long PX_WAIT_CYCLES = 4000000000LL;  // ~2 s

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait until flags[0..W-1] >= epoch.
__device__ bool px_wait_flags(const uint64_t *flags, int W, uint64_t epoch, long long wait) {
    const long long budget = wait > 0 ? wait : PX_WAIT_CYCLES;
    const long long t0 = clock64();
    for (int s = 0; s < W; s++)
        while (ld_acquire_sys(flags + s) < epoch) {
            if (clock64() - t0 > budget) return false;
            __nanosleep(64);
        }
    return true;
}

__device__ __forceinline__ uint8_t *px_base(const PxArgs &a, int r) { return a.bases[r]; }
__device__ __forceinline__ uint64_t *px_flag(const PxArgs &a, int r, int kind, int s) {
    return reinterpret_cast<uint64_t *>(px_base(a, r) + kind * PX_FLAG_BLOCK) + s;
}
__device__ __forceinline__ int32_t *px_inbox(const PxArgs &a, int r) {
    return reinterpret_cast<int32_t *>(px_base(a, r) + a.off_inbox);
}
__device__ __forceinline__ uint64_t px_epoch(const PxArgs &a) {
    return *reinterpret_cast<volatile uint64_t *>(px_base(a, a.me) + a.off_epoch);
}

// Rows this rank sends to key (d, g) = expert_off[key+1] - expert_off[key].
__device__ __forceinline__ int px_my_count(const PxArgs &a, const int32_t *expert_off, int key) {
    const int E = a.W * a.G;
    return (key + 1 < E ? expert_off[key + 1] : a.T * a.k) - expert_off[key];
}

// 1 CTA: epoch += 1; broadcast my count matrix; publish cnt[me].
__global__ void k_px_counts(PxArgs a, const int32_t *__restrict__ expert_off, int *err) {
    __shared__ uint64_t s_epoch;
    const int tid = threadIdx.x;
    if (tid == 0) {
        uint64_t *ep = reinterpret_cast<uint64_t *>(px_base(a, a.me) + a.off_epoch);
        s_epoch = *ep + 1;
        *ep = s_epoch;
    }
    __syncthreads();
    const int WG = a.W * a.G;
    for (int i = tid; i < a.W * WG; i += blockDim.x) {
        const int r = i / WG, key = i - r * WG;  // destination inbox r, my row (key = d*G + g)
        px_inbox(a, r)[a.me * WG + key] = px_my_count(a, expert_off, key);
    }
    __threadfence_system();
    __syncthreads();
    if (tid < a.W) st_release_sys(px_flag(a, tid, PX_CNT, a.me), s_epoch);
}

// Every rank's count matrix into shared memory: cnt[(s*W + d)*G + g].
__device__ void px_load_counts(const PxArgs &a, int32_t *cnt) {
    const int n = a.W * a.W * a.G;
    const int32_t *in = px_inbox(a, a.me);
    for (int i = threadIdx.x; i < n; i += blockDim.x) cnt[i] = __ldcv(in + i);
}

// Warp per row: x[token] (f32) -> fp16 into the owner's grouped buffer.
__global__ void __launch_bounds__(256)
k_px_send(PxArgs a, const float *__restrict__ x, const int32_t *__restrict__ expert_off,
          const int32_t *__restrict__ slot_token, int *err) {
    extern __shared__ int32_t px_sm[];
    const int W = a.W, G = a.G, WG = W * G;
    int32_t *cnt = px_sm;                 // [W][W][G]
    int32_t *pos = cnt + W * WG;          // [W*G] base position of my (d, g) rows at d
    int32_t *off = pos + WG;              // [W*G] my expert_off
    __shared__ int s_ok, s_last;
    __shared__ uint64_t s_epoch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_epoch = px_epoch(a);
        s_ok = px_wait_flags(px_flag(a, a.me, PX_CNT, 0), W, s_epoch, a.wait);
        if (!s_ok) atomicOr(err, QG_FLAG_TIMEOUT);
    }
    __syncthreads();
    if (!s_ok) return;
    px_load_counts(a, cnt);
    for (int i = tid; i < WG; i += blockDim.x) off[i] = expert_off[i];
    __syncthreads();
    // position at d of my rows for d's local expert g: the rows of d's local
    // experts before g (all sources), then the rows of the sources that come
    // before me in d's order (d, d+1, ..., d-1 mod W) for g
    for (int key = tid; key < WG; key += blockDim.x) {
        const int d = key / G, g = key - d * G;
        int p = 0;
        for (int g2 = 0; g2 < g; g2++)
            for (int s = 0; s < W; s++) p += cnt[(s * W + d) * G + g2];
        for (int s = d; s != a.me; s = s + 1 == W ? 0 : s + 1) p += cnt[(s * W + d) * G + g];
        pos[key] = p;
    }
    __syncthreads();
    // warp slot j (global warp index mod W) sends to destination (me + j) mod W
    const int nw = gridDim.x * (blockDim.x >> 5);
    const int wg = blockIdx.x * (blockDim.x >> 5) + warp;
    const int j = wg % W;
    const int d = (a.me + j) % W;
    const int wi = wg / W, nwd = (nw - j + W - 1) / W;  // my index among d's warps
    const int p_end = d + 1 < W ? off[(d + 1) * G] : a.T * a.k;
    for (int p = off[d * G] + wi; p < p_end; p += nwd) {
        int lo = d * G, hi = d * G + G - 1;  // last key of d with off[key] <= p
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (off[mid] <= p) lo = mid; else hi = mid - 1;
        }
        const int64_t row = pos[lo] + (p - off[lo]);
        if (row < 0 || row >= (int64_t)a.recv_cap) {
            if (lane == 0) atomicOr(err, QG_FLAG_BAD_SLOT);
            continue;
        }
        const float *src = x + (size_t)slot_token[p] * a.H;
        __half *dst = reinterpret_cast<__half *>(px_base(a, d) + a.off_recv) + row * a.H;
        for (int c = lane * 8; c < a.H; c += 256) {
            const float4 v0 = *reinterpret_cast<const float4 *>(src + c);
            const float4 v1 = *reinterpret_cast<const float4 *>(src + c + 4);
            __half2 h[4] = {__floats2half2_rn(v0.x, v0.y), __floats2half2_rn(v0.z, v0.w),
                            __floats2half2_rn(v1.x, v1.y), __floats2half2_rn(v1.z, v1.w)};
            *reinterpret_cast<uint4 *>(dst + c) = *reinterpret_cast<uint4 *>(h);
        }
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        int *ticket = reinterpret_cast<int *>(px_base(a, a.me) + a.off_ticket);
        s_last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
        if (s_last) *ticket = 0;
    }
    __syncthreads();
    if (s_last && tid < W) st_release_sys(px_flag(a, tid, PX_DATA, a.me), s_epoch);
}

// Wait for every rank's rows; build this rank's expert tables and the
// return address (source rank << 24 | send position) of each received row.
// CTA 0 writes the tables; every CTA fills its share of out_map.
__global__ void __launch_bounds__(256)
k_px_tables(PxArgs a, int tile_tokens, PxTables t, int *err) {
    extern __shared__ int32_t px_sm[];
    const int W = a.W, G = a.G, WG = W * G;
    int32_t *cnt = px_sm;                  // [W][W][G]
    int32_t *gbase = cnt + W * WG;         // [G+1] first grouped row of local expert g
    int32_t *seg = gbase + G + 1;          // [G][W] first grouped row of (g, j-th source)
    int32_t *dst0 = seg + WG;              // [G][W] send position of that source's row 0
    __shared__ int s_ok;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_ok = px_wait_flags(px_flag(a, a.me, PX_DATA, 0), W, px_epoch(a), a.wait);
        if (!s_ok) atomicOr(err, QG_FLAG_TIMEOUT);
    }
    __syncthreads();
    if (!s_ok) {
        if (blockIdx.x == 0 && tid == 0) {  // no units: the GEMMs run empty
            *t.n_act = 0;
            t.tile_prefix[0] = 0;
        }
        return;
    }
    px_load_counts(a, cnt);
    __syncthreads();
    const int me = a.me;
    if (warp == 0) {
        // per local expert g: rows from every source (exclusive scan over g)
        int carry = 0;
        for (int g0 = 0; g0 < G; g0 += 32) {
            const int g = g0 + lane;
            int n = 0;
            if (g < G)
                for (int s = 0; s < W; s++) n += cnt[(s * W + me) * G + g];
            int incl = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            if (g < G) gbase[g] = carry + incl - n;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) gbase[G] = carry;
    }
    __syncthreads();
    // within expert g the sources follow each other as me, me+1, ..., me-1 (mod W)
    for (int i = tid; i < WG; i += blockDim.x) {
        const int g = i / W, j = i - g * W, s = (me + j) % W;
        int r = gbase[g];
        for (int s2 = me; s2 != s; s2 = s2 + 1 == W ? 0 : s2 + 1) r += cnt[(s2 * W + me) * G + g];
        seg[i] = r;
        // position of s's first row for (me, g) in s's send order: s's rows
        // for ranks before me, then for my experts before g
        int p = 0;
        for (int d = 0; d < me; d++)
            for (int g2 = 0; g2 < G; g2++) p += cnt[(s * W + d) * G + g2];
        for (int g2 = 0; g2 < g; g2++) p += cnt[(s * W + me) * G + g2];
        dst0[i] = p;
    }
    __syncthreads();
    const int R = gbase[G];
    if (blockIdx.x == 0 && warp == 0) {
        const int tsh = __ffs(tile_tokens) - 1;
        int na_base = 0, tb_base = 0;
        for (int g0 = 0; g0 < G; g0 += 32) {
            const int g = g0 + lane;
            const int n = g < G ? gbase[g + 1] - gbase[g] : 0;
            const int act = n > 0, tl = (n + tile_tokens - 1) >> tsh;
            int ai = act, ti = tl;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, ai, o);
                const int w = __shfl_up_sync(0xffffffffu, ti, o);
                if (lane >= o) {
                    ai += v;
                    ti += w;
                }
            }
            if (act) {
                const int slot = na_base + ai - 1;
                t.act_group[slot] = g;
                t.act_begin[slot] = gbase[g];
                t.act_n[slot] = n;
                t.tile_prefix[slot] = tb_base + ti - tl;
            }
            na_base += __shfl_sync(0xffffffffu, ai, 31);
            tb_base += __shfl_sync(0xffffffffu, ti, 31);
        }
        if (lane == 0) {
            t.tile_prefix[na_base] = tb_base;
            *t.n_act = na_base;
            *t.n_rows = R;
        }
    }
    for (int r = blockIdx.x * blockDim.x + tid; r < R; r += gridDim.x * blockDim.x) {
        int lo = 0, hi = G - 1;  // local expert of row r
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (gbase[mid] <= r) lo = mid; else hi = mid - 1;
        }
        int j = W - 1;
        while (j > 0 && seg[lo * W + j] > r) j--;
        const int s = (me + j) % W;
        t.out_map[r] = (s << 24) | (dst0[lo * W + j] + (r - seg[lo * W + j]));
    }
}

// After the down GEMM: my outputs for every source are in place.
__global__ void k_px_signal(PxArgs a) {
    __threadfence_system();
    if ((int)threadIdx.x < a.W)
        st_release_sys(px_flag(a, threadIdx.x, PX_BACK, a.me), px_epoch(a));
}

// Before the combine: every owner has returned my rows.
__global__ void k_px_wait(PxArgs a, int *err) {
    if (threadIdx.x == 0 && !px_wait_flags(px_flag(a, a.me, PX_BACK, 0), a.W, px_epoch(a), a.wait))
        atomicOr(err, QG_FLAG_TIMEOUT);
}

static size_t px_smem(const PxArgs &a) {
    return sizeof(int32_t) * ((size_t)a.W * a.W * a.G + 3 * (size_t)a.W * a.G + a.G + 1);
}

int launch_px_counts(const PxArgs &a, const int32_t *expert_off, int *err, cudaStream_t s) {
    k_px_counts<<<1, 256, 0, s>>>(a, expert_off, err);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_px_send(const PxArgs &a, const float *x, const int32_t *expert_off,
                   const int32_t *slot_token, int *err, cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int rows = a.T * a.k;
    int blocks = (rows + 7) / 8;
    const int cap = num_sms(dev) * 4;
    if (blocks > cap) blocks = cap;
    if (blocks < (a.W + 7) / 8) blocks = (a.W + 7) / 8;  // at least one warp per destination
    k_px_send<<<blocks, 256, px_smem(a), s>>>(a, x, expert_off, slot_token, err);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_px_tables(const PxArgs &a, int tile_tokens, const PxTables &t, int *err,
                     cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    k_px_tables<<<num_sms(dev), 256, px_smem(a), s>>>(a, tile_tokens, t, err);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_px_signal(const PxArgs &a, cudaStream_t s) {
    k_px_signal<<<1, 32, 0, s>>>(a);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

int launch_px_wait(const PxArgs &a, int *err, cudaStream_t s) {
    k_px_wait<<<1, 32, 0, s>>>(a, err);
    QG_CUDA(cudaGetLastError());
    return QGMOE_OK;
}

}  // namespace qg
