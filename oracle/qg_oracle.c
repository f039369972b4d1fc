/*
 * qg_oracle.c -- CPU restatement of qwen-go's MoE layer and QuantLinear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in qwen-go_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * path never calls into it and has no CPU fallback.
 *
 * Parity status: the reference (jackkey143084/qwen-go) is pure Go and no Go
 * toolchain exists on the build or GPU machines, so the reference cannot be
 * run to produce golden values.  The restatement is pinned only against the
 * reference's own test fixtures (TestMoERouting, model/model_test.go:182-201;
 * TestQuantRoundTrip, model/model_test.go:130-147) and hand-derived known
 * answers; value-level parity with the Go binary is UNPINNED.
 *
 * Arithmetic rules followed (Go on amd64 does not contract a*b+c into FMA,
 * so this file is compiled with -ffp-contract=off):
 *   - every dot product is a serial float32 sum in index order
 *     (matmulVec, model/tensors.go:77-89);
 *   - exp() is evaluated in float64 and rounded to float32
 *     (silu/sigmoid1/softmax, model/tensors.go:91-121);
 *   - rounding is half away from zero (math.Round, model/moe.go:258),
 *     which is C round().
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QG_GROUP 32 /* quantGroup, model/moe.go:124 */

/* ------------------------------------------------------------------------ */
/* Deterministic synthetic inputs: counter-based splitmix64 + Box-Muller.    */
/* Value i of (seed, stream) depends only on (seed, stream, i).             */
/* ------------------------------------------------------------------------ */
static inline uint64_t qg_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static inline double qg_uniform(uint64_t key, uint64_t ctr) {
    /* (0, 1]: never 0, so log() is finite */
    uint64_t r = qg_mix64(key ^ qg_mix64(ctr));
    return ((double)(r >> 11) + 1.0) * (1.0 / 9007199254740992.0);
}

uint64_t qgo_stream_key(uint64_t seed, uint64_t stream) {
    return qg_mix64(qg_mix64(seed) + stream * 0xD1B54A32D192ED03ULL);
}

/* out[i] = std * N(0,1)_i for i in [offset, offset+n) of stream (seed, stream) */
void qgo_randn(uint64_t seed, uint64_t stream, uint64_t offset, int64_t n, float stdv,
               float *out) {
    const uint64_t key = qgo_stream_key(seed, stream);
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t j = 0; j < n; j++) {
        uint64_t i = offset + (uint64_t)j;
        uint64_t pair = i >> 1;
        double u1 = qg_uniform(key, 2 * pair);
        double u2 = qg_uniform(key, 2 * pair + 1);
        double r = sqrt(-2.0 * log(u1));
        double z = (i & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
        out[j] = (float)(z * (double)stdv);
    }
}

/* ------------------------------------------------------------------------ */
/* fp16 helpers.  Decode restates f16to32 (safetensors/safetensors.go:182-207);
 * encode is IEEE round-to-nearest-even (the reference has no encoder: its
 * fp16 scales come from quantize.py-style checkpoints).                    */
/* ------------------------------------------------------------------------ */
float qgo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u;
    uint32_t ex = (uint32_t)(h >> 10) & 0x1Fu;
    uint32_t frac = (uint32_t)h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (frac == 0) {
            bits = sign << 31;
        } else {
            uint32_t e = 127 - 15 + 1;
            while ((frac & 0x400u) == 0) {
                frac <<= 1;
                e--;
            }
            frac &= 0x3FFu;
            bits = sign << 31 | e << 23 | frac << 13;
        }
    } else if (ex == 0x1F) {
        bits = sign << 31 | 0xFFu << 23 | frac << 13;
    } else {
        bits = sign << 31 | (ex - 15 + 127) << 23 | frac << 13;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t qgo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
    if (ax >= 0x477FF000u) /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7C00u);
    if (ax < 0x38800000u) { /* below 2^-14: subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25 -> 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

void qgo_f16_encode(const float *in, int64_t n, uint16_t *out) {
    for (int64_t i = 0; i < n; i++) out[i] = qgo_f32_to_f16(in[i]);
}
void qgo_f16_decode(const uint16_t *in, int64_t n, float *out) {
    for (int64_t i = 0; i < n; i++) out[i] = qgo_f16_to_f32(in[i]);
}

/* ------------------------------------------------------------------------ */
/* QuantLinear: model/moe.go:124-258                                        */
/* ------------------------------------------------------------------------ */
static inline float qg_abs32(float x) { return x < 0 ? -x : x; }   /* moe.go:241 */
static inline float qg_clamp(float x, float lo, float hi) {           /* moe.go:248 */
    if (x < lo) return lo;
    if (x > hi) return hi;
    return x;
}
static inline float qg_round32(float x) { return (float)round((double)x); } /* moe.go:258 */

/* quantizeInt8, model/moe.go:165-188 */
void qgo_quantize_int8(const float *w, int out_dim, int in_dim, uint8_t *q, float *scale) {
    const int ng = in_dim / QG_GROUP;
    for (int o = 0; o < out_dim; o++) {
        for (int b = 0; b < ng; b++) {
            float amax = 0;
            for (int j = 0; j < QG_GROUP; j++) {
                float a = qg_abs32(w[(size_t)o * in_dim + b * QG_GROUP + j]);
                if (a > amax) amax = a;
            }
            float s = amax / 127;
            if (s < 1e-8f) s = 1e-8f;
            scale[(size_t)o * ng + b] = s;
            for (int j = 0; j < QG_GROUP; j++) {
                float v = qg_round32(w[(size_t)o * in_dim + b * QG_GROUP + j] / s);
                q[(size_t)o * in_dim + b * QG_GROUP + j] = (uint8_t)(int8_t)qg_clamp(v, -127, 127);
            }
        }
    }
}

/* quantizeInt4, model/moe.go:190-217: even j -> high nibble, stored +8 */
void qgo_quantize_int4(const float *w, int out_dim, int in_dim, uint8_t *q, float *scale) {
    const int ng = in_dim / QG_GROUP;
    memset(q, 0, (size_t)out_dim * in_dim / 2);
    for (int o = 0; o < out_dim; o++) {
        for (int b = 0; b < ng; b++) {
            float amax = 0;
            for (int j = 0; j < QG_GROUP; j++) {
                float a = qg_abs32(w[(size_t)o * in_dim + b * QG_GROUP + j]);
                if (a > amax) amax = a;
            }
            float s = amax / 7;
            if (s < 1e-8f) s = 1e-8f;
            scale[(size_t)o * ng + b] = s;
            for (int j = 0; j < QG_GROUP; j++) {
                float v = qg_clamp(qg_round32(w[(size_t)o * in_dim + b * QG_GROUP + j] / s), -7, 7) + 8;
                size_t at = (size_t)o * (in_dim / 2) + b * QG_GROUP / 2 + j / 2;
                if (j % 2 == 0)
                    q[at] |= (uint8_t)(((int)v & 0xF) << 4);
                else
                    q[at] |= (uint8_t)((int)v & 0xF);
            }
        }
    }
}

/* quantLinear.dequantize, model/moe.go:134-157 */
void qgo_dequantize(int bits, int out_dim, int in_dim, const uint8_t *q, const float *scale,
                    float *w) {
    const int ng = in_dim / QG_GROUP;
    if (bits == 8) {
        for (int o = 0; o < out_dim; o++)
            for (int c = 0; c < in_dim; c++) {
                int8_t v = (int8_t)q[(size_t)o * in_dim + c];
                w[(size_t)o * in_dim + c] = (float)v * scale[(size_t)o * ng + c / QG_GROUP];
            }
        return;
    }
    for (int o = 0; o < out_dim; o++)
        for (int c = 0; c < in_dim / 2; c++) {
            uint8_t b = q[(size_t)o * (in_dim / 2) + c];
            float hi = (float)((int)(b >> 4) & 0xF) - 8;
            float lo = (float)((int)b & 0xF) - 8;
            w[(size_t)o * in_dim + 2 * c] = hi * scale[(size_t)o * ng + (2 * c) / QG_GROUP];
            w[(size_t)o * in_dim + 2 * c + 1] = lo * scale[(size_t)o * ng + (2 * c + 1) / QG_GROUP];
        }
}

/* ------------------------------------------------------------------------ */
/* Tensor ops: model/tensors.go                                             */
/* ------------------------------------------------------------------------ */
/* matmulVec, tensors.go:77-89: y = x @ W^T, serial f32 sum per row */
void qgo_matmul_vec(const float *x, const float *w, int in_dim, int out_dim, float *y) {
    for (int o = 0; o < out_dim; o++) {
        const float *wr = w + (size_t)o * in_dim;
        float s = 0;
        for (int k = 0; k < in_dim; k++) s += x[k] * wr[k];
        y[o] = s;
    }
}

/* silu, tensors.go:91-95 */
static void qg_silu(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = x[i] / (1 + (float)exp(-(double)x[i]));
}

/* sigmoid1, tensors.go:97 */
static float qg_sigmoid1(float x) { return 1 / (1 + (float)exp(-(double)x)); }

/* softmax, tensors.go:106-121 */
void qgo_softmax(float *v, int n) {
    float mx = v[0];
    for (int i = 1; i < n; i++)
        if (v[i] > mx) mx = v[i];
    float sum = 0;
    for (int i = 0; i < n; i++) {
        v[i] = (float)exp((double)(v[i] - mx));
        sum += v[i];
    }
    for (int i = 0; i < n; i++) v[i] /= sum;
}

/* ------------------------------------------------------------------------ */
/* MoE layer: model/moe.go:10-99 and denseMLP.forward model/model.go:350-358 */
/* ------------------------------------------------------------------------ */
enum { QGO_ROUTER_TOPK = 0, QGO_ROUTER_PREFIX = 1 };

/* One linear in either format: f32 rows (bits 32) or quantLinear (8/4). */
typedef struct {
    const float *w;       /* bits == 32: [out, in] */
    const uint8_t *q;     /* bits 8/4: codes */
    const float *scale;   /* bits 8/4: [out, in/32] as float32 values */
} qgo_lin;

typedef struct {
    int n_embed, n_experts, top_k, n_moe_mlp, n_shared_mlp;
    int bits;         /* 32, 8, 4: routed experts */
    int router_mode;  /* QGO_ROUTER_TOPK / QGO_ROUTER_PREFIX */
    const float *router;       /* [E, H] f32 (moeMLP.gate), router_bits 32 */
    const float *shared_gate;  /* [H] (moeMLP.sharedGate), used when n_shared_mlp > 0 */
    qgo_lin gate_up;           /* stacked [E, 2I, H] */
    qgo_lin down;              /* stacked [E, H, I] */
    qgo_lin sh_gate, sh_up;    /* [Is, H] */
    qgo_lin sh_down;           /* [H, Is] */
    int shared_bits;           /* 32, 8, 4: the shared expert's format */
    int router_bits;           /* 32: router rows; 8 / 4: routerQuant (moe.go:16) */
    qgo_lin router_q;          /* router_bits 8 / 4: codes + scales */
} qgo_moe;

/* proj(x, 1, ...) on one row block of a stacked tensor (model.go:196-205;
 * quantLinear.forward moe.go:159-162 dequantizes the whole matrix, then
 * matmulVec).  For stacked experts `row0` selects expert e's rows; a stacked
 * [E*O, I] matrix quantised row-wise equals per-expert quantisation.       */
static void qg_linear_forward(const qgo_lin *l, int bits, size_t row0, int out_dim, int in_dim,
                              const float *x, float *y, float *scratch) {
    if (bits == 32) {
        qgo_matmul_vec(x, l->w + row0 * in_dim, in_dim, out_dim, y);
        return;
    }
    const uint8_t *q = l->q + (bits == 8 ? row0 * in_dim : row0 * in_dim / 2);
    const float *s = l->scale + row0 * (in_dim / QG_GROUP);
    qgo_dequantize(bits, out_dim, in_dim, q, s, scratch); /* transient, as moe.go:160 */
    qgo_matmul_vec(x, scratch, in_dim, out_dim, y);
}

/* Router selection for one token: softmax(logits) then the insertion sort of
 * moe.go:45-52.  PREFIX keeps the literal loop bound (i < topK, so only
 * idx[0..k-1] = experts 0..k-1 are ever ordered); TOPK runs the same loop
 * over all n experts.  Writes idx[k], renormalised w[k] (moe.go:53-63).     */
void qgo_route_token(const float *probs_in, int n, int k, int mode, int32_t *idx_out,
                     float *w_out) {
    float *p = (float *)malloc(sizeof(float) * n);
    int *idx = (int *)malloc(sizeof(int) * n);
    memcpy(p, probs_in, sizeof(float) * n);
    qgo_softmax(p, n);
    for (int i = 0; i < n; i++) idx[i] = i;
    int lim = mode == QGO_ROUTER_PREFIX ? k : n;
    for (int i = 1; i < lim && i < n; i++)
        for (int j = i; j > 0 && p[idx[j]] > p[idx[j - 1]]; j--) {
            int t = idx[j];
            idx[j] = idx[j - 1];
            idx[j - 1] = t;
        }
    float wsum = 0;
    for (int i = 0; i < k; i++) wsum += p[idx[i]];
    for (int i = 0; i < k; i++) {
        idx_out[i] = idx[i];
        w_out[i] = p[idx[i]] / (wsum + 1e-9f);
    }
    free(p);
    free(idx);
}

/* moeMLP.forward for one token (moe.go:41-99).  probs_out[E] receives the
 * softmax probabilities (for tie analysis in tests); may be NULL.          */
static void qg_moe_token(const qgo_moe *m, const float *x, float *out, int32_t *idx_out,
                         float *w_out, float *sg_out, float *probs_out) {
    const int H = m->n_embed, E = m->n_experts, K = m->top_k, I = m->n_moe_mlp;
    const int Is = m->n_shared_mlp;
    float *logits = (float *)malloc(sizeof(float) * E);
    float *rscratch = m->router_bits == 32 ? NULL : (float *)malloc(sizeof(float) * (size_t)E * H);
    /* proj(x, 1, &m.gate, m.routerQuant, E), moe.go:42 and model.go:196-205:
     * the router rows, or quantLinear.forward = dequantize, then matmulVec */
    if (m->router_bits == 32)
        qgo_matmul_vec(x, m->router, H, E, logits);
    else
        qg_linear_forward(&m->router_q, m->router_bits, 0, E, H, x, logits, rscratch);
    free(rscratch);
    if (probs_out) {
        memcpy(probs_out, logits, sizeof(float) * E);
        qgo_softmax(probs_out, E);
    }
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * K);
    float *w = (float *)malloc(sizeof(float) * K);
    qgo_route_token(logits, E, K, m->router_mode, idx, w);

    int maxdim = 2 * I > Is ? 2 * I : Is;
    size_t scratch_n = (size_t)(2 * I) * H;
    if ((size_t)H * I > scratch_n) scratch_n = (size_t)H * I;
    if ((size_t)Is * H > scratch_n) scratch_n = (size_t)Is * H;
    float *scratch = (float *)malloc(sizeof(float) * (scratch_n ? scratch_n : 1));
    float *gu = (float *)malloc(sizeof(float) * (maxdim > H ? maxdim : H));
    float *d = (float *)malloc(sizeof(float) * H);
    for (int j = 0; j < H; j++) out[j] = 0;
    for (int r = 0; r < K; r++) {
        int e = idx[r];
        /* gate_up matvec moe.go:64-69 */
        qg_linear_forward(&m->gate_up, m->bits, (size_t)e * 2 * I, 2 * I, H, x, gu, scratch);
        float *g = gu, *u = gu + I; /* moe.go:70-71 */
        qg_silu(g, I);
        for (int j = 0; j < I; j++) g[j] *= u[j];
        /* down matvec moe.go:77-81 */
        qg_linear_forward(&m->down, m->bits, (size_t)e * H, H, I, g, d, scratch);
        for (int j = 0; j < H; j++) out[j] += w[r] * d[j]; /* moe.go:82-85 */
        if (idx_out) idx_out[r] = e;
        if (w_out) w_out[r] = w[r];
    }
    if (Is > 0) {
        /* denseMLP.forward, model.go:350-358 */
        float *g = (float *)malloc(sizeof(float) * Is);
        float *u = (float *)malloc(sizeof(float) * Is);
        float *s = (float *)malloc(sizeof(float) * H);
        qg_linear_forward(&m->sh_gate, m->shared_bits, 0, Is, H, x, g, scratch);
        qg_linear_forward(&m->sh_up, m->shared_bits, 0, Is, H, x, u, scratch);
        qg_silu(g, Is);
        for (int i = 0; i < Is; i++) g[i] *= u[i];
        qg_linear_forward(&m->sh_down, m->shared_bits, 0, H, Is, g, s, scratch);
        /* sigmoid(shared_gate . x), moe.go:87-97 */
        float gd = 0;
        for (int i = 0; i < H; i++) gd += x[i] * m->shared_gate[i];
        float sg = qg_sigmoid1(gd);
        for (int j = 0; j < H; j++) out[j] += sg * s[j];
        if (sg_out) *sg_out = sg;
        free(g);
        free(u);
        free(s);
    } else if (sg_out) {
        *sg_out = 0;
    }
    free(scratch);
    free(gu);
    free(d);
    free(logits);
    free(idx);
    free(w);
}

/* T tokens, one after another, as decodeLayers calls mlp.forward per token
 * (model/model.go:507-514).  idx/w: [T, k]; sg: [T]; probs: [T, E]; any of
 * them may be NULL.                                                        */
void qgo_moe_forward(const qgo_moe *m, const float *x, int T, float *out, int32_t *idx,
                     float *w, float *sg, float *probs) {
    const int H = m->n_embed, K = m->top_k, E = m->n_experts;
    for (int t = 0; t < T; t++)
        qg_moe_token(m, x + (size_t)t * H, out + (size_t)t * H, idx ? idx + (size_t)t * K : NULL,
                     w ? w + (size_t)t * K : NULL, sg ? sg + t : NULL,
                     probs ? probs + (size_t)t * E : NULL);
}

/* Token-parallel variant (NOT the reference's behaviour, which is serial per
 * token): T independent tokens split over n_threads pthreads.  Each token's
 * arithmetic is qg_moe_token's, so the results equal qgo_moe_forward's bit
 * for bit.  Used as the labelled all-cores CPU baseline and by the tests to
 * check hundreds of full-size tokens; idx/w/sg/probs may be NULL.          */
typedef struct {
    const qgo_moe *m;
    const float *x;
    float *out;
    int32_t *idx;
    float *w, *sg, *probs;
    int t0, t1;
} qg_job;

static void *qg_worker(void *arg) {
    qg_job *j = (qg_job *)arg;
    const int H = j->m->n_embed, K = j->m->top_k, E = j->m->n_experts;
    for (int t = j->t0; t < j->t1; t++)
        qg_moe_token(j->m, j->x + (size_t)t * H, j->out + (size_t)t * H,
                     j->idx ? j->idx + (size_t)t * K : NULL, j->w ? j->w + (size_t)t * K : NULL,
                     j->sg ? j->sg + t : NULL, j->probs ? j->probs + (size_t)t * E : NULL);
    return NULL;
}

int qgo_moe_forward_mt(const qgo_moe *m, const float *x, int T, float *out, int32_t *idx,
                       float *w, float *sg, float *probs, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > T) n_threads = T > 0 ? T : 1;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * n_threads);
    qg_job *jobs = (qg_job *)malloc(sizeof(qg_job) * n_threads);
    int chunk = (T + n_threads - 1) / n_threads;
    int spawned = 0;
    for (int i = 0; i < n_threads; i++) {
        int t0 = i * chunk, t1 = t0 + chunk > T ? T : t0 + chunk;
        if (t0 >= t1) break;
        jobs[i] = (qg_job){m, x, out, idx, w, sg, probs, t0, t1};
        if (pthread_create(&th[i], NULL, qg_worker, &jobs[i]) != 0) {
            qg_worker(&jobs[i]);
            th[i] = 0;
        }
        spawned++;
    }
    for (int i = 0; i < spawned; i++)
        if (th[i]) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
    return spawned;
}

/* Plain QuantLinear / linear forward over T rows (proj with T rows,
 * model.go:196-205: quantised weights dequantised once, then per-row
 * serial dot products as matmulRange, tensors.go:61-74).                   */
void qgo_linear_forward_rows(int bits, int out_dim, int in_dim, const float *wf,
                             const uint8_t *q, const float *scale, const float *x, int T,
                             float *y) {
    const float *w = wf;
    float *tmp = NULL;
    if (bits != 32) {
        tmp = (float *)malloc(sizeof(float) * (size_t)out_dim * in_dim);
        qgo_dequantize(bits, out_dim, in_dim, q, scale, tmp);
        w = tmp;
    }
    for (int t = 0; t < T; t++)
        qgo_matmul_vec(x + (size_t)t * in_dim, w, in_dim, out_dim, y + (size_t)t * out_dim);
    free(tmp);
}
