/* A plain-C host that drives a stack of MoE layers through the C ABI the
 * way qwen-go's decodeLayers (model/model.go:473-526) would through cgo:
 * per layer, h = rmsnorm(x) on the host, out = moe_l(h) with qgmoe_forward
 * (host pointers, blocking: the Go shim's call), x += out (the block's
 * residual).  Attention, embeddings and the LM head are outside the rebuilt
 * path; the activations stand in for the post-attention rows.
 *
 *   stack_host bench <layers> <H> <E> <k> <I> <bits> <prefill> <decode> <seed>
 *       generates <layers> layers on the GPU with the library's generator and
 *       quantiser (qg_randn_device, qgql_quantize_device; layer l uses
 *       generator seed <seed>*1000+l, streams 0 router, 1 gate_up, 2 down),
 *       then runs a prefill of <prefill> tokens (one call per layer) and
 *       <decode> single-token steps (one call per layer per step) and prints
 *       one JSON line: MoE tokens/s (time inside qgmoe_forward) and the whole
 *       loop's tokens/s.
 *   stack_host check <layer.safetensors> <prefix> <top_k> <x.f32> <T> <out.f32> <idx.i32>
 *       creates the layer from the file, runs one qgmoe_forward on x [T, H]
 *       and writes out [T, H] and the selected experts [T, k].
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <cuda_runtime_api.h>

#include "qgmoe.h"

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static int fail(const char *what, int rc) {
    fprintf(stderr, "%s: %s (%d): %s\n", what, qgmoe_strerror(rc), rc, qgmoe_last_error());
    return 1;
}

#define CK(call)                                  \
    do {                                          \
        int rc_ = (call);                         \
        if (rc_ != QGMOE_OK) return fail(#call, rc_); \
    } while (0)
#define CKC(call)                                                            \
    do {                                                                     \
        cudaError_t e_ = (call);                                             \
        if (e_ != cudaSuccess) {                                             \
            fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));      \
            return 1;                                                        \
        }                                                                    \
    } while (0)

/* h = x / sqrt(mean(x^2) + 1e-6), row by row (the block's pre-MLP norm
 * without its weight vector). */
static void rmsnorm_rows(const float *x, float *h, int T, int H) {
    for (int t = 0; t < T; t++) {
        const float *r = x + (size_t)t * H;
        double ss = 0;
        for (int i = 0; i < H; i++) ss += (double)r[i] * r[i];
        const float inv = (float)(1.0 / sqrt(ss / H + 1e-6));
        for (int i = 0; i < H; i++) h[(size_t)t * H + i] = r[i] * inv;
    }
}

static int bench(int argc, char **argv) {
    if (argc != 11) return 2;
    const int L = atoi(argv[2]), H = atoi(argv[3]), E = atoi(argv[4]), k = atoi(argv[5]),
              I = atoi(argv[6]), bits = atoi(argv[7]), P = atoi(argv[8]), D = atoi(argv[9]);
    const unsigned long long seed = strtoull(argv[10], NULL, 10);
    if (L <= 0 || P <= 0 || D < 0 || (bits != 8 && bits != 4)) return 2;
    const size_t gu_rows = (size_t)E * 2 * I, dn_rows = (size_t)E * H;
    const size_t gu_n = gu_rows * H, dn_n = dn_rows * I;
    const size_t big = gu_n > dn_n ? gu_n : dn_n;
    float *w = NULL, *router = NULL;
    CKC(cudaMalloc((void **)&w, sizeof(float) * big));
    CKC(cudaMalloc((void **)&router, sizeof(float) * (size_t)E * H));
    unsigned char *gu_q = NULL, *dn_q = NULL;
    unsigned short *gu_s = NULL, *dn_s = NULL;
    CKC(cudaMalloc((void **)&gu_q, gu_n * bits / 8));
    CKC(cudaMalloc((void **)&dn_q, dn_n * bits / 8));
    CKC(cudaMalloc((void **)&gu_s, sizeof(unsigned short) * (gu_n / 32)));
    CKC(cudaMalloc((void **)&dn_s, sizeof(unsigned short) * (dn_n / 32)));
    qgmoe_t **layers = (qgmoe_t **)calloc((size_t)L, sizeof(qgmoe_t *));
    const double tg = now_s();
    for (int l = 0; l < L; l++) {
        const unsigned long long ls = seed * 1000ULL + (unsigned long long)l;
        CK(qg_randn_device(ls, 0, 0, (long long)E * H, 0.02f, router, NULL));
        CK(qg_randn_device(ls, 1, 0, (long long)gu_n, 0.02f, w, NULL));
        CK(qgql_quantize_device(bits, (int)gu_rows, H, w, gu_q, NULL, gu_s, NULL));
        CK(qg_randn_device(ls, 2, 0, (long long)dn_n, 0.02f, w, NULL));
        CK(qgql_quantize_device(bits, (int)dn_rows, I, w, dn_q, NULL, dn_s, NULL));
        CKC(cudaDeviceSynchronize());
        qgmoe_desc d;
        memset(&d, 0, sizeof d);
        d.n_embed = H;
        d.n_experts = E;
        d.top_k = k;
        d.n_moe_mlp = I;
        d.bits = bits;
        d.router_mode = QGMOE_ROUTER_TOPK;
        d.scale_dtype = QGMOE_SCALE_F16;
        d.weights_on_device = 1;
        d.device = 0;
        d.router = router;
        d.gate_up_q = gu_q;
        d.gate_up_scale = gu_s;
        d.down_q = dn_q;
        d.down_scale = dn_s;
        CK(qgmoe_create(&d, &layers[l]));
    }
    const double gen_s = now_s() - tg;
    cudaFree(w);
    cudaFree(router);
    cudaFree(gu_q);
    cudaFree(dn_q);
    cudaFree(gu_s);
    cudaFree(dn_s);
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);

    float *x = (float *)malloc(sizeof(float) * (size_t)P * H);
    float *h = (float *)malloc(sizeof(float) * (size_t)P * H);
    float *o = (float *)malloc(sizeof(float) * (size_t)P * H);
    /* activations: N(0,1) rows from the same generator (stream 100), via the device */
    float *xd = NULL;
    CKC(cudaMalloc((void **)&xd, sizeof(float) * (size_t)P * H));
    CK(qg_randn_device(seed, 100, 0, (long long)P * H, 1.0f, xd, NULL));
    CKC(cudaMemcpy(x, xd, sizeof(float) * (size_t)P * H, cudaMemcpyDeviceToHost));
    cudaFree(xd);

    /* one untimed pass to warm every layer (workspace, graphs) at both sizes */
    for (int l = 0; l < L; l++) {
        rmsnorm_rows(x, h, P, H);
        CK(qgmoe_forward(layers[l], h, P, o, NULL, NULL));
        CK(qgmoe_forward(layers[l], h, 1, o, NULL, NULL));
        CK(qgmoe_forward(layers[l], h, 1, o, NULL, NULL));
    }
    /* prefill: P tokens through every layer */
    double moe_p = 0, t0 = now_s();
    for (int l = 0; l < L; l++) {
        rmsnorm_rows(x, h, P, H);
        const double a = now_s();
        CK(qgmoe_forward(layers[l], h, P, o, NULL, NULL));
        moe_p += now_s() - a;
        for (size_t i = 0; i < (size_t)P * H; i++) x[i] += o[i];
    }
    const double all_p = now_s() - t0;
    /* decode: D steps of one token (the last prefill row carries on) */
    float *xt = x + (size_t)(P - 1) * H;
    double moe_d = 0;
    t0 = now_s();
    for (int step = 0; step < D; step++) {
        for (int l = 0; l < L; l++) {
            rmsnorm_rows(xt, h, 1, H);
            const double a = now_s();
            CK(qgmoe_forward(layers[l], h, 1, o, NULL, NULL));
            moe_d += now_s() - a;
            for (int i = 0; i < H; i++) xt[i] += o[i];
        }
    }
    const double all_d = now_s() - t0;
    int finite = 1;
    for (size_t i = 0; i < (size_t)P * H; i++)
        if (!isfinite(x[i])) finite = 0;
    printf("{\"layers\": %d, \"H\": %d, \"E\": %d, \"top_k\": %d, \"I\": %d, \"bits\": %d, "
           "\"prefill_tokens\": %d, \"decode_steps\": %d, \"weights_gb\": %.2f, "
           "\"create_s\": %.2f, "
           "\"prefill_moe_tokens_per_s\": %.1f, \"prefill_loop_tokens_per_s\": %.1f, "
           "\"prefill_moe_ms_per_layer\": %.4f, "
           "\"decode_moe_tokens_per_s\": %.2f, \"decode_loop_tokens_per_s\": %.2f, "
           "\"decode_moe_us_per_layer\": %.2f, \"finite\": %s, \"device_free_gb\": %.1f}\n",
           L, H, E, k, I, bits, P, D,
           (double)L * ((double)(gu_n + dn_n) * bits / 8 + (double)(gu_n + dn_n) / 32 * 2 +
                        (double)E * H * 4) / 1e9,
           gen_s, P / moe_p, P / all_p, 1e3 * moe_p / L, D > 0 ? D / moe_d : 0.0,
           D > 0 ? D / all_d : 0.0, D > 0 ? 1e6 * moe_d / ((double)D * L) : 0.0,
           finite ? "true" : "false", free_b / 1e9);
    for (int l = 0; l < L; l++) qgmoe_destroy(layers[l]);
    free(layers);
    free(x);
    free(h);
    free(o);
    return 0;
}

static int check(int argc, char **argv) {
    if (argc != 9) return 2;
    qgmoe_file_t *f = NULL;
    CK(qgmoe_file_open(argv[2], &f));
    qgmoe_desc d;
    CK(qgmoe_file_layer_desc(f, argv[3], atoi(argv[4]), QGMOE_ROUTER_TOPK, 0, &d));
    qgmoe_t *m = NULL;
    CK(qgmoe_create(&d, &m));
    qgmoe_file_close(f);
    const int T = atoi(argv[6]), H = d.n_embed, k = d.top_k;
    float *x = (float *)malloc(sizeof(float) * (size_t)T * H);
    float *out = (float *)malloc(sizeof(float) * (size_t)T * H);
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)T * k);
    FILE *fx = fopen(argv[5], "rb");
    if (!fx || fread(x, sizeof(float), (size_t)T * H, fx) != (size_t)T * H) return 3;
    fclose(fx);
    CK(qgmoe_forward(m, x, T, out, idx, NULL));
    FILE *fo = fopen(argv[7], "wb");
    FILE *fi = fopen(argv[8], "wb");
    if (!fo || !fi) return 3;
    fwrite(out, sizeof(float), (size_t)T * H, fo);
    fwrite(idx, sizeof(int32_t), (size_t)T * k, fi);
    fclose(fo);
    fclose(fi);
    qgmoe_destroy(m);
    free(x);
    free(out);
    free(idx);
    printf("ok T=%d H=%d k=%d\n", T, H, k);
    return 0;
}

int main(int argc, char **argv) {
    if (argc >= 2 && !strcmp(argv[1], "bench")) return bench(argc, argv);
    if (argc >= 2 && !strcmp(argv[1], "check")) return check(argc, argv);
    fprintf(stderr,
            "usage: stack_host bench <layers> <H> <E> <k> <I> <bits> <prefill> <decode> <seed>\n"
            "       stack_host check <file> <prefix> <top_k> <x.f32> <T> <out.f32> <idx.i32>\n");
    return 2;
}
