/* A plain-C host of the C ABI, the way the cgo shim uses it (C99, no C++):
 * maps a layer file, builds the layer descriptor, and tries to create the
 * layer.  Compiled and run by tests/test_abi.py; needs no GPU (create then
 * reports that no sm_100 device is present, or succeeds on a B200).
 * usage: abi_host <file.safetensors> <prefix> <top_k> */
#include <stdio.h>
#include <stdlib.h>

#include "qgmoe.h"

int main(int argc, char **argv) {
    if (argc != 4) return 2;
    qgmoe_file_t *f = NULL;
    int rc = qgmoe_file_open(argv[1], &f);
    if (rc != QGMOE_OK) {
        printf("open %d %s\n", rc, qgmoe_last_error());
        return 1;
    }
    int32_t dtype = -1, rank = 0;
    int64_t shape[8] = {0};
    const void *data = NULL;
    int64_t nbytes = 0;
    char name[256];
    snprintf(name, sizeof name, "%sgate.weight", argv[2]);
    rc = qgmoe_file_tensor(f, name, &dtype, &rank, shape, &data, &nbytes);
    printf("router rc=%d dtype=%d rank=%d shape=%lld,%lld bytes=%lld\n", rc, dtype, rank,
           (long long)shape[0], (long long)shape[1], (long long)nbytes);
    qgmoe_desc d;
    rc = qgmoe_file_layer_desc(f, argv[2], atoi(argv[3]), QGMOE_ROUTER_TOPK, 0, &d);
    printf("desc rc=%d H=%d E=%d k=%d I=%d Is=%d bits=%d scale=%d\n", rc, d.n_embed, d.n_experts,
           d.top_k, d.n_moe_mlp, d.n_shared_mlp, d.bits, d.scale_dtype);
    qgmoe_t *h = NULL;
    rc = qgmoe_create(&d, &h);
    printf("create rc=%d (%s)\n", rc, qgmoe_strerror(rc));
    if (h) qgmoe_destroy(h);
    qgmoe_file_close(f);
    return 0;
}
