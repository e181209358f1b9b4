/* moe_host.c -- a C host of libinzg, the way the reference engine (C11) would drive it: open the model's GGUF, create
 * a context, fill the expert pool of every layer from the file, then run one MoE forward on a small batch.
 * Built and run by tests/test_abi.py to show the public header compiles as plain C and links; the router weights
 * are zeros here (a real engine passes its layer's F16 router view).
 *
 *   moe_host <model.gguf> [hidden ff n_expert topk]
 *
 * Exit status: 0 forward done; 1 bad usage or GGUF; 2 no context (e.g. no CUDA device); 3 a later call failed. */
#include <stdio.h>
#include <stdlib.h>

#include "inzg.h"

int main(int argc, char **argv) {
    if (argc != 2 && argc != 6) {
        fprintf(stderr, "usage: %s <model.gguf> [hidden ff n_expert topk]\n", argv[0]);
        return 1;
    }
    inzg_gguf_info gi;
    char err[256];
    inzg_gguf *g = inzg_gguf_open(argv[1], &gi, err, sizeof(err));
    if (!g) {
        fprintf(stderr, "%s\n", err);
        return 1;
    }
    printf("gguf: expert_type %d blob_bytes %llu layers %d mtp %d\n", gi.expert_type,
           (unsigned long long)gi.blob_bytes, gi.n_layers, gi.has_mtp);
    inzg_config cfg = {2048, 640, 512, 10, 8, gi.n_layers + gi.has_mtp, 0};
    if (argc == 6) {
        cfg.hidden = atoi(argv[2]);
        cfg.ff = atoi(argv[3]);
        cfg.n_expert = atoi(argv[4]);
        cfg.topk = atoi(argv[5]);
    }
    inzg_status st;
    inzg_ctx *ctx = inzg_create(&cfg, &st);
    if (!ctx) {
        printf("inzg_create: %s\n", inzg_status_str(st));
        inzg_gguf_close(g);
        return 2;
    }
    int rc = 0;
    uint16_t *router = calloc((size_t)cfg.n_expert * cfg.hidden, sizeof(uint16_t));
    float *x = calloc((size_t)4 * cfg.hidden, sizeof(float)), *y = calloc((size_t)4 * cfg.hidden, sizeof(float));
    for (int l = 0; l < cfg.n_layers && !rc; l++)
        if (inzg_pool_add_layer_gguf(ctx, l, g, l) != INZG_OK || inzg_set_router(ctx, l, router, cfg.n_expert, cfg.hidden) != INZG_OK) {
            fprintf(stderr, "layer %d: %s\n", l, inzg_last_error(ctx));
            rc = 3;
        }
    if (!rc && inzg_moe_forward(ctx, 0, 4, x, y, NULL) != INZG_OK) {
        fprintf(stderr, "forward: %s\n", inzg_last_error(ctx));
        rc = 3;
    }
    if (!rc) {
        double sum = 0;
        for (int i = 0; i < 4 * cfg.hidden; i++) sum += y[i];
        printf("forward: y sum %.6g\n", sum);
    }
    free(router);
    free(x);
    free(y);
    inzg_destroy(ctx);
    inzg_gguf_close(g);
    return rc;
}
