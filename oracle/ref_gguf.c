/* ref_gguf.c -- TEST INFRASTRUCTURE ONLY: the reference's own GGUF reader and writer (src/gguf.c, compiled from the
 * reference tree by oracle/Makefile into _ref/libinzref_gguf.so) behind two calls the parity tests of the product's
 * GGUF expert reader (inferenz_b200/csrc/host/gguf.c) use:
 *
 *   ref_gguf_tensor  -- what setup_experts sees for one tensor name (src/engine.c:337-350): gguf_open, the expert
 *                       type and blob size with the engine's defaults, gguf_find_tensor's absolute offset and size;
 *   ref_gguf_write   -- a model-shaped file written by the reference's writer: metadata of several types, a leading
 *                       non-expert tensor, then the per-layer "blk.%d.experts" tensors and optionally "mtp.experts",
 *                       experts last as the converter writes them (src/convert.c:461-466).
 */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "gguf.h"

#define REF_T_F32 0
#define REF_T_EXPERTS 120 /* INZ_T_EXPERTS, src/quant.h:36 */
#define REF_T_Q8G 103

__attribute__((visibility("default"))) int ref_gguf_tensor(const char *path, const char *name, uint64_t *abs_offset,
                                                           uint64_t *nbytes, int64_t *expert_type,
                                                           int64_t *blob_bytes, uint64_t *alignment, char *err,
                                                           size_t err_len) {
    gguf_file *g = gguf_open(path, err, err_len);
    if (!g) return 1;
    *expert_type = gguf_get_int(g, "inz.expert_type", REF_T_Q8G);
    *blob_bytes = gguf_get_int(g, "inz.expert_blob_bytes", 0);
    *alignment = g->alignment;
    const gguf_tensor *t = gguf_find_tensor(g, name);
    int rc = 2;
    if (t) {
        *abs_offset = g->data_offset + t->offset;
        *nbytes = t->nbytes;
        rc = 0;
    }
    gguf_close(g);
    return rc;
}

/* blobs: the expert tensors of every layer written (n_layers, then mtp.experts), n_expert * blob_bytes bytes each, back
 * to back; extra_floats: length of the leading F32 tensor "token_embd.weight" (0: none). */
__attribute__((visibility("default"))) int ref_gguf_write(const char *path, uint64_t alignment, int n_layers, int mtp,
                                                          uint32_t expert_type, uint64_t blob_bytes, int n_expert,
                                                          const uint8_t *blobs, uint64_t extra_floats) {
    gguf_writer *w = gguf_writer_new(path, alignment);
    if (!w) return 1;
    static const char *const names[] = {"alpha", "", "gamma"};
    const int32_t ints[3] = {7, -1, 42};
    gguf_w_str(w, "general.architecture", "qwen38flash");
    gguf_w_arr_str(w, "tokenizer.ggml.tokens", names, 3);
    gguf_w_f32(w, "inz.rope_theta", 1.0e6f);
    gguf_w_arr_i32(w, "inz.some_ints", ints, 3);
    gguf_w_bool(w, "inz.flag", true);
    gguf_w_u32(w, "inz.expert_type", expert_type);
    gguf_w_u64(w, "inz.expert_blob_bytes", blob_bytes);
    char name[64];
    const uint64_t layer_bytes = blob_bytes * (uint64_t)n_expert;
    if (extra_floats) {
        const uint64_t ne[1] = {extra_floats};
        gguf_w_tensor(w, "token_embd.weight", REF_T_F32, 1, ne, extra_floats * 4);
    }
    const int nt = n_layers + (mtp ? 1 : 0);
    for (int l = 0; l < nt; l++) {
        const uint64_t ne[2] = {blob_bytes, (uint64_t)n_expert};
        if (l < n_layers) snprintf(name, sizeof(name), "blk.%d.experts", l);
        else snprintf(name, sizeof(name), "mtp.experts");
        gguf_w_tensor(w, name, REF_T_EXPERTS, 2, ne, layer_bytes);
    }
    int ok = gguf_w_header(w);
    if (ok && extra_floats) {
        float v = 0.5f;
        for (uint64_t i = 0; ok && i < extra_floats; i++) ok = gguf_w_data(w, &v, 4);
        ok = ok && gguf_w_tensor_done(w);
    }
    for (int l = 0; ok && l < nt; l++)
        ok = gguf_w_data(w, blobs + (uint64_t)l * layer_bytes, layer_bytes) && gguf_w_tensor_done(w);
    return gguf_writer_close(w) && ok ? 0 : 1;
}
