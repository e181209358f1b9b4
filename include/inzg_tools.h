/*
 * inzg_tools.h -- host-side tools exported by libinzg next to the MoE C ABI (inzg.h): the engine's expert
 * quantizer and the seeded synthetic inputs of the benchmark configurations. No CUDA types.
 *
 * inzg_quantize / inzg_encode_expert replace the converter's expert path (encode, src/convert.c:190-200, over
 * inz_quantize, src/quant.c:422-556) and write byte-identical blobs; inzg_synth_* draw from the LCG + Box-Muller
 * normal of the reference's tests (tests/test_quant.c:10-17).
 */
#ifndef INZG_TOOLS_H
#define INZG_TOOLS_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define INZG_API __attribute__((visibility("default")))
#else
#define INZG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* generator state after n_normals draws of randn (each draw takes two LCG steps) */
INZG_API uint64_t inzg_synth_jump(uint64_t state, uint64_t n_normals);
/* out[i] = randn * scale for i < n; returns the new state */
INZG_API uint64_t inzg_synth_randn(uint64_t state, int64_t n, float scale, float *out);
/* fp32 -> IEEE half, round to nearest even (the reference's inz_f32_to_f16, src/util.c:117) */
INZG_API uint16_t inzg_f32_to_f16(float f);
/* expert e of a layer seeded `seed`: gu [2FF][H] (gate rows then up rows), dn [H][FF], N(0, 1/H) */
INZG_API void inzg_synth_expert(uint64_t seed, int H, int FF, int e, float *gu, float *dn);
/* router [E][H] f16 from N(0, 0.02^2) */
INZG_API void inzg_synth_router(uint64_t seed, int E, int H, uint16_t *w);
/* hidden states [n][H] from N(0, 1), each row RMS-normalised */
INZG_API void inzg_synth_hidden(uint64_t seed, int n, int H, float *x);

/* bytes of one quantized matrix incl. its 64-byte header (inz_qmat_bytes, src/quant.c:30-36) */
INZG_API size_t inzg_qmat_bytes(int type, int rows, int cols);
/* automatic rotation block (inz_auto_rot_block, src/quant.c:166-170) */
INZG_API int inzg_auto_rot_block(int cols);
/* quantize W [rows][cols] to Q4L / Q8G (inz_quantize, src/quant.c:422-556; rot_block 0 = auto, < 0 = none);
 * returns 0, or -1 for an unsupported type or shape */
INZG_API int inzg_quantize(const float *W, int rows, int cols, int type, int rot_block, uint32_t rot_seed, int threads,
                           void *out);
/* bytes of one expert blob (convert_expert_blob_bytes, src/convert.c:179-182) */
INZG_API uint64_t inzg_blob_bytes(int type, int H, int FF);
/* one expert blob from fp32 gate|up and down (the converter's recipe, src/convert.c:190-200, 565-584) */
INZG_API int inzg_encode_expert(const float *GU, const float *D, int type, int H, int FF, void *blob);
/* experts [e0, e1) of a synthetic layer, generated and encoded in parallel: blobs [e1-e0][blob_bytes] */
INZG_API int inzg_synth_layer_blobs(uint64_t seed, int type, int H, int FF, int e0, int e1, void *blobs);
/* only the listed experts generated (in parallel); the others get valid headers and a zero payload */
INZG_API int inzg_synth_layer_blobs_subset(uint64_t seed, int type, int H, int FF, int E, const int32_t *experts,
                                           int n_experts, void *blobs);

#ifdef __cplusplus
}
#endif
#endif
