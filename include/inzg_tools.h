/*
 * inzg_tools.h -- host-side tools exported by libinzg next to the MoE C ABI (inzg.h): the engine's expert
 * quantizer and the seeded synthetic inputs of the benchmark configurations. No CUDA types.
 *
 * inzg_quantize* / inzg_encode_expert* replace the converter's expert path (encode, src/convert.c:190-200, over
 * inz_quantize, src/quant.c:422-556) with a GPU encoder that writes byte-identical blobs; inzg_synth_* draw from the
 * LCG + Box-Muller normal of the reference's tests (tests/test_quant.c:10-17).
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
/* bytes of one expert blob (convert_expert_blob_bytes, src/convert.c:179-182) */
INZG_API uint64_t inzg_blob_bytes(int type, int H, int FF);

/* ---- The expert quantizer, on the GPU (the current CUDA device). It writes the bytes of the reference quantizer
 * (inz_quantize, src/quant.c:422-556) without an importance matrix, as the converter encodes experts
 * (src/convert.c:190-200). Each returns 0, or -1 for an unsupported type or shape, a rotation block other than
 * 64/128/256, or a failed CUDA call. */

/* W_dev [rows][cols] fp32 -> out_dev (inzg_qmat_bytes bytes), Q4L or Q8G; rot_block 0 = auto, < 0 = none
 * (Q8G: rotated only for rot_block > 0); rot_seed 0 = the reference's default 0x5EED. Ordered on `stream`
 * (cudaStream_t, NULL = legacy default); returns after the stream has finished. */
INZG_API int inzg_quantize_device(const float *W_dev, int rows, int cols, int type, int rot_block, uint32_t rot_seed,
                                  void *out_dev, void *stream);
/* the same from and to host memory */
INZG_API int inzg_quantize(const float *W, int rows, int cols, int type, int rot_block, uint32_t rot_seed, void *out);
/* n expert blobs from device fp32 gate|up [n][2FF][H] and down [n][H][FF] (the converter's recipe: Q4L with the
 * automatic rotation, Q8G rotated with the automatic block, src/convert.c:157, 190-200, 565-584) */
INZG_API int inzg_encode_experts_device(const float *gu_dev, const float *dn_dev, int n, int type, int H, int FF,
                                        void *blobs_dev, void *stream);
/* one expert blob from host fp32 gate|up and down */
INZG_API int inzg_encode_expert(const float *GU, const float *D, int type, int H, int FF, void *blob);
/* experts [e0, e1) of a synthetic layer: drawn on the host (the reference tests' exact stream) and encoded on the GPU;
 * blobs [e1-e0][blob_bytes] in host memory */
INZG_API int inzg_synth_layer_blobs(uint64_t seed, int type, int H, int FF, int e0, int e1, void *blobs);
/* only the listed experts generated; the others get valid headers and a zero payload */
INZG_API int inzg_synth_layer_blobs_subset(uint64_t seed, int type, int H, int FF, int E, const int32_t *experts,
                                           int n_experts, void *blobs);
/* the fp32 draws of experts [e0, e0 + n) on the GPU: gu_dev [n][2FF][H], dn_dev [n][H][FF] (the same LCG stream as
 * inzg_synth_expert, with CUDA's double log/cos/sqrt in the Box-Muller step: see inzg_synth_layer_blobs_device) */
INZG_API int inzg_synth_experts_device(uint64_t seed, int H, int FF, int e0, int n, float *gu_dev, float *dn_dev,
                                       void *stream);
/* experts [e0, e1) drawn AND encoded on the GPU into device memory blobs_dev [e1-e0][blob_bytes]: the same LCG
 * stream, with CUDA's double log/cos/sqrt in the Box-Muller step (a float draw can differ from the host stream's
 * where the double result lies within an ulp or two of a float rounding boundary) */
INZG_API int inzg_synth_layer_blobs_device(uint64_t seed, int type, int H, int FF, int e0, int e1, void *blobs_dev,
                                           void *stream);

/* ---- Roofline probe (the counterpart of the reference's bandwidth probe in its diagnostics, src/diag.c:363-394):
 * the int8 tensor-pipe throughput of `device` measured with tcgen05.mma kind::i8 (128 x 256 x 32 MMAs from shared
 * memory on every SM, `iters` x 4 per SM). *tops = int8 tera-operations per second (2 per multiply-add), *ms the
 * timed kernel's duration (optional). Returns 0, or -1 on a CUDA failure or a wait that ran out. */
INZG_API int inzg_probe_tensor_i8(int device, int iters, double *tops, double *ms);
/* the architecture of the library's kernels as loaded on `device` (cudaFuncGetAttributes): binaryVersion 100 for
 * sm_100 SASS; ptxVersion the PTX ISA target. Returns 0, or -1 without a usable device. */
INZG_API int inzg_kernel_arch(int device, int *binary_version, int *ptx_version);

#ifdef __cplusplus
}
#endif
#endif
