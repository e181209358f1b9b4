/* inzg_host.h -- host-side tools of libinzg: the public declarations live in include/inzg_tools.h. */
#ifndef INZG_HOST_H
#define INZG_HOST_H

#include "../../../include/inzg_tools.h"

#define INZG_T_F16 1
#define INZG_T_Q4L 102
#define INZG_T_Q8G 103

#ifdef __cplusplus
extern "C" {
#endif

/* experts[i] of a synthetic layer (inzg_synth_expert) into gu + i * 2FF*H and dn + i * H*FF, experts in parallel
 * (OpenMP); internal to libinzg */
void inzg__synth_experts_host(uint64_t seed, int H, int FF, const int32_t *experts, int n, float *gu, float *dn);

#ifdef __cplusplus
}
#endif
#endif
