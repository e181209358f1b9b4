/* inzg_host.h -- host-side tools of libinzg: the public declarations live in include/inzg_tools.h. */
#ifndef INZG_HOST_H
#define INZG_HOST_H

#include "../../../include/inzg_tools.h"

#define INZG_T_F16 1
#define INZG_T_Q4L 102
#define INZG_T_Q8G 103

#endif
