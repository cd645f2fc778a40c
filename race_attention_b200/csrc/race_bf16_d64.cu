// bf16 instantiations of the RACE attention kernels for head dim 64.
#define RACE_ELEM __nv_bfloat16
#define RACE_DIM 64
#define RACE_TABLE_FN kernels_bf16_d64
#include "race_instances.inc"
