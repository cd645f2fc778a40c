// f32 instantiations of the RACE attention kernels for head dim 64.
#define RACE_ELEM float
#define RACE_DIM 64
#define RACE_TABLE_FN kernels_f32_d64
#include "race_instances.inc"
