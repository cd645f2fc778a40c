// f32 instantiations of the RACE attention kernels for head dim 32.
#define RACE_ELEM float
#define RACE_DIM 32
#define RACE_TABLE_FN kernels_f32_d32
#include "race_instances.inc"
