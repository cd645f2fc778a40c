// float32 instantiations of the RACE attention kernels.
#define RACE_ELEM float
#define RACE_TABLE_FN kernels_f32
#include "race_instances.inc"
