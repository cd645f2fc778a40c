// bfloat16 instantiations of the RACE attention kernels (fp32 accumulation).
#define RACE_ELEM __nv_bfloat16
#define RACE_TABLE_FN kernels_bf16
#include "race_instances.inc"
