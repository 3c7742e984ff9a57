// Verify kernel variants for activation dtype __nv_bfloat16.
#include "verify_launch.cuh"

GDN_RSSM_VERIFY_TU(__nv_bfloat16, bf16)
