// Verify kernel variants for activation dtype float.
#include "verify_launch.cuh"

GDN_RSSM_VERIFY_TU(float, f32)
