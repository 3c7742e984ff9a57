// Verify kernel variants for activation dtype __half.
#include "verify_launch.cuh"

GDN_RSSM_VERIFY_TU(__half, f16)
