// Host versions of the device intrinsics the product's physics headers use,
// mapped as in the reference's host build (oracle/refshim/carl_host_shim.h):
// rsqrtf -> 1/sqrtf, __sincosf -> sinf/cosf.  TEST INFRASTRUCTURE.
#pragma once
#include <cmath>

inline float rsqrtf(float x) { return 1.f / sqrtf(x); }
inline void fast_sincos(float x, float* s, float* c)
{
    *s = sinf(x);
    *c = cosf(x);
}
