/*
 * Pre-include (g++ -include) that lets the reference's CUDA device headers
 * compile as ordinary host C++ for the CPU oracle.
 *
 * It maps the handful of CUDA device built-ins those headers use onto host
 * equivalents:
 *   __ldg(p)           -> *p                       (read-only cache load)
 *   rsqrtf(x)          -> 1 / sqrtf(x)             (device: approximate)
 *   __sincosf(x,&s,&c) -> sinf / cosf              (device: fast intrinsic)
 *   atomicAdd(p, v)    -> non-atomic add; the CPU driver processes each car's
 *                         triangle candidates serially, so slots are assigned
 *                         in candidate order
 *   float4/int4/int2   -> plain structs
 * and turns the execution-space qualifiers into nothing.  Together with the
 * host-memory hip runtime in refshim/hip/ this builds the reference's own
 * physics (include/Physics/**, include/State/**, include/Arena/**) unchanged.
 * TEST INFRASTRUCTURE: only tests, smoke() and bench.py's CPU baseline use it.
 */
#pragma once

#include <algorithm>
#include <array>
#include <bit>
#include <cassert>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <fstream>
#include <initializer_list>
#include <map>
#include <optional>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#define CARL_USE_HIP 1

#define __host__
#define __device__
#define __global__
#define __constant__
#define __shared__
#define __forceinline__ inline
#define __noinline__
#define __restrict__ __restrict
#define __align__(n) alignas(n)

struct float4 { float x, y, z, w; };
struct int4 { int x, y, z, w; };
struct int2 { int x, y; };
struct dim3
{
    unsigned x = 1, y = 1, z = 1;
    dim3() = default;
    dim3(unsigned a, unsigned b = 1, unsigned c = 1) : x(a), y(b), z(c) {}
};

template <class T>
inline T __ldg(const T* p) { return *p; }

inline float rsqrtf(float x) { return 1.f / sqrtf(x); }

inline void __sincosf(float x, float* s, float* c)
{
    *s = sinf(x);
    *c = cosf(x);
}

inline int atomicAdd(int* p, int v)
{
    const int old = *p;
    *p = old + v;
    return old;
}
