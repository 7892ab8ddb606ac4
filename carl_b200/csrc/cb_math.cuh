// Device/host vector math for the tick.
//
// V3 is a packed 12-byte float triple and Q4 a quaternion (x, y, z, w).  Every
// operation evaluates its float arithmetic in the same order, with the same
// intrinsics, as the reference's math layer (jwmccarthy/CARL
// include/Cuda/Math.cuh:31-331): the tick is compiled with --fmad=false, so equal
// inputs give bit-equal outputs to the reference build.  Examples of order that
// matters: dot = (x*a.x + y*a.y) + z*a.z; Q4 dot = (x*b.x + z*b.z) + (y*b.y + w*b.w);
// normalise divides each component by the length; rotation uses the
// two-cross-product form v + t*w + q x t with t = (q x v) * (2 / |q|^2).
#pragma once

#include <cmath>
#include <cstdint>

#if defined(__CUDACC__)
#define CB_HD __host__ __device__ __forceinline__
#define CB_D __device__ __forceinline__
#else
#define CB_HD inline
#define CB_D inline
#endif

struct V3
{
    float x, y, z;
};

struct Q4
{
    float x, y, z, w;
};

struct I3
{
    int x, y, z;
};

CB_HD V3 v3(float x, float y, float z) { return V3{ x, y, z }; }
CB_HD V3 v3zero() { return V3{ 0.f, 0.f, 0.f }; }
CB_HD V3 v3fill(float s) { return V3{ s, s, s }; }

CB_HD V3 operator+(V3 a, V3 b) { return V3{ a.x + b.x, a.y + b.y, a.z + b.z }; }
CB_HD V3 operator-(V3 a, V3 b) { return V3{ a.x - b.x, a.y - b.y, a.z - b.z }; }
CB_HD V3 operator*(V3 a, V3 b) { return V3{ a.x * b.x, a.y * b.y, a.z * b.z }; }
CB_HD V3 operator/(V3 a, V3 b) { return V3{ a.x / b.x, a.y / b.y, a.z / b.z }; }
CB_HD V3 operator+(V3 a, float s) { return V3{ a.x + s, a.y + s, a.z + s }; }
CB_HD V3 operator-(V3 a, float s) { return V3{ a.x - s, a.y - s, a.z - s }; }
CB_HD V3 operator*(V3 a, float s) { return V3{ a.x * s, a.y * s, a.z * s }; }
CB_HD V3 operator/(V3 a, float s) { return V3{ a.x / s, a.y / s, a.z / s }; }

CB_HD V3 neg(V3 a) { return V3{ -a.x, -a.y, -a.z }; }
CB_HD V3 vabs(V3 a) { return V3{ fabsf(a.x), fabsf(a.y), fabsf(a.z) }; }
CB_HD V3 vsign(V3 a)
{
    return V3{ a.x >= 0.f ? 1.f : -1.f, a.y >= 0.f ? 1.f : -1.f, a.z >= 0.f ? 1.f : -1.f };
}
CB_HD float dot(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
CB_HD V3 cross(V3 a, V3 b)
{
    return V3{ a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x };
}
CB_HD float lensq(V3 a) { return dot(a, a); }
CB_HD float len(V3 a) { return sqrtf(lensq(a)); }
CB_HD V3 normalized(V3 a) { return a / len(a); }
CB_HD V3 vmax(V3 a, V3 b) { return V3{ fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z) }; }
CB_HD V3 vmin(V3 a, V3 b) { return V3{ fminf(a.x, b.x), fminf(a.y, b.y), fminf(a.z, b.z) }; }
CB_HD V3 vmax(V3 a, float s) { return V3{ fmaxf(a.x, s), fmaxf(a.y, s), fmaxf(a.z, s) }; }
CB_HD V3 vmin(V3 a, float s) { return V3{ fminf(a.x, s), fminf(a.y, s), fminf(a.z, s) }; }
CB_HD bool allGe(V3 a, float s) { return a.x >= s && a.y >= s && a.z >= s; }
CB_HD int argMax(V3 a) { return a.y > a.x ? (a.y > a.z ? 1 : 2) : (a.x > a.z ? 0 : 2); }
CB_HD float vget(V3 a, int i) { return i == 0 ? a.x : (i == 1 ? a.y : a.z); }
CB_HD void vset(V3& a, int i, float s)
{
    if (i == 0) a.x = s;
    else if (i == 1) a.y = s;
    else a.z = s;
}
CB_HD V3 axisVec(int i)
{
    return V3{ i == 0 ? 1.f : 0.f, i == 1 ? 1.f : 0.f, i == 2 ? 1.f : 0.f };
}

CB_HD float clampf(float value, float lo, float hi) { return fmaxf(lo, fminf(hi, value)); }

// ---- quaternions -------------------------------------------------------------

CB_HD Q4 operator*(Q4 q, float s) { return Q4{ q.x * s, q.y * s, q.z * s, q.w * s }; }
CB_HD V3 qvec(Q4 q) { return V3{ q.x, q.y, q.z }; }
CB_HD float qdot(Q4 a, Q4 b) { return (a.x * b.x + a.z * b.z) + (a.y * b.y + a.w * b.w); }
CB_HD float qlensq(Q4 q) { return qdot(q, q); }
CB_HD Q4 qnormalized(Q4 q) { return q * (1.f / sqrtf(qlensq(q))); }
CB_HD Q4 qconj(Q4 q) { return Q4{ -q.x, -q.y, -q.z, q.w }; }
CB_HD Q4 qyaw(float a) { return Q4{ 0.f, 0.f, sinf(a / 2), cosf(a / 2) }; }

// Hamilton product a * b.
CB_HD Q4 qmul(Q4 a, Q4 b)
{
    return Q4{
        (a.w * b.x - a.z * b.y) + (a.x * b.w + a.y * b.z),
        (a.w * b.y - a.x * b.z) + (a.y * b.w + a.z * b.x),
        (a.w * b.z - a.y * b.x) + (a.z * b.w + a.x * b.y),
        (a.w * b.w - a.z * b.z) - (a.x * b.x + a.y * b.y)
    };
}

CB_HD V3 rotate(Q4 q, V3 v)
{
    const V3 u = qvec(q);
    const V3 t = cross(u, v) * (2.f / qlensq(q));
    return v + t * q.w + cross(u, t);
}

CB_HD V3 unrotate(Q4 q, V3 v) { return rotate(qconj(q), v); }

// Quaternion from the columns of a rotation matrix (forward, right, up).
CB_HD Q4 qfromAxes(V3 f, V3 r, V3 u)
{
    const float trace = f.x + r.y + u.z;
    const V3 t = V3{ f.x, r.y, u.z } * 2.f + (1.f - trace);
    const V3 sum = { r.z + u.y, u.x + f.z, f.y + r.x };
    const V3 diff = { r.z - u.y, u.x - f.z, f.y - r.x };

    if (trace > 0.f)
    {
        const float tw = 1.f + trace;
        return Q4{ diff.x, diff.y, diff.z, tw } * (.5f / sqrtf(tw));
    }
    switch (argMax(t))
    {
    case 0: return Q4{ t.x, sum.z, sum.y, diff.x } * (.5f / sqrtf(t.x));
    case 1: return Q4{ sum.z, t.y, sum.x, diff.y } * (.5f / sqrtf(t.y));
    default: return Q4{ sum.y, sum.x, t.z, diff.z } * (.5f / sqrtf(t.z));
    }
}

// Rodrigues rotation of v about unit axis ax by angle a.
CB_HD V3 rotateAbout(V3 v, V3 ax, float a)
{
    return v * cosf(a) + cross(ax, v) * sinf(a) + ax * (dot(ax, v) * (1.f - cosf(a)));
}

#if defined(__CUDACC__)
// Fast-intrinsic sine/cosine (the reference uses __sincosf for steering).
CB_D void fast_sincos(float x, float* s, float* c) { __sincosf(x, s, c); }
#endif
