// Car-vs-car collision for one sim: 15-axis OBB SAT (face axes in Bullet
// units), reference-face clipping or support-point contacts, the two-body
// split-impulse + normal/friction solver, demolitions and bumps.
//
// Follows jwmccarthy/CARL include/Physics/CarCar/{Types,SAT,Clip,Solver,
// Response,Solve}.cuh with the same fp32 operation order.  Pairs are visited in
// the reference's order: for a < b, pair (A = b, B = a).
#pragma once

#include "cb_cararena.cuh"
#include "cb_state.cuh"

namespace cb {

struct Box
{
    V3 cen;
    Q4 rot;
};

CB_D V3 boxAxis(const Box& b, int i) { return rotate(b.rot, axisVec(i)); }

CB_D V3 boxSupport(const Box& b, V3 dir)
{
    const V3 l = unrotate(b.rot, dir);
    const V3 local = { copysignf(CAR_HALF_X, l.x), copysignf(CAR_HALF_Y, l.y), copysignf(CAR_HALF_Z, l.z) };
    return b.cen + rotate(b.rot, local);
}

struct CCContact
{
    V3 carPosA, carPosB, normal;
    float depth;
};

// ---- SAT -------------------------------------------------------------------------------

CB_D void ccEdgeAxis(V3 axis, const Box& A, const Box& B, int axisIdx, Sat& r)
{
    const float ls = lensq(axis);
    if (ls < 1e-12f) return;
    axis = axis * rsqrtf(ls);
    const float ra = dot(vabs(unrotate(A.rot, axis)), carHalfExtents());
    const float ca = dot(A.cen, axis);
    const float rb = dot(vabs(unrotate(B.rot, axis)), carHalfExtents());
    const float cbp = dot(B.cen, axis);
    const float aMin = ca - ra, aMax = ca + ra, bMin = cbp - rb, bMax = cbp + rb;
    if (aMax < bMin || bMax < aMin)
    {
        r.overlap = false;
        return;
    }
    const float depthAB = aMax - bMin;
    const float depthBA = bMax - aMin;
    const float depth = fminf(depthAB, depthBA);
    if (depth * (axisIdx >= 6 ? 1.05f : 1.f) >= r.minPen) return;
    r.minPen = depth;
    r.minAxis = depthAB < depthBA ? neg(axis) : axis;
    r.axisIdx = axisIdx;
}

CB_D Sat carCarSat(const Box& A, const Box& B)
{
    Sat r{ true, 0, 3.402823466e+38f, v3zero() };
    V3 ax[3], bx[3];
    #pragma unroll
    for (int i = 0; i < 3; i++)
    {
        ax[i] = boxAxis(A, i);
        bx[i] = boxAxis(B, i);
    }
    const V3 delta = B.cen * .02f - A.cen * .02f;
    const V3 half = carHalfExtents() * .02f;
    float al[3][3];
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) al[i][j] = fabsf(dot(ax[i], bx[j]));

    #pragma unroll
    for (int i = 0; i < 3; i++)
    {
        const float distance = dot(delta, ax[i]);
        const float radius = vget(half, i) + half.x * al[i][0] + half.y * al[i][1] + half.z * al[i][2];
        const float depth = (radius - fabsf(distance)) * 50.f;
        if (depth < 0.f)
        {
            r.overlap = false;
            return r;
        }
        if (depth < r.minPen)
        {
            r.minPen = depth;
            r.minAxis = distance > 0 ? neg(ax[i]) : ax[i];
            r.axisIdx = i;
        }
    }
    #pragma unroll
    for (int i = 0; i < 3; i++)
    {
        const float distance = dot(delta, bx[i]);
        const float radius = half.x * al[0][i] + half.y * al[1][i] + half.z * al[2][i] + vget(half, i);
        const float depth = (radius - fabsf(distance)) * 50.f;
        if (depth < 0.f)
        {
            r.overlap = false;
            return r;
        }
        if (depth < r.minPen)
        {
            r.minPen = depth;
            r.minAxis = distance > 0 ? neg(bx[i]) : bx[i];
            r.axisIdx = 3 + i;
        }
    }
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++)
        {
            ccEdgeAxis(cross(ax[i], bx[j]), A, B, 6 + i * 3 + j, r);
            if (!r.overlap) return r;
        }
    return r;
}

// ---- contacts ------------------------------------------------------------------------------

// `clip` holds 16 vertices: the two clip polygon buffers, placed by the caller in
// shared memory (indexed by a vertex count, they would otherwise live in local
// memory).  `out` is written only at unrolled constant slots, so the caller's
// array stays in registers.
CB_D int ccContacts(const Sat& s, const Box& A, const Box& B, CCContact* out, V3* clip)
{
    if (s.axisIdx >= 6)
    {
        const V3 pa = boxSupport(A, neg(s.minAxis));
        const V3 pb = boxSupport(B, s.minAxis);
        out[0] = CCContact{ unrotate(A.rot, pa - A.cen), unrotate(B.rot, pb - B.cen), s.minAxis, s.minPen };
        return 1;
    }
    const bool refIsA = s.axisIdx < 3;
    const Box& ref = refIsA ? A : B;
    const Box& inc = refIsA ? B : A;
    const int faceAxis = refIsA ? s.axisIdx : s.axisIdx - 3;

    V3 refNormal = boxAxis(ref, faceAxis);
    if (dot(refNormal, inc.cen - ref.cen) < 0.f) refNormal = neg(refNormal);

    // Incident face of `inc`: the axis most aligned with the reference normal.
    int incAxis = 0;
    V3 incNormal = v3zero();
    float bestAlign = -1.f;
    #pragma unroll
    for (int a = 0; a < 3; a++)
    {
        const V3 n = boxAxis(inc, a);
        const float d = dot(n, refNormal);
        const float align = fabsf(d);
        if (align <= bestAlign) continue;
        bestAlign = align;
        incAxis = a;
        incNormal = d > 0.f ? neg(n) : n;
    }
    const int au = (incAxis + 1) % 3, av = (incAxis + 2) % 3;
    const V3 eu = boxAxis(inc, au) * vget(carHalfExtents(), au);
    const V3 ev = boxAxis(inc, av) * vget(carHalfExtents(), av);
    const V3 center = inc.cen + incNormal * vget(carHalfExtents(), incAxis);

    V3* bufA = clip;
    V3* bufB = clip + 8;
    bufA[0] = center - eu - ev;
    bufA[1] = center + eu - ev;
    bufA[2] = center + eu + ev;
    bufA[3] = center - eu + ev;
    V3* in = bufA;
    V3* outp = bufB;
    int n = 4;
    for (int axis = 0; axis < 3 && n > 0; axis++)
    {
        if (axis == faceAxis) continue;
        const V3 side = boxAxis(ref, axis);
        const float extent = vget(carHalfExtents(), axis);
        const float maxDist = dot(ref.cen, side) + extent;
        const float minDist = dot(ref.cen, neg(side)) + extent;
        n = clipPolygon(in, n, outp, side, maxDist);
        { V3* t = in; in = outp; outp = t; }
        if (n == 0) break;
        n = clipPolygon(in, n, outp, neg(side), minDist);
        { V3* t = in; in = outp; outp = t; }
    }

    const V3 refCenter = ref.cen + refNormal * vget(carHalfExtents(), faceAxis);
    int count = 0;
    for (int i = 0; i < n && count < MAX_CAR_MANIFOLD_POINTS; i++)
    {
        const float depth = dot(refCenter - in[i], refNormal);
        if (depth < -CAR_CONTACT_BREAK) continue;
        const V3 onRef = in[i] + refNormal * depth;
        const V3 pa = refIsA ? onRef : in[i];
        const V3 pb = refIsA ? in[i] : onRef;
        const CCContact cc{ unrotate(A.rot, pa - A.cen), unrotate(B.rot, pb - B.cen), s.minAxis, fmaxf(depth, 0.f) };
        #pragma unroll
        for (int k = 0; k < MAX_CAR_MANIFOLD_POINTS; k++)
            if (k == count) out[k] = cc;
        count++;
    }
    if (count > 0) return count;
    out[0] = CCContact{ unrotate(A.rot, refCenter - A.cen), unrotate(B.rot, refCenter - B.cen), s.minAxis, s.minPen };
    return 1;
}

// ---- two-body solver -----------------------------------------------------------------------

struct PairRow
{
    V3 axis, relCrossA, relCrossB, angularA, angularB;
    float jacInv, rhs, rhsPen, applied, appliedPush;
};

CB_D PairRow pairAxisRow(const Body& a, const Body& b, V3 axis, V3 relA, V3 relB)
{
    PairRow r;
    r.axis = axis;
    r.relCrossA = cross(relA, axis);
    r.relCrossB = cross(relB, axis);
    r.angularA = invInertiaWorld(a.rot, r.relCrossA);
    r.angularB = invInertiaWorld(b.rot, r.relCrossB);
    const float denom = 2.f * CAR_INV_MASS + dot(axis, cross(r.angularA, relA)) + dot(axis, cross(r.angularB, relB));
    r.jacInv = 1.f / fmaxf(denom, 1e-8f);
    r.rhs = 0.f;
    r.rhsPen = 0.f;
    r.applied = 0.f;
    r.appliedPush = 0.f;
    return r;
}

CB_D float pairVel(const PairRow& r, V3 la, V3 aa, V3 lb, V3 ab)
{
    return dot(r.axis, la) + dot(r.relCrossA, aa) - dot(r.axis, lb) - dot(r.relCrossB, ab);
}

CB_D void pairApply(Body& a, Body& b, const PairRow& r, float impulse, bool split)
{
    V3& la = split ? a.pushVel : a.deltaVel;
    V3& aa = split ? a.turnVel : a.deltaAng;
    V3& lb = split ? b.pushVel : b.deltaVel;
    V3& ab = split ? b.turnVel : b.deltaAng;
    la = la + r.axis * (CAR_INV_MASS * impulse);
    aa = aa + r.angularA * impulse;
    lb = lb - r.axis * (CAR_INV_MASS * impulse);
    ab = ab - r.angularB * impulse;
}

// Two-body solve of `count` contacts.  The row arrays have the compile-time
// capacity N so they stay in registers; rows at and beyond `count` are skipped,
// so every lane of a warp runs the same code whatever its contact count.
template <int N>
CB_D void solvePairN(Body& a, Body& b, const CCContact* c, int count)
{
    PairRow nr[N], fr[N];
    #pragma unroll
    for (int i = 0; i < N; i++)
    {
        if (i >= count) break;
        const V3 relA = a.cen - a.pos + rotate(a.rot, c[i].carPosA);
        const V3 relB = b.cen - b.pos + rotate(b.rot, c[i].carPosB);

        PairRow n = pairAxisRow(a, b, c[i].normal, relA, relB);
        const float relVel = pairVel(n, a.vel, a.ang, b.vel, b.ang);
        const float bounce = relVel < -CAR_RESTITUTION_VEL_THRESH ? CARCAR_COLLISION_RESTITUTION * -relVel : 0.f;
        const float penetration = fmaxf(c[i].depth - CAR_SOLVER_LINEAR_SLOP, 0.f);
        n.rhs = (bounce - relVel) * n.jacInv;
        n.rhsPen = penetration * CAR_CONTACT_ERP / PHYS_DT * n.jacInv;
        nr[i] = n;

        const V3 velA = a.vel + cross(a.ang, relA);
        const V3 velB = b.vel + cross(b.ang, relB);
        const V3 rel = velA - velB;
        const float normalVel = dot(c[i].normal, rel);
        V3 tangent = rel - c[i].normal * normalVel;
        const float tl = lensq(tangent);
        const float threshold = fmaxf(FLOAT_EPSILON, normalVel * normalVel * 1e-8f);
        tangent = tl > threshold ? tangent * rsqrtf(tl) : fallbackTangent(c[i].normal);
        PairRow f = pairAxisRow(a, b, tangent, relA, relB);
        f.rhs = -pairVel(f, a.vel, a.ang, b.vel, b.ang) * f.jacInv;
        fr[i] = f;
    }
    for (int iter = 0; iter < CAR_SOLVER_ITERS; iter++)
        #pragma unroll
        for (int i = 0; i < N; i++)
        {
            if (i >= count) break;
            PairRow& r = nr[i];
            const float rv = pairVel(r, a.pushVel, a.turnVel, b.pushVel, b.turnVel);
            pairApply(a, b, r, solveLowerImpulse(r.rhsPen, 0.f, r.jacInv, rv, 0.f, r.appliedPush), true);
        }
    for (int iter = 0; iter < CAR_SOLVER_ITERS; iter++)
    {
        #pragma unroll
        for (int i = 0; i < N; i++)
        {
            if (i >= count) break;
            PairRow& r = nr[i];
            const float rv = pairVel(r, a.deltaVel, a.deltaAng, b.deltaVel, b.deltaAng);
            pairApply(a, b, r, solveLowerImpulse(r.rhs, 0.f, r.jacInv, rv, 0.f, r.applied), false);
        }
        #pragma unroll
        for (int i = 0; i < N; i++)
        {
            if (i >= count) break;
            const float maxImpulse = CARCAR_COLLISION_FRICTION * nr[i].applied;
            if (maxImpulse <= 0.f) continue;
            PairRow& f = fr[i];
            const float rv = pairVel(f, a.deltaVel, a.deltaAng, b.deltaVel, b.deltaAng);
            pairApply(a, b, f, solveImpulse(f.rhs, 0.f, f.jacInv, rv, -maxImpulse, maxImpulse, f.applied), false);
        }
    }
}

CB_D void solvePair(Body& a, Body& b, const CCContact* c, int count)
{
    if (count > 0) solvePairN<MAX_CAR_MANIFOLD_POINTS>(a, b, c, count);
}

CB_D void finishPairBody(Body& b)
{
    b.vel = b.vel + b.deltaVel;
    b.ang = b.ang + b.deltaAng;
    b.pos = b.pos + b.pushVel * PHYS_DT;
    b.rot = integrateQuat(b.rot, b.turnVel * CAR_SPLIT_IMPULSE_TURN_ERP);
    b.cen = b.pos + carOffsetWorld(b.rot);
    clampCarVelocity(b.vel, b.ang);
}

// ---- demolition and bump responses -------------------------------------------------------------

CB_D float bumpGround(float s)
{
    if (s <= 0.f) return 5.f / 6.f;
    if (s <= 1400.f) return 5.f / 6.f + (1100.f - 5.f / 6.f) * (s / 1400.f);
    if (s <= 2200.f) return 1100.f + (1530.f - 1100.f) * ((s - 1400.f) / 800.f);
    return 1530.f;
}
CB_D float bumpAir(float s)
{
    if (s <= 0.f) return 5.f / 6.f;
    if (s <= 1400.f) return 5.f / 6.f + (1390.f - 5.f / 6.f) * (s / 1400.f);
    if (s <= 2200.f) return 1390.f + (1945.f - 1390.f) * ((s - 1400.f) / 800.f);
    return 1945.f;
}
CB_D float bumpUp(float s)
{
    if (s <= 0.f) return 2.f / 6.f;
    if (s <= 1400.f) return 2.f / 6.f + (278.f - 2.f / 6.f) * (s / 1400.f);
    if (s <= 2200.f) return 278.f + (417.f - 278.f) * ((s - 1400.f) / 800.f);
    return 417.f;
}

CB_D bool frontHit(const CCContact* c, int count, bool aIsBumper, V3 delta, Q4 bumperRot)
{
    if (unrotate(bumperRot, delta).x > BUMP_MIN_FORWARD_DIST) return true;
    for (int i = 0; i < count; i++)
    {
        const V3 p = aIsBumper ? c[i].carPosA : c[i].carPosB;
        if (p.x + CAR_OFF_X > BUMP_MIN_FORWARD_DIST) return true;
    }
    return false;
}

// Context of one sim's cars inside a state array.
template <class S>
struct SimCars
{
    S cars;            // car words
    int base;          // index of the sim's car 0 in `cars`
    int nCars, nBlue;
    int globalBase;    // env-global index of the sim's car 0
    int tick;
    int seed;
    V3* clip;          // this thread's clip polygon storage: 2 x 8 vertices (shared memory)
};

template <class S>
CB_D Body loadCarBody(const S& c, int i)
{
    return makeBody(c.v(C_POS, i), c.v(C_VEL, i), c.v(C_ANG, i), c.v(C_CEN, i), c.q(C_ROT, i));
}

template <class S>
CB_D void storeCarBody(const S& c, int i, const Body& b)
{
    c.setv(C_POS, i, b.pos);
    c.setv(C_VEL, i, b.vel);
    c.setv(C_ANG, i, b.ang);
    c.setv(C_CEN, i, b.cen);
    c.setq(C_ROT, i, b.rot);
}

// Car-car stage of one pair (ia = A, ib = B are sim-local car numbers).
// Returns the number of manifold points kept for the diagnostics.
template <class S>
CB_D int solveCarCarPair(const SimCars<S>& sc, int ia, int ib)
{
    const S& c = sc.cars;
    const int A = sc.base + ia, B = sc.base + ib;
    if (c.n(C_DEMOED, A) || c.n(C_DEMOED, B)) return 0;

    Box boxA, boxB;
    boxA.cen = c.v(C_CEN, A);
    boxB.cen = c.v(C_CEN, B);
    const V3 centerDelta = boxB.cen - boxA.cen;
    const float maxDist = 2.f * len(carHalfExtents());
    if (lensq(centerDelta) > maxDist * maxDist) return 0;
    boxA.rot = c.q(C_ROT, A);
    boxB.rot = c.q(C_ROT, B);

    const Sat sat = carCarSat(boxA, boxB);
    if (!sat.overlap) return 0;
    CCContact contacts[MAX_CAR_MANIFOLD_POINTS];
    const int count = ccContacts(sat, boxA, boxB, contacts, sc.clip);
    if (count == 0) return 0;

    // Demolition test on pre-solve state.
    int demoBumper = -1, demoVictim = -1;
    const bool sameTeam = (ia < sc.nBlue) == (ib < sc.nBlue);
    if (!(sameTeam || sat.minPen < 5.f))
    {
        const V3 velA = c.v(C_VEL, A), velB = c.v(C_VEL, B);
        const V3 posA = c.v(C_POS, A), posB = c.v(C_POS, B);
        for (int side = 0; side < 2; side++)
        {
            const bool aIsBumper = side == 0;
            const V3 bumperVel = aIsBumper ? velA : velB;
            const V3 victimVel = aIsBumper ? velB : velA;
            const V3 delta = (aIsBumper ? posB : posA) - (aIsBumper ? posA : posB);
            const float speed = len(bumperVel);
            if (speed < SUPERSONIC_START_SPEED) continue;
            if (dot(bumperVel, delta) <= 0.f) continue;
            const V3 velDir = bumperVel / speed;
            const V3 hitDir = normalized(delta);
            const float closing = dot(bumperVel, hitDir);
            if (closing <= dot(victimVel, velDir)) continue;
            if (!frontHit(contacts, count, aIsBumper, delta, aIsBumper ? boxA.rot : boxB.rot)) continue;
            demoBumper = aIsBumper ? A : B;
            demoVictim = aIsBumper ? B : A;
            break;
        }
    }

    Body a = loadCarBody(c, A);
    Body b = loadCarBody(c, B);
    const V3 preVelA = a.vel, preVelB = b.vel;
    solvePair(a, b, contacts, count);
    finishPairBody(a);
    finishPairBody(b);
    storeCarBody(c, A, a);
    storeCarBody(c, B, b);

    if (demoVictim >= 0)
    {
        V3 pos = c.v(C_POS, demoVictim), cen;
        Q4 rot = c.q(C_ROT, demoVictim);
        integratePose(pos, cen, rot, c.v(C_VEL, demoVictim), c.v(C_ANG, demoVictim));
        c.setv(C_POS, demoVictim, pos);
        c.setv(C_CEN, demoVictim, cen);
        c.setq(C_ROT, demoVictim, rot);
        c.n(C_DEMOED, demoVictim) = 1;
        c.f(C_DEMO_TIMER, demoVictim) = DEMO_RESPAWN_TIME + PHYS_DT;
        const int victimGlobal = sc.globalBase + (demoVictim - sc.base);
        c.n(C_CONTACT_IDX, demoBumper) = victimGlobal;
        c.f(C_CONTACT_CD, demoBumper) = BUMP_COOLDOWN_TIME;
        const uint32_t seed = (uint32_t)sc.seed ^ (uint32_t)victimGlobal * 0x9e3779b9u ^ (uint32_t)sc.tick;
        c.n(C_INT + I_RESPAWN_IDX, demoVictim) = randomIndex(seed, 4);
        c.n(C_INT + I_LAST_RESPAWN_DIR, demoVictim) = 0;
        return 0;
    }

    for (int side = 0; side < 2; side++)
    {
        const bool aIsBumper = side == 0;
        const int bumper = aIsBumper ? A : B;
        const int victim = aIsBumper ? B : A;
        const V3 bumperVel = aIsBumper ? preVelA : preVelB;
        const V3 victimVel = aIsBumper ? preVelB : preVelA;
        const V3 bumperPos = aIsBumper ? a.pos : b.pos;
        const V3 victimPos = aIsBumper ? b.pos : a.pos;
        const Q4 bumperRot = aIsBumper ? a.rot : b.rot;
        const Q4 victimRot = aIsBumper ? b.rot : a.rot;
        const int victimGlobal = sc.globalBase + (victim - sc.base);

        if (c.n(C_CONTACT_IDX, bumper) == victimGlobal && c.f(C_CONTACT_CD, bumper) > 0.f) continue;
        const V3 delta = victimPos - bumperPos;
        if (dot(bumperVel, delta) <= 0.f) continue;
        const float speed = len(bumperVel);
        if (speed < 1e-6f) continue;
        const V3 velDir = bumperVel / speed;
        const V3 hitDir = normalized(delta);
        const float closing = dot(bumperVel, hitDir);
        if (closing <= dot(victimVel, velDir)) continue;
        if (!frontHit(contacts, count, aIsBumper, delta, bumperRot)) continue;

        const bool grounded = c.n(C_INT + I_ON_GROUND, victim) != 0;
        const float forwardScale = grounded ? bumpGround(closing) : bumpAir(closing);
        const V3 up = grounded ? rotate(victimRot, axisVec(2)) : axisVec(2);
        const V3 impulse = velDir * forwardScale + up * bumpUp(closing);
        c.setv(C_IMP, victim, c.v(C_IMP, victim) + impulse);
        c.n(C_CONTACT_IDX, bumper) = victimGlobal;
        c.f(C_CONTACT_CD, bumper) = BUMP_COOLDOWN_TIME;
    }
    return count;
}

// Distance gate of a pair (the only test that needs no state update).
template <class S>
CB_D bool carCarGate(const S& c, int A, int B);

// The lanes of `mask` that are still stepping meet here (a warp vote on the
// device; on the host, a single sim, nothing to meet).
#if defined(__CUDA_ARCH__)
#define CB_LANES_MEET(mask, pred) __ballot_sync((mask), (pred))
#else
#define CB_LANES_MEET(mask, pred) ((pred) ? 1u : 0u)
#endif

// All pairs of one sim in the reference's order (a < b, pair solved as (b, a)).
// Each round first skips to the sim's next pair within reach, then the lanes
// still stepping a sim meet (a vote over `lanes`, the warp's lanes that call this
// together) and run their pair solves side by side.  Without the meeting point
// the lanes leave the skip loop at different pairs and the warp runs their solves
// one after another: 3v3 crowd steps took 3.11 ms instead of 2.65.  The pairs a
// sim solves, and their order, are the sequential ones (solveCarCarPair re-checks
// the gate itself).  kept[pair] receives the manifold point count of every pair
// (0 when skipped).
template <class S>
CB_D void solveCarCarSim(const SimCars<S>& sc, int* kept, int maxKept, unsigned lanes)
{
    const int nCars = sc.nCars;
    const int nPairs = nCars * (nCars - 1) / 2;
    for (int q = 0; q < nPairs && q < maxKept; q++) kept[q] = 0;
    int a = 0, b = 1, pair = 0;
    while (true)
    {
        while (pair < nPairs && !carCarGate(sc.cars, sc.base + b, sc.base + a))
        {
            pair++;
            if (++b == nCars)
            {
                a++;
                b = a + 1;
            }
        }
        lanes = CB_LANES_MEET(lanes, pair < nPairs);
        if (pair >= nPairs) break;
        const int k = solveCarCarPair(sc, b, a);
        if (pair < maxKept) kept[pair] = k;
        pair++;
        if (++b == nCars)
        {
            a++;
            b = a + 1;
        }
    }
}

template <class S>
CB_D bool carCarGate(const S& c, int A, int B)
{
    if (c.n(C_DEMOED, A) || c.n(C_DEMOED, B)) return false;
    const V3 d = c.v(C_CEN, B) - c.v(C_CEN, A);
    const float maxDist = 2.f * len(carHalfExtents());
    return !(lensq(d) > maxDist * maxDist);
}

}  // namespace cb
