// Car-vs-arena narrow phase and solve: 13-axis box/triangle SAT in the car
// frame, edge-edge or Sutherland-Hodgman face contacts, internal-edge normal
// correction, the four analytic arena planes plus the single best mesh contact
// as a <=4 point manifold, and the split-impulse + normal/friction solver.
//
// Follows jwmccarthy/CARL include/Physics/CarArena/SAT.cuh:16-125,
// Clip.cuh:32-324, Manifold.cuh:73-310, Solve.cuh:13-327,
// include/Physics/Collision/{SAT,Clip,Solver}.cuh, with the same fp32 operation
// order.  SAT hits are processed in candidate order (the reference assigns
// them with atomicAdd, so its order is not fixed).
#pragma once

#include "cb_suspension.cuh"

namespace cb {

// ---- SAT -----------------------------------------------------------------------------

struct LocalTri
{
    V3 v0, v1, v2, e0, e1, e2;
};

CB_D LocalTri makeLocalTri(V3 a, V3 b, V3 c)
{
    LocalTri t;
    t.v0 = a;
    t.v1 = b;
    t.v2 = c;
    t.e0 = b - a;
    t.e1 = c - b;
    t.e2 = a - c;
    return t;
}
CB_D V3 triVert(const LocalTri& t, int i) { return i == 0 ? t.v0 : (i == 1 ? t.v1 : t.v2); }
CB_D V3 triEdge(const LocalTri& t, int i) { return i == 0 ? t.e0 : (i == 1 ? t.e1 : t.e2); }
CB_D V3 triCenter(const LocalTri& t) { return (t.v0 + t.v1 + t.v2) / 3.f; }

// Triangle vertices relative to the car, in the car frame.
CB_D LocalTri localTriangle(V3 cen, Q4 rot, V3 a, V3 b, V3 c)
{
    return makeLocalTri(unrotate(rot, a - cen), unrotate(rot, b - cen), unrotate(rot, c - cen));
}

struct Sat
{
    bool overlap;
    int axisIdx;
    float minPen;
    V3 minAxis;
};

CB_D void satAxis(V3 ax, const LocalTri& t, V3 delta, int idx, bool norm, Sat& r)
{
    if (!r.overlap) return;
    const float ls = lensq(ax);
    if (ls < 1e-12f) return;
    if (norm) ax = ax * rsqrtf(ls);
    ax = ax * copysignf(1.f, dot(ax, delta));

    const float rad = dot(vabs(ax), carHalfExtents());
    const float cMin = -rad, cMax = rad;
    const float d0 = dot(t.v0, ax), d1 = dot(t.v1, ax), d2 = dot(t.v2, ax);
    const float tMin = fminf(fminf(d0, d1), d2);
    const float tMax = fmaxf(fmaxf(d0, d1), d2);
    if (cMax < tMin || tMax < cMin)
    {
        r.overlap = false;
        return;
    }
    const float depth = fminf(cMax - tMin, tMax - cMin);
    if (depth < r.minPen)
    {
        r.minPen = depth;
        r.minAxis = ax;
        r.axisIdx = idx;
    }
}

CB_D Sat carTriSat(const LocalTri& t)
{
    Sat r{ true, 0, 3.402823466e+38f, v3zero() };
    const V3 delta = neg(triCenter(t));
    satAxis(cross(t.e0, t.e1), t, delta, 0, true, r);
    if (!r.overlap) return r;
    satAxis(axisVec(0), t, delta, 1, false, r);
    satAxis(axisVec(1), t, delta, 2, false, r);
    satAxis(axisVec(2), t, delta, 3, false, r);
    #pragma unroll
    for (int a = 0; a < 3; a++)
    {
        satAxis(cross(t.e0, axisVec(a)), t, delta, 4 + 3 * a, true, r);
        satAxis(cross(t.e1, axisVec(a)), t, delta, 5 + 3 * a, true, r);
        satAxis(cross(t.e2, axisVec(a)), t, delta, 6 + 3 * a, true, r);
    }
    return r;
}

// ---- contacts ------------------------------------------------------------------------------

struct Contact
{
    V3 carPos, arenaPos, normal;
    float depth;
};

CB_D Contact edgeEdgeContact(const LocalTri& t, float minPen, int axisIdx, V3 sep)
{
    const int carAxisIdx = (axisIdx - 4) / 3;
    const int triEdgeIdx = (axisIdx - 4) % 3;
    const V3 center = triCenter(t);
    if (dot(sep, center) > 0.f) sep = neg(sep);

    V3 carPoint = vsign(neg(sep)) * carHalfExtents();
    vset(carPoint, carAxisIdx, 0.f);
    const V3 carAxis = axisVec(carAxisIdx);

    const V3 triPoint = triVert(t, triEdgeIdx);
    const V3 edge = triEdge(t, triEdgeIdx);
    const float triLength = len(edge);
    const V3 triAxis = edge / triLength;

    const V3 carToTri = triPoint - carPoint;
    const float axisDot = dot(carAxis, triAxis);
    const float denom = 1.f - axisDot * axisDot;
    V3 pointOnTri = triPoint;
    if (denom > 1e-6f)
    {
        const float carProj = dot(carToTri, carAxis);
        const float triProj = dot(carToTri, triAxis);
        const float unclamped = (axisDot * carProj - triProj) / denom;
        pointOnTri = triPoint + triAxis * clampf(unclamped, 0.f, triLength);
    }
    const float half = vget(carHalfExtents(), carAxisIdx);
    const float carParam = clampf(dot(carAxis, pointOnTri - carPoint), -half, half);
    const V3 pointOnCar = carPoint + carAxis * carParam;
    const V3 separation = pointOnTri - pointOnCar;
    const float sepSq = lensq(separation);
    if (sepSq > 1e-8f)
    {
        V3 n = separation * rsqrtf(sepSq);
        if (dot(n, center) > 0.f) n = neg(n);
        return Contact{ pointOnCar, pointOnTri, n, minPen };
    }
    return Contact{ pointOnCar, pointOnTri, sep, minPen };
}

CB_D int clipPolygon(const V3* in, int n, V3* out, V3 planeNormal, float planeDist)
{
    if (n == 0) return 0;
    int m = 0;
    for (int i = 0; i < n; i++)
    {
        const V3 cur = in[i];
        const V3 next = in[(i + 1) % n];
        const float cd = dot(planeNormal, cur) - planeDist;
        const float nd = dot(planeNormal, next) - planeDist;
        const bool cin = cd <= 0.f;
        const bool nin = nd <= 0.f;
        if (cin) out[m++] = cur;
        if (cin != nin)
        {
            const float s = cd / (cd - nd);
            out[m++] = cur + (next - cur) * s;
        }
    }
    return m;
}

// Clips the triangle to the car box's side planes around `faceAxis`; the
// polygon ends in *poly (up to 8 vertices).
CB_D int clipTriToFace(const LocalTri& t, int faceAxis, V3* bufA, V3* bufB, V3** poly)
{
    V3* in = bufA;
    V3* out = bufB;
    in[0] = t.v0;
    in[1] = t.v1;
    in[2] = t.v2;
    int n = 3;
    for (int axis = 0; axis < 3 && n > 0; axis++)
    {
        if (axis == faceAxis) continue;
        for (int sign = 1; sign >= -1 && n > 0; sign -= 2)
        {
            n = clipPolygon(in, n, out, axisVec(axis) * (float)sign, vget(carHalfExtents(), axis));
            V3* s = in;
            in = out;
            out = s;
        }
    }
    *poly = in;
    return n;
}

// Emits the contacts of one SAT pair through `emit(const Contact&)`, in the
// order the reference writes them.  bufA and bufB hold MAX_PAIR_CONTACTS
// vertices each: the clip polygon's storage, which the caller places in shared
// memory (indexed by a vertex count, it would otherwise live in local memory).
template <class Emit>
CB_D void pairContacts(const LocalTri& t, const Sat& s, V3* bufA, V3* bufB, Emit&& emit)
{
    if (s.axisIdx >= 4)
    {
        emit(edgeEdgeContact(t, s.minPen, s.axisIdx, s.minAxis));
        return;
    }
    V3* poly;
    const int faceAxis = argMax(vabs(s.minAxis));
    const int n = clipTriToFace(t, faceAxis, bufA, bufB, &poly);

    const V3 faceNormal = axisVec(faceAxis) * -copysignf(1.f, vget(s.minAxis, faceAxis));
    const float faceDistance = vget(carHalfExtents(), faceAxis);
    const float minDepth = -(s.minPen + CAR_CONTACT_BREAK);
    for (int i = 0; i < n; i++)
    {
        float depth = dot(faceNormal, poly[i]) - faceDistance;
        depth = fmaxf(depth, minDepth);
        if (depth > CAR_CONTACT_BREAK) continue;
        emit(Contact{ poly[i] + s.minAxis * depth, poly[i], s.minAxis, -depth });
    }
}

// ---- internal-edge correction ------------------------------------------------------------------

CB_D bool clampEdgeNormal(V3 edgeAxis, V3 triNormal, V3 contactNormal, float edgeAngle, V3& clamped)
{
    V3 edgeCross = cross(edgeAxis, triNormal);
    const float cl = lensq(edgeCross);
    if (cl <= 1e-12f) return false;
    edgeCross = edgeCross * rsqrtf(cl);
    const float tangentProj = dot(contactNormal, edgeCross);
    const float normalProj = dot(contactNormal, triNormal);
    const float current = atan2f(tangentProj, normalProj);
    const bool outside = edgeAngle < 0.f ? current < edgeAngle : current > edgeAngle;
    if (!outside) return false;
    clamped = rotateAbout(contactNormal, edgeAxis, edgeAngle - current);
    return true;
}

CB_D void adjustInternalEdge(const LocalTri& t, V3 angles, Contact& c)
{
    if (allGe(angles, BOUNDARY_EDGE_ANGLE)) return;
    const V3 faceNormal = normalized(cross(t.e0, t.v2 - t.v0));

    int bestEdge = -1;
    float bestDistSq = 3.402823466e+38f;
    for (int e = 0; e < 3; e++)
    {
        if (fabsf(vget(angles, e)) >= BOUNDARY_EDGE_ANGLE) continue;
        const V3 start = triVert(t, e);
        const V3 seg = triVert(t, (e + 1) % 3) - start;
        const float proj = dot(c.arenaPos - start, seg) / lensq(seg);
        const V3 nearest = start + seg * clampf(proj, 0.f, 1.f);
        const float d = lensq(c.arenaPos - nearest);
        if (d < bestDistSq)
        {
            bestDistSq = d;
            bestEdge = e;
        }
    }
    if (bestEdge < 0 || bestDistSq >= TRI_EDGE_DIST_MAX_SQ) return;

    const V3 localNormal = normalized(c.normal);
    const float angle = vget(angles, bestEdge);
    const bool faceAligned = dot(faceNormal, localNormal) >= 0.f;
    if (angle == 0.f)
    {
        if (faceAligned)
        {
            c.normal = faceNormal;
            c.arenaPos = c.carPos + faceNormal * c.depth;
        }
        return;
    }

    const float side = angle > 0.f ? 1.f : -1.f;
    const V3 edgeAxis = normalized(triEdge(t, bestEdge));
    const V3 normalA = faceNormal * side;
    const V3 normalB = rotateAbout(faceNormal, edgeAxis, angle) * side;
    if (dot(localNormal, normalA) < 0.f && dot(localNormal, normalB) < 0.f)
    {
        if (faceAligned)
        {
            c.normal = faceNormal;
            c.arenaPos = c.carPos + faceNormal * c.depth;
        }
        return;
    }
    V3 clamped;
    if (clampEdgeNormal(edgeAxis, normalA, localNormal, angle, clamped) && dot(clamped, faceNormal) > 0.f)
    {
        c.normal = normalized(clamped);
        c.arenaPos = c.carPos + c.normal * c.depth;
    }
}

// ---- manifold -------------------------------------------------------------------------------------

struct MPoint
{
    V3 carPos, worldPos, worldNormal;
    float dist;
};

// The manifold helpers index the point array only with unrolled constants (a
// point is written to slot k where k equals its index), so a caller's MPoint[4]
// stays in registers instead of local memory.
CB_D bool nearManifoldPoint(const MPoint* p, int count, V3 carPos)
{
    bool near = false;
    #pragma unroll
    for (int i = 0; i < MAX_CAR_MANIFOLD_POINTS; i++)
        near |= i < count && lensq(p[i].carPos - carPos) < CAR_MANIFOLD_BREAK_SQ;
    return near;
}

CB_D int manifoldReplacement(const MPoint* p, const MPoint& cand)
{
    int deepest = -1;
    float deepestPen = -cand.dist;
    for (int i = 0; i < MAX_CAR_MANIFOLD_POINTS; i++)
    {
        const float pen = -p[i].dist;
        if (pen > deepestPen)
        {
            deepest = i;
            deepestPen = pen;
        }
    }
    float area[4] = { 0.f, 0.f, 0.f, 0.f };
    if (deepest != 0) area[0] = lensq(cross(cand.carPos - p[1].carPos, p[3].carPos - p[2].carPos));
    if (deepest != 1) area[1] = lensq(cross(cand.carPos - p[0].carPos, p[3].carPos - p[2].carPos));
    if (deepest != 2) area[2] = lensq(cross(cand.carPos - p[0].carPos, p[3].carPos - p[1].carPos));
    if (deepest != 3) area[3] = lensq(cross(cand.carPos - p[0].carPos, p[2].carPos - p[1].carPos));
    int best = 0;
    float bestArea = area[0];
    #pragma unroll
    for (int i = 1; i < 4; i++)
        if (area[i] > bestArea)
        {
            best = i;
            bestArea = area[i];
        }
    return best;
}

CB_D void addManifoldPoint(MPoint* p, int& count, const MPoint& point)
{
    int idx = count;
    if (idx == MAX_CAR_MANIFOLD_POINTS) idx = manifoldReplacement(p, point);
    else count++;
    #pragma unroll
    for (int k = 0; k < MAX_CAR_MANIFOLD_POINTS; k++)
        if (k == idx) p[k] = point;
}

// Contacts with the floor (z = 0), ceiling (z = 2044), and side walls (x = +-4096).
// Deepest box corner towards analytic plane k (floor, ceiling, +x wall, -x wall)
// and its signed distance from the plane.
CB_D void planeCorner(int k, V3 cen, Q4 rot, V3& n, V3& carPos, V3& worldCar, float& dist)
{
    const float offsets[4] = { 0.f, -2044.f, -4096.f, -4096.f };
    const V3 normals[4] = { { 0.f, 0.f, 1.f }, { 0.f, 0.f, -1.f }, { 1.f, 0.f, 0.f }, { -1.f, 0.f, 0.f } };
    n = normals[k];
    const V3 dir = unrotate(rot, neg(n));
    carPos = V3{ dir.x >= 0 ? CAR_HALF_X : -CAR_HALF_X, dir.y >= 0 ? CAR_HALF_Y : -CAR_HALF_Y,
                 dir.z >= 0 ? CAR_HALF_Z : -CAR_HALF_Z };
    worldCar = cen + rotate(rot, carPos);
    dist = dot(n, worldCar) - offsets[k];
}

CB_D int planeManifold(V3 cen, Q4 rot, MPoint* p)
{
    int count = 0;
    #pragma unroll
    for (int k = 0; k < 4; k++)
    {
        V3 n, carPos, worldCar;
        float dist;
        planeCorner(k, cen, rot, n, carPos, worldCar, dist);
        if (dist < CAR_CONTACT_BREAK && !nearManifoldPoint(p, count, carPos))
            addManifoldPoint(p, count, MPoint{ carPos, worldCar - n * dist, n, dist });
    }
    return count;
}

// Whether planeManifold would add any point (the first plane within the contact
// break always adds one).
CB_D bool planeContactAny(V3 cen, Q4 rot)
{
    bool any = false;
    #pragma unroll
    for (int k = 0; k < 4; k++)
    {
        V3 n, carPos, worldCar;
        float dist;
        planeCorner(k, cen, rot, n, carPos, worldCar, dist);
        any |= dist < CAR_CONTACT_BREAK;
    }
    return any;
}

CB_D MPoint contactToManifold(const Contact& c, V3 cen, Q4 rot)
{
    return MPoint{ c.carPos, cen + rotate(rot, c.arenaPos), rotate(rot, c.normal), -c.depth };
}

// ---- solver ---------------------------------------------------------------------------------------

CB_D V3 fallbackTangent(V3 n)
{
    if (fabsf(n.z) > SQRT_1_2)
    {
        const float ls = n.y * n.y + n.z * n.z;
        const float inv = rsqrtf(ls);
        return V3{ 0.f, -n.z * inv, n.y * inv };
    }
    const float ls = n.x * n.x + n.y * n.y;
    const float inv = rsqrtf(ls);
    return V3{ -n.y * inv, n.x * inv, 0.f };
}

CB_D float restitutionVelocity(float relVel, float restitution)
{
    if (fabsf(relVel) < CAR_RESTITUTION_VEL_THRESH) return 0.f;
    return restitution * -relVel;
}

CB_D float solveImpulse(float rhs, float cfm, float jacInv, float relVel, float lo, float hi, float& applied)
{
    const float prev = applied;
    const float delta = rhs - applied * cfm - relVel * jacInv;
    applied = clampf(prev + delta, lo, hi);
    return applied - prev;
}

CB_D float solveLowerImpulse(float rhs, float cfm, float jacInv, float relVel, float lo, float& applied)
{
    const float prev = applied;
    const float delta = rhs - applied * cfm - relVel * jacInv;
    applied = fmaxf(prev + delta, lo);
    return applied - prev;
}

struct Row
{
    V3 axis, relCross, angular;
    float jacInv, rhs, rhsPen, lower, upper, applied, appliedPush;
};

CB_D Row axisRow(const Body& b, V3 axis, V3 relPos)
{
    Row r;
    r.axis = axis;
    r.relCross = cross(relPos, axis);
    r.angular = invInertiaWorld(b.rot, r.relCross);
    const V3 linearResponse = cross(r.angular, relPos);
    const float denom = CAR_INV_MASS + dot(axis, linearResponse);
    r.jacInv = 1.f / fmaxf(denom, 1e-8f);
    r.rhs = 0.f;
    r.rhsPen = 0.f;
    r.lower = 0.f;
    r.upper = 1e10f;
    r.applied = 0.f;
    r.appliedPush = 0.f;
    return r;
}

CB_D float rowVel(const Row& r, V3 lin, V3 ang) { return dot(r.axis, lin) + dot(r.relCross, ang); }

CB_D void applyRow(Body& b, const Row& r, float impulse)
{
    b.deltaVel = b.deltaVel + r.axis * (CAR_INV_MASS * impulse);
    b.deltaAng = b.deltaAng + r.angular * impulse;
}

// Solves one car against its manifold of `count` points; updates the body's delta /
// push velocities.  The row arrays have the compile-time capacity N so they stay in
// registers; rows at and beyond `count` are skipped, so every lane of a warp runs
// the same code whatever its contact count.
template <int N>
CB_D void solveCarManifoldN(Body& b, const MPoint* p, int count)
{
    Row normalRow[N], frictionRow[N];
    const V3 centerOffset = b.cen - b.pos;
    const V3 totalVel = b.vel + b.extVel;
    const V3 totalAng = b.ang + b.extAng;
    constexpr float invDt = 1.f / PHYS_DT;

    #pragma unroll
    for (int i = 0; i < N; i++)
    {
        if (i >= count) break;
        const V3 relPos = centerOffset + rotate(b.rot, p[i].carPos);

        Row n = axisRow(b, p[i].worldNormal, relPos);
        const float relVelNoExt = rowVel(n, b.vel, b.ang);
        const float relVel = rowVel(n, totalVel, totalAng);
        const float restitution = restitutionVelocity(relVelNoExt, CAR_WORLD_RESTITUTION);
        const float penetration = p[i].dist + CAR_SOLVER_LINEAR_SLOP;
        float posError = 0.f;
        const float velError = restitution - relVel;
        if (penetration <= 0.f) posError = -penetration * CAR_CONTACT_ERP * invDt;
        const float posImpulse = posError * n.jacInv;
        const float velImpulse = velError * n.jacInv;
        if (penetration > CAR_SPLIT_PENETRATION_THRESH)
        {
            n.rhs = posImpulse + velImpulse;
        }
        else
        {
            n.rhs = velImpulse;
            n.rhsPen = posImpulse;
        }
        n.applied = 0.f * CAR_SOLVER_WARMSTART;
        normalRow[i] = n;

        const V3 contactVel = totalVel + cross(totalAng, relPos);
        const float normalVel = dot(p[i].worldNormal, contactVel);
        V3 tangent = contactVel - p[i].worldNormal * normalVel;
        const float tl = lensq(tangent);
        tangent = tl > 1e-8f ? tangent * rsqrtf(tl) : fallbackTangent(p[i].worldNormal);
        Row f = axisRow(b, tangent, relPos);
        const float tangentVel = rowVel(f, totalVel, b.ang);
        f.rhs = -tangentVel * f.jacInv;
        f.upper = 0.f;
        f.applied = 0.f;
        frictionRow[i] = f;

        applyRow(b, normalRow[i], normalRow[i].applied);  // warm start (zero impulse)
    }

    // Split impulses: position correction without changing reported velocity.
    for (int iter = 0; iter < CAR_SOLVER_ITERS; iter++)
    {
        #pragma unroll
        for (int i = 0; i < N; i++)
        {
            if (i >= count) break;
            Row& r = normalRow[i];
            if (r.rhsPen == 0.f) continue;
            const float rv = rowVel(r, b.pushVel, b.turnVel);
            const float imp = solveLowerImpulse(r.rhsPen, 0.f, r.jacInv, rv, r.lower, r.appliedPush);
            b.pushVel = b.pushVel + r.axis * (CAR_INV_MASS * imp);
            b.turnVel = b.turnVel + r.angular * imp;
        }
    }

    for (int iter = 0; iter < CAR_SOLVER_ITERS; iter++)
    {
        #pragma unroll
        for (int i = 0; i < N; i++)
        {
            if (i >= count) break;
            Row& r = normalRow[i];
            const float rv = rowVel(r, b.deltaVel, b.deltaAng);
            applyRow(b, r, solveLowerImpulse(r.rhs, 0.f, r.jacInv, rv, r.lower, r.applied));
        }
        #pragma unroll
        for (int i = 0; i < N; i++)
        {
            if (i >= count) break;
            const float maxImpulse = CAR_WORLD_FRICTION * normalRow[i].applied;
            if (maxImpulse <= 0.f) continue;
            Row& f = frictionRow[i];
            f.lower = -maxImpulse;
            f.upper = maxImpulse;
            const float rv = rowVel(f, b.deltaVel, b.deltaAng);
            applyRow(b, f, solveImpulse(f.rhs, 0.f, f.jacInv, rv, f.lower, f.upper, f.applied));
        }
    }
}

CB_D void solveCarManifold(Body& b, const MPoint* p, int count)
{
    if (count > 0) solveCarManifoldN<MAX_CAR_MANIFOLD_POINTS>(b, p, count);
}

CB_D void integrateSplitCorrection(Body& b)
{
    if (lensq(b.pushVel) == 0.f && lensq(b.turnVel) == 0.f) return;
    const V3 splitAng = b.turnVel * CAR_SPLIT_IMPULSE_TURN_ERP;
    integratePose(b.pos, b.cen, b.rot, b.pushVel, splitAng);
}

}  // namespace cb
