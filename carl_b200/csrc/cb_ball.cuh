// Ball physics for one sim: sphere-vs-triangle arena contacts with
// internal-edge normal correction and 4-point reduction, the averaged-contact
// arena solver with per-contact split impulses, sphere-vs-car-core contacts
// and solver, the "extra hit" impulse, Bullet-unit integration and goals.
//
// Follows jwmccarthy/CARL include/Physics/BallArena/{Contact,Solver,Solve}.cuh
// (the default arena path and the native-metadata path), include/Physics/CarBall/
// {Contact,Solve,ExtraImpulse}.cuh and include/Physics/Goals.cuh:6-32, with the
// same fp32 operation order.  The arena triangles near the ball are visited in
// ascending triangle order, as the reference's per-cell merge does.
#pragma once

#include "cb_carcar.cuh"

namespace cb {

// ---- sphere vs triangle ---------------------------------------------------------------

// Whether a car touched the ball on the tick before `tick` (arena contacts are
// solved before car-ball contacts, so that is the hit that matters).
CB_HD bool ballHitPreviousTick(int hitTick, int tick) { return hitTick >= 0 && tick > 0 && hitTick == tick - 1; }

struct BallContact
{
    V3 point, relPos, normal;
    float depth;
    int tri;
};

CB_D V3 closestPointOnTriangle(V3 p, V3 a, V3 b, V3 c)
{
    const V3 ab = b - a;
    const V3 ac = c - a;
    const V3 ap = p - a;
    const float abAp = dot(ab, ap);
    const float acAp = dot(ac, ap);
    if (abAp <= 0.f && acAp <= 0.f) return a;

    const V3 bp = p - b;
    const float abBp = dot(ab, bp);
    const float acBp = dot(ac, bp);
    if (abBp >= 0.f && acBp <= abBp) return b;

    const float wc = abAp * acBp - abBp * acAp;
    if (wc <= 0.f && abAp >= 0.f && abBp <= 0.f) return a + ab * (abAp / (abAp - abBp));

    const V3 cp = p - c;
    const float abCp = dot(ab, cp);
    const float acCp = dot(ac, cp);
    if (acCp >= 0.f && abCp <= acCp) return c;

    const float wb = abCp * acAp - abAp * acCp;
    if (wb <= 0.f && acAp >= 0.f && acCp <= 0.f) return a + ac * (acAp / (acAp - acCp));

    const float wa = abBp * acCp - abCp * acBp;
    if (wa <= 0.f && acBp >= abBp && abCp >= acCp)
    {
        const float e = acBp - abBp;
        return b + (c - b) * (e / (e + abCp - acCp));
    }
    const float inv = 1.f / (wa + wb + wc);
    return a + ab * (wb * inv) + ac * (wc * inv);
}

CB_D bool sphereTriangle(V3 center, float radius, V3 v0, V3 v1, V3 v2, BallContact& c)
{
    const V3 point = closestPointOnTriangle(center, v0, v1, v2);
    const V3 delta = center - point;
    const float distSq = lensq(delta);
    const float contactRadius = radius + BALL_ARENA_CONTACT_BREAK;
    if (distSq >= contactRadius * contactRadius) return false;

    V3 normal = cross(v1 - v0, v2 - v0);
    const float nl = lensq(normal);
    if (nl < 1e-12f) return false;
    normal = normal * rsqrtf(nl);
    if (distSq > 1e-8f && dot(normal, delta) < 0.f) normal = neg(normal);
    if (distSq > 1e-8f) normal = delta * rsqrtf(distSq);

    c.point = point;
    c.relPos = normal * -radius;
    c.normal = normal;
    c.depth = distSq > 1e-8f ? radius - sqrtf(distSq) : radius;
    return true;
}

// Index of the contact to replace among four (reduction by depth and spread).
CB_D int ballContactReplacement(const BallContact* c, const BallContact& cand)
{
    int deepest = -1;
    float depth = cand.depth;
    for (int i = 0; i < 4; i++)
    {
        if (c[i].depth > depth)
        {
            deepest = i;
            depth = c[i].depth;
        }
    }
    float area[4] = { 0.f, 0.f, 0.f, 0.f };
    const V3 p = cand.relPos;
    if (deepest != 0) area[0] = lensq(cross(p - c[1].relPos, c[3].relPos - c[2].relPos));
    if (deepest != 1) area[1] = lensq(cross(p - c[0].relPos, c[3].relPos - c[2].relPos));
    if (deepest != 2) area[2] = lensq(cross(p - c[0].relPos, c[3].relPos - c[1].relPos));
    if (deepest != 3) area[3] = lensq(cross(p - c[0].relPos, c[2].relPos - c[1].relPos));
    int best = 0;
    for (int i = 1; i < 4; i++)
        if (area[i] > area[best]) best = i;
    return best;
}

// Internal-edge correction of a sphere contact normal.
CB_D void adjustBallEdgeNormal(BallContact& c, V3 v0, V3 v1, V3 v2, V3 angles)
{
    const V3 verts[3] = { v0, v1, v2 };
    int bestEdge = -1;
    float bestDistSq = 25.f;  // 0.1 m in uu^2... Bullet's edge distance threshold
    for (int e = 0; e < 3; e++)
    {
        if (fabsf(vget(angles, e)) >= BOUNDARY_EDGE_ANGLE) continue;
        const V3 start = verts[e];
        const V3 edge = verts[(e + 1) % 3] - start;
        const float t = clampf(dot(c.point - start, edge) / lensq(edge), 0.f, 1.f);
        const V3 nearest = start + edge * t;
        const float d = lensq(c.point - nearest);
        if (d < bestDistSq)
        {
            bestDistSq = d;
            bestEdge = e;
        }
    }
    if (bestEdge < 0) return;

    const V3 faceNormal = normalized(cross(v1 - v0, v2 - v0));
    const float angle = vget(angles, bestEdge);
    if (angle == 0.f)
    {
        if (dot(faceNormal, c.normal) >= 0.f) c.normal = faceNormal;
        return;
    }
    const float side = angle > 0.f ? 1.f : -1.f;
    const V3 edgeAxis = normalized(verts[(bestEdge + 1) % 3] - verts[bestEdge]);
    const V3 normalA = faceNormal * side;
    const V3 normalB = rotateAbout(faceNormal, edgeAxis, angle) * side;
    if (dot(c.normal, normalA) < 0.f && dot(c.normal, normalB) < 0.f)
    {
        if (dot(faceNormal, c.normal) >= 0.f) c.normal = faceNormal;
        return;
    }
    V3 clamped;
    if (clampEdgeNormal(edgeAxis, normalA, c.normal, angle, clamped) && dot(clamped, faceNormal) > 0.f)
        c.normal = normalized(clamped);
}

// Inserts a contact (found on triangle `tri`, in ascending triangle order)
// into the <=4 contact set, then applies the edge correction.
CB_D void insertBallContact(BallContact* set, int& count, BallContact c, V3 center, V3 v0, V3 v1, V3 v2,
                            V3 angles)
{
    int slot;
    if (count < 4) slot = count++;
    else slot = ballContactReplacement(set, c);
    adjustBallEdgeNormal(c, v0, v1, v2, angles);
    c.point = center + c.relPos + c.normal * c.depth;
    set[slot] = c;
}

// ---- native mesh branch ------------------------------------------------------------------------
// With native mesh metadata (src/ArenaMesh.cu:69-99) the ball meets the arena in
// Bullet units against the native triangles (BallArena/Contact.cuh:161-201,
// 292-343, 478-593): contacts are reduced to four per native mesh, the edge
// correction uses the native angles and edge flags, and the four arena planes
// are added as contacts after the mesh contacts are scaled back to Unreal units.

constexpr int MAX_BALL_ARENA_CONTACTS = 68;  // four per native mesh (16 meshes) plus the four planes

// Sphere (the ball in Bullet units, centre `center`) against a native triangle.
CB_D bool nativeSphereTriangle(V3 center, V3 v0, V3 v1, V3 v2, BallContact& c)
{
    constexpr float radius = BALL_COLLISION_RADIUS * .02f;
    constexpr float extent = radius + BALL_ARENA_CONTACT_BREAK * .02f;
    const V3 e01 = v1 - v0, e02 = v2 - v0, off = center - v0;
    const V3 fn = cross(e01, e02);
    const float nl = lensq(fn);
    if (nl < 1e-14f) return false;
    V3 normal = fn * (1.f / sqrtf(nl));
    float planeDist = dot(off, normal);
    if (planeDist < 0.f)
    {
        planeDist = -planeDist;
        normal = neg(normal);
    }
    if (planeDist >= extent) return false;
    // Barycentric coordinates of the centre's projection.
    const float gamma = dot(cross(e01, off), fn) / nl;
    const float beta = dot(cross(off, e02), fn) / nl;
    const float alpha = 1.f - gamma - beta;
    const bool inside = alpha >= 0.f && alpha <= 1.f && beta >= 0.f && beta <= 1.f && gamma >= 0.f && gamma <= 1.f;
    c.point = inside ? center - normal * planeDist : closestPointOnTriangle(center, v0, v1, v2);
    const V3 delta = center - c.point;
    const float distSq = lensq(delta);
    if (distSq >= extent * extent) return false;
    const float distance = sqrtf(distSq);
    c.normal = distSq > FLOAT_EPSILON ? delta * (1.f / distance) : normal;
    c.depth = distSq > FLOAT_EPSILON ? radius - distance : radius;
    c.relPos = (c.point - c.normal * c.depth) - center;
    return true;
}

// Internal-edge correction of a native contact (point and normal in Bullet
// units).  Edge e runs v_e -> v_(e+1)%3; flag bit e says the face normal points
// to the positive side of its edge, bit e + 3 that the neighbour's normal is
// flipped; a zero angle marks a concave edge.
CB_D void adjustNativeBallEdgeNormal(BallContact& c, V3 v0, V3 v1, V3 v2, V3 angles, int flags)
{
    constexpr float edgeDistance = .1f;
    const V3 verts[3] = { v0, v1, v2 };
    int bestEdge = -1;
    float bestDistSq = edgeDistance * edgeDistance;
    for (int e = 0; e < 3; e++)
    {
        if (fabsf(vget(angles, e)) >= BOUNDARY_EDGE_ANGLE) continue;
        const V3 start = verts[e];
        const V3 edge = verts[(e + 1) % 3] - start;
        const float t = clampf(dot(c.point - start, edge) / lensq(edge), 0.f, 1.f);
        const V3 nearest = start + edge * t;
        const float d = lensq(c.point - nearest);
        if (d < bestDistSq)
        {
            bestDistSq = d;
            bestEdge = e;
        }
    }
    if (bestEdge < 0) return;

    const V3 faceNormal = normalized(cross(v1 - v0, v2 - v0));
    const V3 edgeDir = normalized(verts[bestEdge] - verts[(bestEdge + 1) % 3]);
    const float angle = vget(angles, bestEdge);
    bool concave = angle == 0.f;
    if (!concave)
    {
        const float sign = (flags & (1 << bestEdge)) ? 1.f : -1.f;
        V3 other = rotateAbout(faceNormal, edgeDir, angle);
        if (flags & (1 << (bestEdge + 3))) other = neg(other);
        concave = dot(c.normal, faceNormal * sign) < 0.f && dot(c.normal, other * sign) < 0.f;
        if (!concave)
        {
            V3 clamped;
            if (clampEdgeNormal(edgeDir, faceNormal * sign, c.normal, angle, clamped) && dot(clamped, faceNormal) > 0.f)
                c.normal = clamped;
        }
    }
    if (concave && dot(faceNormal, c.normal) >= 0.f) c.normal = faceNormal;
}

// Scales the native contacts back to Unreal units and adds a contact for each
// arena plane (floor, ceiling, the two side walls) within the contact break.
CB_D int finishNativeBallContacts(BallContact* set, int count, V3 center)
{
    for (int i = 0; i < count; i++)
    {
        set[i].point = set[i].point * 50.f;
        set[i].relPos = set[i].relPos * 50.f;
        set[i].depth *= 50.f;
    }
    const V3 normals[4] = { V3{ 0.f, 0.f, 1.f }, V3{ 0.f, 0.f, -1.f }, V3{ 1.f, 0.f, 0.f }, V3{ -1.f, 0.f, 0.f } };
    const float offsets[4] = { 0.f, -2044.f, -4096.f, -4096.f };
    for (int k = 0; k < 4; k++)
    {
        const float depth = BALL_COLLISION_RADIUS - (dot(normals[k], center) - offsets[k]);
        if (depth > -BALL_ARENA_CONTACT_BREAK && count < MAX_BALL_ARENA_CONTACTS)
        {
            BallContact c;
            c.point = center - normals[k] * (BALL_COLLISION_RADIUS - depth);
            c.relPos = normals[k] * -BALL_COLLISION_RADIUS;
            c.normal = normals[k];
            c.depth = depth;
            c.tri = -1;
            set[count++] = c;
        }
    }
    return count;
}

// ---- ball-arena solver ----------------------------------------------------------------------------

struct BallRow
{
    V3 axis, relCross;
    float jacInv, rhs, rhsPen, applied, appliedPush;
};

struct BallBody
{
    V3 pos, vel, velNoExt, ang, deltaVel, deltaAng, pushVel, pushAng;
};

CB_D BallRow ballAxisRow(V3 axis, V3 relPos)
{
    BallRow r;
    r.axis = axis;
    r.relCross = cross(relPos, axis);
    const float denom = BALL_INV_MASS + BALL_INV_INERTIA * lensq(r.relCross);
    r.jacInv = 1.f / fmaxf(denom, 1e-8f);
    r.rhs = 0.f;
    r.rhsPen = 0.f;
    r.applied = 0.f;
    r.appliedPush = 0.f;
    return r;
}

CB_D float ballRowVel(const BallRow& r, V3 lin, V3 ang) { return dot(r.axis, lin) + dot(r.relCross, ang); }

CB_D BallRow ballNormalRow(const BallBody& b, V3 normal, float depth, V3 relPos, bool split)
{
    BallRow r = ballAxisRow(normal, relPos);
    const float relVel = ballRowVel(r, b.vel, b.ang);
    const float restVel = ballRowVel(r, b.velNoExt, b.ang);
    float bounce = fabsf(restVel) >= CAR_RESTITUTION_VEL_THRESH ? BALL_WORLD_RESTITUTION * -restVel : 0.f;
    bounce = fmaxf(bounce, 0.f);
    const float posError = fmaxf(depth, 0.f) * CAR_CONTACT_ERP / PHYS_DT;
    const float posImpulse = posError * r.jacInv;
    const float velImpulse = (bounce - relVel) * r.jacInv;
    if (!split) r.rhs = velImpulse;
    else if (-depth > CAR_SPLIT_PENETRATION_THRESH) r.rhs = posImpulse + velImpulse;
    else
    {
        r.rhs = velImpulse;
        r.rhsPen = posImpulse;
    }
    return r;
}

CB_D void ballApply(BallBody& b, const BallRow& r, float impulse, bool split)
{
    V3& lin = split ? b.pushVel : b.deltaVel;
    V3& ang = split ? b.pushAng : b.deltaAng;
    lin = lin + r.axis * (BALL_INV_MASS * impulse);
    ang = ang + r.relCross * (BALL_INV_INERTIA * impulse);
}

CB_D void clampBallVelocity(V3& vel, V3& ang)
{
    const float v2 = lensq(vel);
    if (v2 > BALL_MAX_SPEED * BALL_MAX_SPEED) vel = vel * (BALL_MAX_SPEED * rsqrtf(v2));
    const float a2 = lensq(ang);
    if (a2 > BALL_MAX_ANG_SPEED * BALL_MAX_ANG_SPEED) ang = ang * (BALL_MAX_ANG_SPEED * rsqrtf(a2));
}

// Averaged-contact solve of `count` (<= CAP) contacts.
template <int CAP>
CB_D void solveBallArenaN(BallBody& b, const BallContact* c, int count, bool ballWasHit)
{
    if (count == 0) return;
    BallRow split[CAP];
    V3 totalNormal = v3zero();
    float totalRadius = 0.f;
    const bool splitCorrection = !ballWasHit || count != 1 || c[0].normal.z < 0.999f;
    for (int i = 0; i < count; i++)
    {
        split[i] = ballNormalRow(b, c[i].normal, c[i].depth, c[i].relPos, splitCorrection);
        totalNormal = totalNormal + c[i].normal;
        totalRadius += sqrtf(lensq(c[i].relPos));
    }
    const V3 avgNormal = totalNormal * (1.f / count);
    const V3 avgRel = avgNormal * (-totalRadius / count);
    const float avgDepth = -totalRadius / count;

    BallRow nrow = ballNormalRow(b, avgNormal, avgDepth, avgRel, false);
    const V3 pointVel = b.vel + cross(b.ang, avgRel);
    const float normalVel = dot(avgNormal, pointVel);
    V3 tangent = pointVel - avgNormal * normalVel;
    const float tl = lensq(tangent);
    tangent = tl > 1e-8f ? tangent * rsqrtf(tl) : fallbackTangent(avgNormal);
    BallRow frow = ballAxisRow(tangent, avgRel);
    frow.rhs = -ballRowVel(frow, b.vel, b.ang) * frow.jacInv;

    for (int iter = 0; iter < CAR_SOLVER_ITERS; iter++)
        for (int i = 0; i < count; i++)
        {
            BallRow& r = split[i];
            if (r.rhsPen == 0.f) continue;
            const float rv = ballRowVel(r, b.pushVel, b.pushAng);
            ballApply(b, r, solveLowerImpulse(r.rhsPen, 0.f, r.jacInv, rv, 0.f, r.appliedPush), true);
        }
    for (int iter = 0; iter < CAR_SOLVER_ITERS; iter++)
    {
        const float rv = ballRowVel(nrow, b.deltaVel, b.deltaAng);
        ballApply(b, nrow, solveLowerImpulse(nrow.rhs, 0.f, nrow.jacInv, rv, 0.f, nrow.applied), false);
        const float maxImpulse = BALL_WORLD_FRICTION * nrow.applied;
        if (maxImpulse > 0.f)
        {
            const float fv = ballRowVel(frow, b.deltaVel, b.deltaAng);
            ballApply(b, frow, solveImpulse(frow.rhs, 0.f, frow.jacInv, fv, -maxImpulse, maxImpulse, frow.applied), false);
        }
    }
    b.vel = b.vel + b.deltaVel;
    b.ang = b.ang + b.deltaAng;
    clampBallVelocity(b.vel, b.ang);
}

CB_D void solveBallArena(BallBody& b, const BallContact* c, int count, bool ballWasHit)
{
    solveBallArenaN<4>(b, c, count, ballWasHit);
}

// ---- ball vs car -----------------------------------------------------------------------------------

struct BallCarHit
{
    V3 point, normal;
    float depth;
    bool hit;
};

CB_D BallCarHit sphereCarContact(V3 ballPos, V3 carCen, Q4 carRot)
{
    BallCarHit h{ v3zero(), v3zero(), 0.f, false };
    const V3 local = unrotate(carRot, ballPos - carCen);
    const V3 clamped = { clampf(local.x, -CB_CORE_HALF_X, CB_CORE_HALF_X), clampf(local.y, -CB_CORE_HALF_Y, CB_CORE_HALF_Y),
                         clampf(local.z, -CB_CORE_HALF_Z, CB_CORE_HALF_Z) };
    const V3 delta = local - clamped;
    const float distSq = lensq(delta);
    const float intersect = BALL_RADIUS + CAR_BALL_SHAPE_MARGIN;
    const float accept = intersect + CAR_BALL_CONTACT_BREAK;
    if (distSq > 1e-8f)
    {
        if (distSq >= accept * accept) return h;
        const float dist = sqrtf(distSq);
        const V3 ln = delta * (1.f / dist);
        h.point = carCen + rotate(carRot, clamped + ln * CAR_BALL_SHAPE_MARGIN);
        h.normal = rotate(carRot, ln);
        h.depth = intersect - dist;
        h.hit = true;
        return h;
    }
    const V3 faceDist = V3{ CB_CORE_HALF_X, CB_CORE_HALF_Y, CB_CORE_HALF_Z } - vabs(local);
    int axis = 0;
    float minDist = faceDist.x;
    if (faceDist.y < minDist)
    {
        axis = 1;
        minDist = faceDist.y;
    }
    if (faceDist.z < minDist)
    {
        axis = 2;
        minDist = faceDist.z;
    }
    V3 ln = v3zero();
    vset(ln, axis, vget(local, axis) >= 0.f ? 1.f : -1.f);
    h.point = carCen + rotate(carRot, clamped + ln * CAR_BALL_SHAPE_MARGIN);
    h.normal = rotate(carRot, ln);
    h.depth = intersect + minDist;
    h.hit = true;
    return h;
}

struct BCRow
{
    V3 axis, ballTorque, carAngular;
    float jacInv, applied;
};

CB_D BCRow bcRow(Q4 carRot, V3 axis, V3 ballOffset, V3 carOffset)
{
    BCRow r;
    r.axis = axis;
    r.ballTorque = cross(ballOffset, axis);
    const V3 carTorque = cross(carOffset, axis);
    r.carAngular = rotate(carRot, unrotate(carRot, carTorque) * carInvInertia());
    const float denom = BALL_INV_MASS + CAR_INV_MASS + BALL_INV_INERTIA * lensq(r.ballTorque) + dot(r.carAngular, carTorque);
    r.jacInv = 1.f / fmaxf(denom, 1e-8f);
    r.applied = 0.f;
    return r;
}

CB_D float bcVel(const BCRow& r, V3 bv, V3 ba, V3 cv, V3 ca, V3 ballOffset, V3 carOffset)
{
    const V3 bp = bv + cross(ba, ballOffset);
    const V3 cp = cv + cross(ca, carOffset);
    return dot(r.axis, bp - cp);
}

CB_D void bcApply(V3& bv, V3& ba, V3& cv, V3& ca, const BCRow& r, float impulse)
{
    bv = bv + r.axis * (impulse * BALL_INV_MASS);
    ba = ba + r.ballTorque * (impulse * BALL_INV_INERTIA);
    cv = cv - r.axis * (impulse * CAR_INV_MASS);
    ca = ca - r.carAngular * impulse;
}

CB_D float extraImpulseCurve(float s)
{
    if (s <= 500.f) return 0.65f;
    if (s <= 2300.f) return 0.65f + (0.55f - 0.65f) * ((s - 500.f) / 1800.f);
    if (s <= 4600.f) return 0.55f + (0.30f - 0.55f) * ((s - 2300.f) / 2300.f);
    return 0.30f;
}

CB_D V3 extraHitVelocity(V3 ballPos, V3 carPos, V3 carVel, Q4 carRot, V3 preSolveBallVel)
{
    const V3 relVel = preSolveBallVel - carVel;
    const float rawSpeed = sqrtf(lensq(relVel));
    const float speed = fminf(rawSpeed, BALL_CAR_EXTRA_IMPULSE_MAXDELTAVEL_UU);
    if (speed <= 0.f) return v3zero();
    const V3 relPos = ballPos - carPos;
    V3 hitDir = { relPos.x, relPos.y, relPos.z * BALL_CAR_EXTRA_IMPULSE_Z_SCALE };
    const float dl = lensq(hitDir);
    if (dl <= 1e-12f) return v3zero();
    hitDir = hitDir * rsqrtf(dl);
    const V3 forward = rotate(carRot, axisVec(0));
    const float forwardScale = dot(hitDir, forward) * (1.f - BALL_CAR_EXTRA_IMPULSE_FORWARD_SCALE);
    hitDir = hitDir - forward * forwardScale;
    const float al = lensq(hitDir);
    if (al > 1e-12f) hitDir = hitDir * rsqrtf(al);
    return hitDir * (speed * extraImpulseCurve(speed));
}

// Ball state of one sim inside a sim-word array.
template <class T>
struct SimBall
{
    T sims;
    int idx;
};

// Solves the ball against car `car` (index into `cars`); `localCar` is the
// car's number inside the sim.  Returns true when the pair touched.
template <class S, class T>
CB_D bool solveBallCar(const S& cars, int car, const T& sims, int sim, V3 preSolveBallVel, int tick)
{
    if (cars.n(C_DEMOED, car)) return false;
    const V3 ballPos = sims.v(S_BPOS, sim);
    V3 bv = sims.v(S_BVEL, sim);
    V3 ba = sims.v(S_BANG, sim);
    const V3 carPos = cars.v(C_POS, car);
    const V3 carCen = cars.v(C_CEN, car);
    V3 cv = cars.v(C_VEL, car);
    V3 ca = cars.v(C_ANG, car);
    const Q4 carRot = cars.q(C_ROT, car);
    const V3 preSolveCarVel = cv;

    const BallCarHit hit = sphereCarContact(ballPos, carCen, carRot);
    if (!hit.hit) return false;

    const V3 ballOffset = hit.normal * -BALL_RADIUS;
    const V3 carOffset = hit.point - carPos;
    BCRow nrow = bcRow(carRot, hit.normal, ballOffset, carOffset);
    const float relNormal = bcVel(nrow, bv, ba, cv, ca, ballOffset, carOffset);
    V3 tangent = (bv + cross(ba, ballOffset)) - (cv + cross(ca, carOffset));
    tangent = tangent - hit.normal * relNormal;
    const float tl = lensq(tangent);
    const float restitution = fabsf(relNormal) > CAR_RESTITUTION_VEL_THRESH ? CAR_BALL_RESTITUTION * -relNormal : 0.f;
    tangent = tl > FLOAT_EPSILON ? tangent * rsqrtf(tl) : fallbackTangent(hit.normal);
    BCRow frow = bcRow(carRot, tangent, ballOffset, carOffset);

    for (int iter = 0; iter < CAR_SOLVER_ITERS; iter++)
    {
        const float rn = bcVel(nrow, bv, ba, cv, ca, ballOffset, carOffset);
        bcApply(bv, ba, cv, ca, nrow, solveLowerImpulse(restitution * nrow.jacInv, 0.f, nrow.jacInv, rn, 0.f, nrow.applied));
        const float rt = bcVel(frow, bv, ba, cv, ca, ballOffset, carOffset);
        const float maxFriction = CAR_BALL_FRICTION * nrow.applied;
        bcApply(bv, ba, cv, ca, frow, solveImpulse(0.f, 0.f, frow.jacInv, rt, -maxFriction, maxFriction, frow.applied));
    }
    sims.setv(S_BVEL, sim, bv);
    sims.setv(S_BANG, sim, ba);
    cars.setv(C_VEL, car, cv);
    cars.setv(C_ANG, car, ca);

    // Split correction of both positions.
    const float penetration = hit.depth - CAR_SOLVER_LINEAR_SLOP;
    if (penetration > 0.f)
    {
        const float push = penetration * CAR_CONTACT_ERP / PHYS_DT * nrow.jacInv;
        const V3 ballCorr = hit.normal * (push * BALL_INV_MASS * PHYS_DT);
        const V3 carCorr = hit.normal * (-push * CAR_INV_MASS * PHYS_DT);
        const V3 carTurn = nrow.carAngular * -push;
        sims.setv(S_BPOS, sim, sims.v(S_BPOS, sim) + ballCorr);
        const V3 newPos = cars.v(C_POS, car) + carCorr;
        cars.setv(C_POS, car, newPos);
        const Q4 newRot = integrateQuat(cars.q(C_ROT, car), carTurn * CAR_SPLIT_IMPULSE_TURN_ERP);
        cars.setq(C_ROT, car, newRot);
        cars.setv(C_CEN, car, newPos + carOffsetWorld(newRot));
    }

    // Touch bookkeeping and the extra hit impulse (once per hit streak).
    cars.n(C_BALL_CONTACT_TICK, car) = tick;
    sims.n(S_LAST_TOUCH, sim) = tick;
    const int lastTick = cars.n(C_BALL_HIT_TICK, car);
    if (!(tick <= lastTick + 1 && lastTick <= tick))
    {
        cars.n(C_BALL_HIT_TICK, car) = tick;
        const V3 added = extraHitVelocity(ballPos, carPos, preSolveCarVel, carRot, preSolveBallVel);
        sims.setv(S_BIMP, sim, sims.v(S_BIMP, sim) + added);
    }
    return true;
}

CB_D bool ballCarGate(V3 ballPos, V3 carCen)
{
    const float maxDist = BALL_RADIUS + len(V3{ CB_SOLVER_HALF_X, CB_SOLVER_HALF_Y, CB_SOLVER_HALF_Z });
    return !(lensq(ballPos - carCen) > maxDist * maxDist);
}

template <class T>
CB_D void detectGoal(const T& sims, int sim, V3 ballPos, int tick)
{
    const float threshold = SOCCAR_GOAL_SCORE_BASE_THRESHOLD_Y + BALL_RADIUS;
    const int scorer = ballPos.y > threshold ? 1 : (ballPos.y < -threshold ? -1 : 0);
    if (!scorer || sims.n(S_GOALS + G_LAST_SCORER, sim) != 0) return;
    if (scorer > 0) sims.n(S_GOALS + G_BLUE, sim) += 1;
    else sims.n(S_GOALS + G_ORANGE, sim) += 1;
    sims.n(S_GOALS + G_LAST_SCORER, sim) = scorer;
    sims.n(S_GOALS + G_TICK, sim) = tick;
}

}  // namespace cb
