// Host build of the product's physics (carl_b200/csrc/cb_*.cuh) stepped
// serially in the fused kernel's stage order, for CPU-side parity tests.
//
// The device intrinsics map onto host math exactly as in the reference's host
// build (oracle/refshim/carl_host_shim.h): rsqrtf -> 1/sqrtf, __sincosf ->
// sinf/cosf.  With those shared, the product's arithmetic must match the
// reference's host build bit for bit; any difference is a porting error.
// The stage split mirrors carl_b200/csrc/tick.cu: candidate rays and SAT in
// candidate order, the first 32 SAT hits, per-sim car-car pairs then ball with
// ball-arena triangles in ascending order.  TEST INFRASTRUCTURE.
#include "host_intrinsics.h"

#include <cstring>
#include <string>
#include <vector>

#include "../../carl_b200/csrc/arena.hpp"
#include "../../carl_b200/csrc/cb_misc.cuh"
#include "../../include/carlb.h"

using namespace cb;

namespace {

thread_local std::string g_error;

struct HostEnv
{
    int nSim, nCars, nBlue, nOrange, seed;
    long long n;
    std::vector<float> car, out, sim;
    std::vector<int> simOut;
    std::vector<int> diagCar, diagSim;
    ArenaHost arena;
    Tables T;
    int tick = 0;

    SmemSoa cars() { return SmemSoa{ car.data(), (int)n }; }
    SmemSoa outs() { return SmemSoa{ out.data(), (int)n }; }
    SmemSoa sims() { return SmemSoa{ sim.data(), nSim }; }

    void triVerts(int tri, V3& v0, V3& v1, V3& v2) const
    {
        auto vert = [&](int v) { return V3{ arena.verts[3 * v], arena.verts[3 * v + 1], arena.verts[3 * v + 2] }; };
        v0 = vert(arena.tris[3 * tri]);
        v1 = vert(arena.tris[3 * tri + 1]);
        v2 = vert(arena.tris[3 * tri + 2]);
    }
    V3 triAngles(int tri) const
    {
        return V3{ arena.edgeAngles[3 * tri], arena.edgeAngles[3 * tri + 1], arena.edgeAngles[3 * tri + 2] };
    }

    void step(const Controls* ctl);
};

void HostEnv::step(const Controls* ctl)
{
    const SmemSoa C = cars(), O = outs(), S = sims();
    tick++;
    for (int s = 0; s < nSim; s++) S.n(S_EP_TICKS, s) += 1;

    std::vector<int> cell(n), cnt(n);
    std::vector<std::vector<int>> hits(n);
    std::vector<float> rayDist(4 * n);
    std::vector<V3> rayNormal(4 * n);
    std::vector<int> src(4 * n);

    // Broadphase, candidate rays + SAT, other-car / ball rays.
    for (long long i = 0; i < n; i++)
    {
        const V3 pos = C.v(C_POS, i), vel = C.v(C_VEL, i), ang = C.v(C_ANG, i), cen = C.v(C_CEN, i);
        const Q4 rot = C.q(C_ROT, i);
        cell[i] = broadphaseCell(pos, vel, ang, cen, rot);
        const int first = arena.cellStart[cell[i]];
        cnt[i] = arena.cellStart[cell[i] + 1] - first;
        const V3 up = rotate(rot, axisVec(2));
        const V3 dir = neg(up);
        V3 start[4];
        float dist[4];
        int bestK[4];
        for (int w = 0; w < 4; w++)
        {
            start[w] = cen + rotate(rot, suspConnection(w));
            dist[w] = suspRayLength(w) + 1.f;
            bestK[w] = -1;
        }
        for (int k = 0; k < cnt[i]; k++)
        {
            const int tri = arena.cellTris[first + k];
            V3 v0, v1, v2;
            triVerts(tri, v0, v1, v2);
            const V3 e1 = v1 - v0, e2 = v2 - v0;
            const V3 pv = cross(dir, e2);
            const float det = dot(e1, pv);
            if (!(fabsf(det) < RAY_PARALLEL_EPS))
            {
                const float invDet = 1.f / det;
                for (int w = 0; w < 4; w++)
                {
                    const V3 tv = start[w] - v0;
                    const float u = invDet * dot(tv, pv);
                    if (u < 0.f || u > 1.f) continue;
                    const V3 qv = cross(tv, e1);
                    const float v = invDet * dot(dir, qv);
                    if (v < 0.f || u + v > 1.f) continue;
                    const float d = invDet * dot(e2, qv);
                    if (d <= 0.f || !(d < dist[w])) continue;
                    dist[w] = d;
                    bestK[w] = k;
                }
            }
            if (!(arena.triFlags[tri] & TRI_ANALYTIC_PLANE))
                if (carTriSat(localTriangle(cen, rot, v0, v1, v2)).overlap) hits[i].push_back(k);
        }
        for (int w = 0; w < 4; w++)
        {
            float& d = rayDist[4 * i + w];
            V3& nn = rayNormal[4 * i + w];
            int& sc = src[4 * i + w];
            d = dist[w];
            if (bestK[w] >= 0)
            {
                V3 v0, v1, v2;
                triVerts(arena.cellTris[first + bestK[w]], v0, v1, v2);
                V3 fn = cross(v1 - v0, v2 - v0);
                fn = fn * rsqrtf(lensq(fn));
                if (dot(fn, dir) > 0.f) fn = neg(fn);
                nn = fn;
                sc = WHEEL_ARENA;
            }
            else
            {
                nn = up;
                sc = WHEEL_NONE;
            }
        }
        const int sim = (int)(i / nCars);
        for (int k = 0; k < nCars; k++)
        {
            const long long o = (long long)sim * nCars + k;
            if (o == i || C.n(C_DEMOED, o)) continue;
            const V3 oc = C.v(C_CEN, o);
            const Q4 orot = C.q(C_ROT, o);
            for (int w = 0; w < 4; w++)
            {
                const V3 ls = unrotate(orot, start[w] - oc);
                const V3 ld = unrotate(orot, dir);
                float entry = 0.f, exitD = suspRayLength(w);
                int hitAxis = -1;
                bool miss = false;
                for (int a = 0; a < 3 && !miss; a++)
                {
                    const float h = vget(carHalfExtents(), a), dd = vget(ld, a), s0 = vget(ls, a);
                    if (fabsf(dd) < RAY_PARALLEL_EPS)
                    {
                        if (fabsf(s0) > h) miss = true;
                        continue;
                    }
                    const float inv = 1.f / dd;
                    const float t1 = (-h - s0) * inv, t2 = (h - s0) * inv;
                    const float tn = fminf(t1, t2);
                    if (tn > entry) { entry = tn; hitAxis = a; }
                    exitD = fminf(exitD, fmaxf(t1, t2));
                    if (entry > exitD) miss = true;
                }
                if (miss || hitAxis < 0 || entry >= rayDist[4 * i + w]) continue;
                V3 ln = v3zero();
                vset(ln, hitAxis, vget(ld, hitAxis) > 0.f ? -1.f : 1.f);
                rayDist[4 * i + w] = entry;
                rayNormal[4 * i + w] = rotate(orot, ln);
                src[4 * i + w] = WHEEL_CAR;
            }
        }
        const V3 bp = S.v(S_BPOS, sim);
        const float invR = 1.f / BALL_COLLISION_RADIUS;
        for (int w = 0; w < 4; w++)
        {
            const V3 off = start[w] - bp;
            const float b = dot(off, dir);
            const float cc = lensq(off) - BALL_COLLISION_RADIUS * BALL_COLLISION_RADIUS;
            if (cc < 0.f) continue;
            const float disc = b * b - cc;
            if (disc < 0.f) continue;
            const float d = -b - sqrtf(disc);
            if (!(d > 0.f && d <= suspRayLength(w)) || d >= rayDist[4 * i + w]) continue;
            rayDist[4 * i + w] = d;
            rayNormal[4 * i + w] = (start[w] + dir * d - bp) * invR;
            src[4 * i + w] = WHEEL_BALL;
        }
        if (!diagCar.empty())
        {
            diagCar[0 * n + i] = cell[i];
            diagCar[1 * n + i] = cnt[i];
            const int nh = (int)std::min<size_t>(hits[i].size(), MAX_CAR_TRI_PAIRS);
            diagCar[2 * n + i] = nh;
            for (int r = 0; r < MAX_CAR_TRI_PAIRS; r++)
                diagCar[(3 + r) * n + i] = r < nh ? arena.cellTris[first + hits[i][r]] : -1;
        }
    }
    // Controls.
    for (long long i = 0; i < n; i++)
    {
        V3 vel = C.v(C_VEL, i), ang = C.v(C_ANG, i);
        Internal s = loadInternal(C, i);
        Susp su = loadSusp(C, i);
        processControls(ctl[i], C.n(C_DEMOED, i) != 0, C.q(C_ROT, i), vel, ang, s, su, &rayDist[4 * i],
                        C.n(C_MAN_COUNT, i), C.v(C_MAN_N0, i));
        C.setv(C_VEL, i, vel);
        C.setv(C_ANG, i, ang);
        storeInternal(C, i, s);
        storeSusp(C, i, su);
    }
    // Suspension, manifold, solve.
    for (long long i = 0; i < n; i++)
    {
        if (C.n(C_DEMOED, i)) continue;
        const V3 cen = C.v(C_CEN, i);
        const Q4 rot = C.q(C_ROT, i);
        Body body = loadCarBody(C, (int)i);
        Susp su = loadSusp(C, i);
        float lat[4], lon[4];
        for (int w = 0; w < 4; w++)
        {
            lat[w] = C.f(C_LAT + w, i);
            lon[w] = C.f(C_LON + w, i);
        }
        applySuspension(body, su, lat, lon, &rayDist[4 * i], &rayNormal[4 * i], C.n(C_MAN_COUNT, i),
                        C.v(C_MAN_N0, i), tick);
        MPoint pts[4];
        int count = planeManifold(cen, rot, pts);
        const int planeCount = count;
        Contact best{};
        float bestDist = 3.402823466e+38f;
        int bestTri = -1;
        const int first = arena.cellStart[cell[i]];
        for (size_t h = 0; h < hits[i].size() && h < (size_t)MAX_CAR_TRI_PAIRS; h++)
        {
            const int tri = arena.cellTris[first + hits[i][h]];
            V3 v0, v1, v2;
            triVerts(tri, v0, v1, v2);
            const LocalTri lt = localTriangle(cen, rot, v0, v1, v2);
            const Sat sat = carTriSat(lt);
            V3 clip[2 * MAX_PAIR_CONTACTS];
            pairContacts(lt, sat, clip, clip + MAX_PAIR_CONTACTS, [&](const Contact& c) {
                if (nearManifoldPoint(pts, planeCount, c.carPos)) return;
                const float d = -c.depth;
                if (d < bestDist) { bestDist = d; best = c; bestTri = tri; }
            });
        }
        if (bestTri >= 0)
        {
            V3 v0, v1, v2;
            triVerts(bestTri, v0, v1, v2);
            adjustInternalEdge(localTriangle(cen, rot, v0, v1, v2), triAngles(bestTri), best);
            addManifoldPoint(pts, count, contactToManifold(best, cen, rot));
        }
        if (count > 0)
        {
            solveCarManifold(body, pts, count);
            integrateSplitCorrection(body);
        }
        C.n(C_MAN_COUNT, i) = count;
        C.setv(C_MAN_N0, i, count > 0 ? pts[0].worldNormal : v3zero());
        body.vel = body.vel + body.extVel + body.deltaVel;
        body.ang = body.ang + body.extAng + body.deltaAng;
        storeCarBody(C, (int)i, body);
        storeSusp(C, i, su);
        for (int w = 0; w < 4; w++)
        {
            C.f(C_LAT + w, i) = lat[w];
            C.f(C_LON + w, i) = lon[w];
        }
    }
    // Per sim: car-car, then ball.
    for (int s = 0; s < nSim; s++)
    {
        const int sb = s * nCars;
        V3 clip[16];
        SimCars<SmemSoa> sc{ C, sb, nCars, nBlue, sb, tick, seed, clip };
        int pair = 0;
        for (int a = 0; a < nCars - 1; a++)
            for (int b = a + 1; b < nCars; b++, pair++)
            {
                const int kept = solveCarCarPair(sc, b, a);
                if (!diagSim.empty() && pair < DIAG_SIM_WORDS) diagSim[pair * nSim + s] = kept;
            }

        const V3 ballVel = S.v(S_BVEL, s), ballAng = S.v(S_BANG, s);
        const bool sleeping = lensq(ballVel) == 0.f && lensq(ballAng) == 0.f;
        const V3 exportedPos = S.v(S_BPOS, s);
        const bool valid = S.n(S_IVALID, s) != 0;
        V3 posBT = valid && lensq(exportedPos - S.v(S_EPOS, s)) == 0.f ? S.v(S_IPOS, s) : exportedPos * .02f;
        V3 velBT = valid && lensq(ballVel - S.v(S_EVEL, s)) == 0.f ? S.v(S_IVEL, s) : ballVel * .02f;
        const V3 dampedBT = sleeping ? velBT : velBT * powf(1.f - BALL_DRAG, PHYS_DT);
        const V3 preSolveBT = sleeping ? velBT : dampedBT + (V3{ 0.f, 0.f, GRAVITY_Z } * .02f) * PHYS_DT;
        const V3 velNoExt = dampedBT * 50.f;
        const V3 preSolveVel = preSolveBT * 50.f;
        V3 pushVel = v3zero();
        if (!sleeping)
        {
            const V3 center = exportedPos;
            const V3 ext = v3fill(BALL_COLLISION_RADIUS + BALL_ARENA_CONTACT_BREAK);
            const I3 lo = gridCell(center - ext), hi = gridCell(center + ext);
            std::vector<int> tris;
            for (int z = lo.z; z <= hi.z; z++)
                for (int y = lo.y; y <= hi.y; y++)
                    for (int x = lo.x; x <= hi.x; x++)
                    {
                        const int c = flatCell(I3{ x, y, z });
                        for (int e = arena.cellStart[c]; e < arena.cellStart[c + 1]; e++) tris.push_back(arena.cellTris[e]);
                    }
            std::sort(tris.begin(), tris.end());
            tris.erase(std::unique(tris.begin(), tris.end()), tris.end());
            BallContact set[4];
            int count = 0;
            for (int tri : tris)
            {
                V3 v0, v1, v2;
                triVerts(tri, v0, v1, v2);
                BallContact c;
                if (sphereTriangle(center, BALL_COLLISION_RADIUS, v0, v1, v2, c))
                    insertBallContact(set, count, c, center, v0, v1, v2, triAngles(tri));
            }
            bool wasHit = false;
            for (int k = 0; k < nCars; k++)
            {
                const int ht = C.n(C_BALL_HIT_TICK, sb + k);
                wasHit |= ballHitPreviousTick(ht, tick);
            }
            BallBody body;
            body.pos = center;
            body.vel = preSolveVel;
            body.velNoExt = velNoExt;
            body.ang = ballAng;
            body.deltaVel = body.deltaAng = body.pushVel = body.pushAng = v3zero();
            solveBallArena(body, set, count, wasHit);
            S.setv(S_BVEL, s, body.vel);
            S.setv(S_BANG, s, body.ang);
            pushVel = body.pushVel;
        }
        for (int k = 0; k < nCars; k++)
        {
            const int i = sb + k;
            if (!C.n(C_DEMOED, i) && ballCarGate(exportedPos, C.v(C_CEN, i)))
                solveBallCar(C, i, S, s, preSolveVel, tick);
        }
        const V3 corrected = S.v(S_BPOS, s);
        if (lensq(corrected - exportedPos) != 0.f) posBT = corrected * .02f;
        const V3 finalVel = S.v(S_BVEL, s);
        velBT = lensq(finalVel - preSolveVel) == 0.f ? preSolveBT : finalVel * .02f;
        posBT = posBT + (pushVel * .02f) * PHYS_DT;
        posBT = posBT + velBT * PHYS_DT;
        const V3 ballPos = posBT * 50.f;
        S.setv(S_BPOS, s, ballPos);
        S.setv(S_IPOS, s, posBT);
        S.setv(S_IVEL, s, velBT);
        S.setv(S_EPOS, s, ballPos);
        S.setv(S_EVEL, s, finalVel);
        S.n(S_IVALID, s) = 1;
        detectGoal(S, s, ballPos, tick);
    }
    // Integrate, finish.
    for (long long i = 0; i < n; i++)
    {
        if (!C.n(C_DEMOED, i))
        {
            V3 pos = C.v(C_POS, i), cen, vel = C.v(C_VEL, i), ang = C.v(C_ANG, i);
            Q4 rot = C.q(C_ROT, i);
            integratePose(pos, cen, rot, vel, ang);
            clampCarVelocity(vel, ang);
            C.setv(C_POS, i, pos);
            C.setv(C_VEL, i, vel);
            C.setv(C_ANG, i, ang);
            C.setv(C_CEN, i, cen);
            C.setq(C_ROT, i, rot);
        }
        const bool respawned = finishCar(C, (int)i, ctl[i].steer, (i % nCars) >= nBlue, T);
        for (int w = 0; w < 4; w++)
        {
            O.f(O_RAY_DIST + w, i) = rayDist[4 * i + w];
            O.setv(O_RAY_NORMAL + 3 * w, i, rayNormal[4 * i + w]);
            O.n(O_WHEEL_SRC + w, i) = src[4 * i + w];
            O.n(O_WHEEL_CON + w, i) = respawned ? 0 : (src[4 * i + w] != WHEEL_NONE && rayDist[4 * i + w] <= suspRayLength(w));
        }
        O.f(O_CONTROLS + 0, i) = ctl[i].throttle;
        O.f(O_CONTROLS + 1, i) = ctl[i].steer;
        O.f(O_CONTROLS + 2, i) = ctl[i].yaw;
        O.f(O_CONTROLS + 3, i) = ctl[i].pitch;
        O.f(O_CONTROLS + 4, i) = ctl[i].roll;
        O.n(O_CONTROLS + 5, i) = ctl[i].jump;
        O.n(O_CONTROLS + 6, i) = ctl[i].boost;
        O.n(O_CONTROLS + 7, i) = ctl[i].slide;
    }
    for (int s = 0; s < nSim; s++) finishBall(S, s);
    for (int s = 0; s < nSim; s++)
        for (int p = 0; p < NUM_BOOST_PADS; p++) boostPad(C, s * nCars, nCars, S, s, p, T);
}

struct Map
{
    float* base;
    long long stride, rows;
    int word, width;
    bool tick = false;
};

bool mapField(HostEnv* e, int f, Map& m)
{
    auto carW = [&](int w, int k) { m = Map{ e->car.data(), e->n, e->n, w, k }; };
    auto outW = [&](int w, int k) { m = Map{ e->out.data(), e->n, e->n, w, k }; };
    auto simW = [&](int w, int k) { m = Map{ e->sim.data(), e->nSim, e->nSim, w, k }; };
    switch (f)
    {
    case CARLB_F_CAR_POS: carW(C_POS, 3); return true;
    case CARLB_F_CAR_VEL: carW(C_VEL, 3); return true;
    case CARLB_F_CAR_ANG: carW(C_ANG, 3); return true;
    case CARLB_F_CAR_ROT: carW(C_ROT, 4); return true;
    case CARLB_F_CAR_CEN: carW(C_CEN, 3); return true;
    case CARLB_F_CAR_IMP: carW(C_IMP, 3); return true;
    case CARLB_F_CAR_IS_DEMOED: carW(C_DEMOED, 1); return true;
    case CARLB_F_CAR_DEMO_TIMER: carW(C_DEMO_TIMER, 1); return true;
    case CARLB_F_CAR_CONTACT_IDX: carW(C_CONTACT_IDX, 1); return true;
    case CARLB_F_CAR_CONTACT_COOLDOWN: carW(C_CONTACT_CD, 1); return true;
    case CARLB_F_CAR_BALL_HIT_TICK: carW(C_BALL_HIT_TICK, 1); return true;
    case CARLB_F_CAR_BALL_CONTACT_TICK: carW(C_BALL_CONTACT_TICK, 1); return true;
    case CARLB_F_CAR_WHEEL_SOURCE: outW(O_WHEEL_SRC, 4); return true;
    case CARLB_F_CAR_WHEEL_CONTACT: outW(O_WHEEL_CON, 4); return true;
    case CARLB_F_CAR_ARENA_CONTACT_TICK: outW(O_ARENA_CONTACT_TICK, 1); return true;
    case CARLB_F_CAR_CONTROLS: outW(O_CONTROLS, 8); return true;
    case CARLB_F_CAR_INTERNAL: carW(C_INT, 24); return true;
    case CARLB_F_SUSP_SCALARS: carW(C_SUSP, 15); return true;
    case CARLB_F_SUSP_RAY_DIST: outW(O_RAY_DIST, 4); return true;
    case CARLB_F_SUSP_RAY_NORMAL: outW(O_RAY_NORMAL, 12); return true;
    case CARLB_F_SUSP_LAT_FRICTION: carW(C_LAT, 4); return true;
    case CARLB_F_SUSP_LON_FRICTION: carW(C_LON, 4); return true;
    case CARLB_F_MAN_COUNT: carW(C_MAN_COUNT, 1); return true;
    case CARLB_F_MAN_NORMAL0: carW(C_MAN_N0, 3); return true;
    case CARLB_F_BALL_POS: simW(S_BPOS, 3); return true;
    case CARLB_F_BALL_VEL: simW(S_BVEL, 3); return true;
    case CARLB_F_BALL_ANG: simW(S_BANG, 3); return true;
    case CARLB_F_BALL_IMP: simW(S_BIMP, 3); return true;
    case CARLB_F_BALL_INT_POS: simW(S_IPOS, 3); return true;
    case CARLB_F_BALL_INT_VEL: simW(S_IVEL, 3); return true;
    case CARLB_F_BALL_EXP_POS: simW(S_EPOS, 3); return true;
    case CARLB_F_BALL_EXP_VEL: simW(S_EVEL, 3); return true;
    case CARLB_F_BALL_INT_VALID: simW(S_IVALID, 1); return true;
    case CARLB_F_EPISODE_TICKS: simW(S_EP_TICKS, 1); return true;
    case CARLB_F_LAST_TOUCH_TICKS: simW(S_LAST_TOUCH, 1); return true;
    case CARLB_F_BALL_ARENA_CONTACT_TICK:
        m = Map{ reinterpret_cast<float*>(e->simOut.data()), e->nSim, e->nSim, 0, 1 }; return true;
    case CARLB_F_GOALS: simW(S_GOALS, 5); return true;
    case CARLB_F_PAD_COOLDOWNS: simW(S_PADS, NUM_BOOST_PADS); return true;
    case CARLB_F_TICK_COUNT: m.tick = true; m.rows = 1; m.width = 1; return true;
    case CARLB_F_DIAG_CELL_IDX:
        m = Map{ reinterpret_cast<float*>(e->diagCar.data()), e->n, e->n, 0, 1 }; return true;
    case CARLB_F_DIAG_NUM_TRIS:
        m = Map{ reinterpret_cast<float*>(e->diagCar.data()), e->n, e->n, 1, 1 }; return true;
    case CARLB_F_DIAG_SAT_PAIRS:
        m = Map{ reinterpret_cast<float*>(e->diagCar.data()), e->n, e->n, 2, 33 }; return true;
    case CARLB_F_DIAG_CC_COUNT:
    {
        const int pairs = e->nCars * (e->nCars - 1) / 2;
        m = Map{ reinterpret_cast<float*>(e->diagSim.data()), e->nSim, e->nSim, 0, pairs > 0 ? pairs : 1 };
        return true;
    }
    default: return false;
    }
}

}  // namespace

extern "C" {

const char* hosttick_error() { return g_error.c_str(); }

void* hosttick_create(const char* arenaPath, int nSim, int nBlue, int nOrange, int seed)
{
    auto* e = new HostEnv;
    e->nSim = nSim;
    e->nBlue = nBlue;
    e->nOrange = nOrange;
    e->nCars = nBlue + nOrange;
    e->seed = seed;
    e->n = (long long)nSim * e->nCars;
    g_error = buildArena(arenaPath, e->arena);
    if (!g_error.empty())
    {
        delete e;
        return nullptr;
    }
    buildTables(e->T);
    e->car.assign((size_t)NCW * e->n, 0.f);
    e->out.assign((size_t)NOW * e->n, 0.f);
    e->sim.assign((size_t)NSW * nSim, 0.f);
    e->simOut.assign(nSim, -1);
    e->diagCar.assign((size_t)DIAG_CAR_WORDS * e->n, 0);
    e->diagSim.assign((size_t)DIAG_SIM_WORDS * nSim, 0);
    return e;
}

void hosttick_destroy(void* h) { delete static_cast<HostEnv*>(h); }

int hosttick_read_field(void* h, int f, uint32_t* out)
{
    auto* e = static_cast<HostEnv*>(h);
    Map m;
    if (!mapField(e, f, m)) return 1;
    if (m.tick)
    {
        out[0] = (uint32_t)e->tick;
        return 0;
    }
    const uint32_t* base = reinterpret_cast<const uint32_t*>(m.base);
    for (long long r = 0; r < m.rows; r++)
        for (int k = 0; k < m.width; k++) out[r * m.width + k] = base[(m.word + k) * m.stride + r];
    return 0;
}

int hosttick_write_field(void* h, int f, const uint32_t* in)
{
    auto* e = static_cast<HostEnv*>(h);
    Map m;
    if (!mapField(e, f, m) || f >= CARLB_F_DIAG_CELL_IDX) return 1;
    if (m.tick)
    {
        e->tick = (int)in[0];
        return 0;
    }
    uint32_t* base = reinterpret_cast<uint32_t*>(m.base);
    for (long long r = 0; r < m.rows; r++)
        for (int k = 0; k < m.width; k++) base[(m.word + k) * m.stride + r] = in[r * m.width + k];
    return 0;
}

// Direct controls ([n, 8] words), `ticks` ticks.
int hosttick_ticks(void* h, const uint32_t* controls, int ticks)
{
    auto* e = static_cast<HostEnv*>(h);
    std::vector<Controls> ctl(e->n);
    for (long long i = 0; i < e->n; i++)
    {
        const uint32_t* w = controls + 8 * i;
        std::memcpy(&ctl[i].throttle, &w[0], 4);
        std::memcpy(&ctl[i].steer, &w[1], 4);
        std::memcpy(&ctl[i].yaw, &w[2], 4);
        std::memcpy(&ctl[i].pitch, &w[3], 4);
        std::memcpy(&ctl[i].roll, &w[4], 4);
        ctl[i].jump = (int)w[5];
        ctl[i].boost = (int)w[6];
        ctl[i].slide = (int)w[7];
    }
    for (int t = 0; t < ticks; t++) e->step(ctl.data());
    return 0;
}

}  // extern "C"

extern "C" {

// Product arena build (carl_b200/csrc/arena.cpp) for the arena parity test:
// sizes = {nVerts, nTris, nCells, nRefs}.
int hosttick_arena_sizes(void* h, int* sizes)
{
    auto* e = static_cast<HostEnv*>(h);
    sizes[0] = e->arena.nVerts();
    sizes[1] = e->arena.nTris();
    sizes[2] = (int)e->arena.cellStart.size() - 1;
    sizes[3] = e->arena.cellStart.back();
    return 0;
}

int hosttick_arena_tables(void* h, float* verts, int* tris, int* cellStart, int* cellTris, float* edgeAngles,
                          float* normals, int* flags)
{
    auto* e = static_cast<HostEnv*>(h);
    const ArenaHost& a = e->arena;
    std::memcpy(verts, a.verts.data(), a.verts.size() * 4);
    std::memcpy(tris, a.tris.data(), a.tris.size() * 4);
    std::memcpy(cellStart, a.cellStart.data(), a.cellStart.size() * 4);
    std::memcpy(cellTris, a.cellTris.data(), a.cellTris.size() * 4);
    std::memcpy(edgeAngles, a.edgeAngles.data(), a.edgeAngles.size() * 4);
    std::memcpy(normals, a.normals.data(), a.normals.size() * 4);
    std::memcpy(flags, a.triFlags.data(), a.triFlags.size() * 4);
    return 0;
}

}  // extern "C"

extern "C" int hosttick_kickoff_table(void* h, int* out)
{
    auto* e = static_cast<HostEnv*>(h);
    for (int r = 0; r < 120; r++)
        for (int k = 0; k < 4; k++) out[4 * r + k] = e->T.kickoffPerm[r][k];
    return 0;
}

// Product ball grid (carl_b200/csrc/arena.cpp) for the ball-grid coverage test:
// geom = {origin x, y, z, cell size}, dims = {x, y, z, entries}.
extern "C" int hosttick_ball_grid(void* h, float* geom, int* dims)
{
    auto* e = static_cast<HostEnv*>(h);
    for (int k = 0; k < 3; k++)
    {
        geom[k] = e->arena.ballOrigin[k];
        dims[k] = e->arena.ballDims[k];
    }
    geom[3] = e->arena.ballCell;
    dims[3] = (int)e->arena.ballCellTris.size();
    return 0;
}

// Loads native mesh metadata into the env's arena tables (carl_b200/csrc/arena.cpp
// loadNativeMetadata): 0, or 1 with the error in hosttick_error().
extern "C" int hosttick_load_metadata(void* h, const char* path)
{
    auto* e = static_cast<HostEnv*>(h);
    g_error = loadNativeMetadata(path, e->arena);
    return g_error.empty() ? 0 : 1;
}

extern "C" int hosttick_ball_lists(void* h, int* start, int* tris)
{
    auto* e = static_cast<HostEnv*>(h);
    std::memcpy(start, e->arena.ballCellStart.data(), e->arena.ballCellStart.size() * 4);
    std::memcpy(tris, e->arena.ballCellTris.data(), e->arena.ballCellTris.size() * 4);
    return 0;
}
