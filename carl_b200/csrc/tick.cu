// The batched tick as a sequence of sm_100a stage kernels.
//
// Every stage kernel works on the persistent state in global memory (word-major
// SoA, resident in the 126 MB L2 between stages), so each stage runs at its own
// occupancy and no warp waits on a CTA barrier for unrelated work.  Within a tick
// the stages run in the reference's order (jwmccarthy/CARL src/Kernels.cu:15-202,
// src/RLEnvironment.cu:166-211):
//
//   begin step -> broadphase -> suspension raycast -> controls -> SAT/clip ->
//   suspension + manifold + solve -> car-car -> ball (arena, cars, integrate,
//   goal) -> integrate cars -> finish tick (impulses, demo respawn) -> pads
//
// The (car, candidate triangle) work of the raycasts and the SAT is flattened over
// a CTA with a block scan and spread evenly over its threads (cells hold 0-262
// triangles, so per-car loops would leave most lanes idle); the wheel ray minimum
// is an atomicMin on (distance bits, candidate) keys, which picks the same
// triangle as the reference's first-minimum scan; SAT hits are a per-car bitmask
// of candidate numbers, processed in candidate order.  All physics arithmetic
// lives in cb_*.cuh and keeps the reference's fp32 operation order (the file is
// compiled with --fmad=false).
#include "tick.cuh"

#include "../../include/carlb.h"

#include <algorithm>
#include <mutex>

#include <cuda_runtime.h>

#include "cb_misc.cuh"

namespace cb {

namespace {

constexpr int WARP_HIT_BUF = 256;    // ball-arena triangle hits gathered per warp
constexpr int WARP_WORDS = WARP_HIT_BUF + 8;
constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ float rayLen(int w) { return suspRayLength(w); }

__device__ __forceinline__ void loadTri(const ArenaDev& a, int tri, V3& v0, V3& v1, V3& v2, int& flags)
{
    const float4 p0 = __ldg(&a.triV[3 * tri]);
    const float4 p1 = __ldg(&a.triV[3 * tri + 1]);
    const float4 p2 = __ldg(&a.triV[3 * tri + 2]);
    v0 = V3{ p0.x, p0.y, p0.z };
    v1 = V3{ p1.x, p1.y, p1.z };
    v2 = V3{ p2.x, p2.y, p2.z };
    flags = __float_as_int(p0.w);
}

__device__ __forceinline__ V3 triAngles(const ArenaDev& a, int tri)
{
    const float4 g = __ldg(&a.triAng[tri]);
    return V3{ g.x, g.y, g.z };
}

__device__ __forceinline__ unsigned long long rayKey(float dist, unsigned cand)
{
    return ((unsigned long long)__float_as_uint(dist) << 32) | cand;
}

// Decodes the controls of car `gi` (env-global row in the action array).
__device__ Controls decodeAction(const void* actions, int kind, long long row)
{
    if (kind == ACT_DISCRETE)
    {
        const int32_t* a = static_cast<const int32_t*>(actions) + row * 7;
        int32_t v[7];
        #pragma unroll
        for (int k = 0; k < 7; k++) v[k] = a[k];
        return decodeDiscrete(v);
    }
    if (kind == ACT_CONTINUOUS)
    {
        const float* a = static_cast<const float*>(actions) + row * 7;
        float v[7];
        #pragma unroll
        for (int k = 0; k < 7; k++) v[k] = a[k];
        return decodeContinuous(v);
    }
    const float* a = static_cast<const float*>(actions) + row * 8;
    Controls c;
    c.throttle = a[0];
    c.steer = a[1];
    c.yaw = a[2];
    c.pitch = a[3];
    c.roll = a[4];
    c.jump = __float_as_int(a[5]);
    c.boost = __float_as_int(a[6]);
    c.slide = __float_as_int(a[7]);
    return c;
}

// ---- ball stage, part 1: arena contacts of one sim ------------------------------------------
//
// Per-sim values handed between the parts (15 scratch words, one row per sim):
// 0-2 the exported position at stage start, 3-5 posBT, 6-8 preSolveBT, 9-11 pushVel,
// 12-14 velNoExt.

struct BallPre
{
    V3 exportedPos, posBT, preSolveBT, velNoExt;
    bool sleeping;
};

// The ball's integration inputs at stage start (include/Physics/BallArena/Solve.cuh:61-82).
template <class T>
CB_D BallPre ballPre(const T& sims, int s)
{
    const V3 ballVel = sims.v(S_BVEL, s);
    const V3 ballAng = sims.v(S_BANG, s);
    BallPre b;
    b.sleeping = lensq(ballVel) == 0.f && lensq(ballAng) == 0.f;
    b.exportedPos = sims.v(S_BPOS, s);
    const bool valid = sims.n(S_IVALID, s) != 0;
    b.posBT = valid && lensq(b.exportedPos - sims.v(S_EPOS, s)) == 0.f ? sims.v(S_IPOS, s) : b.exportedPos * .02f;
    const V3 velBT = valid && lensq(ballVel - sims.v(S_EVEL, s)) == 0.f ? sims.v(S_IVEL, s) : ballVel * .02f;
    const V3 dampedBT = b.sleeping ? velBT : velBT * powf(1.f - BALL_DRAG, PHYS_DT);
    b.preSolveBT = b.sleeping ? velBT : dampedBT + (V3{ 0.f, 0.f, GRAVITY_Z } * .02f) * PHYS_DT;
    b.velNoExt = dampedBT * 50.f;
    return b;
}

CB_D void storeBallScratch(float* scratch, int stride, int s, const V3* v, int first, int count)
{
    for (int k = first; k < first + count; k++)
    {
        scratch[(3 * k) * stride + s] = v[k - first].x;
        scratch[(3 * k + 1) * stride + s] = v[k - first].y;
        scratch[(3 * k + 2) * stride + s] = v[k - first].z;
    }
}

CB_D V3 loadBallScratch(const float* scratch, int stride, int s, int k)
{
    return V3{ scratch[(3 * k) * stride + s], scratch[(3 * k + 1) * stride + s], scratch[(3 * k + 2) * stride + s] };
}

// Native-metadata arena contacts of the ball (lane 0): entry `e` of the ball-cell
// list (triangles in traversal-key order) is offered to the per-mesh reduction.
// Returns false when the triangle makes no contact.
__device__ bool nativeBallContact(const ArenaDev& arena, int tri, V3 centerBT, BallContact& c, int& mesh)
{
    const float4 p0 = __ldg(&arena.nativeV[3 * tri]), p1 = __ldg(&arena.nativeV[3 * tri + 1]);
    const float4 p2 = __ldg(&arena.nativeV[3 * tri + 2]);
    mesh = __float_as_int(p0.w);
    if (mesh < 0) return false;
    return nativeSphereTriangle(centerBT, V3{ p0.x, p0.y, p0.z }, V3{ p1.x, p1.y, p1.z }, V3{ p2.x, p2.y, p2.z }, c);
}

// Reduction state of the native branch: contacts are kept four per native mesh
// (meshes arrive in traversal order, so each mesh's contacts are contiguous).
struct NativeBallSet
{
    BallContact set[MAX_BALL_ARENA_CONTACTS];
    int count = 0, mesh = -1, base = 0, local = 0;

    __device__ void offer(const ArenaDev& arena, int tri, V3 center, V3 centerBT, BallContact c, int cmesh)
    {
        if (cmesh != mesh)
        {
            base = count;
            local = 0;
            mesh = cmesh;
        }
        int slot;
        if (local < 4)
        {
            // Room for the four plane contacts stays reserved (more than 16
            // contacting meshes would overflow the reference's own arrays).
            if (count >= MAX_BALL_ARENA_CONTACTS - 4) return;
            slot = local++;
            count++;
        }
        else
        {
            slot = ballContactReplacement(set + base, c);
        }
        const float4 p0 = __ldg(&arena.nativeV[3 * tri]), p1 = __ldg(&arena.nativeV[3 * tri + 1]);
        const float4 p2 = __ldg(&arena.nativeV[3 * tri + 2]);
        const float4 ang = __ldg(&arena.nativeAng[tri]);
        adjustNativeBallEdgeNormal(c, V3{ p0.x, p0.y, p0.z }, V3{ p1.x, p1.y, p1.z }, V3{ p2.x, p2.y, p2.z },
                                   V3{ ang.x, ang.y, ang.z }, __float_as_int(ang.w));
        c.point = centerBT + c.relPos + c.normal * c.depth;
        c.tri = tri;
        set[base + slot] = c;
    }
};

// Arena contacts and solve of a moving ball with native mesh metadata, one warp:
// the ball-cell list is tested across lanes, the per-mesh reduction in
// traversal order and the solve run on lane 0, which returns the push velocity.
__device__ V3 ballArenaSolveNative(const SmemSoa& cars, const SmemSoa& sims, int s, int nCars, int tick,
                                   const ArenaDev& arena, int* wbuf, int lane, const BallPre& b, int start, int end)
{
    const V3 center = b.exportedPos;
    const V3 centerBT = center * .02f;
    int& hitCount = wbuf[WARP_HIT_BUF];
    if (lane == 0) hitCount = 0;
    __syncwarp();
    for (int e = start + lane; e < end; e += 32)
    {
        BallContact c;
        int mesh;
        if (nativeBallContact(arena, __ldg(&arena.ballCellTris[e]), centerBT, c, mesh))
        {
            const int slot = atomicAdd(&hitCount, 1);
            if (slot < WARP_HIT_BUF) wbuf[slot] = e;
        }
    }
    __syncwarp();
    V3 pushVel = v3zero();
    if (lane == 0)
    {
        NativeBallSet ns;
        const int n = hitCount;
        if (n <= WARP_HIT_BUF)
        {
            // Entry order is traversal-key order.
            for (int i = 1; i < n; i++)
            {
                const int v = wbuf[i];
                int j = i - 1;
                while (j >= 0 && wbuf[j] > v)
                {
                    wbuf[j + 1] = wbuf[j];
                    j--;
                }
                wbuf[j + 1] = v;
            }
            for (int i = 0; i < n; i++)
            {
                const int tri = __ldg(&arena.ballCellTris[wbuf[i]]);
                BallContact c;
                int mesh;
                nativeBallContact(arena, tri, centerBT, c, mesh);
                ns.offer(arena, tri, center, centerBT, c, mesh);
            }
        }
        else
        {
            for (int e = start; e < end; e++)
            {
                const int tri = __ldg(&arena.ballCellTris[e]);
                BallContact c;
                int mesh;
                if (nativeBallContact(arena, tri, centerBT, c, mesh)) ns.offer(arena, tri, center, centerBT, c, mesh);
            }
        }
        const int count = finishNativeBallContacts(ns.set, ns.count, center);
        bool wasHit = false;
        for (int k = 0; k < nCars; k++) wasHit |= ballHitPreviousTick(cars.n(C_BALL_HIT_TICK, s * nCars + k), tick);
        BallBody body;
        body.pos = center;
        body.vel = b.preSolveBT * 50.f;
        body.velNoExt = b.velNoExt;
        body.ang = sims.v(S_BANG, s);
        body.deltaVel = body.deltaAng = body.pushVel = body.pushAng = v3zero();
        solveBallArenaN<MAX_BALL_ARENA_CONTACTS>(body, ns.set, count, wasHit);
        sims.setv(S_BVEL, s, body.vel);
        sims.setv(S_BANG, s, body.ang);
        pushVel = body.pushVel;
    }
    return pushVel;
}

// Arena contacts and solve of a moving ball, executed by one warp: triangles of
// the grid cells around the ball are tested across lanes, the order-dependent
// contact reduction and solve run on lane 0, which returns the push velocity.
__device__ V3 ballArenaSolve(const SmemSoa& cars, const SmemSoa& sims, int s, int nCars, int tick,
                             const ArenaDev& arena, int* wbuf, int lane, const BallPre& b)
{
    const int carBase = s * nCars;
    const V3 ballAng = sims.v(S_BANG, s);
    const V3 preSolveVel = b.preSolveBT * 50.f;
    const V3 velNoExt = b.velNoExt;
    const V3 exportedPos = b.exportedPos;
    V3 pushVel = v3zero();
    // Arena triangles of the ball-grid cell holding the ball centre (it lists every
    // triangle within the contact reach of any point of the cell), tested across lanes.
    const V3 center = exportedPos;
    const float4 g = arena.ballGrid;
    const float fx = (center.x - g.x) * g.w, fy = (center.y - g.y) * g.w, fz = (center.z - g.z) * g.w;
    int start = 0, end = 0;
    if (fx >= 0.f && fx < (float)arena.ballDimX && fy >= 0.f && fy < (float)arena.ballDimY && fz >= 0.f &&
        fz < (float)arena.ballDimZ)
    {
        const int c = (int)fx + arena.ballDimX * ((int)fy + arena.ballDimY * (int)fz);
        start = __ldg(&arena.ballCellStart[c]);
        end = __ldg(&arena.ballCellStart[c + 1]);
    }
    if (arena.hasNative) return ballArenaSolveNative(cars, sims, s, nCars, tick, arena, wbuf, lane, b, start, end);
    int& hitCount = wbuf[WARP_HIT_BUF];
    if (lane == 0) hitCount = 0;
    __syncwarp();
    for (int e = start + lane; e < end; e += 32)
    {
        // A triangle beyond the contact radius (plus 1 uu) cannot touch the ball.
        const float4 sph = __ldg(&arena.ballCellSph[e]);
        const float dx = sph.x - center.x, dy = sph.y - center.y, dz = sph.z - center.z;
        const float rr = sph.w + (BALL_COLLISION_RADIUS + BALL_ARENA_CONTACT_BREAK + 1.f);
        if (dx * dx + dy * dy + dz * dz > rr * rr) continue;
        const int tri = __ldg(&arena.ballCellTris[e]);
        V3 v0, v1, v2;
        int flags;
        loadTri(arena, tri, v0, v1, v2, flags);
        BallContact c;
        if (sphereTriangle(center, BALL_COLLISION_RADIUS, v0, v1, v2, c))
        {
            const int slot = atomicAdd(&hitCount, 1);
            if (slot < WARP_HIT_BUF) wbuf[slot] = tri;
        }
    }
    __syncwarp();

    if (lane == 0)
    {
        BallContact set[4];
        int count = 0;
        const int n = hitCount;
        if (n <= WARP_HIT_BUF)
        {
            // Ascending triangle order (the reference merges the per-cell lists in
            // triangle order; the ball cell's list has no repeats).
            for (int i = 1; i < n; i++)
            {
                const int v = wbuf[i];
                int j = i - 1;
                while (j >= 0 && wbuf[j] > v)
                {
                    wbuf[j + 1] = wbuf[j];
                    j--;
                }
                wbuf[j + 1] = v;
            }
            for (int i = 0; i < n; i++)
            {
                const int tri = wbuf[i];
                V3 v0, v1, v2;
                int flags;
                loadTri(arena, tri, v0, v1, v2, flags);
                BallContact c;
                sphereTriangle(center, BALL_COLLISION_RADIUS, v0, v1, v2, c);
                insertBallContact(set, count, c, center, v0, v1, v2, triAngles(arena, tri));
            }
        }
        else
        {
            // Too many hits to buffer: walk the (ascending) cell list directly.
            for (int e = start; e < end; e++)
            {
                const int tri = __ldg(&arena.ballCellTris[e]);
                V3 v0, v1, v2;
                int flags;
                loadTri(arena, tri, v0, v1, v2, flags);
                BallContact c;
                if (sphereTriangle(center, BALL_COLLISION_RADIUS, v0, v1, v2, c))
                    insertBallContact(set, count, c, center, v0, v1, v2, triAngles(arena, tri));
            }
        }

        bool wasHit = false;
        for (int k = 0; k < nCars; k++)
        {
            const int hitTick = cars.n(C_BALL_HIT_TICK, carBase + k);
            wasHit |= ballHitPreviousTick(hitTick, tick);
        }
        BallBody body;
        body.pos = center;
        body.vel = preSolveVel;
        body.velNoExt = velNoExt;
        body.ang = ballAng;
        body.deltaVel = body.deltaAng = body.pushVel = body.pushAng = v3zero();
        solveBallArena(body, set, count, wasHit);
        sims.setv(S_BVEL, s, body.vel);
        sims.setv(S_BANG, s, body.ang);
        pushVel = body.pushVel;
    }
    return pushVel;
}

// ---- ball stage, part 2: ball vs cars (in car order), integration, goal; one thread ----------
// `gate[k]` is the distance gate of the sim's car k against the ball's
// pre-contact position (computed by the car's own thread: a solve only moves its
// own car and the ball, so gating each car before the first solve is the same
// as gating it just before its own).
__device__ void ballFinishStage(const SmemSoa& cars, const SmemSoa& sims, int s, int nCars, int tick,
                                const float* scratch, int scratchStride, const unsigned char* gate)
{
    V3 in[4];
    #pragma unroll
    for (int k = 0; k < 4; k++)
        in[k] = V3{ scratch[(3 * k) * scratchStride + s], scratch[(3 * k + 1) * scratchStride + s],
                    scratch[(3 * k + 2) * scratchStride + s] };
    const V3 exportedPos = in[0];
    V3 posBT = in[1];
    const V3 preSolveBT = in[2];
    const V3 pushVel = in[3];
    const V3 preSolveVel = preSolveBT * 50.f;

    const int carBase = s * nCars;
    for (int k = 0; k < nCars; k++)
        if (gate[k]) solveBallCar(cars, carBase + k, sims, s, preSolveVel, tick);

    const V3 corrected = sims.v(S_BPOS, s);
    if (lensq(corrected - exportedPos) != 0.f) posBT = corrected * .02f;
    const V3 finalVel = sims.v(S_BVEL, s);
    const V3 velBT = lensq(finalVel - preSolveVel) == 0.f ? preSolveBT : finalVel * .02f;
    posBT = posBT + (pushVel * .02f) * PHYS_DT;
    posBT = posBT + velBT * PHYS_DT;
    const V3 ballPos = posBT * 50.f;
    sims.setv(S_BPOS, s, ballPos);
    sims.setv(S_IPOS, s, posBT);
    sims.setv(S_IVEL, s, velBT);
    sims.setv(S_EPOS, s, ballPos);
    sims.setv(S_EVEL, s, finalVel);
    sims.n(S_IVALID, s) = 1;
    detectGoal(sims, s, ballPos, tick);
}

// =========================================================================================
// Stage kernels, per tick and sim slice:
//   flatKernel     begin step, broadphase, (car, candidate) wheel rays + SAT, per CTA of cars
//   rayKernel      ray finish (arena hit, other cars' boxes, ball)
//   ctlSuspKernel  controls, then suspension; cars that may touch a plane or the mesh are listed
//   contactKernel  plane + mesh manifold and car-arena solve of the listed cars
//   ballPrepKernel ball prelude (moving balls are listed)
//   carCarKernel   car-car pairs per sim
//   ballKernel     ball arena contacts, one warp per listed ball
//   finishKernel   ball vs cars + integration + goal, car integration + finish, boost pads
// =========================================================================================

// Tick count before the first tick of the launch (device counter when set).
__device__ __forceinline__ int tickBase(const TickParams& p) { return p.tickDev ? *p.tickDev : p.tick0; }

__global__ void setTickKernel(int* dst, int value) { *dst = value; }

constexpr int CAND_BLOCK = 384;   // cars per flatKernel CTA: at 78 registers, 2 CTAs (768 threads) fill an SM's
                                  // register file; 128 and 256 measured slower (C3 880 and 898 against 905 M)
constexpr int CAND_MAP_CAP = 12288;  // items per CTA resolved through the shared item -> car map
constexpr int RAY_BLOCK = 128;    // cars per rayKernel CTA
constexpr int SOLVE_BLOCK = 128;  // cars per ctlSuspKernel / contactKernel CTA
constexpr int CC_BLOCK = 128;     // sims per carCarKernel CTA
constexpr int BALL_WARPS = 4;     // sims (warps) per ballKernel CTA
constexpr int FIN_THREADS = 256;  // threads per finishKernel CTA
constexpr int STAGE_MAX_GROUPS = 8;  // sim slices stepped on separate streams

using CarSoa = Soa<int>;  // int indexing: NCW * carStride < 2^31 is checked at launch

__global__ void __launch_bounds__(CAND_BLOCK) flatKernel(TickParams p, ArenaDev arena, StageScratch x, int t)
{
    extern __shared__ __align__(16) float sm[];
    const int B = CAND_BLOCK, HW = arena.hitWords;
    int* cntS = reinterpret_cast<int*>(sm);                 // [B]
    int* firstS = cntS + B;                                  // [B]
    int* preS = firstS + B;                                  // [B + 1]
    int* wsumS = preS + B + 1;                               // [32]
    float* rsS = reinterpret_cast<float*>(wsumS + 32);       // [15][B] ray starts (12), dir (3)
    float* poseS = rsS + 15 * B;                             // [7][B] cen (3), rot (4)
    unsigned* hitS = reinterpret_cast<unsigned*>(poseS + 7 * B);  // [HW][B]
    const size_t keyOff = ((size_t)(hitS + HW * B) - (size_t)sm + 7) & ~(size_t)7;
    unsigned long long* keyS = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(sm) + keyOff);  // [4][B]
    unsigned short* mapS = reinterpret_cast<unsigned short*>(keyS + 4 * B);  // [CAND_MAP_CAP] item -> car

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = p.nSim * p.nCars;
    const int first = blockIdx.x * B;
    const int here = min(B, n - first);
    const int i = first + tid;
    const bool valid = tid < here;
    const CarSoa cars{ p.car, (int)p.carStride };
    const CarSoa sims{ p.sim, (int)p.simStride };
    const bool lastTick = t == p.nTicks - 1;

    V3 cen = v3zero(), up = v3zero();
    Q4 rot = Q4{ 0.f, 0.f, 0.f, 1.f };
    if (valid)
    {
        if (i % p.nCars == 0) sims.n(S_EP_TICKS, i / p.nCars) += 1;
        const V3 pos = cars.v(C_POS, i), vel = cars.v(C_VEL, i), ang = cars.v(C_ANG, i);
        cen = cars.v(C_CEN, i);
        rot = cars.q(C_ROT, i);
        const int cell = broadphaseCell(pos, vel, ang, cen, rot);
        const int f0 = __ldg(&arena.cellStart[cell]);
        firstS[tid] = f0;
        cntS[tid] = __ldg(&arena.cellStart[cell + 1]) - f0;
        if (lastTick && p.diagCar) p.diagCar[0 * p.carStride + i] = cell;
        up = rotate(rot, axisVec(2));
        #pragma unroll
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            const V3 st = cen + rotate(rot, suspConnection(w));
            rsS[(3 * w) * B + tid] = st.x;
            rsS[(3 * w + 1) * B + tid] = st.y;
            rsS[(3 * w + 2) * B + tid] = st.z;
            keyS[w * B + tid] = rayKey(rayLen(w) + 1.f, 0xffffffffu);
        }
        const V3 dir = neg(up);
        rsS[12 * B + tid] = dir.x;
        rsS[13 * B + tid] = dir.y;
        rsS[14 * B + tid] = dir.z;
        poseS[0 * B + tid] = cen.x;
        poseS[1 * B + tid] = cen.y;
        poseS[2 * B + tid] = cen.z;
        poseS[3 * B + tid] = rot.x;
        poseS[4 * B + tid] = rot.y;
        poseS[5 * B + tid] = rot.z;
        poseS[6 * B + tid] = rot.w;
        for (int h = 0; h < HW; h++) hitS[h * B + tid] = 0u;
    }
    else
    {
        cntS[tid] = 0;
    }

    // Block exclusive scan of candidate counts.
    {
        int v = cntS[tid];
        #pragma unroll
        for (int d = 1; d < 32; d <<= 1)
        {
            const int u = __shfl_up_sync(FULL, v, d);
            if (lane >= d) v += u;
        }
        if (lane == 31) wsumS[warp] = v;
        __syncthreads();
        if (warp == 0)
        {
            int q = lane < B / 32 ? wsumS[lane] : 0;
            #pragma unroll
            for (int d = 1; d < 32; d <<= 1)
            {
                const int u = __shfl_up_sync(FULL, q, d);
                if (lane >= d) q += u;
            }
            if (lane < B / 32) wsumS[lane] = q;
        }
        __syncthreads();
        if (warp > 0) v += wsumS[warp - 1];
        preS[tid + 1] = v;
        if (tid == 0) preS[0] = 0;
        // Item -> car map for the first CAND_MAP_CAP items (later items search preS).
        const int cnt = cntS[tid];
        for (int k = v - cnt; k < v && k < CAND_MAP_CAP; k++) mapS[k] = (unsigned short)tid;
    }
    __syncthreads();

    // Flattened (car, candidate) work: wheel rays and SAT.  Two items per thread
    // per round, their loads issued together, to keep more of them in flight.
    const int total = preS[here];
    auto carOf = [&](int it) -> int {
        if (it < CAND_MAP_CAP) return mapS[it];
        int lo = 0, hi = here - 1;
        while (lo < hi)
        {
            const int mid = (lo + hi + 1) >> 1;
            if (preS[mid] <= it) lo = mid;
            else hi = mid - 1;
        }
        return lo;
    };
    auto inReach = [&](int c, float4 sph) -> bool {
        // Triangles out of reach of the box and the wheel rays cannot produce a
        // ray hit or a SAT overlap.
        const float dx = sph.x - poseS[0 * B + c], dy = sph.y - poseS[1 * B + c], dz = sph.z - poseS[2 * B + c];
        const float rr = sph.w + arena.carReach;
        return !(dx * dx + dy * dy + dz * dz > rr * rr);
    };
    auto process = [&](int c, int k, float4 q0, float4 q1, float4 q2) {
        const V3 v0 = { q0.x, q0.y, q0.z }, v1 = { q1.x, q1.y, q1.z }, v2 = { q2.x, q2.y, q2.z };
        const int flags = __float_as_int(q0.w);
        const V3 dir = { rsS[12 * B + c], rsS[13 * B + c], rsS[14 * B + c] };
        const V3 e1 = v1 - v0;
        const V3 e2 = v2 - v0;
        const V3 pv = cross(dir, e2);
        const float det = dot(e1, pv);
        if (!(fabsf(det) < RAY_PARALLEL_EPS))
        {
            const float invDet = 1.f / det;
            #pragma unroll
            for (int w = 0; w < NUM_WHEELS; w++)
            {
                const V3 st = { rsS[(3 * w) * B + c], rsS[(3 * w + 1) * B + c], rsS[(3 * w + 2) * B + c] };
                const V3 tv = st - v0;
                const float u = invDet * dot(tv, pv);
                if (u < 0.f || u > 1.f) continue;
                const V3 qv = cross(tv, e1);
                const float v = invDet * dot(dir, qv);
                if (v < 0.f || u + v > 1.f) continue;
                const float dist = invDet * dot(e2, qv);
                if (dist <= 0.f || !(dist < rayLen(w) + 1.f)) continue;
                atomicMin(&keyS[w * B + c], rayKey(dist, (unsigned)k));
            }
        }
        if (!(flags & 1))
        {
            const V3 cc = { poseS[0 * B + c], poseS[1 * B + c], poseS[2 * B + c] };
            const Q4 cr = { poseS[3 * B + c], poseS[4 * B + c], poseS[5 * B + c], poseS[6 * B + c] };
            // Plane pre-test in world space: a box whose centre is farther from the
            // triangle's plane than the box reaches along the normal, by more than the
            // entry's margin (q1.w, scaled by |n|; it bounds the rounding of this test
            // and of the car-frame one), is separated on the triangle-normal axis,
            // where the car-frame SAT would report no overlap too.  Only the other
            // triangles go through the exact SAT.
            const V3 nw = cross(e1, e2);
            const float off = dot(nw, cc - v0);
            const float ext = dot(vabs(unrotate(cr, nw)), carHalfExtents());
            if (!(fabsf(off) > ext + q1.w))
            {
                const LocalTri lt = localTriangle(cc, cr, v0, v1, v2);
                if (carTriSat(lt).overlap) atomicOr(&hitS[(k >> 5) * B + c], 1u << (k & 31));
            }
        }
    };
    for (int itA = tid; itA < total; itA += 2 * B)
    {
        const int itB = itA + B;
        const bool hasB = itB < total;
        const int cA = carOf(itA);
        const int cB = hasB ? carOf(itB) : cA;
        const int kA = itA - preS[cA];
        const int kB = hasB ? itB - preS[cB] : kA;
        const int eA = firstS[cA] + kA;
        const int eB = firstS[cB] + kB;
        const float4 sA = __ldg(&arena.cellSph[eA]);
        const float4 sB = __ldg(&arena.cellSph[eB]);
        const bool keepA = inReach(cA, sA);
        const bool keepB = hasB && inReach(cB, sB);
        float4 a0, a1, a2, b0, b1, b2;
        if (keepA)
        {
            a0 = __ldg(&arena.cellV[3 * eA]);
            a1 = __ldg(&arena.cellV[3 * eA + 1]);
            a2 = __ldg(&arena.cellV[3 * eA + 2]);
        }
        if (keepB)
        {
            b0 = __ldg(&arena.cellV[3 * eB]);
            b1 = __ldg(&arena.cellV[3 * eB + 1]);
            b2 = __ldg(&arena.cellV[3 * eB + 2]);
        }
        if (keepA) process(cA, kA, a0, a1, a2);
        if (keepB) process(cB, kB, b0, b1, b2);
    }
    __syncthreads();
    if (!valid) return;
    x.first[i] = firstS[tid];
    x.cnt[i] = cntS[tid];
    for (int h = 0; h < HW; h++) x.hits[(long long)h * p.carStride + i] = hitS[h * B + tid];
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++) x.keys[(long long)w * p.carStride + i] = keyS[w * B + tid];
}

// Wheel rays of a car: the arena hit found by the flat stage, then the other
// cars' boxes (car order) and the ball.  No control state is touched here, so
// the kernel needs few registers and a slice runs in one wave.
__global__ void __launch_bounds__(RAY_BLOCK) rayKernel(TickParams p, ArenaDev arena, StageScratch x, int t)
{
    const int n = p.nSim * p.nCars;
    const int i = blockIdx.x * RAY_BLOCK + threadIdx.x;
    if (i >= n) return;
    const CarSoa cars{ p.car, (int)p.carStride };
    const CarSoa sims{ p.sim, (int)p.simStride };
    const bool lastTick = t == p.nTicks - 1;
    const V3 cen = cars.v(C_CEN, i);
    const Q4 rot = cars.q(C_ROT, i);
    const V3 up = rotate(rot, axisVec(2));

    // Finish the wheel rays: arena hit, other cars' boxes (in car order), ball.
    const V3 dir = neg(up);
    float rayDist[NUM_WHEELS];
    V3 rayNormal[NUM_WHEELS];
    int src[NUM_WHEELS];
    V3 start[NUM_WHEELS];
    const int cellFirst = x.first[i];
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        start[w] = cen + rotate(rot, suspConnection(w));
        const unsigned long long key = x.keys[(long long)w * p.carStride + i];
        const unsigned cand = (unsigned)(key & 0xffffffffu);
        if (cand != 0xffffffffu)
        {
            rayDist[w] = __uint_as_float((unsigned)(key >> 32));
            V3 v0, v1, v2;
            int flags;
            loadTri(arena, __ldg(&arena.cellTris[cellFirst + (int)cand]), v0, v1, v2, flags);
            V3 nrm = cross(v1 - v0, v2 - v0);
            const float nl = lensq(nrm);
            nrm = nrm * rsqrtf(nl);
            if (dot(nrm, dir) > 0.f) nrm = neg(nrm);
            rayNormal[w] = nrm;
            src[w] = WHEEL_ARENA;
        }
        else
        {
            rayDist[w] = rayLen(w) + 1.f;
            rayNormal[w] = up;
            src[w] = WHEEL_NONE;
        }
    }
    const int mySim = i / p.nCars;
    const int sb = mySim * p.nCars;
    for (int k = 0; k < p.nCars; k++)
    {
        const int o = sb + k;
        if (o == i || cars.n(C_DEMOED, o)) continue;
        const V3 oc = cars.v(C_CEN, o);
        if (lensq(oc - cen) > 250.f * 250.f) continue;  // beyond any wheel ray + box reach
        const Q4 orot = cars.q(C_ROT, o);
        #pragma unroll
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            const V3 ls = unrotate(orot, start[w] - oc);
            const V3 ld = unrotate(orot, dir);
            float entry = 0.f, exitD = rayLen(w);
            int hitAxis = -1;
            bool miss = false;
            #pragma unroll
            for (int a = 0; a < 3; a++)
            {
                const float h = vget(carHalfExtents(), a);
                const float d = vget(ld, a), s0 = vget(ls, a);
                if (fabsf(d) < RAY_PARALLEL_EPS)
                {
                    if (fabsf(s0) > h) { miss = true; break; }
                    continue;
                }
                const float inv = 1.f / d;
                const float t1 = (-h - s0) * inv;
                const float t2 = (h - s0) * inv;
                const float tn = fminf(t1, t2);
                if (tn > entry)
                {
                    entry = tn;
                    hitAxis = a;
                }
                exitD = fminf(exitD, fmaxf(t1, t2));
                if (entry > exitD) { miss = true; break; }
            }
            if (miss || hitAxis < 0 || entry >= rayDist[w]) continue;
            V3 ln = v3zero();
            vset(ln, hitAxis, vget(ld, hitAxis) > 0.f ? -1.f : 1.f);
            rayDist[w] = entry;
            rayNormal[w] = rotate(orot, ln);
            src[w] = WHEEL_CAR;
        }
    }
    {
        const V3 bp = sims.v(S_BPOS, mySim);
        const float invR = 1.f / BALL_COLLISION_RADIUS;
        #pragma unroll
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            const V3 off = start[w] - bp;
            const float b = dot(off, dir);
            const float cq = lensq(off) - BALL_COLLISION_RADIUS * BALL_COLLISION_RADIUS;
            if (cq < 0.f) continue;
            const float disc = b * b - cq;
            if (disc < 0.f) continue;
            const float dist = -b - sqrtf(disc);
            if (!(dist > 0.f && dist <= rayLen(w))) continue;
            if (dist >= rayDist[w]) continue;
            rayDist[w] = dist;
            rayNormal[w] = (start[w] + dir * dist - bp) * invR;
            src[w] = WHEEL_BALL;
        }
    }
    unsigned wheelBits = 0;
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
        if (src[w] != WHEEL_NONE && rayDist[w] <= rayLen(w)) wheelBits |= 1u << w;
    x.wheelBits[i] = wheelBits;
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        x.ray[(long long)w * p.carStride + i] = rayDist[w];
        x.ray[(long long)(4 + 3 * w) * p.carStride + i] = rayNormal[w].x;
        x.ray[(long long)(5 + 3 * w) * p.carStride + i] = rayNormal[w].y;
        x.ray[(long long)(6 + 3 * w) * p.carStride + i] = rayNormal[w].z;
    }
    if (lastTick)
    {
        #pragma unroll
        for (int w = 0; w < NUM_WHEELS; w++)
        {
            p.carOut[(long long)(O_RAY_DIST + w) * p.carStride + i] = rayDist[w];
            p.carOut[(long long)(O_RAY_NORMAL + 3 * w) * p.carStride + i] = rayNormal[w].x;
            p.carOut[(long long)(O_RAY_NORMAL + 3 * w + 1) * p.carStride + i] = rayNormal[w].y;
            p.carOut[(long long)(O_RAY_NORMAL + 3 * w + 2) * p.carStride + i] = rayNormal[w].z;
            reinterpret_cast<int*>(p.carOut)[(long long)(O_WHEEL_SRC + w) * p.carStride + i] = src[w];
        }
    }

}

// Controls and suspension of a car, one thread each: the control state machine's
// outputs (velocities, suspension staging) feed the suspension in registers.
// Capped at 168 registers (3 CTAs per SM; 16 bytes spilled).
__global__ void __launch_bounds__(SOLVE_BLOCK, 3) ctlSuspKernel(TickParams p, ArenaDev arena, StageScratch x, int t)
{
    const int n = p.nSim * p.nCars;
    const int i = blockIdx.x * SOLVE_BLOCK + threadIdx.x;
    if (i >= n) return;
    const CarSoa cars{ p.car, (int)p.carStride };
    const int tick = tickBase(p) + t + 1;
    const bool lastTick = t == p.nTicks - 1;
    const int HW = arena.hitWords;
    const int cellFirst = x.first[i];
    bool anyHit = false;
    for (int h = 0; h < HW; h++) anyHit |= x.hits[(long long)h * p.carStride + i] != 0u;
    if (lastTick && p.diagCar)
    {
        p.diagCar[1 * p.carStride + i] = x.cnt[i];
        int nh = 0;
        for (int h = 0; h < HW && nh < MAX_CAR_TRI_PAIRS; h++)
            for (unsigned m = x.hits[(long long)h * p.carStride + i]; m && nh < MAX_CAR_TRI_PAIRS; m &= m - 1)
            {
                const int k = h * 32 + __ffs(m) - 1;
                p.diagCar[(3 + nh) * p.carStride + i] = __ldg(&arena.cellTris[cellFirst + k]);
                nh++;
            }
        p.diagCar[2 * p.carStride + i] = nh;
        for (int r = nh; r < MAX_CAR_TRI_PAIRS; r++) p.diagCar[(3 + r) * p.carStride + i] = -1;
    }
    // Controls (the ray stage has finished the wheel rays).
    float rayDist[NUM_WHEELS];
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++) rayDist[w] = x.ray[(long long)w * p.carStride + i];
    const bool demoed = cars.n(C_DEMOED, i) != 0;
    Susp su = loadSusp(cars, i);
    V3 velC = cars.v(C_VEL, i), angC = cars.v(C_ANG, i);
    {
        const Controls ctl = decodeAction(p.actions, p.actionKind, i);
        Internal st = loadInternal(cars, i);
        processControls(ctl, demoed, cars.q(C_ROT, i), velC, angC, st, su, rayDist, cars.n(C_MAN_COUNT, i),
                        cars.v(C_MAN_N0, i));
        storeInternal(cars, i, st);
    }
    if (demoed)
    {
        cars.setv(C_VEL, i, velC);
        cars.setv(C_ANG, i, angC);
        storeSusp(cars, i, su);
        return;
    }

    V3 rayNormal[NUM_WHEELS];
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
        rayNormal[w] = V3{ x.ray[(long long)(4 + 3 * w) * p.carStride + i], x.ray[(long long)(5 + 3 * w) * p.carStride + i],
                           x.ray[(long long)(6 + 3 * w) * p.carStride + i] };
    Body body = makeBody(cars.v(C_POS, i), velC, angC, cars.v(C_CEN, i), cars.q(C_ROT, i));
    float lat[NUM_WHEELS], lon[NUM_WHEELS];
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        lat[w] = cars.f(C_LAT + w, i);
        lon[w] = cars.f(C_LON + w, i);
    }
    applySuspension(body, su, lat, lon, rayDist, rayNormal, cars.n(C_MAN_COUNT, i), cars.v(C_MAN_N0, i), tick,
                    (p.compatFlags & CARLB_SOURCE_LAGGED_LATERAL_FRICTION) == 0);
    storeSusp(cars, i, su);
    #pragma unroll
    for (int w = 0; w < NUM_WHEELS; w++)
    {
        cars.f(C_LAT + w, i) = lat[w];
        cars.f(C_LON + w, i) = lon[w];
    }
    if (anyHit || planeContactAny(body.cen, body.rot))
    {
        // Plane or mesh contacts possible: the velocities after the suspension go
        // to the contact kernel, which builds the manifold and solves it.
        const V3 hv[6] = { body.vel, body.ang, body.extVel, body.extAng, body.deltaVel, body.deltaAng };
        #pragma unroll
        for (int k = 0; k < 6; k++)
        {
            x.heavyBody[(long long)(3 * k) * p.carStride + i] = hv[k].x;
            x.heavyBody[(long long)(3 * k + 1) * p.carStride + i] = hv[k].y;
            x.heavyBody[(long long)(3 * k + 2) * p.carStride + i] = hv[k].z;
        }
        // Two lists: cars with SAT hits (a warp each in the contact kernel, lanes
        // over the hits) and cars with plane contacts only (a thread each).
        const int cls = anyHit ? 1 : 0;
        x.heavyList[(long long)cls * p.carStride + atomicAdd(&x.heavyCount[cls], 1)] = i;
        return;
    }
    cars.n(C_MAN_COUNT, i) = 0;
    cars.setv(C_MAN_N0, i, v3zero());
    cars.setv(C_VEL, i, body.vel + body.extVel + body.deltaVel);
    cars.setv(C_ANG, i, body.ang + body.extAng + body.deltaAng);
}

// Velocities after the suspension of a listed car (from ctlSuspKernel).
__device__ __forceinline__ Body loadHeavyBody(const CarSoa& cars, const StageScratch& x, long long stride, int i)
{
    Body body = loadCarBody(cars, i);
    V3 hv[6];
    #pragma unroll
    for (int k = 0; k < 6; k++)
        hv[k] = V3{ x.heavyBody[(3 * k) * stride + i], x.heavyBody[(3 * k + 1) * stride + i],
                    x.heavyBody[(3 * k + 2) * stride + i] };
    body.vel = hv[0];
    body.ang = hv[1];
    body.extVel = hv[2];
    body.extAng = hv[3];
    body.deltaVel = hv[4];
    body.deltaAng = hv[5];
    return body;
}

// Manifold solve and final store of a listed car (src/Physics/CarArena/Solve.cuh order).
// Inlined, so the body and the manifold stay in registers (through a call they
// are passed in local memory, whose loads sit on the car's dependency chain).
// With the clip polygons in shared memory, the 3v3 bench measured 869-874 M
// agent-steps/s inlined with register manifolds against 866-870 out of line.
__device__ __forceinline__ void finishContactCar(const CarSoa& cars, int i, Body& body, MPoint* pts, int cnt)
{
    if (cnt > 0)
    {
        solveCarManifold(body, pts, cnt);
        integrateSplitCorrection(body);
    }
    cars.n(C_MAN_COUNT, i) = cnt;
    cars.setv(C_MAN_N0, i, cnt > 0 ? pts[0].worldNormal : v3zero());
    body.vel = body.vel + body.extVel + body.deltaVel;
    body.ang = body.ang + body.extAng + body.deltaAng;
    storeCarBody(cars, i, body);
}

// Plane and mesh contacts and the car-arena solve of the listed cars.  The first
// `planeBlocks` CTAs take the plane-only cars, a thread each; the others take the
// cars with SAT hits, a warp each: lane r builds the contacts of the r-th hit (in
// candidate order) and keeps its deepest (first on ties), and a warp reduction in
// hit order then picks exactly the contact the sequential loop over hits keeps.
__global__ void __launch_bounds__(SOLVE_BLOCK) contactKernel(TickParams p, ArenaDev arena, StageScratch x, int t,
                                                            int planeBlocks)
{
    const CarSoa cars{ p.car, (int)p.carStride };
    const long long stride = p.carStride;
    if ((int)blockIdx.x < planeBlocks)
    {
        const int count = x.heavyCount[0];
        for (int j = blockIdx.x * SOLVE_BLOCK + threadIdx.x; j < count; j += planeBlocks * SOLVE_BLOCK)
        {
            const int i = x.heavyList[j];
            Body body = loadHeavyBody(cars, x, stride, i);
            MPoint pts[MAX_CAR_MANIFOLD_POINTS];
            const int cnt = planeManifold(body.cen, body.rot, pts);
            finishContactCar(cars, i, body, pts, cnt);
        }
        return;
    }
    // Each thread's two clip polygons in shared memory, an odd number of words
    // apart, so the lanes of a warp touch distinct banks at any one vertex.
    constexpr int CLIP_WORDS = 2 * MAX_PAIR_CONTACTS * 3 + 1;
    __shared__ float clipS[SOLVE_BLOCK * CLIP_WORDS];
    V3* bufA = reinterpret_cast<V3*>(clipS + threadIdx.x * CLIP_WORDS);
    V3* bufB = bufA + MAX_PAIR_CONTACTS;
    const int HW = arena.hitWords;
    const int lane = threadIdx.x & 31;
    const int warpsPer = SOLVE_BLOCK / 32;
    const int count = x.heavyCount[1];
    const int* list = x.heavyList + stride;
    for (int j = ((int)blockIdx.x - planeBlocks) * warpsPer + (threadIdx.x >> 5); j < count;
         j += ((int)gridDim.x - planeBlocks) * warpsPer)
    {
        const int i = list[j];
        Body body = loadHeavyBody(cars, x, stride, i);
        const V3 cen = body.cen;
        const Q4 rot = body.rot;
        const int cellFirst = x.first[i];
        MPoint pts[MAX_CAR_MANIFOLD_POINTS];
        int cnt = planeManifold(cen, rot, pts);
        const int planeCount = cnt;

        // Entry of this lane's hit: the lane-th set bit over the hit words (the
        // first MAX_CAR_TRI_PAIRS hits are used, as in the reference's slots).
        int myEntry = -1;
        {
            int base = 0;
            for (int h = 0; h < HW && myEntry < 0; h++)
            {
                unsigned m = x.hits[h * stride + i];
                const int c = __popc(m);
                if (lane < base + c)
                {
                    for (int r = base; r < lane; r++) m &= m - 1;
                    myEntry = cellFirst + h * 32 + __ffs(m) - 1;
                }
                base += c;
            }
            if (lane >= MAX_CAR_TRI_PAIRS) myEntry = -1;
        }
        Contact best{};
        float bestDist = 3.402823466e+38f;
        bool have = false;
        if (myEntry >= 0)
        {
            const float4 q0 = __ldg(&arena.cellV[3 * myEntry]);
            const float4 q1 = __ldg(&arena.cellV[3 * myEntry + 1]);
            const float4 q2 = __ldg(&arena.cellV[3 * myEntry + 2]);
            const LocalTri lt = localTriangle(cen, rot, V3{ q0.x, q0.y, q0.z }, V3{ q1.x, q1.y, q1.z },
                                              V3{ q2.x, q2.y, q2.z });
            const Sat sat = carTriSat(lt);
            pairContacts(lt, sat, bufA, bufB, [&](const Contact& c) {
                if (nearManifoldPoint(pts, planeCount, c.carPos)) return;
                const float d = -c.depth;
                if (d < bestDist)
                {
                    bestDist = d;
                    best = c;
                    have = true;
                }
            });
        }
        // Deepest over the hits, the earliest hit on ties.
        float key = have ? bestDist : 3.402823466e+38f;
        int owner = have ? lane : 32;
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1)
        {
            const float ok = __shfl_xor_sync(FULL, key, off);
            const int oo = __shfl_xor_sync(FULL, owner, off);
            if (ok < key || (ok == key && oo < owner))
            {
                key = ok;
                owner = oo;
            }
        }
        if (owner < 32)
        {
            Contact c;
            c.carPos = V3{ __shfl_sync(FULL, best.carPos.x, owner), __shfl_sync(FULL, best.carPos.y, owner),
                           __shfl_sync(FULL, best.carPos.z, owner) };
            c.arenaPos = V3{ __shfl_sync(FULL, best.arenaPos.x, owner), __shfl_sync(FULL, best.arenaPos.y, owner),
                             __shfl_sync(FULL, best.arenaPos.z, owner) };
            c.normal = V3{ __shfl_sync(FULL, best.normal.x, owner), __shfl_sync(FULL, best.normal.y, owner),
                           __shfl_sync(FULL, best.normal.z, owner) };
            c.depth = __shfl_sync(FULL, best.depth, owner);
            const int e = __shfl_sync(FULL, myEntry, owner);
            const float4 q0 = __ldg(&arena.cellV[3 * e]);
            const float4 q1 = __ldg(&arena.cellV[3 * e + 1]);
            const float4 q2 = __ldg(&arena.cellV[3 * e + 2]);
            const int tri = __ldg(&arena.cellTris[e]);
            adjustInternalEdge(localTriangle(cen, rot, V3{ q0.x, q0.y, q0.z }, V3{ q1.x, q1.y, q1.z },
                                             V3{ q2.x, q2.y, q2.z }),
                               triAngles(arena, tri), c);
            addManifoldPoint(pts, cnt, contactToManifold(c, cen, rot));
        }
        if (lane == 0) finishContactCar(cars, i, body, pts, cnt);
        __syncwarp();
    }
}

__global__ void __launch_bounds__(CC_BLOCK) carCarKernel(TickParams p, StageScratch x, int t)
{
    __shared__ int activeS[CC_BLOCK];
    __shared__ int nActive;
    const int tid = threadIdx.x;
    const int s = blockIdx.x * CC_BLOCK + tid;
    const CarSoa cars{ p.car, (int)p.carStride };
    const int nCars = p.nCars;
    const int tick = tickBase(p) + t + 1;
    const bool lastTick = t == p.nTicks - 1;
    const int nPairs = nCars * (nCars - 1) / 2;
    if (tid == 0) nActive = 0;
    __syncthreads();
    if (s < p.nSim)
    {
        const int sb = s * nCars;
        bool gate = false;
        for (int a = 0; a < nCars - 1 && !gate; a++)
            for (int b = a + 1; b < nCars && !gate; b++) gate = carCarGate(cars, sb + b, sb + a);
        if (gate) activeS[atomicAdd(&nActive, 1)] = s;
        else if (lastTick && p.diagSim)
            for (int q = 0; q < nPairs && q < DIAG_SIM_WORDS; q++) p.diagSim[q * p.simStride + s] = 0;
    }
    __syncthreads();
    if (tid == 0 && nActive) atomicAdd(x.ccCount, nActive);
    // The active sims are packed into the first lanes; those lanes of each warp
    // step their sims together.
    const unsigned lanes = __ballot_sync(FULL, tid < nActive);
    if (tid >= nActive) return;
    const int sIdx = activeS[tid];
    const int sb = sIdx * nCars;
    // Each thread's clip polygons (16 vertices) in shared memory, an odd number of
    // words apart: the lanes of a warp touch distinct banks at any one vertex.
    constexpr int CC_CLIP_WORDS = 16 * 3 + 1;
    __shared__ float ccClipS[CC_BLOCK * CC_CLIP_WORDS];
    SimCars<CarSoa> sc{ cars, sb, nCars, p.nBlue, (int)(p.globalCarBase + sb), tick, p.seed,
                        reinterpret_cast<V3*>(ccClipS + tid * CC_CLIP_WORDS) };
    int kept[DIAG_SIM_WORDS];
    const bool diag = lastTick && p.diagSim;
    solveCarCarSim(sc, kept, diag ? DIAG_SIM_WORDS : 0, lanes);
    if (diag)
        for (int q = 0; q < nPairs && q < DIAG_SIM_WORDS; q++) p.diagSim[q * p.simStride + sIdx] = kept[q];
}

// Ball stage prelude, one thread per sim: hand-over values for every sim and the
// list of moving balls (the only ones with arena work).  It reads only the ball,
// which no car stage of the tick writes before the finish kernel.
__global__ void __launch_bounds__(256) ballPrepKernel(TickParams p, StageScratch x)
{
    const int s = blockIdx.x * 256 + threadIdx.x;
    if (s >= p.nSim) return;
    const CarSoa sims{ p.sim, (int)p.simStride };
    const BallPre bp = ballPre(sims, s);
    const V3 out[5] = { bp.exportedPos, bp.posBT, bp.preSolveBT, v3zero(), bp.velNoExt };
    storeBallScratch(x.ball, (int)p.simStride, s, out, 0, 5);
    if (!bp.sleeping) x.ballList[atomicAdd(x.ballCount, 1)] = s;
}

__global__ void __launch_bounds__(BALL_WARPS * 32) ballKernel(TickParams p, ArenaDev arena, StageScratch x, int t)
{
    __shared__ int wbufS[BALL_WARPS][WARP_WORDS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const CarSoa cars{ p.car, (int)p.carStride };
    const CarSoa sims{ p.sim, (int)p.simStride };
    const int stride = (int)p.simStride;
    const int count = *x.ballCount;
    for (int j = blockIdx.x * BALL_WARPS + warp; j < count; j += gridDim.x * BALL_WARPS)
    {
        const int s = x.ballList[j];
        BallPre b;
        b.sleeping = false;
        b.exportedPos = loadBallScratch(x.ball, stride, s, 0);
        b.posBT = loadBallScratch(x.ball, stride, s, 1);
        b.preSolveBT = loadBallScratch(x.ball, stride, s, 2);
        b.velNoExt = loadBallScratch(x.ball, stride, s, 4);
        const V3 pushVel = ballArenaSolve(cars, sims, s, p.nCars, tickBase(p) + t + 1, arena, wbufS[warp], lane, b);
        if (lane == 0) storeBallScratch(x.ball, stride, s, &pushVel, 3, 1);
        __syncwarp();
    }
}

// The boost pad whose pickup cylinder holds a car at `pos`, or -1
// (include/Physics/BoostPads.cuh:70-106 test, same arithmetic).  The pads'
// pickup disks are disjoint, so at most one pad holds a car; the cell list
// narrows the pads tested to those that reach the car's cell.
__device__ __forceinline__ int padUnderCar(V3 pos)
{
    const int cx = (int)floorf((pos.x - PAD_GRID_X0) * (1.f / PAD_CELL));
    const int cy = (int)floorf((pos.y - PAD_GRID_Y0) * (1.f / PAD_CELL));
    if (cx < 0 || cx >= PAD_GRID_NX || cy < 0 || cy >= PAD_GRID_NY) return -1;
    const unsigned word = c_tables.padCell[cy * PAD_GRID_NX + cx];
    const int n = word == 0xfffffffeu ? NUM_BOOST_PADS : 4;
    for (int j = 0; j < n; j++)
    {
        const int pad = n == 4 ? (int)((word >> (8 * j)) & 0xffu) : j;
        if (pad == 0xff) break;
        const float radius = c_tables.padBig[pad] ? BIG_PAD_RADIUS : SMALL_PAD_RADIUS;
        const float dx = pos.x - c_tables.padX[pad];
        const float dy = pos.y - c_tables.padY[pad];
        const float distSq = dx * dx + dy * dy;
        if (distSq < radius * radius && fabsf(pos.z - c_tables.padZ[pad]) < BOOST_PAD_HEIGHT) return pad;
    }
    return -1;
}

// Finish of a CTA of `simsPerBlock` whole sims, in four phases:
//   1. a thread per car: the car's ball gate;
//   2. a thread per sim: ball vs its gated cars (car order), ball integration, goal;
//   3. a thread per car: integration and finish (demo timer, respawn, outputs),
//      then the pad under the car; a thread per sim: the ball's finish;
//   4. a thread per (pad, sim): cooldown, and the last car (in car order) on the
//      pad takes it (include/Physics/BoostPads.cuh:89-97).  A car is on at most
//      one pad, so the pads of a sim are independent.
__global__ void __launch_bounds__(FIN_THREADS, 3) finishKernel(TickParams p, StageScratch x, int t,
                                                                int simsPerBlock)
{
    __shared__ unsigned char gateS[FIN_THREADS];
    __shared__ signed char padS[FIN_THREADS];
    const int tid = threadIdx.x;
    const int nCars = p.nCars;
    const int s0 = blockIdx.x * simsPerBlock;
    const int simsHere = min(simsPerBlock, p.nSim - s0);
    const int carsHere = simsHere * nCars;
    const CarSoa cars{ p.car, (int)p.carStride };
    const CarSoa sims{ p.sim, (int)p.simStride };
    const int tick = tickBase(p) + t + 1;
    const bool lastTick = t == p.nTicks - 1;

    if (blockIdx.x == 0 && tid == 0)
    {
        // The per-tick work lists are consumed; keep their sizes and empty them
        // for the next tick.
        for (int c = 0; c < HEAVY_CLASSES; c++) x.stats[c] = x.heavyCount[c];
        x.stats[HEAVY_CLASSES] = *x.ballCount;
        x.stats[HEAVY_CLASSES + 1] = *x.ccCount;
        *x.ballCount = 0;
        *x.ccCount = 0;
        for (int c = 0; c < HEAVY_CLASSES; c++) x.heavyCount[c] = 0;
    }
    if (tid < carsHere)
    {
        const int i = s0 * nCars + tid;
        const int s = s0 + tid / nCars;
        const V3 exportedPos{ x.ball[0 * p.simStride + s], x.ball[1 * p.simStride + s], x.ball[2 * p.simStride + s] };
        gateS[tid] = !cars.n(C_DEMOED, i) && ballCarGate(exportedPos, cars.v(C_CEN, i));
    }
    __syncthreads();
    if (tid < simsHere)
        ballFinishStage(cars, sims, s0 + tid, nCars, tick, x.ball, (int)p.simStride, gateS + tid * nCars);
    __syncthreads();
    if (tid < carsHere)
    {
        const int i = s0 * nCars + tid;
        if (!cars.n(C_DEMOED, i))
        {
            V3 pos = cars.v(C_POS, i), cen, vel = cars.v(C_VEL, i), ang = cars.v(C_ANG, i);
            Q4 rot = cars.q(C_ROT, i);
            integratePose(pos, cen, rot, vel, ang);
            clampCarVelocity(vel, ang);
            cars.setv(C_POS, i, pos);
            cars.setv(C_VEL, i, vel);
            cars.setv(C_ANG, i, ang);
            cars.setv(C_CEN, i, cen);
            cars.setq(C_ROT, i, rot);
        }
        const Controls ctl = decodeAction(p.actions, p.actionKind, i);
        const bool respawned = finishCar(cars, i, ctl.steer, (i % nCars) >= p.nBlue, c_tables);
        padS[tid] = cars.n(C_DEMOED, i) ? -1 : (signed char)padUnderCar(cars.v(C_POS, i));
        if (lastTick)
        {
            const unsigned bits = x.wheelBits[i];
            int* outI = reinterpret_cast<int*>(p.carOut);
            #pragma unroll
            for (int w = 0; w < NUM_WHEELS; w++)
                outI[(long long)(O_WHEEL_CON + w) * p.carStride + i] = respawned ? 0 : (int)((bits >> w) & 1u);
            p.carOut[(long long)(O_CONTROLS + 0) * p.carStride + i] = ctl.throttle;
            p.carOut[(long long)(O_CONTROLS + 1) * p.carStride + i] = ctl.steer;
            p.carOut[(long long)(O_CONTROLS + 2) * p.carStride + i] = ctl.yaw;
            p.carOut[(long long)(O_CONTROLS + 3) * p.carStride + i] = ctl.pitch;
            p.carOut[(long long)(O_CONTROLS + 4) * p.carStride + i] = ctl.roll;
            outI[(long long)(O_CONTROLS + 5) * p.carStride + i] = ctl.jump;
            outI[(long long)(O_CONTROLS + 6) * p.carStride + i] = ctl.boost;
            outI[(long long)(O_CONTROLS + 7) * p.carStride + i] = ctl.slide;
        }
    }
    if (tid < simsHere) finishBall(sims, s0 + tid);
    __syncthreads();
    for (int it = tid; it < simsHere * NUM_BOOST_PADS; it += blockDim.x)
    {
        const int pad = it / simsHere;
        const int ls = it - pad * simsHere;
        const int s = s0 + ls;
        float cd = sims.f(S_PADS + pad, s);
        if (cd > 0.f)
        {
            cd = fmaxf(cd - PHYS_DT, 0.f);
            sims.f(S_PADS + pad, s) = cd;
        }
        if (cd > 0.f) continue;
        int locked = -1;
        for (int k = 0; k < nCars; k++)
            if (padS[ls * nCars + k] == pad) locked = s * nCars + k;
        if (locked < 0) continue;
        const bool big = c_tables.padBig[pad] != 0;
        const float boost = cars.f(C_INT + I_BOOST, locked);
        if (boost >= BOOST_MAX) continue;
        cars.f(C_INT + I_BOOST, locked) = fminf(boost + (big ? BIG_PAD_AMOUNT : SMALL_PAD_AMOUNT), BOOST_MAX);
        sims.f(S_PADS + pad, s) = big ? BIG_PAD_COOLDOWN : SMALL_PAD_COOLDOWN;
    }
}

}  // namespace

int uploadTickTables(const Tables& t)
{
    return (int)cudaMemcpyToSymbol(c_tables, &t, sizeof(Tables));
}

// ---- fixed-size scratch for carlb_ticks_static_scratch --------------------------------------
// A file-scope device array, so that entry point allocates nothing at call time
// (for callers that cannot call cudaMalloc while stepping).  Every GPU that loads
// the library holds it until the process exits.  Host code must not use its name
// as an address (on the host it is only a stand-in): staticScratchAddress looks
// the device address up.  Calls that overlap on the GPU (any env, any stream)
// share it and race.
static __device__ __align__(256) unsigned char g_staticScratch[STATIC_SCRATCH_BYTES];

int stagedSetup();

int staticScratchAddress(void** ptr, size_t* bytes, void** lastUse)
{
    static std::mutex lock;
    static void* cached[64] = {};
    static cudaEvent_t used[64] = {};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return (int)err;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> guard(lock);
    if (!cached[dev])
    {
        // Load every kernel the static-scratch ticks launch, and set the flat
        // stage's shared-memory opt-in, now: with lazy module loading a kernel's
        // first launch would otherwise load its code and may allocate device
        // memory inside a call that promises to allocate nothing.
        const void* kernels[] = { (const void*)ballPrepKernel, (const void*)flatKernel, (const void*)rayKernel,
                                  (const void*)ctlSuspKernel, (const void*)contactKernel, (const void*)carCarKernel,
                                  (const void*)ballKernel, (const void*)finishKernel };
        for (const void* k : kernels)
        {
            cudaFuncAttributes attr;
            err = cudaFuncGetAttributes(&attr, k);
            if (err != cudaSuccess) return (int)err;
        }
        if (const int e = stagedSetup()) return e;
        err = cudaEventCreateWithFlags(&used[dev], cudaEventDisableTiming);
        if (err != cudaSuccess) return (int)err;
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_staticScratch);
        if (err != cudaSuccess) return (int)err;
        if (!p) return (int)cudaErrorInvalidSymbol;
        cached[dev] = p;
    }
    *ptr = cached[dev];
    *bytes = STATIC_SCRATCH_BYTES;
    if (lastUse) *lastUse = used[dev];
    return 0;
}

size_t stageCandSmemBytes(int hitWords)
{
    const int B = CAND_BLOCK;
    size_t words = (size_t)B + B + (B + 1) + 32 + 15 * B + 7 * B + (size_t)hitWords * B;
    size_t bytes = (words * 4 + 7) & ~(size_t)7;
    return bytes + 8 * 4 * (size_t)B + 2 * CAND_MAP_CAP;
}

int stagedSetup()
{
    static std::mutex lock;
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return (int)err;
    std::lock_guard<std::mutex> guard(lock);
    if (dev < 0 || dev >= 64 || !configured[dev])
    {
        err = cudaFuncSetAttribute(flatKernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
        if (err != cudaSuccess) return (int)err;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    return 0;
}

int launchSetTick(int* dst, int value, void* stream)
{
    setTickKernel<<<1, 1, 0, (cudaStream_t)stream>>>(dst, value);
    return (int)cudaGetLastError();
}

int launchTickStaged(const TickParams& p, const ArenaDev& a, const StageScratch& x, void* stream,
                     const StageStreams& aux)
{
    if (p.nTicks <= 0 || p.nSim <= 0) return 0;
    if ((long long)NCW * p.carStride >= (1LL << 31) || (long long)NSW * p.simStride >= (1LL << 31))
        return (int)cudaErrorInvalidValue;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t candSmem = stageCandSmemBytes(a.hitWords);
    if (const int e = stagedSetup()) return e;
    int dev = 0;
    cudaGetDevice(&dev);
    if (candSmem > 128 * 1024) return (int)cudaErrorInvalidValue;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);

    // Sims are independent, so the env's sims are split into `groups` contiguous
    // slices, each stepped on its own stream: while one slice runs a stage that
    // leaves the GPU half idle (the contact solve of a few cars, the ball arena
    // stage), another slice's wide stages fill it.  A slice is the env itself seen
    // through shifted base pointers (every array is word-major with the env's
    // strides), with its own work-list counters.
    const int groups = std::max(1, std::min(aux.groups, STAGE_MAX_GROUPS));
    cudaError_t err = cudaEventRecord((cudaEvent_t)aux.fork, st);
    if (err != cudaSuccess) return (int)err;
    TickParams gp[STAGE_MAX_GROUPS];
    StageScratch gx[STAGE_MAX_GROUPS];
    cudaStream_t gs[STAGE_MAX_GROUPS];
    int nG = 0;
    for (int g = 0; g < groups; g++)
    {
        int s0 = 0, ns = 0;
        stageSlice(p.nSim, groups, g, &s0, &ns);
        if (ns <= 0) break;
        const long long c0 = (long long)s0 * p.nCars;
        TickParams q = p;
        q.car = p.car + c0;
        q.sim = p.sim + s0;
        q.carOut = p.carOut + c0;
        q.diagCar = p.diagCar ? p.diagCar + c0 : nullptr;
        q.diagSim = p.diagSim ? p.diagSim + s0 : nullptr;
        const size_t rowBytes = p.actionKind == ACT_DIRECT ? 32 : 28;
        q.actions = static_cast<const char*>(p.actions) + c0 * rowBytes;
        q.globalCarBase = p.globalCarBase + c0;
        q.nSim = ns;
        StageScratch y = x;
        y.first = x.first + c0;
        y.cnt = x.cnt + c0;
        y.ray = x.ray + c0;
        y.hits = x.hits + c0;
        y.wheelBits = x.wheelBits + c0;
        y.keys = x.keys + c0;
        y.heavyBody = x.heavyBody + c0;
        y.heavyList = x.heavyList + c0;
        y.heavyCount = x.heavyCount + g * HEAVY_CLASSES;
        y.ball = x.ball + s0;
        y.ballList = x.ballList + s0;
        y.ballCount = x.ballCount + g;
        y.ccCount = x.ccCount + g;
        y.stats = x.stats + g * STAGE_WORK;
        gp[nG] = q;
        gx[nG] = y;
        gs[nG] = groups == 1 ? st : (cudaStream_t)aux.streams[g];
        if (gs[nG] != st && (err = cudaStreamWaitEvent(gs[nG], (cudaEvent_t)aux.fork, 0)) != cudaSuccess) return (int)err;
        nG++;
    }
    for (int t = 0; t < p.nTicks; t++)
        for (int g = 0; g < nG; g++)
        {
            const TickParams& q = gp[g];
            const StageScratch& y = gx[g];
            cudaStream_t sq = gs[g];
            const int n = q.nSim * q.nCars;
            // Sims per finish CTA: up to a CTA's threads' worth of cars, but spread over
            // at least one wave (3 CTAs per SM) when the slice is small, so the per-sim
            // and per-(pad, sim) phases of a small env run on many SMs (1v1, 1024 sims:
            // 4 sims per CTA, 256 CTAs, against 128 sims in 8 CTAs).
            const int simsPerFin = std::max(1, std::min(FIN_THREADS / q.nCars,
                                                        std::max(4, (q.nSim + 3 * sms / nG - 1) / (3 * sms / nG))));
            const int ballBlocks = std::max(1, std::min((q.nSim + BALL_WARPS - 1) / BALL_WARPS, sms * 8 / nG));
            const int contactBlocks = std::max(1, std::min((n + SOLVE_BLOCK - 1) / SOLVE_BLOCK, sms * 2 / nG));
            const int meshBlocks = std::max(1, std::min((n + SOLVE_BLOCK - 1) / SOLVE_BLOCK, sms * 4 / nG));
            const bool timed = g == 0 && t == p.nTicks - 1 && aux.stageEvents[0];
            // Events around stage k: stageEvents[2k] (start), [2k + 1] (end), on the
            // stream the stage kernel runs on.
            // Under stream capture the record becomes an event node of the graph
            // (a plain record there is only an ordering edge).
            auto mark = [&](int k, bool end, cudaStream_t on) {
                if (!timed) return;
                cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
                cudaStreamIsCapturing(on, &cs);
                cudaEventRecordWithFlags((cudaEvent_t)aux.stageEvents[2 * k + (end ? 1 : 0)], on,
                                         cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal
                                                                             : cudaEventRecordDefault);
            };
            // The ball's arena stage reads only the ball and the cars' last-hit ticks,
            // which no car stage of this tick writes before the finish kernel, so with
            // a side stream it runs beside the car stages.
            cudaStream_t sb = aux.ballStreams[g] ? (cudaStream_t)aux.ballStreams[g] : sq;
            if (sb != sq)
            {
                if ((err = cudaEventRecord((cudaEvent_t)aux.tickStart[g], sq)) != cudaSuccess) return (int)err;
                if ((err = cudaStreamWaitEvent(sb, (cudaEvent_t)aux.tickStart[g], 0)) != cudaSuccess) return (int)err;
            }
            mark(0, false, sb);
            ballPrepKernel<<<(q.nSim + 255) / 256, 256, 0, sb>>>(q, y);
            mark(0, true, sb);
            mark(6, false, sb);
            ballKernel<<<ballBlocks, BALL_WARPS * 32, 0, sb>>>(q, a, y, t);
            mark(6, true, sb);
            if (sb != sq && (err = cudaEventRecord((cudaEvent_t)aux.ballDone[g], sb)) != cudaSuccess) return (int)err;
            // Phase offset between slices: slice g starts its wide stages (flat, ray
            // finish, suspension) only after the previous slice's wide stages of this
            // tick (slice 0: the last slice's, previous tick), so one slice's
            // latency-bound contact / car-car stages overlap another's wide stages.
            if (nG > 1 && aux.wideDone[0])
            {
                const int prev = g == 0 ? nG - 1 : g - 1;
                if ((g > 0 || t > 0) &&
                    (err = cudaStreamWaitEvent(sq, (cudaEvent_t)aux.wideDone[prev], 0)) != cudaSuccess)
                    return (int)err;
            }
            mark(1, false, sq);
            flatKernel<<<(n + CAND_BLOCK - 1) / CAND_BLOCK, CAND_BLOCK, candSmem, sq>>>(q, a, y, t);
            mark(1, true, sq);
            mark(2, false, sq);
            rayKernel<<<(n + RAY_BLOCK - 1) / RAY_BLOCK, RAY_BLOCK, 0, sq>>>(q, a, y, t);
            mark(2, true, sq);
            // Actions copied in per slice beside the launch: the controls stage is the
            // first reader (the finish after it the only other), so the copy overlaps
            // the first tick's broadphase and ray stages.
            if (t == 0 && aux.actionsReady[g])
            {
                cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
                cudaStreamIsCapturing(sq, &cs);
                if ((err = cudaStreamWaitEvent(sq, (cudaEvent_t)aux.actionsReady[g],
                                               cs == cudaStreamCaptureStatusActive ? cudaEventWaitExternal
                                                                                   : cudaEventWaitDefault)) != cudaSuccess)
                    return (int)err;
            }
            mark(3, false, sq);
            ctlSuspKernel<<<(n + SOLVE_BLOCK - 1) / SOLVE_BLOCK, SOLVE_BLOCK, 0, sq>>>(q, a, y, t);
            mark(3, true, sq);
            if (nG > 1 && aux.wideDone[0] && (err = cudaEventRecord((cudaEvent_t)aux.wideDone[g], sq)) != cudaSuccess)
                return (int)err;
            mark(4, false, sq);
            contactKernel<<<contactBlocks + meshBlocks, SOLVE_BLOCK, 0, sq>>>(q, a, y, t, contactBlocks);
            mark(4, true, sq);
            mark(5, false, sq);
            carCarKernel<<<(q.nSim + CC_BLOCK - 1) / CC_BLOCK, CC_BLOCK, 0, sq>>>(q, y, t);
            mark(5, true, sq);
            if (sb != sq && (err = cudaStreamWaitEvent(sq, (cudaEvent_t)aux.ballDone[g], 0)) != cudaSuccess)
                return (int)err;
            mark(7, false, sq);
            finishKernel<<<(q.nSim + simsPerFin - 1) / simsPerFin, FIN_THREADS, 0, sq>>>(q, y, t, simsPerFin);
            mark(7, true, sq);
        }
    for (int g = 0; g < nG; g++)
    {
        if (gs[g] == st) continue;
        if ((err = cudaEventRecord((cudaEvent_t)aux.join[g], gs[g])) != cudaSuccess) return (int)err;
        if ((err = cudaStreamWaitEvent(st, (cudaEvent_t)aux.join[g], 0)) != cudaSuccess) return (int)err;
    }
    return (int)cudaGetLastError();
}

}  // namespace cb
