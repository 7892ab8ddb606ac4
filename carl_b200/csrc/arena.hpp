// Host-side arena build: collision mesh -> device tables.
//
// Produces the same tables as the reference's ArenaMesh constructor
// (jwmccarthy/CARL src/ArenaMesh.cu:15-125 with include/Arena/ObjLoader.cuh:91-126,
// TriMesh.cuh:21-66, BroadPhaseGrid.cuh:12-78, EdgeInfo.cuh:61-125): OBJ vertices
// read as (y, x, z), exact-bit vertex welding, unit face normals, a 48x48x10
// uniform grid whose cells list every triangle whose (one-cell-dilated) AABB
// overlaps them in ascending triangle order, and the signed dihedral angle of
// every shared edge (2*pi on boundary edges).  Only the default arena path is
// built (no native-metadata override), so the ball's per-cell triangle order is
// the car's order.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace cb {

// Triangle flag bits (ArenaHost::triFlags).
enum : int32_t {
    TRI_ANALYTIC_PLANE = 1,  // floor, ceiling or flat side wall: skipped by car-vs-mesh SAT
};

struct ArenaHost
{
    std::vector<float> verts;       // [nVerts][3]
    std::vector<int32_t> tris;      // [nTris][3] welded vertex ids
    std::vector<float> normals;     // [nTris][3]
    std::vector<float> edgeAngles;  // [nTris][3], edge i = (v_i, v_(i+1)%3)
    std::vector<int32_t> triFlags;  // [nTris]
    std::vector<int32_t> cellStart; // [NUM_CELLS + 1]
    std::vector<int32_t> cellTris;  // [cellStart[NUM_CELLS]]
    int32_t maxCellTris = 0;

    // Ball grid: cubic cells of ballCell uu from ballOrigin; a cell lists, in
    // ascending order, every triangle whose bounding box grown by the ball's
    // contact reach (plus a margin) overlaps it, so one cell holds every triangle
    // a ball centred in it can touch.  A ball outside the grid touches nothing.
    float ballOrigin[3] = { 0.f, 0.f, 0.f };
    float ballCell = 128.f;
    int32_t ballDims[3] = { 0, 0, 0 };
    std::vector<int32_t> ballCellStart;  // [ballDims product + 1]
    std::vector<int32_t> ballCellTris;   // [ballCellStart.back()]

    // Native mesh metadata ($CARL_ARENA_METADATA, src/ArenaMesh.cu:69-99): per
    // triangle its native mesh (negative: no ball contact) and traversal order
    // within it, its edge angles and edge flags in the native mesh, and its
    // vertices in Bullet units.  With it the ball's arena contacts take the
    // native branch, and every ball-cell list is ordered by the traversal key
    // mesh * 10000 + order (the order the reference merges its cell lists in).
    bool hasNative = false;
    std::vector<int32_t> nativeMesh, nativeOrder, nativeFlags;  // [nTris]
    std::vector<float> nativeAngles;                            // [nTris][3]
    std::vector<float> nativeVerts;                             // [nTris][3 vertices][3]

    int nVerts() const { return (int)verts.size() / 3; }
    int nTris() const { return (int)tris.size() / 3; }
    // Traversal key of a triangle for the ball (triangle index without metadata).
    int32_t ballKey(int t) const { return hasNative ? nativeMesh[t] * 10000 + nativeOrder[t] : t; }
};

// Path of the native metadata file: $CARL_ARENA_METADATA, or empty.
std::string arenaMetadataPath();

// Reads the native metadata file (format of src/ArenaMesh.cu:69-99: the triangle
// count, then per triangle `mesh order a0 a1 a2 flags` and its three vertices)
// into `a` and reorders the ball-cell lists by traversal key.  Returns an empty
// string on success, else the error (the reference's messages).
std::string loadNativeMetadata(const std::string& path, ArenaHost& a);

// Path of the arena mesh: $CARL_ARENA_OBJ if set, else `fallback`.
std::string arenaObjPath(const std::string& fallback);

// Builds the tables; returns an empty string on success, else the error.
std::string buildArena(const std::string& objPath, ArenaHost& out);

}  // namespace cb
