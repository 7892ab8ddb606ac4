// Host-side arena build (see arena.hpp).  Compiled with -ffp-contract=off so
// the normals, cell indices and edge angles are bit-identical to the
// reference's host build of the same tables.
#include "arena.hpp"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <unordered_map>

#include "cb_consts.cuh"

namespace cb {

std::string arenaObjPath(const std::string& fallback)
{
    const char* env = std::getenv("CARL_ARENA_OBJ");
    if (env && *env) return env;
    return fallback;
}

std::string arenaMetadataPath()
{
    const char* env = std::getenv("CARL_ARENA_METADATA");
    return env ? std::string(env) : std::string();
}

std::string loadNativeMetadata(const std::string& path, ArenaHost& a)
{
    std::ifstream file(path);
    if (!file.is_open()) return "cannot open CARL arena metadata '" + path + "'";
    const int nTris = a.nTris();
    int count = 0;
    file >> count;
    if (count != nTris) return "CARL arena metadata triangle count mismatch";
    a.nativeMesh.assign(nTris, 0);
    a.nativeOrder.assign(nTris, 0);
    a.nativeFlags.assign(nTris, 0);
    a.nativeAngles.assign((size_t)nTris * 3, 0.f);
    a.nativeVerts.assign((size_t)nTris * 9, 0.f);
    for (int t = 0; t < nTris; t++)
    {
        file >> a.nativeMesh[t] >> a.nativeOrder[t];
        for (int k = 0; k < 3; k++) file >> a.nativeAngles[3 * t + k];
        file >> a.nativeFlags[t];
        for (int k = 0; k < 9; k++) file >> a.nativeVerts[9 * t + k];
    }
    if (!file) return "Invalid CARL arena metadata";
    a.hasNative = true;
    // Ball-cell lists in traversal-key order; equal keys keep ascending triangle
    // order (a stable sort of the ascending lists).
    const size_t nb = a.ballCellStart.size() - 1;
    for (size_t c = 0; c < nb; c++)
        std::stable_sort(a.ballCellTris.begin() + a.ballCellStart[c], a.ballCellTris.begin() + a.ballCellStart[c + 1],
                         [&](int x, int y) { return a.ballKey(x) < a.ballKey(y); });
    return "";
}

namespace {

uint32_t weldBits(float v)
{
    const float canon = v == 0.f ? 0.f : v;  // -0 and +0 weld together
    uint32_t bits;
    std::memcpy(&bits, &canon, 4);
    return bits;
}

I3 cellOf(V3 p)
{
    // ((p - ARENA_MIN) / CELL_SIZE) clamped to [0, GRID - 1], truncated.
    const float gx = fminf(fmaxf((p.x - ARENA_MIN_X) / CELL_X, 0.f), GRID_X - 1.f);
    const float gy = fminf(fmaxf((p.y - ARENA_MIN_Y) / CELL_Y, 0.f), GRID_Y - 1.f);
    const float gz = fminf(fmaxf((p.z - ARENA_MIN_Z) / CELL_Z, 0.f), GRID_Z - 1.f);
    return I3{ (int)gx, (int)gy, (int)gz };
}

V3 vert(const ArenaHost& a, int i) { return V3{ a.verts[3 * i], a.verts[3 * i + 1], a.verts[3 * i + 2] }; }

}  // namespace

std::string buildArena(const std::string& path, ArenaHost& a)
{
    std::ifstream file(path);
    if (!file.is_open()) return "cannot open arena mesh '" + path + "' (set CARL_ARENA_OBJ)";

    std::vector<float> raw;
    std::vector<int32_t> faces;
    std::string line;
    while (std::getline(file, line))
    {
        const char* s = line.c_str();
        while (*s == ' ' || *s == '\t') s++;
        if (s[0] == 'v' && (s[1] == ' ' || s[1] == '\t'))
        {
            char* end = nullptr;
            const float y = std::strtof(s + 1, &end);  // file order is (y, x, z)
            const char* p = end;
            const float x = std::strtof(p, &end);
            if (end == p) return "invalid OBJ vertex: " + line;
            p = end;
            const float z = std::strtof(p, &end);
            if (end == p) return "invalid OBJ vertex: " + line;
            raw.insert(raw.end(), { x, y, z });
        }
        else if (s[0] == 'f' && (s[1] == ' ' || s[1] == '\t'))
        {
            std::istringstream in(s + 1);
            int i0, i1, i2;
            if (!(in >> i0 >> i1 >> i2)) return "invalid OBJ face: " + line;
            faces.insert(faces.end(), { i0 - 1, i1 - 1, i2 - 1 });
        }
    }

    // Exact-bit weld, first occurrence keeps its position.
    const int nRaw = (int)raw.size() / 3;
    std::map<std::array<uint32_t, 3>, int> ids;
    std::vector<int> remap(nRaw);
    a.verts.clear();
    for (int i = 0; i < nRaw; i++)
    {
        const std::array<uint32_t, 3> key = { weldBits(raw[3 * i]), weldBits(raw[3 * i + 1]),
                                              weldBits(raw[3 * i + 2]) };
        const auto [it, inserted] = ids.emplace(key, (int)a.verts.size() / 3);
        if (inserted) a.verts.insert(a.verts.end(), { raw[3 * i], raw[3 * i + 1], raw[3 * i + 2] });
        remap[i] = it->second;
    }
    a.tris.resize(faces.size());
    for (size_t k = 0; k < faces.size(); k++)
    {
        if (faces[k] < 0 || faces[k] >= nRaw) return "OBJ triangle index is out of range";
        a.tris[k] = remap[faces[k]];
    }

    const int nTris = a.nTris();
    a.normals.resize((size_t)nTris * 3);
    a.triFlags.assign(nTris, 0);
    std::vector<V3> lo(nTris), hi(nTris);
    for (int t = 0; t < nTris; t++)
    {
        const V3 v0 = vert(a, a.tris[3 * t]), v1 = vert(a, a.tris[3 * t + 1]), v2 = vert(a, a.tris[3 * t + 2]);
        const V3 c = cross(v1 - v0, v2 - v0);
        const float ls = lensq(c);
        if (ls <= 1e-12f) return "degenerate triangle in arena mesh";
        const V3 n = c * (1.f / sqrtf(ls));
        a.normals[3 * t] = n.x;
        a.normals[3 * t + 1] = n.y;
        a.normals[3 * t + 2] = n.z;
        lo[t] = vmin(vmin(v0, v1), v2);
        hi[t] = vmax(vmax(v0, v1), v2);

        const bool horizontal = v0.z == v1.z && v0.z == v2.z && (v0.z == 0.f || v0.z == 2048.f);
        const bool sideWall = v0.x == v1.x && v0.x == v2.x && fabsf(v0.x) == 4096.f;
        if (horizontal || sideWall) a.triFlags[t] |= TRI_ANALYTIC_PLANE;
    }

    // Uniform grid: each triangle spans [cell(min) - 1, cell(max)] per axis.
    std::vector<std::vector<int32_t>> cells(NUM_CELLS);
    for (int t = 0; t < nTris; t++)
    {
        const I3 c0 = cellOf(lo[t]);
        const I3 c1 = cellOf(hi[t]);
        const int x0 = c0.x - 1 > 0 ? c0.x - 1 : 0;
        const int y0 = c0.y - 1 > 0 ? c0.y - 1 : 0;
        const int z0 = c0.z - 1 > 0 ? c0.z - 1 : 0;
        for (int x = x0; x <= c1.x; x++)
            for (int y = y0; y <= c1.y; y++)
                for (int z = z0; z <= c1.z; z++)
                    cells[x + y * GRID_W + z * GRID_W * GRID_H].push_back(t);
    }
    a.cellStart.assign(NUM_CELLS + 1, 0);
    a.maxCellTris = 0;
    for (int c = 0; c < NUM_CELLS; c++)
    {
        a.cellStart[c + 1] = a.cellStart[c] + (int)cells[c].size();
        if ((int)cells[c].size() > a.maxCellTris) a.maxCellTris = (int)cells[c].size();
    }
    a.cellTris.resize(a.cellStart[NUM_CELLS]);
    for (int c = 0; c < NUM_CELLS; c++)
        std::copy(cells[c].begin(), cells[c].end(), a.cellTris.begin() + a.cellStart[c]);

    // Ball grid (see ArenaHost): reach = contact radius + 2 uu of margin, which
    // covers float rounding in the device's cell lookup.
    {
        const double reach = (double)BALL_COLLISION_RADIUS + (double)BALL_ARENA_CONTACT_BREAK + 2.0;
        const double cell = a.ballCell;
        double o[3] = { 1e30, 1e30, 1e30 }, e[3] = { -1e30, -1e30, -1e30 };
        for (int t = 0; t < nTris; t++)
        {
            const double l[3] = { lo[t].x, lo[t].y, lo[t].z }, h[3] = { hi[t].x, hi[t].y, hi[t].z };
            for (int k = 0; k < 3; k++)
            {
                o[k] = std::min(o[k], l[k] - reach);
                e[k] = std::max(e[k], h[k] + reach);
            }
        }
        for (int k = 0; k < 3; k++)
        {
            a.ballOrigin[k] = (float)std::floor(o[k]);
            a.ballDims[k] = (int)std::ceil((e[k] - a.ballOrigin[k]) / cell) + 1;
        }
        const size_t nb = (size_t)a.ballDims[0] * a.ballDims[1] * a.ballDims[2];
        std::vector<std::vector<int32_t>> bcells(nb);
        for (int t = 0; t < nTris; t++)
        {
            const double l[3] = { lo[t].x, lo[t].y, lo[t].z }, h[3] = { hi[t].x, hi[t].y, hi[t].z };
            int c0[3], c1[3];
            for (int k = 0; k < 3; k++)
            {
                c0[k] = std::max(0, (int)std::floor((l[k] - reach - a.ballOrigin[k]) / cell));
                c1[k] = std::min(a.ballDims[k] - 1, (int)std::floor((h[k] + reach - a.ballOrigin[k]) / cell));
            }
            for (int z = c0[2]; z <= c1[2]; z++)
                for (int y = c0[1]; y <= c1[1]; y++)
                    for (int x = c0[0]; x <= c1[0]; x++)
                        bcells[x + (size_t)a.ballDims[0] * (y + (size_t)a.ballDims[1] * z)].push_back(t);
        }
        a.ballCellStart.assign(nb + 1, 0);
        for (size_t c = 0; c < nb; c++) a.ballCellStart[c + 1] = a.ballCellStart[c] + (int)bcells[c].size();
        a.ballCellTris.resize(a.ballCellStart[nb]);
        for (size_t c = 0; c < nb; c++)
            std::copy(bcells[c].begin(), bcells[c].end(), a.ballCellTris.begin() + a.ballCellStart[c]);
    }

    // Signed dihedral angle across every shared edge.
    a.edgeAngles.assign((size_t)nTris * 3, BOUNDARY_EDGE_ANGLE);
    struct EdgeRef { int tri, slot, start, end; bool paired; };
    std::map<std::pair<int, int>, EdgeRef> edges;
    for (int t = 0; t < nTris; t++)
    {
        for (int slot = 0; slot < 3; slot++)
        {
            const int s0 = a.tris[3 * t + slot];
            const int s1 = a.tris[3 * t + (slot + 1) % 3];
            const std::pair<int, int> key = s0 < s1 ? std::make_pair(s0, s1) : std::make_pair(s1, s0);
            auto [it, inserted] = edges.try_emplace(key, EdgeRef{ t, slot, s0, s1, false });
            if (inserted) continue;
            EdgeRef& first = it->second;
            if (first.paired) return "non-manifold edge in arena mesh";
            first.paired = true;
            if (first.start != s1 || first.end != s0) return "inconsistent triangle winding in arena mesh";

            const V3 ev = vert(a, first.end) - vert(a, first.start);
            const float el = lensq(ev);
            if (el <= 1e-12f) return "degenerate edge in arena mesh";
            const V3 edge = ev * (1.f / sqrtf(el));
            const V3 na = { a.normals[3 * first.tri], a.normals[3 * first.tri + 1], a.normals[3 * first.tri + 2] };
            const V3 nb = { a.normals[3 * t], a.normals[3 * t + 1], a.normals[3 * t + 2] };
            const V3 nc = cross(na, nb);
            float nd = dot(na, nb);
            nd = nd < -1.f ? -1.f : (nd > 1.f ? 1.f : nd);
            float angle = 0.f;
            if (lensq(nc) <= 1e-4f)
            {
                if (nd < 0.f) return "opposing triangle normals in arena mesh";
            }
            else
            {
                angle = atan2f(dot(edge, nc), nd);
            }
            a.edgeAngles[3 * first.tri + first.slot] = angle;
            a.edgeAngles[3 * t + slot] = angle;
        }
    }
    return "";
}

}  // namespace cb
