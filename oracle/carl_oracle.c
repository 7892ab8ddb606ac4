/*
 * carl_oracle.c - plain-C restatement of the reference's integer / index
 * paths (see carl_oracle.h).  Float steps that feed an index (the swept car
 * box of the broadphase) keep the reference's fp32 operation order; the file
 * is compiled with -ffp-contract=off.  TEST INFRASTRUCTURE: only tests use it.
 */
#include "carl_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---- arena (include/Arena/ObjLoader.cuh:56-126, TriMesh.cuh:45-66,
 *      BroadPhaseGrid.cuh:9-78, src/ArenaMesh.cu:15-42) ---------------------- */

#define GRID_X 48
#define GRID_Y 48
#define GRID_Z 10

static const float AMIN[3] = { -4108.f, -6000.f, -14.f };
static const float AMAX[3] = { 4108.f, 6000.f, 2076.f };
static const float GDIM[3] = { 48.f, 48.f, 10.f };

/* aabbToCell3D: ((p - ARENA_MIN) / CELL_SIZE) clamped to [0, dims-1], truncated. */
static void cell_of(const float p[3], int c[3])
{
    for (int k = 0; k < 3; k++)
    {
        const float cell = (AMAX[k] - AMIN[k]) / GDIM[k];
        float g = (p[k] - AMIN[k]) / cell;
        g = fmaxf(g, 0.f);
        g = fminf(g, GDIM[k] - 1.f);
        c[k] = (int)g;
    }
}

static int flat(int x, int y, int z) { return x + y * GRID_X + z * GRID_X * GRID_Y; }

static uint32_t canon_bits(float v)
{
    const float c = v == 0.f ? 0.f : v;
    uint32_t b;
    memcpy(&b, &c, 4);
    return b;
}

typedef struct { uint32_t k[3]; int id; int used; } slot_t;

int co_arena_build(const char* path, co_arena* a)
{
    memset(a, 0, sizeof(*a));
    FILE* f = fopen(path, "r");
    if (!f) return 1;
    int cap_v = 1024, cap_f = 1024, nv = 0, nf = 0;
    float* raw = malloc(sizeof(float) * 3 * cap_v);
    int32_t* faces = malloc(sizeof(int32_t) * 3 * cap_f);
    char line[512];
    while (fgets(line, sizeof line, f))
    {
        const char* s = line;
        while (*s == ' ' || *s == '\t') s++;
        if (s[0] == 'v' && (s[1] == ' ' || s[1] == '\t'))
        {
            char* e;
            const float y = strtof(s + 1, &e);  /* file order (y, x, z) */
            const float x = strtof(e, &e);
            const float z = strtof(e, &e);
            if (nv == cap_v) raw = realloc(raw, sizeof(float) * 3 * (cap_v *= 2));
            raw[3 * nv] = x; raw[3 * nv + 1] = y; raw[3 * nv + 2] = z;
            nv++;
        }
        else if (s[0] == 'f' && (s[1] == ' ' || s[1] == '\t'))
        {
            char* e;
            const long i0 = strtol(s + 1, &e, 10), i1 = strtol(e, &e, 10), i2 = strtol(e, &e, 10);
            if (nf == cap_f) faces = realloc(faces, sizeof(int32_t) * 3 * (cap_f *= 2));
            faces[3 * nf] = (int32_t)i0 - 1; faces[3 * nf + 1] = (int32_t)i1 - 1; faces[3 * nf + 2] = (int32_t)i2 - 1;
            nf++;
        }
    }
    fclose(f);

    /* Exact-bit weld: ids in order of first occurrence (open addressing). */
    int cap = 1;
    while (cap < 4 * nv) cap <<= 1;
    slot_t* table = calloc(cap, sizeof(slot_t));
    int* remap = malloc(sizeof(int) * nv);
    a->verts = malloc(sizeof(float) * 3 * nv);
    for (int i = 0; i < nv; i++)
    {
        uint32_t k[3] = { canon_bits(raw[3 * i]), canon_bits(raw[3 * i + 1]), canon_bits(raw[3 * i + 2]) };
        uint32_t h = (k[0] * 73856093u) ^ (k[1] * 19349663u) ^ (k[2] * 83492791u);
        int pos = (int)(h & (cap - 1));
        while (table[pos].used && memcmp(table[pos].k, k, sizeof k) != 0) pos = (pos + 1) & (cap - 1);
        if (!table[pos].used)
        {
            table[pos].used = 1;
            memcpy(table[pos].k, k, sizeof k);
            table[pos].id = a->n_verts;
            memcpy(&a->verts[3 * a->n_verts], &raw[3 * i], sizeof(float) * 3);
            a->n_verts++;
        }
        remap[i] = table[pos].id;
    }
    a->n_tris = nf;
    a->tris = malloc(sizeof(int32_t) * 3 * nf);
    for (int i = 0; i < 3 * nf; i++)
    {
        if (faces[i] < 0 || faces[i] >= nv) return 2;
        a->tris[i] = remap[faces[i]];
    }

    /* Grid: count, prefix, fill (triangle order within each cell). */
    a->n_cells = GRID_X * GRID_Y * GRID_Z;
    int32_t* lo = malloc(sizeof(int32_t) * 3 * nf);
    int32_t* hi = malloc(sizeof(int32_t) * 3 * nf);
    a->prefix = calloc(a->n_cells + 1, sizeof(int32_t));
    for (int t = 0; t < nf; t++)
    {
        float mn[3], mx[3];
        for (int k = 0; k < 3; k++)
        {
            const float v0 = a->verts[3 * a->tris[3 * t] + k];
            const float v1 = a->verts[3 * a->tris[3 * t + 1] + k];
            const float v2 = a->verts[3 * a->tris[3 * t + 2] + k];
            mn[k] = fminf(fminf(v0, v1), v2);
            mx[k] = fmaxf(fmaxf(v0, v1), v2);
        }
        int c0[3], c1[3];
        cell_of(mn, c0);
        cell_of(mx, c1);
        for (int k = 0; k < 3; k++)
        {
            lo[3 * t + k] = c0[k] - 1 > 0 ? c0[k] - 1 : 0;
            hi[3 * t + k] = c1[k];
        }
        for (int x = lo[3 * t]; x <= hi[3 * t]; x++)
            for (int y = lo[3 * t + 1]; y <= hi[3 * t + 1]; y++)
                for (int z = lo[3 * t + 2]; z <= hi[3 * t + 2]; z++) a->prefix[flat(x, y, z) + 1]++;
    }
    for (int c = 0; c < a->n_cells; c++) a->prefix[c + 1] += a->prefix[c];
    a->n_refs = a->prefix[a->n_cells];
    a->tri_idx = malloc(sizeof(int32_t) * (a->n_refs > 0 ? a->n_refs : 1));
    int32_t* fill = calloc(a->n_cells, sizeof(int32_t));
    for (int t = 0; t < nf; t++)
        for (int x = lo[3 * t]; x <= hi[3 * t]; x++)
            for (int y = lo[3 * t + 1]; y <= hi[3 * t + 1]; y++)
                for (int z = lo[3 * t + 2]; z <= hi[3 * t + 2]; z++)
                {
                    const int c = flat(x, y, z);
                    a->tri_idx[a->prefix[c] + fill[c]++] = t;
                }
    free(fill); free(lo); free(hi); free(table); free(remap); free(raw); free(faces);
    return 0;
}

void co_arena_free(co_arena* a)
{
    free(a->verts); free(a->tris); free(a->prefix); free(a->tri_idx);
    memset(a, 0, sizeof(*a));
}

/* ---- broadphase (include/Physics/CarArena/BroadPhase.cuh:10-28,
 *      include/Physics/Integration.cuh:6-69, include/AABB.cuh:11-34,
 *      include/Cuda/Math.cuh:228-331) ---------------------------------------- */

static void cross3(const float a[3], const float b[3], float o[3])
{
    o[0] = a[1] * b[2] - a[2] * b[1];
    o[1] = a[2] * b[0] - a[0] * b[2];
    o[2] = a[0] * b[1] - a[1] * b[0];
}

/* Quaternion rotation v + t*w + q x t, t = (q x v) * (2 / |q|^2). */
static void qrot(const float q[4], const float v[3], float o[3])
{
    const float ls = (q[0] * q[0] + q[2] * q[2]) + (q[1] * q[1] + q[3] * q[3]);
    const float s = 2.f / ls;
    float c[3], t[3], c2[3];
    cross3(q, v, c);
    for (int k = 0; k < 3; k++) t[k] = c[k] * s;
    cross3(q, t, c2);
    for (int k = 0; k < 3; k++) o[k] = (v[k] + t[k] * q[3]) + c2[k];
}

static void qscale(float q[4], float s)
{
    for (int k = 0; k < 4; k++) q[k] = q[k] * s;
}

static void integrate_rot(const float rot[4], const float ang[3], float out[4])
{
    const float dt = 1.f / 120;
    const float maxMotion = (3.1415926535897932384626433832795029f / 4);
    const float sq = (ang[0] * ang[0] + ang[1] * ang[1]) + ang[2] * ang[2];
    float speed = sq > 1e-8f ? sqrtf(sq) : 0.f;
    if (speed * dt > maxMotion) speed = maxMotion / dt;
    float axis[3];
    if (speed < 0.001f)
    {
        const float scale = 0.5f * dt - dt * dt * dt * 0.020833333333f * speed * speed;
        for (int k = 0; k < 3; k++) axis[k] = ang[k] * scale;
    }
    else
    {
        const float s = sinf(0.5f * speed * dt) / speed;
        for (int k = 0; k < 3; k++) axis[k] = ang[k] * s;
    }
    const float d[4] = { axis[0], axis[1], axis[2], cosf(0.5f * speed * dt) };

    /* Basis quaternion from the rotated axes (Quat::fromAxes). */
    const float ex[3] = { 1.f, 0.f, 0.f }, ey[3] = { 0.f, 1.f, 0.f }, ez[3] = { 0.f, 0.f, 1.f };
    float f[3], r[3], u[3];
    qrot(rot, ex, f);
    qrot(rot, ey, r);
    qrot(rot, ez, u);
    const float trace = f[0] + r[1] + u[2];
    const float t[3] = { f[0] * 2.f + (1.f - trace), r[1] * 2.f + (1.f - trace), u[2] * 2.f + (1.f - trace) };
    const float sum[3] = { r[2] + u[1], u[0] + f[2], f[1] + r[0] };
    const float diff[3] = { r[2] - u[1], u[0] - f[2], f[1] - r[0] };
    float b[4];
    if (trace > 0.f)
    {
        const float tw = 1.f + trace;
        b[0] = diff[0]; b[1] = diff[1]; b[2] = diff[2]; b[3] = tw;
        qscale(b, .5f / sqrtf(tw));
    }
    else
    {
        const int am = t[1] > t[0] ? (t[1] > t[2] ? 1 : 2) : (t[0] > t[2] ? 0 : 2);
        if (am == 0) { b[0] = t[0]; b[1] = sum[2]; b[2] = sum[1]; b[3] = diff[0]; qscale(b, .5f / sqrtf(t[0])); }
        else if (am == 1) { b[0] = sum[2]; b[1] = t[1]; b[2] = sum[0]; b[3] = diff[1]; qscale(b, .5f / sqrtf(t[1])); }
        else { b[0] = sum[1]; b[1] = sum[0]; b[2] = t[2]; b[3] = diff[2]; qscale(b, .5f / sqrtf(t[2])); }
    }
    /* delta * basis, then normalise. */
    float p[4];
    p[0] = (d[3] * b[0] - d[2] * b[1]) + (d[0] * b[3] + d[1] * b[2]);
    p[1] = (d[3] * b[1] - d[0] * b[2]) + (d[1] * b[3] + d[2] * b[0]);
    p[2] = (d[3] * b[2] - d[1] * b[0]) + (d[2] * b[3] + d[0] * b[1]);
    p[3] = (d[3] * b[3] - d[2] * b[2]) - (d[0] * b[0] + d[1] * b[1]);
    const float pl = (p[0] * p[0] + p[2] * p[2]) + (p[1] * p[1] + p[3] * p[3]);
    qscale(p, 1.f / sqrtf(pl));
    memcpy(out, p, sizeof p);
}

static void box_min(const float cen[3], const float rot[4], float o[3])
{
    static const float H[3] = { 60.186455f, 43.282655f, 19.262505f };
    const float ex[3] = { 1.f, 0.f, 0.f }, ey[3] = { 0.f, 1.f, 0.f }, ez[3] = { 0.f, 0.f, 1.f };
    float rx[3], ry[3], rz[3];
    qrot(rot, ex, rx);
    qrot(rot, ey, ry);
    qrot(rot, ez, rz);
    for (int k = 0; k < 3; k++)
    {
        const float half = (fabsf(rx[k]) * H[0] + fabsf(ry[k]) * H[1]) + fabsf(rz[k]) * H[2];
        o[k] = cen[k] - half;
    }
}

int32_t co_broadphase_cell(const float pos[3], const float vel[3], const float ang[3],
                           const float cen[3], const float rot[4])
{
    static const float OFF[3] = { 13.87566f, 0.f, 20.755f };
    const float dt = 1.f / 120;
    float ppos[3], prot[4], off[3], pcen[3];
    for (int k = 0; k < 3; k++) ppos[k] = pos[k] + vel[k] * dt;
    integrate_rot(rot, ang, prot);
    qrot(prot, OFF, off);
    for (int k = 0; k < 3; k++) pcen[k] = ppos[k] + off[k];
    float m0[3], m1[3], sw[3];
    box_min(cen, rot, m0);
    box_min(pcen, prot, m1);
    for (int k = 0; k < 3; k++) sw[k] = fminf(m0[k], m1[k]);
    int c[3];
    cell_of(sw, c);
    return flat(c[0], c[1], c[2]);
}

/* ---- kickoff (include/Cuda/Random.cuh:7-17, include/State/Reset.cuh:52-63,
 *      src/RLConstants.cu:4-29) --------------------------------------------- */

uint32_t co_hash32(uint32_t v)
{
    v = ((v >> 16) ^ v) * 0x45d9f3bu;
    v = ((v >> 16) ^ v) * 0x45d9f3bu;
    return (v >> 16) ^ v;
}

int32_t co_kickoff_row(int32_t seed, int32_t sim, int32_t tick)
{
    const uint32_t h = co_hash32((uint32_t)seed) ^ co_hash32((uint32_t)sim) ^ co_hash32((uint32_t)tick);
    return (int32_t)(co_hash32(h) % 120u);
}

void co_kickoff_table(int32_t out[120][4])
{
    int row = 0;
    for (int skip = 0; skip < 5; skip++)
        for (int a = 0; a < 5; a++)
            for (int b = 0; b < 5; b++)
                for (int c = 0; c < 5; c++)
                    for (int d = 0; d < 5; d++)
                    {
                        const int v[4] = { a, b, c, d };
                        int ok = 1;
                        for (int i = 0; i < 4; i++)
                        {
                            if (v[i] == skip) ok = 0;
                            for (int j = 0; j < i; j++)
                                if (v[i] == v[j]) ok = 0;
                        }
                        if (!ok) continue;
                        for (int i = 0; i < 4; i++) out[row][i] = v[i];
                        row++;
                    }
}
