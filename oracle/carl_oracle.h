/*
 * carl_oracle.h - plain-C restatement of the reference's integer / index paths
 * of the tick, used only as a test checker (never by the product).
 *
 * Covered: arena mesh parse + exact-bit weld + uniform-grid CSR build,
 * the broadphase grid cell of a car pose, the kickoff permutation table and the
 * per-sim kickoff hash.  Each function cites the reference code it restates.
 * TEST INFRASTRUCTURE.
 */
#ifndef CARL_ORACLE_H
#define CARL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Arena tables (default mesh path).  Arrays are malloc'd; free with co_arena_free. */
typedef struct co_arena {
    int n_verts, n_tris, n_cells, n_refs;
    float* verts;      /* [n_verts][3] */
    int32_t* tris;     /* [n_tris][3]  */
    int32_t* prefix;   /* [n_cells+1]  */
    int32_t* tri_idx;  /* [n_refs]     */
} co_arena;

int co_arena_build(const char* obj_path, co_arena* out);
void co_arena_free(co_arena* a);

/* Grid cell (flat index) of the minimum corner of a car's box swept over one tick. */
int32_t co_broadphase_cell(const float pos[3], const float vel[3], const float ang[3],
                           const float cen[3], const float rot[4]);

uint32_t co_hash32(uint32_t v);
/* Row of the kickoff permutation table chosen for (seed, sim, tick). */
int32_t co_kickoff_row(int32_t seed, int32_t sim, int32_t tick);
/* The 120 x 4 kickoff permutation table. */
void co_kickoff_table(int32_t out[120][4]);

#ifdef __cplusplus
}
#endif

#endif
