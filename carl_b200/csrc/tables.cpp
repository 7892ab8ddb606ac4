// Host construction of the game tables uploaded to constant memory.
//
// Boost pads, kickoff and respawn spots are the soccar values used by the
// reference (jwmccarthy/CARL include/Physics/BoostPads.cuh:21-56,
// include/RLConstants.cuh:53-67).  Two tables are derived instead of listed:
//   * kickoffPerm: every ordered arrangement of 4 of the 5 kickoff spots,
//     grouped by the spot left out (0..4) and lexicographic within a group,
//     which is the order of the reference's KICKOFF_PERMUTATIONS
//     (src/RLConstants.cu:4-29);
//   * padMirror: the pad at (-x, -y) of each pad, which is what an inverted
//     (orange) observer sees at that index (include/Physics/Observations.cuh:86-94).
#include <algorithm>
#include <cmath>

#include "cb_tables.hpp"

namespace cb {

void buildTables(Tables& t)
{
    struct Pad { float x, y, z; int big; };
    static const Pad pads[NUM_BOOST_PADS] = {
        { -3584.f, 0.f, 73.f, 1 },     { 3584.f, 0.f, 73.f, 1 },      { -3072.f, 4096.f, 73.f, 1 },
        { 3072.f, 4096.f, 73.f, 1 },   { -3072.f, -4096.f, 73.f, 1 }, { 3072.f, -4096.f, 73.f, 1 },
        { 0.f, -4240.f, 70.f, 0 },     { -1792.f, -4184.f, 70.f, 0 }, { 1792.f, -4184.f, 70.f, 0 },
        { -940.f, -3308.f, 70.f, 0 },  { 940.f, -3308.f, 70.f, 0 },   { 0.f, -2816.f, 70.f, 0 },
        { -3584.f, -2484.f, 70.f, 0 }, { 3584.f, -2484.f, 70.f, 0 },  { -1788.f, -2300.f, 70.f, 0 },
        { 1788.f, -2300.f, 70.f, 0 },  { -2048.f, -1036.f, 70.f, 0 }, { 0.f, -1024.f, 70.f, 0 },
        { 2048.f, -1036.f, 70.f, 0 },  { -1024.f, 0.f, 70.f, 0 },     { 1024.f, 0.f, 70.f, 0 },
        { -2048.f, 1036.f, 70.f, 0 },  { 0.f, 1024.f, 70.f, 0 },      { 2048.f, 1036.f, 70.f, 0 },
        { -1788.f, 2300.f, 70.f, 0 },  { 1788.f, 2300.f, 70.f, 0 },   { -3584.f, 2484.f, 70.f, 0 },
        { 3584.f, 2484.f, 70.f, 0 },   { 0.f, 2816.f, 70.f, 0 },      { -940.f, 3308.f, 70.f, 0 },
        { 940.f, 3308.f, 70.f, 0 },    { -1792.f, 4184.f, 70.f, 0 },  { 1792.f, 4184.f, 70.f, 0 },
        { 0.f, 4240.f, 70.f, 0 },
    };
    for (int p = 0; p < NUM_BOOST_PADS; p++)
    {
        t.padX[p] = pads[p].x;
        t.padY[p] = pads[p].y;
        t.padZ[p] = pads[p].z;
        t.padBig[p] = pads[p].big;
    }
    // Pad cell lists: every pad whose pickup disk comes within 2 uu of the cell
    // (the margin covers a car's cell being rounded to a neighbour).  The disks
    // are disjoint (pads are at least 1000 uu apart, radii at most 208), so a
    // car is on at most one pad and at most 4 pads reach a cell.
    for (int cy = 0; cy < PAD_GRID_NY; cy++)
        for (int cx = 0; cx < PAD_GRID_NX; cx++)
        {
            const double x0 = PAD_GRID_X0 + (double)cx * PAD_CELL, y0 = PAD_GRID_Y0 + (double)cy * PAD_CELL;
            unsigned word = 0xffffffffu;
            int n = 0;
            for (int p = 0; p < NUM_BOOST_PADS; p++)
            {
                const double px = pads[p].x, py = pads[p].y;
                const double dx = px < x0 ? x0 - px : (px > x0 + PAD_CELL ? px - x0 - PAD_CELL : 0.0);
                const double dy = py < y0 ? y0 - py : (py > y0 + PAD_CELL ? py - y0 - PAD_CELL : 0.0);
                const double reach = (pads[p].big ? BIG_PAD_RADIUS : SMALL_PAD_RADIUS) + 2.0;
                if (dx * dx + dy * dy >= reach * reach) continue;
                if (n < 4) word = (word & ~(0xffu << (8 * n))) | ((unsigned)p << (8 * n));
                n++;
            }
            t.padCell[cy * PAD_GRID_NX + cx] = n <= 4 ? word : 0xfffffffeu;  // 0xfffffffe: more than 4 (never)
        }
    for (int p = 0; p < NUM_BOOST_PADS; p++)
    {
        t.padMirror[p] = p;
        for (int q = 0; q < NUM_BOOST_PADS; q++)
            if (pads[q].x == -pads[p].x && pads[q].y == -pads[p].y) t.padMirror[p] = q;
    }

    int row = 0;
    for (int skip = 0; skip < 5; skip++)
    {
        int spots[4], n = 0;
        for (int s = 0; s < 5; s++)
            if (s != skip) spots[n++] = s;
        do
        {
            for (int k = 0; k < 4; k++) t.kickoffPerm[row][k] = spots[k];
            row++;
        } while (std::next_permutation(spots, spots + 4));
    }

    const float kx[5] = { -2048.f, 2048.f, -256.f, 256.f, 0.f };
    const float ky[5] = { -2560.f, -2560.f, -3840.f, -3840.f, -4608.f };
    const float kyaw[5] = { PI_4 * 1, PI_4 * 3, PI_4 * 2, PI_4 * 2, PI_4 * 2 };
    for (int k = 0; k < 5; k++)
    {
        t.kickX[k] = kx[k];
        t.kickY[k] = ky[k];
        t.kickYaw[k] = kyaw[k];
    }
    const float rx[4] = { 2688.f, 2304.f, -2304.f, -2688.f };
    for (int k = 0; k < 4; k++)
    {
        t.respX[k] = rx[k];
        t.respY[k] = -4608.f;
        t.respYaw[k] = PI_2 * 1;
    }
}

}  // namespace cb
