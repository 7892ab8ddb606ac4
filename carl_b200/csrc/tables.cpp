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
