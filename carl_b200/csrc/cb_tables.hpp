// Game tables kept in constant memory (built on the host by tables.cpp).
#pragma once

#include "cb_consts.cuh"

namespace cb {

constexpr int PAD_CELL = 512;
constexpr int PAD_GRID_NX = 16, PAD_GRID_NY = 20;
constexpr float PAD_GRID_X0 = -4096.f, PAD_GRID_Y0 = -5120.f;

struct Tables
{
    float padX[NUM_BOOST_PADS], padY[NUM_BOOST_PADS], padZ[NUM_BOOST_PADS];
    int padBig[NUM_BOOST_PADS];
    int padMirror[NUM_BOOST_PADS];   // pad seen at index p by an inverted (orange) observer
    int kickoffPerm[120][4];         // ordered 4-subsets of the 5 kickoff spots
    float kickX[5], kickY[5], kickYaw[5];
    float respX[4], respY[4], respYaw[4];
    // Boost pads whose pickup disk reaches each PAD_CELL-sized cell of the field
    // (x from PAD_GRID_X0, y from PAD_GRID_Y0), up to 4 pad numbers a word, one
    // byte each, 0xff = none.  A car outside the grid is near no pad.
    unsigned padCell[PAD_GRID_NX * PAD_GRID_NY];
};

void buildTables(Tables& t);

}  // namespace cb
