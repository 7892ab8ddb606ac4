// Game tables kept in constant memory (built on the host by tables.cpp).
#pragma once

#include "cb_consts.cuh"

namespace cb {

struct Tables
{
    float padX[NUM_BOOST_PADS], padY[NUM_BOOST_PADS], padZ[NUM_BOOST_PADS];
    int padBig[NUM_BOOST_PADS];
    int padMirror[NUM_BOOST_PADS];   // pad seen at index p by an inverted (orange) observer
    int kickoffPerm[120][4];         // ordered 4-subsets of the 5 kickoff spots
    float kickX[5], kickY[5], kickYaw[5];
    float respX[4], respY[4], respYaw[4];
};

void buildTables(Tables& t);

}  // namespace cb
