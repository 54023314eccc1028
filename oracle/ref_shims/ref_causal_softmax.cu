// Exposes logit() of the reference's tests/tile_causal_softmax.cu (:270-273).
#define main tkref_tile_causal_softmax_main
#include "tile_causal_softmax.cu"
#undef main

extern "C" double tkref_causal_logit(int row, int col, int extreme) {
    return logit(row, col, extreme != 0);
}
