// Exposes the logit generators of the reference's tests/tile_softmax.cu
// (logits :97-108) and tests/tile_causal_softmax.cu (logit :270-273).
#define main tkref_tile_softmax_main
#include "tile_softmax.cu"
#undef main

extern "C" float tkref_softmax_logit(int group, int row, int col, int kind) {
    return logits(group, row, col, kind);
}
