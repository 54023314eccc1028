// Exposes the host fixtures (fill_* :40-83), the FP64 reference with
// FP16-rounded probabilities (make_reference :97-140) and midpoint_margin
// (:149-159) of the reference's tests/attention_correctness.cu.
#include <cstdint>
#include <cstring>
#define main tkref_attention_main
#include "attention_correctness.cu"
#undef main

// which: 0 uniform, 1 shifted one-hot with identity V, 2 shifted one-hot with
// asymmetric V, 3 large scores, 4 aliased input (only q is written).
extern "C" void tkref_attention_fill(int which, uint16_t* q, uint16_t* k, uint16_t* v) {
    static Data data;
    std::memset(&data, 0, sizeof(data));
    switch (which) {
        case 0: fill_uniform(&data); break;
        case 1: fill_shifted_one_hot(&data, true); break;
        case 2: fill_shifted_one_hot(&data, false); break;
        case 3: fill_large_scores(&data); break;
        default: fill_alias_input(&data); break;
    }
    std::memcpy(q, data.q, sizeof(data.q));
    std::memcpy(k, data.k, sizeof(data.k));
    std::memcpy(v, data.v, sizeof(data.v));
}

extern "C" void tkref_attention_reference(const uint16_t* q, const uint16_t* k,
                                          const uint16_t* v, int causal,
                                          double* probability, uint16_t* rounded,
                                          double* out) {
    const Reference r = make_reference(reinterpret_cast<const __half*>(q),
                                       reinterpret_cast<const __half*>(k),
                                       reinterpret_cast<const __half*>(v), causal != 0);
    std::memcpy(probability, r.probability, sizeof(r.probability));
    std::memcpy(rounded, r.rounded_probability, sizeof(r.rounded_probability));
    std::memcpy(out, r.out, sizeof(r.out));
}

extern "C" double tkref_midpoint_margin(double probability, uint16_t rounded) {
    __half h;
    std::memcpy(&h, &rounded, sizeof(h));
    return midpoint_margin(probability, h);
}
