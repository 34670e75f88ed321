// common.h - internal declarations shared by the host loader and the engine.
#pragma once
#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/bnn_b200.h"

#define BNN_API extern "C" __attribute__((visibility("default")))

namespace bnn {

// thread-local last-error message + status helper
int set_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

// engine lifetime (engine.cu): attached to a parsed Model by the loader
void* engine_create();
// the engine of a v2 (spectral-stem) model: the stem records it runs before
// the body (arrays borrowed from the StemModel, which outlives the engine)
void* engine_create_stem(const Conv* stem_conv, const Act* stem_act);
// stem width of the engine's model, 0 for a v1 model
int engine_stem_c(const void* e);
void engine_destroy(void* e);

// topology of a validated v1 model, derived once at load
struct Topology {
    int stem;       // v2 stem width (enc1.conv1 is binary on it), 0 for v1
    int enc[4];     // encoder widths (conv1/conv2 Cout per stage)
    int bott;       // bottleneck width
    int dec[4];     // decoder widths dec4..dec1
    int bands, classes;
};
// stem_c > 0: the body of a v2 model whose stem has stem_c channels
int validate_topology(const Model* m, Topology* t, int stem_c = 0);

// Debug fill of the activation arenas before every forward (engine.cu):
// the byte to write, or -1 for none. Read from BNN_ARENA_POISON (its value
// & 255, as csrc/bnn_react_arena.c:30-32 reads it) on first use unless
// bnn_set_arena_poison set it.
int arena_poison_byte();

}  // namespace bnn
