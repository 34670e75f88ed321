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
void engine_destroy(void* e);

// topology of a validated v1 model, derived once at load
struct Topology {
    int enc[4];     // encoder widths (conv1/conv2 Cout per stage)
    int bott;       // bottleneck width
    int dec[4];     // decoder widths dec4..dec1
    int bands, classes;
};
int validate_topology(const Model* m, Topology* t);

}  // namespace bnn
