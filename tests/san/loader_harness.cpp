// Host-only harness for a sanitizer build of the blob loaders (loader.cpp,
// loader_react.cpp) with the device engine stubbed out. Test
// infrastructure: tests/test_sanitize_cpu.py compiles it with
// -fsanitize=address,undefined and feeds it corrupted blobs.
//
//   loader_harness <v1|stem|react> FILE...
//
// Per file, one line: "<status>\t<bnn_last_error()>" from the status loader
// given the file as an exactly sized heap buffer (so an over-read past the
// blob is a sanitizer report), after checking that the path loader agrees.
// A model that loads is freed again (leak checks see the whole lifetime).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "bnn_b200.h"
#include "bnn_model.h"
#include "bnn_model_react.h"
#include "bnn_model_stem.h"

namespace bnn {
// the engine hooks the loaders call (engine.cu, react.cu), without a device
struct StubEngine {
    int stem_c;
};
void* engine_create() { return new StubEngine{0}; }
void* engine_create_stem(const Conv* stem_conv, const Act*) { return new StubEngine{stem_conv->Cout}; }
int engine_stem_c(const void* e) { return e ? static_cast<const StubEngine*>(e)->stem_c : 0; }
void engine_destroy(void* e) { delete static_cast<StubEngine*>(e); }
void* react_engine_create() { return new int(0); }
void react_engine_destroy(void* e) { delete static_cast<int*>(e); }
}  // namespace bnn

extern "C" void bnn_forward(const Model*, const float*, int, int, float*) {
    fprintf(stderr, "loader harness: no forward\n");
    abort();
}

static bool read_file(const char* path, std::vector<unsigned char>* out) {
    FILE* f = fopen(path, "rb");
    if (!f) return false;
    unsigned char chunk[1 << 16];
    size_t k;
    while ((k = fread(chunk, 1, sizeof chunk, f)) > 0) out->insert(out->end(), chunk, chunk + k);
    fclose(f);
    return true;
}

template <class M, class LoadMem, class LoadPath, class Free>
static int run(const char* path, LoadMem load_mem, LoadPath load_path, Free free_model) {
    std::vector<unsigned char> bytes;
    if (!read_file(path, &bytes)) {
        fprintf(stderr, "cannot read %s\n", path);
        return 2;
    }
    // exactly sized copy: reading one byte past the blob is a heap overflow
    unsigned char* buf = static_cast<unsigned char*>(malloc(bytes.size() ? bytes.size() : 1));
    if (!bytes.empty()) memcpy(buf, bytes.data(), bytes.size());
    M* m = nullptr;
    const int rc = load_mem(buf, bytes.size(), &m);
    const std::string msg = bnn_last_error();
    free(buf);
    if (m) free_model(m);
    M* m2 = nullptr;
    const int rc2 = load_path(path, &m2);
    const std::string msg2 = bnn_last_error();
    if (m2) free_model(m2);
    if (rc != rc2 || msg != msg2) {
        fprintf(stderr, "%s: memory load (%d, %s) != path load (%d, %s)\n", path, rc, msg.c_str(), rc2,
                msg2.c_str());
        return 3;
    }
    printf("%d\t%s\n", rc, msg.c_str());
    return 0;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: %s <v1|stem|react> FILE...\n", argv[0]);
        return 2;
    }
    const std::string kind = argv[1];
    for (int i = 2; i < argc; ++i) {
        int r;
        if (kind == "v1")
            r = run<Model>(argv[i], bnn_load_mem, bnn_load_ex, bnn_free);
        else if (kind == "stem")
            r = run<StemModel>(argv[i], bnn_stem_load_mem, bnn_stem_load_ex, bnn_stem_free);
        else if (kind == "react")
            r = run<ModelR>(argv[i], bnn_react_load_mem, bnn_react_load_ex, bnn_free_react);
        else {
            fprintf(stderr, "unknown kind %s\n", kind.c_str());
            return 2;
        }
        if (r) return r;
    }
    return 0;
}
