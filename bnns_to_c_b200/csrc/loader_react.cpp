// loader_react.cpp - blob v3 (ReActNet) parser behind bnn_load_react /
// bnn_react_load_ex / bnn_react_load_mem.
//
// Record for record the reference's loader (csrc/bnn_model_react.c:42-135):
// magic, version 3 ("blob version %d, this engine reads v3 (ReActNet)"),
// upsampler 0 ("only nearest upsampler supported"), 4 DownBlocks, the
// bottleneck and 4 PlainBlocks ([tap1] conv1 proj1 epi1 tap2 conv2 epi_a
// [epi_b]) with the same structural checks ("blob layout mismatch: ..."),
// head tag 4, no trailing byte. Then the topology the forward needs is
// validated (channel chains, 3x3 pad 1 stride 1 convs, head width), which the
// reference leaves to crash; violations are BNN_ERR_UNSUPPORTED.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.h"
#include "../../include/bnn_model_react.h"

namespace bnn {

void* react_engine_create();
void react_engine_destroy(void* e);

namespace {

struct Rd {
    const unsigned char* p;
    size_t n, off;
    int status = BNN_OK;
    bool fail(int code, const char* msg) {
        if (status == BNN_OK) status = set_error(code, "%s", msg);
        return false;
    }
    bool bytes(void* d, size_t k) {
        if (status != BNN_OK) return false;
        if (n - off < k) return fail(BNN_ERR_FORMAT, "short read");
        memcpy(d, p + off, k);
        off += k;
        return true;
    }
    int i32() {
        int32_t v = 0;
        bytes(&v, 4);
        return v;
    }
    template <class T>
    T* arr(size_t count) {
        if (status != BNN_OK) return nullptr;
        const size_t k = count * sizeof(T);
        if (n - off < k) { fail(BNN_ERR_FORMAT, "short read"); return nullptr; }
        T* q = (T*)malloc(k ? k : 1);
        if (!q) { fail(BNN_ERR_OOM, "OOM"); return nullptr; }
        bytes(q, k);
        return q;
    }
    void tag(int want, const char* what) {
        int t = i32();
        if (status == BNN_OK && t != want) {
            char m[64];
            snprintf(m, sizeof m, "bad %s tag %d", what, t);
            fail(BNN_ERR_FORMAT, m);
        }
    }
};

void rd_conv(Rd& r, ConvR* c) {
    memset(c, 0, sizeof *c);
    c->tag = r.i32();
    c->Cout = r.i32(); c->Cin = r.i32(); c->kh = r.i32(); c->kw = r.i32(); c->pad = r.i32(); c->stride = r.i32();
    if (r.status != BNN_OK) return;
    if (c->tag == 1) {
        c->nwords = r.i32();
        if (r.status == BNN_OK && (c->Cout < 0 || c->nwords < 0)) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
        c->packed = r.arr<uint64_t>((size_t)c->Cout * c->nwords);
    } else if (c->tag == 2) {
        if (c->Cout < 0 || c->Cin < 0 || c->kh < 0 || c->kw < 0) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
        c->wsign = r.arr<int8_t>((size_t)c->Cout * c->Cin * c->kh * c->kw);
        c->alpha = r.arr<float>((size_t)c->Cout);
    } else {
        char m[64];
        snprintf(m, sizeof m, "bad conv tag %d", c->tag);
        r.fail(BNN_ERR_FORMAT, m);
    }
}

void rd_proj(Rd& r, ProjR* p) {
    r.tag(5, "proj");
    p->Cout = r.i32(); p->Cin = r.i32();
    if (r.status == BNN_OK && (p->Cout < 0 || p->Cin < 0)) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
    p->W = r.arr<float>((size_t)p->Cout * p->Cin);
}

void rd_epi(Rd& r, EpiR* e) {
    r.tag(6, "epi");
    e->kind = r.i32(); e->C = r.i32();
    if (r.status == BNN_OK && e->C < 0) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
    e->A = r.arr<float>(e->C); e->B = r.arr<float>(e->C);
    e->move1 = r.arr<float>(e->C); e->prelu_w = r.arr<float>(e->C);
}

void rd_tap(Rd& r, TapR* t) {
    r.tag(7, "tap");
    t->C = r.i32();
    if (r.status == BNN_OK && t->C < 0) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
    t->rsign = r.arr<float>(t->C);
}

// csrc/bnn_model_react.c:85-106
void rd_block(Rd& r, BlockR* b, int is_down, int input_real) {
    memset(b, 0, sizeof *b);
    b->is_down = is_down; b->input_real = input_real;
    if (!input_real) rd_tap(r, &b->tap1);
    rd_conv(r, &b->conv1);
    rd_proj(r, &b->proj1);
    rd_epi(r, &b->epi1);
    rd_tap(r, &b->tap2);
    rd_conv(r, &b->conv2);
    rd_epi(r, &b->epi_a);
    if (is_down) rd_epi(r, &b->epi_b);
    if (r.status != BNN_OK) return;
    auto check = [&](bool ok, const char* what) {
        if (!ok && r.status == BNN_OK) {
            char m[96];
            snprintf(m, sizeof m, "blob layout mismatch: %s", what);
            r.fail(BNN_ERR_FORMAT, m);
        }
    };
    check(b->conv1.tag == (input_real ? 2 : 1), "conv1 tag");
    check(b->conv2.tag == 1, "conv2 tag");
    check(b->proj1.Cin == b->conv1.Cin && b->proj1.Cout == b->conv1.Cout, "proj1 dims");
    check(input_real || b->tap1.C == b->conv1.Cin, "tap1 channels");
    check(b->tap2.C == b->conv2.Cin, "tap2 channels");
    check(b->epi1.C == b->conv1.Cout && b->epi1.kind == (input_real ? 1 : 0), "epi1");
    check(b->epi_a.C == b->conv2.Cout && b->epi_a.kind == 0, "epi_a");
    check(!is_down || (b->epi_b.C == b->conv2.Cout && b->epi_b.kind == 0), "epi_b");
}

void free_block(BlockR* b) {
    free(b->tap1.rsign); free(b->tap2.rsign);
    free(b->conv1.packed); free(b->conv1.wsign); free(b->conv1.alpha);
    free(b->conv2.packed); free(b->conv2.wsign); free(b->conv2.alpha);
    free(b->proj1.W);
    EpiR* e[3] = {&b->epi1, &b->epi_a, &b->epi_b};
    for (EpiR* x : e) { free(x->A); free(x->B); free(x->move1); free(x->prelu_w); }
}

void free_arrays(ModelR* m) {
    for (int i = 0; i < 4; ++i) { free_block(&m->enc[i]); free_block(&m->dec[i]); }
    free_block(&m->bott);
    free(m->head_W); free(m->head_bias);
}

int unsupported(const char* blk, const char* what) {
    return set_error(BNN_ERR_UNSUPPORTED, "%s: %s", blk, what);
}

int check_bin(const ConvR& c, const char* blk, int cin) {
    char m[128];
    if (c.kh != 3 || c.kw != 3 || c.pad != 1 || c.stride != 1) {
        snprintf(m, sizeof m, "%dx%d pad %d stride %d conv, the forward runs 3x3 pad 1 stride 1", c.kh, c.kw, c.pad,
                 c.stride);
        return unsupported(blk, m);
    }
    if (c.Cin != cin || c.Cout <= 0) {
        snprintf(m, sizeof m, "conv Cin %d Cout %d, its input has %d channels", c.Cin, c.Cout, cin);
        return unsupported(blk, m);
    }
    if (c.tag == 1 && c.nwords != (9 * c.Cin + 63) / 64) return unsupported(blk, "nwords != ceil(9*Cin/64)");
    return BNN_OK;
}

}  // namespace

// The channel chain of csrc/bnn_model_react.c:395-441: enc i takes the
// previous level's width, conv2 keeps conv1's width, the bottleneck takes
// enc4's, dec i takes skip + previous widths, the head takes dec1's; enc1's
// real conv weights are -1 / 0 / +1 (every product of its sum exact).
int react_validate(const ModelR* m) {
    static const char* EN[4] = {"enc1", "enc2", "enc3", "enc4"};
    static const char* DN[4] = {"dec4", "dec3", "dec2", "dec1"};
    int rc;
    if (m->n_bands <= 0 || m->n_classes <= 0)
        return set_error(BNN_ERR_UNSUPPORTED, "n_bands %d / n_classes %d", m->n_bands, m->n_classes);
    int cin = m->n_bands, skipc[4];
    for (int i = 0; i < 4; ++i) {
        const BlockR& b = m->enc[i];
        if ((rc = check_bin(b.conv1, EN[i], cin)) || (rc = check_bin(b.conv2, EN[i], b.conv1.Cout))) return rc;
        if (b.conv2.Cout != b.conv1.Cout) return unsupported(EN[i], "conv2 width != conv1 width");
        cin = skipc[i] = b.conv2.Cout;
    }
    {
        const ConvR& c1 = m->enc[0].conv1;
        for (size_t k = 0; k < (size_t)c1.Cout * c1.Cin * 9; ++k)
            if (c1.wsign[k] < -1 || c1.wsign[k] > 1) return unsupported("enc1", "real conv wsign outside -1, 0, +1");
    }
    if ((rc = check_bin(m->bott.conv1, "bottleneck", cin)) ||
        (rc = check_bin(m->bott.conv2, "bottleneck", m->bott.conv1.Cout)))
        return rc;
    if (m->bott.conv2.Cout != m->bott.conv1.Cout) return unsupported("bottleneck", "conv2 width != conv1 width");
    int prev = m->bott.conv2.Cout;
    for (int i = 0; i < 4; ++i) {
        const BlockR& b = m->dec[i];
        if ((rc = check_bin(b.conv1, DN[i], skipc[3 - i] + prev)) || (rc = check_bin(b.conv2, DN[i], b.conv1.Cout)))
            return rc;
        if (b.conv2.Cout != b.conv1.Cout) return unsupported(DN[i], "conv2 width != conv1 width");
        prev = b.conv2.Cout;
    }
    if (m->dec[0].conv1.Cin > 3072 || m->n_bands > 3072)
        return set_error(BNN_ERR_UNSUPPORTED, "block input wider than 3072 channels (projection tile limit)");
    if (m->head_Cin != prev) return unsupported("head", "Cin != dec1 width");
    if (m->head_Cout != m->n_classes) return unsupported("head", "Cout != n_classes");
    return BNN_OK;
}

static int parse_react(const unsigned char* data, size_t n, ModelR** out) {
    *out = nullptr;
    Rd r{data, n, 0};
    char magic[4] = {0, 0, 0, 0};
    r.bytes(magic, 4);
    if (r.status == BNN_OK && memcmp(magic, "BNNC", 4) != 0) r.fail(BNN_ERR_FORMAT, "bad magic");
    if (r.status != BNN_OK) return r.status;
    ModelR* m = (ModelR*)calloc(1, sizeof(ModelR));
    if (!m) return set_error(BNN_ERR_OOM, "OOM %zu", sizeof(ModelR));
    m->version = r.i32();
    if (r.status == BNN_OK && m->version != 3) {
        char msg[96];
        snprintf(msg, sizeof msg, "blob version %d, this engine reads v3 (ReActNet)", m->version);
        r.fail(BNN_ERR_FORMAT, msg);
    }
    m->base_channels = r.i32(); m->n_bands = r.i32(); m->n_classes = r.i32(); m->upsampler = r.i32();
    if (r.status == BNN_OK && m->upsampler != 0) r.fail(BNN_ERR_FORMAT, "only nearest upsampler supported");
    for (int i = 0; i < 4 && r.status == BNN_OK; ++i) rd_block(r, &m->enc[i], 1, i == 0);
    if (r.status == BNN_OK) rd_block(r, &m->bott, 0, 0);
    for (int i = 0; i < 4 && r.status == BNN_OK; ++i) rd_block(r, &m->dec[i], 0, 0);
    r.tag(4, "head");
    m->head_Cout = r.i32(); m->head_Cin = r.i32();
    if (r.status == BNN_OK && (m->head_Cout < 0 || m->head_Cin < 0)) r.fail(BNN_ERR_FORMAT, "short read");
    m->head_W = r.arr<float>((size_t)m->head_Cout * m->head_Cin);
    m->head_bias = r.arr<float>((size_t)m->head_Cout);
    if (r.status == BNN_OK && r.off != r.n) r.fail(BNN_ERR_FORMAT, "trailing bytes in blob");
    int rc = r.status;
    if (rc == BNN_OK) rc = react_validate(m);
    if (rc == BNN_OK && !(m->engine = react_engine_create())) rc = set_error(BNN_ERR_OOM, "OOM engine");
    if (rc != BNN_OK) {
        free_arrays(m);
        free(m);
        return rc;
    }
    *out = m;
    return BNN_OK;
}

void react_free_model(ModelR* m) {
    if (!m) return;
    react_engine_destroy(m->engine);
    free_arrays(m);
    free(m);
}

}  // namespace bnn

using namespace bnn;

BNN_API int bnn_react_load_mem(const void* data, size_t n, ModelR** out) {
    if (!out) return set_error(BNN_ERR_ARG, "out is NULL");
    clear_error();
    return parse_react((const unsigned char*)data, n, out);
}

BNN_API int bnn_react_load_ex(const char* path, ModelR** out) {
    if (!out) return set_error(BNN_ERR_ARG, "out is NULL");
    *out = nullptr;
    clear_error();
    FILE* f = fopen(path, "rb");
    if (!f) return set_error(BNN_ERR_IO, "cannot open %s", path);
    std::string buf;
    char chunk[1 << 16];
    size_t k;
    while ((k = fread(chunk, 1, sizeof chunk, f)) > 0) buf.append(chunk, k);
    int err = ferror(f);
    fclose(f);
    if (err) return set_error(BNN_ERR_IO, "short read");
    return parse_react((const unsigned char*)buf.data(), buf.size(), out);
}

BNN_API ModelR* bnn_load_react(const char* path) {
    ModelR* m = nullptr;
    if (bnn_react_load_ex(path, &m) != BNN_OK) {
        fprintf(stderr, "%s\n", bnn_last_error());
        exit(1);
    }
    return m;
}

BNN_API void bnn_free_react(ModelR* m) { react_free_model(m); }
