// loader.cpp - blob v1 parser behind bnn_load / bnn_load_ex / bnn_load_mem.
//
// Parsing follows the reference loader record for record (csrc/bnn_model.c:
// 27-96): magic "BNNC", five header ints (version is read, not checked, as
// there), 4 x [conv, act, conv, act, act], [conv, act] x 2, 4 x [conv, act,
// conv, act], head tag 4, and no trailing byte. The same conditions fail with
// the same messages ("cannot open", "short read", "bad magic", "bad conv
// tag", "bad act tag", "bad head tag", "trailing bytes in blob").
//
// After parsing, the topology bnn_forward needs is validated (the reference
// would crash or read out of bounds on such blobs instead); violations are
// BNN_ERR_UNSUPPORTED with a message naming the record.
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.h"
#include "../../include/bnn_model_stem.h"

namespace bnn {

static thread_local std::string g_err;

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

void clear_error() { g_err.clear(); }

namespace {

struct Reader {
    const unsigned char* p;
    size_t n, off;
    int status = BNN_OK;

    bool fail(int code, const char* msg) {
        if (status == BNN_OK) status = set_error(code, "%s", msg);
        return false;
    }
    bool bytes(void* dst, size_t k) {
        if (status != BNN_OK) return false;
        if (n - off < k) return fail(BNN_ERR_FORMAT, "short read");
        memcpy(dst, p + off, k);
        off += k;
        return true;
    }
    int i32() {
        int32_t v = 0;
        bytes(&v, 4);
        return v;
    }
    void* alloc_read(size_t k) {
        if (status != BNN_OK) return nullptr;
        if (n - off < k) { fail(BNN_ERR_FORMAT, "short read"); return nullptr; }
        void* q = malloc(k ? k : 1);
        if (!q) { fail(BNN_ERR_OOM, "OOM"); return nullptr; }
        bytes(q, k);
        return q;
    }
};

void read_conv(Reader& r, Conv* c) {
    memset(c, 0, sizeof *c);
    c->tag = r.i32();
    c->Cout = r.i32(); c->Cin = r.i32(); c->kh = r.i32(); c->kw = r.i32();
    c->pad = r.i32(); c->stride = r.i32();
    if (r.status != BNN_OK) return;
    if (c->tag == 1) {
        c->nwords = r.i32();
        if (r.status != BNN_OK) return;
        if (c->Cout < 0 || c->nwords < 0) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
        c->packed = (uint64_t*)r.alloc_read((size_t)c->Cout * (size_t)c->nwords * 8);
    } else if (c->tag == 2) {
        if (c->Cout < 0 || c->Cin < 0 || c->kh < 0 || c->kw < 0) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
        c->wsign = (int8_t*)r.alloc_read((size_t)c->Cout * c->Cin * c->kh * c->kw);
        c->alpha = (float*)r.alloc_read((size_t)c->Cout * 4);
    } else {
        char m[64];
        snprintf(m, sizeof m, "bad conv tag %d", c->tag);
        r.fail(BNN_ERR_FORMAT, m);
    }
}

void read_act(Reader& r, Act* a) {
    memset(a, 0, sizeof *a);
    int tag = r.i32();
    if (r.status != BNN_OK) return;
    if (tag != 3) {
        char m[64];
        snprintf(m, sizeof m, "bad act tag %d", tag);
        r.fail(BNN_ERR_FORMAT, m);
        return;
    }
    a->kind = r.i32(); a->C = r.i32();
    if (r.status != BNN_OK) return;
    if (a->C < 0) { r.fail(BNN_ERR_FORMAT, "short read"); return; }
    size_t k = (size_t)a->C * 4;
    if (a->kind == 0) {
        a->type = (int32_t*)r.alloc_read(k); a->t = (int32_t*)r.alloc_read(k);
        a->lo = (int32_t*)r.alloc_read(k);   a->hi = (int32_t*)r.alloc_read(k);
    } else {
        a->A = (float*)r.alloc_read(k);     a->B = (float*)r.alloc_read(k);
        a->slope = (float*)r.alloc_read(k); a->rsign = (float*)r.alloc_read(k);
    }
}

void free_conv(Conv* c) { free(c->packed); free(c->wsign); free(c->alpha); }
void free_act(Act* a) {
    free(a->type); free(a->t); free(a->lo); free(a->hi);
    free(a->A); free(a->B); free(a->slope); free(a->rsign);
}

void free_model_arrays(Model* m) {
    for (int i = 0; i < 4; ++i) {
        free_conv(&m->enc_conv1[i]); free_conv(&m->enc_conv2[i]);
        free_act(&m->enc_act1[i]); free_act(&m->enc_act2_skip[i]); free_act(&m->enc_act2_down[i]);
        free_conv(&m->dec_conv1[i]); free_conv(&m->dec_conv2[i]);
        free_act(&m->dec_act1[i]); free_act(&m->dec_act2[i]);
    }
    free_conv(&m->bott_conv1); free_conv(&m->bott_conv2);
    free_act(&m->bott_act1); free_act(&m->bott_act2);
    free(m->head_W); free(m->head_bias);
}

// everything after the header (and, for v2, the stem records): the body
// records, the head and the end-of-blob check (csrc/bnn_model.c:74-95,
// csrc/bnn_model_stem.c:95-114 read the same sequence)
void parse_body(Reader& r, Model* m) {
    for (int i = 0; i < 4; ++i) {
        read_conv(r, &m->enc_conv1[i]); read_act(r, &m->enc_act1[i]);
        read_conv(r, &m->enc_conv2[i]); read_act(r, &m->enc_act2_skip[i]);
        read_act(r, &m->enc_act2_down[i]);
    }
    read_conv(r, &m->bott_conv1); read_act(r, &m->bott_act1);
    read_conv(r, &m->bott_conv2); read_act(r, &m->bott_act2);
    for (int i = 0; i < 4; ++i) {
        read_conv(r, &m->dec_conv1[i]); read_act(r, &m->dec_act1[i]);
        read_conv(r, &m->dec_conv2[i]); read_act(r, &m->dec_act2[i]);
    }
    int tag = r.i32();
    if (r.status == BNN_OK && tag != 4) {
        char msg[64];
        snprintf(msg, sizeof msg, "bad head tag %d", tag);
        r.fail(BNN_ERR_FORMAT, msg);
    }
    m->head_Cout = r.i32(); m->head_Cin = r.i32();
    if (r.status == BNN_OK && (m->head_Cout < 0 || m->head_Cin < 0)) r.fail(BNN_ERR_FORMAT, "short read");
    m->head_W = (float*)r.alloc_read((size_t)m->head_Cout * m->head_Cin * 4);
    m->head_bias = (float*)r.alloc_read((size_t)m->head_Cout * 4);
    if (r.status == BNN_OK && r.off != r.n) r.fail(BNN_ERR_FORMAT, "trailing bytes in blob");
}

int parse(const unsigned char* data, size_t n, Model** out) {
    *out = nullptr;
    Reader r{data, n, 0};
    char magic[4] = {0, 0, 0, 0};
    r.bytes(magic, 4);
    if (r.status == BNN_OK && memcmp(magic, "BNNC", 4) != 0) r.fail(BNN_ERR_FORMAT, "bad magic");
    if (r.status != BNN_OK) return r.status;
    Model* m = (Model*)calloc(1, sizeof(Model));
    if (!m) return set_error(BNN_ERR_OOM, "OOM %zu", sizeof(Model));
    m->version = r.i32(); m->base_channels = r.i32();
    m->n_bands = r.i32(); m->n_classes = r.i32(); m->upsampler = r.i32();
    parse_body(r, m);
    if (r.status != BNN_OK) {
        free_model_arrays(m);
        free(m);
        return r.status;
    }
    Topology t;
    int rc = validate_topology(m, &t);
    if (rc != BNN_OK) {
        free_model_arrays(m);
        free(m);
        return rc;
    }
    m->engine = engine_create();
    if (!m->engine) {
        free_model_arrays(m);
        free(m);
        return set_error(BNN_ERR_OOM, "OOM engine");
    }
    *out = m;
    return BNN_OK;
}

// v2 records are the v1 records under another name
void conv_to_s(const Conv& c, ConvS* s) {
    s->tag = c.tag; s->Cout = c.Cout; s->Cin = c.Cin; s->kh = c.kh; s->kw = c.kw;
    s->pad = c.pad; s->stride = c.stride; s->nwords = c.nwords;
    s->packed = c.packed; s->wsign = c.wsign; s->alpha = c.alpha;
}
void act_to_s(const Act& a, ActS* s) {
    s->kind = a.kind; s->C = a.C;
    s->type = a.type; s->t = a.t; s->lo = a.lo; s->hi = a.hi;
    s->A = a.A; s->B = a.B; s->slope = a.slope; s->rsign = a.rsign;
}

int validate_stem(const Model* body, const Conv* sc, const Act* sa);

// v2 blob (csrc/bnn_model_stem.c:77-115): header with has_stem and
// n_stem_layers, the stem conv + act, then the v1 body sequence. The parsed
// arrays are owned by the StemModel; `body` (its engine handle) is a Model
// whose records alias them.
int parse_stem(const unsigned char* data, size_t n, StemModel** out) {
    *out = nullptr;
    Reader r{data, n, 0};
    char magic[4] = {0, 0, 0, 0};
    r.bytes(magic, 4);
    if (r.status == BNN_OK && memcmp(magic, "BNNC", 4) != 0) r.fail(BNN_ERR_FORMAT, "bad magic");
    if (r.status != BNN_OK) return r.status;
    StemModel* sm = (StemModel*)calloc(1, sizeof(StemModel));
    Model* m = (Model*)calloc(1, sizeof(Model));
    if (!sm || !m) {
        free(sm);
        free(m);
        return set_error(BNN_ERR_OOM, "OOM %zu", sizeof(StemModel) + sizeof(Model));
    }
    m->version = r.i32();
    if (r.status == BNN_OK && m->version != 2) {
        char msg[128];
        snprintf(msg, sizeof msg, "bnn_stem: expected v2 blob, got v%d (use the v1 engine for non-stem models)",
                 m->version);
        r.fail(BNN_ERR_FORMAT, msg);
    }
    m->base_channels = r.i32();
    m->n_bands = r.i32(); m->n_classes = r.i32(); m->upsampler = r.i32();
    const int has_stem = r.i32(), n_stem = r.i32();
    if (r.status == BNN_OK && (has_stem != 1 || n_stem != 1))
        r.fail(BNN_ERR_FORMAT, "bnn_stem: only has_stem=1, n_stem_layers=1 supported");
    Conv sc;
    Act sa;
    memset(&sc, 0, sizeof sc);
    memset(&sa, 0, sizeof sa);
    if (r.status == BNN_OK) read_conv(r, &sc);
    if (r.status == BNN_OK) read_act(r, &sa);
    if (r.status == BNN_OK) parse_body(r, m);
    int rc = r.status;
    if (rc == BNN_OK) rc = validate_stem(m, &sc, &sa);
    if (rc == BNN_OK) {
        m->engine = engine_create_stem(&sc, &sa);
        if (!m->engine) rc = set_error(BNN_ERR_OOM, "OOM engine");
    }
    if (rc != BNN_OK) {
        free_conv(&sc);
        free_act(&sa);
        free_model_arrays(m);
        free(m);
        free(sm);
        return rc;
    }
    sm->version = m->version; sm->base_channels = m->base_channels; sm->n_bands = m->n_bands;
    sm->n_classes = m->n_classes; sm->upsampler = m->upsampler;
    sm->has_stem = has_stem; sm->n_stem_layers = n_stem;
    conv_to_s(sc, &sm->stem_conv);
    act_to_s(sa, &sm->stem_act);
    for (int i = 0; i < 4; ++i) {
        conv_to_s(m->enc_conv1[i], &sm->enc_conv1[i]); conv_to_s(m->enc_conv2[i], &sm->enc_conv2[i]);
        act_to_s(m->enc_act1[i], &sm->enc_act1[i]); act_to_s(m->enc_act2_skip[i], &sm->enc_act2_skip[i]);
        act_to_s(m->enc_act2_down[i], &sm->enc_act2_down[i]);
        conv_to_s(m->dec_conv1[i], &sm->dec_conv1[i]); conv_to_s(m->dec_conv2[i], &sm->dec_conv2[i]);
        act_to_s(m->dec_act1[i], &sm->dec_act1[i]); act_to_s(m->dec_act2[i], &sm->dec_act2[i]);
    }
    conv_to_s(m->bott_conv1, &sm->bott_conv1); conv_to_s(m->bott_conv2, &sm->bott_conv2);
    act_to_s(m->bott_act1, &sm->bott_act1); act_to_s(m->bott_act2, &sm->bott_act2);
    sm->head_Cout = m->head_Cout; sm->head_Cin = m->head_Cin;
    sm->head_W = m->head_W; sm->head_bias = m->head_bias;
    sm->engine = m;
    *out = sm;
    return BNN_OK;
}

int check_conv(const Conv* c, const char* name, int want_tag, int cin) {
    if (c->tag != want_tag)
        return set_error(BNN_ERR_UNSUPPORTED, "%s: conv tag %d, the v1 forward needs %d", name, c->tag, want_tag);
    if (c->kh != 3 || c->kw != 3 || c->pad != 1 || c->stride != 1)
        return set_error(BNN_ERR_UNSUPPORTED, "%s: %dx%d pad %d stride %d, the v1 forward needs 3x3 pad 1 stride 1",
                         name, c->kh, c->kw, c->pad, c->stride);
    if (c->Cin != cin)
        return set_error(BNN_ERR_UNSUPPORTED, "%s: Cin %d, its input has %d channels", name, c->Cin, cin);
    if (c->Cout <= 0 || c->Cin <= 0)
        return set_error(BNN_ERR_UNSUPPORTED, "%s: empty conv (%d -> %d)", name, c->Cin, c->Cout);
    if (want_tag == 1 && c->nwords != (9 * c->Cin + 63) / 64)
        return set_error(BNN_ERR_UNSUPPORTED, "%s: nwords %d != ceil(9*Cin/64) = %d", name, c->nwords,
                         (9 * c->Cin + 63) / 64);
    return BNN_OK;
}

int check_act(const Act* a, const char* name, int want_kind_real, int C) {
    if ((a->kind != 0) != (want_kind_real != 0))
        return set_error(BNN_ERR_UNSUPPORTED, "%s: fold kind %d, the v1 forward needs %s", name, a->kind,
                         want_kind_real ? "a real fold" : "an integer fold (0)");
    if (a->C != C) return set_error(BNN_ERR_UNSUPPORTED, "%s: C %d != conv Cout %d", name, a->C, C);
    return BNN_OK;
}

// the reference's blob writer stores a real conv's weights as np.sign (-1,
// 0, +1; python/bnn2c/blob.py:80-88), for which every x*w of the reference's
// sum is exact; the tensor-core first conv and the stem rely on that
int check_wsign(const Conv* c, const char* name) {
    const size_t n = (size_t)c->Cout * c->Cin * c->kh * c->kw;
    for (size_t i = 0; i < n; ++i)
        if (c->wsign[i] < -1 || c->wsign[i] > 1)
            return set_error(BNN_ERR_UNSUPPORTED, "%s: wsign[%zu] = %d, only -1, 0, +1 are supported", name, i,
                             (int)c->wsign[i]);
    return BNN_OK;
}

// The stem this engine runs: real-input 1x1 pad 0 stride 1 on the bands
// (what python/bnn2c/blob.py writes for the A1b stem) and a real fold; its
// width is the Cin of the binary enc1.conv1.
int validate_stem(const Model* body, const Conv* sc, const Act* sa) {
    if (body->n_bands <= 0 || body->n_bands > 1024)
        return set_error(BNN_ERR_UNSUPPORTED, "n_bands %d outside [1, 1024] (stem tile limit)", body->n_bands);
    if (sc->tag != 2) return set_error(BNN_ERR_UNSUPPORTED, "stem.conv: conv tag %d, the v2 forward needs 2", sc->tag);
    if (sc->kh != 1 || sc->kw != 1 || sc->pad != 0 || sc->stride != 1)
        return set_error(BNN_ERR_UNSUPPORTED, "stem.conv: %dx%d pad %d stride %d, this engine runs a 1x1 pad 0 "
                         "stride 1 stem", sc->kh, sc->kw, sc->pad, sc->stride);
    if (sc->Cin != body->n_bands)
        return set_error(BNN_ERR_UNSUPPORTED, "stem.conv: Cin %d, the input has %d bands", sc->Cin, body->n_bands);
    if (sc->Cout <= 0 || sc->Cout > 256)
        return set_error(BNN_ERR_UNSUPPORTED, "stem.conv: Cout %d outside [1, 256]", sc->Cout);
    int rc = check_wsign(sc, "stem.conv");
    if (rc) return rc;
    if ((rc = check_act(sa, "stem.act", 1, sc->Cout))) return rc;
    Topology t;
    return validate_topology(body, &t, sc->Cout);
}

}  // namespace

// The forward of csrc/bnn_model.c:150-253 assumes: enc1.conv1 real, all
// other convs binary, all 3x3/p1/s1 (output planes are allocated HxW), the
// channel counts chaining as the UNet does, enc1.act1 the only real fold
// (act() passes xreal = NULL everywhere else), and head_Cout == n_classes
// (main.c sizes the logits by n_classes). The v2 body
// (csrc/bnn_model_stem.c:189-255) is the same with enc1.conv1 binary on the
// stem's stem_c channels.
int validate_topology(const Model* m, Topology* t, int stem_c) {
    static const char* EN[4] = {"enc1", "enc2", "enc3", "enc4"};
    static const char* DN[4] = {"dec4", "dec3", "dec2", "dec1"};
    char nm[48];
    int rc;
    if (m->n_bands <= 0 || m->n_classes <= 0)
        return set_error(BNN_ERR_UNSUPPORTED, "n_bands %d / n_classes %d", m->n_bands, m->n_classes);
    if (!stem_c && m->n_bands > 256)
        return set_error(BNN_ERR_UNSUPPORTED, "n_bands %d > 256 (first-conv tile limit)", m->n_bands);
    int cin = stem_c ? stem_c : m->n_bands;
    t->stem = stem_c;
    for (int i = 0; i < 4; ++i) {
        const Conv* c1 = &m->enc_conv1[i];
        const bool real = i == 0 && !stem_c;
        snprintf(nm, sizeof nm, "%s.conv1", EN[i]);
        if ((rc = check_conv(c1, nm, real ? 2 : 1, cin))) return rc;
        if (real && (rc = check_wsign(c1, nm))) return rc;
        snprintf(nm, sizeof nm, "%s.act1", EN[i]);
        if ((rc = check_act(&m->enc_act1[i], nm, real, c1->Cout))) return rc;
        snprintf(nm, sizeof nm, "%s.conv2", EN[i]);
        if ((rc = check_conv(&m->enc_conv2[i], nm, 1, c1->Cout))) return rc;
        int c = m->enc_conv2[i].Cout;
        snprintf(nm, sizeof nm, "%s.act2_skip", EN[i]);
        if ((rc = check_act(&m->enc_act2_skip[i], nm, 0, c))) return rc;
        snprintf(nm, sizeof nm, "%s.act2_down", EN[i]);
        if ((rc = check_act(&m->enc_act2_down[i], nm, 0, c))) return rc;
        t->enc[i] = c;
        cin = c;
    }
    if ((rc = check_conv(&m->bott_conv1, "bottleneck.conv1", 1, cin))) return rc;
    if ((rc = check_act(&m->bott_act1, "bottleneck.act1", 0, m->bott_conv1.Cout))) return rc;
    if ((rc = check_conv(&m->bott_conv2, "bottleneck.conv2", 1, m->bott_conv1.Cout))) return rc;
    if ((rc = check_act(&m->bott_act2, "bottleneck.act2", 0, m->bott_conv2.Cout))) return rc;
    t->bott = m->bott_conv2.Cout;
    int prev = t->bott;
    for (int i = 0; i < 4; ++i) {
        int skip = t->enc[3 - i];
        snprintf(nm, sizeof nm, "%s.conv1", DN[i]);
        if ((rc = check_conv(&m->dec_conv1[i], nm, 1, skip + prev))) return rc;
        snprintf(nm, sizeof nm, "%s.act1", DN[i]);
        if ((rc = check_act(&m->dec_act1[i], nm, 0, m->dec_conv1[i].Cout))) return rc;
        snprintf(nm, sizeof nm, "%s.conv2", DN[i]);
        if ((rc = check_conv(&m->dec_conv2[i], nm, 1, m->dec_conv1[i].Cout))) return rc;
        snprintf(nm, sizeof nm, "%s.act2", DN[i]);
        if ((rc = check_act(&m->dec_act2[i], nm, 0, m->dec_conv2[i].Cout))) return rc;
        prev = m->dec_conv2[i].Cout;
        t->dec[i] = prev;
    }
    if (m->head_Cin != prev)
        return set_error(BNN_ERR_UNSUPPORTED, "head: Cin %d != dec1 width %d", m->head_Cin, prev);
    if (m->head_Cout != m->n_classes)
        return set_error(BNN_ERR_UNSUPPORTED, "head: Cout %d != n_classes %d", m->head_Cout, m->n_classes);
    t->bands = m->n_bands;
    t->classes = m->n_classes;
    return BNN_OK;
}

}  // namespace bnn

using namespace bnn;

BNN_API const char* bnn_last_error(void) { return g_err.c_str(); }

BNN_API int bnn_load_mem(const void* data, size_t n, Model** out) {
    if (!out) return set_error(BNN_ERR_ARG, "out is NULL");
    clear_error();
    return parse((const unsigned char*)data, n, out);
}

BNN_API int bnn_load_ex(const char* path, Model** out) {
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
    return parse((const unsigned char*)buf.data(), buf.size(), out);
}

BNN_API Model* bnn_load(const char* path) {
    Model* m = nullptr;
    if (bnn_load_ex(path, &m) != BNN_OK) {
        fprintf(stderr, "%s\n", bnn_last_error());
        exit(1);
    }
    return m;
}

BNN_API void bnn_free(Model* m) {
    if (!m) return;
    if (engine_stem_c(m->engine) > 0) return;  // the engine handle of a StemModel: bnn_stem_free owns it
    engine_destroy(m->engine);
    free_model_arrays(m);
    free(m);
}

BNN_API int bnn_stem_load_mem(const void* data, size_t n, StemModel** out) {
    if (!out) return set_error(BNN_ERR_ARG, "out is NULL");
    clear_error();
    return parse_stem((const unsigned char*)data, n, out);
}

BNN_API int bnn_stem_load_ex(const char* path, StemModel** out) {
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
    return parse_stem((const unsigned char*)buf.data(), buf.size(), out);
}

BNN_API StemModel* bnn_stem_load(const char* path) {
    StemModel* m = nullptr;
    if (bnn_stem_load_ex(path, &m) != BNN_OK) {
        fprintf(stderr, "%s\n", bnn_last_error());
        exit(1);
    }
    return m;
}

BNN_API Model* bnn_stem_as_model(StemModel* m) { return m ? (Model*)m->engine : nullptr; }

BNN_API void bnn_stem_forward(const StemModel* m, const float* input, int H, int W, float* logits) {
    if (!m) {
        fprintf(stderr, "bnn_stem_forward: NULL model\n");
        exit(1);
    }
    bnn_forward((const Model*)m->engine, input, H, W, logits);
}

BNN_API void bnn_stem_free(StemModel* sm) {
    if (!sm) return;
    Model* m = (Model*)sm->engine;
    if (m) {
        engine_destroy(m->engine);
        free_model_arrays(m);  // the body arrays (aliased by sm's records)
        free(m);
    }
    free(sm->stem_conv.packed); free(sm->stem_conv.wsign); free(sm->stem_conv.alpha);
    ActS* a = &sm->stem_act;
    free(a->type); free(a->t); free(a->lo); free(a->hi);
    free(a->A); free(a->B); free(a->slope); free(a->rsign);
    free(sm);
}
