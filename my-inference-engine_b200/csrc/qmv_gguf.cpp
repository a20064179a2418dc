// GGUF v3 model images behind the C ABI (qmv_gguf_*, declared in
// include/qmv_b200.h): the tensor-directory walk that makes every packed
// tensor of a model resident on the GPU once, and the metadata reads that
// configure the Qwen2 decoder from the same image.
//
// The reference maps the file and parses it in gguf_open
// (src/gguf_reader.cpp:617-786); its callers then re-derive a
// GgufQuantizedTensorView per projection call (src/qwen2_architecture.cpp:
// 585-595).  Here the image (the caller's mapping, or one made by
// qmv_gguf_open_file) is parsed once with the same acceptance rules, so a file
// the reference rejects is rejected here too:
//   header      "GGUF", version 3, 1..1e6 tensors, <= 1e6 metadata entries
//   metadata    typed values (GGUF value types 0..12); arrays of <= 1e6
//               elements nest at most two levels below the entry; a bool
//               byte is 0 or 1
//   alignment   general.alignment when stored as an unsigned integer: a
//               power of two in [8, 4096]; 32 otherwise
//   required    a non-empty general.architecture string
//   tensors     1..4 non-zero dimensions; F32, Q5_0, Q8_0, Q4_K or Q6_K;
//               whole blocks; offsets on the alignment; unique names; data
//               section at the aligned end of the directory; every tensor
//               inside the file
// qmv_gguf_upload then walks the directory and registers each packed 2-D
// tensor in the residency registry keyed by its mapped address, which is the
// address the reference's views point at: a later drop-in
// quantized_tensor_matvec_f32 on such a view finds its weight resident.
// qmv_gguf_close releases the resident copies keyed inside the image, since
// its addresses may be reused by a later mapping.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <limits.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <string>
#include <vector>

#include "qmv_b200.h"
#include "qmv_internal.h"

#define QMV_EXPORT extern "C" __attribute__((visibility("default")))

struct QmvGguf {
    struct Meta {
        std::string key;
        uint32_t type = 0;
        uint64_t value_at = 0;  // file offset of the value
        uint32_t array_type = 0;
        uint64_t array_count = 0;
    };
    struct Tensor {
        std::string name;
        uint32_t n_dims = 0;
        uint64_t dims[4] = {0, 0, 0, 0};
        uint32_t type = 0;
        uint64_t offset = 0;  // from the start of the data section
        uint64_t bytes = 0;
    };
    const unsigned char *data = nullptr;
    uint64_t size = 0;
    void *mapping = nullptr;  // owned mapping (qmv_gguf_open_file)
    uint32_t version = 0;
    uint32_t alignment = 32;
    uint64_t data_offset = 0;
    std::vector<Meta> meta;
    std::vector<Tensor> tensors;
};

namespace {

constexpr uint64_t kMaxEntries = 1000000;  // tensors, metadata entries, array elements
constexpr uint64_t kHeaderBytes = 24;      // magic, version, two counts

// Bounds-checked little-endian reads over the image.
struct Cursor {
    const unsigned char *p;
    uint64_t size;
    uint64_t at;

    bool has(uint64_t n) const { return at <= size && n <= size - at; }
    bool le(int bytes, uint64_t *v)
    {
        if (!has((uint64_t)bytes)) return false;
        uint64_t r = 0;
        for (int i = 0; i < bytes; ++i) r |= (uint64_t)p[at + (uint64_t)i] << (8 * i);
        at += (uint64_t)bytes;
        *v = r;
        return true;
    }
    bool u32(uint32_t *v)
    {
        uint64_t r = 0;
        if (!le(4, &r)) return false;
        *v = (uint32_t)r;
        return true;
    }
    bool u64(uint64_t *v) { return le(8, v); }
    bool text(std::string *s)
    {
        uint64_t n = 0;
        if (!u64(&n) || !has(n)) return false;
        s->assign((const char *)p + at, (size_t)n);
        at += n;
        return true;
    }
};

// Width of a fixed-size GGUF value: u8 i8 u16 i16 u32 i32 f32 bool (0-7),
// u64 i64 f64 (10-12); 0 for string (8), array (9) and unknown types.
int value_width(uint32_t t)
{
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

bool is_unsigned(uint32_t t) { return t == 0 || t == 2 || t == 4 || t == 10; }

// Step over one value of type t at nesting level `level` (0 = the entry's own
// value).  Elements below the second array level are refused.
bool skip_value(Cursor &c, uint32_t t, int level, QmvGguf::Meta *top)
{
    if (level > 2) return false;
    if (t == 8) {
        uint64_t n = 0;
        if (!c.u64(&n) || !c.has(n)) return false;
        c.at += n;
        return true;
    }
    if (t == 9) {
        uint32_t et = 0;
        uint64_t count = 0;
        if (!c.u32(&et) || !c.u64(&count) || count > kMaxEntries) return false;
        if (top != nullptr) {
            top->array_type = et;
            top->array_count = count;
        }
        for (uint64_t i = 0; i < count; ++i)
            if (!skip_value(c, et, level + 1, nullptr)) return false;
        return true;
    }
    const int w = value_width(t);
    if (w == 0 || !c.has((uint64_t)w)) return false;
    if (t == 7 && c.p[c.at] > 1) return false;
    c.at += (uint64_t)w;
    return true;
}

// Elements per block and bytes per block of the tensor types a model may hold.
bool type_blocks(uint32_t t, uint64_t *elems, uint64_t *bytes)
{
    switch (t) {
    case 0: *elems = 1; *bytes = 4; return true;
    case qmv::kQ5_0: *elems = 32; *bytes = 22; return true;
    case qmv::kQ8_0: *elems = 32; *bytes = 34; return true;
    case qmv::kQ4_K: *elems = 256; *bytes = 144; return true;
    case qmv::kQ6_K: *elems = 256; *bytes = 210; return true;
    default: return false;
    }
}

// Element count (no zero dimension, no overflow); false otherwise.
bool element_count(const QmvGguf::Tensor &t, uint64_t *n)
{
    uint64_t e = 1;
    for (uint32_t i = 0; i < t.n_dims; ++i) {
        if (t.dims[i] == 0 || e > UINT64_MAX / t.dims[i]) return false;
        e *= t.dims[i];
    }
    *n = e;
    return true;
}

const QmvGguf::Meta *find_meta(const QmvGguf *g, const char *key)
{
    if (g == nullptr || key == nullptr) return nullptr;
    // C-string comparison, as the reference's (a key holding a NUL byte
    // matches up to it)
    for (const QmvGguf::Meta &m : g->meta)
        if (strcmp(m.key.c_str(), key) == 0) return &m;  // the first entry of that name
    return nullptr;
}

const QmvGguf::Tensor *find_tensor(const QmvGguf *g, const char *name)
{
    if (g == nullptr || name == nullptr) return nullptr;
    for (const QmvGguf::Tensor &t : g->tensors)
        if (strcmp(t.name.c_str(), name) == 0) return &t;
    return nullptr;
}

bool read_uint(const QmvGguf *g, const char *key, uint64_t *v)
{
    const QmvGguf::Meta *m = find_meta(g, key);
    if (m == nullptr || !is_unsigned(m->type)) return false;
    Cursor c{g->data, g->size, m->value_at};
    return c.le(value_width(m->type), v);
}

int parse(QmvGguf *g)
{
    if (g->size < kHeaderBytes) return qmv::set_error("GGUF image is smaller than its header");
    if (memcmp(g->data, "GGUF", 4) != 0) return qmv::set_error("GGUF magic is missing");
    Cursor c{g->data, g->size, 4};
    uint64_t n_tensors = 0, n_meta = 0;
    if (!c.u32(&g->version) || !c.u64(&n_tensors) || !c.u64(&n_meta) || g->version != 3 || n_tensors == 0 ||
        n_tensors > kMaxEntries || n_meta > kMaxEntries)
        return qmv::set_error("GGUF header is malformed or not version 3");
    // entries are appended as they parse: a count the image cannot hold
    // fails at its first missing entry without a large allocation
    for (uint64_t i = 0; i < n_meta; ++i) {
        QmvGguf::Meta m;
        if (!c.text(&m.key) || !c.u32(&m.type)) return qmv::set_error("GGUF metadata section is malformed");
        m.value_at = c.at;
        if (!skip_value(c, m.type, 0, &m)) return qmv::set_error("GGUF metadata section is malformed");
        g->meta.push_back(std::move(m));
    }
    uint64_t align = 0;
    if (read_uint(g, "general.alignment", &align)) {
        if (align < 8 || align > 4096 || (align & (align - 1)) != 0)
            return qmv::set_error("GGUF general.alignment is invalid");
        g->alignment = (uint32_t)align;
    }
    const char *arch = nullptr;
    uint64_t arch_len = 0;
    if (!qmv_gguf_get_string(g, "general.architecture", &arch, &arch_len) || arch_len == 0)
        return qmv::set_error("GGUF general.architecture is missing");
    for (uint64_t i = 0; i < n_tensors; ++i) {
        g->tensors.emplace_back();
        QmvGguf::Tensor &t = g->tensors.back();
        uint64_t elems = 0, be = 0, bb = 0;
        if (!c.text(&t.name) || !c.u32(&t.n_dims) || t.n_dims == 0 || t.n_dims > 4)
            return qmv::set_error("GGUF tensor directory is malformed");
        for (uint32_t d = 0; d < t.n_dims; ++d)
            if (!c.u64(&t.dims[d])) return qmv::set_error("GGUF tensor directory is malformed");
        if (!c.u32(&t.type) || !c.u64(&t.offset)) return qmv::set_error("GGUF tensor directory is malformed");
        if (!type_blocks(t.type, &be, &bb)) return qmv::set_error("GGUF tensor type is not F32, Q5_0, Q8_0, Q4_K or Q6_K");
        if (!element_count(t, &elems) || elems % be != 0 || elems / be > UINT64_MAX / bb)
            return qmv::set_error("GGUF tensor shape does not hold whole blocks");
        t.bytes = elems / be * bb;
        if (t.offset % g->alignment != 0) return qmv::set_error("GGUF tensor offset is not aligned");
    }
    for (size_t i = 0; i < g->tensors.size(); ++i)
        for (size_t j = 0; j < i; ++j)
            if (strcmp(g->tensors[i].name.c_str(), g->tensors[j].name.c_str()) == 0)
                return qmv::set_error("GGUF tensor directory has duplicate names");
    const uint64_t end = c.at;
    if (end > UINT64_MAX - (g->alignment - 1)) return qmv::set_error("GGUF tensor directory size overflows");
    g->data_offset = (end + g->alignment - 1) & ~(uint64_t)(g->alignment - 1);
    if (g->data_offset > g->size) return qmv::set_error("GGUF data section starts past the end of the image");
    const uint64_t room = g->size - g->data_offset;
    for (const QmvGguf::Tensor &t : g->tensors)
        if (t.offset > room || t.bytes > room - t.offset)
            return qmv::set_error("GGUF tensor data extends past the end of the image");
    return 1;
}

void fill_info(const QmvGguf *g, const QmvGguf::Tensor &t, QmvGgufTensor *out)
{
    memset(out, 0, sizeof(*out));
    out->name = t.name.c_str();
    out->ggml_type = t.type;
    out->dimension_count = t.n_dims;
    for (uint32_t d = 0; d < t.n_dims; ++d) out->dimensions[d] = t.dims[d];
    out->offset = t.offset;
    out->byte_size = t.bytes;
    out->data = g->data + g->data_offset + t.offset;
}

}  // namespace

QMV_EXPORT int qmv_gguf_open(const void *data, uint64_t size, QmvGguf **out)
{
    if (out == nullptr) return qmv::set_error("output handle pointer is null");
    *out = nullptr;
    if (data == nullptr) return qmv::set_error("GGUF image is null");
    QmvGguf *g = new QmvGguf();
    g->data = (const unsigned char *)data;
    g->size = size;
    if (!parse(g)) {
        delete g;
        return 0;
    }
    *out = g;
    return 1;
}

QMV_EXPORT int qmv_gguf_open_file(const char *path, QmvGguf **out)
{
    if (out == nullptr) return qmv::set_error("output handle pointer is null");
    *out = nullptr;
    if (path == nullptr || path[0] == '\0') return qmv::set_error("model path is empty");
    const int fd = open(path, O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st) != 0 || st.st_size < (off_t)kHeaderBytes) {
        if (fd >= 0) close(fd);
        return qmv::set_error("could not open the model file, or it is smaller than a GGUF header");
    }
    void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);  // the mapping stays valid
    if (map == MAP_FAILED) return qmv::set_error("could not map the model file");
    QmvGguf *g = new QmvGguf();
    g->data = (const unsigned char *)map;
    g->size = (uint64_t)st.st_size;
    g->mapping = map;
    if (!parse(g)) {
        munmap(map, (size_t)g->size);
        delete g;
        return 0;
    }
    *out = g;
    return 1;
}

QMV_EXPORT int qmv_gguf_close(QmvGguf *g)
{
    if (g == nullptr) return qmv::set_error("null GGUF handle");
    // resident copies keyed by addresses inside the image go with it
    qmv::release_resident_range(g->data, g->data + g->size);
    if (g->mapping != nullptr) munmap(g->mapping, (size_t)g->size);
    delete g;
    return 1;
}

QMV_EXPORT int qmv_gguf_info(const QmvGguf *g, uint64_t *tensor_count, uint64_t *metadata_count,
                             uint64_t *data_offset, uint32_t *alignment)
{
    if (g == nullptr) return qmv::set_error("null GGUF handle");
    if (tensor_count) *tensor_count = g->tensors.size();
    if (metadata_count) *metadata_count = g->meta.size();
    if (data_offset) *data_offset = g->data_offset;
    if (alignment) *alignment = g->alignment;
    return 1;
}

QMV_EXPORT int qmv_gguf_tensor(const QmvGguf *g, uint64_t index, QmvGgufTensor *out)
{
    if (g == nullptr || out == nullptr) return qmv::set_error("null GGUF handle or output");
    if (index >= g->tensors.size()) return qmv::set_error("tensor index out of range");
    fill_info(g, g->tensors[(size_t)index], out);
    return 1;
}

QMV_EXPORT int qmv_gguf_find_tensor(const QmvGguf *g, const char *name, QmvGgufTensor *out)
{
    if (out == nullptr) return qmv::set_error("null output");
    const QmvGguf::Tensor *t = find_tensor(g, name);
    if (t == nullptr) return qmv::set_error("tensor not found");
    fill_info(g, *t, out);
    return 1;
}

QMV_EXPORT int qmv_gguf_get_uint(const QmvGguf *g, const char *key, uint64_t *value)
{
    if (value == nullptr) return 0;
    return read_uint(g, key, value) ? 1 : 0;
}

QMV_EXPORT int qmv_gguf_get_float(const QmvGguf *g, const char *key, double *value)
{
    const QmvGguf::Meta *m = find_meta(g, key);
    if (m == nullptr || value == nullptr || (m->type != 6 && m->type != 12)) return 0;
    Cursor c{g->data, g->size, m->value_at};
    uint64_t bits = 0;
    if (!c.le(m->type == 6 ? 4 : 8, &bits)) return 0;
    double v;
    if (m->type == 6) {
        float f;
        const uint32_t b32 = (uint32_t)bits;
        memcpy(&f, &b32, sizeof(f));
        v = (double)f;
    } else {
        memcpy(&v, &bits, sizeof(v));
    }
    if (!isfinite(v)) return 0;
    *value = v;
    return 1;
}

QMV_EXPORT int qmv_gguf_get_string(const QmvGguf *g, const char *key, const char **value, uint64_t *length)
{
    const QmvGguf::Meta *m = find_meta(g, key);
    if (m == nullptr || value == nullptr || length == nullptr || m->type != 8) return 0;
    Cursor c{g->data, g->size, m->value_at};
    uint64_t n = 0;
    if (!c.u64(&n) || !c.has(n)) return 0;
    *value = (const char *)(g->data + c.at);
    *length = n;
    return 1;
}

QMV_EXPORT int qmv_gguf_get_array_info(const QmvGguf *g, const char *key, uint32_t *element_type,
                                       uint64_t *count)
{
    const QmvGguf::Meta *m = find_meta(g, key);
    if (m == nullptr || element_type == nullptr || count == nullptr || m->type != 9) return 0;
    *element_type = m->array_type;
    *count = m->array_count;
    return 1;
}

// gguf_get_bool (src/gguf_reader.cpp:375-388): a bool entry's byte != 0.
QMV_EXPORT int qmv_gguf_get_bool(const QmvGguf *g, const char *key, int *value)
{
    const QmvGguf::Meta *m = find_meta(g, key);
    if (m == nullptr || value == nullptr || m->type != 7 || m->value_at >= g->size) return 0;
    *value = g->data[m->value_at] != 0;
    return 1;
}

// Sequential reads of one top-level array (gguf_array_cursor_init and the
// next_* readers, src/gguf_reader.cpp:390-489): the cursor sits on the next
// element; each read checks the element type and the image bounds.
QMV_EXPORT int qmv_gguf_array_cursor_init(const QmvGguf *g, const char *key, QmvGgufArrayCursor *cursor)
{
    const QmvGguf::Meta *m = find_meta(g, key);
    if (m == nullptr || cursor == nullptr || m->type != 9) return 0;
    Cursor c{g->data, g->size, m->value_at};
    uint32_t et = 0;
    uint64_t count = 0;
    if (!c.u32(&et) || !c.u64(&count) || et != m->array_type || count != m->array_count) return 0;
    cursor->gguf = g;
    cursor->position = c.at;
    cursor->remaining = count;
    cursor->element_type = et;
    return 1;
}

QMV_EXPORT int qmv_gguf_array_next_string(QmvGgufArrayCursor *cursor, const char **value, uint64_t *length)
{
    if (cursor == nullptr || value == nullptr || length == nullptr || cursor->gguf == nullptr ||
        cursor->remaining == 0 || cursor->element_type != 8)
        return 0;
    Cursor c{cursor->gguf->data, cursor->gguf->size, cursor->position};
    uint64_t n = 0;
    if (!c.u64(&n) || !c.has(n)) return 0;
    *value = (const char *)(c.p + c.at);
    *length = n;
    cursor->position = c.at + n;
    --cursor->remaining;
    return 1;
}

QMV_EXPORT int qmv_gguf_array_next_uint(QmvGgufArrayCursor *cursor, uint64_t *value)
{
    if (cursor == nullptr || value == nullptr || cursor->gguf == nullptr || cursor->remaining == 0 ||
        !is_unsigned(cursor->element_type))
        return 0;
    Cursor c{cursor->gguf->data, cursor->gguf->size, cursor->position};
    uint64_t v = 0;
    if (!c.le(value_width(cursor->element_type), &v)) return 0;
    cursor->position = c.at;
    --cursor->remaining;
    *value = v;
    return 1;
}

QMV_EXPORT int qmv_gguf_array_next_int(QmvGgufArrayCursor *cursor, int64_t *value)
{
    const uint32_t t = cursor ? cursor->element_type : 0u;
    if (cursor == nullptr || value == nullptr || cursor->gguf == nullptr || cursor->remaining == 0 ||
        !(t == 1 || t == 3 || t == 5 || t == 11))
        return 0;
    const int w = value_width(t);
    Cursor c{cursor->gguf->data, cursor->gguf->size, cursor->position};
    uint64_t bits = 0;
    if (!c.le(w, &bits)) return 0;
    if (w < 8 && (bits >> (8 * w - 1)) & 1u) bits |= ~((1ull << (8 * w)) - 1ull);  // sign-extend
    cursor->position = c.at;
    --cursor->remaining;
    *value = (int64_t)bits;
    return 1;
}

// gguf_get_f32_tensor_view (src/gguf_reader.cpp:514-571): F32 tensors only;
// the view is cleared on every failure.
QMV_EXPORT int qmv_gguf_f32_view(const QmvGguf *g, const char *name, QmvGgufF32View *view)
{
    if (view == nullptr) return 0;
    memset(view, 0, sizeof(*view));
    if (g == nullptr || name == nullptr || g->tensors.empty()) return 0;
    const QmvGguf::Tensor *t = find_tensor(g, name);
    uint64_t elems = 0;
    if (t == nullptr || t->type != 0 || t->n_dims == 0 || t->n_dims > 4 || !element_count(*t, &elems)) return 0;
    if (elems > UINT64_MAX / sizeof(float) || t->bytes != elems * sizeof(float)) return 0;
    if (t->offset > g->size - g->data_offset) return 0;
    view->data = (const float *)(g->data + g->data_offset + t->offset);
    view->element_count = elems;
    view->dimension_count = t->n_dims;
    for (uint32_t d = 0; d < t->n_dims; ++d) view->dimensions[d] = t->dims[d];
    return 1;
}

// The reference's gguf_get_quantized_tensor_view (src/gguf_reader.cpp:690-741):
// a cleared view on every failure; packed types only; whole blocks whose
// byte count matches the directory; data inside the image.
QMV_EXPORT int qmv_gguf_quantized_view(const QmvGguf *g, const char *name, GgufQuantizedTensorView *view)
{
    if (view == nullptr) return 0;
    memset(view, 0, sizeof(*view));
    const QmvGguf::Tensor *t = find_tensor(g, name);
    uint64_t be = 0, bb = 0, elems = 0;
    if (t == nullptr || t->type == 0 || !type_blocks(t->type, &be, &bb) || !element_count(*t, &elems) ||
        elems % be != 0)
        return 0;
    const uint64_t blocks = elems / be;
    if (blocks > UINT64_MAX / bb || t->bytes != blocks * bb || g->data_offset > g->size ||
        t->offset > g->size - g->data_offset || t->bytes > g->size - g->data_offset - t->offset)
        return 0;
    view->data = g->data + g->data_offset + t->offset;
    view->ggml_type = t->type;
    view->dimension_count = t->n_dims;
    for (uint32_t d = 0; d < t->n_dims; ++d) view->dimensions[d] = t->dims[d];
    view->element_count = elems;
    view->block_elements = be;
    view->block_bytes = bb;
    view->block_count = blocks;
    return 1;
}

// Every packed 2-D tensor of the image becomes resident on the calling
// thread's device (qmv_resident_weight: one upload and repack per mapped
// address); F32 and packed 1-D tensors stay on the host.
QMV_EXPORT int qmv_gguf_upload(const QmvGguf *g, int *tensors, uint64_t *device_bytes)
{
    if (g == nullptr) return qmv::set_error("null GGUF handle");
    int n = 0;
    uint64_t bytes = 0;
    for (const QmvGguf::Tensor &t : g->tensors) {
        if (t.type == 0 || t.n_dims != 2) continue;
        GgufQuantizedTensorView view;
        if (!qmv_gguf_quantized_view(g, t.name.c_str(), &view))
            return qmv::set_error("GGUF tensor cannot be viewed as packed blocks");
        QmvWeight *w = nullptr;
        if (!qmv_resident_weight(&view, &w)) return 0;
        size_t b = 0;
        if (!qmv_weight_info(w, nullptr, nullptr, nullptr, nullptr, &b)) return 0;
        ++n;
        bytes += b;
    }
    if (tensors) *tensors = n;
    if (device_bytes) *device_bytes = bytes;
    return 1;
}

// The reference's Qwen2 configuration (qwen2_configure_model,
// src/qwen2_architecture.cpp:105-257, with the vocabulary size taken from
// tokenizer.ggml.tokens as engine_load_model does, src/engine.cpp:64-72) and
// its context rule (qwen2_state_init, :286-291: 1 <= max_context <=
// qwen2.context_length); then qmv_qwen2_create on the image's tensors.
QMV_EXPORT int qmv_qwen2_create_from_gguf(const QmvGguf *g, int max_context, QmvQwen2 **out)
{
    if (out == nullptr) return qmv::set_error("output handle pointer is null");
    *out = nullptr;
    if (g == nullptr) return qmv::set_error("null GGUF handle");
    const char *arch = nullptr;
    uint64_t arch_len = 0;
    if (!qmv_gguf_get_string(g, "general.architecture", &arch, &arch_len) || arch_len != 5 ||
        memcmp(arch, "qwen2", 5) != 0)
        return qmv::set_error("GGUF architecture is not qwen2");
    uint32_t tok_type = 0;
    uint64_t vocab = 0;
    if (!qmv_gguf_get_array_info(g, "tokenizer.ggml.tokens", &tok_type, &vocab) || tok_type != 8 || vocab == 0 ||
        vocab > INT_MAX)
        return qmv::set_error("GGUF tokenizer.ggml.tokens metadata is missing or invalid");
    static const char *const kKeys[] = {"qwen2.embedding_length", "qwen2.feed_forward_length", "qwen2.block_count",
                                        "qwen2.attention.head_count", "qwen2.attention.head_count_kv",
                                        "qwen2.context_length"};
    int v[6];
    for (int i = 0; i < 6; ++i) {
        uint64_t u = 0;
        if (!qmv_gguf_get_uint(g, kKeys[i], &u) || u == 0 || u > INT_MAX)
            return qmv::set_error("Qwen2 GGUF metadata is missing or invalid");
        v[i] = (int)u;
    }
    double eps = 0, rope = 0;
    if (!qmv_gguf_get_float(g, "qwen2.attention.layer_norm_rms_epsilon", &eps) ||
        !qmv_gguf_get_float(g, "qwen2.rope.freq_base", &rope))
        return qmv::set_error("Qwen2 normalization or RoPE metadata is missing or invalid");
    const float epsf = (float)eps, ropef = (float)rope;
    if (!(eps > 0.0) || !(rope > 0.0) || !isfinite(epsf) || !(epsf > 0.f) || !isfinite(ropef) || !(ropef > 0.f))
        return qmv::set_error("Qwen2 normalization or RoPE metadata is out of range");
    if (v[0] % v[3] != 0 || v[4] > v[3] || v[3] % v[4] != 0)
        return qmv::set_error("Qwen2 head dimensions in GGUF metadata are inconsistent");
    if (max_context <= 0 || max_context > v[5])
        return qmv::set_error("max_context must be in 1..qwen2.context_length");
    QmvQwen2Config cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.dim = v[0];
    cfg.hidden_dim = v[1];
    cfg.n_layers = v[2];
    cfg.n_heads = v[3];
    cfg.n_kv_heads = v[4];
    cfg.vocab_size = (int)vocab;
    cfg.max_context = max_context;
    cfg.rms_norm_epsilon = epsf;
    cfg.rope_frequency_base = ropef;
    std::vector<QmvQwen2Tensor> list;
    list.reserve(g->tensors.size());
    for (const QmvGguf::Tensor &t : g->tensors) {
        QmvQwen2Tensor q;
        q.name = t.name.c_str();
        q.ggml_type = t.type;
        q.cols = t.dims[0];
        q.rows = t.n_dims == 1 ? 0 : t.dims[1];
        if (t.n_dims > 2) continue;  // not a Qwen2 tensor shape
        q.data = g->data + g->data_offset + t.offset;
        list.push_back(q);
    }
    return qmv_qwen2_create(&cfg, list.data(), (int)list.size(), out);
}
