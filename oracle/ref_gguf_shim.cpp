// TEST INFRASTRUCTURE ONLY — compiled by oracle/Makefile together with the
// reference engine's own src/gguf_reader.cpp (read in place from the
// reference checkout) into oracle/_ref/.  It exposes the reference's GGUF
// reader (gguf_open and its metadata / view accessors, src/gguf_reader.h:
// 71-142) through plain C entry points so the tests can parse the same image
// with the reference and with the product's qmv_gguf_* and compare.  Nothing
// in the product links this file.
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "gguf_reader.h"

extern "C" {

// Opens `path` with the reference's gguf_open; null on rejection, with the
// reference's message in `error`.
void *ref_gguf_open(const char *path, char *error, int capacity)
{
    GgufFile *f = (GgufFile *)calloc(1, sizeof(GgufFile));
    if (f == nullptr) return nullptr;
    if (!gguf_open(path, f, error, capacity)) {
        free(f);
        return nullptr;
    }
    return f;
}

void ref_gguf_close(void *h)
{
    if (h == nullptr) return;
    gguf_close((GgufFile *)h);
    free(h);
}

int ref_gguf_info(void *h, uint64_t *tensor_count, uint64_t *metadata_count, uint64_t *data_offset,
                  uint32_t *alignment)
{
    const GgufFile *f = (const GgufFile *)h;
    *tensor_count = f->tensor_count;
    *metadata_count = f->metadata_count;
    *data_offset = f->tensor_data_offset;
    *alignment = f->alignment;
    return 1;
}

int ref_gguf_tensor(void *h, uint64_t index, const char **name, uint32_t *type, uint32_t *dimension_count,
                    uint64_t *dimensions, uint64_t *offset, uint64_t *byte_size)
{
    const GgufFile *f = (const GgufFile *)h;
    if (index >= f->tensor_count) return 0;
    const GgufTensorInfo *t = &f->tensors[index];
    *name = t->name;
    *type = t->type;
    *dimension_count = t->dimension_count;
    for (int i = 0; i < 4; ++i) dimensions[i] = t->dimensions[i];
    *offset = t->offset;
    *byte_size = t->byte_size;
    return 1;
}

int ref_gguf_get_uint(void *h, const char *key, uint64_t *value) { return gguf_get_uint((GgufFile *)h, key, value); }

int ref_gguf_get_float(void *h, const char *key, double *value) { return gguf_get_float((GgufFile *)h, key, value); }

int ref_gguf_get_string(void *h, const char *key, const char **value, uint64_t *length)
{
    return gguf_get_string((GgufFile *)h, key, value, length);
}

int ref_gguf_get_array_info(void *h, const char *key, uint32_t *element_type, uint64_t *count)
{
    return gguf_get_array_info((GgufFile *)h, key, element_type, count);
}

// View offsets are returned relative to the mapped image, since the two
// parsers map the file at different addresses.
int ref_gguf_quantized_view(void *h, const char *name, GgufQuantizedTensorView *view, uint64_t *data_at)
{
    const GgufFile *f = (const GgufFile *)h;
    const int ok = gguf_get_quantized_tensor_view(f, name, view);
    *data_at = ok ? (uint64_t)(view->data - f->data) : 0;
    return ok;
}

int ref_gguf_get_bool(void *h, const char *key, int *value) { return gguf_get_bool((GgufFile *)h, key, value); }

// Every element of a top-level array through the reference's cursor readers:
// kind 0 strings (each as length then bytes into `bytes`), 1 unsigned, 2
// signed (into `ints`).  Returns the elements read before the first failure
// (-1 when the cursor does not open).
int ref_gguf_array_read(void *h, const char *key, int kind, int max, uint64_t *ints, uint8_t *bytes,
                        uint64_t bytes_cap, uint64_t *bytes_used)
{
    GgufArrayCursor cur;
    if (!gguf_array_cursor_init((GgufFile *)h, key, &cur)) return -1;
    int n = 0;
    uint64_t used = 0;
    for (; n < max; ++n) {
        if (kind == 0) {
            const char *v = nullptr;
            uint64_t len = 0;
            if (!gguf_array_next_string(&cur, &v, &len) || used + 8 + len > bytes_cap) break;
            memcpy(bytes + used, &len, 8);
            memcpy(bytes + used + 8, v, (size_t)len);
            used += 8 + len;
        } else if (kind == 1) {
            if (!gguf_array_next_uint(&cur, &ints[n])) break;
        } else {
            int64_t v = 0;
            if (!gguf_array_next_int(&cur, &v)) break;
            ints[n] = (uint64_t)v;
        }
    }
    *bytes_used = used;
    return n;
}

// The reference's F32 view, its data as an offset into the mapped image.
int ref_gguf_f32_view(void *h, const char *name, GgufF32TensorView *view, uint64_t *data_at)
{
    const GgufFile *f = (const GgufFile *)h;
    const int ok = gguf_get_f32_tensor_view(f, name, view);
    *data_at = ok ? (uint64_t)((const unsigned char *)view->data - f->data) : 0;
    return ok;
}

}  // extern "C"
