/* gguf.c — GGUF v2/v3 reader: mmap the file, decode the KV metadata and the
 * tensor index, leave tensor bytes in the mapping.
 *
 * Behaviour follows the reference parser (src/gguf.c:216-325): version 2 or 3,
 * at most 4 dims per tensor, data section aligned to `general.alignment`
 * (default 32), tensor lookup by exact name. Unlike the reference, every read is
 * bounds-checked through a cursor with a sticky error flag, counts are checked
 * against the bytes left before anything is allocated, and each tensor's
 * [offset, offset+size) must lie inside the file: a truncated or corrupted file
 * returns NULL rather than reading past the mapping.
 */
#include "gguf.h"

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* Block geometry of each ggml type: {bytes per block, elements per block}.
 * These are properties of the on-disk formats (the same numbers as the
 * reference's table, src/gguf.c:21-51). */
static int type_geometry(ggml_type_t t, size_t *bytes, size_t *elems) {
    size_t b = 0, e = 0;
    switch (t) {
    case GGML_TYPE_F32: b = 4; e = 1; break;
    case GGML_TYPE_F16: b = 2; e = 1; break;
    case GGML_TYPE_BF16: b = 2; e = 1; break;
    case GGML_TYPE_I8: b = 1; e = 1; break;
    case GGML_TYPE_I16: b = 2; e = 1; break;
    case GGML_TYPE_I32: b = 4; e = 1; break;
    case GGML_TYPE_I64: b = 8; e = 1; break;
    case GGML_TYPE_F64: b = 8; e = 1; break;
    case GGML_TYPE_Q4_0: b = 18; e = 32; break;
    case GGML_TYPE_Q4_1: b = 20; e = 32; break;
    case GGML_TYPE_Q5_0: b = 22; e = 32; break;
    case GGML_TYPE_Q5_1: b = 24; e = 32; break;
    case GGML_TYPE_Q8_0: b = 34; e = 32; break;
    case GGML_TYPE_Q8_1: b = 36; e = 32; break;
    case GGML_TYPE_IQ4_NL: b = 18; e = 32; break;
    case GGML_TYPE_IQ4_XS: b = 36; e = 32; break;
    case GGML_TYPE_Q2_K: b = 84; e = 256; break;
    case GGML_TYPE_Q3_K: b = 110; e = 256; break;
    case GGML_TYPE_Q4_K: b = 144; e = 256; break;
    case GGML_TYPE_Q5_K: b = 176; e = 256; break;
    case GGML_TYPE_Q6_K: b = 210; e = 256; break;
    case GGML_TYPE_Q8_K: b = 292; e = 256; break;
    case GGML_TYPE_IQ2_XXS: b = 66; e = 256; break;
    case GGML_TYPE_IQ2_XS: b = 74; e = 256; break;
    case GGML_TYPE_IQ3_XXS: b = 98; e = 256; break;
    case GGML_TYPE_IQ1_S: b = 50; e = 256; break;
    case GGML_TYPE_IQ3_S: b = 110; e = 256; break;
    case GGML_TYPE_IQ2_S: b = 82; e = 256; break;
    case GGML_TYPE_IQ1_M: b = 56; e = 256; break;
    default: return 0;
    }
    if (bytes) *bytes = b;
    if (elems) *elems = e;
    return 1;
}

size_t ggml_type_size(ggml_type_t type) {
    size_t b = 0;
    return type_geometry(type, &b, NULL) ? b : 0;
}

size_t ggml_block_size(ggml_type_t type) {
    size_t e = 0;
    return type_geometry(type, NULL, &e) ? e : 0;
}

const char *ggml_type_name(ggml_type_t type) {
    switch (type) {
    case GGML_TYPE_F32: return "F32";
    case GGML_TYPE_F16: return "F16";
    case GGML_TYPE_Q4_0: return "Q4_0";
    case GGML_TYPE_Q4_1: return "Q4_1";
    case GGML_TYPE_Q5_0: return "Q5_0";
    case GGML_TYPE_Q5_1: return "Q5_1";
    case GGML_TYPE_Q8_0: return "Q8_0";
    case GGML_TYPE_Q8_1: return "Q8_1";
    case GGML_TYPE_Q2_K: return "Q2_K";
    case GGML_TYPE_Q3_K: return "Q3_K";
    case GGML_TYPE_Q4_K: return "Q4_K";
    case GGML_TYPE_Q5_K: return "Q5_K";
    case GGML_TYPE_Q6_K: return "Q6_K";
    case GGML_TYPE_Q8_K: return "Q8_K";
    case GGML_TYPE_IQ2_XXS: return "IQ2_XXS";
    case GGML_TYPE_IQ2_XS: return "IQ2_XS";
    case GGML_TYPE_IQ3_XXS: return "IQ3_XXS";
    case GGML_TYPE_IQ1_S: return "IQ1_S";
    case GGML_TYPE_IQ4_NL: return "IQ4_NL";
    case GGML_TYPE_IQ3_S: return "IQ3_S";
    case GGML_TYPE_IQ2_S: return "IQ2_S";
    case GGML_TYPE_IQ4_XS: return "IQ4_XS";
    case GGML_TYPE_I8: return "I8";
    case GGML_TYPE_I16: return "I16";
    case GGML_TYPE_I32: return "I32";
    case GGML_TYPE_I64: return "I64";
    case GGML_TYPE_F64: return "F64";
    case GGML_TYPE_IQ1_M: return "IQ1_M";
    case GGML_TYPE_BF16: return "BF16";
    default: return "UNKNOWN";
    }
}

const char *gguf_type_name(gguf_type_t type) {
    static const char *const names[] = {"UINT8", "INT8", "UINT16", "INT16", "UINT32",
                                        "INT32", "FLOAT32", "BOOL", "STRING", "ARRAY",
                                        "UINT64", "INT64", "FLOAT64"};
    if ((unsigned)type < sizeof(names) / sizeof(names[0])) return names[type];
    return "UNKNOWN";
}

/* ---- bounds-checked cursor ------------------------------------------------ */

typedef struct {
    const uint8_t *base;
    size_t size;
    size_t pos;
    int bad; /* sticky: set on the first read past the end */
} cursor_t;

static int cur_take(cursor_t *c, void *dst, size_t n) {
    if (c->bad || n > c->size - c->pos) {
        c->bad = 1;
        if (dst) memset(dst, 0, n);
        return 0;
    }
    if (dst) memcpy(dst, c->base + c->pos, n);
    c->pos += n;
    return 1;
}

static uint32_t cur_u32(cursor_t *c) {
    uint32_t v;
    cur_take(c, &v, 4);
    return v;
}

static uint64_t cur_u64(cursor_t *c) {
    uint64_t v;
    cur_take(c, &v, 8);
    return v;
}

static gguf_string_t cur_str(cursor_t *c) {
    gguf_string_t s = {0, NULL};
    uint64_t n = cur_u64(c);
    if (c->bad || n > c->size - c->pos) {
        c->bad = 1;
        return s;
    }
    s.len = n;
    s.str = (const char *)(c->base + c->pos);
    c->pos += (size_t)n;
    return s;
}

static size_t scalar_width(gguf_type_t t) {
    switch (t) {
    case GGUF_TYPE_UINT8:
    case GGUF_TYPE_INT8:
    case GGUF_TYPE_BOOL: return 1;
    case GGUF_TYPE_UINT16:
    case GGUF_TYPE_INT16: return 2;
    case GGUF_TYPE_UINT32:
    case GGUF_TYPE_INT32:
    case GGUF_TYPE_FLOAT32: return 4;
    case GGUF_TYPE_UINT64:
    case GGUF_TYPE_INT64:
    case GGUF_TYPE_FLOAT64: return 8;
    default: return 0;
    }
}

static int decode_value(cursor_t *c, gguf_kv_t *kv) {
    switch (kv->type) {
    case GGUF_TYPE_UINT8: cur_take(c, &kv->value.u8, 1); break;
    case GGUF_TYPE_INT8: cur_take(c, &kv->value.i8, 1); break;
    case GGUF_TYPE_UINT16: cur_take(c, &kv->value.u16, 2); break;
    case GGUF_TYPE_INT16: cur_take(c, &kv->value.i16, 2); break;
    case GGUF_TYPE_UINT32: cur_take(c, &kv->value.u32, 4); break;
    case GGUF_TYPE_INT32: cur_take(c, &kv->value.i32, 4); break;
    case GGUF_TYPE_FLOAT32: cur_take(c, &kv->value.f32, 4); break;
    case GGUF_TYPE_UINT64: cur_take(c, &kv->value.u64, 8); break;
    case GGUF_TYPE_INT64: cur_take(c, &kv->value.i64, 8); break;
    case GGUF_TYPE_FLOAT64: cur_take(c, &kv->value.f64, 8); break;
    case GGUF_TYPE_BOOL: {
        uint8_t b = 0;
        cur_take(c, &b, 1);
        kv->value.b = b != 0;
        break;
    }
    case GGUF_TYPE_STRING: kv->value.str = cur_str(c); break;
    case GGUF_TYPE_ARRAY: {
        gguf_type_t et = (gguf_type_t)cur_u32(c);
        uint64_t count = cur_u64(c);
        kv->value.arr.elem_type = et;
        kv->value.arr.count = count;
        kv->value.arr.data = c->base + c->pos;
        if (et == GGUF_TYPE_STRING) {
            /* every string carries at least its 8-byte length */
            if (count > (c->size - c->pos) / 8) {
                c->bad = 1;
                break;
            }
            for (uint64_t i = 0; i < count && !c->bad; i++) cur_str(c);
        } else {
            size_t w = scalar_width(et);
            if (w == 0 || count > (c->size - c->pos) / w) {
                c->bad = 1;
                break;
            }
            c->pos += (size_t)(count * w);
        }
        break;
    }
    default:
        fprintf(stderr, "gguf: unknown KV type %d\n", (int)kv->type);
        return 0;
    }
    return !c->bad;
}

/* ---- public API ------------------------------------------------------------ */

void gguf_close(gguf_file_t *gf) {
    if (!gf) return;
    if (gf->kv_cstr) {
        for (uint64_t i = 0; i < gf->n_kv; i++) free(gf->kv_cstr[i]);
        free(gf->kv_cstr);
    }
    if (gf->data && gf->data != MAP_FAILED) munmap(gf->data, gf->file_size);
    if (gf->fd >= 0) close(gf->fd);
    free(gf->kv);
    free(gf->tensors);
    free(gf);
}

gguf_file_t *gguf_open(const char *path) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        perror("gguf: open");
        return NULL;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        perror("gguf: fstat");
        close(fd);
        return NULL;
    }
    size_t fsize = (size_t)st.st_size;
    if (fsize < 24) {
        fprintf(stderr, "gguf: file too small (%zu bytes)\n", fsize);
        close(fd);
        return NULL;
    }
    void *map = mmap(NULL, fsize, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
        perror("gguf: mmap");
        close(fd);
        return NULL;
    }

    gguf_file_t *gf = (gguf_file_t *)calloc(1, sizeof(*gf));
    if (!gf) {
        munmap(map, fsize);
        close(fd);
        return NULL;
    }
    gf->fd = fd;
    gf->data = map;
    gf->file_size = fsize;

    cursor_t c = {(const uint8_t *)map, fsize, 0, 0};
    uint32_t magic = cur_u32(&c);
    if (magic != GGUF_MAGIC) {
        fprintf(stderr, "gguf: bad magic 0x%08x (expected 0x%08x)\n", magic, GGUF_MAGIC);
        gguf_close(gf);
        return NULL;
    }
    gf->version = cur_u32(&c);
    gf->n_tensors = cur_u64(&c);
    gf->n_kv = cur_u64(&c);
    if (gf->version < 2 || gf->version > 3) {
        fprintf(stderr, "gguf: unsupported version %u (need 2 or 3)\n", gf->version);
        gguf_close(gf);
        return NULL;
    }
    /* Each KV needs >= 12 header bytes and each tensor >= 24: reject counts that
     * cannot fit before allocating for them. */
    if (gf->n_kv > fsize / 12 || gf->n_tensors > fsize / 24) {
        fprintf(stderr, "gguf: implausible counts (kv=%llu tensors=%llu)\n",
                (unsigned long long)gf->n_kv, (unsigned long long)gf->n_tensors);
        gf->n_kv = 0;
        gguf_close(gf);
        return NULL;
    }

    gf->kv = (gguf_kv_t *)calloc(gf->n_kv ? gf->n_kv : 1, sizeof(gguf_kv_t));
    gf->kv_cstr = (char **)calloc(gf->n_kv ? gf->n_kv : 1, sizeof(char *));
    if (!gf->kv || !gf->kv_cstr) {
        gguf_close(gf);
        return NULL;
    }
    for (uint64_t i = 0; i < gf->n_kv; i++) {
        gguf_kv_t *kv = &gf->kv[i];
        kv->key = cur_str(&c);
        kv->type = (gguf_type_t)cur_u32(&c);
        if (c.bad || !decode_value(&c, kv)) {
            fprintf(stderr, "gguf: error parsing KV %llu\n", (unsigned long long)i);
            gguf_close(gf);
            return NULL;
        }
        if (kv->type == GGUF_TYPE_STRING) {
            char *s = (char *)malloc((size_t)kv->value.str.len + 1);
            if (!s) {
                gguf_close(gf);
                return NULL;
            }
            memcpy(s, kv->value.str.str, (size_t)kv->value.str.len);
            s[kv->value.str.len] = '\0';
            gf->kv_cstr[i] = s;
        }
    }

    gf->tensors = (gguf_tensor_info_t *)calloc(gf->n_tensors ? gf->n_tensors : 1,
                                               sizeof(gguf_tensor_info_t));
    if (!gf->tensors) {
        gguf_close(gf);
        return NULL;
    }
    for (uint64_t i = 0; i < gf->n_tensors; i++) {
        gguf_tensor_info_t *ti = &gf->tensors[i];
        ti->name = cur_str(&c);
        ti->n_dims = cur_u32(&c);
        if (c.bad) break;
        if (ti->n_dims > 4) {
            fprintf(stderr, "gguf: tensor %llu has %u dims (max 4)\n",
                    (unsigned long long)i, ti->n_dims);
            gguf_close(gf);
            return NULL;
        }
        uint64_t ne = 1;
        for (uint32_t d = 0; d < 4; d++) {
            ti->dims[d] = d < ti->n_dims ? cur_u64(&c) : 1;
            if (ti->dims[d] && ne > UINT64_MAX / ti->dims[d]) c.bad = 1;
            ne *= ti->dims[d];
        }
        ti->n_elements = ne;
        ti->type = (ggml_type_t)cur_u32(&c);
        ti->offset = cur_u64(&c);
        size_t bb = 0, be = 0;
        if (type_geometry(ti->type, &bb, &be) && be > 0)
            ti->size_bytes = (size_t)((ne / be) * bb);
        else
            ti->size_bytes = 0;
    }
    if (c.bad) {
        fprintf(stderr, "gguf: truncated header\n");
        gguf_close(gf);
        return NULL;
    }

    size_t align = 32;
    const gguf_kv_t *akv = gguf_find_kv(gf, "general.alignment");
    if (akv && akv->type == GGUF_TYPE_UINT32) align = akv->value.u32;
    if (align == 0 || (align & (align - 1)) != 0) {
        fprintf(stderr, "gguf: bad general.alignment %zu\n", align);
        gguf_close(gf);
        return NULL;
    }
    gf->data_offset = (c.pos + align - 1) & ~(align - 1);
    if (gf->data_offset > fsize) {
        fprintf(stderr, "gguf: data section starts past end of file\n");
        gguf_close(gf);
        return NULL;
    }
    size_t data_bytes = fsize - gf->data_offset;
    for (uint64_t i = 0; i < gf->n_tensors; i++) {
        const gguf_tensor_info_t *ti = &gf->tensors[i];
        if (ti->offset > data_bytes || ti->size_bytes > data_bytes - ti->offset) {
            fprintf(stderr, "gguf: tensor %.*s [%llu, +%zu) outside data section (%zu bytes)\n",
                    (int)ti->name.len, ti->name.str, (unsigned long long)ti->offset,
                    ti->size_bytes, data_bytes);
            gguf_close(gf);
            return NULL;
        }
    }
    madvise(map, fsize, MADV_RANDOM);
    return gf;
}

const void *gguf_tensor_data(const gguf_file_t *gf, const gguf_tensor_info_t *ti) {
    return (const uint8_t *)gf->data + gf->data_offset + ti->offset;
}

static int name_eq(gguf_string_t s, const char *name, size_t n) {
    return s.len == n && memcmp(s.str, name, n) == 0;
}

const gguf_tensor_info_t *gguf_find_tensor(const gguf_file_t *gf, const char *name) {
    size_t n = strlen(name);
    for (uint64_t i = 0; i < gf->n_tensors; i++)
        if (name_eq(gf->tensors[i].name, name, n)) return &gf->tensors[i];
    return NULL;
}

const gguf_kv_t *gguf_find_kv(const gguf_file_t *gf, const char *key) {
    size_t n = strlen(key);
    for (uint64_t i = 0; i < gf->n_kv; i++)
        if (name_eq(gf->kv[i].key, key, n)) return &gf->kv[i];
    return NULL;
}

uint32_t gguf_get_u32(const gguf_file_t *gf, const char *key, uint32_t default_val) {
    const gguf_kv_t *kv = gguf_find_kv(gf, key);
    if (!kv) return default_val;
    if (kv->type == GGUF_TYPE_UINT32) return kv->value.u32;
    if (kv->type == GGUF_TYPE_INT32) return (uint32_t)kv->value.i32;
    return default_val;
}

uint64_t gguf_get_u64(const gguf_file_t *gf, const char *key, uint64_t default_val) {
    const gguf_kv_t *kv = gguf_find_kv(gf, key);
    if (!kv) return default_val;
    if (kv->type == GGUF_TYPE_UINT64) return kv->value.u64;
    if (kv->type == GGUF_TYPE_UINT32) return kv->value.u32;
    return default_val;
}

float gguf_get_f32(const gguf_file_t *gf, const char *key, float default_val) {
    const gguf_kv_t *kv = gguf_find_kv(gf, key);
    if (!kv || kv->type != GGUF_TYPE_FLOAT32) return default_val;
    return kv->value.f32;
}

const char *gguf_get_str(const gguf_file_t *gf, const char *key) {
    const gguf_kv_t *kv = gguf_find_kv(gf, key);
    if (!kv || kv->type != GGUF_TYPE_STRING) return NULL;
    return gf->kv_cstr[kv - gf->kv];
}
