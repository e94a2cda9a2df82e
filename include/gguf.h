/* gguf.h — GGUF v2/v3 container reader (host side, mmap, zero-copy).
 *
 * Same entry points, types and error behaviour as the reference's GGUF parser
 * (src/gguf.h:131-155 of Fiber-Inference): functions return NULL / defaults on
 * failure and print a one-line reason to stderr. The implementation
 * (fiber-inference_b200/host/gguf.c) is written independently and additionally
 * validates every offset against the file size, so a truncated or corrupted
 * file is rejected instead of read out of bounds.
 *
 * The enum values below are fixed by the GGUF file format (they are written
 * into files), so they are identical to the reference's (src/gguf.h:15-62).
 */
#ifndef FIBER_GGUF_H
#define FIBER_GGUF_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGUF_MAGIC 0x46554747u /* "GGUF" read as a little-endian uint32 */

typedef enum {
    GGUF_TYPE_UINT8 = 0,
    GGUF_TYPE_INT8 = 1,
    GGUF_TYPE_UINT16 = 2,
    GGUF_TYPE_INT16 = 3,
    GGUF_TYPE_UINT32 = 4,
    GGUF_TYPE_INT32 = 5,
    GGUF_TYPE_FLOAT32 = 6,
    GGUF_TYPE_BOOL = 7,
    GGUF_TYPE_STRING = 8,
    GGUF_TYPE_ARRAY = 9,
    GGUF_TYPE_UINT64 = 10,
    GGUF_TYPE_INT64 = 11,
    GGUF_TYPE_FLOAT64 = 12,
} gguf_type_t;

typedef enum {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6,
    GGML_TYPE_Q5_1 = 7,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_Q8_1 = 9,
    GGML_TYPE_Q2_K = 10,
    GGML_TYPE_Q3_K = 11,
    GGML_TYPE_Q4_K = 12,
    GGML_TYPE_Q5_K = 13,
    GGML_TYPE_Q6_K = 14,
    GGML_TYPE_Q8_K = 15,
    GGML_TYPE_IQ2_XXS = 16,
    GGML_TYPE_IQ2_XS = 17,
    GGML_TYPE_IQ3_XXS = 18,
    GGML_TYPE_IQ1_S = 19,
    GGML_TYPE_IQ4_NL = 20,
    GGML_TYPE_IQ3_S = 21,
    GGML_TYPE_IQ2_S = 22,
    GGML_TYPE_IQ4_XS = 23,
    GGML_TYPE_I8 = 24,
    GGML_TYPE_I16 = 25,
    GGML_TYPE_I32 = 26,
    GGML_TYPE_I64 = 27,
    GGML_TYPE_F64 = 28,
    GGML_TYPE_IQ1_M = 29,
    GGML_TYPE_BF16 = 30,
} ggml_type_t;

/* Length-prefixed string inside the mapping (not NUL-terminated). */
typedef struct {
    uint64_t len;
    const char *str;
} gguf_string_t;

/* One metadata key/value. Scalars are decoded; arrays point into the mapping. */
typedef struct {
    gguf_string_t key;
    gguf_type_t type;
    union {
        uint8_t u8;
        int8_t i8;
        uint16_t u16;
        int16_t i16;
        uint32_t u32;
        int32_t i32;
        float f32;
        bool b;
        uint64_t u64;
        int64_t i64;
        double f64;
        gguf_string_t str;
        struct {
            gguf_type_t elem_type;
            uint64_t count;
            const void *data;
        } arr;
    } value;
} gguf_kv_t;

/* Tensor index entry. dims[0] is the innermost (row length) dimension. */
typedef struct {
    gguf_string_t name;
    uint32_t n_dims;
    uint64_t dims[4];
    ggml_type_t type;
    uint64_t offset;   /* relative to the data section */
    size_t size_bytes; /* computed from dims and the type table */
    uint64_t n_elements;
} gguf_tensor_info_t;

typedef struct {
    int fd;
    void *data; /* mmap base */
    size_t file_size;
    uint32_t version;
    uint64_t n_tensors;
    uint64_t n_kv;
    gguf_kv_t *kv;
    gguf_tensor_info_t *tensors;
    size_t data_offset; /* absolute file offset of the tensor data section */
    /* NUL-terminated copies of string-valued KVs, indexed like kv[] (NULL for
     * non-strings); gguf_get_str returns these, valid until gguf_close. */
    char **kv_cstr;
} gguf_file_t;

gguf_file_t *gguf_open(const char *path);
void gguf_close(gguf_file_t *gf);
const void *gguf_tensor_data(const gguf_file_t *gf, const gguf_tensor_info_t *ti);
const gguf_tensor_info_t *gguf_find_tensor(const gguf_file_t *gf, const char *name);
const gguf_kv_t *gguf_find_kv(const gguf_file_t *gf, const char *key);
uint32_t gguf_get_u32(const gguf_file_t *gf, const char *key, uint32_t default_val);
uint64_t gguf_get_u64(const gguf_file_t *gf, const char *key, uint64_t default_val);
float gguf_get_f32(const gguf_file_t *gf, const char *key, float default_val);
const char *gguf_get_str(const gguf_file_t *gf, const char *key);

size_t ggml_type_size(ggml_type_t type);  /* bytes per block */
size_t ggml_block_size(ggml_type_t type); /* elements per block */
const char *ggml_type_name(ggml_type_t type);
const char *gguf_type_name(gguf_type_t type);

#ifdef __cplusplus
}
#endif
#endif /* FIBER_GGUF_H */
