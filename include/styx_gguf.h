/*
 * styx_gguf.h -- the GGUF container reader of the model loader, part of
 * libstyx_moe.so.
 *
 * Gguf::open (crates/gguf-rs/src/lib.rs:41-120): the header, the metadata
 * key/values, the tensor infos and the aligned start of the tensor data,
 * with the same checks, limits and messages:
 *
 *   magic 0x46554747                       else STYX_EDATA "Invalid GGUF magic"
 *   version 2 or 3                         else STYX_EDATA "Unsupported GGUF version"
 *   string length <= 2^24                  else STYX_EDATA "String too long"
 *   strings valid UTF-8                    else STYX_EDATA "Invalid UTF-8: ..."
 *   value types 0-12                       else STYX_EDATA "Unknown value type: N"
 *   array length <= 2^28                   else STYX_EDATA "Array too long"
 *   known ggml type (compute_size_bytes)   else STYX_EDATA "Unknown ggml_type: N"
 *   element count a multiple of the block  else STYX_EDATA "First dimension not
 *                                              multiple of block size"
 *   any field cut short by the end of file: STYX_EEOF (the reader's
 *   UnexpectedEof, "failed to fill whole buffer").
 *
 * data_start = the position after the tensor infos rounded up to
 * general.alignment (only when that key is a u32, else 32), with the
 * reference's round-up formula.  A later duplicate metadata key replaces the
 * earlier value (HashMap insert).  The file is memory-mapped, so
 * styx_gguf_tensor_data returns the tensor's bytes in place (the MmapFile
 * view of MoeModel::load, crates/model/src/moe.rs:593-599); unlike the
 * reference, which indexes the mapping without a check, it refuses a tensor
 * whose bytes do not lie inside the file.
 *
 * Every function returns STYX_OK (0) or a negative code and leaves a message
 * for styx_last_error().  Strings and arrays returned by the accessors stay
 * valid until styx_gguf_close.
 */
#ifndef STYX_GGUF_H
#define STYX_GGUF_H

#include <stddef.h>
#include <stdint.h>

#include "styx_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

#define STYX_EIO (-6)         /* the file could not be opened, sized or mapped */
#define STYX_EEOF (-7)        /* a field runs past the end of the file */
#define STYX_EDATA (-8)       /* invalid content (the reference's InvalidData) */

/* metadata value types (read_value, lib.rs:155-176) */
typedef enum {
    STYX_GGUF_U8 = 0,
    STYX_GGUF_I8 = 1,
    STYX_GGUF_U16 = 2,
    STYX_GGUF_I16 = 3,
    STYX_GGUF_U32 = 4,
    STYX_GGUF_I32 = 5,
    STYX_GGUF_F32 = 6,
    STYX_GGUF_BOOL = 7,
    STYX_GGUF_STRING = 8,
    STYX_GGUF_ARRAY = 9,
    STYX_GGUF_U64 = 10,
    STYX_GGUF_I64 = 11,
    STYX_GGUF_F64 = 12
} styx_gguf_vtype;

typedef struct styx_gguf styx_gguf;

/* TensorInfo (lib.rs:23-30) */
typedef struct {
    const char *name;      /* NUL-terminated */
    uint32_t n_dims;
    const uint64_t *dims;  /* n_dims entries, innermost first (GGUF order) */
    uint32_t ggml_type;
    uint64_t offset;       /* from data_start */
    uint64_t size_bytes;   /* compute_size_bytes(dims, ggml_type) */
} styx_gguf_tensor_info;

/* Gguf::open (lib.rs:41-120) on a file, mapped read-only. */
int styx_gguf_open(const char *path, styx_gguf **out);
/* The same parse over `bytes` bytes at `data`, which the caller keeps alive
 * and unchanged until styx_gguf_close. */
int styx_gguf_open_memory(const void *data, uint64_t bytes, styx_gguf **out);
void styx_gguf_close(styx_gguf *g);

uint32_t styx_gguf_version(const styx_gguf *g);
uint64_t styx_gguf_data_start(const styx_gguf *g);
uint64_t styx_gguf_file_bytes(const styx_gguf *g);

/* ---- metadata.  Keys in first-seen order; a value is a node: a scalar, a
 * string, or an array of `count` elements of one type (nested arrays are
 * nodes too). */
uint64_t styx_gguf_kv_count(const styx_gguf *g);
int styx_gguf_kv_key(const styx_gguf *g, uint64_t i, const char **key);
/* the value node of key i */
int styx_gguf_kv_value(const styx_gguf *g, uint64_t i, uint64_t *node);
/* index of `key`, or -1 */
int64_t styx_gguf_find_kv(const styx_gguf *g, const char *key);
/* a node's type; for an array also its element type and length (count 1 and
 * elem_type = vtype for a scalar or string) */
int styx_gguf_node_type(const styx_gguf *g, uint64_t node, uint32_t *vtype, uint32_t *elem_type, uint64_t *count);
/* a scalar node's value, or element `index` of an array of scalars, stored
 * at `out` in its own type (1, 2, 4 or 8 bytes; bool as one byte 0/1) */
int styx_gguf_node_scalar(const styx_gguf *g, uint64_t node, uint64_t index, void *out);
/* a string node, or element `index` of an array of strings (not
 * NUL-terminated in general: use len) */
int styx_gguf_node_string(const styx_gguf *g, uint64_t node, uint64_t index, const char **s, uint64_t *len);
/* element `index` of an array of arrays, as a node */
int styx_gguf_node_elem(const styx_gguf *g, uint64_t node, uint64_t index, uint64_t *elem);

/* MoeModel::load's typed lookups (moe.rs:538-549): `key` must be present
 * with exactly this type, else STYX_EINVAL. */
int styx_gguf_get_u32(const styx_gguf *g, const char *key, uint32_t *out);
int styx_gguf_get_f32(const styx_gguf *g, const char *key, float *out);
int styx_gguf_get_str(const styx_gguf *g, const char *key, const char **s, uint64_t *len);

/* ---- tensors, in file order */
uint64_t styx_gguf_tensor_count(const styx_gguf *g);
int styx_gguf_tensor(const styx_gguf *g, uint64_t i, styx_gguf_tensor_info *out);
/* index of the first tensor named `name`, or -1 */
int64_t styx_gguf_find_tensor(const styx_gguf *g, const char *name);
/* the tensor's bytes [data_start + offset, + size_bytes) in the mapping */
int styx_gguf_tensor_data(const styx_gguf *g, uint64_t i, const void **data);

/* compute_size_bytes (lib.rs:243-332): elements per block and bytes per
 * block of a ggml type, and the bytes of a tensor of that type and shape. */
int styx_gguf_type_size(uint32_t ggml_type, uint64_t *block_elems, uint64_t *block_bytes);
int styx_gguf_tensor_bytes(uint32_t ggml_type, const uint64_t *dims, uint32_t n_dims, uint64_t *out);

#ifdef __cplusplus
}
#endif

#endif
