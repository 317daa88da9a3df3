/*
 * vbq_gguf.h -- C ABI of the GGUF weight source: read a GGUF file's metadata and tensor
 * table, and upload tensors (or block-aligned tensor-parallel shards of them) into device
 * memory as the raw blocks the vbq_* kernels read.
 *
 * Replaces the reference engine's reader, vibeblade::GGUFFile (kevin046/VibeBlade
 * cpp/include/gguf.h, cpp/src/gguf.cpp:14-280): the same parse rules and error messages
 * (status VBQ_ERR_FORMAT / VBQ_ERR_IO and vbq_gguf_last_error()), and the same accessors --
 * tensor_info / tensor_data (gguf.h, gguf.cpp:253-268) as vbq_gguf_find + vbq_gguf_tensor /
 * vbq_gguf_tensor_data, meta_string / meta_int / meta_float / meta_bool and the array
 * accessors (gguf.cpp:270-320) as vbq_gguf_meta_*.  The file is memory-mapped read-only
 * (the reference reads it into one heap buffer).  A handle may be read from several
 * threads; vbq_gguf_upload uses the handle's staging buffers, so uploads from one handle
 * must not run concurrently.
 *
 * A tensor is K rows of N values: N = dims[0] (the fastest dimension), K = the product of
 * the other dims -- the layout gemv_dequant reads (cpp/src/dequant.cpp:739-771).
 */
#ifndef VBQ_GGUF_H
#define VBQ_GGUF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct vbq_gguf vbq_gguf;

typedef struct vbq_gguf_tensor_info {
  const char* name;  /* valid until vbq_gguf_close */
  int32_t n_dims;
  int64_t dims[4];   /* dims past n_dims are 1 */
  int32_t type;      /* ggml type id */
  uint64_t offset;   /* bytes from the start of the data section */
  uint64_t size;     /* tensor_nbytes(type, values) (cpp/include/ggml_types.h:195-199) */
} vbq_gguf_tensor_info;

/* metadata kinds (vbq_gguf_meta_count) */
#define VBQ_GGUF_META_INT 1
#define VBQ_GGUF_META_FLOAT 2
#define VBQ_GGUF_META_BOOL 3
#define VBQ_GGUF_META_STRING 4
#define VBQ_GGUF_META_INT_ARRAY 5
#define VBQ_GGUF_META_FLOAT_ARRAY 6
#define VBQ_GGUF_META_STRING_ARRAY 7

/* Message of the last failing vbq_gguf_* call on this thread. */
const char* vbq_gguf_last_error(void);

/* Open and parse (GGUFFile::GGUFFile, cpp/src/gguf.cpp:229-237).  *out is NULL on failure. */
int vbq_gguf_open(const char* path, vbq_gguf** out);
void vbq_gguf_close(vbq_gguf* g);

int vbq_gguf_version(const vbq_gguf* g, uint32_t* out);
int vbq_gguf_file_size(const vbq_gguf* g, uint64_t* out);
/* file offset of the data section (the tensor table's end, rounded up to 32 bytes) */
int vbq_gguf_data_offset(const vbq_gguf* g, uint64_t* out);

/* The tensor table, in file order (GGUFFile::tensors). */
int vbq_gguf_n_tensors(const vbq_gguf* g, int64_t* out);
int vbq_gguf_tensor(const vbq_gguf* g, int64_t index, vbq_gguf_tensor_info* out);
/* Index of the tensor named `name` (the last one of that name), or -1 (GGUFFile::tensor_info). */
int vbq_gguf_find(const vbq_gguf* g, const char* name, int64_t* index);
/* Host address of a tensor's bytes inside the mapping; VBQ_ERR_FORMAT when they run past
 * the end of the file (GGUFFile::tensor_data, cpp/src/gguf.cpp:253-260). */
int vbq_gguf_tensor_data(const vbq_gguf* g, int64_t index, const void** data);

/* Metadata (GGUFFile::meta_*, cpp/src/gguf.cpp:270-320).  As in the reference, each kind
 * of value has its own table (an integer and a string may share a key; a later key
 * replaces an earlier one of its kind), and 16-bit integer values are not kept.
 * vbq_gguf_meta_count: VBQ_OK and the string or array length (1 for a scalar) when `key`
 * holds a value of `kind`, else VBQ_ERR_NOT_FOUND.  The typed getters return
 * VBQ_ERR_NOT_FOUND when the key has no value of their kind (the reference then returns
 * its default). */
int vbq_gguf_meta_count(const vbq_gguf* g, const char* key, int32_t kind, int64_t* count);
int vbq_gguf_meta_int(const vbq_gguf* g, const char* key, int64_t* out);
int vbq_gguf_meta_float(const vbq_gguf* g, const char* key, double* out);
int vbq_gguf_meta_bool(const vbq_gguf* g, const char* key, int32_t* out);
int vbq_gguf_meta_string(const vbq_gguf* g, const char* key, const char** str, int64_t* len);
/* copies min(cap, count) elements into out (out may be NULL to ask for count only) */
int vbq_gguf_meta_int_array(const vbq_gguf* g, const char* key, int64_t* out, int64_t cap,
                            int64_t* count);
int vbq_gguf_meta_float_array(const vbq_gguf* g, const char* key, float* out, int64_t cap,
                              int64_t* count);
int vbq_gguf_meta_string_at(const vbq_gguf* g, const char* key, int64_t j, const char** str,
                            int64_t* len);

/*
 * Upload rows [row0, row1) x columns [col0, col1) of tensor `index` to device memory at
 * dst, each destination row dst_row_bytes apart (>= the shard's row bytes; the bytes past
 * them are zeroed, e.g. to pad rows to 16 bytes).  Columns must be whole blocks.  A
 * tensor-parallel column shard is a column range of every row, a row shard a row range;
 * both arrive packed as their own block matrix.  The bytes pass through two pinned 32 MiB
 * staging buffers (allocated by the first upload of the handle, freed by vbq_gguf_close)
 * with one 2-D copy per chunk on `stream`; the call returns when the copies are done.
 * This replaces the reference's raw-block upload (cpp/src/cuda_kernels.cu:152-156,
 * cpp/include/cuda_backend.h:108-120).
 */
int vbq_gguf_upload(vbq_gguf* g, int64_t index, int64_t row0, int64_t row1, int64_t col0,
                    int64_t col1, void* dst, int64_t dst_row_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VBQ_GGUF_H */
