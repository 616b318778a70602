/*
 * smeai_gguf.h -- GGUF model-file reader feeding the sm_100a Q2_K path.
 *
 * The reference runs GGUF models through llama.cpp (the TinyLlama Q2_K file
 * of llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:28-59: 201 tensors, Q2_K / Q3_K /
 * Q6_K / F32), whose loader is ggml's gguf reader (gguf_init_from_file,
 * gguf_get_n_tensors, gguf_find_tensor, gguf_get_tensor_{name,type,offset,
 * size}, gguf_find_key, gguf_get_val_{u32,str}, gguf_free in ggml 0.9.8;
 * its sources are not part of the reference tree).  These entry points
 * cover the same ground under an smeai_ prefix (so a process may also link
 * ggml) and add the step the reference's CPU_REPACK buffer does at load
 * time: a Q2_K tensor goes straight into the device tile layout.
 *
 * Format handled: GGUF versions 2 and 3, little-endian; metadata of every
 * value type (arrays are skipped, their type and length kept); tensor infos
 * with up to 4 dimensions; data section aligned to general.alignment
 * (default 32).  ne[0] is the innermost dimension (a weight's row length).
 *
 * Status codes: 0 = OK; -1 bad argument or malformed file; -2 allocation
 * failure; -3 unsupported (type, version, endianness); -5 CUDA error.
 * smeai_last_error() (smeai_q2k.h) says what went wrong.  A context is
 * read-only after smeai_gguf_open and may be shared between threads.
 */
#ifndef SMEAI_GGUF_H
#define SMEAI_GGUF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids used below (ggml.h numbering). */
enum {
  SMEAI_GGML_F32 = 0,
  SMEAI_GGML_F16 = 1,
  SMEAI_GGML_Q2_K = 10,
  SMEAI_GGML_Q3_K = 11,
  SMEAI_GGML_Q4_K = 12,
  SMEAI_GGML_Q5_K = 13,
  SMEAI_GGML_Q6_K = 14,
  SMEAI_GGML_Q8_K = 15
};

/* Parse the header, metadata and tensor infos of `path` (gguf_init_from_file
 * with no_alloc: tensor data stays in the file).  *ctx_out gets the context. */
int smeai_gguf_open(const char *path, void **ctx_out);
/* gguf_free. */
void smeai_gguf_close(void *ctx);

/* GGUF version, data alignment, byte offset of the data section. */
int smeai_gguf_version(const void *ctx);
uint64_t smeai_gguf_alignment(const void *ctx);
uint64_t smeai_gguf_data_offset(const void *ctx);

/* gguf_get_n_tensors / gguf_find_tensor (-1 when absent). */
int64_t smeai_gguf_n_tensors(const void *ctx);
int64_t smeai_gguf_find_tensor(const void *ctx, const char *name);

/* Tensor `id`: name (valid while ctx is open), ggml type, number of
 * dimensions, ne[0..3] (1 past n_dims), offset of its data relative to the
 * data section (gguf_get_tensor_offset) and its size in bytes (0 when the
 * type's block size is unknown to this reader).  Any output may be NULL. */
int smeai_gguf_tensor_info(const void *ctx, int64_t id, const char **name, int *ggml_type, int *n_dims,
                           int64_t ne[4], uint64_t *offset, uint64_t *nbytes);

/* Copy tensor `id`'s raw bytes (ggml's block layout) into host memory;
 * dst_bytes must be at least its size. */
int smeai_gguf_read_tensor(const void *ctx, int64_t id, void *dst, uint64_t dst_bytes);

/* Load a 2-D Q2_K tensor (ne[0] = k, a multiple of 256; ne[1] = rows) into
 * the device tile layout: the same handle smeai_q2k_repack returns (free it
 * with smeai_q2k_free).  Other types are refused with -3. */
int smeai_gguf_load_q2k(const void *ctx, int64_t id, void **w_dev_out);

/* The same for a 2-D Q3_K / Q6_K tensor (smeai_q3k_repack's / smeai_q6k_repack's handle). */
int smeai_gguf_load_q3k(const void *ctx, int64_t id, void **w_dev_out);
int smeai_gguf_load_q6k(const void *ctx, int64_t id, void **w_dev_out);

/* Metadata: gguf_get_n_kv / gguf_find_key (-1 when absent), the value type
 * of a key (GGUF value-type numbering: 0 u8 .. 12 f64, 8 = string,
 * 9 = array), and typed getters.  smeai_gguf_get_u64 accepts any integer
 * type holding a non-negative value; smeai_gguf_get_str returns a pointer
 * valid while ctx is open. */
int64_t smeai_gguf_n_kv(const void *ctx);
int64_t smeai_gguf_find_key(const void *ctx, const char *key);
int smeai_gguf_key_type(const void *ctx, const char *key);
int smeai_gguf_get_u64(const void *ctx, const char *key, uint64_t *out);
int smeai_gguf_get_f64(const void *ctx, const char *key, double *out);
int smeai_gguf_get_str(const void *ctx, const char *key, const char **out);

#ifdef __cplusplus
}
#endif

#endif /* SMEAI_GGUF_H */
