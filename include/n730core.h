/*
 * n730core.h - .n730 file reader and host dequant (library: n730core.so).
 *
 * Drop-in for the reference C++ core src-code/cpp/n730core.cpp, whose ctypes
 * binding is src-code/scheduler.py:24-84.  Same symbols, argument types and
 * error codes.  All functions are thread-safe (pread-based).
 *
 * Error codes (n730core.cpp:22-28): -1 BAD_MAGIC, -2 FILE, -3 ALLOC,
 * -4 BAD_LAYER, -5 BAD_PREC, -6 NULL.
 */
#ifndef N730CORE_H
#define N730CORE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Open a .n730 file; returns a handle > 0 or a negative error.
 * Replaces n730core.cpp:162-182 (n730_open). */
int64_t n730_open(const char* path);

/* Close a handle.  Replaces n730core.cpp:184-190. */
void n730_close(int64_t handle);

/* Read the block at an absolute offset and dequantise it to fp32
 * ((float)q - zero_point) * scale into out[rows*cols]; also decodes the
 * group-wise ids 0x42/0x44/0x48.  Replaces n730core.cpp:192-248. */
int32_t n730_read_layer(int64_t handle, int64_t file_offset, float* out, int32_t* out_rows,
                        int32_t* out_cols, int32_t* out_prec_id);

/* rows*cols of the block at file_offset.  Replaces n730core.cpp:272-283. */
int32_t n730_layer_elements(int64_t handle, int64_t file_offset);

/* Same as n730_layer_elements (the reference's variant reads through a NULL
 * pointer, n730core.cpp:265).  Replaces n730core.cpp:250-270. */
int32_t n730_probe_layer_size(int64_t handle, int64_t file_offset);

/* Version string.  Replaces n730core.cpp:285-287. */
const char* n730_version(void);

/* New (no reference counterpart): header fields and raw payload of one block.
 * hdr[8] = layer_idx, prec_id, rows, cols, data_size, group_size (0 for
 * per-tensor), scale and zero-point as float32 bit patterns.  With payload ==
 * NULL only the header is read.  Used to upload packed codes to the GPU. */
int32_t n730_read_block(int64_t handle, int64_t file_offset, int64_t* hdr, uint8_t* payload,
                        int64_t capacity);

#ifdef __cplusplus
}
#endif
#endif
