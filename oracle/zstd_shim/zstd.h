/* Declarations of the four libzstd (1.5.x) entry points the reference's
 * src/quant_format.cpp calls.  The container ships the library
 * (libzstd.so.1) but not its header; these prototypes follow zstd's public,
 * stable API.  Test infrastructure for oracle/_ref only. */
#ifndef PF_ZSTD_SHIM_H
#define PF_ZSTD_SHIM_H
#include <stddef.h>
#ifdef __cplusplus
extern "C" {
#endif
size_t ZSTD_compressBound(size_t srcSize);
size_t ZSTD_compress(void* dst, size_t dstCapacity, const void* src, size_t srcSize,
                     int compressionLevel);
size_t ZSTD_decompress(void* dst, size_t dstCapacity, const void* src, size_t compressedSize);
unsigned ZSTD_isError(size_t code);
#ifdef __cplusplus
}
#endif
#endif
