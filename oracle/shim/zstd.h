/* Declarations of the five libzstd functions the reference reader and encoder call. The image ships only the runtime
   library (libzstd.so.1, 1.5.x) without its header; these are the library's public prototypes, and the build links
   the runtime library by path. */
#pragma once
#include <stddef.h>
#ifdef __cplusplus
extern "C" {
#endif
unsigned long long ZSTD_getFrameContentSize(const void* src, size_t srcSize);
size_t ZSTD_findFrameCompressedSize(const void* src, size_t srcSize);
size_t ZSTD_decompress(void* dst, size_t dstCapacity, const void* src, size_t compressedSize);
size_t ZSTD_compressBound(size_t srcSize);
size_t ZSTD_compress(void* dst, size_t dstCapacity, const void* src, size_t srcSize, int compressionLevel);
unsigned ZSTD_isError(size_t code);
#ifdef __cplusplus
}
#endif
