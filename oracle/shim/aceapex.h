/* The reference encoder's sources include aceapex.h for its pre-v1 container paths only (refrel.cpp region decode).
   The v1 encoder never calls it; this declaration plus the failing stub in aceapex_stub.c let it link. */
#pragma once
#include <stddef.h>
#include <stdint.h>
int64_t aceapex_decompress_region(const uint8_t* src, size_t n, uint8_t* dst, size_t cap, uint64_t off, uint64_t len);
