// Failing stand-in for the aceapex library call that only the reference encoder's pre-v1 paths make.
#include "aceapex.h"
int64_t aceapex_decompress_region(const uint8_t*, size_t, uint8_t*, size_t, uint64_t, uint64_t) { return -1; }
