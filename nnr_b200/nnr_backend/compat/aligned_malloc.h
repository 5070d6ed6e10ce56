/* Build shim for compiling nnr's sources with GCC on Linux: nnr calls the
 * MSVC names for aligned allocation (_aligned_malloc / _aligned_free). */
#pragma once
#include <stdlib.h>
static inline void* _aligned_malloc(size_t size, size_t align) {
  size_t rounded = (size + align - 1) / align * align;
  return aligned_alloc(align, rounded ? rounded : align);
}
static inline void _aligned_free(void* p) { free(p); }
