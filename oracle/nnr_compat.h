/* Build shim for compiling nnr x64 headers with GCC on Linux (test
 * infrastructure only): nnr calls the MSVC names for aligned allocation. */
#pragma once
#include <stdlib.h>
static inline void* _aligned_malloc(size_t size, size_t align) {
  size_t rounded = (size + align - 1) / align * align;
  return aligned_alloc(align, rounded ? rounded : align);
}
static inline void _aligned_free(void* p) { free(p); }
