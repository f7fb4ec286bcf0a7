// Borrowed, strided views of caller-owned integer buffers (NumPy arrays or
// pinned host tensors).  The proposer never copies a whole padded buffer: it
// reads boundary windows and the per-step delta through these views.
#pragma once
#include <cstddef>
#include <cstdint>
#include <stdexcept>

namespace sh {

struct IntMatrix {
  const char* base = nullptr;
  ptrdiff_t s0 = 0, s1 = 0;  // byte strides
  size_t rows = 0, cols = 0;
  int itemsize = 8;  // 4 (int32) or 8 (int64)

  inline int64_t at(size_t i, size_t j) const {
    const char* p = base + static_cast<ptrdiff_t>(i) * s0 + static_cast<ptrdiff_t>(j) * s1;
    return itemsize == 8 ? *reinterpret_cast<const int64_t*>(p) : static_cast<int64_t>(*reinterpret_cast<const int32_t*>(p));
  }
  // Contiguous int64 row (the fast path), or nullptr.
  inline const int64_t* row64(size_t i) const {
    return (itemsize == 8 && s1 == 8) ? reinterpret_cast<const int64_t*>(base + static_cast<ptrdiff_t>(i) * s0) : nullptr;
  }
};

struct IntVector {
  const char* base = nullptr;
  ptrdiff_t s = 0;
  size_t n = 0;
  int itemsize = 8;
  inline int64_t at(size_t i) const {
    const char* p = base + static_cast<ptrdiff_t>(i) * s;
    return itemsize == 8 ? *reinterpret_cast<const int64_t*>(p) : static_cast<int64_t>(*reinterpret_cast<const int32_t*>(p));
  }
};

// Python ValueError.
struct ValueError : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};

}  // namespace sh
