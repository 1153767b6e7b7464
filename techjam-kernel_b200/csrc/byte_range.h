// byte_range.h — address ranges of row-major operands, for the host-side
// overlap checks of the entry points (an output whose stores race the reads
// of an input is rejected before launch).
#pragma once

#include <cstdint>

namespace b200attn {

struct ByteRange {
  uintptr_t lo = 0, hi = 0;  // [lo, hi)
  bool overlaps(const ByteRange& o) const { return lo < o.hi && o.lo < hi; }
};

// Bytes spanned by a [rows, cols] matrix of `elem`-byte elements whose rows
// start `ld` elements apart (the last dimension contiguous).
inline ByteRange rows_range(const void* base, int64_t rows, int64_t cols, int64_t ld,
                            int64_t elem = 2) {
  const uintptr_t lo = reinterpret_cast<uintptr_t>(base);
  const int64_t span = (rows > 1 ? (rows - 1) * ld : 0) + cols;
  return ByteRange{lo, lo + static_cast<uintptr_t>(span * elem)};
}

}  // namespace b200attn
