// Host-side helpers of the control plane (no CUDA dependency; built with the host compiler).
//
//  afd_mismatch_i32 / afd_mismatch_i64  first index at which two token-id arrays differ: the
//      inner loop of radix prefix matching (reference behaviour:
//      python/minisgl/kernel/csrc/src/radix.cpp, `fast_compare_key`).
//  afd_decode_out_loc                   KV slot of every request's next token from its page-table
//      row: slot = page_table[row][pos / page_size] * page_size + pos % page_size. Returns the
//      index of the first request whose page is missing (-1 entry) or out of range, else -1.
#include <algorithm>
#include <cstdint>

namespace {

template <typename T>
int64_t mismatch(const T* a, const T* b, int64_t n) {
  const T* end = a + n;
  return std::mismatch(a, end, b).first - a;
}

}  // namespace

extern "C" {

int64_t afd_mismatch_i32(const int32_t* a, const int32_t* b, int64_t n) { return mismatch(a, b, n); }

int64_t afd_mismatch_i64(const int64_t* a, const int64_t* b, int64_t n) { return mismatch(a, b, n); }

int64_t afd_decode_out_loc(const int32_t* page_table, int64_t row_stride, const int32_t* rows,
                           const int32_t* positions, int64_t n, int32_t page_size, int64_t num_pages,
                           int32_t* out_loc) {
  for (int64_t i = 0; i < n; ++i) {
    const int32_t pos = positions[i];
    const int64_t col = pos / page_size;
    if (pos < 0 || col >= row_stride) return i;
    const int32_t page = page_table[static_cast<int64_t>(rows[i]) * row_stride + col];
    if (page < 0 || page >= num_pages) return i;
    out_loc[i] = page * page_size + pos % page_size;
  }
  return -1;
}

}  // extern "C"
