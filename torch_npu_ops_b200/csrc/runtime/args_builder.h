// Byte-packed kernel argument buffer with natural alignment, the same
// interface as the reference's ArgsBuilder (triton_npu/args_builder.h:34-302):
// constructArgs / add / add_aligned / pad_to and the hex-dump and diff
// helpers used when debugging argument-packing mismatches.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <iomanip>
#include <sstream>
#include <string>
#include <type_traits>
#include <vector>

namespace xllm::kernel::npu {

class ArgsBuilder final {
 public:
  ArgsBuilder() { buf_.reserve(256); }

  const void* data() const { return buf_.data(); }
  size_t size() const { return buf_.size(); }
  void clear() { buf_.clear(); }

  template <typename... Ts>
  void constructArgs(const Ts&... args) {
    (add(args), ...);
  }

  template <typename T>
  void add(const T& v) {
    static_assert(std::is_trivially_copyable_v<T>, "kernel arguments must be trivially copyable");
    add_aligned<T>(v, alignof(T));
  }

  template <typename T>
  void add_aligned(const T& v, size_t alignment) {
    static_assert(std::is_trivially_copyable_v<T>, "kernel arguments must be trivially copyable");
    pad_to(alignment);
    const size_t at = buf_.size();
    buf_.resize(at + sizeof(T));
    std::memcpy(buf_.data() + at, &v, sizeof(T));
  }

  void pad_to(size_t alignment) {
    if (alignment > 1) buf_.resize((buf_.size() + alignment - 1) / alignment * alignment, 0);
  }

  std::string hex_dump() const {
    std::ostringstream os;
    os << std::hex << std::uppercase << std::setfill('0');
    for (size_t i = 0; i < buf_.size(); ++i) {
      if (i && i % 16 == 0) os << '\n';
      else if (i) os << ' ';
      os << std::setw(2) << static_cast<unsigned>(buf_[i]);
    }
    return os.str();
  }

  bool compare_with(const void* other, size_t n) const {
    return n == buf_.size() && std::memcmp(buf_.data(), other, n) == 0;
  }

  // Byte offsets where this buffer and `other` differ (empty when equal).
  std::vector<size_t> diff_with(const void* other, size_t n) const {
    std::vector<size_t> out;
    const auto* o = static_cast<const unsigned char*>(other);
    const size_t m = n < buf_.size() ? n : buf_.size();
    for (size_t i = 0; i < m; ++i)
      if (buf_[i] != o[i]) out.push_back(i);
    for (size_t i = m; i < (n > buf_.size() ? n : buf_.size()); ++i) out.push_back(i);
    return out;
  }

 private:
  std::vector<unsigned char> buf_;
};

}  // namespace xllm::kernel::npu
