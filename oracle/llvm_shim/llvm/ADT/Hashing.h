// ORACLE support - test infrastructure only. Clean-room stand-in for the LLVM
// hash_combine interface. Only equal inputs must give equal codes (callers
// compare the hashed payloads afterwards); the mixing is 64-bit FNV-1a.
#ifndef CIM22_SHIM_LLVM_ADT_HASHING_H
#define CIM22_SHIM_LLVM_ADT_HASHING_H

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <type_traits>

namespace llvm {

class hash_code {
public:
  hash_code() = default;
  explicit hash_code(uint64_t v) : value_(v) {}
  operator size_t() const { return static_cast<size_t>(value_); }
  uint64_t value() const { return value_; }

private:
  uint64_t value_ = 0;
};

namespace shim_detail {
inline uint64_t mix_bytes(uint64_t h, const void *data, size_t n) {
  const unsigned char *p = static_cast<const unsigned char *>(data);
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 0x100000001b3ull;
  }
  return h;
}
constexpr uint64_t kSeed = 0xcbf29ce484222325ull;

template <typename T> uint64_t mix(uint64_t h, const T &v) {
  if constexpr (std::is_same_v<T, hash_code>) {
    const uint64_t x = v.value();
    return mix_bytes(h, &x, sizeof x);
  } else {
    static_assert(std::is_integral_v<T> || std::is_enum_v<T>,
                  "hash_combine of integral values and hash codes");
    return mix_bytes(h, &v, sizeof v);
  }
}
} // namespace shim_detail

template <typename It> hash_code hash_combine_range(It first, It last) {
  uint64_t h = shim_detail::kSeed;
  for (; first != last; ++first)
    h = shim_detail::mix(h, *first);
  return hash_code(h);
}

template <typename... Ts> hash_code hash_combine(const Ts &...values) {
  uint64_t h = shim_detail::kSeed;
  ((h = shim_detail::mix(h, values)), ...);
  return hash_code(h);
}

} // namespace llvm

#endif
