// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// StringRef interface: a non-owning view of characters.
#ifndef CIM22_SHIM_LLVM_ADT_STRINGREF_H
#define CIM22_SHIM_LLVM_ADT_STRINGREF_H

#include <cstddef>
#include <cstring>
#include <ostream>
#include <string>
#include <string_view>

namespace llvm {

class StringRef {
public:
  StringRef() = default;
  StringRef(const char *s) : ptr_(s), len_(s ? std::strlen(s) : 0) {}
  StringRef(const char *s, size_t n) : ptr_(s), len_(n) {}
  StringRef(const std::string &s) : ptr_(s.data()), len_(s.size()) {}
  StringRef(std::string_view s) : ptr_(s.data()), len_(s.size()) {}

  const char *data() const { return ptr_; }
  size_t size() const { return len_; }
  bool empty() const { return len_ == 0; }
  const char *begin() const { return ptr_; }
  const char *end() const { return ptr_ + len_; }
  char operator[](size_t i) const { return ptr_[i]; }
  std::string str() const { return std::string(ptr_, len_); }
  operator std::string_view() const { return std::string_view(ptr_, len_); }
  bool equals(StringRef o) const {
    return len_ == o.len_ && (len_ == 0 || std::memcmp(ptr_, o.ptr_, len_) == 0);
  }

private:
  const char *ptr_ = nullptr;
  size_t len_ = 0;
};

inline bool operator==(StringRef a, StringRef b) { return a.equals(b); }
inline bool operator!=(StringRef a, StringRef b) { return !a.equals(b); }
inline std::ostream &operator<<(std::ostream &os, StringRef s) {
  return os.write(s.data(), static_cast<std::streamsize>(s.size()));
}

} // namespace llvm

#endif
