// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// ArrayRef / MutableArrayRef interface: non-owning views of contiguous
// elements.
#ifndef CIM22_SHIM_LLVM_ADT_ARRAYREF_H
#define CIM22_SHIM_LLVM_ADT_ARRAYREF_H

#include <array>
#include <cassert>
#include <cstddef>
#include <initializer_list>
#include <vector>

namespace llvm {

template <typename T> class ArrayRef {
public:
  using value_type = T;
  using iterator = const T *;
  using const_iterator = const T *;
  using size_type = size_t;

  ArrayRef() = default;
  ArrayRef(const T &one) : ptr_(&one), len_(1) {}
  ArrayRef(const T *data, size_t length) : ptr_(data), len_(length) {}
  ArrayRef(const T *first, const T *last) : ptr_(first), len_(last - first) {}
  template <typename A>
  ArrayRef(const std::vector<T, A> &v) : ptr_(v.data()), len_(v.size()) {}
  template <size_t N>
  ArrayRef(const std::array<T, N> &a) : ptr_(a.data()), len_(N) {}
  template <size_t N> ArrayRef(const T (&a)[N]) : ptr_(a), len_(N) {}
  ArrayRef(const std::initializer_list<T> &list)
      : ptr_(list.begin() == list.end() ? nullptr : list.begin()), len_(list.size()) {}

  const T *begin() const { return ptr_; }
  const T *end() const { return ptr_ + len_; }
  const T *data() const { return ptr_; }
  size_t size() const { return len_; }
  bool empty() const { return len_ == 0; }
  const T &front() const { return ptr_[0]; }
  const T &back() const { return ptr_[len_ - 1]; }
  const T &operator[](size_t i) const { return ptr_[i]; }

  ArrayRef slice(size_t start, size_t count) const {
    assert(start + count <= len_ && "slice out of range");
    return ArrayRef(ptr_ + start, count);
  }
  ArrayRef slice(size_t start) const { return slice(start, len_ - start); }
  ArrayRef drop_front(size_t n = 1) const { return slice(n); }
  ArrayRef take_front(size_t n = 1) const { return slice(0, n); }

  bool equals(ArrayRef other) const {
    if (len_ != other.len_)
      return false;
    for (size_t i = 0; i < len_; ++i)
      if (!(ptr_[i] == other.ptr_[i]))
        return false;
    return true;
  }

  std::vector<T> vec() const { return std::vector<T>(begin(), end()); }

private:
  const T *ptr_ = nullptr;
  size_t len_ = 0;
};

template <typename T> class MutableArrayRef : public ArrayRef<T> {
public:
  using iterator = T *;

  MutableArrayRef() = default;
  MutableArrayRef(T &one) : ArrayRef<T>(one) {}
  MutableArrayRef(T *data, size_t length) : ArrayRef<T>(data, length) {}
  MutableArrayRef(T *first, T *last) : ArrayRef<T>(first, last) {}
  template <typename A> MutableArrayRef(std::vector<T, A> &v) : ArrayRef<T>(v) {}
  template <size_t N> MutableArrayRef(std::array<T, N> &a) : ArrayRef<T>(a) {}
  template <size_t N> MutableArrayRef(T (&a)[N]) : ArrayRef<T>(a) {}

  T *data() const { return const_cast<T *>(ArrayRef<T>::data()); }
  T *begin() const { return data(); }
  T *end() const { return data() + this->size(); }
  T &front() const { return data()[0]; }
  T &back() const { return data()[this->size() - 1]; }
  T &operator[](size_t i) const { return data()[i]; }

  MutableArrayRef slice(size_t start, size_t count) const {
    assert(start + count <= this->size() && "slice out of range");
    return MutableArrayRef(data() + start, count);
  }
  MutableArrayRef slice(size_t start) const { return slice(start, this->size() - start); }
  MutableArrayRef drop_front(size_t n = 1) const { return slice(n); }
  MutableArrayRef take_front(size_t n = 1) const { return slice(0, n); }
};

// Class template argument deduction, as llvm::ArrayRef(container) is written.
template <typename T> ArrayRef(const T &) -> ArrayRef<T>;
template <typename T> ArrayRef(const T *, size_t) -> ArrayRef<T>;
template <typename T, typename A> ArrayRef(const std::vector<T, A> &) -> ArrayRef<T>;
template <typename T, size_t N> ArrayRef(const std::array<T, N> &) -> ArrayRef<T>;
template <typename T, size_t N> ArrayRef(const T (&)[N]) -> ArrayRef<T>;
template <typename T> MutableArrayRef(T &) -> MutableArrayRef<T>;
template <typename T> MutableArrayRef(T *, size_t) -> MutableArrayRef<T>;
template <typename T, typename A> MutableArrayRef(std::vector<T, A> &) -> MutableArrayRef<T>;
template <typename T, size_t N> MutableArrayRef(std::array<T, N> &) -> MutableArrayRef<T>;

template <typename T> inline bool operator==(ArrayRef<T> a, ArrayRef<T> b) {
  return a.equals(b);
}
template <typename T> inline bool operator!=(ArrayRef<T> a, ArrayRef<T> b) {
  return !a.equals(b);
}

template <typename T> ArrayRef<T> makeArrayRef(const T *data, size_t length) {
  return ArrayRef<T>(data, length);
}

} // namespace llvm

#endif
