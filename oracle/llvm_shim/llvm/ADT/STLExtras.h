// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// STLExtras range helpers.
#ifndef CIM22_SHIM_LLVM_ADT_STLEXTRAS_H
#define CIM22_SHIM_LLVM_ADT_STLEXTRAS_H

#include <algorithm>
#include <cassert>
#include <cstddef>
#include <iterator>
#include <tuple>
#include <utility>

namespace llvm {

template <typename R, typename P> bool all_of(R &&range, P pred) {
  return std::all_of(std::begin(range), std::end(range), pred);
}
template <typename R, typename P> bool any_of(R &&range, P pred) {
  return std::any_of(std::begin(range), std::end(range), pred);
}
template <typename R, typename P> bool none_of(R &&range, P pred) {
  return std::none_of(std::begin(range), std::end(range), pred);
}
template <typename R, typename E> bool is_contained(R &&range, const E &element) {
  return std::find(std::begin(range), std::end(range), element) != std::end(range);
}
template <typename R> void sort(R &&range) { std::sort(std::begin(range), std::end(range)); }
template <typename R, typename C> void sort(R &&range, C cmp) {
  std::sort(std::begin(range), std::end(range), cmp);
}
template <typename R, typename O, typename F> O transform(R &&range, O out, F fn) {
  return std::transform(std::begin(range), std::end(range), out, fn);
}

// enumerate(range): (index, element reference) pairs, usable with
// structured bindings.
template <typename R> class Enumerator {
  using It = decltype(std::begin(std::declval<R &>()));

public:
  explicit Enumerator(R &&range) : range_(std::forward<R>(range)) {}

  class iterator {
  public:
    iterator(It it, size_t index) : it_(it), index_(index) {}
    std::pair<size_t, decltype(*std::declval<It>())> operator*() const {
      return {index_, *it_};
    }
    iterator &operator++() {
      ++it_;
      ++index_;
      return *this;
    }
    bool operator!=(const iterator &o) const { return it_ != o.it_; }
    bool operator==(const iterator &o) const { return it_ == o.it_; }

  private:
    It it_;
    size_t index_;
  };

  iterator begin() { return iterator(std::begin(range_), 0); }
  iterator end() { return iterator(std::end(range_), 0); }

private:
  R range_;
};

template <typename R> Enumerator<R> enumerate(R &&range) {
  return Enumerator<R>(std::forward<R>(range));
}

// zip_equal(a, b): element pairs of two ranges of equal length.
template <typename A, typename B> class ZipEqual {
  using ItA = decltype(std::begin(std::declval<A &>()));
  using ItB = decltype(std::begin(std::declval<B &>()));

public:
  ZipEqual(A &&a, B &&b) : a_(std::forward<A>(a)), b_(std::forward<B>(b)) {
    assert(std::distance(std::begin(a_), std::end(a_)) ==
               std::distance(std::begin(b_), std::end(b_)) &&
           "zip_equal ranges differ in length");
  }

  class iterator {
  public:
    iterator(ItA a, ItB b) : a_(a), b_(b) {}
    std::tuple<decltype(*std::declval<ItA>()), decltype(*std::declval<ItB>())>
    operator*() const {
      return {*a_, *b_};
    }
    iterator &operator++() {
      ++a_;
      ++b_;
      return *this;
    }
    bool operator!=(const iterator &o) const { return a_ != o.a_; }
    bool operator==(const iterator &o) const { return a_ == o.a_; }

  private:
    ItA a_;
    ItB b_;
  };

  iterator begin() { return iterator(std::begin(a_), std::begin(b_)); }
  iterator end() { return iterator(std::end(a_), std::end(b_)); }

private:
  A a_;
  B b_;
};

template <typename A, typename B> ZipEqual<A, B> zip_equal(A &&a, B &&b) {
  return ZipEqual<A, B>(std::forward<A>(a), std::forward<B>(b));
}

} // namespace llvm

#endif
