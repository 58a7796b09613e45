// ORACLE support - test infrastructure only. Clean-room subset of the LLVM
// APFloat interface for two formats, written from IEEE 754:
//   BFloat      1 sign, 8 exponent (bias 127), 7 fraction bits; subnormals
//   IEEEdouble  binary64
// Values are held exactly in a double (every BFloat value is a double).
// Conversions to BFloat and scalbn round to nearest, ties to even, with
// gradual underflow and overflow to infinity; only that rounding mode is
// provided.
#ifndef CIM22_SHIM_LLVM_ADT_APFLOAT_H
#define CIM22_SHIM_LLVM_ADT_APFLOAT_H

#include "llvm/ADT/APInt.h"

#include <cassert>
#include <cmath>
#include <cstdint>
#include <cstring>

namespace llvm {

struct fltSemantics {
  unsigned bits; // 16: BFloat, 64: IEEEdouble
};

class APFloat {
public:
  enum roundingMode { rmNearestTiesToEven, rmTowardPositive, rmTowardNegative, rmTowardZero,
                      rmNearestTiesToAway };
  enum opStatus { opOK = 0, opInvalidOp = 1, opDivByZero = 2, opOverflow = 4,
                  opUnderflow = 8, opInexact = 16 };

  static const fltSemantics &BFloat() {
    static const fltSemantics s{16};
    return s;
  }
  static const fltSemantics &IEEEdouble() {
    static const fltSemantics s{64};
    return s;
  }

  APFloat(const fltSemantics &sem, const APInt &bits) : sem_(&sem) {
    if (sem.bits == 16) {
      assert(bits.getBitWidth() == 16);
      value_ = decodeBF16(static_cast<uint16_t>(bits.getZExtValue()));
    } else {
      assert(sem.bits == 64 && bits.getBitWidth() == 64);
      const uint64_t raw = bits.getZExtValue();
      std::memcpy(&value_, &raw, sizeof value_);
    }
  }
  explicit APFloat(double value) : sem_(&IEEEdouble()), value_(value) {}

  bool isFinite() const { return std::isfinite(value_); }
  bool isNaN() const { return std::isnan(value_); }
  bool isInfinity() const { return std::isinf(value_); }
  bool isZero() const { return value_ == 0.0; }
  bool isNegative() const { return std::signbit(value_); }

  opStatus convert(const fltSemantics &to, roundingMode mode, bool *losesInfo) {
    assert(mode == rmNearestTiesToEven && "only round-to-nearest-even is provided");
    (void)mode;
    opStatus status = opOK;
    bool inexact = false;
    if (to.bits == 16 && sem_->bits == 64) {
      bool overflow = false;
      value_ = decodeBF16(encodeBF16(value_, &inexact, &overflow));
      status = static_cast<opStatus>((inexact ? opInexact : 0) | (overflow ? opOverflow : 0));
    }
    sem_ = &to;
    if (losesInfo)
      *losesInfo = inexact;
    return status;
  }

  double convertToDouble() const {
    assert(sem_->bits == 64 && "convertToDouble of a non-double value");
    return value_;
  }

  APInt bitcastToAPInt() const {
    if (sem_->bits == 16) {
      bool inexact = false, overflow = false;
      return APInt(16, encodeBF16(value_, &inexact, &overflow));
    }
    uint64_t raw;
    std::memcpy(&raw, &value_, sizeof raw);
    return APInt(64, raw);
  }

  // x * 2^exponent rounded once to x's format (llvm::scalbn).
  static APFloat scaled(APFloat x, int exponent, roundingMode mode) {
    assert(mode == rmNearestTiesToEven && "only round-to-nearest-even is provided");
    (void)mode;
    if (!std::isfinite(x.value_) || x.value_ == 0.0)
      return x;
    // Exact in binary64 for the exponents of both formats; beyond that the
    // result is an overflow or an underflow to zero in either format.
    const int e = exponent > 4000 ? 4000 : exponent < -4000 ? -4000 : exponent;
    double scaled = std::ldexp(x.value_, e);
    if (x.sem_->bits == 16) {
      bool inexact = false, overflow = false;
      scaled = decodeBF16(encodeBF16(scaled, &inexact, &overflow));
    }
    x.value_ = scaled;
    return x;
  }

private:
  static double decodeBF16(uint16_t bits) {
    const bool negative = bits & 0x8000u;
    const int exponent = (bits >> 7) & 0xff;
    const int fraction = bits & 0x7f;
    double v;
    if (exponent == 0xff)
      v = fraction ? std::nan("") : INFINITY;
    else if (exponent == 0)
      v = std::ldexp(static_cast<double>(fraction), -133);
    else
      v = std::ldexp(static_cast<double>(128 + fraction), exponent - 134);
    return negative ? -v : v;
  }

  // Round a binary64 value to the nearest BFloat, ties to even.
  static uint16_t encodeBF16(double v, bool *inexact, bool *overflow) {
    *inexact = false;
    *overflow = false;
    const uint16_t sign = std::signbit(v) ? 0x8000u : 0u;
    if (std::isnan(v))
      return sign | 0x7fc0u;
    const double a = std::fabs(v);
    if (a == 0.0)
      return sign;
    if (std::isinf(a))
      return sign | 0x7f80u;
    int e2 = 0;
    std::frexp(a, &e2);
    int e = e2 - 1; // a is in [2^e, 2^(e+1))
    const int quantum = e >= -126 ? e - 7 : -133;
    const double scaled = std::ldexp(a, -quantum);
    // nearbyint rounds to nearest, ties to even, in the default FP mode.
    double r = std::nearbyint(scaled);
    *inexact = r != scaled;
    if (e >= -126) {
      if (r == 256.0) {
        r = 128.0;
        ++e;
      }
      if (e > 127) {
        *overflow = true;
        *inexact = true;
        return sign | 0x7f80u;
      }
      return static_cast<uint16_t>(sign | ((e + 127) << 7) | (static_cast<int>(r) - 128));
    }
    // Subnormal range: r * 2^-133, or the smallest normal when r == 128.
    return static_cast<uint16_t>(sign | static_cast<int>(r));
  }

  const fltSemantics *sem_;
  double value_ = 0.0;
};

inline APFloat scalbn(APFloat x, int exponent, APFloat::roundingMode mode) {
  return APFloat::scaled(x, exponent, mode);
}

} // namespace llvm

#endif
