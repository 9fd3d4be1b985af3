// Double-double arithmetic for the DoubleDouble precisions (double_double.rs): a value
// is the unevaluated sum hi + lo of two doubles (about a 106-bit significand), kept
// normalised (|lo| <= ulp(hi) / 2).  Built from the error-free transformations of
// Knuth (TwoSum), Dekker (Fast2Sum) and the FMA product (TwoProd), combined into the
// accurate addition and the product of Hida, Li and Bailey's double-double library.
// Division refines the leading quotient twice; the square root takes one Newton step
// from the double root.  Host and device (the CPU emulator and the kernels share it).
#pragma once

#include "dft_codelets.cuh"

namespace b200fft {

struct dd;
B200FFT_HD dd dd_sqrt(dd a);

struct dd {
    double hi, lo;
    dd() = default;
    B200FFT_HD constexpr dd(double h) : hi(h), lo(0.0) {}
    B200FFT_HD constexpr dd(double h, double l) : hi(h), lo(l) {}
    // found by argument-dependent lookup only: float / double sqrt stay unaffected
    friend B200FFT_HD dd sqrt(dd a) { return dd_sqrt(a); }
};

namespace ddops {

B200FFT_HD double two_sum(double a, double b, double &e) {
    const double s = a + b;
    const double bb = s - a;
    e = (a - (s - bb)) + (b - bb);
    return s;
}

B200FFT_HD double fast_two_sum(double a, double b, double &e) {
    const double s = a + b;
    e = b - (s - a);
    return s;
}

B200FFT_HD double two_prod(double a, double b, double &e) {
    const double p = a * b;
    e = fma(a, b, -p);
    return p;
}

}  // namespace ddops

B200FFT_HD dd operator+(dd a, dd b) {
    double e1, e2;
    double s = ddops::two_sum(a.hi, b.hi, e1);
    const double t = ddops::two_sum(a.lo, b.lo, e2);
    e1 += t;
    s = ddops::fast_two_sum(s, e1, e1);
    e1 += e2;
    double lo;
    const double hi = ddops::fast_two_sum(s, e1, lo);
    return dd(hi, lo);
}

B200FFT_HD dd operator-(dd a) { return dd(-a.hi, -a.lo); }
B200FFT_HD dd operator-(dd a, dd b) { return a + (-b); }

B200FFT_HD dd operator*(dd a, dd b) {
    double e;
    const double p = ddops::two_prod(a.hi, b.hi, e);
    e = fma(a.hi, b.lo, e);
    e = fma(a.lo, b.hi, e);
    e = fma(a.lo, b.lo, e);
    double lo;
    const double hi = ddops::fast_two_sum(p, e, lo);
    return dd(hi, lo);
}

B200FFT_HD dd operator/(dd a, dd b) {
    const double q1 = a.hi / b.hi;
    dd r = a - b * dd(q1);
    const double q2 = r.hi / b.hi;
    r = r - b * dd(q2);
    const double q3 = r.hi / b.hi;
    double lo;
    const double hi = ddops::fast_two_sum(q1, q2, lo);
    return dd(hi, lo) + dd(q3);
}

B200FFT_HD dd &operator+=(dd &a, dd b) { return a = a + b; }
B200FFT_HD dd &operator-=(dd &a, dd b) { return a = a - b; }
B200FFT_HD dd &operator*=(dd &a, dd b) { return a = a * b; }

// Square root: one Newton step from the double root (dd's sqrt forwards here).
B200FFT_HD dd dd_sqrt(dd a) {
    if (a.hi <= 0.0) return dd(0.0);
    const double s = ::sqrt(a.hi);
    double e;
    const double p = ddops::two_prod(s, s, e);
    const dd r = a - dd(p, e);
    return dd(s) + dd(r.hi / (2.0 * s));
}

}  // namespace b200fft

template <> struct KConst<b200fft::dd> {
    static B200FFT_HD b200fft::dd make(double hi, double lo) { return b200fft::dd(hi, lo); }
};
