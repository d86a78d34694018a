// vw_libm_exp.h -- fp64 exp with the host libm's exact results, for host and device code.
//
// voxwerk computes every softmax numerator with Math.Exp (src/Voxwerk/Talker/Sampler.cs:57), which .NET on Linux
// takes from the C runtime: glibc's exp.  glibc's exp is not correctly rounded (on this path's arguments about 1 in
// 1000 values differ from the correctly rounded one), and CUDA's exp differs from both, so matching the reference's
// sums bit for bit needs glibc's own function.  This file restates its published algorithm: glibc >= 2.28 took it
// from Arm's Optimized Routines (exp.c, Szabolcs Nagy, 2018); the x86-64 build that runs on FMA-capable CPUs
// evaluates it with the multiply-adds fused as below.  The table (vw_libm_exp_table.h) is computed from its
// definition by gen_exp_table.py.  tests/test_exp_cpu.py compiles this same file for the host and checks it against
// the C library's exp on every softmax argument of the five benchmark configurations (8.7 million values).
//
// Algorithm, for |x| < 512: k = round(x * 128 / ln 2) (by adding 1.5 * 2^52), r = x - k ln2/128 (two-part
// constant, fused), exp(x) = 2^(k/128) (1 + tail + r + r^2 (C2 + C3 r) + r^4 (C4 + C5 r)) with 2^(k/128) from the
// table.  |x| >= 512 rescales to keep 2^(k/128) normal and, for results below 2^-1022, rounds once more in a
// double-double step.  Only ieee binary64 operations and fma are used, so host and device results are identical.
// Compile device code with -fmad=false (and host code with -ffp-contract=off): no contraction other than the
// explicit fma calls may happen.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)   // device code (the table lives in device memory)
#define VW_HD __device__ __forceinline__
#define VW_EXP_TABLE_STORAGE __device__
#else
#define VW_HD inline
#define VW_EXP_TABLE_STORAGE static
#endif

#include "vw_libm_exp_table.h"

namespace vw {
namespace libm {

VW_HD uint64_t as_u64(double x) {
#if defined(__CUDA_ARCH__)
    return static_cast<uint64_t>(__double_as_longlong(x));
#else
    uint64_t u;
    std::memcpy(&u, &x, sizeof u);
    return u;
#endif
}
VW_HD double as_f64(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double(static_cast<long long>(u));
#else
    double x;
    std::memcpy(&x, &u, sizeof x);
    return x;
#endif
}
VW_HD uint64_t table(int i) {
#if defined(__CUDA_ARCH__)
    return __ldg(&kExpTab[i]);
#else
    return kExpTab[i];
#endif
}

constexpr double kInvLn2N = 0x1.71547652b82fep0 * 128;   // 128 / ln 2
constexpr double kNegLn2HiN = -0x1.62e42fefa0000p-8;     // -ln2/128, high part
constexpr double kNegLn2LoN = -0x1.cf79abc9e3b3ap-47;    // -ln2/128, low part
constexpr double kShift = 0x1.8p52;                      // rounds to an integer in the low bits
constexpr double kC2 = 0x1.ffffffffffdbdp-2;             // polynomial for e^r - 1 - r on |r| <= ln2/256
constexpr double kC3 = 0x1.555555555543cp-3;
constexpr double kC4 = 0x1.55555cf172b91p-5;
constexpr double kC5 = 0x1.1111167a4d017p-7;

}  // namespace libm

// exp(x) with the exact result of glibc's exp (x86-64, FMA build).
VW_HD double libm_exp(double x) {
    using namespace libm;
    const uint64_t ux = as_u64(x);
    const uint32_t abstop = static_cast<uint32_t>(ux >> 52) & 0x7ffu;
    // |x| < 2^-54, |x| >= 512, inf and nan
    if (abstop - 0x3c9u >= 0x408u - 0x3c9u) {
        if (static_cast<int32_t>(abstop - 0x3c9u) < 0) return 1.0 + x;   // tiny: 1 + x rounds correctly
        if (abstop >= 0x409u) {                                           // |x| >= 1024, inf, nan
            if (ux == 0xfff0000000000000ull) return 0.0;
            if (abstop >= 0x7ffu) return 1.0 + x;
            return (ux >> 63) ? 0.0 : as_f64(0x7ff0000000000000ull);
        }
    }
    double kd = fma(kInvLn2N, x, kShift);
    const uint64_t ki = as_u64(kd);
    kd = kd - kShift;
    const double r = fma(kd, kNegLn2LoN, fma(kd, kNegLn2HiN, x));
    const int idx = 2 * static_cast<int>(ki & 127u);
    const uint64_t top = ki << 45;
    const double tail = as_f64(table(idx));
    uint64_t sbits = table(idx + 1) + top;
    const double r2 = r * r;
    double tmp = tail + r;
    tmp = fma(r2, fma(r, kC3, kC2), tmp);
    tmp = fma(r2 * r2, fma(r, kC5, kC4), tmp);
    if (abstop >= 0x408u) {   // |x| >= 512: keep the scale normal, round the product unfused
        if ((ki & 0x80000000u) == 0) {
            sbits -= 1009ull << 52;
            const double scale = as_f64(sbits);
            return 0x1p1009 * (scale + scale * tmp);
        }
        sbits += 1022ull << 52;
        const double scale = as_f64(sbits);
        const double st = scale * tmp;
        double y = scale + st;
        if (y < 1.0) {   // the result is subnormal: round scale (1 + tmp) once, at 2^-1022 * ulp(1)
            double lo = (scale - y) + st;
            const double hi = 1.0 + y;
            lo = ((1.0 - hi) + y) + lo;
            y = (hi + lo) - 1.0;
            if (y == 0.0) y = 0.0;   // no negative zero
        }
        return 0x1p-1022 * y;
    }
    const double scale = as_f64(sbits);
    return fma(scale, tmp, scale);
}

}  // namespace vw
