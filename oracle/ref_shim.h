/*
 * ref_shim.h -- the few HIP names the reference's CPU verification code uses,
 * so that code compiles with plain g++ (TEST INFRASTRUCTURE ONLY).
 *
 * The reference's host drivers run their CPU GEMMs, codecs and byte layouts
 * over __hip_fp8_e4m3 (OCP E4M3FN on gfx950) and mark a few helpers
 * __host__ __device__.  Nothing else from HIP is needed by the functions that
 * oracle/ref_extract.py cuts out of the reference sources, so this header
 * supplies exactly:
 *   - __host__ / __device__ as empty markers;
 *   - __hip_fp8_e4m3: one byte of storage (__x), conversion to float by the
 *     OCP E4M3FN decode (bias 7, no infinities, S.1111.111 is NaN), and
 *     construction from float by round-to-nearest-even with saturation to
 *     +-448 (HIP's default __HIP_SATFINITE), NaN -> 0x7F.
 * The decode is this project's own code, checked against torch's
 * float8_e4m3fn for all 256 codes by tests/test_ref_pin.py.
 */
#ifndef BSGEMM_REF_SHIM_H
#define BSGEMM_REF_SHIM_H

#include <algorithm>
#include <cerrno>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>
#include <omp.h>

#define __host__
#define __device__

struct __hip_fp8_e4m3 {
    std::uint8_t __x;

    __hip_fp8_e4m3() = default;
    explicit __hip_fp8_e4m3(float f) : __x(encode(f)) {}

    explicit operator float() const {
        // built from the bit fields: no libm call in the GEMM loops
        const std::uint32_t s = (__x & 0x80u) << 24, e = (__x >> 3) & 15u, m = __x & 7u;
        if (e == 15 && m == 7) return std::numeric_limits<float>::quiet_NaN();
        if (e == 0) {                                    // subnormal: m * 2^-9
            const float mag = static_cast<float>(m) * 0.001953125f;
            return s ? -mag : mag;
        }
        const std::uint32_t bits = s | ((e + 120u) << 23) | (m << 20);
        float f;
        std::memcpy(&f, &bits, 4);
        return f;
    }

  private:
    static std::uint8_t encode(float f) {
        if (std::isnan(f)) return 0x7F;
        const std::uint8_t sign = std::signbit(f) ? 0x80 : 0x00;
        const double a = std::fabs(static_cast<double>(f));
        if (a >= 448.0) return sign | 0x7E;
        if (a == 0.0) return sign;
        int e2;
        std::frexp(a, &e2);
        const int e = e2 - 1;                            // a in [2^e, 2^(e+1))
        if (e < -6)                                      // subnormal: units of 2^-9
            return sign | static_cast<std::uint8_t>(std::nearbyint(std::ldexp(a, 9)));
        int q = static_cast<int>(std::nearbyint(std::ldexp(a, 3 - e)));   // 8..16
        int ee = e;
        if (q == 16) { q = 8; ++ee; }
        int code = ((ee + 7) << 3) | (q - 8);
        if (code > 0x7E) code = 0x7E;
        return sign | static_cast<std::uint8_t>(code);
    }
};
static_assert(sizeof(__hip_fp8_e4m3) == 1, "one byte per element");

#endif
