// detmath.cuh -- exp and log that give the same bits on the host and on the
// device.
//
// The connectivity generators decide each synapse by comparing a Philox
// word with a probability; a probability computed with the platform's exp
// or log can differ in its last bit between the CPU and the GPU, and a
// single such difference changes the network.  These functions use only
// IEEE double additions, multiplications, divisions (each rounded once;
// the library is compiled without fused multiply-adds) and exact scaling by
// powers of two, so every platform computes the same result:
//   * exp(-x), x >= 0: Cody and Waite's argument reduction x = k ln2 + r
//     with ln2 split into a high part exact in 32 bits and a low part, then
//     the Taylor series of exp(-r) to 22 terms (r < 0.7: error below 1e-19),
//     scaled by 2^-k;
//   * log(u), u > 0: u = m 2^e with m in [1/2, 1), then
//     ln m = 2 atanh(z), z = (m - 1)/(m + 1), |z| <= 1/3, by its series to
//     the z^45 term, plus e ln2.
// Accuracy is a few ulps; reproducibility is what matters here.
#pragma once
#include <cmath>

#if defined(__CUDACC__)
#define NRN_HD __host__ __device__ __forceinline__
#else
#define NRN_HD inline
#endif

namespace nrn {

constexpr double kLn2Hi = 6.93147180369123816490e-01;   // ln 2, high bits (exact product with k < 2^20)
constexpr double kLn2Lo = 1.90821492927058770002e-10;   // ln 2 - kLn2Hi
constexpr double kLn2 = 6.93147180559945309417e-01;

NRN_HD double det_exp_neg(double x) {
    if (!(x > 0.0)) return 1.0;
    if (x > 745.0) return 0.0;
    const double k = floor(x / kLn2);
    const double r = (x - k * kLn2Hi) - k * kLn2Lo;   // in [0, ln 2) up to rounding
    double s = 1.0;
    for (int i = 22; i >= 1; --i) s = 1.0 - (r / static_cast<double>(i)) * s;
    return ldexp(s, -static_cast<int>(k));
}

NRN_HD double det_log(double u) {
    int e = 0;
    const double m = frexp(u, &e);                     // u = m 2^e, m in [1/2, 1)
    const double z = (m - 1.0) / (m + 1.0);
    const double z2 = z * z;
    double s = 0.0;
    for (int i = 45; i >= 3; i -= 2) s = (s + 1.0 / static_cast<double>(i)) * z2;
    return 2.0 * z * (1.0 + s) + static_cast<double>(e) * kLn2;
}

}  // namespace nrn
