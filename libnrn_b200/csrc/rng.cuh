// rng.cuh -- counter-based random numbers on the device.
//
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) and the samplers built
// on it.  The samplers use only binary32 +, -, *, / and sqrt, each rounded
// on its own: the translation units that include this file are compiled
// with -fmad=false, so a host implementation of the same formulas (with
// contraction off) draws identical values.
#pragma once
#include <cstdint>

namespace nrn {

constexpr uint32_t kStreamDrive = 0x44524956u;
constexpr uint32_t kStreamConn = 0x434F4E4Eu;
constexpr uint32_t kStreamInit = 0x494E4954u;

struct U4 {
    uint32_t x, y, z, w;
};

__device__ __forceinline__ U4 philox4x32_10(U4 c, uint64_t seed) {
    uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
        uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
        c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

// Uniform in (0,1): odd multiples of 2^-24, exactly representable.
__device__ __forceinline__ float u01(uint32_t x) {
    return __uint2float_rn(((x >> 9) << 1) | 1u) * 5.9604644775390625e-8f;
}

// Poisson(lambda) by sequential inversion (Devroye 1986, X.3); exp_neg_lam
// = expf(-lambda) from the host.  At most 255 events.
__device__ __forceinline__ int poisson_inv(float u, float lam, float exp_neg_lam) {
    int k = 0;
    float p = exp_neg_lam;
    float F = p;
    while (u > F && k < 255) {
        k += 1;
        p = __fdiv_rn(__fmul_rn(p, lam), __int2float_rn(k));
        F = __fadd_rn(F, p);
    }
    return k;
}

// Natural log of a normal positive float: x = m 2^e, m in [sqrt(1/2), sqrt 2),
// ln m = 2 atanh(s) with s = (m-1)/(m+1), series to s^11; ln 2 split in two.
__device__ __forceinline__ float log_series(float x) {
    uint32_t b = __float_as_uint(x);
    int e = static_cast<int>((b >> 23) & 0xffu) - 127;
    float m = __uint_as_float((b & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421353816986083984375f) { m = __fmul_rn(m, 0.5f); e += 1; }
    float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
    float s2 = __fmul_rn(s, s);
    float poly = 1.0f / 11.0f;
    poly = __fadd_rn(__fmul_rn(poly, s2), 1.0f / 9.0f);
    poly = __fadd_rn(__fmul_rn(poly, s2), 1.0f / 7.0f);
    poly = __fadd_rn(__fmul_rn(poly, s2), 1.0f / 5.0f);
    poly = __fadd_rn(__fmul_rn(poly, s2), 1.0f / 3.0f);
    poly = __fadd_rn(__fmul_rn(poly, s2), 1.0f);
    float lnm = __fmul_rn(__fmul_rn(2.0f, s), poly);
    float fe = __int2float_rn(e);
    return __fadd_rn(__fmul_rn(fe, 0.693145751953125f),
                     __fadd_rn(__fmul_rn(fe, 1.428606765330187045e-06f), lnm));
}

// cos(2 pi u), u in [0,1): quadrant k = round(4u), r = u - k/4 (exact),
// Taylor series of sin and cos of 2 pi r on [-pi/4, pi/4].
__device__ __forceinline__ float cos_2pi_series(float u) {
    float q = __fmul_rn(u, 4.0f);
    int k = static_cast<int>(__fadd_rn(q, 0.5f));
    float r = __fsub_rn(u, __fmul_rn(__int2float_rn(k), 0.25f));
    float x = __fmul_rn(r, 6.28318548202514648438f);
    float x2 = __fmul_rn(x, x);
    float c = 1.0f / 40320.0f;
    c = __fsub_rn(__fmul_rn(c, x2), 1.0f / 720.0f);
    c = __fadd_rn(__fmul_rn(c, x2), 1.0f / 24.0f);
    c = __fsub_rn(__fmul_rn(c, x2), 0.5f);
    c = __fadd_rn(__fmul_rn(c, x2), 1.0f);
    float s = 1.0f / 362880.0f;
    s = __fsub_rn(__fmul_rn(s, x2), 1.0f / 5040.0f);
    s = __fadd_rn(__fmul_rn(s, x2), 1.0f / 120.0f);
    s = __fsub_rn(__fmul_rn(s, x2), 1.0f / 6.0f);
    s = __fadd_rn(__fmul_rn(__fmul_rn(s, x2), x), x);
    switch (k & 3) {
        case 0: return c;
        case 1: return -s;
        case 2: return -c;
        default: return s;
    }
}

// Standard normal (Box & Muller 1958).
__device__ __forceinline__ float normal_bm(float u1, float u2) {
    float l = log_series(u1);
    float rad = __fsqrt_rn(__fmul_rn(-2.0f, l));
    return __fmul_rn(rad, cos_2pi_series(u2));
}

}  // namespace nrn
