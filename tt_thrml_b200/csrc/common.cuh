// Shared helpers of the sweep kernels: error reporting, Philox4x32-10 and
// the uniform / normal / Gumbel transforms every kernel draws from.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/tthrml.h"

namespace tthrml {

// Thread-local last error message (read by tthrml_last_error()).
void set_error(const char* fmt, ...);

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TTHRML_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return TTHRML_ERR_CUDA;
}

// Checks the launch just made (configuration errors surface here; the kernel
// itself runs asynchronously).
inline int launch_status(const char* what) { return cuda_status(cudaGetLastError(), what); }

// Salts of the Philox counter word 3: one per variate kind so the spin,
// categorical and gaussian streams of one (chain, row, sweep) never overlap.
constexpr uint32_t kSaltSpin = 0x5350494eu;      // "SPIN"
constexpr uint32_t kSaltGauss = 0x47415553u;     // "GAUS"
constexpr uint32_t kSaltCat = 0x43415400u;       // "CAT\0"
// Dense (tensor-core) blocks draw along the unit axis of one chain: counter
// (chain, row/4, sweep, salt) gives the spins of four consecutive rows, or
// the normals of four gaussian rows: Box-Muller on words 2p, 2p+1 gives rows
// 4j+2p (r cos theta) and 4j+2p+1 (r sin theta).
constexpr uint32_t kSaltDenseSpin = 0x44535049u;   // "DSPI"
constexpr uint32_t kSaltDenseGauss = 0x44474155u;  // "DGAU"
// Lattice (threshold-table) spin draws use split uniforms: the 23-bit draw
// m = (h << 7) | f takes its top 16 bits h from a counter shared by eight
// draws (two per 32-bit word: low half first) and its low 7 bits f from a
// counter of its own, (chain, row, sweep, "LREF") word 0 >> 25.  A draw
// compares h with the threshold's top 16 bits first and needs f only when
// they are equal (probability 2^-16), so a lattice site costs an eighth of a
// Philox call instead of a quarter; m is uniform on [0, 2^23) as before.
constexpr uint32_t kSaltLatticeSpin = 0x4C535049u;    // "LSPI"
constexpr uint32_t kSaltLatticeRefill = 0x4C524546u;  // "LREF"
// Bit-sliced lattice draws: plane b of a 32-site group from salt "LPL0" + b / 4.
constexpr uint32_t kSaltLatticePlanes = 0x4C504C30u;  // "LPL0"
// Chunks of four planes the bit-sliced kernels draw before testing for ties.
#ifndef TTHRML_PLANES_EAGER
#define TTHRML_PLANES_EAGER 3
#endif

struct u32x4 {
  uint32_t x, y, z, w;
};

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as
// easy as 1, 2, 3", SC'11): ten rounds of two 32x32->64 multiplies with the
// published multipliers and Weyl key increments.
__host__ __device__ __forceinline__ u32x4 philox4x32_10(u32x4 c, uint32_t k0, uint32_t k1) {
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int r = 0; r < 10; ++r) {
#ifdef __CUDA_ARCH__
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
#else
    const uint64_t p0 = (uint64_t)0xD2511F53u * c.x, p1 = (uint64_t)0xCD9E8D57u * c.z;
    const uint32_t lo0 = (uint32_t)p0, hi0 = (uint32_t)(p0 >> 32);
    const uint32_t lo1 = (uint32_t)p1, hi1 = (uint32_t)(p1 >> 32);
#endif
    c = u32x4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// Philox4x32-10 with its ten round keys precomputed once per thread: the key
// schedule of a persistent kernel is loop-invariant, so each call is left
// with the multiplies and XORs of the rounds.
struct PhiloxKeys {
  uint32_t a[10], b[10];
};
__host__ __device__ __forceinline__ PhiloxKeys philox_keys(uint32_t k0, uint32_t k1) {
  PhiloxKeys k;
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int r = 0; r < 10; ++r) {
    k.a[r] = k0 + (uint32_t)r * 0x9E3779B9u;
    k.b[r] = k1 + (uint32_t)r * 0xBB67AE85u;
  }
  return k;
}
__host__ __device__ __forceinline__ u32x4 philox4x32_10(u32x4 c, const PhiloxKeys& k) {
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int r = 0; r < 10; ++r) {
#if defined(__CUDA_ARCH__) && !defined(TTHRML_PHILOX_WIDE)
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
#else
    const uint64_t p0 = (uint64_t)0xD2511F53u * c.x, p1 = (uint64_t)0xCD9E8D57u * c.z;
    const uint32_t lo0 = (uint32_t)p0, hi0 = (uint32_t)(p0 >> 32);
    const uint32_t lo1 = (uint32_t)p1, hi1 = (uint32_t)(p1 >> 32);
#endif
    c = u32x4{hi1 ^ c.y ^ k.a[r], lo1, hi0 ^ c.w ^ k.b[r], lo0};
  }
  return c;
}

// n / d for 0 <= n < 2^31 as (umulhi(n, m) + n) >> l with a host-computed
// magic number (Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994).
struct FastDiv {
  uint32_t d, m, l;
};
inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, l};
}
#ifdef __CUDACC__
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) { return (__umulhi(n, f.m) + n) >> f.l; }
#endif

__host__ __device__ __forceinline__ uint32_t word_of(const u32x4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// Uniform on the open interval (0, 1): odd multiples of 2^-24 built from the
// top 23 bits, exact in float32 and identical on host and device.
__host__ __device__ __forceinline__ float uniform_open(uint32_t bits) {
  return (float)(((bits >> 9) << 1) | 1u) * 5.9604644775390625e-08f;  // 2^-24
}

#ifdef __CUDACC__
// Open uniform (2m+1)/2^24, m = bits >> 9, built without an int->float
// conversion: 1 + m/2^23 from the mantissa, minus (1 - 2^-24); both steps exact,
// so the value equals uniform_open(bits) bit for bit.
__device__ __forceinline__ float uniform_open_alu(uint32_t bits) {
  return __uint_as_float(0x3F800000u | (bits >> 9)) - 0.99999994039535522461f;
}
#endif

__host__ __device__ __forceinline__ uint32_t seed_lo(uint64_t s) { return (uint32_t)s; }
__host__ __device__ __forceinline__ uint32_t seed_hi(uint64_t s) { return (uint32_t)(s >> 32); }

#ifdef __CUDACC__
// PTX prmt in its default mode: each selector nibble picks one of the eight
// bytes of {b, a} (low 3 bits); with the nibble's top bit set the picked
// byte's sign bit is replicated over the result byte.
__device__ __forceinline__ uint32_t prmt_sign(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Bit-sliced lattice decision for 32 spins at once (count-symmetric threshold
// tables).  L, R, U, D: the spins' left / right / up / down neighbour bits
// (set = -1).  MS[i][n]: bit 23 - i of the count-n threshold as a 0 / ~0 mask.
// The draw m of each spin (23 bits, bit 22 - b from word b % 4 of counter
// (c0, c1, sweep, "LPL0" + b / 4), the spin's own bit position) is compared
// with T(n) from the top bit down; the result has a bit set where m >= T(n),
// i.e. where the spin goes to -1.  The first TTHRML_PLANES_EAGER chunks of four
// planes are drawn unconditionally, the rest only while some spin is tied.
// The bit-sliced decision of planes_decide in steps, for kernels that finish the rare undecided words
// later (same planes in the same order, so the same result): PlaneState holds the neighbour-count
// planes and the decided / tied masks; planes_chunk applies the four planes of Philox chunk ch.
struct PlaneState {
  uint32_t n0, n1, n2, lt, eq;
};
__device__ __forceinline__ uint32_t plane_tbit(const uint32_t (*MS)[8], const PlaneState& s, int i) {
  const uint4 a = *reinterpret_cast<const uint4*>(&MS[i][0]);
  const uint32_t m4 = MS[i][4];
  const uint32_t lo = (s.n0 & a.y) | (~s.n0 & a.x), hi = (s.n0 & a.w) | (~s.n0 & a.z);
  const uint32_t g = (s.n1 & hi) | (~s.n1 & lo);
  return (s.n2 & m4) | (~s.n2 & g);
}
__device__ __forceinline__ void plane_counts(PlaneState& s, uint32_t L, uint32_t R, uint32_t U, uint32_t D) {
  const uint32_t s1 = L ^ R, k1 = L & R, s2 = U ^ D, k2 = U & D;
  const uint32_t t = s1 & s2;
  s.n0 = s1 ^ s2;
  s.n1 = k1 ^ k2 ^ t;
  s.n2 = (k1 & k2) | (t & (k1 | k2));
}
__device__ __forceinline__ void planes_begin(PlaneState& s, uint32_t L, uint32_t R, uint32_t U, uint32_t D,
                                             const uint32_t (*MS)[8]) {
  plane_counts(s, L, R, U, D);
  s.lt = plane_tbit(MS, s, 0);
  s.eq = ~s.lt;
}
__device__ __forceinline__ void planes_chunk(PlaneState& s, const uint32_t (*MS)[8], const u32x4& r, int ch) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int b = 4 * ch + q;
    if (b < 23) {
      const uint32_t tb = plane_tbit(MS, s, b + 1), ub = word_of(r, q);
      s.lt |= s.eq & tb & ~ub;
      s.eq &= ~(tb ^ ub);
    }
  }
}

// The eager chunks' Philox words of one word's draws (they depend on the counter only, so a kernel may
// compute them before the state they decide is ready).
__device__ __forceinline__ void planes_eager(u32x4 (&pre)[TTHRML_PLANES_EAGER], uint32_t c0, uint32_t c1,
                                             uint32_t sweep, const PhiloxKeys& keys) {
#pragma unroll
  for (int ch = 0; ch < TTHRML_PLANES_EAGER; ++ch)
    pre[ch] = philox4x32_10(u32x4{c0, c1, sweep, kSaltLatticePlanes + (uint32_t)ch}, keys);
}

template <bool PRE>
__device__ __forceinline__ uint32_t planes_decide_impl(uint32_t L, uint32_t R, uint32_t U, uint32_t D,
                                                       const uint32_t (*MS)[8], const u32x4* pre, uint32_t c0,
                                                       uint32_t c1, uint32_t sweep, const PhiloxKeys& keys) {
  // n = L + R + U + D in bit-planes n0, n1, n2 (n2 set only for n = 4)
  const uint32_t s1 = L ^ R, k1 = L & R, s2 = U ^ D, k2 = U & D;
  const uint32_t n0 = s1 ^ s2, t = s1 & s2;
  const uint32_t n1 = k1 ^ k2 ^ t, n2 = (k1 & k2) | (t & (k1 | k2));
  auto tbit = [&](int i) -> uint32_t {  // the threshold bit of every spin, from its count
    const uint4 a = *reinterpret_cast<const uint4*>(&MS[i][0]);
    const uint32_t m4 = MS[i][4];
    const uint32_t lo = (n0 & a.y) | (~n0 & a.x), hi = (n0 & a.w) | (~n0 & a.z);
    const uint32_t g = (n1 & hi) | (~n1 & lo);
    return (n2 & m4) | (~n2 & g);
  };
  uint32_t lt = tbit(0);  // decided "m < T" (only T = 2^23 so far)
  uint32_t eq = ~lt;      // still tied with T
  auto planes4 = [&](int ch) {
    const u32x4 r = (PRE && ch < TTHRML_PLANES_EAGER)
                        ? pre[ch]
                        : philox4x32_10(u32x4{c0, c1, sweep, kSaltLatticePlanes + (uint32_t)ch}, keys);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int b = 4 * ch + q;
      if (b < 23) {
        const uint32_t tb = tbit(b + 1), ub = word_of(r, q);
        lt |= eq & tb & ~ub;
        eq &= ~(tb ^ ub);
      }
    }
  };
#pragma unroll
  for (int ch = 0; ch < TTHRML_PLANES_EAGER; ++ch) planes4(ch);
#pragma unroll 1
  for (int ch = TTHRML_PLANES_EAGER; ch < 6 && eq; ++ch) planes4(ch);
  return ~lt;
}

__device__ __forceinline__ uint32_t planes_decide(uint32_t L, uint32_t R, uint32_t U, uint32_t D,
                                                  const uint32_t (*MS)[8], uint32_t c0, uint32_t c1, uint32_t sweep,
                                                  const PhiloxKeys& keys) {
  return planes_decide_impl<false>(L, R, U, D, MS, nullptr, c0, c1, sweep, keys);
}

// planes_decide with the eager chunks' words given (planes_eager of the same counter).
__device__ __forceinline__ uint32_t planes_decide_pre(uint32_t L, uint32_t R, uint32_t U, uint32_t D,
                                                      const uint32_t (*MS)[8], const u32x4 (&pre)[TTHRML_PLANES_EAGER],
                                                      uint32_t c0, uint32_t c1, uint32_t sweep,
                                                      const PhiloxKeys& keys) {
  return planes_decide_impl<true>(L, R, U, D, MS, pre, c0, c1, sweep, keys);
}

// Fills MS[24][8] (see planes_decide) from a 16-entry threshold table whose
// entry 2^n - 1 holds the count-n threshold; call with all threads, then sync.
__device__ __forceinline__ void planes_masks(uint32_t (*MS)[8], const uint32_t* __restrict__ thresholds) {
  if (threadIdx.x < 24 * 5) {
    const int i = threadIdx.x / 5, n = threadIdx.x - 5 * i;
    const uint32_t t = thresholds[(1u << n) - 1u];  // the pattern with the n lowest neighbours at -1
    MS[i][n] = ((t >> (23 - i)) & 1u) ? 0xFFFFFFFFu : 0u;
  }
}

// Byte-transposed 32-site masks (site s = 4j + k at bit 8k + j): the mask of
// sites s - 1 (e = the bit of site -1) and s + 1 (e = the bit of site 32).
__device__ __forceinline__ uint32_t sites_minus1(uint32_t M, uint32_t e) {
  return (M << 8) | ((M >> 23) & 0xFEu) | e;
}
__device__ __forceinline__ uint32_t sites_plus1(uint32_t M, uint32_t e) {
  return (M >> 8) | ((M << 23) & 0x7F000000u) | (e << 31);
}

// Categorical draw in Philox mode by inverse CDF from one uniform u, a sample
// of softmax(theta): e_k = 2^((theta_k - max theta) * log2 e) (ex2.approx),
// and the draw is the number of boundaries k < q - 1 that u reaches,
// u >= C_k / S with C_k = e_0 + ... + e_k and S = C_(q-1).  For u < 1/2 the
// boundaries are decided on head sums, C_k <= u*S; otherwise the categories
// are taken in reverse order, so the running sums are the tail sums T_(k+1) =
// e_(k+1) + ... + e_(q-1) (summed from the end), decided against (1 - u)*S
// (1 - u is exact in float32), and the count is mirrored.  Either way every
// boundary close to u is decided by a sum that is small where the decision is
// close, so the float32 error of a decision stays near 1e-6 in logit units at
// both ends of the CDF, inside the 1e-5 threshold band of the parity criteria;
// one pass of running sums and one compare per boundary serve both ends.
// Small QMAX (unrolled, registers) reverses over QMAX entries with e_k = 0
// past q, which leaves the same sums with leading zeros.
template <int QMAX>
__device__ __forceinline__ int categorical_icdf(const float (&theta)[QMAX], int q, float u) {
  constexpr bool kUnroll = QMAX <= 16;  // small bounds stay in registers
  float m = theta[0];
#pragma unroll(kUnroll ? QMAX : 1)
  for (int k = 1; k < QMAX; ++k)
    if (k < q) m = fmaxf(m, theta[k]);
  const float ml = m * 1.44269502162933349609375f;
  const bool low = u < 0.5f;
  float e[QMAX];
  int cnt = 0;
  if constexpr (kUnroll) {
#pragma unroll
    for (int k = 0; k < QMAX; ++k) {
      float v = 0.0f;
      if (k < q) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(v) : "f"(__fmaf_rn(theta[k], 1.44269502162933349609375f, -ml)));
      e[k] = v;
    }
    float h[QMAX];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < QMAX; ++j) {
      const float x = low ? e[j] : e[QMAX - 1 - j];
      s = j == 0 ? x : __fadd_rn(s, x);
      h[j] = s;
    }
    const float t = __fmul_rn(low ? u : 1.0f - u, s);
#pragma unroll
    for (int j = 0; j < QMAX - 1; ++j) cnt += h[j] <= t ? 1 : 0;
    return low ? cnt : QMAX - 1 - cnt;
  } else {
    for (int k = 0; k < q; ++k)
      asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e[k]) : "f"(__fmaf_rn(theta[k], 1.44269502162933349609375f, -ml)));
    float s = 0.0f;  // the total, in the order of the running sums below
    for (int j = 0; j < q; ++j) {
      const float x = low ? e[j] : e[q - 1 - j];
      s = j == 0 ? x : __fadd_rn(s, x);
    }
    const float t = __fmul_rn(low ? u : 1.0f - u, s);
    float h = 0.0f;
    for (int j = 0; j < q - 1; ++j) {
      const float x = low ? e[j] : e[q - 1 - j];
      h = j == 0 ? x : __fadd_rn(h, x);
      cnt += h <= t ? 1 : 0;
    }
    return low ? cnt : q - 1 - cnt;
  }
}

// The same inverse-CDF draw from unnormalised weights e_k (e_k = 0 for k >= q):
// the count of boundaries u reaches, decided on head sums for u < 1/2 and on
// tail sums against (1 - u) * S otherwise.  Returns -1 when the total S is not
// a normal float32 number (the weights underflowed), so the caller can decide
// from theta instead.
template <int QMAX>
__device__ __forceinline__ int categorical_icdf_weights(const float (&e)[QMAX], float u) {
  const bool low = u < 0.5f;
  float h[QMAX];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < QMAX; ++j) {
    const float x = low ? e[j] : e[QMAX - 1 - j];
    s = j == 0 ? x : __fadd_rn(s, x);
    h[j] = s;
  }
  if (!(s >= 1.17549435e-38f)) return -1;
  const float t = __fmul_rn(low ? u : 1.0f - u, s);
  int cnt = 0;
  if constexpr (QMAX == 8) {
    // h is non-decreasing, so the count of h[0..6] <= t is found by a three-step binary search
    // (the same count as the linear one): h[3], then h[1] or h[5], then one of h[0], h[2], h[4], h[6]
    const bool c2 = h[3] <= t;
    const bool c1 = (c2 ? h[5] : h[1]) <= t;
    const bool c0 = (c2 ? (c1 ? h[6] : h[4]) : (c1 ? h[2] : h[0])) <= t;
    cnt = (c2 ? 4 : 0) + (c1 ? 2 : 0) + (c0 ? 1 : 0);
  } else {
#pragma unroll
    for (int j = 0; j < QMAX - 1; ++j) cnt += h[j] <= t ? 1 : 0;
  }
  return low ? cnt : QMAX - 1 - cnt;
}

// Heat-bath spin decision in Philox mode: +1 with probability sigmoid(2*gamma)
// (thrml's SpinGibbsConditional; tt_thrml/compiler.py:321-324), written as
// u * (1 + exp(-2 gamma)) < 1 so a single exponential decides it.
__device__ __forceinline__ bool spin_up_philox(float gamma, uint32_t bits) {
  const float u = uniform_open(bits);
  return u * (1.0f + __expf(-2.0f * gamma)) < 1.0f;
}
#endif

}  // namespace tthrml
