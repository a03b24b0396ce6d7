// Device helpers shared by the sparse spin kernels (int8 and bit-packed state).
#pragma once

#include "common.cuh"

namespace tthrml {
namespace {

constexpr int kTableBits = 8;  // neighbours folded into one partial-sum table

// +1 with probability sigmoid(2*gamma): u * (1 + 2^(-2*gamma*log2(e))) < 1.
__device__ __forceinline__ bool spin_up_fast(float gamma, uint32_t bits) {
  const float u = uniform_open_alu(bits);
  float t;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(gamma * -2.8853900817779268f));
  return __fmaf_rn(u, t, u) < 1.0f;
}

template <int BYTES>
__device__ __forceinline__ void cp_async_bytes(void* smem_dst, const void* gmem_src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
  if constexpr (BYTES == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src));
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(d), "l"(gmem_src), "n"(BYTES));
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

struct RowInfo {
  int64_t r;   // block-local row
  int64_t e0;  // first term
  int32_t deg;
  int32_t col;  // lane k holds column k (k < 32)
  float w;      // lane k holds weight k
  float b;
};

__device__ __forceinline__ void load_row(int64_t r, int64_t n_rows, const int64_t* __restrict__ rp,
                                         const int32_t* __restrict__ cols, const float* __restrict__ vals,
                                         const float* __restrict__ bias, int lane, RowInfo& m) {
  if (r >= n_rows) return;
  m.r = r;
  m.e0 = __ldg(rp + r);
  m.deg = (int)(__ldg(rp + r + 1) - m.e0);
  const int n = m.deg < 32 ? m.deg : 32;
  m.col = lane < n ? __ldg(cols + m.e0 + lane) : 0;
  m.w = lane < n ? __ldg(vals + m.e0 + lane) : 0.0f;
  m.b = bias ? __ldg(bias + r) : 0.0f;
}

__device__ __forceinline__ float flip(float w, uint32_t sign) { return __uint_as_float(__float_as_uint(w) ^ sign); }

// Writes the 2^t partial-sum table of the row (t in 5..8) into T.
__device__ __forceinline__ void build_table(float* T, float wl, int t, int lane) {
  float w[kTableBits];
#pragma unroll
  for (int k = 0; k < kTableBits; ++k) w[k] = __shfl_sync(0xffffffffu, wl, k);
  const uint32_t l = (uint32_t)lane;
  float p = __fadd_rn(flip(w[0], (l & 1u) << 31), flip(w[1], ((l >> 1) & 1u) << 31));
  p = __fadd_rn(p, flip(w[2], ((l >> 2) & 1u) << 31));
  p = __fadd_rn(p, flip(w[3], ((l >> 3) & 1u) << 31));
  p = __fadd_rn(p, flip(w[4], ((l >> 4) & 1u) << 31));
  if (t == 5) {
    T[l] = p;
  } else {
    const float a0 = __fadd_rn(p, w[5]), a1 = __fadd_rn(p, -w[5]);
    if (t == 6) {
      T[l] = a0;
      T[l | 32] = a1;
    } else {
      const float b0 = __fadd_rn(a0, w[6]), b1 = __fadd_rn(a1, w[6]);
      const float b2 = __fadd_rn(a0, -w[6]), b3 = __fadd_rn(a1, -w[6]);
      if (t == 7) {
        T[l] = b0;
        T[l | 32] = b1;
        T[l | 64] = b2;
        T[l | 96] = b3;
      } else {
        T[l] = __fadd_rn(b0, w[7]);
        T[l | 32] = __fadd_rn(b1, w[7]);
        T[l | 64] = __fadd_rn(b2, w[7]);
        T[l | 96] = __fadd_rn(b3, w[7]);
        T[l | 128] = __fadd_rn(b0, -w[7]);
        T[l | 160] = __fadd_rn(b1, -w[7]);
        T[l | 192] = __fadd_rn(b2, -w[7]);
        T[l | 224] = __fadd_rn(b3, -w[7]);
      }
    }
  }
}

// 8x8 bit-matrix transpose of the bytes of (lo, hi): bit j of byte i moves to
// bit i of byte j (three masked swap rounds; Warren, "Hacker's Delight", 7-3).
__device__ __forceinline__ void transpose8x8(uint32_t& lo, uint32_t& hi) {
  uint32_t t;
  t = (lo ^ (lo >> 7)) & 0x00AA00AAu;
  lo = lo ^ t ^ (t << 7);
  t = (hi ^ (hi >> 7)) & 0x00AA00AAu;
  hi = hi ^ t ^ (t << 7);
  t = (lo ^ (lo >> 14)) & 0x0000CCCCu;
  lo = lo ^ t ^ (t << 14);
  t = (hi ^ (hi >> 14)) & 0x0000CCCCu;
  hi = hi ^ t ^ (t << 14);
  t = (lo ^ (hi << 4)) & 0xF0F0F0F0u;
  lo ^= t;
  hi ^= t >> 4;
}

}  // namespace
}  // namespace tthrml
