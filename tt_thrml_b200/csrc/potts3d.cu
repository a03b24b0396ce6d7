// 3-D q-state Potts stencil kernel (checkerboard colour block of a periodic
// X x Y x Z lattice).
//
// State layout: the flat int8 state [rows][n_chains] (chain innermost) of the
// executor; colour block c holds the colour-c sites in increasing linear index
// L = (z*Y + y)*X + x, so site L sits at block row L/2.  One thread updates
// one 32-bit word of a row, i.e. four chains of one site: it loads the
// matching word of its six neighbour rows (x-, x+, y-, y+, z-, z+, all of the
// other colour), forms the q category fields
//   theta_k = ((b_k + (Jx[k][s_x-] + Jx[k][s_x+])) + (Jy[k][s_y-] + Jy[k][s_y+]))
//             + (Jz[k][s_z-] + Jz[k][s_z+])
// (interactions summed over their terms first, then accumulated in program
// order: tt_thrml/compiler.py:289-318), draws, and writes the word back.  Each
// CTA first tabulates the rounded pair sums P_a[s0][s1][k] = J_a[k][s0] +
// J_a[k][s1] in shared memory, so an axis costs one 32-byte lookup and q adds
// per chain; categories outside [0, q) select all-zero matrix rows, as the
// reference's one-hot selection gives them no weight.  Site coordinates come
// from 32-bit divisions by invariant integers (multiply-high and shift).
//
// Draws: variates mode takes argmax(theta + g) over uploaded Gumbels
// (tt_thrml/compiler.py:327-344, first maximum wins); Philox mode takes one
// uniform from counter (chain/4, row, sweep, "CAT") and draws by inverse CDF
// (categorical_icdf), exactly as the generic kernel does, so both kernels give
// identical states.
#include "common.cuh"

namespace tthrml {
namespace {

constexpr int kPottsThreads = 256;
constexpr int kPottsQ = 8;  // categories handled by this kernel
constexpr int kRows = kPottsQ + 1;  // matrix rows per neighbour category, the last one all zero
#ifndef TTHRML_POTTS_ROW_FLOATS
#define TTHRML_POTTS_ROW_FLOATS 12
#endif
// a pair-sum row holds kPottsQ floats padded to kRowFloats: rows 48 bytes apart
// spread the random per-lane row reads over all shared-memory banks
constexpr int kRowFloats = TTHRML_POTTS_ROW_FLOATS;
#ifndef TTHRML_POTTS_WIDE
#define TTHRML_POTTS_WIDE 1
#endif
#ifndef TTHRML_POTTS_WPT
#define TTHRML_POTTS_WPT 2  // chain words per thread when n_chains allows
#endif
#ifndef TTHRML_POTTS_EXP
#define TTHRML_POTTS_EXP 1  // Philox mode, q = 8: the exponential-table kernel
#endif
#ifndef TTHRML_POTTS_EXP_MINB
#define TTHRML_POTTS_EXP_MINB 2  // resident blocks per SM the exponential-table kernel is compiled for
#endif
#ifndef TTHRML_POTTS_V_UNROLL
#define TTHRML_POTTS_V_UNROLL 4  // chains of a word unrolled in the exponential-table kernel
#endif

// QC: the category count as a compile-time constant (8, the common case: no
// per-category predicates) or 0 (any q <= 8, read from the argument).
// WPT: chain words (4 chains each) per thread; 2 shares a site's coordinates,
// neighbour addresses and bias row between 8 chains.
template <bool VARIATES, int QC, int WPT>
__global__ void __launch_bounds__(kPottsThreads) k_potts3d(
    int8_t* state, int64_t C, int32_t X, int32_t Y, int32_t Z, FastDiv div_words, FastDiv div_x, FastDiv div_y,
    int32_t colour, int64_t target_row0, int64_t source_row0, const float* __restrict__ J,
    const float* __restrict__ bias, int32_t q_arg, int64_t chain_offset, const float* __restrict__ variates,
    int64_t variates_sweeps, uint64_t seed, uint32_t sweep_base, const tthrml_run_ctl* __restrict__ ctl) {
  const int q = QC ? QC : q_arg;
  // P[a][s0][s1][k] = J[a][k][s0] + J[a][k][s1] (float32), with J[a][k][s] = 0
  // for s >= q (rows kPottsQ: categories out of range) and for k >= q
  __shared__ __align__(16) float P[3][kRows][kRows][kRowFloats];
  for (int i = threadIdx.x; i < 3 * kRows * kRows * kRowFloats; i += blockDim.x) {
    const int k = i % kRowFloats, s1 = (i / kRowFloats) % kRows, s0 = (i / (kRowFloats * kRows)) % kRows;
    const int a = i / (kRowFloats * kRows * kRows);
    const float j0 = (s0 < q && k < q) ? J[((int64_t)a * q + k) * q + s0] : 0.0f;
    const float j1 = (s1 < q && k < q) ? J[((int64_t)a * q + k) * q + s1] : 0.0f;
    (&P[0][0][0][0])[i] = __fadd_rn(j0, j1);
  }
  __syncthreads();

  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  const uint32_t words = div_words.d;  // thread items per site
  const int64_t half = (int64_t)X * Y * Z / 2;
  const uint32_t items = (uint32_t)(half * words);  // < 2^31, checked by the host
  const uint32_t XY = (uint32_t)X * (uint32_t)Y;  // sites < 2^31, checked by the host: 32-bit coordinates
  const int64_t vs = VARIATES ? (int64_t)(sweep % (uint32_t)(variates_sweeps > 0 ? variates_sweeps : 1)) : 0;

  for (uint32_t it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
    const uint32_t r = fdiv(it, div_words);
    const uint32_t w = (it - r * words) * WPT;  // first chain word of this thread
    const uint32_t even = 2 * r;
    const uint32_t yz = fdiv(even, div_x);
    const int32_t z = (int32_t)fdiv(yz, div_y);
    const int32_t y = (int32_t)yz - z * Y;
    const int32_t x = (int32_t)(even - yz * (uint32_t)X) + ((y + z + colour) & 1);
    const int32_t xm = x == 0 ? X - 1 : x - 1, xp = x == X - 1 ? 0 : x + 1;
    const int32_t ym = y == 0 ? Y - 1 : y - 1, yp = y == Y - 1 ? 0 : y + 1;
    const int32_t zm = z == 0 ? Z - 1 : z - 1, zp = z == Z - 1 ? 0 : z + 1;
    const uint32_t zXY = (uint32_t)z * XY, yX = (uint32_t)y * (uint32_t)X;
    uint32_t nb[6];  // neighbour block rows
    nb[0] = (zXY + yX + (uint32_t)xm) >> 1;
    nb[1] = (zXY + yX + (uint32_t)xp) >> 1;
    nb[2] = (zXY + (uint32_t)ym * (uint32_t)X + (uint32_t)x) >> 1;
    nb[3] = (zXY + (uint32_t)yp * (uint32_t)X + (uint32_t)x) >> 1;
    nb[4] = ((uint32_t)zm * XY + yX + (uint32_t)x) >> 1;
    nb[5] = ((uint32_t)zp * XY + yX + (uint32_t)x) >> 1;
    uint32_t nw[6][WPT];
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(state + (uint64_t)((uint32_t)source_row0 + nb[j]) *
                                                                          (uint32_t)C) + w;
      if (WPT == 4) {
        const uint4 v4 = __ldg(reinterpret_cast<const uint4*>(src));
        nw[j][0] = v4.x;
        nw[j][1 % WPT] = v4.y;
        nw[j][2 % WPT] = v4.z;
        nw[j][3 % WPT] = v4.w;
      } else if (WPT == 2) {
        const uint2 v2 = __ldg(reinterpret_cast<const uint2*>(src));
        nw[j][0] = v2.x;
        nw[j][WPT - 1] = v2.y;
      } else {
        nw[j][0] = __ldg(src);
      }
    }

    float b[kPottsQ];
    if (QC == kPottsQ) {  // the site's bias row as two 16-byte loads (the host checks the alignment)
      const float4* bp = reinterpret_cast<const float4*>(bias + (size_t)r * kPottsQ);
      const float4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
      b[0] = b0.x, b[1] = b0.y, b[2] = b0.z, b[3] = b0.w, b[4] = b1.x, b[5] = b1.y, b[6] = b1.z, b[7] = b1.w;
    } else {
#pragma unroll
      for (int k = 0; k < kPottsQ; ++k) b[k] = k < q ? __ldg(bias + r * q + k) : 0.0f;
    }

    const int64_t row = target_row0 + r;
    uint32_t out[WPT];
#pragma unroll
    for (int ww = 0; ww < WPT; ++ww) {
    out[ww] = 0u;
    u32x4 rr{0u, 0u, 0u, 0u};
    if (!VARIATES)
      rr = philox4x32_10(u32x4{(uint32_t)((chain_offset >> 2) + w + ww), (uint32_t)row, sweep, kSaltCat}, keys);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      float theta[kPottsQ];
#pragma unroll
      for (int k = 0; k < kPottsQ; ++k) theta[k] = b[k];
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const uint32_t s0 = min(__byte_perm(nw[2 * a][ww], 0u, 0x4440u + v), (uint32_t)kPottsQ);
        const uint32_t s1 = min(__byte_perm(nw[2 * a + 1][ww], 0u, 0x4440u + v), (uint32_t)kPottsQ);
        const float4* pp = reinterpret_cast<const float4*>(&P[a][s0][s1][0]);
        const float4 p0 = pp[0], p1 = pp[1];
        theta[0] = __fadd_rn(theta[0], p0.x);
        theta[1] = __fadd_rn(theta[1], p0.y);
        theta[2] = __fadd_rn(theta[2], p0.z);
        theta[3] = __fadd_rn(theta[3], p0.w);
        theta[4] = __fadd_rn(theta[4], p1.x);
        theta[5] = __fadd_rn(theta[5], p1.y);
        theta[6] = __fadd_rn(theta[6], p1.z);
        theta[7] = __fadd_rn(theta[7], p1.w);
      }
      int cat;
      if (VARIATES) {
        const float* g = variates + ((vs * half + r) * q) * C + 4 * (w + ww) + v;
        cat = 0;
        float best = 0.0f;
#pragma unroll
        for (int k = 0; k < kPottsQ; ++k) {
          if (k < q) {
            const float val = __fadd_rn(theta[k], __ldg(g + (int64_t)k * C));
            if (k == 0 || val > best) {
              best = val;
              cat = k;
            }
          }
        }
      } else {
        cat = categorical_icdf(theta, q, uniform_open(word_of(rr, v)));
      }
      out[ww] |= (uint32_t)cat << (8 * v);
    }
    }
    uint32_t* dst = reinterpret_cast<uint32_t*>(state + row * C) + w;
    if (WPT == 4)
      *reinterpret_cast<uint4*>(dst) = make_uint4(out[0], out[1 % WPT], out[2 % WPT], out[3 % WPT]);
    else if (WPT == 2)
      *reinterpret_cast<uint2*>(dst) = make_uint2(out[0], out[WPT - 1]);
    else
      *dst = out[0];
  }
}

// ---------------------------------------------------------------------------
// Philox-mode kernel on exponential tables.
//
// The inverse-CDF draw needs the unnormalised weights e^(theta_k) only up to
// a common factor per site and chain, and
//   e^(theta_k) = e^(b_k) * e^(Px_k) * e^(Py_k) * e^(Pz_k)
// with P_a = J_a[k][s-] + J_a[k][s+] the pair sum of axis a.  Each CTA
// tabulates E_a[s0][s1][k] = e^(P_a[s0][s1][k] - max_k P_a[s0][s1][.]) (every
// row's largest entry is 1, so products cannot overflow), and a thread turns
// its site's bias row into e^(b_k - max b) once for its 8 chains.  A chain's
// weights are then three 8-wide products of table rows and no exponential at
// all (the theta kernel above evaluates 8 per chain).  The weights are those
// of the reference's theta up to float32 rounding (a few 1e-7 relative, i.e.
// decisions move by ~1e-6 in logit units, inside the threshold band).  When
// the normalised product underflows (couplings spanning more than ~80 in
// theta), the chain falls back to theta from the matrices and the ex2 draw.
//
// Shared-memory layout: a row of 8 floats is two 16-byte chunks, each stored
// 8 times, [axis][s0][s1][chunk][copy][4 floats]; lane l reads copy l % 8, and
// a quarter-warp (the 8 lanes one 16-byte load serves at a time) then always
// touches 8 different bank groups: the lookups are free of bank conflicts.
// The fallback draw: theta of one chain from the matrices and the bias row (global memory), then the
// inverse-CDF draw with exponentials (categorical_icdf).
template <int WPT>
__device__ __forceinline__ int potts_theta_draw(const uint32_t (&nw)[6][WPT], int ww, int v,
                                                const float* __restrict__ J, const float* __restrict__ bias,
                                                uint32_t r, int q, float u) {
  float theta[kPottsQ];
#pragma unroll
  for (int k = 0; k < kPottsQ; ++k) {
    float acc = k < q ? __ldg(bias + (size_t)r * kPottsQ + k) : 0.0f;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const uint32_t s0 = __byte_perm(nw[2 * a][ww], 0u, 0x4440u + v);
      const uint32_t s1 = __byte_perm(nw[2 * a + 1][ww], 0u, 0x4440u + v);
      const float j0 = (s0 < (uint32_t)q && k < q) ? __ldg(J + (a * q + k) * q + s0) : 0.0f;
      const float j1 = (s1 < (uint32_t)q && k < q) ? __ldg(J + (a * q + k) * q + s1) : 0.0f;
      acc = __fadd_rn(acc, __fadd_rn(j0, j1));
    }
    theta[k] = acc;
  }
  return categorical_icdf(theta, q, u);
}

constexpr int kPottsVUnroll = TTHRML_POTTS_V_UNROLL;
#ifndef TTHRML_POTTS_EXP_COPIES
#define TTHRML_POTTS_EXP_COPIES 8
#endif
constexpr int kExpCopies = TTHRML_POTTS_EXP_COPIES;
// one table row: 2 chunks x copies x 4 floats; a single copy is padded to 3 chunks (rows 48 bytes apart)
constexpr int kExpRowFloats = kExpCopies == 1 ? 12 : 2 * kExpCopies * 4;
constexpr int kExpSmemBytes = 3 * kRows * kRows * kExpRowFloats * 4;

#ifndef TTHRML_POTTS_F32X2
#define TTHRML_POTTS_F32X2 1  // packed f32x2 category products (0: scalar)
#endif

// e^(b_k - max b) of one site's bias row (16-byte loads; the host checks the alignment), k < q, else 0.
__device__ __forceinline__ void site_bias_weights(const float* __restrict__ bias, int64_t r, int32_t q,
                                                  float (&eb)[kPottsQ]) {
  float b[kPottsQ];
  const float4* bp = reinterpret_cast<const float4*>(bias + (size_t)r * kPottsQ);
  const float4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
  b[0] = b0.x, b[1] = b0.y, b[2] = b0.z, b[3] = b0.w, b[4] = b1.x, b[5] = b1.y, b[6] = b1.z, b[7] = b1.w;
  float mb = b[0];
#pragma unroll
  for (int k = 1; k < kPottsQ; ++k)
    if (k < q) mb = fmaxf(mb, b[k]);
  const float ml = mb * 1.44269502162933349609375f;
#pragma unroll
  for (int k = 0; k < kPottsQ; ++k) {
    float v = 0.0f;
    if (k < q) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(v) : "f"(__fmaf_rn(b[k], 1.44269502162933349609375f, -ml)));
    eb[k] = v;
  }
}

// The bias weights of every site once (they do not change between sweeps): the sweep kernel then reads
// e^(b - max b) instead of computing it per site and launch, with the same values.
__global__ void k_potts_bias_weights(const float* __restrict__ bias, int64_t n, int32_t q, float* __restrict__ w) {
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
    float eb[kPottsQ];
    site_bias_weights(bias, r, q, eb);
    float4* dst = reinterpret_cast<float4*>(w + (size_t)r * kPottsQ);
    dst[0] = make_float4(eb[0], eb[1], eb[2], eb[3]);
    dst[1] = make_float4(eb[4], eb[5], eb[6], eb[7]);
  }
}

// Bytes of x clamped to at most c (each byte unsigned).
__device__ __forceinline__ uint32_t clamp_bytes(uint32_t x, uint32_t c) {
  uint32_t y = 0u;
#pragma unroll
  for (int k = 0; k < 4; ++k) y |= min((x >> (8 * k)) & 0xFFu, c) << (8 * k);
  return y;
}

template <int WPT>
__global__ void __launch_bounds__(kPottsThreads, TTHRML_POTTS_EXP_MINB) k_potts3d_exp(
    int8_t* state, int64_t C, int32_t X, int32_t Y, int32_t Z, FastDiv div_words, FastDiv div_x, FastDiv div_y,
    int32_t colour, int64_t target_row0, int64_t source_row0, const float* __restrict__ J,
    const float* __restrict__ bias, int32_t q, int64_t chain_offset, uint64_t seed, uint32_t sweep_base,
    const tthrml_run_ctl* __restrict__ ctl, const float* __restrict__ bias_w) {
  extern __shared__ __align__(16) float E[];  // [3][kRows][kRows][2][kExpCopies][4]
  for (int row = threadIdx.x; row < 3 * kRows * kRows; row += blockDim.x) {
    const int s1 = row % kRows, s0 = (row / kRows) % kRows, a = row / (kRows * kRows);
    float p[kPottsQ];
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kPottsQ; ++k) {
      const float j0 = (s0 < q && k < q) ? J[((int64_t)a * q + k) * q + s0] : 0.0f;
      const float j1 = (s1 < q && k < q) ? J[((int64_t)a * q + k) * q + s1] : 0.0f;
      p[k] = __fadd_rn(j0, j1);
      if (k < q) m = fmaxf(m, p[k]);
    }
    float e[kPottsQ];
#pragma unroll
    for (int k = 0; k < kPottsQ; ++k) e[k] = k < q ? expf(p[k] - m) : 0.0f;
    float4* dst = reinterpret_cast<float4*>(E + (size_t)row * kExpRowFloats);
#pragma unroll
    for (int c = 0; c < kExpCopies; ++c) {
      dst[c] = make_float4(e[0], e[1], e[2], e[3]);
      dst[kExpCopies + c] = make_float4(e[4], e[5], e[6], e[7]);
    }
  }
  __syncthreads();

  const int copy = threadIdx.x & (kExpCopies - 1);
  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const PhiloxKeys keys = philox_keys(seed_lo(sd), seed_hi(sd));
  const uint32_t words = div_words.d;
  const int64_t half = (int64_t)X * Y * Z / 2;
  const uint32_t items = (uint32_t)(half * words);
  const uint32_t XY = (uint32_t)X * (uint32_t)Y;

  for (uint32_t it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
    const uint32_t r = fdiv(it, div_words);
    const uint32_t w = (it - r * words) * WPT;
    const uint32_t even = 2 * r;
    const uint32_t yz = fdiv(even, div_x);
    const int32_t z = (int32_t)fdiv(yz, div_y);
    const int32_t y = (int32_t)yz - z * Y;
    const int32_t x = (int32_t)(even - yz * (uint32_t)X) + ((y + z + colour) & 1);
    const int32_t xm = x == 0 ? X - 1 : x - 1, xp = x == X - 1 ? 0 : x + 1;
    const int32_t ym = y == 0 ? Y - 1 : y - 1, yp = y == Y - 1 ? 0 : y + 1;
    const int32_t zm = z == 0 ? Z - 1 : z - 1, zp = z == Z - 1 ? 0 : z + 1;
    const uint32_t zXY = (uint32_t)z * XY, yX = (uint32_t)y * (uint32_t)X;
    uint32_t nb[6];
    nb[0] = (zXY + yX + (uint32_t)xm) >> 1;
    nb[1] = (zXY + yX + (uint32_t)xp) >> 1;
    nb[2] = (zXY + (uint32_t)ym * (uint32_t)X + (uint32_t)x) >> 1;
    nb[3] = (zXY + (uint32_t)yp * (uint32_t)X + (uint32_t)x) >> 1;
    nb[4] = ((uint32_t)zm * XY + yX + (uint32_t)x) >> 1;
    nb[5] = ((uint32_t)zp * XY + yX + (uint32_t)x) >> 1;
    uint32_t nw[6][WPT];
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(state + (uint64_t)((uint32_t)source_row0 + nb[j]) *
                                                                          (uint32_t)C) + w;
      if (WPT == 4) {
        const uint4 v4 = __ldg(reinterpret_cast<const uint4*>(src));
        nw[j][0] = v4.x;
        nw[j][1 % WPT] = v4.y;
        nw[j][2 % WPT] = v4.z;
        nw[j][3 % WPT] = v4.w;
      } else if (WPT == 2) {
        const uint2 v2 = __ldg(reinterpret_cast<const uint2*>(src));
        nw[j][0] = v2.x;
        nw[j][WPT - 1] = v2.y;
      } else {
        nw[j][0] = __ldg(src);
      }
    }
    // the site's bias row as e^(b_k - max b): from the precomputed table, or computed here
    float eb[kPottsQ];
    if (bias_w) {
      const float4* wp = reinterpret_cast<const float4*>(bias_w + (size_t)r * kPottsQ);
      const float4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
      eb[0] = w0.x, eb[1] = w0.y, eb[2] = w0.z, eb[3] = w0.w, eb[4] = w1.x, eb[5] = w1.y, eb[6] = w1.z, eb[7] = w1.w;
    } else {
      site_bias_weights(bias, r, q, eb);
    }

    const int64_t row = target_row0 + r;
    uint32_t out[WPT];
#pragma unroll
    for (int ww = 0; ww < WPT; ++ww) {
      out[ww] = 0u;
      const u32x4 rr =
          philox4x32_10(u32x4{(uint32_t)((chain_offset >> 2) + w + ww), (uint32_t)row, sweep, kSaltCat}, keys);
      // table rows of the 4 chains of this word, one byte each: 9 * s0 + s1 per axis (<= 80, so the
      // byte-wise sums never carry), neighbour categories above kPottsQ taken as the zero row kPottsQ
      uint32_t chk = 0u;
#pragma unroll
      for (int j = 0; j < 6; ++j) chk |= nw[j][ww] | (nw[j][ww] + 0x77777777u);  // bit 7 of a byte: >= 9
      const bool clean = !(chk & 0x80808080u);
      uint32_t I[3];
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        uint32_t s0w = nw[2 * a][ww], s1w = nw[2 * a + 1][ww];
        if (!clean) {  // only with neighbour categories outside [0, kPottsQ]
          s0w = clamp_bytes(s0w, kPottsQ);
          s1w = clamp_bytes(s1w, kPottsQ);
        }
        I[a] = (s0w << 3) + s0w + s1w;
      }
#pragma unroll kPottsVUnroll
      for (int v = 0; v < 4; ++v) {
        float e[kPottsQ];
#pragma unroll
        for (int k = 0; k < kPottsQ; ++k) e[k] = eb[k];
#pragma unroll
        for (int a = 0; a < 3; ++a) {
          const uint32_t idx = __byte_perm(I[a], 0u, 0x4440u + v);
          const float4* pp = reinterpret_cast<const float4*>(
              E + (size_t)(a * kRows * kRows + (int)idx) * kExpRowFloats) + copy;
          const float4 p0 = pp[0], p1 = pp[kExpCopies];
#if TTHRML_POTTS_F32X2  // two categories per packed multiply (each product rounded as alone)
          const float2 q01 = __fmul2_rn(make_float2(e[0], e[1]), make_float2(p0.x, p0.y));
          const float2 q23 = __fmul2_rn(make_float2(e[2], e[3]), make_float2(p0.z, p0.w));
          const float2 q45 = __fmul2_rn(make_float2(e[4], e[5]), make_float2(p1.x, p1.y));
          const float2 q67 = __fmul2_rn(make_float2(e[6], e[7]), make_float2(p1.z, p1.w));
          e[0] = q01.x, e[1] = q01.y, e[2] = q23.x, e[3] = q23.y;
          e[4] = q45.x, e[5] = q45.y, e[6] = q67.x, e[7] = q67.y;
#else
          e[0] = __fmul_rn(e[0], p0.x);
          e[1] = __fmul_rn(e[1], p0.y);
          e[2] = __fmul_rn(e[2], p0.z);
          e[3] = __fmul_rn(e[3], p0.w);
          e[4] = __fmul_rn(e[4], p1.x);
          e[5] = __fmul_rn(e[5], p1.y);
          e[6] = __fmul_rn(e[6], p1.z);
          e[7] = __fmul_rn(e[7], p1.w);
#endif
        }
        const float u = uniform_open_alu(word_of(rr, v));
        int cat = categorical_icdf_weights<kPottsQ>(e, u);
        if (cat < 0) cat = potts_theta_draw(nw, ww, v, J, bias, r, q, u);  // the weights underflowed
        out[ww] |= (uint32_t)cat << (8 * v);
      }
    }
    uint32_t* dst = reinterpret_cast<uint32_t*>(state + row * C) + w;
    if (WPT == 4)
      *reinterpret_cast<uint4*>(dst) = make_uint4(out[0], out[1 % WPT], out[2 % WPT], out[3 % WPT]);
    else if (WPT == 2)
      *reinterpret_cast<uint2*>(dst) = make_uint2(out[0], out[WPT - 1]);
    else
      *dst = out[0];
  }
}

template <int WPT>
int launch_potts_exp(int8_t* state, int64_t C, int32_t X, int32_t Y, int32_t Z, int32_t colour, int64_t target_row0,
                     int64_t source_row0, const float* J, const float* bias, int32_t q, int64_t chain_offset,
                     uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, const float* bias_w, cudaStream_t s) {
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_potts3d_exp<WPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kExpSmemBytes);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_potts3d_exp<WPT>, kPottsThreads, kExpSmemBytes);
    if (e != cudaSuccess) return cuda_status(e, "k_potts3d_exp set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t items = (int64_t)X * Y * Z / 2 * (C / (4 * WPT));
  const int64_t need = (items + kPottsThreads - 1) / kPottsThreads;
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_potts3d_exp<WPT><<<grid, kPottsThreads, kExpSmemBytes, s>>>(
      state, C, X, Y, Z, make_fastdiv((uint32_t)(C / (4 * WPT))), make_fastdiv((uint32_t)X),
      make_fastdiv((uint32_t)Y), colour, target_row0, source_row0, J, bias, q, chain_offset, seed, sweep, ctl,
      bias_w);
  return launch_status("k_potts3d_exp launch");
}

template <bool VARIATES, int QC, int WPT>
int launch_potts(int8_t* state, int64_t C, int32_t X, int32_t Y, int32_t Z, int32_t colour, int64_t target_row0,
                 int64_t source_row0, const float* J, const float* bias, int32_t q, int64_t chain_offset,
                 const float* variates, int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                 const tthrml_run_ctl* ctl, cudaStream_t s) {
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_potts3d<VARIATES, QC, WPT>, kPottsThreads, 0);
    if (e != cudaSuccess) return cuda_status(e, "k_potts3d set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t items = (int64_t)X * Y * Z / 2 * (C / (4 * WPT));
  const int64_t need = (items + kPottsThreads - 1) / kPottsThreads;
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_potts3d<VARIATES, QC, WPT><<<grid, kPottsThreads, 0, s>>>(state, C, X, Y, Z,
                                                     make_fastdiv((uint32_t)(C / (4 * WPT))),
                                                     make_fastdiv((uint32_t)X), make_fastdiv((uint32_t)Y), colour,
                                                     target_row0, source_row0, J, bias, q, chain_offset, variates,
                                                     variates_sweeps, seed, sweep, ctl);
  return launch_status("k_potts3d launch");
}

}  // namespace
}  // namespace tthrml

namespace {
int potts3d_step(int8_t* state, int64_t n_chains, int32_t X, int32_t Y, int32_t Z, int32_t colour,
                 int64_t target_row0, int64_t source_row0, const float* J, const float* bias, int32_t q,
                 int64_t chain_offset, const float* variates, int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                 const tthrml_run_ctl* ctl, const float* bias_w, void* stream) {
  using namespace tthrml;
  if (!state || !J || !bias || X <= 0 || Y <= 0 || Z <= 0 || (X | Y | Z) & 1 || (colour != 0 && colour != 1)) {
    set_error("tthrml_potts3d_step: invalid arguments (dimensions must be positive and even, colour 0 or 1)");
    return TTHRML_ERR_ARG;
  }
  if (q < 1 || q > kPottsQ) {
    set_error("tthrml_potts3d_step: q must be in [1, %d] (got %d)", kPottsQ, (int)q);
    return TTHRML_ERR_ARG;
  }
  if (n_chains <= 0 || n_chains % 4 || chain_offset % 4 || ((uintptr_t)state % 16) ||
      (variates && ((uintptr_t)variates % 16))) {
    set_error("tthrml_potts3d_step: n_chains and chain_offset must be multiples of 4 and buffers 16-byte aligned");
    return TTHRML_ERR_ARG;
  }
  const int64_t half = (int64_t)X * Y * Z / 2;
  if (half * (n_chains / 4) >= (1ll << 31) || (int64_t)X * Y * Z >= (1ll << 31)) {
    set_error("tthrml_potts3d_step: sites x chain words must stay below 2^31 per launch");
    return TTHRML_ERR_UNSUPPORTED;
  }
  if (source_row0 + half >= (1ll << 31) || target_row0 + half >= (1ll << 31)) {
    set_error("tthrml_potts3d_step: block rows must stay below 2^31");
    return TTHRML_ERR_UNSUPPORTED;
  }
  if (target_row0 < 0 || source_row0 < 0 || (target_row0 < source_row0 + half && source_row0 < target_row0 + half)) {
    set_error("tthrml_potts3d_step: target and source blocks must be disjoint row ranges");
    return TTHRML_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
#define TTHRML_POTTS_LAUNCH(V, QC)                                                                              \
  return (wide ? launch_potts<V, QC, TTHRML_POTTS_WPT> : launch_potts<V, QC, 1>)(state, n_chains, X, Y, Z, colour,  \
                                                                  target_row0,                                    \
                                                                  source_row0, J, bias, q, chain_offset, variates, \
                                                                  variates_sweeps, seed, sweep, ctl, s)
  const bool q8 = q == kPottsQ && (uintptr_t)bias % 16 == 0;  // the q = 8 kernel reads 16-byte bias vectors
  const bool wide = TTHRML_POTTS_WIDE && n_chains % (4 * TTHRML_POTTS_WPT) == 0;  // several chain words per thread
  if (!variates && q8 && TTHRML_POTTS_EXP) {
    // 4 chain words (16 chains) per thread when the chain count allows: the site's neighbour addresses and
    // bias weights serve more chains (measured 2.35e11 -> 2.46e11 updates/s over 2 words at 64 chains)
    auto launch = n_chains % 16 == 0 ? launch_potts_exp<4> : (n_chains % 8 == 0 ? launch_potts_exp<2>
                                                                                  : launch_potts_exp<1>);
    return launch(state, n_chains, X, Y, Z, colour, target_row0, source_row0, J, bias, q, chain_offset, seed, sweep,
                  ctl, bias_w, s);
  }
  if (variates) {
    if (q8) TTHRML_POTTS_LAUNCH(true, kPottsQ);
    TTHRML_POTTS_LAUNCH(true, 0);
  }
  if (q8) TTHRML_POTTS_LAUNCH(false, kPottsQ);
  TTHRML_POTTS_LAUNCH(false, 0);
#undef TTHRML_POTTS_LAUNCH
}
}  // namespace

extern "C" int tthrml_potts3d_step(int8_t* state, int64_t n_chains, int32_t X, int32_t Y, int32_t Z, int32_t colour,
                                   int64_t target_row0, int64_t source_row0, const float* J, const float* bias,
                                   int32_t q, int64_t chain_offset, const float* variates, int64_t variates_sweeps,
                                   uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, void* stream) {
  return potts3d_step(state, n_chains, X, Y, Z, colour, target_row0, source_row0, J, bias, q, chain_offset, variates,
                      variates_sweeps, seed, sweep, ctl, nullptr, stream);
}

extern "C" int tthrml_potts3d_step_weights(int8_t* state, int64_t n_chains, int32_t X, int32_t Y, int32_t Z,
                                           int32_t colour, int64_t target_row0, int64_t source_row0, const float* J,
                                           const float* bias, int32_t q, int64_t chain_offset, const float* variates,
                                           int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                                           const tthrml_run_ctl* ctl, const float* bias_weights, void* stream) {
  if (!bias_weights || ((uintptr_t)bias_weights % 16)) {
    tthrml::set_error("tthrml_potts3d_step_weights: bias_weights must be a 16-byte aligned device array");
    return TTHRML_ERR_ARG;
  }
  return potts3d_step(state, n_chains, X, Y, Z, colour, target_row0, source_row0, J, bias, q, chain_offset, variates,
                      variates_sweeps, seed, sweep, ctl, bias_weights, stream);
}

extern "C" int tthrml_potts3d_bias_weights(const float* bias, int64_t n_sites, int32_t q, float* bias_weights,
                                           void* stream) {
  using namespace tthrml;
  if (!bias || !bias_weights || n_sites < 0 || q != kPottsQ || ((uintptr_t)bias % 16) ||
      ((uintptr_t)bias_weights % 16)) {
    set_error("tthrml_potts3d_bias_weights: q must be %d and both arrays 16-byte aligned [n_sites][%d]", kPottsQ,
              kPottsQ);
    return TTHRML_ERR_ARG;
  }
  if (n_sites == 0) return TTHRML_OK;
  const int64_t blocks = (n_sites + 255) / 256;
  k_potts_bias_weights<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, (cudaStream_t)stream>>>(bias, n_sites, q,
                                                                                                   bias_weights);
  return launch_status("k_potts_bias_weights launch");
}
