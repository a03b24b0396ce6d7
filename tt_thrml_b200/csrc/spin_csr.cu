// Sparse spin block kernel on int8 ±1 state, chain-innermost.
//
// One warp per (row, 32*VEC-chain slice): each lane owns VEC consecutive
// chains, so every neighbour fetch is one coalesced 32*VEC-byte read of the
// neighbour's state row.  The row's (col, weight) pairs are read once per warp
// with a coalesced load and broadcast by shuffles, and up to UNROLL neighbour
// rows are in flight before any is accumulated.  The accumulation itself runs
// in CSR order so the field is bit-identical to a sequential float32 sum of
// the reference's terms (tt_thrml/compiler.py:303-318).
#include "common.cuh"

namespace tthrml {
namespace {

template <int VEC>
struct Vec;
template <>
struct Vec<1> {
  using T = int8_t;
};
template <>
struct Vec<2> {
  using T = int16_t;
};
template <>
struct Vec<4> {
  using T = int32_t;
};
template <>
struct Vec<8> {
  using T = int2;
};
template <>
struct Vec<16> {
  using T = int4;
};

template <int VEC>
__device__ __forceinline__ void unpack(const typename Vec<VEC>::T& v, int8_t (&out)[VEC]) {
  const int8_t* p = reinterpret_cast<const int8_t*>(&v);
#pragma unroll
  for (int i = 0; i < VEC; ++i) out[i] = p[i];
}

template <int VEC, bool VARIATES>
__global__ void __launch_bounds__(256) k_spin_csr(const int64_t* __restrict__ row_ptr,
                                                  const int32_t* __restrict__ cols,
                                                  const float* __restrict__ vals,
                                                  const float* __restrict__ bias, int64_t row_start,
                                                  int64_t n_rows, int8_t* state, int64_t C,
                                                  int64_t chain_offset,
                                                  const float* __restrict__ variates,
                                                  int64_t variates_sweeps, uint64_t seed, uint32_t sweep_base,
                                                  const tthrml_run_ctl* __restrict__ ctl) {
  using V = typename Vec<VEC>::T;
  constexpr int UNROLL = 8;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t slices = C / (32 * VEC);
  const int64_t r = warp / slices;
  if (r >= n_rows) return;
  const int64_t c0 = (warp - r * slices) * (32 * VEC) + lane * VEC;
  const int64_t e0 = row_ptr[r], e1 = row_ptr[r + 1];
  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);

  float acc[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc[v] = 0.0f;

  for (int64_t eb = e0; eb < e1; eb += 32) {
    const int n = (int)min((int64_t)32, e1 - eb);
    const int32_t my_col = lane < n ? __ldg(cols + eb + lane) : 0;
    const float my_w = lane < n ? __ldg(vals + eb + lane) : 0.0f;
    for (int k0 = 0; k0 < n; k0 += UNROLL) {
      V sv[UNROLL];
      float w[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int32_t j = __shfl_sync(0xffffffffu, my_col, (k0 + u) & 31);
        w[u] = __shfl_sync(0xffffffffu, my_w, (k0 + u) & 31);
        if (k0 + u < n) sv[u] = *reinterpret_cast<const V*>(state + (int64_t)j * C + c0);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (k0 + u < n) {
          int8_t s[VEC];
          unpack<VEC>(sv[u], s);
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[v] = __fadd_rn(acc[v], __fmul_rn(w[u], (float)s[v]));
        }
      }
    }
  }

  const int64_t row = row_start + r;
  const float b = bias ? __ldg(bias + r) : 0.0f;
  int8_t out[VEC];
  if (VARIATES) {
    // the host never runs past variates_sweeps; the modulo keeps misuse in bounds
    const int64_t vs = (int64_t)(sweep % (uint32_t)(variates_sweeps > 0 ? variates_sweeps : 1));
    const float* lrow = variates + (vs * n_rows + r) * C + c0;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const float gamma = bias ? __fadd_rn(b, acc[v]) : acc[v];
      out[v] = __fmul_rn(2.0f, gamma) > __ldg(lrow + v) ? 1 : -1;
    }
  } else {
    const uint64_t sd = ctl ? ctl->seed : seed;
    const uint32_t k0 = seed_lo(sd), k1 = seed_hi(sd);
    const int64_t g0 = chain_offset + c0;
    if (VEC >= 4) {
#pragma unroll
      for (int v = 0; v < VEC; v += 4) {
        const u32x4 rr = philox4x32_10(u32x4{(uint32_t)((g0 + v) >> 2), (uint32_t)row, sweep, kSaltSpin}, k0, k1);
#pragma unroll
        for (int t = 0; t < 4 && v + t < VEC; ++t) {
          const float gamma = bias ? __fadd_rn(b, acc[v + t]) : acc[v + t];
          out[v + t] = spin_up_philox(gamma, word_of(rr, t)) ? 1 : -1;
        }
      }
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const int64_t gc = g0 + v;
        const u32x4 rr = philox4x32_10(u32x4{(uint32_t)(gc >> 2), (uint32_t)row, sweep, kSaltSpin}, k0, k1);
        const float gamma = bias ? __fadd_rn(b, acc[v]) : acc[v];
        out[v] = spin_up_philox(gamma, word_of(rr, (int)(gc & 3))) ? 1 : -1;
      }
    }
  }
  V packed;
  int8_t* pp = reinterpret_cast<int8_t*>(&packed);
#pragma unroll
  for (int v = 0; v < VEC; ++v) pp[v] = out[v];
  *reinterpret_cast<V*>(state + row * C + c0) = packed;
}

template <int VEC>
int launch(const int64_t* rp, const int32_t* cols, const float* vals, const float* bias, int64_t row_start,
           int64_t n_rows, int8_t* state, int64_t C, int64_t chain_offset, const float* variates,
           int64_t variates_sweeps, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, cudaStream_t s) {
  const int64_t warps = n_rows * (C / (32 * VEC));
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) {
    set_error("tthrml_spin_csr_step: block too large");
    return TTHRML_ERR_ARG;
  }
  if (variates)
    k_spin_csr<VEC, true><<<(unsigned)blocks, threads, 0, s>>>(rp, cols, vals, bias, row_start, n_rows, state, C,
                                                               chain_offset, variates, variates_sweeps, seed, sweep,
                                                               ctl);
  else
    k_spin_csr<VEC, false><<<(unsigned)blocks, threads, 0, s>>>(rp, cols, vals, bias, row_start, n_rows, state, C,
                                                                chain_offset, variates, variates_sweeps, seed, sweep,
                                                                ctl);
  return launch_status("k_spin_csr launch");
}

}  // namespace
}  // namespace tthrml

extern "C" int tthrml_spin_csr_step(const int64_t* row_ptr, const int32_t* cols, const float* vals,
                                    const float* bias, int64_t row_start, int64_t n_rows, int8_t* state,
                                    int64_t n_chains, int64_t chain_offset, const float* variates,
                                    int64_t variates_sweeps, uint64_t seed, uint32_t sweep,
                                    const tthrml_run_ctl* ctl, void* stream) {
  using namespace tthrml;
  if (n_rows == 0) return TTHRML_OK;
  if (!row_ptr || !cols || !vals || !state || n_rows < 0 || row_start < 0) {
    set_error("tthrml_spin_csr_step: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  if (n_chains <= 0 || n_chains % 32 || chain_offset % 4) {
    set_error("tthrml_spin_csr_step: n_chains must be a positive multiple of 32 and chain_offset a multiple of 4 "
              "(got %lld, %lld)", (long long)n_chains, (long long)chain_offset);
    return TTHRML_ERR_ARG;
  }
  if (((uintptr_t)state) % 16) {
    set_error("tthrml_spin_csr_step: state must be 16-byte aligned");
    return TTHRML_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t per_lane = n_chains / 32;
  if (per_lane % 16 == 0)
    return launch<16>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates, variates_sweeps, seed, sweep, ctl, s);
  if (per_lane % 8 == 0)
    return launch<8>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates, variates_sweeps, seed, sweep, ctl, s);
  if (per_lane % 4 == 0)
    return launch<4>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates, variates_sweeps, seed, sweep, ctl, s);
  if (per_lane % 2 == 0)
    return launch<2>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates, variates_sweeps, seed, sweep, ctl, s);
  return launch<1>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates, variates_sweeps, seed, sweep, ctl, s);
}
