// State load / read-back / reduction kernels and the library's plain C entry
// points (error text, ABI version, host graph colouring).
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace tthrml {

namespace {
thread_local std::string g_last_error;
}

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

namespace {

// Tiled transpose between chain-innermost state [row][chain] and chain-major
// host order [chain][row]; 32x32 tiles through shared memory keep both sides
// coalesced.
template <typename S>
__global__ void k_decode(const S* __restrict__ state, int64_t C, int64_t row_start, int64_t n_rows, int out_kind,
                         void* __restrict__ out) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.x * 32, c0 = (int64_t)blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t r = r0 + k, c = c0 + threadIdx.x;
    if (r < n_rows && c < C) tile[k][threadIdx.x] = (float)state[(row_start + r) * C + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t c = c0 + k, r = r0 + threadIdx.x;
    if (r < n_rows && c < C) {
      const float v = tile[threadIdx.x][k];
      const int64_t o = c * n_rows + r;
      if (out_kind == 0)
        ((uint8_t*)out)[o] = v > 0.0f ? 1 : 0;
      else if (out_kind == 1)
        ((int32_t*)out)[o] = (int32_t)rintf(v);
      else
        ((float*)out)[o] = v;
    }
  }
}

template <typename I, typename S>
__global__ void k_encode(const I* __restrict__ in, int as_spin, int64_t n_rows, int64_t C, int64_t row_start,
                         S* __restrict__ state) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.x * 32, c0 = (int64_t)blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t c = c0 + k, r = r0 + threadIdx.x;
    if (r < n_rows && c < C) tile[threadIdx.x][k] = (float)in[c * n_rows + r];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t r = r0 + k, c = c0 + threadIdx.x;
    if (r < n_rows && c < C) {
      float v = tile[k][threadIdx.x];
      if (as_spin) v = v > 0.0f ? 1.0f : -1.0f;
      if (sizeof(S) == 1)
        state[(row_start + r) * C + c] = (S)__float2int_rn(v);
      else
        state[(row_start + r) * C + c] = (S)v;
    }
  }
}

// Per-chain sum over a row range: each thread owns one chain column and walks
// a strip of rows; one atomic per (strip, chain).
template <typename S>
__global__ void k_sum_rows(const S* __restrict__ state, int64_t C, int64_t row_start, int64_t n_rows,
                           int64_t rows_per_strip, double* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_strip;
  const int64_t r1 = min(n_rows, r0 + rows_per_strip);
  float acc = 0.0f;
  double dacc = 0.0;
  int64_t cnt = 0;
  for (int64_t r = r0; r < r1; ++r) {
    acc += (float)state[(row_start + r) * C + c];
    if (++cnt == 4096) {  // keep the float partial exact for ±1 / small integers
      dacc += acc;
      acc = 0.0f;
      cnt = 0;
    }
  }
  dacc += acc;
  if (r1 > r0) atomicAdd(out + c, dacc);
}

__global__ void k_ctl_advance(tthrml_run_ctl* c, uint32_t d) { c->sweep += d; }

// Bit-packed spin state (TTHRML_STATE_BITS): row r = W words, bit c set = chain c is -1.
template <typename I>
__global__ void k_encode_bits(const I* __restrict__ in, int64_t n_rows, int64_t W, int64_t row_start,
                              uint32_t* __restrict__ state) {
  __shared__ float tile[32][33];  // [chain][row]
  const int64_t r0 = (int64_t)blockIdx.x * 32, w = blockIdx.y;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t c = w * 32 + k, r = r0 + threadIdx.x;
    tile[k][threadIdx.x] = r < n_rows ? (float)in[c * n_rows + r] : 1.0f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {  // warp y packs row r0 + k
    const unsigned down = __ballot_sync(0xffffffffu, !(tile[threadIdx.x][k] > 0.0f));
    if (threadIdx.x == 0 && r0 + k < n_rows) state[(row_start + r0 + k) * W + w] = down;
  }
}

__global__ void k_decode_bits(const uint32_t* __restrict__ state, int64_t W, int64_t row_start, int64_t n_rows,
                              int out_kind, void* __restrict__ out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t C = W * 32;
  if (r >= n_rows) return;
  for (int64_t c = blockIdx.y; c < C; c += gridDim.y) {
    const bool up = ((state[(row_start + r) * W + (c >> 5)] >> (c & 31)) & 1u) == 0u;
    const int64_t o = c * n_rows + r;
    if (out_kind == 0)
      ((uint8_t*)out)[o] = up ? 1 : 0;
    else if (out_kind == 1)
      ((int32_t*)out)[o] = up ? 1 : -1;
    else
      ((float*)out)[o] = up ? 1.0f : -1.0f;
  }
}

__global__ void k_sum_rows_bits(const uint32_t* __restrict__ state, int64_t W, int64_t row_start, int64_t n_rows,
                                int64_t rows_per_strip, double* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= W * 32) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_strip;
  const int64_t r1 = min(n_rows, r0 + rows_per_strip);
  int64_t down = 0;
  for (int64_t r = r0; r < r1; ++r) down += (state[(row_start + r) * W + (c >> 5)] >> (c & 31)) & 1u;
  if (r1 > r0) atomicAdd(out + c, (double)((r1 - r0) - 2 * down));
}

}  // namespace
}  // namespace tthrml

using namespace tthrml;

extern "C" int tthrml_ctl_advance(tthrml_run_ctl* ctl, uint32_t delta, void* stream) {
  if (!ctl) {
    set_error("tthrml_ctl_advance: ctl is NULL");
    return TTHRML_ERR_ARG;
  }
  k_ctl_advance<<<1, 1, 0, (cudaStream_t)stream>>>(ctl, delta);
  return launch_status("k_ctl_advance launch");
}

extern "C" int tthrml_decode_rows(const void* state, int32_t dtype, int64_t C, int64_t row_start, int64_t n_rows,
                                  int32_t out_kind, void* out, void* stream) {
  if (n_rows == 0 || C == 0) return TTHRML_OK;
  if (!state || !out || n_rows < 0 || C < 0 || out_kind < 0 || out_kind > 2) {
    set_error("tthrml_decode_rows: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  dim3 grid((unsigned)((n_rows + 31) / 32), (unsigned)((C + 31) / 32)), block(32, 8);
  if ((n_rows + 31) / 32 > 0x7fffffffLL || (C + 31) / 32 > 65535) {
    set_error("tthrml_decode_rows: sizes exceed the launch grid");
    return TTHRML_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == TTHRML_STATE_BITS) {
    if (C % 32) {
      set_error("tthrml_decode_rows: bit-packed state needs n_chains %% 32 == 0");
      return TTHRML_ERR_ARG;
    }
    dim3 g((unsigned)((n_rows + 255) / 256), (unsigned)(C < 1024 ? C : 1024));
    k_decode_bits<<<g, 256, 0, s>>>((const uint32_t*)state, C / 32, row_start, n_rows, out_kind, out);
    return launch_status("k_decode_bits launch");
  }
  if (dtype == TTHRML_STATE_F32)
    k_decode<float><<<grid, block, 0, s>>>((const float*)state, C, row_start, n_rows, out_kind, out);
  else if (dtype == TTHRML_STATE_I8)
    k_decode<int8_t><<<grid, block, 0, s>>>((const int8_t*)state, C, row_start, n_rows, out_kind, out);
  else {
    set_error("tthrml_decode_rows: unknown dtype %d", dtype);
    return TTHRML_ERR_ARG;
  }
  return launch_status("k_decode launch");
}

extern "C" int tthrml_encode_rows(const void* in, int32_t in_dtype, int32_t as_spin, int64_t n_rows, int32_t dtype,
                                  int64_t C, int64_t row_start, void* state, void* stream) {
  if (n_rows == 0 || C == 0) return TTHRML_OK;
  if (!state || !in || n_rows < 0 || C < 0) {
    set_error("tthrml_encode_rows: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  if ((n_rows + 31) / 32 > 0x7fffffffLL || (C + 31) / 32 > 65535) {
    set_error("tthrml_encode_rows: sizes exceed the launch grid");
    return TTHRML_ERR_ARG;
  }
  dim3 grid((unsigned)((n_rows + 31) / 32), (unsigned)((C + 31) / 32)), block(32, 8);
  cudaStream_t s = (cudaStream_t)stream;
  const bool in_f32 = in_dtype == TTHRML_STATE_F32;
  if (!in_f32 && in_dtype != TTHRML_STATE_I8) {
    set_error("tthrml_encode_rows: unknown input dtype %d", in_dtype);
    return TTHRML_ERR_ARG;
  }
  if (dtype == TTHRML_STATE_BITS) {
    if (C % 32 || !as_spin) {
      set_error("tthrml_encode_rows: bit-packed state holds spins only and needs n_chains %% 32 == 0");
      return TTHRML_ERR_ARG;
    }
    dim3 g((unsigned)((n_rows + 31) / 32), (unsigned)(C / 32));
    if (in_f32)
      k_encode_bits<float><<<g, block, 0, s>>>((const float*)in, n_rows, C / 32, row_start, (uint32_t*)state);
    else
      k_encode_bits<int8_t><<<g, block, 0, s>>>((const int8_t*)in, n_rows, C / 32, row_start, (uint32_t*)state);
    return launch_status("k_encode_bits launch");
  }
  if (dtype == TTHRML_STATE_F32) {
    if (in_f32)
      k_encode<float, float><<<grid, block, 0, s>>>((const float*)in, as_spin, n_rows, C, row_start, (float*)state);
    else
      k_encode<int8_t, float><<<grid, block, 0, s>>>((const int8_t*)in, as_spin, n_rows, C, row_start, (float*)state);
  } else if (dtype == TTHRML_STATE_I8) {
    if (in_f32)
      k_encode<float, int8_t><<<grid, block, 0, s>>>((const float*)in, as_spin, n_rows, C, row_start, (int8_t*)state);
    else
      k_encode<int8_t, int8_t><<<grid, block, 0, s>>>((const int8_t*)in, as_spin, n_rows, C, row_start, (int8_t*)state);
  } else {
    set_error("tthrml_encode_rows: unknown dtype %d", dtype);
    return TTHRML_ERR_ARG;
  }
  return launch_status("k_encode launch");
}

extern "C" int tthrml_sum_rows(const void* state, int32_t dtype, int64_t C, int64_t row_start, int64_t n_rows,
                               double* out, void* stream) {
  if (n_rows == 0 || C == 0) return TTHRML_OK;
  if (!state || !out || n_rows < 0 || C < 0) {
    set_error("tthrml_sum_rows: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  const int threads = 128;
  const int64_t strips_wanted = 1184;  // 8 per SM on 148 SMs
  int64_t rows_per_strip = (n_rows + strips_wanted - 1) / strips_wanted;
  if (rows_per_strip < 64) rows_per_strip = 64;
  const int64_t strips = (n_rows + rows_per_strip - 1) / rows_per_strip;
  dim3 grid((unsigned)((C + threads - 1) / threads), (unsigned)strips);
  if (strips > 65535) {
    set_error("tthrml_sum_rows: too many strips");
    return TTHRML_ERR_ARG;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == TTHRML_STATE_BITS) {
    if (C % 32) {
      set_error("tthrml_sum_rows: bit-packed state needs n_chains %% 32 == 0");
      return TTHRML_ERR_ARG;
    }
    k_sum_rows_bits<<<grid, threads, 0, s>>>((const uint32_t*)state, C / 32, row_start, n_rows, rows_per_strip, out);
    return launch_status("k_sum_rows_bits launch");
  }
  if (dtype == TTHRML_STATE_F32)
    k_sum_rows<float><<<grid, threads, 0, s>>>((const float*)state, C, row_start, n_rows, rows_per_strip, out);
  else if (dtype == TTHRML_STATE_I8)
    k_sum_rows<int8_t><<<grid, threads, 0, s>>>((const int8_t*)state, C, row_start, n_rows, rows_per_strip, out);
  else {
    set_error("tthrml_sum_rows: unknown dtype %d", dtype);
    return TTHRML_ERR_ARG;
  }
  return launch_status("k_sum_rows launch");
}

namespace tthrml {
namespace {

// Value of (row, chain) for the moment products: spins as +-1 (spin_as_bool:
// 1 for +1, 0 for -1, the reference's boolean spin state), other states as
// stored (categorical index, gaussian value).
template <typename T>
__device__ __forceinline__ double moment_value(const T* state, int64_t C, int64_t row, int64_t chain, bool spin_row,
                                               int32_t spin_as_bool) {
  const double v = (double)state[row * C + chain];
  return spin_row && spin_as_bool ? (v > 0 ? 1.0 : 0.0) : v;
}
__device__ __forceinline__ double moment_value_bits(const uint32_t* state, int64_t W, int64_t row, int64_t chain,
                                                    int32_t spin_as_bool) {
  const bool minus = (state[row * W + (chain >> 5)] >> (chain & 31)) & 1u;
  return spin_as_bool ? (minus ? 0.0 : 1.0) : (minus ? -1.0 : 1.0);
}

// acc[m][chain] += prod_k value(rows[m][k], chain) over the k < order with rows >= 0.
template <typename T, bool BITS>
__global__ void k_moments(const T* state, int64_t C, const int64_t* __restrict__ rows, const uint8_t* __restrict__ spin,
                          int32_t order, int64_t n_moments, int32_t spin_as_bool, double* acc) {
  const int64_t m = blockIdx.y;
  for (int64_t chain = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; chain < C; chain += (int64_t)gridDim.x * blockDim.x) {
    double p = 1.0;
    for (int k = 0; k < order; ++k) {
      const int64_t r = rows[m * order + k];
      if (r < 0) break;
      if (BITS)
        p *= moment_value_bits(reinterpret_cast<const uint32_t*>(state), C / 32, r, chain, spin_as_bool);
      else
        p *= moment_value(state, C, r, chain, spin[m * order + k] != 0, spin_as_bool);
    }
    acc[m * C + chain] += p;
  }
}

}  // namespace
}  // namespace tthrml

extern "C" int tthrml_moments_accumulate(const void* state, int32_t dtype, int64_t C, const int64_t* rows,
                                         const uint8_t* spin_rows, int32_t order, int64_t n_moments,
                                         int32_t spin_as_bool, double* acc, void* stream) {
  using namespace tthrml;
  if (n_moments == 0 || C == 0) return TTHRML_OK;
  if (!state || !rows || !acc || order < 1 || n_moments < 0 || C < 0 || n_moments > 65535 ||
      (dtype != TTHRML_STATE_BITS && !spin_rows)) {
    set_error("tthrml_moments_accumulate: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  const int threads = 128;
  const int64_t bx = (C + threads - 1) / threads;
  dim3 grid((unsigned)(bx < 1024 ? bx : 1024), (unsigned)n_moments);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == TTHRML_STATE_BITS) {
    if (C % 32) {
      set_error("tthrml_moments_accumulate: bit-packed state needs n_chains %% 32 == 0");
      return TTHRML_ERR_ARG;
    }
    k_moments<uint32_t, true><<<grid, threads, 0, s>>>((const uint32_t*)state, C, rows, spin_rows, order, n_moments,
                                                       spin_as_bool, acc);
  } else if (dtype == TTHRML_STATE_I8) {
    k_moments<int8_t, false><<<grid, threads, 0, s>>>((const int8_t*)state, C, rows, spin_rows, order, n_moments,
                                                      spin_as_bool, acc);
  } else if (dtype == TTHRML_STATE_F32) {
    k_moments<float, false><<<grid, threads, 0, s>>>((const float*)state, C, rows, spin_rows, order, n_moments,
                                                     spin_as_bool, acc);
  } else {
    set_error("tthrml_moments_accumulate: unknown dtype %d", dtype);
    return TTHRML_ERR_ARG;
  }
  return launch_status("k_moments launch");
}

extern "C" int tthrml_greedy_colouring(int64_t n, const int64_t* row_ptr, const int32_t* cols, int32_t* colour,
                                       int32_t* n_colours) {
  if (n < 0 || (n > 0 && (!row_ptr || !cols || !colour)) || !n_colours) {
    set_error("tthrml_greedy_colouring: invalid arguments");
    return TTHRML_ERR_ARG;
  }
  std::vector<int64_t> mark;  // mark[c] == v  <=>  colour c is taken by a neighbour of v
  int32_t k = 0;
  for (int64_t v = 0; v < n; ++v) colour[v] = -1;
  for (int64_t v = 0; v < n; ++v) {
    for (int64_t e = row_ptr[v]; e < row_ptr[v + 1]; ++e) {
      const int64_t u = cols[e];
      if (u < 0 || u >= n) {
        set_error("tthrml_greedy_colouring: column %lld out of range", (long long)u);
        return TTHRML_ERR_ARG;
      }
      const int32_t cu = colour[u];
      if (cu >= 0) {
        if ((int64_t)mark.size() <= cu) mark.resize(cu + 1, -1);
        mark[cu] = v;
      }
    }
    int32_t c = 0;
    while (c < (int32_t)mark.size() && mark[c] == v) ++c;
    colour[v] = c;
    if (c + 1 > k) k = c + 1;
  }
  *n_colours = k;
  return TTHRML_OK;
}

extern "C" int tthrml_set_device(int32_t device) { return cuda_status(cudaSetDevice(device), "cudaSetDevice"); }

extern "C" const char* tthrml_last_error(void) { return g_last_error.c_str(); }
extern "C" int tthrml_abi_version(void) { return TTHRML_ABI_VERSION; }
