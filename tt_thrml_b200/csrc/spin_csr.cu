// Sparse spin block kernel on int8 ±1 state, chain-innermost.
//
// Work item = (row, slice of 32*VEC chains); one warp per item, each lane owns
// VEC consecutive chains, so every neighbour fetch is one coalesced
// 32*VEC-byte read of the neighbour's state row.  Warps are persistent: each
// walks items with a grid stride and prefetches the next item's CSR offsets,
// columns, weights and bias while the current item's neighbour rows are in
// flight.  Up to UNROLL neighbour rows are loaded before any is accumulated.
//
// Field arithmetic is bit-identical to a sequential float32 sum of w*s in CSR
// order (tt_thrml/compiler.py:303-318): with s = ±1 the product w*s is w with
// its sign bit flipped where s = -1, taken straight from the int8 sign bit, so
// no integer-to-float conversion is issued per neighbour.
#include "spin_common.cuh"

// Tuning: neighbour rows in flight per warp and the occupancy floor the
// register allocator must honour (blocks of 256 threads per SM).
#ifndef TTHRML_SPIN_UNROLL
#define TTHRML_SPIN_UNROLL 4
#endif
#ifndef TTHRML_SPIN_MIN_BLOCKS
#define TTHRML_SPIN_MIN_BLOCKS 3
#endif
#ifndef TTHRML_SPIN_ASYNC
#define TTHRML_SPIN_ASYNC 1
#endif
#ifndef TTHRML_ASYNC_MIN_BLOCKS
#define TTHRML_ASYNC_MIN_BLOCKS 5
#endif
#ifndef TTHRML_ASYNC_STAGE_ROWS
#define TTHRML_ASYNC_STAGE_ROWS 16
#endif

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
  using T = uint32_t;
};
template <>
struct Vec<8> {
  using T = uint2;
};
template <>
struct Vec<16> {
  using T = uint4;
};

// 32-bit words of a VEC-byte vector (VEC >= 4).
template <int VEC>
__device__ __forceinline__ uint32_t word(const typename Vec<VEC>::T& v, int i) {
  if constexpr (VEC == 4) {
    return v;
  } else if constexpr (VEC == 8) {
    return i == 0 ? v.x : v.y;
  } else if constexpr (VEC == 16) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
  } else {
    return 0u;
  }
}

// acc[v] += w * s_v for the VEC int8 spins of one neighbour row.
template <int VEC>
__device__ __forceinline__ void accumulate(float (&acc)[VEC], const typename Vec<VEC>::T& sv, float w) {
  const uint32_t wb = __float_as_uint(w);
  if constexpr (VEC >= 4) {
#pragma unroll
    for (int q = 0; q < VEC / 4; ++q) {
      const uint32_t x = word<VEC>(sv, q);
      acc[4 * q + 0] = __fadd_rn(acc[4 * q + 0], __uint_as_float(wb ^ ((x << 24) & 0x80000000u)));
      acc[4 * q + 1] = __fadd_rn(acc[4 * q + 1], __uint_as_float(wb ^ ((x << 16) & 0x80000000u)));
      acc[4 * q + 2] = __fadd_rn(acc[4 * q + 2], __uint_as_float(wb ^ ((x << 8) & 0x80000000u)));
      acc[4 * q + 3] = __fadd_rn(acc[4 * q + 3], __uint_as_float(wb ^ (x & 0x80000000u)));
    }
  } else {
    const int8_t* p = reinterpret_cast<const int8_t*>(&sv);
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const uint32_t sign = ((uint32_t)(uint8_t)p[v] << 24) & 0x80000000u;
      acc[v] = __fadd_rn(acc[v], __uint_as_float(wb ^ sign));
    }
  }
}

struct RowMeta {
  int64_t r;
  int64_t e0, e1;
  int32_t col;
  float w;
  float b;
};

__device__ __forceinline__ void load_meta(int64_t item, int64_t items, int64_t slices, const int64_t* __restrict__ rp,
                                          const int32_t* __restrict__ cols, const float* __restrict__ vals,
                                          const float* __restrict__ bias, int lane, RowMeta& m) {
  if (item >= items) return;
  m.r = item / slices;
  m.e0 = __ldg(rp + m.r);
  m.e1 = __ldg(rp + m.r + 1);
  const int64_t n = min((int64_t)32, m.e1 - m.e0);
  m.col = lane < n ? __ldg(cols + m.e0 + lane) : 0;
  m.w = lane < n ? __ldg(vals + m.e0 + lane) : 0.0f;
  m.b = bias ? __ldg(bias + m.r) : 0.0f;
}

template <int VEC, bool VARIATES>
__global__ void __launch_bounds__(256, TTHRML_SPIN_MIN_BLOCKS) k_spin_csr(const int64_t* __restrict__ row_ptr,
                                                  const int32_t* __restrict__ cols,
                                                  const float* __restrict__ vals,
                                                  const float* __restrict__ bias, int64_t row_start,
                                                  int64_t n_rows, int8_t* state, int64_t C,
                                                  int64_t chain_offset,
                                                  const float* __restrict__ variates,
                                                  int64_t variates_sweeps, uint64_t seed, uint32_t sweep_base,
                                                  const tthrml_run_ctl* __restrict__ ctl) {
  using V = typename Vec<VEC>::T;
  constexpr int UNROLL = TTHRML_SPIN_UNROLL;
  const int lane = threadIdx.x & 31;
  const int64_t slices = C / (32 * VEC);
  const int64_t items = n_rows * slices;
  const int64_t stride = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const uint32_t k0 = seed_lo(sd), k1 = seed_hi(sd);

  RowMeta cur{};
  load_meta(item, items, slices, row_ptr, cols, vals, bias, lane, cur);
  while (item < items) {
    const int64_t next = item + stride;
    const int64_t c0 = (item - cur.r * slices) * (32 * VEC) + lane * VEC;
    const int deg0 = (int)min((int64_t)32, cur.e1 - cur.e0);

    float acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0.0f;

    // first (up to) 32 neighbours: their columns are already in registers
    RowMeta nxt{};
    bool prefetched = false;
    for (int kb = 0; kb < deg0; kb += UNROLL) {
      V sv[UNROLL];
      float w[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int32_t j = __shfl_sync(0xffffffffu, cur.col, (kb + u) & 31);
        w[u] = __shfl_sync(0xffffffffu, cur.w, (kb + u) & 31);
        if (kb + u < deg0) sv[u] = *reinterpret_cast<const V*>(state + (int64_t)j * C + c0);
      }
      if (!prefetched) {  // the next item's metadata travels while these rows arrive
        load_meta(next, items, slices, row_ptr, cols, vals, bias, lane, nxt);
        prefetched = true;
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        if (kb + u < deg0) accumulate<VEC>(acc, sv[u], w[u]);
    }
    if (!prefetched) load_meta(next, items, slices, row_ptr, cols, vals, bias, lane, nxt);

    // rare: rows with more than 32 neighbours
    for (int64_t eb = cur.e0 + 32; eb < cur.e1; eb += 32) {
      const int n = (int)min((int64_t)32, cur.e1 - eb);
      const int32_t my_col = lane < n ? __ldg(cols + eb + lane) : 0;
      const float my_w = lane < n ? __ldg(vals + eb + lane) : 0.0f;
      for (int kb = 0; kb < n; kb += UNROLL) {
        V sv[UNROLL];
        float w[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const int32_t j = __shfl_sync(0xffffffffu, my_col, (kb + u) & 31);
          w[u] = __shfl_sync(0xffffffffu, my_w, (kb + u) & 31);
          if (kb + u < n) sv[u] = *reinterpret_cast<const V*>(state + (int64_t)j * C + c0);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u)
          if (kb + u < n) accumulate<VEC>(acc, sv[u], w[u]);
      }
    }

    const int64_t row = row_start + cur.r;
    int8_t out[VEC];
    if (VARIATES) {
      // the host never runs past variates_sweeps; the modulo keeps misuse in bounds
      const int64_t vs = (int64_t)(sweep % (uint32_t)(variates_sweeps > 0 ? variates_sweeps : 1));
      const float* lrow = variates + (vs * n_rows + cur.r) * C + c0;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
        out[v] = __fmul_rn(2.0f, gamma) > __ldg(lrow + v) ? 1 : -1;
      }
    } else {
      const int64_t g0 = chain_offset + c0;
      if (VEC >= 4) {
#pragma unroll
        for (int v = 0; v < VEC; v += 4) {
          const u32x4 rr = philox4x32_10(u32x4{(uint32_t)((g0 + v) >> 2), (uint32_t)row, sweep, kSaltSpin}, k0, k1);
#pragma unroll
          for (int t = 0; t < 4 && v + t < VEC; ++t) {
            const float gamma = bias ? __fadd_rn(cur.b, acc[v + t]) : acc[v + t];
            out[v + t] = spin_up_fast(gamma, word_of(rr, t)) ? 1 : -1;
          }
        }
      } else {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          const int64_t gc = g0 + v;
          const u32x4 rr = philox4x32_10(u32x4{(uint32_t)(gc >> 2), (uint32_t)row, sweep, kSaltSpin}, k0, k1);
          const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
          out[v] = spin_up_fast(gamma, word_of(rr, (int)(gc & 3))) ? 1 : -1;
        }
      }
    }
    V packed;
    int8_t* pp = reinterpret_cast<int8_t*>(&packed);
#pragma unroll
    for (int v = 0; v < VEC; ++v) pp[v] = out[v];
    *reinterpret_cast<V*>(state + row * C + c0) = packed;

    cur = nxt;
    item = next;
  }
}

// ----------------------------------------------------------------------------
// Shared-memory staged variant (VEC >= 4): each warp keeps two items in flight.
// While item i is summed from shared memory, the neighbour rows of item i+1
// stream in with cp.async (no registers held for data in flight), the metadata
// of item i+2 is being fetched, and the Philox words of item i are computed
// before its data is waited for.  Rows beyond kStageRows neighbours (rare at
// mean degree 8) are read directly.
//
// Field by table lookup: for a row with d >= 5 neighbours the warp first
// writes the 2^t sequential partial sums (t = min(d, 8)) of +-w_0, ..., +-w_(t-1)
// into shared memory, entry bit k set meaning spin k is -1.  Lane l owns the
// entries whose low five bits equal l: it sums its five-term prefix and
// extends it over neighbours 5..t-1 as a binary tree (510 additions per row
// for t = 8, spread over 32 lanes).  Each chain then ORs its t sign bits into
// an index and reads its field with one shared-memory load; neighbours past
// the first t are added afterwards in order.  Every entry is a left-to-right
// float32 sum in CSR order, so the field equals the sequential sum exactly.
// ----------------------------------------------------------------------------
constexpr int kStageRows = TTHRML_ASYNC_STAGE_ROWS;
constexpr int kAsyncThreads = 128;

template <int VEC>
__device__ __forceinline__ void issue_rows(const RowInfo& m, int64_t c0, bool valid, const int8_t* state, int64_t C,
                                           unsigned char* stage_buf, int lane) {
  if (!valid) return;
  const int deg = m.deg < kStageRows ? m.deg : kStageRows;
  for (int k = 0; k < deg; ++k) {
    const int32_t j = __shfl_sync(0xffffffffu, m.col, k);
    cp_async_bytes<VEC>(stage_buf + k * (32 * VEC) + lane * VEC, state + (int64_t)j * C + c0);
  }
}

template <int VEC, bool VARIATES>
__global__ void __launch_bounds__(kAsyncThreads, TTHRML_ASYNC_MIN_BLOCKS) k_spin_csr_async(
    const int64_t* __restrict__ row_ptr, const int32_t* __restrict__ cols, const float* __restrict__ vals,
    const float* __restrict__ bias, int64_t row_start, int64_t n_rows, int8_t* state, int64_t C, int64_t chain_offset,
    const float* __restrict__ variates, int64_t variates_sweeps, uint64_t seed, uint32_t sweep_base,
    const tthrml_run_ctl* __restrict__ ctl) {
  using V = typename Vec<VEC>::T;
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr int kStageBytes = kStageRows * 32 * VEC;
  constexpr int kWarpBytes = 2 * kStageBytes + (1 << kTableBits) * 4;
  const int lane = threadIdx.x & 31;
  unsigned char* wbuf = smem + (size_t)(threadIdx.x >> 5) * kWarpBytes;
  float* table = reinterpret_cast<float*>(wbuf + 2 * kStageBytes);
  const int64_t slices = C / (32 * VEC);
  const int64_t items = n_rows * slices;
  const int64_t stride = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int64_t item = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t sweep = sweep_base + (ctl ? ctl->sweep : 0u);
  const uint64_t sd = ctl ? ctl->seed : seed;
  const uint32_t k0 = seed_lo(sd), k1 = seed_hi(sd);
  // item = row * slices + slice; with one slice per row (the common case) no division is needed
  auto row_of = [&](int64_t it) -> int64_t { return slices == 1 ? it : (int64_t)((uint64_t)it / (uint64_t)slices); };
  auto col0_of = [&](int64_t it, int64_t r) -> int64_t { return (it - r * slices) * (32 * VEC) + lane * VEC; };

  RowInfo cur{}, nxt{};
  load_row(row_of(item), n_rows, row_ptr, cols, vals, bias, lane, cur);
  int stage = 0;
  issue_rows<VEC>(cur, col0_of(item, cur.r), item < items, state, C, wbuf, lane);
  cp_async_commit();
  int64_t next = item + stride;
  if (next < items) load_row(row_of(next), n_rows, row_ptr, cols, vals, bias, lane, nxt);

  while (item < items) {
    issue_rows<VEC>(nxt, col0_of(next, nxt.r), next < items, state, C, wbuf + (stage ^ 1) * kStageBytes, lane);
    cp_async_commit();
    RowInfo after{};
    if (next + stride < items) load_row(row_of(next + stride), n_rows, row_ptr, cols, vals, bias, lane, after);

    const int64_t c0 = col0_of(item, cur.r);
    const int64_t row = row_start + cur.r;
    uint32_t bits[VEC];
    if (!VARIATES) {  // independent of the neighbour data: computed while it is in flight
      const int64_t g0 = chain_offset + c0;
#pragma unroll
      for (int v = 0; v < VEC; v += 4) {
        const u32x4 rr = philox4x32_10(u32x4{(uint32_t)((g0 + v) >> 2), (uint32_t)row, sweep, kSaltSpin}, k0, k1);
        bits[v] = rr.x;
        bits[v + 1] = rr.y;
        bits[v + 2] = rr.z;
        bits[v + 3] = rr.w;
      }
    }

    const int deg = cur.deg;
    const int staged = deg < kStageRows ? deg : kStageRows;
    const unsigned char* sbuf = wbuf + stage * kStageBytes + lane * VEC;
    float acc[VEC];
    int done = 0;
    if (deg >= 5) {
      const int t = deg < kTableBits ? deg : kTableBits;
      __syncwarp();  // the previous item's lookups are finished before the table is rewritten
      build_table(table, cur.w, t, lane);
      cp_async_wait<1>();
      __syncwarp();  // table and this item's staged rows are visible to the warp
      uint32_t ix[VEC / 4];
#pragma unroll
      for (int q = 0; q < VEC / 4; ++q) ix[q] = 0u;
      for (int k = 0; k < t; ++k) {
        const V sv = *reinterpret_cast<const V*>(sbuf + k * (32 * VEC));
#pragma unroll
        for (int q = 0; q < VEC / 4; ++q) ix[q] |= (word<VEC>(sv, q) >> (7 - k)) & (0x01010101u << k);
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = table[(ix[v >> 2] >> (8 * (v & 3))) & 0xFFu];
      done = t;
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = 0.0f;
      cp_async_wait<1>();
      __syncwarp();
    }
    for (int k = done; k < staged; ++k) {
      const float w = __shfl_sync(0xffffffffu, cur.w, k);
      accumulate<VEC>(acc, *reinterpret_cast<const V*>(sbuf + k * (32 * VEC)), w);
    }
    // neighbours kStageRows..31: columns in registers, rows read directly
    const int first_chunk = deg < 32 ? deg : 32;
    for (int k = kStageRows; k < first_chunk; ++k) {
      const int32_t j = __shfl_sync(0xffffffffu, cur.col, k);
      const float w = __shfl_sync(0xffffffffu, cur.w, k);
      accumulate<VEC>(acc, *reinterpret_cast<const V*>(state + (int64_t)j * C + c0), w);
    }
    for (int64_t eb = cur.e0 + 32; eb < cur.e0 + deg; eb += 32) {  // more than 32 neighbours
      const int n = (int)min((int64_t)32, cur.e0 + deg - eb);
      const int32_t my_col = lane < n ? __ldg(cols + eb + lane) : 0;
      const float my_w = lane < n ? __ldg(vals + eb + lane) : 0.0f;
      for (int k = 0; k < n; ++k) {
        const int32_t j = __shfl_sync(0xffffffffu, my_col, k);
        const float w = __shfl_sync(0xffffffffu, my_w, k);
        accumulate<VEC>(acc, *reinterpret_cast<const V*>(state + (int64_t)j * C + c0), w);
      }
    }

    int8_t out[VEC];
    if (VARIATES) {
      // the host never runs past variates_sweeps; the modulo keeps misuse in bounds
      const int64_t vs = (int64_t)(sweep % (uint32_t)(variates_sweeps > 0 ? variates_sweeps : 1));
      const float* lrow = variates + (vs * n_rows + cur.r) * C + c0;
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
        out[v] = __fmul_rn(2.0f, gamma) > __ldg(lrow + v) ? 1 : -1;
      }
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float gamma = bias ? __fadd_rn(cur.b, acc[v]) : acc[v];
        out[v] = spin_up_fast(gamma, bits[v]) ? 1 : -1;
      }
    }
    V packed;
    int8_t* pp = reinterpret_cast<int8_t*>(&packed);
#pragma unroll
    for (int v = 0; v < VEC; ++v) pp[v] = out[v];
    *reinterpret_cast<V*>(state + row * C + c0) = packed;

    __syncwarp();  // every lane is done with this stage before it is refilled
    stage ^= 1;
    cur = nxt;
    nxt = after;
    item = next;
    next += stride;
  }
  cp_async_wait<0>();
}

template <int VEC, bool VARIATES>
int launch_async(const int64_t* rp, const int32_t* cols, const float* vals, const float* bias, int64_t row_start,
                 int64_t n_rows, int8_t* state, int64_t C, int64_t chain_offset, const float* variates,
                 int64_t variates_sweeps, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, cudaStream_t s) {
  constexpr int smem = (kAsyncThreads / 32) * (2 * kStageRows * 32 * VEC + (1 << kTableBits) * 4);
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_spin_csr_async<VEC, VARIATES>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_spin_csr_async<VEC, VARIATES>, kAsyncThreads, smem);
    if (e != cudaSuccess) return cuda_status(e, "k_spin_csr_async set-up");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t items = n_rows * (C / (32 * VEC));
  const int64_t need = (items + kAsyncThreads / 32 - 1) / (kAsyncThreads / 32);
  const int64_t full = (int64_t)sms * per_sm;
  const int grid = (int)(need < full ? (need > 0 ? need : 1) : full);
  k_spin_csr_async<VEC, VARIATES><<<grid, kAsyncThreads, smem, s>>>(rp, cols, vals, bias, row_start, n_rows, state, C,
                                                                    chain_offset, variates, variates_sweeps, seed,
                                                                    sweep, ctl);
  return launch_status("k_spin_csr_async launch");
}

// Persistent grid: every SM filled to its occupancy limit, or fewer blocks for
// small launches.  Cached per template instance after the first query.
template <int VEC, bool VARIATES>
int grid_for(int64_t items, int threads, int* grid) {
  static int per_sm = 0, sms = 0;  // same values from every thread: a benign race
  if (!per_sm) {
    int dev = 0, n = 0, b = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_spin_csr<VEC, VARIATES>, threads, 0);
    if (e != cudaSuccess) return cuda_status(e, "k_spin_csr occupancy query");
    sms = n;
    per_sm = b > 0 ? b : 1;
  }
  const int64_t warps_per_block = threads / 32;
  const int64_t need = (items + warps_per_block - 1) / warps_per_block;
  const int64_t full = (int64_t)sms * per_sm;
  *grid = (int)(need < full ? need : full);
  if (*grid < 1) *grid = 1;
  return TTHRML_OK;
}

template <int VEC>
int launch(const int64_t* rp, const int32_t* cols, const float* vals, const float* bias, int64_t row_start,
           int64_t n_rows, int8_t* state, int64_t C, int64_t chain_offset, const float* variates,
           int64_t variates_sweeps, uint64_t seed, uint32_t sweep, const tthrml_run_ctl* ctl, cudaStream_t s) {
#if TTHRML_SPIN_ASYNC
  if constexpr (VEC >= 4) {
    if (variates)
      return launch_async<VEC, true>(rp, cols, vals, bias, row_start, n_rows, state, C, chain_offset, variates,
                                     variates_sweeps, seed, sweep, ctl, s);
    return launch_async<VEC, false>(rp, cols, vals, bias, row_start, n_rows, state, C, chain_offset, variates,
                                    variates_sweeps, seed, sweep, ctl, s);
  }
#endif
  const int threads = 256;
  const int64_t items = n_rows * (C / (32 * VEC));
  int grid = 0;
  const int rc = variates ? grid_for<VEC, true>(items, threads, &grid) : grid_for<VEC, false>(items, threads, &grid);
  if (rc) return rc;
  if (variates)
    k_spin_csr<VEC, true><<<grid, threads, 0, s>>>(rp, cols, vals, bias, row_start, n_rows, state, C, chain_offset,
                                                   variates, variates_sweeps, seed, sweep, ctl);
  else
    k_spin_csr<VEC, false><<<grid, threads, 0, s>>>(rp, cols, vals, bias, row_start, n_rows, state, C, chain_offset,
                                                    variates, variates_sweeps, seed, sweep, ctl);
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
    return launch<16>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates,
                      variates_sweeps, seed, sweep, ctl, s);
  if (per_lane % 8 == 0)
    return launch<8>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates,
                     variates_sweeps, seed, sweep, ctl, s);
  if (per_lane % 4 == 0)
    return launch<4>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates,
                     variates_sweeps, seed, sweep, ctl, s);
  if (per_lane % 2 == 0)
    return launch<2>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates,
                     variates_sweeps, seed, sweep, ctl, s);
  return launch<1>(row_ptr, cols, vals, bias, row_start, n_rows, state, n_chains, chain_offset, variates,
                   variates_sweeps, seed, sweep, ctl, s);
}
